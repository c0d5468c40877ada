"""cfg1 MLP training step (784 -> 256 -> 128 -> 10, batch 128, softmax cross-entropy, SGD
lr 0.01) on the bit-exact fp32 kernels against the oracle's composition of the same step.

Forward logits are bit-exact: the region, matmul and ReLU kernels reproduce the reference's
fp32 loop order. expf / logf (CUDA vs the host libm) may differ by an ulp, so the loss and
everything downstream of it are compared within fp32 tolerance: max |diff| / max |ref| <=
1e-5 per tensor."""
import numpy as np
import pytest
import torch

import oracle
from c3_b200 import mlp

pytestmark = pytest.mark.gpu


def _np(p):
    return {k: v.detach().cpu().numpy().copy() for k, v in p.items()}


def _close(a, b, what, tol=1e-5):
    err = float(np.abs(a - b).max())
    ref = float(np.abs(b).max())
    assert err <= tol * max(ref, 1e-30), f"{what}: max |diff| {err:.3e} vs max |ref| {ref:.3e}"


def test_forward_logits_bit_exact_and_step_parity(cuda_device):
    params = mlp.init_params(1234, cuda_device)
    ref = _np(params)
    step = mlp.MLPTrainStep(params, batch=128, lr=0.01)
    for s in range(3):
        x, y = mlp.synthetic_batch(100 + s, 128, cuda_device)
        loss = step.step(x, y)
        torch.cuda.synchronize()
        r_loss, r_logits, r_grads, ref = oracle.mlp_train_step(ref, x.cpu().numpy(), y.cpu().numpy(), 0.01)
        if s == 0:
            assert np.array_equal(step.z3.cpu().numpy(), r_logits), "step 0 logits differ from the oracle"
        else:
            _close(step.z3.cpu().numpy(), r_logits, f"step {s} logits")
        assert abs(float(loss.item()) - r_loss) <= 1e-5 * abs(r_loss), (float(loss.item()), r_loss)
        for k in mlp.PARAM_NAMES:
            _close(step.g[k].cpu().numpy(), r_grads[k], f"step {s} grad {k}")
            _close(params[k].cpu().numpy(), ref[k], f"step {s} param {k}")


def test_graph_replay_matches_eager(cuda_device):
    p_eager = mlp.init_params(7, cuda_device)
    p_graph = {k: v.clone() for k, v in p_eager.items()}
    eager = mlp.MLPTrainStep(p_eager, batch=128)
    graphed = mlp.MLPTrainStep(p_graph, batch=128)
    graphed.capture()
    for s in range(4):
        x, y = mlp.synthetic_batch(200 + s, 128, cuda_device)
        l1 = eager.step(x, y).clone()
        l2 = graphed.replay(x, y).clone()
        torch.cuda.synchronize()
        assert torch.equal(l1, l2)
    for k in mlp.PARAM_NAMES:
        assert torch.equal(p_eager[k], p_graph[k]), k


def test_loss_decreases_over_steps(cuda_device):
    params = mlp.init_params(3, cuda_device)
    step = mlp.MLPTrainStep(params, batch=128, lr=0.1)
    x, y = mlp.synthetic_batch(9, 128, cuda_device)
    first = float(step.step(x, y).item())
    for _ in range(30):
        last = float(step.step(x, y).item())
    assert last < first * 0.9, (first, last)


def test_invalid_label_gives_nan_loss(cuda_device):
    params = mlp.init_params(4, cuda_device)
    step = mlp.MLPTrainStep(params, batch=128)
    x, y = mlp.synthetic_batch(5, 128, cuda_device)
    y[3] = 10
    loss = step.step(x, y)
    torch.cuda.synchronize()
    assert np.isnan(float(loss.item()))
