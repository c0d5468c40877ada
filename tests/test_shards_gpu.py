"""The exchange-free data-parallel shards on one GPU: each shard runs on its own slice, one after
another, and the shards must reassemble the full run bit for bit, since no output element
depends on another shard's inputs:
- the fused Linear+bias+ReLU forward by rows (shard_rows; Y and the ReLU bit mask);
- the cfg4 elementwise chain by vector-aligned element ranges (shard_range);
- the causal FlashAttention forward by (batch, head) pairs (shard_heads; O and LSE).
On several GPUs each rank runs exactly one of these slices."""
import pytest
import torch

from c3_b200 import elementwise, linear
from c3_b200.attention import flash_attn_fwd
from c3_b200.data_parallel import shard_heads, shard_range, shard_rows

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3, 8])
def test_forward_row_shards_reassemble(cuda_device, world):
    M, N, K = 1000, 512, 384
    g = torch.Generator(device=cuda_device).manual_seed(21)
    X = torch.randn((M, K), generator=g, device=cuda_device).to(torch.bfloat16)
    W = (torch.randn((N, K), generator=g, device=cuda_device) * 0.05).to(torch.bfloat16)
    b = torch.randn((N,), generator=g, device=cuda_device) * 0.05
    Y, mask = linear.forward(X, W, b, "nk")
    for r in range(world):
        lo, hi = shard_rows(M, world, r)
        Ys, ms = linear.forward(X[lo:hi].contiguous(), W, b, "nk")
        torch.cuda.synchronize()
        assert torch.equal(Ys, Y[lo:hi]), f"rank {r} of {world}: Y"
        assert torch.equal(ms, mask[lo:hi]), f"rank {r} of {world}: mask"


@pytest.mark.parametrize("n,world", [(4099, 2), ((1 << 22) + 5, 8), (1000, 3)])
def test_chain_range_shards_reassemble(cuda_device, n, world):
    g = torch.Generator(device=cuda_device).manual_seed(n)
    A = torch.rand(n, generator=g, device=cuda_device) * 8 - 4
    B = torch.rand(n, generator=g, device=cuda_device) * 16 - 8
    C = torch.rand(n, generator=g, device=cuda_device) * 8 - 4
    full = elementwise.chain_cfg4(A, B, C)
    out = torch.full_like(full, float("nan"))
    for r in range(world):
        lo, hi = shard_range(n, world, r)
        if hi > lo:
            elementwise.chain_cfg4(A[lo:hi], B[lo:hi], C[lo:hi], out[lo:hi])
    torch.cuda.synchronize()
    assert torch.equal(out, full)


@pytest.mark.parametrize("world", [2, 3])
def test_attention_head_shards_reassemble(cuda_device, world):
    Bt, H, S, D = 2, 3, 384, 128
    g = torch.Generator(device=cuda_device).manual_seed(5)
    Q, K, V = (torch.randn((Bt, H, S, D), generator=g, device=cuda_device).to(torch.bfloat16) for _ in range(3))
    O, L = flash_attn_fwd(Q, K, V, causal=True)
    flat = lambda t: t.view(1, Bt * H, *t.shape[2:])
    for r in range(world):
        lo, hi = shard_heads(Bt, H, world, r)
        Os, Ls = flash_attn_fwd(flat(Q)[:, lo:hi], flat(K)[:, lo:hi], flat(V)[:, lo:hi], causal=True)
        torch.cuda.synchronize()
        assert torch.equal(Os, flat(O)[:, lo:hi]), f"rank {r} of {world}: O"
        assert torch.equal(Ls, L.view(1, Bt * H, S)[:, lo:hi]), f"rank {r} of {world}: LSE"


def test_one_process_on_two_devices(cuda_device):
    """A host that drives two GPUs from one process, with cuda:0 current throughout: the
    wrappers run each call on its tensors' device, every kernel's launch setup (shared memory
    limits, workspaces, tensor maps) is per device, and both devices give the same bits for the
    same inputs. Tensors on different devices are refused before any launch."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from c3_b200 import _lib, mlp
    torch.cuda.set_device(0)
    outs = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        g = torch.Generator(device=dev).manual_seed(9)
        X = torch.randn((1024, 768), generator=g, device=dev).to(torch.bfloat16)
        W = (torch.randn((512, 768), generator=g, device=dev) * 0.05).to(torch.bfloat16)
        b = torch.randn((512,), generator=g, device=dev) * 0.05
        dY = (torch.randn((1024, 512), generator=g, device=dev) * 1e-2).to(torch.bfloat16)
        Y, mask = linear.forward(X, W, b, "nk")
        dZ, db = linear.relu_mask_db(dY, mask)
        dW = linear.grad_weight(dZ, X, "nk")
        Q, K, V = (torch.randn((1, 2, 256, 128), generator=g, device=dev).to(torch.bfloat16)
                   for _ in range(3))
        O, L = flash_attn_fwd(Q, K, V, causal=True)
        params = mlp.init_params(3, dev)
        x, y = mlp.synthetic_batch(4, 128, dev)
        loss = mlp.MLPTrainStep(params, batch=128).step(x, y)
        torch.cuda.synchronize(dev)
        assert torch.cuda.current_device() == 0
        outs.append([t.cpu() for t in (Y, mask, dZ, db, dW, O, L, loss, params["W1"])])
        if d == 1:
            with pytest.raises(_lib.C3CUError):
                linear.forward(X, W.to("cuda:0"), b, "nk")
    for name, a, c in zip(("Y", "mask", "dZ", "db", "dW", "O", "LSE", "loss", "W1"), *outs):
        assert torch.equal(a, c), name
