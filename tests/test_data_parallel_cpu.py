"""Host logic of the data-parallel step on CPU: row sharding, dW band schedule, and the
gradient sum over a world_size-2 gloo process group (c3_b200.data_parallel.GradientSync,
"group" collective), checked against the oracle's full-batch backward of the MatMul+Add+ReLU
region (src/C3/C3BackwardCapture.cpp:501-528, 618-644, 681-723). Each rank's local gradients
come from the oracle on its rows; the test checks that the sharding and the banded sums
reassemble the full-batch gradients. A rank that leaves before the exchange makes the other
rank's sum end with an error instead of hanging it.

Also: the exchange-free shards of the elementwise chain (element ranges) and of attention
((batch, head) pairs), and the cfg1 MLP step's gradient exchange (c3_b200.mlp: flat gradient
+ loss buffer, one all-reduce, lr / world) against the oracle's full-batch step."""
import os
import socket

import numpy as np
import pytest

from c3_b200.data_parallel import dw_bands, shard_heads, shard_range, shard_rows


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("m,world", [(0, 1), (1, 2), (7, 2), (16384, 8), (37, 4), (5, 8), (129, 3)])
def test_shard_rows_cover_and_balance(m, world):
    ranges = [shard_rows(m, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == m
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0, "ranges must be contiguous"
    sizes = [hi - lo for lo, hi in ranges]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_shard_rows_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)
    with pytest.raises(ValueError):
        shard_rows(10, 0, 0)


@pytest.mark.parametrize("n,world,align", [(0, 2, 4), (3, 2, 4), (4099, 2, 4), (1 << 28, 8, 4),
                                           (1001, 3, 4), (17, 8, 4), (100, 3, 1)])
def test_shard_range_covers_aligned_and_balanced(n, world, align):
    ranges = [shard_range(n, world, r, align) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for lo, hi in ranges:
        assert (lo % align == 0 or lo == n) and lo <= hi  # an empty last shard sits at n
        assert hi % align == 0 or hi == n
    vecs = [(hi - lo + align - 1) // align for lo, hi in ranges]
    assert max(vecs) - min(vecs) <= 1


@pytest.mark.parametrize("b,h,world", [(8, 32, 8), (8, 32, 3), (1, 2, 4), (0, 4, 2)])
def test_shard_heads_cover_all_pairs(b, h, world):
    ranges = [shard_heads(b, h, world, r) for r in range(world)]
    covered = [i for lo, hi in ranges for i in range(lo, hi)]
    assert covered == list(range(b * h))
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


@pytest.mark.parametrize("n,chunks,expect", [
    (4096, 1, [(0, 4096)]),
    (4096, 4, [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]),
    (24, 3, [(0, 8), (8, 16), (16, 24)]),
    (20, 2, [(0, 20)]),      # 10-row bands are not 8-row aligned: one band
    (4096, 0, [(0, 4096)]),
])
def test_dw_bands(n, chunks, expect):
    assert dw_bands(n, chunks) == expect


def _problem(M, N, K, seed=5):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, K)).astype(np.float32)
    Z = rng.standard_normal((M, N)).astype(np.float32)  # pre-activation of the forward
    Z[::5, ::3] = 0.0                                    # ReLU'(0) = 0 (CmpF OGT)
    dY = (rng.standard_normal((M, N)) * 1e-2).astype(np.float32)
    return X, Z, dY


def _local_grads(X, Z, dY, lo, hi):
    import oracle
    dZ = oracle.relu_bwd(dY[lo:hi], Z[lo:hi])
    dW = oracle.matmul(dZ, X[lo:hi], transA=True) if hi > lo else np.zeros((dY.shape[1], X.shape[1]), np.float32)
    db = oracle.sum_reduce(dZ, 0) if hi > lo else np.zeros(dY.shape[1], np.float32)
    return dW, db


def _worker(rank, world, port, q, mode):
    try:
        import datetime

        import torch
        import torch.distributed as dist
        from c3_b200.data_parallel import GradientSync
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=20))
        M, N, K = 37, 24, 20
        X, Z, dY = _problem(M, N, K)
        lo, hi = shard_rows(M, world, rank)
        dW_r, db_r = _local_grads(X, Z, dY, lo, hi)
        if mode == "mlp":
            q.put((rank, "ok", _mlp_dp_rank(rank, world)))
            dist.barrier()
            dist.destroy_process_group()
            return
        if mode == "leave":
            # rank 1 leaves between steps, before its exchange; rank 0's sum must end with an
            # error (peer closed or process-group timeout), not wait for ever
            if rank == 1:
                q.put((rank, "ok", "left"))
                return
            sync = GradientSync(N, K, torch.device("cpu"), torch.float32, "group")
            sync.dW.copy_(torch.from_numpy(dW_r))
            sync.db.copy_(torch.from_numpy(db_r))
            try:
                sync.reduce_()
            except Exception as exc:  # the failure surfaced on the host
                q.put((rank, "ok", f"detected: {type(exc).__name__}"))
                return
            q.put((rank, "error", "the sum returned although the peer left"))
            return
        out = {}
        for chunks in (1, 3):
            sync = GradientSync(N, K, torch.device("cpu"), torch.float32, "group")
            sync.dW.copy_(torch.from_numpy(dW_r))
            sync.db.copy_(torch.from_numpy(db_r))
            bands = dw_bands(N, chunks)
            for i, band in enumerate(bands):
                sync.reduce_(band, with_db=i == len(bands) - 1)
            out[chunks] = (sync.dW.numpy().copy(), sync.db.numpy().copy())
        q.put((rank, "ok", out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc)))


_MLP_BATCH, _MLP_LR = 128, 0.05


def _mlp_problem():
    from c3_b200 import mlp
    params = {k: v.numpy() for k, v in mlp.init_params(11).items()}
    x, y = mlp.synthetic_batch(12, _MLP_BATCH)
    return params, x.numpy(), y.numpy()


def _mlp_dp_rank(rank, world):
    """One data-parallel cfg1 step of one rank: oracle gradients on the rank's rows, packed in
    the step's flat buffer layout, summed by mlp.reduce_gradients over gloo, SGD at
    mlp.data_parallel_lr."""
    import torch

    import oracle
    from c3_b200 import mlp
    params, x, y = _mlp_problem()
    lo, hi = mlp.shard_batch(_MLP_BATCH, world, rank)
    loss, _, g, _ = oracle.mlp_train_step(params, x[lo:hi], y[lo:hi], _MLP_LR)
    shapes = {k: params[k].shape for k in mlp.PARAM_NAMES}
    flat = torch.zeros(mlp.flat_numel(shapes))
    views, loss_slot = mlp.gradient_views(flat, shapes)
    for k in mlp.PARAM_NAMES:
        views[k].copy_(torch.from_numpy(g[k]))
    loss_slot.fill_(loss)
    mlp.reduce_gradients(flat, world)
    lr = mlp.data_parallel_lr(_MLP_LR, world)
    new = {k: oracle.sgd(params[k], views[k].numpy(), lr) for k in mlp.PARAM_NAMES}
    grads = {k: views[k].numpy() / world for k in mlp.PARAM_NAMES}
    return float(loss_slot.item()), grads, new


def _run(world, mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = [q.get(timeout=120) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return {rank: (status, res) for rank, status, res in out}


def test_gradient_sum_world2_gloo():
    import oracle
    res = _run(2, "sum")
    M, N, K = 37, 24, 20
    X, Z, dY = _problem(M, N, K)
    dW_full, db_full = _local_grads(X, Z, dY, 0, M)
    # sequential-k fp32 sums over all rows vs the sum of two partial sums: bounded by a few
    # ulp of the sum of |terms|
    dZ = oracle.relu_bwd(dY, Z)
    bound_w = 1e-6 * (np.abs(dZ).T @ np.abs(X)) + 1e-12
    bound_b = 1e-6 * np.abs(dZ).sum(axis=0) + 1e-12
    for rank in range(2):
        status, out = res[rank]
        assert status == "ok", f"rank {rank}: {out}"
        for chunks, (dW, db) in out.items():
            assert (np.abs(dW - dW_full) <= bound_w).all(), f"rank {rank}, {chunks} band(s): dW"
            assert (np.abs(db - db_full) <= bound_b).all(), f"rank {rank}, {chunks} band(s): db"
        # both ranks hold the same bits after the sum
    for chunks in res[0][1]:
        assert np.array_equal(res[0][1][chunks][0], res[1][1][chunks][0])


def test_rank_leaving_is_detected_world2_gloo():
    res = _run(2, "leave")
    assert res[1] == ("ok", "left")
    status, msg = res[0]
    assert status == "ok", msg
    assert msg.startswith("detected")


def test_mlp_step_gradient_exchange_world2_gloo():
    import oracle
    from c3_b200 import mlp
    res = _run(2, "mlp")
    params, x, y = _mlp_problem()
    loss, _, g, new = oracle.mlp_train_step(params, x, y, _MLP_LR)
    for rank in range(2):
        status, out = res[rank]
        assert status == "ok", f"rank {rank}: {out}"
        r_loss, r_grads, r_new = out
        # the mean of the ranks' means is the full-batch mean, up to fp32 rounding
        assert abs(r_loss - loss) <= 1e-5 * abs(loss), (r_loss, loss)
        for k in mlp.PARAM_NAMES:
            ref = float(np.abs(g[k]).max())
            assert float(np.abs(r_grads[k] - g[k]).max()) <= 1e-5 * max(ref, 1e-30), f"rank {rank} grad {k}"
            assert float(np.abs(r_new[k] - new[k]).max()) <= 1e-6 * float(np.abs(new[k]).max()) + 1e-9, \
                f"rank {rank} param {k}"
    for k in mlp.PARAM_NAMES:  # every rank applies the same update
        assert np.array_equal(res[0][1][2][k], res[1][1][2][k]), k


def test_mlp_shard_batch_needs_equal_shares():
    from c3_b200 import mlp
    assert mlp.shard_batch(128, 4, 3) == (96, 128)
    with pytest.raises(ValueError):
        mlp.shard_batch(128, 3, 0)


# Property tests of the shard arithmetic over arbitrary sizes and world sizes.
from hypothesis import given, settings, strategies as st  # noqa: E402


@settings(max_examples=300, deadline=None)
@given(n=st.integers(0, 1 << 40), world=st.integers(1, 64), align=st.sampled_from([1, 2, 4, 8, 16]))
def test_shard_range_properties(n, world, align):
    ranges = [shard_range(n, world, r, align) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for lo, hi in ranges:
        assert 0 <= lo <= hi <= n
        assert lo % align == 0 or lo == n
    vecs = [(hi - lo + align - 1) // align for lo, hi in ranges]
    assert max(vecs) - min(vecs) <= 1


@settings(max_examples=300, deadline=None)
@given(m=st.integers(0, 1 << 40), world=st.integers(1, 64))
def test_shard_rows_properties(m, world):
    ranges = [shard_rows(m, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == m
    sizes = [hi - lo for lo, hi in ranges]
    assert all(s >= 0 for s in sizes) and max(sizes) - min(sizes) <= 1 and sum(sizes) == m


@settings(max_examples=200, deadline=None)
@given(b=st.integers(0, 64), h=st.integers(0, 128), world=st.integers(1, 16))
def test_shard_heads_properties(b, h, world):
    covered = [i for r in range(world) for i in range(*shard_heads(b, h, world, r))]
    assert covered == list(range(b * h))


@settings(max_examples=200, deadline=None)
@given(n=st.integers(1, 1 << 16), chunks=st.integers(0, 16))
def test_dw_bands_properties(n, chunks):
    bands = dw_bands(n, chunks)
    assert bands[0][0] == 0 and bands[-1][1] == n
    for (a0, a1), (b0, b1) in zip(bands, bands[1:]):
        assert a1 == b0
    if len(bands) > 1:
        assert all((hi - lo) % 8 == 0 for lo, hi in bands) and len(bands) == chunks


@given(st.integers(0, 1 << 20).map(lambda v: v * 8), st.floats(0.0, 1.0))
@settings(max_examples=200, deadline=None)
def test_split_point_properties(count, frac):
    """The switch / peer boundary of the split all-reduce: whole 8-element vectors, the peer part
    within half a vector of the asked fraction, and the whole range at the ends."""
    from c3_b200.collective import split_point
    p = split_point(count, frac)
    assert p % 8 == 0 and 0 <= p <= count
    assert abs((count - p) - frac * count) <= 4
    assert split_point(count, 0.0) == count and split_point(count, 1.0) == 0


def test_split_options_are_checked():
    from c3_b200.collective import split_point
    from c3_b200.data_parallel import GradientSync
    with pytest.raises(ValueError):
        split_point(64, 1.5)
    for frac, ctas in ((0.3, 0), (0.3, 16), (-0.1, 1), (1.2, 1)):
        with pytest.raises(ValueError, match="peer_frac"):
            GradientSync(64, 64, "cpu", collective="group", num_ctas=16, peer_frac=frac, peer_ctas=ctas)


def test_nvls_ranges_are_checked_against_the_regions():
    """The in-switch all-reduce calls take bare offsets; a range outside its region is refused
    on the host (no buffer is needed to check it)."""
    from c3_b200.collective import NvlsAllReduce
    ar = object.__new__(NvlsAllReduce)
    ar.numel, ar.numel_bf16 = 100, 64
    assert ar._ranges((8, 64), (0, 100)) == (8, 64, 0, 100)
    assert ar._ranges(None, None) == (0, 0, 0, 0)
    for bad in ((0, 72), (4, 64), (16, 8), (-8, 8)):
        with pytest.raises(ValueError, match="bf16 range"):
            ar._ranges(bad, None)
    for bad in ((0, 104), (2, 8), (8, 4)):
        with pytest.raises(ValueError, match="fp32 range"):
            ar._ranges(None, bad)
