"""Data-parallel path on 2 GPUs (child processes, one per GPU): the in-switch all-reduce kernels
(including the split call that sums part of the buffer from peer loads) against NCCL's
all_reduce on the same buffers, the dW GEMM with the all-reduce fused into its
epilogue against NCCL's sum of the same partials, the row-sharded training step against the
one-GPU step on the full batch, and the data-parallel cfg1 MLP step (eager and CUDA-graph
replay, one NCCL all-reduce of gradients + loss per step) against the one-GPU full-batch step.
Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        import datetime

        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        import c3_b200
        from c3_b200.collective import NvlsAllReduce
        n = 1 << 20
        ar = NvlsAllReduce(n + 7, dev, num_ctas=8)
        results = {}
        for trial in range(3):
            g = torch.Generator(device=dev).manual_seed(100 * trial + rank)
            x = torch.randn(n + 7, generator=g, device=dev)
            ar.data().copy_(x)
            ref = x.clone()
            dist.all_reduce(ref)
            # two calls per trial: a partial range, then the rest
            ar.allreduce_(0, 3000)
            ar.allreduce_(3000, n + 7)
            torch.cuda.synchronize()
            results[trial] = float((ar.data() - ref).abs().max() / ref.abs().max())
        # bf16 region (fp32 accumulation in the switch, one rounding) and fp32 region in one call
        nb, nf = 1 << 20, 1024
        arb = NvlsAllReduce(nf, dev, num_ctas=8, numel_bf16=nb)
        for trial in range(2):
            g = torch.Generator(device=dev).manual_seed(7 + 10 * trial + rank)
            xb = torch.randn(nb, generator=g, device=dev).to(torch.bfloat16)
            xf = torch.randn(nf, generator=g, device=dev)
            arb.bf16.copy_(xb)
            arb.f32.copy_(xf)
            ref_b = xb.float()
            ref_f = xf.clone()
            dist.all_reduce(ref_b)
            dist.all_reduce(ref_f)
            arb.allreduce2_((0, nb // 2), None)
            arb.allreduce2_((nb // 2, nb), (0, nf))
            torch.cuda.synchronize()
            # within one bf16 ulp of the exact sum: the switch accumulates in fp32 and converts
            # to bf16 once, and that conversion is not assumed to round to nearest
            err_b = (arb.bf16.float() - ref_b).abs()
            ok_b = bool((err_b <= 2.0 ** -7 * ref_b.abs() + 1e-6).all())
            results[f"bf16_{trial}"] = 0.0 if ok_b else float(err_b.max())
            results[f"bf16_ratio_{trial}"] = 0.0  # informational below
            print(f"rank {rank} bf16 max err/|sum| = {float((err_b / ref_b.abs().clamp_min(1e-3)).max()):.3e}",
                  flush=True)
            results[f"f32_{trial}"] = float((arb.f32 - ref_f).abs().max() / ref_f.abs().max())
        # split call (c3cu_nvls_allreduce_split): the peer part is an fp32 sum in rank order
        # rounded once to nearest, so with two ranks (one fp32 addition, the same IEEE result in
        # either order) it equals NCCL's fp32 sum rounded to bf16 bit for bit; the switch part
        # as above
        from c3_b200.collective import split_point
        for trial, (frac, pctas, lo, hi, with_f32) in enumerate(
                [(0.3, 3, 0, nb, True), (0.5, 1, 8 * 1001, nb - 8 * 77, False), (1.0, 7, 0, nb, True),
                 (1.0, 8, 8, 8 * 5003, False)]):
            g = torch.Generator(device=dev).manual_seed(500 + 10 * trial + rank)
            xb = torch.randn(nb, generator=g, device=dev).to(torch.bfloat16)
            xf = torch.randn(nf, generator=g, device=dev)
            arb.bf16.copy_(xb)
            arb.f32.copy_(xf)
            ref_b = xb.float()
            ref_f = xf.clone()
            dist.all_reduce(ref_b)
            dist.all_reduce(ref_f)
            arb.allreduce_split_((lo, hi), (0, nf) if with_f32 else None, frac, pctas)
            torch.cuda.synchronize()
            got = arb.bf16.float()
            pf = lo + split_point(hi - lo, frac)
            sw = slice(lo, pf)
            err_sw = (got[sw] - ref_b[sw]).abs()
            ok_sw = bool((err_sw <= 2.0 ** -7 * ref_b[sw].abs() + 1e-6).all())
            peer_exact = torch.equal(arb.bf16[pf:hi], ref_b[pf:hi].to(torch.bfloat16))
            untouched = torch.equal(arb.bf16[:lo], xb[:lo]) and torch.equal(arb.bf16[hi:], xb[hi:])
            results[f"split_{trial}"] = 0.0 if (ok_sw and peer_exact and untouched) else \
                float(1 + (not ok_sw) + 2 * (not peer_exact) + 4 * (not untouched))
            f_err = float((arb.f32 - ref_f).abs().max() / ref_f.abs().max()) if with_f32 else \
                float((arb.f32 - xf).abs().max())
            results[f"split_f32_{trial}"] = f_err
        # NCCL through the C ABI (c3cu_allreduce_grads) against torch's all_reduce
        from c3_b200.collective import NcclComm
        nc = NcclComm(dev)
        for dt in (torch.float32, torch.bfloat16):
            g = torch.Generator(device=dev).manual_seed(31 + rank)
            x = torch.randn(4099, generator=g, device=dev).to(dt)
            ref = x.clone()
            dist.all_reduce(ref)
            nc.allreduce_(x)
            torch.cuda.synchronize()
            results[f"nccl_abi_{dt}"] = float((x.float() - ref.float()).abs().max())
        nc.close()
        c3_b200.fault_status()
        q.put((rank, "ok", results))
        dist.barrier()
        del ar, arb
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc)))


def test_nvls_allreduce_matches_nccl(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, status, res in out:
        assert status == "ok", f"rank {rank}: {res}"
        # fp32 sums of two values: the switch and NCCL may round in a different order;
        # bf16 results are within one bf16 rounding of the exact fp32 sum (0.0 when so)
        assert all(v <= 1e-6 for v in res.values()), res


def _fused_worker(rank, world, port, q):
    """c3cu_gemm_dw_allreduce on `world` GPUs: dW = sum over ranks of dZ_rᵀ X_r (bf16) and db
    summed in place, against torch.distributed's fp32 all_reduce of the same partials, over
    several epochs with fresh data each call. Shapes: ragged (K not a multiple of the tile) and
    one whose tiles run as split-K halves (fewer tiles than clusters, long reduction)."""
    try:
        import datetime

        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        import c3_b200
        from c3_b200 import _lib, linear
        from c3_b200.collective import NvlsAllReduce
        res = {}
        for (m, n, k) in ((500, 512, 384), (4096, 1024, 1024), (300 + 37 * rank, 384, 1032)):
            words = 4 + 16 * ((n + 255) // 256) * ((k + 255) // 256)
            buf = NvlsAllReduce(n, dev, num_ctas=8, numel_bf16=n * k, ar_flag_words=words)
            dW, db = buf.bf16.view(n, k), buf.f32
            worst_ulp, worst_db = 0.0, 0.0
            for epoch in range(3):
                g = torch.Generator(device=dev).manual_seed(1000 * epoch + 17 * rank + m)
                dZ = (torch.randn((m, n), generator=g, device=dev) * 1e-2).to(torch.bfloat16)
                X = torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16)
                db_part = torch.randn(n, generator=g, device=dev)
                db.copy_(db_part)
                dW.fill_(float("nan"))  # every element must be written by this call
                torch.cuda.synchronize()
                buf.gemm_dw_allreduce_(dZ, X, n, k)
                part = linear.grad_weight(dZ, X, "nk", out_dtype=torch.bfloat16)
                ref = part.float()
                dist.all_reduce(ref)
                ref_db = db_part.clone()
                dist.all_reduce(ref_db)
                absdb = db_part.abs()
                dist.all_reduce(absdb)
                torch.cuda.synchronize()
                ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(2.0 ** -126))) - 7)
                worst_ulp = max(worst_ulp, float(((dW.float() - ref).abs() / ulp).max()))
                worst_db = max(worst_db, float(((db - ref_db).abs() / (absdb + 1e-30)).max()))
            res[f"{m}x{n}x{k}_ulp"] = worst_ulp
            res[f"{m}x{n}x{k}_db"] = worst_db
            del buf
        res["fault"] = c3_b200.fault_status()
        q.put((rank, "ok", res))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc)))


def test_fused_dw_allreduce_matches_nccl(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, status, res in out:
        assert status == "ok", f"rank {rank}: {res}"
        assert res["fault"] == 0, res
        for key, v in res.items():
            if key.endswith("_ulp"):  # fp32 sum in the switch, one conversion to bf16
                assert v <= 1.0, (key, res)
            elif key.endswith("_db"):
                assert v <= 1e-6, (key, res)


def _step_worker(rank, world, port, q):
    """The row-sharded training step (c3_b200.data_parallel.LinearReluTrainStep) on `world`
    GPUs against the one-GPU kernels on the full batch."""
    try:
        import datetime

        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        import c3_b200
        from c3_b200 import linear
        from c3_b200.data_parallel import LinearReluTrainStep, shard_rows
        M, N, K = 1000, 512, 384
        g = torch.Generator(device=dev).manual_seed(11)  # the same full batch on every rank
        X = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        W = (torch.randn((N, K), generator=g, device=dev) * 0.05).to(torch.bfloat16)
        b = torch.randn((N,), generator=g, device=dev) * 0.05
        dY = (torch.randn((M, N), generator=g, device=dev) * 1e-2).to(torch.bfloat16)
        lo, hi = shard_rows(M, world, rank)
        res = {}
        for grad_dtype, chunks, coll in ((torch.bfloat16, 1, "fused"), (torch.bfloat16, 1, "nvls"),
                                         (torch.bfloat16, 4, "nvls"),
                                         (torch.float32, 2, "nvls"), (torch.bfloat16, 2, "nccl"),
                                         (torch.float32, 1, "nccl")):
            step = LinearReluTrainStep(hi - lo, N, K, dev, grad_dtype, collective=coll, chunks=chunks,
                                       num_ctas=8)
            Xs, dYs = X[lo:hi].contiguous(), dY[lo:hi].contiguous()
            step(Xs, W, b, dYs)
            step(Xs, W, b, dYs)  # a second step re-uses the buffers and the barrier epochs
            torch.cuda.synchronize()
            # one-GPU reference on the full batch (fp32 dW), and this rank's fp32 partial
            Y, mask = linear.forward(X, W, b, "nk")
            dZ, db = linear.relu_mask_db(dY, mask)
            dW = linear.grad_weight(dZ, X, "nk")
            dX = linear.grad_input(dZ, W, "nk")
            part = linear.grad_weight(dZ[lo:hi].contiguous(), Xs, "nk").abs()
            dist.all_reduce(part)  # sum over ranks of |partial dW|
            torch.cuda.synchronize()
            tol = (2.0 ** -6 if grad_dtype == torch.bfloat16 else 1e-5) * part + 1e-6
            key = f"{grad_dtype}_{chunks}_{coll}"
            res[key + "_collective"] = step.sync.collective == coll
            res[key + "_dW_ok"] = bool(((step.dW.float() - dW).abs() <= tol).all())
            res[key + "_db_err"] = float((step.db - db).abs().max() / db.abs().max())
            res[key + "_dX_equal"] = bool(torch.equal(step.dX, dX[lo:hi]))
            res[key + "_Y_equal"] = bool(torch.equal(step.Y, Y[lo:hi]))
            step.close()
            del step
        c3_b200.fault_status()
        q.put((rank, "ok", res))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc)))


def test_sharded_step_matches_full_batch(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_step_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, status, res in out:
        assert status == "ok", f"rank {rank}: {res}"
        for key, v in res.items():
            if key.endswith("_collective") or key.endswith("_ok") or key.endswith("_equal"):
                assert v is True, (key, res)
            else:  # db: fp32 sums of two row blocks vs one pass, and summation order
                assert v <= 1e-5, (key, res)


def _mlp_worker(rank, world, port, q):
    """The data-parallel cfg1 MLP step (c3_b200.mlp.MLPTrainStep with a process group) on its
    share of the batch against the one-GPU step on the full batch, on this rank's GPU."""
    try:
        import datetime
        import gc
        import hashlib

        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        import c3_b200
        from c3_b200 import mlp
        B, lr = 128, 0.05
        params = mlp.init_params(31, dev)
        full = {k: v.clone() for k, v in params.items()}
        lo, hi = mlp.shard_batch(B, world, rank)
        dp = mlp.MLPTrainStep(params, batch=hi - lo, lr=lr, group=dist.group.WORLD)
        one = mlp.MLPTrainStep(full, batch=B, lr=lr)
        res = {"loss_err": 0.0, "param_err": 0.0}

        def compare(l_dp, l_one):
            torch.cuda.synchronize()
            res["loss_err"] = max(res["loss_err"], abs(float(l_dp) - float(l_one)) / abs(float(l_one)))
            for k in mlp.PARAM_NAMES:
                e = float((params[k] - full[k]).abs().max() / full[k].abs().max())
                res["param_err"] = max(res["param_err"], e)

        for s in range(3):
            x, y = mlp.synthetic_batch(40 + s, B, dev)
            l_dp = dp.step(x[lo:hi].contiguous(), y[lo:hi].contiguous()).clone()
            l_one = one.step(x, y).clone()
            compare(l_dp.item(), l_one.item())
        dp.capture()  # the NCCL all-reduce is recorded in the graph with the kernels
        one.capture()
        for s in range(3):
            x, y = mlp.synthetic_batch(50 + s, B, dev)
            l_dp = dp.replay(x[lo:hi], y[lo:hi]).clone()
            l_one = one.replay(x, y).clone()
            compare(l_dp.item(), l_one.item())
        torch.cuda.synchronize()
        h = hashlib.sha256()
        for k in mlp.PARAM_NAMES:
            h.update(params[k].cpu().numpy().tobytes())
        res["params_sha"] = h.hexdigest()
        res["fault"] = c3_b200.fault_status()
        dp.graph = None  # release the graph that holds NCCL calls before the group goes
        one.graph = None
        del dp, one
        gc.collect()
        q.put((rank, "ok", res))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc)))


def test_data_parallel_mlp_step_matches_full_batch(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mlp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    res = {}
    for rank, status, r in out:
        assert status == "ok", f"rank {rank}: {r}"
        # the sum of two half-batch means against one full-batch mean: fp32 rounding only
        assert r["loss_err"] <= 1e-5 and r["param_err"] <= 1e-5, r
        assert r["fault"] == 0
        res[rank] = r
    assert res[0]["params_sha"] == res[1]["params_sha"], "ranks hold different parameters"
