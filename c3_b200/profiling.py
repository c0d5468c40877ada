"""Runs one hot-path kernel repeatedly on cuda:0, for timing and for ncu captures.

    python -m c3_b200.profiling <case> [--iters N] [--m M] [--n N] [--k K] [--elems E]
                                [--variant V] [--dw-dtype bf16|fp32]

cases: gemm-fwd, gemm-dw, gemm-dx, prepass, ew-cfg4, sum-rows, step, attn, mlp-step,
       mlp-step-graph (the cfg1 training step, eager launches or one CUDA graph),
       pcie-h2d, pcie-d2h, pcie-bidir (pinned host <-> device copies of the cfg3 step's
       inputs X, dY, W, b and results Y, dX, dW, db, one direction or both at once: the link
       that bounds the end-to-end measurement)
Prints the CUDA-event time per launch and the algorithmic rate (TFLOP/s or GB/s)."""
from __future__ import annotations

import argparse
import json

import torch

from . import elementwise, linear


def _case(args, dev):
    g = torch.Generator(device=dev).manual_seed(0)
    M, N, K = args.m, args.n, args.k
    if args.case.startswith("gemm") or args.case in ("prepass", "step"):
        X = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        W = (torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        b = torch.randn((N,), generator=g, device=dev) * 0.01
        dY = (torch.randn((M, N), generator=g, device=dev) * 1e-3).to(torch.bfloat16)
        Y, mask = linear.forward(X, W, b)
        dZ, db = linear.relu_mask_db(dY, mask)
        dW = torch.empty((N, K), dtype=torch.bfloat16 if args.dw_dtype == "bf16" else torch.float32,
                         device=dev)
        dX = torch.empty((M, K), dtype=torch.bfloat16, device=dev)
        fl = 2.0 * M * N * K
        if args.case == "gemm-fwd":
            return (lambda: linear.forward(X, W, b, "nk", Y, mask)), fl, "TFLOP/s"
        if args.case == "gemm-dw":
            return (lambda: linear.grad_weight(dZ, X, "nk", dW)), fl, "TFLOP/s"
        if args.case == "gemm-dx":
            return (lambda: linear.grad_input(dZ, W, "nk", dX)), fl, "TFLOP/s"
        if args.case == "prepass":
            nbytes = M * N * 2 * 2 + M * ((N + 31) // 32) * 4 + N * 4
            return (lambda: linear.relu_mask_db(dY, mask, dZ, db)), nbytes, "GB/s"

        def step():
            linear.forward(X, W, b, "nk", Y, mask)
            linear.relu_mask_db(dY, mask, dZ, db)
            linear.grad_weight(dZ, X, "nk", dW)
            linear.grad_input(dZ, W, "nk", dX)
        return step, 3 * fl, "TFLOP/s"
    if args.case == "ew-cfg4":
        n = args.elems
        A = torch.rand(n, generator=g, device=dev) * 8 - 4
        B = torch.rand(n, generator=g, device=dev) * 16 - 8
        C = torch.rand(n, generator=g, device=dev) * 8 - 4
        out = torch.empty_like(A)
        return (lambda: elementwise.chain_cfg4(A, B, C, out)), 16.0 * n, "GB/s"
    if args.case == "attn":
        from .attention import flash_attn_fwd
        B, H, S = args.b, args.h, args.s
        Q, K, V = [torch.randn((B, H, S, 128), generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
        O = torch.empty_like(Q)
        L = torch.empty((B, H, S), device=dev)
        flops = 2.0 * B * H * S * S * 128  # causal: half of 4 B H S^2 D
        return (lambda: flash_attn_fwd(Q, K, V, True, None, O, L)), flops, "TFLOP/s"
    if args.case in ("mlp-step", "mlp-step-graph"):
        from . import mlp
        params = mlp.init_params(1234, dev)
        step = mlp.MLPTrainStep(params, batch=128, lr=0.01)
        x, y = mlp.synthetic_batch(1, 128, dev)
        d = mlp.LAYERS
        fl = 2.0 * 128 * sum(a * b for a, b in zip(d[:-1], d[1:]))  # forward
        fl += fl + 2.0 * 128 * (d[1] * d[2] + d[2] * d[3])  # dW of all layers + dX of layers 2, 3
        if args.case == "mlp-step":
            return (lambda: step.step(x, y)), fl, "TFLOP/s"
        step.capture()
        step.x_static.copy_(x)
        step.y_static.copy_(y)
        return (lambda: step.replay()), fl, "TFLOP/s"
    if args.case.startswith("pcie-"):
        shapes = [((M, K), torch.bfloat16), ((M, N), torch.bfloat16), ((N, K), torch.bfloat16),
                  ((N,), torch.float32)]
        host_in = [torch.ones(s, dtype=t, pin_memory=True) for s, t in shapes]
        host_out = [torch.empty(s, dtype=t, pin_memory=True) for s, t in shapes]
        dev_in = [torch.empty(s, dtype=t, device=dev) for s, t in shapes]
        dev_out = [torch.ones(s, dtype=t, device=dev) for s, t in shapes]
        nbytes = sum(t.numel() * t.element_size() for t in host_in)
        up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ups = args.case in ("pcie-h2d", "pcie-bidir")
        downs = args.case in ("pcie-d2h", "pcie-bidir")

        def copies():
            cur = torch.cuda.current_stream(dev)
            active = [(st, pairs) for st, on, pairs in ((up, ups, list(zip(dev_in, host_in))),
                                                        (down, downs, list(zip(host_out, dev_out)))) if on]
            for st, _ in active:  # both directions start after the start event, neither waits on the other
                st.wait_stream(cur)
            for st, pairs in active:
                with torch.cuda.stream(st):
                    for dst, src in pairs:
                        dst.copy_(src, non_blocking=True)
            for st, _ in active:
                cur.wait_stream(st)
        return copies, nbytes * (2 if args.case == "pcie-bidir" else 1), "GB/s"
    if args.case == "sum-rows":
        x = torch.randn((M, N), generator=g, device=dev)
        out = torch.empty(N, device=dev)
        return (lambda: elementwise.sum_rows(x, out)), 4.0 * M * N, "GB/s"
    raise SystemExit(f"unknown case {args.case}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--elems", type=int, default=1 << 28)
    ap.add_argument("--b", type=int, default=8)
    ap.add_argument("--h", type=int, default=32)
    ap.add_argument("--s", type=int, default=8192)
    ap.add_argument("--variant", type=int, default=0, help="GEMM kernel variant (c3cu_set_gemm_variant)")
    ap.add_argument("--dw-dtype", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--attn-variant", type=int, default=0, help="c3cu_set_attn_variant")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from . import _lib
    _lib.check(_lib.load().c3cu_set_gemm_variant(args.variant), "c3cu_set_gemm_variant")
    _lib.check(_lib.load().c3cu_set_attn_variant(args.attn_variant), "c3cu_set_attn_variant")
    fn, work, unit = _case(args, dev)
    fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    from . import fault_status
    fault_status()
    best, avg = min(times), sum(times) / len(times)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    print(json.dumps({"case": args.case, "variant": args.variant, "attn_variant": args.attn_variant, "m": args.m, "n": args.n, "k": args.k, "elems": args.elems,
                      "ms_avg": avg, "ms_best": best, "rate_avg": work / (avg * 1e-3) / scale,
                      "rate_best": work / (best * 1e-3) / scale, "unit": unit,
                      "times_ms": [round(t, 4) for t in times]}))


if __name__ == "__main__":
    main()
