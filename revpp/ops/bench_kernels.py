"""Per-kernel microbenchmarks of the sm_100a extension (CUDA-event timing).

    python -m revpp.ops.bench_kernels gemm --M 16384 --N 4096 --K 1024 --epi gelu --variant 2
    python -m revpp.ops.bench_kernels attn-fwd --B 16 --S 512 --heads 16
    python -m revpp.ops.bench_kernels attn-bwd --B 16 --S 512 --heads 16
    python -m revpp.ops.bench_kernels layernorm --M 16384 --H 1024
    python -m revpp.ops.bench_kernels adamw --n 335000000
    python -m revpp.ops.bench_kernels suite --B 16 --S 512 --heads 16   # every kernel of one layer

Each run warms up, then times ``--iters`` launches between CUDA events and prints one JSON
line with the time per launch and the achieved TFLOP/s or GB/s.  ``--iters 1 --warmup 1``
gives a short, fixed launch sequence for profiler captures.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

EPIS = {"bf16": 0, "gelu": 1, "resid": 2, "atomic": 3, "dgelu": 4, "f32": 5}


def _time(fn, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def bench_gemm(a, C):
    M, N, K = a.M, a.N, a.K
    epi = EPIS[a.epi]
    dev = "cuda"
    splits = 1
    if a.layout == "wgrad":  # C[N_out, K_in] += dY[T, N]^T X[T, K]
        A = torch.randn(K, M, device=dev).to(torch.bfloat16)
        B = torch.randn(K, N, device=dev).to(torch.bfloat16)
        out = torch.zeros(M, N, device=dev)
        splits = a.splits if a.splits > 0 else C.gemm_suggest_splits(M, N, K)
        fn = lambda: C.gemm_tc(A, True, B, True, M, N, K, 3, out, splits=splits, variant=a.variant)  # noqa: E731
    elif a.layout == "dgrad":
        A = torch.randn(M, K, device=dev).to(torch.bfloat16)
        B = (torch.randn(K, N, device=dev) * 0.05).to(torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        aux = torch.randn(M, N, device=dev).to(torch.bfloat16) if epi == 4 else None
        cs = torch.zeros(N, device=dev) if (epi == 4 and a.colsum) else None
        fn = lambda: C.gemm_tc(A, False, B, True, M, N, K, epi, out, aux=aux, variant=a.variant,  # noqa: E731
                               colsum=cs)
    else:
        A = torch.randn(M, K, device=dev).to(torch.bfloat16)
        B = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
        bias = torch.zeros(N, device=dev, dtype=torch.bfloat16)
        f32 = epi in (2, 5)
        out = torch.empty(M, N, device=dev, dtype=torch.float32 if f32 else torch.bfloat16)
        aux = torch.empty(M, N, device=dev, dtype=torch.bfloat16) if (epi == 1 and not a.no_aux_out) else None
        resid = torch.randn(M, N, device=dev) if epi == 2 else None
        fn = lambda: C.gemm_tc(A, False, B, False, M, N, K, epi, out, bias=bias, aux_out=aux,  # noqa: E731
                               resid=resid, variant=a.variant)
    if a.cublas:  # the same product through cuBLAS (torch.matmul, bf16 out), for comparison
        if a.layout == "wgrad":
            fn = lambda: torch.matmul(A.t(), B)  # noqa: E731
        elif a.layout == "dgrad":
            fn = lambda: torch.matmul(A, B)  # noqa: E731
        else:
            fn = lambda: torch.matmul(A, B.t())  # noqa: E731
    ms = _time(fn, a.warmup, a.iters)
    return {"op": "gemm" + ("-cublas" if a.cublas else ""), "layout": a.layout, "epi": a.epi, "variant": a.variant, "M": M, "N": N, "K": K,
            "colsum": bool(a.colsum), "aux_out": a.epi == "gelu" and not a.no_aux_out,
            "splits": splits if a.layout == "wgrad" else 1, "ms": ms, "tflops": 2.0 * M * N * K / ms / 1e9}


def bench_attn(a, C, backward: bool):
    B, S, heads = a.B, a.S, a.heads
    H = heads * 64
    qkv = torch.randn(B * S, 3 * H, device="cuda").to(torch.bfloat16)
    out = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, heads, S, device="cuda")
    fwd = {"persistent": C.attn_fwd_persistent, "tc": C.attn_fwd_tc, "mma": C.attn_fwd}[a.impl]
    fwd(qkv, out, lse, B, S, heads)
    flops = 4.0 * B * S * S * H
    if not backward:
        ms = _time(lambda: fwd(qkv, out, lse, B, S, heads), a.warmup, a.iters)
        return {"op": "attn-fwd", "impl": a.impl, "B": B, "S": S, "heads": heads, "ms": ms,
                "tflops": flops / ms / 1e9}
    dout = torch.randn_like(out)
    dqkv = torch.empty_like(qkv)
    dq = torch.empty(B * S, H, device="cuda")
    D = torch.empty(B, heads, S, device="cuda")
    tc = a.impl in ("tc", "persistent")
    bwd = C.attn_bwd_tc if tc else C.attn_bwd
    if tc:  # with the fused q/k/v bias-gradient column sums, as in training
        cs = torch.zeros(3 * H, device="cuda")
        ms = _time(lambda: bwd(qkv, out, dout, lse, dqkv, dq, D, B, S, heads, colsum=cs), a.warmup, a.iters)
    else:
        ms = _time(lambda: bwd(qkv, out, dout, lse, dqkv, dq, D, B, S, heads), a.warmup, a.iters)
    return {"op": "attn-bwd", "impl": a.impl, "B": B, "S": S, "heads": heads, "ms": ms,
            "tflops": 2.5 * flops / ms / 1e9}


def attn_phases(a, C):
    """Per-CTA phase times of the tcgen05 attention kernels (globaltimer stamps written by
    the kernels when given a phase buffer): median time from the CTA's start to each
    phase, the median CTA duration and the kernel span.  Forward phases: 1 Q and first K
    landed, 2 first scores ready, 3 last P handed over, 4 merge starts, 5 merge done,
    6 end.  Backward (persistent: phases 1-6 of the CTA's first work item): 1 K, V, Q0, dO0
    landed, 2 first S^T/dP^T ready, 3 last P^T/dS^T handed over, 4 dK/dV complete, 5 dK
    written + column sums, 6 its dQ reductions issued, 7 the CTA's end (all its items)."""
    B, S, heads = a.B, a.S, a.heads
    H = heads * 64
    qkv = torch.randn(B * S, 3 * H, device="cuda").to(torch.bfloat16)
    out = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, heads, S, device="cuda")
    res = {"op": "attn-phases", "B": B, "S": S, "heads": heads}
    for kind in ("fwd", "bwd"):
        grid = ((S + 127) // 128) * heads * B
        ph = torch.zeros(grid * 32, dtype=torch.int64, device="cuda")
        if kind == "fwd":
            C.attn_fwd_tc(qkv, out, lse, B, S, heads)
            torch.cuda.synchronize()
            C.attn_fwd_tc(qkv, out, lse, B, S, heads, phase_ns=ph)
            nph = 7
        else:
            dout = torch.randn_like(out)
            dqkv = torch.empty_like(qkv)
            dq = torch.empty(B * S, H, device="cuda")
            D = torch.empty(B, heads, S, device="cuda")
            cs = torch.zeros(3 * H, device="cuda")
            C.attn_bwd_tc(qkv, out, dout, lse, dqkv, dq, D, B, S, heads, colsum=cs)
            torch.cuda.synchronize()
            C.attn_bwd_tc(qkv, out, dout, lse, dqkv, dq, D, B, S, heads, colsum=cs, phase_ns=ph)
            nph = 8
        torch.cuda.synchronize()
        full = ph.view(grid, 32).double()
        full = full[full[:, 0] > 0]  # the persistent backward runs fewer CTAs than work items
        t = full[:, :nph]
        rel = (t - t[:, :1]) / 1e3  # us from the CTA's start
        res[kind] = {"phase_us_median": [round(float(x), 2) for x in rel.median(0).values],
                     "cta_us_median": round(float(rel[:, -1].median()), 2),
                     "span_us": round(float((t[:, -1].max() - t[:, 0].min()) / 1e3), 2)}
        if kind == "bwd":  # the CTA's first item; per query tile: softmax start, hand-over, next S, MMAs
            res[kind]["first_item_us_median"] = round(float(rel[:, 5].median()), 2)
            res[kind]["ctas"] = int(full.shape[0])
            nt = min(4, (S + 127) // 128)
            tiles = (full[:, 8:8 + 4 * nt] - full[:, :1]) / 1e3
            med = [round(float(x), 2) for x in tiles.median(0).values]
            res[kind]["tiles_us_median"] = [med[4 * i:4 * i + 4] for i in range(nt)]
    return res


def bench_layernorm(a, C):
    M, H = a.M, a.H
    x = torch.randn(M, H, device="cuda")
    g = torch.ones(H, device="cuda")
    b = torch.zeros(H, device="cuda")
    y = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    mean = torch.empty(M, device="cuda")
    rstd = torch.empty(M, device="cuda")
    C.layernorm_fwd(x, g, b, 1e-5, y_bf16=y, mean=mean, rstd=rstd)
    t_f = _time(lambda: C.layernorm_fwd(x, g, b, 1e-5, y_bf16=y, mean=mean, rstd=rstd), a.warmup, a.iters)
    dy = torch.randn(M, H, device="cuda").to(torch.bfloat16)
    resid = torch.randn(M, H, device="cuda")
    dx = torch.empty(M, H, device="cuda")
    dxb = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    dg = torch.zeros(H, device="cuda")
    db = torch.zeros(H, device="cuda")
    cs = torch.zeros(H, device="cuda")
    t_b = _time(lambda: C.layernorm_bwd(dy, x, g, mean, rstd, dgamma=dg, dbeta=db, resid=resid, dx_f32=dx,
                                        dx_bf16=dxb, colsum=cs), a.warmup, a.iters)
    fwd_bytes = M * H * (4 + 2)
    bwd_bytes = M * H * (2 + 4 + 4 + 4 + 2)
    return {"op": "layernorm", "M": M, "H": H, "fwd_ms": t_f, "fwd_gbs": fwd_bytes / t_f / 1e6, "bwd_ms": t_b,
            "bwd_gbs": bwd_bytes / t_b / 1e6}


def bench_adamw(a, C):
    n = (a.n + 63) // 64 * 64
    p, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    v.abs_()
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    ss = torch.zeros(1, device="cuda")
    step = [0]

    def fn():
        step[0] += 1
        ss.zero_()
        C.grad_sumsq(g, ss)
        C.adamw_step(p, g, m, v, shadow=sh, lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-6, wd=0.01, step=step[0],
                     max_norm=1.0, sumsq=ss, zero_grad=False)

    ms = _time(fn, a.warmup, a.iters)
    bytes_ = n * (4 + 4 * 4 + 4 * 3 + 2)  # norm read + (g, p, m, v) read + (p, m, v) write + shadow
    return {"op": "adamw", "n": n, "ms": ms, "gbs": bytes_ / ms / 1e6}


def layer_suite(a):
    """Argument lists of every kernel of one reversible encoder layer for one micro-batch
    (tokens T = B*S, hidden H, FFN 4H): forward / reconstruction GEMMs with their
    epilogues, input-gradient and weight-gradient GEMMs, attention forward / backward,
    LayerNorm."""
    T, H, I = a.B * a.S, a.heads * 64, 4 * a.heads * 64
    g = ["gemm", "--M", str(T)]
    return [
        g + ["--N", str(3 * H), "--K", str(H), "--epi", "bf16"],                      # QKV
        g + ["--N", str(H), "--K", str(H), "--epi", "resid"],                         # out-proj + residual
        g + ["--N", str(I), "--K", str(H), "--epi", "gelu", "--no-aux-out"],          # FFN1 + GELU
        g + ["--N", str(I), "--K", str(H), "--epi", "gelu"],                          # FFN1 + GELU, saves u
        g + ["--N", str(H), "--K", str(I), "--epi", "resid"],                         # FFN2 + residual
        g + ["--N", str(I), "--K", str(H), "--layout", "dgrad", "--epi", "dgelu"],    # du
        g + ["--N", str(I), "--K", str(H), "--layout", "dgrad", "--epi", "dgelu", "--colsum"],
        g + ["--N", str(H), "--K", str(I), "--layout", "dgrad", "--epi", "bf16"],     # d LN2 out
        g + ["--N", str(H), "--K", str(H), "--layout", "dgrad", "--epi", "bf16"],     # d attn out
        g + ["--N", str(H), "--K", str(3 * H), "--layout", "dgrad", "--epi", "bf16"],  # d LN1 out
        ["gemm", "--M", str(H), "--N", str(I), "--K", str(T), "--layout", "wgrad", "--epi", "atomic"],   # dW2
        ["gemm", "--M", str(I), "--N", str(H), "--K", str(T), "--layout", "wgrad", "--epi", "atomic"],   # dW1
        ["gemm", "--M", str(H), "--N", str(H), "--K", str(T), "--layout", "wgrad", "--epi", "atomic"],   # dWo
        ["gemm", "--M", str(3 * H), "--N", str(H), "--K", str(T), "--layout", "wgrad", "--epi", "atomic"],  # dWqkv
        ["attn-fwd", "--B", str(a.B), "--S", str(a.S), "--heads", str(a.heads)],
        ["attn-bwd", "--B", str(a.B), "--S", str(a.S), "--heads", str(a.heads)],
        ["layernorm", "--M", str(T), "--H", str(H)],
    ]


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser()
    p.add_argument("op", choices=["gemm", "attn-fwd", "attn-bwd", "attn-phases", "layernorm", "adamw", "suite"])
    p.add_argument("--M", type=int, default=16384)
    p.add_argument("--N", type=int, default=4096)
    p.add_argument("--K", type=int, default=1024)
    p.add_argument("--H", type=int, default=1024)
    p.add_argument("--epi", choices=list(EPIS), default="bf16")
    p.add_argument("--layout", choices=["fwd", "dgrad", "wgrad"], default="fwd")
    p.add_argument("--variant", type=int, default=0)
    p.add_argument("--splits", type=int, default=0, help="wgrad: split-K count (0: the heuristic's)")
    p.add_argument("--colsum", action="store_true", help="dgelu: fused bias-gradient column sums")
    p.add_argument("--no-aux-out", action="store_true", help="gelu: do not write the pre-activation")
    p.add_argument("--B", type=int, default=16)
    p.add_argument("--S", type=int, default=512)
    p.add_argument("--heads", type=int, default=16)
    p.add_argument("--impl", choices=["persistent", "tc", "mma"], default="tc",
                   help="attention kernels: persistent / one-CTA-per-tile tcgen05 forward, or mma.sync")
    p.add_argument("--cublas", action="store_true", help="gemm: time torch.matmul on the same shape instead")
    p.add_argument("--n", type=int, default=335_000_000)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=20)
    return p


def main(argv=None):
    p = build_parser()
    a = p.parse_args(argv)
    from revpp.ops import ext

    C = ext()
    if a.op == "suite":
        extra = ["--warmup", str(a.warmup), "--iters", str(a.iters)]
        for args in layer_suite(a):
            if a.cublas and args[0] != "gemm":
                continue
            main(args + extra + (["--cublas"] if a.cublas else []))
        return
    if a.op == "gemm":
        r = bench_gemm(a, C)
    elif a.op == "attn-fwd":
        r = bench_attn(a, C, False)
    elif a.op == "attn-bwd":
        r = bench_attn(a, C, True)
    elif a.op == "attn-phases":
        r = attn_phases(a, C)
    elif a.op == "layernorm":
        r = bench_layernorm(a, C)
    else:
        r = bench_adamw(a, C)
    r["status"] = C.status_read_and_clear()
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
