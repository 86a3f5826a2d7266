"""Per-kernel timings at the d512 depth-8 production shapes, against library baselines.

  python benchmarks/kernels.py [--tokens 262144] [--json out.json] [--only tags|=tag] [--pair on|off|all]

Each kernel is timed with CUDA events on the launching stream after warm-up (median of R repeats);
inputs of the large shapes exceed the 126 MB L2. FLOP/s and bytes/s are reported as fractions of the
measured bf16 GEMM peak and copy bandwidth of ``MEASURED_PEAKS.json`` (fallback 1590 TFLOP/s,
6650 GB/s). Library rows (cuBLAS via ``torch.matmul``, ``F.scaled_dot_product_attention``) are the
baselines the sm_100a kernels replace.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"] * 1e12, d["hbm_gbs"] * 1e9, "measured"
    except Exception:
        return 1590e12, 6650e9, "fallback"


def timeit(fn, reps=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=262144)
    ap.add_argument("--json", default="")
    ap.add_argument("--only", default="")
    ap.add_argument("--pair", default="on", choices=["on", "off", "all"],
                    help="256-column GEMM tiles on CTA pairs (cta_group::2): on / all (the default policy puts "
                         "every such GEMM on pairs) or off (single CTAs)")
    args = ap.parse_args()
    from bitresearch_b200.ops import gemm
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    E.gemm_set_pair({"off": 0, "on": 1, "all": 2}[args.pair])
    dev = torch.device("cuda", 0)
    FLOPS, BW, src = peaks()
    M, D, F4, V, T, H = args.tokens, 512, 2048, 8192, 2048, 4
    B = M // T
    rows = []

    def report(name, ms, flops=0.0, nbytes=0.0, lib=None):
        r = {"kernel": name, "ms": ms}
        if flops:
            r["tflops"] = flops / ms / 1e9
            r["frac_peak"] = flops / ms / 1e-3 / FLOPS
        if nbytes:
            r["gbs"] = nbytes / ms / 1e6
            r["frac_bw"] = nbytes / ms / 1e-3 / BW
        if lib is not None:
            r["lib_ms"] = lib
            r["speedup_vs_lib"] = lib / ms
        rows.append(r)
        extra = " ".join(f"{k}={v:.3f}" for k, v in r.items() if k not in ("kernel",) and isinstance(v, float))
        print(f"{name:44s} {extra}", flush=True)

    bf = dict(device=dev, dtype=torch.bfloat16)
    sel = args.only.split(",") if args.only else None

    def want(tag):  # a selector matches tags that contain it; "=tag" matches that tag only
        return sel is None or any(s[1:] == tag if s.startswith("=") else s in tag for s in sel)

    # ------------------------------------------------------------------ GEMMs
    shapes = [  # name, (M, K, N), a transposed?, b transposed?, epilogue
        ("qkv_fwd", (M, D, 3 * D), False, False, gemm.BF16),
        ("proj_fwd_resid", (M, D, D), False, False, gemm.F32),
        ("fc_fwd_relu2", (M, D, F4), False, False, gemm.RELU2),
        ("mlp_proj_fwd_resid", (M, F4, D), False, False, gemm.F32),
        ("lm_head_fwd_softcap", (M, D, V), False, True, gemm.SOFTCAP),
        ("lm_head_dx", (M, V, D), False, False, gemm.BF16),
        ("mlp_proj_dx_relu2bwd", (M, D, F4), False, True, gemm.RELU2_BWD),
        ("fc_dx", (M, F4, D), False, True, gemm.BF16),
        ("qkv_dx", (M, 3 * D, D), False, True, gemm.BF16),
        ("dW_fc", (D, M, F4), True, False, gemm.ATOMIC),
        ("dW_mlp_proj", (F4, M, D), True, False, gemm.ATOMIC),
        ("dW_q", (D, M, D), True, False, gemm.ATOMIC),
        ("dW_lm_head", (V, M, D), True, False, gemm.ATOMIC),
    ]
    for name, (m, k, n), at, bt, epi in shapes:
        if not want(name):
            continue
        a = torch.randn(k, m, **bf).t() if at else torch.randn(m, k, **bf)
        b = torch.randn(n, k, **bf).t() if bt else torch.randn(k, n, **bf)
        if epi in (gemm.F32, gemm.ATOMIC):
            out = torch.zeros(m, n, device=dev)
        else:
            out = torch.empty(m, n, **bf)
        aux = None
        kw = {}
        if epi == gemm.F32:
            aux = out
            kw = dict(beta=1.0)
        elif epi == gemm.RELU2_BWD:
            aux = torch.rand(m, n, **bf)
        elif epi == gemm.SOFTCAP:
            kw = dict(alpha=1 / 15, beta=15.0)
        splits = 0 if epi == gemm.ATOMIC else 1
        ms = timeit(lambda: gemm.matmul(a, b, out=out, epi=epi, aux=aux, k_splits=splits, **kw))
        lib = timeit(lambda: torch.matmul(a, b))
        report(f"gemm/{name} {m}x{k}x{n}", ms, flops=2.0 * m * n * k, lib=lib)
    torch.cuda.synchronize()
    assert check_status() == 0

    # ------------------------------------------------------------------ attention
    if want("attn"):
        for window in (1024, 2048):
            qkv = torch.randn(M, 3 * D, **bf)
            q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
            o = torch.empty(M, D, **bf)
            lse = torch.empty(B, H, T, device=dev)
            # causal/window FLOPs actually computed: 4*hd per (query, visible key) pair, fwd
            vis = sum(min(i + 1, window) for i in range(T))
            f_fwd = 4.0 * 128 * vis * B * H
            ms = timeit(lambda: E.attn_fwd(q, k, v, o, lse, B, T, H, H, 128, window), reps=5)
            qs, ks, vs = (t.reshape(B, T, H, 128).transpose(1, 2) for t in (q, k, v))
            if window >= T:
                lib = timeit(lambda: F.scaled_dot_product_attention(qs, ks, vs, is_causal=True), reps=5)
            else:
                ii = torch.arange(T, device=dev)
                mask = (ii[None] <= ii[:, None]) & (ii[None] > ii[:, None] - window)
                lib = timeit(lambda: F.scaled_dot_product_attention(qs, ks, vs, attn_mask=mask), reps=5)
            report(f"attn_fwd w={window} B={B} T={T} H={H}", ms, flops=f_fwd, lib=lib)
            do = torch.randn(M, D, **bf)
            dqkv = torch.empty(M, 3 * D, **bf)
            delta = torch.empty(B, H, T, device=dev)
            ms = timeit(lambda: E.attn_bwd(q, k, v, o, do, lse, dqkv[:, :D], dqkv[:, D:2 * D], dqkv[:, 2 * D:], delta,
                                           delta, B, T, H, H, 128, window), reps=5)
            report(f"attn_bwd w={window} (2.5x fwd FLOPs)", ms, flops=2.5 * f_fwd)
            o2 = torch.empty(M, D, **bf)
            ms = timeit(lambda: E.attn_fwd_tc(qkv, o2, lse, B, T, H, H, 128, window), reps=5)
            report(f"attn_fwd_tc w={window}", ms, flops=f_fwd, lib=lib)
            ms = timeit(lambda: E.attn_bwd_tc(qkv, o2, do, lse, dqkv, delta, B, T, H, H, 128, window), reps=5)
            report(f"attn_bwd_tc w={window} (2.5x fwd FLOPs)", ms, flops=2.5 * f_fwd)
            ms = timeit(lambda: E.attn_bwd_tc(qkv, o2, do, lse, dqkv, delta, B, T, H, H, 128, window, 1), reps=5)
            report(f"  attn_bwd_tc dq only (1.5x fwd)", ms, flops=1.5 * f_fwd)
            ms = timeit(lambda: E.attn_bwd_tc(qkv, o2, do, lse, dqkv, delta, B, T, H, H, 128, window, 2), reps=5)
            report(f"  attn_bwd_tc dkdv only (2x fwd)", ms, flops=2.0 * f_fwd)

    # ------------------------------------------------------------------ RoPE fusion A/B
    if want("fusion"):
        # QKV projection + RoPE/QK-norm (+ value embedding): one GEMM with the epilogue vs GEMM + kernel
        xq = torch.randn(M, D, **bf)
        wq = torch.randn(D, 3 * D, **bf) * D ** -0.5
        qkv = torch.empty(M, 3 * D, **bf)
        pos = torch.arange(T, device=dev, dtype=torch.float32)[:, None]
        inv = 10000.0 ** (-torch.arange(0, 128, 2, device=dev, dtype=torch.float32) / 128)
        cos, sin = torch.cos(pos * inv).contiguous(), torch.sin(pos * inv).contiguous()
        idx = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        rq, rk = torch.empty(M, H, device=dev), torch.empty(M, H, device=dev)
        ve = torch.randn(V, D, device=dev)
        curx = torch.randn(M, D, device=dev)
        wg = torch.randn(32, H, device=dev) * 0.3
        gate = torch.empty(M, H, device=dev)
        for tag, vea in (("", (idx, None, None, None, None)), (" +VE", (idx, ve, curx, wg, gate))):
            ms_sep = timeit(lambda: (gemm.matmul(xq, wq, out=qkv),
                                     E.rope_fwd(qkv, T, H, H, 128, cos, sin, rq, rk, *vea)))
            ms_fused = timeit(lambda: gemm.qkv_rope(xq, wq, qkv, cos, sin, rq, rk, T, H, H, *vea))
            report(f"qkv+rope{tag}: gemm then rope_fwd", ms_sep, flops=2.0 * M * D * 3 * D)
            report(f"qkv+rope{tag}: fused epilogue", ms_fused, flops=2.0 * M * D * 3 * D)

    # ------------------------------------------------------------------ lm_head + softcap + CE
    if want("head"):
        # the fused form (the logits never reach memory) against the two-pass form it replaced
        # (softcapped bf16 logits written by the GEMM, read and overwritten by softcap_ce)
        xf = torch.randn(M, D, **bf)
        w = (torch.randn(V, D, device=dev) * 0.05)
        wb = w.to(torch.bfloat16)
        tgt = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        G = torch.empty(M, V, **bf)
        part = torch.empty(2 * ((V + 255) // 256), M, device=dev)
        zt, rs, cf = (torch.empty(M, device=dev) for _ in range(3))
        nats = torch.empty(M, device=dev)
        ls = torch.zeros(1, device=dev)
        xs = torch.empty(M, D, **bf)
        dw = torch.zeros(V, D, device=dev)
        f_head = 2.0 * M * D * V
        ms = timeit(lambda: E.gemm_softcap_ce(xf, wb, G, tgt, part, zt, 15.0, True))
        report(f"head: gemm_softcap_ce {M}x{D}x{V}", ms, flops=f_head)
        ms_fin = timeit(lambda: E.ce_finalize(part, zt, tgt, V, 15.0, 1.0 / M, nats=nats, loss_sum=ls, rowscale=rs,
                                              x=xf, xs=xs, g=G))
        report("head: ce_finalize", ms_fin, nbytes=M * (4 * (V // 256) + 2 * D * 2))
        ms_old = timeit(lambda: (gemm.matmul(xf, wb.t(), out=G, epi=gemm.SOFTCAP, alpha=1 / 15, beta=15.0),
                                 E.softcap_ce(G, tgt, 15.0, 1.0 / M, nats, ls, True)))
        report("head: two-pass (softcap GEMM + softcap_ce)", ms_old, flops=f_head)
        ms_eval = timeit(lambda: E.gemm_softcap_ce(xf, wb, G, tgt, part, zt, 15.0, False))
        report("head: gemm_softcap_ce, statistics only (eval)", ms_eval, flops=f_head)

    # ------------------------------------------------------------------ row kernels
    if want("rows"):
        x = torch.randn(M, D, device=dev)
        x0 = torch.randn(M, D, device=dev)
        lam = torch.ones(8, device=dev)
        cur = torch.empty(M, D, device=dev)
        xn = torch.empty(M, D, **bf)
        rs = torch.empty(M, device=dev)
        ms = timeit(lambda: E.ladder_rms_fwd(x, x0, lam, lam, 0, cur, xn, rs))
        report("ladder_rms_fwd", ms, nbytes=M * D * (4 + 4 + 4 + 2))
        ms = timeit(lambda: E.rms_fwd(x, xn, rs))
        report("rms_fwd", ms, nbytes=M * D * (4 + 2))
        dxn = torch.randn(M, D, **bf)
        dres = torch.randn(M, D, device=dev)
        dx = torch.empty(M, D, device=dev)
        ms = timeit(lambda: E.rms_bwd(x, rs, dxn, dres, dx, xn))
        report("rms_bwd (+residual, fp32+bf16 out)", ms, nbytes=M * D * (4 + 2 + 4 + 4 + 2))
        dx0 = torch.zeros(M, D, device=dev)
        g = torch.zeros(8, device=dev)
        ms = timeit(lambda: E.ladder_bwd(x, x0, lam, lam, 1, rs, dxn, dres, None, dx, dx0, g, g, False))
        report("ladder_bwd", ms, nbytes=M * D * (4 + 4 + 2 + 4 + 4 + 4 + 4))
        qkv = torch.randn(M, 3 * D, **bf)
        cos = torch.randn(T, 64, device=dev)
        idx = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        rq = torch.empty(M, H, device=dev)
        ms = timeit(lambda: E.rope_fwd(qkv, T, H, H, 128, cos, cos, rq, rq, idx, None, None, None, None))
        report("rope_qknorm_fwd", ms, nbytes=M * 2 * D * 2 * 2)
        logits = torch.randn(M, V, **bf)
        tgt = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        nats = torch.empty(M, device=dev)
        ls = torch.zeros(1, device=dev)
        ms = timeit(lambda: E.softcap_ce(logits, tgt, 15.0, 1.0 / M, nats, ls, True))
        report("softcap_ce fwd+bwd", ms, nbytes=M * V * 2 * 2)
        wte = torch.randn(V, D, device=dev)
        dw = torch.zeros(V, D, device=dev)
        ms = timeit(lambda: E.embed_bwd(idx, wte, rs, x, dw))
        report("embed_bwd (uniform ids)", ms, nbytes=M * D * 4 * 3)
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"peaks": src, "rows": rows}, f, indent=1)


if __name__ == "__main__":
    main()
