"""Small, fixed workloads of each kernel for profiling (ncu) and quick timing.

    python minimaxh3-on-a100-x4_b200/profile_cases.py CASE [--reps N]

Every case allocates a few GB at most, runs the kernel once to warm up and then N more times
(default 1), and checks the device status word. Cases:
  attn       attention, S=8192, 56 heads (Q/K/V 0.35 GB)
  pack       qk-RMSNorm + RoPE + pack, S=8192 tokens, 56 heads
  gemm_qkv   projection GEMM M=8192, K=5376, N=21504
  gemm_out   projection GEMM M=8192, K=7168, N=5376 (A read head-major [56][8192][128])
  gemm_fc1   fc1 + SwiGLU epilogue M=8192, K=5376, F=14336
  gemm_fc2   projection GEMM M=8192, K=14336, N=5376
  norm_mod   attention residual + LayerNorm + modulation, 42000 x 5376
  residual   gated residual, 42000 x 5376
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

import h3_model  # noqa: E402
import h3attn  # noqa: E402

CASES = ("attn", "pack", "gemm_qkv", "gemm_out", "gemm_fc1", "gemm_fc2", "norm_mod", "residual")


def build(case: str, dev):
    g = torch.Generator(device=dev).manual_seed(7)
    rnd = lambda *shape, std=1.0: (torch.randn(shape, generator=g, device=dev) * std).to(torch.bfloat16)
    H, D = 56, 128
    if case in ("attn", "pack"):
        S = 8192
        qkv = rnd(S, 3 * H * D)
        rope = h3_model.rope_freqs_1d(S, device=dev)[0].contiguous()
        q, k, v = qkv.split(H * D, -1)
        if case == "pack":
            out = torch.empty((1, 3, H, S, D), dtype=torch.bfloat16, device=dev)
            return lambda: h3attn.qknorm_rope_pack(q, k, v, rope, None, None, 1e-6, 1, out=out)
        send = h3attn.qknorm_rope_pack(q, k, v, rope, None, None, 1e-6, 1)
        o = torch.empty((S, H * D), dtype=torch.bfloat16, device=dev)
        return lambda: h3attn.attention(send[0, 0], send[0, 1], send[0, 2], layout="token", out=o)
    if case.startswith("gemm"):
        M = 8192
        if case == "gemm_out":
            a, w, ep = rnd(H, M, D), rnd(5376, H * D, std=0.02), "none"
        elif case == "gemm_qkv":
            a, w, ep = rnd(M, 5376), rnd(3 * H * D, 5376, std=0.02), "none"
        elif case == "gemm_fc1":
            a, w, ep = rnd(M, 5376), rnd(2 * 14336, 5376, std=0.02), "swiglu"
        else:
            a, w, ep = rnd(M, 14336), rnd(5376, 14336, std=0.02), "none"
        n = w.shape[0] // 2 if ep == "swiglu" else w.shape[0]
        c = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
        return lambda: h3attn.linear(a, w, out=c, epilogue=ep)
    rows, hidden = 42000, 5376
    x, y = rnd(rows, hidden), rnd(rows, hidden)
    mods = rnd(4, 6 * hidden, std=0.1).chunk(6, dim=-1)
    seg = h3attn.segment_rows(h3_model.H3_SEGMENTS, rows, dev)
    out, x1 = torch.empty_like(x), torch.empty_like(x)
    if case == "norm_mod":
        return lambda: h3attn.norm_modulate(x, mods[3], mods[4], seg, 1e-6, y=y, gate=mods[2], x_out=x1, out=out)
    return lambda: h3attn.gated_residual(x, y, mods[5], seg, out=out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=CASES)
    ap.add_argument("--reps", type=int, default=1)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    fn = build(args.case, dev)
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    h3attn.check_status()
    print(f"{args.case}: {e0.elapsed_time(e1) / max(args.reps, 1):.3f} ms per launch", flush=True)


if __name__ == "__main__":
    main()
