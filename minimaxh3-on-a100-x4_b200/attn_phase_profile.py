"""Phase profile of the attention kernel (diagnostics; the counterpart of the reference kernel's
clock64 phase counters and report scripts, attn_sm80/fa3_sm80_h3.cu:96-105, attn_sm80/report_v2.py).

    python minimaxh3-on-a100-x4_b200/attn_phase_profile.py [--seq 8192] [--heads 56] [--variant 0 ...]

Runs h3_attn_fwd_profile on one GPU and prints, per KV iteration of CTA (0, 0), the mean clock64
duration of each phase (iterations 8..55) for the two softmax warpgroups and the MMA-issuing thread:
softmax: wait for S, S loaded, first-half max/rescale, first-half exp + P hand-off, second-half
max/rescale, second-half exp + P hand-off; MMA thread: the spans between its recorded points.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402

import h3_model  # noqa: E402
import h3attn  # noqa: E402

SOFTMAX = ["wait_S", "load_S", "max_a", "exp_a+P_a", "max_b", "exp_b+P_b"]


def profile(seq: int, heads: int, variant: int, iters: int = 64):
    L = h3attn.lib()
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    L.h3_attn_fwd_profile.argtypes = [vp] * 4 + [i64] * 11 + [ctypes.c_float, vp, ctypes.c_int32, vp, i64, vp]
    L.h3_attn_fwd_profile.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    qkv = torch.randn((seq, 3 * heads * 128), generator=g, device=dev).to(torch.bfloat16)
    rope = h3_model.rope_freqs_1d(seq, device=dev)[0].contiguous()
    q, k, v = qkv.split(heads * 128, -1)
    send = h3attn.qknorm_rope_pack(q, k, v, rope, None, None, 1e-6, 1)
    qh, kh, vh = send[0]
    o = torch.empty_like(qh)
    trace = torch.zeros(3 * iters * 8, dtype=torch.int64, device=dev)
    n = seq * 128
    for _ in range(2):
        rc = L.h3_attn_fwd_profile(qh.data_ptr(), kh.data_ptr(), vh.data_ptr(), o.data_ptr(), heads, seq, seq, n, 128,
                                   n, 128, seq, 0, n, 128, ctypes.c_float(128 ** -0.5),
                                   h3attn.status_word().data_ptr(), variant, trace.data_ptr(), iters,
                                   torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(f"h3_attn_fwd_profile returned {rc}")
    torch.cuda.synchronize()
    h3attn.check_status()
    t = trace.view(3, iters, 8).cpu().double()
    lo, hi = 8, min(56, max(9, (seq + 127) // 128 - 1))
    res = {}
    for role in (0, 1):
        r = t[role, lo:hi]
        res[f"softmax_tile{role}"] = {nm: (r[:, i + 1] - r[:, i]).mean().item() for i, nm in enumerate(SOFTMAX)}
        res[f"softmax_tile{role}"]["iteration"] = (t[role, lo + 1:hi + 1, 0] - t[role, lo:hi, 0]).mean().item()
    m = t[2, lo:hi]
    npts = int((m != 0).sum(dim=0).gt(0).sum().item())
    res["mma"] = {f"p{i}-p{i + 1}": (m[:, i + 1] - m[:, i]).mean().item() for i in range(max(npts - 1, 0))}
    res["mma"]["iteration"] = (t[2, lo + 1:hi + 1, 0] - t[2, lo:hi, 0]).mean().item()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--heads", type=int, default=56)
    ap.add_argument("--variant", type=int, nargs="+", default=[0])
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    out = {}
    for var in args.variant:
        res = profile(args.seq, args.heads, var)
        out[f"variant{var}"] = res
        print(f"S={args.seq} heads={args.heads} variant={var} (clk, mean over KV iterations 8..55 of CTA 0)")
        for k, v in res.items():
            print("  " + k + ": " + ", ".join(f"{a}={b:.0f}" for a, b in v.items()))
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
