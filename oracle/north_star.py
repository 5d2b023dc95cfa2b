"""Inputs and ground truths of the north-star accuracy check (BASELINE configs 0 and 1).

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU legs
may import this module, and only as the checker; the product path never calls it.

The configs:
  config 0  B=1, H=56, D=128, S=4096,  seed 0, fp32, on the CPU through the reference's own
            SDPA FLASH call (harness/sp_runtime.py:119-121)
  config 1  B=1, H=56, D=128, S=42000, seed 1, bf16 kernel inputs, fp32 ground truth
Both draw Q, K, V ~ N(0, 1) (in that order, from one generator seeded with `seed`), apply
per-head RMSNorm (eps 1e-6, unit weight) and then 1-D RoPE (theta 10000, positions
0..S-1) to Q and K; V stays raw. The RoPE pairs (x[i], x[i+64]) as the library's pack
does (the "split half" convention named by the reference's rms_rope_split_half_ call,
sp_runtime.py:98). Scale 1/sqrt(128), non-causal, every key live.

The geometry and the error measures follow the reference's own attention check
(attn_sm80/bench_attn.py:11-32: [B, H, N, 128], max error and rel_mean =
mean|err| / mean|ref|); the thresholds are the north star's (max-abs 2e-2, mean-abs 2e-3
against an fp32 ground truth) plus the reference's rel_mean < 5e-3.
"""
from __future__ import annotations

import math

import numpy as np
import torch

D = 128
EPS = 1e-6
MAX_ABS = 2e-2
MEAN_ABS = 2e-3
REL_MEAN = 5e-3


def rope_matrices(s: int, device, theta: float = 10000.0) -> torch.Tensor:
    """[s, 64, 2, 2] fp32 rotation matrices [[cos, -sin], [sin, cos]], angle pos * theta^(-2i/128),
    computed in float64."""
    inv = theta ** (-torch.arange(D // 2, dtype=torch.float64) * 2.0 / D)
    ang = torch.arange(s, dtype=torch.float64)[:, None] * inv[None, :]
    c, sn = torch.cos(ang), torch.sin(ang)
    m = torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2)
    return m.to(torch.float32).to(device)


def norm_rope(x: torch.Tensor, rope: torch.Tensor | None) -> torch.Tensor:
    """Per-head RMSNorm (unit weight, eps 1e-6) then RoPE on x [H, S, 128] fp32, all in fp32."""
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + EPS)
    if rope is None:
        return y
    a, b = y[..., :64], y[..., 64:]
    m = rope[None]  # [1, S, 64, 2, 2]
    return torch.cat([m[..., 0, 0] * a + m[..., 0, 1] * b, m[..., 1, 0] * a + m[..., 1, 1] * b], -1)


def config_inputs(seed: int, heads: int, s: int, device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """fp32 q, k, v [heads, s, 128] of a config (normalised and rotated q, k; raw v). The
    generator lives on `device` (torch's CPU or CUDA generator: the same seed gives different
    draws on the two, so config 0 is drawn on the CPU and config 1 on the GPU)."""
    device = torch.device(device)
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn((heads, s, D), generator=g, device=device)
    k = torch.randn((heads, s, D), generator=g, device=device)
    v = torch.randn((heads, s, D), generator=g, device=device)
    rope = rope_matrices(s, device)
    return norm_rope(q, rope), norm_rope(k, rope), v


@torch.no_grad()
def fp32_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows: int = 8192) -> torch.Tensor:
    """Plain fp32 softmax(Q K^T / sqrt(128)) V by head and by blocks of `rows` queries (TF32 off)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = torch.empty_like(q)
        scale = 1.0 / math.sqrt(D)
        for h in range(q.shape[0]):
            kt = k[h].T.contiguous()
            for r0 in range(0, q.shape[1], rows):
                s = (q[h, r0:r0 + rows] @ kt) * scale
                s = torch.softmax(s, dim=-1)
                out[h, r0:r0 + rows] = s @ v[h]
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def f64_rows(q: np.ndarray, k: np.ndarray, v: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """float64 attention of the query rows `rows` of one head (q, k, v: [S, 128] float arrays)."""
    qr = q[rows].astype(np.float64)
    s = (qr @ k.astype(np.float64).T) / math.sqrt(D)
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    return (p @ v.astype(np.float64)) / p.sum(axis=1, keepdims=True)


def errors(out: torch.Tensor, ref: torch.Tensor) -> dict:
    """max-abs, mean-abs and rel_mean of out against ref (both any float dtype, same shape)."""
    err = (out.float() - ref.float()).abs()
    mean_ref = ref.float().abs().mean().item()
    return {"max_abs": err.max().item(), "mean_abs": err.mean().item(),
            "rel_mean": err.mean().item() / (mean_ref + 1e-30)}


def within(e: dict) -> bool:
    return e["max_abs"] <= MAX_ABS and e["mean_abs"] <= MEAN_ABS and e["rel_mean"] < REL_MEAN
