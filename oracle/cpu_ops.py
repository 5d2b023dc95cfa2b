"""CPU stand-in for the kernel binding (h3attn) used ONLY by tests that drive sp_runtime's
host logic on CPU gloo ranks. Same call signatures as h3attn; the arithmetic is the
oracle's (qk-RMSNorm + RoPE) and the reference's SDPA call (attention). Tests install it
explicitly with `sp_runtime._ops = cpu_ops`; the runtime never selects it by itself.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from oracle import h3_oracle as O
from oracle import sdpa_ref

D = 128


def qknorm_rope_pack(q, k, v, rope, q_weight, k_weight, eps, world, out=None):
    sl = q.shape[0]
    H = q.reshape(sl, -1).shape[1] // D
    f = lambda t: O.bf16_round(t.detach().float().reshape(sl, H, D).numpy())
    w = lambda t: None if t is None else O.bf16_round(t.detach().float().numpy())
    r = None if rope is None else (rope[0] if rope.dim() == 5 else rope).detach().float().numpy()
    send = O.qknorm_rope_pack(f(q), f(k), v.detach().float().reshape(sl, H, D).numpy(), r, w(q_weight),
                              w(k_weight), float(eps), world)
    res = torch.from_numpy(send).to(q.dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res


def seq_to_head_unpack(recv, out=None):
    W, T, hl, sl, d = recv.shape
    res = recv.permute(1, 2, 0, 3, 4).reshape(T, hl, W * sl, d).contiguous()
    if out is not None:
        out.copy_(res)
        return out
    return res


def attention(q, k, v, s_kv=None, scale=None, out=None, layout="head", world=1):
    H, sq, _ = q.shape
    s_kv = k.shape[1] if s_kv is None else s_kv
    assert scale is None or abs(scale - 1 / math.sqrt(D)) < 1e-12
    o = sdpa_ref.attention(q[None], k[None, :, :s_kv], v[None, :, :s_kv])[0]  # [H, sq, D]
    if layout == "head":
        res = o.contiguous()
    elif layout == "token":
        res = o.transpose(0, 1).reshape(sq, H * D).contiguous()
    elif layout == "send":
        res = o.reshape(H, world, sq // world, D).permute(1, 0, 2, 3).contiguous()
    else:
        raise ValueError(layout)
    if out is not None:
        out.copy_(res)
        return out
    return res


def head_to_seq_unpack(recv, out=None):
    H, sl, d = recv.shape
    res = recv.transpose(0, 1).reshape(sl, H * d).contiguous()
    if out is not None:
        out.copy_(res)
        return out
    return res


def linear(a, weight, out=None, epilogue="none"):
    """The projection GEMM as the host model computes it: nn.Linear without bias (a [m, k], or
    head-major [H, m, 128] read as [m, H*128]); "swiglu": chunk(2) -> silu(gate) * up."""
    if a.dim() == 3:
        a = a.transpose(0, 1).reshape(a.shape[1], -1)
    y = torch.nn.functional.linear(a, weight)
    if epilogue == "swiglu":
        g, u = y.chunk(2, dim=-1)
        y = torch.nn.functional.silu(g) * u
    if out is not None:
        out.copy_(y)
        return out
    return y
