"""CPU oracle for the MiniMax-H3 Ulysses attention path.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs may import this module, and only as the checker. The product path
(libh3attn.so behind sp_runtime) never calls into it and has no CPU fallback.

What it restates (citations are paths inside the reference project):
  * attention: O = softmax(Q K^T * d^-1/2) V, non-causal, over the first s_kv keys --
    the SDPA FLASH call at harness/sp_runtime.py:119-121 with the pad-path K/V slice of
    :106-109. torch.nn.functional.scaled_dot_product_attention is third-party (PyTorch;
    the reference ran 2.13.0+cu130, README.md:119); its published algorithm is the
    plain softmax formula above, restated here in float64.
  * a2a layouts: a2a_seq_to_head / a2a_head_to_seq, sp_runtime.py:67-77.
  * pad + shard: sp_runtime.py:224-239, _shard_segments :196-201, _piece_bounds :136-144.
  * qk-RMSNorm + RoPE: stands in for comfy_kitchen's rms_rope_split_half_ (called at
    sp_runtime.py:93-99), whose source is not part of the reference. The convention is
    this build's own: y = x * (1/sqrt(mean(x^2) + eps)) * w, then rotation of the pairs
    (x[i], x[i+64]) by the [S][64][2][2] matrix table. PARITY UNPINNED for this part:
    no reference test or fixture fixes it. The restatement reproduces the CUDA kernel's
    fp32 operation order exactly (bit-exact check), so the GPU path is pinned to it.

Pinning: tests/golden/ holds vectors produced by running the reference's own code here
(harness/sp_runtime.py with a stub `comfy` package, CPU gloo ranks, and its SDPA call);
tests/test_oracle.py checks every function below against them.
"""
from __future__ import annotations

import math

import numpy as np

D = 128
ROPE_PAIRS = 64


# ----------------------------------------------------------------------------- bf16
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.float32("nan")
    return out


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- RoPE table
def rope_table(s: int, theta: float = 10000.0, pos0: int = 0, rot_dim: int = D) -> np.ndarray:
    """[1, s, rot_dim/2, 2, 2] float32 rotation matrices [[cos, -sin], [sin, cos]] for 1-D
    positions pos0..pos0+s-1 with angle pos * theta^(-2i/rot_dim); computed in float64."""
    half = rot_dim // 2
    inv = theta ** (-np.arange(half, dtype=np.float64) * 2.0 / rot_dim)
    ang = np.arange(pos0, pos0 + s, dtype=np.float64)[:, None] * inv[None, :]
    c, sn = np.cos(ang), np.sin(ang)
    m = np.empty((1, s, half, 2, 2), dtype=np.float64)
    m[0, :, :, 0, 0] = c
    m[0, :, :, 0, 1] = -sn
    m[0, :, :, 1, 0] = sn
    m[0, :, :, 1, 1] = c
    return m.astype(np.float32)


# ----------------------------------------------------------------------------- qk-RMSNorm + RoPE
def qknorm_rope(x: np.ndarray, weight: np.ndarray | None, rope: np.ndarray | None, eps: float) -> np.ndarray:
    """x: [S, H, 128] bf16 values (float32 array). weight: [128] bf16 values or None.
    rope: [S, 64, 2, 2] float32 or None. Returns bf16-rounded float32 [S, H, 128].

    Operation order (every step a separately rounded fp32 op), as in the CUDA kernel:
      lane g in 0..7 owns elements [8g, 8g+8) and [64+8g, 64+8g+8); its partial sum of
      squares runs over those 16 elements in that order; partials combine by an xor
      butterfly at distances 4, 2, 1; mean = sum * 2^-7; r = 1 / sqrt(mean + eps);
      y = (x * r) * w; pair i: (m00*a + m01*b, m10*a + m11*b)."""
    f32 = np.float32
    x = np.asarray(x, dtype=f32)
    S, H, d = x.shape
    assert d == D
    idx = np.concatenate([np.arange(8 * g, 8 * g + 8).tolist() + np.arange(64 + 8 * g, 72 + 8 * g).tolist()
                          for g in range(8)]).reshape(8, 16)
    xg = x[:, :, idx]  # [S, H, 8 lanes, 16]
    sq = (xg * xg).astype(f32)
    acc = sq[..., 0].copy()
    for i in range(1, 16):
        acc = (acc + sq[..., i]).astype(f32)
    # butterfly: after distance 4 lane g holds acc[g] + acc[g^4], etc. (commutative adds)
    a4 = (acc + acc[..., [4, 5, 6, 7, 0, 1, 2, 3]]).astype(f32)
    a2 = (a4 + a4[..., [2, 3, 0, 1, 6, 7, 4, 5]]).astype(f32)
    a1 = (a2 + a2[..., [1, 0, 3, 2, 5, 4, 7, 6]]).astype(f32)
    total = a1[..., 0]
    mean = (total * f32(0.0078125)).astype(f32)
    r = (f32(1.0) / np.sqrt((mean + f32(eps)).astype(f32))).astype(f32)
    y = (x * r[..., None]).astype(f32)
    if weight is not None:
        y = (y * np.asarray(weight, dtype=f32)[None, None, :]).astype(f32)
    if rope is not None:
        rope = np.asarray(rope, dtype=f32)
        a = y[:, :, :64]
        b = y[:, :, 64:]
        m00 = rope[:, None, :, 0, 0]
        m01 = rope[:, None, :, 0, 1]
        m10 = rope[:, None, :, 1, 0]
        m11 = rope[:, None, :, 1, 1]
        ya = ((m00 * a).astype(f32) + (m01 * b).astype(f32)).astype(f32)
        yb = ((m10 * a).astype(f32) + (m11 * b).astype(f32)).astype(f32)
        y = np.concatenate([ya, yb], axis=-1)
    return bf16_round(y)


def qknorm_rope_pack(q, k, v, rope, qw, kw, eps, world: int) -> np.ndarray:
    """The fused pack: q, k, v [S_l, H, 128] -> send buffer [world, 3, H/world, S_l, 128]
    (rank r receives heads [r*Hl, (r+1)*Hl) of every tensor)."""
    S, H, _ = q.shape
    hl = H // world
    qn = qknorm_rope(q, qw, rope, eps)
    kn = qknorm_rope(k, kw, rope, eps)
    out = np.empty((world, 3, hl, S, D), dtype=np.float32)
    for t, src in enumerate((qn, kn, np.asarray(v, dtype=np.float32))):
        out[:, t] = src.transpose(1, 0, 2).reshape(world, hl, S, D)
    return out


# ----------------------------------------------------------------------------- attention
def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None,
              s_kv: int | None = None) -> np.ndarray:
    """q: [H, Sq, 128], k/v: [H, Skv, 128] -> [H, Sq, 128] float64 (keys >= s_kv ignored)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    if s_kv is not None:
        k = k[:, :s_kv]
        v = v[:, :s_kv]
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    out = np.empty(q.shape, dtype=np.float64)
    for h in range(q.shape[0]):
        for a in range(0, q.shape[1], 1024):
            s = (q[h, a:a + 1024] @ k[h].T) * scale
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            out[h, a:a + 1024] = (p @ v[h]) / p.sum(axis=1, keepdims=True)
    return out


# ----------------------------------------------------------------------------- Ulysses layouts
def a2a_seq_to_head(xs: list[np.ndarray]) -> list[np.ndarray]:
    """Per-rank inputs [1, H, Sl, d] -> per-rank outputs [1, Hl, W*Sl, d]
    (harness/sp_runtime.py:67-71: rank r receives heads [r*Hl, (r+1)*Hl) of every rank's
    tokens, concatenated in rank order)."""
    W = len(xs)
    _, H, Sl, d = xs[0].shape
    hl = H // W
    return [np.concatenate([xs[src][:, r * hl:(r + 1) * hl] for src in range(W)], axis=2) for r in range(W)]


def a2a_head_to_seq(xs: list[np.ndarray]) -> list[np.ndarray]:
    """Per-rank inputs [1, Hl, S, d] -> per-rank outputs [1, H, S/W, d]
    (harness/sp_runtime.py:73-77)."""
    W = len(xs)
    _, hl, S, d = xs[0].shape
    sl = S // W
    return [np.concatenate([xs[src][:, :, r * sl:(r + 1) * sl] for src in range(W)], axis=1) for r in range(W)]


def seq_to_head_unpack(recv: np.ndarray, world: int) -> np.ndarray:
    """recv [W(src), T, Hl, Sl, d] -> [T, Hl, W*Sl, d]."""
    W, T, hl, sl, d = recv.shape
    return recv.transpose(1, 2, 0, 3, 4).reshape(T, hl, W * sl, d)


def head_to_seq_unpack(recv: np.ndarray) -> np.ndarray:
    """[H, Sl, d] -> [Sl, H*d]."""
    H, sl, d = recv.shape
    return recv.transpose(1, 0, 2).reshape(sl, H * d)


# ----------------------------------------------------------------------------- pad / shard
def pad_len(s: int, world: int) -> int:
    """S_pad = ceil(S / W) * W (harness/sp_runtime.py:229)."""
    return ((s + world - 1) // world) * world


def shard_segments(segs, lo: int, hi: int):
    """Re-base (a, b, row) segments into the shard [lo, hi) (sp_runtime.py:196-201)."""
    out = []
    for a, b, row in segs:
        A, B = max(a, lo), min(b, hi)
        if A < B:
            out.append((A - lo, B - lo, row))
    return out


def piece_bounds(n: int, p: int):
    """Split n rows into p near-equal pieces, the longer ones first (sp_runtime.py:136-144)."""
    base, rem = divmod(n, p)
    out, s = [], 0
    for i in range(p):
        ln = base + (1 if i < rem else 0)
        if ln == 0:
            continue
        out.append((s, s + ln))
        s += ln
    return out


def pad_shard(h: np.ndarray, rope: np.ndarray | None, segs, world: int, rank: int):
    """Zero-pad h [S, hidden] (and rope along dim 1) to S_pad, take rank's row shard
    (sp_runtime.py:229-239). Returns (h_loc, rope_loc, segs_loc, S_pad)."""
    S = h.shape[0]
    sp = pad_len(S, world)
    P = sp - S
    if P:
        h = np.concatenate([h, np.zeros((P, h.shape[1]), h.dtype)], 0)
        if rope is not None:
            rope = np.concatenate([rope, np.zeros((rope.shape[0], P) + rope.shape[2:], rope.dtype)], 1)
    sl = sp // world
    lo, hi = rank * sl, (rank + 1) * sl
    return h[lo:hi], (rope[:, lo:hi] if rope is not None else None), shard_segments(segs, lo, hi), sp


# ----------------------------------------------------------------------------- seeded inputs
def make_qkv(seed: int, h: int, s: int, d: int = D, dtype=np.float32):
    """Config-0 style raw inputs: Q, K, V ~ N(0, 1) as [S, H, d], rounded to bf16 values."""
    rng = np.random.default_rng(seed)
    return tuple(bf16_round(rng.standard_normal((s, h, d), dtype=np.float32)) for _ in range(3))


def flops(s_q: int, s_kv: int, heads: int, d: int = D) -> float:
    """Attention FLOPs 4 * S_q * S_kv * d * H (two GEMMs)."""
    return 4.0 * s_q * s_kv * d * heads
