"""Stand-in for ComfyUI's `comfy.ldm.minimax.model` (MiniMax-H3 DiT), which the reference
patches but does not contain. It has the classes, attributes and call signatures that
harness/sp_runtime.py relies on, and the behaviour-identical `run_blocks` seam of
patches/model_run_blocks_seam.md:13-34, so `sp_runtime.install(module)` patches it exactly
as it patches ComfyUI:

  MiniMaxH3Model.run_blocks(h, t_emb, mod_segments, rope_freqs, transformer_options={})
  DiTBlock.forward(x, t_emb, mod_segments, rope_freqs, transformer_options={})
  Attention.forward(x, rope_freqs=None, transformer_options={})   (.qkv_proj .q_norm .k_norm
                                                                   .out_proj .heads .head_dim)
  _mod_scale_shift(x, shift, scale, mod_segments), _mod_gate(x, gate, y, mod_segments)

The block structure follows the timed replica at sp_runtime.py:203-218 (adaln -> norm1 +
modulation -> attention -> gated residual -> norm2 + modulation -> SwiGLU MLP -> gated
residual). Everything here is plain PyTorch: it is the host model, not this library's
product. Weights are random (the H3 checkpoint is not available), ~N(0, 0.02).

mod_segments is a list of (a, b, row): tokens [a, b) use modulation row `row`; tokens
outside every segment (the pad tail of the SP runtime) are left unmodulated and get no
residual update.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

HIDDEN = 5376
HEADS = 56
HEAD_DIM = 128
FFN = 14336
N_BLOCKS = 50
T_DIM = 256


class RMSNorm(nn.Module):
    """Per-head RMSNorm holder (weight + eps), computed in fp32."""

    def __init__(self, dim, eps=1e-6, dtype=None, device=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype, device=device))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()
        return y.to(x.dtype)


def rope_freqs_1d(s: int, theta: float = 10000.0, pos0: int = 0, rot_dim: int = HEAD_DIM,
                  device=None) -> torch.Tensor:
    """[1, s, rot_dim/2, 2, 2] fp32 rotation matrices [[cos, -sin], [sin, cos]] for positions
    pos0..pos0+s-1, angle = pos * theta^(-2i/rot_dim), computed in fp64."""
    half = rot_dim // 2
    inv = theta ** (-torch.arange(half, dtype=torch.float64) * 2.0 / rot_dim)
    ang = torch.arange(pos0, pos0 + s, dtype=torch.float64)[:, None] * inv[None, :]
    c, sn = torch.cos(ang), torch.sin(ang)
    m = torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2)  # [s, half, 2, 2]
    return m[None].to(torch.float32).to(device)


def rms_rope_ref(x: torch.Tensor, w: torch.Tensor | None, rope: torch.Tensor | None, eps: float) -> torch.Tensor:
    """Host-model qk-RMSNorm + RoPE on [S, H, 128] (fp32 math, split-half pairs (i, i+64))."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if w is not None:
        y = y * w.float()
    if rope is not None:
        r = rope[0] if rope.dim() == 5 else rope  # [S, 64, 2, 2]
        half = r.shape[1]
        a, b = y[..., :half], y[..., half:2 * half]
        m = r[:, None].float()
        ya = m[..., 0, 0] * a + m[..., 0, 1] * b
        yb = m[..., 1, 0] * a + m[..., 1, 1] * b
        y = torch.cat([ya, yb, y[..., 2 * half:]], -1)
    return y.to(x.dtype)


class Attention(nn.Module):
    def __init__(self, hidden=HIDDEN, heads=HEADS, head_dim=HEAD_DIM, dtype=None, device=None):
        super().__init__()
        self.heads, self.head_dim = heads, head_dim
        self.qkv_proj = nn.Linear(hidden, 3 * heads * head_dim, bias=False, dtype=dtype, device=device)
        self.q_norm = RMSNorm(head_dim, eps=1e-6, dtype=dtype, device=device)
        self.k_norm = RMSNorm(head_dim, eps=1e-6, dtype=dtype, device=device)
        self.out_proj = nn.Linear(heads * head_dim, hidden, bias=False, dtype=dtype, device=device)

    def forward(self, x, rope_freqs=None, transformer_options={}):
        s = x.shape[0]
        q, k, v = self.qkv_proj(x).split(self.heads * self.head_dim, dim=-1)
        q = rms_rope_ref(q.reshape(s, self.heads, self.head_dim), self.q_norm.weight, rope_freqs, self.q_norm.eps)
        k = rms_rope_ref(k.reshape(s, self.heads, self.head_dim), self.k_norm.weight, rope_freqs, self.q_norm.eps)
        v = v.reshape(s, self.heads, self.head_dim)
        o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None])
        return self.out_proj(o[0].transpose(0, 1).reshape(s, self.heads * self.head_dim))


class MLP(nn.Module):
    """SwiGLU: fc1 -> (a, b) -> silu(a) * b -> fc2."""

    def __init__(self, hidden=HIDDEN, ffn=FFN, dtype=None, device=None):
        super().__init__()
        self.fc1 = nn.Linear(hidden, 2 * ffn, bias=False, dtype=dtype, device=device)
        self.fc2 = nn.Linear(ffn, hidden, bias=False, dtype=dtype, device=device)

    def forward(self, x):
        a, b = self.fc1(x).chunk(2, dim=-1)
        return self.fc2(F.silu(a) * b)


class AdalnProj(nn.Module):
    """t_emb [rows, t_dim] -> six modulation tensors [rows, hidden]."""

    def __init__(self, hidden=HIDDEN, t_dim=T_DIM, dtype=None, device=None):
        super().__init__()
        self.lin = nn.Linear(t_dim, 6 * hidden, bias=True, dtype=dtype, device=device)

    def forward(self, t_emb):
        return self.lin(F.silu(t_emb)).chunk(6, dim=-1)


def _mod_scale_shift(x, shift, scale, mod_segments):
    out = x.clone()
    for a, b, row in mod_segments:
        out[a:b] = x[a:b] * (1 + scale[row]) + shift[row]
    return out


def _mod_gate(x, gate, y, mod_segments):
    out = x.clone()
    for a, b, row in mod_segments:
        out[a:b] = x[a:b] + gate[row] * y[a:b]
    return out


class DiTBlock(nn.Module):
    def __init__(self, hidden=HIDDEN, heads=HEADS, head_dim=HEAD_DIM, ffn=FFN, t_dim=T_DIM, dtype=None, device=None):
        super().__init__()
        kw = dict(dtype=dtype, device=device)
        self.adaln_proj = AdalnProj(hidden, t_dim, **kw)
        self.norm1 = nn.LayerNorm(hidden, eps=1e-6, elementwise_affine=False, **kw)
        self.attn = Attention(hidden, heads, head_dim, **kw)
        self.norm2 = nn.LayerNorm(hidden, eps=1e-6, elementwise_affine=False, **kw)
        self.mlp = MLP(hidden, ffn, **kw)

    def forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options={}):
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.adaln_proj(t_emb)
        h = _mod_scale_shift(self.norm1(x), shift_msa, scale_msa, mod_segments)
        a = self.attn(h, rope_freqs=rope_freqs, transformer_options=transformer_options)
        x = _mod_gate(x, gate_msa, a, mod_segments)
        h = _mod_scale_shift(self.norm2(x), shift_mlp, scale_mlp, mod_segments)
        return _mod_gate(x, gate_mlp, self.mlp(h), mod_segments)


class MiniMaxH3Model(nn.Module):
    def __init__(self, n_blocks=N_BLOCKS, hidden=HIDDEN, heads=HEADS, head_dim=HEAD_DIM, ffn=FFN, t_dim=T_DIM,
                 dtype=None, device=None):
        super().__init__()
        self.blocks = nn.ModuleList(DiTBlock(hidden, heads, head_dim, ffn, t_dim, dtype=dtype, device=device)
                                    for _ in range(n_blocks))

    def run_blocks(self, h, t_emb, mod_segments, rope_freqs, transformer_options={}):
        # The seam: the default single-GPU block loop (patches/model_run_blocks_seam.md:13-34).
        for block in self.blocks:
            h = block(h, t_emb, mod_segments, rope_freqs, transformer_options=transformer_options)
        return h


def timestep_embedding(t: torch.Tensor, dim: int = T_DIM, max_period: float = 10000.0) -> torch.Tensor:
    """Sinusoidal embedding of timesteps t [rows] -> [rows, dim] (cos half, then sin half)."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32) / half).to(t.device)
    args = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def init_weights(model: nn.Module, seed: int, std: float = 0.02) -> None:
    """Random init ~N(0, std) for every Linear weight (bias zero); norms keep unit weight."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, nn.Linear):
                w = torch.empty(m.weight.shape, dtype=torch.float32).normal_(0.0, std, generator=g)
                m.weight.copy_(w.to(m.weight.dtype))
                if m.bias is not None:
                    m.bias.zero_()


H3_SEGMENTS = ((0, 512, 0), (512, 1536, 1), (1536, 3000, 2), (3000, 42000, 3))  # text | cond | audio | video
