"""Torch-facing binding of libh3attn.so (the sm_100a kernels behind include/h3attn.h).

Every function here validates its tensors, passes raw device pointers, element strides
and the current CUDA stream through ctypes, and raises on a negative return code. There
is no CPU path: a missing library or a non-CUDA tensor is an error.

Reference counterparts:
  attention            SDPA FLASH call, harness/sp_runtime.py:119-121 (and the unwired
                       fa3(q, k, v, o) of attn_sm80/attn_sm80.py:26-31)
  qknorm_rope_pack     ck.rms_rope_split_half_ + transposes + send reshape, sp_runtime.py:93-104, :69
  seq_to_head_unpack   receive-side permute copy, sp_runtime.py:71
  head_to_seq_unpack   transpose/reshape ahead of out_proj, sp_runtime.py:125
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libh3attn.so")
D = 128

_ERRORS = {
    -1: "a required pointer is NULL",
    -2: "a pointer is not 16-byte aligned",
    -3: "a size is out of range",
    -4: "a stride is not a multiple of 8 elements or is too small",
    -5: "the CUDA runtime refused the launch",
    -6: "cuTensorMapEncodeTiled rejected the layout",
    -7: "driver entry point unavailable",
    -8: "unsupported configuration",
    -9: "a CUDA runtime call failed",
    -10: "the call needs more than the no-alloc entry point's static scratch",
    -11: "a kernel gave up waiting (bounded-wait timeout)",
}
STATUS_NAMES = {
    0: "ok", 1: "timeout waiting for Q tiles", 2: "timeout in the K/V ring", 3: "timeout waiting for S",
    4: "timeout waiting for P", 5: "timeout waiting for O", 6: "timeout draining copies", 7: "timeout in a tile KAT",
}

_lib = None
_status = {}


class H3Error(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load libh3attn.so once. Raises ImportError when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python {os.path.join(HERE, 'build.py')}`")
        L = ctypes.CDLL(LIB_PATH)
        i64, vp, f32, i32p = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p
        L.h3_version.restype = ctypes.c_int
        L.h3_attn_fwd.argtypes = [vp, vp, vp, vp] + [i64] * 11 + [f32, i32p, vp]
        L.h3_attn_fwd.restype = ctypes.c_int
        L.h3_attn_fwd_variant.argtypes = [vp, vp, vp, vp] + [i64] * 11 + [f32, i32p, ctypes.c_int32, vp]
        L.h3_attn_fwd_variant.restype = ctypes.c_int
        L.h3_qknorm_rope_pack.argtypes = [vp, vp, vp, i64, vp, i64, vp, vp, f32, vp, vp, vp, i64, i64, i64, i64,
                                          i64, vp]
        L.h3_qknorm_rope_pack.restype = ctypes.c_int
        L.h3_seq_to_head_unpack.argtypes = [vp, vp] + [i64] * 7 + [vp]
        L.h3_seq_to_head_unpack.restype = ctypes.c_int
        L.h3_head_to_seq_unpack.argtypes = [vp, vp, i64, i64, vp]
        L.h3_head_to_seq_unpack.restype = ctypes.c_int
        L.h3_tile_kat_qk.argtypes = [vp, vp, vp, i32p, vp]
        L.h3_tile_kat_qk.restype = ctypes.c_int
        L.h3_tile_kat_pv.argtypes = [vp, vp, vp, i32p, vp]
        L.h3_tile_kat_pv.restype = ctypes.c_int
        L.h3_wait_kat.argtypes = [vp, i64, i32p, vp]
        L.h3_wait_kat.restype = ctypes.c_int
        for name in ("h3_tile_kat_pair_qk", "h3_tile_kat_pair_pv"):
            getattr(L, name).argtypes = [vp, vp, vp, i32p, vp]
            getattr(L, name).restype = ctypes.c_int
        L.h3_gemm_bf16.argtypes = [vp, i64, i64, i64, i64, i64, vp, i64, i64, vp, i64, ctypes.c_int32, i32p, vp]
        L.h3_gemm_bf16.restype = ctypes.c_int
        L.h3_norm_modulate.argtypes = [vp, i64, vp, i64, vp, vp, i64, vp, vp, i64, vp, vp, i64, i64, i64,
                                       ctypes.c_float, vp]
        L.h3_norm_modulate.restype = ctypes.c_int
        L.h3_gated_residual.argtypes = [vp, i64, vp, i64, vp, i64, vp, vp, i64, i64, i64, vp]
        L.h3_gated_residual.restype = ctypes.c_int
        L.h3_qknorm_rope_pack_peer.argtypes = [vp, vp, vp, i64, vp, i64, vp, vp, ctypes.c_float, vp, i64, i64, i64,
                                               i64, i64, i64, i64, vp]
        L.h3_qknorm_rope_pack_peer.restype = ctypes.c_int
        L.h3_attn_fwd_peer.argtypes = [vp] * 5 + [i64] * 11 + [ctypes.c_float, i32p, vp]
        L.h3_attn_fwd_peer.restype = ctypes.c_int
        L.h3_copy_2d.argtypes = [vp, i64, vp, i64, i64, i64, vp]
        L.h3_copy_2d.restype = ctypes.c_int
        L.h3_status_read.argtypes = [i32p, vp]
        L.h3_status_read.restype = ctypes.c_int
        _lib = L
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise H3Error(f"{what}: {_ERRORS.get(rc, 'error')} (code {rc})")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _cuda(t: torch.Tensor, name: str, dtype=torch.bfloat16) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise H3Error(f"{name} must be a CUDA tensor (this library has no CPU path)")
    if t.dtype != dtype:
        raise H3Error(f"{name} must be {dtype}, got {t.dtype}")


def status_word(device=None) -> torch.Tensor:
    """The int32 device status word this process hands to every kernel on `device`."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
    st = _status.get(dev.index)
    if st is None:
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        _status[dev.index] = st
    return st


def check_status(device=None) -> None:
    """Synchronise and raise if a kernel on `device` reported a bounded-wait timeout."""
    st = status_word(device)
    code = lib().h3_status_read(ctypes.c_void_p(st.data_ptr()), ctypes.c_void_p(_stream()))
    if code < 0:
        _check(code, "h3_status_read")
    if code != 0:
        st.zero_()
        raise H3Error(f"device status {code}: {STATUS_NAMES.get(code, 'unknown')}")


# ----------------------------------------------------------------------------- attention
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, s_kv: int | None = None,
              scale: float | None = None, out: torch.Tensor | None = None, layout: str = "head",
              world: int = 1, variant: int | None = None) -> torch.Tensor:
    """Exact attention over heads: q [H, Sq, 128], k/v [H, Skv, 128] (bf16, last dim
    contiguous, any head/row strides that are multiples of 8). Keys/values stop at s_kv
    (default Skv). Output layout:
      "head":  [H, Sq, 128]
      "token": [Sq, H*128] (what out_proj consumes)
      "send":  [world, H, Sq/world, 128] -- the head->seq all-to-all send buffer
    """
    for n, t in (("q", q), ("k", k), ("v", v)):
        _cuda(t, n)
        if t.dim() != 3 or t.shape[-1] != D or t.stride(-1) != 1:
            raise H3Error(f"{n} must be [heads, rows, 128] with a contiguous last dim, got {tuple(t.shape)}")
    H, sq, _ = q.shape
    if k.shape[0] != H or v.shape[0] != H or k.shape[1] != v.shape[1]:
        raise H3Error("q, k, v disagree on heads or key count")
    if k.stride() != v.stride():
        raise H3Error("k and v must share strides")
    skv_alloc = k.shape[1]
    s_kv = skv_alloc if s_kv is None else int(s_kv)
    if not 1 <= s_kv <= skv_alloc:
        raise H3Error(f"s_kv={s_kv} outside [1, {skv_alloc}]")
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    if layout == "head":
        shape, rank_rows, rank_stride, head_stride, row_stride = (H, sq, D), sq, 0, sq * D, D
    elif layout == "token":
        shape, rank_rows, rank_stride, head_stride, row_stride = (sq, H * D), sq, 0, D, H * D
    elif layout == "send":
        if sq % world:
            raise H3Error(f"send layout needs rows {sq} divisible by world {world}")
        sl = sq // world
        shape, rank_rows, rank_stride, head_stride, row_stride = (world, H, sl, D), sl, H * sl * D, sl * D, D
    else:
        raise H3Error(f"unknown layout {layout!r}")
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=q.device)
    else:
        _cuda(out, "out")
        if tuple(out.shape) != tuple(shape) or not out.is_contiguous():
            raise H3Error(f"out must be contiguous {shape}, got {tuple(out.shape)}")
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), H, sq, s_kv, q.stride(0), q.stride(1),
            k.stride(0), k.stride(1), rank_rows, rank_stride, head_stride, row_stride, scale,
            status_word(q.device).data_ptr())
    if variant is None:
        rc = lib().h3_attn_fwd(*args, _stream())
    else:
        rc = lib().h3_attn_fwd_variant(*args, int(variant), _stream())
    _check(rc, "h3_attn_fwd")
    return out


# ----------------------------------------------------------------------------- fused exchanges (peer memory)
def qknorm_rope_pack_peer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rope: torch.Tensor | None,
                          q_weight: torch.Tensor | None, k_weight: torch.Tensor | None, eps: float, world: int,
                          rank_base: torch.Tensor, tensor_stride: int, head_stride: int, row_offset: int) -> None:
    """The pack with the seq->head exchange fused in: head g of each token goes straight to rank
    g // (H/world)'s buffer at rank_base[rank] (int64 device tensor [world] of addresses mapped in
    this process) + tensor*tensor_stride + local_head*head_stride + (row_offset + token)*128."""
    q2, k2, v2, sl, H, rope_ptr, rope_stride, wptr = _pack_args(q, k, v, rope, q_weight, k_weight)
    if H % world:
        raise H3Error(f"heads {H} not divisible by world {world}")
    _cuda(rank_base, "rank_base", torch.int64)
    if tuple(rank_base.shape) != (world,) or not rank_base.is_contiguous():
        raise H3Error("rank_base must be a contiguous int64 [world] device tensor")
    rc = lib().h3_qknorm_rope_pack_peer(q2.data_ptr(), k2.data_ptr(), v2.data_ptr(), q2.stride(0), rope_ptr,
                                        rope_stride, wptr[0], wptr[1], float(eps), rank_base.data_ptr(), world,
                                        tensor_stride, head_stride, row_offset, sl, H, H // world, _stream())
    _check(rc, "h3_qknorm_rope_pack_peer")


def attention_peer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o_local: torch.Tensor, o_peer: torch.Tensor,
                   rank_rows: int, head_stride: int, row_stride: int, s_kv: int | None = None,
                   scale: float | None = None) -> None:
    """Attention with the head->seq exchange fused into the epilogue: query row i of head h goes to
    o_peer[i // rank_rows] + h*head_stride + (i % rank_rows)*row_stride (elements)."""
    for n, t in (("q", q), ("k", k), ("v", v)):
        _cuda(t, n)
        if t.dim() != 3 or t.shape[-1] != D or t.stride(-1) != 1:
            raise H3Error(f"{n} must be [heads, rows, 128] with a contiguous last dim")
    _cuda(o_local, "o_local")
    _cuda(o_peer, "o_peer", torch.int64)
    H, sq, _ = q.shape
    if k.shape[0] != H or v.shape[0] != H or k.shape[1] != v.shape[1] or k.stride() != v.stride():
        raise H3Error("q, k, v disagree on heads, key count or strides")
    if o_peer.dim() != 1 or o_peer.shape[0] * rank_rows < sq or not o_peer.is_contiguous():
        raise H3Error("o_peer must hold one address per destination rank")
    s_kv = k.shape[1] if s_kv is None else int(s_kv)
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    rc = lib().h3_attn_fwd_peer(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_local.data_ptr(), o_peer.data_ptr(),
                                o_peer.shape[0], H, sq, s_kv, q.stride(0), q.stride(1), k.stride(0), k.stride(1), rank_rows, head_stride,
                                row_stride, scale, status_word(q.device).data_ptr(), _stream())
    _check(rc, "h3_attn_fwd_peer")


# ----------------------------------------------------------------------------- pack / unpack
def _pack_args(q, k, v, rope, q_weight, k_weight):
    """Checks shared by the pack entry points; returns (q2, k2, v2, tokens, heads, rope_ptr,
    rope_row_stride, [q_weight_ptr, k_weight_ptr])."""
    for n, t in (("q", q), ("k", k), ("v", v)):
        _cuda(t, n)
        if t.dim() == 3:
            t = t.reshape(t.shape[0], -1)
        if t.dim() != 2 or t.stride(-1) != 1:
            raise H3Error(f"{n} must be [tokens, heads*128] with a contiguous last dim")
    q2, k2, v2 = (t.reshape(t.shape[0], -1) if t.dim() == 3 else t for t in (q, k, v))
    sl, hd = q2.shape
    if hd % D or k2.shape != q2.shape or v2.shape != q2.shape:
        raise H3Error("q, k, v must share shape [tokens, heads*128]")
    if not (q2.stride(0) == k2.stride(0) == v2.stride(0)):
        raise H3Error("q, k, v must share a row stride")
    rope_ptr, rope_stride = None, 0
    if rope is not None:
        _cuda(rope, "rope", torch.float32)
        if rope.dim() == 5:
            if rope.shape[0] != 1:
                raise H3Error("rope batch dim must be 1")
            rope = rope[0]
        if tuple(rope.shape[1:]) != (64, 2, 2) or rope.shape[0] != sl or not rope[0].is_contiguous():
            raise H3Error(f"rope must be [tokens, 64, 2, 2] fp32 (rot_dim 128), got {tuple(rope.shape)}")
        rope_ptr, rope_stride = rope.data_ptr(), rope.stride(0)
    wptr = []
    for n, w in (("q_weight", q_weight), ("k_weight", k_weight)):
        if w is None:
            wptr.append(None)
            continue
        _cuda(w, n)
        if tuple(w.shape) != (D,) or not w.is_contiguous():
            raise H3Error(f"{n} must be contiguous [128] bf16")
        wptr.append(w.data_ptr())
    return q2, k2, v2, sl, hd // D, rope_ptr, rope_stride, wptr


def qknorm_rope_pack(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rope: torch.Tensor | None,
                     q_weight: torch.Tensor | None, k_weight: torch.Tensor | None, eps: float, world: int,
                     out: torch.Tensor | None = None, head_major: bool = False) -> torch.Tensor:
    """q, k, v: [S_l, H*128] (views of the fused QKV output are fine; rows may be strided).
    rope: fp32 [S_l, 64, 2, 2] or None. Returns the seq->head send buffer
    [world, 3, H/world, S_l, 128] with q and k RMS-normalised (+ rotated); head_major=True lays
    it out [H/world, world, 3, S_l, 128] instead, so each local head's blocks for all peers are
    one contiguous all-to-all buffer (head-by-head pipelining)."""
    q2, k2, v2, sl, H, rope_ptr, rope_stride, wptr = _pack_args(q, k, v, rope, q_weight, k_weight)
    if H % world:
        raise H3Error(f"heads {H} not divisible by world {world}")
    hl = H // world
    shape = (hl, world, 3, sl, D) if head_major else (world, 3, hl, sl, D)
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=q.device)
    elif tuple(out.shape) != shape or not out.is_contiguous():
        raise H3Error(f"out must be contiguous {shape}")
    if head_major:  # element (h, rank, tensor, row) at ((h*world + rank)*3 + tensor)*sl + row
        tstride, rank_stride, head_stride = sl * D, 3 * sl * D, world * 3 * sl * D
    else:           # element (rank, tensor, h, row) at ((rank*3 + tensor)*hl + h)*sl + row
        tstride, rank_stride, head_stride = hl * sl * D, 3 * hl * sl * D, sl * D
    base = out.data_ptr()
    rc = lib().h3_qknorm_rope_pack(q2.data_ptr(), k2.data_ptr(), v2.data_ptr(), q2.stride(0), rope_ptr, rope_stride,
                                   wptr[0], wptr[1], float(eps), base, base + 2 * tstride, base + 4 * tstride, sl, H,
                                   hl, rank_stride, head_stride, _stream())
    _check(rc, "h3_qknorm_rope_pack")
    return out


def seq_to_head_unpack(recv: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """recv [W, T, Hl, Sl, 128] (one block per source rank) -> [T, Hl, W*Sl, 128]."""
    _cuda(recv, "recv")
    if recv.dim() != 5 or recv.shape[-1] != D or not recv.is_contiguous():
        raise H3Error("recv must be contiguous [world, tensors, heads, tokens, 128]")
    W, T, hl, sl, _ = recv.shape
    if out is None:
        out = torch.empty((T, hl, W * sl, D), dtype=torch.bfloat16, device=recv.device)
    elif tuple(out.shape) != (T, hl, W * sl, D) or not out.is_contiguous():
        raise H3Error("out has the wrong shape")
    rc = lib().h3_seq_to_head_unpack(recv.data_ptr(), out.data_ptr(), W, hl, sl, T, T * hl * sl * D, hl * sl * D,
                                     hl * W * sl * D, _stream())
    _check(rc, "h3_seq_to_head_unpack")
    return out


def copy_2d(dst_ptr: int, dst_pitch: int, src_ptr: int, src_pitch: int, width: int, rows: int,
            stream: torch.cuda.Stream | None = None) -> None:
    """Copy-engine copy of `rows` rows of `width` bytes (pitches in bytes) on `stream` (default: the
    current one); either address may be a peer GPU's mapped memory. Used for the all-to-all
    exchanges of SP_OVERLAP=ce: each rank writes its chunk straight into every destination's
    attention / out_proj input."""
    st = (stream or torch.cuda.current_stream()).cuda_stream
    _check(lib().h3_copy_2d(dst_ptr, dst_pitch, src_ptr, src_pitch, width, rows, st), "h3_copy_2d")


def head_to_seq_unpack(recv: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[H, Sl, 128] head-major -> [Sl, H*128] token-major."""
    _cuda(recv, "recv")
    if recv.dim() != 3 or recv.shape[-1] != D or not recv.is_contiguous():
        raise H3Error("recv must be contiguous [heads, tokens, 128]")
    H, sl, _ = recv.shape
    if out is None:
        out = torch.empty((sl, H * D), dtype=torch.bfloat16, device=recv.device)
    elif tuple(out.shape) != (sl, H * D) or not out.is_contiguous():
        raise H3Error("out has the wrong shape")
    rc = lib().h3_head_to_seq_unpack(recv.data_ptr(), out.data_ptr(), H, sl, _stream())
    _check(rc, "h3_head_to_seq_unpack")
    return out


# ----------------------------------------------------------------------------- projection GEMM
def linear(a: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None,
           epilogue: str = "none") -> torch.Tensor:
    """Row-independent a @ weight.T (bf16, fp32 accumulate): the bits of an output row depend only
    on that row of `a`, never on how many rows the call has.
      a: [m, k] with a contiguous last dim, or head-major [H, m, 128] (read in place as [m, H*128]);
      weight: [n, k] (nn.Linear layout); epilogue "swiglu": weight = [gate; up] (2F rows) and the
      result is silu(a @ gate.T) * (a @ up.T), [m, F]."""
    _cuda(a, "a")
    _cuda(weight, "weight")
    if weight.dim() != 2 or weight.stride(-1) != 1:
        raise H3Error("weight must be [out, in] with a contiguous last dim")
    if a.dim() == 2:
        if a.stride(-1) != 1:
            raise H3Error("a must have a contiguous last dim")
        m, k = a.shape
        chunks, chunk_cols, chunk_stride, row_stride = 1, k, 0, a.stride(0)
    elif a.dim() == 3:
        if a.stride(-1) != 1:
            raise H3Error("a must have a contiguous last dim")
        chunks, m, chunk_cols = a.shape
        chunk_stride, row_stride = a.stride(0), a.stride(1)
        k = chunks * chunk_cols
    else:
        raise H3Error(f"a must be 2-D or 3-D, got {tuple(a.shape)}")
    if weight.shape[1] != k:
        raise H3Error(f"weight has {weight.shape[1]} inputs, a has {k}")
    ep = {"none": 0, "swiglu": 1}.get(epilogue)
    if ep is None:
        raise H3Error(f"unknown epilogue {epilogue!r}")
    n = weight.shape[0] // 2 if ep == 1 else weight.shape[0]
    if ep == 1 and weight.shape[0] % 2:
        raise H3Error("swiglu weight needs an even row count")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    else:
        _cuda(out, "out")
        if tuple(out.shape) != (m, n) or out.stride(-1) != 1:
            raise H3Error(f"out must be [{m}, {n}] with a contiguous last dim")
    rc = lib().h3_gemm_bf16(a.data_ptr(), m, chunks, chunk_cols, chunk_stride, row_stride, weight.data_ptr(), n,
                            weight.stride(0), out.data_ptr(), out.stride(0), ep, status_word(a.device).data_ptr(),
                            _stream())
    _check(rc, "h3_gemm_bf16")
    return out


# ----------------------------------------------------------------------------- AdaLN modulation
def segment_rows(mod_segments, rows: int, device) -> torch.Tensor:
    """int32 [rows]: the modulation row of each token ((a, b, row) segments, later ones win as in
    the host model's per-segment assignments), -1 outside every segment."""
    seg = torch.full((rows,), -1, dtype=torch.int32, device=device)
    for a, b, row in mod_segments:
        a, b = max(int(a), 0), min(int(b), rows)
        if a < b:
            seg[a:b] = int(row)
    return seg


def _rows2d(t: torch.Tensor, name: str, hidden: int) -> None:
    _cuda(t, name)
    if t.dim() != 2 or t.shape[1] != hidden or t.stride(1) != 1:
        raise H3Error(f"{name} must be [rows, {hidden}] with a contiguous last dim, got {tuple(t.shape)}")


def norm_modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, seg_row: torch.Tensor, eps: float,
                  y: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                  x_out: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """h = LN(xr) * (1 + scale[seg]) + shift[seg] with xr = x + gate[seg] * y when y is given
    (xr also written to x_out). x, y: [rows, hidden]; shift/scale/gate: [mod_rows, hidden] views
    sharing one row stride; seg_row: int32 [rows]."""
    rows, hidden = x.shape
    _rows2d(x, "x", hidden)
    for n, t in (("shift", shift), ("scale", scale)) + ((("gate", gate),) if y is not None else ()):
        _rows2d(t, n, hidden)
    if scale.stride(0) != shift.stride(0) or (y is not None and gate.stride(0) != shift.stride(0)):
        raise H3Error("shift, scale and gate must share a row stride")
    if y is not None:
        _rows2d(y, "y", hidden)
        if y.shape[0] != rows:
            raise H3Error("y and x disagree on rows")
    _cuda(seg_row, "seg_row", torch.int32)
    if seg_row.shape != (rows,) or not seg_row.is_contiguous():
        raise H3Error("seg_row must be a contiguous int32 [rows]")
    if x_out is not None:
        _rows2d(x_out, "x_out", hidden)
    if out is None:
        out = torch.empty((rows, hidden), dtype=torch.bfloat16, device=x.device)
    else:
        _rows2d(out, "out", hidden)
    rc = lib().h3_norm_modulate(x.data_ptr(), x.stride(0), y.data_ptr() if y is not None else None,
                                y.stride(0) if y is not None else 0, gate.data_ptr() if y is not None else None,
                                x_out.data_ptr() if x_out is not None else None,
                                x_out.stride(0) if x_out is not None else 0, shift.data_ptr(), scale.data_ptr(),
                                shift.stride(0), seg_row.data_ptr(), out.data_ptr(), out.stride(0), rows, hidden,
                                float(eps), _stream())
    _check(rc, "h3_norm_modulate")
    return out


def gated_residual(x: torch.Tensor, y: torch.Tensor, gate: torch.Tensor, seg_row: torch.Tensor,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """out = x + gate[seg] * y on segment tokens, x elsewhere."""
    rows, hidden = x.shape
    for n, t in (("x", x), ("y", y), ("gate", gate)):
        _rows2d(t, n, hidden)
    _cuda(seg_row, "seg_row", torch.int32)
    if y.shape[0] != rows or seg_row.shape != (rows,) or not seg_row.is_contiguous():
        raise H3Error("x, y and seg_row disagree on rows")
    if out is None:
        out = torch.empty((rows, hidden), dtype=torch.bfloat16, device=x.device)
    else:
        _rows2d(out, "out", hidden)
    rc = lib().h3_gated_residual(x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), gate.data_ptr(), gate.stride(0),
                                 seg_row.data_ptr(), out.data_ptr(), out.stride(0), rows, hidden, _stream())
    _check(rc, "h3_gated_residual")
    return out


# ----------------------------------------------------------------------------- tile KATs
def tile_kat_qk(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    _cuda(q, "q")
    _cuda(k, "k")
    assert q.shape == (128, 128) and k.shape == (128, 128) and q.is_contiguous() and k.is_contiguous()
    s = torch.empty((128, 128), dtype=torch.float32, device=q.device)
    _check(lib().h3_tile_kat_qk(q.data_ptr(), k.data_ptr(), s.data_ptr(), status_word(q.device).data_ptr(),
                                _stream()), "h3_tile_kat_qk")
    return s


def tile_kat_pv(p: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    _cuda(p, "p")
    _cuda(v, "v")
    assert p.shape == (128, 128) and v.shape == (128, 128) and p.is_contiguous() and v.is_contiguous()
    o = torch.empty((128, 128), dtype=torch.float32, device=p.device)
    _check(lib().h3_tile_kat_pv(p.data_ptr(), v.data_ptr(), o.data_ptr(), status_word(p.device).data_ptr(),
                                _stream()), "h3_tile_kat_pv")
    return o


def tile_kat_pair_qk(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """S[256][128] = q[256][128] . k[128][128]^T through an SM pair (cta_group::2)."""
    _cuda(q, "q")
    _cuda(k, "k")
    assert q.shape == (256, 128) and k.shape == (128, 128) and q.is_contiguous() and k.is_contiguous()
    s = torch.empty((256, 128), dtype=torch.float32, device=q.device)
    _check(lib().h3_tile_kat_pair_qk(q.data_ptr(), k.data_ptr(), s.data_ptr(), status_word(q.device).data_ptr(),
                                     _stream()), "h3_tile_kat_pair_qk")
    return s


def tile_kat_pair_pv(p: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """O[256][128] = p[256][128] . v[128][128] through an SM pair (cta_group::2)."""
    _cuda(p, "p")
    _cuda(v, "v")
    assert p.shape == (256, 128) and v.shape == (128, 128) and p.is_contiguous() and v.is_contiguous()
    o = torch.empty((256, 128), dtype=torch.float32, device=p.device)
    _check(lib().h3_tile_kat_pair_pv(p.data_ptr(), v.data_ptr(), o.data_ptr(), status_word(p.device).data_ptr(),
                                     _stream()), "h3_tile_kat_pair_pv")
    return o


def wait_kat(tile: torch.Tensor, limit_ns: int) -> None:
    """Launch the bounded-wait KAT: one CTA loads `tile` [128, 128] bf16 by TMA, then waits up to
    limit_ns on a barrier nothing completes, reports H3_STATUS_TIMEOUT_KAT in the status word and
    returns. Read the outcome with check_status() (which raises on it)."""
    _cuda(tile, "tile")
    if tuple(tile.shape) != (128, 128) or not tile.is_contiguous():
        raise H3Error("tile must be a contiguous [128, 128] bf16 tensor")
    _check(lib().h3_wait_kat(tile.data_ptr(), int(limit_ns), status_word(tile.device).data_ptr(), _stream()),
           "h3_wait_kat")
