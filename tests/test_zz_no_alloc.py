"""h3_attn_layer_noalloc: the single-GPU attention layer for callers that cannot allocate device
memory (C or FFI code inside an application whose caching allocator owns the GPU's memory). It
keeps its intermediate and status word in the library's static device array instead of asking the
caller for a workspace.

Called through the C ABI (ctypes) twice in a row with different shapes, and compared with the
existing entry points (h3_qknorm_rope_pack into a caller-allocated buffer, then h3_attn_fwd)
within the attention tolerance used everywhere in these tests; the same kernels run on the same
inputs, so the rows also match exactly. The first call's output is also checked against the CPU
oracle (pack restatement + float64 attention). A call larger than the static array, a qkv row
stride too small to hold q, k and v, and a head count beyond the attention grid are rejected
before anything is enqueued. This file is named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
H3_ERR_SHAPE, H3_ERR_STRIDE, H3_ERR_SCRATCH_LIMIT = -3, -4, -10


def _lib():
    import h3attn
    L = h3attn.lib()
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    L.h3_attn_layer_noalloc.argtypes = [vp, i64, vp, i64, vp, vp, ctypes.c_float, vp, i64, i64, ctypes.c_float, vp]
    L.h3_attn_layer_noalloc.restype = ctypes.c_int
    return L


def _case(dev, seed, S, H, with_weights):
    rng = np.random.default_rng(seed)
    qkv = torch.from_numpy(O.bf16_round(rng.standard_normal((S, 3 * H * 128), dtype=np.float32))).to(dev)
    qkv = qkv.to(torch.bfloat16)
    rope = torch.from_numpy(O.rope_table(S)[0]).to(dev)
    if with_weights:
        qw = torch.from_numpy(O.bf16_round(1 + 0.1 * rng.standard_normal(128, dtype=np.float32))).to(dev).to(torch.bfloat16)
        kw = torch.from_numpy(O.bf16_round(1 + 0.1 * rng.standard_normal(128, dtype=np.float32))).to(dev).to(torch.bfloat16)
    else:
        qw = kw = None
    return qkv, rope, qw, kw


def _existing(qkv, rope, qw, kw, H):
    import h3attn
    q, k, v = qkv.split(H * 128, dim=-1)
    send = h3attn.qknorm_rope_pack(q, k, v, rope, qw, kw, 1e-6, 1)
    return h3attn.attention(send[0, 0], send[0, 1], send[0, 2], layout="token")


def test_noalloc_layer_matches_existing_entry_points(cuda_dev):
    L = _lib()
    for seed, S, H, w in [(1, 700, 8, True), (2, 301, 4, False)]:  # two calls in a row, different shapes
        qkv, rope, qw, kw = _case(cuda_dev, seed, S, H, w)
        out = torch.empty((S, H * 128), dtype=torch.bfloat16, device=cuda_dev)
        rc = L.h3_attn_layer_noalloc(qkv.data_ptr(), qkv.stride(0), rope.data_ptr(), rope.stride(0),
                                     qw.data_ptr() if qw is not None else None,
                                     kw.data_ptr() if kw is not None else None, ctypes.c_float(1e-6),
                                     out.data_ptr(), S, H, ctypes.c_float(128 ** -0.5),
                                     torch.cuda.current_stream().cuda_stream)
        assert rc == 0, rc
        ref = _existing(qkv, rope, qw, kw, H)
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert err.max().item() < MAX_ABS and err.mean().item() < MEAN_ABS
        assert torch.equal(out, ref)
        if seed == 1:  # and against the CPU oracle on the same inputs
            x = qkv.float().cpu().numpy().reshape(S, 3, H, 128)
            wq = qw.float().cpu().numpy() if qw is not None else None
            wk = kw.float().cpu().numpy() if kw is not None else None
            send = O.qknorm_rope_pack(x[:, 0], x[:, 1], x[:, 2], rope.cpu().numpy(), wq, wk, 1e-6, 1)
            oref = O.attention(send[0, 0], send[0, 1], send[0, 2])  # [H, S, 128]
            got = out.float().cpu().numpy().reshape(S, H, 128).transpose(1, 0, 2)
            e = np.abs(got - oref)
            assert e.max() < MAX_ABS and e.mean() < MEAN_ABS, (e.max(), e.mean())


def test_noalloc_layer_rejects_sizes_beyond_its_scratch(cuda_dev):
    L = _lib()
    S, H = 1561, 56  # 3 * 1561 * 56 * 128 * 2 bytes > 64 MiB
    qkv = torch.zeros((8, 3 * H * 128), dtype=torch.bfloat16, device=cuda_dev)  # never read
    out = torch.zeros((8, H * 128), dtype=torch.bfloat16, device=cuda_dev)
    rc = L.h3_attn_layer_noalloc(qkv.data_ptr(), qkv.stride(0), None, 0, None, None, ctypes.c_float(1e-6),
                                 out.data_ptr(), S, H, ctypes.c_float(128 ** -0.5),
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == H3_ERR_SCRATCH_LIMIT


def test_noalloc_layer_rejects_bad_layouts_before_any_work(cuda_dev):
    """A row stride that cannot hold q, k and v, or more heads than the attention grid takes, is
    refused up front (nothing is enqueued, the shared array is untouched)."""
    L = _lib()
    S, H = 64, 4
    qkv = torch.zeros((S, 3 * H * 128), dtype=torch.bfloat16, device=cuda_dev)
    out = torch.zeros((S, H * 128), dtype=torch.bfloat16, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    rc = L.h3_attn_layer_noalloc(qkv.data_ptr(), H * 128, None, 0, None, None, ctypes.c_float(1e-6), out.data_ptr(),
                                 S, H, ctypes.c_float(128 ** -0.5), st)
    assert rc == H3_ERR_STRIDE
    rc = L.h3_attn_layer_noalloc(qkv.data_ptr(), 3 * 70000 * 128, None, 0, None, None, ctypes.c_float(1e-6),
                                 out.data_ptr(), 1, 70000, ctypes.c_float(128 ** -0.5), st)
    assert rc == H3_ERR_SHAPE
    torch.cuda.synchronize()
    assert bool((out == 0).all())
