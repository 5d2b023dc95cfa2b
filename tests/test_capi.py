"""The C ABI (include/h3attn.h) on CPU: the library loads, exports every declared entry
point, and rejects bad arguments before any CUDA work. No kernel runs here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "h3attn.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*int\s+(h3_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def L():
    import h3attn
    if not os.path.exists(h3attn.LIB_PATH):
        from build import build
        build()
    return h3attn.lib()


def test_header_declares_entry_points():
    names = declared()
    for n in ("h3_attn_fwd", "h3_qknorm_rope_pack", "h3_seq_to_head_unpack", "h3_head_to_seq_unpack",
              "h3_status_read", "h3_version", "h3_tile_kat_qk", "h3_tile_kat_pv"):
        assert n in names


def test_library_exports_every_declared_symbol(L):
    for n in declared():
        assert hasattr(L, n), n


def test_version(L):
    assert L.h3_version() == 1


def test_attn_rejects_bad_arguments_before_launch(L):
    args = lambda q: [q, q, q, q, 2, 128, 128, 128 * 128, 128, 128 * 128, 128, 128, 0, 128 * 128, 128,
                      ctypes.c_float(0.088), ctypes.c_void_p(0x1000), None]
    assert L.h3_attn_fwd(*args(None)) == -1                      # NULL
    assert L.h3_attn_fwd(*args(ctypes.c_void_p(0x1008))) == -2   # not 16-byte aligned
    a = args(ctypes.c_void_p(0x1000))
    a[5] = 0                                                     # s_q = 0
    assert L.h3_attn_fwd(*a) == -3
    a = args(ctypes.c_void_p(0x1000))
    a[8] = 100                                                   # row stride not a multiple of 8
    assert L.h3_attn_fwd(*a) == -4
    a = args(ctypes.c_void_p(0x1000))
    a[15] = ctypes.c_float(-1.0)                                 # scale must be positive
    assert L.h3_attn_fwd(*a) == -3


def test_pack_rejects_bad_arguments_before_launch(L):
    p = ctypes.c_void_p(0x1000)
    ok = [p, p, p, 3 * 4 * 128, None, 0, None, None, ctypes.c_float(1e-6), p, p, p, 10, 4, 2, 4 * 10 * 128,
          10 * 128, None]
    bad = list(ok)
    bad[0] = None
    assert L.h3_qknorm_rope_pack(*bad) == -1
    bad = list(ok)
    bad[14] = 3  # heads not divisible into ranks
    assert L.h3_qknorm_rope_pack(*bad) == -3
    bad = list(ok)
    bad[3] = 4 * 128 - 8  # row stride smaller than a row
    assert L.h3_qknorm_rope_pack(*bad) == -4


def test_copy_2d_rejects_bad_arguments_before_any_copy(L):
    p = ctypes.c_void_p(0x1000)
    assert L.h3_copy_2d(None, 256, p, 256, 256, 4, None) == -1      # no destination
    assert L.h3_copy_2d(p, 128, p, 256, 256, 4, None) == -3         # destination pitch below the row width
    assert L.h3_copy_2d(p, 256, p, 256, 256, 0, None) == -3         # no rows


def test_unpack_rejects_bad_arguments_before_launch(L):
    p = ctypes.c_void_p(0x1000)
    assert L.h3_seq_to_head_unpack(None, p, 2, 2, 8, 3, 0, 0, 0, None) == -1
    assert L.h3_seq_to_head_unpack(p, p, 0, 2, 8, 3, 0, 0, 0, None) == -3
    assert L.h3_head_to_seq_unpack(p, ctypes.c_void_p(0x1004), 4, 8, None) == -2
    assert L.h3_status_read(None, None) == -1


def test_gemm_rejects_bad_arguments_before_launch(L):
    p, st = ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000)
    # a [1][300][512], w [256][512], c [300][256]
    ok = [p, 300, 1, 512, 0, 512, p, 256, 512, p, 256, 0, st, None]
    bad = list(ok)
    bad[6] = None
    assert L.h3_gemm_bf16(*bad) == -1                    # NULL weight
    bad = list(ok)
    bad[9] = ctypes.c_void_p(0x1004)
    assert L.h3_gemm_bf16(*bad) == -2                    # output not 16-byte aligned
    bad = list(ok)
    bad[7] = 100
    assert L.h3_gemm_bf16(*bad) == -3                    # n_out not a multiple of 8
    bad = list(ok)
    bad[11] = 1
    bad[7] = 192
    assert L.h3_gemm_bf16(*bad) == -3                    # swiglu width not a multiple of 128
    bad = list(ok)
    bad[2], bad[3] = 4, 96
    assert L.h3_gemm_bf16(*bad) == -3                    # chunked a needs 64-column chunks
    bad = list(ok)
    bad[8] = 256
    assert L.h3_gemm_bf16(*bad) == -4                    # weight rows shorter than k
    bad = list(ok)
    bad[10] = 128
    assert L.h3_gemm_bf16(*bad) == -4                    # output rows shorter than n_out


def test_peer_entry_points_reject_bad_arguments_before_launch(L):
    p, st = ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000)
    # pack: q, k, v [10][4*128], 2 ranks, table of 2 addresses
    ok = [p, p, p, 4 * 128, None, 0, None, None, ctypes.c_float(1e-6), p, 2, 20 * 128, 10 * 128, 0, 10, 4, 2, None]
    bad = list(ok)
    bad[9] = None
    assert L.h3_qknorm_rope_pack_peer(*bad) == -1                 # no address table
    bad = list(ok)
    bad[9] = ctypes.c_void_p(0x1004)
    assert L.h3_qknorm_rope_pack_peer(*bad) == -2                 # table not 8-byte aligned
    bad = list(ok)
    bad[16] = 3
    assert L.h3_qknorm_rope_pack_peer(*bad) == -3                 # heads not divisible into ranks
    bad = list(ok)
    bad[10] = 1
    assert L.h3_qknorm_rope_pack_peer(*bad) == -3                 # table shorter than the destination ranks
    bad = list(ok)
    bad[11] = 20 * 128 + 4
    assert L.h3_qknorm_rope_pack_peer(*bad) == -4                 # tensor stride not a multiple of 8
    # attention: [2][128][128] q/k/v, two destination ranks of 64 rows
    a = [p, p, p, p, p, 2, 2, 128, 128, 128 * 128, 128, 128 * 128, 128, 64, 128, 256, ctypes.c_float(0.088), st,
         None]
    bad = list(a)
    bad[4] = None
    assert L.h3_attn_fwd_peer(*bad) == -1                         # no address table
    bad = list(a)
    bad[4] = ctypes.c_void_p(0x1004)
    assert L.h3_attn_fwd_peer(*bad) == -2
    bad = list(a)
    bad[7] = 0
    assert L.h3_attn_fwd_peer(*bad) == -3                         # no query rows
    bad = list(a)
    bad[5] = 1
    assert L.h3_attn_fwd_peer(*bad) == -3                         # 128 rows, one table entry of 64 rows


def test_noalloc_rejects_bad_arguments_before_any_work(L):
    """Every argument of h3_attn_layer_noalloc is checked before anything is enqueued, so a
    rejected call never leaves the shared static array half-written."""
    L.h3_attn_layer_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p]
    p = ctypes.c_void_p(0x1000)
    ok = [p, 3 * 4 * 128, None, 0, None, None, ctypes.c_float(1e-6), p, 100, 4, ctypes.c_float(0.088), None]
    bad = list(ok)
    bad[0] = None
    assert L.h3_attn_layer_noalloc(*bad) == -1
    bad = list(ok)
    bad[7] = ctypes.c_void_p(0x1008)
    assert L.h3_attn_layer_noalloc(*bad) == -2                    # output not 16-byte aligned
    bad = list(ok)
    bad[1] = 4 * 128                                              # row holds q only: k, v reads would overrun
    assert L.h3_attn_layer_noalloc(*bad) == -4
    bad = list(ok)
    bad[1] = 3 * 4 * 128 - 8
    assert L.h3_attn_layer_noalloc(*bad) == -4
    bad = list(ok)
    bad[9], bad[8], bad[1] = 70000, 1, 3 * 70000 * 128
    assert L.h3_attn_layer_noalloc(*bad) == -3                    # more heads than the attention grid takes
    bad = list(ok)
    bad[8] = 1 << 60                                              # absurd length: rejected, no overflow
    assert L.h3_attn_layer_noalloc(*bad) == -3
    bad = list(ok)
    bad[10] = ctypes.c_float(0.0)
    assert L.h3_attn_layer_noalloc(*bad) == -3                    # scale must be positive
    bad = list(ok)
    bad[8], bad[9], bad[1] = 1561, 56, 3 * 56 * 128
    assert L.h3_attn_layer_noalloc(*bad) == -10                   # beyond the static scratch


def test_no_cpu_path():
    """The binding refuses host tensors instead of computing on the CPU."""
    import torch
    import h3attn
    q = torch.zeros(1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(h3attn.H3Error):
        h3attn.attention(q, q, q)
    with pytest.raises(h3attn.H3Error):
        h3attn.qknorm_rope_pack(q[0], q[0], q[0], None, None, None, 1e-6, 1)
