"""Host-side decisions of the runtime and the binding that need no GPU: the per-token modulation
row table, when the projection GEMM and the fused modulation kernels apply (and when the host
module's own ops run instead), and the address arithmetic of the head-major and peer layouts."""
import os
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "minimaxh3-on-a100-x4_b200")
sys.path.insert(0, PKG)


def test_segment_rows_last_segment_wins_and_pads_are_unmodulated():
    import h3_model as M
    import h3attn
    rows = 40
    segs = [(0, 10, 0), (5, 20, 1), (18, 50, 2)]  # overlapping, the last reaches past the end
    seg = h3attn.segment_rows(segs, rows, "cpu")
    assert seg.dtype == torch.int32 and seg.shape == (rows,)
    # the host's per-segment assignments in order: later segments overwrite earlier ones
    x = torch.zeros(rows, 1)
    ref = M._mod_scale_shift(x, torch.arange(3, dtype=torch.float32)[:, None] + 1, torch.zeros(3, 1), segs)
    assert torch.equal(seg.float() + 1, ref[:, 0])
    seg2 = h3attn.segment_rows([(0, 10, 1)], 16, "cpu")
    assert seg2[10:].eq(-1).all() and seg2[:10].eq(1).all()


def test_gemm_weight_only_for_bias_free_bf16_linears():
    import sp_runtime
    x = torch.zeros(4, 16, dtype=torch.bfloat16)
    lin = torch.nn.Linear(16, 32, bias=False, dtype=torch.bfloat16)
    assert sp_runtime._gemm_weight(lin, x) is lin.weight
    assert sp_runtime._gemm_weight(torch.nn.Linear(16, 32, bias=True, dtype=torch.bfloat16), x) is None
    assert sp_runtime._gemm_weight(torch.nn.Linear(16, 32, bias=False), x) is None  # fp32 weight
    assert sp_runtime._gemm_weight(lin, x.float()) is None                           # fp32 activations


def test_fused_block_only_for_affine_free_layernorms_on_gpu():
    import h3_model as M
    import sp_runtime
    blk = M.DiTBlock(hidden=64, heads=1, head_dim=64, ffn=128, t_dim=16, dtype=torch.bfloat16)
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    assert not sp_runtime._fusable(blk, x)  # host tensors: the host block runs
    blk.norm1 = torch.nn.LayerNorm(64, elementwise_affine=True, dtype=torch.bfloat16)
    x_meta = torch.empty(4, 64, dtype=torch.bfloat16, device="meta")
    assert not sp_runtime._fusable(blk, x_meta)


@pytest.mark.parametrize("world,hl,sl", [(2, 3, 5), (4, 2, 7)])
def test_head_major_pack_layout_is_contiguous_per_head(world, hl, sl):
    """The strides handed to the pack kernel for head_major=True put (h, rank, tensor, row) at
    ((h*world + rank)*3 + tensor)*sl + row rows of 128: each local head's blocks for all peers form
    one contiguous all-to-all buffer send[h] of shape [world, 3, sl, 128]."""
    D = 128
    tstride, rank_stride, head_stride = sl * D, 3 * sl * D, world * 3 * sl * D
    buf = torch.empty((hl, world, 3, sl, D))
    for h in range(hl):
        for r in range(world):
            for t in range(3):
                off = t * tstride + r * rank_stride + h * head_stride
                assert off == buf[h, r, t].storage_offset()


def test_peer_layout_offsets():
    """Peer pack: head g of token t lands in rank g // hl's [3][hl][S][128] buffer at row
    rank*sl + t; peer attention: query row i lands in rank i // sl's [sl][H*128] buffer at column
    block (this rank*hl + h)."""
    W, H, sl, D = 4, 8, 6, 128
    hl, S = H // W, W * sl
    me = 2
    qkv = torch.empty((3, hl, S, D))
    for g in range(H):
        dest, h = divmod(g, hl)
        for t in range(3):
            off = t * (hl * S * D) + h * (S * D) + (me * sl + 1) * D
            assert off == qkv[t, h, me * sl + 1].storage_offset()
    o = torch.empty((sl, H * D))
    for h in range(hl):
        i = 3 * sl + 4  # query row 3*sl + 4 belongs to rank 3, local row 4
        base = me * hl * D
        off = base + h * D + (i % sl) * (H * D)
        assert off == o[i % sl, (me * hl + h) * D:].storage_offset()


def test_host_fallback_reported_once_or_refused_in_strict_mode():
    import warnings

    import sp_runtime
    sp_runtime._fallbacks_seen.clear()
    old = sp_runtime._STRICT
    try:
        sp_runtime._STRICT = False
        with warnings.catch_warnings(record=True) as w:
            warnings.simplefilter("always")
            sp_runtime._host_fallback("a projection", "the linear has a bias")
            sp_runtime._host_fallback("a projection", "the linear has a bias")
        assert len([x for x in w if "host module's ops" in str(x.message)]) == 1
        sp_runtime._STRICT = True
        with pytest.raises(RuntimeError, match="SP_STRICT"):
            sp_runtime._host_fallback("a projection", "the linear has a bias")
    finally:
        sp_runtime._STRICT = old
        sp_runtime._fallbacks_seen.clear()


@pytest.mark.parametrize("S,world", [(42000, 8), (41999, 8), (67, 4), (3, 4), (64, 1)])
def test_shard_bounds_follow_the_pad_rule(S, world):
    """S_pad = ceil(S / world) * world; rank r holds rows [r * S_pad/world, (r+1) * S_pad/world)."""
    import sp_runtime
    spans = [sp_runtime._shard_bounds(S, world, r) for r in range(world)]
    S_pad = spans[0][0]
    assert S_pad % world == 0 and S <= S_pad < S + world
    assert spans[0][1] == 0 and spans[-1][2] == S_pad
    assert all(a[2] == b[1] for a, b in zip(spans, spans[1:]))
    assert len({hi - lo for _, lo, hi in spans}) == 1


def test_timeline_books_host_spans_by_category():
    import time

    import sp_runtime
    tl = sp_runtime._Timeline(on_gpu=False)
    with tl.span("qkv"):
        time.sleep(0.01)
    with tl.span("qkv"):
        pass
    with tl.span("gather"):
        pass
    tot = tl.totals()
    assert set(tot) == {"qkv", "gather"} and tot["qkv"] >= 9.0 and tot["gather"] >= 0.0


@pytest.mark.parametrize("world,H,s", [(2, 4, 5), (4, 8, 3), (8, 56, 2)])
def test_copy_engine_exchange_geometry_reproduces_the_all_to_alls(world, H, s):
    """SP_OVERLAP=ce: every rank copies rows of its send chunks straight into each destination's
    buffers with the geometry _ce_geometry plans. Replayed on byte buffers for all ranks, the copies
    must leave each rank's attention input equal to all-to-all + seq->head unpack of the blocking
    path, and each rank's out_proj input equal to the head->seq all-to-all (oracle layouts)."""
    import numpy as np
    import sp_runtime
    from oracle import h3_oracle as O

    D, hl = 2, H // world  # a short head_dim keeps the replay small; the geometry is per element size
    rng = np.random.default_rng(world * 100 + H)
    sends = [rng.integers(0, 2 ** 16, size=(world, 3, hl, s, D), dtype=np.uint16) for _ in range(world)]
    attn_in = [np.zeros(3 * hl * world * s * D, dtype=np.uint16) for _ in range(world)]
    o_sends = [rng.integers(0, 2 ** 16, size=(world, hl, s, D), dtype=np.uint16) for _ in range(world)]
    o_in = [np.zeros(H * s * D, dtype=np.uint16) for _ in range(world)]
    for r in range(world):
        geo = sp_runtime._ce_geometry(s, H, D, world, r)
        off, pitch, width, rows = geo["qkv"]
        o_off, o_bytes = geo["o"]
        for d in range(world):
            src = sends[r][d].reshape(-1).view(np.uint8)
            dst = attn_in[d].view(np.uint8)
            for i in range(rows):
                dst[off + i * pitch:off + i * pitch + width] = src[i * width:(i + 1) * width]
            o_in[d].view(np.uint8)[o_off:o_off + o_bytes] = o_sends[r][d].reshape(-1).view(np.uint8)
    for d in range(world):
        # blocking path: rank d receives chunk d of every source rank, then unpacks to [3][hl][W*s][D]
        recv = np.stack([sends[r][d] for r in range(world)])
        assert np.array_equal(attn_in[d].reshape(3, hl, world * s, D), O.seq_to_head_unpack(recv, world))
    # head->seq: per-rank [1, hl, W*s, D] attention outputs -> per-rank [1, H, s, D]
    o_full = [np.concatenate([o_sends[r][d] for d in range(world)], axis=1)[None] for r in range(world)]
    want = O.a2a_head_to_seq(o_full)
    for d in range(world):
        assert np.array_equal(o_in[d].reshape(1, H, s, D), want[d])
