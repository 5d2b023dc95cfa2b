"""Pin the CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py ran harness/sp_runtime.py and its SDPA call)."""
import glob
import json
import os

import numpy as np
import pytest
import torch

from oracle import h3_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_bf16_round_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(10000, dtype=np.float32) * 10 ** rng.uniform(-30, 30, 10000).astype(np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf, 3.3895314e38, 1e-40, -1e-42], np.float32)])
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    got = O.bf16_round(x)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert np.isnan(O.bf16_round(np.array([np.nan], np.float32))).all()


def test_attention_oracle_matches_reference_sdpa():
    g = np.load(os.path.join(GOLD, "sdpa.npz"))
    names = sorted({k.rsplit("_", 1)[0] for k in g.files})
    assert len(names) == 8
    for n in names:
        q, k, v = (O.from_bf16_bits(g[f"{n}_{t}"]) for t in "qkv")
        ref = g[f"{n}_o"]
        s_kv = 301 if n.startswith("pad") else None
        got = O.attention(q, k, v, s_kv=s_kv)
        assert np.abs(got - ref).max() < 2e-5, n


def test_a2a_layout_restatement_matches_reference():
    for W in (2, 4):
        files = [os.path.join(GOLD, f"a2a_W{W}.npz")] + [os.path.join(GOLD, f"a2a_W{W}_r{r}.npz") for r in range(1, W)]
        data = [np.load(f) for f in files]
        xs = list(data[0]["x"])
        ys = O.a2a_seq_to_head(xs)
        zs = O.a2a_head_to_seq(ys)
        for r in range(W):
            assert np.array_equal(ys[r], data[r]["y"])
            assert np.array_equal(zs[r], data[r]["z"])
            assert np.array_equal(zs[r], xs[r])  # round trip


def test_unpack_layouts_compose_to_reference_a2a():
    """send layout [W,T,Hl,Sl,d] exchanged then unpacked == reference a2a_seq_to_head."""
    W, H, Sl = 4, 8, 5
    data = [np.load(os.path.join(GOLD, f"a2a_W{W}.npz" if r == 0 else f"a2a_W{W}_r{r}.npz")) for r in range(W)]
    xs = list(data[0]["x"])  # [W][1, H, Sl, d]
    hl = H // W
    for r in range(W):
        recv = np.stack([xs[src][0].reshape(W, 1, hl, Sl, 128)[r] for src in range(W)])  # [W, 1, Hl, Sl, d]
        assert np.array_equal(O.seq_to_head_unpack(recv, W)[0], data[r]["y"][0])


def test_host_helpers_match_reference():
    with open(os.path.join(GOLD, "host.json")) as f:
        g = json.load(f)
    for c in g["shard_segments"]:
        assert [list(t) for t in O.shard_segments([tuple(s) for s in c["segs"]], c["lo"], c["hi"])] == c["out"]
    for c in g["piece_bounds"]:
        assert [list(t) for t in O.piece_bounds(c["n"], c["p"])] == c["out"]


def test_pad_shard_restatement():
    h = np.arange(67 * 3, dtype=np.float32).reshape(67, 3)
    rope = O.rope_table(67)
    for W in (1, 2, 4, 8):
        parts = [O.pad_shard(h, rope, [(0, 67, 0)], W, r) for r in range(W)]
        sp = parts[0][3]
        assert sp == O.pad_len(67, W) and sp % W == 0 and sp - 67 < W
        cat = np.concatenate([p[0] for p in parts])
        assert np.array_equal(cat[:67], h) and not cat[67:].any()
        rcat = np.concatenate([p[1] for p in parts], 1)
        assert np.array_equal(rcat[:, :67], rope) and not rcat[:, 67:].any()


def test_rope_table_is_rotation():
    r = O.rope_table(100).astype(np.float64)[0]
    det = r[..., 0, 0] * r[..., 1, 1] - r[..., 0, 1] * r[..., 1, 0]
    assert np.allclose(det, 1, atol=1e-6)
    assert np.array_equal(r[0], np.tile(np.eye(2), (64, 1, 1)))


def test_qknorm_rope_properties():
    """Size-independent properties of the restatement: unit RMS after the norm (rotation
    preserves pair norms), weight scaling, and the no-rope path equals plain RMSNorm."""
    q, _, _ = O.make_qkv(3, 4, 50)
    y0 = O.qknorm_rope(q, None, None, 1e-6)
    assert np.allclose(np.sqrt((y0.astype(np.float64) ** 2).mean(-1)), 1, atol=4e-3)
    y1 = O.qknorm_rope(q, None, O.rope_table(50)[0], 1e-6)
    assert np.allclose((y1.astype(np.float64) ** 2).mean(-1), 1, atol=1e-2)
    ref = q / np.sqrt((q.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6)
    assert np.abs(y0 - ref).max() < 2 ** -7 * np.abs(ref).max()
