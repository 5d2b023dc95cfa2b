"""Parity of the sm_100a kernels against the CPU oracle (and fp32 torch for the tile KATs).

Tolerances (north star): attention within max-abs 2e-2 and mean-abs 2e-3 of an fp32/fp64
ground truth; pack/unpack kernels bit-exact; KATs within fp32 summation-order noise.
"""
import numpy as np
import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


def _inputs(seed, H, S, dev):
    """Config-0 style: raw N(0,1) -> qk-RMSNorm + RoPE (oracle) for q, k; v raw. [H, S, 128]."""
    q, k, v = O.make_qkv(seed, H, S)
    rope = O.rope_table(S)[0]
    qn = O.qknorm_rope(q, None, rope, 1e-6)
    kn = O.qknorm_rope(k, None, rope, 1e-6)
    to = lambda a: a.transpose(1, 0, 2).copy()
    return to(qn), to(kn), to(v)


def test_library_loads():
    import h3attn
    assert h3attn.lib().h3_version() == 1


def test_tile_kat_qk(cuda_dev):
    import h3attn
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    s = h3attn.tile_kat_qk(q.to(cuda_dev), k.to(cuda_dev))
    h3attn.check_status()
    ref = q.double() @ k.double().T
    err = (s.cpu().double() - ref).abs()
    assert err.max().item() < 1e-3, err.max().item()


def test_tile_kat_pv(cuda_dev):
    import h3attn
    g = torch.Generator(device="cpu").manual_seed(1)
    p = torch.rand(128, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    o = h3attn.tile_kat_pv(p.to(cuda_dev), v.to(cuda_dev))
    h3attn.check_status()
    ref = p.double() @ v.double()
    err = (o.cpu().double() - ref).abs()
    assert err.max().item() < 1e-3, err.max().item()


def test_tile_kat_pair_qk(cuda_dev):
    import h3attn
    g = torch.Generator(device="cpu").manual_seed(2)
    q = torch.randn(256, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    s = h3attn.tile_kat_pair_qk(q.to(cuda_dev), k.to(cuda_dev))
    h3attn.check_status()
    err = (s.cpu().double() - q.double() @ k.double().T).abs()
    assert err.max().item() < 1e-3, err.max().item()


def test_tile_kat_pair_pv(cuda_dev):
    import h3attn
    g = torch.Generator(device="cpu").manual_seed(3)
    p = torch.rand(256, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    o = h3attn.tile_kat_pair_pv(p.to(cuda_dev), v.to(cuda_dev))
    h3attn.check_status()
    err = (o.cpu().double() - p.double() @ v.double()).abs()
    assert err.max().item() < 1e-3, err.max().item()


@pytest.mark.parametrize("H,S", [(2, 1), (2, 15), (2, 127), (2, 128), (2, 129), (2, 255), (2, 256), (3, 300),
                                 (2, 1000), (1, 4095)])
def test_attention_vs_oracle(cuda_dev, H, S):
    import h3attn
    q, k, v = _inputs(S * 7 + H, H, S, cuda_dev)
    o = h3attn.attention(_bf16(q, cuda_dev), _bf16(k, cuda_dev), _bf16(v, cuda_dev))
    h3attn.check_status()
    ref = O.attention(q, k, v)
    err = np.abs(o.float().cpu().numpy() - ref)
    assert err.max() < MAX_ABS and err.mean() < MEAN_ABS, (err.max(), err.mean())


def test_attention_pad_path(cuda_dev):
    """Queries over S_pad rows, keys/values stopped at the real length (sp_runtime.py:106-109)."""
    import h3attn
    H, S_real, S_pad = 2, 301, 304
    q, k, v = _inputs(11, H, S_pad, cuda_dev)
    o = h3attn.attention(_bf16(q, cuda_dev), _bf16(k, cuda_dev), _bf16(v, cuda_dev), s_kv=S_real)
    h3attn.check_status()
    ref = O.attention(q, k, v, s_kv=S_real)
    err = np.abs(o.float().cpu().numpy() - ref)
    assert err.max() < MAX_ABS and err.mean() < MEAN_ABS, (err.max(), err.mean())


def test_attention_layouts_bit_exact(cuda_dev):
    import h3attn
    H, S, W = 4, 512, 2
    q, k, v = (_bf16(a, cuda_dev) for a in _inputs(5, H, S, cuda_dev))
    o_head = h3attn.attention(q, k, v, layout="head")
    o_tok = h3attn.attention(q, k, v, layout="token")
    o_send = h3attn.attention(q, k, v, layout="send", world=W)
    torch.cuda.synchronize()
    assert torch.equal(o_tok.view(S, H, 128).transpose(0, 1), o_head)
    assert torch.equal(o_send.permute(1, 0, 2, 3).reshape(H, S, 128), o_head)


def test_attention_subsets_bit_exact(cuda_dev):
    """A row's result depends only on that row and K/V: head and row subsets match bitwise."""
    import h3attn
    H, S = 4, 700
    q, k, v = (_bf16(a, cuda_dev) for a in _inputs(9, H, S, cuda_dev))
    full = h3attn.attention(q, k, v)
    sub_h = h3attn.attention(q[1:3], k[1:3], v[1:3])
    sub_r = h3attn.attention(q[:, 37:500], k, v)
    torch.cuda.synchronize()
    assert torch.equal(sub_h, full[1:3])
    assert torch.equal(sub_r, full[:, 37:500])


@pytest.mark.parametrize("world", [1, 2, 4])
def test_pack_bit_exact(cuda_dev, world):
    import h3attn
    S, H = 67, 8
    rng = np.random.default_rng(world)
    qkv = O.bf16_round(rng.standard_normal((S, 3, H, 128), dtype=np.float32) * 3)
    qw = O.bf16_round(1 + 0.1 * rng.standard_normal(128, dtype=np.float32))
    kw = O.bf16_round(1 + 0.1 * rng.standard_normal(128, dtype=np.float32))
    rope = O.rope_table(S, pos0=5)[0]
    x = _bf16(qkv.reshape(S, 3 * H * 128), cuda_dev)
    q, k, v = x.split(H * 128, dim=-1)
    out = h3attn.qknorm_rope_pack(q, k, v, torch.from_numpy(rope).to(cuda_dev), _bf16(qw, cuda_dev),
                                  _bf16(kw, cuda_dev), 1e-6, world)
    torch.cuda.synchronize()
    ref = O.qknorm_rope_pack(qkv[:, 0], qkv[:, 1], qkv[:, 2], rope, qw, kw, 1e-6, world)
    got = out.float().cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("S,H,world,head_major", [
    (1, 3, 1, False),        # one token, q/k rows fewer than one step of the lane groups
    (16, 8, 2, False),
    (2369, 12, 2, False),    # 2 * 12 q/k rows: a partial last step of the row walk
    (5003, 56, 8, True),     # the H3 head count, head-major layout, several grid-stride passes
    (4099, 56, 4, False),
])
def test_pack_strided_inputs_bit_exact(cuda_dev, S, H, world, head_major):
    """Padded input rows and rope rows, head counts that leave partial steps of the kernel's row walk,
    token counts beyond one grid-stride pass and the head-major layout all give the oracle's bits."""
    import h3attn
    rng = np.random.default_rng(S + H)
    qkv = O.bf16_round(rng.standard_normal((S, 3, H, 128), dtype=np.float32) * 2)
    qw = O.bf16_round(1 + 0.1 * rng.standard_normal(128, dtype=np.float32))
    kw = O.bf16_round(1 + 0.1 * rng.standard_normal(128, dtype=np.float32))
    rope = O.rope_table(S, pos0=11)[0]
    # rows padded past the three column blocks, rope rows padded past 256 floats
    x = torch.zeros((S, 3 * H * 128 + 64), dtype=torch.bfloat16, device=cuda_dev)
    x[:, :3 * H * 128] = _bf16(qkv.reshape(S, 3 * H * 128), cuda_dev)
    q, k, v = x[:, :H * 128], x[:, H * 128:2 * H * 128], x[:, 2 * H * 128:3 * H * 128]
    rope_pad = torch.zeros((S, 320), dtype=torch.float32, device=cuda_dev)
    rope_pad[:, :256] = torch.from_numpy(rope.reshape(S, 256)).to(cuda_dev)
    out = h3attn.qknorm_rope_pack(q, k, v, rope_pad[:, :256].view(S, 64, 2, 2), _bf16(qw, cuda_dev),
                                  _bf16(kw, cuda_dev), 1e-6, world, head_major=head_major)
    torch.cuda.synchronize()
    h3attn.check_status()
    if head_major:  # [hl, world, 3, S, D] -> [world, 3, hl, S, D]
        out = out.permute(1, 2, 0, 3, 4)
    ref = O.qknorm_rope_pack(qkv[:, 0], qkv[:, 1], qkv[:, 2], rope, qw, kw, 1e-6, world)
    got = out.float().cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_pack_no_rope_no_weight(cuda_dev):
    import h3attn
    S, H = 33, 4
    rng = np.random.default_rng(3)
    qkv = O.bf16_round(rng.standard_normal((S, 3, H, 128), dtype=np.float32))
    x = _bf16(qkv.reshape(S, 3 * H * 128), cuda_dev)
    q, k, v = x.split(H * 128, dim=-1)
    out = h3attn.qknorm_rope_pack(q, k, v, None, None, None, 1e-5, 1)
    torch.cuda.synchronize()
    ref = O.qknorm_rope_pack(qkv[:, 0], qkv[:, 1], qkv[:, 2], None, None, None, 1e-5, 1)
    assert np.array_equal(out.float().cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_unpack_kernels_bit_exact(cuda_dev):
    import h3attn
    W, T, hl, sl = 4, 3, 2, 45
    rng = np.random.default_rng(4)
    recv = O.bf16_round(rng.standard_normal((W, T, hl, sl, 128), dtype=np.float32))
    out = h3attn.seq_to_head_unpack(_bf16(recv, cuda_dev))
    o2 = h3attn.head_to_seq_unpack(_bf16(recv[:, 0].reshape(W * hl, sl, 128), cuda_dev))
    torch.cuda.synchronize()
    assert np.array_equal(out.float().cpu().numpy(), O.seq_to_head_unpack(recv, W))
    assert np.array_equal(o2.float().cpu().numpy(), O.head_to_seq_unpack(recv[:, 0].reshape(W * hl, sl, 128)))


def test_bad_arguments_rejected(cuda_dev):
    import h3attn
    q = torch.zeros(2, 128, 128, dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(h3attn.H3Error):
        h3attn.attention(q.float(), q, q)
    with pytest.raises(h3attn.H3Error):
        h3attn.attention(q, q, q, s_kv=0)
    with pytest.raises(h3attn.H3Error):
        h3attn.attention(q.cpu(), q, q)
    with pytest.raises(h3attn.H3Error):
        h3attn.attention(q, q, q, layout="send", world=3)


# schedule variant -> (FMA-pipe exp2 pair positions in a 32-key chunk, chunks using them). Variants
# with the same placement run the same arithmetic (1-SM or SM-pair MMAs, another P hand-off) and
# are bit-identical.
VARIANT_EMU = {0: (0, 0), 1: (0, 0), 2: (0, 0), 3: (0, 0), 4: (0x5555, 6), 5: (0x1111, 7), 6: (0x4444, 6),
               7: (0, 0), 8: (0x5555, 6)}


@pytest.mark.parametrize("variant", sorted(VARIANT_EMU))
def test_attention_variants_vs_oracle(cuda_dev, variant):
    """Every kernel schedule meets the tolerance; schedules that only change the MMA form or the
    P hand-off are bit-identical to the first variant with the same exp2 placement."""
    import h3attn
    H, S_real, S_pad = 2, 1001, 1004
    q, k, v = _inputs(21, H, S_pad, cuda_dev)
    qd, kd, vd = (_bf16(a, cuda_dev) for a in (q, k, v))
    o = h3attn.attention(qd, kd, vd, s_kv=S_real, variant=variant)
    h3attn.check_status()
    ref = O.attention(q, k, v, s_kv=S_real)
    err = np.abs(o.float().cpu().numpy() - ref)
    assert err.max() < MAX_ABS and err.mean() < MEAN_ABS, (err.max(), err.mean())
    first = min(w for w, e in VARIANT_EMU.items() if e == VARIANT_EMU[variant])
    if first != variant:  # same arithmetic in another schedule
        assert torch.equal(o, h3attn.attention(qd, kd, vd, s_kv=S_real, variant=first))
    # every variant keeps rows independent of each other: a row subset is bit-identical
    sub = h3attn.attention(qd[:, 129:700], kd, vd, s_kv=S_real, variant=variant)
    torch.cuda.synchronize()
    assert torch.equal(sub, o[:, 129:700])


def test_removed_variants_rejected(cuda_dev):
    import h3attn
    q = torch.zeros(1, 128, 128, dtype=torch.bfloat16, device=cuda_dev)
    for variant in (9, 13, 20, 99, -1):
        with pytest.raises(h3attn.H3Error):
            h3attn.attention(q, q, q, variant=variant)
