"""AdaLN modulation / gated-residual kernels against the host model's own torch ops on the GPU.

The gated residual is pure bf16 elementwise arithmetic in the host's rounding order, so it must
match bit for bit. The modulation also depends on the LayerNorm statistics, whose fp32 summation
order differs from torch's; results may differ by one bf16 rounding step in rare elements
(|diff| <= 2^-7 |ref| + 2^-9, at most 1 % of elements). Rows are independent: a row subset
reproduces the same bits. Tokens outside every segment are normalised but not modulated."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _setup(dev, rows=777, hidden=5376, mod_rows=3, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(rows, hidden, generator=g) * 2 + 0.5).to(torch.bfloat16).to(dev)
    y = torch.randn(rows, hidden, generator=g).to(torch.bfloat16).to(dev)
    mods = (torch.randn(mod_rows, 6 * hidden, generator=g) * 0.3).to(torch.bfloat16).to(dev)
    segs = [(0, 100, 0), (100, 500, 1), (450, rows - 20, 2)]  # overlapping: the later segment wins
    return x, y, mods.chunk(6, dim=-1), segs


def _close(out, ref, shift_tok=None):
    """One bf16 step of the LayerNorm value survives the modulation in absolute terms, so the bound
    scales with the magnitude before the shift is added (|ref - shift|) as well as with |ref|."""
    d = (out.float() - ref.float()).abs()
    mag = ref.float().abs()
    if shift_tok is not None:
        mag = torch.maximum(mag, (ref.float() - shift_tok.float()).abs())
    bad = d > 2 ** -7 * mag + 2 ** -9
    assert not bool(bad.any()), d.max().item()
    assert (out != ref).float().mean().item() < 0.01


def test_norm_modulate_matches_host(cuda_dev):
    import h3attn
    import h3_model as M
    x, y, (shift, scale, gate, _, _, _), segs = _setup(cuda_dev)
    seg = h3attn.segment_rows(segs, x.shape[0], cuda_dev)
    out = h3attn.norm_modulate(x, shift, scale, seg, 1e-6)
    ref = M._mod_scale_shift(F.layer_norm(x, (x.shape[1],), eps=1e-6), shift, scale, segs)
    torch.cuda.synchronize()
    _close(out, ref, M._mod_scale_shift(torch.zeros_like(x), shift, scale, segs))
    # tail rows (outside every segment): plain LayerNorm
    _close(out[-20:], F.layer_norm(x[-20:], (x.shape[1],), eps=1e-6))


def test_norm_modulate_with_residual_matches_host(cuda_dev):
    import h3attn
    import h3_model as M
    x, y, (shift, scale, gate, _, _, _), segs = _setup(cuda_dev, seed=1)
    seg = h3attn.segment_rows(segs, x.shape[0], cuda_dev)
    x1 = torch.empty_like(x)
    out = h3attn.norm_modulate(x, shift, scale, seg, 1e-6, y=y, gate=gate, x_out=x1)
    x1_ref = M._mod_gate(x, gate, y, segs)
    ref = M._mod_scale_shift(F.layer_norm(x1_ref, (x.shape[1],), eps=1e-6), shift, scale, segs)
    torch.cuda.synchronize()
    assert torch.equal(x1, x1_ref)
    _close(out, ref, M._mod_scale_shift(torch.zeros_like(x), shift, scale, segs))


def test_gated_residual_bit_exact(cuda_dev):
    import h3attn
    import h3_model as M
    x, y, (_, _, gate, _, _, _), segs = _setup(cuda_dev, rows=1001, seed=2)
    seg = h3attn.segment_rows(segs, x.shape[0], cuda_dev)
    out = h3attn.gated_residual(x, y, gate, seg)
    torch.cuda.synchronize()
    assert torch.equal(out, M._mod_gate(x, gate, y, segs))


def test_rows_independent(cuda_dev):
    import h3attn
    x, y, (shift, scale, gate, _, _, _), segs = _setup(cuda_dev, seed=3)
    seg = h3attn.segment_rows(segs, x.shape[0], cuda_dev)
    full = h3attn.norm_modulate(x, shift, scale, seg, 1e-6, y=y, gate=gate)
    part = h3attn.norm_modulate(x[300:700].contiguous(), shift, scale, seg[300:700].contiguous(), 1e-6,
                                y=y[300:700].contiguous(), gate=gate)
    torch.cuda.synchronize()
    assert torch.equal(part, full[300:700])


def test_many_rows_and_in_place(cuda_dev):
    """Thousands of rows per call give the same bits as row subsets, and x_out / h may be x itself
    (a row is read completely before any of it is written)."""
    import h3attn
    import h3_model as M
    x, y, (shift, scale, gate, _, _, _), segs = _setup(cuda_dev, rows=9001, seed=5)
    seg = h3attn.segment_rows(segs, x.shape[0], cuda_dev)
    x1 = torch.empty_like(x)
    out = h3attn.norm_modulate(x, shift, scale, seg, 1e-6, y=y, gate=gate, x_out=x1)
    part = h3attn.norm_modulate(x[4000:4100].contiguous(), shift, scale, seg[4000:4100].contiguous(), 1e-6,
                                y=y[4000:4100].contiguous(), gate=gate)
    xi = x.clone()
    h_in = h3attn.norm_modulate(xi, shift, scale, seg, 1e-6, y=y, gate=gate, x_out=xi)  # residual in place
    xh = x.clone()
    h3attn.norm_modulate(xh, shift, scale, seg, 1e-6, out=xh)                           # h over x
    plain = h3attn.norm_modulate(x, shift, scale, seg, 1e-6)
    torch.cuda.synchronize()
    h3attn.check_status()
    assert torch.equal(x1, M._mod_gate(x, gate, y, segs))
    assert torch.equal(part, out[4000:4100])
    assert torch.equal(xi, x1) and torch.equal(h_in, out)
    assert torch.equal(xh, plain)


@pytest.mark.parametrize("hidden", [8, 1000, 1024, 8192])
def test_widths(cuda_dev, hidden):
    import h3attn
    import h3_model as M
    x, y, (shift, scale, gate, _, _, _), _ = _setup(cuda_dev, rows=64, hidden=hidden, seed=4)
    segs = [(0, 64, 1)]
    seg = h3attn.segment_rows(segs, 64, cuda_dev)
    out = h3attn.norm_modulate(x, shift, scale, seg, 1e-6)
    ref = M._mod_scale_shift(F.layer_norm(x, (hidden,), eps=1e-6), shift, scale, segs)
    torch.cuda.synchronize()
    _close(out, ref, M._mod_scale_shift(torch.zeros_like(x), shift, scale, segs))


def test_bad_arguments(cuda_dev):
    import h3attn
    x, y, (shift, scale, gate, _, _, _), segs = _setup(cuda_dev, rows=16, hidden=64)
    seg = h3attn.segment_rows(segs, 16, cuda_dev)
    with pytest.raises(h3attn.H3Error):
        h3attn.norm_modulate(x, shift, scale, seg.long(), 1e-6)      # seg dtype
    with pytest.raises(h3attn.H3Error):
        h3attn.norm_modulate(x[:, :60], shift[:, :60], scale[:, :60], seg, 1e-6)  # width not a multiple of 8
    with pytest.raises(h3attn.H3Error):
        h3attn.gated_residual(x, y[:8], gate, seg)                    # rows mismatch
