"""The row-independent projection GEMM (h3_gemm_bf16) on the GPU.

Tolerance: against an fp32 torch product of the same bf16 inputs, rounded once to bf16, the
result may differ by fp32 summation-order noise plus one bf16 rounding step:
|c - ref| <= 2^-7 * |ref| + 1e-2 * sqrt(k / 1024) * rms(ref). Bit-exact properties: an output row
does not change with the row count or the row's position (the basis of W-way exactness), and the
head-major A read equals the same matrix laid out row-major."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(shape, seed, dev, std=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(torch.bfloat16).to(dev)


def _check_close(c, ref, k, rel=2 ** -7):
    ref = ref.float()
    err = (c.float() - ref).abs()
    rms = ref.pow(2).mean().sqrt().item()
    bound = rel * ref.abs() + 1e-2 * math.sqrt(k / 1024) * rms
    bad = (err > bound).sum().item()
    assert bad == 0, (bad, err.max().item(), rms)


@pytest.mark.parametrize("m,k,n", [(1, 64, 256), (100, 200, 264), (256, 1024, 512), (257, 576, 256),
                                   (700, 5376, 768), (3000, 128, 8)])
def test_gemm_vs_fp32(cuda_dev, m, k, n):
    import h3attn
    a = _rand((m, k), 1, cuda_dev)
    w = _rand((n, k), 2, cuda_dev, 0.02)
    c = h3attn.linear(a, w)
    torch.cuda.synchronize()
    h3attn.check_status()
    _check_close(c, a.float() @ w.float().T, k)


def test_gemm_rows_independent_of_call_shape(cuda_dev):
    import h3attn
    m, k, n = 1200, 1088, 512
    a = _rand((m, k), 3, cuda_dev)
    w = _rand((n, k), 4, cuda_dev, 0.02)
    full = h3attn.linear(a, w)
    for lo, hi in [(1, 1200), (100, 357), (129, 130), (256, 1200), (600, 1100)]:
        part = h3attn.linear(a[lo:hi].contiguous(), w)
        torch.cuda.synchronize()
        assert torch.equal(part, full[lo:hi]), (lo, hi)
    h3attn.check_status()


def test_gemm_head_major_a_equals_row_major(cuda_dev):
    """out_proj reads the head->seq receive buffer [H, s, 128] in place."""
    import h3attn
    H, s, n = 12, 333, 256
    a_heads = _rand((H, s, 128), 5, cuda_dev)
    w = _rand((n, H * 128), 6, cuda_dev, 0.02)
    a_rows = a_heads.transpose(0, 1).reshape(s, H * 128).contiguous()
    c_heads = h3attn.linear(a_heads, w)
    c_rows = h3attn.linear(a_rows, w)
    torch.cuda.synchronize()
    h3attn.check_status()
    assert torch.equal(c_heads, c_rows)
    _check_close(c_heads, a_rows.float() @ w.float().T, H * 128)


def test_gemm_strided_output_and_input(cuda_dev):
    import h3attn
    m, k, n = 300, 256, 256
    big = _rand((m, k + 64), 7, cuda_dev)
    a = big[:, 32:32 + k]  # row stride k + 64, 64-byte offset
    w = _rand((n, k), 8, cuda_dev, 0.02)
    out = torch.full((m, n + 16), 3.0, dtype=torch.bfloat16, device=cuda_dev)
    c = h3attn.linear(a, w, out=out[:, :n])
    torch.cuda.synchronize()
    assert torch.equal(c, h3attn.linear(a.contiguous(), w))
    assert bool((out[:, n:] == 3.0).all())


@pytest.mark.parametrize("m,k,f", [(1, 64, 128), (300, 640, 384), (513, 1024, 256)])
def test_gemm_swiglu_epilogue(cuda_dev, m, k, f):
    """silu(a @ gate.T) * (a @ up.T) with the host model's roundings; gate/up rows are the two
    halves of the fc1 weight (MLP.forward: fc1(x).chunk(2))."""
    import h3attn
    a = _rand((m, k), 9, cuda_dev)
    w = _rand((2 * f, k), 10, cuda_dev, 0.05)
    c = h3attn.linear(a, w, epilogue="swiglu")
    plain = h3attn.linear(a, w)  # [m, 2f]: the same rounded gate / up values
    torch.cuda.synchronize()
    h3attn.check_status()
    g, u = plain.float().chunk(2, dim=-1)
    s = (g * torch.sigmoid(g)).to(torch.bfloat16).float()
    ref = (s * u).to(torch.bfloat16)
    err = (c.float() - ref.float()).abs()
    assert (err <= 2 ** -7 * ref.float().abs() + 1e-6).all(), err.max().item()
    # against the unrounded fp32 model: three bf16 roundings (g, silu(g), product), the first
    # amplified up to ~4x by silu's relative slope at negative g
    af = a.float() @ w.float().T
    gf, uf = af.chunk(2, dim=-1)
    _check_close(c, torch.nn.functional.silu(gf) * uf, k, rel=2 ** -5)


def test_gemm_bad_arguments(cuda_dev):
    import h3attn
    a = _rand((64, 128), 11, cuda_dev)
    w = _rand((256, 128), 12, cuda_dev)
    with pytest.raises(h3attn.H3Error):
        h3attn.linear(a, w[:, :64])            # k mismatch
    with pytest.raises(h3attn.H3Error):
        h3attn.linear(a.float(), w)            # dtype
    with pytest.raises(h3attn.H3Error):
        h3attn.linear(a, w[:100])              # n not a multiple of 8
    with pytest.raises(h3attn.H3Error):
        h3attn.linear(a, w[:192], epilogue="swiglu")  # F = 96 not a multiple of 128
    with pytest.raises(h3attn.H3Error):
        h3attn.linear(a[:, 1:121], w[:, :120])  # misaligned base
