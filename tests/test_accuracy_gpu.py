"""The north star's accuracy clause at the configs it names, through the library's attention.

  config 1  B=1, H=56, D=128, S=42000 (328 full 128-key tiles and a 16-key tail), seed 1:
            h3_attn_fwd on the bf16-rounded inputs against an fp32 ground truth computed on
            the GPU (torch fp32 math by head, TF32 off), plus 64 sampled query rows of every
            head against float64 on the CPU. The reference's own GPU call (torch SDPA, FLASH
            backend, sp_runtime.py:119-121) runs on the same bf16 inputs and is held to the
            same bar beside it.
  config 0  B=1, H=56, D=128, S=4096, seed 0: h3_attn_fwd against the reference's SDPA FLASH
            call in fp32 on the CPU (oracle/sdpa_ref.py).
  fixtures  the inputs of tests/golden/sdpa.npz (produced by running the reference's SDPA call)
            fed straight to the kernel and compared with the reference's stored outputs.

Bar: max-abs <= 2e-2 and mean-abs <= 2e-3 (north star), rel_mean < 5e-3 (the reference's own
check, attn_sm80/bench_attn.py:26-33). The measured errors are printed (pytest -s)."""
import os

import numpy as np
import pytest
import torch

from oracle import h3_oracle as O
from oracle import north_star as NS

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _report(name, e):
    print(f"[accuracy] {name}: max_abs={e['max_abs']:.3e} mean_abs={e['mean_abs']:.3e} rel_mean={e['rel_mean']:.3e}")


@pytest.fixture(scope="module")
def config1(cuda_dev):
    H, S = 56, 42000
    q, k, v = NS.config_inputs(1, H, S, cuda_dev)
    qb, kb, vb = (t.to(torch.bfloat16) for t in (q, k, v))
    truth = NS.fp32_attention(q, k, v)
    return q, k, v, qb, kb, vb, truth


def test_config1_against_fp32_ground_truth(cuda_dev, config1):
    import h3attn
    q, k, v, qb, kb, vb, truth = config1
    o = h3attn.attention(qb, kb, vb, layout="head")
    h3attn.check_status()
    e = NS.errors(o, truth)
    _report("config 1, h3_attn_fwd vs fp32", e)
    assert NS.within(e), e
    assert bool(torch.isfinite(o).all())


def test_config1_sampled_rows_against_float64(cuda_dev, config1):
    """64 query rows of every head (the 16 rows of the tail tile among them) in float64 on the CPU,
    also checking the GPU fp32 ground truth itself."""
    import h3attn
    q, k, v, qb, kb, vb, truth = config1
    o = h3attn.attention(qb, kb, vb, layout="head")
    h3attn.check_status()
    S = q.shape[1]
    rng = np.random.default_rng(1)
    worst_kernel, worst_truth = 0.0, 0.0
    errs = []
    for h in range(q.shape[0]):
        rows = np.concatenate([np.arange(S - 16, S), rng.choice(S - 16, 48, replace=False)])
        qf, kf, vf = (t[h].float().cpu().numpy() for t in (qb, kb, vb))
        ref = NS.f64_rows(qf, kf, vf, rows)
        got = o[h, torch.from_numpy(rows).to(o.device)].float().cpu().numpy()
        err = np.abs(got - ref)
        errs.append(err)
        worst_kernel = max(worst_kernel, float(err.max()))
        # the fp32 truth was computed from the unrounded inputs: compare it on its own inputs
        ref_unrounded = NS.f64_rows(q[h].cpu().numpy(), k[h].cpu().numpy(), v[h].cpu().numpy(), rows)
        tr = truth[h, torch.from_numpy(rows).to(truth.device)].cpu().numpy()
        worst_truth = max(worst_truth, float(np.abs(tr - ref_unrounded).max()))
    allerr = np.concatenate(errs)
    print(f"[accuracy] config 1 sampled rows vs float64: kernel max {worst_kernel:.3e} mean {allerr.mean():.3e}; "
          f"fp32 ground truth max {worst_truth:.3e}")
    assert worst_kernel <= NS.MAX_ABS and allerr.mean() <= NS.MEAN_ABS
    assert worst_truth < 1e-4  # the fp32 ground truth itself is accurate to fp32 summation noise


def test_config1_reference_gpu_call_same_bar(cuda_dev, config1):
    """The reference's own attention call on the same bf16 inputs, against the same truth: the
    library's kernel must be at least as close (within a small margin)."""
    import h3attn
    from torch.nn.attention import SDPBackend, sdpa_kernel
    q, k, v, qb, kb, vb, truth = config1
    try:
        with sdpa_kernel([SDPBackend.FLASH_ATTENTION]):
            ref = torch.nn.functional.scaled_dot_product_attention(qb[None], kb[None], vb[None])[0]
    except RuntimeError as exc:  # the backend may not support this GPU
        pytest.skip(f"torch SDPA FLASH unavailable: {exc}")
    o = h3attn.attention(qb, kb, vb, layout="head")
    h3attn.check_status()
    e_ref, e_ours = NS.errors(ref, truth), NS.errors(o, truth)
    _report("config 1, torch SDPA FLASH (reference call) vs fp32", e_ref)
    _report("config 1, h3_attn_fwd vs fp32", e_ours)
    assert e_ours["mean_abs"] <= 1.25 * e_ref["mean_abs"] + 1e-6


def test_config0_against_reference_sdpa_on_cpu(cuda_dev):
    import h3attn
    from oracle import sdpa_ref
    H, S = 56, 4096
    q, k, v = NS.config_inputs(0, H, S, "cpu")
    torch.set_num_threads(os.cpu_count() or 1)
    ref = sdpa_ref.attention(q[None], k[None], v[None])[0]  # the reference's call, fp32, CPU
    qb, kb, vb = (t.to(torch.bfloat16).to(cuda_dev) for t in (q, k, v))
    o = h3attn.attention(qb, kb, vb, layout="head")
    h3attn.check_status()
    e = NS.errors(o.cpu(), ref)
    _report("config 0, h3_attn_fwd vs reference SDPA (CPU fp32)", e)
    assert NS.within(e), e


def _golden_cases():
    z = np.load(os.path.join(GOLDEN, "sdpa.npz"))
    return sorted({f[:-2] for f in z.files})


@pytest.mark.parametrize("case", _golden_cases())
def test_reference_sdpa_fixtures_through_the_kernel(cuda_dev, case):
    """Inputs the reference's SDPA call consumed when the fixtures were made, straight into the
    kernel; compared with the reference's stored fp32 outputs (the pad case keeps keys to 301)."""
    import h3attn
    z = np.load(os.path.join(GOLDEN, "sdpa.npz"))
    q, k, v = (O.from_bf16_bits(z[f"{case}_{t}"]) for t in "qkv")
    ref = z[f"{case}_o"]
    s_kv = int(case.split("kv")[1]) if "kv" in case else k.shape[1]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_dev).to(torch.bfloat16)
    o = h3attn.attention(dev(q), dev(k), dev(v), s_kv=s_kv, layout="head")
    h3attn.check_status()
    got = o.float().cpu().numpy()
    assert got.shape == ref.shape
    err = np.abs(got - ref)
    assert err.max() <= NS.MAX_ABS and err.mean() <= NS.MEAN_ABS, (case, err.max(), err.mean())
