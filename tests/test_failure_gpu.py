"""Device-side failure detection, exercised without faulting or hanging the GPU.

Every wait in the library's kernels is bounded: when one runs out, the kernel records a code in
the caller's status word, winds down (drains its copies, frees its tensor memory) and returns.
  * h3_wait_kat waits, with a 1 ms limit, on an mbarrier that nothing ever completes: the call
    must come back with H3_STATUS_TIMEOUT_KAT in the status word, and the device must then run
    a normal attention launch correctly.
  * A status word set non-zero by the host (a failure reported earlier) makes an attention grid
    stop before any work: no output row is written.
  * The installed runtime reads the status word at the end of run_blocks and raises instead of
    returning activations computed by kernels that gave up.
"""
import time

import numpy as np
import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu

H3_STATUS_TIMEOUT_KAT = 7


def _small_attention_case(dev, seed=5, H=2, S=300):
    q, k, v = O.make_qkv(seed, H, S)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a.transpose(1, 0, 2))).to(dev).to(torch.bfloat16)
    qd, kd, vd = to(q), to(k), to(v)
    ref = O.attention(qd.float().cpu().numpy(), kd.float().cpu().numpy(), vd.float().cpu().numpy())
    return qd, kd, vd, ref


def test_bounded_wait_runs_out_and_device_stays_usable(cuda_dev):
    import h3attn
    st = h3attn.status_word(cuda_dev)
    st.zero_()
    tile = torch.randn(128, 128, device=cuda_dev).to(torch.bfloat16)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    h3attn.wait_kat(tile, limit_ns=1_000_000)
    code = h3attn.lib().h3_status_read(st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    elapsed = time.perf_counter() - t0
    assert code == H3_STATUS_TIMEOUT_KAT, code
    assert elapsed < 2.0, elapsed  # the 1 ms limit, not the 2 s default, ended the wait
    with pytest.raises(h3attn.H3Error, match="tile KAT"):
        h3attn.check_status()  # raises and clears the word
    assert int(st.item()) == 0
    # the same device still computes correctly
    qd, kd, vd, ref = _small_attention_case(cuda_dev)
    o = h3attn.attention(qd, kd, vd)
    h3attn.check_status()
    err = np.abs(o.float().cpu().numpy() - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3


def test_preset_status_stops_attention_before_any_write(cuda_dev):
    import h3attn
    qd, kd, vd, ref = _small_attention_case(cuda_dev, seed=6)
    st = h3attn.status_word(cuda_dev)
    canary = torch.full((2, 300, 128), 3.0, dtype=torch.bfloat16, device=cuda_dev)
    st.fill_(5)  # an earlier kernel's failure, injected by the host
    h3attn.attention(qd, kd, vd, out=canary)
    code = h3attn.lib().h3_status_read(st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert code == 5
    assert bool((canary == 3.0).all())  # the grid wrote nothing
    st.zero_()
    h3attn.attention(qd, kd, vd, out=canary)
    h3attn.check_status()
    err = np.abs(canary.float().cpu().numpy() - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3


def test_runtime_raises_on_a_reported_failure(cuda_dev):
    import h3attn
    import h3_model as M
    import sp_runtime
    model = M.MiniMaxH3Model(2, 1024, 8, 128, 2048, 256, dtype=torch.bfloat16, device=cuda_dev)
    M.init_weights(model, 3, std=0.02)
    S = 300
    h = torch.randn(S, 1024, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(cuda_dev)
    t_emb = M.timestep_embedding(torch.tensor([500.0]), 256).to(torch.bfloat16).to(cuda_dev)
    segs = [(0, S, 0)]
    rope = M.rope_freqs_1d(S, device=cuda_dev)
    sp_runtime.init()
    sp_runtime.install(M)
    try:
        st = h3attn.status_word(cuda_dev)
        with torch.no_grad():
            good = model.run_blocks(h, t_emb, segs, rope, {})  # clean run: no error
            st.fill_(2)  # a K/V ring timeout reported by an earlier launch
            with pytest.raises(h3attn.H3Error, match="K/V ring"):
                model.run_blocks(h, t_emb, segs, rope, {})
            assert int(st.item()) == 0  # the runtime cleared the word when it raised
            again = model.run_blocks(h, t_emb, segs, rope, {})
        assert torch.equal(good, again)
    finally:
        sp_runtime.uninstall()
