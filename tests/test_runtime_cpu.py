"""Host logic of the drop-in runtime on CPU gloo ranks (world size 2 and 4).

The runtime's kernel binding is swapped for oracle/cpu_ops (same signatures; the
reference's SDPA call for attention), so everything else -- pad, shard, segment
re-basing, the fused send layout, both all-to-alls, the unpacks, the all-gather and
the unpad -- is the product code. Outputs must equal, bit for bit, what the reference's
own harness/sp_runtime.py produced on the same inputs (tests/golden/seam_*.npz).
"""
import os
import socket
import sys
import tempfile
import time

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "minimaxh3-on-a100-x4_b200")
GOLD = os.path.join(HERE, "golden")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_env(rank, world, port):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      SP_BACKEND="gloo")
    for p in (os.path.join(HERE, "stub_comfy"), PKG, ROOT, HERE):
        if p not in sys.path:
            sys.path.insert(0, p)


def _seam_worker(rank, world, port, out_dir, cases, overlap, timing=False):
    _setup_env(rank, world, port)
    if overlap:
        os.environ["SP_OVERLAP"] = "1"
    if timing:
        os.environ["SP_TIMING"] = "1"
    import sp_runtime
    from oracle import cpu_ops
    from golden.make_golden import seam_setup
    import comfy.ldm.minimax.model as MM
    sp_runtime._ops = cpu_ops
    sp_runtime.init(timeout_s=60)
    sp_runtime.install()
    res, timing = {}, {}
    for S in cases:
        model, h, t_emb, segs, rope = seam_setup(S)
        with torch.no_grad():
            res[S] = MM.MiniMaxH3Model.run_blocks(model, h.clone(), t_emb, segs, rope, {}).numpy()
        timing[S] = sp_runtime.get_timing()
    # the reference API a2a helpers
    H, Sl = 8, 5
    g = torch.Generator().manual_seed(7)
    xs = [torch.randn(1, H, Sl, 128, generator=g) for _ in range(world)]
    y = sp_runtime.a2a_seq_to_head(xs[rank].clone(), world)
    z = sp_runtime.a2a_head_to_seq(y.clone(), world, H)
    sp_runtime.uninstall()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), y=y.numpy(), z=z.numpy(),
             **{f"seam_{S}": v for S, v in res.items()},
             **{f"timing_{S}": np.array(sorted(t.items()), dtype=object) for S, t in timing.items()})
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _run(world, cases, overlap=False, timing=False):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_seam_worker, args=(world, _free_port(), d, cases, overlap, timing), nprocs=world,
                           start_method="spawn")
        return [dict(np.load(os.path.join(d, f"r{r}.npz"), allow_pickle=True)) for r in range(world)]


def test_sp_timing_reports_the_reference_categories():
    """SP_TIMING=1: get_timing() after run_blocks holds exactly the categories that
    harness/sp_full_step.py:66 reads, each a non-negative ms figure, and the output is unchanged."""
    outs = _run(2, [67], timing=True)
    ref = np.load(os.path.join(GOLD, "seam_W2_S67.npz"))["out"]
    keys = {"norm_mod", "qkv", "a2a_fwd", "fa2_local", "a2a_inv", "out_proj", "residual", "ffn", "gather"}
    for r in range(2):
        t = dict(outs[r]["timing_67"])
        assert set(t) == keys, sorted(t)
        assert all(float(v) >= 0.0 for v in t.values())
        assert np.array_equal(outs[r]["seam_67"], ref)


@pytest.mark.parametrize("world", [2, 4])
def test_seam_bit_exact_vs_reference_runtime(world):
    outs = _run(world, [67, 64])
    for S in (67, 64):
        ref = np.load(os.path.join(GOLD, f"seam_W{world}_S{S}.npz"))["out"]
        for r in range(world):
            got = outs[r][f"seam_{S}"]
            assert got.shape == ref.shape == (S, 96)
            assert np.array_equal(got, ref), (world, S, r, np.abs(got - ref).max())


@pytest.mark.parametrize("world", [2, 4])
def test_a2a_api_matches_reference(world):
    outs = _run(world, [])
    for r in range(world):
        g = np.load(os.path.join(GOLD, f"a2a_W{world}.npz" if r == 0 else f"a2a_W{world}_r{r}.npz"))
        assert np.array_equal(outs[r]["y"], g["y"])
        assert np.array_equal(outs[r]["z"], g["z"])


def test_world1_seam_runs_same_path():
    """WORLD=1 goes through the same seam (pack -> attention -> out_proj, no exchange)."""
    outs = _run(1, [67])
    ref = np.load(os.path.join(GOLD, "seam_W2_S67.npz"))["out"]
    got = outs[0]["seam_67"]
    # same math as the W=2 reference path up to GEMM row-blocking: equal within fp32 noise
    assert np.abs(got - ref).max() < 1e-4


def _dropout_worker(rank, world, port, out_dir):
    """Rank 1 leaves between steps; rank 0 must get an error from its next collective in
    bounded time instead of hanging."""
    _setup_env(rank, world, port)
    import sp_runtime
    sp_runtime.init(timeout_s=5)
    x = torch.ones(1, 4, 3, 128) * rank
    sp_runtime._ops = __import__("oracle.cpu_ops", fromlist=["x"])
    sp_runtime.a2a_seq_to_head(x, world)  # step 1: everybody participates
    if rank == 1:
        return  # leaves without joining step 2
    t0 = time.time()
    err = ""
    try:
        sp_runtime.a2a_seq_to_head(x, world)
    except Exception as e:  # noqa: BLE001 - any backend error is the expected outcome
        err = type(e).__name__
    with open(os.path.join(out_dir, "r0.txt"), "w") as f:
        f.write(f"{err} {time.time() - t0:.1f}")


def test_rank_dropout_raises_in_bounded_time():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_dropout_worker, args=(2, _free_port(), d), nprocs=2, start_method="spawn")
        err, dt = open(os.path.join(d, "r0.txt")).read().split()
    assert err, "the surviving rank's collective did not fail"
    assert float(dt) < 60
