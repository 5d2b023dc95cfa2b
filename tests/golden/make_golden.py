"""Generate the golden vectors in tests/golden/ by running the REFERENCE's own code.

    python tests/golden/make_golden.py --ref <checkout of shi3z/MinimaxH3-on-A100-x4>

Runs here (CPU, gloo ranks); the GPU box never needs the reference. It imports
harness/sp_runtime.py from the reference checkout (read-only) with the test stub `comfy`
package (tests/stub_comfy: ComfyUI-shaped H3 model, qk-RMSNorm+RoPE restated by the
oracle) and records:

  a2a.npz        a2a_seq_to_head / a2a_head_to_seq round trips      (sp_runtime.py:67-77)
  seam_W{W}_S{S}.npz  install() + run_blocks through the seam on W gloo ranks, including
                 the uneven-S pad path (sp_runtime.py:220-271, :85-127)
  sdpa.npz       the reference's attention call (SDPA FLASH, sp_runtime.py:119-121) on
                 config-0 style inputs at small / ragged sizes and the pad (s_kv < s_q) case
  host.json      _shard_segments / _piece_bounds on a table of cases (:196-201, :136-144)
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import socket
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
TESTS = os.path.dirname(HERE)
ROOT = os.path.dirname(TESTS)
PKG = os.path.join(ROOT, "minimaxh3-on-a100-x4_b200")

# seam case definition (shared with tests/test_runtime_cpu.py through seam_setup())
SEAM = dict(n_blocks=2, hidden=96, heads=4, head_dim=128, ffn=192, t_dim=32, seed=0)


def _paths():
    for p in (os.path.join(TESTS, "stub_comfy"), PKG, ROOT, TESTS):
        if p not in sys.path:
            sys.path.insert(0, p)


def seam_setup(S: int):
    """Model + inputs of the seam case (fp32, CPU): (model, h, t_emb, segs, rope)."""
    _paths()
    import h3_model as M
    model = M.MiniMaxH3Model(SEAM["n_blocks"], SEAM["hidden"], SEAM["heads"], SEAM["head_dim"], SEAM["ffn"],
                             SEAM["t_dim"])
    M.init_weights(model, SEAM["seed"], std=0.05)
    g = torch.Generator().manual_seed(100 + S)
    h = torch.randn(S, SEAM["hidden"], generator=g)
    t_emb = M.timestep_embedding(torch.tensor([500.0, 250.0, 750.0]), SEAM["t_dim"])
    segs = [(0, 10, 0), (10, 40, 1), (40, S, 2)]
    rope = M.rope_freqs_1d(S)
    return model, h, t_emb, segs, rope


def load_reference_runtime(ref_root: str):
    path = os.path.join(ref_root, "harness", "sp_runtime.py")
    spec = importlib.util.spec_from_file_location("ref_sp_runtime", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, ref_root, out_dir, cases):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    _paths()
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ref = load_reference_runtime(ref_root)  # reads RANK / WORLD_SIZE at import, as in production
    res = {}
    if "a2a" in cases:
        H, Sl = 8, 5
        g = torch.Generator().manual_seed(7)
        xs = [torch.randn(1, H, Sl, 128, generator=g) for _ in range(world)]
        y = ref.a2a_seq_to_head(xs[rank].clone(), world)
        z = ref.a2a_head_to_seq(y.clone(), world, H)
        res["a2a"] = dict(x=np.stack([x.numpy() for x in xs]), y=y.numpy(), z=z.numpy())
    for S in cases.get("seam", []):
        import comfy.ldm.minimax.model as MM
        model, h, t_emb, segs, rope = seam_setup(S)
        ref.install()
        with torch.no_grad():
            out = MM.MiniMaxH3Model.run_blocks(model, h.clone(), t_emb, segs, rope, {})
        MM.MiniMaxH3Model.run_blocks = ref._orig_run_blocks
        MM.Attention.forward = ref._orig_attn_forward
        res[f"seam_{S}"] = out.numpy()
    dist.barrier()
    if rank == 0:
        if "a2a" in res:
            np.savez_compressed(os.path.join(out_dir, f"a2a_W{world}.npz"), **res["a2a"])
        for S in cases.get("seam", []):
            np.savez_compressed(os.path.join(out_dir, f"seam_W{world}_S{S}.npz"), out=res[f"seam_{S}"])
    else:
        if "a2a" in res:
            np.savez_compressed(os.path.join(out_dir, f"a2a_W{world}_r{rank}.npz"), **res["a2a"])
    dist.destroy_process_group()


def run_ranks(world, ref_root, out_dir, cases):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _free_port(), ref_root, out_dir, cases), nprocs=world,
                       start_method="spawn")


def sdpa_golden(out_dir):
    _paths()
    from oracle import h3_oracle as O
    from oracle import sdpa_ref
    rec = {}
    for H, S in [(2, 1), (2, 15), (2, 127), (2, 128), (2, 129), (2, 255), (3, 300)]:
        q, k, v = O.make_qkv(S * 7 + H, H, S)
        rope = O.rope_table(S)[0]
        qn = O.qknorm_rope(q, None, rope, 1e-6).transpose(1, 0, 2).copy()
        kn = O.qknorm_rope(k, None, rope, 1e-6).transpose(1, 0, 2).copy()
        vt = v.transpose(1, 0, 2).copy()
        o = sdpa_ref.attention(*(torch.from_numpy(a)[None] for a in (qn, kn, vt)))[0].numpy()
        rec[f"H{H}_S{S}"] = (qn, kn, vt, o)
    # pad path: queries over 304 rows, keys/values over the first 301
    q, k, v = O.make_qkv(11, 2, 304)
    qt, kt, vt = (a.transpose(1, 0, 2).copy() for a in (q, k, v))
    o = sdpa_ref.attention(torch.from_numpy(qt)[None], torch.from_numpy(kt[:, :301])[None],
                           torch.from_numpy(vt[:, :301])[None])[0].numpy()
    rec["pad_S304_kv301"] = (qt, kt, vt, o)
    arrays = {}
    for name, (q, k, v, o) in rec.items():
        arrays[name + "_q"] = O.to_bf16_bits(q)
        arrays[name + "_k"] = O.to_bf16_bits(k)
        arrays[name + "_v"] = O.to_bf16_bits(v)
        arrays[name + "_o"] = o.astype(np.float32)
    np.savez_compressed(os.path.join(out_dir, "sdpa.npz"), **arrays)


def host_golden(ref_root, out_dir):
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    _paths()
    ref = load_reference_runtime(ref_root)
    segs = [(0, 512, 0), (512, 1536, 1), (1536, 3000, 2), (3000, 42000, 3)]
    shard = []
    for W in (1, 2, 4, 8):
        for S in (42000, 42003, 67):
            sp = ((S + W - 1) // W) * W
            sl = sp // W
            s2 = [(a, min(b, S), r) for a, b, r in segs if a < S]
            for r in range(W):
                shard.append(dict(segs=s2, lo=r * sl, hi=(r + 1) * sl, out=ref._shard_segments(s2, r * sl, (r + 1) * sl)))
    pieces = [dict(n=n, p=p, out=ref._piece_bounds(n, p)) for n in (0, 1, 3, 7, 5250, 10500, 21000) for p in (1, 2, 3, 4, 8)]
    with open(os.path.join(out_dir, "host.json"), "w") as f:
        json.dump(dict(shard_segments=shard, piece_bounds=pieces), f)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of a read-only checkout of the reference project")
    args = ap.parse_args()
    out_dir = HERE
    host_golden(args.ref, out_dir)
    sdpa_golden(out_dir)
    for W in (2, 4):
        run_ranks(W, args.ref, out_dir, {"a2a": True, "seam": [67, 64]})
    print("golden vectors written to", out_dir)


if __name__ == "__main__":
    main()
