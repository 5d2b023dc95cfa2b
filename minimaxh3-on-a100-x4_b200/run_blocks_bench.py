"""50-block MiniMax-H3 denoiser forward (run_blocks) through the installed runtime, 1..8 GPUs.

    python minimaxh3-on-a100-x4_b200/run_blocks_bench.py [--blocks 50] [--seq 42000] [--steps 2]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 minimaxh3-on-a100-x4_b200/run_blocks_bench.py

The reference's block-loop benchmark (harness/sp_blockloop.py:141-200: 50 blocks, random init,
token-sharded run_blocks with the Ulysses attention, all-gather at the end, CUDA-event timing,
max over ranks). Model: hidden 5376, 56x128 heads, SwiGLU FFN 14336, AdaLN from a sinusoidal
t=500 embedding, bf16 weights ~N(0, 0.02) (the checkpoint is not available); input: the packed
[text 512 | cond 1024 | audio 1464 | video 39000] = 42000-token sequence, x ~N(0, 1).
Prints one JSON line (rank 0): ms per forward (max over ranks), the per-category split of one
extra timed forward (SP_TIMING categories of the runtime), and the TFLOP/s of the whole forward.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def forward_flops(s: int, blocks: int, hidden=5376, heads=56, head_dim=128, ffn=14336) -> float:
    hd = heads * head_dim
    gemm = 2.0 * s * (hidden * 3 * hd + hd * hidden + hidden * 2 * ffn + ffn * hidden)
    attn = 4.0 * s * s * head_dim * heads
    return blocks * (gemm + attn)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--blocks", type=int, default=50)
    ap.add_argument("--seq", type=int, default=42000)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    args = ap.parse_args()
    os.environ.setdefault("SP_TIMING", "0")
    import sp_runtime
    import h3_model as M
    import h3attn

    sp_runtime.init(timeout_s=600)
    rank, world = sp_runtime.RANK, sp_runtime.WORLD
    dev = torch.device("cuda", torch.cuda.current_device())
    model = M.MiniMaxH3Model(n_blocks=args.blocks, dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)  # same weights on every rank
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, torch.nn.Linear):
                m.weight.normal_(0.0, 0.02, generator=g)
                if m.bias is not None:
                    m.bias.zero_()
    S = args.seq
    segs = [(a, min(b, S), r) for a, b, r in M.H3_SEGMENTS if a < S]
    h = torch.randn((S, M.HIDDEN), generator=torch.Generator(device=dev).manual_seed(4), device=dev).to(torch.bfloat16)
    t_emb = M.timestep_embedding(torch.full((len(segs),), 500.0, device=dev)).to(torch.bfloat16)
    rope = M.rope_freqs_1d(S, device=dev)
    sp_runtime.install(M)

    def fwd():
        with torch.no_grad():
            return model.run_blocks(h, t_emb, segs, rope, {})

    def sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        fwd()
    h3attn.check_status()
    sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = fwd()
    e1.record()
    sync()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    h3attn.check_status()
    assert tuple(out.shape) == (S, M.HIDDEN) and bool(torch.isfinite(out.float()).all())
    # one more forward with per-category CUDA-event timing
    sp_runtime._TIMING = True
    fwd()
    sync()
    cats = sp_runtime.get_timing()
    sp_runtime._TIMING = False
    if rank == 0:
        fl = forward_flops(S, args.blocks)
        print(json.dumps({
            "metric": "run_blocks forward ms/step", "value": ms, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "scaling": "strong",
            "tflops": fl / (ms * 1e-3) / 1e12, "flop_per_step": fl, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C3 50-block run_blocks", "blocks": args.blocks, "seq_len": S, "hidden": M.HIDDEN,
                       "heads": M.HEADS, "ffn": M.FFN, "segments": segs, "parallelism": f"ulysses{world}"},
            "categories_ms_rank0": {k: round(v, 2) for k, v in cats.items()},
        }), flush=True)
    sp_runtime.uninstall()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
