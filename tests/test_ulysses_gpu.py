"""W-way Ulysses attention layer on real GPUs (NCCL over NVLink), one spawned process per
GPU: the W-way output of every rank must equal, bit for bit, the 1-GPU kernel's output on
that rank's token rows (the exactness the reference reports as max_err 0.0,
bench/ulysses_attn_microbench.py:57-70), including an uneven S that takes the pad path.
Skipped when fewer GPUs are visible than the world size."""
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "minimaxh3-on-a100-x4_b200")
H, D = 8, 128


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, S, result_dir, peer=False):
    for p in (PKG, ROOT):
        sys.path.insert(0, p)
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from datetime import timedelta
    import h3attn
    import h3_model
    import sp_runtime
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        g = torch.Generator().manual_seed(5)
        qkv_full = torch.randn(S, 3 * H * D, generator=g).to(torch.bfloat16).to(dev)
        rope_full = h3_model.rope_freqs_1d(S, device=dev)
        S_pad = ((S + world - 1) // world) * world
        sl = S_pad // world
        # 1-GPU reference on the full sequence (same kernels, W = 1 layout)
        q, k, v = qkv_full.split(H * D, -1)
        send1 = h3attn.qknorm_rope_pack(q, k, v, rope_full[0], None, None, 1e-6, 1)
        ref = h3attn.attention(send1[0, 0], send1[0, 1], send1[0, 2], layout="token")  # [S, H*D]
        # W-way: pad, shard, fused pack, exchange, unpack, attention into the send layout, exchange back
        qkv_pad = torch.cat([qkv_full, qkv_full.new_zeros(S_pad - S, qkv_full.shape[1])]) if S_pad > S else qkv_full
        rope_pad = torch.cat([rope_full, rope_full.new_zeros(1, S_pad - S, 64, 2, 2)], 1) if S_pad > S else rope_full
        loc = qkv_pad[rank * sl:(rank + 1) * sl].contiguous()
        rope_loc = rope_pad[0, rank * sl:(rank + 1) * sl].contiguous()
        q, k, v = loc.split(H * D, -1)
        if peer:  # both exchanges fused into the kernels over NVLink peer memory
            hl = H // world
            buf = sp_runtime._peer_buffers(sl, H, D, dev)[0]
            h3attn.qknorm_rope_pack_peer(q, k, v, rope_loc, None, None, 1e-6, world, buf["qkv_ptrs"],
                                         hl * S_pad * D, S_pad * D, rank * sl)
            dist.all_reduce(buf["flag"])
            qkvh = buf["qkv"]
            h3attn.attention_peer(qkvh[0], qkvh[1], qkvh[2], buf["o"], buf["o_ptrs"], sl, D, H * D, s_kv=S)
            dist.all_reduce(buf["flag"])
            out = buf["o"]
        else:
            send = h3attn.qknorm_rope_pack(q, k, v, rope_loc, None, None, 1e-6, world)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send)
            qkvh = h3attn.seq_to_head_unpack(recv)
            o_send = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=S, layout="send", world=world)
            o_recv = torch.empty_like(o_send)
            dist.all_to_all_single(o_recv, o_send)
            out = h3attn.head_to_seq_unpack(o_recv.view(H, sl, D))
        h3attn.check_status()
        lo, hi = rank * sl, min((rank + 1) * sl, S)
        ok = torch.equal(out[:hi - lo], ref[lo:hi]) if hi > lo else True
        # reference-API helpers round-trip on this rank's shard
        xs = torch.randn(1, H, sl, D, generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16).to(dev)
        y = sp_runtime.a2a_seq_to_head(xs, world)
        z = sp_runtime.a2a_head_to_seq(y, world, H)
        ok = ok and torch.equal(z, xs) and tuple(y.shape) == (1, H // world, world * sl, D)
        torch.cuda.synchronize()
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,S,peer", [(2, 4096, False), (2, 3001, False), (4, 4096, False), (8, 4099, False),
                                          (2, 3001, True), (4, 4096, True), (8, 4099, True)])
def test_ulysses_layer_bit_exact_vs_single_gpu(world, S, peer, tmp_path):
    """peer: the exchanges fused into the pack and attention kernels (stores into the destination
    ranks' symmetric buffers) instead of NCCL all-to-alls plus unpack kernels."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _port(), S, str(tmp_path), peer), nprocs=world, start_method="spawn")
    for r in range(world):
        assert (tmp_path / f"r{r}").read_text() == "ok", r
