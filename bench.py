"""Benchmark of the B200 Ulysses attention layer (the BASELINE.json headline metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--seq S]
    (N > 1: python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...)

One step = one exact 56x128-head attention layer over S = 42,000 tokens (config 1 at N=1,
the Ulysses layer of config 2 at N>1): each rank starts from its token shard of the fused
QKV projection output, runs the fused qk-RMSNorm + RoPE + send pack, the seq->head
all-to-all (N>1), attention over its 56/N heads and the full sequence, and the head->seq
all-to-all back to token-major rows (N>1). FLOPs per step = 4*S^2*128*56 (5.058e13).

Printed by rank 0 as ONE JSON line: value = whole-job TFLOP/s from CUDA events (max over
ranks), e2e = the same through the public API with the step's input copied from pinned
host memory and its output read back inside the timed region, roofline of the attention
kernel against MEASURED_PEAKS.json, the CPU baseline (the reference's own SDPA call on
this host's cores, bounded sample), and SM clocks sampled during the timed region.

--impl reference times the reference's CPU path for this op (torch SDPA FLASH on the host
cores, harness/sp_runtime.py:119-121) on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "minimaxh3-on-a100-x4_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "ms/layer & TFLOP/s, 56x128 attn S=42k bf16, 1/2/4/8 B200; % dense bf16 peak"
UNIT = "TFLOP/s"
HEADS, D = 56, 128
NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool's B200s (nominal 900)


def flops_layer(s: int, heads: int = HEADS) -> float:
    return 4.0 * s * s * D * heads


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j.get("bf16_tflops"), j.get("bf16_tflops_sustained"), j.get("hbm_gbs"), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def profiled_traffic(name: str, seq: int, heads: int):
    """DRAM bytes (read + write) of one attention launch at `seq` x `heads`, scaled from the
    ncu capture summarised in profiles/<name> ('capture_seq:' and 'dram_bytes_per_launch:'
    lines, 56 heads). Q, K, V are read once and O written once, so traffic is linear in
    S and in the head count. None when no capture has been summarised."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    vals = {}
    with open(p) as f:
        for line in f:
            for key in ("capture_seq:", "dram_bytes_per_launch:"):
                if line.startswith(key):
                    vals[key] = float(line.split(":", 1)[1].strip())
    if len(vals) != 2:
        return None
    return int(vals["dram_bytes_per_launch:"] * seq / vals["capture_seq:"] * heads / HEADS)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms from before the warm-up
    until after the timed region; summary() keeps the samples stamped inside the timed
    window (mark_start / mark_end), falling back to the whole run when the window was too
    short to catch one."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, n_gpus: int):
        self.n = n_gpus
        self.proc = None
        self.t_start = self.t_end = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_bench_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def mark_start(self):
        self.t_start = time.time()

    def mark_end(self):
        self.t_end = time.time()

    def stop(self):
        if self.proc is not None:
            time.sleep(0.25)  # one more sample after the window
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def _rows(self):
        with open(self.path) as f:
            for line in f:
                c = [x.strip() for x in line.split(",")]
                if len(c) < 10 or not c[1].isdigit() or int(c[1]) >= self.n:
                    continue
                try:
                    ts = time.mktime(time.strptime(c[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                    ts += float("0." + c[0].split(".")[1]) if "." in c[0] else 0.0
                    yield ts, float(c[2]), float(c[3]), c[6:10]
                except ValueError:
                    continue

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = list(self._rows())
        win = [r for r in rows if self.t_start is not None and self.t_start - 0.2 <= r[0] <= self.t_end + 0.2]
        scope = "timed region"
        if not win:
            win, scope = rows, "whole run (timed region shorter than the sampling period)"
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        reasons = sorted({nm for r in win for nm, val in zip(self.NAMES, r[3]) if val.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in win), "sm_max_mhz": max(r[2] for r in win),
                "reasons": reasons, "samples": len(win), "scope": scope}


def cpu_sdpa_sample(s_kv: int, heads: int, rows: int, reps: int, threads: int):
    """The reference's attention call (SDPA FLASH, sp_runtime.py:119-121) in fp32 on the host
    cores for `heads` heads x `rows` query rows against all s_kv keys. Returns the per-rep times."""
    from oracle import sdpa_ref
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, heads, rows, D, generator=g)
    k = torch.randn(1, heads, s_kv, D, generator=g)
    v = torch.randn(1, heads, s_kv, D, generator=g)
    sdpa_ref.attention(q[:, :, :64], k[:, :, :256], v[:, :, :256])  # warm-up
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        sdpa_ref.attention(q, k, v)
        times.append(time.perf_counter() - t0)
    return times


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    heads, rows = 1, 4096  # one bounded sample per step: 1 head x 4096 query rows x all keys
    torch.set_num_threads(threads)
    times = cpu_sdpa_sample(args.seq, heads, rows, args.warmup + args.steps, threads)[args.warmup:]
    per = statistics.median(times)
    fl = 4.0 * rows * args.seq * D * heads
    val = fl / per / 1e12
    sample = f"{heads} head x {rows} query rows x {args.seq} keys fp32 per step ({fl:.3g} FLOP)"
    line = {
        "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": config(args),
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample + "; torch SDPA FLASH on CPU, the reference's attention call"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config(args):
    return {"workload": "ulysses attention layer: qk-RMSNorm+RoPE pack, seq->head all-to-all, exact attention, "
                        "head->seq all-to-all", "heads": HEADS, "head_dim": D, "seq_len": args.seq,
            "batch": args.batch, "parallelism": f"ulysses{args.gpus}",
            "overlap": args.overlap if args.gpus > 1 else "none",
            "l2": f"inputs larger than L2: {args.batch * args.seq * 3 * HEADS * D * 2 / 1e9:.2f} GB of QKV per step"}


def run_ours(args, rank: int, world: int, local: int) -> None:
    import h3attn
    import h3_model

    dev = torch.device("cuda", local)
    S, H, W = args.seq, HEADS, world
    sampler = ClockSampler(W).start() if rank == 0 else None  # started early: nvidia-smi needs ~1 s
    if S % W or H % W:
        raise SystemExit(f"seq {S} and heads {H} must divide by {W}")
    sl, hl = S // W, H // W
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    B = args.batch  # independent sequences per step (config 4: CFG cond/uncond, separate seeds)
    qkv = torch.stack([torch.randn((sl, 3 * H * D), generator=torch.Generator(device=dev).manual_seed(1000 + rank + 7919 * b),
                                   device=dev, dtype=torch.float32).to(torch.bfloat16) for b in range(B)])
    rope = h3_model.rope_freqs_1d(sl, pos0=rank * sl, device=dev)[0].contiguous()
    ones = torch.ones(D, dtype=torch.bfloat16, device=dev)
    eps = 1e-6
    ev_att, ev_a2a = [], []

    def exchange(send, timed):
        recv = torch.empty_like(send)
        if timed:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        dist.all_to_all_single(recv, send)
        if timed:
            b.record()
            ev_a2a.append((a, b, send.numel() * send.element_size() * (W - 1) // W))
        return recv

    def layer(x, out=None, timed=False):
        q, k, v = x.split(H * D, dim=-1)
        send = h3attn.qknorm_rope_pack(q, k, v, rope, ones, ones, eps, W)
        if W > 1:
            qkvh = h3attn.seq_to_head_unpack(exchange(send, timed))
        else:
            qkvh = send[0]
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        if W > 1:
            o_send = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], layout="send", world=W)
        else:
            o = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], layout="token", out=out)
        if timed:
            e1.record()
            ev_att.append((e0, e1))
        if W > 1:
            o_recv = exchange(o_send, timed)
            o = h3attn.head_to_seq_unpack(o_recv.view(H, sl, D), out=out)
        return o

    comm, side = (torch.cuda.Stream(), torch.cuda.Stream()) if W > 1 else (None, None)

    def layer_heads(x, out=None, timed=False):
        """The same layer pipelined head by head: each local head's q/k/v and O travel in their own
        all-to-all on a side stream while other heads compute; consecutive heads alternate between
        two compute streams so one head's tail wave overlaps the next head."""
        q, k, v = x.split(H * D, dim=-1)
        send = h3attn.qknorm_rope_pack(q, k, v, rope, ones, ones, eps, W, head_major=True)  # [hl, W, 3, sl, D]
        default = torch.cuda.current_stream()
        comm.wait_stream(default)
        side.wait_stream(default)
        send.record_stream(comm)
        o_heads = torch.empty((W, hl, sl, D), dtype=torch.bfloat16, device=dev)
        o_heads.record_stream(comm)
        recvs, arrived = [], []
        with torch.cuda.stream(comm):
            for h in range(hl):
                recvs.append(exchange(send[h], timed))
                arrived.append(torch.cuda.Event())
                arrived[-1].record(comm)
        for h in range(hl):
            cs = default if h % 2 == 0 else side
            cs.wait_event(arrived[h])
            recvs[h].record_stream(cs)
            with torch.cuda.stream(cs):
                qkvh = h3attn.seq_to_head_unpack(recvs[h].view(W, 3, 1, sl, D))
                if timed:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(cs)
                o_send = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], layout="send", world=W)
                if timed:
                    e1.record(cs)
                    ev_att.append((e0, e1))
                done = torch.cuda.Event()
                done.record(cs)
            o_send.record_stream(comm)
            with torch.cuda.stream(comm):
                comm.wait_event(done)
                o_heads[:, h].copy_(exchange(o_send, timed).view(W, sl, D))
        default.wait_stream(side)
        default.wait_stream(comm)
        return h3attn.head_to_seq_unpack(o_heads.view(H, sl, D), out=out)

    peer_bufs, peer_step = None, [0]
    if W > 1 and args.overlap == "peer":
        import sp_runtime
        peer_bufs = sp_runtime._peer_buffers(sl, H, D, dev, slots=2)

    def layer_peer(x, out=None, timed=False):
        """The same layer with both exchanges fused into the kernels over NVLink peer memory: the
        pack writes every head into its destination rank's attention input, the attention epilogue
        writes every row into its destination rank's token-major output; a stream-ordered barrier
        after each. Two buffer slots alternate so a step's readback never meets the next step's
        peer writes. Returns this rank's [Sl, H*D] output (a symmetric buffer)."""
        buf = peer_bufs[peer_step[0] % 2]
        peer_step[0] += 1
        q, k, v = x.split(H * D, dim=-1)
        h3attn.qknorm_rope_pack_peer(q, k, v, rope, ones, ones, eps, W, buf["qkv_ptrs"], hl * S * D, S * D, rank * sl)
        barrier(buf["flag"], timed)
        qkvh = buf["qkv"]
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        h3attn.attention_peer(qkvh[0], qkvh[1], qkvh[2], buf["o"], buf["o_ptrs"], sl, D, H * D)
        if timed:
            e1.record()
            ev_att.append((e0, e1))
        barrier(buf["flag"], timed)
        return buf["o"]

    def barrier(flag, timed):
        if timed:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        dist.all_reduce(flag)
        if timed:
            b.record()
            ev_a2a.append((a, b, 0))

    heads_per_launch = hl
    if W > 1 and args.overlap == "heads":
        layer = layer_heads  # noqa: F811
        heads_per_launch = 1
    if W > 1 and args.overlap == "peer":
        layer = layer_peer  # noqa: F811

    def sync_all():
        torch.cuda.synchronize()
        if W > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if W == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def step(x, out=None, timed=False):
        """One step: the layer over each of the B sequences of x [B, Sl, 3*H*D]; returns the B
        outputs (views of `out` when given and the layer writes there)."""
        return [layer(x[b], out=None if out is None else out[b], timed=timed) for b in range(B)]

    # correctness guard: the status word must stay clean
    for _ in range(args.warmup):
        step(qkv)
    h3attn.check_status()
    sync_all()

    # ---- device-timed region
    ev_att.clear()
    ev_a2a.clear()
    sync_all()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.mark_start()
    t0.record()
    for _ in range(args.steps):
        step(qkv, timed=True)
    t1.record()
    sync_all()
    if sampler:
        sampler.mark_end()
        sampler.stop()
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    att_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in ev_att))
    if W > 1:  # the blocking layer: both exchanges are exposed (nothing runs beside them)
        a2a_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b, _ in ev_a2a) / args.steps)
        a2a_bytes = sum(n for _, _, n in ev_a2a) / args.steps
    h3attn.check_status()

    # ---- end-to-end through the public API: every step copies its input from pinned host
    # memory and reads its output back. Copies run on their own streams with two device
    # buffers each way, so step i+1's upload and step i-1's readback overlap step i's layer.
    host_in = torch.empty(qkv.shape, dtype=qkv.dtype, pin_memory=True)
    host_in.copy_(qkv)
    host_out = [torch.empty((B, sl, H * D), dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
    dev_in = [torch.empty_like(qkv) for _ in range(2)]
    dev_out = [torch.empty((B, sl, H * D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    compute = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()
    in_ready, in_free, done, out_free = ([ev() for _ in range(2)] for _ in range(4))
    for b in range(2):
        in_free[b].record(compute)
        out_free[b].record(compute)

    def e2e_steps(n, start=None):
        """n pipelined steps; t0 is recorded on the compute stream when step `start` is due (the
        pipeline is already running: its input was uploaded under the previous step's layer)."""
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(in_free[b])
                dev_in[b].copy_(host_in, non_blocking=True)
                in_ready[b].record(s_in)
            if i == start:
                t0.record(compute)
            compute.wait_event(in_ready[b])
            compute.wait_event(out_free[b])
            res = step(dev_in[b], out=None if peer_bufs is not None else dev_out[b])
            in_free[b].record(compute)
            done[b].record(compute)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done[b])
                for bb in range(B):
                    host_out[b][bb].copy_(res[bb], non_blocking=True)
                out_free[b].record(s_out)
        compute.wait_stream(s_in)
        compute.wait_stream(s_out)

    # steady state: two warm-up steps, then e2e_n timed steps of the same running pipeline; the
    # timed region ends when the last step's result has reached host memory
    e2e_n = max(3, min(args.steps, 10))
    e2e_warm = 2
    sync_all()
    e2e_steps(e2e_warm + e2e_n, start=e2e_warm)
    t1.record(compute)
    sync_all()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1) / e2e_n)
    if not torch.equal(host_out[(e2e_warm + e2e_n - 1) % 2], torch.stack([r.cpu() for r in step(qkv)])):
        raise SystemExit("end-to-end output differs from the device-resident run")

    if rank != 0:
        return
    fl = flops_layer(S) * B
    burst, sustained, hbm, kind = peaks()
    att_fl = 4.0 * S * S * D * heads_per_launch  # one attention launch
    achieved = att_fl / (att_ms * 1e-3) / 1e12
    traffic = profiled_traffic("attn_fwd_s8192_h56_full.md", S, hl)
    # our kernels per step: pack, attention (W=1); + seq->head unpack and head->seq unpack (W>1),
    # the unpack and attention once per local head when pipelined by heads
    per_step = 2 if W == 1 or peer_bufs is not None else (4 if heads_per_launch == hl else 2 + 2 * hl)
    launches = per_step * B * args.steps
    line = {
        "metric": METRIC, "value": fl / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": W, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config(args),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                     "frac": achieved / sustained, "peak_kind": f"{kind} sustained bf16 (cuBLAS 8192^3 loop)",
                     "frac_of_burst_peak": achieved / burst, "traffic": traffic, "kernel": "attn_fwd_kernel",
                     "kernel_ms": att_ms, "flop_per_launch": att_fl},
        "e2e": {"value": fl / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                "method": "steady-state pipeline: step i+1's upload and step i-1's readback overlap step i",
                "h2d_bytes_per_step": qkv.numel() * 2 * W, "d2h_bytes_per_step": B * sl * H * D * 2 * W},
        "gpu_launches": launches,
        "clocks": sampler.summary() if sampler else None,
    }
    if W > 1 and peer_bufs is not None:
        # the exchanges are stores of the pack and attention kernels; only the barriers stand alone
        sent = B * 4 * sl * H * D * 2 * (W - 1) / W  # q, k, v and O rows bound for other ranks
        line["a2a"] = {"barrier_ms_per_step": a2a_ms, "bytes_sent_per_gpu_per_step": sent,
                       "mode": "fused into the pack and attention kernels (NVLink peer stores)",
                       "frac_of_step": a2a_ms / ms}
    elif W > 1:
        gbs = a2a_bytes / (a2a_ms * 1e-3) / 1e9
        key = "exposed_ms_per_step" if args.overlap == "none" else "comm_stream_ms_per_step_overlapped"
        line["a2a"] = {key: a2a_ms, "bytes_sent_per_gpu_per_step": a2a_bytes,
                       "achieved_gbs_per_gpu": gbs, "frac_of_nvlink": gbs / NVLINK_GBS,
                       "nvlink_ref": f"{NVLINK_GBS:.0f} GB/s per direction per GPU (measured peer copy on this pool)",
                       "frac_of_step": a2a_ms / ms}
    if W == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        heads, rows = 4, 4096
        times = cpu_sdpa_sample(S, heads, rows, 5, threads)
        per = statistics.median(times)
        cfl = 4.0 * rows * S * D * heads
        line["cpu_baseline"] = {"value": cfl / per / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": f"{heads} heads x {rows} query rows x {S} keys fp32 ({cfl:.3g} FLOP), "
                                          f"median of 5; torch SDPA FLASH on CPU (the reference's attention call)"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seq", type=int, default=42000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=1, help="independent sequences per step (config 4: 2)")
    ap.add_argument("--overlap", default="none", choices=["none", "heads", "peer"],
                    help="W>1: exchanges pipelined head by head, or fused into the kernels over peer memory")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
