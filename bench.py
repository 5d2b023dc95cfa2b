"""Benchmark of the B200 Ulysses attention layer (the BASELINE.json headline metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--seq S]
    (N > 1: python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...)

One step = one exact 56x128-head attention layer over S = 42,000 tokens (config 1 at N=1,
the Ulysses layer of config 2 at N>1): each rank starts from its token shard of the fused
QKV projection output, runs the fused qk-RMSNorm + RoPE + send pack, the seq->head
all-to-all (N>1), attention over its 56/N heads and the full sequence, and the head->seq
all-to-all back to token-major rows (N>1). FLOPs per step = 4*S^2*128*56 (5.058e13). An S
that does not divide by N takes the runtime's pad path (pad rows at the tail, keys stop at S).

Printed by rank 0 as ONE JSON line:
  value          whole-job TFLOP/s from CUDA events (max over ranks)
  e2e            the same through the public API with the step's input copied from pinned host
                 memory and its output read back inside the timed region, with the per-rank copy
                 rates and a plain pinned-copy ceiling measured at the same concurrency
  roofline       the attention kernel against MEASURED_PEAKS.json
  cpu_baseline   the reference's own SDPA call at config 0 on this host's cores
  clocks         SM clocks sampled during the timed region
  bit_exact_vs_w1 (N>1) every rank's output rows equal, bit for bit, the 1-GPU layer on the
                 gathered input; the run exits non-zero otherwise
  vendor_attention (N=1) the reference's GPU call (torch SDPA) at config 1 on the same box
  run_blocks     config 3: the 50-block MiniMax-H3 forward through the installed runtime (ms per
                 forward, max over ranks, its own clock record, per-category split; at N>1 also
                 bit-exact against the 1-GPU forward)

--case <kernel> times one kernel of the path alone (attn, pack, gemm_qkv/out/fc1/fc2, norm_mod,
residual) at --seq rows: the entry point of the profile summaries under profiles/.

--impl reference times the reference's CPU path for this op (torch SDPA FLASH on the host
cores, harness/sp_runtime.py:119-121) at config 0 (H=56, S=4096, fp32, seed 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
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
NVLINK_GBS = 770.0  # measured peer copy per direction per B200 (nominal 900)


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
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms from start() to stop();
    summary(window) keeps the samples stamped inside a named window (mark(name, "start"/"end")),
    falling back to the whole run when the window was too short to catch one."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, n_gpus: int):
        self.n = n_gpus
        self.proc = None
        self.windows = {}
        self.tmp = tempfile.TemporaryDirectory(prefix="h3_clocks_")
        self.path = os.path.join(self.tmp.name, "clocks.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def mark(self, window: str, edge: str):
        self.windows.setdefault(window, {})[edge] = time.time()

    def stop(self):
        if self.proc is not None:
            time.sleep(0.25)  # one more sample after the last window
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()
            self.proc_done = True

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

    def summary(self, window: str):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = list(self._rows())
        w = self.windows.get(window, {})
        t0, t1 = w.get("start"), w.get("end")
        win = [r for r in rows if t0 is not None and t1 is not None and t0 - 0.2 <= r[0] <= t1 + 0.2]
        scope = "timed region"
        if not win:
            win, scope = rows, "whole run (timed region shorter than the sampling period)"
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        reasons = sorted({nm for r in win for nm, val in zip(self.NAMES, r[3]) if val.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in win), "sm_max_mhz": max(r[2] for r in win),
                "reasons": reasons, "samples": len(win), "scope": scope}


# ----------------------------------------------------------------------------- the CPU baseline
def cpu_config0(reps: int, threads: int, warm: int = 1):
    """The reference's attention call (SDPA FLASH, sp_runtime.py:119-121) at config 0 (H=56,
    S=4096, D=128, fp32, seed 0, RMSNorm + RoPE on q and k) on the host cores. `warm` warm-up runs,
    then `reps` timed runs; returns (per-run seconds, FLOPs per run, sample description)."""
    from oracle import north_star, sdpa_ref
    torch.set_num_threads(threads)
    H, S = 56, 4096
    q, k, v = north_star.config_inputs(0, H, S, "cpu")
    q, k, v = q[None], k[None], v[None]
    for _ in range(warm):
        sdpa_ref.attention(q, k, v)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        sdpa_ref.attention(q, k, v)
        times.append(time.perf_counter() - t0)
    sample = (f"config 0: B=1 H={H} S={S} D=128 fp32 seed 0 (RMSNorm + RoPE), the reference's SDPA FLASH call "
              f"on the CPU, {threads} threads, median of {reps} after {warm} warm-up run(s)")
    return times, flops_layer(S, H), sample


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    times, fl, sample = cpu_config0(args.steps, threads, warm=args.warmup)
    per = statistics.median(times)
    val = fl / per / 1e12
    line = {
        "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": config(args),
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                         "ms": per * 1e3},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "ms_per_layer_at_s": {"s": args.seq, "ms": flops_layer(args.seq) / (val * 1e12) * 1e3,
                              "how": "config-0 throughput applied to the arm's layer (4*S^2*128*56 FLOP)"},
    }
    print(json.dumps(line), flush=True)


def config(args):
    return {"workload": "ulysses attention layer: qk-RMSNorm+RoPE pack, seq->head all-to-all, exact attention, "
                        "head->seq all-to-all", "heads": HEADS, "head_dim": D, "seq_len": args.seq,
            "batch": args.batch, "parallelism": f"ulysses{args.gpus}",
            "overlap": args.overlap if args.gpus > 1 else "none",
            "l2": f"inputs larger than L2: {args.batch * args.seq * 3 * HEADS * D * 2 / 1e9:.2f} GB of QKV per step"}


# ----------------------------------------------------------------------------- helpers
def gpu_local_cpus(dev: torch.device):
    """CPUs on the NUMA node of `dev` (from sysfs), or None when unknown."""
    try:
        p = torch.cuda.get_device_properties(dev)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as f:
            spec = f.read().strip()
    except (AttributeError, OSError, RuntimeError):
        return None
    cpus = set()
    for part in spec.split(","):
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        elif part:
            cpus.add(int(part))
    return cpus or None


def run_ours(args, rank: int, world: int, local: int) -> None:
    import h3attn
    import h3_model

    dev = torch.device("cuda", local)
    S, H, W = args.seq, HEADS, world
    sampler = ClockSampler(W).start() if rank == 0 else None  # started early: nvidia-smi needs ~1 s
    if H % W:
        raise SystemExit(f"heads {H} must divide by {W}")
    sl, hl = -(-S // W), H // W
    S_pad = sl * W
    real = max(0, min(sl, S - rank * sl))  # this rank's real (non-pad) rows
    # host buffers on the GPU's own NUMA node: bind before any pinned allocation (first touch)
    numa = None
    if not args.no_numa_bind:
        cpus = gpu_local_cpus(dev)
        if cpus:
            try:
                os.sched_setaffinity(0, cpus)
                numa = f"{len(cpus)} CPUs local to the GPU"
            except OSError:
                numa = None
    B = args.batch  # independent sequences per step (config 4: CFG cond/uncond, separate seeds)

    def make_qkv(b):
        g = torch.Generator(device=dev).manual_seed(1000 + rank + 7919 * b)
        x = torch.randn((sl, 3 * H * D), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
        x[real:] = 0  # pad rows (S not a multiple of W)
        return x

    qkv = torch.stack([make_qkv(b) for b in range(B)])
    rope = h3_model.rope_freqs_1d(sl, pos0=rank * sl, device=dev)[0].contiguous()
    rope[real:] = 0
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
            o_send = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=S, layout="send", world=W)
        else:
            o = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=S, layout="token", out=out)
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
                o_send = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=S, layout="send", world=W)
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
        h3attn.qknorm_rope_pack_peer(q, k, v, rope, ones, ones, eps, W, buf["qkv_ptrs"], hl * S_pad * D, S_pad * D,
                                     rank * sl)
        barrier(buf["flag"], timed)
        qkvh = buf["qkv"]
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        h3attn.attention_peer(qkvh[0], qkvh[1], qkvh[2], buf["o"], buf["o_ptrs"], sl, D, H * D, s_kv=S)
        if timed:
            e1.record()
            ev_att.append((e0, e1))
        barrier(buf["flag"], timed)
        return buf["o"]

    ce_bufs, ce_step, ce_streams = None, [0], None
    if W > 1 and args.overlap == "ce":
        import sp_runtime
        ce_bufs = sp_runtime._peer_buffers(sl, H, D, dev, slots=2)
        ce_streams = [torch.cuda.Stream() for _ in range(W)]
        for b in ce_bufs:  # every rank's buffer bases, on the host
            b["qkv_base"] = b["qkv_ptrs"].tolist()
            b["o_base"] = [p - rank * hl * D * 2 for p in b["o_ptrs"].tolist()]

    def layer_ce(x, out=None, timed=False):
        """The same layer with both exchanges done by the copy engines: the pack writes the usual
        send buffer, then one 2-D copy per destination rank puts this rank's q/k/v rows straight into
        that rank's attention input [3][H/W][S][D] (rows rank*Sl...), and one contiguous copy per
        destination puts this rank's attention output heads into that rank's [H][Sl][D] out_proj
        input; the copies to different ranks run on their own streams, and a stream-ordered barrier
        follows each exchange. No unpack kernel runs on the receive side of the q/k/v exchange."""
        buf = ce_bufs[ce_step[0] % 2]
        ce_step[0] += 1
        cur = torch.cuda.current_stream()
        q, k, v = x.split(H * D, dim=-1)
        send = h3attn.qknorm_rope_pack(q, k, v, rope, ones, ones, eps, W)  # [W, 3, hl, sl, D]
        if timed:
            a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        row = sl * D * 2
        for d in range(W):
            st = ce_streams[d]
            st.wait_stream(cur)
            h3attn.copy_2d(buf["qkv_base"][d] + rank * row, S_pad * D * 2, send[d].data_ptr(), row, row, 3 * hl,
                           stream=st)
        for st in ce_streams:
            cur.wait_stream(st)
        dist.all_reduce(buf["flag"])  # every rank's rows have landed
        if timed:
            b_.record()
            ev_a2a.append((a, b_, send.numel() * 2 * (W - 1) // W))
        qkvh = buf["qkv"]
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        o_send = h3attn.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=S, layout="send", world=W)  # [W, hl, sl, D]
        if timed:
            e1.record()
            ev_att.append((e0, e1))
            a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        blk = hl * sl * D * 2
        for d in range(W):
            st = ce_streams[d]
            st.wait_stream(cur)
            h3attn.copy_2d(buf["o_base"][d] + rank * blk, blk, o_send[d].data_ptr(), blk, blk, 1, stream=st)
        for st in ce_streams:
            cur.wait_stream(st)
        dist.all_reduce(buf["flag"])  # every rank's heads for this rank have landed
        if timed:
            b_.record()
            ev_a2a.append((a, b_, o_send.numel() * 2 * (W - 1) // W))
        return h3attn.head_to_seq_unpack(buf["o"].view(H, sl, D), out=out)

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
    if W > 1 and args.overlap == "ce":
        layer = layer_ce  # noqa: F811

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
        sampler.mark("layer", "start")
    t0.record()
    for _ in range(args.steps):
        step(qkv, timed=True)
    t1.record()
    sync_all()
    if sampler:
        sampler.mark("layer", "end")
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    att_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in ev_att))
    if W > 1:  # the blocking layer: both exchanges are exposed (nothing runs beside them)
        a2a_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b, _ in ev_a2a) / args.steps)
        a2a_bytes = sum(n for _, _, n in ev_a2a) / args.steps
    h3attn.check_status()

    # ---- W-way output against the 1-GPU layer on the gathered input, bit for bit
    bit_exact = None
    if W > 1:
        mine = torch.stack([o.clone() for o in step(qkv)])  # [B, sl, H*D]
        ok = True
        for b in range(B):
            full = torch.empty((S_pad, 3 * H * D), dtype=torch.bfloat16, device=dev)
            dist.all_gather_into_tensor(full, qkv[b].contiguous())
            rope_full = h3_model.rope_freqs_1d(S_pad, device=dev)[0].contiguous()
            rope_full[S:] = 0
            q, k, v = full.split(H * D, dim=-1)
            send1 = h3attn.qknorm_rope_pack(q, k, v, rope_full, ones, ones, eps, 1)
            ref = h3attn.attention(send1[0, 0], send1[0, 1], send1[0, 2], s_kv=S, layout="token")
            ok = ok and torch.equal(ref[rank * sl:rank * sl + real], mine[b, :real])
            del full, send1, ref
        flag = torch.tensor([0 if ok else 1], device=dev, dtype=torch.int32)
        dist.all_reduce(flag)
        bit_exact = int(flag.item()) == 0
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

    # the copies alone, every rank at once: the ceiling the e2e pipeline runs against
    def copy_ms(dst, src, reps=3):
        sync_all()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b) / reps)

    def both_ms(reps=3):
        """Upload and readback at once, each on its own stream as the e2e pipeline runs them."""
        sync_all()
        cur = torch.cuda.current_stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            for _ in range(reps):
                dev_in[0].copy_(host_in, non_blocking=True)
        with torch.cuda.stream(s_out):
            for _ in range(reps):
                host_out[0].copy_(dev_out[0], non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        b.record(cur)
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b) / reps)

    h2d_bytes, d2h_bytes = qkv.numel() * 2, B * sl * H * D * 2  # per rank per step
    h2d_alone = copy_ms(dev_in[0], host_in)
    d2h_alone = copy_ms(host_out[0], dev_out[0])
    copies_together = both_ms()
    del dev_in, dev_out, host_in, host_out

    # ---- the reference's own GPU call at config 1 on the same box (context for the kernel's speed)
    vendor = None
    if W == 1 and B == 1 and not args.no_vendor:
        vendor = vendor_attention(qkv[0], rope, ones, eps, S, att_ms)
    del qkv
    torch.cuda.empty_cache()

    # ---- config 3: the 50-block run_blocks forward through the installed runtime
    rb = None
    if args.rb_blocks > 0 and B == 1:
        rb = run_blocks_bench(args, rank, W, dev, sampler, max_over_ranks, sync_all)

    if sampler:
        sampler.stop()
    if rank != 0:
        return
    fl = flops_layer(S) * B
    burst, sustained, hbm, kind = peaks()
    att_fl = 4.0 * S * S * D * heads_per_launch  # one attention launch
    achieved = att_fl / (att_ms * 1e-3) / 1e12
    traffic = profiled_traffic("attn_fwd_s8192_h56_full.md", S, hl)
    # our kernels per step: pack, attention (W=1); + seq->head unpack and head->seq unpack (W>1),
    # the unpack and attention once per local head when pipelined by heads
    per_step = 2 if W == 1 or peer_bufs is not None else (
        3 if ce_bufs is not None else (4 if heads_per_launch == hl else 2 + 2 * hl))
    launches = per_step * B * args.steps
    e2e_bound_ms = max(ms, h2d_alone, d2h_alone, copies_together)
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
                "h2d_bytes_per_step": h2d_bytes * W, "d2h_bytes_per_step": d2h_bytes * W,
                "h2d_gbs_per_rank": h2d_bytes / (e2e_ms * 1e-3) / 1e9,
                "d2h_gbs_per_rank": d2h_bytes / (e2e_ms * 1e-3) / 1e9,
                "copy_ceiling": {"h2d_ms": h2d_alone, "d2h_ms": d2h_alone, "h2d_and_d2h_together_ms": copies_together,
                                 "h2d_gbs_per_rank": h2d_bytes / (h2d_alone * 1e-3) / 1e9,
                                 "d2h_gbs_per_rank": d2h_bytes / (d2h_alone * 1e-3) / 1e9,
                                 "how": f"each copy alone, then both at once on their own streams, all {W} ranks"
                                        f" at once, pinned host memory"
                                        + (f" on {numa}" if numa else "")},
                "bound_ms": e2e_bound_ms, "frac_of_bound": e2e_bound_ms / e2e_ms},
        "gpu_launches": launches,
        "clocks": sampler.summary("layer") if sampler else None,
    }
    if W > 1 and peer_bufs is not None:
        # the exchanges are stores of the pack and attention kernels; only the barriers stand alone
        sent = B * 4 * sl * H * D * 2 * (W - 1) / W  # q, k, v and O rows bound for other ranks
        line["a2a"] = {"barrier_ms_per_step": a2a_ms, "bytes_sent_per_gpu_per_step": sent,
                       "mode": "fused into the pack and attention kernels (NVLink peer stores)",
                       "frac_of_step": a2a_ms / ms}
    elif W > 1:
        gbs = a2a_bytes / (a2a_ms * 1e-3) / 1e9
        key = "exposed_ms_per_step" if args.overlap in ("none", "ce") else "comm_stream_ms_per_step_overlapped"
        line["a2a"] = {key: a2a_ms, "bytes_sent_per_gpu_per_step": a2a_bytes,
                       "mode": "copy engines into peers' buffers + barrier" if args.overlap == "ce" else "NCCL all_to_all_single",
                       "achieved_gbs_per_gpu": gbs, "frac_of_nvlink": gbs / NVLINK_GBS,
                       "nvlink_ref": f"{NVLINK_GBS:.0f} GB/s per direction per GPU (measured peer copy)",
                       "frac_of_step": a2a_ms / ms}
    if W == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        times, cfl, sample = cpu_config0(3, threads)
        per = statistics.median(times)
        line["cpu_baseline"] = {"value": cfl / per / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": sample, "ms": per * 1e3}
    if vendor is not None:
        line["vendor_attention"] = vendor
    if rb is not None:
        line["run_blocks"] = rb
    if bit_exact is not None:
        line["bit_exact_vs_w1"] = bit_exact
    print(json.dumps(line), flush=True)
    if bit_exact is False or (rb is not None and rb.get("bit_exact_vs_w1") is False):
        raise SystemExit("W-way output differs from the 1-GPU output")


def vendor_attention(x, rope, ones, eps, S, our_ms):
    """torch SDPA (the reference's call, sp_runtime.py:119-121) on the bench's own packed q, k, v
    [1, 56, S, 128] bf16, by backend: 1 warm-up + 3 timed calls each, CUDA events."""
    import h3attn
    from torch.nn.attention import SDPBackend, sdpa_kernel
    q, k, v = x.split(HEADS * D, dim=-1)
    send = h3attn.qknorm_rope_pack(q, k, v, rope, ones, ones, eps, 1)
    qh, kh, vh = (send[0, i][None] for i in range(3))
    out = {}
    for name, backend in (("flash", SDPBackend.FLASH_ATTENTION), ("cudnn", SDPBackend.CUDNN_ATTENTION)):
        try:
            with sdpa_kernel([backend]):
                torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(3):
                    torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
                b.record()
                torch.cuda.synchronize()
            ms = a.elapsed_time(b) / 3
            out[name] = {"ms": ms, "tflops": flops_layer(S) / (ms * 1e-3) / 1e12, "ours_speedup": ms / our_ms}
        except RuntimeError as exc:
            out[name] = {"unavailable": str(exc).splitlines()[0][:160]}
    out["call"] = "torch.nn.functional.scaled_dot_product_attention, [1,56,S,128] bf16, per SDPBackend"
    return out


def run_blocks_bench(args, rank, W, dev, sampler, max_over_ranks, sync_all):
    """Config 3: the 50-block MiniMax-H3 denoiser forward (run_blocks) through the installed runtime,
    as the reference's full-step harness measures it (harness/sp_full_step.py:48-93): hidden 5376,
    56x128 heads, SwiGLU 14336, AdaLN from a sinusoidal t=500 embedding, bf16 weights and biases ~N(0, 0.02),
    the packed [512 | 1024 | 1464 | 39000] sequence of x ~N(0, 1). Returns the run_blocks record."""
    import h3_model as M
    import h3attn
    import sp_runtime

    sp_runtime.init()
    S = args.rb_seq
    blocks = args.rb_blocks
    model = M.MiniMaxH3Model(n_blocks=blocks, dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)  # the same parameters on every rank
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, torch.nn.Linear):
                m.weight.normal_(0.0, 0.02, generator=g)
                if m.bias is not None:  # nn.Linear's default bias init would differ between ranks
                    m.bias.normal_(0.0, 0.02, generator=g)
    segs = [(a, min(b, S), r) for a, b, r in M.H3_SEGMENTS if a < S]
    h = torch.randn((S, M.HIDDEN), generator=torch.Generator(device=dev).manual_seed(4), device=dev).to(torch.bfloat16)
    t_emb = M.timestep_embedding(torch.full((len(segs),), 500.0, device=dev)).to(torch.bfloat16)
    rope = M.rope_freqs_1d(S, device=dev)
    sp_runtime.install(M)

    def fwd():
        with torch.no_grad():
            return model.run_blocks(h, t_emb, segs, rope, {})

    fwd()  # warm-up (also runs the runtime's status check)
    sync_all()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.mark("run_blocks", "start")
    a.record()
    for _ in range(args.rb_steps):
        out = fwd()
    b.record()
    sync_all()
    if sampler:
        sampler.mark("run_blocks", "end")
    ms = max_over_ranks(a.elapsed_time(b) / args.rb_steps)
    h3attn.check_status()
    # one more forward with the runtime's per-category CUDA-event timing (SP_TIMING), MAX over ranks
    sp_runtime._TIMING = True
    fwd()
    sp_runtime._TIMING = False
    cats = sp_runtime.get_timing()
    cat_ms = {k: max_over_ranks(cats.get(k, 0.0)) for k in sp_runtime.CATEGORIES}
    rec = {"ms": ms, "forwards": args.rb_steps, "blocks": blocks, "seq_len": S,
           "tflops": forward_flops(S, blocks) / (ms * 1e-3) / 1e12, "flop_per_forward": forward_flops(S, blocks),
           "categories_ms": {k: round(v, 1) for k, v in cat_ms.items()},
           "clocks": sampler.summary("run_blocks") if sampler else None}
    if W > 1:
        # the same forward on this GPU alone (the runtime's W=1 seam, same kernels), compared bit for bit
        world, rnk = sp_runtime.WORLD, sp_runtime.RANK
        sp_runtime.WORLD, sp_runtime.RANK = 1, 0
        try:
            one = fwd()
        finally:
            sp_runtime.WORLD, sp_runtime.RANK = world, rnk
        flag = torch.tensor([0 if torch.equal(one, out) else 1], device=dev, dtype=torch.int32)
        dist.all_reduce(flag)
        rec["bit_exact_vs_w1"] = int(flag.item()) == 0
    sp_runtime.uninstall()
    del model, h, out
    torch.cuda.empty_cache()
    return rec


def forward_flops(s: int, blocks: int, hidden=5376, heads=56, head_dim=128, ffn=14336) -> float:
    """Projection GEMMs (qkv, out, fc1 with both SwiGLU halves, fc2) plus attention, per forward."""
    hd = heads * head_dim
    gemm = 2.0 * s * (hidden * 3 * hd + hd * hidden + hidden * 2 * ffn + ffn * hidden)
    return blocks * (gemm + flops_layer(s, heads))


# ----------------------------------------------------------------------------- single-kernel cases
CASES = ("attn", "pack", "gemm_qkv", "gemm_out", "gemm_fc1", "gemm_fc2", "norm_mod", "residual")


def run_case(args) -> None:
    """One kernel of the path at a chosen size, for profiling (ncu -k <kernel> python bench.py --case ...):
    `warmup` untimed launches, then `steps` launches timed with CUDA events; prints one JSON line with the
    per-launch time and the kernel's rate against its roofline unit. Sizes: --seq rows (tokens), 56 heads,
    hidden 5376, FFN 14336; inputs are seeded N(0, 1) (weights N(0, 0.02))."""
    import h3attn
    import h3_model

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    S, hidden, ffn = args.seq, 5376, 14336
    rnd = lambda *shape, s=1.0: (torch.randn(shape, device=dev, generator=g) * s).to(torch.bfloat16)
    if args.case == "attn":
        q, k, v = (rnd(HEADS, S, D) for _ in range(3))
        o = torch.empty_like(q)
        fn = lambda: h3attn.attention(q, k, v, out=o)
        work, unit = flops_layer(S), "TFLOP/s"
    elif args.case == "pack":
        x = rnd(S, 3 * HEADS * D)
        rope = h3_model.rope_freqs_1d(S, device=dev)[0].contiguous()
        ones = torch.ones(D, dtype=torch.bfloat16, device=dev)
        q, k, v = x.split(HEADS * D, dim=-1)
        fn = lambda: h3attn.qknorm_rope_pack(q, k, v, rope, ones, ones, 1e-6, 1)
        work, unit = S * 3 * HEADS * D * 2 * 2 + S * 1024, "GB/s"
    elif args.case.startswith("gemm_"):
        k_in, n_out, ep = {"gemm_qkv": (hidden, 3 * HEADS * D, "none"), "gemm_out": (HEADS * D, hidden, "none"),
                           "gemm_fc1": (hidden, 2 * ffn, "swiglu"), "gemm_fc2": (ffn, hidden, "none")}[args.case]
        a, w = rnd(S, k_in), rnd(n_out, k_in, s=0.02)
        out = h3attn.linear(a, w, epilogue=ep)
        fn = lambda: h3attn.linear(a, w, out=out, epilogue=ep)
        work, unit = 2.0 * S * k_in * n_out, "TFLOP/s"
    else:
        x, y = rnd(S, hidden), rnd(S, hidden)
        mods = rnd(4, hidden, s=0.1)
        seg = h3attn.segment_rows([(0, S // 2, 0), (S // 2, S, 1)], S, dev)
        if args.case == "norm_mod":
            xo, ho = torch.empty_like(x), torch.empty_like(x)
            fn = lambda: h3attn.norm_modulate(x, mods[0:2], mods[2:4], seg, 1e-6, y=y, gate=mods[0:2], x_out=xo,
                                              out=ho)
            work = S * hidden * 2 * 4  # read x, y; write x_out, h
        else:
            ro = torch.empty_like(x)
            fn = lambda: h3attn.gated_residual(x, y, mods[0:2], seg, out=ro)
            work = S * hidden * 2 * 3  # read x, y; write out
        unit = "GB/s"
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        fn()
    ev1.record()
    torch.cuda.synchronize()
    h3attn.check_status()
    ms = ev0.elapsed_time(ev1) / args.steps
    rate = work / (ms * 1e-3) / (1e12 if unit == "TFLOP/s" else 1e9)
    print(json.dumps({"case": args.case, "rows": S, "ms_per_launch": ms, "achieved": rate, "unit": unit,
                      "launches": args.steps}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seq", type=int, default=42000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-vendor", action="store_true", help="skip timing torch SDPA at N=1")
    ap.add_argument("--no-numa-bind", action="store_true", help="leave host buffers wherever the OS puts them")
    ap.add_argument("--batch", type=int, default=1, help="independent sequences per step (config 4: 2)")
    ap.add_argument("--overlap", default="none", choices=["none", "heads", "peer", "ce"],
                    help="W>1: exchanges pipelined head by head, fused into the kernels over peer memory, "
                         "or done by the copy engines straight into peers' buffers")
    ap.add_argument("--rb-blocks", type=int, default=50, help="config 3 run_blocks forward depth (0: skip)")
    ap.add_argument("--rb-seq", type=int, default=42000)
    ap.add_argument("--rb-steps", type=int, default=2, help="timed run_blocks forwards")
    ap.add_argument("--case", choices=CASES, default=None,
                    help="time one kernel of the path alone at --seq rows (profiling); 1 GPU, no JSON contract")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.case is not None:
        run_case(args)
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
