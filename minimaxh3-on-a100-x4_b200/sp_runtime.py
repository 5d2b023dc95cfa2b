"""B200 drop-in for the reference's Ulysses sequence-parallel runtime (harness/sp_runtime.py).

Same module API and behaviour, B200 data path underneath:

  init()                       process group (NCCL) + device          (ref :60-65)
  install(module=None)         patch MiniMaxH3Model.run_blocks,        (ref :258-271)
                               Attention.forward and MLP.forward of the host model module
  a2a_seq_to_head(x, world)    [1, H, Sl, d] -> [1, H/W, S, d]         (ref :67-71)
  a2a_head_to_seq(x, world, H) [1, H/W, S, d] -> [1, H, Sl, d]         (ref :73-77)
  get_timing()                 per-category ms of the last run_blocks  (ref :57-58)
  RANK, WORLD                  module constants from the environment   (ref :16-17)
  env SP_TIMING=1, SP_OVERLAP=1, SP_PIECES=N                           (ref :32, :133, :265)
  env SP_OVERLAP=heads         head-by-head all-to-all / attention pipelining (this build)
  env SP_OVERLAP=peer          all-to-alls fused into pack / attention over peer memory (this build)
  env SP_OVERLAP=ce            all-to-alls as copy-engine copies into peers' final buffers (this build)

What differs, by design:
  * The attention layer runs on libh3attn.so (sm_100a): one fused kernel does the q/k
    RMSNorm + RoPE and writes q, k, v straight into the all-to-all send buffer (one
    exchange for all three), the attention kernel reads the unpacked receive buffer and
    writes O straight into the head->seq send layout (or, at W=1, token-major for out_proj).
  * The projections run on the library's row-independent GEMM (h3_gemm_bf16): qkv_proj,
    out_proj (at W > 1 reading the head->seq receive buffer in place, no unpack pass) and,
    through a patched MLP.forward (the reference's block-loop harness patches the same method,
    harness/sp_blockloop.py:167-170), fc1 with the SwiGLU fused into its epilogue, then fc2.
    An output row's bits do not depend on the shard it is computed in, so the whole layer and
    block loop are bit-exact across W. A projection whose weight is not a bias-free bf16
    matrix falls back to the host module's own op.
  * The block's AdaLN modulation and gated residuals run as three fused passes per block
    (h3_norm_modulate, h3_gated_residual) when its norms are affine-free LayerNorms and the
    activations are bf16 on the GPU; otherwise the host block runs.
  * WORLD == 1 runs the same seam with this library's attention instead of falling through
    to the host model's own loop (ref :222-223), so W-way output is bit-exact against the
    1-GPU output of the same kernels.
  * The SLA sparse-attention branch (ref :79-83, :111-118) is not carried: attention is
    always the exact dense op.
  * install() takes the host module as an optional argument (default: ComfyUI's
    comfy.ldm.minimax.model, as in the reference) and uninstall() restores it.
  * SP_BACKEND selects the process-group backend (default nccl); LOCAL_RANK, when set,
    picks the device (torchrun); otherwise cuda:0 as in the reference.

There is no CPU path: the kernels live in h3attn (libh3attn.so) and raise if it is absent.
"""
from __future__ import annotations

import contextlib
import os
import time
import warnings
from datetime import timedelta

import torch
import torch.distributed as dist

RANK = int(os.environ.get("RANK", "0"))
WORLD = int(os.environ.get("WORLD_SIZE", "1"))
_INIT = False

# SP attention is scoped to the block loop: run_blocks sets _SP_ACTIVE while the sharded
# loop runs and the patched attention defers to the host model's own forward otherwise.
# _SP_REAL_S is the unpadded sequence length: keys/values stop there (pad path).
_SP_ACTIVE = False
_SP_REAL_S = None
_orig_attn_forward = None
_orig_run_blocks = None
_orig_mlp_forward = None
_MODULE = None

_ops = None  # the kernel library binding (h3attn); resolved on first use


def ops():
    global _ops
    if _ops is None:
        import h3attn
        h3attn.lib()  # fail loudly here if libh3attn.so is missing
        _ops = h3attn
    return _ops


# ---- per-category timing of run_blocks (SP_TIMING=1) ----
# The categories are the reference's (sp_runtime.py:31-58, consumed by harness/sp_full_step.py:66):
# norm_mod, qkv, a2a_fwd, fa2_local, a2a_inv, out_proj, residual, ffn, gather.
_TIMING = os.environ.get("SP_TIMING") == "1"
CATEGORIES = ("norm_mod", "qkv", "a2a_fwd", "fa2_local", "a2a_inv", "out_proj", "residual", "ffn", "gather")
_timeline = None   # the _Timeline of the run_blocks call in progress, when timing
_last_totals = {}  # category -> ms of the last finished run_blocks call


class _Timeline:
    """Spans of one run_blocks call. On the GPU each span is a pair of CUDA events recorded on the
    current stream, so totals are device time and reading them needs one synchronisation at the end
    of the call; on host tensors (the CPU gloo tests) the host clock brackets the span."""

    def __init__(self, on_gpu: bool):
        self.on_gpu = on_gpu
        self.marks = []  # (category, start, end)

    def _stamp(self):
        if self.on_gpu:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            return ev
        return time.perf_counter()

    @contextlib.contextmanager
    def span(self, cat: str):
        t0 = self._stamp()
        try:
            yield
        finally:
            self.marks.append((cat, t0, self._stamp()))

    def totals(self) -> dict:
        if self.on_gpu:
            torch.cuda.synchronize()
        out = {}
        for cat, a, b in self.marks:
            ms = a.elapsed_time(b) if self.on_gpu else (b - a) * 1e3
            out[cat] = out.get(cat, 0.0) + ms
        return out


def _span(cat: str):
    """Context manager booking the enclosed work under `cat` while a timed run_blocks is running."""
    return _timeline.span(cat) if _timeline is not None else contextlib.nullcontext()


def get_timing():
    """Per-category ms of the last run_blocks call (empty unless SP_TIMING=1)."""
    return dict(_last_totals)


def init(timeout_s: float | None = None):
    """Join the process group (when WORLD > 1) and select this rank's device."""
    global _INIT
    if torch.cuda.is_available():
        local = int(os.environ.get("LOCAL_RANK", "0")) if torch.cuda.device_count() > 1 else 0
        torch.cuda.set_device(local)
    if WORLD > 1 and not dist.is_initialized():
        backend = os.environ.get("SP_BACKEND", "nccl")
        kw = {"timeout": timedelta(seconds=timeout_s)} if timeout_s else {}
        dist.init_process_group(backend, rank=RANK, world_size=WORLD, **kw)
    _INIT = True


def _exchange(send: torch.Tensor) -> torch.Tensor:
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)
    return recv


def a2a_seq_to_head(x, world):  # [1,H,Sl,d] -> [1,Hl,S,d]
    _, H, Sl, d = x.shape
    hl = H // world
    send = x.reshape(world, 1, hl, Sl, d).contiguous()
    recv = _exchange(send) if world > 1 else send
    return ops().seq_to_head_unpack(recv)[0].unsqueeze(0)


def a2a_head_to_seq(x, world, H):  # [1,Hl,S,d] -> [1,H,Sl,d]
    _, hl, S, d = x.shape
    Sl = S // world
    send = x[0].view(hl, world, Sl, d).permute(1, 0, 2, 3).contiguous()
    recv = _exchange(send) if world > 1 else send
    return recv.reshape(1, H, Sl, d)


def _h3sla_schedule(transformer_options):
    """The reference's SLA hook (sp_runtime.py:79-83). Sparse attention is not carried:
    this runtime always runs the exact dense op, so there is never a schedule."""
    return None


def _norm_inputs(self, x, rope_freqs):
    rope = None
    if rope_freqs is not None:
        rot = rope_freqs.shape[-3] * 2
        if rot != self.head_dim:
            raise NotImplementedError(f"rotary dim {rot} != head_dim {self.head_dim} is not supported")
        rope = rope_freqs[0] if rope_freqs.dim() == 5 else rope_freqs
        if rope.dtype != torch.float32:
            rope = rope.float()
    qw = getattr(self.q_norm, "weight", None)
    kw = getattr(self.k_norm, "weight", None)
    if qw is not None:
        qw = qw.to(device=x.device, dtype=x.dtype).contiguous()
    if kw is not None:
        kw = kw.to(device=x.device, dtype=x.dtype).contiguous()
    return rope, qw, kw


_STRICT = os.environ.get("SP_STRICT") == "1"
_fallbacks_seen = set()


def _host_fallback(what: str, why: str) -> None:
    """A projection or block the library's kernels cannot take runs on the host module's own torch
    ops. Said once per kind on rank 0; with SP_STRICT=1 it is an error instead."""
    if _STRICT:
        raise RuntimeError(f"sp_runtime: {what} would fall back to the host module's ops ({why}); SP_STRICT=1")
    key = (what, why)
    if key not in _fallbacks_seen:
        _fallbacks_seen.add(key)
        if RANK == 0:
            warnings.warn(f"sp_runtime: {what} runs on the host module's ops ({why})", RuntimeWarning, stacklevel=3)


def _gemm_weight(lin, x):
    """The weight of a bias-free bf16 Linear that the projection GEMM takes for input x, or None
    (then the host module's own op runs, as in the reference, and the fallback is reported)."""
    w = getattr(lin, "weight", None)
    why = None
    if not isinstance(w, torch.Tensor):
        why = "no weight tensor"
    elif getattr(lin, "bias", None) is not None:
        why = "the linear has a bias"
    elif w.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
        why = f"dtype {w.dtype} weight / {x.dtype} input (bf16 needed)"
    elif w.dim() != 2 or w.device != x.device:
        why = "weight shape or device"
    if why is not None:
        if x.is_cuda:
            _host_fallback("a projection", why)
        return None
    return w


def _sp_mlp_forward(self, x):
    """SwiGLU FFN (fc1 -> chunk(2) -> silu(gate) * up -> fc2) as two projection GEMMs, the
    SwiGLU fused into fc1's epilogue (cf. harness/sp_blockloop.py:167-170)."""
    w1, w2 = _gemm_weight(self.fc1, x), _gemm_weight(self.fc2, x)
    if not _SP_ACTIVE or w1 is None or w2 is None or x.dim() != 2:
        return _orig_mlp_forward(self, x)
    O = ops()
    return O.linear(O.linear(x, w1, epilogue="swiglu"), w2)


def _sp_attn_forward(self, x, rope_freqs=None, transformer_options={}):
    if not _SP_ACTIVE:
        return _orig_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    O = ops()
    s = x.shape[0]
    H, D, W = self.heads, self.head_dim, WORLD
    with _span("qkv"):
        w_qkv = _gemm_weight(self.qkv_proj, x)
        qkv = O.linear(x, w_qkv) if w_qkv is not None else self.qkv_proj(x)
        q, k, v = qkv.split(H * D, dim=-1)
        rope, qw, kw = _norm_inputs(self, x, rope_freqs)
        send = O.qknorm_rope_pack(q, k, v, rope, qw, kw, self.q_norm.eps, W)  # [W, 3, H/W, s, D]
    with _span("a2a_fwd"):
        qkvh = O.seq_to_head_unpack(_exchange(send)) if W > 1 else send[0]  # [3, H/W, W*s, D]
    with _span("fa2_local"):
        S_pad = W * s
        s_kv = _SP_REAL_S if (_SP_REAL_S is not None and _SP_REAL_S < S_pad) else S_pad
        if W > 1:
            o_send = O.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=s_kv, layout="send", world=W)
        else:
            o = O.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=s_kv, layout="token")
    with _span("a2a_inv"):
        if W > 1:
            o_recv = _exchange(o_send)  # [W, H/W, s, D] == [H, s, D]
    with _span("out_proj"):
        w_out = _gemm_weight(self.out_proj, x)
        if W > 1:
            o_heads = o_recv.view(H, s, D)
            if w_out is not None:
                return O.linear(o_heads, w_out)  # reads [H, s, D] as [s, H*D] in place
            o = O.head_to_seq_unpack(o_heads)
        return O.linear(o, w_out) if w_out is not None else self.out_proj(o)


# ---- comm/compute overlap (exact): Q and O exchanged in token pieces on a side stream ----
_PIECES = int(os.environ.get("SP_PIECES", "4"))
_comm_stream = None
_side_stream = None


def _piece_bounds(n, p):
    base, rem = divmod(n, p)
    out, s = [], 0
    for i in range(p):
        ln = base + (1 if i < rem else 0)
        if ln == 0:
            continue
        out.append((s, s + ln))
        s += ln
    return out


def _sp_attn_forward_overlap(self, x, rope_freqs=None, transformer_options={}):
    if not _SP_ACTIVE:
        return _orig_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    if WORLD == 1:
        return _sp_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    global _comm_stream
    if _comm_stream is None:
        _comm_stream = torch.cuda.Stream()
    O = ops()
    s = x.shape[0]
    H, D, W = self.heads, self.head_dim, WORLD
    w_qkv = _gemm_weight(self.qkv_proj, x)
    qkv = O.linear(x, w_qkv) if w_qkv is not None else self.qkv_proj(x)
    q, k, v = qkv.split(H * D, dim=-1)
    rope, qw, kw = _norm_inputs(self, x, rope_freqs)
    send = O.qknorm_rope_pack(q, k, v, rope, qw, kw, self.q_norm.eps, W)  # [W, 3, H/W, s, D]
    kvh = O.seq_to_head_unpack(_exchange(send[:, 1:].contiguous()))  # K, V first (blocking)
    S_pad = W * s
    s_kv = _SP_REAL_S if (_SP_REAL_S is not None and _SP_REAL_S < S_pad) else S_pad
    pieces = _piece_bounds(s, _PIECES)
    default = torch.cuda.current_stream()
    _comm_stream.wait_stream(default)
    o = torch.empty((s, H * D), dtype=x.dtype, device=x.device)

    def q_piece(lo, hi):
        qh = O.seq_to_head_unpack(_exchange(send[:, 0:1, :, lo:hi].contiguous()))[0]  # [H/W, W*n, D]
        qh.record_stream(default)
        return qh

    with torch.cuda.stream(_comm_stream):
        qh_next = q_piece(*pieces[0])
    for i, (lo, hi) in enumerate(pieces):
        default.wait_stream(_comm_stream)
        qh_p = qh_next
        if i + 1 < len(pieces):
            with torch.cuda.stream(_comm_stream):
                qh_next = q_piece(*pieces[i + 1])
        o_send = O.attention(qh_p, kvh[0], kvh[1], s_kv=s_kv, layout="send", world=W)
        with torch.cuda.stream(_comm_stream):
            _comm_stream.wait_stream(default)
            o_send.record_stream(_comm_stream)
            O.head_to_seq_unpack(_exchange(o_send).view(H, hi - lo, D), out=o[lo:hi])
    default.wait_stream(_comm_stream)
    w_out = _gemm_weight(self.out_proj, x)
    return O.linear(o, w_out) if w_out is not None else self.out_proj(o)


def _sp_attn_forward_heads(self, x, rope_freqs=None, transformer_options={}):
    """Same math, pipelined by heads (this build's SP_OVERLAP=heads; the reference pipelines token
    pieces): the pack writes the send buffer head-major, each local head's q/k/v travels in its own
    all-to-all on a side stream, and head h's attention and O exchange overlap the exchanges of the
    heads after it. Consecutive heads alternate between two compute streams: one head's attention
    grid is about one wave, so the next head fills the SMs its tail leaves idle. Heads are
    independent, so the output is bit-identical to the blocking path."""
    if not _SP_ACTIVE:
        return _orig_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    if WORLD == 1:
        return _sp_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    global _comm_stream, _side_stream
    if _comm_stream is None:
        _comm_stream = torch.cuda.Stream()
    if _side_stream is None:
        _side_stream = torch.cuda.Stream()
    O = ops()
    s = x.shape[0]
    H, D, W = self.heads, self.head_dim, WORLD
    hl = H // W
    with _span("qkv"):
        w_qkv = _gemm_weight(self.qkv_proj, x)
        qkv = O.linear(x, w_qkv) if w_qkv is not None else self.qkv_proj(x)
        q, k, v = qkv.split(H * D, dim=-1)
        rope, qw, kw = _norm_inputs(self, x, rope_freqs)
        send = O.qknorm_rope_pack(q, k, v, rope, qw, kw, self.q_norm.eps, W, head_major=True)  # [hl, W, 3, s, D]
    S_pad = W * s
    s_kv = _SP_REAL_S if (_SP_REAL_S is not None and _SP_REAL_S < S_pad) else S_pad
    default = torch.cuda.current_stream()
    o_heads = torch.empty((W, hl, s, D), dtype=x.dtype, device=x.device)  # == [H, s, D], head g = src*hl + h
    with _span("fa2_local"):
        _comm_stream.wait_stream(default)
        _side_stream.wait_stream(default)
        send.record_stream(_comm_stream)
        o_heads.record_stream(_comm_stream)
        recvs, arrived = [], []
        with torch.cuda.stream(_comm_stream):
            for h in range(hl):
                recvs.append(_exchange(send[h]))  # [W(src), 3, s, D]
                arrived.append(torch.cuda.Event())
                arrived[-1].record(_comm_stream)
        for h in range(hl):
            cs = default if h % 2 == 0 else _side_stream
            cs.wait_event(arrived[h])
            recvs[h].record_stream(cs)
            with torch.cuda.stream(cs):
                qkvh = O.seq_to_head_unpack(recvs[h].view(W, 3, 1, s, D))  # [3, 1, W*s, D]
                o_send = O.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=s_kv, layout="send", world=W)  # [W, 1, s, D]
                done = torch.cuda.Event()
                done.record(cs)
            o_send.record_stream(_comm_stream)
            with torch.cuda.stream(_comm_stream):
                _comm_stream.wait_event(done)
                o_heads[:, h].copy_(_exchange(o_send).view(W, s, D))
        default.wait_stream(_side_stream)
        default.wait_stream(_comm_stream)
    with _span("out_proj"):
        w_out = _gemm_weight(self.out_proj, x)
        o_hsd = o_heads.view(H, s, D)
        return O.linear(o_hsd, w_out) if w_out is not None else self.out_proj(O.head_to_seq_unpack(o_hsd))


_peer_cache = {}


def _peer_buffers(s, H, D, dev, slots=1):
    """Symmetric-memory buffers for the fused exchanges of one layer shape, allocated and
    rendezvoused once (a collective: every rank reaches it with the same shape): per slot the
    attention input [3][H/W][W*s][D] that every rank's pack writes into, and the out_proj input
    [s][H*D] that every rank's attention writes into; device tables of every rank's addresses."""
    key = (s, H, D, str(dev), slots)
    if key in _peer_cache:
        return _peer_cache[key]
    # plain peer mappings only: the kernels store into peers' buffers, nothing uses multicast
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    import torch.distributed._symmetric_memory as symm
    W, hl = WORLD, H // WORLD
    group = dist.group.WORLD
    if hasattr(symm, "enable_symm_mem_for_group"):
        symm.enable_symm_mem_for_group(group.group_name)

    def table(t, extra_bytes):
        h = symm.rendezvous(t, group)
        ptrs = [int(p) + int(h.offset) for p in h.buffer_ptrs]
        if ptrs[RANK] != t.data_ptr():
            raise RuntimeError("symmetric buffer addresses do not match the local tensor")
        return h, torch.tensor([p + extra_bytes for p in ptrs], dtype=torch.int64, device=dev)

    out = []
    for _ in range(slots):
        qkv = symm.empty((3, hl, W * s, D), dtype=torch.bfloat16, device=dev)
        o = symm.empty((s, H * D), dtype=torch.bfloat16, device=dev)
        hq, qkv_ptrs = table(qkv, 0)
        ho, o_ptrs = table(o, RANK * hl * D * 2)  # this rank's column block of every peer's [s][H*D]
        out.append({"qkv": qkv, "o": o, "qkv_ptrs": qkv_ptrs, "o_ptrs": o_ptrs, "handles": (hq, ho)})
    flag = torch.zeros(1, dtype=torch.float32, device=dev)
    for b in out:
        b["flag"] = flag
    _peer_cache[key] = out
    return out


def _peer_barrier(flag):
    """Stream-ordered barrier: an NCCL all-reduce of one element completes on a rank only after
    every rank has enqueued it, i.e. after every rank's preceding kernels (whose peer stores end
    with a system-scope fence)."""
    dist.all_reduce(flag)


def _sp_attn_forward_peer(self, x, rope_freqs=None, transformer_options={}):
    """Same math with both all-to-alls fused into the kernels over NVLink peer memory (this build's
    SP_OVERLAP=peer): the pack writes every head straight into its destination rank's attention
    input, the attention epilogue writes every query row straight into its destination rank's
    out_proj input; two stream-ordered barriers per layer. Bit-identical to the blocking path."""
    if not _SP_ACTIVE:
        return _orig_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    if WORLD == 1:
        return _sp_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    O = ops()
    s = x.shape[0]
    H, D, W = self.heads, self.head_dim, WORLD
    hl = H // W
    buf = _peer_buffers(s, H, D, x.device)[0]
    S_pad = W * s
    s_kv = _SP_REAL_S if (_SP_REAL_S is not None and _SP_REAL_S < S_pad) else S_pad
    with _span("qkv"):
        w_qkv = _gemm_weight(self.qkv_proj, x)
        qkv = O.linear(x, w_qkv) if w_qkv is not None else self.qkv_proj(x)
        q, k, v = qkv.split(H * D, dim=-1)
        rope, qw, kw = _norm_inputs(self, x, rope_freqs)
        O.qknorm_rope_pack_peer(q, k, v, rope, qw, kw, self.q_norm.eps, W, buf["qkv_ptrs"], hl * S_pad * D,
                                S_pad * D, RANK * s)
    with _span("a2a_fwd"):
        _peer_barrier(buf["flag"])  # every rank's q/k/v rows have landed
    with _span("fa2_local"):
        qkvh = buf["qkv"]
        O.attention_peer(qkvh[0], qkvh[1], qkvh[2], buf["o"], buf["o_ptrs"], s, D, H * D, s_kv=s_kv)
    with _span("a2a_inv"):
        _peer_barrier(buf["flag"])  # every rank's output rows for this rank have landed
    with _span("out_proj"):
        w_out = _gemm_weight(self.out_proj, x)
        return O.linear(buf["o"], w_out) if w_out is not None else self.out_proj(buf["o"].clone())


_ce_streams = {}


def _ce_geometry(s: int, H: int, D: int, W: int, rank: int) -> dict:
    """Byte geometry of this rank's two copy-engine exchanges, the same for every destination:
    qkv: (offset into the destination's [3][H/W][W*s][D] attention input, its row pitch, bytes per
         row, rows) -- row (t, h) of this rank's send chunk [3][H/W][s][D] lands at rows rank*s...;
    o:   (offset into the destination's [H][s][D] out_proj input, bytes) -- this rank's H/W heads.
    Elements are 2-byte bf16."""
    hl = H // W
    row = s * D * 2
    return {"qkv": (rank * row, W * s * D * 2, row, 3 * hl), "o": (rank * hl * s * D * 2, hl * s * D * 2)}


def _ce_copies(bases, offset, dst_pitch, chunks, width, rows, dev):
    """One copy-engine copy per destination rank d: `rows` rows of `width` bytes from chunks[d] to
    bases[d] + offset (row pitch dst_pitch), each on its own side stream ordered after the current
    stream's work; the current stream then waits for all of them."""
    cur = torch.cuda.current_stream()
    streams = _ce_streams.get(str(dev))
    if streams is None:
        streams = _ce_streams[str(dev)] = [torch.cuda.Stream(device=dev) for _ in range(WORLD)]
    for d in range(WORLD):
        st = streams[d]
        st.wait_stream(cur)
        chunks[d].record_stream(st)
        ops().copy_2d(bases[d] + offset, dst_pitch, chunks[d].data_ptr(), width, width, rows, stream=st)
    for st in streams:
        cur.wait_stream(st)


def _sp_attn_forward_ce(self, x, rope_freqs=None, transformer_options={}):
    """Same math with both all-to-alls done by the GPU's copy engines (this build's SP_OVERLAP=ce):
    the pack writes the usual send buffer; one 2-D copy per destination rank puts this rank's q/k/v
    rows straight into that rank's attention input [3][H/W][W*s][D] (symmetric memory, rows
    RANK*s...), and one contiguous copy per destination puts this rank's attention output heads into
    that rank's [H][s][D] out_proj input, which out_proj reads in place. No kernel spends SMs on the
    exchanges and no unpack runs; a stream-ordered barrier follows each exchange. Bit-identical to
    the blocking path."""
    if not _SP_ACTIVE:
        return _orig_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    if WORLD == 1:
        return _sp_attn_forward(self, x, rope_freqs=rope_freqs, transformer_options=transformer_options)
    O = ops()
    s = x.shape[0]
    H, D, W = self.heads, self.head_dim, WORLD
    hl = H // W
    buf = _peer_buffers(s, H, D, x.device)[0]
    if "qkv_base" not in buf:  # every rank's buffer bases, on the host
        buf["qkv_base"] = buf["qkv_ptrs"].tolist()
        buf["o_base"] = [p - RANK * hl * D * 2 for p in buf["o_ptrs"].tolist()]
    S_pad = W * s
    s_kv = _SP_REAL_S if (_SP_REAL_S is not None and _SP_REAL_S < S_pad) else S_pad
    with _span("qkv"):
        w_qkv = _gemm_weight(self.qkv_proj, x)
        qkv = O.linear(x, w_qkv) if w_qkv is not None else self.qkv_proj(x)
        q, k, v = qkv.split(H * D, dim=-1)
        rope, qw, kw = _norm_inputs(self, x, rope_freqs)
        send = O.qknorm_rope_pack(q, k, v, rope, qw, kw, self.q_norm.eps, W)  # [W, 3, H/W, s, D]
    geo = _ce_geometry(s, H, D, W, RANK)
    with _span("a2a_fwd"):
        off, pitch, row, rows = geo["qkv"]
        _ce_copies(buf["qkv_base"], off, pitch, send, row, rows, x.device)
        _peer_barrier(buf["flag"])  # every rank's q/k/v rows have landed
    with _span("fa2_local"):
        qkvh = buf["qkv"]
        o_send = O.attention(qkvh[0], qkvh[1], qkvh[2], s_kv=s_kv, layout="send", world=W)  # [W, H/W, s, D]
    with _span("a2a_inv"):
        off, blk = geo["o"]
        _ce_copies(buf["o_base"], off, blk, o_send, blk, 1, x.device)
        _peer_barrier(buf["flag"])  # every rank's output heads for this rank have landed
    with _span("out_proj"):
        o_heads = buf["o"].view(H, s, D)
        w_out = _gemm_weight(self.out_proj, x)
        if w_out is not None:
            return O.linear(o_heads, w_out)  # reads [H, s, D] as [s, H*D] in place
        return self.out_proj(O.head_to_seq_unpack(o_heads))


def _shard_segments(segs, lo, hi):
    out = []
    for a, b, row in segs:
        A, B = max(a, lo), min(b, hi)
        if A < B:
            out.append((A - lo, B - lo, row))
    return out


def _host_block_timed(self, x, t_emb, mod_segments, rope_freqs, transformer_options={}):
    """The host DiTBlock.forward, op for op, with each step booked under its timing category
    (used instead of the block's own forward only while SP_TIMING=1 and only for blocks the fused
    kernels cannot take; the patched attention books its own sub-steps)."""
    MM = _MODULE
    with _span("norm_mod"):
        mods = self.adaln_proj(t_emb)
        shift1, scale1, gate1, shift2, scale2, gate2 = mods
        h = MM._mod_scale_shift(self.norm1(x), shift1, scale1, mod_segments)
    attn_out = self.attn(h, rope_freqs=rope_freqs, transformer_options=transformer_options)
    with _span("residual"):
        x = MM._mod_gate(x, gate1, attn_out, mod_segments)
    with _span("norm_mod"):
        h = MM._mod_scale_shift(self.norm2(x), shift2, scale2, mod_segments)
    with _span("ffn"):
        ffn_out = self.mlp(h)
    with _span("residual"):
        return MM._mod_gate(x, gate2, ffn_out, mod_segments)


def _fusable(blk, x) -> bool:
    """The block's norms are affine-free LayerNorms over the hidden width and x is bf16 on the GPU,
    so the fused modulation kernels reproduce the host ops (else the host block runs, reported once)."""
    if not x.is_cuda:
        return False
    why = None
    if not (x.dtype == torch.bfloat16 and x.dim() == 2 and x.shape[1] % 8 == 0 and x.shape[1] <= 8192):
        why = f"activations {x.dtype} {tuple(x.shape)} (bf16, hidden <= 8192 and a multiple of 8 needed)"
    else:
        for n in (getattr(blk, "norm1", None), getattr(blk, "norm2", None)):
            if not isinstance(n, torch.nn.LayerNorm) or n.weight is not None or n.bias is not None:
                why = "a norm that is not an affine-free LayerNorm"
            elif tuple(n.normalized_shape) != (x.shape[1],):
                why = "a norm over another width"
    if why is not None:
        _host_fallback("the AdaLN modulation of a block", why)
        return False
    return True


def _sp_block(self, x, t_emb, seg_row, rope_freqs, transformer_options={}):
    """The host block's op order (DiTBlock.forward, as the reference's timed replica walks it at
    sp_runtime.py:203-218) with the AdaLN modulation and gated residuals on the library's kernels:
    three passes over [rows, hidden]: norm1 + modulation; attention residual + norm2 + modulation;
    FFN residual."""
    O = ops()
    with _span("norm_mod"):
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.adaln_proj(t_emb)
        h = O.norm_modulate(x, shift_msa, scale_msa, seg_row, self.norm1.eps)
    a = self.attn(h, rope_freqs=rope_freqs, transformer_options=transformer_options)
    # one pass does the attention residual, norm2 and its modulation: booked as norm_mod (its bulk);
    # residual then holds the closing gated residual only
    with _span("norm_mod"):
        x1 = torch.empty_like(x)
        h = O.norm_modulate(x, shift_mlp, scale_mlp, seg_row, self.norm2.eps, y=a, gate=gate_msa, x_out=x1)
    with _span("ffn"):
        m = self.mlp(h)
    with _span("residual"):
        return O.gated_residual(x1, m, gate_mlp, seg_row)


def _gather_rows(h_loc: torch.Tensor) -> torch.Tensor:
    out = torch.empty((WORLD * h_loc.shape[0],) + tuple(h_loc.shape[1:]), dtype=h_loc.dtype, device=h_loc.device)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, h_loc.contiguous())
    else:
        dist.all_gather(list(out.chunk(WORLD, 0)), h_loc.contiguous())
    return out


def _shard_bounds(S: int, world: int, rank: int) -> tuple[int, int, int]:
    """(S_pad, lo, hi): the sequence is padded to the next multiple of world and rank holds rows
    [lo, hi) of the padded sequence (the reference's pad rule, sp_runtime.py:224-239)."""
    rows = -(-S // world)
    return rows * world, rank * rows, (rank + 1) * rows


def _sp_run_blocks(self, h, t_emb, mod_segments, rope_freqs, transformer_options={}):
    global _SP_ACTIVE, _SP_REAL_S, _timeline
    S = h.shape[0]
    S_pad, lo, hi = _shard_bounds(S, WORLD, RANK)
    # Pad rows sit after the last token: they belong to no modulation segment (scale, shift and
    # gate leave them alone), their keys are cut off inside attention (_SP_REAL_S), and the
    # all-gather's tail drops them again.
    h_loc = h[lo:min(hi, S)]
    rope_loc = rope_freqs[:, lo:min(hi, S)] if rope_freqs is not None else None
    if hi > S:
        h_loc = torch.cat([h_loc, h.new_zeros(hi - max(lo, S), h.shape[1])], dim=0)
        if rope_freqs is not None:
            tail = rope_freqs.new_zeros((rope_freqs.shape[0], hi - max(lo, S)) + tuple(rope_freqs.shape[2:]))
            rope_loc = torch.cat([rope_loc, tail], dim=1)
    h_loc = h_loc.contiguous()
    rope_loc = rope_loc.contiguous() if rope_loc is not None else None
    segs_loc = _shard_segments(mod_segments, lo, hi)
    host_block = _host_block_timed if _TIMING else None
    _timeline = _Timeline(h_loc.is_cuda) if _TIMING else None
    _SP_ACTIVE, _SP_REAL_S = True, S
    seg_row = None
    try:
        for blk in self.blocks:
            if _fusable(blk, h_loc):
                if seg_row is None:
                    seg_row = ops().segment_rows(segs_loc, h_loc.shape[0], h_loc.device)
                h_loc = _sp_block(blk, h_loc, t_emb, seg_row, rope_loc, transformer_options=transformer_options)
            elif host_block is not None:
                h_loc = host_block(blk, h_loc, t_emb, segs_loc, rope_loc, transformer_options=transformer_options)
            else:
                h_loc = blk(h_loc, t_emb, segs_loc, rope_loc, transformer_options=transformer_options)
        with _span("gather"):
            out = _gather_rows(h_loc) if WORLD > 1 else h_loc
    finally:
        _SP_ACTIVE, _SP_REAL_S = False, None
        timeline, _timeline = _timeline, None
    if timeline is not None:
        _last_totals.clear()
        _last_totals.update(timeline.totals())
    # A kernel that gave up a bounded wait leaves a code in the device status word and its output
    # rows unwritten: raise here rather than hand back such activations (one sync per call).
    check = getattr(ops(), "check_status", None)
    if check is not None and out.is_cuda:
        check(out.device)
    return out[:S] if S_pad > S else out


def install(module=None):
    """Patch the host model module (default: ComfyUI's comfy.ldm.minimax.model)."""
    global _orig_run_blocks, _orig_attn_forward, _orig_mlp_forward, _MODULE
    if module is None:
        import comfy.ldm.minimax.model as module
    if _MODULE is not None and _MODULE is not module:
        uninstall()
    _MODULE = module
    if _orig_run_blocks is None:
        _orig_run_blocks = module.MiniMaxH3Model.run_blocks
    if _orig_attn_forward is None:
        _orig_attn_forward = module.Attention.forward
    if _orig_mlp_forward is None and hasattr(module, "MLP"):
        _orig_mlp_forward = module.MLP.forward
    mode = os.environ.get("SP_OVERLAP", "0")
    overlap = mode == "1"
    module.Attention.forward = {"1": _sp_attn_forward_overlap, "heads": _sp_attn_forward_heads,
                                "peer": _sp_attn_forward_peer, "ce": _sp_attn_forward_ce}.get(mode, _sp_attn_forward)
    module.MiniMaxH3Model.run_blocks = _sp_run_blocks
    if _orig_mlp_forward is not None:
        module.MLP.forward = _sp_mlp_forward
    if RANK == 0:
        mode = f"overlap(P={_PIECES})" if overlap else {"heads": "overlap(heads)", "peer": "fused exchanges (peer)",
                                                         "ce": "copy-engine exchanges"}.get(mode, "blocking")
        print(f"[sp_runtime] installed (WORLD={WORLD}) - run_blocks + Ulysses attention patched [{mode}]"
              + (" [SP_TIMING]" if _TIMING else ""), flush=True)


def uninstall():
    """Restore the host module's original run_blocks / Attention.forward / MLP.forward."""
    global _orig_run_blocks, _orig_attn_forward, _orig_mlp_forward, _MODULE
    if _MODULE is not None:
        if _orig_run_blocks is not None:
            _MODULE.MiniMaxH3Model.run_blocks = _orig_run_blocks
        if _orig_attn_forward is not None:
            _MODULE.Attention.forward = _orig_attn_forward
        if _orig_mlp_forward is not None:
            _MODULE.MLP.forward = _orig_mlp_forward
    _orig_run_blocks = _orig_attn_forward = _orig_mlp_forward = _MODULE = None
