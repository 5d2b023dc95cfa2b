/* C ABI of the B200 (sm_100a) MiniMax-H3 Ulysses attention library, libh3attn.so.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer, every
 * size and stride is an int64 count of ELEMENTS (bf16 unless stated), and every call
 * takes the caller's CUDA stream as `void*` (a cudaStream_t; NULL = legacy default
 * stream). Calls are asynchronous: they validate arguments, enqueue kernels and return.
 * Nothing here allocates device memory; callers pass every buffer, including the
 * int32 device status word that bounded in-kernel waits report into.
 *
 * Return values: 0 on success, a negative H3_ERR_* on a rejected argument or a failed
 * launch. A kernel that gave up waiting (it never hangs the GPU) leaves a positive
 * H3_STATUS_* code in the status word; read it with h3_status_read(). The status word
 * must be zero before a launch; it is sticky (kernels only ever write non-zero codes).
 *
 * Threading: calls keep no global mutable state; distinct streams may call concurrently.
 * The one exception is h3_attn_layer_noalloc: every call shares one static device array, so
 * its calls must not overlap on the GPU (see its comment).
 */
#ifndef H3ATTN_H_
#define H3ATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3ATTN_VERSION 1

/* return codes */
#define H3_OK 0
#define H3_ERR_NULL (-1)        /* a required pointer is NULL */
#define H3_ERR_ALIGN (-2)       /* a pointer is not 16-byte aligned */
#define H3_ERR_SHAPE (-3)       /* a size is out of range */
#define H3_ERR_STRIDE (-4)      /* a stride is not a multiple of 8 elements / too small */
#define H3_ERR_LAUNCH (-5)      /* the CUDA runtime refused the launch */
#define H3_ERR_TENSOR_MAP (-6)  /* cuTensorMapEncodeTiled rejected the layout */
#define H3_ERR_DRIVER (-7)      /* driver entry point unavailable */
#define H3_ERR_UNSUPPORTED (-8) /* a configuration this build does not implement */
#define H3_ERR_CUDA (-9)        /* a CUDA runtime call failed (h3_status_read) */
#define H3_ERR_SCRATCH_LIMIT (-10)  /* h3_attn_layer_noalloc: the call needs more than its static scratch */
#define H3_ERR_DEVICE_TIMEOUT (-11) /* h3_attn_layer_noalloc: a kernel gave up waiting (bounded wait) */

/* device status codes (positive, written by kernels into the status word) */
#define H3_STATUS_OK 0
#define H3_STATUS_TIMEOUT_Q 1
#define H3_STATUS_TIMEOUT_KV 2
#define H3_STATUS_TIMEOUT_S 3
#define H3_STATUS_TIMEOUT_P 4
#define H3_STATUS_TIMEOUT_O 5
#define H3_STATUS_TIMEOUT_DRAIN 6
#define H3_STATUS_TIMEOUT_KAT 7

/* Library build version (H3ATTN_VERSION). */
int h3_version(void);

/* Exact non-causal attention, head_dim 128, bf16 in / fp32 accumulate / bf16 out:
 *   O[h, i, :] = softmax_j( Q[h, i, :] . K[h, j, :] * softmax_scale ) V[h, j, :],  j < s_kv
 * Replaces the SDPA FLASH call of the Ulysses runtime, harness/sp_runtime.py:119-121
 * (and the unwired fa3(q,k,v,o) binding, attn_sm80/fa3_sm80_h3.cu:584-593), including
 * the pad path of sp_runtime.py:106-109: queries run over s_q rows while keys and
 * values stop at the real length s_kv.
 *   q: [n_heads][s_q][128] with strides (q_head_stride, q_row_stride)
 *   k, v: [n_heads][s_kv][128] with strides (kv_head_stride, kv_row_stride)
 *   o: row i of head h is written at
 *        o + (i / o_rank_rows) * o_rank_stride + h * o_head_stride + (i % o_rank_rows) * o_row_stride
 *      so one launch can write [n_heads][s_q][128], token-major [s_q][n_heads][128], or the
 *      head->seq all-to-all send layout [world][n_heads][s_q/world][128] directly.
 * A query row's result depends only on that row, K and V: running any subset of
 * heads or of rows gives bit-identical rows. */
int h3_attn_fwd(const void* q, const void* k, const void* v, void* o, int64_t n_heads, int64_t s_q, int64_t s_kv,
                int64_t q_head_stride, int64_t q_row_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                int64_t o_rank_rows, int64_t o_rank_stride, int64_t o_head_stride, int64_t o_row_stride,
                float softmax_scale, int32_t* status, void* stream);

/* h3_attn_fwd with an explicit kernel schedule (a tuning hook; h3_attn_fwd uses the
 * default). All variants compute the same attention within the same tolerance; variants with
 * the same exp2 placement are bit-identical to each other (0, 1, 2, 3, 7 | 4, 8):
 *   0  one CTA per SM, exp2 on MUFU, P handed over after 3 of its 4 32-key chunks (the default)
 *   1  SM pairs: tcgen05 cta_group::2 MMAs over two CTAs on two SMs, each staging half of every
 *      K and V tile; otherwise as 0
 *   2  as 0 with P handed over after 2 of 4 chunks; 7 the same after all 4
 *   3  as 0 with the two softmax warpgroups taking turns for their exponentials
 *   4  as 0 with every other key pair of 32-key chunks 1-2 on the FMA pipe (a degree-3
 *      polynomial exp2); 5 key pairs 0, 4, 8, 12 of chunks 0-2; 6 key pairs 2, 6, 10, 14 of
 *      chunks 1-2
 *   8  as 1 with the exp2 placement of 4
 * Returns H3_ERR_UNSUPPORTED for any other value. */
int h3_attn_fwd_variant(const void* q, const void* k, const void* v, void* o, int64_t n_heads, int64_t s_q,
                        int64_t s_kv, int64_t q_head_stride, int64_t q_row_stride, int64_t kv_head_stride,
                        int64_t kv_row_stride, int64_t o_rank_rows, int64_t o_rank_stride, int64_t o_head_stride,
                        int64_t o_row_stride, float softmax_scale, int32_t* status, int32_t variant, void* stream);

/* Phase profiler (diagnostics; cf. the clock64 phase counters of the reference kernel,
 * attn_sm80/fa3_sm80_h3.cu:96-105, :572-582): runs any variant above and records clock64()
 * stamps of CTA (0, 0) for the first trace_iters KV iterations into the device buffer
 *   trace[((role * trace_iters) + j) * 8 + point]   (int64, 3 * trace_iters * 8 entries)
 * role 0/1 = softmax warpgroup of Q tile 0/1: points 0 before the S wait, 1 S ready,
 *   2 S in registers (second half's load done), 3 row max and any rescale done, 4 first P chunks
 *   handed over, 5 all of P handed over;
 * role 2 = MMA thread: 0 iteration start, 1 V ready, 2 first P chunks of tile 0 ready, 3 all of
 *   P_0 ready, 4 next S_0 issued, 5-7 the same for tile 1. */
int h3_attn_fwd_profile(const void* q, const void* k, const void* v, void* o, int64_t n_heads, int64_t s_q,
                        int64_t s_kv, int64_t q_head_stride, int64_t q_row_stride, int64_t kv_head_stride,
                        int64_t kv_row_stride, int64_t o_rank_rows, int64_t o_rank_stride, int64_t o_head_stride,
                        int64_t o_row_stride, float softmax_scale, int32_t* status, int32_t variant,
                        long long* trace, int64_t trace_iters, void* stream);

/* Fused per-head qk-RMSNorm + RoPE + seq->head send-buffer pack for one token shard.
 * Replaces comfy_kitchen's in-place rms_rope_split_half_ call (harness/sp_runtime.py:93-99,
 * or q_norm/k_norm when rope is absent, :100-101), the head transposes (:102) and the
 * send-side reshape copy of a2a_seq_to_head (:69).
 *   q, k, v: [s_l][n_heads*128] rows with row stride in_row_stride (views of the fused QKV
 *            projection output are fine)
 *   rope: fp32 [s_l][64][2][2] rotation matrices, token row stride rope_row_stride
 *         (elements); pair i rotates (x[i], x[i+64]):
 *           out[i] = m00*x[i] + m01*x[i+64],  out[i+64] = m10*x[i] + m11*x[i+64]
 *         NULL = no rotary embedding (plain RMSNorm)
 *   q_weight, k_weight: bf16 [128] RMSNorm weights, NULL = unit weight
 *   y = x * (1 / sqrt(mean(x^2) + eps)) * w, computed in fp32, rounded once to bf16.
 *   outputs: head h, token j of q (k, v) lands at
 *     out + (h / heads_per_rank) * out_rank_stride + (h % heads_per_rank) * out_head_stride + j * 128
 *   v is copied unchanged. */
int h3_qknorm_rope_pack(const void* q, const void* k, const void* v, int64_t in_row_stride, const float* rope,
                        int64_t rope_row_stride, const void* q_weight, const void* k_weight, float eps, void* q_out,
                        void* k_out, void* v_out, int64_t s_l, int64_t n_heads, int64_t heads_per_rank,
                        int64_t out_rank_stride, int64_t out_head_stride, void* stream);

/* Receive-side reorder of the seq->head all-to-all: the permute copy of
 * harness/sp_runtime.py:71. recv holds, for each source rank r, n_tensors tensors of
 * [heads_per_rank][s_l][128]:
 *   recv + r * recv_rank_stride + t * recv_tensor_stride + h * s_l*128 + j*128
 * and tensor t lands as [heads_per_rank][world*s_l][128] at out + t * out_tensor_stride. */
int h3_seq_to_head_unpack(const void* recv, void* out, int64_t world, int64_t heads_per_rank, int64_t s_l,
                          int64_t n_tensors, int64_t recv_rank_stride, int64_t recv_tensor_stride,
                          int64_t out_tensor_stride, void* stream);

/* Head-major [n_heads][s_l][128] -> token-major [s_l][n_heads*128]: the
 * transpose(1, 2).reshape(s, H*D) copy ahead of out_proj (harness/sp_runtime.py:125)
 * applied to the head->seq all-to-all receive buffer (:76-77). */
int h3_head_to_seq_unpack(const void* recv, void* out, int64_t n_heads, int64_t s_l, void* stream);

/* The two all-to-alls of the Ulysses layer fused into the kernels that produce their data, over
 * NVLink peer memory (replacing a2a_seq_to_head + its receive permute, harness/sp_runtime.py:67-71,
 * and a2a_head_to_seq + the head->seq transpose, :73-77 and :125). rank_base / o_peer are DEVICE
 * arrays of n_ranks addresses, one per destination rank, each mapped into this process (e.g. symmetric
 * memory); the caller orders the writes of all ranks before any read with a stream-ordered barrier.
 * A table too short for the call (n_heads / heads_per_rank > n_ranks for the pack, s_q > n_ranks *
 * o_rank_rows for the attention) is rejected with H3_ERR_SHAPE before anything is enqueued.
 *
 * h3_qknorm_rope_pack_peer: as h3_qknorm_rope_pack, but head g of token t goes to rank
 *   r = g / heads_per_rank at rank_base[r] + tensor*tensor_stride + (g % heads_per_rank)*head_stride
 *   + (row_offset + t)*128 (elements): each rank's attention input [3][H/W][S][128] is written by all
 *   ranks directly, no send buffer, exchange or unpack.
 * h3_attn_fwd_peer: as h3_attn_fwd (default schedule), but query row i goes to rank
 *   r = i / o_rank_rows at o_peer[r] + head*o_head_stride + (i % o_rank_rows)*o_row_stride, e.g. the
 *   destination's token-major out_proj input [S/W][H*128] at this rank's column block. o_local is
 *   this rank's own output buffer (argument checks only). Both kernels end with a system-scope
 *   fence so their peer stores are visible to the barrier that follows. */
int h3_qknorm_rope_pack_peer(const void* q, const void* k, const void* v, int64_t in_row_stride, const float* rope,
                             int64_t rope_row_stride, const void* q_weight, const void* k_weight, float eps,
                             const uint64_t* rank_base, int64_t n_ranks, int64_t tensor_stride, int64_t head_stride,
                             int64_t row_offset, int64_t s_l, int64_t n_heads, int64_t heads_per_rank, void* stream);
int h3_attn_fwd_peer(const void* q, const void* k, const void* v, void* o_local, const uint64_t* o_peer,
                     int64_t n_ranks, int64_t n_heads, int64_t s_q, int64_t s_kv, int64_t q_head_stride,
                     int64_t q_row_stride, int64_t kv_head_stride, int64_t kv_row_stride, int64_t o_rank_rows,
                     int64_t o_head_stride, int64_t o_row_stride, float softmax_scale, int32_t* status, void* stream);

/* Row-independent projection GEMM, bf16 in, fp32 accumulate, bf16 out:
 *   epilogue 0: c[m][n] = sum_k a[m][k] * w[n][k]                  (w has n_out rows)
 *   epilogue 1: c[m][n] = silu(a . w[n]) * (a . w[n_out + n])       (w = [gate; up], 2*n_out rows;
 *               both products and silu rounded to bf16 as the host model's fc1 -> chunk -> silu -> mul)
 * Replaces the projection linears around the attention op: qkv_proj (harness/sp_runtime.py:91) and
 * out_proj (:126), and the FFN's fc1 and swiglu-into-fc2 linears (harness/sp_blockloop.py:169-170).
 * w is an nn.Linear weight [out][in] (row stride w_row_stride). a is read as [a_chunks][m][a_chunk_cols]
 * (element strides a_chunk_stride, a_row_stride) and multiplied as the row-major [m][a_chunks*a_chunk_cols]
 * matrix: a_chunks = 1 is a plain row-major a; a_chunks = H, a_chunk_cols = 128 reads the head->seq
 * receive buffer [H][s_l][128] in place (no unpack pass). Each output row is computed by one tile with
 * one fixed reduction order, so the bits of a row do not depend on m or on the row's position: token
 * shards on W ranks reproduce the 1-GPU result exactly. Requires 16-byte aligned pointers, strides and
 * a_chunk_cols multiples of 8, a_chunk_cols a multiple of 64 when a_chunks > 1, n_out a multiple of 8
 * (of 128 for epilogue 1). Allocates nothing. */
int h3_gemm_bf16(const void* a, int64_t m, int64_t a_chunks, int64_t a_chunk_cols, int64_t a_chunk_stride,
                 int64_t a_row_stride, const void* w, int64_t n_out, int64_t w_row_stride, void* c,
                 int64_t c_row_stride, int32_t epilogue, int32_t* status, void* stream);

/* AdaLN modulation of the DiT block (the host model's norm + _mod_scale_shift, harness/sp_runtime.py:
 * 209-210 and :214-215), optionally after its gated residual (_mod_gate, :212-213), in one pass:
 *   xr = x + gate[seg] * y   (when y != NULL and the token is in a segment; else xr = x), stored to
 *        x_out when x_out != NULL
 *   h  = LN(xr) * (1 + scale[seg]) + shift[seg]   (LN(xr) alone for tokens outside every segment)
 * LN is the affine-free LayerNorm (biased variance, eps), computed in fp32; every torch op of the
 * host path rounds to bf16 and so does this kernel, in the same order. seg_row[token] is the
 * modulation row of the token's segment or -1; gate / shift / scale are [rows][hidden] bf16 with
 * row stride mod_row_stride. hidden <= 8192, a multiple of 8. */
int h3_norm_modulate(const void* x, int64_t x_row_stride, const void* y, int64_t y_row_stride, const void* gate,
                     void* x_out, int64_t x_out_row_stride, const void* shift, const void* scale,
                     int64_t mod_row_stride, const int32_t* seg_row, void* h, int64_t h_row_stride, int64_t rows,
                     int64_t hidden, float eps, void* stream);
/* The block's closing gated residual (_mod_gate after the FFN, harness/sp_runtime.py:217-218):
 * out = x + gate[seg] * y on segment tokens, x elsewhere (bf16 roundings as the host ops). */
int h3_gated_residual(const void* x, int64_t x_row_stride, const void* y, int64_t y_row_stride, const void* gate,
                      int64_t gate_row_stride, const int32_t* seg_row, void* out, int64_t out_row_stride,
                      int64_t rows, int64_t hidden, void* stream);

/* Tile known-answer tests of the tcgen05 path (cf. attn_sm80/microtest.py:10-26):
 *   h3_tile_kat_qk: s_out[128][128] fp32 = q[128][128] . k[128][128]^T
 *   h3_tile_kat_pv: o_out[128][128] fp32 = p[128][128] . v[128][128]  (p written to TMEM
 *                   exactly as the softmax warps write P) */
int h3_tile_kat_qk(const void* q, const void* k, float* s_out, int32_t* status, void* stream);
int h3_tile_kat_pv(const void* p, const void* v, float* o_out, int32_t* status, void* stream);
/* Bounded-wait known-answer test (the failure path of every kernel here, on purpose): one CTA
 * starts a TMA load of tile[128][128] bf16, then waits up to limit_ns nanoseconds (1 us .. 10 s)
 * on an mbarrier that nothing ever completes. When the limit passes it writes
 * H3_STATUS_TIMEOUT_KAT into *status, drains its copy, frees its tensor memory and returns,
 * leaving the device usable; h3_status_read() then returns H3_STATUS_TIMEOUT_KAT. */
int h3_wait_kat(const void* tile, int64_t limit_ns, int32_t* status, void* stream);
/* The same through an SM pair (tcgen05.mma.cta_group::2, M = 256, two-CTA cluster):
 *   h3_tile_kat_pair_qk: s_out[256][128] = q[256][128] . k[128][128]^T (CTA r: q rows 128r.., keys 64r..)
 *   h3_tile_kat_pair_pv: o_out[256][128] = p[256][128] . v[128][128]   (CTA r: p rows 128r.., v cols 64r..) */
int h3_tile_kat_pair_qk(const void* q, const void* k, float* s_out, int32_t* status, void* stream);
int h3_tile_kat_pair_pv(const void* p, const void* v, float* o_out, int32_t* status, void* stream);

/* No counterpart in the reference. The single-GPU attention layer -- h3_qknorm_rope_pack into
 * head-major q/k/v, then h3_attn_fwd into token-major o -- for callers that cannot allocate device
 * memory themselves (e.g. C or FFI code inside an application whose caching allocator owns all device
 * memory). The caller passes only inputs and outputs: qkv [s][3*n_heads*128] bf16 (q, k, v column
 * blocks, row stride qkv_row_stride), rope fp32 [s][64][2][2] or NULL, bf16 weights or NULL,
 * o [s][n_heads*128] bf16. The packed intermediate and the status word live in a static device array
 * of 64 MiB + 256 B that every GPU loading the library keeps until exit; calls needing more
 * (3*s*n_heads*128*2 bytes > 64 MiB, i.e. s*n_heads > 87381) return H3_ERR_SCRATCH_LIMIT. The first
 * call on a device looks up the array's device address (make it before any stream capture on that
 * device). All calls share the array, so calls that overlap on the GPU race. The call waits for
 * `stream` to drain and returns H3_ERR_DEVICE_TIMEOUT if a kernel reported a bounded-wait timeout. */
int h3_attn_layer_noalloc(const void* qkv, int64_t qkv_row_stride, const float* rope, int64_t rope_row_stride,
                          const void* q_weight, const void* k_weight, float eps, void* o, int64_t s, int64_t n_heads,
                          float softmax_scale, void* stream);

/* Synchronise `stream`, then return the status word's value (>= 0), or H3_ERR_CUDA. */
int h3_status_read(const int32_t* status, void* stream);

/* Copy-engine exchange step: `rows` rows of `width` bytes from src (row pitch src_pitch bytes) to
 * dst (row pitch dst_pitch bytes), ordered on `stream`; either side may be a peer GPU's memory
 * mapped into this process (CUDA IPC, cuMem or torch symmetric memory). One call moves one rank's
 * chunk of an all-to-all straight into the destination's final layout (the attention input
 * [3][H/W][S][128] at this rank's rows, or the out_proj input [H][S/W][128] at this rank's heads),
 * the transfer the NCCL all-to-all plus unpack of harness/sp_runtime.py:67-77 performs. No kernel
 * runs: the GPU's copy engines move the bytes. */
int h3_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width, int64_t rows,
               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* H3ATTN_H_ */
