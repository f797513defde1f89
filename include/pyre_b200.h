/*
 * pyre_b200.h — C ABI of the B200 (sm_100a) tensor-parallel forward hot path.
 *
 * Every entry point:
 *   - takes plain device pointers and sizes (no framework types),
 *   - is asynchronous on the caller-supplied stream (a cudaStream_t passed as void*;
 *     NULL means the legacy default stream),
 *   - returns an int status: PYRE_OK (0) or one of the PYRE_E* codes below. The message
 *     of the last failure on the calling thread is available through pyre_last_error().
 *
 * The caller owns every buffer it passes in. The library never frees caller memory;
 * pyre_comm_t owns only what pyre_comm_create() allocates (peer table, status word).
 *
 * Q8_0 format. The reference quantizes a weight stored as [K, N] row-major float
 * (K = input dim, N = output dim) in flattened C order in 32-element blocks
 * (src/orchestrator/quantizer.py:11-26, src/orchestrator/llama_loader.py:1132-1134), so
 * every block runs along N: q int8 [K, N], scale [K, N/32], scale[k, j/32] for q[k, j].
 *
 * Packed device weight layout (used by the FFN entry points). A group of M matrices that
 * share [K, N] (M = 2: gate and up; M = 1: one matrix) is stored as contiguous blocks, one
 * per (slab of 256 output columns j, unit of R = 64 / M input rows u), in (j, u) order:
 *   [q of matrix 0: R x 256 int8] ... [q of matrix M-1] [scales of matrix 0: R x 8] ...
 * with K padded to a multiple of R and N to a multiple of 256 by zeros. The int8 values and
 * scales are exactly the reference's blocks; a block (~17 KB) is one pipeline stage that the
 * kernels move with a single bulk copy. pyre_q80_pack() builds it from the plain form.
 */
#ifndef PYRE_B200_H
#define PYRE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define PYRE_API __attribute__((visibility("default")))
#else
#define PYRE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define PYRE_OK        0
#define PYRE_EINVAL    1  /* bad argument: null pointer, size, alignment, dtype        */
#define PYRE_ECUDA     2  /* a CUDA runtime/driver call failed                          */
#define PYRE_ETIMEOUT  3  /* a bounded device-side wait on a peer ran out               */
#define PYRE_ENOMEM    4  /* caller-supplied workspace too small / allocation failed    */
#define PYRE_ERANGE    5  /* device status: an FFN partial sum was not finite or >= 2^30 */

/* ---- element types ----------------------------------------------------------------- */
#define PYRE_F32   0
#define PYRE_BF16  1
#define PYRE_F16   2

typedef struct pyre_comm pyre_comm_t;

/* Library version (major*10000 + minor*100 + patch). */
PYRE_API int pyre_version(void);

/* Copies the last error message of the calling thread into buf (NUL-terminated,
 * truncated to len). Returns the length of the full message. */
PYRE_API int pyre_last_error(char* buf, int len);

/* One call of a captured op, end to end (the compiled model's execute(), root_node.py:574-580):
 * copies in_bytes from host src into the pinned staging buffer stage_in that the graph's
 * first node copies to the device, launches the instantiated CUDA graph exec
 * (cudaGraphExec_t) on stream, and waits for it; the graph's last node has written the
 * result to its pinned output buffer. in_bytes may be 0 (input already staged). */
PYRE_API int pyre_graph_run(void* exec, void* stream, const void* src, void* stage_in, int64_t in_bytes);

/* ---- Q8_0 format ------------------------------------------------------------------
 * pyre_q80_quantize replaces quantize_q80 (src/orchestrator/quantizer.py:11-26):
 *   flatten -> zero-pad to a multiple of 32 -> per block absmax (0 -> 1.0) ->
 *   scale = f32(absmax / 127) -> q = clip(round_half_even(x / scale), -128, 127).
 * Bit-exact with the reference for finite inputs. src is f32 or bf16 (src_dtype).
 * q receives ceil(n/32)*32 bytes; scale_f32 and scale_f16 receive ceil(n/32)
 * entries each; either scale pointer may be NULL (not both). scale_f16 holds
 * f16(scale_f32), round-to-nearest-even. */
PYRE_API int pyre_q80_quantize(const void* src, int src_dtype, int64_t n,
                      int8_t* q, float* scale_f32, uint16_t* scale_f16, void* stream);

/* pyre_q80_dequantize replaces dequantize_q80 (src/orchestrator/quantizer.py:29-40)
 * and pyre_kernels.q80_dequantize (src/kernels/mojo/pyre_kernels.mojo:172-185):
 * out[i] = f32(q[i]) * scale[i/32], for i < n. scale_dtype is PYRE_F32 or PYRE_F16. */
PYRE_API int pyre_q80_dequantize(const int8_t* q, const void* scale, int scale_dtype, int64_t n,
                        float* out, void* stream);

/* Bytes of the packed layout of M (1 or 2) [K, N] matrices with scales of scale_dtype. */
PYRE_API int pyre_q80_packed_bytes(int M, int K, int N, int scale_dtype, int64_t* bytes);

/* Plain -> packed: q0/q1 int8 [K, N] row-major (16-byte aligned), s0/s1 scales [K, N/32]
 * (the reference's flat Q8_0 tuple of a stored [in, out] weight, reshaped); M == 2 packs
 * q0/s0 (gate) with q1/s1 (up) block by block. out: pyre_q80_packed_bytes() bytes. */
PYRE_API int pyre_q80_pack(int M, const int8_t* q0, const void* s0, const int8_t* q1, const void* s1,
                  int K, int N, int scale_dtype, void* out, void* stream);

/* ---- gated-SiLU FFN shard ---------------------------------------------------------
 * The shard [ffn_start, ffn_end) of width W of the intermediate dim, as built by
 * build_ffn_graph (src/ffn/builder.py:20-53) and run by the root's decode FFN
 * (src/orchestrator/root_node.py:956-980).
 *
 * Bytes of scratch the FFN calls below need for T tokens, hidden H, width W (256-byte
 * aligned, zero-initialised once by the caller). */
PYRE_API int pyre_ffn_workspace_bytes(int T, int H, int W, int64_t* bytes);

/* h[T, W] = silu(x @ Wg) * (x @ Wu)      (gated,   src/ffn/builder.py:37-43)
 * h[T, W] = silu(x @ Wu)                 (ungated, src/ffn/builder.py:47-49; gated == 0)
 * x: [T, H] of x_dtype (PYRE_F32 or PYRE_BF16), 16-byte aligned rows. wgu: gate and up
 * [H, W] packed together (M = 2), or up alone (M = 1) when gated == 0, scales of
 * scale_dtype. h: [T, W] of h_dtype (PYRE_F32 or PYRE_BF16; also PYRE_F16 for
 * T > PYRE_FUSED_REDUCE_MAX_T, where the tensor-core GEMM takes f16 operands and flags
 * PYRE_ERANGE in the workspace status word for values beyond f16). silu(g) = g / (1 + exp(-g))
 * as in pyre_kernels.silu_mul (src/kernels/mojo/pyre_kernels.mojo:121-129).
 * workspace: zero-initialised device memory of at least pyre_ffn_workspace_bytes();
 * it is left zeroed where it must start at zero, so it can be reused call after call on
 * one stream (calls that overlap on the GPU need separate workspaces). */
PYRE_API int pyre_ffn_gateup_silu_q80(const void* x, int x_dtype, int T, int H,
                             const void* wgu, int gated, int scale_dtype, int W,
                             void* h, int h_dtype, void* workspace, int64_t ws_bytes,
                             void* stream);

/* The whole shard FFN for T <= PYRE_FUSED_REDUCE_MAX_T tokens in one persistent launch:
 *   out[T, H] = (silu(x @ Wg) * (x @ Wu)) @ Wd          (src/ffn/builder.py:37-45, the
 *   root's decode FFN src/orchestrator/root_node.py:956-980; gated == 0: silu(x @ Wu) @ Wd)
 * and, with comm != NULL, the sum over the ranks of comm in rank order
 * (src/orchestrator/root_node.py:982-995), reduced in the down-projection epilogue through
 * NVLink peer stores. The gate/up product h lives in the workspace; the down projection of
 * rows k..k+31 of h starts as soon as the gate/up slab holding them is finished.
 * x: [T, H] (PYRE_F32 or PYRE_BF16, 16-byte aligned rows); wgu: gate/up [H, W] packed as a
 * pair (or up alone), wd: down [W, H] packed; H and W multiples of 32; out: f32 [T, H]. */
PYRE_API int pyre_ffn_decode_q80(const void* x, int x_dtype, int T, int H,
                                 const void* wgu, int gated, const void* wd, int scale_dtype, int W,
                                 float* out, void* workspace, int64_t ws_bytes,
                                 pyre_comm_t* comm, void* stream);

/* No counterpart in the reference: this library's own entry point for callers that cannot
 * allocate device memory (a host program that binds only this C ABI with no CUDA allocator
 * of its own, or a runtime whose device memory all belongs to its own pool, where a
 * cudaMalloc fails or synchronises the device mid-serving).
 * Same computation, inputs and outputs as pyre_ffn_decode_q80 on one GPU (no communicator),
 * but the scratch is a static device array of PYRE_NOALLOC_SCRATCH_BYTES inside the library,
 * so the call allocates nothing. Limits and rules:
 *   - sizes whose workspace (pyre_ffn_workspace_bytes) exceeds PYRE_NOALLOC_SCRATCH_BYTES are
 *     rejected with PYRE_EINVAL;
 *   - every GPU that loads the library holds the array until the process exits;
 *   - the first call on a device looks up the array's address on that device (with that
 *     device current); make it before any stream capture;
 *   - calls on one device share the array: each call clears it on its stream first (after
 *     its argument checks pass; a rejected call queues nothing), and calls that overlap on
 *     the GPU race (serialise them on one stream);
 *   - the kernel's status word is not cleared by the calls: it keeps the first problem since
 *     it was last read (PYRE_ERANGE: a partial sum was not finite or too large and that
 *     call's out is wrong; PYRE_ETIMEOUT: a bounded wait ran out, and calls return incomplete
 *     output until the word is read). Read it with pyre_ffn_decode_q80_noalloc_status. */
#define PYRE_NOALLOC_SCRATCH_BYTES (4 << 20)
PYRE_API int pyre_ffn_decode_q80_noalloc(const void* x, int x_dtype, int T, int H,
                                         const void* wgu, int gated, const void* wd, int scale_dtype,
                                         int W, float* out, void* stream);
/* No counterpart in the reference. Synchronises stream, then returns in *status the status
 * word of pyre_ffn_decode_q80_noalloc's static scratch on the current device (PYRE_OK,
 * PYRE_ERANGE or PYRE_ETIMEOUT, the first since the last read) and clears it. */
PYRE_API int pyre_ffn_decode_q80_noalloc_status(int* status, void* stream);

/* out[T, H] = h @ Wd   (src/ffn/builder.py:44), and with comm != NULL also the sum of
 * that partial over every rank of comm (src/orchestrator/root_node.py:582-594 and
 * :982-995, `ffn_out += partial`), in rank order 0..world-1 on every rank. For
 * T <= PYRE_FUSED_REDUCE_MAX_T the reduction happens in the GEMV epilogue through
 * NVLink peer stores and bounded flag waits; above it a two-shot peer-memory
 * all-reduce follows the GEMM. h: [T, W] of h_dtype; wd: [W, H] packed (M = 1); out: f32 [T, H]. */
#define PYRE_FUSED_REDUCE_MAX_T 4
PYRE_API int pyre_ffn_down_q80(const void* h, int h_dtype, int T, int W,
                      const void* wd, int scale_dtype, int H,
                      float* out, void* workspace, int64_t ws_bytes,
                      pyre_comm_t* comm, void* stream);

/* ---- peer-memory communicator (one process per GPU, NVLink / NVSwitch) ------------
 * Replaces the reference's TCP gather of FFN partials (src/orchestrator/net.py:18-48
 * used at src/orchestrator/root_node.py:582-594) inside one box.
 *
 * Bytes of the symmetric receive buffer each rank allocates for world ranks, up to
 * max_tokens tokens of a hidden-wide f32 row. */
PYRE_API int pyre_comm_buffer_bytes(int world, int max_tokens, int hidden, int64_t* bytes);
/* cudaMalloc + zero a receive buffer and export its IPC handle (64 bytes). */
PYRE_API int pyre_comm_alloc(int64_t bytes, void** dev_ptr, void* ipc_handle_out);
PYRE_API int pyre_comm_free(void* dev_ptr);
/* Map a peer's exported buffer into this process (cudaIpcOpenMemHandle). */
PYRE_API int pyre_comm_open_peer(const void* ipc_handle, void** peer_ptr);
PYRE_API int pyre_comm_close_peer(void* peer_ptr);
/* bufs[r] is rank r's receive buffer as seen from this process (bufs[rank] is the
 * local one). All ranks must pass the same world, max_tokens and hidden. */
PYRE_API int pyre_comm_create(int rank, int world, void* const* bufs, int max_tokens, int hidden,
                     pyre_comm_t** out);
PYRE_API int pyre_comm_destroy(pyre_comm_t* comm);
/* Limit of every device-side wait on a peer flag, in nanoseconds (default 2 s). */
PYRE_API int pyre_comm_set_timeout_ns(pyre_comm_t* comm, uint64_t ns);
/* Synchronises stream, then reads and clears the device status word of comm:
 * *status = PYRE_OK, or PYRE_ETIMEOUT if some wait since the last check ran out. */
PYRE_API int pyre_comm_check(pyre_comm_t* comm, int* status, void* stream);
/* Recovery after a wait ran out (no counterpart in the reference, whose TCP receive just
 * blocks): synchronises stream, then zeroes this rank's flag words, collective epoch, arrival
 * counter and status word. Every rank calls it, between host-side barriers and with none of
 * its collectives in flight; the ranks then start again from a common state. */
PYRE_API int pyre_comm_reset(pyre_comm_t* comm, void* stream);
/* In-place sum over ranks of a f32 buffer of n elements (two-shot: reduce-scatter then
 * all-gather through peer memory), rank order 0..world-1. n <= max_tokens * hidden. */
PYRE_API int pyre_allreduce_sum_f32(pyre_comm_t* comm, float* buf, int64_t n, void* stream);
/* Greedy token over a vocabulary split across the ranks of comm (Generator._sample at
 * temperature < 0.01, src/orchestrator/generator.py:51-53, np.argmax over the whole logit row):
 * key[T] is this rank's best (value, index) key per row from pyre_lm_head_argmax on its rows of
 * the table; every rank gets token[t] = the index of the largest key over the ranks (equal
 * values: the lower index) and, when key_out is not NULL, that key. T <= 4. */
PYRE_API int pyre_argmax_combine(pyre_comm_t* comm, const long long* key, int T, int* token, long long* key_out,
                                 void* stream);

/* ---- attention path ------------------------------------------------------------------
 * out[T, N] (f32) = x[T, K] @ W, W a packed single Q8_0 matrix [K, N] (pyre_q80_pack with
 * M = 1): the Q, K, V and O projections of src/attention/builder.py:56-58 (x @ Wq ...) and
 * root_node.py:866-897 (matmul_f32 of the normed token with the projection weights), on the
 * Q8_0 weights a reference worker holds. x: f32 or bf16 (f16 too for T > 4). workspace:
 * zero-initialised, pyre_ffn_workspace_bytes(T, K, N) bytes. */
PYRE_API int pyre_q80_linear(const void* x, int x_dtype, int T, int K, const void* w, int scale_dtype, int N,
                             float* out, void* workspace, int64_t ws_bytes, void* stream);
/* The same with an f32 bias [N] added to every output row (bias may be NULL): the Q/K/V
 * projections with q_bias / k_bias / v_bias that the reference adds right after x @ W, before
 * RoPE (src/orchestrator/root_node.py:443-451 prefill, :786-799 decode; Qwen2-style models). The
 * bias joins the finished f32 dot product in the kernel's epilogue. */
PYRE_API int pyre_q80_linear_bias(const void* x, int x_dtype, int T, int K, const void* w, int scale_dtype, int N,
                                  const float* bias, float* out, void* workspace, int64_t ws_bytes, void* stream);

/* out[r, :] = f32(x[r, :] * rstd_r * w) with rstd_r = 1 / sqrt(mean(x[r, :]^2) + eps), the sum
 * of squares in f64 (pyre_kernels.mojo:18-35; the reference uses eps = 1e-6). x, out: f32
 * [rows, H]; w: f32 [H]. */
PYRE_API int pyre_rms_norm(const float* x, int rows, int H, const float* w, double eps, float* out, void* stream);

/* h = x + delta (f32, the residual adds h = x + attn_out and out = h + ffn_out of
 * src/orchestrator/root_node.py:947, :997), then norm = rms_norm(h, w) exactly as
 * pyre_rms_norm (the next RMSNorm, root_node.py:951 / :752): one launch for the glue between
 * the attention, the FFN and the next layer. h may alias x. w and norm both null: add only.
 * x, delta, h, norm: f32 [rows, H]; w: f32 [H]. */
PYRE_API int pyre_add_rms_norm(const float* x, const float* delta, int rows, int H, const float* w, double eps,
                               float* h, float* norm, void* stream);

/* Softmax over the last axis of an f32 [rows, cols] matrix, max initialised to -1e10 and
 * exp(x - max) * (1 / sum) (pyre_kernels.mojo:39-58). */
PYRE_API int pyre_softmax_rows(const float* x, int64_t rows, int cols, float* out, void* stream);

/* Host function: the RoPE table of pyre_kernels.mojo:86-89 for positions 0..n_pos-1, as f32
 * [n_pos, dims/2, 2] (cos, sin) with dims = int(hd * rope_fraction), freq_i =
 * 1 / theta^(2i/dims) and the angle pos * freq_i in f64 (C library pow / cos / sin), cast to
 * f32. host_out holds n_pos * (dims/2) * 2 floats; the caller copies it to the device. */
PYRE_API int pyre_rope_table(double theta, double rope_fraction, int hd, int n_pos, float* host_out);

/* RoPE + clip + KV-cache append for T new tokens at positions start_pos..start_pos+T-1
 * (pyre_kernels.mojo:62-96 apply_rope, root_node.py:283-290 and :905-929): q [T, nq, hd] and
 * k, v [T, nkv, hd] f32 with row strides q_stride / kv_stride elements (one fused QKV
 * projection output can be passed as three offset pointers). q and k are rotated over the
 * first int(hd * rope_fraction) dims with the device copy of pyre_rope_table (covering the
 * positions used), q, k and v clipped to +-1000; q_out f16 [nq, T, hd]; k, v appended to the
 * f16 caches [nkv, max_t, hd]. */
PYRE_API int pyre_rope_kv_append(const float* q, const float* k, const float* v, int64_t q_stride,
                                 int64_t kv_stride, int T, int nq, int nkv, int hd, int start_pos,
                                 const float* rope_table, double rope_fraction, uint16_t* q_out, uint16_t* k_cache,
                                 uint16_t* v_cache, int max_t, void* stream);

/* Causal prefill attention over positions 0..T-1 of the caches (root_node.py:292-307:
 * GQA q head h -> kv head h / (nq / nkv), q k^T / sqrt(hd), -inf above the diagonal, softmax,
 * probs @ v), f16 operands on the tcgen05 tensor cores, f32 accumulation. q: f16 [nq, T, hd]
 * (pyre_rope_kv_append); out: f32 [T, nq * hd]. hd: 64 or 128. */
PYRE_API int pyre_attn_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int T, int nq,
                               int nkv, int hd, int max_t, float* out, void* stream);

/* Device status of the prefill attention kernels on the current device (PYRE_OK, or
 * PYRE_ETIMEOUT if a bounded pipeline wait ran out; that launch's output is incomplete).
 * Synchronous: waits for the device, returns the word and clears it. No counterpart in the
 * reference (its attention is host numpy). */
PYRE_API int pyre_attn_status(int* status);

/* Decode attention of one query token over cache positions 0..t-1 (root_node.py:1009-1031):
 * positions in [mask_lo, mask_hi) are masked (the reference's padded prefill). q: f16
 * [nq, hd]; out: f32 [nq * hd]. Split over the cache (flash-decoding), chunks combined in
 * order (deterministic). workspace: zero-initialised once, pyre_attn_decode_workspace_bytes
 * bytes, reused call after call on one stream. nq / nkv <= 8, hd 64 or 128. */
PYRE_API int pyre_attn_decode_workspace_bytes(int nq, int nkv, int hd, int t, int64_t* bytes);
PYRE_API int pyre_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int t, int nq,
                              int nkv, int hd, int max_t, int mask_lo, int mask_hi, float* out, void* workspace,
                              int64_t ws_bytes, void* stream);

/* One decode step of the attention block in one launch (root_node.py:900-933 then
 * :1009-1031): RoPE of the token's q and k at position start_pos (the cache length before
 * the step; table from pyre_rope_table), clip +-1000, append of k and v at row start_pos,
 * then decode attention over positions 0..start_pos as pyre_attn_decode. q: f32 [nq * hd];
 * k, v: f32 [nkv * hd]; same workspace as pyre_attn_decode. */
PYRE_API int pyre_attn_decode_step(const float* q, const float* k, const float* v, int start_pos,
                                   const float* rope_table, double rope_fraction, int nq, int nkv, int hd,
                                   uint16_t* k_cache, uint16_t* v_cache, int max_t, int mask_lo, int mask_hi,
                                   float* out, void* workspace, int64_t ws_bytes, void* stream);

/* ---- last decode step: final norm, lm_head, greedy token ------------------------------
 * Replaces Generator._rms_norm / _compute_logits / _sample at temperature < 0.01
 * (src/orchestrator/generator.py:40-53): rows of h f32 [T, H] (T <= 4) are normalised
 * (f64 mean of squares, x / sqrt(var + eps) in f64, times norm_w f32 [H]; norm_w NULL: no
 * norm), logits = h_norm . lm_head^T with the f16 table lm_head [V, H] (f32 accumulation),
 * token[t] = index of the largest logit of row t (the first among equal maxima, like
 * np.argmax). Rows of lm_head are the global vocabulary indices v0 .. v0 + V - 1 (a
 * vocab-sharded table: one shard per rank). logits f32 [T, V] and key [T] may be NULL; key
 * gets an int64 that orders (value, lower index) like the argmax, so the shards' keys combine
 * with a signed max reduction (index = 0xFFFFFFFF - (low 32 bits)). workspace:
 * pyre_lm_head_workspace_bytes, zeroed once, reused call after call on one stream. */
/* x[t, :] = f32(table[ids[t], :]) for T token ids (Generator._embed,
 * src/orchestrator/generator.py:38-39, on the f16 table), then norm = rms_norm(x, w) as
 * pyre_rms_norm (the first layer's input RMSNorm, root_node.py:752); w and norm both null:
 * gather only. ids: int32 on the device. An id outside [0, V) gives a zero row and writes
 * PYRE_EINVAL to *status (when status is not null). */
PYRE_API int pyre_embed_rms_norm(const int* ids, int T, const void* table, int V, int H, const float* w, double eps,
                                 float* x, float* norm, int* status, void* stream);
PYRE_API int pyre_lm_head_workspace_bytes(int T, int64_t* bytes);
PYRE_API int pyre_lm_head_argmax(const float* h, int T, int H, const float* norm_w, double eps,
                                 const uint16_t* lm_head, int V, int64_t v0, float* logits, int* token,
                                 long long* key, void* workspace, int64_t ws_bytes, void* stream);

/* ---- decode step of a whole decoder ----------------------------------------------------
 * One greedy token of a Llama-style decoder (src/orchestrator/generator.py:117-131 over
 * RootNode._decode_single_layer, root_node.py:739-1007, head-partitioned with every head
 * local) as the launch sequence embed_rms_norm -> per layer {q80_linear [Wq|Wk|Wv],
 * attn_decode_step, q80_linear Wo, add_rms_norm, ffn_decode_q80, add_rms_norm} ->
 * lm_head_argmax, issued from one host call. All pointers are device memory the caller
 * allocated; the structs are read on every call (nothing is retained). */
typedef struct pyre_decoder_layer {
  const void* qkv_w;   /* packed single Q8_0 matrix [H, (nq + 2 nkv) hd] (pyre_q80_pack, M = 1) */
  void* qkv_ws;        /* pyre_ffn_workspace_bytes(1, H, (nq + 2 nkv) hd), zeroed once */
  int64_t qkv_ws_bytes;
  const void* o_w;     /* packed [nq hd, H] */
  void* o_ws;
  int64_t o_ws_bytes;
  const void* gateup_w; /* FFN gate/up pair (or up alone) and down, as pyre_ffn_decode_q80 */
  const void* down_w;
  int gated;
  void* ffn_ws;
  int64_t ffn_ws_bytes;
  const float* ln1;    /* input_layernorm [H] */
  const float* ln2;    /* post_attention_layernorm [H] */
  uint16_t* k_cache;   /* f16 [nkv, max_t, hd] */
  uint16_t* v_cache;
  const float* rope;   /* pyre_rope_table for max_t positions */
  void* attn_ws;       /* pyre_attn_decode_workspace_bytes */
  int64_t attn_ws_bytes;
  const float* qkv_bias; /* f32 [(nq + 2 nkv) hd]: [q_bias | k_bias | v_bias], or NULL */
} pyre_decoder_layer;

typedef struct pyre_decoder_desc {
  int n_layers, H, nq, nkv, hd, ffn_width, V, max_t;
  int scale_dtype;     /* PYRE_F32 or PYRE_F16, every matrix */
  double eps, rope_fraction;
  const pyre_decoder_layer* layers; /* host array of n_layers */
  const void* embedding; /* f16 [V, H] */
  const uint16_t* lm_head; /* f16 [V, H] (the embedding when tied) */
  const float* final_norm; /* [H] or NULL */
  void* lm_ws;         /* pyre_lm_head_workspace_bytes(1) */
  int64_t lm_ws_bytes;
  float *x, *xn, *hn, *qkv, *attn, *ao, *f; /* scratch: [H] x3, [(nq + 2 nkv) hd], [nq hd], [H] x2 */
  int* status;         /* embedding status word */
  long long* key;      /* [1] */
  int* pos_dev;        /* NULL, or int32 [1] on the device: the step's position is read there
                        * (the pos argument only plans the attention grid and must not exceed
                        * it), and the step ends with history[*pos_dev + 1] = token_out and
                        * *pos_dev += 1, so the step can be captured once in a CUDA graph and
                        * replayed for positions pos, pos + 1, ... */
  int* history;        /* with pos_dev: int32 [max_t + 1], token at each position */
  /* Tensor parallelism (NULL: one GPU). Rank r of comm holds heads nq, nkv of this struct (its
   * share), the QKV columns and O rows of those heads, an FFN shard of ffn_width, and lm_head
   * rows lm_v0 .. lm_v0 + lm_V - 1 of the vocabulary; the O projection and the FFN sum their
   * partials over the ranks in their epilogues (NVLink peer stores), and the ranks' best
   * (value, index) keys are combined over comm into the greedy token. Every rank makes the same
   * calls in the same order. */
  pyre_comm_t* comm;
  int64_t lm_v0;       /* first vocabulary row of lm_head (0 without a vocabulary split) */
  int lm_V;            /* rows of lm_head; 0: V (the whole table) */
  /* Static batch (0 or 1: one sequence): B sequences decoded in lockstep at one position.
   * token_in / token_out hold B ids, the scratch vectors are [B, ...], each layer's caches
   * [B, nkv, max_t, hd] with attn_ws of pyre_attn_decode_workspace_bytes(B nq, B nkv, hd,
   * max_t), logits [B, lm_V], history [B, max_t + 1]; the projections and the FFN run on row
   * groups of at most 4 tokens, so every sequence's arithmetic equals a one-sequence step's. */
  int batch;
} pyre_decoder_desc;

/* One decode step: token_in (int32 [1], device) at position pos (= tokens already in the
 * caches), positions [mask_lo, mask_hi) masked (the reference's padded prefill; 0, 0: none).
 * Writes the greedy token to token_out (int32 [1], device) and, when logits is not NULL, the
 * logits f32 [V]. */
/* The fused attention decode step of pyre_attn_decode_step with the position in device memory
 * (int32 *pos_dev, read by the kernel): valid for every position p with plan_pos <= p < max_t,
 * the grid being planned for plan_pos. A position outside that range makes the kernel do
 * nothing and report PYRE_EINVAL through pyre_attn_status. For steps captured in CUDA graphs. */
PYRE_API int pyre_attn_decode_step_dev(const float* q, const float* k, const float* v, const int* pos_dev,
                                       int plan_pos, const float* rope_table, double rope_fraction, int nq, int nkv,
                                       int hd, uint16_t* k_cache, uint16_t* v_cache, int max_t, int mask_lo,
                                       int mask_hi, float* out, void* workspace, int64_t ws_bytes, void* stream);

/* The fused decode step for B sequences at one position (a static batch decoded in lockstep):
 * q, k, v of sequence b start at q + b * qkv_stride, k + b * qkv_stride, v + b * qkv_stride (one
 * fused QKV projection output [B, (nq + 2 nkv) hd] passed as three offset pointers); the caches
 * are [B, nkv, max_t, hd] f16 and out [B, nq * hd] f32. Every sequence's cache is split as in a
 * single-sequence step, so each sequence's result equals pyre_attn_decode_step_dev's bit for
 * bit. pos_dev (nullable) as in pyre_attn_decode_step_dev, else the position is plan_pos.
 * workspace: pyre_attn_decode_workspace_bytes(B * nq, B * nkv, hd, max_t), zeroed once. */
PYRE_API int pyre_attn_decode_step_batch(const float* q, const float* k, const float* v, int64_t qkv_stride, int B,
                                         const int* pos_dev, int plan_pos, const float* rope_table,
                                         double rope_fraction, int nq, int nkv, int hd, uint16_t* k_cache,
                                         uint16_t* v_cache, int max_t, float* out, void* workspace, int64_t ws_bytes,
                                         void* stream);

/* sizeof(pyre_decoder_layer) and sizeof(pyre_decoder_desc), for bindings that lay the
 * structs out themselves (ctypes, cgo) to check their layout against. */
PYRE_API int pyre_decoder_struct_sizes(int64_t* layer_bytes, int64_t* desc_bytes);

PYRE_API int pyre_decoder_step(const pyre_decoder_desc* d, const int* token_in, int pos, int mask_lo, int mask_hi,
                               int* token_out, float* logits, void* stream);

/* The same decode step with every layer in ONE persistent launch (RootNode._decode_single_layer,
 * root_node.py:739-1007, for all layers; Generator's decode loop, generator.py:117-131):
 * embedding gather -> decode_persistent_kernel (one CTA per SM for the whole token: a work queue
 * of QKV, attention, O, FFN gate/up and down items over all layers, weight blocks and KV rows
 * streamed through a shared-memory ring while the consumers wait on the previous stage's
 * flags) -> lm_head_argmax (-> position advance with pos_dev). Same arguments and results as
 * pyre_decoder_step for one sequence on one GPU (batch <= 1, comm NULL, f16 scales, head_dim 64
 * or 128, (nq / nkv) * head_dim <= 512, H, nq * hd and ffn_width multiples of 64), no prefill
 * mask; the per-layer scratch workspaces of the descriptor are not used. workspace:
 * pyre_decoder_persistent_workspace_bytes(d) bytes, 256-byte aligned, zeroed once and reused
 * call after call on one stream (every call leaves it ready for the next). A bounded wait that
 * ran out, an out-of-range partial or a graphed position outside the cache leaves PYRE_ETIMEOUT /
 * PYRE_ERANGE / PYRE_EINVAL in the workspace's status word (pyre_decoder_persistent_status). */
PYRE_API int pyre_decoder_persistent_workspace_bytes(const pyre_decoder_desc* d, int64_t* bytes);
PYRE_API int pyre_decoder_step_persistent(const pyre_decoder_desc* d, void* workspace, int64_t ws_bytes,
                                          const int* token_in, int pos, int* token_out, float* logits, void* stream);
/* Reads the persistent workspace's status word (synchronous copy; 0 = no problem). */
PYRE_API int pyre_decoder_persistent_status(const void* workspace, int* status);

/* ---- Ulysses sequence parallelism over NVLink (one process per GPU, P <= 16) ----------
 * Replaces the gather of every node's q/k/v at the root over TCP and the full-sequence
 * attention there (src/orchestrator/root_node.py:250-314; Ulysses mode :110): rank r owns
 * tokens [r*S/P, (r+1)*S/P) and heads [r*nq/P, ..) / [r*nkv/P, ..). Each rank allocates one
 * buffer of pyre_ulysses_buffer_bytes() with pyre_comm_alloc() (zeroed) and maps its peers'
 * (pyre_comm_open_peer); bufs[i] is rank i's buffer as seen from this process. Per call,
 * on one stream: pyre_ulysses_rope_scatter (RoPE at the tokens' global positions, clip, and
 * NVLink stores of every head into its owner's buffer), pyre_ulysses_barrier(phase 0),
 * pyre_ulysses_attention (causal attention of the owned heads over the whole sequence, each
 * output row stored into its token owner's buffer), pyre_ulysses_barrier(phase 1), then
 * pyre_ulysses_finish (sync, status, and the rank's [S/P, nq*hd] f32 output). Barrier waits
 * are bounded by timeout_ns and report PYRE_ETIMEOUT through pyre_ulysses_finish. */
PYRE_API int pyre_ulysses_buffer_bytes(int S, int P, int nq, int nkv, int hd, int64_t* bytes);
PYRE_API int pyre_ulysses_rope_scatter(void* const* bufs, int rank, int P, const float* q, const float* k,
                                       const float* v, int64_t q_stride, int64_t kv_stride, int S, int nq, int nkv,
                                       int hd, const float* rope_table, double rope_fraction, void* stream);
PYRE_API int pyre_ulysses_barrier(void* const* bufs, int rank, int P, int S, int nq, int nkv, int hd, int phase,
                                  uint64_t timeout_ns, void* stream);
PYRE_API int pyre_ulysses_attention(void* const* bufs, int rank, int P, int S, int nq, int nkv, int hd,
                                    void* stream);
PYRE_API int pyre_ulysses_finish(void* local_buf, int P, int S, int nq, int nkv, int hd, float* out, int* status,
                                 void* stream);
/* After a call whose barrier timed out: zeroes this rank's Ulysses flags, epoch and status word
 * (every rank, between host barriers, nothing in flight), as pyre_comm_reset does for comm. */
PYRE_API int pyre_ulysses_reset(void* local_buf, int P, int S, int nq, int nkv, int hd, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PYRE_B200_H */
