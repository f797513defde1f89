// Gated-SiLU FFN shard on Q8_0 weights, two-call form: gate/up + SiLU·mul, then down
// (+ the cross-rank sum). Decode (T <= 4) runs the streaming kernel of ffn_stream.cuh;
// larger T runs the tensor-core GEMM of gemm_tc.cu.
//
// Reference semantics (src/ffn/builder.py:37-45, src/orchestrator/root_node.py:972-980):
//   gate = x @ Wg, up = x @ Wu, h = silu(gate) * up, partial = h @ Wd
// with silu(g) = g / (1 + exp(-g)) (src/kernels/mojo/pyre_kernels.mojo:121-129) and the
// weights dequantized from Q8_0 (src/orchestrator/quantizer.py:29-40) as a reference worker
// does (src/orchestrator/worker_node.py:59-69). Accumulation is f32.
//
// Weights are in the packed block layout of gemv_common.cuh (gate and up interleaved per
// block for the gated form).
#include "ffn_internal.cuh"

namespace pyre {
namespace ffn {

using namespace gemv;

}  // namespace ffn

int ffn_check_common(const void* x, int x_dtype, int T, int K, int N, int scale_dtype, const void* out,
                     const void* ws, int64_t ws_bytes, const char* fn) {
  std::string f(fn);
  PYRE_CHECK_ARG(x != nullptr && out != nullptr, f + ": null input/output");
  PYRE_CHECK_ARG(T >= 1 && K >= 1 && N >= 32, f + ": sizes must be positive (N >= 32)");
  PYRE_CHECK_ARG(N % 32 == 0, f + ": output width must be a multiple of 32 (Q8_0 blocks run along it)");
  PYRE_CHECK_ARG(x_dtype == PYRE_F32 || x_dtype == PYRE_BF16 || (x_dtype == PYRE_F16 && T > PYRE_FUSED_REDUCE_MAX_T),
                 f + ": activation dtype must be f32 or bf16 (or f16 for T > PYRE_FUSED_REDUCE_MAX_T)");
  PYRE_CHECK_ARG(scale_dtype == PYRE_F32 || scale_dtype == PYRE_F16, f + ": scale dtype must be f32 or f16");
  PYRE_CHECK_ARG(gemv::tiles_of(N) <= gemv::kMaxTiles, f + ": output width too large");
  PYRE_CHECK_ARG(T > PYRE_FUSED_REDUCE_MAX_T || (static_cast<int64_t>(K) * (x_dtype == PYRE_BF16 ? 2 : 4)) % 16 == 0,
                 f + ": activation rows must be 16-byte multiples");
  PYRE_CHECK_ARG(ws != nullptr, f + ": null workspace");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(ws) % 256 == 0, f + ": workspace must be 256-byte aligned");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(x) % 16 == 0, f + ": activations must be 16-byte aligned");
  PYRE_CHECK_ARG(ws_bytes >= gemv::kHeaderBytes, f + ": workspace smaller than pyre_ffn_workspace_bytes()");
  return PYRE_OK;
}

// The T > 4 path keeps its f16 activation staging and stream-K partial tiles at the END of
// the workspace, clear of the decode accumulators at its start (which must be zero on entry
// to a decode call), so one workspace serves prefill and decode calls in any order.
struct GemmRegion {
  char* stage;
  int64_t stage_bytes;
  char* part;
  int64_t part_bytes;
};

int gemm_region(void* workspace, int64_t ws_bytes, int T, int K, int N, int nmat, GemmRegion* r, const char* f) {
  const int64_t stage = ffn_gemm_staging_bytes(T, K, N);
  const int64_t part = ffn_gemm_partial_bytes(T, N, nmat);
  const int64_t base = (ws_bytes - stage - part) / 256 * 256;
  if (base < gemv::kHeaderBytes)
    return set_error(PYRE_ENOMEM, std::string(f) + ": workspace smaller than pyre_ffn_workspace_bytes()");
  char* wsc = static_cast<char*>(workspace);
  *r = GemmRegion{wsc + base, stage, wsc + base + stage, part};
  return PYRE_OK;
}

}  // namespace pyre

using namespace pyre;
using namespace pyre::ffn;

extern "C" int pyre_ffn_gateup_silu_q80(const void* x, int x_dtype, int T, int H, const void* wgu, int gated,
                                        int scale_dtype, int W, void* h, int h_dtype, void* workspace,
                                        int64_t ws_bytes, void* stream) {
  int rc = ffn_check_common(x, x_dtype, T, H, W, scale_dtype, h, workspace, ws_bytes, "pyre_ffn_gateup_silu_q80");
  if (rc) return rc;
  PYRE_CHECK_ARG(wgu != nullptr && reinterpret_cast<uintptr_t>(wgu) % 16 == 0,
                 "pyre_ffn_gateup_silu_q80: packed gate/up weights must be non-null and 16-byte aligned");
  PYRE_CHECK_ARG(h_dtype == PYRE_F32 || h_dtype == PYRE_BF16 || (h_dtype == PYRE_F16 && T > PYRE_FUSED_REDUCE_MAX_T),
                 "pyre_ffn_gateup_silu_q80: h dtype must be f32 or bf16 (or f16 for T > PYRE_FUSED_REDUCE_MAX_T)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T <= PYRE_FUSED_REDUCE_MAX_T)
    return ffn_stream_gateup(x, x_dtype, T, H, wgu, gated, scale_dtype, W, h, h_dtype, workspace, ws_bytes, s);
  char* wsc = static_cast<char*>(workspace);
  GemmRegion g;
  rc = gemm_region(workspace, ws_bytes, T, H, W, gated ? 2 : 1, &g, "pyre_ffn_gateup_silu_q80");
  if (rc) return rc;
  return ffn_gemm_tc(x, x_dtype, T, H, wgu, gated ? 2 : 1, gated ? EPI_SILU_MUL : EPI_SILU, scale_dtype, W, h,
                     h_dtype, g.stage, g.stage_bytes, g.part, g.part_bytes,
                     reinterpret_cast<unsigned int*>(wsc + kHdrCntA), reinterpret_cast<int*>(wsc + kHdrStatus), s);
}

extern "C" int pyre_ffn_down_q80(const void* h, int h_dtype, int T, int W, const void* wd, int scale_dtype, int H,
                                 float* out, void* workspace, int64_t ws_bytes, pyre_comm_t* comm, void* stream) {
  int rc = ffn_check_common(h, h_dtype, T, W, H, scale_dtype, out, workspace, ws_bytes, "pyre_ffn_down_q80");
  if (rc) return rc;
  PYRE_CHECK_ARG(wd != nullptr && reinterpret_cast<uintptr_t>(wd) % 16 == 0,
                 "pyre_ffn_down_q80: packed down weights must be non-null and 16-byte aligned");
  if (comm != nullptr) {
    PYRE_CHECK_ARG(comm->hidden == H, "pyre_ffn_down_q80: communicator hidden size differs from H");
    PYRE_CHECK_ARG(T <= comm->max_tokens, "pyre_ffn_down_q80: T exceeds the communicator's max_tokens");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T <= PYRE_FUSED_REDUCE_MAX_T)
    return ffn_stream_down(h, h_dtype, T, W, wd, scale_dtype, H, out, workspace, ws_bytes, comm, s);
  char* wsc = static_cast<char*>(workspace);
  GemmRegion g;
  rc = gemm_region(workspace, ws_bytes, T, W, H, 1, &g, "pyre_ffn_down_q80");
  if (rc) return rc;
  rc = ffn_gemm_tc(h, h_dtype, T, W, wd, 1, EPI_STORE, scale_dtype, H, out, PYRE_F32, g.stage, g.stage_bytes, g.part,
                   g.part_bytes, reinterpret_cast<unsigned int*>(wsc + kHdrCntA),
                   reinterpret_cast<int*>(wsc + kHdrStatus), s);
  const bool tp = comm != nullptr && comm->world > 1;
  if (rc || !tp) return rc;
  return allreduce_sum_f32(comm, out, static_cast<int64_t>(T) * H, s);
}

extern "C" int pyre_q80_linear_bias(const void* x, int x_dtype, int T, int K, const void* w, int scale_dtype,
                                    int N, const float* bias, float* out, void* workspace, int64_t ws_bytes,
                                    void* stream) {
  int rc = ffn_check_common(x, x_dtype, T, K, N, scale_dtype, out, workspace, ws_bytes, "pyre_q80_linear");
  if (rc) return rc;
  PYRE_CHECK_ARG(w != nullptr && reinterpret_cast<uintptr_t>(w) % 16 == 0,
                 "pyre_q80_linear: packed weights must be non-null and 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* wsc = static_cast<char*>(workspace);
  if (T <= PYRE_FUSED_REDUCE_MAX_T) {
    // matrices up to K = 8192 (the attention projections): one cluster per column slab, every
    // weight copy in flight at once, the split-K reduction in distributed shared memory
    if (gemv_cluster_eligible(K, N))
      return gemv_cluster(x, x_dtype, T, K, w, scale_dtype, N, bias, out, reinterpret_cast<int*>(wsc + kHdrStatus), s);
    return ffn_stream_down(x, x_dtype, T, K, w, scale_dtype, N, out, workspace, ws_bytes, nullptr, s, bias);
  }
  GemmRegion g;
  rc = gemm_region(workspace, ws_bytes, T, K, N, 1, &g, "pyre_q80_linear");
  if (rc) return rc;
  return ffn_gemm_tc(x, x_dtype, T, K, w, 1, EPI_STORE, scale_dtype, N, out, PYRE_F32, g.stage, g.stage_bytes, g.part,
                     g.part_bytes, reinterpret_cast<unsigned int*>(wsc + kHdrCntA),
                     reinterpret_cast<int*>(wsc + kHdrStatus), s, bias);
}

extern "C" int pyre_q80_linear(const void* x, int x_dtype, int T, int K, const void* w, int scale_dtype, int N,
                               float* out, void* workspace, int64_t ws_bytes, void* stream) {
  return pyre_q80_linear_bias(x, x_dtype, T, K, w, scale_dtype, N, nullptr, out, workspace, ws_bytes, stream);
}
