// Gated-SiLU FFN shard on Q8_0 weights, two-call form: gate/up + SiLU·mul, then down
// (+ the cross-rank sum). Decode (T <= 4) runs the streaming kernel of ffn_stream.cuh;
// larger T runs a SIMT dequant GEMM (placeholder for the tensor-core path).
//
// Reference semantics (src/ffn/builder.py:37-45, src/orchestrator/root_node.py:972-980):
//   gate = x @ Wg, up = x @ Wu, h = silu(gate) * up, partial = h @ Wd
// with silu(g) = g / (1 + exp(-g)) (src/kernels/mojo/pyre_kernels.mojo:121-129) and the
// weights dequantized from Q8_0 (src/orchestrator/quantizer.py:29-40) as a reference worker
// does (src/orchestrator/worker_node.py:59-69). Accumulation is f32.
//
// Weights are in the packed block layout of gemv_common.cuh (gate and up interleaved per
// block for the gated form).
#include <algorithm>

#include "ffn_internal.cuh"

namespace pyre {
namespace ffn {

using namespace gemv;

template <typename ST>
__device__ __forceinline__ float ld_scale(const void* s, int64_t i) {
  return to_f32(__ldg(static_cast<const ST*>(s) + i));
}

template <typename XT>
__device__ __forceinline__ float ld_x(const void* x, int64_t i) {
  return to_f32(__ldg(static_cast<const XT*>(x) + i));
}

// ---- SIMT GEMM for T > 4 --------------------------------------------------------------
// CTA tile: 64 tokens x 64 columns, K step 32. Weights are dequantized into shared
// memory as f32; each thread owns a 4x4 block of outputs per matrix.
constexpr int kGM = 64, kGN = 64, kGK = 32;

template <int NMAT, int EPI, typename XT, typename ST>
__global__ void __launch_bounds__(256) q80_gemm_simt_kernel(const Params p) {
  __shared__ float xs[kGK][kGM + 4];
  __shared__ float wsm[NMAT][kGK][kGN + 4];
  const int tx = threadIdx.x & 15;   // column group
  const int ty = threadIdx.x >> 4;   // token group
  const int n0 = blockIdx.x * kGN;
  const int t0 = blockIdx.y * kGM;
  float acc[NMAT][4][4];
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[m][i][j] = 0.f;
  constexpr int R = UnitRows<NMAT>::value;
  const int64_t bbytes = packed_block_bytes(NMAT, sizeof(ST));

  for (int k0 = 0; k0 < p.K; k0 += kGK) {
    for (int i = threadIdx.x; i < kGM * kGK; i += 256) {
      const int tt = i / kGK, kk = i % kGK;
      const int t = t0 + tt, k = k0 + kk;
      xs[kk][tt] = (t < p.T && k < p.K) ? ld_x<XT>(p.x, static_cast<int64_t>(t) * p.K + k) : 0.f;
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      for (int i = threadIdx.x; i < kGK * kGN; i += 256) {
        const int kk = i / kGN, nn = i % kGN;
        const int k = k0 + kk, n = n0 + nn;
        float w = 0.f;
        if (k < p.K && n < p.N) {
          const uint8_t* blk = p.w + (static_cast<int64_t>(n / kTileN) * p.upt + k / R) * bbytes;
          const int rr = k % R, cn = n % kTileN;
          const int8_t q = reinterpret_cast<const int8_t*>(blk)[(m * R + rr) * kTileN + cn];
          const ST* sc = reinterpret_cast<const ST*>(blk + NMAT * R * kTileN);
          w = static_cast<float>(q) * to_f32(sc[(m * R + rr) * 8 + (cn >> 5)]);
        }
        wsm[m][kk][nn] = w;
      }
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kGK; ++kk) {
      float a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        float b[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = wsm[m][kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[m][i][j] = fmaf(a[i], b[j], acc[m][i][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= p.T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= p.N) continue;
      float v;
      if constexpr (EPI == EPI_SILU_MUL) {
        v = silu_f32(acc[0][i][j]) * acc[NMAT - 1][i][j];
      } else if constexpr (EPI == EPI_SILU) {
        v = silu_f32(acc[0][i][j]);
      } else {
        v = acc[0][i][j];
      }
      store_out(p.out, p.out_bf16, p.N, t, n, v);
    }
  }
}

// ---- host side ------------------------------------------------------------------------

template <int NMAT, int EPI, typename XT, typename ST>
int dispatch_T(Params p, cudaStream_t s) {
  static_assert(EPI != EPI_TP || NMAT == 1, "TP epilogue is single-matrix");
  dim3 grid((p.N + kGN - 1) / kGN, (p.T + kGM - 1) / kGM);
  constexpr int GEPI = EPI == EPI_TP ? EPI_STORE : EPI;
  q80_gemm_simt_kernel<NMAT, GEPI, XT, ST><<<grid, 256, 0, s>>>(p);
  PYRE_LAUNCH_CHECK("q80_gemm_simt_kernel");
  return PYRE_OK;
}

template <int NMAT, int EPI>
int dispatch_types(Params p, int x_dtype, int scale_dtype, cudaStream_t s) {
  if (x_dtype == PYRE_BF16) {
    if (scale_dtype == PYRE_F16) return dispatch_T<NMAT, EPI, __nv_bfloat16, __half>(p, s);
    return dispatch_T<NMAT, EPI, __nv_bfloat16, float>(p, s);
  }
  if (scale_dtype == PYRE_F16) return dispatch_T<NMAT, EPI, float, __half>(p, s);
  return dispatch_T<NMAT, EPI, float, float>(p, s);
}

}  // namespace ffn

int ffn_check_common(const void* x, int x_dtype, int T, int K, int N, int scale_dtype, const void* out,
                     const void* ws, int64_t ws_bytes, const char* fn) {
  std::string f(fn);
  PYRE_CHECK_ARG(x != nullptr && out != nullptr, f + ": null input/output");
  PYRE_CHECK_ARG(T >= 1 && K >= 1 && N >= 32, f + ": sizes must be positive (N >= 32)");
  PYRE_CHECK_ARG(N % 32 == 0, f + ": output width must be a multiple of 32 (Q8_0 blocks run along it)");
  PYRE_CHECK_ARG(x_dtype == PYRE_F32 || x_dtype == PYRE_BF16, f + ": activation dtype must be f32 or bf16");
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
  PYRE_CHECK_ARG(h_dtype == PYRE_F32 || h_dtype == PYRE_BF16, "pyre_ffn_gateup_silu_q80: h dtype must be f32 or bf16");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T <= PYRE_FUSED_REDUCE_MAX_T)
    return ffn_stream_gateup(x, x_dtype, T, H, wgu, gated, scale_dtype, W, h, h_dtype, workspace, ws_bytes, s);
  const int R = gated ? kUnitRowsPair : kUnitRowsSingle;
  char* wsc = static_cast<char*>(workspace);
  Params p{};
  p.x = x;
  p.w = static_cast<const uint8_t*>(wgu);
  p.K = H;
  p.N = W;
  p.T = T;
  p.tiles = tiles_of(W);
  p.upt = (H + R - 1) / R;
  p.total_units = static_cast<int64_t>(p.tiles) * p.upt;
  p.counters = reinterpret_cast<unsigned int*>(wsc + kHdrCntA);
  p.status = reinterpret_cast<int*>(wsc + kHdrStatus);
  p.ws = reinterpret_cast<float*>(wsc + kHeaderBytes);
  p.ws_cap = ws_bytes - kHeaderBytes;
  p.out = h;
  p.out_bf16 = h_dtype == PYRE_BF16;
  if (gated) return dispatch_types<2, EPI_SILU_MUL>(p, x_dtype, scale_dtype, s);
  return dispatch_types<1, EPI_SILU>(p, x_dtype, scale_dtype, s);
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
  Params p{};
  p.x = h;
  p.w = static_cast<const uint8_t*>(wd);
  p.K = W;
  p.N = H;
  p.T = T;
  p.tiles = tiles_of(H);
  p.upt = (W + kUnitRowsSingle - 1) / kUnitRowsSingle;
  p.total_units = static_cast<int64_t>(p.tiles) * p.upt;
  p.counters = reinterpret_cast<unsigned int*>(wsc + kHdrCntB);
  p.status = reinterpret_cast<int*>(wsc + kHdrStatus);
  p.ws = reinterpret_cast<float*>(wsc + kHeaderBytes);
  p.ws_cap = ws_bytes - kHeaderBytes;
  p.out = out;
  p.out_bf16 = 0;
  const bool tp = comm != nullptr && comm->world > 1;
  rc = dispatch_types<1, EPI_STORE>(p, h_dtype, scale_dtype, s);
  if (rc || !tp) return rc;
  return allreduce_sum_f32(comm, out, static_cast<int64_t>(T) * H, s);
}
