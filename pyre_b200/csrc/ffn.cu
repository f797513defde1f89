// Gated-SiLU FFN shard on Q8_0 weights: decode GEMV (T <= 4) and a SIMT GEMM for larger T.
//
// Reference semantics (src/ffn/builder.py:37-45, src/orchestrator/root_node.py:972-980):
//   gate = x @ Wg, up = x @ Wu, h = silu(gate) * up, partial = h @ Wd
// with silu(g) = g / (1 + exp(-g)) (src/kernels/mojo/pyre_kernels.mojo:121-129) and
// Wg, Wu, Wd dequantized from Q8_0 (src/orchestrator/quantizer.py:29-40) as a reference
// worker does (src/orchestrator/worker_node.py:59-69). Accumulation is f32.
//
// Decode GEMV layout. A weight is int8 [K, N] row-major with scales [K, N/32]. The output
// columns are cut into tiles of 128; a tile is covered by work units of 32 input rows.
// A warp reads 4 rows x 128 columns per unit step: lane (rs, cc) streams the 16 bytes
// q[k, 16cc .. 16cc+15] of row k = 4*warp + rs with one 128-bit load, so each row
// segment is a full 128-byte line. The (tile, unit) space is split evenly over a grid of
// co-resident CTAs (stream-K): a CTA sums its units of a tile in registers, reduces across
// its warps in shared memory and, when the tile is shared with other CTAs, the last CTA
// to finish adds the pieces in CTA order (deterministic) and runs the epilogue.
#include <algorithm>

#include "comm.cuh"

namespace pyre {
namespace ffn {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCols = 128;
constexpr int kUnitRows = 32;
constexpr int kMaxGrid = 1024;
constexpr int kCounterWords = 2048;  // tiles <= 2048 (N <= 262144)

enum Epi : int { EPI_SILU_MUL = 0, EPI_SILU = 1, EPI_STORE = 2, EPI_TP = 3 };

struct Params {
  const void* x;             // [T, K]
  const int8_t* q0;          // gate (NMAT == 2) or the single matrix
  const void* s0;
  const int8_t* q1;          // up (NMAT == 2)
  const void* s1;
  int K, N, T;
  int tiles;                 // ceil(N / kCols)
  int upt;                   // units per tile = ceil(K / kUnitRows)
  int64_t total_units;       // tiles * upt
  int pmax;                  // piece slots per tile in ws
  int64_t ws_cap;            // bytes of ws (after the counters)
  float* ws;                 // [tiles, pmax, NMAT, T, kCols]
  unsigned int* counters;    // [tiles], zero between calls
  void* out;                 // [T, N]
  int out_bf16;
  comm::DevComm comm;        // EPI_TP only
};

__device__ __forceinline__ float silu_f32(float g) { return __fdiv_rn(g, 1.0f + expf(-g)); }

template <typename ST>
__device__ __forceinline__ float ld_scale(const void* s, int64_t i) {
  return to_f32(__ldg(static_cast<const ST*>(s) + i));
}

template <typename XT>
__device__ __forceinline__ float ld_x(const void* x, int64_t i) {
  return to_f32(__ldg(static_cast<const XT*>(x) + i));
}

__device__ __forceinline__ void store_out(const Params& p, int t, int col, float v) {
  const int64_t o = static_cast<int64_t>(t) * p.N + col;
  if (p.out_bf16)
    static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(p.out)[o] = v;
}

// First / last CTA whose unit range [c*U/G, (c+1)*U/G) contains unit index x.
__host__ __device__ __forceinline__ int cta_of_unit(int64_t x, int64_t U, int G) {
  return static_cast<int>(((x + 1) * G - 1) / U);
}

// Epilogue over the finished tile sums vals(m, t, c) held in shared memory `fin`
// ([NMAT][T][kCols]).
template <int T, int NMAT, int EPI>
__device__ void tile_epilogue(const Params& p, int tile, const float* fin, uint32_t epoch) {
  const int col_base = tile * kCols;
  if constexpr (EPI == EPI_TP) {
    const comm::DevComm& c = p.comm;
    const int slot = epoch & 1u;
    const int n = T * kCols;
    // push this rank's tile partial into every rank's receive slot (self included)
    for (int peer = 0; peer < c.world; ++peer) {
      float* dst = comm::fused_slot(c, peer, slot, c.rank) + static_cast<int64_t>(tile) * n;
      for (int i = threadIdx.x; i < n; i += kThreads) dst[i] = fin[i];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < c.world) st_release_sys(comm::fused_flag(c, threadIdx.x, slot, c.rank, tile), epoch);
    if (threadIdx.x < c.world) {
      if (!wait_flag_eq(comm::fused_flag(c, c.rank, slot, threadIdx.x, tile), epoch, c.timeout_ns))
        atomicExch(c.status, PYRE_ETIMEOUT);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const int t = i / kCols, cc = i % kCols;
      const int col = col_base + cc;
      if (col >= p.N) continue;
      float acc = 0.f;
      for (int src = 0; src < c.world; ++src)
        acc += __ldcg(comm::fused_slot(c, c.rank, slot, src) + static_cast<int64_t>(tile) * n + i);
      store_out(p, t, col, acc);
    }
  } else {
    for (int i = threadIdx.x; i < T * kCols; i += kThreads) {
      const int t = i / kCols, cc = i % kCols;
      const int col = col_base + cc;
      if (col >= p.N) continue;
      float v;
      if constexpr (EPI == EPI_SILU_MUL) {
        v = silu_f32(fin[i]) * fin[T * kCols + i];
      } else if constexpr (EPI == EPI_SILU) {
        v = silu_f32(fin[i]);
      } else {
        v = fin[i];
      }
      store_out(p, t, col, v);
    }
  }
}

template <int T, int NMAT>
struct GemvCfg {
  static constexpr int kUnroll = (T * NMAT <= 2) ? 4 : 2;
  static constexpr int kMinBlocks = (T * NMAT <= 2) ? 2 : 1;
};

template <int T, int NMAT, int EPI, typename XT, typename ST>
__global__ void __launch_bounds__(kThreads, (GemvCfg<T, NMAT>::kMinBlocks))
q80_gemv_kernel(const Params p) {
  constexpr int UNR = GemvCfg<T, NMAT>::kUnroll;
  __shared__ float red[kWarps][NMAT * T * kCols];
  __shared__ float fin[NMAT * T * kCols];
  __shared__ int s_last;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int rs = lane >> 3;
  const int cc = lane & 7;
  const int G = gridDim.x;
  const int c = blockIdx.x;
  const int64_t U = p.total_units;
  int64_t u = (static_cast<int64_t>(c) * U) / G;
  const int64_t u_end = (static_cast<int64_t>(c + 1) * U) / G;
  const int nsb = p.N / 32;
  const int8_t* qm[2] = {p.q0, p.q1};
  const void* sm[2] = {p.s0, p.s1};
  uint32_t epoch = 0;
  if constexpr (EPI == EPI_TP) epoch = comm::epoch_begin(p.comm);

  while (u < u_end) {
    const int tile = static_cast<int>(u / p.upt);
    const int64_t tile_u0 = static_cast<int64_t>(tile) * p.upt;
    const int64_t seg_end = min(u_end, tile_u0 + p.upt);
    const int col0 = tile * kCols + cc * 16;
    const bool col_ok = col0 < p.N;

    float acc[NMAT][T][16];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int t = 0; t < T; ++t)
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[m][t][i] = 0.f;

    for (int64_t ub = u; ub < seg_end; ub += UNR) {
      int4 wv[UNR][NMAT];
      float sv[UNR][NMAT];
      float xv[UNR][T];
#pragma unroll
      for (int j = 0; j < UNR; ++j) {
        const int64_t uj = ub + j;
        const int k = static_cast<int>((uj - tile_u0) * kUnitRows) + warp * 4 + rs;
        const bool ok = col_ok && (uj < seg_end) && (k < p.K);
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          if (ok) {
            wv[j][m] = ld_stream16(qm[m] + static_cast<int64_t>(k) * p.N + col0);
            sv[j][m] = ld_scale<ST>(sm[m], static_cast<int64_t>(k) * nsb + (col0 >> 5));
          } else {
            wv[j][m] = make_int4(0, 0, 0, 0);
            sv[j][m] = 0.f;
          }
        }
#pragma unroll
        for (int t = 0; t < T; ++t) xv[j][t] = ok ? ld_x<XT>(p.x, static_cast<int64_t>(t) * p.K + k) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < UNR; ++j) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          const uint32_t words[4] = {static_cast<uint32_t>(wv[j][m].x), static_cast<uint32_t>(wv[j][m].y),
                                     static_cast<uint32_t>(wv[j][m].z), static_cast<uint32_t>(wv[j][m].w)};
          float a[T];
#pragma unroll
          for (int t = 0; t < T; ++t) a[t] = xv[j][t] * sv[j][m];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            float f[4];
            s8x4_to_f32(words[w], f);
#pragma unroll
            for (int t = 0; t < T; ++t)
#pragma unroll
              for (int i = 0; i < 4; ++i) acc[m][t][w * 4 + i] = fmaf(a[t], f[i], acc[m][t][w * 4 + i]);
          }
        }
      }
    }

    u = seg_end;

    // reduce the 4 row lanes of each column chunk, then across warps
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int t = 0; t < T; ++t)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float v = acc[m][t][i];
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          acc[m][t][i] = v;
        }
    if (rs == 0) {
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int t = 0; t < T; ++t)
#pragma unroll
          for (int i = 0; i < 16; ++i) red[warp][(m * T + t) * kCols + cc * 16 + i] = acc[m][t][i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NMAT * T * kCols; i += kThreads) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += red[w][i];
      fin[i] = v;
    }
    __syncthreads();

    const int cf = cta_of_unit(tile_u0, U, G);
    const int cl = cta_of_unit(tile_u0 + p.upt - 1, U, G);
    if (cf == cl) {
      tile_epilogue<T, NMAT, EPI>(p, tile, fin, epoch);
    } else {
      const int piece = c - cf;
      const int np = cl - cf + 1;
      float* slot = p.ws + (static_cast<int64_t>(tile) * p.pmax + piece) * (NMAT * T * kCols);
      for (int i = threadIdx.x; i < NMAT * T * kCols; i += kThreads) __stcg(slot + i, fin[i]);
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(p.counters + tile, 1u);
        s_last = (prev == static_cast<unsigned>(np - 1));
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        const float* base = p.ws + static_cast<int64_t>(tile) * p.pmax * (NMAT * T * kCols);
        for (int i = threadIdx.x; i < NMAT * T * kCols; i += kThreads) {
          float v = 0.f;
          for (int pc = 0; pc < np; ++pc) v += __ldcg(base + static_cast<int64_t>(pc) * (NMAT * T * kCols) + i);
          fin[i] = v;
        }
        __syncthreads();
        tile_epilogue<T, NMAT, EPI>(p, tile, fin, epoch);
        if (threadIdx.x == 0) p.counters[tile] = 0u;
      }
    }
    __syncthreads();
  }
  if constexpr (EPI == EPI_TP) comm::epoch_end(p.comm, epoch);
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
  const int nsb = p.N / 32;
  float acc[NMAT][4][4];
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[m][i][j] = 0.f;
  const int8_t* qm[2] = {p.q0, p.q1};
  const void* sm[2] = {p.s0, p.s1};

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
        if (k < p.K && n < p.N)
          w = static_cast<float>(qm[m][static_cast<int64_t>(k) * p.N + n]) *
              ld_scale<ST>(sm[m], static_cast<int64_t>(k) * nsb + (n >> 5));
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
      store_out(p, t, n, v);
    }
  }
}

// ---- host side ------------------------------------------------------------------------

int tiles_of(int N) { return (N + kCols - 1) / kCols; }

// Grid of the GEMV for one instantiation: every CTA co-resident, capped by the work.
template <typename K>
int gemv_grid(K kernel, int64_t units) {
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kThreads, 0) != cudaSuccess || occ < 1) occ = 1;
  int64_t g = static_cast<int64_t>(occ) * sm_count();
  if (g > kMaxGrid) g = kMaxGrid;
  if (g > units) g = units;
  return static_cast<int>(g < 1 ? 1 : g);
}

int pmax_for(int tiles, int upt, int G) {
  const int64_t U = static_cast<int64_t>(tiles) * upt;
  int pm = 1;
  for (int t = 0; t < tiles; ++t) {
    const int64_t u0 = static_cast<int64_t>(t) * upt;
    const int np = cta_of_unit(u0 + upt - 1, U, G) - cta_of_unit(u0, U, G) + 1;
    pm = std::max(pm, np);
  }
  return pm;
}

// Upper bound of the piece workspace for any grid <= kMaxGrid.
int64_t gemv_ws_bytes(int T, int K, int N, int nmat) {
  const int tiles = tiles_of(N);
  const int64_t pmax = (kMaxGrid + tiles - 1) / tiles + 1;
  (void)K;
  return static_cast<int64_t>(tiles) * pmax * nmat * T * kCols * 4;
}

constexpr int64_t kCounterBytes = kCounterWords * 4;

template <int T, int NMAT, int EPI, typename XT, typename ST>
int launch_gemv(Params p, cudaStream_t s) {
  auto kern = q80_gemv_kernel<T, NMAT, EPI, XT, ST>;
  const int G = gemv_grid(kern, p.total_units);
  p.pmax = pmax_for(p.tiles, p.upt, G);
  if (static_cast<int64_t>(p.tiles) * p.pmax * NMAT * T * kCols * 4 > p.ws_cap)
    return set_error(PYRE_ENOMEM, "q80_gemv: stream-K workspace too small for this grid");
  kern<<<G, kThreads, 0, s>>>(p);
  PYRE_LAUNCH_CHECK("q80_gemv_kernel");
  return PYRE_OK;
}

template <int NMAT, int EPI, typename XT, typename ST>
int dispatch_T(Params p, cudaStream_t s) {
  switch (p.T) {
    case 1: return launch_gemv<1, NMAT, EPI, XT, ST>(p, s);
    case 2: return launch_gemv<2, NMAT, EPI, XT, ST>(p, s);
    case 3: return launch_gemv<3, NMAT, EPI, XT, ST>(p, s);
    case 4: return launch_gemv<4, NMAT, EPI, XT, ST>(p, s);
    default: break;
  }
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

int check_common(const void* x, int x_dtype, int T, int K, int N, int scale_dtype, const void* out,
                 const void* ws, int64_t ws_bytes, const char* fn) {
  std::string f(fn);
  PYRE_CHECK_ARG(x != nullptr && out != nullptr, f + ": null input/output");
  PYRE_CHECK_ARG(T >= 1 && K >= 1 && N >= 32, f + ": sizes must be positive (N >= 32)");
  PYRE_CHECK_ARG(N % 32 == 0, f + ": output width must be a multiple of 32 (Q8_0 blocks run along it)");
  PYRE_CHECK_ARG(x_dtype == PYRE_F32 || x_dtype == PYRE_BF16, f + ": activation dtype must be f32 or bf16");
  PYRE_CHECK_ARG(scale_dtype == PYRE_F32 || scale_dtype == PYRE_F16, f + ": scale dtype must be f32 or f16");
  PYRE_CHECK_ARG(tiles_of(N) <= kCounterWords, f + ": output width too large");
  PYRE_CHECK_ARG(ws != nullptr || T > PYRE_FUSED_REDUCE_MAX_T, f + ": null workspace");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(ws) % 16 == 0, f + ": workspace must be 16-byte aligned");
  PYRE_CHECK_ARG(ws_bytes >= 0, f + ": negative workspace size");
  return PYRE_OK;
}

int64_t ws_need(int T, int K, int N, int nmat) {
  if (T > PYRE_FUSED_REDUCE_MAX_T) return 0;
  return kCounterBytes + gemv_ws_bytes(T, K, N, nmat);
}

}  // namespace ffn
}  // namespace pyre

using namespace pyre;
using namespace pyre::ffn;

extern "C" int pyre_ffn_workspace_bytes(int T, int H, int W, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_ffn_workspace_bytes: null bytes");
  PYRE_CHECK_ARG(T >= 1 && H >= 1 && W >= 1, "pyre_ffn_workspace_bytes: sizes must be positive");
  const int64_t a = ws_need(T, H, W, 2);   // gate/up: K = H, N = W
  const int64_t b = ws_need(T, W, H, 1);   // down:    K = W, N = H
  int64_t need = std::max(a, b);
  if (need < kCounterBytes) need = kCounterBytes;
  *bytes = need;
  return PYRE_OK;
}

extern "C" int pyre_ffn_gateup_silu_q80(const void* x, int x_dtype, int T, int H, const int8_t* qg,
                                        const void* sg, const int8_t* qu, const void* su, int scale_dtype,
                                        int W, void* h, int h_dtype, void* workspace, int64_t ws_bytes,
                                        void* stream) {
  int rc = check_common(x, x_dtype, T, H, W, scale_dtype, h, workspace, ws_bytes, "pyre_ffn_gateup_silu_q80");
  if (rc) return rc;
  PYRE_CHECK_ARG(qu != nullptr && su != nullptr, "pyre_ffn_gateup_silu_q80: null up weight");
  PYRE_CHECK_ARG((qg == nullptr) == (sg == nullptr), "pyre_ffn_gateup_silu_q80: gate q/scale mismatch");
  PYRE_CHECK_ARG(h_dtype == PYRE_F32 || h_dtype == PYRE_BF16, "pyre_ffn_gateup_silu_q80: h dtype must be f32 or bf16");
  const bool gated = qg != nullptr;
  const int64_t need = ws_need(T, H, W, gated ? 2 : 1);
  if (ws_bytes < need)
    return set_error(PYRE_ENOMEM, "pyre_ffn_gateup_silu_q80: workspace smaller than pyre_ffn_workspace_bytes()");
  Params p{};
  p.x = x;
  p.K = H;
  p.N = W;
  p.T = T;
  p.tiles = tiles_of(W);
  p.upt = (H + kUnitRows - 1) / kUnitRows;
  p.total_units = static_cast<int64_t>(p.tiles) * p.upt;
  p.counters = static_cast<unsigned int*>(workspace);
  p.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  p.ws_cap = ws_bytes - kCounterBytes;
  p.out = h;
  p.out_bf16 = h_dtype == PYRE_BF16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gated) {
    p.q0 = qg; p.s0 = sg; p.q1 = qu; p.s1 = su;
    return dispatch_types<2, EPI_SILU_MUL>(p, x_dtype, scale_dtype, s);
  }
  p.q0 = qu; p.s0 = su; p.q1 = nullptr; p.s1 = nullptr;
  return dispatch_types<1, EPI_SILU>(p, x_dtype, scale_dtype, s);
}

extern "C" int pyre_ffn_down_q80(const void* h, int h_dtype, int T, int W, const int8_t* qd, const void* sd,
                                 int scale_dtype, int H, float* out, void* workspace, int64_t ws_bytes,
                                 pyre_comm_t* comm, void* stream) {
  int rc = check_common(h, h_dtype, T, W, H, scale_dtype, out, workspace, ws_bytes, "pyre_ffn_down_q80");
  if (rc) return rc;
  PYRE_CHECK_ARG(qd != nullptr && sd != nullptr, "pyre_ffn_down_q80: null weight");
  const int64_t need = ws_need(T, W, H, 1);
  if (ws_bytes < need)
    return set_error(PYRE_ENOMEM, "pyre_ffn_down_q80: workspace smaller than pyre_ffn_workspace_bytes()");
  if (comm != nullptr) {
    PYRE_CHECK_ARG(comm->hidden == H, "pyre_ffn_down_q80: communicator hidden size differs from H");
    PYRE_CHECK_ARG(T <= comm->max_tokens, "pyre_ffn_down_q80: T exceeds the communicator's max_tokens");
  }
  Params p{};
  p.x = h;
  p.q0 = qd; p.s0 = sd; p.q1 = nullptr; p.s1 = nullptr;
  p.K = W;
  p.N = H;
  p.T = T;
  p.tiles = tiles_of(H);
  p.upt = (W + kUnitRows - 1) / kUnitRows;
  p.total_units = static_cast<int64_t>(p.tiles) * p.upt;
  p.counters = static_cast<unsigned int*>(workspace);
  p.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  p.ws_cap = ws_bytes - kCounterBytes;
  p.out = out;
  p.out_bf16 = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tp = comm != nullptr && comm->world > 1;
  if (tp && T <= PYRE_FUSED_REDUCE_MAX_T) {
    p.comm = comm::device_view(comm);
    return dispatch_types<1, EPI_TP>(p, h_dtype, scale_dtype, s);
  }
  rc = dispatch_types<1, EPI_STORE>(p, h_dtype, scale_dtype, s);
  if (rc || !tp) return rc;
  return allreduce_sum_f32(comm, out, static_cast<int64_t>(T) * H, s);
}
