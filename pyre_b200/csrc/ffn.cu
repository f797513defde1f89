// Gated-SiLU FFN shard on Q8_0 weights: decode GEMV (T <= 4) and a SIMT GEMM for larger T.
//
// Reference semantics (src/ffn/builder.py:37-45, src/orchestrator/root_node.py:972-980):
//   gate = x @ Wg, up = x @ Wu, h = silu(gate) * up, partial = h @ Wd
// with silu(g) = g / (1 + exp(-g)) (src/kernels/mojo/pyre_kernels.mojo:121-129) and
// Wg, Wu, Wd dequantized from Q8_0 (src/orchestrator/quantizer.py:29-40) as a reference
// worker does (src/orchestrator/worker_node.py:59-69). Accumulation is f32.
//
// Device weight layout (column-slab tiled Q8_0). A [K, N] weight is cut into slabs of
// 256 output columns; slab j stores q[:, 256j : 256j+256] row-major (K x 256 int8,
// contiguous) and its scales [:, 8j : 8j+8] (K x 8), N padded with zeros to a multiple of
// 256. The values are exactly the reference's Q8_0 blocks; only the order differs, so a
// 32-row x 256-column work unit is one contiguous 8 KB run of HBM.
//
// Decode GEMV: the output columns of a slab form a tile; a tile is covered by work units
// of 32 input rows. The (tile, unit) space is split evenly over one CTA per SM
// (stream-K); a CTA streams its units through a shared-memory ring with bulk copies,
// sums them in registers, reduces across its warps and, when the tile is shared with
// other CTAs, the last CTA to finish adds the pieces in CTA order (deterministic) and
// runs the epilogue.
#include <algorithm>

#include "comm.cuh"
#include "tma.cuh"

namespace pyre {
namespace ffn {

#ifndef PYRE_GEMV_CONSUMER_WARPS
#define PYRE_GEMV_CONSUMER_WARPS 8
#endif
constexpr int kTileN = 256;           // output columns per tile
constexpr int kUnitRows = 32;         // input rows per work unit = one pipeline stage
constexpr int kConsumerWarps = PYRE_GEMV_CONSUMER_WARPS;
constexpr int kPasses = kUnitRows / (2 * kConsumerWarps);   // row pairs per warp per unit
static_assert(kPasses >= 1 && kPasses * 2 * kConsumerWarps == kUnitRows, "consumer warps must divide 16");
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;   // + one producer warp
constexpr int kMaxGrid = 1024;
constexpr int kCounterWords = 2048;         // word kCounterWords-1 is the status word
constexpr int kMaxTiles = kCounterWords - 1;

enum Epi : int { EPI_SILU_MUL = 0, EPI_SILU = 1, EPI_STORE = 2, EPI_TP = 3 };

struct alignas(64) Params {
  CUtensorMap tx;            // activations [T, K], box T x 32
  const void* x;
  const int8_t* q0;          // tiled q [tiles, K, 256]; gate (NMAT == 2) or the single matrix
  const void* s0;            // tiled scales [tiles, K, 8]
  const int8_t* q1;          // up (NMAT == 2)
  const void* s1;
  int K, N, T;
  int tiles;                 // ceil(N / kTileN)
  int upt;                   // units per tile = ceil(K / kUnitRows)
  int64_t total_units;       // tiles * upt
  int pmax;                  // piece slots per tile in ws
  int64_t ws_cap;            // bytes of ws (after the counters)
  float* ws;                 // [tiles, pmax, NMAT, T, kTileN]
  unsigned int* counters;    // [tiles], zero between calls
  int* status;               // device status word (bounded waits)
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

// CTA whose unit range [c*U/G, (c+1)*U/G) contains unit index x.
__host__ __device__ __forceinline__ int cta_of_unit(int64_t x, int64_t U, int G) {
  return static_cast<int>(((x + 1) * G - 1) / U);
}

__device__ __forceinline__ void consumer_sync() { named_bar(1, kConsumers); }

// Epilogue over the finished tile sums held in shared memory `fin` ([NMAT][T][kTileN]).
// Runs on the consumer threads only (tid in [0, kConsumers)).
template <int T, int NMAT, int EPI>
__device__ void tile_epilogue(const Params& p, int tile, const float* fin, uint32_t epoch, int tid) {
  const int col_base = tile * kTileN;
  if constexpr (EPI == EPI_TP) {
    const comm::DevComm& c = p.comm;
    const int slot = epoch & 1u;
    const int n = T * kTileN;
    // push this rank's tile partial into every rank's receive slot (self included)
    for (int peer = 0; peer < c.world; ++peer) {
      float* dst = comm::fused_slot(c, peer, slot, c.rank) + static_cast<int64_t>(tile) * n;
      for (int i = tid; i < n; i += kConsumers) dst[i] = fin[i];
    }
    __threadfence_system();
    consumer_sync();
    if (tid < c.world) st_release_sys(comm::fused_flag(c, tid, slot, c.rank, tile), epoch);
    if (tid < c.world) {
      if (!wait_flag_eq(comm::fused_flag(c, c.rank, slot, tid, tile), epoch, c.timeout_ns))
        atomicExch(c.status, PYRE_ETIMEOUT);
    }
    consumer_sync();
    for (int i = tid; i < n; i += kConsumers) {
      const int t = i / kTileN, cc = i % kTileN;
      const int col = col_base + cc;
      if (col >= p.N) continue;
      float acc = 0.f;
      for (int src = 0; src < c.world; ++src)
        acc += __ldcg(comm::fused_slot(c, c.rank, slot, src) + static_cast<int64_t>(tile) * n + i);
      store_out(p, t, col, acc);
    }
  } else {
    for (int i = tid; i < T * kTileN; i += kConsumers) {
      const int t = i / kTileN, cc = i % kTileN;
      const int col = col_base + cc;
      if (col >= p.N) continue;
      float v;
      if constexpr (EPI == EPI_SILU_MUL) {
        v = silu_f32(fin[i]) * fin[T * kTileN + i];
      } else if constexpr (EPI == EPI_SILU) {
        v = silu_f32(fin[i]);
      } else {
        v = fin[i];
      }
      store_out(p, t, col, v);
    }
  }
}

#ifndef PYRE_GEMV_STAGES
#define PYRE_GEMV_STAGES 4
#endif
template <int T, int NMAT, typename XT, typename ST>
struct GemvCfg {
  // T <= 2: two CTAs per SM with a 4-stage ring each; T >= 3 (larger reduction buffers):
  // one CTA per SM with 5 stages.
  static constexpr int kCtasPerSm = (T <= 2) ? 2 : 1;
  static constexpr int kStages = (T <= 2) ? PYRE_GEMV_STAGES : 5;
  static constexpr int kQBytes = kUnitRows * kTileN;                       // 8 KB per matrix
  static constexpr int kSBytes = kUnitRows * 8 * static_cast<int>(sizeof(ST));   // 8 scale columns
  static constexpr int kXBytes = T * kUnitRows * static_cast<int>(sizeof(XT));
  static constexpr int kTxBytes = NMAT * (kQBytes + kSBytes) + kXBytes;
  static constexpr int kStageBytes = (kTxBytes + 127) / 128 * 128;
  static constexpr int kRedFloats = kConsumerWarps * NMAT * T * kTileN;
  static constexpr int kFinFloats = NMAT * T * kTileN;
  static constexpr int kSmemBytes = kStages * kStageBytes + (kRedFloats + kFinFloats) * 4 + 2 * kStages * 8 + 16;
};

// Decode GEMV over Q8_0 weights, TMA-fed.
//   warp 8 (producer): lane 0 streams, per unit, the int8 tile [32 rows x 256 cols] and
//     its scale tile [32 x 8] of each matrix plus the activation slice [T x 32] into an
//     mbarrier ring of kStages stages.
//   warps 0-7 (consumers): lane (rs, cc) owns columns 16cc..16cc+15 and rows
//     2*warp + rs (+16) of each unit; int8 -> f32 by byte-permute, scale folded into the
//     activation, packed f32x2 FMA into f32 accumulators.
// The (tile, unit) space is split evenly over the grid (stream-K); CTAs that share a
// tile add their pieces in CTA order, so the result is deterministic.
template <int T, int NMAT, int EPI, typename XT, typename ST>
__global__ void __launch_bounds__(kThreads, (GemvCfg<T, NMAT, XT, ST>::kCtasPerSm))
q80_gemv_kernel(const __grid_constant__ Params p) {
  using C = GemvCfg<T, NMAT, XT, ST>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  float* red = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  float* fin = red + C::kRedFloats;
  uint64_t* full = reinterpret_cast<uint64_t*>(fin + C::kFinFloats);
  uint64_t* empty = full + C::kStages;
  int* s_last = reinterpret_cast<int*>(empty + C::kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int c = blockIdx.x;
  const int64_t U = p.total_units;
  const int64_t u_begin = (static_cast<int64_t>(c) * U) / G;
  const int64_t u_end = (static_cast<int64_t>(c + 1) * U) / G;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t epoch = 0;
  if constexpr (EPI == EPI_TP) epoch = comm::epoch_begin(p.comm);

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&p.tx);
      const int8_t* qm[2] = {p.q0, p.q1};
      const uint8_t* sm[2] = {static_cast<const uint8_t*>(p.s0), static_cast<const uint8_t*>(p.s1)};
      int s = 0;
      uint32_t ph = 0;
      for (int64_t u = u_begin; u < u_end; ++u) {
        const int tile = static_cast<int>(u / p.upt);
        const int k0 = static_cast<int>(u - static_cast<int64_t>(tile) * p.upt) * kUnitRows;
        mbar_wait(&empty[s], ph ^ 1u, p.status);
        uint8_t* st = stages + s * C::kStageBytes;
        mbar_arrive_expect_tx(&full[s], C::kTxBytes);
        const int64_t row0 = static_cast<int64_t>(tile) * p.K + k0;
        for (int m = 0; m < NMAT; ++m) {
          bulk_load(st + m * C::kQBytes, qm[m] + row0 * kTileN, C::kQBytes, &full[s]);
          bulk_load(st + NMAT * C::kQBytes + m * C::kSBytes, sm[m] + row0 * (C::kSBytes / kUnitRows), C::kSBytes,
                    &full[s]);
        }
        tma_load_2d(st + NMAT * (C::kQBytes + C::kSBytes), &p.tx, k0, 0, &full[s]);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else {
    // ---------------- consumers ----------------
    const int tid = threadIdx.x;
    const int rs = lane >> 4;
    const int cc = lane & 15;
    int s = 0;
    uint32_t ph = 0;
    int64_t u = u_begin;
    while (u < u_end) {
      const int tile = static_cast<int>(u / p.upt);
      const int64_t tile_u0 = static_cast<int64_t>(tile) * p.upt;
      const int64_t seg_end = min(u_end, tile_u0 + p.upt);

      float2 acc[NMAT][T][8];
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int t = 0; t < T; ++t)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[m][t][i] = make_float2(0.f, 0.f);

      for (; u < seg_end; ++u) {
        mbar_wait(&full[s], ph, p.status);
        const uint8_t* st = stages + s * C::kStageBytes;
        const ST* ss = reinterpret_cast<const ST*>(st + NMAT * C::kQBytes);
        const XT* xs = reinterpret_cast<const XT*>(st + NMAT * (C::kQBytes + C::kSBytes));
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
          const int r = pass * (2 * kConsumerWarps) + warp * 2 + rs;
          float xv[T];
#pragma unroll
          for (int t = 0; t < T; ++t) xv[t] = to_f32(xs[t * kUnitRows + r]);
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const float sc = to_f32(ss[m * (C::kSBytes / sizeof(ST)) + r * 8 + (cc >> 1)]);
            const int4 w = *reinterpret_cast<const int4*>(st + m * C::kQBytes + r * kTileN + cc * 16);
            const uint32_t words[4] = {static_cast<uint32_t>(w.x), static_cast<uint32_t>(w.y),
                                       static_cast<uint32_t>(w.z), static_cast<uint32_t>(w.w)};
            float2 a2[T];
#pragma unroll
            for (int t = 0; t < T; ++t) {
              const float a = xv[t] * sc;
              a2[t] = make_float2(a, a);
            }
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const uint32_t uu = words[wi] ^ 0x80808080u;
              const float2 magic = make_float2(-8388736.0f, -8388736.0f);
              const float2 f01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(uu, 0x4B000000u, 0x7540u)),
                                                        __uint_as_float(__byte_perm(uu, 0x4B000000u, 0x7541u))),
                                            magic);
              const float2 f23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(uu, 0x4B000000u, 0x7542u)),
                                                        __uint_as_float(__byte_perm(uu, 0x4B000000u, 0x7543u))),
                                            magic);
#pragma unroll
              for (int t = 0; t < T; ++t) {
                acc[m][t][wi * 2] = __ffma2_rn(a2[t], f01, acc[m][t][wi * 2]);
                acc[m][t][wi * 2 + 1] = __ffma2_rn(a2[t], f23, acc[m][t][wi * 2 + 1]);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }

      // reduce the two row lanes of each column chunk, then across warps
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int t = 0; t < T; ++t)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float2 v = acc[m][t][i];
            v.x += __shfl_xor_sync(0xffffffffu, v.x, 16);
            v.y += __shfl_xor_sync(0xffffffffu, v.y, 16);
            acc[m][t][i] = v;
          }
      if (rs == 0) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
          for (int t = 0; t < T; ++t) {
            float4* dst = reinterpret_cast<float4*>(red + static_cast<int64_t>(warp) * NMAT * T * kTileN +
                                                    (m * T + t) * kTileN + cc * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_float4(acc[m][t][2 * i].x, acc[m][t][2 * i].y, acc[m][t][2 * i + 1].x,
                                   acc[m][t][2 * i + 1].y);
          }
      }
      consumer_sync();
      for (int i = tid; i < NMAT * T * kTileN; i += kConsumers) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) v += red[w * NMAT * T * kTileN + i];
        fin[i] = v;
      }
      consumer_sync();

      const int cf = cta_of_unit(tile_u0, U, G);
      const int cl = cta_of_unit(tile_u0 + p.upt - 1, U, G);
      if (cf == cl) {
        tile_epilogue<T, NMAT, EPI>(p, tile, fin, epoch, tid);
      } else {
        const int piece = c - cf;
        const int np = cl - cf + 1;
        float* slot = p.ws + (static_cast<int64_t>(tile) * p.pmax + piece) * (NMAT * T * kTileN);
        for (int i = tid; i < NMAT * T * kTileN; i += kConsumers) __stcg(slot + i, fin[i]);
        __threadfence();
        consumer_sync();
        if (tid == 0) {
          const unsigned prev = atomicAdd(p.counters + tile, 1u);
          *s_last = (prev == static_cast<unsigned>(np - 1));
        }
        consumer_sync();
        if (*s_last) {
          __threadfence();
          const float* base = p.ws + static_cast<int64_t>(tile) * p.pmax * (NMAT * T * kTileN);
          for (int i = tid; i < NMAT * T * kTileN; i += kConsumers) {
            // all piece loads in flight at once, then summed in piece order
            float v = 0.f;
            for (int pc0 = 0; pc0 < np; pc0 += 16) {
              float pv[16];
#pragma unroll
              for (int j = 0; j < 16; ++j)
                pv[j] = (pc0 + j < np) ? __ldcg(base + static_cast<int64_t>(pc0 + j) * (NMAT * T * kTileN) + i) : 0.f;
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (pc0 + j < np) v += pv[j];
            }
            fin[i] = v;
          }
          consumer_sync();
          tile_epilogue<T, NMAT, EPI>(p, tile, fin, epoch, tid);
          if (tid == 0) p.counters[tile] = 0u;
        }
      }
      consumer_sync();
    }
  }
  __syncthreads();
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
        if (k < p.K && n < p.N) {
          const int64_t row = static_cast<int64_t>(n / kTileN) * p.K + k;
          w = static_cast<float>(qm[m][row * kTileN + (n % kTileN)]) *
              ld_scale<ST>(sm[m], row * 8 + ((n % kTileN) >> 5));
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
      store_out(p, t, n, v);
    }
  }
}

// ---- host side ------------------------------------------------------------------------

int tiles_of(int N) { return (N + kTileN - 1) / kTileN; }

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
int64_t gemv_ws_bytes(int T, int N, int nmat) {
  const int tiles = tiles_of(N);
  const int64_t pmax = (kMaxGrid + tiles - 1) / tiles + 1;
  return static_cast<int64_t>(tiles) * pmax * nmat * T * kTileN * 4;
}

constexpr int64_t kCounterBytes = kCounterWords * 4;

template <typename XT>
CUtensorMapDataType tma_dtype();
template <>
CUtensorMapDataType tma_dtype<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <>
CUtensorMapDataType tma_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <>
CUtensorMapDataType tma_dtype<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }

template <int T, int NMAT, int EPI, typename XT, typename ST>
int launch_gemv(Params p, cudaStream_t s) {
  using C = GemvCfg<T, NMAT, XT, ST>;
  auto kern = q80_gemv_kernel<T, NMAT, EPI, XT, ST>;
  static bool attr_set[64] = {};  // per instantiation and device
  int dev = 0;
  PYRE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    PYRE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  int rc = make_tmap_2d(&p.tx, p.x, tma_dtype<XT>(), sizeof(XT), p.T, p.K, static_cast<uint64_t>(p.K) * sizeof(XT),
                        T, kUnitRows);
  if (rc) return rc;
  // every CTA must be co-resident (the tensor-parallel epilogue waits on peers), so the
  // grid never exceeds what the occupancy calculator says fits at once
  int occ = 0;
  PYRE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, C::kSmemBytes));
  if (occ < 1) return set_error(PYRE_ECUDA, "q80_gemv: kernel does not fit on an SM");
  if (occ > C::kCtasPerSm) occ = C::kCtasPerSm;
  int64_t g = static_cast<int64_t>(occ) * sm_count();
  if (g > kMaxGrid) g = kMaxGrid;
  if (g > p.total_units) g = p.total_units;
  const int G = static_cast<int>(g < 1 ? 1 : g);
  p.pmax = pmax_for(p.tiles, p.upt, G);
  if (static_cast<int64_t>(p.tiles) * p.pmax * NMAT * T * kTileN * 4 > p.ws_cap)
    return set_error(PYRE_ENOMEM, "q80_gemv: stream-K workspace too small for this grid");
  kern<<<G, kThreads, C::kSmemBytes, s>>>(p);
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
  PYRE_CHECK_ARG(T > PYRE_FUSED_REDUCE_MAX_T || K % 32 == 0, f + ": the input dim must be a multiple of 32");
  PYRE_CHECK_ARG(tiles_of(N) <= kMaxTiles, f + ": output width too large");
  PYRE_CHECK_ARG(T > PYRE_FUSED_REDUCE_MAX_T || (static_cast<int64_t>(K) * (x_dtype == PYRE_BF16 ? 2 : 4)) % 16 == 0,
                 f + ": activation rows must be 16-byte multiples");
  PYRE_CHECK_ARG(ws != nullptr || T > PYRE_FUSED_REDUCE_MAX_T, f + ": null workspace");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(ws) % 16 == 0, f + ": workspace must be 16-byte aligned");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(x) % 16 == 0, f + ": activations must be 16-byte aligned");
  PYRE_CHECK_ARG(ws_bytes >= 0, f + ": negative workspace size");
  return PYRE_OK;
}

int64_t ws_need(int T, int N, int nmat) {
  if (T > PYRE_FUSED_REDUCE_MAX_T) return 0;
  return kCounterBytes + gemv_ws_bytes(T, N, nmat);
}

}  // namespace ffn
}  // namespace pyre

using namespace pyre;
using namespace pyre::ffn;

extern "C" int pyre_ffn_workspace_bytes(int T, int H, int W, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_ffn_workspace_bytes: null bytes");
  PYRE_CHECK_ARG(T >= 1 && H >= 1 && W >= 1, "pyre_ffn_workspace_bytes: sizes must be positive");
  const int64_t a = ws_need(T, W, 2);   // gate/up: K = H, N = W
  const int64_t b = ws_need(T, H, 1);   // down:    K = W, N = H
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
  const int64_t need = ws_need(T, W, gated ? 2 : 1);
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
  p.status = static_cast<int*>(workspace) + (kCounterWords - 1);
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
  const int64_t need = ws_need(T, H, 1);
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
  p.status = static_cast<int*>(workspace) + (kCounterWords - 1);
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
