// Building blocks of the Q8_0 decode GEMV kernels (T <= 4 tokens).
//
// Work decomposition. A [K, N] weight in the column-slab tiled layout is covered by tiles of
// 256 output columns; a tile is covered by units of 32 input rows. One unit of one matrix
// is a contiguous 8 KB int8 run plus 32 x 8 scales; a pipeline stage holds one unit of each
// matrix the kernel multiplies plus the [T x 32] activation slice.
//
// Consumer mapping. 8 consumer warps; lane (rs, cc) owns columns 16cc..16cc+15 and, for
// pass p, row p*16 + 2*warp + rs of the unit. int8 -> f32 is exact: the byte b becomes the
// float 0x4B0000uu (2^23 + u, u = b ^ 0x80) minus 2^23 + 128, done for pairs with one
// byte-permute each and one packed f32x2 add; the block scale is folded into the
// activation and the products accumulate with packed f32x2 FMA in f32.
#pragma once

#include "comm.cuh"
#include "tma.cuh"

namespace pyre {
namespace gemv {

#ifndef PYRE_GEMV_CONSUMER_WARPS
#define PYRE_GEMV_CONSUMER_WARPS 8
#endif
constexpr int kTileN = 256;            // output columns per tile (= slab width)
constexpr int kUnitRows = 32;          // input rows per unit
constexpr int kConsumerWarps = PYRE_GEMV_CONSUMER_WARPS;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;   // + one producer warp
constexpr int kPasses = kUnitRows / (2 * kConsumerWarps);
static_assert(kPasses >= 1 && kPasses * 2 * kConsumerWarps == kUnitRows, "consumer warps must divide 16");
constexpr int kMaxGrid = 1024;
constexpr int kMaxTiles = 2048;        // N <= 524288

// Workspace header shared by all FFN entry points (bytes): epoch, done counter, status word,
// then three arrays of kMaxTiles u32 (counters A, counters B, per-slab ready flags).
constexpr int64_t kHdrEpoch = 0;
constexpr int64_t kHdrDone = 4;
constexpr int64_t kHdrStatus = 8;
constexpr int64_t kHdrCntA = 1024;
constexpr int64_t kHdrCntB = kHdrCntA + kMaxTiles * 4;
constexpr int64_t kHdrReady = kHdrCntB + kMaxTiles * 4;
constexpr int64_t kHeaderBytes = 32768;
static_assert(kHdrReady + kMaxTiles * 4 <= kHeaderBytes, "workspace header overflow");

template <int T, int NMAT, typename XT, typename ST>
struct StageLayout {
  static constexpr int kQBytes = kUnitRows * kTileN;                                 // 8 KB
  static constexpr int kSBytes = kUnitRows * 8 * static_cast<int>(sizeof(ST));
  static constexpr int kXBytes = T * kUnitRows * static_cast<int>(sizeof(XT));
  static constexpr int kSOff = NMAT * kQBytes;
  static constexpr int kXOff = NMAT * (kQBytes + kSBytes);
  static constexpr int kTxBytes = kXOff + kXBytes;
  static constexpr int kBytes = (kTxBytes + 127) / 128 * 128;
};

__device__ __forceinline__ float silu_f32(float g) { return __fdiv_rn(g, 1.0f + expf(-g)); }

template <int NMAT, int T>
__device__ __forceinline__ void zero_acc(float2 (&acc)[NMAT][T][8]) {
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int t = 0; t < T; ++t)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[m][t][i] = make_float2(0.f, 0.f);
}

// Accumulates one unit held in stage memory `st` into acc.
template <int T, int NMAT, typename XT, typename ST>
__device__ __forceinline__ void consume_unit(const uint8_t* st, float2 (&acc)[NMAT][T][8], int warp, int rs, int cc) {
  using L = StageLayout<T, NMAT, XT, ST>;
  const ST* ss = reinterpret_cast<const ST*>(st + L::kSOff);
  const XT* xs = reinterpret_cast<const XT*>(st + L::kXOff);
#pragma unroll
  for (int pass = 0; pass < kPasses; ++pass) {
    const int r = pass * (2 * kConsumerWarps) + warp * 2 + rs;
    float xv[T];
#pragma unroll
    for (int t = 0; t < T; ++t) xv[t] = to_f32(xs[t * kUnitRows + r]);
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const float sc = to_f32(ss[m * (L::kSBytes / static_cast<int>(sizeof(ST))) + r * 8 + (cc >> 1)]);
      const int4 w = *reinterpret_cast<const int4*>(st + m * L::kQBytes + r * kTileN + cc * 16);
      const uint32_t words[4] = {static_cast<uint32_t>(w.x), static_cast<uint32_t>(w.y), static_cast<uint32_t>(w.z),
                                 static_cast<uint32_t>(w.w)};
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
}

__device__ __forceinline__ void consumer_sync() { named_bar(1, kConsumers); }

// Sums acc over the two row lanes and all consumer warps into fin[NMAT][T][kTileN].
// red: shared scratch of kConsumerWarps * NMAT * T * kTileN floats.
template <int T, int NMAT>
__device__ __forceinline__ void reduce_tile(float2 (&acc)[NMAT][T][8], float* red, float* fin, int warp, int rs,
                                            int cc, int tid) {
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
          dst[i] = make_float4(acc[m][t][2 * i].x, acc[m][t][2 * i].y, acc[m][t][2 * i + 1].x, acc[m][t][2 * i + 1].y);
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
}

// CTA whose unit range [c*U/G, (c+1)*U/G) contains unit index x.
__host__ __device__ __forceinline__ int cta_of_unit(int64_t x, int64_t U, int G) {
  return static_cast<int>(((x + 1) * G - 1) / U);
}

// Stream-K fix-up of a tile shared by CTAs cf..cl: every CTA stores its piece; the last to
// arrive adds all pieces in piece (= CTA) order into fin and returns true. A CTA that owns
// the whole tile returns true at once. ws holds [tiles, pmax, NMAT*T*kTileN] floats.
template <int T, int NMAT>
__device__ __forceinline__ bool fixup_tile(float* fin, float* ws, unsigned int* counters, int pmax, int tile, int c,
                                           int cf, int cl, int* s_last, int tid) {
  if (cf == cl) return true;
  constexpr int kItems = NMAT * T * kTileN;
  const int piece = c - cf;
  const int np = cl - cf + 1;
  float* slot = ws + (static_cast<int64_t>(tile) * pmax + piece) * kItems;
  for (int i = tid; i < kItems; i += kConsumers) __stcg(slot + i, fin[i]);
  __threadfence();
  consumer_sync();
  if (tid == 0) {
    const unsigned prev = atomicAdd(counters + tile, 1u);
    *s_last = (prev == static_cast<unsigned>(np - 1));
  }
  consumer_sync();
  if (!*s_last) return false;
  __threadfence();
  const float* base = ws + static_cast<int64_t>(tile) * pmax * kItems;
  for (int i = tid; i < kItems; i += kConsumers) {
    // all piece loads in flight at once, then summed in piece order
    float v = 0.f;
    for (int pc0 = 0; pc0 < np; pc0 += 16) {
      float pv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        pv[j] = (pc0 + j < np) ? __ldcg(base + static_cast<int64_t>(pc0 + j) * kItems + i) : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (pc0 + j < np) v += pv[j];
    }
    fin[i] = v;
  }
  consumer_sync();
  if (tid == 0) counters[tile] = 0u;
  return true;
}

// Largest number of pieces any tile has for a grid of G CTAs.
inline int pmax_for(int tiles, int upt, int G) {
  const int64_t U = static_cast<int64_t>(tiles) * upt;
  int pm = 1;
  for (int t = 0; t < tiles; ++t) {
    const int64_t u0 = static_cast<int64_t>(t) * upt;
    const int np = cta_of_unit(u0 + upt - 1, U, G) - cta_of_unit(u0, U, G) + 1;
    pm = pm > np ? pm : np;
  }
  return pm;
}

inline int tiles_of(int N) { return (N + kTileN - 1) / kTileN; }

// Upper bound of a piece region for any grid <= kMaxGrid.
inline int64_t pieces_bytes(int T, int N, int nmat) {
  const int tiles = tiles_of(N);
  const int64_t pmax = (kMaxGrid + tiles - 1) / tiles + 1;
  return static_cast<int64_t>(tiles) * pmax * nmat * T * kTileN * 4;
}

template <typename XT>
inline CUtensorMapDataType tma_dtype();
template <>
inline CUtensorMapDataType tma_dtype<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <>
inline CUtensorMapDataType tma_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }

}  // namespace gemv
}  // namespace pyre
