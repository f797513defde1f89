// Building blocks of the Q8_0 decode GEMV kernels (T <= 4 tokens).
//
// Packed device weight layout. A group of M matrices (M = 1, or M = 2 for gate and up,
// which share [K, N]) is stored as blocks: for every slab of 256 output columns j and every
// unit of R = 64 / M input rows u, one contiguous block
//     [q of matrix 0: R x 256 int8] ... [q of matrix M-1] [scales of matrix 0: R x 8] ...
// in (j, u) order, K padded to a multiple of R and N to a multiple of 256 with zeros. The
// int8 values and scales are exactly the reference's Q8_0 blocks (each scale covers 32
// consecutive output columns of one row). One block is one pipeline stage: the producer
// moves it with a single bulk copy (~17 KB), plus the [T x R] activation slice.
//
// Consumer mapping. 8 consumer warps; lane (rs, cc) owns columns 16cc..16cc+15 and, for
// pass p (R / 16 passes), row p*16 + 2*warp + rs of the unit. int8 -> f32 is exact: the byte b becomes the
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
constexpr int kUnitRowsPair = 32;      // unit rows of a packed gate/up pair
constexpr int kUnitRowsSingle = 64;    // unit rows of a packed single matrix
template <int NMAT>
struct UnitRows {
  static constexpr int value = NMAT == 2 ? kUnitRowsPair : kUnitRowsSingle;
};
constexpr int kConsumerWarps = PYRE_GEMV_CONSUMER_WARPS;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;   // + one producer warp
constexpr int kRowsPerPass = 2 * kConsumerWarps;
static_assert(kUnitRowsPair % kRowsPerPass == 0 && kUnitRowsSingle % kRowsPerPass == 0, "consumer warps must divide 16");
constexpr int kMaxGrid = 1024;
constexpr int kMaxTiles = 2048;        // N <= 524288

// Workspace header shared by all FFN entry points (bytes): epoch, done counter, status word,
// then three arrays of kMaxTiles u32 (counters A, counters B, per-slab ready flags).
constexpr int64_t kHdrEpoch = 0;
constexpr int64_t kHdrDone = 4;
constexpr int64_t kHdrStatus = 8;
constexpr int64_t kHdrNext = 16;       // two u32 chunk counters (dynamic scheduling)
constexpr int64_t kHdrAbCalls = 64;    // u32: one-launch decode FFN calls made on this workspace
constexpr int64_t kHdrCntA = 1024;
constexpr int64_t kHdrCntB = kHdrCntA + kMaxTiles * 4;
constexpr int64_t kHdrReady = kHdrCntB + kMaxTiles * 4;
constexpr int64_t kHeaderBytes = 32768;
static_assert(kHdrReady + kMaxTiles * 4 <= kHeaderBytes, "workspace header overflow");

// One pipeline stage: a packed weight block followed by the activation slice.
template <int T, int NMAT, typename XT, typename ST>
struct StageLayout {
  static constexpr int kRows = UnitRows<NMAT>::value;
  static constexpr int kQBytes = kRows * kTileN;                                     // 16 KB / NMAT
  static constexpr int kSBytes = kRows * 8 * static_cast<int>(sizeof(ST));
  static constexpr int kSOff = NMAT * kQBytes;
  static constexpr int kWBytes = NMAT * (kQBytes + kSBytes);                         // packed block
  static constexpr int kXOff = kWBytes;
  static constexpr int kXBytes = T * kRows * static_cast<int>(sizeof(XT));
  static constexpr int kTxBytes = kXOff + kXBytes;
  static constexpr int kBytes = (kTxBytes + 127) / 128 * 128;
};

// Bytes of one packed block of M matrices with scales of es bytes.
__host__ __device__ __forceinline__ int64_t packed_block_bytes(int M, int es) {
  const int R = M == 2 ? kUnitRowsPair : kUnitRowsSingle;
  return static_cast<int64_t>(M) * R * (kTileN + 8 * es);
}

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
  for (int pass = 0; pass < L::kRows / kRowsPerPass; ++pass) {
    const int r = pass * kRowsPerPass + warp * 2 + rs;
    float xv[T];
#pragma unroll
    for (int t = 0; t < T; ++t) xv[t] = to_f32(xs[t * L::kRows + r]);
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

inline int tiles_of(int N) { return (N + kTileN - 1) / kTileN; }

template <typename XT>
inline CUtensorMapDataType tma_dtype();
template <>
inline CUtensorMapDataType tma_dtype<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <>
inline CUtensorMapDataType tma_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }

}  // namespace gemv
}  // namespace pyre
