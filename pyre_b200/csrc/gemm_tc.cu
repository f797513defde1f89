// Tensor-core (tcgen05) Q8_0 GEMM for the FFN at T > 4 tokens (prefill):
//   gate/up:  h[T, W]   = silu(x @ Wg) * (x @ Wu)   (or silu(x @ Wu))     NMAT = 2 (or 1)
//   down:     out[T, H] = h @ Wd                                            NMAT = 1
// Reference semantics: src/ffn/builder.py:37-45 (the graph), src/orchestrator/quantizer.py:29-40
// (Q8_0 dequantization, done here in shared memory), pyre_kernels.mojo:121-129 (silu).
//
// CTA tile: 128 tokens x 256 output columns (one packed slab) per matrix, the whole K.
// One packed weight block (R = 32 rows of a gate/up pair, or 64 rows of one matrix) is one
// pipeline stage; 3 stages. Per stage:
//   producer warp   : TMA of the [128 x R] f16 activation tile (K-major, R*2-byte swizzle)
//                     + one bulk copy of the ~17 KB int8 block;
//   dequant warps   : int8 * scale -> f16 into the B operand (MN-major, 128-byte swizzle),
//                     the layout the MMA reads directly (byte-permute into f16 1024 + u,
//                     one packed subtract, one packed multiply by the f16 scale);
//   MMA warp (1 thr): tcgen05.mma M=128 N=256 K=16, R/16 per matrix, accumulators in tensor
//                     memory (256 columns per matrix); tcgen05.commit frees the stage.
// The dequant warps then read the accumulators (tcgen05.ld) and run the epilogue. Bulk
// copies and TMA loads only; no cluster multicast. Every mbarrier wait is bounded.
//
// Operands are f16: the weights as f16(q * scale) (q exact in f16, one rounding of the product,
// 2^-11 relative), the activations converted to f16 in the workspace unless they already are
// (the gate/up epilogue writes h in f16 for the down GEMM). Accumulation is f32. A value whose
// magnitude does not fit f16 (>= 65520 after rounding, or not finite) flags PYRE_ERANGE.
#include <algorithm>

#include "ffn_internal.cuh"
#include "umma.cuh"

namespace pyre {
namespace tc {

using namespace gemv;

constexpr int kBM = 128;
constexpr int kMaxSplits = 4;
constexpr int kBN = 256;
constexpr int kStages = 3;
constexpr int kDequantWarps = 8;
constexpr int kDequant = kDequantWarps * 32;
constexpr int kThreads = 64 + kDequant;   // warp 0 producer + TMEM allocator, warp 1 MMA, then dequant/epilogue

template <int NMAT>
constexpr int64_t kPartBytes() { return static_cast<int64_t>(NMAT) * 256 * 128 * 4; }

template <int NMAT, typename ST>
struct Cfg {
  static constexpr int R = NMAT == 2 ? kUnitRowsPair : kUnitRowsSingle;   // K per stage
  static constexpr int kABytes = kBM * R * 2;                              // f16 activation tile
  static constexpr int kBMatBytes = kBN * R * 2;                           // f16 B per matrix
  static constexpr int kBBytes = NMAT * kBMatBytes;
  static constexpr int kWBytes = NMAT * R * kTileN + NMAT * R * 8 * static_cast<int>(sizeof(ST));
  static constexpr int kAOff = 0;
  static constexpr int kBOff = kABytes;                                    // multiple of 1024
  static constexpr int kWOff = kBOff + kBBytes;
  static constexpr int kStageBytes = (kWOff + kWBytes + 1023) / 1024 * 1024;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;   // align slack + barriers
  static constexpr int kTmemCols = NMAT * kBN;
  static constexpr uint32_t kSwizzleA = R * 2 == 128 ? umma::kLayoutSW128 : umma::kLayoutSW64;
  static constexpr uint32_t kSboA = 8 * R * 2;                             // 8 rows of one swizzle atom
  static_assert(kABytes % 1024 == 0 && kBMatBytes % 1024 == 0, "operand tiles must keep 1024-byte alignment");
};

struct Params {
  CUtensorMap ta;           // activations [T, K] f16, box 128 x R
  const uint8_t* w;         // packed weights
  int T, K, N;
  int tiles, upt, mtiles;
  void* out;                // [T, N]
  int out_bf16, out_f16;
  int* status;
  int splits;               // split-K factor (1: no split)
  int64_t partial_cap;      // bytes available at partial
  float* partial;           // [tiles, splits, NMAT, 128 x 256] f32 partial tiles (splits > 1)
  unsigned int* counters;   // [tiles] splits finished, zero between calls
};

// Stores 16 consecutive outputs of row t starting at column col0 (bounds-checked on N).
template <typename P>
__device__ __forceinline__ void store_row16(const P& p, int t, int col0, const float (&v)[16]) {
  const int64_t o = static_cast<int64_t>(t) * p.N + col0;
  if (p.out_f16) {
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 16; ++i) bad |= !(fabsf(v[i]) < 65504.0f);
    if (bad) atomicCAS(p.status, PYRE_OK, PYRE_ERANGE);
  }
  if (col0 + 16 <= p.N) {
    if (p.out_f16) {
      uint4 pk[2];
      uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __half2 hh = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        pw[i] = *reinterpret_cast<uint32_t*>(&hh);
      }
      uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + o);
      dst[0] = pk[0];
      dst[1] = pk[1];
    } else if (p.out_bf16) {
      uint4 pk[2];
      uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __nv_bfloat162 bb = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        pw[i] = *reinterpret_cast<uint32_t*>(&bb);
      }
      uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + o);
      dst[0] = pk[0];
      dst[1] = pk[1];
    } else {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + o);
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
  } else {
    for (int i = 0; i < 16 && col0 + i < p.N; ++i) {
      if (p.out_f16)
        static_cast<__half*>(p.out)[o + i] = __float2half_rn(v[i]);
      else
        ffn::store_out(p.out, p.out_bf16, p.N, t, col0 + i, v[i]);
    }
  }
}

__device__ __forceinline__ __half to_f16(__half v) { return v; }
__device__ __forceinline__ __half to_f16(float v) { return __float2half_rn(v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Byte offset of element (n, k) inside a [256 x R] MN-major, 128-byte-swizzled B tile:
// atoms of 64 columns x 8 rows (1 KB), atoms along N 1 KB apart, 8-row groups 4 KB apart.
__device__ __forceinline__ uint32_t b_offset(int n, int k) {
  return static_cast<uint32_t>((n >> 6) * 1024 + (k >> 3) * 4096 + (k & 7) * 128 + ((((n & 63) >> 3) ^ (k & 7)) << 4));
}

template <int NMAT, int EPI, typename ST>
__global__ void __launch_bounds__(kThreads, 1) q80_gemm_tc_kernel(const __grid_constant__ Params p) {
  using C = Cfg<NMAT, ST>;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB alignment for the swizzled operand tiles
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_u32 & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * C::kStageBytes);
  uint64_t* bfull = full + kStages;
  uint64_t* empty = bfull + kStages;
  uint64_t* accfull = empty + kStages;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accfull + 1);
  int* s_last = reinterpret_cast<int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA order: split (fastest), then token tile, then slab, so the CTAs sharing a weight slab
  // run together and its blocks are read from HBM about once
  const int ks = blockIdx.x % p.splits;
  const int tile = blockIdx.x / p.splits;
  const int slab = tile / p.mtiles;
  const int mt = tile - slab * p.mtiles;
  const int m0 = mt * kBM;
  const int kbeg = static_cast<int>(static_cast<int64_t>(ks) * p.upt / p.splits);
  const int nj = static_cast<int>(static_cast<int64_t>(ks + 1) * p.upt / p.splits) - kbeg;   // k-steps here

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&bfull[i], kDequant / 32);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accfull, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0) {
    umma::tmem_alloc(s_tmem, C::kTmemCols);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&p.ta);
      const uint8_t* wslab = p.w + static_cast<int64_t>(slab) * p.upt * C::kWBytes;
      int issued = 0;
      for (int j = 0; j < nj; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) break;
        uint8_t* st = smem + s * C::kStageBytes;
        const int kt = kbeg + j;
        mbar_arrive_expect_tx(&full[s], C::kABytes + C::kWBytes);
        tma_load_2d(st + C::kAOff, &p.ta, kt * C::R, m0, &full[s]);
        bulk_load(st + C::kWOff, wslab + static_cast<int64_t>(kt) * C::kWBytes, C::kWBytes, &full[s]);
        issued = j + 1;
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (int j = issued - kStages < 0 ? 0 : issued - kStages; j < issued; ++j)
        mbar_wait(&full[j % kStages], (j / kStages) & 1u, nullptr, 500000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma::idesc_f16_f32_kmaj_mnmaj<kBM, kBN>();
      for (int j = 0; j < nj; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1u;
        if (!mbar_wait(&bfull[s], ph, p.status)) break;
        umma::fence_after_sync();
        const uint32_t a_base = smem_u32(smem + s * C::kStageBytes + C::kAOff);
        const uint32_t b_base = smem_u32(smem + s * C::kStageBytes + C::kBOff);
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
#pragma unroll
          for (int kk = 0; kk < C::R / 16; ++kk) {
            const uint64_t ad = umma::smem_desc(a_base + kk * 32, 16, C::kSboA, C::kSwizzleA);
            const uint64_t bd = umma::smem_desc(b_base + m * C::kBMatBytes + kk * 2 * 4096, 1024, 4096,
                                                umma::kLayoutSW128);
            umma::mma_f16(tmem + m * kBN, ad, bd, idesc, (j | kk) != 0 ? 1u : 0u);
          }
        }
        umma::mma_commit(&empty[s]);   // the stage is free once these MMAs have read it
      }
      umma::mma_commit(accfull);       // all MMAs (also after an early stop) have completed
    }
  } else {
    // ---------------- dequant, then epilogue ----------------
    const int dt = threadIdx.x - 64;
    for (int j = 0; j < nj; ++j) {
      const int s = j % kStages;
      const uint32_t ph = (j / kStages) & 1u;
      if (!mbar_wait(&full[s], ph, p.status)) break;
      uint8_t* st = smem + s * C::kStageBytes;
      const uint8_t* wq = st + C::kWOff;
      const ST* ws = reinterpret_cast<const ST*>(st + C::kWOff + NMAT * C::R * kTileN);
      uint8_t* bt = st + C::kBOff;
      constexpr int kGroups = NMAT * C::R * 32;   // 8-column groups per stage
#pragma unroll 2
      for (int g = dt; g < kGroups; g += kDequant) {
        const int m = g / (C::R * 32);
        const int rem = g - m * (C::R * 32);
        const int k = rem >> 5;
        const int n8 = rem & 31;
        const uint2 q = *reinterpret_cast<const uint2*>(wq + m * C::R * kTileN + k * kTileN + n8 * 8);
        const __half2 sc = __half2half2(to_f16(ws[m * C::R * 8 + k * 8 + (n8 >> 2)]));
        // byte b (offset by 128) -> f16 1024 + b -> minus 1152 = the int8 value, exactly
        const uint32_t w0 = q.x ^ 0x80808080u, w1 = q.y ^ 0x80808080u;
        const __half2 k1152 = __half2half2(__ushort_as_half(0x6480u));
        uint4 o;
        o.x = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w0, 0x64646464u, 0x4140u)), k1152), sc));
        o.y = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w0, 0x64646464u, 0x4342u)), k1152), sc));
        o.z = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w1, 0x64646464u, 0x4140u)), k1152), sc));
        o.w = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w1, 0x64646464u, 0x4342u)), k1152), sc));
        *reinterpret_cast<uint4*>(bt + m * C::kBMatBytes + b_offset(n8 * 8, k)) = o;
      }
      umma::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bfull[s]);
    }
    // epilogue: this warp reads TMEM lanes 32*(warp % 4) .. +31 = tile rows
    mbar_wait(accfull, 0, p.status);
    umma::fence_after_sync();
    // warps 2..9: TMEM lane quarter = warp % 4, column half = (warp - 2) / 4
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int t = m0 + row;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr int kColsPerWarp = kBN * 4 / kDequantWarps;
    const int cbeg = ((warp - 2) / 4) * kColsPerWarp;
    // split-K: every split stores its partial tile (thread-major, coalesced); the split that
    // counts last adds them in split order (deterministic) and runs the epilogue
    constexpr int kPartFloats = NMAT * kBN * kBM;
    float* part = p.partial + static_cast<int64_t>(tile) * p.splits * kPartFloats;
    auto part_at = [&](int split, int m, int c0) {
      return part + static_cast<int64_t>(split) * kPartFloats + ((m * (kBN / 16) + c0 / 16) * kBM + row) * 16;
    };
    if (p.splits > 1) {
      for (int c0 = cbeg; c0 < cbeg + kColsPerWarp; c0 += 16) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          uint32_t a[16];
          umma::tmem_ld16(trow + m * kBN + c0, a);
          umma::tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(part_at(ks, m, c0));
#pragma unroll
          for (int i = 0; i < 4; ++i)
            __stcg(dst + i, make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                                        __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3])));
        }
      }
      named_bar(1, kDequant);
      if (dt == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(p.counters + tile, 1u);
        const int last = prev == static_cast<unsigned>(p.splits - 1);
        if (last) {
          __threadfence();
          p.counters[tile] = 0u;
        }
        *s_last = last;
      }
      named_bar(1, kDequant);
    }
    if (p.splits == 1 || *s_last) {
      for (int c0 = cbeg; c0 < cbeg + kColsPerWarp; c0 += 16) {
        float acc[NMAT][16];
        if (p.splits == 1) {
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            uint32_t a[16];
            umma::tmem_ld16(trow + m * kBN + c0, a);
            umma::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[m][i] = __uint_as_float(a[i]);
          }
        } else {
#pragma unroll
          for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[m][i] = 0.f;
          for (int sp = 0; sp < p.splits; ++sp) {
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
              const float4* src = reinterpret_cast<const float4*>(part_at(sp, m, c0));
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 v = __ldcg(src + i);
                acc[m][4 * i] += v.x;
                acc[m][4 * i + 1] += v.y;
                acc[m][4 * i + 2] += v.z;
                acc[m][4 * i + 3] += v.w;
              }
            }
          }
        }
        if (t >= p.T) continue;
        const int col0 = slab * kTileN + c0;
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if constexpr (EPI == ffn::EPI_SILU_MUL) {
            v[i] = silu_f32(acc[0][i]) * acc[NMAT - 1][i];
          } else if constexpr (EPI == ffn::EPI_SILU) {
            v[i] = silu_f32(acc[0][i]);
          } else {
            v[i] = acc[0][i];
          }
        }
        store_row16(p, t, col0, v);
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// f32 or bf16 -> f16 conversion of an activation matrix (row-major, n elements); a value
// that does not fit f16 flags PYRE_ERANGE.
template <typename XT>
__global__ void cvt_f16_kernel(const XT* __restrict__ src, __half* __restrict__ dst, int64_t n, int* status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  bool bad = false;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = to_f32(src[i]);
    bad |= !(fabsf(v) < 65504.0f);
    dst[i] = __float2half_rn(v);
  }
  if (bad) atomicCAS(status, PYRE_OK, PYRE_ERANGE);
}

template <int NMAT, int EPI, typename ST>
int launch(Params p, const void* a_f16, cudaStream_t s) {
  using C = Cfg<NMAT, ST>;
  auto kern = q80_gemm_tc_kernel<NMAT, EPI, ST>;
  int rc = ffn::set_smem_once(kern, C::kSmemBytes);
  if (rc) return rc;
  rc = make_tmap_2d(&p.ta, a_f16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.T, p.K, static_cast<uint64_t>(p.K) * 2,
                    kBM, C::R, C::R * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  p.upt = (p.K + C::R - 1) / C::R;
  p.tiles = tiles_of(p.N);
  p.mtiles = (p.T + kBM - 1) / kBM;
  const int64_t tiles = static_cast<int64_t>(p.tiles) * p.mtiles;
  if (tiles > 0x7fffffff / kMaxSplits) return set_error(PYRE_EINVAL, "q80_gemm_tc_kernel: too many tiles");
  // split K when the tiles alone leave SMs idle (one CTA per SM), keeping >= 8 k-steps per
  // split and the partial tiles within the workspace
  int splits = 1;
  const int sms = sm_count();
  if (tiles < sms && tiles <= kMaxTiles && p.partial != nullptr) {
    splits = static_cast<int>(sms / tiles);
    if (splits > kMaxSplits) splits = kMaxSplits;
    while (splits > 1 && (p.upt / splits < 8 || tiles * splits * kPartBytes<NMAT>() > p.partial_cap)) --splits;
  }
  p.splits = splits;
  kern<<<static_cast<int>(tiles * splits), kThreads, C::kSmemBytes, s>>>(p);
  PYRE_LAUNCH_CHECK("q80_gemm_tc_kernel");
  return PYRE_OK;
}

}  // namespace tc

// Bytes of split-K partial tiles the GEMM over [T, K] x [K, N] may use (0 when the tiles
// alone can fill the GPU): at most 160 CTAs (>= the SM count of a B200) of partial tiles.
int64_t ffn_gemm_partial_bytes(int T, int N, int nmat) {
  const int64_t tiles = static_cast<int64_t>(gemv::tiles_of(N)) * ((T + tc::kBM - 1) / tc::kBM);
  if (tiles >= 160) return 0;
  int64_t ctas = tiles * tc::kMaxSplits;
  if (ctas > 160) ctas = 160;
  return ctas * nmat * 256 * 128 * 4;
}

// Tensor-core GEMM form of the FFN halves for T > 4 (used by ffn.cu).
//   nmat = 2: out = silu(a @ W0) * (a @ W1) (epi EPI_SILU_MUL); nmat = 1: EPI_SILU or EPI_STORE.
// a: [T, K] f32, bf16 or f16; f32 and bf16 are converted to f16 in `staging` (>= T*K*2 bytes).
// out: [T, N] of out_dtype (f32, bf16 or f16).
int ffn_gemm_tc(const void* a, int a_dtype, int T, int K, const void* w, int nmat, int epi, int scale_dtype, int N,
                void* out, int out_dtype, void* staging, int64_t staging_bytes, void* partial, int64_t partial_bytes,
                unsigned int* counters, int* status, cudaStream_t s) {
  const void* a_f16 = a;
  if (a_dtype != PYRE_F16) {
    const int64_t n = static_cast<int64_t>(T) * K;
    if (staging == nullptr || staging_bytes < n * 2)
      return set_error(PYRE_ENOMEM, "FFN GEMM: workspace too small for the f16 copy of the activations");
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * 148));
    if (a_dtype == PYRE_F32)
      tc::cvt_f16_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(a), static_cast<__half*>(staging), n,
                                                       status);
    else
      tc::cvt_f16_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(a),
                                                               static_cast<__half*>(staging), n, status);
    PYRE_LAUNCH_CHECK("cvt_f16_kernel");
    a_f16 = staging;
  }
  PYRE_CHECK_ARG((static_cast<int64_t>(K) * 2) % 16 == 0, "FFN GEMM: activation rows must be 16-byte multiples");
  tc::Params p{};
  p.w = static_cast<const uint8_t*>(w);
  p.T = T;
  p.K = K;
  p.N = N;
  p.out = out;
  p.out_bf16 = out_dtype == PYRE_BF16;
  p.out_f16 = out_dtype == PYRE_F16;
  p.status = status;
  p.partial = static_cast<float*>(partial);
  p.partial_cap = partial_bytes;
  p.counters = counters;
  const bool f16s = scale_dtype == PYRE_F16;
  if (nmat == 2)
    return f16s ? tc::launch<2, ffn::EPI_SILU_MUL, __half>(p, a_f16, s)
                : tc::launch<2, ffn::EPI_SILU_MUL, float>(p, a_f16, s);
  if (epi == ffn::EPI_SILU)
    return f16s ? tc::launch<1, ffn::EPI_SILU, __half>(p, a_f16, s) : tc::launch<1, ffn::EPI_SILU, float>(p, a_f16, s);
  return f16s ? tc::launch<1, ffn::EPI_STORE, __half>(p, a_f16, s) : tc::launch<1, ffn::EPI_STORE, float>(p, a_f16, s);
}

}  // namespace pyre
