// Tensor-core (tcgen05) Q8_0 GEMM for the FFN at T > 4 tokens (prefill):
//   gate/up:  h[T, W]   = silu(x @ Wg) * (x @ Wu)   (or silu(x @ Wu))     NMAT = 2 (or 1)
//   down:     out[T, H] = h @ Wd                                            NMAT = 1
// Reference semantics: src/ffn/builder.py:37-45 (the graph), src/orchestrator/quantizer.py:29-40
// (Q8_0 dequantization, done here in shared memory), pyre_kernels.mojo:121-129 (silu).
//
// CTA tile: 128 tokens x 256 output columns (one packed slab) per matrix, the whole K.
// One packed weight block (R = 32 rows of a gate/up pair, or 64 rows of one matrix) is one
// pipeline stage; 3 stages. Per stage:
//   producer warp   : TMA of the [128 x R] bf16 activation tile (K-major, R*2-byte swizzle)
//                     + one bulk copy of the ~17 KB int8 block;
//   dequant warps   : int8 * scale -> bf16 into the B operand (MN-major, 128-byte swizzle),
//                     the layout the MMA reads directly;
//   MMA warp (1 thr): tcgen05.mma M=128 N=256 K=16, R/16 per matrix, accumulators in tensor
//                     memory (256 columns per matrix); tcgen05.commit frees the stage.
// The dequant warps then read the accumulators (tcgen05.ld) and run the epilogue. Bulk
// copies and TMA loads only; no cluster multicast. Every mbarrier wait is bounded.
//
// Activations must be bf16 (the tensor-core operand type); f32 activations are converted
// into the workspace first. Weights are bf16(q * scale) in the MMA (relative rounding
// 2^-9 per weight), accumulated in f32.
#include <algorithm>

#include "ffn_internal.cuh"
#include "umma.cuh"

namespace pyre {
namespace tc {

using namespace gemv;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kStages = 3;
constexpr int kThreads = 192;      // warp 0 producer + TMEM allocator, warp 1 MMA, warps 2-5 dequant/epilogue
constexpr int kDequant = 128;

template <int NMAT, typename ST>
struct Cfg {
  static constexpr int R = NMAT == 2 ? kUnitRowsPair : kUnitRowsSingle;   // K per stage
  static constexpr int kABytes = kBM * R * 2;                              // bf16 activation tile
  static constexpr int kBMatBytes = kBN * R * 2;                           // bf16 B per matrix
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
  CUtensorMap ta;           // activations [T, K] bf16, box 128 x R
  const uint8_t* w;         // packed weights
  int T, K, N;
  int tiles, upt, mtiles;
  void* out;                // [T, N]
  int out_bf16;
  int* status;
};

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

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int slab = blockIdx.x / p.mtiles;
  const int mt = blockIdx.x - slab * p.mtiles;
  const int m0 = mt * kBM;
  const int nk = p.upt;

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
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % kStages;
        const uint32_t ph = (kt / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) break;
        uint8_t* st = smem + s * C::kStageBytes;
        mbar_arrive_expect_tx(&full[s], C::kABytes + C::kWBytes);
        tma_load_2d(st + C::kAOff, &p.ta, kt * C::R, m0, &full[s]);
        bulk_load(st + C::kWOff, wslab + static_cast<int64_t>(kt) * C::kWBytes, C::kWBytes, &full[s]);
        issued = kt + 1;
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (int kt = issued - kStages < 0 ? 0 : issued - kStages; kt < issued; ++kt)
        mbar_wait(&full[kt % kStages], (kt / kStages) & 1u, nullptr, 500000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma::idesc_bf16_f32_kmaj_mnmaj<kBM, kBN>();
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % kStages;
        const uint32_t ph = (kt / kStages) & 1u;
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
            umma::mma_bf16(tmem + m * kBN, ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
          }
        }
        umma::mma_commit(&empty[s]);   // the stage is free once these MMAs have read it
      }
      umma::mma_commit(accfull);       // all MMAs (also after an early stop) have completed
    }
  } else {
    // ---------------- dequant, then epilogue ----------------
    const int dt = threadIdx.x - 64;
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % kStages;
      const uint32_t ph = (kt / kStages) & 1u;
      if (!mbar_wait(&full[s], ph, p.status)) break;
      uint8_t* st = smem + s * C::kStageBytes;
      const uint8_t* wq = st + C::kWOff;
      const ST* ws = reinterpret_cast<const ST*>(st + C::kWOff + NMAT * C::R * kTileN);
      uint8_t* bt = st + C::kBOff;
      constexpr int kGroups = NMAT * C::R * 32;   // 8-column groups per stage
#pragma unroll 4
      for (int g = dt; g < kGroups; g += kDequant) {
        const int m = g / (C::R * 32);
        const int rem = g - m * (C::R * 32);
        const int k = rem >> 5;
        const int n8 = rem & 31;
        const uint2 q = *reinterpret_cast<const uint2*>(wq + m * C::R * kTileN + k * kTileN + n8 * 8);
        const float sc = to_f32(ws[m * C::R * 8 + k * 8 + (n8 >> 2)]);
        const uint32_t w0 = q.x ^ 0x80808080u, w1 = q.y ^ 0x80808080u;
        float f[8];
        f[0] = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7540u)) - 8388736.0f;
        f[1] = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7541u)) - 8388736.0f;
        f[2] = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7542u)) - 8388736.0f;
        f[3] = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7543u)) - 8388736.0f;
        f[4] = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7540u)) - 8388736.0f;
        f[5] = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7541u)) - 8388736.0f;
        f[6] = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7542u)) - 8388736.0f;
        f[7] = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7543u)) - 8388736.0f;
        uint4 o;
        __nv_bfloat162 b0 = __floats2bfloat162_rn(f[0] * sc, f[1] * sc);
        __nv_bfloat162 b1 = __floats2bfloat162_rn(f[2] * sc, f[3] * sc);
        __nv_bfloat162 b2 = __floats2bfloat162_rn(f[4] * sc, f[5] * sc);
        __nv_bfloat162 b3 = __floats2bfloat162_rn(f[6] * sc, f[7] * sc);
        o.x = *reinterpret_cast<uint32_t*>(&b0);
        o.y = *reinterpret_cast<uint32_t*>(&b1);
        o.z = *reinterpret_cast<uint32_t*>(&b2);
        o.w = *reinterpret_cast<uint32_t*>(&b3);
        *reinterpret_cast<uint4*>(bt + m * C::kBMatBytes + b_offset(n8 * 8, k)) = o;
      }
      umma::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bfull[s]);
    }
    // epilogue: this warp reads TMEM lanes 32*(warp % 4) .. +31 = tile rows
    mbar_wait(accfull, 0, p.status);
    umma::fence_after_sync();
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int t = m0 + row;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    for (int c0 = 0; c0 < kBN; c0 += 16) {
      uint32_t a[16];
      umma::tmem_ld16(trow + c0, a);
      uint32_t b[16];
      if constexpr (NMAT == 2) umma::tmem_ld16(trow + kBN + c0, b);
      umma::tmem_wait_ld();
      if (t >= p.T) continue;
      const int col0 = slab * kTileN + c0;
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float g = __uint_as_float(a[i]);
        if constexpr (EPI == ffn::EPI_SILU_MUL) {
          v[i] = silu_f32(g) * __uint_as_float(b[i]);
        } else if constexpr (EPI == ffn::EPI_SILU) {
          v[i] = silu_f32(g);
        } else {
          v[i] = g;
        }
      }
      const int64_t o = static_cast<int64_t>(t) * p.N + col0;
      if (col0 + 16 <= p.N) {
        if (p.out_bf16) {
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
        for (int i = 0; i < 16 && col0 + i < p.N; ++i) ffn::store_out(p.out, p.out_bf16, p.N, t, col0 + i, v[i]);
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

// f32 -> bf16 conversion of an activation matrix (row-major, n elements).
__global__ void cvt_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n) {
      const float4 v = *reinterpret_cast<const float4*>(src + i);
      __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
      reinterpret_cast<__nv_bfloat162*>(dst + i)[0] = a;
      reinterpret_cast<__nv_bfloat162*>(dst + i)[1] = b;
    } else {
      for (int64_t j = i; j < n; ++j) dst[j] = __float2bfloat16_rn(src[j]);
    }
  }
}

template <int NMAT, int EPI, typename ST>
int launch(Params p, const void* a_bf16, cudaStream_t s) {
  using C = Cfg<NMAT, ST>;
  auto kern = q80_gemm_tc_kernel<NMAT, EPI, ST>;
  int rc = ffn::set_smem_once(kern, C::kSmemBytes);
  if (rc) return rc;
  rc = make_tmap_2d(&p.ta, a_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.T, p.K, static_cast<uint64_t>(p.K) * 2,
                    kBM, C::R, C::R * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  p.upt = (p.K + C::R - 1) / C::R;
  p.tiles = tiles_of(p.N);
  p.mtiles = (p.T + kBM - 1) / kBM;
  const int64_t grid = static_cast<int64_t>(p.tiles) * p.mtiles;
  if (grid > 0x7fffffff) return set_error(PYRE_EINVAL, "q80_gemm_tc_kernel: too many tiles");
  kern<<<static_cast<int>(grid), kThreads, C::kSmemBytes, s>>>(p);
  PYRE_LAUNCH_CHECK("q80_gemm_tc_kernel");
  return PYRE_OK;
}

}  // namespace tc

// Tensor-core GEMM form of the FFN halves for T > 4 (used by ffn.cu).
//   nmat = 2: out = silu(a @ W0) * (a @ W1) (epi EPI_SILU_MUL); nmat = 1: EPI_SILU or EPI_STORE.
// a: [T, K] f32 or bf16; f32 is converted to bf16 in `staging` (>= T*K*2 bytes).
int ffn_gemm_tc(const void* a, int a_dtype, int T, int K, const void* w, int nmat, int epi, int scale_dtype, int N,
                void* out, int out_bf16, void* staging, int64_t staging_bytes, int* status, cudaStream_t s) {
  const void* a_bf16 = a;
  if (a_dtype == PYRE_F32) {
    const int64_t n = static_cast<int64_t>(T) * K;
    if (staging == nullptr || staging_bytes < n * 2)
      return set_error(PYRE_ENOMEM, "FFN GEMM: workspace too small for the bf16 copy of the activations");
    const int64_t blocks = std::min<int64_t>((n / 4 + 255) / 256 + 1, 4096);
    tc::cvt_bf16_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(static_cast<const float*>(a),
                                                                  static_cast<__nv_bfloat16*>(staging), n);
    PYRE_LAUNCH_CHECK("cvt_bf16_kernel");
    a_bf16 = staging;
  }
  PYRE_CHECK_ARG((static_cast<int64_t>(K) * 2) % 16 == 0, "FFN GEMM: activation rows must be 16-byte multiples");
  tc::Params p{};
  p.w = static_cast<const uint8_t*>(w);
  p.T = T;
  p.K = K;
  p.N = N;
  p.out = out;
  p.out_bf16 = out_bf16;
  p.status = status;
  const bool f16s = scale_dtype == PYRE_F16;
  if (nmat == 2)
    return f16s ? tc::launch<2, ffn::EPI_SILU_MUL, __half>(p, a_bf16, s)
                : tc::launch<2, ffn::EPI_SILU_MUL, float>(p, a_bf16, s);
  if (epi == ffn::EPI_SILU)
    return f16s ? tc::launch<1, ffn::EPI_SILU, __half>(p, a_bf16, s) : tc::launch<1, ffn::EPI_SILU, float>(p, a_bf16, s);
  return f16s ? tc::launch<1, ffn::EPI_STORE, __half>(p, a_bf16, s) : tc::launch<1, ffn::EPI_STORE, float>(p, a_bf16, s);
}

}  // namespace pyre
