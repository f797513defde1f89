// Q8_0 block quantization / dequantization on the device.
//
// Bit-exact restatement of quantize_q80 (src/orchestrator/quantizer.py:11-26):
//   absmax = max |x| over the 32-element block (zero padding past n),
//   absmax == 0 -> 1.0, scale = f32(absmax / 127) (IEEE f32 division),
//   q = clip(round_half_even(f32(x / scale)), -128, 127).
// The kernels use __fdiv_rn and rintf, so the build must not use fast-math.
#include "gemv_common.cuh"

namespace pyre {
namespace {

constexpr int kBlock = 32;

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 f = *reinterpret_cast<const float4*>(p);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xFFFF0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xFFFF0000u);
  }
};

// Eight threads per 32-element block, four elements per thread. VEC selects aligned
// vector loads for the fully in-range quads; the tail always goes element by element.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) q80_quantize_kernel(const T* __restrict__ src, int64_t n,
                                                           int8_t* __restrict__ q,
                                                           float* __restrict__ scale_f32,
                                                           __half* __restrict__ scale_f16,
                                                           int64_t n_quads) {
  const int lane = threadIdx.x & 31;
  // Every thread of a warp runs the same number of iterations (the quad range is padded
  // to whole warps), so the shuffles below always see all 32 lanes.
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t quad = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       quad - lane < n_quads; quad += stride) {
    const bool active = quad < n_quads;
    const int64_t e0 = quad * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (active) {
      if (VEC && e0 + 4 <= n) {
        Vec4<T>::load(src + e0, v);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (e0 + i < n) v[i] = to_f32(src[e0 + i]);
      }
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int off = 1; off < 8; off <<= 1)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (!active) continue;
    if (amax == 0.f) amax = 1.0f;
    const float scale = __fdiv_rn(amax, 127.0f);
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float r = rintf(__fdiv_rn(v[i], scale));
      r = fminf(fmaxf(r, -128.f), 127.f);
      packed |= (static_cast<uint32_t>(static_cast<int32_t>(r)) & 0xFFu) << (8 * i);
    }
    *reinterpret_cast<uint32_t*>(q + e0) = packed;
    if ((lane & 7) == 0) {
      const int64_t b = quad >> 3;
      if (scale_f32) scale_f32[b] = scale;
      if (scale_f16) scale_f16[b] = __float2half_rn(scale);
    }
  }
}

template <typename S>
__global__ void __launch_bounds__(256) q80_dequantize_kernel(const int8_t* __restrict__ q,
                                                             const S* __restrict__ scale,
                                                             int64_t n, float* __restrict__ out) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    out[i] = static_cast<float>(q[i]) * to_f32(scale[i / kBlock]);
  }
}

// Plain reference-orientation Q8_0 (q [K, N] int8, scales [K, N/32]) -> packed blocks
// (see gemv_common.cuh): one thread per 16-byte chunk of a block's int8 part, one per
// scale entry; rows past K and columns past N become zeros.
template <typename S>
__global__ void __launch_bounds__(256) q80_pack_kernel(const int8_t* __restrict__ q0, const S* __restrict__ s0,
                                                       const int8_t* __restrict__ q1, const S* __restrict__ s1, int M,
                                                       int K, int N, int upt, int64_t nblocks,
                                                       uint8_t* __restrict__ out) {
  const int R = M == 2 ? gemv::kUnitRowsPair : gemv::kUnitRowsSingle;
  const int64_t bbytes = gemv::packed_block_bytes(M, sizeof(S));
  const int64_t q_chunks = static_cast<int64_t>(M) * R * (gemv::kTileN / 16);   // per block
  const int64_t s_items = static_cast<int64_t>(M) * R * 8;                        // per block
  const int64_t per_block = q_chunks + s_items;
  const int64_t total = nblocks * per_block;
  const int nsb = N / 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t blk = i / per_block;
    const int64_t w = i - blk * per_block;
    const int j = static_cast<int>(blk / upt);
    const int u = static_cast<int>(blk - static_cast<int64_t>(j) * upt);
    uint8_t* base = out + blk * bbytes;
    if (w < q_chunks) {
      const int m = static_cast<int>(w / (R * 16));
      const int rr = static_cast<int>((w / 16) % R);
      const int c16 = static_cast<int>(w % 16);
      const int k = u * R + rr;
      const int n = j * gemv::kTileN + c16 * 16;
      int4 v = make_int4(0, 0, 0, 0);
      if (k < K && n < N) v = *reinterpret_cast<const int4*>((m == 0 ? q0 : q1) + static_cast<int64_t>(k) * N + n);
      *reinterpret_cast<int4*>(base + (static_cast<int64_t>(m) * R + rr) * gemv::kTileN + c16 * 16) = v;
    } else {
      const int64_t e = w - q_chunks;
      const int m = static_cast<int>(e / (R * 8));
      const int rr = static_cast<int>((e / 8) % R);
      const int sc = static_cast<int>(e % 8);
      const int k = u * R + rr;
      const int bc = j * 8 + sc;
      S v = S(0.f);
      if (k < K && bc < nsb) v = (m == 0 ? s0 : s1)[static_cast<int64_t>(k) * nsb + bc];
      S* sbase = reinterpret_cast<S*>(base + static_cast<int64_t>(M) * R * gemv::kTileN);
      sbase[(static_cast<int64_t>(m) * R + rr) * 8 + sc] = v;
    }
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t want = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace
}  // namespace pyre

extern "C" int pyre_q80_quantize(const void* src, int src_dtype, int64_t n, int8_t* q,
                                 float* scale_f32, uint16_t* scale_f16, void* stream) {
  using namespace pyre;
  PYRE_CHECK_ARG(n >= 0, "pyre_q80_quantize: n must be >= 0");
  if (n == 0) return PYRE_OK;
  PYRE_CHECK_ARG(src != nullptr && q != nullptr, "pyre_q80_quantize: null src or q");
  PYRE_CHECK_ARG(scale_f32 != nullptr || scale_f16 != nullptr,
                 "pyre_q80_quantize: need scale_f32 or scale_f16");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 4 == 0, "pyre_q80_quantize: q must be 4-byte aligned");
  PYRE_CHECK_ARG(src_dtype == PYRE_F32 || src_dtype == PYRE_BF16,
                 "pyre_q80_quantize: src_dtype must be PYRE_F32 or PYRE_BF16");
  const int64_t n_blocks = (n + kBlock - 1) / kBlock;
  const int64_t n_quads = n_blocks * 8;
  const int threads = 256;
  const int grid = grid_for(n_quads, threads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  __half* s16 = reinterpret_cast<__half*>(scale_f16);
  if (src_dtype == PYRE_F32) {
    const float* p = static_cast<const float*>(src);
    if (reinterpret_cast<uintptr_t>(p) % 16 == 0)
      q80_quantize_kernel<float, true><<<grid, threads, 0, s>>>(p, n, q, scale_f32, s16, n_quads);
    else
      q80_quantize_kernel<float, false><<<grid, threads, 0, s>>>(p, n, q, scale_f32, s16, n_quads);
  } else {
    const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(src);
    if (reinterpret_cast<uintptr_t>(p) % 8 == 0)
      q80_quantize_kernel<__nv_bfloat16, true><<<grid, threads, 0, s>>>(p, n, q, scale_f32, s16, n_quads);
    else
      q80_quantize_kernel<__nv_bfloat16, false><<<grid, threads, 0, s>>>(p, n, q, scale_f32, s16, n_quads);
  }
  PYRE_LAUNCH_CHECK("q80_quantize_kernel");
  return PYRE_OK;
}

extern "C" int pyre_q80_dequantize(const int8_t* q, const void* scale, int scale_dtype, int64_t n,
                                   float* out, void* stream) {
  using namespace pyre;
  PYRE_CHECK_ARG(n >= 0, "pyre_q80_dequantize: n must be >= 0");
  if (n == 0) return PYRE_OK;
  PYRE_CHECK_ARG(q != nullptr && scale != nullptr && out != nullptr, "pyre_q80_dequantize: null pointer");
  PYRE_CHECK_ARG(scale_dtype == PYRE_F32 || scale_dtype == PYRE_F16,
                 "pyre_q80_dequantize: scale_dtype must be PYRE_F32 or PYRE_F16");
  const int threads = 256;
  const int grid = grid_for(n, threads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (scale_dtype == PYRE_F32)
    q80_dequantize_kernel<float><<<grid, threads, 0, s>>>(q, static_cast<const float*>(scale), n, out);
  else
    q80_dequantize_kernel<__half><<<grid, threads, 0, s>>>(q, static_cast<const __half*>(scale), n, out);
  PYRE_LAUNCH_CHECK("q80_dequantize_kernel");
  return PYRE_OK;
}

extern "C" int pyre_q80_packed_bytes(int M, int K, int N, int scale_dtype, int64_t* bytes) {
  using namespace pyre;
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_q80_packed_bytes: null bytes");
  PYRE_CHECK_ARG(M == 1 || M == 2, "pyre_q80_packed_bytes: M must be 1 or 2");
  PYRE_CHECK_ARG(K >= 1 && N >= 32 && N % 32 == 0, "pyre_q80_packed_bytes: need K >= 1 and N a multiple of 32");
  PYRE_CHECK_ARG(scale_dtype == PYRE_F32 || scale_dtype == PYRE_F16, "pyre_q80_packed_bytes: bad scale dtype");
  const int R = M == 2 ? gemv::kUnitRowsPair : gemv::kUnitRowsSingle;
  const int64_t nt = (N + gemv::kTileN - 1) / gemv::kTileN, upt = (K + R - 1) / R;
  *bytes = nt * upt * gemv::packed_block_bytes(M, scale_dtype == PYRE_F16 ? 2 : 4);
  return PYRE_OK;
}

extern "C" int pyre_q80_pack(int M, const int8_t* q0, const void* s0, const int8_t* q1, const void* s1, int K, int N,
                             int scale_dtype, void* out, void* stream) {
  using namespace pyre;
  int64_t bytes = 0;
  int rc = pyre_q80_packed_bytes(M, K, N, scale_dtype, &bytes);
  if (rc) return rc;
  PYRE_CHECK_ARG(q0 != nullptr && s0 != nullptr && out != nullptr, "pyre_q80_pack: null pointer");
  PYRE_CHECK_ARG(M == 1 || (q1 != nullptr && s1 != nullptr), "pyre_q80_pack: M == 2 needs both matrices");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(q0) % 16 == 0 && (q1 == nullptr || reinterpret_cast<uintptr_t>(q1) % 16 == 0) &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0,
                 "pyre_q80_pack: q and out must be 16-byte aligned");
  const int R = M == 2 ? gemv::kUnitRowsPair : gemv::kUnitRowsSingle;
  const int upt = (K + R - 1) / R;
  const int64_t nblocks = static_cast<int64_t>((N + gemv::kTileN - 1) / gemv::kTileN) * upt;
  const int64_t work = nblocks * (static_cast<int64_t>(M) * R * 16 + static_cast<int64_t>(M) * R * 8);
  const int grid = grid_for(work, 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (scale_dtype == PYRE_F16)
    q80_pack_kernel<__half><<<grid, 256, 0, s>>>(q0, static_cast<const __half*>(s0), q1, static_cast<const __half*>(s1),
                                                 M, K, N, upt, nblocks, static_cast<uint8_t*>(out));
  else
    q80_pack_kernel<float><<<grid, 256, 0, s>>>(q0, static_cast<const float*>(s0), q1, static_cast<const float*>(s1),
                                                M, K, N, upt, nblocks, static_cast<uint8_t*>(out));
  PYRE_LAUNCH_CHECK("q80_pack_kernel");
  return PYRE_OK;
}
