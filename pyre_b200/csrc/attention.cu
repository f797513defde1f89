// Attention path of the layer (reference: src/orchestrator/root_node.py:250-314 prefill,
// :900-933 decode block, :1009-1031 decode attention; src/kernels/mojo/pyre_kernels.mojo
// rms_norm :18-35, softmax :39-58, apply_rope :62-96).
//
// Device layout:
//   q, k, v projections : f32 [T, heads, hd]   (the reference's [1, S, heads, hd])
//   rotated queries     : f16 [nq, T, hd]
//   KV cache            : f16 [n_kv, max_t, hd] per layer, position-major inside a head.
//                         Values are clipped to +-1000 before they are stored (the reference
//                         clips q, k and v, and clipping is idempotent), so f16 holds them;
//                         f16 keeps 11 significant bits (the reference keeps f32).
// Kernels:
//   rms_norm_kernel       one CTA per row, f64 sum of squares like the reference
//   softmax_rows_kernel   one CTA per row (max initialised to -1e10 like the reference)
//   rope_append_kernel    RoPE of q and k at positions start_pos.., clip, f16 store / append
//                         (one CTA per token, shared cos/sin table)
//   attn_decode_kernel    flash-decoding: CTAs split the cache of a kv head, f16 mma.sync
//                         scores / weighted values with an online softmax, partials added
//                         in order through a cluster's distributed shared memory
//                         (deterministic)
//   attn_prefill_tc_kernel causal attention on tcgen05: 128 queries x 128 keys per step, S and
//                         O accumulated in tensor memory, online softmax by one warpgroup,
//                         TMA-fed, GQA by kv head = h / rep
#include <cmath>

#include <algorithm>
#include <cooperative_groups.h>
#include <mutex>

#include "common.cuh"
#include "umma.cuh"

namespace pyre {
namespace attn {

// ---------------------------------------------------------------------------------------
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
                                int H, double eps) {
  const int64_t row = blockIdx.x;
  const float* xr = x + row * H;
  double sq = 0.0;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const double v = xr[i];
    sq += v * v;
  }
  __shared__ double red[32];
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const double rstd = 1.0 / sqrt(red[0] / H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[row * H + i] = static_cast<float>(static_cast<double>(xr[i]) * rstd * static_cast<double>(w[i]));
}

// h = x + delta (the f32 residual add of root_node.py:947 / :997), then norm = rms_norm(h, w)
// as rms_norm_kernel; one CTA per row. h may alias x; norm may be null (add only).
__global__ void add_rms_norm_kernel(const float* x, const float* __restrict__ delta, float* h,
                                    const float* __restrict__ w, float* __restrict__ norm, int H, double eps) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const float* xr = x + row * H;
  const float* dr = delta + row * H;
  float* hr = h + row * H;
  double sq = 0.0;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = __fadd_rn(xr[i], dr[i]);
    hr[i] = v;
    sq += static_cast<double>(v) * static_cast<double>(v);
  }
  if (norm == nullptr) return;
  __shared__ double red[32];
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const double rstd = 1.0 / sqrt(red[0] / H + eps);
  // each thread reads back only the elements it wrote above
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    norm[row * H + i] = static_cast<float>(static_cast<double>(hr[i]) * rstd * static_cast<double>(w[i]));
}

// add_rms_norm_kernel for H % 4 == 0 and H <= 4 * kNormVec * blockDim: every x and delta
// value is loaded (16 bytes at a time) into registers before anything is stored, so the loads
// of a row overlap instead of waiting one after another behind stores that may alias them.
constexpr int kNormVec = 4;
__global__ void __launch_bounds__(1024) add_rms_norm_vec_kernel(const float* x, const float* __restrict__ delta,
                                                                float* h, const float* __restrict__ w,
                                                                float* __restrict__ norm, int H, double eps) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int n4 = H >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + row * H);
  const float4* dr = reinterpret_cast<const float4*>(delta + row * H);
  float4 v[kNormVec];
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < n4) {
      const float4 a = xr[i], b = __ldg(dr + i);
      v[j] = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
    }
  }
  double sq = 0.0;
  float4* hr = reinterpret_cast<float4*>(h + row * H);
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < n4) {
      hr[i] = v[j];
      sq += static_cast<double>(v[j].x) * v[j].x + static_cast<double>(v[j].y) * v[j].y +
            static_cast<double>(v[j].z) * v[j].z + static_cast<double>(v[j].w) * v[j].w;
    }
  }
  if (norm == nullptr) return;
  __shared__ double red[32];
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const double rstd = 1.0 / sqrt(red[0] / H + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4* nr = reinterpret_cast<float4*>(norm + row * H);
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < n4) {
      const float4 g = __ldg(wr + i);
      nr[i] = make_float4(static_cast<float>(static_cast<double>(v[j].x) * rstd * static_cast<double>(g.x)),
                          static_cast<float>(static_cast<double>(v[j].y) * rstd * static_cast<double>(g.y)),
                          static_cast<float>(static_cast<double>(v[j].z) * rstd * static_cast<double>(g.z)),
                          static_cast<float>(static_cast<double>(v[j].w) * rstd * static_cast<double>(g.w)));
    }
  }
}

// ---------------------------------------------------------------------------------------
__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ out, int C) {
  const int64_t row = blockIdx.x;
  const float* xr = x + row * C;
  __shared__ float red[32];
  float mx = -1e10f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) mx = fmaxf(mx, xr[i]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -1e10f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float sum = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) sum += expf(xr[i] - mx);
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / red[0];
  for (int i = threadIdx.x; i < C; i += blockDim.x) out[row * C + i] = expf(xr[i] - mx) * inv;
}

// ---------------------------------------------------------------------------------------
// RoPE + clip + append. The cos/sin of a token's position for the rotated half-dims come
// from the table of pyre_rope_table (f64 on the host, as the reference computes them); every
// q and k head of the token is rotated in f32 (pair (i, i+half)), clipped to +-1000 and
// stored as f16; v is clipped and appended. rope_append_vec_kernel handles hd 64 / 128 with
// half a multiple of 4 (16-byte loads); rope_append_kernel (one CTA per token and group of
// heads, scalar) everything else.
constexpr int kRopeMaxHalf = 256;
constexpr int kRopeHeadsPerCta = 8;

// The rotate-half pair (x1, x2) = (src[j], src[j + half]) -> (x1 c - x2 s, x1 s + x2 c), each
// product and sum rounded separately in f32 like the reference's numpy arithmetic (no FMA),
// so that every kernel that rotates stores the same bits.
__device__ __forceinline__ float rope_lo(float x1, float x2, float c, float s) {
  return __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
}
__device__ __forceinline__ float rope_hi(float x1, float x2, float c, float s) {
  return __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
}
__device__ __forceinline__ float clip1000(float r) { return fminf(fmaxf(r, -1000.f), 1000.f); }

// Element i of a rotated, clipped head (rotate-half pairs (i, i + half), cos/sin from the
// table row of the position, dims >= 2 * half pass through), as the fused decode step and
// the scalar append kernel store it.
__device__ __forceinline__ float rope_clip(const float* __restrict__ src, int i, int half, float c, float s) {
  float r;
  if (i < 2 * half) {
    const int jj = i < half ? i : i - half;
    const float x1 = __ldg(src + jj), x2 = __ldg(src + jj + half);
    r = i < half ? rope_lo(x1, x2, c, s) : rope_hi(x1, x2, c, s);
  } else {
    r = __ldg(src + i);
  }
  return clip1000(r);
}

__device__ __forceinline__ uint32_t pack_h2_rn(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Vectorised RoPE + clip + append for hd in {64, 128} with half a multiple of 4: one CTA per
// token, one thread per 4 consecutive dims of a q, k or v row (float4 loads of the dims and
// of their rotation partners, 8-byte f16 stores), all heads of the token.
template <int HD>
__global__ void __launch_bounds__(256) rope_append_vec_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, int64_t q_stride,
                                                               int64_t kv_stride, int T, int nq, int nkv,
                                                               int start_pos, const float2* __restrict__ table,
                                                               int half, __half* __restrict__ q_out,
                                                               __half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                                               int max_t) {
  constexpr int U = HD / 4;
  const int t = blockIdx.x;
  const int pos = start_pos + t;
  const float2* row_cs = table + static_cast<int64_t>(pos) * half;
  const int units = (nq + 2 * nkv) * U;
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int r = u / U, c4 = (u - r * U) * 4;
    const float* src;
    __half* dst;
    bool rot = true;
    if (r < nq) {
      src = q + t * q_stride + static_cast<int64_t>(r) * HD;
      dst = q_out + (static_cast<int64_t>(r) * T + t) * HD;
    } else if (r < nq + nkv) {
      src = k + t * kv_stride + static_cast<int64_t>(r - nq) * HD;
      dst = k_cache + (static_cast<int64_t>(r - nq) * max_t + pos) * HD;
    } else {
      src = v + t * kv_stride + static_cast<int64_t>(r - nq - nkv) * HD;
      dst = v_cache + (static_cast<int64_t>(r - nq - nkv) * max_t + pos) * HD;
      rot = false;
    }
    const float4 x = __ldg(reinterpret_cast<const float4*>(src + c4));
    float o[4] = {x.x, x.y, x.z, x.w};
    if (rot && c4 < 2 * half) {
      const bool lo = c4 < half;
      const int j = lo ? c4 : c4 - half;
      const float4 pr = __ldg(reinterpret_cast<const float4*>(src + (lo ? c4 + half : c4 - half)));
      const float4 cs01 = __ldg(reinterpret_cast<const float4*>(row_cs + j));
      const float4 cs23 = __ldg(reinterpret_cast<const float4*>(row_cs + j + 2));
      const float p[4] = {pr.x, pr.y, pr.z, pr.w};
      const float c[4] = {cs01.x, cs01.z, cs23.x, cs23.z}, sn[4] = {cs01.y, cs01.w, cs23.y, cs23.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = lo ? rope_lo(o[e], p[e], c[e], sn[e]) : rope_hi(p[e], o[e], c[e], sn[e]);
    }
    uint2 h;
    h.x = pack_h2_rn(clip1000(o[0]), clip1000(o[1]));
    h.y = pack_h2_rn(clip1000(o[2]), clip1000(o[3]));
    *reinterpret_cast<uint2*>(dst + c4) = h;
  }
}


__global__ void __launch_bounds__(256) rope_append_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                           const float* __restrict__ v, int64_t q_stride,
                                                           int64_t kv_stride, int T, int nq, int nkv, int hd,
                                                           int start_pos, const float2* __restrict__ table, int dims,
                                                           __half* __restrict__ q_out, __half* __restrict__ k_cache,
                                                           __half* __restrict__ v_cache, int max_t) {
  __shared__ float cs[kRopeMaxHalf], sn[kRopeMaxHalf];
  const int t = blockIdx.x;
  const int pos = start_pos + t;
  const int half = dims >= 2 ? dims / 2 : 0;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float2 c = table[static_cast<int64_t>(pos) * half + j];
    cs[j] = c.x;
    sn[j] = c.y;
  }
  __syncthreads();
  // this CTA's heads: q heads then k heads, kRopeHeadsPerCta of them starting at y * that
  const int h0 = blockIdx.y * kRopeHeadsPerCta;
  const int h1 = min(h0 + kRopeHeadsPerCta, nq + nkv);
#pragma unroll 4
  for (int e = threadIdx.x; e < (h1 - h0) * hd; e += blockDim.x) {
    const int hh = h0 + e / hd, i = e % hd;
    const bool is_q = hh < nq;
    const int h = is_q ? hh : hh - nq;
    const float* src = is_q ? q + t * q_stride + static_cast<int64_t>(h) * hd : k + t * kv_stride + static_cast<int64_t>(h) * hd;
    const int jj = i < 2 * half ? (i < half ? i : i - half) : 0;
    const float r = rope_clip(src, i, half, half ? cs[jj] : 0.f, half ? sn[jj] : 0.f);
    if (is_q)
      q_out[(static_cast<int64_t>(h) * T + t) * hd + i] = __float2half_rn(r);
    else
      k_cache[(static_cast<int64_t>(h) * max_t + pos) * hd + i] = __float2half_rn(r);
  }
  // v heads with the k heads of this CTA
  const int v0 = max(h0, nq) - nq, v1 = max(h1, nq) - nq;
#pragma unroll 4
  for (int e = threadIdx.x; e < (v1 - v0) * hd; e += blockDim.x) {
    const int h = v0 + e / hd, i = e % hd;
    const float x = __ldg(v + t * kv_stride + static_cast<int64_t>(h) * hd + i);
    v_cache[(static_cast<int64_t>(h) * max_t + pos) * hd + i] = __float2half_rn(fminf(fmaxf(x, -1000.f), 1000.f));
  }
}

// ---------------------------------------------------------------------------------------
// Warp-level f16 MMA (m16n8k16, f32 accumulation) and f16 packing, used by decode attention.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------------------
// Decode attention (flash-decoding on mma.sync). grid (S, nkv), 256 threads, clusters of
// C = min(S, 8) CTAs along x; S = C * X splits of the cache of kv head g. CTA (s, g) takes
// positions [s*t/S, (s+1)*t/S) and its 8 warps take batches of 16 positions in turn, the
// loads of a warp's next batch issued before its current batch is computed. Per batch a
// warp computes S^T[16 pos x 8 heads] = K . Q^T with f16 MMAs (the rep <= 8 query heads of
// the kv head are the N = 8 columns), an online softmax per head, and
// O^T[hd x 8 heads] += V^T . P^T. The operands go from global memory straight to registers,
// every load instruction reading whole 32-byte sectors:
//   * a dot product may take its terms in any order, so lane (g, c) of the score MMA holds
//     dims {32j + 8c + e : e < 8} of key rows g, g+8 and of query head g;
//   * the value MMA's A operand (rows = dims, columns = positions) is built with byte
//     permutes from 16-byte pieces of 4 value rows (positions 2c, 2c+1, 2c+8, 2c+9): lane
//     (g, c) reads the hd/8 dims dec_vdim(g, j) + [0, 8) of each; m-tile mt takes the pair of
//     dims in word mt of that slice (row g the even one, row g + 8 the odd one);
//   * P^T (positions x heads) is the score accumulator transposed with movmatrix.
// Partials (running max, sum of exponentials, weighted values) are rescaled to the CTA's
// maximum and added in warp order in shared memory; each CTA of a cluster stores its partial
// into rank 0's shared memory (distributed shared memory), and rank 0 adds the C partials in
// rank order. With X > 1, rank 0 of each cluster writes its partial to the workspace and the
// cluster that arrives last for its kv head (an arrival counter, reset by it) adds the X
// partials in order. No waits on other CTAs beyond the cluster barrier; deterministic for a
// given S.
constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecBatch = 16;
constexpr int kDecMaxRep = 8;
constexpr int kDecCluster = 8;
constexpr int kDecMaxGroups = 8;       // X, clusters per kv head
constexpr int kDecMinChunk = 128;      // positions per CTA at least (one batch per warp)
constexpr int kDecGroupChunk = 2048;   // positions per cluster before another cluster is added

constexpr int64_t kDecPrefetchBytes = 32768;   // bytes per L2 prefetch instruction

// Brings [src, src + bytes) into L2 (16-byte aligned, bytes % 16 == 0); nothing to wait for.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Status word of the attention kernels (read and cleared by pyre_attn_status).
__device__ int g_attn_status;

struct DecodeParams {
  const __half* q;       // [nq, hd] rotated, clipped (attention alone)
  const __half* kc;      // [nkv, max_t, hd]
  const __half* vc;
  const float* qf;       // fused decode step: the token's f32 q [nq * hd], k and v [nkv * hd],
  const float* kf;       // rotated at position t - 1 (rope row), clipped, k and v appended
  const float* vf;       // to the caches at row t - 1 by the CTAs of the last split
  const float2* rope;    // (cos, sin) [half] of position t - 1
  int half;
  __half* kw;            // kc, vc as written by the append
  __half* vw;
  float* out;            // [nq * hd]
  float* part;           // [nkv][X][2 * rep + rep * hd]: max, sum, weighted values per cluster
  unsigned* count;       // [nkv] arrival counters, zero between launches
  int nq, nkv, t, max_t, mask_lo, mask_hi;
  float scale2;          // log2(e) / sqrt(hd): exponentials are taken base 2
  const int* pos_dev;    // fused step with the position in device memory (a step captured in
                         // a CUDA graph): t = *pos_dev + 1, rope row *pos_dev of rope_base;
                         // t and rope above are then only the host's plan of the grid
  const float2* rope_base;
  // Batched fused step: B sequences at one position, their caches [B][nkv_seq] stacked as
  // nkv = B * nkv_seq kv heads (out likewise [B][nq_seq * hd]); kv head g belongs to sequence
  // g / nkv_seq, whose q, k, v rows start at qf + b * q_bstride, kf / vf + b * kv_bstride.
  int nkv_seq;
  int64_t q_bstride, kv_bstride;
};

// Shared memory: the static part below, then (dynamic) the warps' rescaled partials
// [kDecWarps][rep][HD + 8] and the cluster ranks' partials [kDecCluster][rep][HD].
struct DecodeSmem {
  float wm[kDecWarps][kDecMaxRep], wl[kDecWarps][kDecMaxRep];
  float cm[kDecCluster * kDecMaxGroups][kDecMaxRep], cl[kDecCluster * kDecMaxGroups][kDecMaxRep];
  int last;
};
template <int HD>
constexpr int dec_dyn_bytes(int rep) {
  return (kDecWarps * rep * (HD + 8) + kDecCluster * rep * HD) * 4;
}

template <int HD>
struct DecodeRows {                            // one batch of 16 positions, per lane
  uint4 ka[HD / 32], kb[HD / 32];              // key rows base+g, base+g+8
  uint4 va[HD / 64], vb[HD / 64], vc[HD / 64], vd[HD / 64];   // value rows base+2c, +1, +8, +9
};

__device__ __forceinline__ uint32_t u4w(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// 2^x (PTX ex2.approx: relative error below 2^-22, far inside the path's tolerance).
__device__ __forceinline__ float dec_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// exp((m - M) / sqrt(hd)) with scale2 = log2(e) / sqrt(hd); 0 for an empty partial (m = -inf).
__device__ __forceinline__ float dec_weight(float m, float M, float scale2) {
  return m == -INFINITY ? 0.f : dec_exp2((m - M) * scale2);
}
// First dim of 16-byte piece j of lane group g's value slice: lanes 2k, 2k+1 read the two
// halves of one 32-byte sector in each load.
template <int HD>
__device__ __forceinline__ int dec_vdim(int g, int j) {
  return HD == 128 ? 32 * (g >> 1) + 16 * j + 8 * (g & 1) : 8 * g;
}
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// 16 bytes of the cache: through the read-only path, or (COH, when this kernel appends a
// row that its own CTA then reads) a plain load, ordered after the appending stores by the
// CTA barrier.
template <bool COH>
__device__ __forceinline__ uint4 ld_row16(const __half* p) {
  if constexpr (!COH) {
    return __ldg(reinterpret_cast<const uint4*>(p));
  } else {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
  }
}

// Rows past the chunk end (last) are clamped to it; their scores are masked.
template <int HD, bool COH>
__device__ __forceinline__ void dec_load(DecodeRows<HD>& b, const __half* kh, const __half* vh, int base, int last,
                                         int lg, int lc) {
  const __half* ka = kh + static_cast<int64_t>(min(base + lg, last)) * HD + 8 * lc;
  const __half* kb = kh + static_cast<int64_t>(min(base + lg + 8, last)) * HD + 8 * lc;
#pragma unroll
  for (int j = 0; j < HD / 32; ++j) {
    b.ka[j] = ld_row16<COH>(ka + 32 * j);
    b.kb[j] = ld_row16<COH>(kb + 32 * j);
  }
  const __half* va = vh + static_cast<int64_t>(min(base + 2 * lc, last)) * HD;
  const __half* vb = vh + static_cast<int64_t>(min(base + 2 * lc + 1, last)) * HD;
  const __half* vc = vh + static_cast<int64_t>(min(base + 2 * lc + 8, last)) * HD;
  const __half* vd = vh + static_cast<int64_t>(min(base + 2 * lc + 9, last)) * HD;
#pragma unroll
  for (int j = 0; j < HD / 64; ++j) {
    const int d = dec_vdim<HD>(lg, j);
    b.va[j] = ld_row16<COH>(va + d);
    b.vb[j] = ld_row16<COH>(vb + d);
    b.vc[j] = ld_row16<COH>(vc + d);
    b.vd[j] = ld_row16<COH>(vd + d);
  }
}

struct DecodeState {
  float m0, m1, l0, l1;    // heads 2c, 2c+1: running max (raw score units), this lane's sum
};

template <int HD>
__device__ __forceinline__ void dec_batch(const DecodeRows<HD>& b, const uint4 (&qv)[HD / 32], float (&o)[HD / 16][4],
                                          DecodeState& st, int base, int c1, int mask_lo, int mask_hi, float scale2,
                                          int lg) {
  constexpr int KS = HD / 16;
  // scores: s[0], s[1] = position base+lg, heads 2c, 2c+1; s[2], s[3] = position base+lg+8
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    const int j = i >> 1, w = 2 * (i & 1);
    const uint32_t a[4] = {u4w(b.ka[j], w), u4w(b.kb[j], w), u4w(b.ka[j], w + 1), u4w(b.kb[j], w + 1)};
    mma16816(s, a, u4w(qv[j], w), u4w(qv[j], w + 1));
  }
  const int pa = base + lg, pb = base + lg + 8;
  if (pa >= c1 || (pa >= mask_lo && pa < mask_hi)) s[0] = s[1] = -INFINITY;
  if (pb >= c1 || (pb >= mask_lo && pb < mask_hi)) s[2] = s[3] = -INFINITY;
  float x0 = fmaxf(s[0], s[2]), x1 = fmaxf(s[1], s[3]);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, off));
    x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, off));
  }
  const float n0 = fmaxf(st.m0, x0), n1 = fmaxf(st.m1, x1);
  const float al0 = dec_weight(st.m0, n0, scale2), al1 = dec_weight(st.m1, n1, scale2);
  const float p0 = n0 == -INFINITY ? 0.f : dec_exp2((s[0] - n0) * scale2);
  const float p1 = n1 == -INFINITY ? 0.f : dec_exp2((s[1] - n1) * scale2);
  const float p2 = n0 == -INFINITY ? 0.f : dec_exp2((s[2] - n0) * scale2);
  const float p3 = n1 == -INFINITY ? 0.f : dec_exp2((s[3] - n1) * scale2);
  st.l0 = st.l0 * al0 + p0 + p2;     // this lane's positions only; summed over lanes at the end
  st.l1 = st.l1 * al1 + p1 + p3;
  // the weighted sums are rescaled only when a running maximum of the warp has grown
  if (__any_sync(0xffffffffu, n0 > st.m0 || n1 > st.m1)) {
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      o[mt][0] *= al0;
      o[mt][2] *= al0;
      o[mt][1] *= al1;
      o[mt][3] *= al1;
    }
  }
  st.m0 = n0;
  st.m1 = n1;
  const uint32_t b0 = movmatrix_t(pack_h2(p0, p1)), b1 = movmatrix_t(pack_h2(p2, p3));
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) {
    const int j = mt >> 2, w = mt & 3;
    const uint32_t wa = u4w(b.va[j], w), wb = u4w(b.vb[j], w), wc = u4w(b.vc[j], w), wd = u4w(b.vd[j], w);
    const uint32_t a[4] = {__byte_perm(wa, wb, 0x5410), __byte_perm(wa, wb, 0x7632), __byte_perm(wc, wd, 0x5410),
                           __byte_perm(wc, wd, 0x7632)};
    mma16816(o[mt], a, b0, b1);
  }
}

template <int HD, bool FUSED>
__global__ void __launch_bounds__(kDecThreads, 1) attn_decode_kernel(const DecodeParams p) {
  namespace cg = cooperative_groups;
  constexpr int KS = HD / 16;
  constexpr int KQ = HD / 32;
  constexpr int WP = HD + 8;            // row pitch of the warp partials
  __shared__ DecodeSmem sm;
  extern __shared__ float4 dec_dyn[];
  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int split = blockIdx.x, S = gridDim.x, g = blockIdx.y;
  {
    // This CTA's K and V rows into L2 while the previous kernel finishes. A prefetch only
    // warms L2 (the loads below read whatever the rows hold after the wait), so the position it
    // is planned from may be read before the wait.
    int tp = p.t;
    if constexpr (FUSED) {
      if (p.pos_dev != nullptr) {
        const int q = *reinterpret_cast<const volatile int*>(p.pos_dev);
        if (q >= 0 && q < p.max_t) tp = q + 1;
      }
    }
    if (threadIdx.x == 0) {
      const int a0 = static_cast<int>(static_cast<int64_t>(tp) * split / S);
      const int a1 = static_cast<int>(static_cast<int64_t>(tp) * (split + 1) / S);
      if (a1 > a0) {
        const int64_t off = (static_cast<int64_t>(g) * p.max_t + a0) * HD;
        const int64_t bytes = static_cast<int64_t>(a1 - a0) * HD * 2;
        for (int64_t b = 0; b < bytes; b += kDecPrefetchBytes) {
          const uint32_t n = static_cast<uint32_t>(bytes - b < kDecPrefetchBytes ? bytes - b : kDecPrefetchBytes);
          prefetch_l2(reinterpret_cast<const char*>(p.kc + off) + b, n);
          prefetch_l2(reinterpret_cast<const char*>(p.vc + off) + b, n);
        }
      }
    }
  }
  pdl_wait();      // q, k, v (and the position) come from the previous kernels of the stream
  pdl_trigger();
  int t = p.t;
  const float2* rope = p.rope;
  (void)rope;
  if constexpr (FUSED) {
    if (p.pos_dev != nullptr) {
      // every CTA reads the same position, so all of them take the same branch, before any
      // cluster barrier, counter or cache write
      const int pos = *p.pos_dev;
      if (pos < 0 || pos >= p.max_t || pos + 1 < S) {
        if (threadIdx.x == 0 && split == 0 && g == 0) atomicExch(&g_attn_status, PYRE_EINVAL);
        return;
      }
      t = pos + 1;
      rope = p.half ? p.rope_base + static_cast<int64_t>(pos) * p.half : nullptr;
    }
  }
  if (C > 1) cluster_arrive_relaxed();  // every CTA of the cluster has started (waited on below)
  const int X = S / C, grp = split / C;
  const int rep = p.nq / p.nkv;
  const int E = rep * HD;
  float* wo = reinterpret_cast<float*>(dec_dyn);                 // [kDecWarps][rep][WP]
  float* co = wo + kDecWarps * rep * WP;                         // [kDecCluster][rep][HD]
  const int c0 = static_cast<int>(static_cast<int64_t>(t) * split / S);
  const int c1 = static_cast<int>(static_cast<int64_t>(t) * (split + 1) / S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, lg = lane >> 2, lc = lane & 3;

  uint4 qv[KQ];
  if constexpr (FUSED) {
    // RoPE + clip of this kv head's query heads into shared memory; the last split appends
    // the token's rotated k and clipped v at row t - 1 before any of its warps reads it
    __shared__ __align__(16) __half qs[kDecMaxRep * HD];
    const int pos = t - 1;
    const int gb = g / p.nkv_seq, gl = g - gb * p.nkv_seq;     // sequence, kv head within it
    const float* qf = p.qf + gb * p.q_bstride;
    const float* kf = p.kf + gb * p.kv_bstride;
    const float* vf = p.vf + gb * p.kv_bstride;
    for (int e = threadIdx.x; e < E; e += kDecThreads) {
      const int r = e / HD, i = e - r * HD;
      const int jj = i < 2 * p.half ? (i < p.half ? i : i - p.half) : 0;
      const float2 cs = p.half ? __ldg(rope + jj) : make_float2(0.f, 0.f);
      qs[e] = __float2half_rn(rope_clip(qf + (static_cast<int64_t>(gl) * rep + r) * HD, i, p.half, cs.x, cs.y));
    }
    if (split == S - 1) {
      for (int i = threadIdx.x; i < HD; i += kDecThreads) {
        const int jj = i < 2 * p.half ? (i < p.half ? i : i - p.half) : 0;
        const float2 cs = p.half ? __ldg(rope + jj) : make_float2(0.f, 0.f);
        const int64_t row = (static_cast<int64_t>(g) * p.max_t + pos) * HD;
        p.kw[row + i] = __float2half_rn(rope_clip(kf + static_cast<int64_t>(gl) * HD, i, p.half, cs.x, cs.y));
        p.vw[row + i] = __float2half_rn(fminf(fmaxf(__ldg(vf + static_cast<int64_t>(gl) * HD + i), -1000.f), 1000.f));
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < KQ; ++j)
      qv[j] = lg < rep ? *reinterpret_cast<const uint4*>(qs + lg * HD + 32 * j + 8 * lc) : make_uint4(0u, 0u, 0u, 0u);
  } else {
#pragma unroll
    for (int j = 0; j < KQ; ++j)
      qv[j] = lg < rep ? __ldg(reinterpret_cast<const uint4*>(p.q + (static_cast<int64_t>(g) * rep + lg) * HD +
                                                              32 * j + 8 * lc))
                       : make_uint4(0u, 0u, 0u, 0u);
  }
  const __half* kh = p.kc + static_cast<int64_t>(g) * p.max_t * HD;
  const __half* vh = p.vc + static_cast<int64_t>(g) * p.max_t * HD;
  float o[KS][4];
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  DecodeState st{-INFINITY, -INFINITY, 0.f, 0.f};

  constexpr int kStep = kDecWarps * kDecBatch;
  DecodeRows<HD> r0, r1;
  int base = c0 + warp * kDecBatch;
  if (base < c1) dec_load<HD, FUSED>(r0, kh, vh, base, c1 - 1, lg, lc);
  while (base < c1) {
    if (base + kStep < c1) dec_load<HD, FUSED>(r1, kh, vh, base + kStep, c1 - 1, lg, lc);
    dec_batch(r0, qv, o, st, base, c1, p.mask_lo, p.mask_hi, p.scale2, lg);
    base += kStep;
    if (base >= c1) break;
    if (base + kStep < c1) dec_load<HD, FUSED>(r0, kh, vh, base + kStep, c1 - 1, lg, lc);
    dec_batch(r1, qv, o, st, base, c1, p.mask_lo, p.mask_hi, p.scale2, lg);
    base += kStep;
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, off);
    st.l1 += __shfl_xor_sync(0xffffffffu, st.l1, off);
  }
  if (lg == 0) {
    sm.wm[warp][2 * lc] = st.m0;
    sm.wm[warp][2 * lc + 1] = st.m1;
  }
  __syncthreads();
  // rescale this warp's partial to the CTA maximum of each head
  float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) {
    M0 = fmaxf(M0, sm.wm[w][2 * lc]);
    M1 = fmaxf(M1, sm.wm[w][2 * lc + 1]);
  }
  const float f0 = dec_weight(st.m0, M0, p.scale2), f1 = dec_weight(st.m1, M1, p.scale2);
  if (lg == 0) {
    sm.wl[warp][2 * lc] = st.l0 * f0;
    sm.wl[warp][2 * lc + 1] = st.l1 * f1;
  }
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) {
    const int d = dec_vdim<HD>(lg, mt >> 2) + 2 * (mt & 3);
    if (2 * lc < rep)
      *reinterpret_cast<float2*>(wo + (warp * rep + 2 * lc) * WP + d) = make_float2(o[mt][0] * f0, o[mt][2] * f0);
    if (2 * lc + 1 < rep)
      *reinterpret_cast<float2*>(wo + (warp * rep + 2 * lc + 1) * WP + d) = make_float2(o[mt][1] * f1, o[mt][3] * f1);
  }
  __syncthreads();

  // this CTA's partial (warps in order), into rank 0's shared memory when C > 1
  if (C > 1) cluster_wait();            // rank 0 has started: its shared memory can be written
  float* dst_o = C > 1 ? cluster.map_shared_rank(co, 0) + rank * E : nullptr;
  float* dst_m = C > 1 ? cluster.map_shared_rank(&sm.cm[0][0], 0) + rank * kDecMaxRep : nullptr;
  float* dst_l = C > 1 ? cluster.map_shared_rank(&sm.cl[0][0], 0) + rank * kDecMaxRep : nullptr;
  for (int i = threadIdx.x; i < E; i += kDecThreads) {
    const int r = i / HD, d = i - r * HD;
    float O = 0.f, L = 0.f, M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      O += wo[(w * rep + r) * WP + d];
      L += sm.wl[w][r];
      M = fmaxf(M, sm.wm[w][r]);
    }
    if (C == 1 && X == 1) {
      p.out[static_cast<int64_t>(g) * E + i] = O / L;
    } else if (C == 1) {
      co[i] = O;
      if (d == 0) {
        sm.cm[0][r] = M;
        sm.cl[0][r] = L;
      }
    } else {
      dst_o[i] = O;
      if (d == 0) {
        dst_m[r] = M;
        dst_l[r] = L;
      }
    }
  }
  if (C > 1) {
    cluster_arrive();                   // release: the stores above are visible to rank 0
    cluster_wait();
    if (rank != 0) return;              // nothing reads this CTA's shared memory any more
  } else {
    if (X == 1) return;
    __syncthreads();
  }

  // rank 0: the C partials of this cluster, in rank order (weights recomputed per element)
  const int stride = 2 * rep + E;
  float* gpart = X > 1 ? p.part + (static_cast<int64_t>(g) * X + grp) * stride : nullptr;
  for (int i = threadIdx.x; i < E; i += kDecThreads) {
    const int r = i / HD;
    float M = -INFINITY;
#pragma unroll
    for (int cc = 0; cc < kDecCluster; ++cc)
      if (cc < C) M = fmaxf(M, sm.cm[cc][r]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int cc = 0; cc < kDecCluster; ++cc)
      if (cc < C) {
        const float wt = dec_weight(sm.cm[cc][r], M, p.scale2);
        O += co[cc * E + i] * wt;
        L += sm.cl[cc][r] * wt;
      }
    if (X == 1) {
      p.out[static_cast<int64_t>(g) * E + i] = O / L;
    } else {
      gpart[2 * rep + i] = O;
      if (i - r * HD == 0) {
        gpart[r] = M;
        gpart[rep + r] = L;
      }
    }
  }
  if (X == 1) return;
  // arrival: the barrier orders this CTA's stores before thread 0's fence and atomic
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const bool last = atomicAdd(p.count + g, 1u) == static_cast<unsigned>(X - 1);
    if (last) __threadfence();
    sm.last = last;
  }
  __syncthreads();
  if (!sm.last) return;
  // the last cluster of kv head g adds the X cluster partials in order
  const float* pg = p.part + static_cast<int64_t>(g) * X * stride;
  for (int i = threadIdx.x; i < E; i += kDecThreads) {
    const int r = i / HD;
    float m[kDecMaxGroups], l[kDecMaxGroups], v[kDecMaxGroups];
#pragma unroll
    for (int x = 0; x < kDecMaxGroups; ++x) {
      m[x] = x < X ? __ldcg(pg + x * stride + r) : -INFINITY;
      l[x] = x < X ? __ldcg(pg + x * stride + rep + r) : 0.f;
      v[x] = x < X ? __ldcg(pg + x * stride + 2 * rep + i) : 0.f;
    }
    float M = -INFINITY;
#pragma unroll
    for (int x = 0; x < kDecMaxGroups; ++x) M = fmaxf(M, m[x]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int x = 0; x < kDecMaxGroups; ++x) {
      const float wt = dec_weight(m[x], M, p.scale2);
      O += v[x] * wt;
      L += l[x] * wt;
    }
    p.out[static_cast<int64_t>(g) * E + i] = O / L;
  }
  if (threadIdx.x == 0) p.count[g] = 0u;
}

struct PrefillParams {
  const __half* q;     // [nq, T, hd]
  const __half* kc;    // [nkv, max_t, hd]
  const __half* vc;
  float* out;          // [T, nq * hd]
  int T, nq, nkv, max_t;
  float scale_log2;    // log2(e) / sqrt(hd)
  // Ulysses output scatter (scatter != 0): row t goes to rank t / rows_per_rank, into its
  // [rows_per_rank, nq_total * hd] f32 buffer at head column head_off + h
  int scatter, rows_per_rank, head_off, nq_total;
  float* out_peers[16];
};

// ---------------------------------------------------------------------------------------
// Causal prefill attention on the 5th-generation tensor cores. CTA = (q head h, block of
// 128 queries), heaviest blocks first; 192 threads:
//   warp 0     TMA producer (Q once; K and V tiles of 128 keys into a 2-stage ring) and
//              tensor-memory allocator;
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into S buffer j % 2 of tensor memory
//              (M = 128 queries, N = 128 keys, K = hd) and O += P_j V_j (N = hd, K = 128
//              keys); S_{j+1} is issued before O += P_j V_j so the tensor core works while
//              the softmax does;
//   warps 2-5  softmax (thread = query row = tensor-memory lane): reads S_j, masks, runs the
//              online softmax in base 2, writes P_j (f16) into shared memory in the A-operand
//              layout; at the end O / l to the output.
// The running maximum of a row is raised only when the row's maximum grows by more than 8
// (base 2), so P <= 2^8 fits f16 and O (in tensor memory) is rescaled rarely; the rescale
// waits for the previous O += P V. Q, K, V arrive by 3-D TMA with 128-byte swizzle
// (positions past T read as zero); P is written in the same swizzled K-major layout.
// Every mbarrier wait is bounded; a timeout is recorded in the attention status word.
constexpr int kTcBM = 128, kTcBN = 128;
constexpr int kTcThreads = 192;
constexpr int kTcTmemCols = 512;   // S buffers 0..255, O 256..256+hd

struct PrefillTcParams {
  CUtensorMap tq, tk, tv;          // q [nq][T][hd]; k, v [nkv][T][hd] with row stride max_t * hd
  float* out;                      // [T, nq * hd]
  int T, nq, nkv;
  float scale_log2;                // log2(e) / sqrt(hd)
  int scatter, rows_per_rank, head_off, nq_total;
  float* out_peers[16];
  int* status;
};

template <int HD>
struct TcLayout {
  static constexpr int kRegion = kTcBM * 128;                 // 128 rows x 128 bytes, swizzled
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + (HD / 64) * kRegion;          // 2 stages
  static constexpr int kV = kK + 2 * (HD / 64) * kRegion;      // 2 stages
  static constexpr int kP = kV + 2 * (HD / 64) * kRegion;      // 2 buffers x (128 keys = 2 regions)
  static constexpr int kBar = kP + 2 * 2 * kRegion;
  static constexpr int kBytes = 1024 + kBar + 256;             // alignment slack, barriers
};

// Waits for the tensor-memory loads in flight; r is passed through so that no use of the
// loaded registers is scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads, 1) attn_prefill_tc_kernel(const __grid_constant__ PrefillTcParams p) {
  using L = TcLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 7;
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 11;
  uint64_t* mma_done = bars + 13;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 14);

  const int qb = static_cast<int>(gridDim.y) - 1 - static_cast<int>(blockIdx.y), h = blockIdx.x;
  const int g = h / (p.nq / p.nkv);
  const int q0 = qb * kTcBM;
  const int nkb = qb + 1;                 // causal: key blocks 0..qb (kTcBN == kTcBM)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t kTileBytes = kTcBN * HD * 2;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0) {
    umma::tmem_alloc(s_tmem, kTcTmemCols);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&p.tq);
      prefetch_tmap(&p.tk);
      prefetch_tmap(&p.tv);
      mbar_arrive_expect_tx(q_full, kTcBM * HD * 2);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) tma_load_3d(sm + L::kQ + c * L::kRegion, &p.tq, 64 * c, q0, h, q_full);
      int issued = 0;
      for (int j = 0; j < nkb; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_3d(sm + L::kK + (s * (HD / 64) + c) * L::kRegion, &p.tk, 64 * c, j * kTcBN, g, &kv_full[s]);
          tma_load_3d(sm + L::kV + (s * (HD / 64) + c) * L::kRegion, &p.tv, 64 * c, j * kTcBN, g, &kv_full[s]);
        }
        issued = j + 1;
      }
      // no copy may still be landing in shared memory when the CTA exits
      mbar_wait(q_full, 0, nullptr, 500000000ull);
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j)
        mbar_wait(&kv_full[j & 1], (j >> 1) & 1, nullptr, 500000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_s = umma::idesc_f16_f32_kmaj_kmaj<kTcBM, kTcBN>();
      constexpr uint32_t id_o = umma::idesc_f16_f32_kmaj_mnmaj<kTcBM, HD>();
      const uint32_t q_base = smem_u32(sm + L::kQ);
      auto issue_s = [&](int j) {   // S_j = Q K_j^T into S buffer j & 1
        const uint32_t k_base = smem_u32(sm + L::kK + (j & 1) * (HD / 64) * L::kRegion);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kRegion + (kk & 3) * 32;
          umma::mma_f16(tmem + (j & 1) * kTcBN, umma::smem_desc(q_base + off, 16, 1024, umma::kLayoutSW128),
                        umma::smem_desc(k_base + off, 16, 1024, umma::kLayoutSW128), id_s, kk ? 1u : 0u);
        }
        umma::mma_commit(&s_full[j & 1]);
      };
      bool ok = mbar_wait(q_full, 0, p.status) && mbar_wait(&kv_full[0], 0, p.status);
      if (ok) {
        umma::fence_after_sync();
        issue_s(0);
      }
      for (int j = 0; ok && j < nkb; ++j) {
        if (j + 1 < nkb) {
          const int n = j + 1;
          ok = mbar_wait(&kv_full[n & 1], (n >> 1) & 1, p.status);
          if (ok && n >= 2) ok = mbar_wait(&s_free[n & 1], ((n >> 1) - 1) & 1, p.status);
          if (!ok) break;
          umma::fence_after_sync();
          issue_s(n);
        }
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.status)) break;
        umma::fence_after_sync();
        const uint32_t p_base = smem_u32(sm + L::kP + (j & 1) * 2 * L::kRegion);
        const uint32_t v_base = smem_u32(sm + L::kV + (j & 1) * (HD / 64) * L::kRegion);
#pragma unroll
        for (int kk = 0; kk < kTcBN / 16; ++kk) {
          const uint64_t ad =
              umma::smem_desc(p_base + (kk >> 2) * L::kRegion + (kk & 3) * 32, 16, 1024, umma::kLayoutSW128);
          const uint64_t bd = umma::smem_desc(v_base + kk * 2048, L::kRegion, 1024, umma::kLayoutSW128);
          umma::mma_f16(tmem + 2 * kTcBN, ad, bd, id_o, (j | kk) ? 1u : 0u);
        }
        umma::mma_commit(&pv_done[j & 1]);
        umma::mma_commit(&kv_empty[j & 1]);
      }
      umma::mma_commit(mma_done);   // every MMA issued (also after an early stop) has completed
    }
  } else {
    // ---------------- softmax (thread = query row = tensor-memory lane) ----------------
    const int quarter = warp & 3;                      // warps 2, 3, 4, 5 -> lanes 64, 96, 0, 32
    const int row = quarter * 32 + lane;
    const int qrow = q0 + row;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (j >> 1) & 1, p.status));
      if (!ok) break;
      umma::fence_after_sync();
      float x[kTcBN];
      {
        uint32_t r[kTcBN / 16][16];
#pragma unroll
        for (int c = 0; c < kTcBN / 16; ++c) umma::tmem_ld16(tmem + lane_addr + b * kTcBN + c * 16, r[c]);
#pragma unroll
        for (int c = 0; c < kTcBN / 16; ++c) {
          tmem_wait_ld_regs(r[c]);
#pragma unroll
          for (int e = 0; e < 16; ++e) x[c * 16 + e] = __uint_as_float(r[c][e]);
        }
      }
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      // mask (causal on the diagonal block, keys past T), scale to base 2
      const int k0 = j * kTcBN;
      const int klim = min(p.T - 1, qrow);             // last valid key of this row
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTcBN; ++c) {
        x[c] = k0 + c <= klim ? x[c] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, x[c]);
      }
      const bool grow = mx > m_run + 8.f;
      if (__any_sync(0xffffffffu, grow)) {
        const float alpha = !grow ? 1.f : (m_run == -INFINITY ? 0.f : dec_exp2(m_run - mx));
        if (grow) {
          l_run *= alpha;
          m_run = mx;
        }
        if (j > 0) {
          // O holds P_0..P_{j-1} V: wait for the last of those, rescale the row in place
          ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.status));
          if (!ok) break;
          umma::fence_after_sync();
#pragma unroll
          for (int c = 0; c < HD / 16; ++c) {
            uint32_t r[16];
            umma::tmem_ld16(tmem + lane_addr + 2 * kTcBN + c * 16, r);
            tmem_wait_ld_regs(r);
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            umma::tmem_st16(tmem + lane_addr + 2 * kTcBN + c * 16, r);
          }
          umma::tmem_wait_st();
        }
      }
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kTcBN; ++c) {
        x[c] = m_run == -INFINITY ? 0.f : dec_exp2(x[c] - m_run);
        rs += x[c];
      }
      l_run += rs;
      // P buffer b was last read by O += P_{j-2} V_{j-2}
      if (j >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[b], ((j - 2) >> 1) & 1, p.status));
        if (!ok) break;
      }
      uint8_t* prow = sm + L::kP + b * 2 * L::kRegion + row * 128;
#pragma unroll
      for (int ch = 0; ch < kTcBN / 8; ++ch) {
        uint4 v;
        v.x = pack_h2(x[ch * 8 + 0], x[ch * 8 + 1]);
        v.y = pack_h2(x[ch * 8 + 2], x[ch * 8 + 3]);
        v.z = pack_h2(x[ch * 8 + 4], x[ch * 8 + 5]);
        v.w = pack_h2(x[ch * 8 + 6], x[ch * 8 + 7]);
        const int region = ch >> 3, c16 = ch & 7;
        *reinterpret_cast<uint4*>(prow + region * L::kRegion + ((c16 ^ (row & 7)) << 4)) = v;
      }
      umma::fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1, p.status));
    if (ok) {
      umma::fence_after_sync();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      float* dst = nullptr;
      if (qrow < p.T) {
        if (!p.scatter) {
          dst = p.out + static_cast<int64_t>(qrow) * p.nq * HD + static_cast<int64_t>(h) * HD;
        } else {
          // NVLink peer stores into the owning rank's output rows
          dst = p.out_peers[qrow / p.rows_per_rank] +
                static_cast<int64_t>(qrow % p.rows_per_rank) * p.nq_total * HD + static_cast<int64_t>(p.head_off + h) * HD;
        }
      }
#pragma unroll
      for (int c = 0; c < HD / 16; ++c) {
        uint32_t r[16];
        umma::tmem_ld16(tmem + lane_addr + 2 * kTcBN + c * 16, r);
        tmem_wait_ld_regs(r);
        if (dst != nullptr) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            *reinterpret_cast<float4*>(dst + c * 16 + 4 * e) =
                make_float4(__uint_as_float(r[4 * e]) * inv, __uint_as_float(r[4 * e + 1]) * inv,
                            __uint_as_float(r[4 * e + 2]) * inv, __uint_as_float(r[4 * e + 3]) * inv);
        }
      }
    }
    umma::fence_before_sync();
  }
  __syncthreads();
  if (warp == 0) {
    mbar_wait(mma_done, 0, nullptr, 500000000ull);   // no MMA still uses tensor memory
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, kTcTmemCols);
  }
}

}  // namespace attn
}  // namespace pyre

using namespace pyre;
using namespace pyre::attn;

extern "C" int pyre_rms_norm(const float* x, int rows, int H, const float* w, double eps, float* out, void* stream) {
  PYRE_CHECK_ARG(x != nullptr && w != nullptr && out != nullptr, "pyre_rms_norm: null pointer");
  PYRE_CHECK_ARG(rows >= 0 && H >= 1, "pyre_rms_norm: bad sizes");
  if (rows == 0) return PYRE_OK;
  rms_norm_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, w, out, H, eps);
  PYRE_LAUNCH_CHECK("rms_norm_kernel");
  return PYRE_OK;
}

extern "C" int pyre_add_rms_norm(const float* x, const float* delta, int rows, int H, const float* w, double eps,
                                 float* h, float* norm, void* stream) {
  PYRE_CHECK_ARG(x != nullptr && delta != nullptr && h != nullptr, "pyre_add_rms_norm: null pointer");
  PYRE_CHECK_ARG((norm == nullptr) == (w == nullptr), "pyre_add_rms_norm: norm and w go together");
  PYRE_CHECK_ARG(rows >= 0 && H >= 1, "pyre_add_rms_norm: bad sizes");
  if (rows == 0) return PYRE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto a16 = [](const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const int n4 = H / 4;
  if (H % 4 == 0 && n4 <= 1024 * kNormVec && a16(x) && a16(delta) && a16(h) && a16(w) && a16(norm)) {
    int threads = (n4 + kNormVec - 1) / kNormVec;
    threads = std::min(1024, std::max(32, (threads + 31) / 32 * 32));
    PYRE_CUDA_TRY(launch_pdl(add_rms_norm_vec_kernel, dim3(static_cast<unsigned>(rows)), dim3(threads), 0, s, x,
                             delta, h, w, norm, H, eps));
    return PYRE_OK;
  }
  PYRE_CUDA_TRY(launch_pdl(add_rms_norm_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, s, x, delta, h, w,
                           norm, H, eps));
  return PYRE_OK;
}

extern "C" int pyre_softmax_rows(const float* x, int64_t rows, int cols, float* out, void* stream) {
  PYRE_CHECK_ARG(x != nullptr && out != nullptr, "pyre_softmax_rows: null pointer");
  PYRE_CHECK_ARG(rows >= 0 && rows <= 0x7fffffff && cols >= 1, "pyre_softmax_rows: bad sizes");
  if (rows == 0) return PYRE_OK;
  softmax_rows_kernel<<<static_cast<int>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, out, cols);
  PYRE_LAUNCH_CHECK("softmax_rows_kernel");
  return PYRE_OK;
}

extern "C" int pyre_rope_table(double theta, double rope_fraction, int hd, int n_pos, float* host_out) {
  PYRE_CHECK_ARG(host_out != nullptr && hd >= 1 && n_pos >= 1 && theta > 0.0, "pyre_rope_table: bad arguments");
  const int dims = static_cast<int>(static_cast<double>(hd) * rope_fraction);
  PYRE_CHECK_ARG(dims <= hd && dims / 2 <= kRopeMaxHalf, "pyre_rope_table: rope_fraction must be in [0, 1]");
  const int half = dims >= 2 ? dims / 2 : 0;
  for (int i = 0; i < half; ++i) {
    const double freq = 1.0 / std::pow(theta, static_cast<double>(2 * i) / static_cast<double>(dims));
    for (int p = 0; p < n_pos; ++p) {
      const double ang = static_cast<double>(p) * freq;
      host_out[(static_cast<int64_t>(p) * half + i) * 2] = static_cast<float>(std::cos(ang));
      host_out[(static_cast<int64_t>(p) * half + i) * 2 + 1] = static_cast<float>(std::sin(ang));
    }
  }
  return PYRE_OK;
}

extern "C" int pyre_rope_kv_append(const float* q, const float* k, const float* v, int64_t q_stride,
                                   int64_t kv_stride, int T, int nq, int nkv, int hd,
                                   int start_pos, const float* rope_table, double rope_fraction, uint16_t* q_out,
                                   uint16_t* k_cache, uint16_t* v_cache, int max_t, void* stream) {
  PYRE_CHECK_ARG(q && k && v && q_out && k_cache && v_cache, "pyre_rope_kv_append: null pointer");
  PYRE_CHECK_ARG(T >= 1 && nq >= 1 && nkv >= 1 && hd >= 2 && nq % nkv == 0, "pyre_rope_kv_append: bad head counts");
  PYRE_CHECK_ARG(start_pos >= 0 && start_pos + T <= max_t, "pyre_rope_kv_append: positions beyond the cache");
  PYRE_CHECK_ARG(q_stride >= static_cast<int64_t>(nq) * hd && kv_stride >= static_cast<int64_t>(nkv) * hd,
                 "pyre_rope_kv_append: row strides smaller than the heads");
  const int dims = static_cast<int>(static_cast<double>(hd) * rope_fraction);
  PYRE_CHECK_ARG(dims <= hd && dims / 2 <= kRopeMaxHalf, "pyre_rope_kv_append: rope_fraction must be in [0, 1]");
  PYRE_CHECK_ARG(rope_table != nullptr || dims < 2, "pyre_rope_kv_append: null RoPE table");
  const int half = dims >= 2 ? dims / 2 : 0;
  const bool vec = (hd == 64 || hd == 128) && half % 4 == 0 && q_stride % 4 == 0 && kv_stride % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(k) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(v) % 16 == 0 && reinterpret_cast<uintptr_t>(q_out) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(k_cache) % 8 == 0 && reinterpret_cast<uintptr_t>(v_cache) % 8 == 0 &&
                   (half == 0 || reinterpret_cast<uintptr_t>(rope_table) % 16 == 0);
  if (vec) {
    const float2* tab = reinterpret_cast<const float2*>(rope_table);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (hd == 64)
      rope_append_vec_kernel<64><<<T, 256, 0, st>>>(q, k, v, q_stride, kv_stride, T, nq, nkv, start_pos, tab, half,
                                                    reinterpret_cast<__half*>(q_out), reinterpret_cast<__half*>(k_cache),
                                                    reinterpret_cast<__half*>(v_cache), max_t);
    else
      rope_append_vec_kernel<128><<<T, 256, 0, st>>>(q, k, v, q_stride, kv_stride, T, nq, nkv, start_pos, tab, half,
                                                     reinterpret_cast<__half*>(q_out), reinterpret_cast<__half*>(k_cache),
                                                     reinterpret_cast<__half*>(v_cache), max_t);
    PYRE_LAUNCH_CHECK("rope_append_vec_kernel");
    return PYRE_OK;
  }
  dim3 grid(T, (nq + nkv + kRopeHeadsPerCta - 1) / kRopeHeadsPerCta);
  rope_append_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, q_stride, kv_stride, T, nq, nkv, hd, start_pos, reinterpret_cast<const float2*>(rope_table),
      dims < 2 ? 0 : dims, reinterpret_cast<__half*>(q_out),
      reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache), max_t);
  PYRE_LAUNCH_CHECK("rope_append_kernel");
  return PYRE_OK;
}

namespace pyre {
namespace attn {
// Cluster size C: the largest power of two <= 8 that leaves every CTA kDecMinChunk positions.
inline int decode_cluster(int t) {
  int c = 1;
  while (c < kDecCluster && 2 * c * kDecMinChunk <= t) c *= 2;
  return c;
}
// Up to kDecSingleCluster positions one cluster per kv head adds all partials in distributed
// shared memory; longer caches take X clusters of 4 (twice as many of them fit on the device
// at once as clusters of 8) and add the X cluster partials through the workspace.
constexpr int kDecSingleCluster = 6144;
constexpr int kDecLongCluster = 4;
inline int decode_max_groups(int t) {
  return t <= kDecSingleCluster ? 1 : std::min(kDecMaxGroups, (t + kDecGroupChunk - 1) / kDecGroupChunk);
}
inline int64_t decode_counter_bytes(int nkv) { return (static_cast<int64_t>(nkv) * 4 + 255) / 256 * 256; }
inline int64_t decode_group_bytes(int nq, int nkv, int hd) {
  const int rep = nq / nkv;
  return static_cast<int64_t>(2 * rep + rep * hd) * 4;
}

// Clusters of C CTAs the device runs at once (one CTA per SM).
template <int HD>
int decode_active_clusters(int C, int* n) {
  static std::mutex mu;
  static int cached[64][4] = {};
  int dev = 0;
  PYRE_CUDA_TRY(cudaGetDevice(&dev));
  const int slot = C == 8 ? 3 : C == 4 ? 2 : C == 2 ? 1 : 0;
  std::lock_guard<std::mutex> lock(mu);
  int& c = cached[dev & 63][slot];
  if (c == 0) {
    int rc = set_smem_limit(reinterpret_cast<const void*>(attn_decode_kernel<HD, true>), dec_dyn_bytes<HD>(kDecMaxRep));
    if (rc) return rc;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(C), 1, 1);
    cfg.blockDim = dim3(kDecThreads, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(dec_dyn_bytes<HD>(kDecMaxRep));
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(C);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    PYRE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&c, attn_decode_kernel<HD, true>, &cfg));
    c = std::max(1, c);
  }
  *n = c;
  return PYRE_OK;
}

// Splits S = C * X of the cache per kv head, with the grid in one wave.
template <int HD>
int decode_splits(int nkv, int t, int* C, int* X) {
  *C = decode_cluster(t);
  *X = 1;
  if (t <= kDecSingleCluster) return PYRE_OK;
  int n = 0;
  int rc = decode_active_clusters<HD>(kDecLongCluster, &n);
  if (rc) return rc;
  const int x = std::min(decode_max_groups(t), n / nkv);
  if (x >= 2) {
    *C = kDecLongCluster;
    *X = x;
  }
  return PYRE_OK;
}
}  // namespace attn
}  // namespace pyre

extern "C" int pyre_attn_decode_workspace_bytes(int nq, int nkv, int hd, int t, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr && nq >= 1 && nkv >= 1 && hd >= 1 && t >= 1 && nq % nkv == 0,
                 "pyre_attn_decode_workspace_bytes: bad args");
  *bytes = decode_counter_bytes(nkv) + static_cast<int64_t>(nkv) * decode_max_groups(t) * decode_group_bytes(nq, nkv, hd);
  return PYRE_OK;
}

namespace pyre {
namespace attn {
// Shared by the attention-only call and the fused decode step: splits, workspace check,
// cluster launch.
template <int HD, bool FUSED>
int launch_decode(DecodeParams p, void* workspace, int64_t ws_bytes, cudaStream_t stream) {
  int C = 1, X = 1;
  if (p.nkv_seq <= 0) p.nkv_seq = p.nkv;
  // the split plan of ONE sequence, so a batched step splits every sequence's cache exactly as
  // a single-sequence step would (same partial sums in the same order)
  int rc = decode_splits<HD>(p.nkv_seq, p.t, &C, &X);
  if (rc) return rc;
  const int64_t need = decode_counter_bytes(p.nkv) + static_cast<int64_t>(p.nkv) * X * decode_group_bytes(p.nq, p.nkv, HD);
  if (X > 1)
    PYRE_CHECK_ARG(workspace != nullptr && reinterpret_cast<uintptr_t>(workspace) % 16 == 0 && ws_bytes >= need,
                   "pyre_attn_decode: workspace missing, misaligned or smaller than pyre_attn_decode_workspace_bytes");
  p.count = static_cast<unsigned*>(workspace);
  p.part = X > 1 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + decode_counter_bytes(p.nkv)) : nullptr;
  p.scale2 = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
  rc = set_smem_limit(reinterpret_cast<const void*>(attn_decode_kernel<HD, FUSED>), dec_dyn_bytes<HD>(kDecMaxRep));
  if (rc) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(C * X), static_cast<unsigned>(p.nkv), 1);
  cfg.blockDim = dim3(kDecThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(dec_dyn_bytes<HD>(p.nq / p.nkv));
  cfg.stream = stream;
  cudaLaunchAttribute attr[2]{};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see pdl_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  PYRE_CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_decode_kernel<HD, FUSED>, p));
  PYRE_LAUNCH_CHECK("attn_decode_kernel");
  return PYRE_OK;
}
}  // namespace attn
}  // namespace pyre

extern "C" int pyre_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int t, int nq,
                                int nkv, int hd, int max_t, int mask_lo, int mask_hi, float* out, void* workspace,
                                int64_t ws_bytes, void* stream) {
  PYRE_CHECK_ARG(q && k_cache && v_cache && out, "pyre_attn_decode: null pointer");
  PYRE_CHECK_ARG(t >= 1 && t <= max_t && nkv >= 1 && nq % nkv == 0 && nq / nkv <= kDecMaxRep,
                 "pyre_attn_decode: bad sizes (at most 8 query heads per kv head)");
  PYRE_CHECK_ARG(hd == 64 || hd == 128, "pyre_attn_decode: head dim must be 64 or 128");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(k_cache) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(v_cache) % 16 == 0,
                 "pyre_attn_decode: q and the caches must be 16-byte aligned");
  DecodeParams p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.kc = reinterpret_cast<const __half*>(k_cache);
  p.vc = reinterpret_cast<const __half*>(v_cache);
  p.out = out;
  p.nq = nq;
  p.nkv = nkv;
  p.t = t;
  p.max_t = max_t;
  p.mask_lo = mask_lo;
  p.mask_hi = mask_hi;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return hd == 64 ? launch_decode<64, false>(p, workspace, ws_bytes, st)
                  : launch_decode<128, false>(p, workspace, ws_bytes, st);
}

namespace pyre {
namespace attn {
// The fused decode step; pos_dev null: position start_pos; else the position is read from
// *pos_dev on the device and start_pos only plans the grid.
int decode_step(const float* q, const float* k, const float* v, int start_pos, const int* pos_dev,
                const float* rope_table, double rope_fraction, int nq, int nkv, int hd, uint16_t* k_cache,
                uint16_t* v_cache, int max_t, int mask_lo, int mask_hi, float* out, void* workspace,
                int64_t ws_bytes, void* stream, const char* f) {
  const std::string fn(f);
  PYRE_CHECK_ARG(q && k && v && k_cache && v_cache && out, fn + ": null pointer");
  PYRE_CHECK_ARG(start_pos >= 0 && start_pos < max_t && nkv >= 1 && nq % nkv == 0 && nq / nkv <= kDecMaxRep,
                 fn + ": bad sizes (cache full, or more than 8 query heads per kv head)");
  PYRE_CHECK_ARG(hd == 64 || hd == 128, fn + ": head dim must be 64 or 128");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(k_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(v_cache) % 16 == 0,
                 fn + ": the caches must be 16-byte aligned");
  const int dims = static_cast<int>(static_cast<double>(hd) * rope_fraction);
  PYRE_CHECK_ARG(dims >= 0 && dims <= hd, fn + ": rope_fraction must be in [0, 1]");
  const int half = dims >= 2 ? dims / 2 : 0;
  PYRE_CHECK_ARG(rope_table != nullptr || half == 0, fn + ": null RoPE table");
  DecodeParams p{};
  p.kc = reinterpret_cast<const __half*>(k_cache);
  p.vc = reinterpret_cast<const __half*>(v_cache);
  p.kw = reinterpret_cast<__half*>(k_cache);
  p.vw = reinterpret_cast<__half*>(v_cache);
  p.qf = q;
  p.kf = k;
  p.vf = v;
  p.rope = half ? reinterpret_cast<const float2*>(rope_table) + static_cast<int64_t>(start_pos) * half : nullptr;
  p.rope_base = reinterpret_cast<const float2*>(rope_table);
  p.pos_dev = pos_dev;
  p.half = half;
  p.out = out;
  p.nq = nq;
  p.nkv = nkv;
  p.t = start_pos + 1;
  p.max_t = max_t;
  p.mask_lo = mask_lo;
  p.mask_hi = mask_hi;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return hd == 64 ? launch_decode<64, true>(p, workspace, ws_bytes, st)
                  : launch_decode<128, true>(p, workspace, ws_bytes, st);
}
}  // namespace attn
}  // namespace pyre

extern "C" int pyre_attn_decode_step(const float* q, const float* k, const float* v, int start_pos,
                                     const float* rope_table, double rope_fraction, int nq, int nkv, int hd,
                                     uint16_t* k_cache, uint16_t* v_cache, int max_t, int mask_lo, int mask_hi,
                                     float* out, void* workspace, int64_t ws_bytes, void* stream) {
  return attn::decode_step(q, k, v, start_pos, nullptr, rope_table, rope_fraction, nq, nkv, hd, k_cache, v_cache,
                           max_t, mask_lo, mask_hi, out, workspace, ws_bytes, stream, "pyre_attn_decode_step");
}

extern "C" int pyre_attn_decode_step_batch(const float* q, const float* k, const float* v, int64_t qkv_stride,
                                           int B, const int* pos_dev, int plan_pos, const float* rope_table,
                                           double rope_fraction, int nq, int nkv, int hd, uint16_t* k_cache,
                                           uint16_t* v_cache, int max_t, float* out, void* workspace,
                                           int64_t ws_bytes, void* stream) {
  PYRE_CHECK_ARG(B >= 1 && B <= 64, "pyre_attn_decode_step_batch: 1 <= B <= 64 sequences");
  PYRE_CHECK_ARG(qkv_stride >= static_cast<int64_t>(nq + 2 * nkv) * hd,
                 "pyre_attn_decode_step_batch: row stride smaller than the q, k and v of a token");
  PYRE_CHECK_ARG(q && k && v && k_cache && v_cache && out, "pyre_attn_decode_step_batch: null pointer");
  PYRE_CHECK_ARG(plan_pos >= 0 && plan_pos < max_t && nkv >= 1 && nq % nkv == 0 && nq / nkv <= kDecMaxRep,
                 "pyre_attn_decode_step_batch: bad sizes (cache full, or more than 8 query heads per kv head)");
  PYRE_CHECK_ARG(hd == 64 || hd == 128, "pyre_attn_decode_step_batch: head dim must be 64 or 128");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(k_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(v_cache) % 16 == 0,
                 "pyre_attn_decode_step_batch: the caches must be 16-byte aligned");
  const int dims = static_cast<int>(static_cast<double>(hd) * rope_fraction);
  PYRE_CHECK_ARG(dims >= 0 && dims <= hd, "pyre_attn_decode_step_batch: rope_fraction must be in [0, 1]");
  const int half = dims >= 2 ? dims / 2 : 0;
  PYRE_CHECK_ARG(rope_table != nullptr || half == 0, "pyre_attn_decode_step_batch: null RoPE table");
  DecodeParams p{};
  p.kc = reinterpret_cast<const __half*>(k_cache);
  p.vc = reinterpret_cast<const __half*>(v_cache);
  p.kw = reinterpret_cast<__half*>(k_cache);
  p.vw = reinterpret_cast<__half*>(v_cache);
  p.qf = q;
  p.kf = k;
  p.vf = v;
  p.rope = half ? reinterpret_cast<const float2*>(rope_table) + static_cast<int64_t>(plan_pos) * half : nullptr;
  p.rope_base = reinterpret_cast<const float2*>(rope_table);
  p.pos_dev = pos_dev;
  p.half = half;
  p.out = out;
  p.nq = nq * B;
  p.nkv = nkv * B;
  p.nkv_seq = nkv;
  p.q_bstride = qkv_stride;
  p.kv_bstride = qkv_stride;
  p.t = plan_pos + 1;
  p.max_t = max_t;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return hd == 64 ? launch_decode<64, true>(p, workspace, ws_bytes, st)
                  : launch_decode<128, true>(p, workspace, ws_bytes, st);
}

extern "C" int pyre_attn_decode_step_dev(const float* q, const float* k, const float* v, const int* pos_dev,
                                         int plan_pos, const float* rope_table, double rope_fraction, int nq, int nkv,
                                         int hd, uint16_t* k_cache, uint16_t* v_cache, int max_t, int mask_lo,
                                         int mask_hi, float* out, void* workspace, int64_t ws_bytes, void* stream) {
  PYRE_CHECK_ARG(pos_dev != nullptr, "pyre_attn_decode_step_dev: null position");
  return attn::decode_step(q, k, v, plan_pos, pos_dev, rope_table, rope_fraction, nq, nkv, hd, k_cache, v_cache,
                           max_t, mask_lo, mask_hi, out, workspace, ws_bytes, stream, "pyre_attn_decode_step_dev");
}

namespace pyre {
namespace attn {
template <int HD>
int launch_prefill_tc(const PrefillParams& pp, cudaStream_t s) {
  using L = TcLayout<HD>;
  static int* status_of[64] = {};
  int dev = 0;
  PYRE_CUDA_TRY(cudaGetDevice(&dev));
  int*& status = status_of[dev & 63];
  if (status == nullptr) PYRE_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_attn_status));
  PrefillTcParams p{};
  const auto f16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  int rc = make_tmap_3d(&p.tq, pp.q, f16, 2, HD, static_cast<uint64_t>(pp.T), static_cast<uint64_t>(pp.nq), HD * 2,
                        static_cast<uint64_t>(pp.T) * HD * 2, 64, kTcBM, sw);
  if (!rc)
    rc = make_tmap_3d(&p.tk, pp.kc, f16, 2, HD, static_cast<uint64_t>(pp.T), static_cast<uint64_t>(pp.nkv), HD * 2,
                      static_cast<uint64_t>(pp.max_t) * HD * 2, 64, kTcBN, sw);
  if (!rc)
    rc = make_tmap_3d(&p.tv, pp.vc, f16, 2, HD, static_cast<uint64_t>(pp.T), static_cast<uint64_t>(pp.nkv), HD * 2,
                      static_cast<uint64_t>(pp.max_t) * HD * 2, 64, kTcBN, sw);
  if (rc) return rc;
  p.out = pp.out;
  p.T = pp.T;
  p.nq = pp.nq;
  p.nkv = pp.nkv;
  p.scale_log2 = pp.scale_log2;
  p.scatter = pp.scatter;
  p.rows_per_rank = pp.rows_per_rank;
  p.head_off = pp.head_off;
  p.nq_total = pp.nq_total;
  for (int i = 0; i < 16; ++i) p.out_peers[i] = pp.out_peers[i];
  p.status = status;
  rc = set_smem_limit(reinterpret_cast<const void*>(attn_prefill_tc_kernel<HD>), L::kBytes);
  if (rc) return rc;
  const dim3 grid(static_cast<unsigned>(pp.nq), static_cast<unsigned>((pp.T + kTcBM - 1) / kTcBM));
  attn_prefill_tc_kernel<HD><<<grid, kTcThreads, L::kBytes, s>>>(p);
  PYRE_LAUNCH_CHECK("attn_prefill_tc_kernel");
  return PYRE_OK;
}

int launch_prefill(PrefillParams p, int hd, cudaStream_t s) {
  return hd == 64 ? launch_prefill_tc<64>(p, s) : launch_prefill_tc<128>(p, s);
}

}  // namespace attn
}  // namespace pyre

extern "C" int pyre_attn_status(int* status) {
  PYRE_CHECK_ARG(status != nullptr, "pyre_attn_status: null pointer");
  int v = 0;
  PYRE_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(int)));
  if (v != PYRE_OK) {
    const int zero = 0;
    PYRE_CUDA_TRY(cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)));
  }
  *status = v;
  return PYRE_OK;
}

extern "C" int pyre_attn_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int T, int nq,
                                 int nkv, int hd, int max_t, float* out, void* stream) {
  PYRE_CHECK_ARG(q && k_cache && v_cache && out, "pyre_attn_prefill: null pointer");
  PYRE_CHECK_ARG(T >= 1 && T <= max_t && nkv >= 1 && nq % nkv == 0, "pyre_attn_prefill: bad sizes");
  PYRE_CHECK_ARG(hd == 64 || hd == 128, "pyre_attn_prefill: head dim must be 64 or 128");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(k_cache) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(v_cache) % 16 == 0,
                 "pyre_attn_prefill: q and the caches must be 16-byte aligned");
  PrefillParams p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.kc = reinterpret_cast<const __half*>(k_cache);
  p.vc = reinterpret_cast<const __half*>(v_cache);
  p.out = out;
  p.T = T;
  p.nq = nq;
  p.nkv = nkv;
  p.max_t = max_t;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(hd)));
  return launch_prefill(p, hd, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------
// Ulysses sequence parallelism inside one box (P ranks, one GPU each). Rank r owns tokens
// [r*S/P, (r+1)*S/P) and, for attention, q heads [r*nq/P, ..) and kv heads [r*nkv/P, ..).
// Every rank holds one buffer (allocated with pyre_comm_alloc, mapped by its peers):
//   qf  f16 [nq/P, S, hd]      rotated queries of the owned heads, whole sequence
//   kf  f16 [nkv/P, S, hd]     KV cache of the owned kv heads, whole sequence
//   vf  f16 [nkv/P, S, hd]
//   ao  f32 [S/P, nq*hd]       attention output of the owned tokens, all heads
//   flags u32 [2][16], epoch, status (the last two only used locally)
// The QKV "all-gather" is fused into RoPE: each rank rotates its tokens and stores every
// head straight into the owner's qf / kf / vf over NVLink. The output "scatter" is fused
// into the attention epilogue, which stores each row into the owner's ao. A flag barrier
// (release / acquire at system scope, bounded waits) separates the phases.
namespace pyre {
namespace attn {

constexpr int kUlyMaxWorld = 16;

struct UlyLayout {
  int64_t q, k, v, ao, flags, epoch, status, total;
};

inline int64_t a256(int64_t b) { return (b + 255) / 256 * 256; }

UlyLayout uly_layout(int S, int P, int nq, int nkv, int hd) {
  UlyLayout L{};
  L.q = 0;
  L.k = L.q + a256(static_cast<int64_t>(nq / P) * S * hd * 2);
  L.v = L.k + a256(static_cast<int64_t>(nkv / P) * S * hd * 2);
  L.ao = L.v + a256(static_cast<int64_t>(nkv / P) * S * hd * 2);
  L.flags = L.ao + a256(static_cast<int64_t>(S / P) * nq * hd * 4);
  L.epoch = L.flags + 2 * kUlyMaxWorld * 4;
  L.status = L.epoch + 4;
  L.total = a256(L.status + 4);
  return L;
}

struct UlyPeers {
  char* buf[kUlyMaxWorld];
};

__global__ void __launch_bounds__(256) ulysses_rope_scatter_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, int64_t q_stride,
    int64_t kv_stride, int S_local, int seq_off, int S, int nq, int nkv, int hd, const float2* __restrict__ table,
    int dims, int P,
    UlyPeers peers, int64_t off_q, int64_t off_k, int64_t off_v) {
  __shared__ float cs[kRopeMaxHalf], sn[kRopeMaxHalf];
  const int t = blockIdx.x;
  const int pos = seq_off + t;
  const int half = dims >= 2 ? dims / 2 : 0;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float2 c = table[static_cast<int64_t>(pos) * half + j];
    cs[j] = c.x;
    sn[j] = c.y;
  }
  __syncthreads();
  const int qpr = nq / P, kpr = nkv / P;
  for (int e = threadIdx.x; e < (nq + nkv) * hd; e += blockDim.x) {
    const int hh = e / hd, i = e - hh * hd;
    const bool is_q = hh < nq;
    const int h = is_q ? hh : hh - nq;
    const float* src = is_q ? q + t * q_stride + static_cast<int64_t>(h) * hd : k + t * kv_stride + static_cast<int64_t>(h) * hd;
    float r;
    if (i < 2 * half) {
      const int jj = i < half ? i : i - half;
      const float x1 = src[jj], x2 = src[jj + half];
      r = i < half ? rope_lo(x1, x2, cs[jj], sn[jj]) : rope_hi(x1, x2, cs[jj], sn[jj]);
    } else {
      r = src[i];
    }
    const __half hv = __float2half_rn(clip1000(r));
    const int owner = is_q ? h / qpr : h / kpr;
    const int hl = is_q ? h - owner * qpr : h - owner * kpr;
    __half* dst = reinterpret_cast<__half*>(peers.buf[owner] + (is_q ? off_q : off_k));
    dst[(static_cast<int64_t>(hl) * S + pos) * hd + i] = hv;
  }
  for (int e = threadIdx.x; e < nkv * hd; e += blockDim.x) {
    const int h = e / hd, i = e - h * hd;
    const float x = v[t * kv_stride + static_cast<int64_t>(h) * hd + i];
    const int owner = h / kpr, hl = h - owner * kpr;
    __half* dst = reinterpret_cast<__half*>(peers.buf[owner] + off_v);
    dst[(static_cast<int64_t>(hl) * S + pos) * hd + i] = __float2half_rn(fminf(fmaxf(x, -1000.f), 1000.f));
  }
}

// Phase barrier: publish this rank's flag to every peer (after a system-scope fence that
// orders the preceding kernels' peer stores), then wait (bounded) for every peer's flag.
// The epoch of a call is the local epoch word + 1; phase 1 stores it back.
__global__ void ulysses_barrier_kernel(UlyPeers peers, int rank, int P, int phase, int64_t off_flags,
                                       int64_t off_epoch, int64_t off_status, uint64_t timeout_ns) {
  char* mine = peers.buf[rank];
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(mine + off_epoch) + 1u;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < P) {
    uint32_t* f = reinterpret_cast<uint32_t*>(peers.buf[threadIdx.x] + off_flags) + phase * kUlyMaxWorld + rank;
    st_release_sys(f, epoch);
  }
  if (threadIdx.x < P) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + off_flags) + phase * kUlyMaxWorld + threadIdx.x;
    if (!wait_flag_eq(f, epoch, timeout_ns)) atomicExch(reinterpret_cast<int*>(mine + off_status), PYRE_ETIMEOUT);
  }
  __syncthreads();
  if (phase == 1 && threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(mine + off_epoch) = epoch;
}

int uly_peers(void* const* bufs, int P, UlyPeers* out) {
  PYRE_CHECK_ARG(bufs != nullptr && P >= 1 && P <= kUlyMaxWorld, "Ulysses: 1..16 ranks and their buffers");
  for (int i = 0; i < P; ++i) {
    PYRE_CHECK_ARG(bufs[i] != nullptr, "Ulysses: null peer buffer");
    out->buf[i] = static_cast<char*>(bufs[i]);
  }
  return PYRE_OK;
}

int uly_check_shape(int S, int P, int nq, int nkv, int hd) {
  PYRE_CHECK_ARG(P >= 1 && P <= kUlyMaxWorld && S >= P && S % P == 0, "Ulysses: S must be a multiple of P");
  PYRE_CHECK_ARG(nq % P == 0 && nkv % P == 0 && nq % nkv == 0, "Ulysses: head counts must divide by P (and nq by nkv)");
  PYRE_CHECK_ARG(hd == 64 || hd == 128, "Ulysses: head dim must be 64 or 128");
  return PYRE_OK;
}

}  // namespace attn
}  // namespace pyre

extern "C" int pyre_ulysses_buffer_bytes(int S, int P, int nq, int nkv, int hd, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_ulysses_buffer_bytes: null bytes");
  int rc = uly_check_shape(S, P, nq, nkv, hd);
  if (rc) return rc;
  *bytes = uly_layout(S, P, nq, nkv, hd).total;
  return PYRE_OK;
}

extern "C" int pyre_ulysses_rope_scatter(void* const* bufs, int rank, int P, const float* q, const float* k,
                                         const float* v, int64_t q_stride, int64_t kv_stride, int S, int nq, int nkv,
                                         int hd, const float* rope_table, double rope_fraction, void* stream) {
  int rc = uly_check_shape(S, P, nq, nkv, hd);
  if (rc) return rc;
  PYRE_CHECK_ARG(q && k && v && rank >= 0 && rank < P, "pyre_ulysses_rope_scatter: bad arguments");
  PYRE_CHECK_ARG(q_stride >= static_cast<int64_t>(nq) * hd && kv_stride >= static_cast<int64_t>(nkv) * hd,
                 "pyre_ulysses_rope_scatter: row strides smaller than the heads");
  const int dims = static_cast<int>(static_cast<double>(hd) * rope_fraction);
  PYRE_CHECK_ARG(dims <= hd && dims / 2 <= kRopeMaxHalf && (rope_table != nullptr || dims < 2),
                 "pyre_ulysses_rope_scatter: bad RoPE parameters");
  UlyPeers peers{};
  rc = uly_peers(bufs, P, &peers);
  if (rc) return rc;
  const UlyLayout L = uly_layout(S, P, nq, nkv, hd);
  const int S_local = S / P;
  ulysses_rope_scatter_kernel<<<S_local, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, q_stride, kv_stride, S_local, rank * S_local, S, nq, nkv, hd,
      reinterpret_cast<const float2*>(rope_table), dims < 2 ? 0 : dims, P, peers,
      L.q, L.k, L.v);
  PYRE_LAUNCH_CHECK("ulysses_rope_scatter_kernel");
  return PYRE_OK;
}

extern "C" int pyre_ulysses_barrier(void* const* bufs, int rank, int P, int S, int nq, int nkv, int hd, int phase,
                                    uint64_t timeout_ns, void* stream) {
  int rc = uly_check_shape(S, P, nq, nkv, hd);
  if (rc) return rc;
  PYRE_CHECK_ARG(rank >= 0 && rank < P && (phase == 0 || phase == 1), "pyre_ulysses_barrier: bad rank or phase");
  UlyPeers peers{};
  rc = uly_peers(bufs, P, &peers);
  if (rc) return rc;
  const UlyLayout L = uly_layout(S, P, nq, nkv, hd);
  ulysses_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(peers, rank, P, phase, L.flags, L.epoch,
                                                                            L.status, timeout_ns);
  PYRE_LAUNCH_CHECK("ulysses_barrier_kernel");
  return PYRE_OK;
}

extern "C" int pyre_ulysses_attention(void* const* bufs, int rank, int P, int S, int nq, int nkv, int hd,
                                      void* stream) {
  int rc = uly_check_shape(S, P, nq, nkv, hd);
  if (rc) return rc;
  PYRE_CHECK_ARG(rank >= 0 && rank < P, "pyre_ulysses_attention: bad rank");
  UlyPeers peers{};
  rc = uly_peers(bufs, P, &peers);
  if (rc) return rc;
  const UlyLayout L = uly_layout(S, P, nq, nkv, hd);
  PrefillParams p{};
  char* mine = peers.buf[rank];
  p.q = reinterpret_cast<const __half*>(mine + L.q);
  p.kc = reinterpret_cast<const __half*>(mine + L.k);
  p.vc = reinterpret_cast<const __half*>(mine + L.v);
  p.out = nullptr;
  p.T = S;
  p.nq = nq / P;
  p.nkv = nkv / P;
  p.max_t = S;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(hd)));
  p.scatter = 1;
  p.rows_per_rank = S / P;
  p.head_off = rank * (nq / P);
  p.nq_total = nq;
  for (int i = 0; i < P; ++i) p.out_peers[i] = reinterpret_cast<float*>(peers.buf[i] + L.ao);
  return launch_prefill(p, hd, static_cast<cudaStream_t>(stream));
}

// Synchronises the stream, then zeroes this rank's barrier flags, epoch and status word, so the
// ranks start again from a common state after a call that timed out (every rank calls it,
// between host barriers, with none of its Ulysses kernels in flight).
extern "C" int pyre_ulysses_reset(void* local_buf, int P, int S, int nq, int nkv, int hd, void* stream) {
  int rc = uly_check_shape(S, P, nq, nkv, hd);
  if (rc) return rc;
  PYRE_CHECK_ARG(local_buf != nullptr, "pyre_ulysses_reset: null buffer");
  const UlyLayout L = uly_layout(S, P, nq, nkv, hd);
  PYRE_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  PYRE_CUDA_TRY(cudaMemset(static_cast<char*>(local_buf) + L.flags, 0, static_cast<size_t>(L.total - L.flags)));
  PYRE_CUDA_TRY(cudaDeviceSynchronize());
  return PYRE_OK;
}

// Synchronises the stream, returns and clears this rank's status word (PYRE_OK or
// PYRE_ETIMEOUT), and copies its [S/P, nq*hd] attention output into out (device memory).
extern "C" int pyre_ulysses_finish(void* local_buf, int P, int S, int nq, int nkv, int hd, float* out, int* status,
                                   void* stream) {
  int rc = uly_check_shape(S, P, nq, nkv, hd);
  if (rc) return rc;
  PYRE_CHECK_ARG(local_buf != nullptr && status != nullptr, "pyre_ulysses_finish: null pointer");
  const UlyLayout L = uly_layout(S, P, nq, nkv, hd);
  char* mine = static_cast<char*>(local_buf);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (out != nullptr)
    PYRE_CUDA_TRY(cudaMemcpyAsync(out, mine + L.ao, static_cast<size_t>(S / P) * nq * hd * 4, cudaMemcpyDeviceToDevice, s));
  int st = 0;
  PYRE_CUDA_TRY(cudaMemcpyAsync(&st, mine + L.status, 4, cudaMemcpyDeviceToHost, s));
  PYRE_CUDA_TRY(cudaStreamSynchronize(s));
  *status = st;
  if (st != PYRE_OK) PYRE_CUDA_TRY(cudaMemset(mine + L.status, 0, 4));
  return PYRE_OK;
}
