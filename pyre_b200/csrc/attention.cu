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
//   attn_decode_kernel    flash-decoding: (kv head, chunk) CTAs, partials combined in
//                         chunk order by the last CTA of each kv head (deterministic)
//   attn_prefill_kernel   causal attention, 64 queries x 64 keys per step, f16 mma.sync with
//                         f32 accumulation and an online softmax, GQA by kv head = h / rep
#include <cmath>

#include "common.cuh"

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
// One CTA per token: the cos/sin of the token's position for the rotated half-dims are
// computed once (freq_i = 1 / theta^(2i/dims) and pos * freq_i in f64, cast to f32, as the
// reference does), then every q and k head of the token is rotated in f32 (pair (i, i+half)),
// clipped to +-1000 and stored as f16; v is clipped and appended.
constexpr int kRopeMaxHalf = 256;

__global__ void __launch_bounds__(256) rope_append_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                           const float* __restrict__ v, int64_t q_stride,
                                                           int64_t kv_stride, int T, int nq, int nkv, int hd,
                                                           int start_pos, double theta, int dims,
                                                           __half* __restrict__ q_out, __half* __restrict__ k_cache,
                                                           __half* __restrict__ v_cache, int max_t) {
  __shared__ float cs[kRopeMaxHalf], sn[kRopeMaxHalf];
  const int t = blockIdx.x;
  const int pos = start_pos + t;
  const int half = dims >= 2 ? dims / 2 : 0;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const double freq = 1.0 / pow(theta, static_cast<double>(2 * j) / static_cast<double>(dims));
    const double ang = static_cast<double>(pos) * freq;
    cs[j] = static_cast<float>(cos(ang));
    sn[j] = static_cast<float>(sin(ang));
  }
  __syncthreads();
  const int nh = nq + nkv;
  for (int e = threadIdx.x; e < nh * hd; e += blockDim.x) {
    const int hh = e / hd, i = e - hh * hd;
    const bool is_q = hh < nq;
    const int h = is_q ? hh : hh - nq;
    const float* src = is_q ? q + t * q_stride + static_cast<int64_t>(h) * hd : k + t * kv_stride + static_cast<int64_t>(h) * hd;
    float r;
    if (i < 2 * half) {
      const int jj = i < half ? i : i - half;
      const float x1 = src[jj], x2 = src[jj + half];
      r = i < half ? x1 * cs[jj] - x2 * sn[jj] : x1 * sn[jj] + x2 * cs[jj];
    } else {
      r = src[i];
    }
    r = fminf(fmaxf(r, -1000.f), 1000.f);
    if (is_q)
      q_out[(static_cast<int64_t>(h) * T + t) * hd + i] = __float2half_rn(r);
    else
      k_cache[(static_cast<int64_t>(h) * max_t + pos) * hd + i] = __float2half_rn(r);
  }
  for (int e = threadIdx.x; e < nkv * hd; e += blockDim.x) {
    const int h = e / hd, i = e - h * hd;
    const float x = v[t * kv_stride + static_cast<int64_t>(h) * hd + i];
    v_cache[(static_cast<int64_t>(h) * max_t + pos) * hd + i] = __float2half_rn(fminf(fmaxf(x, -1000.f), 1000.f));
  }
}

// ---------------------------------------------------------------------------------------
// Flash-decoding. grid (n_kv, splits), 128 threads. Each CTA scores positions
// [c0, c1) of one kv head for its rep = nq / nkv query heads, keeps the chunk's max, sum of
// exp and exp-weighted V sum per head, and the last CTA of the kv head combines the chunks
// in chunk order.
constexpr int kDecThreads = 128;
constexpr int kDecMaxChunk = 256;
constexpr int kDecMinChunk = 32;
constexpr int kDecMaxRep = 8;

struct DecodeParams {
  const __half* q;       // [nq, hd] rotated, clipped
  const __half* kc;      // [nkv, max_t, hd]
  const __half* vc;
  float* out;            // [nq * hd]
  float* part;           // [nkv, splits, rep, hd + 2]  (m, l, acc[hd])
  unsigned int* counters;// [nkv]
  int nq, nkv, hd, t, max_t, splits, chunk, mask_lo, mask_hi;
  float scale;           // 1 / sqrt(hd)
};

template <int HD>
__global__ void __launch_bounds__(kDecThreads) attn_decode_kernel(const DecodeParams p) {
  const int g = blockIdx.x, sp = blockIdx.y;
  const int rep = p.nq / p.nkv;
  const int c0 = sp * p.chunk, c1 = min(c0 + p.chunk, p.t);
  __shared__ float qs[kDecMaxRep][HD];
  __shared__ float sc[kDecMaxRep][kDecMaxChunk];
  __shared__ float stat[kDecMaxRep][2];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < rep * HD; i += kDecThreads)
    qs[i / HD][i % HD] = __half2float(p.q[(static_cast<int64_t>(g) * rep + i / HD) * HD + i % HD]);
  __syncthreads();
  const __half* kh = p.kc + static_cast<int64_t>(g) * p.max_t * HD;
  const __half* vh = p.vc + static_cast<int64_t>(g) * p.max_t * HD;
  // scores: one warp per position, lanes over hd
  for (int pos = c0 + warp; pos < c1; pos += kDecThreads / 32) {
    float kv[HD / 32];
#pragma unroll
    for (int j = 0; j < HD / 32; ++j) kv[j] = __half2float(kh[static_cast<int64_t>(pos) * HD + lane + 32 * j]);
    for (int r = 0; r < rep; ++r) {
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < HD / 32; ++j) d += qs[r][lane + 32 * j] * kv[j];
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const bool masked = pos >= p.mask_lo && pos < p.mask_hi;
      if (lane == 0) sc[r][pos - c0] = masked ? -INFINITY : d * p.scale;
    }
  }
  __syncthreads();
  // per head: chunk max and sum of exp (one warp per head)
  for (int r = warp; r < rep; r += kDecThreads / 32) {
    float m = -INFINITY;
    for (int i = lane; i < c1 - c0; i += 32) m = fmaxf(m, sc[r][i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int i = lane; i < c1 - c0; i += 32) {
      const float e = m == -INFINITY ? 0.f : expf(sc[r][i] - m);
      sc[r][i] = e;
      l += e;
    }
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      stat[r][0] = m;
      stat[r][1] = l;
    }
  }
  __syncthreads();
  // exp-weighted V sum: thread per dimension
  float* part = p.part + (static_cast<int64_t>(g) * p.splits + sp) * rep * (HD + 2);
  for (int d = threadIdx.x; d < HD; d += kDecThreads) {
    float acc[kDecMaxRep];
#pragma unroll
    for (int r = 0; r < kDecMaxRep; ++r) acc[r] = 0.f;
    for (int pos = c0; pos < c1; ++pos) {
      const float vv = __half2float(vh[static_cast<int64_t>(pos) * HD + d]);
#pragma unroll
      for (int r = 0; r < kDecMaxRep; ++r)
        if (r < rep) acc[r] += sc[r][pos - c0] * vv;
    }
    for (int r = 0; r < rep; ++r) __stcg(part + r * (HD + 2) + 2 + d, acc[r]);
  }
  if (threadIdx.x < rep) {
    __stcg(part + threadIdx.x * (HD + 2), stat[threadIdx.x][0]);
    __stcg(part + threadIdx.x * (HD + 2) + 1, stat[threadIdx.x][1]);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.counters + g, 1u);
    const int last = prev == static_cast<unsigned>(p.splits - 1);
    if (last) {
      __threadfence();
      p.counters[g] = 0u;
    }
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  // combine the chunks of this kv head in chunk order
  const float* base = p.part + static_cast<int64_t>(g) * p.splits * rep * (HD + 2);
  for (int i = threadIdx.x; i < rep * HD; i += kDecThreads) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(base + (static_cast<int64_t>(s) * rep + r) * (HD + 2)));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float* ps = base + (static_cast<int64_t>(s) * rep + r) * (HD + 2);
      const float m = __ldcg(ps);
      const float w = m == -INFINITY ? 0.f : expf(m - M);
      L += __ldcg(ps + 1) * w;
      O += __ldcg(ps + 2 + d) * w;
    }
    p.out[(static_cast<int64_t>(g) * rep + r) * HD + d] = O / L;
  }
}

// ---------------------------------------------------------------------------------------
// Causal prefill attention. grid (ceil(T / 64), nq), 128 threads (4 warps x 16 query rows).
constexpr int kPM = 64, kPN = 64;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
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

template <int HD>
struct PrefillSmem {
  static constexpr int kLd = HD + 8;   // padded row (halves): conflict-free ldmatrix
  static constexpr int kQ = kPM * kLd;
  static constexpr int kKV = kPN * kLd;
  static constexpr int kBytes = (kQ + 4 * kKV) * 2;   // Q + double-buffered K and V
};

template <int HD>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const PrefillParams p) {
  using S = PrefillSmem<HD>;
  extern __shared__ __align__(16) __half sm[];
  __half* qs = sm;
  __half* ks = sm + S::kQ;              // [2][kPN][kLd]
  __half* vs = ks + 2 * S::kKV;
  const int qb = blockIdx.x, h = blockIdx.y;
  const int g = h / (p.nq / p.nkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * kPM;
  const __half* qg = p.q + (static_cast<int64_t>(h) * p.T + q0) * HD;
  const __half* kg = p.kc + static_cast<int64_t>(g) * p.max_t * HD;
  const __half* vg = p.vc + static_cast<int64_t>(g) * p.max_t * HD;
  constexpr int kChunks = HD / 8;       // 16-byte chunks per row
  auto load_kv = [&](int kb, int buf) {
    const int k0 = kb * kPN;
    for (int i = threadIdx.x; i < kPN * kChunks; i += 128) {
      const int r = i / kChunks, c = i % kChunks;
      const bool ok = k0 + r < p.T;
      const int rr = ok ? k0 + r : 0;
      cp_async16(ks + buf * S::kKV + r * S::kLd + c * 8, kg + static_cast<int64_t>(rr) * HD + c * 8, ok);
      cp_async16(vs + buf * S::kKV + r * S::kLd + c * 8, vg + static_cast<int64_t>(rr) * HD + c * 8, ok);
    }
  };
  for (int i = threadIdx.x; i < kPM * kChunks; i += 128) {
    const int r = i / kChunks, c = i % kChunks;
    const bool ok = q0 + r < p.T;
    cp_async16(qs + r * S::kLd + c * 8, qg + static_cast<int64_t>(ok ? r : 0) * HD + c * 8, ok);
  }
  load_kv(0, 0);
  cp_async_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // rows g and g + 8 of this warp
  const int row0 = q0 + warp * 16 + (lane >> 2), row1 = row0 + 8;
  const int nkb = qb + 1;   // causal: key blocks 0..qb
  uint32_t qa[HD / 16][4];
  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) load_kv(kb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk)
        ldsm_x4(qa[kk], qs + (warp * 16 + (lane & 15)) * S::kLd + kk * 16 + (lane >> 4) * 8);
    }
    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[kPN / 8][4];
#pragma unroll
    for (int j = 0; j < kPN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const __half* kt = ks + buf * S::kKV;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int nt = 0; nt < kPN / 16; ++nt) {
        uint32_t b[4];
        ldsm_x4(b, kt + (nt * 16 + (lane >> 4) * 8 + (lane & 7)) * S::kLd + kk * 16 + ((lane >> 3) & 1) * 8);
        mma16816(s[2 * nt], qa[kk], b[0], b[1]);
        mma16816(s[2 * nt + 1], qa[kk], b[2], b[3]);
      }
    }
    // mask (causal and past-the-end keys), online softmax in base 2
    const int k0 = kb * kPN;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < kPN / 8; ++j) {
      const int c = k0 + j * 8 + (lane & 3) * 2;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok0 = c + e <= row0 && c + e < p.T;
        const bool ok1 = c + e <= row1 && c + e < p.T;
        s[j][e] = ok0 ? s[j][e] * p.scale_log2 : -INFINITY;
        s[j][2 + e] = ok1 ? s[j][2 + e] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[j][e]);
        mx1 = fmaxf(mx1, s[j][2 + e]);
      }
    }
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o2));
    }
    const float a0 = mx0 == -INFINITY ? 1.f : exp2f(m0 - mx0);
    const float a1 = mx1 == -INFINITY ? 1.f : exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[kPN / 16][4];
#pragma unroll
    for (int j = 0; j < kPN / 8; ++j) {
      const float p0 = mx0 == -INFINITY ? 0.f : exp2f(s[j][0] - mx0);
      const float p1 = mx0 == -INFINITY ? 0.f : exp2f(s[j][1] - mx0);
      const float p2 = mx1 == -INFINITY ? 0.f : exp2f(s[j][2] - mx1);
      const float p3 = mx1 == -INFINITY ? 0.f : exp2f(s[j][3] - mx1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pa[j / 2][(j & 1) * 2] = pack_h2(p0, p1);
      pa[j / 2][(j & 1) * 2 + 1] = pack_h2(p2, p3);
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      o[j][0] *= a0;
      o[j][1] *= a0;
      o[j][2] *= a1;
      o[j][3] *= a1;
    }
    // O += P V
    const __half* vt = vs + buf * S::kKV;
#pragma unroll
    for (int kk = 0; kk < kPN / 16; ++kk) {
#pragma unroll
      for (int dt = 0; dt < HD / 16; ++dt) {
        uint32_t b[4];
        ldsm_x4_t(b, vt + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * S::kLd + dt * 16 + (lane >> 4) * 8);
        mma16816(o[2 * dt], pa[kk], b[0], b[1]);
        mma16816(o[2 * dt + 1], pa[kk], b[2], b[3]);
      }
    }
    __syncthreads();
  }
  // row sums over the quad, normalise, store f32
#pragma unroll
  for (int o2 = 1; o2 <= 2; o2 <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o2);
  }
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
  float* dst0 = nullptr;
  float* dst1 = nullptr;
  if (!p.scatter) {
    const int64_t ld = static_cast<int64_t>(p.nq) * HD;
    dst0 = p.out + row0 * ld + static_cast<int64_t>(h) * HD;
    dst1 = p.out + row1 * ld + static_cast<int64_t>(h) * HD;
  } else {
    // NVLink peer stores into the owning rank's output rows
    const int64_t ld = static_cast<int64_t>(p.nq_total) * HD;
    const int64_t hc = static_cast<int64_t>(p.head_off + h) * HD;
    if (row0 < p.T) dst0 = p.out_peers[row0 / p.rows_per_rank] + (row0 % p.rows_per_rank) * ld + hc;
    if (row1 < p.T) dst1 = p.out_peers[row1 / p.rows_per_rank] + (row1 % p.rows_per_rank) * ld + hc;
  }
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) {
    const int d = j * 8 + (lane & 3) * 2;
    if (row0 < p.T) *reinterpret_cast<float2*>(dst0 + d) = make_float2(o[j][0] * i0, o[j][1] * i0);
    if (row1 < p.T) *reinterpret_cast<float2*>(dst1 + d) = make_float2(o[j][2] * i1, o[j][3] * i1);
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

extern "C" int pyre_softmax_rows(const float* x, int64_t rows, int cols, float* out, void* stream) {
  PYRE_CHECK_ARG(x != nullptr && out != nullptr, "pyre_softmax_rows: null pointer");
  PYRE_CHECK_ARG(rows >= 0 && rows <= 0x7fffffff && cols >= 1, "pyre_softmax_rows: bad sizes");
  if (rows == 0) return PYRE_OK;
  softmax_rows_kernel<<<static_cast<int>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, out, cols);
  PYRE_LAUNCH_CHECK("softmax_rows_kernel");
  return PYRE_OK;
}

extern "C" int pyre_rope_kv_append(const float* q, const float* k, const float* v, int64_t q_stride,
                                   int64_t kv_stride, int T, int nq, int nkv, int hd,
                                   int start_pos, double theta, double rope_fraction, uint16_t* q_out,
                                   uint16_t* k_cache, uint16_t* v_cache, int max_t, void* stream) {
  PYRE_CHECK_ARG(q && k && v && q_out && k_cache && v_cache, "pyre_rope_kv_append: null pointer");
  PYRE_CHECK_ARG(T >= 1 && nq >= 1 && nkv >= 1 && hd >= 2 && nq % nkv == 0, "pyre_rope_kv_append: bad head counts");
  PYRE_CHECK_ARG(start_pos >= 0 && start_pos + T <= max_t, "pyre_rope_kv_append: positions beyond the cache");
  PYRE_CHECK_ARG(q_stride >= static_cast<int64_t>(nq) * hd && kv_stride >= static_cast<int64_t>(nkv) * hd,
                 "pyre_rope_kv_append: row strides smaller than the heads");
  const int dims = static_cast<int>(static_cast<double>(hd) * rope_fraction);
  PYRE_CHECK_ARG(dims <= hd && dims / 2 <= kRopeMaxHalf, "pyre_rope_kv_append: rope_fraction must be in [0, 1]");
  PYRE_CHECK_ARG(theta > 0.0, "pyre_rope_kv_append: theta must be positive");
  rope_append_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, q_stride, kv_stride, T, nq, nkv, hd, start_pos, theta, dims < 2 ? 0 : dims, reinterpret_cast<__half*>(q_out),
      reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache), max_t);
  PYRE_LAUNCH_CHECK("rope_append_kernel");
  return PYRE_OK;
}

extern "C" int pyre_attn_decode_workspace_bytes(int nq, int nkv, int hd, int t, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr && nq >= 1 && nkv >= 1 && hd >= 1 && t >= 1, "pyre_attn_decode_workspace_bytes: bad args");
  const int64_t splits = (t + kDecMinChunk - 1) / kDecMinChunk;   // the most chunks a call can use
  *bytes = 256 + (static_cast<int64_t>(nq) * splits * (hd + 2) * 4 + 255) / 256 * 256;
  return PYRE_OK;
}

extern "C" int pyre_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, int t, int nq,
                                int nkv, int hd, int max_t, int mask_lo, int mask_hi, float* out, void* workspace,
                                int64_t ws_bytes, void* stream) {
  PYRE_CHECK_ARG(q && k_cache && v_cache && out && workspace, "pyre_attn_decode: null pointer");
  PYRE_CHECK_ARG(t >= 1 && t <= max_t && nkv >= 1 && nq % nkv == 0 && nq / nkv <= kDecMaxRep,
                 "pyre_attn_decode: bad sizes (at most 8 query heads per kv head)");
  PYRE_CHECK_ARG(hd == 64 || hd == 128, "pyre_attn_decode: head dim must be 64 or 128");
  PYRE_CHECK_ARG(nkv <= 64, "pyre_attn_decode: at most 64 kv heads");
  int64_t need = 0;
  pyre_attn_decode_workspace_bytes(nq, nkv, hd, t, &need);
  PYRE_CHECK_ARG(ws_bytes >= need && reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
                 "pyre_attn_decode: workspace too small or not 256-byte aligned");
  DecodeParams p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.kc = reinterpret_cast<const __half*>(k_cache);
  p.vc = reinterpret_cast<const __half*>(v_cache);
  p.out = out;
  p.counters = static_cast<unsigned int*>(workspace);
  p.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  p.nq = nq;
  p.nkv = nkv;
  p.hd = hd;
  p.t = t;
  p.max_t = max_t;
  p.chunk = kDecMaxChunk;
  p.splits = (t + kDecMaxChunk - 1) / kDecMaxChunk;
  // more, smaller chunks while the kv heads alone leave SMs idle
  while (p.chunk > kDecMinChunk && static_cast<int64_t>(nkv) * ((t + p.chunk / 2 - 1) / (p.chunk / 2)) <= 2 * sm_count()) {
    p.chunk /= 2;
    p.splits = (t + p.chunk - 1) / p.chunk;
  }
  p.mask_lo = mask_lo;
  p.mask_hi = mask_hi;
  p.scale = 1.0f / sqrtf(static_cast<float>(hd));
  dim3 grid(nkv, p.splits);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (hd == 64)
    attn_decode_kernel<64><<<grid, kDecThreads, 0, s>>>(p);
  else
    attn_decode_kernel<128><<<grid, kDecThreads, 0, s>>>(p);
  PYRE_LAUNCH_CHECK("attn_decode_kernel");
  return PYRE_OK;
}

namespace pyre {
namespace attn {
int launch_prefill(PrefillParams p, int hd, cudaStream_t s) {
  dim3 grid((p.T + kPM - 1) / kPM, p.nq);
  int rc;
  if (hd == 64) {
    rc = set_smem_limit(reinterpret_cast<const void*>(attn_prefill_kernel<64>), PrefillSmem<64>::kBytes);
    if (rc) return rc;
    attn_prefill_kernel<64><<<grid, 128, PrefillSmem<64>::kBytes, s>>>(p);
  } else {
    rc = set_smem_limit(reinterpret_cast<const void*>(attn_prefill_kernel<128>), PrefillSmem<128>::kBytes);
    if (rc) return rc;
    attn_prefill_kernel<128><<<grid, 128, PrefillSmem<128>::kBytes, s>>>(p);
  }
  PYRE_LAUNCH_CHECK("attn_prefill_kernel");
  return PYRE_OK;
}
}  // namespace attn
}  // namespace pyre

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
    int64_t kv_stride, int S_local, int seq_off, int S, int nq, int nkv, int hd, double theta, int dims, int P,
    UlyPeers peers, int64_t off_q, int64_t off_k, int64_t off_v) {
  __shared__ float cs[kRopeMaxHalf], sn[kRopeMaxHalf];
  const int t = blockIdx.x;
  const int pos = seq_off + t;
  const int half = dims >= 2 ? dims / 2 : 0;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const double freq = 1.0 / pow(theta, static_cast<double>(2 * j) / static_cast<double>(dims));
    const double ang = static_cast<double>(pos) * freq;
    cs[j] = static_cast<float>(cos(ang));
    sn[j] = static_cast<float>(sin(ang));
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
      r = i < half ? x1 * cs[jj] - x2 * sn[jj] : x1 * sn[jj] + x2 * cs[jj];
    } else {
      r = src[i];
    }
    const __half hv = __float2half_rn(fminf(fmaxf(r, -1000.f), 1000.f));
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
                                         int hd, double theta, double rope_fraction, void* stream) {
  int rc = uly_check_shape(S, P, nq, nkv, hd);
  if (rc) return rc;
  PYRE_CHECK_ARG(q && k && v && rank >= 0 && rank < P, "pyre_ulysses_rope_scatter: bad arguments");
  PYRE_CHECK_ARG(q_stride >= static_cast<int64_t>(nq) * hd && kv_stride >= static_cast<int64_t>(nkv) * hd,
                 "pyre_ulysses_rope_scatter: row strides smaller than the heads");
  const int dims = static_cast<int>(static_cast<double>(hd) * rope_fraction);
  PYRE_CHECK_ARG(dims <= hd && theta > 0.0, "pyre_ulysses_rope_scatter: bad RoPE parameters");
  UlyPeers peers{};
  rc = uly_peers(bufs, P, &peers);
  if (rc) return rc;
  const UlyLayout L = uly_layout(S, P, nq, nkv, hd);
  const int S_local = S / P;
  ulysses_rope_scatter_kernel<<<S_local, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, q_stride, kv_stride, S_local, rank * S_local, S, nq, nkv, hd, theta, dims < 2 ? 0 : dims, P, peers,
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
