// Last step of a decode token (reference: src/orchestrator/generator.py:40-53): the final
// RMSNorm of the hidden state (f64 mean of squares, x / sqrt(var + eps) in f64, times the norm
// weight), logits against the f16 lm_head table [V, H] in f32, and the greedy (temperature 0)
// next token, np.argmax semantics: the first index among equal maxima.
//
// One launch: every CTA normalises the T <= 4 rows into shared memory (f32), its warps stream
// rows of the table (4 rows at a time, 16-byte loads, chunks of 8 per lane in flight) and
// keep the best (value, index) per token row as one orderable 64-bit key; the CTA's best key
// goes to the workspace and the last CTA to arrive (a counter it resets) reduces them. The
// key orders by value, then by lower index, so a max over keys is the argmax; with a
// vocab-sharded table (rows v0 .. v0+V-1 on this rank) the ranks' keys combine with a max
// reduction. Deterministic: fixed sum order in every dot product.
#include "common.cuh"

namespace pyre {
namespace lmh {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxT = 4;
constexpr int kMaxH = 8192;
constexpr int kRows = 4;     // table rows per warp step
constexpr int kChunk = 8;    // 16-byte groups per lane per row in flight

struct Params {
  const float* h;            // [T, H]
  const float* norm_w;       // [H] or null (no final norm)
  double eps;
  const uint4* E;            // [V, H] f16, rows of H / 8 16-byte groups
  int T, H, V;
  int64_t v0;                // global index of row 0
  float* logits;             // [T, V] or null
  int* token;                // [T] global index of the maximum
  long long* key;            // [T] orderable (value, index) key of the maximum, or null
  long long* cta_keys;       // [grid][T] workspace
  unsigned* count;           // workspace arrival counter, zero between launches
};

// Orderable key: float bits mapped monotonically to u32 (negative values flipped), index
// complemented so that among equal values the lower index is larger; the top bit is then
// flipped so that signed 64-bit comparison (and a signed max reduction) orders the keys.
__device__ __forceinline__ long long make_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  const unsigned long long k = (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - idx);
  return static_cast<long long>(k ^ 0x8000000000000000ull);
}
__device__ __forceinline__ uint32_t key_index(long long key) {
  const unsigned long long k = static_cast<unsigned long long>(key) ^ 0x8000000000000000ull;
  return 0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull);
}

__device__ __forceinline__ void f16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = a.x;
    f[2 * i + 1] = a.y;
  }
}

template <int T>
__global__ void __launch_bounds__(kThreads, 1) lm_head_kernel(const Params p) {
  pdl_wait();      // h comes from the previous kernel of the stream
  pdl_trigger();
  extern __shared__ float hs[];            // [T][H] normalised rows
  __shared__ double red[kWarps];
  __shared__ long long wkey[kWarps][kMaxT];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H;

  // final RMSNorm of each token row (every CTA; the rows are a few KB and stay in L2)
  for (int t = 0; t < T; ++t) {
    const float* x = p.h + static_cast<int64_t>(t) * H;
    if (p.norm_w == nullptr) {
      for (int i = threadIdx.x; i < H; i += kThreads) hs[t * H + i] = x[i];
      continue;
    }
    double sq = 0.0;
    for (int i = threadIdx.x; i < H; i += kThreads) {
      const double v = x[i];
      sq += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += red[w];
    const double rs = sqrt(tot / H + p.eps);
    for (int i = threadIdx.x; i < H; i += kThreads)
      hs[t * H + i] = static_cast<float>((static_cast<double>(x[i]) / rs) * static_cast<double>(p.norm_w[i]));
    __syncthreads();
  }
  __syncthreads();

  // rows of the table: warp gw takes rows gw*kRows .. +kRows-1, then every nw*kRows later
  const int G8 = H / 8;                    // 16-byte groups per row
  const int nw = gridDim.x * kWarps;
  const int gw = blockIdx.x * kWarps + warp;
  long long best[T];
#pragma unroll
  for (int t = 0; t < T; ++t) best[t] = LLONG_MIN;
  for (int v0 = gw * kRows; v0 < p.V; v0 += nw * kRows) {
    float acc[kRows][T];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int t = 0; t < T; ++t) acc[r][t] = 0.f;
    for (int g0 = lane; g0 < G8; g0 += 32 * kChunk) {
      uint4 e[kRows][kChunk];
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const int v = min(v0 + r, p.V - 1);
        const uint4* row = p.E + static_cast<int64_t>(v) * G8;
#pragma unroll
        for (int c = 0; c < kChunk; ++c) {
          const int g = g0 + 32 * c;
          e[r][c] = g < G8 ? __ldcs(row + g) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int c = 0; c < kChunk; ++c) {
        const int g = g0 + 32 * c;
        if (g >= G8) break;
        float hv[T][8];
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float4 a = *reinterpret_cast<const float4*>(hs + t * H + g * 8);
          const float4 b = *reinterpret_cast<const float4*>(hs + t * H + g * 8 + 4);
          hv[t][0] = a.x; hv[t][1] = a.y; hv[t][2] = a.z; hv[t][3] = a.w;
          hv[t][4] = b.x; hv[t][5] = b.y; hv[t][6] = b.z; hv[t][7] = b.w;
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          float ef[8];
          f16x8_to_f32(e[r][c], ef);
#pragma unroll
          for (int t = 0; t < T; ++t)
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[r][t] = fmaf(hv[t][q], ef[q], acc[r][t]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int t = 0; t < T; ++t) {
        float a = acc[r][t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        const int v = v0 + r;
        if (v < p.V) {
          if (p.logits != nullptr && lane == 0) p.logits[static_cast<int64_t>(t) * p.V + v] = a;
          const long long k = make_key(a, static_cast<uint32_t>(p.v0 + v));
          best[t] = k > best[t] ? k : best[t];
        }
      }
  }
  if (lane == 0)
#pragma unroll
    for (int t = 0; t < T; ++t) wkey[warp][t] = best[t];
  __syncthreads();
  if (threadIdx.x < T) {
    long long k = LLONG_MIN;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) k = wkey[w][threadIdx.x] > k ? wkey[w][threadIdx.x] : k;
    p.cta_keys[static_cast<int64_t>(blockIdx.x) * T + threadIdx.x] = k;
  }
  // the last CTA to arrive reduces the CTAs' keys
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const bool last = atomicAdd(p.count, 1u) == gridDim.x - 1;
    if (last) __threadfence();
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  for (int t = warp; t < T; t += kWarps) {
    long long k = LLONG_MIN;
    for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
      const long long kc = __ldcg(p.cta_keys + static_cast<int64_t>(c) * T + t);
      k = kc > k ? kc : k;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const long long ko = __shfl_xor_sync(0xffffffffu, k, o);
      k = ko > k ? ko : k;
    }
    if (lane == 0) {
      p.token[t] = static_cast<int>(key_index(k));
      if (p.key != nullptr) p.key[t] = k;
    }
  }
  if (threadIdx.x == 0) *p.count = 0u;
}

int grid_ctas() {
  int n = sm_count();
  return n < 1 ? 1 : n;
}

// x[t, :] = f32(table[ids[t], :]) (Generator._embed, generator.py:38-39), then
// norm[t, :] = rms_norm(x[t, :], w) as pyre_rms_norm (the first layer's input RMSNorm,
// root_node.py:752). One CTA per token; an id outside [0, V) yields a zero row and sets
// *status to PYRE_EINVAL.
__global__ void embed_rms_norm_kernel(const int* __restrict__ ids, const __half* __restrict__ table, int V, int H,
                                      const float* __restrict__ w, double eps, float* __restrict__ x,
                                      float* __restrict__ norm, int* status) {
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && status != nullptr) atomicExch(status, PYRE_EINVAL);
  const __half* row = table + static_cast<int64_t>(ok ? id : 0) * H;
  double sq = 0.0;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = ok ? __half2float(row[i]) : 0.0f;
    x[t * H + i] = v;
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
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    norm[t * H + i] = static_cast<float>(static_cast<double>(x[t * H + i]) * rstd * static_cast<double>(w[i]));
}

// embed_rms_norm_kernel for H % 4 == 0 and H <= 4 * kEmbVec * blockDim: each thread loads its
// groups of 4 table entries (8 bytes) into registers up front.
constexpr int kEmbVec = 4;
__global__ void __launch_bounds__(1024) embed_rms_norm_vec_kernel(const int* __restrict__ ids,
                                                                  const __half* __restrict__ table, int V, int H,
                                                                  const float* __restrict__ w, double eps,
                                                                  float* __restrict__ x, float* __restrict__ norm,
                                                                  int* status) {
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && status != nullptr) atomicExch(status, PYRE_EINVAL);
  const uint2* row = reinterpret_cast<const uint2*>(table + static_cast<int64_t>(ok ? id : 0) * H);
  const int n4 = H >> 2;
  float4 v[kEmbVec];
#pragma unroll
  for (int j = 0; j < kEmbVec; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < n4) {
      const uint2 u = __ldg(row + i);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[j] = ok ? make_float4(a.x, a.y, b.x, b.y) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  double sq = 0.0;
  float4* xr = reinterpret_cast<float4*>(x + t * H);
#pragma unroll
  for (int j = 0; j < kEmbVec; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < n4) {
      xr[i] = v[j];
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
    double r = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (threadIdx.x == 0) red[0] = r;
  }
  __syncthreads();
  const double rstd = 1.0 / sqrt(red[0] / H + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4* nr = reinterpret_cast<float4*>(norm + t * H);
#pragma unroll
  for (int j = 0; j < kEmbVec; ++j) {
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

}  // namespace lmh
}  // namespace pyre

using namespace pyre;

extern "C" int pyre_lm_head_workspace_bytes(int T, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr && T >= 1 && T <= lmh::kMaxT, "pyre_lm_head_workspace_bytes: 1 <= T <= 4");
  *bytes = 256 + static_cast<int64_t>(lmh::grid_ctas()) * T * 8;
  return PYRE_OK;
}

extern "C" int pyre_lm_head_argmax(const float* h, int T, int H, const float* norm_w, double eps,
                                   const uint16_t* lm_head, int V, int64_t v0, float* logits, int* token,
                                   long long* key, void* workspace, int64_t ws_bytes, void* stream) {
  PYRE_CHECK_ARG(h != nullptr && lm_head != nullptr && token != nullptr && workspace != nullptr,
                 "pyre_lm_head_argmax: null pointer");
  PYRE_CHECK_ARG(T >= 1 && T <= lmh::kMaxT, "pyre_lm_head_argmax: 1 <= T <= 4 token rows");
  PYRE_CHECK_ARG(H >= 8 && H <= lmh::kMaxH && H % 8 == 0, "pyre_lm_head_argmax: H must be a multiple of 8, <= 8192");
  PYRE_CHECK_ARG(V >= 1 && v0 >= 0 && v0 + V <= 0xFFFFFFFFll, "pyre_lm_head_argmax: bad vocabulary range");
  PYRE_CHECK_ARG(reinterpret_cast<uintptr_t>(lm_head) % 16 == 0 && reinterpret_cast<uintptr_t>(workspace) % 16 == 0,
                 "pyre_lm_head_argmax: lm_head and workspace must be 16-byte aligned");
  const int G = lmh::grid_ctas();
  PYRE_CHECK_ARG(ws_bytes >= 256 + static_cast<int64_t>(G) * T * 8,
                 "pyre_lm_head_argmax: workspace smaller than pyre_lm_head_workspace_bytes");
  lmh::Params p{};
  p.h = h;
  p.norm_w = norm_w;
  p.eps = eps;
  p.E = reinterpret_cast<const uint4*>(lm_head);
  p.T = T;
  p.H = H;
  p.V = V;
  p.v0 = v0;
  p.logits = logits;
  p.token = token;
  p.key = key;
  p.count = static_cast<unsigned*>(workspace);
  p.cta_keys = reinterpret_cast<long long*>(static_cast<char*>(workspace) + 256);
  const int smem = T * H * 4;   // the limit is set once per kernel, for the largest H
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = PYRE_OK;
  switch (T) {
    case 1:
      rc = set_smem_limit(reinterpret_cast<const void*>(lmh::lm_head_kernel<1>), 1 * lmh::kMaxH * 4);
      if (!rc) rc = cuda_status(launch_pdl(lmh::lm_head_kernel<1>, dim3(G), dim3(lmh::kThreads), smem, s, p), "lm_head_kernel");
      break;
    case 2:
      rc = set_smem_limit(reinterpret_cast<const void*>(lmh::lm_head_kernel<2>), 2 * lmh::kMaxH * 4);
      if (!rc) rc = cuda_status(launch_pdl(lmh::lm_head_kernel<2>, dim3(G), dim3(lmh::kThreads), smem, s, p), "lm_head_kernel");
      break;
    case 3:
      rc = set_smem_limit(reinterpret_cast<const void*>(lmh::lm_head_kernel<3>), 3 * lmh::kMaxH * 4);
      if (!rc) rc = cuda_status(launch_pdl(lmh::lm_head_kernel<3>, dim3(G), dim3(lmh::kThreads), smem, s, p), "lm_head_kernel");
      break;
    default:
      rc = set_smem_limit(reinterpret_cast<const void*>(lmh::lm_head_kernel<4>), 4 * lmh::kMaxH * 4);
      if (!rc) rc = cuda_status(launch_pdl(lmh::lm_head_kernel<4>, dim3(G), dim3(lmh::kThreads), smem, s, p), "lm_head_kernel");
      break;
  }
  if (rc) return rc;
  PYRE_LAUNCH_CHECK("lm_head_kernel");
  return PYRE_OK;
}

extern "C" int pyre_embed_rms_norm(const int* ids, int T, const void* table, int V, int H, const float* w, double eps,
                                   float* x, float* norm, int* status, void* stream) {
  PYRE_CHECK_ARG(ids != nullptr && table != nullptr && x != nullptr, "pyre_embed_rms_norm: null pointer");
  PYRE_CHECK_ARG((norm == nullptr) == (w == nullptr), "pyre_embed_rms_norm: norm and w go together");
  PYRE_CHECK_ARG(T >= 0 && V >= 1 && H >= 1, "pyre_embed_rms_norm: bad sizes");
  if (T == 0) return PYRE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto a16 = [](const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const int n4 = H / 4;
  if (H % 4 == 0 && n4 <= 1024 * lmh::kEmbVec && reinterpret_cast<uintptr_t>(table) % 8 == 0 && a16(w) && a16(x) &&
      a16(norm)) {
    int threads = (n4 + lmh::kEmbVec - 1) / lmh::kEmbVec;
    threads = threads < 32 ? 32 : (threads + 31) / 32 * 32;
    PYRE_CUDA_TRY(launch_pdl(lmh::embed_rms_norm_vec_kernel, dim3(static_cast<unsigned>(T)), dim3(threads), 0, s,
                             ids, static_cast<const __half*>(table), V, H, w, eps, x, norm, status));
    return PYRE_OK;
  }
  PYRE_CUDA_TRY(launch_pdl(lmh::embed_rms_norm_kernel, dim3(static_cast<unsigned>(T)), dim3(256), 0, s, ids,
                           static_cast<const __half*>(table), V, H, w, eps, x, norm, status));
  return PYRE_OK;
}
