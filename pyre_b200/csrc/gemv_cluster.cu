// Q8_0 GEMV for T <= 4 tokens on one packed matrix that fits a cluster's shared memory per
// 256-column slab (K <= 8192): the Q/K/V and O projections of a decode step.
//
//   out[T, N] = x[T, K] @ W (+ bias)        (root_node.py:866-897, :851-858; biases :786-799)
//
// Layout: one cluster of C CTAs per 256-column slab of the packed matrix (gemv_common.cuh,
// M = 1: blocks of 64 rows x 256 columns, one bulk copy each). CTA r of the cluster owns the
// contiguous block range [r*upt/C, (r+1)*upt/C) of the slab (upt = blocks per slab, at most 8
// per CTA) and normally keeps ALL of them in flight at once: its producer lane issues every
// bulk copy before griddepcontrol.wait (weights are constant), so under programmatic dependent
// launch the whole weight fetch overlaps the previous kernel's tail. When that leaves too few
// clusters co-resident for one wave, the blocks go through a ring of fewer slots instead (the
// first slots before the wait, each later block as soon as its slot is consumed). After the wait the CTA reads its
// slice of x into shared memory, the consumer warps accumulate block by block (the exact
// int8 -> f32 conversion and packed f32x2 FMA of gemv_common.cuh), reduce over warps into a
// [T, 256] partial, and the cluster reduces the C partials through distributed shared memory:
// rank r adds, in rank order 0..C-1, columns [r*256/C, (r+1)*256/C) of every rank's partial,
// adds the bias and stores the output. No global scratch, atomics or flags: the reduction is
// deterministic and costs one cluster barrier instead of L2 round trips.
//
// Larger matrices (the FFN, and tensor-parallel projections whose epilogue reduces over NVLink)
// use the streaming kernel of ffn_stream.cuh.
#include <cooperative_groups.h>

#include <mutex>
#include <vector>

#include "ffn_internal.cuh"

namespace pyre {
namespace gcl {

using namespace gemv;
namespace cg = cooperative_groups;

constexpr int kRows = kUnitRowsSingle;              // 64 rows per block
constexpr int kMaxUnits = 8;                        // blocks in flight per CTA
constexpr int kMaxCluster = 16;
constexpr int kThreadsC = kConsumers + 32;          // 8 consumer warps + 1 producer warp

template <typename ST>
constexpr int block_bytes() { return kRows * kTileN + kRows * 8 * static_cast<int>(sizeof(ST)); }

// Shared memory: partial [T][256] | barriers (128 B) | x [T][units*64] f32 | blocks, where the
// warp partials ([warps][T][256] f32) reuse the block area once every warp is done with the
// blocks. The partial comes first so that it sits at the same offset in every rank of the
// cluster (the ranks read each other's partials through distributed shared memory at the
// address of their own), whatever each rank's block count. Keeping the head small lets three
// CTAs of four blocks share an SM, so a 24-slab Q/K/V matrix runs as one wave of clusters.
template <int T>
constexpr int head_bytes() { return T * kTileN * 4 + 128; }
template <int T>
constexpr int red_bytes() { return kConsumerWarps * T * kTileN * 4; }
template <int T, typename ST>
constexpr int smem_bytes(int units, int slots) {
  return head_bytes<T>() + T * units * kRows * 4 +
         (slots * block_bytes<ST>() > red_bytes<T>() ? slots * block_bytes<ST>() : red_bytes<T>());
}

struct Params {
  const uint8_t* w;       // packed single matrix [K, N]
  const void* x;          // [T, K] f32 or bf16
  const float* bias;      // [N] or null
  float* out;             // [T, N]
  int* status;            // PYRE_ETIMEOUT if a copy wait ran out
  int K, N, upt, C;
  int slots;              // block slots per CTA (a ring when fewer than the CTA's blocks)
};

template <typename XT>
__device__ __forceinline__ float ld_x(const void* x, int64_t i) {
  return to_f32(static_cast<const XT*>(x)[i]);
}

// One 64 x 256 block at wst into acc; x of the block's rows at xs[t * pitch + r].
template <int T, typename ST>
__device__ __forceinline__ void consume_block(const uint8_t* wst, const float* xs, int pitch, float2 (&acc)[1][T][8],
                                              int warp, int rs, int cc) {
  const ST* ss = reinterpret_cast<const ST*>(wst + kRows * kTileN);
#pragma unroll
  for (int pass = 0; pass < kRows / kRowsPerPass; ++pass) {
    const int r = pass * kRowsPerPass + warp * 2 + rs;
    const float sc = to_f32(ss[r * 8 + (cc >> 1)]);
    const int4 w = *reinterpret_cast<const int4*>(wst + r * kTileN + cc * 16);
    const uint32_t words[4] = {static_cast<uint32_t>(w.x), static_cast<uint32_t>(w.y), static_cast<uint32_t>(w.z),
                               static_cast<uint32_t>(w.w)};
    float2 a2[T];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const float a = xs[t * pitch + r] * sc;
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
        acc[0][t][wi * 2] = __ffma2_rn(a2[t], f01, acc[0][t][wi * 2]);
        acc[0][t][wi * 2 + 1] = __ffma2_rn(a2[t], f23, acc[0][t][wi * 2 + 1]);
      }
    }
  }
}

template <int T, typename XT, typename ST>
__global__ void __launch_bounds__(kThreadsC, 1) q80_gemv_cluster_kernel(const __grid_constant__ Params p) {
  constexpr int kBB = block_bytes<ST>();
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int C = p.C;
  const int rank = static_cast<int>(cluster.block_rank());
  const int tile = blockIdx.y;
  const int u0 = static_cast<int>(static_cast<int64_t>(p.upt) * rank / C);
  const int u1 = static_cast<int>(static_cast<int64_t>(p.upt) * (rank + 1) / C);
  const int nu = u1 - u0;                    // 1..kMaxUnits (the host picks C so)
  const int pitch = nu * kRows;
  float* fin = reinterpret_cast<float*>(smem);                        // same offset in every rank
  uint64_t* full = reinterpret_cast<uint64_t*>(fin + T * kTileN);     // [kMaxUnits]
  uint64_t* empty = full + kMaxUnits;                                 // [kMaxUnits]
  const int S = p.slots < nu ? p.slots : nu;
  float* xs = reinterpret_cast<float*>(smem + head_bytes<T>());
  uint8_t* blocks = smem + head_bytes<T>() + T * pitch * 4;          // 16-byte aligned
  float* red = reinterpret_cast<float*>(blocks);                      // after the last block is read
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const bool producer = warp == kConsumerWarps && lane == 0;
  const uint8_t* src = p.w + (static_cast<int64_t>(tile) * p.upt + u0) * kBB;
  if (producer) {
    // the first S blocks of this CTA (all of them when S == nu) in flight before the wait:
    // weights are constant
    for (int i = 0; i < S; ++i) {
      mbar_arrive_expect_tx(&full[i], kBB);
      bulk_load(blocks + i * kBB, src + static_cast<int64_t>(i) * kBB, kBB, &full[i]);
    }
  }
  pdl_wait();      // x comes from the previous kernel of the stream
  pdl_trigger();
  if (producer) {
    // ring: block i into slot i % S once the consumers have released that slot's previous block
    for (int i = S; i < nu; ++i) {
      const int sl = i % S;
      if (!mbar_wait(&empty[sl], static_cast<uint32_t>((i / S - 1) & 1), p.status)) break;
      mbar_arrive_expect_tx(&full[sl], kBB);
      bulk_load(blocks + sl * kBB, src + static_cast<int64_t>(i) * kBB, kBB, &full[sl]);
    }
  }
  if (warp < kConsumerWarps) {
    const int tid = threadIdx.x;
    const int k0 = u0 * kRows;
    for (int i = tid; i < T * pitch; i += kConsumers) {
      const int t = i / pitch, k = k0 + (i - t * pitch);
      xs[i] = k < p.K ? ld_x<XT>(p.x, static_cast<int64_t>(t) * p.K + k) : 0.f;
    }
    consumer_sync();
    const int rs = lane >> 4, cc = lane & 15;
    float2 acc[1][T][8];
    zero_acc<1, T>(acc);
    for (int i = 0; i < nu; ++i) {
      const int sl = i % S;
      mbar_wait(&full[sl], static_cast<uint32_t>((i / S) & 1), p.status);
      consume_block<T, ST>(blocks + sl * kBB, xs + i * kRows, pitch, acc, warp, rs, cc);
      if (nu > S) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[sl]);
      }
    }
    consumer_sync();   // every warp is done with the blocks: the warp partials go there
    reduce_tile<T, 1>(acc, red, fin, warp, rs, cc, tid);   // fin[t * 256 + c]: this CTA's partial
  }
  cluster.sync();          // every rank's partial is complete and visible
  {
    const int c0 = kTileN * rank / C, c1 = kTileN * (rank + 1) / C;
    const int w = c1 - c0;
    for (int i = threadIdx.x; i < T * w; i += kThreadsC) {
      const int t = i / w, c = c0 + (i - t * w);
      float v = 0.f;
      for (int src = 0; src < C; ++src) v += cluster.map_shared_rank(fin, src)[t * kTileN + c];
      const int col = tile * kTileN + c;
      if (col < p.N) {
        if (p.bias != nullptr) v += __ldg(p.bias + col);
        p.out[static_cast<int64_t>(t) * p.N + col] = v;
      }
    }
  }
  cluster.sync();          // no rank leaves while another still reads its partial
}

// Smallest cluster for [K, N]: enough ranks that each holds at most kMaxUnits blocks (0: K too
// large for this kernel).
int min_cluster(int upt) {
  const int c = (upt + kMaxUnits - 1) / kMaxUnits;
  return c <= kMaxCluster ? (c < 1 ? 1 : c) : 0;
}

template <int T, typename XT, typename ST>
cudaLaunchConfig_t launch_cfg(int C, int slots, int tiles, int upt, cudaStream_t s, cudaLaunchAttribute (&attr)[2]) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(C), static_cast<unsigned>(tiles), 1);
  cfg.blockDim = dim3(kThreadsC, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes<T, ST>((upt + C - 1) / C, slots));
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cfg;
}

// Cluster size and block slots for [K, N] on this device: the pair that runs the tiles'
// clusters in the fewest waves of co-resident one-token clusters (a second wave costs a whole
// second fetch latency); among equals every block in flight at once (no ring) before a ring
// of kRingSlots, then the larger cluster (more SMs fetching). The cluster size fixes how K is
// split into partial sums, so it is decided for the matrix alone (one token, and the same for
// every T and activation type: a row of a batch then gets exactly the sums it gets alone) and
// cached per (device, upt, tiles, scale type).
constexpr int kRingSlots = 3;
template <typename ST>
int pick_cluster(int upt, int tiles, cudaStream_t s, int* C, int* slots) {
  auto kern = q80_gemv_cluster_kernel<1, float, ST>;
  struct Pick { int dev, upt, tiles, C, slots; };
  static std::mutex mu;
  static std::vector<Pick> cache;
  int dev = 0;
  PYRE_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  for (const Pick& q : cache)
    if (q.dev == dev && q.upt == upt && q.tiles == tiles) {
      *C = q.C;
      *slots = q.slots;
      return PYRE_OK;
    }
  int rc = set_smem_limit(reinterpret_cast<const void*>(kern), smem_bytes<1, ST>(kMaxUnits, kMaxUnits));
  if (rc) return rc;
  PYRE_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  const int c0 = min_cluster(upt);
  int best = 0, best_slots = 0, best_waves = 0;
  for (int ring = 0; ring < 2; ++ring) {
    for (int c = c0; c <= kMaxCluster && c <= (upt > c0 ? upt : c0); ++c) {
      const int units = (upt + c - 1) / c;
      const int sl = ring ? kRingSlots : units;
      if (ring && units <= kRingSlots) continue;
      cudaLaunchAttribute attr[2]{};
      cudaLaunchConfig_t cfg = launch_cfg<1, float, ST>(c, sl, tiles, upt, s, attr);
      int active = 0;
      if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess || active < 1) {
        (void)cudaGetLastError();
        continue;
      }
      const int waves = (tiles + active - 1) / active;
      // no ring: the larger cluster among equals; ring: only if it needs fewer waves
      if (best == 0 || waves < best_waves || (!ring && waves == best_waves)) {
        best = c;
        best_slots = sl;
        best_waves = waves;
      }
    }
  }
  if (best == 0) return set_error(PYRE_ECUDA, "q80_gemv_cluster_kernel: no cluster size fits on the device");
  cache.push_back(Pick{dev, upt, tiles, best, best_slots});
  *C = best;
  *slots = best_slots;
  return PYRE_OK;
}

template <int T, typename XT, typename ST>
int launch_t(Params p, int tiles, cudaStream_t s) {
  auto kern = q80_gemv_cluster_kernel<T, XT, ST>;
  int rc = pick_cluster<ST>(p.upt, tiles, s, &p.C, &p.slots);
  if (rc) return rc;
  rc = set_smem_limit(reinterpret_cast<const void*>(kern), smem_bytes<T, ST>(kMaxUnits, kMaxUnits));
  if (rc) return rc;
  if (p.C > 8) {
    static bool nonportable_set[64] = {};
    int d = 0;
    PYRE_CUDA_TRY(cudaGetDevice(&d));
    if (!nonportable_set[d & 63]) {
      PYRE_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                         cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
      nonportable_set[d & 63] = true;
    }
  }
  cudaLaunchAttribute attr[2]{};
  cudaLaunchConfig_t cfg = launch_cfg<T, XT, ST>(p.C, p.slots, tiles, p.upt, s, attr);
  PYRE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
  PYRE_LAUNCH_CHECK("q80_gemv_cluster_kernel");
  return PYRE_OK;
}

template <typename XT, typename ST>
int launch_types(Params p, int T, int tiles, cudaStream_t s) {
  switch (T) {
    case 1: return launch_t<1, XT, ST>(p, tiles, s);
    case 2: return launch_t<2, XT, ST>(p, tiles, s);
    case 3: return launch_t<3, XT, ST>(p, tiles, s);
    case 4: return launch_t<4, XT, ST>(p, tiles, s);
    default: return set_error(PYRE_EINVAL, "q80_gemv_cluster_kernel: T must be in [1, 4]");
  }
}

}  // namespace gcl

// Whether the cluster GEMV serves [K, N] (K <= 8192 at 64 rows per block and 8 blocks per rank).
bool gemv_cluster_eligible(int K, int N) {
  (void)N;
  return gcl::min_cluster((K + gcl::kRows - 1) / gcl::kRows) > 0;
}

int gemv_cluster(const void* x, int x_dtype, int T, int K, const void* w, int scale_dtype, int N, const float* bias,
                 float* out, int* status, cudaStream_t s) {
  gcl::Params p{};
  p.w = static_cast<const uint8_t*>(w);
  p.x = x;
  p.bias = bias;
  p.out = out;
  p.status = status;
  p.K = K;
  p.N = N;
  p.upt = (K + gcl::kRows - 1) / gcl::kRows;
  const int tiles = gemv::tiles_of(N);
  PYRE_CHECK_ARG(gcl::min_cluster(p.upt) > 0, "q80 GEMV: K too large for the cluster kernel");
  const bool f16s = scale_dtype == PYRE_F16;
  if (x_dtype == PYRE_BF16)
    return f16s ? gcl::launch_types<__nv_bfloat16, __half>(p, T, tiles, s)
                : gcl::launch_types<__nv_bfloat16, float>(p, T, tiles, s);
  return f16s ? gcl::launch_types<float, __half>(p, T, tiles, s) : gcl::launch_types<float, float>(p, T, tiles, s);
}

}  // namespace pyre
