// One persistent launch per FFN shard call for decode (T <= 4 tokens):
//   phase A: h[T, W] = silu(x @ Wg) * (x @ Wu)   (stream-K over gate/up slabs)
//   phase B: out[T, H] = h @ Wd (+ the cross-rank sum over NVLink)
// Reference semantics as in ffn.cu (src/ffn/builder.py:37-45, root_node.py:956-995).
//
// Every CTA first works through its share of the phase-A units, then its share of the
// phase-B units, through one shared-memory ring. The producer streams phase-B weights as
// soon as ring slots free up — during the phase-A tail — and only the activation slice of
// a phase-B unit (rows k0..k0+31 of h) waits for the gate/up slab k0/256 that produces
// them: the CTA finishing a slab publishes a per-slab ready flag tagged with the call's
// epoch. Phase A never waits on anything, every CTA is co-resident, so every wait ends.
#include "ffn_internal.cuh"

namespace pyre {
namespace ffn {

struct alignas(64) DecodeParams {
  CUtensorMap tx;            // x [T, H], box T x R_A
  CUtensorMap th;            // h [T, W] f32, box T x R_B
  const uint8_t* wgu;        // packed gate/up pair (or up alone when ungated)
  const uint8_t* wd;         // packed down
  int H, W, T;
  int tilesA, uptA;          // phase A: slabs of W, units of H
  int tilesB, uptB;          // phase B: slabs of H, units of W
  int64_t UA, UB;
  int pmaxA, pmaxB;
  float* h;                  // [T, W]
  float* out;                // [T, H]
  float* wsA;
  float* wsB;
  unsigned int* cntA;
  unsigned int* cntB;
  uint32_t* ready;           // [tilesA]
  uint32_t* ws_epoch;
  unsigned int* ws_done;
  int* status;
  comm::DevComm comm;
};

template <int T, int NA, typename XT, typename ST>
struct DecodeCfg {
  using LA = StageLayout<T, NA, XT, ST>;
  using LB = StageLayout<T, 1, float, ST>;
  static constexpr int kStageBytes = LA::kBytes > LB::kBytes ? LA::kBytes : LB::kBytes;
  static constexpr int kCtasPerSm = (T <= 2) ? 2 : 1;
  static constexpr int kStages = (T <= 2) ? 4 : 5;
  static constexpr int kRedFloats = kConsumerWarps * NA * T * kTileN;
  static constexpr int kFinFloats = NA * T * kTileN;
  static constexpr int kSmemBytes = kStages * kStageBytes + (kRedFloats + kFinFloats) * 4 + 2 * kStages * 8 + 16;
};

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait for a per-slab ready flag (2 s); records PYRE_ETIMEOUT on expiry.
__device__ __forceinline__ void wait_ready(const uint32_t* flag, uint32_t epoch, int* status) {
  if (ld_acquire_gpu(flag) == epoch) return;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_gpu(flag) != epoch) {
    if (globaltimer_ns() - t0 > 2000000000ull) {
      atomicExch(status, PYRE_ETIMEOUT);
      return;
    }
    __nanosleep(20);
  }
}

template <int T, int NA, typename XT, typename ST, bool TP>
__global__ void __launch_bounds__(kThreads, (DecodeCfg<T, NA, XT, ST>::kCtasPerSm))
q80_ffn_decode_kernel(const __grid_constant__ DecodeParams p) {
  using C = DecodeCfg<T, NA, XT, ST>;
  using LA = typename C::LA;
  using LB = typename C::LB;
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
  const int64_t a0 = (static_cast<int64_t>(c) * p.UA) / G, a1 = (static_cast<int64_t>(c + 1) * p.UA) / G;
  const int64_t b0 = (static_cast<int64_t>(c) * p.UB) / G, b1 = (static_cast<int64_t>(c + 1) * p.UB) / G;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // epoch of this call (tags the per-slab ready flags); published by the last CTA to exit
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.ws_epoch) + 1u;
  uint32_t cepoch = 0;
  if constexpr (TP) cepoch = comm::epoch_begin(p.comm);

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&p.tx);
      prefetch_tmap(&p.th);
      int s = 0;
      uint32_t ph = 0;
      for (int64_t u = a0; u < a1; ++u) {
        const int tile = static_cast<int>(u / p.uptA);
        const int k0 = static_cast<int>(u - static_cast<int64_t>(tile) * p.uptA) * LA::kRows;
        mbar_wait(&empty[s], ph ^ 1u, p.status);
        uint8_t* st = stages + s * C::kStageBytes;
        mbar_arrive_expect_tx(&full[s], LA::kTxBytes);
        bulk_load(st, p.wgu + u * LA::kWBytes, LA::kWBytes, &full[s]);
        tma_load_2d(st + LA::kXOff, &p.tx, k0, 0, &full[s]);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      for (int64_t u = b0; u < b1; ++u) {
        const int tile = static_cast<int>(u / p.uptB);
        const int k0 = static_cast<int>(u - static_cast<int64_t>(tile) * p.uptB) * LB::kRows;
        mbar_wait(&empty[s], ph ^ 1u, p.status);
        uint8_t* st = stages + s * C::kStageBytes;
        mbar_arrive_expect_tx(&full[s], LB::kTxBytes);
        bulk_load(st, p.wd + u * LB::kWBytes, LB::kWBytes, &full[s]);
        // rows k0..k0+R_B-1 of h come from gate/up slab k0 / 256 (R_B divides 256)
        wait_ready(p.ready + k0 / kTileN, epoch, p.status);
        fence_proxy_async_global();
        tma_load_2d(st + LB::kXOff, &p.th, k0, 0, &full[s]);
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
    // phase A: gate/up + SiLU·mul into h
    int64_t u = a0;
    while (u < a1) {
      const int tile = static_cast<int>(u / p.uptA);
      const int64_t tile_u0 = static_cast<int64_t>(tile) * p.uptA;
      const int64_t seg_end = min(a1, tile_u0 + p.uptA);
      float2 acc[NA][T][8];
      zero_acc<NA, T>(acc);
      for (; u < seg_end; ++u) {
        mbar_wait(&full[s], ph, p.status);
        consume_unit<T, NA, XT, ST>(stages + s * C::kStageBytes, acc, warp, rs, cc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      reduce_tile<T, NA>(acc, red, fin, warp, rs, cc, tid);
      const int cf = cta_of_unit(tile_u0, p.UA, G);
      const int cl = cta_of_unit(tile_u0 + p.uptA - 1, p.UA, G);
      if (fixup_tile<T, NA>(fin, p.wsA, p.cntA, p.pmaxA, tile, c, cf, cl, s_last, tid)) {
        for (int i = tid; i < T * kTileN; i += kConsumers) {
          const int t = i / kTileN, col = tile * kTileN + (i % kTileN);
          if (col >= p.W) continue;
          const float v = (NA == 2) ? silu_f32(fin[i]) * fin[T * kTileN + i] : silu_f32(fin[i]);
          p.h[static_cast<int64_t>(t) * p.W + col] = v;
        }
        __threadfence();
        fence_proxy_async_global();
        consumer_sync();
        if (tid == 0) st_release_gpu(p.ready + tile, epoch);
      }
      consumer_sync();
    }
    // phase B: down projection (+ cross-rank sum)
    u = b0;
    while (u < b1) {
      const int tile = static_cast<int>(u / p.uptB);
      const int64_t tile_u0 = static_cast<int64_t>(tile) * p.uptB;
      const int64_t seg_end = min(b1, tile_u0 + p.uptB);
      float2 acc[1][T][8];
      zero_acc<1, T>(acc);
      for (; u < seg_end; ++u) {
        mbar_wait(&full[s], ph, p.status);
        consume_unit<T, 1, float, ST>(stages + s * C::kStageBytes, acc, warp, rs, cc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      reduce_tile<T, 1>(acc, red, fin, warp, rs, cc, tid);
      const int cf = cta_of_unit(tile_u0, p.UB, G);
      const int cl = cta_of_unit(tile_u0 + p.uptB - 1, p.UB, G);
      if (fixup_tile<T, 1>(fin, p.wsB, p.cntB, p.pmaxB, tile, c, cf, cl, s_last, tid)) {
        if constexpr (TP) {
          tp_reduce_tile<T>(p.comm, cepoch, tile, fin, p.out, p.H, tid);
        } else {
          for (int i = tid; i < T * kTileN; i += kConsumers) {
            const int t = i / kTileN, col = tile * kTileN + (i % kTileN);
            if (col < p.H) p.out[static_cast<int64_t>(t) * p.H + col] = fin[i];
          }
        }
      }
      consumer_sync();
    }
  }
  __syncthreads();
  if constexpr (TP) comm::epoch_end(p.comm, cepoch);
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.ws_done, 1u);
    if (prev == gridDim.x - 1) {
      *reinterpret_cast<volatile unsigned int*>(p.ws_done) = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(p.ws_epoch) = epoch;
    }
  }
}

inline int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

// Workspace of the one-launch decode: header | h [T, W] f32 | pieces A | pieces B.
int64_t decode_ws_bytes(int T, int H, int W, int na) {
  return kHeaderBytes + align256(static_cast<int64_t>(T) * W * 4) + align256(pieces_bytes(T, W, na)) +
         align256(pieces_bytes(T, H, 1));
}

template <int T, int NA, typename XT, typename ST, bool TP>
int launch_decode(DecodeParams p, const void* x, int64_t ws_cap, cudaStream_t s) {
  using C = DecodeCfg<T, NA, XT, ST>;
  auto kern = q80_ffn_decode_kernel<T, NA, XT, ST, TP>;
  int rc = set_smem_once(kern, C::kSmemBytes);
  if (rc) return rc;
  rc = make_tmap_2d(&p.tx, x, tma_dtype<XT>(), sizeof(XT), T, p.H, static_cast<uint64_t>(p.H) * sizeof(XT), T,
                    C::LA::kRows);
  if (rc) return rc;
  rc = make_tmap_2d(&p.th, p.h, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, T, p.W, static_cast<uint64_t>(p.W) * 4, T,
                    C::LB::kRows);
  if (rc) return rc;
  int G = 1;
  rc = coresident_grid(kern, kThreads, C::kSmemBytes, C::kCtasPerSm, p.UA < p.UB ? p.UA : p.UB, &G);
  if (rc) return rc;
  p.pmaxA = pmax_for(p.tilesA, p.uptA, G);
  p.pmaxB = pmax_for(p.tilesB, p.uptB, G);
  const int64_t needA = align256(static_cast<int64_t>(p.tilesA) * p.pmaxA * NA * T * kTileN * 4);
  const int64_t needB = align256(static_cast<int64_t>(p.tilesB) * p.pmaxB * T * kTileN * 4);
  if (needA + needB > ws_cap) return set_error(PYRE_ENOMEM, "pyre_ffn_decode_q80: workspace too small for this grid");
  p.wsB = reinterpret_cast<float*>(reinterpret_cast<char*>(p.wsA) + needA);
  kern<<<G, kThreads, C::kSmemBytes, s>>>(p);
  PYRE_LAUNCH_CHECK("q80_ffn_decode_kernel");
  return PYRE_OK;
}

template <int T, int NA, typename XT, typename ST>
int decode_tp(DecodeParams p, const void* x, int64_t cap, bool tp, cudaStream_t s) {
  return tp ? launch_decode<T, NA, XT, ST, true>(p, x, cap, s) : launch_decode<T, NA, XT, ST, false>(p, x, cap, s);
}

template <int T, int NA>
int decode_types(DecodeParams p, const void* x, int x_dtype, int scale_dtype, int64_t cap, bool tp, cudaStream_t s) {
  if (x_dtype == PYRE_BF16) {
    if (scale_dtype == PYRE_F16) return decode_tp<T, NA, __nv_bfloat16, __half>(p, x, cap, tp, s);
    return decode_tp<T, NA, __nv_bfloat16, float>(p, x, cap, tp, s);
  }
  if (scale_dtype == PYRE_F16) return decode_tp<T, NA, float, __half>(p, x, cap, tp, s);
  return decode_tp<T, NA, float, float>(p, x, cap, tp, s);
}

template <int NA>
int decode_T(DecodeParams p, const void* x, int x_dtype, int scale_dtype, int64_t cap, bool tp, cudaStream_t s) {
  switch (p.T) {
    case 1: return decode_types<1, NA>(p, x, x_dtype, scale_dtype, cap, tp, s);
    case 2: return decode_types<2, NA>(p, x, x_dtype, scale_dtype, cap, tp, s);
    case 3: return decode_types<3, NA>(p, x, x_dtype, scale_dtype, cap, tp, s);
    case 4: return decode_types<4, NA>(p, x, x_dtype, scale_dtype, cap, tp, s);
    default: return set_error(PYRE_EINVAL, "pyre_ffn_decode_q80: T must be in [1, 4]");
  }
}

// Two-call workspace need (ffn.cu): header + the larger of the two piece regions.
int64_t twocall_ws_bytes(int T, int H, int W) {
  if (T > PYRE_FUSED_REDUCE_MAX_T) return kHeaderBytes;
  const int64_t a = pieces_bytes(T, W, 2), b = pieces_bytes(T, H, 1);
  return kHeaderBytes + (a > b ? a : b);
}

}  // namespace ffn
}  // namespace pyre

using namespace pyre;
using namespace pyre::ffn;

extern "C" int pyre_ffn_workspace_bytes(int T, int H, int W, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_ffn_workspace_bytes: null bytes");
  PYRE_CHECK_ARG(T >= 1 && H >= 1 && W >= 1, "pyre_ffn_workspace_bytes: sizes must be positive");
  int64_t need = twocall_ws_bytes(T, H, W);
  if (T <= PYRE_FUSED_REDUCE_MAX_T) {
    const int64_t d = decode_ws_bytes(T, H, W, 2);
    if (d > need) need = d;
  }
  *bytes = need;
  return PYRE_OK;
}

extern "C" int pyre_ffn_decode_q80(const void* x, int x_dtype, int T, int H, const void* wgu, int gated,
                                   const void* wd, int scale_dtype, int W, float* out, void* workspace,
                                   int64_t ws_bytes, pyre_comm_t* comm, void* stream) {
  int rc = ffn_check_common(x, x_dtype, T, H, W, scale_dtype, out, workspace, ws_bytes, "pyre_ffn_decode_q80");
  if (rc) return rc;
  PYRE_CHECK_ARG(T <= PYRE_FUSED_REDUCE_MAX_T, "pyre_ffn_decode_q80: T must be <= PYRE_FUSED_REDUCE_MAX_T");
  PYRE_CHECK_ARG(H % 32 == 0 && W % 32 == 0, "pyre_ffn_decode_q80: H and W must be multiples of 32");
  PYRE_CHECK_ARG(wgu != nullptr && wd != nullptr && reinterpret_cast<uintptr_t>(wgu) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(wd) % 16 == 0,
                 "pyre_ffn_decode_q80: packed weights must be non-null and 16-byte aligned");
  PYRE_CHECK_ARG(gemv::tiles_of(H) <= gemv::kMaxTiles && gemv::tiles_of(W) <= gemv::kMaxTiles,
                 "pyre_ffn_decode_q80: dims too large");
  if (comm != nullptr) {
    PYRE_CHECK_ARG(comm->hidden == H, "pyre_ffn_decode_q80: communicator hidden size differs from H");
    PYRE_CHECK_ARG(T <= comm->max_tokens, "pyre_ffn_decode_q80: T exceeds the communicator's max_tokens");
  }
  const int64_t need = decode_ws_bytes(T, H, W, gated ? 2 : 1);
  if (ws_bytes < need)
    return set_error(PYRE_ENOMEM, "pyre_ffn_decode_q80: workspace smaller than pyre_ffn_workspace_bytes()");
  char* wsc = static_cast<char*>(workspace);
  DecodeParams p{};
  p.wgu = static_cast<const uint8_t*>(wgu);
  p.wd = static_cast<const uint8_t*>(wd);
  p.H = H;
  p.W = W;
  p.T = T;
  const int ra = gated ? kUnitRowsPair : kUnitRowsSingle;
  p.tilesA = tiles_of(W);
  p.uptA = (H + ra - 1) / ra;
  p.tilesB = tiles_of(H);
  p.uptB = (W + kUnitRowsSingle - 1) / kUnitRowsSingle;
  p.UA = static_cast<int64_t>(p.tilesA) * p.uptA;
  p.UB = static_cast<int64_t>(p.tilesB) * p.uptB;
  p.h = reinterpret_cast<float*>(wsc + kHeaderBytes);
  p.out = out;
  p.wsA = reinterpret_cast<float*>(wsc + kHeaderBytes + align256(static_cast<int64_t>(T) * W * 4));
  p.wsB = nullptr;
  p.cntA = reinterpret_cast<unsigned int*>(wsc + kHdrCntA);
  p.cntB = reinterpret_cast<unsigned int*>(wsc + kHdrCntB);
  p.ready = reinterpret_cast<uint32_t*>(wsc + kHdrReady);
  p.ws_epoch = reinterpret_cast<uint32_t*>(wsc + kHdrEpoch);
  p.ws_done = reinterpret_cast<unsigned int*>(wsc + kHdrDone);
  p.status = reinterpret_cast<int*>(wsc + kHdrStatus);
  const bool tp = comm != nullptr && comm->world > 1;
  if (tp) p.comm = comm::device_view(comm);
  const int64_t cap = ws_bytes - (kHeaderBytes + align256(static_cast<int64_t>(T) * W * 4));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return gated ? decode_T<2>(p, x, x_dtype, scale_dtype, cap, tp, s) : decode_T<1>(p, x, x_dtype, scale_dtype, cap, tp, s);
}
