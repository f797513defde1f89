// The decode-path streaming kernel (T <= 4 tokens), one template for three uses:
//   MODE_A : h[T, N_A] = silu(x @ Wg) * (x @ Wu)  (or silu(x @ Wu))       -> pyre_ffn_gateup_silu_q80
//   MODE_B : out[T, N_B] = x @ Wd (+ cross-rank sum)                      -> pyre_ffn_down_q80
//   MODE_AB: both in one persistent launch, phase B fed by phase A        -> pyre_ffn_decode_q80
// Reference semantics: src/ffn/builder.py:37-45, src/orchestrator/root_node.py:956-995.
//
// Scheduling. A phase's work is its packed weight blocks (one 256-column slab x R rows
// each, see gemv_common.cuh), grouped per slab into chunks of kChunk consecutive blocks.
// The producer lane of every CTA takes chunks from a global atomic counter — all phase-A
// chunks first, then phase-B chunks — so faster SMs simply take more chunks (per-SM memory
// bandwidth on this part is not uniform). Each chunk's partial sums go to a fixed slot
// [slab][chunk]; the CTA finishing the last chunk of a slab adds the slots in chunk order
// (deterministic) and runs the epilogue. In MODE_AB the epilogue of a phase-A slab
// publishes a ready flag tagged with the call's epoch, and the producer waits for the flag
// of the slab holding rows k0.. of h before it loads that h slice for a phase-B block.
// Phase A never waits on phase B, all phase-A chunks are taken before any phase-B chunk,
// and every wait is bounded, so no wait can last forever.
#pragma once

#include "ffn_internal.cuh"

namespace pyre {
namespace ffn {

constexpr int MODE_A = 1;
constexpr int MODE_B = 2;
constexpr int MODE_AB = 3;
constexpr int kChunk = 8;   // blocks per chunk

struct alignas(64) StreamParams {
  CUtensorMap txa;           // phase-A activation x [T, KA], box T x R_A
  CUtensorMap txb;           // phase-B activation [T, KB] (h in MODE_AB), box T x R_B
  const uint8_t* wa;         // packed gate/up pair or up alone
  const uint8_t* wb;         // packed down
  int T;
  int KA, NA, tilesA, uptA, cptA;   // phase A: K, N, slabs, blocks per slab, chunks per slab
  int KB, NB, tilesB, uptB, cptB;
  int ncA, ncB;                     // chunks in each phase
  void* outA;                // [T, NA]: h
  int outA_bf16;
  float* outB;               // [T, NB]
  float* wsA;                // [tilesA, cptA, NMAT_A * T * 256]
  float* wsB;                // [tilesB, cptB, T * 256]
  unsigned int* cntA;        // [tilesA] finished chunks
  unsigned int* cntB;
  uint32_t* ready;           // [tilesA] per-slab ready flags (MODE_AB)
  unsigned int* next;        // [2] chunk counters of phase A and B
  uint32_t* ws_epoch;
  unsigned int* ws_done;
  int* status;
  comm::DevComm comm;
};

constexpr int kMaxOwnedTiles = 64;   // tensor-parallel: slabs one CTA may finish (H <= 16384)

template <int T, int NA, typename XA, typename XB, typename ST>
struct StreamCfg {
  using LA = StageLayout<T, NA, XA, ST>;
  using LB = StageLayout<T, 1, XB, ST>;
  static constexpr int kStageBytes = LA::kBytes > LB::kBytes ? LA::kBytes : LB::kBytes;
  static constexpr int kCtasPerSm = (T <= 2) ? 2 : 1;
  static constexpr int kStages = (T <= 2) ? 4 : 5;
  static constexpr int kRedFloats = kConsumerWarps * NA * T * kTileN;
  static constexpr int kFinFloats = NA * T * kTileN;
  static constexpr int kSmemBytes = kStages * kStageBytes + (kRedFloats + kFinFloats) * 4 + 2 * kStages * 8 +
                                    kStages * 16 + 16 + (kMaxOwnedTiles + 1) * 4;
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

// Bounded wait for a per-slab ready flag (2 s); records PYRE_ETIMEOUT and returns false
// on expiry.
__device__ __forceinline__ bool wait_ready(const uint32_t* flag, uint32_t epoch, int* status) {
  if (ld_acquire_gpu(flag) == epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_gpu(flag) != epoch) {
    if (globaltimer_ns() - t0 > 2000000000ull) {
      atomicExch(status, PYRE_ETIMEOUT);
      return false;
    }
    __nanosleep(20);
  }
  return true;
}

// Stage descriptor written by the producer next to each stage: phase (0 = A, 1 = B,
// -1 = end), slab, chunk within the slab, and whether this block closes its chunk.
struct StageMeta {
  int phase, tile, chunk, last;
};

// Sums the chunk slots of a slab after its last chunk arrived; returns true in the CTA
// that must run the slab epilogue (the sums are then in fin).
template <int T, int NMAT>
__device__ __forceinline__ bool chunk_fixup(float* fin, float* ws, unsigned int* cnt, int cpt, int tile, int chunk,
                                            int* s_last, int tid) {
  constexpr int kItems = NMAT * T * kTileN;
  if (cpt == 1) return true;
  float* slot = ws + (static_cast<int64_t>(tile) * cpt + chunk) * kItems;
  for (int i = tid; i < kItems; i += kConsumers) __stcg(slot + i, fin[i]);
  __threadfence();
  consumer_sync();
  if (tid == 0) {
    const unsigned prev = atomicAdd(cnt + tile, 1u);
    *s_last = (prev == static_cast<unsigned>(cpt - 1));
  }
  consumer_sync();
  if (!*s_last) return false;
  __threadfence();
  const float* base = ws + static_cast<int64_t>(tile) * cpt * kItems;
  for (int i = tid; i < kItems; i += kConsumers) {
    float v = 0.f;
    for (int pc0 = 0; pc0 < cpt; pc0 += 16) {
      float pv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) pv[j] = (pc0 + j < cpt) ? __ldcg(base + static_cast<int64_t>(pc0 + j) * kItems + i) : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (pc0 + j < cpt) v += pv[j];
    }
    fin[i] = v;
  }
  consumer_sync();
  if (tid == 0) cnt[tile] = 0u;
  return true;
}

template <int T, int NA, typename XA, typename XB, typename ST, int MODE, bool TP>
__global__ void __launch_bounds__(kThreads, (StreamCfg<T, NA, XA, XB, ST>::kCtasPerSm))
q80_ffn_stream_kernel(const __grid_constant__ StreamParams p) {
  using C = StreamCfg<T, NA, XA, XB, ST>;
  using LA = typename C::LA;
  using LB = typename C::LB;
  constexpr bool kHasA = (MODE & MODE_A) != 0;
  constexpr bool kHasB = (MODE & MODE_B) != 0;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  float* red = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  float* fin = red + C::kRedFloats;
  uint64_t* full = reinterpret_cast<uint64_t*>(fin + C::kFinFloats);
  uint64_t* empty = full + C::kStages;
  StageMeta* meta = reinterpret_cast<StageMeta*>(empty + C::kStages);
  int* s_last = reinterpret_cast<int*>(meta + C::kStages);
  int* owned = s_last + 4;           // [0]: count, then slab ids (tensor-parallel finish)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    owned[0] = 0;
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
      if constexpr (kHasA) prefetch_tmap(&p.txa);
      if constexpr (kHasB) prefetch_tmap(&p.txb);
      int s = 0;
      uint32_t ph = 0;
      // Failure handling: after any wait runs out (here or in another CTA, seen through the
      // status word) the producer issues no more copies, still tries to hand the consumers
      // their end marker, and waits (bounded) for the copies it already issued, so that no
      // copy into this CTA's shared memory is in flight when it exits.
      bool ok = true;
      uint32_t issued = 0, par = 0;   // stages with an unconfirmed copy, and that copy's parity
      auto acquire = [&]() -> bool {
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) return false;
        issued &= ~(1u << s);           // the consumers released the stage: its copy landed
        return true;
      };
      auto issue_done = [&]() {
        issued |= 1u << s;
        par = (par & ~(1u << s)) | (ph << s);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
      };
      auto failed = [&]() { return *reinterpret_cast<volatile int*>(p.status) != PYRE_OK; };
      if constexpr (kHasA) {
        while (ok) {
          if (failed()) {
            ok = false;
            break;
          }
          const int ch = static_cast<int>(atomicAdd(p.next, 1u));
          if (ch >= p.ncA) break;
          const int tile = ch / p.cptA, chunk = ch - tile * p.cptA;
          const int u0 = chunk * kChunk;
          const int u1 = min(u0 + kChunk, p.uptA);
          for (int u = u0; u < u1; ++u) {
            if (!acquire()) {
              ok = false;
              break;
            }
            meta[s] = StageMeta{0, tile, chunk, u + 1 == u1};
            uint8_t* st = stages + s * C::kStageBytes;
            mbar_arrive_expect_tx(&full[s], LA::kTxBytes);
            bulk_load(st, p.wa + (static_cast<int64_t>(tile) * p.uptA + u) * LA::kWBytes, LA::kWBytes, &full[s]);
            tma_load_2d(st + LA::kXOff, &p.txa, u * LA::kRows, 0, &full[s]);
            issue_done();
          }
        }
      }
      if constexpr (kHasB) {
        while (ok) {
          if (failed()) {
            ok = false;
            break;
          }
          const int ch = static_cast<int>(atomicAdd(p.next + 1, 1u));
          if (ch >= p.ncB) break;
          const int tile = ch / p.cptB, chunk = ch - tile * p.cptB;
          const int u0 = chunk * kChunk;
          const int u1 = min(u0 + kChunk, p.uptB);
          for (int u = u0; u < u1; ++u) {
            if (!acquire()) {
              ok = false;
              break;
            }
            meta[s] = StageMeta{1, tile, chunk, u + 1 == u1};
            uint8_t* st = stages + s * C::kStageBytes;
            mbar_arrive_expect_tx(&full[s], LB::kTxBytes);
            bulk_load(st, p.wb + (static_cast<int64_t>(tile) * p.uptB + u) * LB::kWBytes, LB::kWBytes, &full[s]);
            const int k0 = u * LB::kRows;
            bool rdy = true;
            if constexpr (MODE == MODE_AB) {
              // rows k0..k0+R_B-1 of h come from phase-A slab k0 / 256 (R_B divides 256)
              rdy = wait_ready(p.ready + k0 / kTileN, epoch, p.status);
              fence_proxy_async_global();
            }
            // issued even when the flag wait ran out, so the stage's byte count completes
            tma_load_2d(st + LB::kXOff, &p.txb, k0, 0, &full[s]);
            issue_done();
            if (!rdy) {
              ok = false;
              break;
            }
          }
        }
      }
      // end marker for the consumers
      if (acquire()) {
        meta[s] = StageMeta{-1, 0, 0, 0};
        mbar_arrive(&full[s]);
      }
      if (!ok) {
        for (int i = 0; i < C::kStages; ++i)
          if ((issued >> i) & 1u) mbar_wait(&full[i], (par >> i) & 1u, nullptr, 500000000ull);
      }
    }
  } else {
    // ---------------- consumers ----------------
    const int tid = threadIdx.x;
    const int rs = lane >> 4;
    const int cc = lane & 15;
    int s = 0;
    uint32_t ph = 0;
    float2 acc[NA][T][8];
    zero_acc<NA, T>(acc);
    while (true) {
      // longer than any producer wait, so a producer that gave up reaches us with the end marker
      if (!mbar_wait(&full[s], ph, p.status, 4000000000ull)) break;
      const StageMeta m = meta[s];
      if (m.phase < 0) break;
      const uint8_t* st = stages + s * C::kStageBytes;
      if (kHasA && m.phase == 0) {
        consume_unit<T, NA, XA, ST>(st, acc, warp, rs, cc);
      } else if constexpr (kHasB) {
        float2(&acc1)[1][T][8] = reinterpret_cast<float2(&)[1][T][8]>(acc);
        consume_unit<T, 1, XB, ST>(st, acc1, warp, rs, cc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == C::kStages) {
        s = 0;
        ph ^= 1u;
      }
      if (!m.last) continue;
      // a chunk is complete: reduce it, fix up its slab, run the slab epilogue
      if (kHasA && m.phase == 0) {
        reduce_tile<T, NA>(acc, red, fin, warp, rs, cc, tid);
        zero_acc<NA, T>(acc);
        if (chunk_fixup<T, NA>(fin, p.wsA, p.cntA, p.cptA, m.tile, m.chunk, s_last, tid)) {
          for (int i = tid; i < T * kTileN; i += kConsumers) {
            const int t = i / kTileN, col = m.tile * kTileN + (i % kTileN);
            if (col >= p.NA) continue;
            const float v = (NA == 2) ? silu_f32(fin[i]) * fin[T * kTileN + i] : silu_f32(fin[i]);
            store_out(p.outA, p.outA_bf16, p.NA, t, col, v);
          }
          if constexpr (MODE == MODE_AB) {
            __threadfence();
            fence_proxy_async_global();
            consumer_sync();
            if (tid == 0) st_release_gpu(p.ready + m.tile, epoch);
          }
        }
      } else if constexpr (kHasB) {
        float2(&acc1)[1][T][8] = reinterpret_cast<float2(&)[1][T][8]>(acc);
        reduce_tile<T, 1>(acc1, red, fin, warp, rs, cc, tid);
        zero_acc<NA, T>(acc);
        if (chunk_fixup<T, 1>(fin, p.wsB, p.cntB, p.cptB, m.tile, m.chunk, s_last, tid)) {
          if constexpr (TP) {
            tp_push_tile<T>(p.comm, cepoch, m.tile, fin, tid);
            if (tid == 0) owned[1 + owned[0]++] = m.tile;
          } else {
            for (int i = tid; i < T * kTileN; i += kConsumers) {
              const int t = i / kTileN, col = m.tile * kTileN + (i % kTileN);
              if (col < p.NB) p.outB[static_cast<int64_t>(t) * p.NB + col] = fin[i];
            }
          }
        }
      }
      consumer_sync();
    }
    if constexpr (TP) {
      // every chunk of this CTA is done: now wait for the peers of the slabs it finished
      const int n_owned = owned[0];
      for (int i = 0; i < n_owned; ++i) tp_finish_tile<T>(p.comm, cepoch, owned[1 + i], p.outB, p.NB, tid);
    }
  }
  __syncthreads();
  if constexpr (TP) comm::epoch_end(p.comm, cepoch);
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.ws_done, 1u);
    if (prev == gridDim.x - 1) {
      // last CTA: reset the chunk counters and publish the epoch for the next call
      p.next[0] = 0u;
      p.next[1] = 0u;
      *reinterpret_cast<volatile unsigned int*>(p.ws_done) = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(p.ws_epoch) = epoch;
    }
  }
}

}  // namespace ffn
}  // namespace pyre
