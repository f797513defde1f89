// The decode-path streaming kernel (T <= 4 tokens), one template for three uses:
//   MODE_A : h[T, N_A] = silu(x @ Wg) * (x @ Wu)  (or silu(x @ Wu))       -> pyre_ffn_gateup_silu_q80
//   MODE_B : out[T, N_B] = x @ Wd (+ cross-rank sum)                      -> pyre_ffn_down_q80
//   MODE_AB: both in one persistent launch, phase B fed by phase A        -> pyre_ffn_decode_q80
// Reference semantics: src/ffn/builder.py:37-45, src/orchestrator/root_node.py:956-995.
//
// Scheduling. A phase's work is its packed weight blocks (one 256-column slab x R rows
// each, see gemv_common.cuh), grouped per slab into chunks of kChunk consecutive blocks.
// The producer lane of every CTA takes chunks from one global atomic counter, so faster SMs
// simply take more chunks (per-SM memory bandwidth on this part is not uniform).
//
// Slab sums. Each chunk's partial sums are added into the slab's accumulator as 64-bit
// fixed point (value * 2^32, |value| < 2^30) with integer atomics: integer addition is
// associative, so the sums are bit-identical whatever CTA ran which chunk and in what
// order, and the adds are fire-and-forget. The consumers hand each finished chunk to a
// helper warp, which counts it for its slab (release); the helper that counts a slab's last
// chunk reads the accumulator back, clears it for the next call and runs the slab epilogue
// (SiLU-mul and h store, or the output store / cross-rank push) while its consumers stream on.
//
// MODE_AB keeps no h. The gate/up slab sums are read directly by the phase-B stages that need
// them: the producer waits (acquire) until the slab's chunk count reaches cptA, then copies the
// sums of the stage's R_B rows next to the down block, and each consumer warp computes
// h = silu(g) * u of the rows it reads (the same arithmetic as the slab epilogue). A slab thus
// becomes usable one count after its last chunk instead of after count, read-back, h store and
// flag release, every one a round trip through a fully loaded memory system. The sums and
// counts stay in place until the next call, so there are two sets used by alternate calls
// (ab_calls parity): each call clears the other set, which the previous call used.
//
// MODE_AB queue. Phase-B chunk column c (chunk c of every output slab) reads rows
// [c*512, c*512+512) of h, which phase-A slabs [c*spg, c*spg+spg) produce (group c). The
// queue is: groups 0..slack-1 of phase A, then for each later group g its phase-A chunks
// followed by phase-B column g-slack, then the last `slack` phase-B columns. Phase B thus
// runs alongside phase A instead of after it, each phase-B column comes about `slack`
// groups after the rows it reads, and the tail is short chunks of both phases. The producer
// waits for the chunk count of the slab holding rows k0.. of h before it copies its sums.
// No deadlock: every chunk depends only on phase-A chunks earlier in the queue, chunks are
// taken in queue order by running CTAs, and a CTA's stages are consumed in order, so the
// earliest unfinished chunk can always proceed. Every wait is bounded besides.
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
  int spg, slack;                   // MODE_AB queue: phase-A slabs per group, groups of lead
  void* outA;                // [T, NA]: h
  int outA_bf16;
  float* outB;               // [T, NB]
  const float* biasB;        // MODE_B without tensor parallelism: f32 [NB] added to out, or null
  unsigned long long* accA;  // [tilesA, NMAT_A, T, 256] fixed-point slab sums (zero between calls)
  unsigned long long* accB;  // [tilesB, T, 256]
  unsigned int* cntA;        // [tilesA] finished chunks
  unsigned int* cntB;
  uint32_t* ready;           // [tilesA] per-slab ready flags (MODE_AB)
  unsigned int* next;        // queue position counter
  unsigned long long* sumA;  // MODE_AB: [2][tilesA][kSlabSums] gate/up slab sums, one set per call parity
  unsigned int* cntAB;       // MODE_AB: [2][tilesA] finished phase-A chunks, one set per call parity
  unsigned int* ab_calls;    // MODE_AB: calls made so far on this workspace (its parity picks the set)
  uint32_t* ws_epoch;
  unsigned int* ws_done;
  int* status;
  comm::DevComm comm;
};

constexpr int kMaxOwnedTiles = 64;   // tensor-parallel: slabs one CTA may finish (H <= 16384)

// MODE_AB slab sums: per phase-A slab [2 matrices][PYRE_FUSED_REDUCE_MAX_T tokens][kTileN] int64,
// the same layout for every T and for gated or not, so calls of any shape can share a workspace.
constexpr int kSumT = PYRE_FUSED_REDUCE_MAX_T;
constexpr int kSlabSums = 2 * kSumT * kTileN;

// Warp roles: kConsumerWarps consumers, one producer, kHelperWarps helpers.
constexpr int kHelperWarps = 1;
constexpr int kHelpers = kHelperWarps * 32;
constexpr int kStreamThreads = kThreads + kHelpers;
constexpr int kJobs = 4;             // finished chunks queued from the consumers to the helpers
static_assert(kHelpers == 32, "the slab read-back maps one helper lane to column pairs");

template <int T, int NA, typename XA, typename XB, typename ST>
struct StreamCfg {
  using LA = StageLayout<T, NA, XA, ST>;
  using LB = StageLayout<T, 1, XB, ST>;
  // MODE_AB phase-B stage: packed down block, then h of its rows (f32 [T][R_B], computed by the
  // consumers), then the slab sums those rows come from ([NA][T][R_B] int64, one bulk copy each)
  static constexpr int kSumOff = LB::kXOff + LB::kXBytes;
  static constexpr int kSumBytesMax = 2 * T * LB::kRows * 8;
  static constexpr int kBytesAB = (kSumOff + kSumBytesMax + 127) / 128 * 128;
  static constexpr int kStageBytes = LA::kBytes > kBytesAB ? LA::kBytes : kBytesAB;
  static constexpr int kCtasPerSm = (T <= 2) ? 2 : 1;
  static constexpr int kStages = (T <= 2) ? 4 : 5;
  static constexpr int kRedFloats = kConsumerWarps * NA * T * kTileN;
  static constexpr int kSmemBytes = kStages * kStageBytes + kRedFloats * 4 + 2 * kStages * 8 + kStages * 16 +
                                    2 * kJobs * 8 + kJobs * 16 + 16 + (kMaxOwnedTiles + 1) * 4;
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait (2 s) until a flag or counter word equals `epoch` (acquire); records
// PYRE_ETIMEOUT and returns false on expiry.
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

// A finished chunk handed from the consumers to the helper warps (end = no more chunks).
struct Job {
  int phase, tile, chunk, end;
};

__device__ __forceinline__ void helper_sync() { named_bar(2, kHelpers); }

// Fixed-point slab sums: 2^32 scale; partials are limited to |v| < 2^30, so a slab sum of
// up to 2^32 partials cannot leave int64 (the quantum, 2^-32, is far below f32 rounding of
// the values an FFN produces).
constexpr float kFixScale = 4294967296.0f;            // 2^32
constexpr float kFixInv = 2.3283064365386963e-10f;    // 2^-32
constexpr float kFixLimit = 1073741824.0f;            // 2^30

// Sums acc over the two row lanes and all consumer warps (in warp order) and adds the
// chunk's partial [NMAT][T][kTileN] into the slab accumulator, laid out [NMAT][TS][kTileN]
// (TS >= T tokens of stride). A partial that is not finite or not below 2^30 in magnitude is
// added as 0 and flags PYRE_ERANGE. kProxy: the sums are read next by bulk copies (async
// proxy), so every adding thread fences its adds against that proxy.
// red: kConsumerWarps * NMAT * T * kTileN floats.
template <int T, int NMAT, int TS = T, bool kProxy = false>
__device__ __forceinline__ void reduce_to_acc(float2 (&acc)[NMAT][T][8], float* red, unsigned long long* accum,
                                              int* status, int warp, int rs, int cc, int tid) {
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
  constexpr int kItems = NMAT * T * kTileN;
  for (int i = tid; i < kItems; i += kConsumers) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) v += red[w * kItems + i];
    if (!(fabsf(v) < kFixLimit)) {
      atomicCAS(status, PYRE_OK, PYRE_ERANGE);
      v = 0.f;
    }
    const int row = i / kTileN, m = row / T;
    atomicAdd(accum + (m * TS + (row - m * T)) * kTileN + (i - row * kTileN),
              static_cast<unsigned long long>(__float2ll_rn(v * kFixScale)));
  }
  if constexpr (kProxy) fence_proxy_async_global();
  consumer_sync();   // red is rewritten at the next chunk's end
}

// Helper-warp read-back of a finished slab accumulator: for this lane's column pairs,
// returns the sums of the M rows at row offsets off[m] (in floats of the [.., kTileN] grid)
// as f32 and clears them. kPairs column pairs per call, lane-strided.
template <int M, int kPairs>
__device__ __forceinline__ void take_acc(unsigned long long* base, const int (&off)[M], int pair0, float2 (&out)[kPairs][M]) {
  ulonglong2 v[kPairs][M];
#pragma unroll
  for (int k = 0; k < kPairs; ++k)
#pragma unroll
    for (int m = 0; m < M; ++m)
      v[k][m] = __ldcg(reinterpret_cast<const ulonglong2*>(base + off[m]) + pair0 + k * 32);
#pragma unroll
  for (int k = 0; k < kPairs; ++k)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      __stcg(reinterpret_cast<ulonglong2*>(base + off[m]) + pair0 + k * 32, make_ulonglong2(0ull, 0ull));
      out[k][m] = make_float2(__ll2float_rn(static_cast<long long>(v[k][m].x)) * kFixInv,
                              __ll2float_rn(static_cast<long long>(v[k][m].y)) * kFixInv);
    }
}

// Queue position -> chunk for MODE_AB (see the scheduling note above). Returns false past
// the end; tile may be >= tilesA for the padding slabs of a short last group (skipped).
__host__ __device__ __forceinline__ bool ab_item(const StreamParams& p, int pos, int& phase, int& tile, int& chunk) {
  const int sA = p.spg * p.cptA, sB = p.tilesB, G = p.cptB, D = min(p.slack, G);
  int g, j;
  if (pos < D * sA) {
    g = pos / sA;
    j = pos - g * sA;
  } else {
    const int q = pos - D * sA;
    const int mid = (G - D) * (sA + sB);
    if (q < mid) {
      const int k = q / (sA + sB);
      j = q - k * (sA + sB);
      if (j >= sA) {
        phase = 1;
        chunk = k;
        tile = j - sA;
        return true;
      }
      g = D + k;
    } else {
      const int r = q - mid;
      if (r >= D * sB) return false;
      phase = 1;
      chunk = G - D + r / sB;
      tile = r - (r / sB) * sB;
      return true;
    }
  }
  phase = 0;
  tile = g * p.spg + j / p.cptA;
  chunk = j - (j / p.cptA) * p.cptA;
  return true;
}

template <int T, int NA, typename XA, typename XB, typename ST, int MODE, bool TP>
__global__ void __launch_bounds__(kStreamThreads, (StreamCfg<T, NA, XA, XB, ST>::kCtasPerSm))
q80_ffn_stream_kernel(const __grid_constant__ StreamParams p) {
  using C = StreamCfg<T, NA, XA, XB, ST>;
  using LA = typename C::LA;
  using LB = typename C::LB;
  constexpr bool kHasA = (MODE & MODE_A) != 0;
  constexpr bool kHasB = (MODE & MODE_B) != 0;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  float* red = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + C::kRedFloats);
  uint64_t* empty = full + C::kStages;
  uint64_t* job_full = empty + C::kStages;
  uint64_t* job_empty = job_full + kJobs;
  StageMeta* meta = reinterpret_cast<StageMeta*>(job_empty + kJobs);
  Job* jobs = reinterpret_cast<Job*>(meta + C::kStages);
  int* s_last = reinterpret_cast<int*>(jobs + kJobs);
  int* owned = s_last + 4;           // [0]: count, then slab ids (tensor-parallel finish)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    for (int i = 0; i < kJobs; ++i) {
      mbar_init(&job_full[i], kConsumerWarps);
      mbar_init(&job_empty[i], 1);
    }
    owned[0] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // Programmatic dependent launch: every thread but the producer's waits here until the
  // previous kernel of the stream has finished. The producer first issues the weight copies
  // of its first chunk (weights are constant; the chunk is this CTA's fixed first item, so
  // the workspace is not touched), then waits before any activation load or workspace access.
  const bool producer = warp == kConsumerWarps && lane == 0;
  uint32_t epoch = 0, cepoch = 0, ab_call = 0;
  if (!producer) {
    pdl_wait();
    // epoch of this call; published by the last CTA to exit
    epoch = *reinterpret_cast<volatile uint32_t*>(p.ws_epoch) + 1u;
    if constexpr (MODE == MODE_AB) ab_call = *reinterpret_cast<volatile uint32_t*>(p.ab_calls);
    if constexpr (TP) cepoch = comm::epoch_begin(p.comm);
  }
  // MODE_AB: slab sums and chunk counts of a call parity (this call's: ab_call & 1; the other
  // set is the previous call's, cleared during this call for the next one)
  auto sums_of = [&](uint32_t q) { return p.sumA + static_cast<int64_t>(q & 1u) * p.tilesA * kSlabSums; };
  auto cnt_of = [&](uint32_t q) { return p.cntAB + static_cast<int64_t>(q & 1u) * p.tilesA; };

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      if constexpr (kHasA) prefetch_tmap(&p.txa);
      if constexpr (kHasB && MODE != MODE_AB) prefetch_tmap(&p.txb);
      int s = 0;
      uint32_t ph = 0;
      // activation loads of the stages issued before pdl_wait (at most one ring of stages)
      bool dep = false;
      int ndef = 0;
      int def_s[C::kStages], def_k[C::kStages];
      bool def_b[C::kStages];
      auto resolve = [&]() {
        if (dep) return;
        pdl_wait();
        pdl_trigger();
        dep = true;
        epoch = *reinterpret_cast<volatile uint32_t*>(p.ws_epoch) + 1u;
        if constexpr (MODE == MODE_AB) ab_call = *reinterpret_cast<volatile uint32_t*>(p.ab_calls);
        for (int i = 0; i < ndef; ++i) {
          uint8_t* st = stages + def_s[i] * C::kStageBytes;
          if (def_b[i]) {
            if constexpr (kHasB) tma_load_2d(st + LB::kXOff, &p.txb, def_k[i], 0, &full[def_s[i]]);
          } else {
            if constexpr (kHasA) tma_load_2d(st + LA::kXOff, &p.txa, def_k[i], 0, &full[def_s[i]]);
          }
        }
        ndef = 0;
      };
      // Failure handling: after any wait runs out (here or in another CTA, seen as
      // PYRE_ETIMEOUT in the status word) the producer issues no more copies, still tries to hand the consumers
      // their end marker, and waits (bounded) for the copies it already issued, so that no
      // copy into this CTA's shared memory is in flight when it exits.
      bool ok = true;
      uint32_t issued = 0, par = 0;   // stages with an unconfirmed copy, and that copy's parity
      // MODE_AB: the last phase-A slab this producer has seen complete (its count acquired and
      // the proxy fence done); the following units of the same slab need no second round trip
      int seen_slab = -1;
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
      auto failed = [&]() { return *reinterpret_cast<volatile int*>(p.status) == PYRE_ETIMEOUT; };
      // issues the stages of one chunk; false once a wait ran out
      auto issue_chunk = [&](int phase, int tile, int chunk) -> bool {
        if (phase == 0) {
          if constexpr (kHasA) {
            const int u0 = chunk * kChunk;
            const int u1 = min(u0 + kChunk, p.uptA);
            for (int u = u0; u < u1; ++u) {
              if (ndef == C::kStages) resolve();   // the ring is full of stages waiting for x
              if (!acquire()) return false;
              meta[s] = StageMeta{0, tile, chunk, u + 1 == u1};
              uint8_t* st = stages + s * C::kStageBytes;
              mbar_arrive_expect_tx(&full[s], LA::kTxBytes);
              bulk_load(st, p.wa + (static_cast<int64_t>(tile) * p.uptA + u) * LA::kWBytes, LA::kWBytes, &full[s]);
              if (dep) {
                tma_load_2d(st + LA::kXOff, &p.txa, u * LA::kRows, 0, &full[s]);
              } else {
                def_s[ndef] = s;
                def_k[ndef] = u * LA::kRows;
                def_b[ndef] = false;
                ++ndef;
              }
              issue_done();
            }
          }
        } else {
          if constexpr (kHasB) {
            const int u0 = chunk * kChunk;
            const int u1 = min(u0 + kChunk, p.uptB);
            // MODE_AB: h comes from this kernel's own phase-A sums, read only after the wait
            if (MODE == MODE_AB) resolve();
            for (int u = u0; u < u1; ++u) {
              if (ndef == C::kStages) resolve();
              if (!acquire()) return false;
              meta[s] = StageMeta{1, tile, chunk, u + 1 == u1};
              uint8_t* st = stages + s * C::kStageBytes;
              if constexpr (MODE == MODE_AB) {
                // the down block, and the gate/up slab sums of its R_B rows of h (slab k0 / 256;
                // R_B divides 256) once every chunk of that slab has counted; a slab already
                // seen complete in this call needs no second acquire
                constexpr uint32_t kSumPiece = LB::kRows * 8;
                mbar_arrive_expect_tx(&full[s], LB::kWBytes + NA * T * kSumPiece);
                bulk_load(st, p.wb + (static_cast<int64_t>(tile) * p.uptB + u) * LB::kWBytes, LB::kWBytes, &full[s]);
                const int k0 = u * LB::kRows;
                const int slab = k0 / kTileN;
                bool rdy = true;
                if (slab != seen_slab) {
                  rdy = wait_ready(cnt_of(ab_call) + slab, static_cast<uint32_t>(p.cptA), p.status);
                  fence_proxy_async_global();
                  if (rdy) seen_slab = slab;
                }
                // issued even when the wait ran out, so the stage's byte count completes
                const unsigned long long* src =
                    sums_of(ab_call) + static_cast<int64_t>(slab) * kSlabSums + (k0 - slab * kTileN);
#pragma unroll
                for (int m = 0; m < NA; ++m)
#pragma unroll
                  for (int t = 0; t < T; ++t)
                    bulk_load(st + C::kSumOff + (m * T + t) * kSumPiece, src + (m * kSumT + t) * kTileN, kSumPiece,
                              &full[s]);
                issue_done();
                if (!rdy) return false;
                continue;
              }
              mbar_arrive_expect_tx(&full[s], LB::kTxBytes);
              bulk_load(st, p.wb + (static_cast<int64_t>(tile) * p.uptB + u) * LB::kWBytes, LB::kWBytes, &full[s]);
              const int k0 = u * LB::kRows;
              if (!dep) {
                def_s[ndef] = s;
                def_k[ndef] = k0;
                def_b[ndef] = true;
                ++ndef;
                issue_done();
                continue;
              }
              tma_load_2d(st + LB::kXOff, &p.txb, k0, 0, &full[s]);
              issue_done();
            }
          }
        }
        return true;
      };
      // queue items: blockIdx.x first (fixed, so it can be issued before the wait), then
      // gridDim.x + the shared counter's values
      bool first = true;
      while (ok) {
        int pos = static_cast<int>(blockIdx.x);
        if (!first) {
          resolve();
          if (failed()) {
            ok = false;
            break;
          }
          pos = static_cast<int>(gridDim.x + atomicAdd(p.next, 1u));
        }
        first = false;
        int phase, tile, chunk;
        if constexpr (MODE == MODE_AB) {
          if (!ab_item(p, pos, phase, tile, chunk)) break;
          if (phase == 0 && tile >= p.tilesA) continue;
        } else if constexpr (MODE == MODE_A) {
          if (pos >= p.ncA) break;
          phase = 0;
          tile = pos / p.cptA;
          chunk = pos - tile * p.cptA;
        } else {
          if (pos >= p.ncB) break;
          // chunk-major, like the MODE_AB queue
          phase = 1;
          chunk = pos / p.tilesB;
          tile = pos - chunk * p.tilesB;
        }
        ok = issue_chunk(phase, tile, chunk);
      }
      resolve();   // deferred activation loads, and the wait, even for a CTA with no item
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
  } else if (warp < kConsumerWarps) {
    // ---------------- consumers ----------------
    // Stream stages into register accumulators; at the end of each chunk add it into its
    // slab accumulator and queue it for the helper warp, which counts it and runs the slab
    // epilogue while the consumers go on with the next chunk.
    const int tid = threadIdx.x;
    const int rs = lane >> 4;
    const int cc = lane & 15;
    int s = 0;
    uint32_t ph = 0;
    int jb = 0;
    uint32_t jph = 0;
    auto post_job = [&](const Job& job) {
      // every warp waits for the slot so that no arrival runs a phase ahead of the helpers
      if (lane == 0) mbar_wait(&job_empty[jb], jph ^ 1u, p.status);
      __syncwarp();
      if (tid == 0) jobs[jb] = job;
      __syncwarp();
      if (lane == 0) mbar_arrive(&job_full[jb]);
      if (++jb == kJobs) {
        jb = 0;
        jph ^= 1u;
      }
    };
    float2 acc[NA][T][8];
    zero_acc<NA, T>(acc);
    while (true) {
      // longer than any producer wait, so a producer that gave up reaches us with the end marker
      if (!mbar_wait(&full[s], ph, p.status, 4000000000ull)) break;
      const StageMeta m = meta[s];
      if (m.phase < 0) break;
      const uint8_t* st = stages + s * C::kStageBytes;
      if constexpr (MODE == MODE_AB) {
        if (m.phase == 1) {
          // h of the rows this warp reads (row pass * 16 + 2 * warp + rs of every pass, every
          // token) from the gate/up slab sums, with the arithmetic of the slab epilogue: silu(g) * u
          // of the fixed-point sums scaled back to f32; written where consume_unit reads it
          constexpr int kWarpRows = LB::kRows / kRowsPerPass * 2;
          if (lane < T * kWarpRows) {
            const int t = lane / kWarpRows, j = lane - t * kWarpRows;
            const int r = (j >> 1) * kRowsPerPass + warp * 2 + (j & 1);
            const long long* sm = reinterpret_cast<const long long*>(st + C::kSumOff);
            float h = silu_f32(__ll2float_rn(sm[t * LB::kRows + r]) * kFixInv);
            if constexpr (NA == 2) h *= __ll2float_rn(sm[(T + t) * LB::kRows + r]) * kFixInv;
            reinterpret_cast<float*>(stages + s * C::kStageBytes + LB::kXOff)[t * LB::kRows + r] = h;
          }
          __syncwarp();
        }
      }
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
      if (MODE == MODE_AB && m.phase == 0) {
        reduce_to_acc<T, NA, kSumT, true>(acc, red, sums_of(ab_call) + static_cast<int64_t>(m.tile) * kSlabSums,
                                          p.status, warp, rs, cc, tid);
      } else if (kHasA && m.phase == 0) {
        reduce_to_acc<T, NA>(acc, red, p.accA + static_cast<int64_t>(m.tile) * (NA * T * kTileN), p.status, warp, rs,
                             cc, tid);
      } else if constexpr (kHasB) {
        float2(&acc1)[1][T][8] = reinterpret_cast<float2(&)[1][T][8]>(acc);
        reduce_to_acc<T, 1>(acc1, red, p.accB + static_cast<int64_t>(m.tile) * (T * kTileN), p.status, warp, rs, cc,
                            tid);
      }
      zero_acc<NA, T>(acc);
      post_job(Job{m.phase, m.tile, m.chunk, 0});
    }
    post_job(Job{0, 0, 0, 1});
  } else {
    // ---------------- helpers ----------------
    // Per finished chunk: count it for its slab (release); the CTA that counts a slab's
    // last chunk reads the slab sums back and runs the slab epilogue.
    const int htid = threadIdx.x - (kThreads);
    int jb = 0;
    uint32_t jph = 0;
    while (true) {
      if (!mbar_wait(&job_full[jb], jph, p.status, 8000000000ull)) break;
      const Job job = jobs[jb];
      helper_sync();
      if (htid == 0) mbar_arrive(&job_empty[jb]);
      if (++jb == kJobs) {
        jb = 0;
        jph ^= 1u;
      }
      if (job.end) break;
      const bool isA = kHasA && job.phase == 0;
      if constexpr (MODE == MODE_AB) {
        if (isA) {
          // count the chunk for its slab: the consumers' sum adds (each fenced against the async
          // proxy) are ordered before this (barrier, then mbarrier release/acquire) and the fence
          // makes them visible GPU-wide before the count; the phase-B producers wait for the
          // count to reach cptA, then read the sums with bulk copies
          if (htid == 0) {
            __threadfence();
            atomicAdd(cnt_of(ab_call) + job.tile, 1u);
          }
          // clear this chunk's share of the slab's sums and count of the previous call (the
          // other set), which the next call uses: blocks of 32 words, block b for chunk b % cptA
          unsigned long long* old = sums_of(ab_call ^ 1u) + static_cast<int64_t>(job.tile) * kSlabSums;
          for (int i = job.chunk * 32 + htid; i < kSlabSums; i += p.cptA * 32) old[i] = 0ull;
          if (job.chunk == 0 && htid == 0) cnt_of(ab_call ^ 1u)[job.tile] = 0u;
          continue;
        }
      }
      const int cpt = isA ? p.cptA : p.cptB;
      if (htid == 0) {
        // the consumers' accumulator adds are ordered before this (barrier, then mbarrier
        // release/acquire); the fence makes them visible GPU-wide before the count
        unsigned int* cnt = (isA ? p.cntA : p.cntB) + job.tile;
        __threadfence();
        const unsigned prev = atomicAdd(cnt, 1u);
        const int last = prev == static_cast<unsigned>(cpt - 1);
        if (last) {
          __threadfence();
          *cnt = 0u;      // every chunk of the slab has counted: reset for the next call
        }
        *s_last = last;
      }
      helper_sync();
      const int last = *s_last;
      helper_sync();    // s_last is rewritten for the next job
      if (!last) continue;
      if (isA) {
        if constexpr (kHasA) {
          // h[t, col] for this slab: lane owns column pairs lane, lane + 32, .. (kTileN / 64)
          constexpr int kPairs = kTileN / 64;
          unsigned long long* base = p.accA + static_cast<int64_t>(job.tile) * (NA * T * kTileN);
#pragma unroll 1
          for (int t = 0; t < T; ++t) {
            int off[NA];
#pragma unroll
            for (int m = 0; m < NA; ++m) off[m] = (m * T + t) * kTileN;
            float2 gu[kPairs][NA];
            take_acc<NA, kPairs>(base, off, htid, gu);
#pragma unroll
            for (int k = 0; k < kPairs; ++k) {
              const int col = job.tile * kTileN + 2 * (htid + 32 * k);
              const float2 g = gu[k][0];
              float h0 = silu_f32(g.x), h1 = silu_f32(g.y);
              if constexpr (NA == 2) {
                h0 *= gu[k][1].x;
                h1 *= gu[k][1].y;
              }
              if (col < p.NA) store_out(p.outA, p.outA_bf16, p.NA, t, col, h0);
              if (col + 1 < p.NA) store_out(p.outA, p.outA_bf16, p.NA, t, col + 1, h1);
            }
          }
        }
      } else {
        if constexpr (kHasB) {
          constexpr int kPairs = kTileN / 64;
          unsigned long long* base = p.accB + static_cast<int64_t>(job.tile) * (T * kTileN);
          const int slotp = TP ? static_cast<int>(cepoch & 1u) : 0;
#pragma unroll 1
          for (int t = 0; t < T; ++t) {
            const int off[1] = {t * kTileN};
            float2 v[kPairs][1];
            take_acc<1, kPairs>(base, off, htid, v);
#pragma unroll
            for (int k = 0; k < kPairs; ++k) {
              const int c = 2 * (htid + 32 * k);
              if constexpr (TP) {
                for (int peer = 0; peer < p.comm.world; ++peer) {
                  float* dst = comm::fused_slot(p.comm, peer, slotp, p.comm.rank) +
                               static_cast<int64_t>(job.tile) * (T * kTileN) + t * kTileN + c;
                  *reinterpret_cast<float2*>(dst) = v[k][0];
                }
              } else {
                const int col = job.tile * kTileN + c;
                float2 r = v[k][0];
                if (p.biasB != nullptr) {   // x @ W + b: the bias joins the finished dot product
                  if (col < p.NB) r.x += __ldg(p.biasB + col);
                  if (col + 1 < p.NB) r.y += __ldg(p.biasB + col + 1);
                }
                if (col < p.NB) p.outB[static_cast<int64_t>(t) * p.NB + col] = r.x;
                if (col + 1 < p.NB) p.outB[static_cast<int64_t>(t) * p.NB + col + 1] = r.y;
              }
            }
          }
          if constexpr (TP) {
            __threadfence_system();
            helper_sync();
            if (htid < p.comm.world)
              st_release_sys(comm::fused_flag(p.comm, htid, slotp, p.comm.rank, job.tile), cepoch);
            if (htid == 0) owned[1 + owned[0]++] = job.tile;
          }
        }
      }
    }
  }
  __syncthreads();
  if constexpr (TP) {
    // every chunk of this CTA is done: now wait for the peers of the slabs it finished
    if (warp < kConsumerWarps) {
      const int n_owned = owned[0];
      for (int i = 0; i < n_owned; ++i) tp_finish_tile<T>(p.comm, cepoch, owned[1 + i], p.outB, p.NB, threadIdx.x);
    }
    __syncthreads();
    comm::epoch_end(p.comm, cepoch);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.ws_done, 1u);
    if (prev == gridDim.x - 1) {
      // last CTA: reset the queue counter and publish the epoch for the next call
      p.next[0] = 0u;
      *reinterpret_cast<volatile unsigned int*>(p.ws_done) = 0u;
      if constexpr (MODE == MODE_AB) *reinterpret_cast<volatile unsigned int*>(p.ab_calls) = ab_call + 1u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(p.ws_epoch) = epoch;
    }
  }
}

}  // namespace ffn
}  // namespace pyre
