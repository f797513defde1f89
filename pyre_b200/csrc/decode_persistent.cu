// Persistent decode step: every layer of one greedy token of a Llama-style decoder in ONE
// launch (batch 1, one GPU). Reference semantics: RootNode._decode_single_layer
// (src/orchestrator/root_node.py:739-1007) per layer, Generator's decode loop
// (src/orchestrator/generator.py:117-131) around it; the launches it replaces are those of
// pyre_decoder_step (decoder.cu): per layer QKV GEMV, fused attention step, O GEMV,
// add + RMSNorm, decode FFN, add + RMSNorm.
//
// Why one launch. At batch 1 a token streams every weight once (7.4 GB at the Mistral-7B
// shape) and each of the ~6 kernels of a layer pays a ramp (launch, first copies) and a tail
// (the last CTAs, the split-K reduction). Here one CTA per SM runs for the whole token and its
// producer warp never waits for activations: weight blocks and KV-cache rows are constant
// during the token, so the producer streams the next work items into a ring of shared-memory
// stages while the consumers wait for the previous stage's results. The dependency chain of a
// layer then costs latency the ring hides instead of idle HBM.
//
// Work queue (one global atomic counter, the same order for every CTA; item blockIdx.x first):
// for every layer L, in order,
//   QKV  chunks of [Wq|Wk|Wv] (8 packed 64-row blocks of one 256-column slab each), chunk-major
//   ATT  (kv head g, position split s): 32-position tiles of the K and V caches
//   O    chunks of Wo
//   FA   chunks of the gate/up pair (32-row blocks), slab-major
//   FB   chunks of down, chunk-major (column c reads h rows [512c, 512c + 512))
// Dependencies (consumer side, epoch-tagged flags in the workspace, acquire/release at GPU
// scope): QKV(L) waits for FB(L-1) complete; ATT(L) for QKV(L); O(L) for ATT(L); FA(L) for
// O(L); an FB chunk for the FA slabs that produce its rows of h. Every item depends only on
// items earlier in the queue, CTAs take items in queue order and consume their own items in
// order, and all CTAs are co-resident (cooperative launch, one CTA per SM), so the earliest
// unfinished item can always proceed. Every wait is bounded besides (PYRE_ETIMEOUT).
//
// Split-K sums are int64 fixed point (value * 2^32) added with integer atomics, so results do
// not depend on which CTA ran which chunk; the CTA that counts a slab's last chunk (helper
// warp) reads the sums back, clears them and runs the slab epilogue:
//   QKV: qkv[col] = sum (+ bias)                     root_node.py:866-897 (:786-799 biases)
//   O  : h1[col] = x[col] + sum                      :940-947
//   FA : h[col]  = silu(gate) * up                   :953-979
//   FB : x'[col] = h1[col] + sum                     :997
// The RMSNorms (input_layernorm of L, post_attention_layernorm of L) are computed by each CTA
// from the full residual vector when it takes its first item of the stage (f64 sum of
// squares, the same thread mapping in every CTA, so every CTA holds the same bits).
// Attention (root_node.py:900-933, :1009-1031): q and the token's k are rotated at position
// pos (f32, rotate-half pairs, no FMA), clipped to +-1000 and rounded to f16 like the cache;
// the new k and v rows are written to the caches at row pos by the split that holds it; each
// split accumulates f32 scores and an online softmax (base 2) over its tiles, the warps' and
// then the splits' partials are combined in a fixed order (deterministic).
#include <cooperative_groups.h>

#include "ffn_stream.cuh"

namespace pyre {
namespace pd {

using namespace gemv;
using ffn::kFixInv;
using ffn::kFixLimit;
using ffn::kFixScale;

constexpr int kMaxLayers = 64;
constexpr int kMaxStages = 12;
constexpr int kBlockBytes = 17408;           // one packed block with f16 scales: 64 x 256 single / 2 x 32 x 256 pair
constexpr int kChunkBlocks = 8;              // blocks per GEMV work item
constexpr int kAttTile = 32;                 // cache positions per attention stage
constexpr int kCW = 8;                       // consumer warps
constexpr int kCtasPerSm = 2;                // persistent CTAs per SM (independent barriers)
constexpr int kCT = kCW * 32;                // consumer threads
constexpr int kRPP = 2 * kCW;                // block rows per consumer pass
constexpr int kAttWarps = 8;                 // consumer warps that run an attention tile
constexpr int kThreadsPD = kCT + 64;         // consumers, producer warp, helper warp
constexpr int kJobsPD = 8;
constexpr int kMaxRepHd = 512;               // (query heads per kv head) x head_dim
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits

enum Kind : int { K_QKV = 0, K_ATT = 1, K_O = 2, K_FA = 3, K_FB = 4, K_END = 5 };
// stage flags per layer
enum Flag : int { F_QKV = 0, F_ATT = 1, F_O = 2, F_FB = 3 };

struct LayerPtrs {
  const uint8_t* qkv_w;     // packed single [H, nqkv], f16 scales
  const float* qkv_bias;    // [nqkv] or null
  const uint8_t* o_w;       // packed single [nq*hd, H]
  const uint8_t* gu_w;      // packed gate/up pair [H, W] (or up alone, single)
  const uint8_t* dn_w;      // packed single [W, H]
  const float* ln1;
  const float* ln2;
  __half* kc;               // [nkv, max_t, hd]
  __half* vc;
  const float2* rope;       // (cos, sin) [max_t, half]
};

struct alignas(16) Params {
  const LayerPtrs* layers;                 // [n_layers] in the workspace (pd_table_kernel)
  int n_layers, H, nq, nkv, hd, rep, W, max_t, half, gated, nqkv;
  int stages;                              // ring stages (runtime, <= kMaxStages)
  int tq, uq, cq;                          // QKV: slabs, 64-row blocks per slab, chunks per slab
  int to, uo, co;                          // O
  int ta, ua, ca;                          // FFN gate/up: slabs, blocks per slab (32 or 64 rows), chunks
  int tb, ub, cb;                          // FFN down
  int ra;                                  // rows per FA block (32 pair, 64 single)
  int smax;                                // attention splits per kv head at most
  int vin_floats;                          // activation vector in shared memory (padded K)
  float scale2;                            // log2(e) / sqrt(hd)
  double eps;
  int pos;                                 // position when pos_dev is null
  const int* pos_dev;
  // workspace
  float* xr[2];                            // residual ping-pong: layer L reads xr[L & 1]
  float* qkv;
  float* attn;
  float* h1;
  float* h;
  float* part;                             // [nkv][smax][2 rep + rep hd]
  unsigned long long* acc_q;
  unsigned long long* acc_o;
  unsigned long long* acc_a;
  unsigned long long* acc_b;
  unsigned* cnt_q;
  unsigned* cnt_o;
  unsigned* cnt_a;
  unsigned* cnt_b;
  unsigned* cnt_att;                       // [nkv]
  unsigned* stage_cnt;                     // [4]
  uint32_t* flags;                         // [n_layers][4]
  uint32_t* ready;                         // [n_layers][ta]
  unsigned* next;
  uint32_t* epoch;
  unsigned* done;
  int* status;
  int* check;                              // [2]: first failed bounds check (site, value)
  int64_t mat_bytes[4];                    // packed QKV, O, gate/up, down matrix bytes (every layer)
  int64_t cache_elems;                     // f16 elements of one layer's K (or V) cache
  int64_t part_floats;
  uint32_t magic;                          // kMagic: the parameter block arrived whole
};
constexpr uint32_t kMagic = 0x50595245u;
static_assert(sizeof(Params) <= 1024, "the parameter block stays small");

// Layer pointer tables are written into the workspace by a small kernel before every step
// (at most kTableChunk layers per launch keep its parameter block small).
constexpr int kTableChunk = 32;
struct TableChunk {
  LayerPtrs L[kTableChunk];
  int first, n;
};

struct Item {
  int kind, layer, a, b;    // GEMV: a = slab, b = chunk; ATT: a = kv head, b = split
};

// Attention split plan for t cache positions (the token included): S splits of ppi positions
// (a multiple of the tile), about one item per CTA over all kv heads.
__device__ __forceinline__ void att_plan(int t, int nkv, int smax, int& S, int& ppi) {
  const int tiles = (t + kAttTile - 1) / kAttTile;
  S = min(tiles, smax);
  const int tps = (tiles + S - 1) / S;     // tiles per split
  ppi = tps * kAttTile;
  S = (t + ppi - 1) / ppi;
}

__device__ __forceinline__ bool item_of(const Params& p, int S, int pos, Item& it) {
  const int nQ = p.tq * p.cq, nA = p.nkv * S, nO = p.to * p.co, nFA = p.ta * p.ca, nFB = p.tb * p.cb;
  const int ipl = nQ + nA + nO + nFA + nFB;
  if (pos < 0 || pos >= ipl * p.n_layers) return false;
  it.layer = pos / ipl;
  int r = pos - it.layer * ipl;
  if (r < nQ) {
    it.kind = K_QKV;
    it.b = r / p.tq;
    it.a = r - it.b * p.tq;
    return true;
  }
  r -= nQ;
  if (r < nA) {
    it.kind = K_ATT;
    it.b = r / p.nkv;
    it.a = r - it.b * p.nkv;
    return true;
  }
  r -= nA;
  if (r < nO) {
    it.kind = K_O;
    it.b = r / p.to;
    it.a = r - it.b * p.to;
    return true;
  }
  r -= nO;
  if (r < nFA) {
    it.kind = K_FA;
    it.a = r / p.ca;
    it.b = r - it.a * p.ca;
    return true;
  }
  r -= nFA;
  it.kind = K_FB;
  it.b = r / p.tb;
  it.a = r - it.b * p.tb;
  return true;
}

// Per-stage descriptor written by the producer next to each ring stage.
struct Meta {
  int kind, layer, a, b;
  int blk;          // GEMV: block index within the slab; ATT: first position of the stage
  int n;            // ATT: positions in the stage
  int first, last;  // first / last stage of the item
};

struct Job {
  int kind, layer, tile, end;
};

__device__ __forceinline__ uint32_t ld_acq(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool failed(const int* status) {
  return *reinterpret_cast<const volatile int*>(status) == PYRE_ETIMEOUT;
}

// Bounded wait for *f == want (one thread). After any timeout in the launch the waits return at
// once, so a failed launch still ends in bounded time.
__device__ bool wait_eq(const uint32_t* f, uint32_t want, int* status) {
  if (ld_acq(f) == want) return true;
  if (failed(status)) return false;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (ld_acq(f) == want) return true;
    if (globaltimer_ns() - t0 > kWaitNs) {
      atomicExch(status, PYRE_ETIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
}

// Bounds check of an index the queue arithmetic guarantees: a violation is recorded (the first
// one's site and value) with PYRE_EINVAL in the status word, and the caller skips the access.
__device__ __forceinline__ bool in_range(const Params& p, int64_t v, int64_t hi, int site) {
  if (v >= 0 && v < hi) return true;
  if (atomicCAS(p.check, 0, site) == 0) p.check[1] = static_cast<int>(v);
  atomicCAS(p.status, PYRE_OK, PYRE_EINVAL);
  return false;
}

__device__ __forceinline__ float clip1000f(float r) { return fminf(fmaxf(r, -1000.f), 1000.f); }

// Element i of a head rotated at one position (rotate-half pairs (j, j + half), each product
// and sum rounded separately like the reference's numpy arithmetic, dims >= 2 half pass
// through), clipped; src is written earlier in this launch, so it is read through L2.
__device__ __forceinline__ float rope_clip_cg(const float* src, int i, int half, const float2* cs) {
  float r;
  if (i < 2 * half) {
    const int jj = i < half ? i : i - half;
    const float x1 = __ldcg(src + jj), x2 = __ldcg(src + jj + half);
    const float2 c = __ldg(cs + jj);
    r = i < half ? __fsub_rn(__fmul_rn(x1, c.x), __fmul_rn(x2, c.y))
                 : __fadd_rn(__fmul_rn(x1, c.y), __fmul_rn(x2, c.x));
  } else {
    r = __ldcg(src + i);
  }
  return clip1000f(r);
}

__device__ __forceinline__ float pd_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void cons_sync() { named_bar(1, kCT); }

// One packed block (NMAT = 1: 64 rows of one matrix; NMAT = 2: 32 rows of the gate/up pair)
// accumulated into acc, for one token whose activations for the block's rows are xs[0..R).
// Consumer mapping, int8 -> f32 conversion and packed f32x2 FMA as consume_unit (gemv_common.cuh).
template <int NMAT>
__device__ __forceinline__ void consume_blk(const uint8_t* st, const float* xs, float2 (&acc)[NMAT][1][8], int warp,
                                            int rs, int cc) {
  constexpr int R = NMAT == 2 ? kUnitRowsPair : kUnitRowsSingle;
  constexpr int kQ = R * kTileN;
  const __half* ss = reinterpret_cast<const __half*>(st + NMAT * kQ);
#pragma unroll
  for (int pass = 0; pass < R / kRPP; ++pass) {
    const int r = pass * kRPP + warp * 2 + rs;
    const float xv = xs[r];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const float sc = __half2float(ss[m * R * 8 + r * 8 + (cc >> 1)]);
      const int4 w = *reinterpret_cast<const int4*>(st + m * kQ + r * kTileN + cc * 16);
      const uint32_t words[4] = {static_cast<uint32_t>(w.x), static_cast<uint32_t>(w.y), static_cast<uint32_t>(w.z),
                                 static_cast<uint32_t>(w.w)};
      const float a = xv * sc;
      const float2 a2 = make_float2(a, a);
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
        acc[m][0][wi * 2] = __ffma2_rn(a2, f01, acc[m][0][wi * 2]);
        acc[m][0][wi * 2 + 1] = __ffma2_rn(a2, f23, acc[m][0][wi * 2 + 1]);
      }
    }
  }
}

// Sums acc over the two row lanes and all consumer warps (in warp order) and adds the chunk's
// partial [NMAT][256] into the slab accumulator as fixed point; a partial that is not finite or
// not below 2^30 in magnitude is added as 0 and flags PYRE_ERANGE. red: kCW * NMAT * 256 floats.
template <int NMAT>
__device__ __forceinline__ void pd_reduce(float2 (&acc)[NMAT][1][8], float* red, unsigned long long* accum,
                                          int* status, int warp, int rs, int cc, int tid) {
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float2 v = acc[m][0][i];
      v.x += __shfl_xor_sync(0xffffffffu, v.x, 16);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, 16);
      acc[m][0][i] = v;
    }
  if (rs == 0) {
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      float4* dst = reinterpret_cast<float4*>(red + (warp * NMAT + m) * kTileN + cc * 16);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        dst[i] = make_float4(acc[m][0][2 * i].x, acc[m][0][2 * i].y, acc[m][0][2 * i + 1].x, acc[m][0][2 * i + 1].y);
    }
  }
  cons_sync();
  constexpr int kItems = NMAT * kTileN;
  for (int i = tid; i < kItems; i += kCT) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kCW; ++w) v += red[w * kItems + i];
    if (!(fabsf(v) < kFixLimit)) {
      atomicCAS(status, PYRE_OK, PYRE_ERANGE);
      v = 0.f;
    }
    atomicAdd(accum + i, static_cast<unsigned long long>(__float2ll_rn(v * kFixScale)));
  }
  cons_sync();   // red is rewritten at the next chunk's end
}

// vin[0..H) = rms_norm(x, w) over the consumer threads: f64 sum of squares in a fixed order
// (the same bits in every CTA), each element rounded once to f32 like rms_norm_kernel. H is a
// multiple of 4; up to 2 float4 loads per thread are issued before any is used.
__device__ void norm_to_vin(const float* x, const float* w, int H, double eps, float* vin, double* dred, int tid,
                            int lane, int warp) {
  const int n4 = H >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4* v4 = reinterpret_cast<float4*>(vin);
  double sq = 0.0;
  for (int b = 0; b < n4; b += 2 * kCT) {
    float4 v[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = b + k * kCT + tid;
      if (i < n4) v[k] = __ldcg(x4 + i);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = b + k * kCT + tid;
      if (i < n4) {
        v4[i] = v[k];
        sq += static_cast<double>(v[k].x) * v[k].x + static_cast<double>(v[k].y) * v[k].y +
              static_cast<double>(v[k].z) * v[k].z + static_cast<double>(v[k].w) * v[k].w;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if (lane == 0) dred[warp] = sq;
  cons_sync();
  double tot = 0.0;
#pragma unroll
  for (int i = 0; i < kCW; ++i) tot += dred[i];
  const double rstd = 1.0 / sqrt(tot / H + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int i = tid; i < n4; i += kCT) {
    const float4 v = v4[i], g = __ldg(w4 + i);
    v4[i] = make_float4(static_cast<float>(static_cast<double>(v.x) * rstd * static_cast<double>(g.x)),
                        static_cast<float>(static_cast<double>(v.y) * rstd * static_cast<double>(g.y)),
                        static_cast<float>(static_cast<double>(v.z) * rstd * static_cast<double>(g.z)),
                        static_cast<float>(static_cast<double>(v.w) * rstd * static_cast<double>(g.w)));
  }
  cons_sync();
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Shared-memory carve-up (host and device agree through these offsets).
struct Smem {
  int stages_off, red_off, vin_off, hsl_off, kv_off, dred_off, bar_off, meta_off, jobs_off, misc_off, total;
};
__host__ __device__ inline Smem smem_layout(int stages, int vin_floats) {
  Smem s{};
  int o = 0;
  s.stages_off = o;
  o += stages * kBlockBytes;
  s.red_off = o;
  o += kCW * kMaxRepHd * 4;
  s.vin_off = o;
  o += vin_floats * 4;
  s.hsl_off = o;
  o += kChunkBlocks * kUnitRowsSingle * 4;
  s.kv_off = o;                                   // knew, vnew: f16 [128] each; qs: f16 [512]
  o += 2 * 128 * 2 + kMaxRepHd * 2;
  s.dred_off = o;
  o += kCW * 8;
  s.bar_off = o;
  o += (2 * kMaxStages + 2 * kJobsPD) * 8;
  s.meta_off = o;
  o += kMaxStages * static_cast<int>(sizeof(Meta));
  s.jobs_off = o;
  o += kJobsPD * static_cast<int>(sizeof(Job));
  s.misc_off = o;
  o += 16;
  s.total = o;
  return s;
}

template <int HD>
__global__ void __maxnreg__(96) decode_persistent_kernel(const __grid_constant__ Params p) {
  constexpr int DPL = HD / 32;              // head dims per lane
  extern __shared__ __align__(128) uint8_t smem[];
  const Smem L = smem_layout(p.stages, p.vin_floats);
  uint8_t* stages = smem + L.stages_off;
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  float* vin = reinterpret_cast<float*>(smem + L.vin_off);
  float* hsl = reinterpret_cast<float*>(smem + L.hsl_off);
  __half* knew = reinterpret_cast<__half*>(smem + L.kv_off);
  __half* vnew = knew + 128;
  __half* qs = vnew + 128;
  double* dred = reinterpret_cast<double*>(smem + L.dred_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + kMaxStages;
  uint64_t* job_full = empty + kMaxStages;
  uint64_t* job_empty = job_full + kJobsPD;
  Meta* meta = reinterpret_cast<Meta*>(smem + L.meta_off);
  Job* jobs = reinterpret_cast<Job*>(smem + L.jobs_off);
  int* misc = reinterpret_cast<int*>(smem + L.misc_off);

  if (p.magic != kMagic || p.stages < 1 || p.stages > kMaxStages) return;   // nothing is touched
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCW);
    }
    for (int i = 0; i < kJobsPD; ++i) {
      mbar_init(&job_full[i], kCW);
      mbar_init(&job_empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(p.epoch) + 1u;
  // (an if statement, not a conditional expression: the position word is loaded only when the
  // pointer is set)
  int pos = p.pos;
  if (p.pos_dev != nullptr) pos = __ldcg(p.pos_dev);
  if (pos < 0 || pos >= p.max_t) {
    // a graphed step replayed past the cache: nothing runs, the host sees PYRE_EINVAL
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicCAS(p.status, PYRE_OK, PYRE_EINVAL);
    return;
  }
  const int t = pos + 1;
  int S, ppi;
  att_plan(t, p.nkv, p.smax, S, ppi);

  if (warp == kCW) {
    // ------------------------------- producer -------------------------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t issued = 0, par = 0;
      auto acquire = [&]() -> bool {
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) return false;
        issued &= ~(1u << s);
        return true;
      };
      auto advance = [&]() {
        issued |= 1u << s;
        par = (par & ~(1u << s)) | (ph << s);
        if (++s == p.stages) {
          s = 0;
          ph ^= 1u;
        }
      };
      int ipos = static_cast<int>(blockIdx.x);
      while (ok) {
        if (failed(p.status)) {
          ok = false;
          break;
        }
        Item it;
        if (!item_of(p, S, ipos, it)) break;
        const LayerPtrs Lp = p.layers[it.layer];
        if (it.kind == K_ATT) {
          const int p0 = it.b * ppi, p1 = min(p0 + ppi, t);
          for (int a = p0; a < p1; a += kAttTile) {
            const int b = min(a + kAttTile, p1);
            const int nb = min(b, t - 1) - a;       // rows already in the cache (row t - 1 is the token's)
            if (!acquire()) {
              ok = false;
              break;
            }
            meta[s] = Meta{K_ATT, it.layer, it.a, it.b, a, b - a, a == p0, b == p1};
            uint8_t* st = stages + s * kBlockBytes;
            const int64_t off = (static_cast<int64_t>(it.a) * p.max_t + a) * HD;
            if (nb > 0 && in_range(p, off + static_cast<int64_t>(nb) * HD - 1, p.cache_elems, 5) &&
                in_range(p, nb, kAttTile + 1, 6)) {
              const uint32_t bytes = static_cast<uint32_t>(nb) * HD * 2;
              mbar_arrive_expect_tx(&full[s], 2 * bytes);
              bulk_load(st, Lp.kc + off, bytes, &full[s]);
              bulk_load(st + kAttTile * HD * 2, Lp.vc + off, bytes, &full[s]);
            } else {
              mbar_arrive(&full[s]);
            }
            advance();
          }
        } else {
          const uint8_t* w;
          int upt, mk;
          if (it.kind == K_QKV) {
            w = Lp.qkv_w;
            upt = p.uq;
            mk = 0;
          } else if (it.kind == K_O) {
            w = Lp.o_w;
            upt = p.uo;
            mk = 1;
          } else if (it.kind == K_FA) {
            w = Lp.gu_w;
            upt = p.ua;
            mk = 2;
          } else {
            w = Lp.dn_w;
            upt = p.ub;
            mk = 3;
          }
          const int u0 = it.b * kChunkBlocks, u1 = min(u0 + kChunkBlocks, upt);
          for (int u = u0; u < u1; ++u) {
            if (!acquire()) {
              ok = false;
              break;
            }
            meta[s] = Meta{it.kind, it.layer, it.a, it.b, u, 0, u == u0, u + 1 == u1};
            const int64_t boff = (static_cast<int64_t>(it.a) * upt + u) * kBlockBytes;
            if (in_range(p, boff + kBlockBytes - 1, p.mat_bytes[mk], 1 + mk)) {
              mbar_arrive_expect_tx(&full[s], kBlockBytes);
              bulk_load(stages + s * kBlockBytes, w + boff, kBlockBytes, &full[s]);
            } else {
              mbar_arrive(&full[s]);
            }
            advance();
          }
        }
        if (!ok) break;
        ipos = static_cast<int>(gridDim.x + atomicAdd(p.next, 1u));
      }
      // end marker for the consumers
      if (acquire()) {
        meta[s] = Meta{K_END, 0, 0, 0, 0, 0, 0, 0};
        mbar_arrive(&full[s]);
      }
      if (!ok) {
        // no copy into this CTA's shared memory may be in flight when it exits
        for (int i = 0; i < p.stages; ++i)
          if ((issued >> i) & 1u) mbar_wait(&full[i], (par >> i) & 1u, nullptr, 500000000ull);
      }
    }
  } else if (warp < kCW) {
    // ------------------------------- consumers -------------------------------
    const int tid = threadIdx.x;
    const int rs = lane >> 4, cc = lane & 15;
    int s = 0;
    uint32_t ph = 0;
    int jb = 0;
    uint32_t jph = 0;
    int vin_tag = -1;        // layer * 8 + kind of the vector held in vin
    int att_layer = -1;      // layer whose QKV flag this CTA has seen
    auto post_job = [&](const Job& job) {
      if (lane == 0) mbar_wait(&job_empty[jb], jph ^ 1u, p.status);
      __syncwarp();
      if (tid == 0) jobs[jb] = job;
      __syncwarp();
      if (lane == 0) mbar_arrive(&job_full[jb]);
      if (++jb == kJobsPD) {
        jb = 0;
        jph ^= 1u;
      }
    };
    // one thread waits for a flag, the others meet it at the barrier
    auto dep_wait = [&](const uint32_t* f) {
      cons_sync();     // nobody still reads what the caller is about to overwrite
      if (tid == 0) wait_eq(f, epoch, p.status);
      cons_sync();
    };
    float2 acc[2][1][8];
    zero_acc<2, 1>(acc);
    // attention state of the current item
    float am = -INFINITY, al = 0.f, ao[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) ao[i] = 0.f;
    while (true) {
      if (!mbar_wait(&full[s], ph, p.status, 4000000000ull)) break;
      const Meta m = meta[s];
      if (m.kind == K_END) break;
      if (!in_range(p, m.layer, p.n_layers, 10) || !in_range(p, m.kind, K_END, 11)) break;
      const uint8_t* st = stages + s * kBlockBytes;
      const LayerPtrs* Lq = p.layers + m.layer;
      if (m.kind == K_ATT) {
        // G warps per query head of kv head g (warps 0 .. rep*G-1, G = 2 for rep <= 4): warp
        // (head r, group gi) takes positions gi*P .. gi*P + P - 1 of each tile (P = 32 / G); for
        // the scores its lanes are (dim part dp, position jj), for the weighted values the head dims
        const int g = m.a;
        const int G = p.rep * 2 <= kAttWarps ? 2 : 1;
        const int P = kAttTile / G;
        if (m.first) {
          if (att_layer != m.layer) {
            dep_wait(p.flags + m.layer * 4 + F_QKV);
            att_layer = m.layer;
          } else {
            cons_sync();   // qs / knew / vnew of the previous item are no longer read
          }
          // q of the kv head's query heads, rotated at position pos, clipped, rounded to f16 like
          // the cache; the split that holds the token's own position rotates k, clips v and
          // appends both to the caches at row pos
          const float2* cs = Lq->rope + static_cast<int64_t>(pos) * p.half;
          for (int e = tid; e < p.rep * HD; e += kCT) {
            const int r = e / HD, d = e - r * HD;
            qs[e] = __float2half_rn(rope_clip_cg(p.qkv + static_cast<int64_t>(g * p.rep + r) * HD, d, p.half, cs));
          }
          if (m.b == S - 1) {
            for (int d = tid; d < HD; d += kCT) {
              const float* kf = p.qkv + static_cast<int64_t>(p.nq) * HD + static_cast<int64_t>(g) * HD;
              const float* vf = p.qkv + static_cast<int64_t>(p.nq + p.nkv) * HD + static_cast<int64_t>(g) * HD;
              const __half kn = __float2half_rn(rope_clip_cg(kf, d, p.half, cs));
              const __half vn = __float2half_rn(clip1000f(__ldcg(vf + d)));
              knew[d] = kn;
              vnew[d] = vn;
              const int64_t row = (static_cast<int64_t>(g) * p.max_t + pos) * HD + d;
              if (in_range(p, row, p.cache_elems, 7)) {
                Lq->kc[row] = kn;
                Lq->vc[row] = vn;
              }
            }
          }
          cons_sync();
          am = -INFINITY;
          al = 0.f;
#pragma unroll
          for (int i = 0; i < DPL; ++i) ao[i] = 0.f;
        }
        if (warp < p.rep * G) {
          const int r = warp / G, gi = warp - r * G;
          const int dp = lane / P, jj = lane - dp * P;
          const int j = gi * P + jj;                     // position within the tile
          const int W2 = HD / (2 * G);                   // half2 dims per part
          // partial score over dim part dp, dims taken in a lane-rotated order: the K rows
          // (HD*2 bytes apart) and q are read from shared memory without bank conflicts
          const __half2* Ks2 = reinterpret_cast<const __half2*>(st);
          const __half* Vs = reinterpret_cast<const __half*>(st + kAttTile * HD * 2);
          const __half2* q2 = reinterpret_cast<const __half2*>(qs) + r * (HD / 2) + dp * W2;
          float sc = 0.f;
          if (j < m.n) {
            const __half2* k2 =
                ((m.blk + j == t - 1) ? reinterpret_cast<const __half2*>(knew) : Ks2 + j * (HD / 2)) + dp * W2;
            float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
            for (int i = 0; i < W2; ++i) {
              const int d2 = (i + lane) & (W2 - 1);
              const float2 kk = __half22float2(k2[d2]);
              const float2 qq = __half22float2(q2[d2]);
              a0 = fmaf(qq.x, kk.x, a0);
              a1 = fmaf(qq.y, kk.y, a1);
            }
            sc = a0 + a1;
          }
          if (G == 2) sc += __shfl_xor_sync(0xffffffffu, sc, 16);
          if (j >= m.n) sc = -INFINITY;
          // online softmax over this warp's positions (base 2, running max in raw score units)
          const float mn = fmaxf(am, warp_max(sc));
          if (mn > am) {
            const float alpha = am == -INFINITY ? 0.f : pd_exp2((am - mn) * p.scale2);
            al *= alpha;
#pragma unroll
            for (int i = 0; i < DPL; ++i) ao[i] *= alpha;
            am = mn;
          }
          const float pj = sc == -INFINITY ? 0.f : pd_exp2((sc - mn) * p.scale2);
          al += warp_sum(dp == 0 ? pj : 0.f);
          // weighted values of this warp's positions: lane owns dims lane*DPL .. +DPL
          const int n = min(P, m.n - gi * P);
          for (int q = 0; q < n; ++q) {
            const float pb = __shfl_sync(0xffffffffu, pj, q);
            const int jq = gi * P + q;
            const __half* vr = (m.blk + jq == t - 1) ? vnew : Vs + jq * HD;
            float vf[DPL];
            if constexpr (DPL == 4) {
              const uint2 raw = *reinterpret_cast<const uint2*>(vr + lane * 4);
              const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
              const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
              vf[0] = a.x;
              vf[1] = a.y;
              vf[2] = b.x;
              vf[3] = b.y;
            } else {
              const float2 a = __half22float2(*reinterpret_cast<const __half2*>(vr + lane * 2));
              vf[0] = a.x;
              vf[1] = a.y;
            }
#pragma unroll
            for (int i = 0; i < DPL; ++i) ao[i] = fmaf(pb, vf[i], ao[i]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == p.stages) {
          s = 0;
          ph ^= 1u;
        }
        if (m.last) {
          // the G warps of each head combine (group order) into this split's partial
          const int stride = 2 * p.rep + p.rep * HD;
          if (warp < p.rep * G) {
            float* wp = red + warp * (HD + 2);
            if (lane == 0) {
              wp[HD] = am;
              wp[HD + 1] = al;
            }
#pragma unroll
            for (int i = 0; i < DPL; ++i) wp[lane * DPL + i] = ao[i];
          }
          cons_sync();
          const int64_t dst_off = (static_cast<int64_t>(g) * p.smax + m.b) * stride;
          if (in_range(p, dst_off + stride - 1, p.part_floats, 8)) {
            float* dst = p.part + dst_off;
            for (int e = tid; e < p.rep * HD; e += kCT) {
              const int r = e / HD, d = e - r * HD;
              float M = -INFINITY;
              for (int q = 0; q < G; ++q) M = fmaxf(M, red[(r * G + q) * (HD + 2) + HD]);
              float Ls = 0.f, O = 0.f;
              for (int q = 0; q < G; ++q) {
                const float* wp = red + (r * G + q) * (HD + 2);
                const float wt = wp[HD] == -INFINITY ? 0.f : pd_exp2((wp[HD] - M) * p.scale2);
                Ls = fmaf(wp[HD + 1], wt, Ls);
                O = fmaf(wp[d], wt, O);
              }
              __stcg(dst + 2 * p.rep + e, O);
              if (d == 0) {
                __stcg(dst + r, M);
                __stcg(dst + p.rep + r, Ls);
              }
            }
          }
          __threadfence();
          cons_sync();
          if (tid == 0) {
            const unsigned prev = atomicAdd(p.cnt_att + g, 1u);
            const int last = prev == static_cast<unsigned>(S - 1);
            if (last) {
              p.cnt_att[g] = 0u;
              __threadfence();
            }
            misc[0] = last;
          }
          cons_sync();
          if (misc[0]) {
            // the last split of kv head g combines the S partials in split order: maxima and
            // weights through shared memory (red is free here), then each output sums its S values
            const float* src = p.part + static_cast<int64_t>(g) * p.smax * stride;
            float* ms = red;                       // [rep][S] maxima, then weights
            float* ls = red + p.rep * S;           // [rep][S] sums
            float* Lr = red + 2 * p.rep * S;       // [rep] totals
            for (int e = tid; e < p.rep * S; e += kCT) {
              const int r = e / S, q = e - r * S;
              ms[e] = __ldcg(src + static_cast<int64_t>(q) * stride + r);
              ls[e] = __ldcg(src + static_cast<int64_t>(q) * stride + p.rep + r);
            }
            cons_sync();
            if (tid < p.rep) {
              float M = -INFINITY;
              for (int q = 0; q < S; ++q) M = fmaxf(M, ms[tid * S + q]);
              float Ls = 0.f;
              for (int q = 0; q < S; ++q) {
                const float mq = ms[tid * S + q];
                const float wt = mq == -INFINITY ? 0.f : pd_exp2((mq - M) * p.scale2);
                ms[tid * S + q] = wt;
                Ls = fmaf(ls[tid * S + q], wt, Ls);
              }
              Lr[tid] = Ls;
            }
            cons_sync();
            for (int e = tid; e < p.rep * HD; e += kCT) {
              const int r = e / HD;
              const float* wr = ms + r * S;
              const float* pe = src + 2 * p.rep + e;
              float O = 0.f;
              int q = 0;
              for (; q + 4 <= S; q += 4) {
                const float o0 = __ldcg(pe + static_cast<int64_t>(q) * stride);
                const float o1 = __ldcg(pe + static_cast<int64_t>(q + 1) * stride);
                const float o2 = __ldcg(pe + static_cast<int64_t>(q + 2) * stride);
                const float o3 = __ldcg(pe + static_cast<int64_t>(q + 3) * stride);
                O = fmaf(o0, wr[q], O);
                O = fmaf(o1, wr[q + 1], O);
                O = fmaf(o2, wr[q + 2], O);
                O = fmaf(o3, wr[q + 3], O);
              }
              for (; q < S; ++q) O = fmaf(__ldcg(pe + static_cast<int64_t>(q) * stride), wr[q], O);
              const int64_t ai = static_cast<int64_t>(g * p.rep) * HD + e;
              if (in_range(p, ai, static_cast<int64_t>(p.nq) * HD, 9)) __stcg(p.attn + ai, __fdiv_rn(O, Lr[r]));
            }
            __threadfence();
            cons_sync();
            if (tid == 0) {
              const unsigned prev = atomicAdd(p.stage_cnt + F_ATT, 1u);
              if (prev == static_cast<unsigned>(p.nkv - 1)) {
                p.stage_cnt[F_ATT] = 0u;
                __threadfence();
                st_release_gpu(p.flags + m.layer * 4 + F_ATT, epoch);
              }
            }
          }
        }
        continue;
      }
      // ---- GEMV stages ----
      if (m.first) {
        if (m.kind == K_QKV) {
          const int want = m.layer * 8 + K_QKV;
          if (vin_tag != want) {
            if (m.layer > 0) dep_wait(p.flags + (m.layer - 1) * 4 + F_FB);
            else cons_sync();
            norm_to_vin(p.xr[m.layer & 1], Lq->ln1, p.H, p.eps, vin, dred, tid, lane, warp);
            vin_tag = want;
          }
        } else if (m.kind == K_O) {
          const int want = m.layer * 8 + K_O;
          if (vin_tag != want) {
            dep_wait(p.flags + m.layer * 4 + F_ATT);
            {
              const float4* a4 = reinterpret_cast<const float4*>(p.attn);
              float4* v4 = reinterpret_cast<float4*>(vin);
              const int n4 = p.nq * HD / 4;
              for (int b = 0; b < n4; b += 2 * kCT) {
                float4 v[2];
#pragma unroll
                for (int k = 0; k < 2; ++k)
                  if (b + k * kCT + tid < n4) v[k] = __ldcg(a4 + b + k * kCT + tid);
#pragma unroll
                for (int k = 0; k < 2; ++k)
                  if (b + k * kCT + tid < n4) v4[b + k * kCT + tid] = v[k];
              }
            }
            cons_sync();
            vin_tag = want;
          }
        } else if (m.kind == K_FA) {
          const int want = m.layer * 8 + K_FA;
          if (vin_tag != want) {
            dep_wait(p.flags + m.layer * 4 + F_O);
            norm_to_vin(p.h1, Lq->ln2, p.H, p.eps, vin, dred, tid, lane, warp);
            vin_tag = want;
          }
        } else {
          // rows [512 c, 512 c + 512) of h come from gate/up slabs 2c, 2c + 1
          const int r0 = m.b * kChunkBlocks * kUnitRowsSingle;
          const int r1 = min(r0 + kChunkBlocks * kUnitRowsSingle, p.W);
          cons_sync();
          if (tid == 0) {
            for (int j = r0 / kTileN; j <= (r1 - 1) / kTileN; ++j)
              wait_eq(p.ready + m.layer * p.ta + j, epoch, p.status);
          }
          cons_sync();
          for (int i = tid; i < r1 - r0; i += kCT) hsl[i] = __ldcg(p.h + r0 + i);
          cons_sync();
        }
      }
      const bool pair = m.kind == K_FA && p.gated;
      if (pair) {
        consume_blk<2>(st, vin + m.blk * kUnitRowsPair, acc, warp, rs, cc);
      } else {
        const float* xs = m.kind == K_FB ? hsl + (m.blk - m.b * kChunkBlocks) * kUnitRowsSingle
                                         : vin + m.blk * kUnitRowsSingle;
        float2(&acc1)[1][1][8] = reinterpret_cast<float2(&)[1][1][8]>(acc);
        consume_blk<1>(st, xs, acc1, warp, rs, cc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == p.stages) {
        s = 0;
        ph ^= 1u;
      }
      if (!m.last) continue;
      unsigned long long* accum = m.kind == K_QKV ? p.acc_q + static_cast<int64_t>(m.a) * kTileN
                                  : m.kind == K_O  ? p.acc_o + static_cast<int64_t>(m.a) * kTileN
                                  : m.kind == K_FA ? p.acc_a + static_cast<int64_t>(m.a) * (p.gated ? 2 : 1) * kTileN
                                                   : p.acc_b + static_cast<int64_t>(m.a) * kTileN;
      if (pair) {
        pd_reduce<2>(acc, red, accum, p.status, warp, rs, cc, tid);
      } else {
        float2(&acc1)[1][1][8] = reinterpret_cast<float2(&)[1][1][8]>(acc);
        pd_reduce<1>(acc1, red, accum, p.status, warp, rs, cc, tid);
      }
      zero_acc<2, 1>(acc);
      post_job(Job{m.kind, m.layer, m.a, 0});
    }
    post_job(Job{0, 0, 0, 1});
  } else {
    // ------------------------------- helper warp -------------------------------
    // Per finished chunk: count it for its slab; the CTA that counts a slab's last chunk reads
    // the slab sums back (clearing them) and runs the slab epilogue, then counts the slab for
    // its stage (or releases the slab's ready flag, FA).
    int jb = 0;
    uint32_t jph = 0;
    while (true) {
      if (!mbar_wait(&job_full[jb], jph, p.status, 8000000000ull)) break;
      const Job job = jobs[jb];
      __syncwarp();
      if (lane == 0) mbar_arrive(&job_empty[jb]);
      if (++jb == kJobsPD) {
        jb = 0;
        jph ^= 1u;
      }
      if (job.end) break;
      unsigned* cnt;
      int cpt, ntiles, flag = -1;
      unsigned long long* accb;
      if (job.kind == K_QKV) {
        cnt = p.cnt_q;
        cpt = p.cq;
        ntiles = p.tq;
        flag = F_QKV;
        accb = p.acc_q;
      } else if (job.kind == K_O) {
        cnt = p.cnt_o;
        cpt = p.co;
        ntiles = p.to;
        flag = F_O;
        accb = p.acc_o;
      } else if (job.kind == K_FA) {
        cnt = p.cnt_a;
        cpt = p.ca;
        ntiles = p.ta;
        accb = p.acc_a;
      } else {
        cnt = p.cnt_b;
        cpt = p.cb;
        ntiles = p.tb;
        flag = F_FB;
        accb = p.acc_b;
      }
      if (!in_range(p, job.tile, ntiles, 12) || !in_range(p, job.layer, p.n_layers, 13)) continue;
      int last = 0;
      if (lane == 0) {
        // the consumers' accumulator adds are ordered before this (barrier, then mbarrier
        // release/acquire); the fence makes them visible GPU-wide before the count
        __threadfence();
        const unsigned prev = atomicAdd(cnt + job.tile, 1u);
        last = prev == static_cast<unsigned>(cpt - 1);
        if (last) {
          __threadfence();
          cnt[job.tile] = 0u;
        }
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      constexpr int kPairs = kTileN / 64;
      const int col0 = job.tile * kTileN;
      if (job.kind == K_FA) {
        if (p.gated) {
          const int off[2] = {0, kTileN};
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {   // two rounds of column pairs (register budget)
            float2 gu[kPairs / 2][2];
            ffn::take_acc<2, kPairs / 2>(accb + static_cast<int64_t>(job.tile) * 2 * kTileN, off, lane + 64 * half, gu);
#pragma unroll
            for (int k = 0; k < kPairs / 2; ++k) {
              const int col = col0 + 2 * (lane + 64 * half + 32 * k);
              const float h0 = silu_f32(gu[k][0].x) * gu[k][1].x, h1v = silu_f32(gu[k][0].y) * gu[k][1].y;
              if (col < p.W) __stcg(p.h + col, h0);
              if (col + 1 < p.W) __stcg(p.h + col + 1, h1v);
            }
          }
        } else {
          const int off[1] = {0};
          float2 u[kPairs][1];
          ffn::take_acc<1, kPairs>(accb + static_cast<int64_t>(job.tile) * kTileN, off, lane, u);
#pragma unroll
          for (int k = 0; k < kPairs; ++k) {
            const int col = col0 + 2 * (lane + 32 * k);
            if (col < p.W) __stcg(p.h + col, silu_f32(u[k][0].x));
            if (col + 1 < p.W) __stcg(p.h + col + 1, silu_f32(u[k][0].y));
          }
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu(p.ready + job.layer * p.ta + job.tile, epoch);
        continue;
      }
      {
        const int off[1] = {0};
        float2 v[kPairs][1];
        ffn::take_acc<1, kPairs>(accb + static_cast<int64_t>(job.tile) * kTileN, off, lane, v);
        const float* qkv_bias = p.layers[job.layer].qkv_bias;
#pragma unroll
        for (int k = 0; k < kPairs; ++k) {
          const int col = col0 + 2 * (lane + 32 * k);
          const float vv[2] = {v[k][0].x, v[k][0].y};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = col + e;
            if (job.kind == K_QKV) {
              if (c < p.nqkv) {
                float r = vv[e];
                if (qkv_bias != nullptr) r += __ldg(qkv_bias + c);
                __stcg(p.qkv + c, r);
              }
            } else if (job.kind == K_O) {
              if (c < p.H) __stcg(p.h1 + c, __fadd_rn(__ldcg(p.xr[job.layer & 1] + c), vv[e]));
            } else {
              if (c < p.H) __stcg(p.xr[(job.layer + 1) & 1] + c, __fadd_rn(__ldcg(p.h1 + c), vv[e]));
            }
          }
        }
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) {
        const unsigned prev = atomicAdd(p.stage_cnt + flag, 1u);
        if (prev == static_cast<unsigned>(ntiles - 1)) {
          p.stage_cnt[flag] = 0u;
          __threadfence();
          st_release_gpu(p.flags + job.layer * 4 + flag, epoch);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1) {
      // last CTA: reset the queue counter and publish the epoch for the next call
      *p.next = 0u;
      *reinterpret_cast<volatile unsigned*>(p.done) = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(p.epoch) = epoch;
    }
  }
}

__global__ void pd_advance_kernel(int* pos, const int* token, int* history, int max_t) {
  pdl_wait();
  pdl_trigger();
  const int q = *pos;
  if (q >= 0 && q < max_t) {
    history[q + 1] = token[0];
    *pos = q + 1;
  }
}

__global__ void pd_table_kernel(const __grid_constant__ TableChunk c, LayerPtrs* table) {
  pdl_wait();
  pdl_trigger();
  if (static_cast<int>(threadIdx.x) < c.n) table[c.first + threadIdx.x] = c.L[threadIdx.x];
}

// ---- host side -------------------------------------------------------------------------
inline int64_t al256(int64_t b) { return (b + 255) / 256 * 256; }

struct Geo {
  int H, nq, nkv, hd, rep, W, nqkv, gated, half;
  int tq, uq, cq, to, uo, co, ta, ua, ca, tb, ub, cb, ra;
  int grid, smax, stages, vin_floats, smem;
};

struct WsLayout {
  int64_t table, flags, ready, cnt_att, cnt_q, cnt_o, cnt_a, cnt_b, acc_q, acc_o, acc_a, acc_b;
  int64_t xr1, qkv, attn, h1, h, part, total;
};

constexpr int kHdrBytes = 64;     // epoch, done, status, next, stage counters [4], check [2]

WsLayout ws_layout(const Geo& g, int n_layers) {
  WsLayout w{};
  int64_t o = al256(kHdrBytes);
  w.table = o;
  o = al256(o + static_cast<int64_t>(n_layers) * static_cast<int64_t>(sizeof(LayerPtrs)));
  w.flags = o;
  o = al256(o + static_cast<int64_t>(n_layers) * 4 * 4);
  w.ready = o;
  o = al256(o + static_cast<int64_t>(n_layers) * g.ta * 4);
  w.cnt_att = o;
  o = al256(o + static_cast<int64_t>(g.nkv) * 4);
  w.cnt_q = o;
  o = al256(o + static_cast<int64_t>(g.tq) * 4);
  w.cnt_o = o;
  o = al256(o + static_cast<int64_t>(g.to) * 4);
  w.cnt_a = o;
  o = al256(o + static_cast<int64_t>(g.ta) * 4);
  w.cnt_b = o;
  o = al256(o + static_cast<int64_t>(g.tb) * 4);
  w.acc_q = o;
  o = al256(o + static_cast<int64_t>(g.tq) * kTileN * 8);
  w.acc_o = o;
  o = al256(o + static_cast<int64_t>(g.to) * kTileN * 8);
  w.acc_a = o;
  o = al256(o + static_cast<int64_t>(g.ta) * (g.gated ? 2 : 1) * kTileN * 8);
  w.acc_b = o;
  o = al256(o + static_cast<int64_t>(g.tb) * kTileN * 8);
  w.xr1 = o;
  o = al256(o + static_cast<int64_t>(g.H) * 4);
  w.qkv = o;
  o = al256(o + static_cast<int64_t>(g.tq) * kTileN * 4);
  w.attn = o;
  o = al256(o + static_cast<int64_t>(g.nq) * g.hd * 4);
  w.h1 = o;
  o = al256(o + static_cast<int64_t>(g.H) * 4);
  w.h = o;
  o = al256(o + static_cast<int64_t>(g.ta) * kTileN * 4);
  w.part = o;
  o = al256(o + static_cast<int64_t>(g.nkv) * g.smax * (2 * g.rep + g.rep * g.hd) * 4);
  w.total = o;
  return w;
}

// Checks that the persistent kernel serves this decoder and fills in its geometry.
int geometry(const pyre_decoder_desc* d, Geo& g, const char* fn) {
  std::string f(fn);
  PYRE_CHECK_ARG(d != nullptr && d->layers != nullptr, f + ": null descriptor");
  PYRE_CHECK_ARG(d->n_layers >= 1 && d->n_layers <= kMaxLayers, f + ": 1 to 64 layers");
  PYRE_CHECK_ARG(d->batch <= 1, f + ": one sequence (batch 1)");
  PYRE_CHECK_ARG(d->comm == nullptr, f + ": one GPU (no communicator)");
  PYRE_CHECK_ARG(d->scale_dtype == PYRE_F16, f + ": Q8_0 matrices with f16 scales");
  PYRE_CHECK_ARG(d->hd == 64 || d->hd == 128, f + ": head_dim 64 or 128");
  PYRE_CHECK_ARG(d->nq >= 1 && d->nkv >= 1 && d->nq % d->nkv == 0, f + ": bad head counts");
  g.H = d->H;
  g.nq = d->nq;
  g.nkv = d->nkv;
  g.hd = d->hd;
  g.rep = d->nq / d->nkv;
  g.W = d->ffn_width;
  PYRE_CHECK_ARG(g.rep * g.hd <= kMaxRepHd, f + ": (query heads per kv head) x head_dim must be <= 512");
  PYRE_CHECK_ARG(g.H % 64 == 0 && (g.nq * g.hd) % 64 == 0 && g.W % 64 == 0 && g.H >= 64,
                 f + ": H, nq * hd and the FFN width must be multiples of 64");
  PYRE_CHECK_ARG(g.H <= 16384 && g.nq * g.hd <= 16384, f + ": H and nq * hd at most 16384");
  g.nqkv = (g.nq + 2 * g.nkv) * g.hd;
  g.gated = d->layers[0].gated ? 1 : 0;
  for (int i = 0; i < d->n_layers; ++i)
    PYRE_CHECK_ARG((d->layers[i].gated ? 1 : 0) == g.gated, f + ": every layer gated alike");
  const int dims = static_cast<int>(g.hd * d->rope_fraction);
  g.half = (dims / 2);
  g.tq = tiles_of(g.nqkv);
  g.uq = g.H / kUnitRowsSingle;
  g.cq = (g.uq + kChunkBlocks - 1) / kChunkBlocks;
  g.to = tiles_of(g.H);
  g.uo = g.nq * g.hd / kUnitRowsSingle;
  g.co = (g.uo + kChunkBlocks - 1) / kChunkBlocks;
  g.ra = g.gated ? kUnitRowsPair : kUnitRowsSingle;
  g.ta = tiles_of(g.W);
  g.ua = g.H / g.ra;
  g.ca = (g.ua + kChunkBlocks - 1) / kChunkBlocks;
  g.tb = tiles_of(g.H);
  g.ub = g.W / kUnitRowsSingle;
  g.cb = (g.ub + kChunkBlocks - 1) / kChunkBlocks;
  g.grid = kCtasPerSm * sm_count();
  g.smax = (g.grid + g.nkv - 1) / g.nkv;
  // the last split's combine keeps [rep][S] maxima and sums in the reduction buffer
  const int smax_red = (kCW * kMaxRepHd - g.rep) / (2 * g.rep);
  if (g.smax > smax_red) g.smax = smax_red;
  const int kin = g.H > g.nq * g.hd ? g.H : g.nq * g.hd;
  g.vin_floats = (kin + 63) / 64 * 64;
  // as many ring stages as fit next to the rest of the shared memory (at most 12)
  const int fixed = smem_layout(0, g.vin_floats).total;
  const int limit = (228 * 1024) / kCtasPerSm - 1024;   // per CTA, with the 1 KB reserved per CTA
  g.stages = (limit - fixed) / kBlockBytes;
  if (g.stages > kMaxStages) g.stages = kMaxStages;
  PYRE_CHECK_ARG(g.stages >= 3, f + ": shared memory too small for the stage ring");
  g.smem = smem_layout(g.stages, g.vin_floats).total;
  return PYRE_OK;
}

}  // namespace pd
}  // namespace pyre

extern "C" int pyre_decoder_persistent_workspace_bytes(const pyre_decoder_desc* d, int64_t* bytes) {
  using namespace pyre::pd;
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_decoder_persistent_workspace_bytes: null pointer");
  Geo g{};
  int rc = geometry(d, g, "pyre_decoder_persistent_workspace_bytes");
  if (rc) return rc;
  *bytes = ws_layout(g, d->n_layers).total;
  return PYRE_OK;
}

extern "C" int pyre_decoder_persistent_status(const void* workspace, int* status) {
  PYRE_CHECK_ARG(workspace != nullptr && status != nullptr, "pyre_decoder_persistent_status: null pointer");
  PYRE_CUDA_TRY(cudaMemcpy(status, static_cast<const uint8_t*>(workspace) + 8, 4, cudaMemcpyDeviceToHost));
  return PYRE_OK;
}

extern "C" int pyre_decoder_step_persistent(const pyre_decoder_desc* d, void* workspace, int64_t ws_bytes,
                                            const int* token_in, int pos, int* token_out, float* logits,
                                            void* stream) {
  using namespace pyre;
  using namespace pyre::pd;
  Geo g{};
  int rc = geometry(d, g, "pyre_decoder_step_persistent");
  if (rc) return rc;
  PYRE_CHECK_ARG(token_in != nullptr && token_out != nullptr, "pyre_decoder_step_persistent: null token pointer");
  PYRE_CHECK_ARG(pos >= 0 && pos < d->max_t, "pyre_decoder_step_persistent: position outside the KV cache");
  PYRE_CHECK_ARG(d->pos_dev == nullptr || d->history != nullptr,
                 "pyre_decoder_step_persistent: pos_dev needs a history buffer");
  PYRE_CHECK_ARG(d->lm_V >= 0 && d->lm_v0 >= 0 && d->lm_v0 + (d->lm_V > 0 ? d->lm_V : d->V) <= d->V,
                 "pyre_decoder_step_persistent: lm_head rows outside the vocabulary");
  const WsLayout w = ws_layout(g, d->n_layers);
  PYRE_CHECK_ARG(workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 "pyre_decoder_step_persistent: workspace must be 256-byte aligned device memory");
  if (ws_bytes < w.total)
    return set_error(PYRE_ENOMEM, "pyre_decoder_step_persistent: workspace smaller than "
                                  "pyre_decoder_persistent_workspace_bytes");
  for (int i = 0; i < d->n_layers; ++i) {
    const pyre_decoder_layer& Ld = d->layers[i];
    PYRE_CHECK_ARG(Ld.qkv_w && Ld.o_w && Ld.gateup_w && Ld.down_w && Ld.ln1 && Ld.ln2 && Ld.k_cache && Ld.v_cache &&
                       Ld.rope,
                   "pyre_decoder_step_persistent: null layer pointer");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  // x = embedding rows (the first RMSNorm is the persistent kernel's)
  rc = pyre_embed_rms_norm(token_in, 1, d->embedding, d->V, d->H, nullptr, d->eps, d->x, nullptr, d->status, stream);
  if (rc) return rc;
  // the layer pointers, read from the descriptor on every call, go to the workspace's table
  LayerPtrs* table = reinterpret_cast<LayerPtrs*>(ws + w.table);
  for (int i0 = 0; i0 < d->n_layers; i0 += kTableChunk) {
    TableChunk c{};
    c.first = i0;
    c.n = d->n_layers - i0 < kTableChunk ? d->n_layers - i0 : kTableChunk;
    for (int j = 0; j < c.n; ++j) {
      const pyre_decoder_layer& Ld = d->layers[i0 + j];
      c.L[j] = LayerPtrs{static_cast<const uint8_t*>(Ld.qkv_w), Ld.qkv_bias, static_cast<const uint8_t*>(Ld.o_w),
                         static_cast<const uint8_t*>(Ld.gateup_w), static_cast<const uint8_t*>(Ld.down_w), Ld.ln1,
                         Ld.ln2, reinterpret_cast<__half*>(Ld.k_cache), reinterpret_cast<__half*>(Ld.v_cache),
                         reinterpret_cast<const float2*>(Ld.rope)};
    }
    PYRE_CUDA_TRY(launch_pdl(pd_table_kernel, dim3(1), dim3(kTableChunk), 0, s, c, table));
  }
  Params p{};
  p.layers = table;
  p.magic = kMagic;
  p.n_layers = d->n_layers;
  p.H = g.H;
  p.nq = g.nq;
  p.nkv = g.nkv;
  p.hd = g.hd;
  p.rep = g.rep;
  p.W = g.W;
  p.max_t = d->max_t;
  p.half = g.half;
  p.gated = g.gated;
  p.nqkv = g.nqkv;
  p.stages = g.stages;
  p.tq = g.tq;
  p.uq = g.uq;
  p.cq = g.cq;
  p.to = g.to;
  p.uo = g.uo;
  p.co = g.co;
  p.ta = g.ta;
  p.ua = g.ua;
  p.ca = g.ca;
  p.tb = g.tb;
  p.ub = g.ub;
  p.cb = g.cb;
  p.ra = g.ra;
  p.smax = g.smax;
  p.vin_floats = g.vin_floats;
  p.scale2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(g.hd)));
  p.eps = d->eps;
  p.pos = pos;
  p.pos_dev = d->pos_dev;
  p.xr[0] = d->x;
  p.xr[1] = reinterpret_cast<float*>(ws + w.xr1);
  p.qkv = reinterpret_cast<float*>(ws + w.qkv);
  p.attn = reinterpret_cast<float*>(ws + w.attn);
  p.h1 = reinterpret_cast<float*>(ws + w.h1);
  p.h = reinterpret_cast<float*>(ws + w.h);
  p.part = reinterpret_cast<float*>(ws + w.part);
  p.acc_q = reinterpret_cast<unsigned long long*>(ws + w.acc_q);
  p.acc_o = reinterpret_cast<unsigned long long*>(ws + w.acc_o);
  p.acc_a = reinterpret_cast<unsigned long long*>(ws + w.acc_a);
  p.acc_b = reinterpret_cast<unsigned long long*>(ws + w.acc_b);
  p.cnt_q = reinterpret_cast<unsigned*>(ws + w.cnt_q);
  p.cnt_o = reinterpret_cast<unsigned*>(ws + w.cnt_o);
  p.cnt_a = reinterpret_cast<unsigned*>(ws + w.cnt_a);
  p.cnt_b = reinterpret_cast<unsigned*>(ws + w.cnt_b);
  p.cnt_att = reinterpret_cast<unsigned*>(ws + w.cnt_att);
  p.stage_cnt = reinterpret_cast<unsigned*>(ws + 16);
  p.flags = reinterpret_cast<uint32_t*>(ws + w.flags);
  p.ready = reinterpret_cast<uint32_t*>(ws + w.ready);
  p.next = reinterpret_cast<unsigned*>(ws + 12);
  p.epoch = reinterpret_cast<uint32_t*>(ws + 0);
  p.done = reinterpret_cast<unsigned*>(ws + 4);
  p.status = reinterpret_cast<int*>(ws + 8);
  p.check = reinterpret_cast<int*>(ws + 32);
  p.mat_bytes[0] = static_cast<int64_t>(g.tq) * g.uq * kBlockBytes;
  p.mat_bytes[1] = static_cast<int64_t>(g.to) * g.uo * kBlockBytes;
  p.mat_bytes[2] = static_cast<int64_t>(g.ta) * g.ua * kBlockBytes;
  p.mat_bytes[3] = static_cast<int64_t>(g.tb) * g.ub * kBlockBytes;
  p.cache_elems = static_cast<int64_t>(g.nkv) * d->max_t * g.hd;
  p.part_floats = static_cast<int64_t>(g.nkv) * g.smax * (2 * g.rep + g.rep * g.hd);
  auto kern = g.hd == 128 ? decode_persistent_kernel<128> : decode_persistent_kernel<64>;
  rc = set_smem_limit(reinterpret_cast<const void*>(kern), 227 * 1024);
  if (rc) return rc;
  int occ = 0;
  PYRE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreadsPD, g.smem));
  if (occ < kCtasPerSm) return set_error(PYRE_ECUDA, "decode_persistent_kernel: two CTAs do not fit on an SM");
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(g.grid));
  cfg.blockDim = dim3(kThreadsPD);
  cfg.dynamicSmemBytes = static_cast<size_t>(g.smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1]{};
  // every CTA waits for results of others: the grid (one CTA per SM) must be co-resident
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PYRE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
  PYRE_LAUNCH_CHECK("decode_persistent_kernel");
  const int lm_V = d->lm_V > 0 ? d->lm_V : d->V;
  rc = pyre_lm_head_argmax(p.xr[d->n_layers & 1], 1, d->H, d->final_norm, d->eps, d->lm_head, lm_V, d->lm_v0, logits,
                           token_out, d->key, d->lm_ws, d->lm_ws_bytes, stream);
  if (rc) return rc;
  if (d->pos_dev == nullptr) return PYRE_OK;
  PYRE_CUDA_TRY(launch_pdl(pd_advance_kernel, dim3(1), dim3(1), 0, s, d->pos_dev, static_cast<const int*>(token_out),
                           d->history, d->max_t));
  return PYRE_OK;
}
