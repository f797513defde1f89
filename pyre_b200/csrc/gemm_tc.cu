// Tensor-core (tcgen05) Q8_0 GEMM for the FFN at T > 4 tokens (prefill):
//   gate/up:  h[T, W]   = silu(x @ Wg) * (x @ Wu)   (or silu(x @ Wu))     NMAT = 2 (or 1)
//   down:     out[T, H] = h @ Wd                                            NMAT = 1
// Reference semantics: src/ffn/builder.py:37-45 (the graph), src/orchestrator/quantizer.py:29-40
// (Q8_0 dequantization, done here in shared memory), pyre_kernels.mojo:121-129 (silu).
//
// CTA tile: 128 tokens x 256 output columns (one packed slab) per matrix, the whole K.
// One packed weight block (R = 32 rows of a gate/up pair, or 64 rows of one matrix) is one
// pipeline stage; 3 stages. Per stage:
//   producer warp   : TMA of the [128 x R] f16 activation tile (K-major, R*2-byte swizzle)
//                     + one bulk copy of the ~17 KB int8 block;
//   dequant warps   : int8 * scale -> f16 into the B operand (MN-major, 128-byte swizzle),
//                     the layout the MMA reads directly (byte-permute into f16 1024 + u,
//                     one packed subtract, one packed multiply by the f16 scale);
//   MMA warp (1 thr): tcgen05.mma M=128 N=256 K=16, R/16 per matrix, accumulators in tensor
//                     memory (256 columns per matrix); tcgen05.commit frees the stage.
// The dequant warps then read the accumulators (tcgen05.ld) and run the epilogue. The
// k-steps of all tiles are split evenly over one CTA per SM (stream-K, below), so no wave
// of tiles leaves SMs idle. Bulk
// copies and TMA loads only; no cluster multicast. Every mbarrier wait is bounded.
//
// Operands are f16: the weights as f16(q * scale) (q exact in f16, one rounding of the product,
// 2^-11 relative), the activations converted to f16 in the workspace unless they already are
// (the gate/up epilogue writes h in f16 for the down GEMM). Accumulation is f32. A value whose
// magnitude does not fit f16 (>= 65520 after rounding, or not finite) flags PYRE_ERANGE.
#include <algorithm>

#include "ffn_internal.cuh"
#include "umma.cuh"

namespace pyre {
namespace tc {

using namespace gemv;

constexpr int kBM = 128;
constexpr int kMaxCtas = 160;     // stream-K CTAs at most (>= the SM count of a B200)
constexpr int kMinSteps = 8;      // k-steps per CTA at least
constexpr int kBN = 256;
constexpr int kStages = 3;
constexpr int kDequantWarps = 8;
constexpr int kDequant = kDequantWarps * 32;
constexpr int kThreads = 64 + kDequant;   // warp 0 producer + TMEM allocator, warp 1 MMA, then dequant/epilogue

template <int NMAT>
constexpr int64_t kPartBytes() { return static_cast<int64_t>(NMAT) * 256 * 128 * 4; }

template <int NMAT, typename ST>
struct Cfg {
  static constexpr int R = NMAT == 2 ? kUnitRowsPair : kUnitRowsSingle;   // K per stage
  static constexpr int kABytes = kBM * R * 2;                              // f16 activation tile
  static constexpr int kBMatBytes = kBN * R * 2;                           // f16 B per matrix
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
  CUtensorMap ta;           // activations [T, K] f16, box 128 x R
  const uint8_t* w;         // packed weights
  int T, K, N;
  int tiles, upt, mtiles;
  void* out;                // [T, N]
  int out_bf16, out_f16;
  int* status;
  int64_t partial_cap;      // bytes available at partial
  float* partial;           // [CTAs][NMAT, 128 x 256] f32: stream-K partial tile of each CTA
  unsigned int* counters;   // [CTAs] partial-ready flags, zero between calls
  const float* bias;        // EPI_STORE: f32 [N] added to every row, or null
};

// Stores 16 consecutive outputs of row t starting at column col0 (bounds-checked on N).
template <typename P>
__device__ __forceinline__ void store_row16(const P& p, int t, int col0, const float (&v)[16]) {
  const int64_t o = static_cast<int64_t>(t) * p.N + col0;
  if (p.out_f16) {
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 16; ++i) bad |= !(fabsf(v[i]) < 65504.0f);
    if (bad) atomicCAS(p.status, PYRE_OK, PYRE_ERANGE);
  }
  if (col0 + 16 <= p.N) {
    if (p.out_f16) {
      uint4 pk[2];
      uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __half2 hh = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        pw[i] = *reinterpret_cast<uint32_t*>(&hh);
      }
      uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + o);
      dst[0] = pk[0];
      dst[1] = pk[1];
    } else if (p.out_bf16) {
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
    for (int i = 0; i < 16 && col0 + i < p.N; ++i) {
      if (p.out_f16)
        static_cast<__half*>(p.out)[o + i] = __float2half_rn(v[i]);
      else
        ffn::store_out(p.out, p.out_bf16, p.N, t, col0 + i, v[i]);
    }
  }
}

__device__ __forceinline__ __half to_f16(__half v) { return v; }
__device__ __forceinline__ __half to_f16(float v) { return __float2half_rn(v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Byte offset of element (n, k) inside a [256 x R] MN-major, 128-byte-swizzled B tile:
// atoms of 64 columns x 8 rows (1 KB), atoms along N 1 KB apart, 8-row groups 4 KB apart.
__device__ __forceinline__ uint32_t b_offset(int n, int k) {
  return static_cast<uint32_t>((n >> 6) * 1024 + (k >> 3) * 4096 + (k & 7) * 128 + ((((n & 63) >> 3) ^ (k & 7)) << 4));
}

// Stream-K schedule: the tiles' k-steps, tile after tile (tile = slab * mtiles + m-tile, so
// consecutive CTAs share weight slabs), are cut into G equal ranges, one per CTA. A CTA's
// range covers segments of one or more tiles:
//   * a whole tile: accumulate, epilogue;
//   * the start of a tile that continues in the next CTAs (always the CTA's last segment):
//     this CTA finishes the tile: it waits (bounded) for the partials of those CTAs, adds
//     them in k order to its own accumulator and runs the epilogue;
//   * a tile's continuation (always the CTA's first segment): the partial goes to this CTA's
//     slot in the workspace and a flag releases it.
// Waits only go to higher CTA indices and all G <= SM-count CTAs are resident, so the
// schedule has no cycles. Results are deterministic: the same ranges, the same order.
struct Seg {
  int tile, k0, k1;   // k-steps [k0, k1) of tile
};
__device__ __forceinline__ int sk_owner(int64_t u, int64_t total, int G) {   // CTA whose range holds u
  return static_cast<int>(((u + 1) * G - 1) / total);
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
  uint64_t* tmem_free = accfull + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(tmem_free + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int64_t total = static_cast<int64_t>(p.tiles) * p.mtiles * p.upt;
  const int64_t ub = total * c / G, ue = total * (c + 1) / G;   // this CTA's k-steps
  const int t_first = static_cast<int>(ub / p.upt);
  const int nseg = ue > ub ? static_cast<int>((ue - 1) / p.upt) - t_first + 1 : 0;
  auto seg_of = [&](int i) {
    Seg sg;
    sg.tile = t_first + i;
    const int64_t base = static_cast<int64_t>(sg.tile) * p.upt;
    sg.k0 = static_cast<int>((ub > base ? ub : base) - base);
    sg.k1 = static_cast<int>((ue < base + p.upt ? ue : base + p.upt) - base);
    return sg;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&bfull[i], kDequant / 32);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(tmem_free, kDequant / 32);
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
      int64_t j = 0, issued = 0;
      bool ok = true;
      for (int i = 0; ok && i < nseg; ++i) {
        const Seg sg = seg_of(i);
        const int slab = sg.tile / p.mtiles, m0 = (sg.tile - slab * p.mtiles) * kBM;
        const uint8_t* wslab = p.w + static_cast<int64_t>(slab) * p.upt * C::kWBytes;
        for (int kt = sg.k0; kt < sg.k1; ++kt, ++j) {
          const int s = static_cast<int>(j % kStages);
          const uint32_t ph = static_cast<uint32_t>(j / kStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * C::kStageBytes;
          mbar_arrive_expect_tx(&full[s], C::kABytes + C::kWBytes);
          tma_load_2d(st + C::kAOff, &p.ta, kt * C::R, m0, &full[s]);
          bulk_load(st + C::kWOff, wslab + static_cast<int64_t>(kt) * C::kWBytes, C::kWBytes, &full[s]);
          issued = j + 1;
        }
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (int64_t q = issued - kStages < 0 ? 0 : issued - kStages; q < issued; ++q)
        mbar_wait(&full[q % kStages], static_cast<uint32_t>(q / kStages) & 1u, nullptr, 500000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma::idesc_f16_f32_kmaj_mnmaj<kBM, kBN>();
      int64_t j = 0;
      bool ok = true;
      for (int i = 0; ok && i < nseg; ++i) {
        const Seg sg = seg_of(i);
        // the accumulator is overwritten: the previous segment's epilogue must have read it
        if (i > 0 && !mbar_wait(tmem_free, static_cast<uint32_t>(i - 1) & 1u, p.status)) break;
        umma::fence_after_sync();
        for (int kt = sg.k0; kt < sg.k1; ++kt, ++j) {
          const int s = static_cast<int>(j % kStages);
          const uint32_t ph = static_cast<uint32_t>(j / kStages) & 1u;
          if (!mbar_wait(&bfull[s], ph, p.status)) {
            ok = false;
            break;
          }
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
              umma::mma_f16(tmem + m * kBN, ad, bd, idesc, (kt != sg.k0 || kk != 0) ? 1u : 0u);
            }
          }
          umma::mma_commit(&empty[s]);   // the stage is free once these MMAs have read it
        }
        umma::mma_commit(accfull);       // this segment's MMAs (also after an early stop) are done
      }
    }
  } else {
    // ---------------- dequant, then the epilogue of each segment ----------------
    const int dt = threadIdx.x - 64;
    // warps 2..9: TMEM lane quarter = warp % 4, column half = (warp - 2) / 4
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr int kColsPerWarp = kBN * 4 / kDequantWarps;
    const int cbeg = ((warp - 2) / 4) * kColsPerWarp;
    constexpr int kPartFloats = NMAT * kBN * kBM;
    auto part_at = [&](int cta, int m, int c0) {   // coalesced: 16 floats per (thread row, column group)
      return p.partial + static_cast<int64_t>(cta) * kPartFloats + ((m * (kBN / 16) + c0 / 16) * kBM + row) * 16;
    };
    int64_t j = 0;
    bool ok = true;
    for (int i = 0; ok && i < nseg; ++i) {
      const Seg sg = seg_of(i);
      for (int kt = sg.k0; kt < sg.k1; ++kt, ++j) {
        const int s = static_cast<int>(j % kStages);
        const uint32_t ph = static_cast<uint32_t>(j / kStages) & 1u;
        if (!mbar_wait(&full[s], ph, p.status)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * C::kStageBytes;
        const uint8_t* wq = st + C::kWOff;
        const ST* ws = reinterpret_cast<const ST*>(st + C::kWOff + NMAT * C::R * kTileN);
        uint8_t* bt = st + C::kBOff;
        constexpr int kGroups = NMAT * C::R * 32;   // 8-column groups per stage
#pragma unroll 2
        for (int g = dt; g < kGroups; g += kDequant) {
          const int m = g / (C::R * 32);
          const int rem = g - m * (C::R * 32);
          const int k = rem >> 5;
          const int n8 = rem & 31;
          const uint2 q = *reinterpret_cast<const uint2*>(wq + m * C::R * kTileN + k * kTileN + n8 * 8);
          const __half2 sc = __half2half2(to_f16(ws[m * C::R * 8 + k * 8 + (n8 >> 2)]));
          // byte b (offset by 128) -> f16 1024 + b -> minus 1152 = the int8 value, exactly
          const uint32_t w0 = q.x ^ 0x80808080u, w1 = q.y ^ 0x80808080u;
          const __half2 k1152 = __half2half2(__ushort_as_half(0x6480u));
          uint4 o;
          o.x = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w0, 0x64646464u, 0x4140u)), k1152), sc));
          o.y = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w0, 0x64646464u, 0x4342u)), k1152), sc));
          o.z = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w1, 0x64646464u, 0x4140u)), k1152), sc));
          o.w = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w1, 0x64646464u, 0x4342u)), k1152), sc));
          *reinterpret_cast<uint4*>(bt + m * C::kBMatBytes + b_offset(n8 * 8, k)) = o;
        }
        umma::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[s]);
      }
      if (!ok) break;
      // epilogue of this segment: this warp reads TMEM lanes 32*(warp % 4) .. +31 = tile rows
      if (!mbar_wait(accfull, static_cast<uint32_t>(i) & 1u, p.status)) break;
      umma::fence_after_sync();
      const int slab = sg.tile / p.mtiles;
      const int t = (sg.tile - slab * p.mtiles) * kBM + row;
      const bool whole = sg.k0 == 0 && sg.k1 == p.upt;
      const bool finisher = sg.k0 == 0 && sg.k1 < p.upt;
      if (!whole && !finisher) {
        // a tile's continuation: partial into this CTA's slot, then release it
        for (int c0 = cbeg; c0 < cbeg + kColsPerWarp; c0 += 16) {
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            uint32_t a[16];
            umma::tmem_ld16(trow + m * kBN + c0, a);
            umma::tmem_wait_ld();
            float4* dst = reinterpret_cast<float4*>(part_at(c, m, c0));
#pragma unroll
            for (int q = 0; q < 4; ++q)
              __stcg(dst + q, make_float4(__uint_as_float(a[4 * q]), __uint_as_float(a[4 * q + 1]),
                                          __uint_as_float(a[4 * q + 2]), __uint_as_float(a[4 * q + 3])));
          }
        }
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(tmem_free);
        __threadfence();
        named_bar(1, kDequant);
        if (dt == 0) st_release_gpu(p.counters + c, 1u);
        continue;
      }
      // whole tile, or the start of a tile finished here with the partials of CTAs c+1..cl
      int cl = c;
      if (finisher) {
        cl = sk_owner(static_cast<int64_t>(sg.tile + 1) * p.upt - 1, total, G);
        if (dt < cl - c) {
          if (!wait_flag_eq(p.counters + c + 1 + dt, 1u, 2000000000ull)) atomicExch(p.status, PYRE_ETIMEOUT);
        }
        named_bar(1, kDequant);
      }
      for (int c0 = cbeg; c0 < cbeg + kColsPerWarp; c0 += 16) {
        float acc[NMAT][16];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          uint32_t a[16];
          umma::tmem_ld16(trow + m * kBN + c0, a);
          umma::tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q) acc[m][q] = __uint_as_float(a[q]);
        }
        for (int src = c + 1; src <= cl; ++src) {
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const float4* pp = reinterpret_cast<const float4*>(part_at(src, m, c0));
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 v = __ldcg(pp + q);
              acc[m][4 * q] += v.x;
              acc[m][4 * q + 1] += v.y;
              acc[m][4 * q + 2] += v.z;
              acc[m][4 * q + 3] += v.w;
            }
          }
        }
        if (t >= p.T) continue;
        const int col0 = slab * kTileN + c0;
        float v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if constexpr (EPI == ffn::EPI_SILU_MUL) {
            v[q] = silu_f32(acc[0][q]) * acc[NMAT - 1][q];
          } else if constexpr (EPI == ffn::EPI_SILU) {
            v[q] = silu_f32(acc[0][q]);
          } else {
            v[q] = acc[0][q];
          }
        }
        if constexpr (EPI == ffn::EPI_STORE) {
          // the projection bias, added to the finished f32 dot product (x @ W + b)
          if (p.bias != nullptr) {
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (col0 + q < p.N) v[q] += __ldg(p.bias + col0 + q);
          }
        }
        store_row16(p, t, col0, v);
      }
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(tmem_free);
      if (finisher) {
        named_bar(1, kDequant);
        if (dt < cl - c) p.counters[c + 1 + dt] = 0u;   // consumed: back to zero for the next call
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

// f32 or bf16 -> f16 conversion of an activation matrix (row-major, n elements); a value
// that does not fit f16 flags PYRE_ERANGE.
template <typename XT>
__global__ void cvt_f16_kernel(const XT* __restrict__ src, __half* __restrict__ dst, int64_t n, int* status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  bool bad = false;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = to_f32(src[i]);
    bad |= !(fabsf(v) < 65504.0f);
    dst[i] = __float2half_rn(v);
  }
  if (bad) atomicCAS(status, PYRE_OK, PYRE_ERANGE);
}

template <int NMAT, int EPI, typename ST>
int launch(Params p, const void* a_f16, cudaStream_t s) {
  using C = Cfg<NMAT, ST>;
  auto kern = q80_gemm_tc_kernel<NMAT, EPI, ST>;
  int rc = ffn::set_smem_once(kern, C::kSmemBytes);
  if (rc) return rc;
  rc = make_tmap_2d(&p.ta, a_f16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.T, p.K, static_cast<uint64_t>(p.K) * 2,
                    kBM, C::R, C::R * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  p.upt = (p.K + C::R - 1) / C::R;
  p.tiles = tiles_of(p.N);
  p.mtiles = (p.T + kBM - 1) / kBM;
  const int64_t steps = static_cast<int64_t>(p.tiles) * p.mtiles * p.upt;
  // stream-K over at most one CTA per SM (all resident: the finishing CTAs wait for the
  // partials of the next ones), at least kMinSteps k-steps each, slots within the workspace
  int64_t G = sm_count();
  if (G > kMaxCtas) G = kMaxCtas;
  if (G > steps / kMinSteps) G = steps / kMinSteps;
  if (G < 1) G = 1;
  if (p.partial == nullptr || G * kPartBytes<NMAT>() > p.partial_cap)
    return set_error(PYRE_ENOMEM, "q80_gemm_tc_kernel: workspace too small for the stream-K partial tiles");
  kern<<<static_cast<int>(G), kThreads, C::kSmemBytes, s>>>(p);
  PYRE_LAUNCH_CHECK("q80_gemm_tc_kernel");
  return PYRE_OK;
}

}  // namespace tc

// Bytes of stream-K partial tiles the GEMM over [T, K] x [K, N] uses: one tile slot per CTA.
int64_t ffn_gemm_partial_bytes(int T, int N, int nmat) {
  (void)T;
  (void)N;
  return static_cast<int64_t>(tc::kMaxCtas) * nmat * 256 * 128 * 4;
}

// Tensor-core GEMM form of the FFN halves for T > 4 (used by ffn.cu).
//   nmat = 2: out = silu(a @ W0) * (a @ W1) (epi EPI_SILU_MUL); nmat = 1: EPI_SILU or EPI_STORE.
// a: [T, K] f32, bf16 or f16; f32 and bf16 are converted to f16 in `staging` (>= T*K*2 bytes).
// out: [T, N] of out_dtype (f32, bf16 or f16). bias (EPI_STORE only, nullable): f32 [N].
int ffn_gemm_tc(const void* a, int a_dtype, int T, int K, const void* w, int nmat, int epi, int scale_dtype, int N,
                void* out, int out_dtype, void* staging, int64_t staging_bytes, void* partial, int64_t partial_bytes,
                unsigned int* counters, int* status, cudaStream_t s, const float* bias) {
  const void* a_f16 = a;
  if (a_dtype != PYRE_F16) {
    const int64_t n = static_cast<int64_t>(T) * K;
    if (staging == nullptr || staging_bytes < n * 2)
      return set_error(PYRE_ENOMEM, "FFN GEMM: workspace too small for the f16 copy of the activations");
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * 148));
    if (a_dtype == PYRE_F32)
      tc::cvt_f16_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(a), static_cast<__half*>(staging), n,
                                                       status);
    else
      tc::cvt_f16_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(a),
                                                               static_cast<__half*>(staging), n, status);
    PYRE_LAUNCH_CHECK("cvt_f16_kernel");
    a_f16 = staging;
  }
  PYRE_CHECK_ARG((static_cast<int64_t>(K) * 2) % 16 == 0, "FFN GEMM: activation rows must be 16-byte multiples");
  tc::Params p{};
  p.w = static_cast<const uint8_t*>(w);
  p.T = T;
  p.K = K;
  p.N = N;
  p.out = out;
  p.out_bf16 = out_dtype == PYRE_BF16;
  p.out_f16 = out_dtype == PYRE_F16;
  p.status = status;
  p.partial = static_cast<float*>(partial);
  p.partial_cap = partial_bytes;
  p.counters = counters;
  p.bias = epi == ffn::EPI_STORE ? bias : nullptr;
  const bool f16s = scale_dtype == PYRE_F16;
  if (nmat == 2)
    return f16s ? tc::launch<2, ffn::EPI_SILU_MUL, __half>(p, a_f16, s)
                : tc::launch<2, ffn::EPI_SILU_MUL, float>(p, a_f16, s);
  if (epi == ffn::EPI_SILU)
    return f16s ? tc::launch<1, ffn::EPI_SILU, __half>(p, a_f16, s) : tc::launch<1, ffn::EPI_SILU, float>(p, a_f16, s);
  return f16s ? tc::launch<1, ffn::EPI_STORE, __half>(p, a_f16, s) : tc::launch<1, ffn::EPI_STORE, float>(p, a_f16, s);
}

}  // namespace pyre
