// Host side of the decode-path streaming kernel (ffn_stream.cuh) and the one-launch decode
// FFN entry point. Reference semantics: src/ffn/builder.py:37-45 and
// src/orchestrator/root_node.py:956-995.
#include "ffn_stream.cuh"

namespace pyre {
namespace ffn {

inline int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

// Fixed-point slab accumulators of one phase: [tiles(N), nmat, T, 256] int64.
int64_t stream_acc_bytes(int T, int N, int nmat) {
  return align256(static_cast<int64_t>(tiles_of(N)) * nmat * T * kTileN * 8);
}

// Workspace layouts (after the kHeaderBytes header):
//   MODE_A / MODE_B : accumulators of that phase, from the start of the lead region
//   MODE_AB         : accumulators B from the start of the lead region; after the lead region
//                     (sized for T = PYRE_FUSED_REDUCE_MAX_T and both phases, so no call of
//                     any T or mode reaches past it) the two sets of gate/up slab sums
//                     [2][tiles(W)][kSlabSums] int64 and chunk counts [2][tiles(W)] u32
// Everything in the lead region must be zero when a call starts (each call zeroes what it
// used); the MODE_AB sets are cleared by alternate calls. The tensor-core GEMM's staging and
// partial tiles are plain data and sit at the END of the workspace, so calls with any T (and
// of either path) can share one workspace.
int64_t lead_bytes(int H, int W) {
  const int64_t a = stream_acc_bytes(PYRE_FUSED_REDUCE_MAX_T, W, 2);
  const int64_t b = stream_acc_bytes(PYRE_FUSED_REDUCE_MAX_T, H, 1);
  return a > b ? a : b;
}
int64_t ab_sums_bytes(int W) { return align256(2 * static_cast<int64_t>(tiles_of(W)) * kSlabSums * 8); }
int64_t decode_ws_bytes(int H, int W) {
  return kHeaderBytes + lead_bytes(H, W) + ab_sums_bytes(W) + align256(2 * static_cast<int64_t>(tiles_of(W)) * 4);
}

struct StreamArgs {
  int mode;
  bool tp;
  const void* xa;      // phase-A activation [T, KA]
  int xa_dtype;
  const void* xb;      // phase-B activation [T, KB] (MODE_B); MODE_AB computes h from the slab sums
  int xb_dtype;
};

template <int T, int NA, typename XA, typename XB, typename ST, int MODE, bool TP>
int launch_stream(StreamParams p, const StreamArgs& a, cudaStream_t s) {
  using C = StreamCfg<T, NA, XA, XB, ST>;
  auto kern = q80_ffn_stream_kernel<T, NA, XA, XB, ST, MODE, TP>;
  int rc = set_smem_once(kern, C::kSmemBytes);
  if (rc) return rc;
  if constexpr ((MODE & MODE_A) != 0) {
    rc = make_tmap_2d(&p.txa, a.xa, tma_dtype<XA>(), sizeof(XA), T, p.KA, static_cast<uint64_t>(p.KA) * sizeof(XA), T,
                      C::LA::kRows);
    if (rc) return rc;
  }
  if constexpr (MODE == MODE_B) {
    rc = make_tmap_2d(&p.txb, a.xb, tma_dtype<XB>(), sizeof(XB), T, p.KB, static_cast<uint64_t>(p.KB) * sizeof(XB), T,
                      C::LB::kRows);
    if (rc) return rc;
  }
  int occ = 0;
  PYRE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kStreamThreads, C::kSmemBytes));
  if (occ < 1) return set_error(PYRE_ECUDA, "q80_ffn_stream_kernel does not fit on an SM");
  if (occ > C::kCtasPerSm) occ = C::kCtasPerSm;
  int64_t g = static_cast<int64_t>(occ) * sm_count();   // co-resident (tensor-parallel waits)
  const int64_t chunks = static_cast<int64_t>(p.ncA) + p.ncB;
  if (g > chunks) g = chunks;
  if (g < 1) g = 1;
  if constexpr (MODE == MODE_AB) {
    // Lead of phase A over phase B in the queue, in groups. A phase-A slab becomes usable
    // several microseconds after its last chunk is streamed (count, read-back, release under
    // full HBM load), so a phase-B chunk queued a round or two after its rows blocks its
    // producer; measured on the 7B decode shape, queueing all of phase A first is faster.
    static_assert((kChunk * C::LB::kRows) % kTileN == 0, "a phase-B chunk must cover whole phase-A slabs");
    p.spg = kChunk * C::LB::kRows / kTileN;
    p.slack = p.cptB;
  }
  // May start while the previous kernel finishes: its first weight copies overlap that tail.
  // Everything else (activations, scratch, and with tensor parallelism the communicator's
  // epoch, peer stores and flag waits) comes after griddepcontrol.wait, i.e. after the previous
  // kernel has completed. A tensor-parallel grid is sized to be co-resident and its CTAs wait
  // only for peer ranks (never for CTAs of their own grid), so an early start cannot deadlock.
  PYRE_CUDA_TRY(launch_pdl(kern, dim3(static_cast<unsigned>(g)), dim3(kStreamThreads),
                           static_cast<size_t>(C::kSmemBytes), s, p));
  return PYRE_OK;
}

template <int T, int NA, typename XA, typename XB, typename ST>
int stream_mode(StreamParams p, const StreamArgs& a, cudaStream_t s) {
  switch (a.mode) {
    case MODE_A: return launch_stream<T, NA, XA, XB, ST, MODE_A, false>(p, a, s);
    case MODE_B:
      return a.tp ? launch_stream<T, NA, XA, XB, ST, MODE_B, true>(p, a, s)
                  : launch_stream<T, NA, XA, XB, ST, MODE_B, false>(p, a, s);
    default:
      return a.tp ? launch_stream<T, NA, XA, XB, ST, MODE_AB, true>(p, a, s)
                  : launch_stream<T, NA, XA, XB, ST, MODE_AB, false>(p, a, s);
  }
}

// Type dispatch. MODE_A: XA = x dtype; MODE_B: XB = x dtype (NA unused, 1);
// MODE_AB: XA = x dtype, XB = f32 (h).
template <int T, int NA>
int stream_types(StreamParams p, const StreamArgs& a, int scale_dtype, cudaStream_t s) {
  const bool f16s = scale_dtype == PYRE_F16;
  if (a.mode == MODE_B) {
    if (a.xb_dtype == PYRE_BF16)
      return f16s ? stream_mode<T, 1, float, __nv_bfloat16, __half>(p, a, s)
                  : stream_mode<T, 1, float, __nv_bfloat16, float>(p, a, s);
    return f16s ? stream_mode<T, 1, float, float, __half>(p, a, s) : stream_mode<T, 1, float, float, float>(p, a, s);
  }
  if (a.xa_dtype == PYRE_BF16)
    return f16s ? stream_mode<T, NA, __nv_bfloat16, float, __half>(p, a, s)
                : stream_mode<T, NA, __nv_bfloat16, float, float>(p, a, s);
  return f16s ? stream_mode<T, NA, float, float, __half>(p, a, s) : stream_mode<T, NA, float, float, float>(p, a, s);
}

template <int NA>
int stream_T(StreamParams p, const StreamArgs& a, int scale_dtype, cudaStream_t s) {
  switch (p.T) {
    case 1: return stream_types<1, NA>(p, a, scale_dtype, s);
    case 2: return stream_types<2, NA>(p, a, scale_dtype, s);
    case 3: return stream_types<3, NA>(p, a, scale_dtype, s);
    case 4: return stream_types<4, NA>(p, a, scale_dtype, s);
    default: return set_error(PYRE_EINVAL, "streaming FFN kernel: T must be in [1, 4]");
  }
}

void fill_phase(StreamParams& p, bool phase_b, int K, int N, int nmat) {
  const int R = nmat == 2 ? kUnitRowsPair : kUnitRowsSingle;
  const int tiles = tiles_of(N), upt = (K + R - 1) / R, cpt = (upt + kChunk - 1) / kChunk;
  if (!phase_b) {
    p.KA = K; p.NA = N; p.tilesA = tiles; p.uptA = upt; p.cptA = cpt; p.ncA = tiles * cpt;
  } else {
    p.KB = K; p.NB = N; p.tilesB = tiles; p.uptB = upt; p.cptB = cpt; p.ncB = tiles * cpt;
  }
}

void fill_header(StreamParams& p, char* wsc) {
  p.cntA = reinterpret_cast<unsigned int*>(wsc + kHdrCntA);
  p.cntB = reinterpret_cast<unsigned int*>(wsc + kHdrCntB);
  p.ready = reinterpret_cast<uint32_t*>(wsc + kHdrReady);
  p.next = reinterpret_cast<unsigned int*>(wsc + kHdrNext);
  p.ws_epoch = reinterpret_cast<uint32_t*>(wsc + kHdrEpoch);
  p.ws_done = reinterpret_cast<unsigned int*>(wsc + kHdrDone);
  p.status = reinterpret_cast<int*>(wsc + kHdrStatus);
}

}  // namespace ffn

// Streaming-kernel forms of the two-call entry points (T <= 4), used by ffn.cu.
int ffn_stream_gateup(const void* x, int x_dtype, int T, int H, const void* wgu, int gated, int scale_dtype, int W,
                      void* h, int h_dtype, void* workspace, int64_t ws_bytes, cudaStream_t s) {
  using namespace ffn;
  const int na = gated ? 2 : 1;
  if (ws_bytes < kHeaderBytes + stream_acc_bytes(T, W, na))
    return set_error(PYRE_ENOMEM, "pyre_ffn_gateup_silu_q80: workspace smaller than pyre_ffn_workspace_bytes()");
  char* wsc = static_cast<char*>(workspace);
  StreamParams p{};
  p.T = T;
  p.wa = static_cast<const uint8_t*>(wgu);
  fill_phase(p, false, H, W, na);
  p.outA = h;
  p.outA_bf16 = h_dtype == PYRE_BF16;
  p.accA = reinterpret_cast<unsigned long long*>(wsc + kHeaderBytes);
  fill_header(p, wsc);
  StreamArgs a{MODE_A, false, x, x_dtype, nullptr, PYRE_F32};
  return gated ? stream_T<2>(p, a, scale_dtype, s) : stream_T<1>(p, a, scale_dtype, s);
}

int ffn_stream_down(const void* h, int h_dtype, int T, int W, const void* wd, int scale_dtype, int H, float* out,
                    void* workspace, int64_t ws_bytes, pyre_comm_t* comm, cudaStream_t s, const float* bias) {
  using namespace ffn;
  if (ws_bytes < kHeaderBytes + stream_acc_bytes(T, H, 1))
    return set_error(PYRE_ENOMEM, "pyre_ffn_down_q80: workspace smaller than pyre_ffn_workspace_bytes()");
  const bool tp = comm != nullptr && comm->world > 1;
  PYRE_CHECK_ARG(!tp || tiles_of(H) <= kMaxOwnedTiles, "pyre_ffn_down_q80: H too large for the fused reduce");
  char* wsc = static_cast<char*>(workspace);
  StreamParams p{};
  p.T = T;
  p.wb = static_cast<const uint8_t*>(wd);
  fill_phase(p, true, W, H, 1);
  p.outB = out;
  p.biasB = tp ? nullptr : bias;
  p.accB = reinterpret_cast<unsigned long long*>(wsc + kHeaderBytes);
  fill_header(p, wsc);
  if (tp) p.comm = comm::device_view(comm);
  StreamArgs a{MODE_B, tp, nullptr, PYRE_F32, h, h_dtype};
  return stream_T<1>(p, a, scale_dtype, s);
}

}  // namespace pyre

using namespace pyre;
using namespace pyre::ffn;

extern "C" int pyre_ffn_workspace_bytes(int T, int H, int W, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_ffn_workspace_bytes: null bytes");
  PYRE_CHECK_ARG(T >= 1 && H >= 1 && W >= 1, "pyre_ffn_workspace_bytes: sizes must be positive");
  // decode (T <= 4, also the two-call forms) at the start and, for larger T, the tensor-core
  // GEMM's f16 activation staging and partial tiles after it (placed from the end by the
  // GEMM calls): the two never overlap, so calls of either kind can follow each other
  int64_t need = decode_ws_bytes(H, W);
  if (T > PYRE_FUSED_REDUCE_MAX_T) {
    const int64_t pg = ffn_gemm_partial_bytes(T, W, 2), pd = ffn_gemm_partial_bytes(T, H, 1);
    need += ffn_gemm_staging_bytes(T, H, W) + (pg > pd ? pg : pd) + 256;
  }
  *bytes = need;
  return PYRE_OK;
}

namespace pyre {
// Every argument check of pyre_ffn_decode_q80, before anything is queued on the stream.
int ffn_decode_check(const void* x, int x_dtype, int T, int H, const void* wgu, int gated, const void* wd,
                     int scale_dtype, int W, const float* out, const void* workspace, int64_t ws_bytes,
                     const pyre_comm_t* comm, const char* fn) {
  using namespace ffn;
  const std::string f(fn);
  int rc = ffn_check_common(x, x_dtype, T, H, W, scale_dtype, out, workspace, ws_bytes, fn);
  if (rc) return rc;
  PYRE_CHECK_ARG(T <= PYRE_FUSED_REDUCE_MAX_T, f + ": T must be <= PYRE_FUSED_REDUCE_MAX_T");
  PYRE_CHECK_ARG(H % 32 == 0 && W % 32 == 0, f + ": H and W must be multiples of 32");
  PYRE_CHECK_ARG(wgu != nullptr && wd != nullptr && reinterpret_cast<uintptr_t>(wgu) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(wd) % 16 == 0,
                 f + ": packed weights must be non-null and 16-byte aligned");
  PYRE_CHECK_ARG(tiles_of(H) <= kMaxTiles && tiles_of(W) <= kMaxTiles, f + ": dims too large");
  if (comm != nullptr) {
    const bool tp = comm->world > 1;
    PYRE_CHECK_ARG(comm->hidden == H, f + ": communicator hidden size differs from H");
    PYRE_CHECK_ARG(T <= comm->max_tokens, f + ": T exceeds the communicator's max_tokens");
    PYRE_CHECK_ARG(!tp || tiles_of(H) <= kMaxOwnedTiles, f + ": H too large for the fused reduce");
  }
  if (ws_bytes < decode_ws_bytes(H, W))
    return set_error(PYRE_ENOMEM, f + ": workspace smaller than pyre_ffn_workspace_bytes()");
  return PYRE_OK;
}
}  // namespace pyre

extern "C" int pyre_ffn_decode_q80(const void* x, int x_dtype, int T, int H, const void* wgu, int gated,
                                   const void* wd, int scale_dtype, int W, float* out, void* workspace,
                                   int64_t ws_bytes, pyre_comm_t* comm, void* stream) {
  int rc = ffn_decode_check(x, x_dtype, T, H, wgu, gated, wd, scale_dtype, W, out, workspace, ws_bytes, comm,
                            "pyre_ffn_decode_q80");
  if (rc) return rc;
  const bool tp = comm != nullptr && comm->world > 1;
  const int na = gated ? 2 : 1;
  char* wsc = static_cast<char*>(workspace);
  StreamParams p{};
  p.T = T;
  p.wa = static_cast<const uint8_t*>(wgu);
  p.wb = static_cast<const uint8_t*>(wd);
  fill_phase(p, false, H, W, na);
  fill_phase(p, true, W, H, 1);
  // phase-B accumulators (zero on entry, zeroed again by the kernel) right after the header;
  // the gate/up slab sums and counts after the lead region (see decode_ws_bytes)
  p.accB = reinterpret_cast<unsigned long long*>(wsc + kHeaderBytes);
  p.sumA = reinterpret_cast<unsigned long long*>(wsc + kHeaderBytes + lead_bytes(H, W));
  p.cntAB = reinterpret_cast<unsigned int*>(reinterpret_cast<char*>(p.sumA) + ab_sums_bytes(W));
  p.ab_calls = reinterpret_cast<unsigned int*>(wsc + kHdrAbCalls);
  p.outB = out;
  fill_header(p, wsc);
  if (tp) p.comm = comm::device_view(comm);
  StreamArgs a{MODE_AB, tp, x, x_dtype, nullptr, PYRE_F32};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return gated ? stream_T<2>(p, a, scale_dtype, s) : stream_T<1>(p, a, scale_dtype, s);
}
