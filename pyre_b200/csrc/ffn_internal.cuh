// Internal pieces shared by ffn.cu (two-call FFN) and ffn_decode.cu (one-launch decode FFN).
#pragma once

#include "gemv_common.cuh"

namespace pyre {
namespace ffn {

using namespace gemv;

enum Epi : int { EPI_SILU_MUL = 0, EPI_SILU = 1, EPI_STORE = 2, EPI_TP = 3 };

struct alignas(64) Params {
  CUtensorMap tx;            // activations [T, K], box T x R
  const void* x;
  const uint8_t* w;          // packed weight group (gate/up pair, or one matrix)
  int K, N, T;
  int tiles;                 // ceil(N / kTileN)
  int upt;                   // units per tile = ceil(K / R)
  int64_t total_units;       // tiles * upt
  int pmax;                  // piece slots per tile in ws
  int64_t ws_cap;            // bytes available for pieces
  float* ws;                 // [tiles, pmax, NMAT, T, kTileN]
  unsigned int* counters;    // [tiles], zero between calls
  int* status;               // device status word (bounded waits)
  void* out;                 // [T, N]
  int out_bf16;
  comm::DevComm comm;        // EPI_TP only
};

__device__ __forceinline__ void store_out(void* out, int out_bf16, int N, int t, int col, float v) {
  const int64_t o = static_cast<int64_t>(t) * N + col;
  if (out_bf16)
    static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(out)[o] = v;
}

// Cross-rank sum of one finished tile (the reference's `ffn_out += partial`,
// src/orchestrator/root_node.py:582-594), split for kernels that schedule work dynamically
// (the chunk to CTA map differs between ranks, so a CTA must never block on a peer while it
// still holds unprocessed work): tp_push_tile() pushes the partial into every rank's receive
// slot (self included) over NVLink and releases a flag per peer without waiting;
// tp_finish_tile() waits (bounded) for every peer's flag of the tile and adds the partials in
// rank order 0..world-1, called after all work is drained.
template <int T>
__device__ void tp_push_tile(const comm::DevComm& c, uint32_t epoch, int tile, const float* fin, int tid) {
  const int slot = epoch & 1u;
  const int n = T * kTileN;
  for (int peer = 0; peer < c.world; ++peer) {
    float* dst = comm::fused_slot(c, peer, slot, c.rank) + static_cast<int64_t>(tile) * n;
    for (int i = tid; i < n; i += kConsumers) dst[i] = fin[i];
  }
  __threadfence_system();
  consumer_sync();
  if (tid < c.world) st_release_sys(comm::fused_flag(c, tid, slot, c.rank, tile), epoch);
}

template <int T>
__device__ void tp_finish_tile(const comm::DevComm& c, uint32_t epoch, int tile, float* out, int N, int tid) {
  const int slot = epoch & 1u;
  const int n = T * kTileN;
  if (tid < c.world) {
    if (!wait_flag_eq(comm::fused_flag(c, c.rank, slot, tid, tile), epoch, c.timeout_ns))
      atomicExch(c.status, PYRE_ETIMEOUT);
  }
  consumer_sync();
  for (int i = tid; i < n; i += kConsumers) {
    const int t = i / kTileN, cc = i % kTileN;
    const int col = tile * kTileN + cc;
    if (col >= N) continue;
    float acc = 0.f;
    for (int src = 0; src < c.world; ++src)
      acc += __ldcg(comm::fused_slot(c, c.rank, slot, src) + static_cast<int64_t>(tile) * n + i);
    out[static_cast<int64_t>(t) * N + col] = acc;
  }
  consumer_sync();
}

template <typename K>
int set_smem_once(K kern, int bytes) {
  return set_smem_limit(reinterpret_cast<const void*>(kern), bytes);
}

}  // namespace ffn

// Argument checks shared by the FFN entry points (defined in ffn.cu).
int ffn_check_common(const void* x, int x_dtype, int T, int K, int N, int scale_dtype, const void* out,
                     const void* ws, int64_t ws_bytes, const char* fn);
// Streaming-kernel forms of the two-call entry points for T <= 4 (defined in ffn_decode.cu).
// Every argument check of pyre_ffn_decode_q80 (defined in ffn_decode.cu); fn names the caller
// in the error text.
int ffn_decode_check(const void* x, int x_dtype, int T, int H, const void* wgu, int gated, const void* wd,
                     int scale_dtype, int W, const float* out, const void* workspace, int64_t ws_bytes,
                     const pyre_comm_t* comm, const char* fn);
// Cluster GEMV of gemv_cluster.cu for T <= 4 on one packed matrix [K, N] (K <= 8192).
bool gemv_cluster_eligible(int K, int N);
int gemv_cluster(const void* x, int x_dtype, int T, int K, const void* w, int scale_dtype, int N, const float* bias,
                 float* out, int* status, cudaStream_t s);
int ffn_gemm_tc(const void* a, int a_dtype, int T, int K, const void* w, int nmat, int epi, int scale_dtype, int N,
                void* out, int out_dtype, void* staging, int64_t staging_bytes, void* partial, int64_t partial_bytes,
                unsigned int* counters, int* status, cudaStream_t s, const float* bias = nullptr);
int64_t ffn_gemm_partial_bytes(int T, int N, int nmat);
// Workspace regions of the T > 4 path after the header: f16 staging of the activations,
// then the stream-K partial tiles of the GEMM (one per CTA).
inline int64_t ffn_gemm_staging_bytes(int T, int H, int W) {
  return (static_cast<int64_t>(T) * (H > W ? H : W) * 2 + 255) / 256 * 256;
}
int ffn_stream_gateup(const void* x, int x_dtype, int T, int H, const void* wgu, int gated, int scale_dtype, int W,
                      void* h, int h_dtype, void* workspace, int64_t ws_bytes, cudaStream_t s);
int ffn_stream_down(const void* h, int h_dtype, int T, int W, const void* wd, int scale_dtype, int H, float* out,
                    void* workspace, int64_t ws_bytes, pyre_comm_t* comm, cudaStream_t s,
                    const float* bias = nullptr);

}  // namespace pyre
