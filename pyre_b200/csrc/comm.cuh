// Peer-memory communicator shared by the FFN epilogue and the all-reduce kernels.
#pragma once

#include "common.cuh"

struct pyre_comm {
  int rank;
  int world;
  int max_tokens;
  int hidden;
  uint64_t timeout_ns;
  uint32_t* d_epoch;       // device sequence number of the last finished collective
  unsigned int* d_done;    // arrival counter of the CTAs of the running collective
  char** d_peers;          // device array [world]: base of every rank's receive buffer
  int* d_status;           // device status word (PYRE_OK / PYRE_ETIMEOUT)
  int64_t fused_floats;    // per (slot, src) capacity of the fused-epilogue region
  int64_t ar_chunk;        // per (slot, phase, src) capacity of the all-reduce region
  char* local;             // this rank's receive buffer (bufs[rank] of pyre_comm_create)
};

namespace pyre {
namespace comm {

// Receive-buffer layout (identical on every rank, so one offset works for all peers):
//   [fused region]  2 slots x world srcs x fused_floats  f32   (decode epilogue pushes)
//   [ar region]     2 slots x 2 phases x world x ar_chunk f32  (two-shot all-reduce)
//   [flags]         kFlagWords u32
// Slot = epoch & 1. A rank can only run two collectives ahead of a peer after that peer
// has consumed the older slot, so two slots are enough.
//
// The epoch lives in device memory: every CTA of a collective kernel reads
// e = *d_epoch + 1 when it starts, and the last CTA to finish stores e back. Kernel
// parameters therefore never carry the epoch, and a captured CUDA graph replays
// correctly (each replay is a new epoch on every rank).
constexpr int kFusedMaxTokens = PYRE_FUSED_REDUCE_MAX_T;
constexpr int kTileCols = 128;
constexpr int kMaxTiles = 1024;          // hidden <= 131072
constexpr int kArMaxCtas = 256;
constexpr int kMaxWorld = 16;
// flags: fused [2][kMaxWorld][kMaxTiles] + ar [2 slots][2 phases][kMaxWorld][kArMaxCtas]
constexpr int64_t kFusedFlagWords = 2LL * kMaxWorld * kMaxTiles;
constexpr int64_t kArFlagWords = 2LL * 2 * kMaxWorld * kArMaxCtas;
constexpr int64_t kFlagWords = kFusedFlagWords + kArFlagWords;

struct Layout {
  int64_t fused_floats;
  int64_t ar_chunk;
  int64_t fused_off;   // bytes
  int64_t ar_off;      // bytes
  int64_t flags_off;   // bytes
  int64_t total;       // bytes
};

inline Layout layout(int world, int max_tokens, int hidden) {
  Layout L;
  const int64_t tiles = (hidden + kTileCols - 1) / kTileCols;
  const int fused_t = max_tokens < kFusedMaxTokens ? max_tokens : kFusedMaxTokens;
  L.fused_floats = tiles * kTileCols * fused_t;
  const int64_t n = static_cast<int64_t>(max_tokens) * hidden;
  int64_t chunk = (n + world - 1) / world;
  chunk = (chunk + 63) / 64 * 64;
  L.ar_chunk = chunk;
  L.fused_off = 0;
  L.ar_off = L.fused_off + 2LL * world * L.fused_floats * 4;
  L.flags_off = L.ar_off + 4LL * world * L.ar_chunk * 4;
  L.total = L.flags_off + kFlagWords * 4;
  L.total = (L.total + 255) / 256 * 256;
  return L;
}

// Device view handed to kernels (by value).
struct DevComm {
  char* const* peers;
  int* status;
  uint32_t* epoch_dev;
  unsigned int* done;
  int rank;
  int world;
  uint64_t timeout_ns;
  int64_t fused_floats;
  int64_t ar_chunk;
  int64_t ar_off;
  int64_t flags_off;
};

__device__ __forceinline__ float* fused_slot(const DevComm& c, int peer, int slot, int src) {
  return reinterpret_cast<float*>(c.peers[peer]) + (static_cast<int64_t>(slot) * c.world + src) * c.fused_floats;
}
__device__ __forceinline__ uint32_t* fused_flag(const DevComm& c, int peer, int slot, int src, int tile) {
  uint32_t* f = reinterpret_cast<uint32_t*>(c.peers[peer] + c.flags_off);
  return f + (static_cast<int64_t>(slot) * kMaxWorld + src) * kMaxTiles + tile;
}
__device__ __forceinline__ float* ar_slot(const DevComm& c, int peer, int slot, int phase, int src) {
  float* base = reinterpret_cast<float*>(c.peers[peer] + c.ar_off);
  return base + ((static_cast<int64_t>(slot) * 2 + phase) * c.world + src) * c.ar_chunk;
}
__device__ __forceinline__ uint32_t* ar_flag(const DevComm& c, int peer, int slot, int phase, int src, int cta) {
  uint32_t* f = reinterpret_cast<uint32_t*>(c.peers[peer] + c.flags_off) + kFusedFlagWords;
  return f + ((static_cast<int64_t>(slot) * 2 + phase) * kMaxWorld + src) * kArMaxCtas + cta;
}

// Epoch of the collective a CTA is part of (read once at kernel start).
__device__ __forceinline__ uint32_t epoch_begin(const DevComm& c) {
  return *reinterpret_cast<volatile uint32_t*>(c.epoch_dev) + 1u;
}

// Called by every CTA once it is done with the collective: the last one to arrive
// resets the arrival counter and publishes the epoch for the next collective.
__device__ __forceinline__ void epoch_end(const DevComm& c, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(c.done, 1u);
    if (prev == gridDim.x - 1) {
      *reinterpret_cast<volatile unsigned int*>(c.done) = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(c.epoch_dev) = epoch;
    }
  }
}

inline DevComm device_view(pyre_comm* c) {
  DevComm d;
  d.peers = c->d_peers;
  d.status = c->d_status;
  d.epoch_dev = c->d_epoch;
  d.done = c->d_done;
  d.rank = c->rank;
  d.world = c->world;
  d.timeout_ns = c->timeout_ns;
  const Layout L = layout(c->world, c->max_tokens, c->hidden);
  d.fused_floats = L.fused_floats;
  d.ar_chunk = L.ar_chunk;
  d.ar_off = L.ar_off;
  d.flags_off = L.flags_off;
  return d;
}

}  // namespace comm

// Launches the two-shot all-reduce of n floats of buf over comm.
int allreduce_sum_f32(pyre_comm* comm, float* buf, int64_t n, cudaStream_t stream);
// Launches the cross-rank maximum of T orderable argmax keys (token[t] = its index).
int argmax_combine(pyre_comm* comm, const long long* key, int T, int* token, long long* key_out,
                   cudaStream_t stream);

}  // namespace pyre
