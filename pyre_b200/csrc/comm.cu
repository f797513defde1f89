// Peer-memory communicator (one process per GPU, buffers shared with CUDA IPC) and the
// two-shot all-reduce used after the prefill down-projection.
//
// The reference gathers FFN partials at the root over TCP and sums them in worker order
// (src/orchestrator/root_node.py:582-594, :982-995). Here every rank sums the same
// partials in rank order 0..world-1, so all ranks hold bit-identical results.
#include <climits>
#include <vector>

#include "comm.cuh"

namespace pyre {
namespace {

using comm::DevComm;

// Two-shot all-reduce. CTA b owns the b-th slice of every rank's chunk. Phase 0: push
// slice b of chunk p to peer p. Phase 1: sum own chunk's slice over ranks (rank order),
// push the sum to every peer. Then copy the gathered sums back into buf. Each CTA only
// waits for the CTAs with the same index on other ranks, and the grid never exceeds one
// CTA per SM, so all waits are between co-resident CTAs. Every wait is bounded.
__global__ void __launch_bounds__(512) allreduce_two_shot_kernel(DevComm c, float* __restrict__ buf,
                                                                 int64_t n, int64_t chunk) {
  const uint32_t epoch = comm::epoch_begin(c);
  const int slot = epoch & 1u;
  const int b = blockIdx.x;
  const int64_t slice = (chunk + gridDim.x - 1) / gridDim.x;
  const int64_t s0 = b * slice;
  const int64_t s1 = s0 + slice < chunk ? s0 + slice : chunk;

  // phase 0: scatter
  for (int p = 0; p < c.world; ++p) {
    float* dst = comm::ar_slot(c, p, slot, 0, c.rank);
    const int64_t base = p * chunk;
    for (int64_t i = s0 + threadIdx.x; i < s1; i += blockDim.x) {
      const int64_t g = base + i;
      dst[i] = g < n ? buf[g] : 0.f;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < c.world)
    st_release_sys(comm::ar_flag(c, threadIdx.x, slot, 0, c.rank, b), epoch);
  if (threadIdx.x < c.world) {
    if (!wait_flag_eq(comm::ar_flag(c, c.rank, slot, 0, threadIdx.x, b), epoch, c.timeout_ns)) {
      atomicExch(c.status, PYRE_ETIMEOUT);
    }
  }
  __syncthreads();

  // phase 1: reduce own chunk slice, broadcast it
  for (int64_t i = s0 + threadIdx.x; i < s1; i += blockDim.x) {
    float acc = 0.f;
    for (int src = 0; src < c.world; ++src) acc += __ldcg(comm::ar_slot(c, c.rank, slot, 0, src) + i);
    for (int p = 0; p < c.world; ++p) comm::ar_slot(c, p, slot, 1, c.rank)[i] = acc;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < c.world)
    st_release_sys(comm::ar_flag(c, threadIdx.x, slot, 1, c.rank, b), epoch);
  if (threadIdx.x < c.world) {
    if (!wait_flag_eq(comm::ar_flag(c, c.rank, slot, 1, threadIdx.x, b), epoch, c.timeout_ns)) {
      atomicExch(c.status, PYRE_ETIMEOUT);
    }
  }
  __syncthreads();

  // gather back into buf
  for (int src = 0; src < c.world; ++src) {
    const float* g = comm::ar_slot(c, c.rank, slot, 1, src);
    const int64_t base = src * chunk;
    for (int64_t i = s0 + threadIdx.x; i < s1; i += blockDim.x) {
      const int64_t o = base + i;
      if (o < n) buf[o] = __ldcg(g + i);
    }
  }
  comm::epoch_end(c, epoch);
}

// Greedy token over a vocabulary split across the ranks: each rank holds the best
// (value, index) key of its vocabulary rows per token row (pyre_lm_head_argmax); the ranks
// exchange them through peer memory and every rank takes the maximum key, whose low half
// names the winning index (0xFFFFFFFF - low: equal values go to the lower index, as
// np.argmax over the whole vocabulary would). One CTA, every wait bounded.
__global__ void __launch_bounds__(32) key_max_kernel(DevComm c, const long long* __restrict__ key, int T,
                                                     int* __restrict__ token, long long* __restrict__ key_out) {
  const uint32_t epoch = comm::epoch_begin(c);
  const int slot = epoch & 1u;
  const int tid = threadIdx.x;
  for (int i = tid; i < c.world * T; i += 32) {
    const int peer = i / T, t = i - peer * T;
    reinterpret_cast<long long*>(comm::ar_slot(c, peer, slot, 0, c.rank))[t] = key[t];
  }
  __threadfence_system();
  __syncwarp();
  if (tid < c.world) st_release_sys(comm::ar_flag(c, tid, slot, 0, c.rank, 0), epoch);
  if (tid < c.world) {
    if (!wait_flag_eq(comm::ar_flag(c, c.rank, slot, 0, tid, 0), epoch, c.timeout_ns))
      atomicExch(c.status, PYRE_ETIMEOUT);
  }
  __syncwarp();
  if (tid < T) {
    long long best = LLONG_MIN;
    for (int src = 0; src < c.world; ++src) {
      const long long k = __ldcg(reinterpret_cast<const long long*>(comm::ar_slot(c, c.rank, slot, 0, src)) + tid);
      best = k > best ? k : best;
    }
    const unsigned long long u = static_cast<unsigned long long>(best) ^ 0x8000000000000000ull;
    token[tid] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(u & 0xFFFFFFFFull));
    if (key_out != nullptr) key_out[tid] = best;
  }
  comm::epoch_end(c, epoch);
}

}  // namespace

int argmax_combine(pyre_comm* c, const long long* key, int T, int* token, long long* key_out, cudaStream_t stream) {
  PYRE_CHECK_ARG(c != nullptr && key != nullptr && token != nullptr, "pyre_argmax_combine: null argument");
  PYRE_CHECK_ARG(T >= 1 && T <= PYRE_FUSED_REDUCE_MAX_T, "pyre_argmax_combine: 1 <= T <= PYRE_FUSED_REDUCE_MAX_T");
  PYRE_CHECK_ARG(2LL * T <= comm::layout(c->world, c->max_tokens, c->hidden).ar_chunk,
                 "pyre_argmax_combine: communicator buffer too small");
  key_max_kernel<<<1, 32, 0, stream>>>(comm::device_view(c), key, T, token, key_out);
  PYRE_LAUNCH_CHECK("key_max_kernel");
  return PYRE_OK;
}

int allreduce_sum_f32(pyre_comm* c, float* buf, int64_t n, cudaStream_t stream) {
  const comm::Layout L = comm::layout(c->world, c->max_tokens, c->hidden);
  PYRE_CHECK_ARG(n <= static_cast<int64_t>(c->max_tokens) * c->hidden,
                 "pyre_allreduce_sum_f32: n exceeds the communicator's max_tokens * hidden");
  if (n == 0) return PYRE_OK;
  if (c->world == 1) return PYRE_OK;
  int64_t chunk = (n + c->world - 1) / c->world;
  chunk = (chunk + 63) / 64 * 64;
  if (chunk > L.ar_chunk) chunk = L.ar_chunk;
  int grid = static_cast<int>((chunk + 2047) / 2048);
  const int cap = sm_count() < comm::kArMaxCtas ? sm_count() : comm::kArMaxCtas;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  allreduce_two_shot_kernel<<<grid, 512, 0, stream>>>(comm::device_view(c), buf, n, chunk);
  PYRE_LAUNCH_CHECK("allreduce_two_shot_kernel");
  return PYRE_OK;
}

}  // namespace pyre

using namespace pyre;

extern "C" int pyre_comm_buffer_bytes(int world, int max_tokens, int hidden, int64_t* bytes) {
  PYRE_CHECK_ARG(bytes != nullptr, "pyre_comm_buffer_bytes: null bytes");
  PYRE_CHECK_ARG(world >= 1 && world <= comm::kMaxWorld, "pyre_comm_buffer_bytes: world must be in [1, 16]");
  PYRE_CHECK_ARG(max_tokens >= 1 && hidden >= 1, "pyre_comm_buffer_bytes: sizes must be positive");
  PYRE_CHECK_ARG((hidden + comm::kTileCols - 1) / comm::kTileCols <= comm::kMaxTiles,
                 "pyre_comm_buffer_bytes: hidden too large");
  *bytes = comm::layout(world, max_tokens, hidden).total;
  return PYRE_OK;
}

extern "C" int pyre_comm_alloc(int64_t bytes, void** dev_ptr, void* ipc_handle_out) {
  PYRE_CHECK_ARG(bytes > 0 && dev_ptr != nullptr && ipc_handle_out != nullptr, "pyre_comm_alloc: bad argument");
  void* p = nullptr;
  PYRE_CUDA_TRY(cudaMalloc(&p, static_cast<size_t>(bytes)));
  cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "pyre_comm_alloc");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(ipc_handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return PYRE_OK;
}

extern "C" int pyre_comm_free(void* dev_ptr) {
  if (dev_ptr == nullptr) return PYRE_OK;
  PYRE_CUDA_TRY(cudaFree(dev_ptr));
  return PYRE_OK;
}

extern "C" int pyre_comm_open_peer(const void* ipc_handle, void** peer_ptr) {
  PYRE_CHECK_ARG(ipc_handle != nullptr && peer_ptr != nullptr, "pyre_comm_open_peer: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  PYRE_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *peer_ptr = p;
  return PYRE_OK;
}

extern "C" int pyre_comm_close_peer(void* peer_ptr) {
  if (peer_ptr == nullptr) return PYRE_OK;
  PYRE_CUDA_TRY(cudaIpcCloseMemHandle(peer_ptr));
  return PYRE_OK;
}

extern "C" int pyre_comm_create(int rank, int world, void* const* bufs, int max_tokens, int hidden,
                                pyre_comm_t** out) {
  PYRE_CHECK_ARG(out != nullptr && bufs != nullptr, "pyre_comm_create: null argument");
  PYRE_CHECK_ARG(world >= 1 && world <= comm::kMaxWorld, "pyre_comm_create: world must be in [1, 16]");
  PYRE_CHECK_ARG(rank >= 0 && rank < world, "pyre_comm_create: rank out of range");
  PYRE_CHECK_ARG(max_tokens >= 1 && hidden >= 1, "pyre_comm_create: sizes must be positive");
  PYRE_CHECK_ARG((hidden + comm::kTileCols - 1) / comm::kTileCols <= comm::kMaxTiles,
                 "pyre_comm_create: hidden too large");
  for (int r = 0; r < world; ++r) PYRE_CHECK_ARG(bufs[r] != nullptr, "pyre_comm_create: null peer buffer");
  pyre_comm* c = new pyre_comm();
  c->rank = rank;
  c->world = world;
  c->max_tokens = max_tokens;
  c->hidden = hidden;
  c->timeout_ns = 2000000000ull;
  c->d_peers = nullptr;
  c->d_status = nullptr;
  c->d_epoch = nullptr;
  c->d_done = nullptr;
  const comm::Layout L = comm::layout(world, max_tokens, hidden);
  c->fused_floats = L.fused_floats;
  c->ar_chunk = L.ar_chunk;
  c->local = static_cast<char*>(bufs[rank]);
  cudaError_t e = cudaMalloc(&c->d_peers, sizeof(char*) * world);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&c->d_epoch, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&c->d_done, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemcpy(c->d_peers, bufs, sizeof(char*) * world, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(c->d_status, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->d_epoch, 0, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(c->d_done, 0, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->d_peers) cudaFree(c->d_peers);
    if (c->d_status) cudaFree(c->d_status);
    if (c->d_epoch) cudaFree(c->d_epoch);
    if (c->d_done) cudaFree(c->d_done);
    delete c;
    return cuda_status(e, "pyre_comm_create");
  }
  *out = c;
  return PYRE_OK;
}

extern "C" int pyre_comm_destroy(pyre_comm_t* c) {
  if (c == nullptr) return PYRE_OK;
  cudaFree(c->d_peers);
  cudaFree(c->d_status);
  cudaFree(c->d_epoch);
  cudaFree(c->d_done);
  delete c;
  return PYRE_OK;
}

extern "C" int pyre_comm_set_timeout_ns(pyre_comm_t* c, uint64_t ns) {
  PYRE_CHECK_ARG(c != nullptr && ns > 0, "pyre_comm_set_timeout_ns: bad argument");
  c->timeout_ns = ns;
  return PYRE_OK;
}

extern "C" int pyre_comm_check(pyre_comm_t* c, int* status, void* stream) {
  PYRE_CHECK_ARG(c != nullptr && status != nullptr, "pyre_comm_check: null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int h = 0;
  PYRE_CUDA_TRY(cudaStreamSynchronize(s));
  PYRE_CUDA_TRY(cudaMemcpy(&h, c->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  PYRE_CUDA_TRY(cudaMemset(c->d_status, 0, sizeof(int)));
  *status = h;
  return PYRE_OK;
}

extern "C" int pyre_comm_reset(pyre_comm_t* c, void* stream) {
  PYRE_CHECK_ARG(c != nullptr, "pyre_comm_reset: null communicator");
  const comm::Layout L = comm::layout(c->world, c->max_tokens, c->hidden);
  PYRE_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  PYRE_CUDA_TRY(cudaMemset(c->local + L.flags_off, 0, static_cast<size_t>(comm::kFlagWords) * 4));
  PYRE_CUDA_TRY(cudaMemset(c->d_epoch, 0, sizeof(uint32_t)));
  PYRE_CUDA_TRY(cudaMemset(c->d_done, 0, sizeof(unsigned int)));
  PYRE_CUDA_TRY(cudaMemset(c->d_status, 0, sizeof(int)));
  PYRE_CUDA_TRY(cudaDeviceSynchronize());
  return PYRE_OK;
}

extern "C" int pyre_argmax_combine(pyre_comm_t* c, const long long* key, int T, int* token, long long* key_out,
                                   void* stream) {
  return argmax_combine(c, key, T, token, key_out, static_cast<cudaStream_t>(stream));
}

extern "C" int pyre_allreduce_sum_f32(pyre_comm_t* c, float* buf, int64_t n, void* stream) {
  PYRE_CHECK_ARG(c != nullptr && (buf != nullptr || n == 0) && n >= 0, "pyre_allreduce_sum_f32: bad argument");
  return allreduce_sum_f32(c, buf, n, static_cast<cudaStream_t>(stream));
}
