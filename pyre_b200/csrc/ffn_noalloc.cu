// pyre_ffn_decode_q80_noalloc: the one-launch decode FFN with its scratch in a static device
// array, for callers that cannot allocate device memory.
//
// Who needs it. pyre_ffn_decode_q80 wants a caller-allocated, zero-initialised workspace.
// Some callers have no way to provide one: a host program that binds only this C ABI (a
// Go, Java or ctypes caller with no CUDA allocator of its own), or a serving runtime whose
// device memory is entirely handed to its own pool, where a cudaMalloc either fails or
// blocks the whole device (it synchronises) in the middle of serving. This entry point takes
// the same inputs and outputs but keeps its scratch in g_decode_scratch below, so it calls
// no cudaMalloc, cudaFree or any other allocating routine.
//
// Rules that follow from a static array:
//   - Every GPU that loads this library holds kNoAllocScratchBytes of device memory for the
//     array until the process exits.
//   - The first call on a device looks up the array's device address on that device
//     (cudaGetSymbolAddress, with that device current) and caches it; make that first call
//     before any stream capture.
//   - All calls on one device share the array and it keeps the last call's contents. Every
//     call therefore clears the parts that must start at zero (counters, flags, slab
//     accumulators) with cudaMemsetAsync on the call's stream before the launch, after all
//     of its argument checks have passed (a rejected call queues nothing).
//   - The kernel's status word (PYRE_ERANGE for a partial sum that is not finite or too
//     large, PYRE_ETIMEOUT for a bounded wait that ran out) is NOT cleared by the calls: it
//     keeps the first problem since it was last read. pyre_ffn_decode_q80_noalloc_status()
//     synchronises the stream, returns the word and clears it.
//   - Calls that overlap on the GPU (different streams, or host threads without ordering)
//     race on the array and give wrong results; serialise them on one stream.
//   - Single GPU only (no tensor-parallel reduce: a communicator needs allocated buffers).
#include <mutex>
#include <string>

#include "ffn_internal.cuh"

namespace pyre {
namespace {

constexpr int kMaxDevices = 64;

// The scratch itself. In host code this name is only a stand-in for the symbol; the device
// address on the current device comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_decode_scratch[PYRE_NOALLOC_SCRATCH_BYTES];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (looked up once per device).
int scratch_on_current_device(void** out) {
  int dev = 0;
  PYRE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(PYRE_EINVAL, "pyre_ffn_decode_q80_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return cuda_status(e, "pyre_ffn_decode_q80_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PYRE_OK;
}

}  // namespace
}  // namespace pyre

extern "C" int pyre_ffn_decode_q80_noalloc(const void* x, int x_dtype, int T, int H, const void* wgu, int gated,
                                           const void* wd, int scale_dtype, int W, float* out, void* stream) {
  using namespace pyre;
  PYRE_CHECK_ARG(T >= 1 && T <= PYRE_FUSED_REDUCE_MAX_T,
                 "pyre_ffn_decode_q80_noalloc: T must be in [1, PYRE_FUSED_REDUCE_MAX_T]");
  PYRE_CHECK_ARG(H >= 1 && W >= 1, "pyre_ffn_decode_q80_noalloc: sizes must be positive");
  int64_t need = 0;
  int rc = pyre_ffn_workspace_bytes(T, H, W, &need);
  if (rc) return rc;
  if (need > PYRE_NOALLOC_SCRATCH_BYTES)
    return set_error(PYRE_EINVAL, "pyre_ffn_decode_q80_noalloc: T=" + std::to_string(T) + ", H=" +
                                      std::to_string(H) + ", W=" + std::to_string(W) + " need " +
                                      std::to_string(need) + " bytes of scratch, more than the built-in " +
                                      std::to_string(PYRE_NOALLOC_SCRATCH_BYTES) +
                                      " (use pyre_ffn_decode_q80 with a workspace)");
  void* scratch = nullptr;
  rc = scratch_on_current_device(&scratch);
  if (rc) return rc;
  // every check the launch will make, before the shared array is touched
  rc = ffn_decode_check(x, x_dtype, T, H, wgu, gated, wd, scale_dtype, W, out, scratch, need, nullptr,
                        "pyre_ffn_decode_q80_noalloc");
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // zeros everywhere but the status word (kept until read) and the h rows (plain data, but
  // clearing them with the rest is one memset either way)
  char* sc = static_cast<char*>(scratch);
  constexpr int64_t kStatusEnd = gemv::kHdrStatus + 4;
  PYRE_CUDA_TRY(cudaMemsetAsync(sc, 0, static_cast<size_t>(gemv::kHdrStatus), s));
  PYRE_CUDA_TRY(cudaMemsetAsync(sc + kStatusEnd, 0, static_cast<size_t>(need - kStatusEnd), s));
  return pyre_ffn_decode_q80(x, x_dtype, T, H, wgu, gated, wd, scale_dtype, W, out, scratch, need, nullptr, stream);
}

extern "C" int pyre_ffn_decode_q80_noalloc_status(int* status, void* stream) {
  using namespace pyre;
  PYRE_CHECK_ARG(status != nullptr, "pyre_ffn_decode_q80_noalloc_status: null status");
  void* scratch = nullptr;
  int rc = scratch_on_current_device(&scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* word = reinterpret_cast<int*>(static_cast<char*>(scratch) + gemv::kHdrStatus);
  int h = 0;
  PYRE_CUDA_TRY(cudaStreamSynchronize(s));
  PYRE_CUDA_TRY(cudaMemcpy(&h, word, sizeof(int), cudaMemcpyDeviceToHost));
  PYRE_CUDA_TRY(cudaMemset(word, 0, sizeof(int)));
  *status = h;
  return PYRE_OK;
}
