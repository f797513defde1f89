// Library-wide C ABI pieces: version, per-thread error text, device queries.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace pyre {

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PYRE_OK;
  return set_error(PYRE_ECUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                   cudaGetErrorString(e) + ")");
}

int sm_count() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("PYRE_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

int set_smem_limit(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  PYRE_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return PYRE_OK;
  PYRE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert({kernel, dev});
  return PYRE_OK;
}

}  // namespace pyre

extern "C" int pyre_version(void) { return 100; }

extern "C" int pyre_last_error(char* buf, int len) {
  const std::string& s = pyre::g_last_error;
  if (buf != nullptr && len > 0) {
    const size_t n = s.size() < static_cast<size_t>(len - 1) ? s.size() : static_cast<size_t>(len - 1);
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
  return static_cast<int>(s.size());
}

extern "C" int pyre_graph_run(void* exec, void* stream, const void* src, void* stage_in, int64_t in_bytes) {
  PYRE_CHECK_ARG(exec != nullptr, "pyre_graph_run: null graph");
  PYRE_CHECK_ARG(in_bytes >= 0 && (in_bytes == 0 || (src != nullptr && stage_in != nullptr)),
                 "pyre_graph_run: bad input copy");
  if (in_bytes > 0) std::memcpy(stage_in, src, static_cast<size_t>(in_bytes));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PYRE_CUDA_TRY(cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), s));
  PYRE_CUDA_TRY(cudaStreamSynchronize(s));
  return PYRE_OK;
}
