// Library-wide C-ABI helpers: version, device status word, last CUDA error.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace hcu {

static thread_local char t_last_error[256] = "";

void set_last_error(cudaError_t e) {
  if (e == cudaSuccess) return;
  std::snprintf(t_last_error, sizeof(t_last_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
}

void set_last_error_msg(const char* a, const char* b) {
  std::snprintf(t_last_error, sizeof(t_last_error), "%s%s", a, b);
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(e);
    return HCU_ERR_LAUNCH;
  }
  return HCU_OK;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace hcu

extern "C" const char* hcu_version(void) { return "hcu_indexer 0.1 sm_100a"; }

extern "C" const char* hcu_last_error_string(void) { return hcu::t_last_error; }

extern "C" int hcu_read_device_status(uint32_t* status, int clear) {
  if (!status) return HCU_ERR_ARG;
  *status = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = hcu::status_dequant(status, clear);
  if (e == cudaSuccess) e = hcu::status_topk(status, clear);
  if (e == cudaSuccess) e = hcu::status_logits(status, clear);
  if (e == cudaSuccess) e = hcu::status_mla(status, clear);
  if (e != cudaSuccess) {
    hcu::set_last_error(e);
    return HCU_ERR_LAUNCH;
  }
  return HCU_OK;
}

extern "C" int hcu_set_wait_limit_ns(uint64_t ns) {
  if (ns == 0) ns = hcu::kWaitLimitNs;
  cudaError_t e = hcu::status_dequant_set_wait_limit(ns);
  if (e == cudaSuccess) e = hcu::status_topk_set_wait_limit(ns);
  if (e == cudaSuccess) e = hcu::status_logits_set_wait_limit(ns);
  if (e == cudaSuccess) e = hcu::status_mla_set_wait_limit(ns);
  if (e != cudaSuccess) {
    hcu::set_last_error(e);
    return HCU_ERR_LAUNCH;
  }
  return HCU_OK;
}
