// pkv_abi.cu — library-wide host plumbing: version, per-thread error text,
// pool validation, device properties.
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "pkv_common.cuh"

namespace pkv {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return PKV_ERR_CUDA;
}

int check_pool(const pkv_pool* p) {
  if (!p) return fail(PKV_ERR_ARG, "pool descriptor is NULL");
  if (!p->base) return fail(PKV_ERR_ARG, "pool base pointer is NULL");
  if (p->num_blocks <= 0 || p->num_layers <= 0 || p->block_size <= 0 || p->n_kv_heads <= 0 ||
      p->head_dim <= 0)
    return fail(PKV_ERR_ARG, "pool geometry must be positive (num_blocks, num_layers, "
                             "block_size, n_kv_heads, head_dim)");
  if (elem_size(p->dtype) == 0) return fail(PKV_ERR_ARG, "unknown pool dtype code");
  if ((reinterpret_cast<uintptr_t>(p->base) & 15) != 0)
    return fail(PKV_ERR_ARG, "pool base must be 16-byte aligned");
  if ((int64_t)p->num_blocks * p->block_size >= (int64_t(1) << 31))
    return fail(PKV_ERR_ARG, "num_blocks * block_size must fit in int32 slot ids");
  return PKV_OK;
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("PKV_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

}  // namespace pkv

extern "C" int pkv_version(void) { return 100; }

extern "C" const char* pkv_last_error(void) { return pkv::g_last_error.c_str(); }
