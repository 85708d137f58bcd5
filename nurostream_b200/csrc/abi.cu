// Error reporting, type layouts and device queries of the ns_b200 C ABI.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace ns {

static thread_local char t_msg[512] = "no error";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof t_msg, fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof t_msg, fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  set_error("%s failed: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return NS_ERR_CUDA;
}

int num_sms(int* out) {
  static int cache[64] = {0};
  int dev = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(NS_ERR_INVALID, "device ordinal %d out of range", dev);
  if (cache[dev] == 0) {
    int n = 0;
    NS_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    cache[dev] = n;
  }
  *out = cache[dev];
  return NS_OK;
}

}  // namespace ns

extern "C" {

const char* ns_last_error(void) { return ns::t_msg; }

int ns_abi_version(void) { return NS_ABI_VERSION; }

int ns_type_layout(int ggml_type, int* block_elems, int* block_bytes) {
  if (!block_elems || !block_bytes) return ns::fail(NS_ERR_INVALID, "ns_type_layout: null output");
  if (!ns::block_layout(ggml_type, block_elems, block_bytes))
    return ns::fail(NS_ERR_UNSUPPORTED, "ns_type_layout: unsupported ggml type %d", ggml_type);
  return NS_OK;
}

int ns_device_error(uint32_t* bits, int clear) {
  if (!bits) return ns::fail(NS_ERR_INVALID, "ns_device_error: null output");
  unsigned int v = 0;
  NS_CUDA_TRY(cudaDeviceSynchronize());
  NS_CUDA_TRY(cudaMemcpyFromSymbol(&v, ns::g_device_error, sizeof v));
  if (clear && v) {
    unsigned int z = 0;
    NS_CUDA_TRY(cudaMemcpyToSymbol(ns::g_device_error, &z, sizeof z));
  }
  *bits = v;
  return NS_OK;
}

}  // extern "C"
