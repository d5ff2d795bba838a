// Status / error plumbing shared by every entry point of libi8moe.
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"

namespace i8moe {

namespace {
thread_local std::string g_last_error;
std::mutex g_sm_mu;
int g_sm_count[64] = {0};
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return set_error(I8MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return I8MOE_OK;
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int num_sms(int device) {
  if (device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> lk(g_sm_mu);
  if (g_sm_count[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[device] = n;
  }
  return g_sm_count[device];
}

// Per-translation-unit device error words (each .cu file owns one).
int read_route_error(uint32_t* w, int clear);
int read_quant_error(uint32_t* w, int clear);
int read_gemm_error(uint32_t* w, int clear);
int read_ep_error(uint32_t* w, int clear);
int read_peak_error(uint32_t* w, int clear);

}  // namespace i8moe

extern "C" {

int i8moe_abi_version(void) { return 1; }

const char* i8moe_last_error(void) { return i8moe::g_last_error.c_str(); }

int i8moe_device_error(int device, uint32_t* word, int clear) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return i8moe::set_error(I8MOE_ERR_CUDA, "cudaGetDevice");
  if (cudaSetDevice(device) != cudaSuccess)
    return i8moe::set_error(I8MOE_ERR_CUDA, "cudaSetDevice failed");
  uint32_t a = 0, b = 0, c = 0;
  int rc = i8moe::read_route_error(&a, clear);
  if (rc == I8MOE_OK) rc = i8moe::read_quant_error(&b, clear);
  if (rc == I8MOE_OK) rc = i8moe::read_gemm_error(&c, clear);
  uint32_t d = 0, e = 0;
  if (rc == I8MOE_OK) rc = i8moe::read_ep_error(&d, clear);
  if (rc == I8MOE_OK) rc = i8moe::read_peak_error(&e, clear);
  cudaSetDevice(prev);
  if (word) *word = a | b | c | d | e;
  return rc;
}

int i8moe_moe_permute_unpermute_supported(void) { return CUDART_VERSION >= 12000 ? 1 : 0; }

}  // extern "C"
