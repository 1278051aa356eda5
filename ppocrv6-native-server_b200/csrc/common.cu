// Per-device bookkeeping shared by all kernels: the error word written by
// kernels whose bounded waits ran out, and the SM count used to size
// persistent grids.
#include "kernels.h"
#include <mutex>

namespace pb2 {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int *g_error_words[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d < 0 || d >= kMaxDevices ? 0 : d;
}
} // namespace

int *device_error_word() {
  const int d = current_device();
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_error_words[d]) {
    int *p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess)
      return nullptr;
    cudaMemset(p, 0, sizeof(int));
    g_error_words[d] = p;
  }
  return g_error_words[d];
}

int take_device_error() {
  int *p = device_error_word();
  if (!p)
    return -1;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return -1;
  if (v)
    cudaMemset(p, 0, sizeof(int));
  return v;
}

int sm_count() {
  const int d = current_device();
  if (!g_sms[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 148;
  }
  return g_sms[d];
}

} // namespace pb2
