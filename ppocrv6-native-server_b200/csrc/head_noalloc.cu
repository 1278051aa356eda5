// Allocation-free variant of the packed vocabulary projection + argmax
// (ppocr_b200_classifier_run_packed_noalloc in include/ppocr_b200_head.h).
//
// Who needs it: hosts that must not call cudaMalloc on the serving path --
// for example a process whose device memory is entirely handed to its own
// pool allocator (a cudaMalloc would fail or fragment that pool), or a
// latency-bound request loop where an allocation would stall the device.
// The regular entry point needs three caller-provided partial buffers; this
// one keeps them in a fixed, file-scope device array instead.
//
// The scratch array below is static device memory of this library: every
// GPU that loads the library holds it (kScratchBytes, about 24 MB) until the
// process exits. All calls on a device share it and it keeps the contents of
// the last call, so calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on it. Every partial the merge
// reads is written earlier in the same call, so nothing needs clearing
// between calls. The first word of the array is this path's wait-timeout
// word: the projection kernel writes a nonzero code there when one of its
// bounded waits runs out (its outputs are then invalid). It is zeroed at
// set-up, and ppocr_b200_device_error() reads and clears it together with
// the library's other error word.
//
// Set-up happens inside the first call on each device (address lookup of
// the array plus a synchronous clear of its first 256 bytes), so make that
// first call before any stream capture on the device. A set-up that failed
// is retried by the next call.
#include "../../include/ppocr_b200_head.h"
#include "kernels.h"
#include <mutex>
#include <string>

namespace {

// Partials are (max, id, sum) per (vocabulary tile of 256, row).
constexpr size_t kMaxPartials = size_t(1) << 21; // rows * ceil(V/256) limit
constexpr size_t kHeaderBytes = 256;              // error word + padding
constexpr size_t kArrayBytes = kMaxPartials * 4;
constexpr size_t kScratchBytes = kHeaderBytes + 3 * kArrayBytes;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup;
unsigned char *g_base[kMaxDevices] = {}; // set once a device's set-up succeeded

// In host code `g_scratch` names a host-side shadow, not device memory: the
// device address is looked up per device, with that device current. A
// failed look-up or clear leaves the entry empty, so the next call retries.
unsigned char *device_scratch(cudaError_t *status) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *status = e;
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    *status = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup);
  if (!g_base[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    // Clear the timeout word (the partials need no clearing).
    if (e == cudaSuccess)
      e = cudaMemset(p, 0, kHeaderBytes);
    if (e != cudaSuccess) {
      *status = e;
      return nullptr;
    }
    g_base[dev] = static_cast<unsigned char *>(p);
  }
  *status = cudaSuccess;
  return g_base[dev];
}

// The current device's timeout word, or null when this path has not been
// set up on it (then no kernel of this path can have written it).
int *set_up_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return nullptr;
  std::lock_guard<std::mutex> lock(g_setup);
  return reinterpret_cast<int *>(g_base[dev]);
}

} // namespace

namespace pb2 {
// Reads and clears the allocation-free path's timeout word on the current
// device (0 when clear or never set up; -1 when the read failed). Used by
// ppocr_b200_device_error().
int take_noalloc_error() {
  int *word = set_up_error_word();
  if (!word)
    return 0;
  int v = 0;
  if (cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return -1;
  if (v && cudaMemset(word, 0, sizeof(int)) != cudaSuccess)
    return -1;
  return v;
}
} // namespace pb2

namespace pb2 {
// Test support for ppocr_b200_test_store_error_code: writes `code` into the
// current device's timeout word of this path, as a kernel whose wait ran out
// would. Sets the path up on the device if needed; allocates nothing.
cudaError_t store_noalloc_error(int code) {
  cudaError_t status;
  unsigned char *base = device_scratch(&status);
  if (!base)
    return status;
  return cudaMemcpy(base, &code, sizeof(int), cudaMemcpyHostToDevice);
}
} // namespace pb2

extern "C" int ppocr_b200_classifier_run_packed_noalloc(
    const void *hidden, const void *packed, const void *bias, int *ids,
    float *prob, float *max_logits, int rows, int hidden_size, int vocab,
    int calc_prob, cudaStream_t stream) {
  if (rows <= 0)
    return 0;
  pb2::set_last_error("");
  if (!hidden || !packed || !bias || !ids || !prob || !max_logits ||
      hidden_size <= 0 || hidden_size % 8 || vocab <= 0) {
    pb2::set_last_error("invalid classifier launch arguments");
    return -1;
  }
  const size_t tiles = static_cast<size_t>(pb2::vocab_tiles(vocab));
  if (static_cast<size_t>(rows) * tiles > kMaxPartials) {
    pb2::set_last_error("rows * ceil(vocab/256) = " +
                        std::to_string(static_cast<size_t>(rows) * tiles) +
                        " exceeds the allocation-free scratch limit of " +
                        std::to_string(kMaxPartials) + " partials");
    return -1;
  }
  cudaError_t status;
  unsigned char *base = device_scratch(&status);
  if (!base) {
    pb2::set_last_error(
        std::string("cannot resolve the static scratch array: ") +
        cudaGetErrorString(status));
    return -1;
  }
  int *err_word = reinterpret_cast<int *>(base);
  float *part_max = reinterpret_cast<float *>(base + kHeaderBytes);
  int *part_id = reinterpret_cast<int *>(base + kHeaderBytes + kArrayBytes);
  float *part_sum =
      reinterpret_cast<float *>(base + kHeaderBytes + 2 * kArrayBytes);
  cudaError_t e = pb2::tc_vocab_partials(
      static_cast<const half *>(hidden), rows, hidden_size,
      static_cast<const half *>(packed), static_cast<const half *>(bias),
      vocab, part_max, part_id, part_sum, calc_prob, stream, err_word);
  if (e == cudaSuccess)
    e = pb2::vocab_merge(part_max, part_id, part_sum, rows,
                         static_cast<int>(tiles), ids, prob, max_logits,
                         calc_prob, stream);
  if (e != cudaSuccess) {
    pb2::set_last_error(std::string("vocab projection: ") +
                        cudaGetErrorString(e));
    return -1;
  }
  return 0;
}
