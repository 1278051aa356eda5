// Model ABI v2 shell (include/ppocr_b200_model_abi.h) around one generated
// graph. Compiled once per shape with -I<dir of model.inc>; links against
// libppocr_b200.so for the Runtime and its kernels.
//
// Behaviour follows the reference shell native/src/compiled/model_library.cu:
// weight loading and FP16 packing (100-129), storage checks (44-66), event
// join with the caller stream, input staging with a zero tail, eager first
// run then CUDA-graph capture and replay (67-96), error strings and the
// stream sync on a failed enqueue (150-176).
//
// Bounded waits: a kernel whose wait ran out sets the library's per-device
// error word and its outputs are invalid. The first (eager) run checks the
// word synchronously; every later enqueue copies the word into pinned host
// memory behind its graph launch, and the next enqueue of the handle fails
// with the code if that copy (already complete) saw one. Serving loops that
// must not wait for the next batch call ppocr_b200_device_error() after their
// stream sync.
#include "../../include/ppocr_b200_model_abi.h"
#include "kernels.h"
#include "runtime.h"
#include <fstream>
#include <memory>
#include <vector>

// The generated graph: kernels, size constants and build_model(Runtime&).
#include "model.inc"

#ifndef PPOCR_MODEL_DETECTOR
#define PPOCR_MODEL_DETECTOR 0
#endif
static_assert(half_storage, "model bundles use FP16 activation storage");

namespace {
thread_local std::string last_error;

constexpr size_t kArenaBytes = (ARENA_ELEMENTS * 2 + 255) & ~size_t(255);

struct Instance {
  Runtime r;
  cudaEvent_t ready = nullptr, done = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool warmed = false;
  int *error_seen = nullptr;     // host-mapped: the error word after the last replay
  int *error_seen_dev = nullptr; // its device address
  bool error_pending = false;

  ~Instance() {
    if (r.stream)
      cudaStreamSynchronize(r.stream);
    if (error_seen)
      cudaFreeHost(error_seen);
    if (exec)
      cudaGraphExecDestroy(exec);
    if (graph)
      cudaGraphDestroy(graph);
    if (ready)
      cudaEventDestroy(ready);
    if (done)
      cudaEventDestroy(done);
  }

  void init(void *weights, void *scratch, size_t bytes,
            PpocrModelResources *resources) {
    if (!resources || !weights || !scratch ||
        bytes < kArenaBytes + Runtime::workspace_limit)
      throw std::runtime_error("Invalid compiled model storage");
    r.weights = static_cast<half *>(weights);
    r.weight_elements = WEIGHT_ELEMENTS;
    r.arena = static_cast<half *>(scratch);
    r.workspace = static_cast<unsigned char *>(scratch) + kArenaBytes;
    r.workspace_bytes = Runtime::workspace_limit;
    build_model(r);
    r.reads({OUTPUT_ID}); // the output leaves through the ABI
    // Input staging writes the channels-last input directly when the graph
    // opens with the exporter's NCHW->NHWC transpose of tensor 0.
    if (r.input_nhwc_id >= 0)
      r.first_op = 1;
    // The per-device error word is allocated here, outside any capture.
    if (!pb2::device_error_word())
      throw std::runtime_error("Cannot allocate device error word");
    CU(cudaHostAlloc(&error_seen, sizeof(int), cudaHostAllocMapped));
    *error_seen = 0;
    CU(cudaHostGetDevicePointer(reinterpret_cast<void **>(&error_seen_dev), error_seen, 0));
    CU(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
    CU(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
  }

  void check_batch(const void *input, void *output, int batch) const {
    if (!input || !output || batch < 1 || batch > MODEL_INPUT_SHAPE[0])
      throw std::runtime_error("Invalid compiled model input/batch");
  }

  // Runs the graph on staged input. The first call runs the launch list
  // eagerly, captures it and then stages the input again: when staging
  // writes a tensor the arena reuses later in the graph (the channels-last
  // input of the fast path), the warm-up run has overwritten it.
  // Fails when the previous replay, now complete, saw a timed-out wait.
  void check_previous() {
    if (!error_pending || cudaEventQuery(done) != cudaSuccess)
      return;
    error_pending = false;
    if (const int code = *reinterpret_cast<volatile int *>(error_seen)) {
      *error_seen = 0;
      pb2::take_device_error(); // clear the word for the next batch
      throw std::runtime_error("kernel wait timed out in the previous batch (code " +
                               std::to_string(code) + "); its output is invalid");
    }
  }

  template <class Stage>
  void execute(const Stage &stage, void *output, int batch,
               cudaStream_t caller) {
    stage();
    if (!warmed) {
      r.run();
      CU(cudaStreamSynchronize(r.stream));
      if (int code = pb2::take_device_error())
        throw std::runtime_error("kernel wait timed out (code " +
                                 std::to_string(code) + ")");
      CU(cudaStreamBeginCapture(r.stream, cudaStreamCaptureModeThreadLocal));
      r.run();
      CU(cudaStreamEndCapture(r.stream, &graph));
      CU(cudaGraphInstantiate(&exec, graph, 0));
      warmed = true;
      stage();
    }
    CU(cudaGraphLaunch(exec, r.stream));
    // One kernel copies the output (widened to f32 for the detector) and
    // mirrors the error word into host-mapped memory for check_previous().
    const size_t output_n = OUTPUT_ELEMENTS / MODEL_INPUT_SHAPE[0] * batch;
    CU(pb2::output_copy(r.t[OUTPUT_ID], output, output_n, PPOCR_MODEL_DETECTOR != 0,
                        pb2::device_error_word(), error_seen_dev, r.stream));
    error_pending = true;
    CU(cudaGetLastError());
    CU(cudaEventRecord(done, r.stream));
    CU(cudaStreamWaitEvent(caller, done));
  }

  void enqueue_f32(const float *input, void *output, int batch,
                   cudaStream_t caller) {
    check_batch(input, output, batch);
    check_previous();
    CU(cudaEventRecord(ready, caller));
    CU(cudaStreamWaitEvent(r.stream, ready));
    auto stage = [&] {
      if (r.first_op == 1) {
        CU(pb2::nchw_f32_to_nhwc_f16(input, r.t[r.input_nhwc_id], batch,
                                     MODEL_INPUT_SHAPE[0], MODEL_INPUT_SHAPE[1],
                                     MODEL_INPUT_SHAPE[2], MODEL_INPUT_SHAPE[3],
                                     r.stream));
      } else {
        const size_t input_n = INPUT_ELEMENTS / MODEL_INPUT_SHAPE[0] * batch;
        CU(pb2::copy_input_f32(input, r.t[0], input_n, INPUT_ELEMENTS,
                               r.stream));
      }
    };
    execute(stage, output, batch, caller);
  }

  void enqueue_nhwc(const void *input, void *output, int batch,
                    cudaStream_t caller) {
    check_batch(input, output, batch);
    check_previous();
    CU(cudaEventRecord(ready, caller));
    CU(cudaStreamWaitEvent(r.stream, ready));
    auto stage = [&] {
      if (r.first_op == 1) {
        // Already channels-last: copy the valid images, zero the rest.
        const size_t per_image = INPUT_ELEMENTS / MODEL_INPUT_SHAPE[0] * 2;
        CU(pb2::stage_bytes(input, r.t[r.input_nhwc_id], per_image * batch,
                            per_image * MODEL_INPUT_SHAPE[0], r.stream));
      } else {
        CU(pb2::copy_input_nhwc_f16(static_cast<const half *>(input), r.t[0],
                                    batch, MODEL_INPUT_SHAPE[0],
                                    MODEL_INPUT_SHAPE[1], MODEL_INPUT_SHAPE[2],
                                    MODEL_INPUT_SHAPE[3], r.stream));
      }
    };
    execute(stage, output, batch, caller);
  }
};
} // namespace

#define API extern "C" __attribute__((visibility("default")))

API const PpocrModelInfo *ppocr_model_info() {
  static const PpocrModelInfo info = {
      PPOCR_MODEL_ABI_VERSION,
      {MODEL_INPUT_SHAPE[0], MODEL_INPUT_SHAPE[1], MODEL_INPUT_SHAPE[2],
       MODEL_INPUT_SHAPE[3]},
      MODEL_OUTPUT_RANK,
      {MODEL_OUTPUT_SHAPE[0], MODEL_OUTPUT_SHAPE[1], MODEL_OUTPUT_SHAPE[2],
       MODEL_OUTPUT_SHAPE[3]},
      PPOCR_MODEL_DETECTOR ? 4 : 2,
      WEIGHT_ELEMENTS * 4,
      kArenaBytes + Runtime::workspace_limit};
  return &info;
}

API void *ppocr_model_load_weights(const char *path) {
  void *device = nullptr;
  try {
    last_error.clear();
    if (!path)
      throw std::runtime_error("Null weights path");
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f || f.tellg() != std::streamoff(WEIGHT_ELEMENTS * 4))
      throw std::runtime_error("Invalid compiled model weight size");
    std::vector<float> host(WEIGHT_ELEMENTS);
    f.seekg(0);
    f.read(reinterpret_cast<char *>(host.data()), host.size() * 4);
    if (!f)
      throw std::runtime_error("Cannot read compiled model weights");
    std::vector<half> packed(WEIGHT_ELEMENTS);
    for (size_t i = 0; i < host.size(); ++i)
      packed[i] = __float2half_rn(host[i]);
    CU(cudaMalloc(&device, WEIGHT_ELEMENTS * 2));
    CU(cudaMemcpy(device, packed.data(), WEIGHT_ELEMENTS * 2,
                  cudaMemcpyHostToDevice));
    return device;
  } catch (const std::exception &e) {
    cudaFree(device);
    last_error = e.what();
    return nullptr;
  }
}

API void *ppocr_model_create(void *weights, void *scratch, size_t bytes,
                             PpocrModelResources *resources) {
  try {
    last_error.clear();
    // Validate borrowed storage before any device object is created.
    if (!resources || !weights || !scratch ||
        bytes < kArenaBytes + Runtime::workspace_limit)
      throw std::runtime_error("Invalid compiled model storage");
    auto p = std::make_unique<Instance>();
    p->init(weights, scratch, bytes, resources);
    return p.release();
  } catch (const std::exception &e) {
    last_error = e.what();
    return nullptr;
  }
}

template <class F> static int guarded(void *handle, F &&f) {
  try {
    last_error.clear();
    if (!handle)
      throw std::runtime_error("Null model handle");
    f(*static_cast<Instance *>(handle));
    return 0;
  } catch (const std::exception &e) {
    // Work may have been submitted without `done` being recorded; keep the
    // borrowed scratch exclusive until it has finished.
    if (handle)
      cudaStreamSynchronize(static_cast<Instance *>(handle)->r.stream);
    last_error = e.what();
    return -1;
  }
}

API int ppocr_model_enqueue(void *handle, const float *input, void *output,
                            int batch, cudaStream_t stream) {
  return guarded(handle, [&](Instance &i) {
    i.enqueue_f32(input, output, batch, stream);
  });
}

API int ppocr_model_enqueue_nhwc_f16(void *handle, const void *input,
                                     void *output, int batch,
                                     cudaStream_t stream) {
  return guarded(handle, [&](Instance &i) {
    i.enqueue_nhwc(input, output, batch, stream);
  });
}

API void ppocr_model_release_resources(PpocrModelResources *resources) {
  if (resources)
    resources->blas = nullptr;
}

API void ppocr_model_destroy(void *handle) {
  delete static_cast<Instance *>(handle);
}

API const char *ppocr_model_error() { return last_error.c_str(); }

API int ppocr_model_op_count(void *handle) {
  if (!handle)
    return -1;
  return static_cast<int>(static_cast<Instance *>(handle)->r.ops.size());
}

API const char *ppocr_model_op_name(void *handle, int index) {
  if (!handle)
    return "";
  auto &r = static_cast<Instance *>(handle)->r;
  if (index < 0 || index >= static_cast<int>(r.ops.size()))
    return "";
  if (index >= static_cast<int>(r.op_names.size()) || r.op_names[index].empty())
    return "generated";
  return r.op_names[index].c_str();
}

API int ppocr_model_profile_ops(void *handle, float *ms, int n) {
  return guarded(handle, [&](Instance &i) {
    auto &r = i.r;
    if (!r.prepared) {
      for (auto &p : r.prepare)
        p();
      r.prepared = true;
    }
    const int count = static_cast<int>(r.ops.size());
    std::vector<cudaEvent_t> ev(count + 1);
    for (auto &e : ev)
      CU(cudaEventCreate(&e));
    CU(cudaEventRecord(ev[0], r.stream));
    // Entries before first_op are replaced by input staging: reported as 0.
    for (int k = 0; k < count; ++k) {
      if (k >= r.first_op)
        r.ops[k]();
      CU(cudaEventRecord(ev[k + 1], r.stream));
    }
    CU(cudaStreamSynchronize(r.stream));
    for (int k = 0; k < count && k < n; ++k)
      CU(cudaEventElapsedTime(&ms[k], ev[k], ev[k + 1]));
    for (auto &e : ev)
      cudaEventDestroy(e);
  });
}
