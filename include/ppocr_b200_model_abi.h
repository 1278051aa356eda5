// Model ABI v2 of the B200 layer path: one shared library per compiled shape
// (model_<name>.so), loadable unchanged by the reference's catalog loader
// (native/src/engine/model_engine_compiled.cpp:43-75, which dlsyms exactly the
// seven functions below and validates PpocrModelInfo).
//
// Structs and functions replace, with identical layout, names, arguments,
// ownership and error behaviour, the reference header
// native/include/ppocrv6_native/compiled/model_abi.h:11-38:
//   - device input is NCHW float32 [batch <= input_shape[0]]; unused batch
//     rows are treated as zero images;
//   - output is contiguous FP16 recognition features (element bytes 2) or
//     float32 detector probabilities (element bytes 4);
//   - calls enqueue work on the supplied stream and join it with events;
//     the first enqueue runs eagerly, then captures a CUDA graph;
//   - failures return nullptr / -1 and leave a thread-local message for
//     ppocr_model_error(); a failed enqueue synchronizes its stream first.
// Handles are not reentrant (one stream per handle).
#pragma once
#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#define PPOCR_MODEL_ABI_VERSION 2

// model_abi.h:12-20
struct PpocrModelInfo {
  uint32_t abi_version;
  int input_shape[4];
  int output_rank;
  int output_shape[4];
  int output_element_bytes;
  size_t weight_file_bytes;
  size_t scratch_bytes;
};
// model_abi.h:22-24. `blas` is kept for layout compatibility; the B200 path
// creates no library handles, so it stays null.
struct PpocrModelResources {
  void *blas;
};

#ifdef __cplusplus
extern "C" {
#endif
// model_abi.h:26 -- static shape/size metadata of this compiled shape.
const struct PpocrModelInfo *ppocr_model_info(void);
// model_abi.h:28 -- reads raw little-endian FP32 weights (export.py layout,
// exact size) and returns a device FP16 copy; release with cudaFree.
void *ppocr_model_load_weights(const char *weights_path);
// model_abi.h:31-32 -- borrows weights and scratch (scratch_bytes or more);
// recreate the handle if the scratch address changes.
void *ppocr_model_create(void *weights, void *scratch, size_t scratch_bytes,
                         struct PpocrModelResources *resources);
// model_abi.h:33
void ppocr_model_release_resources(struct PpocrModelResources *resources);
// model_abi.h:34-35 -- asynchronous forward pass of `batch` images.
int ppocr_model_enqueue(void *handle, const float *device_input,
                        void *device_output, int batch, cudaStream_t stream);
// model_abi.h:36 -- waits for the handle's work, then frees it.
void ppocr_model_destroy(void *handle);
// model_abi.h:37 -- message of the last failure on this thread ("" if none).
const char *ppocr_model_error(void);

// ---- extensions (no counterpart in model_abi.h; the reference loader never
// looks them up, so they do not affect drop-in loading)
// Same as ppocr_model_enqueue, but the device input is FP16 NHWC
// [batch][H][W][3] (the BASELINE benchmark layout).
int ppocr_model_enqueue_nhwc_f16(void *handle, const void *device_input,
                                 void *device_output, int batch,
                                 cudaStream_t stream);
// Number of launch-list entries of a created handle, their kind names, and
// one eager timing pass (milliseconds per entry, CUDA events on the handle's
// stream). Return -1 on error.
int ppocr_model_op_count(void *handle);
const char *ppocr_model_op_name(void *handle, int index);
int ppocr_model_profile_ops(void *handle, float *ms, int count);
#ifdef __cplusplus
}
#endif
