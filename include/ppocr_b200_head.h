// CTC head of the B200 layer path (libppocr_b200.so): vocabulary projection
// with fused argmax / softmax-max, argmax over FP16 logits, the greedy CTC
// collapse on device, and the selected-class probability.
//
// Every function returns 0 on success and -1 on failure; the message of the
// last failure on the calling thread is ppocr_b200_last_error(). Argument
// checks mirror the reference's std::invalid_argument cases. Pointers are
// device pointers unless stated; work is enqueued on `stream`.
#pragma once
#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char *ppocr_b200_last_error(void);
// Reads and clears the current device's error words that kernels set when
// one of their bounded waits ran out (0 = no error; the outputs of the work
// enqueued since the last call are then invalid). Covers every kernel of the
// library, the allocation-free head's own word included. Synchronizes the
// device; a serving loop calls it after its stream sync and fails the batch
// on a nonzero code.
int ppocr_b200_device_error(void);
// Test support, no counterpart in the reference: stores `code` in one of the
// current device's error words, as a kernel whose bounded wait ran out would
// (which = 0: the library-wide word; 1: the allocation-free head's word), so
// tests can check how ppocr_b200_device_error() and the model shells report
// it. The library-wide word is allocated on first use; nothing else is.
int ppocr_b200_test_store_error_code(int which, int code);

// Replaces tiled_classifier_workspace_shape
// (native/include/ppocrv6_native/kernels/classifier.h:16-17,
// classifier.cu:520-536), with the same results: num_row_blocks =
// ceil(rows/row_block_size), num_vocab_blocks = ceil(vocab/vocab_tile_size),
// partial_count = num_row_blocks * num_vocab_blocks * row_block_size.
int ppocr_b200_classifier_workspace(int rows, int vocab_size,
                                    int row_block_size, int vocab_tile_size,
                                    int *num_row_blocks, int *num_vocab_blocks,
                                    size_t *partial_count);

// Replaces cuda_linear_argmax_prob_wmma_mode (classifier.h:38-43,
// classifier.cu:611-659). hidden FP16 [rows][hidden_size], weight FP16
// [hidden_size][vocab_size] (row-major, as the reference loads it), bias FP16
// [vocab_size]. Outputs per row: argmax id (ties -> lowest id), 1/sum
// exp(l - max) (1.0 when calculate_probability is 0) and the max logit.
// partial_* are sized as the reference sizes them for this vocab_tile_size
// (ppocr_b200_classifier_workspace with row_block_size 16). The B200 kernel
// reduces 256-column vocabulary tiles whatever vocab_tile_size says; when the
// caller's partial buffers are too small for that, it uses a workspace of the
// calling stream instead. The weight is transposed per call into that
// per-(device, stream) workspace (allocated stream-ordered on first use and
// grown the same way; callers on different streams never share it), so each
// call depends only on its own arguments. Callers that keep the weight
// resident use ppocr_b200_classifier_pack/_run_packed instead.
int ppocr_b200_linear_argmax_prob(
    const void *hidden, const void *weight, const void *bias, int *out_indices,
    float *out_prob, float *out_max_logits, int rows, int hidden_size,
    int vocab_size, int vocab_tile_size, int *partial_ids, float *partial_max,
    float *partial_sum, int calculate_probability, cudaStream_t stream);

// Extension: one-time transpose of weight [hidden][vocab] into the K-major
// [vocab][hidden] layout the tensor-core projection reads (packed must hold
// vocab*hidden FP16 values, 16-byte aligned).
int ppocr_b200_classifier_pack(const void *weight, void *packed,
                               int hidden_size, int vocab_size,
                               cudaStream_t stream);
// Extension: projection + argmax with a packed weight. partial_* need
// rows * ceil(vocab/256) entries each.
int ppocr_b200_classifier_run_packed(
    const void *hidden, const void *packed, const void *bias, int *out_indices,
    float *out_prob, float *out_max_logits, int rows, int hidden_size,
    int vocab_size, int *partial_ids, float *partial_max, float *partial_sum,
    int calculate_probability, cudaStream_t stream);

// No counterpart in the reference. Allocation-free form of
// ppocr_b200_classifier_run_packed for callers that must not call cudaMalloc
// (their device memory is owned by their own pool allocator, or an
// allocation would stall a latency-bound request loop). Same arguments and
// results minus the partial buffers: the partials live in a file-scope
// device array of this library (about 24 MB per GPU that loads the library,
// held until the process exits). Limit: rows * ceil(vocab_size/256) must not
// exceed 2,097,152 (e.g. 29,127 rows at vocab 18,385); larger calls fail with
// a message. All calls on a device share the array, so calls whose kernels
// may overlap on the GPU race; order them on one stream. The first call on
// each device performs a one-time set-up (array lookup and a synchronous
// clear), so make it before any stream capture on that device; a failed
// set-up is retried by the next call. A projection whose bounded wait ran out
// writes its code into the array's own error word, which
// ppocr_b200_device_error() reads and clears like the library's other word.
int ppocr_b200_classifier_run_packed_noalloc(
    const void *hidden, const void *packed, const void *bias, int *out_indices,
    float *out_prob, float *out_max_logits, int rows, int hidden_size,
    int vocab_size, int calculate_probability, cudaStream_t stream);


// Replaces cuda_selected_class_vs_max_probability (classifier.h:45-49,
// classifier.cu:111-143): p(class) / (p(class) + p(max)) per row.
int ppocr_b200_selected_class_vs_max_probability(
    const void *hidden, const void *weight, const void *bias,
    const float *max_logits, float *out_probability, int rows,
    int hidden_size, int vocab_size, int class_id, cudaStream_t stream);

// Extension (the reference computes this inside the WMMA partial kernel,
// classifier.cu:456-515, from hidden states): argmax and softmax-max over
// FP16 logits [rows][vocab_size] that are already materialised.
int ppocr_b200_logits_argmax_prob(const void *logits, int rows, int vocab_size,
                                  int *out_indices, float *out_prob,
                                  float *out_max_logits,
                                  int calculate_probability,
                                  cudaStream_t stream);

// Replaces the index/score part of ctc_greedy_decode_batch
// (native/include/ppocrv6_native/recognition/ctc_decode.h:21-24,
// ctc_decode.cpp:7-81), on device: per line of `seq_len` ids, skip an id equal
// to the previous id, then skip `blank_id`; out_ids [lines][seq_len] holds
// the kept ids (-1 padded), out_len their count, out_score the float mean of
// the kept probabilities (0 when none; probabilities may be null = 1.0).
// Mapping ids to characters stays on the host.
int ppocr_b200_ctc_collapse(const int *indices, const float *probabilities,
                            int lines, int seq_len, int blank_id,
                            int *out_ids, int *out_len, float *out_score,
                            cudaStream_t stream);

#ifdef __cplusplus
}
#endif
