// C entry points over the reference's own vocabulary-projection kernels,
// compiled from native/src/kernels/classifier.cu where it lies into
// oracle/_ref/ by the Makefile beside this file. TEST INFRASTRUCTURE ONLY:
// run on the GPU box to pin the oracle's argmax/prob restatement.
#include "ppocrv6_native/kernels/classifier.h"

extern "C" int ref_classifier_workspace(int rows, int vocab, int row_block,
                                        int tile, size_t *partial_count) {
  try {
    auto s = ppocrv6_native::kernels::tiled_classifier_workspace_shape(
        rows, vocab, row_block, tile);
    *partial_count = s.partial_count;
    return 0;
  } catch (...) {
    return -1;
  }
}

extern "C" int ref_linear_argmax_prob_wmma(
    const void *hidden, const void *weight, const void *bias, int *ids,
    float *prob, float *max_logits, int rows, int hidden_size, int vocab,
    int tile, int *partial_ids, float *partial_max, float *partial_sum,
    int calc_prob, void *stream) {
  try {
    ppocrv6_native::kernels::cuda_linear_argmax_prob_wmma_mode(
        static_cast<const half *>(hidden), static_cast<const half *>(weight),
        static_cast<const half *>(bias), ids, prob, max_logits, rows,
        hidden_size, vocab, tile, partial_ids, partial_max, partial_sum,
        calc_prob != 0, static_cast<cudaStream_t>(stream));
    return 0;
  } catch (...) {
    return -1;
  }
}

extern "C" int ref_selected_class_vs_max(const void *hidden, const void *weight,
                                         const void *bias,
                                         const float *max_logits,
                                         float *out_probability, int rows,
                                         int hidden_size, int vocab,
                                         int class_id, void *stream) {
  try {
    ppocrv6_native::kernels::cuda_selected_class_vs_max_probability(
        static_cast<const half *>(hidden), static_cast<const half *>(weight),
        static_cast<const half *>(bias), max_logits, out_probability, rows,
        hidden_size, vocab, class_id, static_cast<cudaStream_t>(stream));
    return 0;
  } catch (...) {
    return -1;
  }
}
