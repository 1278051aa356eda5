/* Plain-C restatement of the CTC head on the host. TEST INFRASTRUCTURE ONLY
 * (oracle): used by tests/ as the checker and by bench.py as the timed CPU
 * baseline, never by the product path.
 *
 * oracle_argmax_prob  follows native/src/kernels/classifier.cu:456-515 and
 *                     270-368: per row, argmax with ties -> lowest id, max
 *                     logit, prob = 1 / sum exp(l - max) (double here).
 * oracle_ctc_collapse follows native/src/recognition/ctc_decode.cpp:7-51:
 *                     skip an id equal to the previous id (previous starts
 *                     at -1 and is updated for every id), then skip blank;
 *                     score = float running sum of kept probs / count
 *                     (0 when nothing is kept; probs NULL means 1.0 each).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      exp = 127 - 15 + 1;
      while (!(mant & 0x400)) {
        mant <<= 1;
        --exp;
      }
      mant &= 0x3ff;
      bits = sign | (exp << 23) | (mant << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  union {
    uint32_t u;
    float f;
  } v;
  v.u = bits;
  return v.f;
}

/* logits: fp16 bit patterns [rows][vocab]. */
void oracle_argmax_prob(const uint16_t *logits, long rows, int vocab,
                        int *ids, float *prob, float *max_logit, int threads) {
  (void)threads;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (long r = 0; r < rows; ++r) {
    const uint16_t *row = logits + (size_t)r * vocab;
    float best = -INFINITY;
    int best_id = 0;
    for (int j = 0; j < vocab; ++j) {
      const float v = half_to_float(row[j]);
      if (v > best) {
        best = v;
        best_id = j;
      }
    }
    double sum = 0.0;
    for (int j = 0; j < vocab; ++j)
      sum += exp((double)half_to_float(row[j]) - (double)best);
    ids[r] = best_id;
    max_logit[r] = best;
    prob[r] = (float)(1.0 / sum);
  }
}

void oracle_ctc_collapse(const int *ids, const float *probs, long lines, int T,
                         int blank, int *out_ids, int *out_len,
                         float *out_score) {
  for (long l = 0; l < lines; ++l) {
    const int *row = ids + (size_t)l * T;
    int *dst = out_ids + (size_t)l * T;
    int prev = -1, count = 0;
    float sum = 0.0f;
    for (int t = 0; t < T; ++t) {
      const int id = row[t];
      if (id == prev)
        continue;
      prev = id;
      if (id == blank)
        continue;
      dst[count++] = id;
      sum += probs ? probs[(size_t)l * T + t] : 1.0f;
    }
    for (int t = count; t < T; ++t)
      dst[t] = -1;
    out_len[l] = count;
    out_score[l] = count ? sum / (float)count : 0.0f;
  }
}
