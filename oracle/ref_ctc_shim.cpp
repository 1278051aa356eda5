// C entry points over the reference's own CTC decoder, compiled from its
// source (native/src/recognition/ctc_decode.cpp) into oracle/_ref/ by the
// Makefile beside this file. TEST INFRASTRUCTURE ONLY: pins the oracle's C
// restatement of the collapse against the real reference code.
#include "ppocrv6_native/recognition/ctc_decode.h"

#include <cstring>
#include <span>
#include <string>
#include <vector>

namespace {
std::vector<std::string> split_lines(const char *joined) {
  std::vector<std::string> out;
  if (!joined)
    return out;
  std::string cur;
  for (const char *p = joined; *p; ++p) {
    if (*p == '\n') {
      out.push_back(cur);
      cur.clear();
    } else {
      cur.push_back(*p);
    }
  }
  out.push_back(cur);
  return out;
}
} // namespace

// ids/scores [batch][seq]; scores may be null (empty span). Writes the kept
// class ids (-1 padded) and scores; returns 0, or -1 if the decoder throws.
extern "C" int ref_ctc_decode_batch(const int *ids, const float *scores,
                                    int batch, int seq, int blank,
                                    int *out_ids, int *out_len,
                                    float *out_score) {
  try {
    const size_t n = static_cast<size_t>(batch) * static_cast<size_t>(seq);
    std::span<const int> idx(ids, n);
    std::span<const float> sc =
        scores ? std::span<const float>(scores, n) : std::span<const float>{};
    const std::vector<std::string> characters; // ids map to "<id>"
    auto res = ppocrv6_native::recognition::ctc_greedy_decode_batch(
        idx, sc, batch, seq, characters, blank);
    for (int b = 0; b < batch; ++b) {
      const auto &d = res[static_cast<size_t>(b)];
      for (int t = 0; t < seq; ++t)
        out_ids[static_cast<size_t>(b) * seq + t] =
            t < static_cast<int>(d.class_ids.size()) ? d.class_ids[t] : -1;
      out_len[b] = static_cast<int>(d.class_ids.size());
      out_score[b] = d.score;
    }
    return 0;
  } catch (...) {
    return -1;
  }
}

// Decodes one batch to text with a '\n'-joined character list; the texts
// are written '\n'-joined into `text` (capacity bytes). Returns 0 / -1.
extern "C" int ref_ctc_decode_text(const int *ids, const float *scores,
                                   int batch, int seq, const char *characters,
                                   int blank, char *text, int capacity,
                                   float *out_score) {
  try {
    const size_t n = static_cast<size_t>(batch) * static_cast<size_t>(seq);
    auto res = ppocrv6_native::recognition::ctc_greedy_decode_batch(
        std::span<const int>(ids, n),
        scores ? std::span<const float>(scores, n) : std::span<const float>{},
        batch, seq, split_lines(characters), blank);
    std::string joined;
    for (int b = 0; b < batch; ++b) {
      if (b)
        joined += '\n';
      joined += res[static_cast<size_t>(b)].text;
      out_score[b] = res[static_cast<size_t>(b)].score;
    }
    if (static_cast<int>(joined.size()) + 1 > capacity)
      return -1;
    std::memcpy(text, joined.c_str(), joined.size() + 1);
    return 0;
  } catch (...) {
    return -1;
  }
}
