// Speculative decoding with FlashHead token ids: acceptance of draft tokens.
//
// The target model's FlashHead step returns one token id per position
// (greedy) instead of logits, so verification is an exact comparison: per
// request, draft tokens are accepted while they equal the target's token at
// the same position; the first mismatch is replaced by the target's token and
// ends the row; a row whose drafts are all accepted gets the bonus token (the
// target's token after the last draft) at position n. Every other position
// holds the placeholder id. This is the comparison of the reference's
// RejectionSampler hook (patches/rejection_sampler.py:55-76), done on the
// device instead of in a per-element host loop. Unlike that loop, a request
// with no draft tokens gets its bonus token at position 0, as vLLM's own
// rejection sampler gives it.
#pragma once

#include <cstdint>

namespace fh {

// One warp per request; lanes scan its draft positions 32 at a time and the
// first mismatch (ballot) ends acceptance. cu_num_draft[b] = drafts of
// requests 0..b (inclusive prefix sum, vLLM's cu_num_draft_tokens).
__global__ void k_spec_accept(const int32_t *draft, const int32_t *target, const int32_t *bonus,
                              const int32_t *cu_num_draft, int batch, int max_spec_len,
                              int32_t placeholder, int32_t *out) {
  const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= batch) return;
  const int start = w ? cu_num_draft[w - 1] : 0;
  int n = cu_num_draft[w] - start;
  n = n < 0 ? 0 : (n > max_spec_len ? max_spec_len : n);
  int first = n;  // first rejected position; n: all accepted
  for (int j0 = 0; j0 < n && first == n; j0 += 32) {
    const int j = j0 + lane;
    const bool mismatch = j < n && draft[start + j] != target[start + j];
    const unsigned m = __ballot_sync(0xFFFFFFFFu, mismatch);
    if (m) first = j0 + __ffs(m) - 1;
  }
  int32_t *row = out + (size_t)w * (max_spec_len + 1);
  for (int j = lane; j <= max_spec_len; j += 32) {
    int32_t v = placeholder;
    if (j < first)
      v = draft[start + j];
    else if (j == first)
      v = first < n ? target[start + j] : bonus[w];
    row[j] = v;
  }
}

}  // namespace fh
