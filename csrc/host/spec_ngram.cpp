// Prompt-lookup (n-gram) draft proposals for speculative decoding, batched over sequences.
//
// For each sequence, the longest suffix of its tokens (n from max_n down to min_n) that also occurs
// earlier in the sequence is located (most recent earlier occurrence); the up-to-k tokens that
// followed that occurrence are the draft. No draft model is needed: repetitive text (code, quoted
// context, lists) is verified k tokens at a time by one target forward.
//
// Plays the drafting role of the reference's draft model in
// inference/gollek-runtime-inference/…/runtime/inference/speculative/SpeculativeDecoder.java:1-60.
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <vector>

namespace {

// Draft for one token sequence; returns the number of tokens written to out (<= k).
int propose_one(const int32_t* tok, int64_t len, int min_n, int max_n, int k, int32_t* out) {
  for (int n = std::min<int64_t>(max_n, len - 1); n >= min_n; --n) {
    const int32_t* pat = tok + len - n;
    // scan earlier windows from the most recent backwards; window must end before the suffix
    for (int64_t s = len - n - 1; s >= 0; --s) {
      if (tok[s] != pat[0]) continue;
      bool eq = true;
      for (int j = 1; j < n; ++j)
        if (tok[s + j] != pat[j]) {
          eq = false;
          break;
        }
      if (!eq) continue;
      const int64_t from = s + n;
      const int cnt = (int)std::min<int64_t>(k, len - from);
      for (int j = 0; j < cnt; ++j) out[j] = tok[from + j];
      if (cnt > 0) return cnt;
    }
  }
  return 0;
}

}  // namespace

// tokens: int32 concatenation of every sequence's tokens; offsets: int64 [B + 1].
// Returns (drafts int32 [B, k] (padded with -1), counts int32 [B]).
std::vector<torch::Tensor> ngram_propose(torch::Tensor tokens, torch::Tensor offsets, int64_t min_n, int64_t max_n,
                                         int64_t k) {
  TORCH_CHECK(tokens.dtype() == torch::kInt32 && tokens.is_contiguous() && !tokens.is_cuda(), "tokens: int32 CPU");
  TORCH_CHECK(offsets.dtype() == torch::kInt64 && offsets.is_contiguous() && !offsets.is_cuda(), "offsets: int64 CPU");
  TORCH_CHECK(min_n >= 1 && max_n >= min_n && k >= 1, "ngram: 1 <= min_n <= max_n, k >= 1");
  const int64_t B = offsets.numel() - 1;
  auto drafts = torch::full({B, k}, -1, torch::dtype(torch::kInt32));
  auto counts = torch::zeros({B}, torch::dtype(torch::kInt32));
  const int32_t* tp = tokens.data_ptr<int32_t>();
  const int64_t* op = offsets.data_ptr<int64_t>();
  int32_t* dp = drafts.data_ptr<int32_t>();
  int32_t* cp = counts.data_ptr<int32_t>();
  {
    pybind11::gil_scoped_release release;
    for (int64_t b = 0; b < B; ++b) {
      const int64_t len = op[b + 1] - op[b];
      TORCH_CHECK(len >= 0, "ngram: offsets must be non-decreasing");
      cp[b] = len > 1 ? propose_one(tp + op[b], len, (int)min_n, (int)max_n, (int)k, dp + b * k) : 0;
    }
  }
  return {drafts, counts};
}

void register_spec(pybind11::module& m) {
  m.def("ngram_propose", &ngram_propose, "prompt-lookup draft tokens for a batch of sequences");
}
