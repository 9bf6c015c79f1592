// pm_ngram.cuh -- batched n-gram drafts (reference pagedmoe/lookup_decode.py:184-221
// draft_ngram, which rescans one request's context in Python every step).
//
// One CTA per request.  A window of n tokens ending at position e (e < L, so
// a token follows it) matches the context's last n tokens exactly when the
// prefixes toks[:e] and toks[:L] share a suffix of length >= n, so one pass
// computes, for every end e, that common length c(e) (capped at n_max) and
// records per n: the latest end whose continuation holds k tokens, and the
// earliest end (longest continuation) among the others.  The longest n with
// any match decides: its latest full continuation, else its longest partial
// one -- the reference's choice.
#pragma once

namespace pm {

constexpr int kNgramMax = 32;

__global__ void __launch_bounds__(256) k_draft_ngram(const int32_t* hist, const int32_t* hist_len,
                                                     int64_t hist_stride, int64_t requests, int k, int n_min,
                                                     int n_max, int32_t* drafts, int32_t* draft_len,
                                                     int32_t* match_n) {
  __shared__ int full_e[kNgramMax + 1];
  __shared__ int part_e[kNgramMax + 1];
  const int tid = threadIdx.x;
  for (int64_t b = blockIdx.x; b < requests; b += gridDim.x) {
    const int32_t* toks = hist + b * hist_stride;
    int L = hist_len ? hist_len[b] : (int)hist_stride;
    L = L < 0 ? 0 : (L > hist_stride ? (int)hist_stride : L);
    const int nmax = n_max < L ? n_max : L;
    for (int n = tid; n <= kNgramMax; n += blockDim.x) {
      full_e[n] = -1;
      part_e[n] = 0x7fffffff;
    }
    __syncthreads();
    if (k > 0 && nmax >= n_min) {
      for (int e = n_min + tid; e < L; e += blockDim.x) {
        const int cap = nmax < e ? nmax : e;
        int c = 0;
        while (c < cap && toks[e - 1 - c] == toks[L - 1 - c]) ++c;
        for (int n = n_min; n <= c; ++n) {
          if (e + k <= L) atomicMax(&full_e[n], e);
          else atomicMin(&part_e[n], e);
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      int len = 0, used = 0, at = 0;
      if (k > 0 && nmax >= n_min) {
        for (int n = nmax; n >= n_min; --n) {
          if (full_e[n] >= 0) { at = full_e[n]; len = k; used = n; break; }
          if (part_e[n] != 0x7fffffff) { at = part_e[n]; len = L - part_e[n]; used = n; break; }
        }
      }
      for (int i = 0; i < k; ++i) drafts[b * k + i] = i < len ? toks[at + i] : -1;
      draft_len[b] = len;
      if (match_n) match_n[b] = used;
    }
    __syncthreads();
  }
}

}  // namespace pm
