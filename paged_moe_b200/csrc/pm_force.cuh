// pm_force.cuh -- the forcing hook: ThinkBudget's choice of the next token
// (reference pagedmoe/think_budget.py:75-109) and its effect on a sampled row.
#pragma once

namespace pm {

// A forced row keeps only its forced token: that token is the sample, the
// row's log-sum-exp is its processed value, its log-probability 0 and its
// survivor list the token alone.  A forced token whose processed value is
// -inf leaves a row with no finite value: token 0, as every other pass.
__global__ void __launch_bounds__(256) k_force_rows(const __grid_constant__ SampleArgs a, int dtype,
                                                    const int32_t* forced) {
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < a.rows;
       row += (int64_t)gridDim.x * blockDim.x) {
    const int f = forced[row];
    if (f < 0 || f >= a.vocab) continue;
    const pm_row_params p = row_params(a, row);
    const float x = processed_value(a, dtype, p, row, f);
    const bool fin = x > -INFINITY;
    a.tokens[row] = fin ? f : 0;
    a.status[row] &= ~(1 | 8);  // the row is decided: no unbounded-filter flags
    if (a.lse_out) a.lse_out[row] = x;
    if (a.row_lse) a.row_lse[row] = x;
    if (a.tok_logprob) a.tok_logprob[row] = fin ? 0.0f : __int_as_float(0x7fc00000);
    if (a.n_surv) a.n_surv[row] = fin ? 1 : 0;
    if (a.surv_ids) {
      for (int r = 0; r < a.surv_cap; ++r) {
        a.surv_ids[row * a.surv_cap + r] = (r == 0 && fin) ? f : -1;
        a.surv_probs[row * a.surv_cap + r] = (r == 0 && fin) ? 1.0f : 0.0f;
      }
    }
  }
}

// One warp per row: decoded lengths summed over the counted generation, the
// first position past the budget, the first sentence end (or the slack) at
// or after it, then which close token is due.
__global__ void __launch_bounds__(256) k_think_budget(const int32_t* gen, const int32_t* gen_len, int64_t gen_stride,
                                                      int64_t rows, const int32_t* piece_len,
                                                      const uint8_t* piece_end, int64_t table_size,
                                                      const int32_t* chars, const int32_t* close, int n_close,
                                                      int end_id, int start_id, int slack, int32_t* forced) {
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int32_t* g = gen + row * gen_stride;
    int n = gen_len ? gen_len[row] : (int)gen_stride;
    n = n < 0 ? 0 : (n > gen_stride ? (int)gen_stride : n);
    const int budget = chars[row];
    // where reasoning opens: from the start when the prompt opened it, else
    // after the first start_id (and not at all without one); whether the end
    // tag is already out
    int open_at = start_id < 0 ? -1 : 0x7fffffff;
    bool ended = false;
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lane;
      const int id = i < n ? g[i] : -2;
      if (start_id >= 0) {
        const unsigned b = __ballot_sync(kFull, i < n && id == start_id);
        if (b && open_at == 0x7fffffff) open_at = i0 + __ffs(b) - 1;
      }
      ended |= __any_sync(kFull, i < n && id == end_id) != 0;
    }
    int result = -1;
    if (n > 0 && open_at != 0x7fffffff && !ended) {
      // running sum of the counted pieces: the first position where it reaches
      // the budget, then the first stop at or after it
      int first = -1, stop_at = -1;
      int carry = 0;
      for (int i0 = 0; i0 < n && stop_at < 0; i0 += 32) {
        const int i = i0 + lane;
        int len = 0;
        bool end = false;
        if (i < n) {
          int id = g[i];
          id = id < 0 ? 0 : (id >= table_size ? (int)table_size - 1 : id);
          len = i > open_at ? piece_len[id] : 0;
          end = piece_end[id] != 0;
        }
        const int cum = carry + warp_incl_scan(len);
        carry = __shfl_sync(kFull, cum, 31);
        const bool over = i < n && cum >= budget;
        if (first < 0) {
          const unsigned b = __ballot_sync(kFull, over);
          if (b) first = i0 + __ffs(b) - 1;
        }
        const bool stop = over && first >= 0 && (end || i >= first + slack);
        const unsigned sb = __ballot_sync(kFull, stop);
        if (sb) stop_at = i0 + __ffs(sb) - 1;
      }
      if (stop_at >= 0) {
        const int step = n - 1 - stop_at;
        if (step < n_close) result = close[step];
      }
    }
    if (lane == 0) forced[row] = result;
  }
}

}  // namespace pm
