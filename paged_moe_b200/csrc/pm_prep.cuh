// pm_prep.cuh -- the penalty scatter's host-independent half: per-row sorted
// override lists built from the token histories.
//
// For every row, the ids inside the union of its processors' windows are
// sorted (with their positions) and each distinct id becomes one entry:
// bit0 = inside the repetition window, bit1 = inside the presence window,
// bits 8.. = occurrences inside the frequency window.  Entries are ascending
// by id, and tile_off[t] is the first entry with id >= t * kTile, so the
// streaming kernel finds a tile's overrides in O(1).
//
// Windows follow Python's tokens[-context_size:] (mlx-lm's processors slice
// the running sequence that way; reference verify_decode.py:828-831).
#pragma once

#include "pm_device.cuh"
#include "../../include/pm_sample.h"

namespace pm {

struct PrepArgs {
  const int32_t* hist;
  const int32_t* hist_len;
  int64_t hist_stride;
  const int32_t* feed;
  int32_t feed_group;
  const pm_row_params* params;
  int32_t params_per_row;
  int64_t rows;
  int64_t vocab;
  int64_t id_base;    // first token id of these rows' vocabulary slice (a vocabulary shard), else 0
  int32_t n_tiles;
  int32_t cap;        // entries per row in the output lists (power of two)
  int32_t* ovr_tok;   // [rows, cap]
  uint32_t* ovr_info; // [rows, cap]
  int32_t* ovr_off;   // [rows, n_tiles + 1]
  int32_t* status;    // [rows]
};

__device__ __forceinline__ int window_start(int H, int ctx) {
  if (ctx > 0) return H > ctx ? H - ctx : 0;
  if (ctx == 0) return 0;
  return (-ctx) < H ? -ctx : H;
}

// one CTA of 1024 threads per row; dynamic shared memory: cap u64 keys, 64 ints, cap ints
__global__ void __launch_bounds__(1024) k_prep_overrides(PrepArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem_raw);
  int* wsum = reinterpret_cast<int*>(keys + a.cap);
  const int tid = threadIdx.x, nth = blockDim.x;
  const int64_t r = blockIdx.x;
  if (r >= a.rows) return;
  const pm_row_params p = a.params[a.params_per_row ? r : 0];
  const int64_t b = a.feed ? r / a.feed_group : r;
  const int fi = a.feed ? (int)(r % a.feed_group) : -1;
  int Hb = 0;
  if (a.hist) {
    Hb = a.hist_len ? a.hist_len[b] : (int)a.hist_stride;
    Hb = Hb < 0 ? 0 : (Hb > a.hist_stride ? (int)a.hist_stride : Hb);
  }
  const int H = Hb + (a.feed ? fi + 1 : 0);
  const bool rep = p.flags & PM_F_REP, pres = p.flags & PM_F_PRES, freq = p.flags & PM_F_FREQ;
  const int s_rep = rep ? window_start(H, p.repetition_context_size) : H;
  const int s_pres = pres ? window_start(H, p.presence_context_size) : H;
  const int s_freq = freq ? window_start(H, p.frequency_context_size) : H;
  int s = s_rep < s_pres ? s_rep : s_pres;
  s = s < s_freq ? s : s_freq;
  int n = H - s;
  if (tid == 0) a.status[r] = n > a.cap ? 2 : 0;  // 2: window longer than this build's history cap
  if (n > a.cap) n = 0;
  // load (id << 32 | position); ids outside [0, V) sort last and are dropped
  for (int i = tid; i < a.cap; i += nth) {
    uint64_t k = ~0ull;
    if (i < n) {
      const int pos = s + i;
      const int64_t tok =
          (int64_t)(pos < Hb ? a.hist[b * a.hist_stride + pos] : a.feed[b * a.feed_group + (pos - Hb)]) - a.id_base;
      if (tok >= 0 && tok < a.vocab) k = ((uint64_t)(uint32_t)tok << 32) | (uint32_t)pos;
    }
    keys[i] = k;
  }
  __syncthreads();
  for (int k = 2; k <= a.cap; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < a.cap; i += nth) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = keys[i], y = keys[ixj];
          const bool asc = (i & k) == 0;
          if (asc ? (x > y) : (x < y)) { keys[i] = y; keys[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
  // Runs of equal ids are contiguous and ascending by position.  A run's
  // last element carries its latest position (the repetition / presence
  // windows) and, through two block scans, the run's first index and the
  // number of its positions inside the frequency window.  Each thread owns a
  // contiguous block of E entries.
  const int E = a.cap / nth > 0 ? a.cap / nth : 1;
  const int lo = tid * E;
  int* fpre = reinterpret_cast<int*>(wsum + 64);  // inclusive count of in-window positions, per entry
  int fsum = 0, smax = 0;
  for (int e = 0; e < E; ++e) {
    const int i = lo + e;
    if (i >= a.cap) break;
    const uint64_t k = keys[i];
    const bool valid = k != ~0ull;
    if (valid && (i == 0 || (uint32_t)(keys[i - 1] >> 32) != (uint32_t)(k >> 32))) smax = i;
    fsum += (valid && freq && (int)(uint32_t)k >= s_freq) ? 1 : 0;
  }
  // block scans: exclusive sum of in-window counts, exclusive max of run starts
  {
    const int lane = tid & 31, wid = tid >> 5;
    int is = fsum, im = smax;  // warp-inclusive
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ts = __shfl_up_sync(kFull, is, o), tm = __shfl_up_sync(kFull, im, o);
      if (lane >= o) { is += ts; im = max(im, tm); }
    }
    if (lane == 31) { wsum[wid] = is; wsum[32 + wid] = im; }
    __syncthreads();
    if (wid == 0) {
      const int nw2 = nth >> 5;
      int xs = lane < nw2 ? wsum[lane] : 0, xm = lane < nw2 ? wsum[32 + lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int ts = __shfl_up_sync(kFull, xs, o), tm = __shfl_up_sync(kFull, xm, o);
        if (lane >= o) { xs += ts; xm = max(xm, tm); }
      }
      if (lane < nw2) { wsum[lane] = xs; wsum[32 + lane] = xm; }
    }
    __syncthreads();
    const int prev_m = __shfl_up_sync(kFull, im, 1);
    fsum = (is - fsum) + (wid > 0 ? wsum[wid - 1] : 0);
    smax = max(lane > 0 ? prev_m : 0, wid > 0 ? wsum[32 + wid - 1] : 0);
  }
  __syncthreads();  // wsum is reused for the emit scan below
  int run_start[8];
  int emit_local = 0;
  uint32_t info_loc[8];
  int tok_loc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) { info_loc[e] = 0; tok_loc[e] = -1; run_start[e] = 0; }
  for (int e = 0; e < E && e < 8; ++e) {
    const int i = lo + e;
    if (i >= a.cap) break;
    const uint64_t k = keys[i];
    const bool valid = k != ~0ull;
    if (valid && (i == 0 || (uint32_t)(keys[i - 1] >> 32) != (uint32_t)(k >> 32))) smax = i;
    run_start[e] = smax;
    fsum += (valid && freq && (int)(uint32_t)k >= s_freq) ? 1 : 0;
    fpre[i] = fsum;
  }
  __syncthreads();
  for (int e = 0; e < E && e < 8; ++e) {
    const int i = lo + e;
    if (i >= a.cap) break;
    const uint64_t k = keys[i];
    if (k == ~0ull) continue;
    const uint32_t tok = (uint32_t)(k >> 32);
    if (i + 1 < a.cap && keys[i + 1] != ~0ull && (uint32_t)(keys[i + 1] >> 32) == tok) continue;  // not a run end
    const int last_pos = (int)(uint32_t)k;
    const int st = run_start[e];
    uint32_t info = 0;
    if (rep && last_pos >= s_rep) info |= 1u;
    if (pres && last_pos >= s_pres) info |= 2u;
    if (freq) info |= (uint32_t)(fpre[i] - (st > 0 ? fpre[st - 1] : 0)) << 8;
    if (info) { info_loc[e] = info; tok_loc[e] = (int)tok; ++emit_local; }
  }
  // block exclusive scan of emit counts
  const int lane = tid & 31, wid = tid >> 5;
  const int incl = warp_incl_scan(emit_local);
  if (lane == 31) wsum[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    const int v = lane < (nth >> 5) ? wsum[lane] : 0;
    const int vi = warp_incl_scan(v);
    if (lane < (nth >> 5)) wsum[lane] = vi - v;
  }
  __syncthreads();
  int pos = wsum[wid] + incl - emit_local;
  int32_t* out_tok = a.ovr_tok + r * a.cap;
  uint32_t* out_info = a.ovr_info + r * a.cap;
  for (int e = 0; e < E && e < 8; ++e) {
    if (tok_loc[e] >= 0) { out_tok[pos] = tok_loc[e]; out_info[pos] = info_loc[e]; ++pos; }
  }
  __syncthreads();
  // total count = exclusive start of the last thread + its count
  __shared__ int total_s;
  if (tid == nth - 1) total_s = pos;
  __syncthreads();
  const int total = total_s;
  // tile offsets: lower_bound over the emitted ids (read back from global)
  for (int t = tid; t <= a.n_tiles; t += nth) {
    const int64_t key = (int64_t)t * kTile;
    int lo3 = 0, hi3 = total;
    while (lo3 < hi3) {
      const int mid = (lo3 + hi3) >> 1;
      if ((int64_t)out_tok[mid] >= key) hi3 = mid; else lo3 = mid + 1;
    }
    a.ovr_off[r * (int64_t)(a.n_tiles + 1) + t] = lo3;
  }
}

}  // namespace pm
