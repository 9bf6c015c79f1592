// pm_prep.cuh -- the penalty scatter's host-independent half: per-row
// override lists built from the token histories.
//
// For every row, each distinct id inside the union of its processors'
// windows becomes one entry: bit0 = inside the repetition window, bit1 =
// inside the presence window, bits 8.. = occurrences inside the frequency
// window.  Entries are grouped by 1024-token tile (in no particular order
// inside a tile), and tile_off[t] is the first entry of tile t, so the
// streaming kernels find a tile's overrides in O(1).
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
  uint64_t* row_tau;  // [rows] zeroed here for the streaming pass (or null)
  int32_t* exact_q;   // [1 + rows]: the exact pass's queue count and tile counters, zeroed here (or null)
};

__device__ __forceinline__ int window_start(int H, int ctx) {
  if (ctx > 0) return H > ctx ? H - ctx : 0;
  if (ctx == 0) return 0;
  return (-ctx) < H ? -ctx : H;
}

// One CTA of 1024 threads per row.  The ids of the union window go into a
// shared-memory hash table (open addressing, 2 x cap slots) that keeps each
// distinct id's latest position and its count inside the frequency window;
// the entries with an effect are then bucketed by tile (a counting pass and a
// scatter), in no particular order inside a tile.  Dynamic shared memory:
// 3 x (2 cap) ints + 2 x 264 ints.
__global__ void __launch_bounds__(1024) k_prep_overrides(PrepArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int slots = 2 * a.cap;
  int* hid = reinterpret_cast<int*>(smem_raw);
  int* hlast = hid + slots;
  int* hcnt = hlast + slots;
  int* tcount = hcnt + slots;  // [264]
  int* tcur = tcount + 264;    // [264]
  const int tid = threadIdx.x, nth = blockDim.x;
  const int64_t r = blockIdx.x;
  // the streaming pass may start its prologue (tile loads) now; it waits for
  // this grid before it reads anything written here
  asm volatile("griddepcontrol.launch_dependents;");
  if (r >= a.rows) return;
  if (a.row_tau && tid == 0) a.row_tau[r] = 0;
  if (a.exact_q && tid == 0) {
    a.exact_q[1 + r] = 0;
    if (r == 0) a.exact_q[0] = 0;
  }
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
  for (int i = tid; i < slots; i += nth) { hid[i] = -1; hlast[i] = -1; hcnt[i] = 0; }
  for (int i = tid; i < 264; i += nth) tcount[i] = 0;
  __syncthreads();
  // insert every position of the window; ids outside [0, V) are dropped
  for (int i = tid; i < n; i += nth) {
    const int pos = s + i;
    const int64_t tok =
        (int64_t)(pos < Hb ? a.hist[b * a.hist_stride + pos] : a.feed[b * a.feed_group + (pos - Hb)]) - a.id_base;
    if (tok < 0 || tok >= a.vocab) continue;
    uint32_t h = ((uint32_t)tok * 2654435761u) % (uint32_t)slots;
    for (int probe = 0; probe < slots; ++probe) {
      const int prev = atomicCAS(&hid[h], -1, (int)tok);
      if (prev == -1 || prev == (int)tok) {
        atomicMax(&hlast[h], pos);
        if (freq && pos >= s_freq) atomicAdd(&hcnt[h], 1);
        break;
      }
      h = h + 1 == (uint32_t)slots ? 0u : h + 1;
    }
  }
  __syncthreads();
  // entries with an effect, counted per tile
  for (int i = tid; i < slots; i += nth) {
    const int tok = hid[i];
    if (tok < 0) continue;
    const int last = hlast[i];
    const uint32_t info = (rep && last >= s_rep ? 1u : 0u) | (pres && last >= s_pres ? 2u : 0u) |
                          ((uint32_t)hcnt[i] << 8);
    hcnt[i] = (int)info;  // reuse the slot for the entry's info
    if (info) atomicAdd(&tcount[tok / kTile], 1);
  }
  __syncthreads();
  // tile offsets (exclusive prefix over the tiles, one warp)
  if (tid < 32) {
    const int per = (a.n_tiles + 1 + 31) / 32;  // <= 9 for 257 entries
    int loc[9];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const int t = tid * per + k;
      loc[k] = (k < per && t <= a.n_tiles) ? tcount[t] : 0;
      sum += loc[k];
    }
    const int incl = warp_incl_scan(sum);
    int run = incl - sum;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const int t = tid * per + k;
      if (k < per && t <= a.n_tiles) {
        tcur[t] = run;
        a.ovr_off[r * (int64_t)(a.n_tiles + 1) + t] = run;
        run += loc[k];
      }
    }
  }
  __syncthreads();
  int32_t* out_tok = a.ovr_tok + r * a.cap;
  uint32_t* out_info = a.ovr_info + r * a.cap;
  for (int i = tid; i < slots; i += nth) {
    const int tok = hid[i];
    if (tok < 0) continue;
    const uint32_t info = (uint32_t)hcnt[i];
    if (!info) continue;
    const int at = atomicAdd(&tcur[tok / kTile], 1);
    out_tok[at] = tok;
    out_info[at] = info;
  }
}

}  // namespace pm
