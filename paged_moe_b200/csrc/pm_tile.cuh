// pm_tile.cuh -- one 1024-token tile of one logits row, as a warp sees it.
//
// A warp holds a tile in registers: lane L owns 32 value slots; slot s is
// token  (s / VW) * 32 * VW + L * VW + (s % VW)  of the tile, so every load
// instruction of the warp reads 32 * VW consecutive tokens (512 bytes) with
// one 16-byte access per lane.  VW = 4 for fp32 rows, 8 for bf16 rows.
//
// The raw load of the next tile (values, the lane's allowed-token word and
// the tile's override range) is issued before the current tile is
// processed, so the memory system always has the next tile in flight.
#pragma once

#include "pm_device.cuh"
#include "../../include/pm_sample.h"

namespace pm {

struct TileStat {
  float m;        // max of the tile's (processed) values, -inf if none is finite
  uint32_t pad;
  uint64_t s;     // sum over the tile of floor(e^(x - m) 2^52)
};

// Approximate statistics of one row part (rows whose filters need the
// log-sum-exp only to place the top-p cut): s ~ sum over the part of
// 2^(fl(x L - fl(mref L))), L = fl32(log2 e), from the hardware ex2 and fp32
// sums, with eps a bound on its relative error.  Stored in the row's
// y-statistics slot of the part's first tile (such rows use no y statistics).
struct ApproxStat {
  float mref;   // the part's reference value (-inf: the part holds no finite value)
  float eps;
  double s;
};
static_assert(sizeof(ApproxStat) == sizeof(TileStat), "ApproxStat shares the TileStat slots");

// Everything the streaming kernels read or write.
struct SampleArgs {
  const void* logits;
  int64_t rows, vocab, row_stride;
  bool vec_ok;
  const pm_row_params* params;
  int32_t params_per_row;
  // processors
  const int32_t* ovr_tok;
  const uint32_t* ovr_info;
  const int32_t* ovr_off;   // [rows, n_tiles + 1] or null
  int32_t ovr_cap;
  const int32_t* bias_tok;
  const float* bias_val;
  const int32_t* bias_off;  // [n_tiles + 1] or null
  const uint32_t* mask;
  int64_t mask_stride;
  bool mask_ok;             // mask rows 16-byte aligned: bulk-copyable
  // noise
  int32_t noise_mode;
  uint64_t seed, offset;
  uint32_t row_base;
  const float* gumbel;
  int64_t gumbel_stride;
  const double* uniform;
  // outputs
  int32_t* tokens;
  float* lse_out;
  float* tok_logprob;
  int32_t* surv_ids;
  float* surv_probs;
  int32_t* n_surv;
  int32_t surv_cap;
  bool want_lse;
  // workspace
  TileStat* statx;   // [rows, n_tiles] stats of x (the processed logits)
  TileStat* staty;   // [rows, n_tiles] stats of y = x * inv_temperature (whole-vocabulary draw)
  uint64_t* cand;    // [rows, max_parts, KC] candidate keys of each row part
  int32_t* cand_n;   // [rows, max_parts] count | (1 << 30) when the part was trimmed
  uint64_t* best;    // [rows, max_parts] greedy best key of each row part
  uint64_t* row_tau;   // [rows] largest K-th key any part of the row has proven (0: none)
  int32_t* status;   // [rows] 0 ok, 1 survivors beyond the candidates, 2 history window too long
  bool status_live;  // status[] already holds this call's flags (zeroed, or written by the penalty prep)
  float* row_lse;    // [rows]
  // bracketed statistics: rows with top-k and top-p (no min-p) need the
  // log-sum-exp only to place the top-p cut; with approx_ok the streaming
  // pass writes approximate tile sums for them, the merge places the cut from
  // a rigorous bracket around the exact log-sum-exp, and the rare rows whose
  // cut the bracket does not decide are queued for the exact pass
  bool approx_ok;
  // greedy rows finished inside the streaming pass: the warp that ends a
  // row's last part (a count of finished parts in row_tau, which greedy rows
  // do not otherwise use) takes the parts' best keys and writes the row
  bool merge_greedy;
  int32_t* exact_q;  // [1 + 2 rows]: queued count, per-entry tile counters [rows], queued rows [rows]
  int32_t n_tiles;
  int32_t max_parts;
  int64_t n_warps;   // warps of the launch (the flattened tile range is split over them)
  int32_t fixed_parts;  // > 0: every row has this many parts (the fused LM-head pass's vocabulary slices)
  // verify extension (pm_verify.cu); rows are requests * (k+1) target rows
  int32_t feed_group;
  void* verify;      // VerifyState* or null
};

template <typename T> struct Lay;
template <> struct Lay<float> { static constexpr int VW = 4; };
template <> struct Lay<__nv_bfloat16> { static constexpr int VW = 8; };

template <int VW>
__device__ __forceinline__ int slot_elem(int s, int lane) {
  return (s / VW) * (32 * VW) + lane * VW + (s % VW);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// A tile in flight: raw values plus what the processors need.
struct TileIn {
  float v[32];
  uint32_t mw;   // lane's allowed-token word (mask) of the tile
  int ob, oe;    // override range of the tile in the row's list
  int bb, be;    // logit-bias range of the tile
};

__device__ __forceinline__ int tile_valid(const SampleArgs& a, int tile) {
  const int64_t start = (int64_t)tile * kTile;
  return (int)((a.vocab - start) < kTile ? (a.vocab - start) : kTile);
}

template <typename T>
__device__ __forceinline__ void load_tile(const SampleArgs& a, int64_t row, int tile, TileIn& ti) {
  constexpr int VW = Lay<T>::VW;
  const int lane = threadIdx.x & 31;
  const int64_t start = (int64_t)tile * kTile;
  const int n_valid = tile_valid(a, tile);
  const T* rowp = reinterpret_cast<const T*>(a.logits) + row * a.row_stride;
  if (a.vec_ok && n_valid == kTile) {
    if constexpr (sizeof(T) == 4) {
      const float4* p = reinterpret_cast<const float4*>(rowp + start);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 q = __ldcs(p + j * 32 + lane);
        ti.v[4 * j] = q.x; ti.v[4 * j + 1] = q.y; ti.v[4 * j + 2] = q.z; ti.v[4 * j + 3] = q.w;
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(rowp + start);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 q = __ldcs(p + j * 32 + lane);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          ti.v[8 * j + 2 * h] = bf16_bits_to_f32(w[h] & 0xffffu);
          ti.v[8 * j + 2 * h + 1] = bf16_bits_to_f32(w[h] >> 16);
        }
      }
    }
  } else {
#pragma unroll
    for (int s = 0; s < 32; ++s) {
      const int e = slot_elem<VW>(s, lane);
      float x = -INFINITY;
      if (e < n_valid) {
        if constexpr (sizeof(T) == 4) x = rowp[start + e];
        else x = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(rowp)[start + e]);
      }
      ti.v[s] = x;
    }
  }
  ti.mw = 0xffffffffu;
  if (a.mask) {
    const int nw = (n_valid + 31) >> 5;
    ti.mw = lane < nw ? __ldcs(a.mask + row * a.mask_stride + (start >> 5) + lane) : 0u;
  }
  ti.ob = ti.oe = ti.bb = ti.be = 0;
  if (a.ovr_off) {
    const int32_t* off = a.ovr_off + row * (int64_t)(a.n_tiles + 1) + tile;
    ti.ob = off[0];
    ti.oe = off[1];
  }
  if (a.bias_off) { ti.bb = a.bias_off[tile]; ti.be = a.bias_off[tile + 1]; }
}

// The processors on a loaded tile, in mlx-lm's make_logits_processors order
// (logit bias, repetition, presence, frequency), then the allowed-token mask
// that the reference's own processors apply last (server.py:3045-3049 appends
// them after mlx-lm's; think_budget.py:107-109, rescue.py:240-245).  Overrides
// go through the warp's staging buffer, only for tiles that hold one.
template <int VW>
__device__ __forceinline__ void process_tile(const SampleArgs& a, const pm_row_params& p, int64_t row,
                                             int tile, TileIn& ti, float* wbuf) {
  const int lane = threadIdx.x & 31;
  const int64_t start = (int64_t)tile * kTile;
  if (ti.oe > ti.ob || ti.be > ti.bb) {
#pragma unroll
    for (int s = 0; s < 32; ++s) wbuf[slot_elem<VW>(s, lane)] = ti.v[s];
    __syncwarp();
    for (int i = ti.bb + lane; i < ti.be; i += 32) {
      const int64_t e = a.bias_tok[i] - start;
      if (e >= 0 && e < kTile) wbuf[e] = fadd(wbuf[e], a.bias_val[i]);  // ids out of ascending order: skipped
    }
    __syncwarp();
    const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
    const uint32_t* oinf = a.ovr_info + row * (int64_t)a.ovr_cap;
    for (int i = ti.ob + lane; i < ti.oe; i += 32) {
      const int e = (int)(otok[i] - start);
      const uint32_t info = oinf[i];
      float x = wbuf[e];
      if (info & 1u) x = x < 0.0f ? fmul(x, p.repetition_penalty) : __fdiv_rn(x, p.repetition_penalty);
      if (info & 2u) x = fsub(x, p.presence_penalty);
      const uint32_t cnt = info >> 8;
      if (cnt) x = fsub(x, fmul(p.frequency_penalty, (float)cnt));
      wbuf[e] = x;
    }
    __syncwarp();
#pragma unroll
    for (int s = 0; s < 32; ++s) ti.v[s] = wbuf[slot_elem<VW>(s, lane)];
    __syncwarp();
  }
  if (a.mask) {
#pragma unroll
    for (int j = 0; j < 32 / VW; ++j) {
      const uint32_t w = __shfl_sync(kFull, ti.mw, j * VW + (lane * VW) / 32);
      const uint32_t bits = w >> ((lane * VW) & 31);
#pragma unroll
      for (int c = 0; c < VW; ++c)
        if (!((bits >> c) & 1u)) ti.v[j * VW + c] = -INFINITY;
    }
  }
}

// Exact statistics of one tile held by the warp (warp-uniform result).
__device__ __forceinline__ void tile_stats(const float (&v)[32], float* m_out, uint64_t* s_out) {
  float m = -INFINITY;
#pragma unroll
  for (int s = 0; s < 32; ++s) m = fmaxf(m, v[s]);
  m = warp_max(m);
  uint64_t sum = 0;
  if (m > -INFINITY) {
#pragma unroll
    for (int s = 0; s < 32; s += 2) {
      uint64_t q0, q1;
      q52x2(fsub(v[s], m), fsub(v[s + 1], m), q0, q1);
      sum += q0 + q1;
    }
  }
  *m_out = m;
  *s_out = warp_sum_u64(sum);
}

__device__ __forceinline__ const pm_row_params& row_params(const SampleArgs& a, int64_t row) {
  return a.params[a.params_per_row ? row : 0];
}

enum RowMode { kGreedy = 0, kCand = 1, kFullDraw = 2 };

__device__ __forceinline__ int row_mode(const pm_row_params& p) {
  if (p.flags & PM_F_GREEDY) return kGreedy;
  if (p.top_k > 0 || (p.flags & (PM_F_TOP_P | PM_F_MIN_P))) return kCand;
  return kFullDraw;
}

// Rows filtered by min-p alone (top-k and top-p off, min_tokens_to_keep <= 1):
// nothing below (any part's maximum) + log(min_p) - 1 can survive, so such a
// floor is a candidate threshold that drops no survivor.  The shared row
// threshold of these rows carries floors only.
__device__ __forceinline__ bool minp_floor_row(const pm_row_params& p) {
  return (p.flags & PM_F_MIN_P) && !(p.flags & PM_F_TOP_P) && p.top_k <= 0 && p.min_tokens_to_keep <= 1;
}

// Rows whose exact log-sum-exp is replaced by a bracket (see SampleArgs).
__device__ __forceinline__ bool needs_astats(const SampleArgs& a, const pm_row_params& p, int mode) {
  return a.approx_ok && !a.want_lse && !a.mask && mode == kCand && p.top_k > 0 && (p.flags & PM_F_TOP_P) &&
         !(p.flags & PM_F_MIN_P);
}

__device__ __forceinline__ bool needs_xstats(const SampleArgs& a, const pm_row_params& p, int mode) {
  return a.want_lse || (mode == kCand && (p.flags & (PM_F_TOP_P | PM_F_MIN_P)) && !needs_astats(a, p, mode));
}

// Flattened split of rows * n_tiles tiles over n_warps warps: warp w owns
// [floor(w T / W), floor((w+1) T / W)).  The warp that owns tile g:
__device__ __forceinline__ int64_t owner_warp(int64_t g, int64_t T, int64_t W) {
  return ((g + 1) * W + T - 1) / T - 1;
}

}  // namespace pm
