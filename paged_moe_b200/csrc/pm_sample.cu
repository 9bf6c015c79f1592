// pm_sample.cu -- the fused token-selection kernels for sm_100a.
//
// One streaming pass per row reads the logits once from HBM.  A row is cut
// into chunks of whole 1024-token tiles; a persistent grid walks the
// (row, chunk) work items.  For every tile a warp
//   1. loads the tile with 128-bit streaming loads (one value slot per
//      register, 32 per lane),
//   2. applies the processors: logit bias and penalties through a shared
//      memory staging copy when the tile holds an overridden id (rare), then
//      the allowed-token bitmask,
//   3. writes the tile's exact log-sum-exp statistics (max and the integer
//      sum of floor(e^(x - max) 2^52)) when the row needs them,
//   4. feeds the row's candidate search: the greedy argmax, or a warp
//      candidate buffer behind a running threshold for top-k style filters.
// A second kernel, one warp per row, merges each row's parts: log-sum-exp
// from the tile statistics, the row's top-K candidates, top-p / min-p, and
// the draw.
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "pm_device.cuh"
#include "pm_prep.cuh"
#include "pm_select.cuh"
#include "pm_tile.cuh"
#include "pm_warp.cuh"
#include "pm_stream.cuh"
#include "../../include/pm_sample.h"
#include "pm_host.h"

namespace pm {

constexpr int kWarpsS = 4;                 // warps per CTA of the streaming kernel
constexpr int kThreadsS = kWarpsS * 32;
// Streaming CTAs resident per SM: four at KC = 64 (51.6 KB of shared memory
// each, so 128 registers a thread), three at KC = 256 (57.8 KB each: a
// fourth would not fit in 228 KB, so its registers need no tighter cap).
template <int KC>
constexpr int kStreamBlocks = KC == 64 ? 4 : 3;

// Per-row state of a warp's current row part.
struct PartState {
  pm_row_params p;
  int mode;
  bool needx, needy;
  bool needa;       // approximate statistics (the bracket) instead of needx
  int K;            // candidates kept per part
  float best_x;
  int best_e;
  Cand cd;
  bool published;   // a compaction raised the threshold since the last publish
  uint64_t rtau;    // the row's shared threshold, loaded one tile ahead
  // min-p without top-k / top-p (and min_tokens_to_keep <= 1): nothing below
  // (part maximum) + log(min_p) - 1 can survive, so offers start there
  bool minp_floor;
  float floor;
  uint64_t fkey;    // the floor as a key (what these rows publish)
  // approximate statistics (needa): per lane, a compensated sum of the
  // part's 2^(x L - aLref) against a warp-uniform reference, and the lane's
  // maximum; nres counts the reference's moves
  int t0;           // the part's first tile in its row
  float aref, aLref;
  float as_hi, as_c, amx;
  int nres;
};

__device__ __forceinline__ void part_begin(const SampleArgs& a, int64_t row, int first_tile, int KC,
                                           PartState& ps) {
  ps.p = row_params(a, row);
  ps.mode = row_mode(ps.p);
  ps.needx = needs_xstats(a, ps.p, ps.mode);
  ps.needa = needs_astats(a, ps.p, ps.mode);
  ps.needy = ps.mode == kFullDraw;
  ps.K = (ps.p.top_k > 0 && ps.p.top_k < KC) ? ps.p.top_k : KC;
  ps.best_x = -INFINITY;          // a part whose values are all -inf answers its first token
  ps.best_e = first_tile * kTile;
  cand_reset(ps.cd);
  ps.published = false;
  ps.rtau = 0;
  ps.minp_floor = minp_floor_row(ps.p);
  ps.floor = -INFINITY;
  ps.fkey = 0;
  ps.t0 = first_tile;
  ps.aref = ps.aLref = -INFINITY;
  ps.as_hi = ps.as_c = 0.0f;
  ps.amx = -INFINITY;
  ps.nres = 0;
}

// The threshold a part shares with the other parts of its row: the K-th
// largest key it holds (a lower bound for the row's K-th largest key), or,
// on min-p floor rows, its floor.
__device__ __forceinline__ uint64_t part_bound(const PartState& ps) { return ps.minp_floor ? ps.fkey : ps.cd.tau; }

// Share the part's threshold with the other parts of the row, and adopt
// theirs: keys at or below the largest bound can never be selected.
// Dropping them makes the part's list incomplete ("trimmed"), except below a
// min-p floor, where the list still holds every survivor.
__device__ __forceinline__ void share_threshold(const SampleArgs& a, int64_t row, PartState& ps) {
  if (ps.published) {
    const uint64_t b = part_bound(ps);
    if ((threadIdx.x & 31) == 0 && b) atomicMax(reinterpret_cast<unsigned long long*>(&a.row_tau[row]), b);
    ps.published = false;
  }
  if (ps.rtau > ps.cd.tau) {
    ps.cd.tau = ps.rtau;
    ps.cd.tau_x = key_value(ps.rtau);
    if (!ps.minp_floor) ps.cd.trimmed = true;
  }
}

// The min-p floor as a key threshold, published like a compaction's: every
// part's floor lies below the row's min-p cut, so the largest one serves all
// parts of the row.
__device__ __forceinline__ void raise_to_floor(PartState& ps) {
  const uint64_t fk = (uint64_t)ordkey(ps.floor) << 32;
  if (ps.floor > -INFINITY && fk > ps.fkey) {
    ps.fkey = fk;
    ps.published = true;
    if (fk > ps.cd.tau) {
      ps.cd.tau = fk;
      ps.cd.tau_x = key_value(fk);
    }
  }
}

// Fill stage s of the warp's ring with tile gi by bulk copies (lane 0), when
// the tile is whole and aligned; returns whether it did (warp-uniform).
template <typename T, int KC>
__device__ __forceinline__ bool issue_tile(const SampleArgs& a, int64_t row, int tile, int s, StreamMem<KC>* wm,
                                           uint64_t pol) {
  const bool bulk = a.vec_ok && tile_valid(a, tile) == kTile && (!a.mask || a.mask_ok);
  if (bulk && (threadIdx.x & 31) == 0) {
    const uint32_t bytes = kTile * sizeof(T) + (a.mask ? 128u : 0u);
    mbar_arrive_expect_tx(&wm->bar[s], bytes);
    const T* src = reinterpret_cast<const T*>(a.logits) + row * a.row_stride + (int64_t)tile * kTile;
    bulk_copy_g2s(wm->tile[s], src, kTile * sizeof(T), &wm->bar[s], pol);
    if (a.mask) bulk_copy_g2s(wm->mask[s], a.mask + row * a.mask_stride + (int64_t)tile * 32, 128u, &wm->bar[s], pol);
  }
  return bulk;
}

// A tile that is ragged or unaligned: the warp loads it itself (padding -inf).
template <typename T, int KC>
__device__ __forceinline__ void load_tile_plain(const SampleArgs& a, int64_t row, int tile, int s,
                                                StreamMem<KC>* wm) {
  const int lane = threadIdx.x & 31;
  const int n_valid = tile_valid(a, tile);
  const T* src = reinterpret_cast<const T*>(a.logits) + row * a.row_stride + (int64_t)tile * kTile;
  T* dst = reinterpret_cast<T*>(wm->tile[s]);
  for (int e = lane; e < kTile; e += 32) {
    if constexpr (sizeof(T) == 4) dst[e] = e < n_valid ? src[e] : -INFINITY;
    else reinterpret_cast<uint16_t*>(dst)[e] = e < n_valid ? reinterpret_cast<const uint16_t*>(src)[e] : (uint16_t)0xff80u;
  }
  if (a.mask) {
    const int nw = (n_valid + 31) >> 5;
    wm->mask[s][lane] = lane < nw ? a.mask[row * a.mask_stride + (int64_t)tile * 32 + lane] : 0u;
  }
  __syncwarp();
}

// Per-tile accumulators of a warp's scan.
struct ScanAcc {
  float mx, my;        // maxima of x and of y = x * inv_temperature
  uint64_t sx, sy;     // exact sums relative to the tile maxima
};

// One value of pass PASS (1: maxima + selection, 2: x sums, 3: y sums) for
// rows of mode MODE.
template <int PASS, int MODE, int KC>
__device__ __forceinline__ void scan_value(float x, int e, int start, float mref, float inv_t, PartState& ps,
                                           ScanAcc& acc, StreamMem<KC>* wm) {
  constexpr int CAP = StreamMem<KC>::CAP;
  if constexpr (PASS == 1) {
    acc.mx = fmaxf(acc.mx, x);
    if constexpr (MODE == kFullDraw) {
      if (x > -INFINITY) acc.my = fmaxf(acc.my, fmul(x, inv_t));
    } else if constexpr (MODE == kGreedy) {
      if (x > ps.best_x) { ps.best_x = x; ps.best_e = start + e; }
    } else {
      if (cand_offer_one<CAP>(x, (uint32_t)(start + e), wm->cand, wm->hist, ps.cd, ps.K)) ps.published = true;
    }
  } else if constexpr (PASS == 2) {
    acc.sx += q52(fsub(x, mref));
  } else {
    if (x > -INFINITY) acc.sy += q52(fsub(fmul(x, inv_t), mref));
  }
}

// One pass over the staged tile in increasing token order per lane.  Dense
// when unmasked and whole; otherwise by slot over the allowed (and valid)
// slots, padded so every lane makes the same number of calls.
template <typename S, int PASS, int MODE, int KC>
__device__ __forceinline__ void scan_pass(const float* buf, bool dense, uint32_t slots, int start, float mref,
                                          float inv_t, PartState& ps, ScanAcc& acc, StreamMem<KC>* wm) {
  constexpr int VW = Vec<S>::VW;
  const int lane = threadIdx.x & 31;
  if (dense) {
#pragma unroll 2
    for (int j = 0; j < 32 / VW; ++j) {
      float x[VW];
      read_step<S>(buf, j, lane, x);
      if constexpr (PASS == 1) {
        const int e0 = j * 32 * VW + lane * VW;
        float lmax = x[0];
#pragma unroll
        for (int c = 1; c < VW; ++c) lmax = fmaxf(lmax, x[c]);
        acc.mx = fmaxf(acc.mx, lmax);
        if constexpr (MODE == kFullDraw) {
#pragma unroll
          for (int c = 0; c < VW; ++c)
            if (x[c] > -INFINITY) acc.my = fmaxf(acc.my, fmul(x[c], inv_t));
        } else if constexpr (MODE == kGreedy) {
          if (lmax > ps.best_x) {
#pragma unroll
            for (int c = 0; c < VW; ++c)
              if (x[c] > ps.best_x) { ps.best_x = x[c]; ps.best_e = start + e0 + c; }
          }
        } else {
          if (cand_offer_vec<VW, StreamMem<KC>::CAP>(x, lmax, (uint32_t)(start + e0), wm->cand, wm->hist, ps.cd,
                                                     ps.K))
            ps.published = true;
        }
      } else {
        // exact sums, two values per packed f32x2 evaluation
#pragma unroll
        for (int c = 0; c < VW; c += 2) {
          float d0, d1;
          if constexpr (PASS == 2) {
            d0 = fsub(x[c], mref);
            d1 = fsub(x[c + 1], mref);
          } else {
            d0 = fsub(x[c] > -INFINITY ? fmul(x[c], inv_t) : -INFINITY, mref);
            d1 = fsub(x[c + 1] > -INFINITY ? fmul(x[c + 1], inv_t) : -INFINITY, mref);
          }
          uint64_t q0, q1;
          q52x2(d0, d1, q0, q1);
          if constexpr (PASS == 2) acc.sx += q0 + q1;
          else acc.sy += q0 + q1;
        }
      }
    }
    return;
  }
  uint32_t rem = slots;
  int cnt = __popc(rem);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt = max(cnt, __shfl_xor_sync(kFull, cnt, o));
#pragma unroll 1
  for (int it = 0; it < cnt; ++it) {
    float x = -INFINITY;
    int e = -1;
    if (rem) {
      const int sl = __ffs(rem) - 1;
      rem &= rem - 1;
      e = slot_to_elem<VW>(sl, lane);
      x = read_elem<S>(buf, e);
    }
    scan_value<PASS, MODE, KC>(x, e, start, mref, inv_t, ps, acc, wm);
  }
}

// Exact sums over n compacted fp32 values (two per packed evaluation).
template <int PASS>
__device__ __forceinline__ uint64_t sum_compacted(const float* buf, int n, float mref, float inv_t) {
  const int lane = threadIdx.x & 31;
  uint64_t sum = 0;
  for (int i = 2 * lane; i < n; i += 64) {
    float x0 = buf[i];
    float x1 = i + 1 < n ? buf[i + 1] : -INFINITY;
    if constexpr (PASS == 3) {
      x0 = fmul(x0, inv_t);
      x1 = x1 > -INFINITY ? fmul(x1, inv_t) : -INFINITY;
    }
    uint64_t q0, q1;
    q52x2(fsub(x0, mref), fsub(x1, mref), q0, q1);
    sum += q0 + q1;
  }
  return sum;
}

// A masked (or ragged) tile: one dense pass applies the per-slot allowed
// bits, does the maxima and the selection, and compacts the allowed values
// in place at the front of the buffer (their order is irrelevant to the
// exact integer sums); the sums then run over the compacted values only.
template <int MODE, int KC>
__device__ __forceinline__ void scan_tile_masked(const SampleArgs& a, int64_t row, int tile, float* buf,
                                                 uint32_t slots, PartState& ps, StreamMem<KC>* wm) {
  constexpr int VW = 4;
  const int lane = threadIdx.x & 31;
  const int start = tile * kTile;
  const float inv_t = ps.p.inv_temperature;
  const bool compact = ps.needx || MODE == kFullDraw;
  float mx = -INFINITY, my = -INFINITY;
  int base = 0;
#pragma unroll 2
  for (int j = 0; j < 32 / VW; ++j) {
    float x[VW];
    read_step<float>(buf, j, lane, x);
    const uint32_t bits = (slots >> (j * VW)) & ((1u << VW) - 1u);
#pragma unroll
    for (int c = 0; c < VW; ++c)
      if (!((bits >> c) & 1u)) x[c] = -INFINITY;
    const int e0 = j * 32 * VW + lane * VW;
    float lmax = x[0];
#pragma unroll
    for (int c = 1; c < VW; ++c) lmax = fmaxf(lmax, x[c]);
    mx = fmaxf(mx, lmax);
    if constexpr (MODE == kFullDraw) {
#pragma unroll
      for (int c = 0; c < VW; ++c)
        if (x[c] > -INFINITY) my = fmaxf(my, fmul(x[c], inv_t));
    } else if constexpr (MODE == kGreedy) {
      if (lmax > ps.best_x) {
#pragma unroll
        for (int c = 0; c < VW; ++c)
          if (x[c] > ps.best_x) { ps.best_x = x[c]; ps.best_e = start + e0 + c; }
      }
    } else {
      if (cand_offer_vec<VW, StreamMem<KC>::CAP>(x, lmax, (uint32_t)(start + e0), wm->cand, wm->hist, ps.cd, ps.K))
        ps.published = true;
    }
    if (compact) {
      const int nv = __popc(bits);
      const int incl = warp_incl_scan(nv);
      int pos = base + incl - nv;
      __syncwarp();  // every lane has this step's values in registers
#pragma unroll
      for (int c = 0; c < VW; ++c)
        if ((bits >> c) & 1u) buf[pos++] = x[c];
      base += __shfl_sync(kFull, incl, 31);
    }
  }
  __syncwarp();
  if (ps.needx) {
    const float m = warp_max(mx);
    if (MODE == kCand && ps.minp_floor && m > -INFINITY)
      ps.floor = fmaxf(ps.floor, fsub(fadd(m, ps.p.log_min_p), 1.0f));
    uint64_t sum = 0;
    if (m > -INFINITY) sum = sum_compacted<2>(buf, base, m, inv_t);
    sum = warp_sum_u64(sum);
    if (lane == 0) { TileStat t; t.m = m; t.pad = 0; t.s = sum; a.statx[row * a.n_tiles + tile] = t; }
  }
  if constexpr (MODE == kFullDraw) {
    const float m = warp_max(my);
    uint64_t sum = 0;
    if (m > -INFINITY) sum = sum_compacted<3>(buf, base, m, inv_t);
    sum = warp_sum_u64(sum);
    if (lane == 0) { TileStat t; t.m = m; t.pad = 0; t.s = sum; a.staty[row * a.n_tiles + tile] = t; }
  }
}

// Statistics and selection of one staged tile for rows of mode MODE.
template <typename S, int MODE, int KC>
__device__ __forceinline__ void scan_tile_mode(const SampleArgs& a, int64_t row, int tile, const float* buf,
                                               bool dense, uint32_t slots, PartState& ps, StreamMem<KC>* wm) {
  const int lane = threadIdx.x & 31;
  const int start = tile * kTile;
  const float inv_t = ps.p.inv_temperature;
  ScanAcc acc;
  acc.mx = -INFINITY;
  acc.my = -INFINITY;
  acc.sx = 0;
  acc.sy = 0;
  if (MODE == kCand && dense && ps.minp_floor) {
    // min-p rows: the tile's own maximum raises the floor before its offers
    constexpr int VW = Vec<S>::VW;
    float lm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32 / VW; ++j) {
      float x[VW];
      read_step<S>(buf, j, lane, x);
#pragma unroll
      for (int c = 0; c < VW; ++c) lm = fmaxf(lm, x[c]);
    }
    const float m = warp_max(lm);
    if (m > -INFINITY) {
      ps.floor = fmaxf(ps.floor, fsub(fadd(m, ps.p.log_min_p), 1.0f));
      raise_to_floor(ps);
    }
  }
  if (MODE == kCand && dense && ps.cd.tau == 0 && ps.K <= 128) {
    // the part's first offers: the K-th largest of the tile's 128
    // quarter-lane maxima (8 values each) bounds the part's K-th largest
    // value from below, and so does its upper 16 key bits padded with zeros;
    // the offers start there instead of at nothing.  Warp search, two bits a
    // step.
    constexpr int VW = Vec<S>::VW;
    constexpr int SPQ = 8 / VW;  // steps per quarter (fp32: 2, bf16: 1)
    float h[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 32 / VW; ++j) {
      float x[VW];
      read_step<S>(buf, j, lane, x);
#pragma unroll
      for (int c = 0; c < VW; ++c) h[j / SPQ] = fmaxf(h[j / SPQ], x[c]);
    }
    uint32_t kq[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) kq[q] = h[q] > -INFINITY ? ordkey(h[q]) >> 16 : 0u;
    uint32_t T = 0;
#pragma unroll
    for (int b = 14; b >= 0; b -= 2) {
      const uint32_t c1 = T | (1u << b), c2 = T | (2u << b), c3 = T | (3u << b);
      unsigned n1 = 0, n2 = 0, n3 = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        n1 += kq[q] >= c1 ? 1u : 0u;
        n2 += kq[q] >= c2 ? 1u : 0u;
        n3 += kq[q] >= c3 ? 1u : 0u;
      }
      const uint32_t d = ((int)__reduce_add_sync(kFull, n1) >= ps.K ? 1u : 0u) +
                         ((int)__reduce_add_sync(kFull, n2) >= ps.K ? 1u : 0u) +
                         ((int)__reduce_add_sync(kFull, n3) >= ps.K ? 1u : 0u);
      T |= d << b;
    }
    if (T) {
      ps.cd.tau = (uint64_t)(T << 16) << 32;
      ps.cd.tau_x = key_value(ps.cd.tau);
      ps.cd.trimmed = true;
      ps.published = true;
    }
  }
  scan_pass<S, 1, MODE, KC>(buf, dense, slots, start, 0.0f, inv_t, ps, acc, wm);
  if (ps.needx) {
    const float m = warp_max(acc.mx);
    if (MODE == kCand && ps.minp_floor && m > -INFINITY)
      ps.floor = fmaxf(ps.floor, fsub(fadd(m, ps.p.log_min_p), 1.0f));
    if (m > -INFINITY) scan_pass<S, 2, MODE, KC>(buf, dense, slots, start, m, inv_t, ps, acc, wm);
    const uint64_t sum = warp_sum_u64(acc.sx);
    if (lane == 0) { TileStat t; t.m = m; t.pad = 0; t.s = sum; a.statx[row * a.n_tiles + tile] = t; }
  }
  if constexpr (MODE == kFullDraw) {
    const float m = warp_max(acc.my);
    if (m > -INFINITY) scan_pass<S, 3, MODE, KC>(buf, dense, slots, start, m, inv_t, ps, acc, wm);
    const uint64_t sum = warp_sum_u64(acc.sy);
    if (lane == 0) { TileStat t; t.m = m; t.pad = 0; t.s = sum; a.staty[row * a.n_tiles + tile] = t; }
  }
}

// Offers of a staged tile to the part's candidate buffer: each lane marks
// its values at or above the threshold value (slot layout of read_step), one
// warp scan sizes the appends, and each lane writes the keys of its marks.
// A value equal to the threshold value whose key does not beat the threshold
// leaves a zero key, squeezed out before the count is committed.  When the
// marks would overflow the buffer even after a compaction (a first tile of
// near-equal values), the tile is offered step by step instead.
template <typename S, int KC>
__device__ __forceinline__ uint32_t mark_tile(const float* buf, float tau_x) {
  constexpr int VW = Vec<S>::VW;
  const int lane = threadIdx.x & 31;
  uint32_t mk = 0;
#pragma unroll
  for (int j = 0; j < 32 / VW; ++j) {
    float x[VW];
    read_step<S>(buf, j, lane, x);
#pragma unroll
    for (int c = 0; c < VW; ++c)
      if (x[c] > -INFINITY && x[c] >= tau_x) mk |= 1u << (j * VW + c);
  }
  return mk;
}

template <typename S, int KC>
__device__ __forceinline__ void offer_tile(const float* buf, int start, PartState& ps, StreamMem<KC>* wm) {
  constexpr int VW = Vec<S>::VW;
  constexpr int CAP = StreamMem<KC>::CAP;
  const int lane = threadIdx.x & 31;
  uint32_t mk = mark_tile<S, KC>(buf, ps.cd.tau_x);
  int total = (int)__reduce_add_sync(kFull, (unsigned)__popc(mk));
  if (ps.cd.cnt + total > CAP && ps.cd.cnt > ps.K) {
    cand_compact<CAP>(wm->cand, wm->hist, ps.cd, ps.K);
    ps.published = true;
    mk = mark_tile<S, KC>(buf, ps.cd.tau_x);
    total = (int)__reduce_add_sync(kFull, (unsigned)__popc(mk));
  }
  if (ps.cd.cnt + total > CAP) {
#pragma unroll 1
    for (int j = 0; j < 32 / VW; ++j) {
      float x[VW];
      read_step<S>(buf, j, lane, x);
      float lmax = x[0];
#pragma unroll
      for (int c = 1; c < VW; ++c) lmax = fmaxf(lmax, x[c]);
      if (cand_offer_vec<VW, CAP>(x, lmax, (uint32_t)(start + j * 32 * VW + lane * VW), wm->cand, wm->hist, ps.cd,
                                  ps.K))
        ps.published = true;
    }
    return;
  }
  const int n = __popc(mk);
  const int c0 = ps.cd.cnt;
  int pos = c0 + warp_incl_scan(n) - n;
  bool hole = false;
  while (mk) {
    const int sl = __ffs(mk) - 1;
    mk &= mk - 1;
    const int e = slot_to_elem<VW>(sl, lane);
    const uint64_t key = rankkey(read_elem<S>(buf, e), (uint32_t)(start + e));
    const bool ok = key > ps.cd.tau;
    hole |= !ok;
    wm->cand[pos++] = ok ? key : 0ull;
  }
  __syncwarp();
  if (__any_sync(kFull, hole)) {
    const unsigned below = (1u << lane) - 1u;
    int w = c0;
    for (int r0 = c0; r0 < c0 + total; r0 += 32) {
      const int i = r0 + lane;
      const uint64_t k = i < c0 + total ? wm->cand[i] : 0ull;
      const unsigned bal = __ballot_sync(kFull, k != 0ull);
      __syncwarp();
      if (k) wm->cand[w + __popc(bal & below)] = k;
      w += __popc(bal);
      __syncwarp();
    }
    total = w - c0;
  }
  ps.cd.cnt = c0 + total;
  if (ps.cd.cnt > ps.K + 128) {
    cand_compact<CAP>(wm->cand, wm->hist, ps.cd, ps.K);
    ps.published = true;
  }
}

// One lane's approximate partial of a tile held in registers: the sum of
// ex2(fl(x L - aLref)) over its 32 values, added pairwise in fp32 -- four
// levels over the f32x2 halves, then the two halves.
__device__ __forceinline__ float approx_lane_sum(const float (&v)[32], float aLref) {
  const uint64_t L2 = pk(kLog2eF, kLog2eF), M2 = pk(-aLref, -aLref);
  uint64_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint64_t t = fma2(pk(v[2 * i], v[2 * i + 1]), L2, M2);
    w[i] = pk(ex2_approx(lo_f(t)), ex2_approx(hi_f(t)));
  }
#pragma unroll
  for (int h = 8; h >= 1; h >>= 1)
#pragma unroll
    for (int i = 0; i < h; ++i) w[i] = add2(w[i], w[i + h]);
  return fadd(lo_f(w[0]), hi_f(w[0]));
}

// A tile's share of the part's approximate statistics (lm: the lane's
// maximum of the tile).  The reference is the first finite tile maximum; it
// moves up (the sums rescaled by the hardware ex2 of the step) when a value
// would sit more than 2^64 above it.  A non-finite reference poisons the sum
// (NaN), which sends the row to the exact pass.
__device__ __forceinline__ void approx_tile(const float (&v)[32], float lm, PartState& ps) {
  if (!(ps.aLref > -INFINITY)) {
    const float m = warp_max(lm);
    if (!(m > -INFINITY)) return;  // nothing finite yet
    ps.aref = m;
    ps.aLref = fmul(m, kLog2eF);
    if (!(m < INFINITY)) ps.as_hi = __int_as_float(0x7fc00000);
  } else if (__any_sync(kFull, ffma(lm, kLog2eF, -ps.aLref) > 64.0f)) {
    const float m = warp_max(lm);
    const float nL = fmul(m, kLog2eF);
    const float f = ex2_approx(fsub(ps.aLref, nL));
    ps.as_hi = fmul(ps.as_hi, f);
    ps.as_c = fmul(ps.as_c, f);
    ps.aref = m;
    ps.aLref = nL;
    ps.nres += 1;
    if (!(m < INFINITY)) ps.as_hi = __int_as_float(0x7fc00000);
  }
  // Kahan summation of the tile partials
  const float t = approx_lane_sum(v, ps.aLref);
  const float y = fsub(t, ps.as_c);
  const float u = fadd(ps.as_hi, y);
  ps.as_c = fsub(fsub(u, ps.as_hi), y);
  ps.as_hi = u;
  ps.amx = fmaxf(ps.amx, lm);
}

// The part's approximate statistics at its end (lane 0 writes them to the
// slot of its first tile).  Relative error bound of s, with N <= 8192
// values a lane (A = 25: N A 2^-A < 0.01 of the largest term):
//   hardware ex2                                 2^-20
//   exponent arguments, |rho| <= 2^-24 |a| and
//   sum v|a| <= (A + 0.01 + |a_top|) s           2^-24 ln2 (25.01 + |a_top|)
//   L != log2 e, |x| <= |m_part| + A / L          1.4e-8 (|m_part| + 18)
//   four-level tree, halves, Kahan                8 2^-24
//   each move of the reference                    1.2e-6, and |a| up to 64 + A
// (a_top: the part maximum's argument against the final reference).
__device__ __forceinline__ void approx_part_end(const SampleArgs& a, int64_t row, const PartState& ps) {
  double s = (double)ps.as_hi + (double)ps.as_c;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = dadd(s, __shfl_xor_sync(kFull, s, o));
  const float mp = warp_max(ps.amx);
  if ((threadIdx.x & 31) == 0) {
    const float atop = fabsf(ffma(mp, kLog2eF, -ps.aLref));
    const float argb = ps.nres ? 64.0f + 25.01f : 25.01f + atop;
    ApproxStat st;
    st.mref = ps.aref;
    st.eps = (float)(0x1p-20 + 0x1p-24 * 0.6931471805599453 * (double)argb +
                     1.4e-8 * ((double)fabsf(mp) + 18.0) + 8.0 * 0x1p-24 + 1.2e-6 * ps.nres);
    st.s = ps.aLref > -INFINITY ? s : 0.0;
    reinterpret_cast<ApproxStat*>(a.staty)[row * a.n_tiles + ps.t0] = st;
  }
}

// A whole (or -inf padded ragged) unmasked tile of a filtered row, values of
// type S in buf: the tile in registers, its maxima and its exact or
// approximate statistics; then the first-tile bound and the offers, which
// re-read the staged tile (rarely: most tiles hold nothing above the
// threshold).
template <typename S, int KC>
__device__ __forceinline__ void scan_dense_cand(const SampleArgs& a, int64_t row, int tile, const float* buf,
                                                PartState& ps, StreamMem<KC>* wm) {
  constexpr int VW = Vec<S>::VW;
  const int lane = threadIdx.x & 31;
  const int start = tile * kTile;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32 / VW; ++j) {
    float x[VW];
    read_step<S>(buf, j, lane, x);
#pragma unroll
    for (int c = 0; c < VW; ++c) v[j * VW + c] = x[c];
  }
  // quarter maxima: quarter q of a lane is its slots 8q .. 8q + 7
  float h[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float a0 = fmaxf(v[8 * q], v[8 * q + 1]), a1 = fmaxf(v[8 * q + 2], v[8 * q + 3]);
    const float a2 = fmaxf(v[8 * q + 4], v[8 * q + 5]), a3 = fmaxf(v[8 * q + 6], v[8 * q + 7]);
    h[q] = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
  }
  const float lm = fmaxf(fmaxf(h[0], h[1]), fmaxf(h[2], h[3]));
  float m = -INFINITY;
  if (ps.needx || ps.minp_floor) m = warp_max(lm);
  if (ps.minp_floor && m > -INFINITY) {
    // min-p rows: the tile's own maximum raises the floor before its offers
    ps.floor = fmaxf(ps.floor, fsub(fadd(m, ps.p.log_min_p), 1.0f));
    raise_to_floor(ps);
  }
  if (ps.needx) {
    uint64_t sum = 0;
    if (m > -INFINITY) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        uint64_t q0, q1;
        q52x2(fsub(v[2 * i], m), fsub(v[2 * i + 1], m), q0, q1);
        sum += q0 + q1;
      }
    }
    sum = warp_sum_u64(sum);
    if (lane == 0) { TileStat t; t.m = m; t.pad = 0; t.s = sum; a.statx[row * a.n_tiles + tile] = t; }
  } else if (ps.needa) {
    approx_tile(v, lm, ps);
  }
  if (ps.cd.tau == 0 && ps.K <= 128) {
    // the part's first offers: the K-th largest of the tile's 128 quarter
    // maxima bounds the part's K-th largest value from below, and so does its
    // upper 16 key bits padded with zeros; the offers start there instead of
    // at nothing.  Warp search, two bits a step.
    uint32_t kq[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) kq[q] = h[q] > -INFINITY ? ordkey(h[q]) >> 16 : 0u;
    uint32_t T = 0;
#pragma unroll
    for (int b = 14; b >= 0; b -= 2) {
      const uint32_t c1 = T | (1u << b), c2 = T | (2u << b), c3 = T | (3u << b);
      unsigned n1 = 0, n2 = 0, n3 = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        n1 += kq[q] >= c1 ? 1u : 0u;
        n2 += kq[q] >= c2 ? 1u : 0u;
        n3 += kq[q] >= c3 ? 1u : 0u;
      }
      const uint32_t d = ((int)__reduce_add_sync(kFull, n1) >= ps.K ? 1u : 0u) +
                         ((int)__reduce_add_sync(kFull, n2) >= ps.K ? 1u : 0u) +
                         ((int)__reduce_add_sync(kFull, n3) >= ps.K ? 1u : 0u);
      T |= d << b;
    }
    if (T) {
      ps.cd.tau = (uint64_t)(T << 16) << 32;
      ps.cd.tau_x = key_value(ps.cd.tau);
      ps.cd.trimmed = true;
      ps.published = true;
    }
  }
  if (__any_sync(kFull, lm > -INFINITY && lm >= ps.cd.tau_x)) offer_tile<S, KC>(buf, start, ps, wm);
}

// Statistics and candidate search of one staged tile, values of type S in buf.
template <typename S, int KC>
__device__ __forceinline__ void scan_tile(const SampleArgs& a, int64_t row, int tile, float* buf,
                                          const uint32_t* mw, PartState& ps, StreamMem<KC>* wm) {
  const int lane = threadIdx.x & 31;
  const int n_valid = tile_valid(a, tile);
  const bool masked = a.mask != nullptr;
  if (!masked && ps.mode == kCand) {
    // ragged tiles too: the staged buffer is padded with -inf
    scan_dense_cand<S, KC>(a, row, tile, buf, ps, wm);
    return;
  }
  if (!masked && n_valid == kTile) {
    if (ps.mode == kGreedy) scan_tile_mode<S, kGreedy, KC>(a, row, tile, buf, true, ~0u, ps, wm);
    else if (ps.mode == kCand) scan_tile_mode<S, kCand, KC>(a, row, tile, buf, true, ~0u, ps, wm);
    else scan_tile_mode<S, kFullDraw, KC>(a, row, tile, buf, true, ~0u, ps, wm);
    return;
  }
  // masked or ragged: fp32 slots (a bf16 tile is widened in place first)
  if constexpr (sizeof(S) == 2) expand_bf16_in_place(buf);
  constexpr int VW = 4;
  uint32_t slots = masked ? slot_mask<VW>(mw) : 0xffffffffu;
  if (n_valid < kTile) {
    uint32_t keep = 0;
#pragma unroll
    for (int sl = 0; sl < 32; ++sl)
      if (slot_to_elem<VW>(sl, lane) < n_valid) keep |= 1u << sl;
    slots &= keep;
  }
  int busiest = __popc(slots);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) busiest = max(busiest, __shfl_xor_sync(kFull, busiest, o));
  if (busiest <= 12) {
    // few allowed values: visit them slot by slot
    if (ps.mode == kGreedy) scan_tile_mode<float, kGreedy, KC>(a, row, tile, buf, false, slots, ps, wm);
    else if (ps.mode == kCand) scan_tile_mode<float, kCand, KC>(a, row, tile, buf, false, slots, ps, wm);
    else scan_tile_mode<float, kFullDraw, KC>(a, row, tile, buf, false, slots, ps, wm);
    return;
  }
  if (ps.mode == kGreedy) scan_tile_masked<kGreedy, KC>(a, row, tile, buf, slots, ps, wm);
  else if (ps.mode == kCand) scan_tile_masked<kCand, KC>(a, row, tile, buf, slots, ps, wm);
  else scan_tile_masked<kFullDraw, KC>(a, row, tile, buf, slots, ps, wm);
}

// End of a row part: publish its candidates (or its argmax) for the merge.
template <typename T, int KC>
__device__ __forceinline__ void part_end(const SampleArgs& a, int64_t row, int64_t gw, PartState& ps,
                                         StreamMem<KC>* wm) {
  constexpr int CAP = StreamMem<KC>::CAP;
  const int lane = threadIdx.x & 31;
  const int64_t total = a.rows * a.n_tiles;
  const int part = (int)(gw - owner_warp(row * a.n_tiles, total, a.n_warps));
  if (ps.mode == kGreedy) {
    const uint64_t k = rankkey(ps.best_x, (uint32_t)ps.best_e);
    const uint64_t wk = warp_max_u64(k);
    if (lane == 0) a.best[row * a.max_parts + part] = wk;
    if (a.merge_greedy) {
      // the last part of the row to finish merges it (its own key and
      // statistics are ordered before the count by the fence; the others'
      // before theirs)
      const int n_parts = (int)(owner_warp((row + 1) * a.n_tiles - 1, total, a.n_warps) -
                                owner_warp(row * a.n_tiles, total, a.n_warps) + 1);
      int last = 0;
      if (lane == 0) {
        __threadfence();
        const unsigned long long done = atomicAdd(reinterpret_cast<unsigned long long*>(&a.row_tau[row]), 1ull);
        last = done == (unsigned long long)(n_parts - 1);
        __threadfence();
      }
      last = __shfl_sync(kFull, last, 0);
      if (last) {
        uint64_t bk = 0;
        for (int i = lane; i < n_parts; i += 32) {
          const uint64_t kk = ld_cg(&a.best[row * a.max_parts + i]);
          bk = kk > bk ? kk : bk;
        }
        bk = warp_max_u64(bk);
        float c = __int_as_float(0x7fc00000);
        if (needs_xstats(a, ps.p, kGreedy)) {
          float mx;
          c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &mx);
        }
        if (lane == 0) write_row(a, row, kGreedy, (int)key_index(bk), key_value(bk), c, 0);
      }
    }
  } else if (ps.mode == kCand) {
    if (ps.needa) approx_part_end(a, row, ps);
    if (ps.cd.cnt > ps.K) cand_compact<CAP>(wm->cand, wm->hist, ps.cd, ps.K);
    // the part's final threshold bounds the row's K-th key (or its min-p
    // cut) from below: the merge starts from the largest one
    const uint64_t b = part_bound(ps);
    if (lane == 0 && b) atomicMax(reinterpret_cast<unsigned long long*>(&a.row_tau[row]), b);
    if (lane == 0) a.best[row * a.max_parts + part] = ps.cd.ctau;
    uint64_t* dst = a.cand + (row * a.max_parts + part) * (int64_t)KC;
    for (int i = lane; i < ps.cd.cnt; i += 32) dst[i] = wm->cand[i];
    if (lane == 0) a.cand_n[row * a.max_parts + part] = ps.cd.cnt | (ps.cd.trimmed ? (1 << 30) : 0);
  }
  __syncwarp();
}

// Merge of every row's parts: one CTA (8 warps) per row.  Launched after
// the streaming kernel on the same stream (programmatic dependent launch: it
// may start while the streaming kernel drains, and waits for its results).
// For a filtered row each warp folds every eighth part's candidates into
// its own top-K buffer, the CTA radix-selects the row's top-K from the eight
// lists, warp 0 finishes the log-sum-exp while the other warps compute the
// candidates' Gumbel scores, and warp 0 filters and draws.  Greedy and
// whole-vocabulary rows are merged by warp 0 alone.
template <int KC>
struct MergeCta {
  static constexpr int CAP = StreamMem<KC>::CAP;
  uint64_t cand[8][CAP];
  unsigned hist[8][256];
  uint64_t u[8 * KC];
  uint64_t carry[KC];
  float score[KC];
  unsigned mhist[256];
  int scal[8];
  int wcnt[8];
  int wtrim[8];
  float lse, lse_hi;  // exact log-sum-exp, or the bracket [lse, lse_hi]
  int bracket_ok;
};

template <typename T, int KC>
__global__ void __launch_bounds__(256) k_row_merge_cta(const __grid_constant__ SampleArgs a) {
  using M = MergeCta<KC>;
  constexpr int CAP = M::CAP;
  extern __shared__ __align__(128) unsigned char smem_merge[];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  M* mc = reinterpret_cast<M*>(smem_merge);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t total = a.rows * a.n_tiles;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int n_parts = a.fixed_parts > 0 ? a.fixed_parts
                                          : (int)(owner_warp((row + 1) * a.n_tiles - 1, total, a.n_warps) -
                                                  owner_warp(row * a.n_tiles, total, a.n_warps) + 1);
    const pm_row_params p = row_params(a, row);
    const int mode = row_mode(p);
    if (mode == kFullDraw) {
      // whole-vocabulary draw: warp 0 the log-sum-exp (when asked), warp 1
      // the tile; then all eight warps the tile's q52 masses (four slots a
      // lane each, stored by token index) and a block scan for the token
      constexpr int VW = Lay<T>::VW;
      uint64_t* qbuf = &mc->cand[0][0];                            // [1024] masses
      float* xbuf = reinterpret_cast<float*>(&mc->cand[0][0] + kTile);  // [1024] processed logits
      const bool needx = needs_xstats(a, p, mode);
      if (wid == 0 && needx) {
        float mx;
        const float c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &mx);
        if (lane == 0) mc->lse = c;
      } else if (wid == 1) {
        float mt;
        uint64_t t2;
        const int tt = warp_full_pick(a, row, &mt, &t2);
        if (lane == 0) {
          mc->scal[0] = tt;
          mc->scal[1] = tt >= 0 ? tt * kTile : 0;
          mc->scal[2] = __float_as_int(mt);
          mc->scal[3] = __float_as_int(-INFINITY);
          mc->u[0] = t2;
        }
      }
      __syncthreads();
      const int tt = mc->scal[0];
      if (tt >= 0) {
        const float mt = __int_as_float(mc->scal[2]);
        TileIn ti;
        load_tile<T>(a, row, tt, ti);
        process_tile_regs<VW>(a, p, row, tt, ti);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int sl = wid * 4 + k4;
          const int e = slot_elem<VW>(sl, lane);
          const float x = ti.v[sl];
          const float y = x > -INFINITY ? fmul(x, p.inv_temperature) : -INFINITY;
          qbuf[e] = q52(fsub(y, mt));
          xbuf[e] = x;
        }
        __syncthreads();
        uint64_t loc = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) loc += qbuf[4 * tid + c];
        const uint64_t wincl = warp_incl_scan_u64(loc);
        if (lane == 31) mc->u[1 + wid] = wincl;
        __syncthreads();
        uint64_t base = 0;
        for (int w = 0; w < wid; ++w) base += mc->u[1 + w];
        const uint64_t excl = base + wincl - loc;
        const uint64_t t2 = mc->u[0];
        if (excl <= t2 && t2 < excl + loc) {
          uint64_t run = excl;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            run += qbuf[4 * tid + c];
            if (run > t2) {
              mc->scal[1] = tt * kTile + 4 * tid + c;
              mc->scal[3] = __float_as_int(xbuf[4 * tid + c]);
              break;
            }
          }
        }
      }
      __syncthreads();
      if (tid == 0)
        write_row(a, row, mode, mc->scal[1], __int_as_float(mc->scal[3]), needx ? mc->lse : __int_as_float(0x7fc00000),
                  0);
      __syncthreads();
      continue;
    }
    if (mode != kCand) {
      if (wid == 0) {
        float x_tok, lse;
        int ns;
        const int tok = warp_row_merge<T, KC, CAP>(a, row, n_parts, mc->cand[0], mc->hist[0], &x_tok, &lse, &ns);
        if (lane == 0) write_row(a, row, mode, tok, x_tok, lse, ns);
      }
      __syncthreads();
      continue;
    }
    const int K = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;
    const bool needx = needs_xstats(a, p, mode);
    const bool needa = needs_astats(a, p, mode);
    // Rows of many short part lists (the fused LM-head pass: one part per
    // 128 ids): every count in one load per thread, a block scan, every key
    // copied into the fold buffers, one block radix select of the top K.
    // Keys below the row's shared bound may come along; they cannot reach
    // the top K, since at least K listed keys lie at or above it.  Longer
    // lists fall back to the per-warp fold below.
    int ncarry = 0;
    bool dropped = false;
    bool gathered = false;
    if (a.fixed_parts > 0) {
      uint64_t* U = &mc->cand[0][0];
      constexpr int kUcap = 8 * CAP;
      if (wid == 0) {
        if (needx) {
          float mx;
          const float c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &mx);
          if (lane == 0) mc->lse = c;
        }
      } else {
        // warps 1..7: part q = (wid - 1) * 32 + lane + 224 i
        int mine = 0;
        bool trim = false;
        for (int q = tid - 32; q < n_parts; q += 224) {
          const int raw = ld_cg(&a.cand_n[row * a.max_parts + q]);
          mine += raw & 0x3fffffff;
          trim |= ((raw >> 30) & 1) != 0;
        }
        const int incl = warp_incl_scan(mine);
        if (lane == 31) mc->wcnt[wid] = incl;
        const bool wt = __any_sync(kFull, trim) != 0;
        if (lane == 0) mc->wtrim[wid] = wt;
        mine = incl - mine;  // this thread's offset within its warp
        // stash the offset in the carry's score slots until the scan is done
        reinterpret_cast<int*>(mc->u)[tid] = mine;
      }
      __syncthreads();
      int tot = 0;
      int wbase[8];
#pragma unroll
      for (int w = 1; w < 8; ++w) {
        wbase[w] = tot;
        tot += mc->wcnt[w];
      }
      bool trim_any = false;
#pragma unroll
      for (int w = 1; w < 8; ++w) trim_any |= mc->wtrim[w] != 0;
      gathered = tot <= kUcap;
      if (gathered) {
        if (wid > 0) {
          int o = wbase[wid] + reinterpret_cast<int*>(mc->u)[tid];
          for (int q = tid - 32; q < n_parts; q += 224) {
            const int n = ld_cg(&a.cand_n[row * a.max_parts + q]) & 0x3fffffff;
            const uint64_t* src = a.cand + (row * a.max_parts + q) * (int64_t)KC;
            for (int i = 0; i < n; ++i) U[o + i] = ld_cg(&src[i]);
            o += n;
          }
        }
        __syncthreads();
        ncarry = block_topk_sorted(U, tot, K, mc->carry, KC, mc->mhist, mc->scal);
        dropped = trim_any || tot > K;
        __syncthreads();
      }
    }
    if (!gathered) {
    // 1. warp 0: the row log-sum-exp (or its bracket).  Warps 1..7 (fw = wid - 1): parts fw,
    //    fw + 7, ... into their own top-K, from the row's shared threshold; a
    //    round takes 32 of the warp's parts at once (lane i: part
    //    fw + 7 (p0 + i)), their keys flattened and loaded eight per lane in
    //    flight
    if (wid == 0) {
      if (needx) {
        float mx;
        const float c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &mx);
        if (lane == 0) mc->lse = c;
      } else if (needa) {
        float lo = __int_as_float(0x7fc00000), hi = __int_as_float(0x7fc00000);
        const bool ok = warp_bracket(a, row, n_parts, &lo, &hi);
        if (lane == 0) { mc->lse = lo; mc->lse_hi = hi; mc->bracket_ok = ok; }
      }
      if (lane == 0) { mc->wcnt[0] = 0; mc->wtrim[0] = 0; }
    } else {
      const int fw = wid - 1;
      Cand cd;
      cand_reset(cd);
      const bool minp = minp_floor_row(p);
      const uint64_t rt = ld_cg(&a.row_tau[row]);
      if (rt) {
        cd.tau = merge_floor(rt);
        cd.tau_x = key_value(rt);
        cd.trimmed = !minp;
      }
      bool trimmed = false;
      const int mine_n = n_parts > fw ? (n_parts - fw + 6) / 7 : 0;
      for (int p0 = 0; p0 < mine_n; p0 += 32) {
        const int part = fw + 7 * (p0 + lane);
        const int raw = p0 + lane < mine_n ? ld_cg(&a.cand_n[row * a.max_parts + part]) : 0;
        trimmed |= __any_sync(kFull, part_trimmed(a, row, part, raw, minp, rt)) != 0;
        const int n = raw & 0x3fffffff;
        const int incl = warp_incl_scan(n);
        const int tot = __shfl_sync(kFull, incl, 31);
        for (int f0 = 0; f0 < tot; f0 += 256) {
          uint64_t keys[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int f = f0 + u * 32 + lane;
            int q = 0;  // lanes whose inclusive prefix is <= f
#pragma unroll
            for (int st = 16; st > 0; st >>= 1) {
              const int v = __shfl_sync(kFull, incl, (q + st - 1) & 31);
              if (q + st - 1 < 32 && v <= f) q += st;
            }
            const int qi = q < 32 ? q : 31;
            const int iq = __shfl_sync(kFull, incl, qi);
            const int nq = __shfl_sync(kFull, n, qi);
            keys[u] = 0ull;
            if (f < tot) {
              const uint64_t* src = a.cand + (row * a.max_parts + fw + 7 * (p0 + qi)) * (int64_t)KC;
              keys[u] = ld_cg(&src[f - (iq - nq)]);
            }
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) cand_offer_key<CAP>(keys[u], mc->cand[wid], mc->hist[wid], cd, K);
        }
      }
      if (cd.cnt > K) cand_compact<CAP>(mc->cand[wid], mc->hist[wid], cd, K);
      for (int i = lane; i < cd.cnt; i += 32) mc->u[wid * KC + i] = mc->cand[wid][i];
      if (lane == 0) { mc->wcnt[wid] = cd.cnt; mc->wtrim[wid] = trimmed || cd.trimmed; }
    }
    __syncthreads();
    // 2. the eight lists end to end, then the row's top-K sorted into the carry
    int tot = 0, start[8];
    dropped = false;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      start[w] = tot;
      tot += mc->wcnt[w];
      dropped |= mc->wtrim[w] != 0;
    }
    uint64_t mine[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) mine[w] = tid < mc->wcnt[w] ? mc->u[w * KC + tid] : 0ull;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < 8; ++w)
      if (tid < mc->wcnt[w]) mc->u[start[w] + tid] = mine[w];
    __syncthreads();
    dropped |= tot > K;
    if (tot <= 512) {
      // few keys: rank each by counting the larger ones (unique keys), the K
      // largest land sorted in the carry
      for (int i = tid; i < tot; i += 256) {
        const uint64_t k = mc->u[i];
        int rank = 0;
#pragma unroll 8
        for (int j = 0; j < tot; ++j) rank += mc->u[j] > k;
        if (rank < K) mc->carry[rank] = k;
      }
      ncarry = tot < K ? tot : K;
    } else {
      ncarry = block_topk_sorted(mc->u, tot, K, mc->carry, KC, mc->mhist, mc->scal);
    }
    __syncthreads();
    }
    // 3. the Gumbel scores of the row's top-K
    for (int r = tid; r < ncarry; r += 256)
      mc->score[r] = fadd(fmul(key_value(mc->carry[r]), p.inv_temperature), row_gumbel(a, row, key_index(mc->carry[r])));
    __syncthreads();
    // 4. filters and draw
    if (wid == 0) {
      const float c = (needx || needa) ? mc->lse : __int_as_float(0x7fc00000);
      const float c_hi = needa ? mc->lse_hi : __int_as_float(0x7fc00000);
      int ns = 0;
      float x_tok = -INFINITY;
      const int tok = (needa && !mc->bracket_ok)
                          ? -2
                          : warp_filter_draw(a, p, row, mc->carry, ncarry, !dropped, c, &ns, mc->score, &x_tok, c_hi);
      if (tok == -2) queue_exact<KC>(a, row, mc->carry, ncarry);
      if (tok >= 0 && a.surv_ids && lane == 0) write_survivors(a, p, row, mc->carry, ns);
      if (lane == 0) write_row(a, row, mode, tok, x_tok, needa ? __int_as_float(0x7fc00000) : c, ns);
    }
    __syncthreads();
  }
}

// Merge with one warp per row: for many rows with few parts each.
template <typename T, int KC>
__global__ void __launch_bounds__(256) k_row_merge_warp(const __grid_constant__ SampleArgs a) {
  constexpr int CAP = StreamMem<KC>::CAP;
  struct MergeMem {
    uint64_t cand[CAP];
    unsigned hist[256];
  };
  extern __shared__ __align__(128) unsigned char smem_mwarp[];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  MergeMem* mm = reinterpret_cast<MergeMem*>(smem_mwarp) + wid;
  const int64_t total = a.rows * a.n_tiles;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + wid; row < a.rows;
       row += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int n_parts = a.fixed_parts > 0 ? a.fixed_parts
                                          : (int)(owner_warp((row + 1) * a.n_tiles - 1, total, a.n_warps) -
                                                  owner_warp(row * a.n_tiles, total, a.n_warps) + 1);
    float x_tok, lse;
    int ns;
    const int tok = warp_row_merge<T, KC, CAP>(a, row, n_parts, mm->cand, mm->hist, &x_tok, &lse, &ns);
    if (lane == 0) write_row(a, row, row_mode(row_params(a, row)), tok, x_tok, lse, ns);
    __syncwarp();
  }
}

// The exact pass over the rows whose top-p cut the bracket left open (queued
// by the merges): the grid's warps take the queued rows' tiles in turn and
// write their exact statistics; the warp that writes a row's last tile (a
// counter per queue entry) finishes the row as the merge would have with the
// exact log-sum-exp -- the cut over the row's saved top candidates, the
// draw, the outputs.  With an empty queue every CTA returns after one load.
template <typename T, int KC>
struct ExactMem {
  float wbuf[kTile];
  uint64_t S[KC];
};

template <typename T, int KC>
__global__ void __launch_bounds__(256) k_row_exact(const __grid_constant__ SampleArgs a) {
  constexpr int VW = Lay<T>::VW;
  extern __shared__ __align__(128) unsigned char smem_exact[];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int n = ld_cg(&a.exact_q[0]);
  if (n == 0) return;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  ExactMem<T, KC>* xm = reinterpret_cast<ExactMem<T, KC>*>(smem_exact) + wid;
  int32_t* done = a.exact_q + 1;
  const int32_t* queue = a.exact_q + 1 + a.rows;
  const int64_t total = (int64_t)n * a.n_tiles;
  for (int64_t g = (int64_t)blockIdx.x * 8 + wid; g < total; g += (int64_t)gridDim.x * 8) {
    const int q = (int)(g / a.n_tiles);
    const int t = (int)(g - (int64_t)q * a.n_tiles);
    const int64_t row = ld_cg(&queue[q]);
    const pm_row_params p = row_params(a, row);
    TileIn ti;
    load_tile<T>(a, row, t, ti);
    process_tile<VW>(a, p, row, t, ti, xm->wbuf);
    float m;
    uint64_t s;
    tile_stats(ti.v, &m, &s);
    if (lane == 0) {
      TileStat st;
      st.m = m;
      st.pad = 0;
      st.s = s;
      a.statx[row * a.n_tiles + t] = st;
    }
    __threadfence();
    int prev = 0;
    if (lane == 0) prev = atomicAdd(&done[q], 1);
    prev = __shfl_sync(kFull, prev, 0);
    if (prev != a.n_tiles - 1) continue;
    __threadfence();
    float mx;
    const float c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &mx);
    const int nc = ld_cg(&a.cand_n[row * a.max_parts]);
    const uint64_t* src = a.cand + row * a.max_parts * (int64_t)KC;
    for (int i = lane; i < nc; i += 32) xm->S[i] = ld_cg(&src[i]);
    __syncwarp();
    int ns = 0;
    float x_tok = -INFINITY;
    const int tok = warp_filter_draw(a, p, row, xm->S, nc, true, c, &ns, nullptr, &x_tok);
    if (tok >= 0 && a.surv_ids && lane == 0) write_survivors(a, p, row, xm->S, ns);
    if (lane == 0) write_row(a, row, kCand, tok, x_tok, c, ns);
    __syncwarp();
  }
}

// Largest relative error of ex2_approx over every fp32 a in [-126, 1]
// against the fp64 2^a: a grid-stride walk over the bit patterns of
// [-126, -0] and of [+0, 1]; the maximum (a non-negative double, so its bits
// order like unsigned integers) is folded in with one atomicMax per warp.
__global__ void __launch_bounds__(256) k_selfcheck_ex2(unsigned long long* out) {
  const uint32_t neg_lo = 0x80000000u, neg_hi = 0xC2FC0000u;  // -0 .. -126
  const uint32_t pos_hi = 0x3F800000u;                        // +0 .. 1
  const uint64_t n_neg = (uint64_t)(neg_hi - neg_lo) + 1, n_all = n_neg + (uint64_t)pos_hi + 1;
  double worst = 0.0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_all;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t bits = i < n_neg ? neg_lo + (uint32_t)i : (uint32_t)(i - n_neg);
    const float a = __uint_as_float(bits);
    const double ref = exp2((double)a);
    const double err = fabs((double)ex2_approx(a) - ref) / ref;
    worst = err > worst ? err : worst;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double t = __shfl_xor_sync(kFull, worst, o);
    worst = t > worst ? t : worst;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(out, (unsigned long long)__double_as_longlong(worst));
}

// The streaming kernel.  Warp gw owns the flattened tiles
// [floor(gw T / W), floor((gw+1) T / W)) of the rows * n_tiles tiles and walks
// them in order through its ring of kStages shared-memory tile buffers: the
// next tile is in flight (bulk copy) while the current one is scanned, and
// four CTAs per SM (128 registers a thread) keep 16 warps' copies going.
// A row part closes at a row change or at the end of the range.  Warps never
// wait for one another; the only waits are the bounded mbarrier waits on the
// warp's own copies.
template <typename T, int KC>
__global__ void __launch_bounds__(kThreadsS, kStreamBlocks<KC>) k_sample_stream(const __grid_constant__ SampleArgs a) {
  using SMem = StreamMem<KC>;
  extern __shared__ __align__(128) unsigned char smem_stream[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  SMem* wm = reinterpret_cast<SMem*>(smem_stream) + wid;
  asm volatile("griddepcontrol.launch_dependents;");
  const int64_t total = a.rows * a.n_tiles;
  const int64_t gw = (int64_t)blockIdx.x * kWarpsS + wid;
  if (gw >= a.n_warps) return;
  const int64_t g0 = gw * total / a.n_warps;
  const int64_t g1 = (gw + 1) * total / a.n_warps;
  if (g0 >= g1) return;
  const uint64_t pol = policy_evict_first();
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&wm->bar[s], 1);
    fence_proxy_async_smem();
  }
  __syncwarp();
  uint32_t armed = 0, phase = 0;
  // issue cursor (irow, itile) runs kStages tiles ahead of the scan cursor
  // (row, tile); both advance without divisions
  int64_t row = g0 / a.n_tiles;
  int tile = (int)(g0 - row * a.n_tiles);
  int64_t irow = row;
  int itile = tile;
  for (int s = 0; s < kStages; ++s) {
    if (g0 + s < g1 && issue_tile<T, KC>(a, irow, itile, s, wm, pol)) armed |= 1u << s;
    if (++itile == a.n_tiles) { itile = 0; ++irow; }
  }
  // the kernel before (the penalty prep, when it runs) has finished and its
  // writes are visible past this point
  asm volatile("griddepcontrol.wait;" ::: "memory");
  PartState ps;
  part_begin(a, row, tile, KC, ps);
  int s = 0;
  for (int64_t gi = g0; gi < g1; ++gi) {
    if ((armed >> s) & 1u) {
      if (!mbar_wait(&wm->bar[s], (phase >> s) & 1u)) {
        // copy never completed: flag the row, wait (bounded) for the other
        // armed stages, and leave
        if (lane == 0) atomicOr(reinterpret_cast<unsigned*>(&a.status[row]), 4u);
        for (int o = 0; o < kStages; ++o)
          if (o != s && ((armed >> o) & 1u)) mbar_wait(&wm->bar[o], (phase >> o) & 1u);
        return;
      }
      phase ^= 1u << s;
    } else {
      load_tile_plain<T, KC>(a, row, tile, s, wm);
    }
    float* buf = wm->tile[s];
    int ob = 0, oe = 0, bb = 0, be = 0;
    if (a.ovr_off) {
      const int32_t* off = a.ovr_off + row * (int64_t)(a.n_tiles + 1) + tile;
      ob = off[0];
      oe = off[1];
    }
    if (a.bias_off) { bb = a.bias_off[tile]; be = a.bias_off[tile + 1]; }
    if (ps.mode == kCand) {
      share_threshold(a, row, ps);
      raise_to_floor(ps);
    }
    if (oe > ob || be > bb) {
      if constexpr (sizeof(T) == 2) expand_bf16_in_place(buf);
      apply_overrides_smem(a, ps.p, row, tile, ob, oe, bb, be, buf);
      scan_tile<float, KC>(a, row, tile, buf, wm->mask[s], ps, wm);
    } else {
      scan_tile<T, KC>(a, row, tile, buf, wm->mask[s], ps, wm);
    }
    if (ps.mode == kCand) ps.rtau = ld_cg(&a.row_tau[row]);  // for the next tile, in flight meanwhile
    __syncwarp();
    armed &= ~(1u << s);
    if (gi + kStages < g1) {
      fence_proxy_async_smem();
      if (issue_tile<T, KC>(a, irow, itile, s, wm, pol)) armed |= 1u << s;
      if (++itile == a.n_tiles) { itile = 0; ++irow; }
    }
    if (++s == kStages) s = 0;
    if (tile == a.n_tiles - 1 || gi == g1 - 1) part_end<T, KC>(a, row, gw, ps, wm);
    if (++tile == a.n_tiles) {
      tile = 0;
      ++row;
      if (gi + 1 < g1) part_begin(a, row, 0, KC, ps);
    }
  }
}

// --------------------------------------------------------------------------
// processors / logprobs: per-tile stats pass and a write pass
// --------------------------------------------------------------------------
// out (when given) receives the processed logits, minus the row's
// log-sum-exp sub[row] when sub is given (the log-softmax write pass).
template <typename T>
__global__ void __launch_bounds__(kThreadsS) k_process_rows(const __grid_constant__ SampleArgs a, float* out,
                                                            int64_t out_stride, bool want_stats, const float* sub) {
  constexpr int VW = Lay<T>::VW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* wbuf = reinterpret_cast<float*>(smem_raw) + (threadIdx.x >> 5) * kTile;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * kWarpsS + (threadIdx.x >> 5);
  const int64_t total = a.rows * a.n_tiles;
  for (int64_t w = gw; w < total; w += (int64_t)gridDim.x * kWarpsS) {
    const int64_t row = w / a.n_tiles;
    const int t = (int)(w % a.n_tiles);
    const pm_row_params p = row_params(a, row);
    const int64_t start = (int64_t)t * kTile;
    const int n_valid = tile_valid(a, t);
    TileIn ti;
    load_tile<T>(a, row, t, ti);
    process_tile<VW>(a, p, row, t, ti, wbuf);
    if (want_stats) {
      float m;
      uint64_t s;
      tile_stats(ti.v, &m, &s);
      if (lane == 0) { TileStat ts; ts.m = m; ts.pad = 0; ts.s = s; a.statx[row * a.n_tiles + t] = ts; }
    }
    if (out) {
      float* orow = out + row * out_stride + start;
      const float c = sub ? sub[row] : 0.0f;
#pragma unroll
      for (int s = 0; s < 32; ++s) {
        const int e = slot_elem<VW>(s, lane);
        if (e < n_valid) orow[e] = sub ? fsub(ti.v[s], c) : ti.v[s];
      }
    }
  }
}

// row log-sum-exp from tile stats: one warp per row
__global__ void __launch_bounds__(kThreadsS) k_row_lse(const __grid_constant__ SampleArgs a, float* lse_out) {
  const int64_t gw = (int64_t)blockIdx.x * kWarpsS + (threadIdx.x >> 5);
  for (int64_t row = gw; row < a.rows; row += (int64_t)gridDim.x * kWarpsS) {
    float m;
    const float c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &m);
    if ((threadIdx.x & 31) == 0) { if (lse_out) lse_out[row] = c; a.row_lse[row] = c; }
  }
}

__global__ void k_bias_offsets(const int32_t* tok, int n, int n_tiles, int32_t* off) {
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t <= n_tiles; t += gridDim.x * blockDim.x) {
    const int64_t key = (int64_t)t * kTile;
    int lo = 0, hi = n;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((int64_t)tok[mid] >= key) hi = mid; else lo = mid + 1;
    }
    off[t] = lo;
  }
}

}  // namespace pm

#include "pm_wide.cuh"
#include "pm_verify_impl.cuh"
#include "pm_shard_impl.cuh"
#include "pm_ngram.cuh"
#include "pm_force.cuh"

// ============================================================================
// host side
// ============================================================================
namespace {

using pmh::cuda_fail;
using pmh::current_device;
using pmh::DeviceOnce;
using pmh::kMaxDevices;
using pmh::num_sms;

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int pow2_at_least(int64_t x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

bool penalties_on(const pm_rows* r) {
  return r->hist && (r->flags_any & (PM_F_REP | PM_F_PRES | PM_F_FREQ));
}

template <typename T, int KC>
int stream_occupancy() {
  static int occ[kMaxDevices] = {};
  static DeviceOnce once;
  const int d = current_device();
  int* slot = (d >= 0 && d < kMaxDevices) ? &occ[d] : nullptr;
  int local = 0;
  once([&] {
    const size_t smem = sizeof(pm::StreamMem<KC>) * pm::kWarpsS;
    cudaFuncSetAttribute(pm::k_sample_stream<T, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, pm::k_sample_stream<T, KC>, pm::kThreadsS, smem) !=
            cudaSuccess || v < 1) {
      cudaGetLastError();
      v = pm::kStreamBlocks<KC>;
    }
    if (slot) *slot = v;
    local = v;
  });
  return slot ? *slot : (local ? local : pm::kStreamBlocks<KC>);
}

int occupancy_for(int dtype, int KC) {
  const bool bf = dtype == PM_DTYPE_BF16;
  if (KC == 64) return bf ? stream_occupancy<__nv_bfloat16, 64>() : stream_occupancy<float, 64>();
  return bf ? stream_occupancy<__nv_bfloat16, 256>() : stream_occupancy<float, 256>();
}

struct Layout {
  int n_tiles = 0, KC = 0, ovr_cap = 0, max_parts = 0;
  int64_t n_warps = 0;
  size_t row_tau = 0, status = 0, exact = 0, statx = 0, staty = 0, cand = 0, cand_n = 0, best = 0, ovr_tok = 0,
         ovr_info = 0, ovr_off = 0, bias_off = 0, row_lse = 0, total = 0;
};

int64_t owner(int64_t g, int64_t T, int64_t W) { return ((g + 1) * W + T - 1) / T - 1; }

int plan(const pm_rows* r, Layout* L) {
  if (!r || r->rows < 0 || r->vocab <= 0 || r->row_stride < r->vocab) return PM_ERR_ARG;
  if (r->vocab > (int64_t)32 * pm::kMaxPer * pm::kTile) return PM_ERR_UNSUPPORTED;  // 256 tiles per row at most
  L->n_tiles = (int)((r->vocab + pm::kTile - 1) / pm::kTile);
  int need = r->top_k_max > 0 ? r->top_k_max : 0;
  if (r->flags_any & PM_F_UNBOUNDED) need = need > 256 ? need : 256;
  if (need > 256) return PM_ERR_UNSUPPORTED;
  L->KC = need <= 64 ? 64 : 256;
  const int64_t T = r->rows * (int64_t)L->n_tiles;
  const int64_t wmax = (int64_t)num_sms() * occupancy_for(r->dtype, L->KC) * pm::kWarpsS;
  int64_t nw = (T + 1) / 2;  // at least two tiles per warp
  if (nw > wmax) nw = wmax;
  if (nw < 1) nw = 1;
  L->n_warps = nw;
  int mp = 1;
  for (int64_t row = 0; row < r->rows; ++row) {
    const int64_t n = owner((row + 1) * L->n_tiles - 1, T, nw) - owner(row * L->n_tiles, T, nw) + 1;
    if (n > mp) mp = (int)n;
  }
  L->max_parts = mp;
  L->ovr_cap = 0;
  if (penalties_on(r)) {
    int64_t w = r->hist_stride + (r->feed ? r->feed_group : 0);
    if (w > 8192) return PM_ERR_UNSUPPORTED;
    L->ovr_cap = pow2_at_least(w < 32 ? 32 : w);
  }
  const int64_t R = r->rows;
  size_t o = 0;
  auto take = [&](size_t bytes) { o = align_up(o, 256); const size_t at = o; o += bytes; return at; };
  L->status = take(sizeof(int32_t) * R);
  L->row_tau = take(sizeof(uint64_t) * R);
  L->exact = take(sizeof(int32_t) * (1 + 2 * R));
  L->statx = take(sizeof(pm::TileStat) * R * L->n_tiles);
  L->staty = take(sizeof(pm::TileStat) * R * L->n_tiles);
  L->cand = take(sizeof(uint64_t) * R * L->max_parts * L->KC);
  L->cand_n = take(sizeof(int32_t) * R * L->max_parts);
  L->best = take(sizeof(uint64_t) * R * L->max_parts);
  L->ovr_tok = take(sizeof(int32_t) * R * L->ovr_cap);
  L->ovr_info = take(sizeof(uint32_t) * R * L->ovr_cap);
  L->ovr_off = take(sizeof(int32_t) * R * (L->ovr_cap ? (L->n_tiles + 1) : 0));
  L->bias_off = take(sizeof(int32_t) * (L->n_tiles + 1));
  L->row_lse = take(sizeof(float) * R);
  L->total = align_up(o, 256);
  return PM_OK;
}

int check_rows(const pm_rows* r) {
  if (!r || !r->logits || !r->params) return PM_ERR_ARG;
  if (r->dtype != PM_DTYPE_F32 && r->dtype != PM_DTYPE_BF16) return PM_ERR_ARG;
  if (r->mask && r->mask_stride < (r->vocab + 31) / 32) return PM_ERR_ARG;
  if (r->feed && (r->feed_group <= 0 || r->rows % r->feed_group)) return PM_ERR_ARG;
  if (r->n_bias < 0 || (r->n_bias > 0 && (!r->bias_tokens || !r->bias_values))) return PM_ERR_ARG;
  if (r->hist && r->hist_stride <= 0) return PM_ERR_ARG;
  if (r->rows > 0x7fffffff) return PM_ERR_UNSUPPORTED;
  return PM_OK;
}

// prep kernels shared by every entry point; fills the processor fields of a
int launch_prep(const pm_rows* r, const Layout& L, unsigned char* ws, pm::SampleArgs& a, cudaStream_t st,
                int64_t id_base = 0) {
  a.logits = r->logits;
  a.rows = r->rows;
  a.vocab = r->vocab;
  a.row_stride = r->row_stride;
  const size_t esz = r->dtype == PM_DTYPE_F32 ? 4 : 2;
  a.vec_ok = ((uintptr_t)r->logits % 16 == 0) && ((r->row_stride * esz) % 16 == 0);
  a.mask_ok = r->mask && ((uintptr_t)r->mask % 16 == 0) && ((r->mask_stride * 4) % 16 == 0);
  a.params = r->params;
  a.params_per_row = r->params_per_row;
  a.mask = r->mask;
  a.mask_stride = r->mask_stride;
  a.n_tiles = L.n_tiles;
  a.max_parts = L.max_parts;
  a.n_warps = L.n_warps;
  a.statx = reinterpret_cast<pm::TileStat*>(ws + L.statx);
  a.staty = reinterpret_cast<pm::TileStat*>(ws + L.staty);
  a.cand = reinterpret_cast<uint64_t*>(ws + L.cand);
  a.cand_n = reinterpret_cast<int32_t*>(ws + L.cand_n);
  a.best = reinterpret_cast<uint64_t*>(ws + L.best);
  a.row_tau = reinterpret_cast<uint64_t*>(ws + L.row_tau);
  a.status = reinterpret_cast<int32_t*>(ws + L.status);
  a.row_lse = reinterpret_cast<float*>(ws + L.row_lse);
  a.exact_q = reinterpret_cast<int32_t*>(ws + L.exact);
  a.approx_ok = false;
  a.ovr_tok = nullptr;
  a.ovr_info = nullptr;
  a.ovr_off = nullptr;
  a.ovr_cap = L.ovr_cap;
  a.bias_tok = nullptr;
  a.bias_val = nullptr;
  a.bias_off = nullptr;
  a.status_live = false;
  a.feed_group = r->feed ? r->feed_group : 0;
  a.verify = nullptr;
  cudaError_t e;
  if (penalties_on(r) && r->rows > 0) {
    pm::PrepArgs pa;
    pa.hist = r->hist;
    pa.hist_len = r->hist_len;
    pa.hist_stride = r->hist_stride;
    pa.feed = r->feed;
    pa.feed_group = r->feed_group;
    pa.params = r->params;
    pa.params_per_row = r->params_per_row;
    pa.rows = r->rows;
    pa.vocab = r->vocab;
    pa.id_base = id_base;
    pa.n_tiles = L.n_tiles;
    pa.cap = L.ovr_cap;
    pa.ovr_tok = reinterpret_cast<int32_t*>(ws + L.ovr_tok);
    pa.ovr_info = reinterpret_cast<uint32_t*>(ws + L.ovr_info);
    pa.ovr_off = reinterpret_cast<int32_t*>(ws + L.ovr_off);
    pa.status = a.status;
    pa.row_tau = a.row_tau;
    pa.exact_q = a.exact_q;
    const size_t smem = sizeof(int) * (6 * (size_t)L.ovr_cap + 2 * 264);
    static DeviceOnce once;
    once([&] {
      cudaFuncSetAttribute(pm::k_prep_overrides, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * (6 * 8192 + 2 * 264));
    });
    pm::k_prep_overrides<<<(unsigned)r->rows, 1024, smem, st>>>(pa);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    a.ovr_tok = pa.ovr_tok;
    a.ovr_info = pa.ovr_info;
    a.ovr_off = pa.ovr_off;
    a.status_live = true;
  }
  if (r->n_bias > 0) {
    a.bias_tok = r->bias_tokens;
    a.bias_val = r->bias_values;
    a.bias_off = reinterpret_cast<int32_t*>(ws + L.bias_off);
    pm::k_bias_offsets<<<(L.n_tiles + 256) / 256, 256, 0, st>>>(r->bias_tokens, r->n_bias, L.n_tiles,
                                                                const_cast<int32_t*>(a.bias_off));
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return PM_OK;
}

bool has_cand_rows(const pm_rows* r) {
  return r->top_k_max > 0 || (r->flags_any & (PM_F_TOP_P | PM_F_MIN_P));
}

// The row merges after a pass that wrote the parts' results, chained by
// programmatic dependent launch, then the exact pass when the bracket is on.
template <typename T, int KC>
int launch_merges(const pm::SampleArgs& a, cudaStream_t st) {
  cudaError_t e;
  // the row merges, chained by programmatic dependent launch: one CTA per
  // row when rows are few (every row then has many parts), one warp per row
  // otherwise
  const bool per_cta = a.rows <= (int64_t)num_sms() * 2;
  const size_t msmem = per_cta ? sizeof(pm::MergeCta<KC>) : (sizeof(uint64_t) * pm::StreamMem<KC>::CAP + 1024) * 8;
  static DeviceOnce once;
  once([&] {
    cudaFuncSetAttribute(pm::k_row_merge_cta<T, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(pm::MergeCta<KC>));
    cudaFuncSetAttribute(pm::k_row_merge_warp<T, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)((sizeof(uint64_t) * pm::StreamMem<KC>::CAP + 1024) * 8));
  });
  int64_t mgrid = per_cta ? a.rows : (a.rows + 7) / 8;
  const int64_t mcap = (int64_t)num_sms() * (per_cta ? 3 : 8);
  if (mgrid > mcap) mgrid = mcap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)mgrid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = msmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = per_cta ? cudaLaunchKernelEx(&cfg, pm::k_row_merge_cta<T, KC>, a)
              : cudaLaunchKernelEx(&cfg, pm::k_row_merge_warp<T, KC>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();  // no programmatic launch here: plain stream order
    if (per_cta) pm::k_row_merge_cta<T, KC><<<(unsigned)mgrid, 256, msmem, st>>>(a);
    else pm::k_row_merge_warp<T, KC><<<(unsigned)mgrid, 256, msmem, st>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return cuda_fail(e);
  if (!a.approx_ok) return PM_OK;
  // the exact pass for the rows the bracket left open (usually none)
  const size_t xsmem = sizeof(pm::ExactMem<T, KC>) * 8;
  static DeviceOnce xonce;
  xonce([&] {
    cudaFuncSetAttribute(pm::k_row_exact<T, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)xsmem);
  });
  cfg.gridDim = dim3((unsigned)num_sms());
  cfg.dynamicSmemBytes = xsmem;
  e = cudaLaunchKernelEx(&cfg, pm::k_row_exact<T, KC>, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    pm::k_row_exact<T, KC><<<(unsigned)num_sms(), 256, xsmem, st>>>(a);
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

template <typename T, int KC>
int launch_stream(pm::SampleArgs a, bool cand_rows, cudaStream_t st, bool merge = true) {
  stream_occupancy<T, KC>();
  const size_t smem = sizeof(pm::StreamMem<KC>) * pm::kWarpsS;
  const int64_t grid = (a.n_warps + pm::kWarpsS - 1) / pm::kWarpsS;
  if (grid == 0) return PM_OK;
  cudaError_t e;
  // the row status (the streaming pass ORs a copy timeout into it), the
  // shared row thresholds ("nothing proven") and the exact pass's queue
  // count and tile counters start at zero; the penalty prep zeroes all of
  // them when it runs.  The workspace plan puts the three arrays one after
  // the other, so one memset covers them.
  if (!a.status_live) {
    const char* s0 = reinterpret_cast<const char*>(a.status);
    const char* t0 = reinterpret_cast<const char*>(a.row_tau);
    const char* x0 = reinterpret_cast<const char*>(a.exact_q);
    const size_t sb = sizeof(int32_t) * a.rows, tb = sizeof(uint64_t) * a.rows,
                 xb = sizeof(int32_t) * (1 + a.rows);
    const bool adjacent = t0 >= s0 + sb && t0 <= s0 + sb + 256 && x0 >= t0 + tb && x0 <= t0 + tb + 256;
    // (row_tau also counts the finished parts of greedy rows merged in the pass)
    if ((cand_rows || a.approx_ok || a.merge_greedy) && adjacent) {
      e = cudaMemsetAsync(a.status, 0, (size_t)(x0 - s0) + (a.approx_ok ? xb : 0), st);
    } else {
      e = cudaMemsetAsync(a.status, 0, sb, st);
      if (e == cudaSuccess && (cand_rows || a.merge_greedy)) e = cudaMemsetAsync(a.row_tau, 0, tb, st);
      if (e == cudaSuccess && a.approx_ok) e = cudaMemsetAsync(a.exact_q, 0, xb, st);
    }
    if (e != cudaSuccess) return cuda_fail(e);
    a.status_live = true;
  }
  {
    // programmatic dependent launch: the tile prologue overlaps the tail of
    // the kernel before (the penalty prep); the kernel waits for it before
    // reading its outputs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(pm::kThreadsS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, pm::k_sample_stream<T, KC>, a);
    if (e != cudaSuccess) {
      cudaGetLastError();  // no programmatic launch here: plain stream order
      pm::k_sample_stream<T, KC><<<(unsigned)grid, pm::kThreadsS, smem, st>>>(a);
      e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(e);
    }
  }
  if (!merge) return PM_OK;
  return launch_merges<T, KC>(a, st);
}

int launch_stream_any(int dtype, int KC, const pm::SampleArgs& a, bool cand_rows, cudaStream_t st,
                      bool merge = true) {
  const bool bf = dtype == PM_DTYPE_BF16;
  if (KC == 64)
    return bf ? launch_stream<__nv_bfloat16, 64>(a, cand_rows, st, merge) : launch_stream<float, 64>(a, cand_rows, st, merge);
  return bf ? launch_stream<__nv_bfloat16, 256>(a, cand_rows, st, merge) : launch_stream<float, 256>(a, cand_rows, st, merge);
}

// Masked rows go through the one-CTA-per-row gather pass when their logits
// can be fetched as aligned 4-byte words (always for fp32; bf16 rows need an
// even stride and a 4-byte aligned base).
bool masked_path(const pm_rows* r) {
  if (!r->mask) return false;
  if (r->dtype == PM_DTYPE_F32) return true;
  return ((uintptr_t)r->logits % 4 == 0) && (r->row_stride % 2 == 0);
}

template <typename T>
int launch_wide(const pm::SampleArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(pm::WideMem);
  static DeviceOnce once;
  once([&] {
    cudaFuncSetAttribute(pm::k_row_wide<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  int64_t grid = a.rows;
  if (grid > (int64_t)num_sms() * 2) grid = (int64_t)num_sms() * 2;
  pm::k_row_wide<T><<<(unsigned)grid, pm::kWThreads, smem, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

// The sampling pass over prepared arguments: gather pass for masked rows,
// streaming + merge otherwise; then, when some row has an unbounded filter,
// the exact finish of rows whose survivors outran the candidates.
int launch_rows(const pm_rows* r, int KC, const pm::SampleArgs& a0, cudaStream_t st) {
  const bool bf = r->dtype == PM_DTYPE_BF16;
  int rc;
  pm::SampleArgs a = a0;
  if (masked_path(r)) {
    rc = pm_launch_masked(r->dtype, KC, a, st);
  } else {
    // greedy rows are merged inside the streaming pass; when every row is
    // greedy (no filter of any row, no whole-vocabulary draw) the merge
    // kernel has nothing left to do and is not launched
    a.merge_greedy = true;
    const bool all_greedy = !(r->flags_any & (PM_F_TOP_P | PM_F_MIN_P | PM_F_FULL)) && r->top_k_max <= 0;
    rc = launch_stream_any(r->dtype, KC, a, has_cand_rows(r), st, !all_greedy);
  }
  if (rc) return rc;
  if (r->flags_any & PM_F_UNBOUNDED) {
    rc = bf ? launch_wide<__nv_bfloat16>(a, st) : launch_wide<float>(a, st);
    if (rc) return rc;
  }
  if (r->forced) {
    int64_t grid = (a.rows + 255) / 256;
    if (grid > (int64_t)num_sms() * 4) grid = (int64_t)num_sms() * 4;
    pm::k_force_rows<<<(unsigned)grid, 256, 0, st>>>(a, r->dtype, r->forced);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return PM_OK;
}

int check_noise(const pm_rows* rows, const pm_noise* noise) {
  if (!noise) return PM_ERR_ARG;
  if (noise->mode != PM_NOISE_PHILOX && noise->mode != PM_NOISE_INJECTED) return PM_ERR_ARG;
  if (noise->mode == PM_NOISE_INJECTED) {
    if (has_cand_rows(rows) && (!noise->gumbel || noise->gumbel_stride < rows->vocab)) return PM_ERR_ARG;
    if ((rows->flags_any & PM_F_FULL) && !noise->uniform) return PM_ERR_ARG;
  }
  return PM_OK;
}

void set_noise(const pm_noise* noise, pm::SampleArgs& a) {
  a.noise_mode = noise->mode;
  a.seed = noise->seed;
  a.offset = noise->offset;
  a.row_base = noise->row_base;
  a.gumbel = noise->gumbel;
  a.gumbel_stride = noise->gumbel_stride;
  a.uniform = noise->uniform;
}

// Workspace of a verify call: the sampling layout of the target rows, then
// each row's sample and survivors, the pending residual rows, and the draft
// rows' tile statistics and log-sum-exp.
struct VLayout {
  Layout L;
  int k = 0, scap = 0;
  int64_t B = 0, D = 0;
  size_t rtok = 0, sids = 0, sprobs = 0, ns = 0, pending = 0, dstat = 0, dlse = 0, ylse = 0, rsum = 0, probs = 0,
         total = 0;
};

int plan_verify(const pm_rows* r, const pm_verify_args* v, VLayout* V) {
  if (!r || !v || v->n_draft < 0 || r->rows < 0) return PM_ERR_ARG;
  if (v->mode != PM_VERIFY_MATCH && v->mode != PM_VERIFY_RESIDUAL) return PM_ERR_ARG;
  const int64_t K1 = (int64_t)v->n_draft + 1;
  if (r->rows % K1) return PM_ERR_ARG;
  int rc = plan(r, &V->L);
  if (rc) return rc;
  V->k = v->n_draft;
  V->B = r->rows / K1;
  const bool res = v->mode == PM_VERIFY_RESIDUAL;
  V->D = res ? V->B * V->k : 0;
  V->scap = res ? V->L.KC : 0;
  const int64_t R = r->rows;
  size_t o = V->L.total;
  auto take = [&](size_t bytes) { o = align_up(o, 256); const size_t at = o; o += bytes; return at; };
  V->rtok = take(sizeof(int32_t) * R);
  V->sids = take(sizeof(int32_t) * R * V->scap);
  V->sprobs = take(sizeof(float) * R * V->scap);
  V->ns = take(sizeof(int32_t) * R);
  V->pending = take(sizeof(int32_t) * V->B);
  V->dstat = take(sizeof(pm::TileStat) * V->D * V->L.n_tiles);
  V->dlse = take(sizeof(float) * V->D);
  V->ylse = take(sizeof(float) * V->B);
  V->rsum = take(res ? sizeof(uint64_t) * V->B * V->L.n_tiles : 0);
  V->probs = take(sizeof(pm::AccProb) * V->D);
  V->total = align_up(o, 256);
  return PM_OK;
}

// Tile statistics of the raw draft rows (no processors); k_accept_probs folds
// each row's into its log-sum-exp.
template <typename TD>
int launch_draft_lse(const pm_rows* rows, const pm_verify_args* v, const VLayout& V, unsigned char* ws,
                     cudaStream_t st) {
  pm::SampleArgs da;
  memset(&da, 0, sizeof(da));
  da.logits = v->draft_logits;
  da.rows = V.D;
  da.vocab = rows->vocab;
  da.row_stride = v->draft_row_stride;
  da.vec_ok = ((uintptr_t)v->draft_logits % 16 == 0) && ((v->draft_row_stride * sizeof(TD)) % 16 == 0);
  da.params = rows->params;  // only read when a tile has overrides, and the draft rows have none
  da.params_per_row = 0;
  da.n_tiles = V.L.n_tiles;
  da.statx = reinterpret_cast<pm::TileStat*>(ws + V.dstat);
  const int64_t work = V.D * (int64_t)V.L.n_tiles;
  int64_t grid = (work + pm::kWarpsS - 1) / pm::kWarpsS;
  if (grid > (int64_t)num_sms() * 16) grid = (int64_t)num_sms() * 16;
  pm::k_process_rows<TD><<<(unsigned)grid, pm::kThreadsS, pm::kWarpsS * pm::kTile * 4, st>>>(da, nullptr, 0, true,
                                                                                          nullptr);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

template <int KC>
int launch_accept(const pm::SampleArgs& a, int dtype, const pm::VerifyK& vk, int64_t B, cudaStream_t st) {
  constexpr int kAccWarps = 8;
  const size_t smem = sizeof(uint64_t) * 2 * KC * kAccWarps;
  int64_t grid = (B + kAccWarps - 1) / kAccWarps;
  if (grid > (int64_t)num_sms() * 8) grid = (int64_t)num_sms() * 8;
  pm::k_verify_accept<KC><<<(unsigned)grid, 32 * kAccWarps, smem, st>>>(a, dtype, vk);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

}  // namespace

// The processors' device lists for a pass of another translation unit (the
// fused LM-head pass): the penalty overrides bucketed by 1024-id tile and the
// logit-bias tile offsets, laid out in `region` (pm_prep_bytes of it).
size_t pm_prep_bytes(const pm_rows* r, int n_tiles) {
  int cap = 0;
  if (penalties_on(r)) {
    const int64_t w = r->hist_stride + (r->feed ? r->feed_group : 0);
    if (w > 8192) return 0;
    cap = pow2_at_least(w < 32 ? 32 : w);
  }
  const int64_t R = r->rows;
  return align_up(sizeof(int32_t) * R * cap, 256) + align_up(sizeof(uint32_t) * R * cap, 256) +
         align_up(sizeof(int32_t) * R * (cap ? n_tiles + 1 : 0), 256) + align_up(sizeof(int32_t) * (n_tiles + 1), 256);
}

int pm_prep_launch(const pm_rows* r, int n_tiles, unsigned char* region, pm::SampleArgs& a, cudaStream_t st) {
  Layout L;
  L.n_tiles = n_tiles;
  L.ovr_cap = 0;
  if (penalties_on(r)) {
    const int64_t w = r->hist_stride + (r->feed ? r->feed_group : 0);
    if (w > 8192) return PM_ERR_UNSUPPORTED;
    L.ovr_cap = pow2_at_least(w < 32 ? 32 : w);
  }
  const int64_t R = r->rows;
  size_t o = 0;
  L.ovr_tok = o;
  o += align_up(sizeof(int32_t) * R * L.ovr_cap, 256);
  L.ovr_info = o;
  o += align_up(sizeof(uint32_t) * R * L.ovr_cap, 256);
  L.ovr_off = o;
  o += align_up(sizeof(int32_t) * R * (L.ovr_cap ? n_tiles + 1 : 0), 256);
  L.bias_off = o;
  a.ovr_tok = nullptr;
  a.ovr_info = nullptr;
  a.ovr_off = nullptr;
  a.ovr_cap = L.ovr_cap;
  a.bias_tok = nullptr;
  a.bias_val = nullptr;
  a.bias_off = nullptr;
  cudaError_t e;
  if (L.ovr_cap && R > 0) {
    pm::PrepArgs pa;
    pa.hist = r->hist;
    pa.hist_len = r->hist_len;
    pa.hist_stride = r->hist_stride;
    pa.feed = r->feed;
    pa.feed_group = r->feed_group;
    pa.params = r->params;
    pa.params_per_row = r->params_per_row;
    pa.rows = R;
    pa.vocab = r->vocab;
    pa.id_base = 0;
    pa.n_tiles = n_tiles;
    pa.cap = L.ovr_cap;
    pa.ovr_tok = reinterpret_cast<int32_t*>(region + L.ovr_tok);
    pa.ovr_info = reinterpret_cast<uint32_t*>(region + L.ovr_info);
    pa.ovr_off = reinterpret_cast<int32_t*>(region + L.ovr_off);
    pa.status = a.status;
    pa.row_tau = a.row_tau;
    pa.exact_q = nullptr;
    const size_t smem = sizeof(int) * (6 * (size_t)L.ovr_cap + 2 * 264);
    static DeviceOnce once;
    once([&] {
      cudaFuncSetAttribute(pm::k_prep_overrides, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * (6 * 8192 + 2 * 264));
    });
    pm::k_prep_overrides<<<(unsigned)R, 1024, smem, st>>>(pa);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    a.ovr_tok = pa.ovr_tok;
    a.ovr_info = pa.ovr_info;
    a.ovr_off = pa.ovr_off;
  }
  if (r->n_bias > 0) {
    a.bias_tok = r->bias_tokens;
    a.bias_val = r->bias_values;
    a.bias_off = reinterpret_cast<int32_t*>(region + L.bias_off);
    pm::k_bias_offsets<<<(n_tiles + 256) / 256, 256, 0, st>>>(r->bias_tokens, r->n_bias, n_tiles,
                                                               const_cast<int32_t*>(a.bias_off));
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return PM_OK;
}

// The row merges over parts written by another translation unit's pass (the
// fused LM-head pass): rows never take the whole-vocabulary draw there, so
// the logits type is immaterial.
int pm_launch_merges(int KC, const pm::SampleArgs& a, cudaStream_t st) {
  return KC == 64 ? launch_merges<float, 64>(a, st) : launch_merges<float, 256>(a, st);
}

extern "C" {

int pm_last_cuda_error(void) { return pmh::last_cuda(); }

const char* pm_version(void) { return "pm_sample 0.2 sm_100a"; }

size_t pm_sample_workspace_bytes(const pm_rows* rows) {
  Layout L;
  if (plan(rows, &L) != PM_OK) return 0;
  return L.total;
}

int pm_sample_rows(const pm_rows* rows, const pm_noise* noise, const pm_sample_out* out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int rc = check_rows(rows);
  if (rc) return rc;
  if (!out || !out->tokens || !workspace) return PM_ERR_ARG;
  rc = check_noise(rows, noise);
  if (rc) return rc;
  if (out->surv_ids && (!out->surv_probs || !out->n_surv || out->surv_cap <= 0)) return PM_ERR_ARG;
  Layout L;
  rc = plan(rows, &L);
  if (rc) return rc;
  if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
  if (rows->rows == 0) return PM_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  pm::SampleArgs a;
  memset(&a, 0, sizeof(a));
  rc = launch_prep(rows, L, ws, a, st);
  if (rc) return rc;
  set_noise(noise, a);
  a.tokens = out->tokens;
  a.lse_out = out->lse;
  a.tok_logprob = out->token_logprob;
  a.surv_ids = out->surv_ids;
  a.surv_probs = out->surv_probs;
  a.n_surv = out->n_surv;
  a.surv_cap = out->surv_cap;
  a.want_lse = out->lse != nullptr || out->token_logprob != nullptr;
  // bracketed statistics for top-k + top-p rows when the streaming pass has
  // at least four tiles a warp (below that it is latency-bound, and the
  // exact pass's launch would cost more than it saves)
  a.approx_ok = !a.want_lse && !rows->mask && rows->top_k_max > 0 && (rows->flags_any & PM_F_TOP_P) &&
                rows->rows * (int64_t)L.n_tiles >= 4 * L.n_warps;
  return launch_rows(rows, L.KC, a, st);
}

size_t pm_processors_workspace_bytes(const pm_rows* rows) { return pm_sample_workspace_bytes(rows); }

static int process_common(const pm_rows* rows, float* out, int64_t out_stride, float* lse_out, bool logprobs,
                          void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_rows(rows);
  if (rc) return rc;
  if (!out || out_stride < rows->vocab || !workspace) return PM_ERR_ARG;
  Layout L;
  rc = plan(rows, &L);
  if (rc) return rc;
  if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
  if (rows->rows == 0) return PM_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  pm::SampleArgs a;
  memset(&a, 0, sizeof(a));
  rc = launch_prep(rows, L, ws, a, st);
  if (rc) return rc;
  const size_t smem = pm::kWarpsS * pm::kTile * 4;
  const int64_t work = rows->rows * (int64_t)L.n_tiles;
  int64_t grid = (work + pm::kWarpsS - 1) / pm::kWarpsS;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (grid > cap) grid = cap;
  // processors: one pass writing the processed rows.  log-softmax: a pass
  // for the tile statistics only (nothing written), the row log-sum-exp,
  // then one pass writing processed - log-sum-exp.
  const bool bf = rows->dtype == PM_DTYPE_BF16;
  auto pass = [&](float* o, bool stats, const float* sub) {
    if (bf) pm::k_process_rows<__nv_bfloat16><<<(unsigned)grid, pm::kThreadsS, smem, st>>>(a, o, out_stride, stats, sub);
    else pm::k_process_rows<float><<<(unsigned)grid, pm::kThreadsS, smem, st>>>(a, o, out_stride, stats, sub);
    return cudaGetLastError();
  };
  cudaError_t e = logprobs ? pass(nullptr, true, nullptr) : pass(out, false, nullptr);
  if (e != cudaSuccess) return cuda_fail(e);
  if (logprobs) {
    int64_t g2 = (rows->rows + pm::kWarpsS - 1) / pm::kWarpsS;
    if (g2 > (int64_t)num_sms() * 8) g2 = (int64_t)num_sms() * 8;
    pm::k_row_lse<<<(unsigned)g2, pm::kThreadsS, 0, st>>>(a, lse_out);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    e = pass(out, false, a.row_lse);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return PM_OK;
}

int pm_apply_processors(const pm_rows* rows, float* out, int64_t out_stride, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return process_common(rows, out, out_stride, nullptr, false, workspace, workspace_bytes, stream);
}

int pm_logprobs(const pm_rows* rows, float* out, int64_t out_stride, float* lse_out, void* workspace,
                size_t workspace_bytes, void* stream) {
  return process_common(rows, out, out_stride, lse_out, true, workspace, workspace_bytes, stream);
}

size_t pm_verify_workspace_bytes(const pm_rows* rows, const pm_verify_args* v) {
  VLayout V;
  if (plan_verify(rows, v, &V) != PM_OK) return 0;
  return V.total;
}

int pm_verify(const pm_rows* rows, const pm_noise* noise, const pm_verify_args* v, void* workspace,
              size_t workspace_bytes, void* stream) {
  int rc = check_rows(rows);
  if (rc) return rc;
  if (!v || !workspace || !v->tokens || !v->n_accepted) return PM_ERR_ARG;
  if (v->n_draft > 0 && !v->drafts) return PM_ERR_ARG;
  if (rows->feed && rows->feed_group != v->n_draft + 1) return PM_ERR_ARG;
  const bool res = v->mode == PM_VERIFY_RESIDUAL;
  if (res && v->n_draft > 0) {
    if (!v->draft_logits || v->draft_row_stride < rows->vocab) return PM_ERR_ARG;
    if (v->draft_dtype != PM_DTYPE_F32 && v->draft_dtype != PM_DTYPE_BF16) return PM_ERR_ARG;
  }
  rc = check_noise(rows, noise);
  if (rc) return rc;
  VLayout V;
  rc = plan_verify(rows, v, &V);
  if (rc) return rc;
  if (workspace_bytes < V.total) return PM_ERR_WORKSPACE;
  if (rows->rows == 0) return PM_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  if (V.D > 0) {
    rc = v->draft_dtype == PM_DTYPE_BF16 ? launch_draft_lse<__nv_bfloat16>(rows, v, V, ws, st)
                                         : launch_draft_lse<float>(rows, v, V, ws, st);
    if (rc) return rc;
  }
  pm::SampleArgs a;
  memset(&a, 0, sizeof(a));
  rc = launch_prep(rows, V.L, ws, a, st);
  if (rc) return rc;
  set_noise(noise, a);
  a.tokens = reinterpret_cast<int32_t*>(ws + V.rtok);
  a.n_surv = reinterpret_cast<int32_t*>(ws + V.ns);
  if (res) {
    a.surv_ids = reinterpret_cast<int32_t*>(ws + V.sids);
    a.surv_probs = reinterpret_cast<float*>(ws + V.sprobs);
    a.surv_cap = V.scap;
  }
  rc = launch_rows(rows, V.L.KC, a, st);
  if (rc) return rc;
  pm::VerifyK vk;
  memset(&vk, 0, sizeof(vk));
  vk.mode = v->mode;
  vk.drafts = v->drafts;
  vk.k = v->n_draft;
  vk.dlogits = v->draft_logits;
  vk.ddtype = v->draft_dtype;
  vk.dstride = v->draft_row_stride;
  vk.dlse = reinterpret_cast<float*>(ws + V.dlse);
  vk.dstat = reinterpret_cast<const pm::TileStat*>(ws + V.dstat);
  vk.u_accept = v->u_accept;
  vk.u_residual = v->u_residual;
  vk.tokens = v->tokens;
  vk.n_acc = v->n_accepted;
  vk.row_tokens = v->row_tokens;
  vk.rtok = a.tokens;
  vk.sids = a.surv_ids;
  vk.sprobs = a.surv_probs;
  vk.ns = a.n_surv;
  vk.scap = V.scap;
  vk.pending = reinterpret_cast<int32_t*>(ws + V.pending);
  vk.ylse = reinterpret_cast<float*>(ws + V.ylse);
  vk.rsum = reinterpret_cast<uint64_t*>(ws + V.rsum);
  vk.probs = reinterpret_cast<pm::AccProb*>(ws + V.probs);
  if (res && V.D > 0) {
    int64_t g = (V.D + 7) / 8;
    if (g > (int64_t)num_sms() * 8) g = (int64_t)num_sms() * 8;
    pm::k_accept_probs<<<(unsigned)g, 256, 0, st>>>(a, rows->dtype, vk);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
  }
  rc = V.L.KC == 64 ? launch_accept<64>(a, rows->dtype, vk, V.B, st) : launch_accept<256>(a, rows->dtype, vk, V.B, st);
  if (rc) return rc;
  if (res && V.k > 0 && (rows->flags_any & PM_F_FULL)) {
    // the draft rows as plain rows for the tile loads (no processors)
    pm::SampleArgs da = a;
    da.logits = v->draft_logits;
    da.rows = V.D;
    da.row_stride = v->draft_row_stride;
    const size_t desz = v->draft_dtype == PM_DTYPE_F32 ? 4 : 2;
    da.vec_ok = ((uintptr_t)v->draft_logits % 16 == 0) && ((v->draft_row_stride * desz) % 16 == 0);
    da.mask = nullptr;
    da.mask_ok = false;
    da.ovr_off = nullptr;
    da.bias_off = nullptr;
    int64_t g1 = (V.B * V.L.n_tiles + 7) / 8;
    if (g1 > (int64_t)num_sms() * 16) g1 = (int64_t)num_sms() * 16;
    const bool tb = rows->dtype == PM_DTYPE_BF16, db = v->draft_dtype == PM_DTYPE_BF16;
    if (tb && db) pm::k_residual_tiles<__nv_bfloat16, __nv_bfloat16><<<(unsigned)g1, 256, 0, st>>>(a, da, vk);
    else if (tb) pm::k_residual_tiles<__nv_bfloat16, float><<<(unsigned)g1, 256, 0, st>>>(a, da, vk);
    else if (db) pm::k_residual_tiles<float, __nv_bfloat16><<<(unsigned)g1, 256, 0, st>>>(a, da, vk);
    else pm::k_residual_tiles<float, float><<<(unsigned)g1, 256, 0, st>>>(a, da, vk);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    int64_t g2 = V.B;  // one CTA per request
    if (g2 > (int64_t)num_sms() * 4) g2 = (int64_t)num_sms() * 4;
    if (tb) pm::k_residual_draw<__nv_bfloat16><<<(unsigned)g2, 256, 0, st>>>(a, vk);
    else pm::k_residual_draw<float><<<(unsigned)g2, 256, 0, st>>>(a, vk);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return PM_OK;
}

}  // extern "C"

// ============================================================================
// vocabulary-sharded sampling
// ============================================================================
namespace {

int shard_layout(const pm_rows* r, const pm_shard* sh, pm::ShardLayout* S) {
  if (!r || !sh) return PM_ERR_ARG;
  if (sh->n_shards < 1 || sh->shard_index < 0 || sh->shard_index >= sh->n_shards) return PM_ERR_ARG;
  if (sh->shard_width <= 0 || sh->vocab_total <= 0) return PM_ERR_ARG;
  if (sh->n_shards > 1 && sh->shard_width % pm::kTile) return PM_ERR_ARG;
  const int64_t last = sh->vocab_total - (int64_t)(sh->n_shards - 1) * sh->shard_width;
  if (last <= 0 || last > sh->shard_width) return PM_ERR_ARG;
  if (sh->vocab_total > (int64_t)32 * pm::kMaxPer * pm::kTile) return PM_ERR_UNSUPPORTED;
  int need = r->top_k_max > 0 ? r->top_k_max : 0;
  if (r->flags_any & PM_F_UNBOUNDED) need = need > 256 ? need : 256;
  if (need > 256) return PM_ERR_UNSUPPORTED;
  S->cand_k = need <= 64 ? 64 : 256;
  S->nts = (int)((sh->shard_width + pm::kTile - 1) / pm::kTile);
  S->full = (r->flags_any & PM_F_FULL) != 0;
  size_t o = 16;
  S->keys = o;
  o += sizeof(uint64_t) * S->cand_k;
  S->xst = o;
  o += sizeof(pm::TileStat) * S->nts;
  S->yst = S->ttok = S->tx = o;
  if (S->full) {
    S->yst = o;
    o += sizeof(pm::TileStat) * S->nts;
    S->ttok = o;
    o += sizeof(int32_t) * S->nts;
    S->tx = o;
    o += sizeof(float) * S->nts;
  }
  S->row_bytes = align_up(o, 16);
  return PM_OK;
}

int64_t shard_vocab(const pm_shard* sh) {
  const int64_t last = sh->vocab_total - (int64_t)(sh->n_shards - 1) * sh->shard_width;
  return sh->shard_index == sh->n_shards - 1 ? last : sh->shard_width;
}

template <typename T, int KC>
int launch_shard_pack(const pm::SampleArgs& a, const pm::ShardK& sk, cudaStream_t st) {
  constexpr int kWarpsP = 8;
  const size_t smem = (sizeof(uint64_t) * pm::StreamMem<KC>::CAP + 1024) * kWarpsP;
  static DeviceOnce once;
  once([&] {
    cudaFuncSetAttribute(pm::k_shard_pack<T, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  int64_t grid = (a.rows + kWarpsP - 1) / kWarpsP;
  if (grid > (int64_t)num_sms() * 8) grid = (int64_t)num_sms() * 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(32 * kWarpsP);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, pm::k_shard_pack<T, KC>, a, sk);
  if (e != cudaSuccess) {
    cudaGetLastError();
    pm::k_shard_pack<T, KC><<<(unsigned)grid, 32 * kWarpsP, smem, st>>>(a, sk);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return cuda_fail(e);
  if (sk.full) {
    int64_t g2 = (a.rows * a.n_tiles + 7) / 8;
    if (g2 > (int64_t)num_sms() * 16) g2 = (int64_t)num_sms() * 16;
    pm::k_shard_tiles<T><<<(unsigned)g2, 256, 0, st>>>(a, sk);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return PM_OK;
}

template <typename T, int KC>
int shard_stream_and_pack(const pm::SampleArgs& a, const pm::ShardK& sk, bool cand_rows, cudaStream_t st) {
  const int rc = launch_stream<T, KC>(a, cand_rows, st, false);
  if (rc) return rc;
  return launch_shard_pack<T, KC>(a, sk, st);
}

template <int KC>
int launch_shard_merge(const pm::SampleArgs& a, const pm::MergeK& m, cudaStream_t st) {
  // one CTA per row: the gathered keys of every shard, the row's top K, the
  // radix histogram and its scalars
  const size_t smem = sizeof(uint64_t) * ((size_t)m.n_shards * m.cand_k + KC) + sizeof(unsigned) * 256 +
                      sizeof(int) * 8;
  if (smem > 227 * 1024) return PM_ERR_UNSUPPORTED;
  static DeviceOnce once;
  once([&] {
    cudaFuncSetAttribute(pm::k_shard_merge<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  int64_t grid = a.rows;
  if (grid > (int64_t)num_sms() * 8) grid = (int64_t)num_sms() * 8;
  pm::k_shard_merge<KC><<<(unsigned)grid, 256, smem, st>>>(a, m);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

}  // namespace

extern "C" {

size_t pm_shard_summary_bytes(const pm_rows* rows, const pm_shard* shard) {
  pm::ShardLayout S;
  if (!rows || rows->rows < 0 || shard_layout(rows, shard, &S) != PM_OK) return 0;
  return S.row_bytes * (size_t)rows->rows;
}

int pm_shard_summarize(const pm_rows* rows, const pm_shard* shard, const pm_noise* noise, void* summary,
                       void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_rows(rows);
  if (rc) return rc;
  pm::ShardLayout S;
  rc = shard_layout(rows, shard, &S);
  if (rc) return rc;
  if (rows->vocab != shard_vocab(shard)) return PM_ERR_ARG;
  if (!summary || !workspace) return PM_ERR_ARG;
  rc = check_noise(rows, noise);
  if (rc) return rc;
  Layout L;
  rc = plan(rows, &L);
  if (rc) return rc;
  if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
  if (rows->rows == 0) return PM_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  const int64_t id_base = (int64_t)shard->shard_index * shard->shard_width;
  pm::SampleArgs a;
  memset(&a, 0, sizeof(a));
  rc = launch_prep(rows, L, ws, a, st, id_base);
  if (rc) return rc;
  set_noise(noise, a);
  a.want_lse = true;  // the merge may ask for the log-sum-exp: every row records its x statistics
  pm::ShardK sk;
  sk.rec = reinterpret_cast<unsigned char*>(summary);
  sk.row_bytes = (int64_t)S.row_bytes;
  sk.keys = (int64_t)S.keys;
  sk.xst = (int64_t)S.xst;
  sk.yst = (int64_t)S.yst;
  sk.ttok = (int64_t)S.ttok;
  sk.tx = (int64_t)S.tx;
  sk.cand_k = S.cand_k;
  sk.id_base = (uint32_t)id_base;
  sk.full = S.full;
  const bool bf = rows->dtype == PM_DTYPE_BF16;
  const bool cand = has_cand_rows(rows);
  if (L.KC == 64) rc = bf ? shard_stream_and_pack<__nv_bfloat16, 64>(a, sk, cand, st)
                          : shard_stream_and_pack<float, 64>(a, sk, cand, st);
  else rc = bf ? shard_stream_and_pack<__nv_bfloat16, 256>(a, sk, cand, st)
               : shard_stream_and_pack<float, 256>(a, sk, cand, st);
  return rc;
}

int pm_shard_merge(const pm_rows* rows, const pm_shard* shard, const pm_noise* noise, const void* summaries,
                   const pm_sample_out* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!rows || !rows->params || rows->rows < 0 || !summaries || !out || !out->tokens || !workspace) return PM_ERR_ARG;
  if (rows->vocab != (shard ? shard->vocab_total : -1)) return PM_ERR_ARG;
  if (out->surv_ids && (!out->surv_probs || !out->n_surv || out->surv_cap <= 0)) return PM_ERR_ARG;
  pm::ShardLayout S;
  int rc = shard_layout(rows, shard, &S);
  if (rc) return rc;
  rc = check_noise(rows, noise);
  if (rc) return rc;
  if (workspace_bytes < sizeof(int32_t) * (size_t)rows->rows) return PM_ERR_WORKSPACE;
  if (rows->rows == 0) return PM_OK;
  pm::SampleArgs a;
  memset(&a, 0, sizeof(a));
  a.rows = rows->rows;
  a.vocab = rows->vocab;
  a.params = rows->params;
  a.params_per_row = rows->params_per_row;
  set_noise(noise, a);
  a.tokens = out->tokens;
  a.lse_out = out->lse;
  a.tok_logprob = out->token_logprob;
  a.surv_ids = out->surv_ids;
  a.surv_probs = out->surv_probs;
  a.n_surv = out->n_surv;
  a.surv_cap = out->surv_cap;
  a.want_lse = out->lse != nullptr || out->token_logprob != nullptr;
  a.status = reinterpret_cast<int32_t*>(workspace);
  pm::MergeK m;
  m.recs = reinterpret_cast<const unsigned char*>(summaries);
  m.row_bytes = (int64_t)S.row_bytes;
  m.shard_bytes = (int64_t)S.row_bytes * rows->rows;
  m.keys = (int64_t)S.keys;
  m.xst = (int64_t)S.xst;
  m.yst = (int64_t)S.yst;
  m.ttok = (int64_t)S.ttok;
  m.tx = (int64_t)S.tx;
  m.n_shards = shard->n_shards;
  m.nts = S.nts;
  m.nt = (int)((rows->vocab + pm::kTile - 1) / pm::kTile);
  m.cand_k = S.cand_k;
  a.n_tiles = m.nt;
  return S.cand_k == 64 ? launch_shard_merge<64>(a, m, reinterpret_cast<cudaStream_t>(stream))
                        : launch_shard_merge<256>(a, m, reinterpret_cast<cudaStream_t>(stream));
}

int pm_selfcheck_ex2(double* max_rel_err) {
  if (!max_rel_err) return PM_ERR_ARG;
  unsigned long long* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(unsigned long long));
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaMemset(d, 0, sizeof(unsigned long long));
  if (e == cudaSuccess) {
    pm::k_selfcheck_ex2<<<(unsigned)num_sms() * 8, 256>>>(d);
    e = cudaGetLastError();
  }
  unsigned long long bits = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&bits, d, sizeof(bits), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return cuda_fail(e);
  double v;
  memcpy(&v, &bits, sizeof(v));
  *max_rel_err = v;
  return PM_OK;
}

}  // extern "C"

extern "C" int pm_draft_ngram(const int32_t* hist, const int32_t* hist_len, int64_t hist_stride,
                              int64_t requests, int32_t k, int32_t n_min, int32_t n_max, int32_t* drafts,
                              int32_t* draft_len, int32_t* match_n, void* stream) {
  if (requests < 0 || k < 0 || n_min < 1 || n_max > pm::kNgramMax || hist_stride < 0) return PM_ERR_ARG;
  if (requests == 0 || k == 0) {
    if (requests > 0 && draft_len) {
      cudaError_t e = cudaMemsetAsync(draft_len, 0, sizeof(int32_t) * requests, reinterpret_cast<cudaStream_t>(stream));
      if (e == cudaSuccess && match_n)
        e = cudaMemsetAsync(match_n, 0, sizeof(int32_t) * requests, reinterpret_cast<cudaStream_t>(stream));
      return e == cudaSuccess ? PM_OK : cuda_fail(e);
    }
    return PM_OK;
  }
  if (!hist || !drafts || !draft_len) return PM_ERR_ARG;
  int64_t grid = requests < (int64_t)num_sms() * 8 ? requests : (int64_t)num_sms() * 8;
  pm::k_draft_ngram<<<(unsigned)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      hist, hist_len, hist_stride, requests, k, n_min, n_max, drafts, draft_len, match_n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

extern "C" int pm_think_budget(const int32_t* gen, const int32_t* gen_len, int64_t gen_stride, int64_t rows,
                               const int32_t* piece_len, const uint8_t* piece_end, int64_t table_size,
                               const int32_t* chars, const int32_t* close, int32_t n_close, int32_t end_id,
                               int32_t start_id, int32_t slack, int32_t* forced, void* stream) {
  if (rows < 0 || gen_stride < 0 || table_size <= 0 || n_close <= 0 || slack < 0) return PM_ERR_ARG;
  if (rows == 0) return PM_OK;
  if (!gen || !piece_len || !piece_end || !chars || !close || !forced) return PM_ERR_ARG;
  int64_t grid = (rows + 7) / 8;
  if (grid > (int64_t)num_sms() * 8) grid = (int64_t)num_sms() * 8;
  pm::k_think_budget<<<(unsigned)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      gen, gen_len, gen_stride, rows, piece_len, piece_end, table_size, chars, close, n_close, end_id, start_id,
      slack, forced);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

// ============================================================================
// Fixed-scratch variant of pm_sample_rows
// ============================================================================
// Some callers have no device allocator to take a workspace from: a host
// binding (cgo, JNI, a C server loop) that holds only the logits and output
// pointers, or a decode loop that must not call cudaMalloc between steps
// because it synchronises the whole device and stalls the other streams.
// For them the sampling pass can run out of scratch that the library owns: a
// file-scope device array, placed in device memory by the CUDA driver when it
// loads this module, never by a call.  Its address is looked up once per
// device (cudaGetSymbolAddress with that device current) on the first call
// there, so that first call should come before any stream capture.  Nothing
// in it needs to start at zero: the pass zeroes the row thresholds itself
// (cudaMemsetAsync on the caller's stream) and writes every other byte
// before reading it.  There is one scratch array per device, so calls on the
// same device must not overlap (one stream, or serialised by the caller);
// overlapping calls race on it.
namespace {

static __device__ __align__(256) unsigned char g_static_scratch[PM_STATIC_SCRATCH_BYTES];

std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};

int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return PM_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e);
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return PM_OK;
}

}  // namespace

extern "C" int pm_sample_rows_static(const pm_rows* rows, const pm_noise* noise, const pm_sample_out* out,
                                     void* stream) {
  int rc = check_rows(rows);
  if (rc) return rc;
  Layout L;
  rc = plan(rows, &L);
  if (rc) return rc;
  if (L.total > (size_t)PM_STATIC_SCRATCH_BYTES) return PM_ERR_WORKSPACE;
  void* ws = nullptr;
  rc = static_scratch(&ws);
  if (rc) return rc;
  return pm_sample_rows(rows, noise, out, ws, (size_t)PM_STATIC_SCRATCH_BYTES, stream);
}
