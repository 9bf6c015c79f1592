// pm_masked.cu -- the sampling pass for rows with an allowed-token mask:
// one CTA of 16 warps per row.
//
// A constrained-decoding mask usually allows a small part of the vocabulary
// (a grammar state, a forced token).  Every processed value of a disallowed
// token is -inf and changes nothing (log-sum-exp, candidates, draw), so this
// pass reads the row's mask words first and then fetches only the logits of
// allowed tokens, 4 bytes each, straight into shared memory by asynchronous
// copies, in ascending token order.  HBM traffic: the mask plus the 32-byte
// sectors that hold an allowed token, instead of the whole row.
//
// A row whose allowed tokens fit the kWin-position list (the fast path):
//   1. the mask words -> shared memory (coalesced loads, all issued before
//      the first store); thread t then takes the WPT consecutive words from
//      WPT t on, i.e. warp w the tiles [WPT w, WPT (w + 1)); one warp scan of
//      the threads' allowed counts and one shared-memory atomic allocate the
//      warp's list region, and the warp writes its tokens' ids there;
//   -- barrier: a 4-byte asynchronous copy of each listed logit into its
//      value slot, position-strided over all threads (coalesced along runs
//      of allowed tokens);
//   2. processors on each warp's tiles (logit bias, penalties);
//   -- barrier: exact tile statistics (max, integer sum of
//      floor(e^(x - max) 2^52)) over balanced runs of list positions, a pass
//      of maxima and, after a barrier, a pass of sums; each thread keeps its
//      largest value (and its best key, for greedy rows);
//   -- barrier: warp 0 finds v0, a lower bound of the row's K-th largest
//      value (the K-th largest of the threads' maxima, 16-bit resolution),
//      while warps 8..15 weigh one tile each for the row's log-sum-exp;
//   -- barrier: keys >= v0 -> selection buffer (position-strided);
//   -- barrier: every key ranked by counting the larger ones; the thread
//      that ranks a key also computes its Gumbel score, and the last warp,
//      idle, the row's log-sum-exp;
//   -- barrier: warp 0 filters and draws.
// Windowed path: thread t's words are t + 512 k (k < 16), so round k of warp
// w is exactly tile w + 16 k, one word per lane, and warp w builds the list
// of tiles w, w + 16, ... of each window.
// Rows with more than kWin allowed tokens go in windows of whole tiles (the
// same steps per window; each window's keys are ranked together with the
// running top-K).  Results, tie rules and noise are those of the streaming
// pass and of the oracle.
#include <cstdio>
#include <cstring>

#include "pm_device.cuh"
#include "pm_select.cuh"
#include "pm_tile.cuh"
#include "pm_warp.cuh"
#include "pm_host.h"

namespace pm {

constexpr int kMThreads = 512;
constexpr int kMWarps = kMThreads / 32;            // 16
constexpr int kWin = 4096;                         // allowed tokens per window
constexpr int kMaxTiles = 32 * kMaxPer;            // tiles of the largest row (256)
constexpr int kMRounds = kMaxTiles / kMWarps;      // mask words a thread holds (16)
constexpr int kSel = 1024;                         // keys the fast selection path holds
static_assert(kMThreads == 2 * kMaxTiles, "warps 8..15 weigh one tile per thread for the log-sum-exp");

template <int KC>
struct MaskedMem {
  uint32_t val[kWin];          // gathered logits: raw words, then processed fp32 bits
  uint32_t mw[kMRounds * kMThreads];  // the row's mask words (word w of the row at w)
  uint32_t ids[kWin];          // token id of each list position
  uint64_t sel[kSel + KC];     // selection buffer
  uint64_t carry[KC];          // the row's top-K so far, sorted descending
  float score[KC];             // Gumbel scores of the carried keys
  int tc[kMaxTiles];           // allowed tokens per tile
  int toff[kMaxTiles];         // first list position of each tile (of the window)
  float tmx[kMaxTiles];        // tile maxima of x (-inf: nothing finite)
  float tmy[kMaxTiles];        // tile maxima of y = x * inv_temperature
  uint64_t tsx[kMaxTiles];     // tile sums of q52(x - m_t)
  uint64_t tsy[kMaxTiles];
  uint32_t tkx[kMaxTiles];     // tile maxima while they accumulate (ordered keys; 0: none)
  uint32_t tky[kMaxTiles];
  uint32_t tsx3[kMaxTiles][3];  // tile sums while they accumulate: 21-bit digits of each addend
  uint32_t tsy3[kMaxTiles][3];
  uint32_t lmax[kMThreads];    // each thread's largest value (ordered key; 0: none): bound entries
  unsigned hist[256];
  int scal[8];
  uint64_t wbest[kMWarps];
  double redd[8];              // the log-sum-exp tree's eight warp subtrees
  uint32_t rowmax;             // ordered key of the row's largest x (0: nothing finite)
  int nsel;
  int alloc;                   // list positions handed out to the warps (this row)
  int overflow;                // a warp's region passed kWin: the row takes the windowed path
  int excluded;                // a finite value was left out of the selection buffer
  float v0;
  float lse;                   // the row's log-sum-exp when an idle warp computed it during the ranking
};

// A 64-bit sum accumulated in shared memory as three 32-bit counters, one
// per 21-bit digit of each addend (v < 2^63): three native atomic adds that
// return nothing.  Exact while each counter stays below 2^32, i.e. for fewer
// than 2^11 addends -- here one per lane run of a tile.
__device__ __forceinline__ void smem_add3(uint32_t* c, uint64_t v) {
  atomicAdd(&c[0], (uint32_t)(v & 0x1FFFFFu));
  atomicAdd(&c[1], (uint32_t)((v >> 21) & 0x1FFFFFu));
  atomicAdd(&c[2], (uint32_t)(v >> 42));
}
__device__ __forceinline__ uint64_t sum3(const uint32_t* c) {
  return ((uint64_t)c[2] << 42) + ((uint64_t)c[1] << 21) + (uint64_t)c[0];
}

__device__ __forceinline__ float ord_value(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

template <typename T>
__device__ __forceinline__ float staged_value(uint32_t raw, uint32_t id) {
  if constexpr (sizeof(T) == 4) return __uint_as_float(raw);
  else return bf16_bits_to_f32((id & 1u) ? (raw >> 16) : (raw & 0xffffu));
}

// 4-byte asynchronous copy global -> shared, cached in L1 and L2.
__device__ __forceinline__ void cp_async4(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Descending bitonic sort of S[0..n) (n <= P <= 1024, P a power of two,
// S holds P slots) by the whole CTA.
__device__ __forceinline__ void block_sort_desc(uint64_t* S, int n, int P) {
  for (int i = n + threadIdx.x; i < P; i += kMThreads) S[i] = 0ull;
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += kMThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = S[i], y = S[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) { S[i] = y; S[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
}

// Processors on the overridden ids of tile t, which warp w owns in this
// window: logit bias first, then the penalties (the order of process_tile).
// `word` / `wpre` are this lane's mask word of the tile and the allowed
// tokens before it inside the tile; ts the tile's first list position.
template <int KC>
__device__ __noinline__ void masked_overrides(const SampleArgs& a, const pm_row_params& p, int64_t row, int t,
                                                 uint32_t word, int wpre, int ts, MaskedMem<KC>* mm) {
  const int lane = threadIdx.x & 31;
  const uint32_t t0 = (uint32_t)t * kTile;
  auto locate = [&](int id, bool in) -> int {  // list position of id, -1 if disallowed (all lanes call)
    in = in && (uint32_t)id - t0 < (uint32_t)kTile;  // ids out of ascending order: skipped
    const uint32_t e = in ? (uint32_t)id - t0 : 0u;
    const uint32_t wj = __shfl_sync(kFull, word, (int)(e >> 5));
    const int pj = __shfl_sync(kFull, wpre, (int)(e >> 5));
    const uint32_t b = e & 31u;
    if (!in || !((wj >> b) & 1u)) return -1;
    return ts + pj + __popc(wj & ((1u << b) - 1u));
  };
  if (a.bias_off) {
    const int bb = a.bias_off[t], be = a.bias_off[t + 1];
    for (int i0 = bb; i0 < be; i0 += 32) {
      const int i = i0 + lane;
      const bool in = i < be;
      const int pos = locate(in ? a.bias_tok[i] : 0, in);
      if (pos >= 0) mm->val[pos] = __float_as_uint(fadd(__uint_as_float(mm->val[pos]), a.bias_val[i]));
    }
    __syncwarp();
  }
  if (a.ovr_off) {
    const int32_t* off = a.ovr_off + row * (int64_t)(a.n_tiles + 1);
    const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
    const uint32_t* oinf = a.ovr_info + row * (int64_t)a.ovr_cap;
    const int ob = off[t], oe = off[t + 1];
    for (int i0 = ob; i0 < oe; i0 += 32) {
      const int i = i0 + lane;
      const bool in = i < oe;
      const int pos = locate(in ? otok[i] : 0, in);
      if (pos >= 0) {
        const uint32_t info = oinf[i];
        float x = __uint_as_float(mm->val[pos]);
        if (info & 1u) x = x < 0.0f ? fmul(x, p.repetition_penalty) : __fdiv_rn(x, p.repetition_penalty);
        if (info & 2u) x = fsub(x, p.presence_penalty);
        const uint32_t cnt = info >> 8;
        if (cnt) x = fsub(x, fmul(p.frequency_penalty, (float)cnt));
        mm->val[pos] = __float_as_uint(x);
      }
    }
    __syncwarp();
  }
}

// Tile statistics over the list, in balanced runs: thread i takes the
// positions [i CH, (i + 1) CH) of the n-position list (CH = ceil(n / 512));
// the list holds whole tiles, each as one run, so a thread's positions cover
// a few tile parts.  Pass 1 folds each part's maximum into the tile's slot
// (atomic maximum of ordered keys); after a barrier pass 2 folds each part's
// q52 sum against the finished maximum into three 21-bit digit counters.
// Slots must be zero before pass 1.  Pass 1 also gives the thread's largest
// value (ordered key, 0 if none) and, on greedy rows, its best rank key.
template <int KC>
__device__ __forceinline__ void chunk_max(MaskedMem<KC>* mm, int a0, int a1, bool needy, bool greedy, float inv_t,
                                          uint32_t& lmax, uint64_t& lbest) {
  int cur = -1;
  uint32_t kx = 0, ky = 0;
  for (int q = a0; q < a1; ++q) {
    const float x = __uint_as_float(mm->val[q]);
    const uint32_t id = mm->ids[q];
    const int t = (int)(id >> 10);
    if (t != cur) {
      if (kx) atomicMax(&mm->tkx[cur], kx);
      if (ky) atomicMax(&mm->tky[cur], ky);
      cur = t;
      kx = ky = 0;
    }
    if (x > -INFINITY) {
      const uint32_t o = ordkey(x);
      kx = max(kx, o);
      if (needy) ky = max(ky, ordkey(fmul(x, inv_t)));
      if (greedy) {
        const uint64_t kk = rankkey(x, id);
        lbest = kk > lbest ? kk : lbest;
      }
    }
    lmax = max(lmax, kx);
  }
  if (kx) atomicMax(&mm->tkx[cur], kx);
  if (ky) atomicMax(&mm->tky[cur], ky);
}

template <int KC>
__device__ __forceinline__ void chunk_sum(MaskedMem<KC>* mm, int a0, int a1, bool needx, bool needy, float inv_t) {
  auto mof = [](uint32_t k) { return k ? ord_value(k) : -INFINITY; };
  int cur = -1;
  uint64_t sx = 0, sy = 0;
  for (int q = a0; q < a1; q += 2) {
    const bool two = q + 1 < a1;
    const float x0 = __uint_as_float(mm->val[q]);
    const float x1 = two ? __uint_as_float(mm->val[q + 1]) : -INFINITY;
    const int t0 = (int)(mm->ids[q] >> 10);
    const int t1 = two ? (int)(mm->ids[q + 1] >> 10) : t0;
    uint64_t qx0 = 0, qx1 = 0, qy0 = 0, qy1 = 0;
    if (needx) q52x2(fsub(x0, mof(mm->tkx[t0])), fsub(x1, mof(mm->tkx[t1])), qx0, qx1);
    if (needy) {
      const float y0 = x0 > -INFINITY ? fmul(x0, inv_t) : -INFINITY;
      const float y1 = x1 > -INFINITY ? fmul(x1, inv_t) : -INFINITY;
      q52x2(fsub(y0, mof(mm->tky[t0])), fsub(y1, mof(mm->tky[t1])), qy0, qy1);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h == 0 || two) {
        const int t = h ? t1 : t0;
        if (t != cur) {
          if (sx) smem_add3(mm->tsx3[cur], sx);
          if (sy) smem_add3(mm->tsy3[cur], sy);
          cur = t;
          sx = sy = 0;
        }
        sx += h ? qx1 : qx0;
        sy += h ? qy1 : qy0;
      }
    }
  }
  if (sx) smem_add3(mm->tsx3[cur], sx);
  if (sy) smem_add3(mm->tsy3[cur], sy);
}

template <typename T, int KC>
__global__ void __launch_bounds__(kMThreads, 2) k_sample_masked(const __grid_constant__ SampleArgs a) {
  extern __shared__ __align__(128) unsigned char smem_masked[];
  MaskedMem<KC>* mm = reinterpret_cast<MaskedMem<KC>*>(smem_masked);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nt = a.n_tiles;
  const int nw = (int)((a.vocab + 31) >> 5);
  const int KR = (nt + kMWarps - 1) / kMWarps;     // windowed path: rounds in which some warp has a tile
  const int WPT = (nw + kMThreads - 1) / kMThreads;  // mask words per thread (<= 16)
  const uint32_t sval = (uint32_t)__cvta_generic_to_shared(mm->val);
  if (tid == 0) {
    mm->alloc = 0;
    mm->overflow = 0;
    mm->rowmax = 0u;
  }
  __syncthreads();
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    // the row's mask words are requested first, so their DRAM round trip
    // overlaps the read of the row's settings; every load is issued before
    // the first store waits on one
    const uint32_t* mrow = a.mask + row * a.mask_stride;
    uint32_t w[kMRounds];
    {
      const int g0 = 32 * WPT * wid;
#pragma unroll
      for (int j = 0; j < kMRounds; ++j) {
        const int g = g0 + 32 * j + lane;
        w[j] = (j < WPT && g < nw) ? __ldcs(mrow + g) : 0u;
      }
    }
    const pm_row_params p = row_params(a, row);
    const int mode = row_mode(p);
    const bool needx = needs_xstats(a, p, mode);
    const bool needy = mode == kFullDraw;
    const float inv_t = p.inv_temperature;
    const int K = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;
    const T* rowp = reinterpret_cast<const T*>(a.logits) + row * a.row_stride;
    // fold a tile's accumulated slots into its statistics (and the row maximum)
    auto finish_tile = [&](int t) {
      if (needx) {
        const uint32_t k = mm->tkx[t];
        TileStat st;
        st.m = k ? ord_value(k) : -INFINITY;
        st.pad = 0;
        st.s = sum3(mm->tsx3[t]);
        mm->tmx[t] = st.m;
        mm->tsx[t] = st.s;
        a.statx[row * nt + t] = st;
        if (k) atomicMax(&mm->rowmax, k);
      }
      if (needy) {
        const uint32_t k = mm->tky[t];
        TileStat st;
        st.m = k ? ord_value(k) : -INFINITY;
        st.pad = 0;
        st.s = sum3(mm->tsy3[t]);
        mm->tmy[t] = st.m;
        mm->tsy[t] = st.s;
        a.staty[row * nt + t] = st;
      }
    };
    auto clear_tile = [&](int t) {
      mm->tkx[t] = 0u;
      mm->tky[t] = 0u;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        mm->tsx3[t][j] = 0u;
        mm->tsy3[t][j] = 0u;
      }
    };
    uint32_t lmax = 0;   // this thread's largest value seen (bound entry)
    uint64_t lbest = 0;  // greedy: this thread's best key
    // 1. Warp w takes the mask words [32 WPT w, 32 WPT (w + 1)), i.e. the
    //    tiles [WPT w, WPT (w + 1)); thread t of them the WPT words from
    //    WPT t on.  Words -> shared memory (coalesced loads, cut at the
    //    vocabulary), each thread's words back in registers, one warp scan of
    //    the threads' allowed counts and one shared-memory allocation of the
    //    warp's contiguous list region: every allowed token's list position
    //    is known without a CTA barrier.  Then the token ids (a whole word's
    //    32 ids written by the warp together).  After the first barrier,
    //    4-byte asynchronous copies of the logits position-strided over the
    //    whole list and all 512 threads (balanced even when one warp's tiles
    //    hold a block of allowed tokens; coalesced along runs of them), then
    //    the processors on each warp's own tiles.  A row whose list would
    //    pass kWin positions takes the windowed path instead.
    {
      const int g0 = 32 * WPT * wid;
#pragma unroll
      for (int j = 0; j < kMRounds; ++j) {
        if (j < WPT) {
          const int g = g0 + 32 * j + lane;
          if (g == nw - 1 && (a.vocab & 31)) w[j] &= (1u << (a.vocab & 31)) - 1u;
          mm->mw[g] = w[j];
        }
      }
    }
    __syncwarp();
    uint32_t my[kMRounds];
    int ctot = 0;
#pragma unroll
    for (int i = 0; i < kMRounds; ++i) {
      my[i] = i < WPT ? mm->mw[WPT * tid + i] : 0u;
      ctot += __popc(my[i]);
    }
    const int cincl = warp_incl_scan(ctot);
    const int wtot = __shfl_sync(kFull, cincl, 31);
    int wbase = 0;
    if (lane == 0) wbase = atomicAdd(&mm->alloc, wtot);
    wbase = __shfl_sync(kFull, wbase, 0);
    if (wbase + wtot <= kWin) {  // warp-uniform
      int pos = wbase + cincl - ctot;
#pragma unroll
      for (int i = 0; i < kMRounds; ++i) {
        if (i < WPT) {
          const int g = WPT * tid + i;
          if ((g & 31) == 0 && (g >> 5) < nt) mm->toff[g >> 5] = pos;  // a tile starts at this word
          const uint32_t word = my[i];
          unsigned full = __ballot_sync(kFull, word == 0xffffffffu);
          while (full) {  // a fully allowed word: its 32 ids written by the whole warp
            const int j = __ffs(full) - 1;
            full &= full - 1;
            const int pj = __shfl_sync(kFull, pos, j);
            mm->ids[pj + lane] = (uint32_t)(WPT * (32 * wid + j) + i) * 32u + (uint32_t)lane;
          }
          if (word != 0xffffffffu) {
            uint32_t wv = word;
            int q = pos;
            while (wv) {
              mm->ids[q++] = (uint32_t)g * 32u + (uint32_t)(__ffs(wv) - 1);
              wv &= wv - 1;
            }
          }
          pos += __popc(word);
        }
      }
      __syncwarp();
      const int tw0 = WPT * wid;  // the warp's first tile
      if (lane < WPT && tw0 + lane < nt) {
        const int t = tw0 + lane;
        mm->tc[t] = (lane + 1 < WPT && t + 1 < nt ? mm->toff[t + 1] : wbase + wtot) - mm->toff[t];
        clear_tile(t);
      }
    } else if (lane == 0) {
      mm->overflow = 1;
    }
    __syncthreads();
    if (mm->overflow == 0) {  // CTA-uniform
      // the logit copies, position-strided over the whole list: every thread
      // issues about the same number (a warp holding a block of allowed
      // tokens would otherwise issue hundreds), coalesced along runs of
      // allowed tokens
      const int n_all = mm->alloc;
      for (int q = tid; q < n_all; q += kMThreads) {
        const uint32_t id = mm->ids[q];
        cp_async4(sval + 4u * (uint32_t)q, rowp + (sizeof(T) == 4 ? id : (id & ~1u)));
      }
      cp_async_wait_all();
      __syncthreads();
      if constexpr (sizeof(T) == 2) {
        for (int q = tid; q < n_all; q += kMThreads)
          mm->val[q] = __float_as_uint(staged_value<T>(mm->val[q], mm->ids[q]));
        __syncthreads();
      }
      if (a.bias_off || a.ovr_off) {
        const int tw0 = WPT * wid;
        for (int t = tw0; t < tw0 + WPT && t < nt; ++t) {
          const uint32_t word = mm->mw[t * 32 + lane];
          const int pc = __popc(word);
          masked_overrides<KC>(a, p, row, t, word, warp_incl_scan(pc) - pc, mm->toff[t], mm);
        }
        __syncthreads();
      }
    }
    const bool fast = mm->overflow == 0;  // CTA-uniform
    const int total = fast ? mm->alloc : 0;
    // windowed path only: per tile counts (a warp sum per tile-round of the
    // word layout word = tid + 512 k) and their row prefix (lane l sums
    // tiles 8 l .. 8 l + 7)
    if (!fast) {
      lmax = 0;
      lbest = 0;
#pragma unroll 1
      for (int k = 0; k < KR; ++k) {
        const int t = wid + k * kMWarps;
        const int c = (int)__reduce_add_sync(kFull, (unsigned)__popc(mm->mw[tid + k * kMThreads]));
        if (lane == 0 && t < nt) mm->tc[t] = c;
      }
      __syncthreads();
    }
    int cl[kMaxPer];
    int lsum = 0;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int t = lane * kMaxPer + j;
      cl[j] = (!fast && t < nt) ? mm->tc[t] : 0;
      lsum += cl[j];
    }
    const int lincl = warp_incl_scan(lsum);
    const int wtotal = __shfl_sync(kFull, lincl, 31);
    // start of tile t in the row's list (t warp-uniform; t = nt gives the total)
    auto tile_start = [&](int t) -> int {
      if (t >= nt) return wtotal;
      int s0 = lincl - lsum;
#pragma unroll
      for (int j = 0; j < kMaxPer; ++j)
        if (j < (t & (kMaxPer - 1))) s0 += cl[j];
      return __shfl_sync(kFull, s0, t >> 3);
    };
    // this warp's tiles wid + 16 k all sit at element (wid & 7) of lane (wid >> 3) + 2 k
    int mine = lincl - lsum;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j)
      if (j < (wid & (kMaxPer - 1))) mine += cl[j];

    // the row's log-sum-exp from the tile tree's eight warp subtrees (valid
    // once the last window's tree is built)
    auto row_lse = [&]() -> float {
      const float m_row = mm->rowmax ? ord_value(mm->rowmax) : -INFINITY;
      if (!(m_row > -INFINITY)) return -INFINITY;
      const double z = dadd(dadd(dadd(mm->redd[0], mm->redd[1]), dadd(mm->redd[2], mm->redd[3])),
                            dadd(dadd(mm->redd[4], mm->redd[5]), dadd(mm->redd[6], mm->redd[7])));
      return (float)dadd((double)m_row, det_log64(dmul(z, 0x1p-52)));
    };
    bool lse_early = false;  // mm->lse holds the row's log-sum-exp
    int ncarry = 0;
    bool dropped = false;  // the top-K may not hold every key of the row
    uint64_t tau = 0;      // keys at or below the running K-th key cannot enter
    uint64_t best = 0;
    for (int t0 = 0; t0 < nt;) {
      int base = 0, t1 = nt, n = total;
      if (!fast) {
        // the window: tiles [t0, t1), at most kWin allowed tokens (a tile holds at most 1024)
        base = tile_start(t0);
        if (wtotal - base > kWin) {
          int c = 0, run = lincl - lsum;
#pragma unroll
          for (int j = 0; j < kMaxPer; ++j) {
            const int t = lane * kMaxPer + j;
            run += cl[j];
            c += (t >= t0 && t < nt && run - base <= kWin) ? 1 : 0;
          }
          t1 = t0 + (int)__reduce_add_sync(kFull, (unsigned)c);
        }
        n = tile_start(t1) - base;
        // 2. per owned tile (wid + 16 k): token ids of its set bits -> the
        //    window's list (a lane per mask word), 4-byte asynchronous copies
        //    of their logits, lane-strided over the positions, the processors
        //    and the tile's statistics
#pragma unroll 1
        for (int k = 0; k < KR; ++k) {
          const int t = wid + k * kMWarps;
          if (t < t0 || t >= t1) continue;  // warp-uniform
          const int ts = __shfl_sync(kFull, mine, (wid >> 3) + 2 * k) - base;
          if (lane == 0) {
            mm->toff[t] = ts;
            clear_tile(t);
          }
          const uint32_t word = mm->mw[tid + k * kMThreads];
          const int pc = __popc(word);
          const int wpre = warp_incl_scan(pc) - pc;
          int q = ts + wpre;
          const uint32_t id0 = (uint32_t)t * kTile + (uint32_t)lane * 32u;
          uint32_t wv = word;
          while (wv) {
            mm->ids[q++] = id0 + (uint32_t)(__ffs(wv) - 1);
            wv &= wv - 1;
          }
          __syncwarp();
          const int te = ts + mm->tc[t];
          for (int q2 = ts + lane; q2 < te; q2 += 32) {
            const uint32_t id = mm->ids[q2];
            cp_async4(sval + 4u * (uint32_t)q2, rowp + (sizeof(T) == 4 ? id : (id & ~1u)));
          }
          cp_async_wait_all();
          __syncwarp();
          if constexpr (sizeof(T) == 2) {
            for (int q2 = ts + lane; q2 < te; q2 += 32)
              mm->val[q2] = __float_as_uint(staged_value<T>(mm->val[q2], mm->ids[q2]));
            __syncwarp();
          }
          if (a.bias_off || a.ovr_off) masked_overrides<KC>(a, p, row, t, word, wpre, ts, mm);
        }
        __syncthreads();  // the window's list is complete
      }
      const bool last = t1 == nt;
      // 3. tile statistics in balanced runs of positions (two passes), then
      //    thread t finishes tile t of the window
      {
        const int CH = (n + kMThreads - 1) / kMThreads;
        const int a0 = min(n, tid * CH), a1 = min(n, a0 + CH);
        if (needx || needy || mode != kFullDraw) chunk_max<KC>(mm, a0, a1, needy, mode == kGreedy, inv_t, lmax, lbest);
        if (needx || needy) {
          __syncthreads();
          chunk_sum<KC>(mm, a0, a1, needx, needy, inv_t);
        }
        __syncthreads();
        if (tid >= t0 && tid < t1) finish_tile(tid);
      }
      if (mode == kGreedy) {
        const uint64_t wb = warp_max_u64(lbest);
        if (lane == 0) mm->wbest[wid] = wb;
      }
      mm->lmax[tid] = lmax;
      if (tid == 0) {
        mm->nsel = 0;
        mm->excluded = 0;
      }
      __syncthreads();
      // 4. the log-sum-exp tree, after the last window: thread 256 + t weighs
      //    tile t, each of warps 8..15 sums its 32 tiles pairwise (a complete
      //    subtree of the zero-padded 256-leaf tree)
      if (last && needx && wid >= 8) {
        const int t = tid - 256;
        const float m_row = mm->rowmax ? ord_value(mm->rowmax) : -INFINITY;
        const bool ok = t < nt;
        double v = (ok && m_row > -INFINITY) ? tile_weight_of(mm->tmx[t], mm->tsx[t], m_row) : 0.0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double u = __shfl_down_sync(kFull, v, o);
          if ((lane & (2 * o - 1)) == 0) v = dadd(v, u);
        }
        if (lane == 0) mm->redd[wid - 8] = v;
      }
      if (mode == kGreedy) {
#pragma unroll
        for (int w = 0; w < kMWarps; ++w) best = mm->wbest[w] > best ? mm->wbest[w] : best;
      }
      if (mode == kCand && wid == 0) {
        // 5. v0: the largest 16-bit key prefix T with at least K of the
        //    threads' largest values at or above it -- they are K distinct
        //    values, so the K-th largest is >= T.  Two bits a step.
        uint32_t rv[kMThreads / 32];
#pragma unroll
        for (int j = 0; j < kMThreads / 32; ++j) rv[j] = mm->lmax[lane + 32 * j] >> 16;
        uint32_t T16 = 0;
#pragma unroll 1
        for (int b = 14; b >= 0; b -= 2) {
          unsigned n1 = 0, n2 = 0, n3 = 0;
          const uint32_t c1 = T16 | (1u << b), c2 = T16 | (2u << b), c3 = T16 | (3u << b);
#pragma unroll
          for (int j = 0; j < kMThreads / 32; ++j) {
            n1 += rv[j] >= c1 ? 1u : 0u;
            n2 += rv[j] >= c2 ? 1u : 0u;
            n3 += rv[j] >= c3 ? 1u : 0u;
          }
          const uint32_t d = ((int)__reduce_add_sync(kFull, n1) >= K ? 1u : 0u) +
                             ((int)__reduce_add_sync(kFull, n2) >= K ? 1u : 0u) +
                             ((int)__reduce_add_sync(kFull, n3) >= K ? 1u : 0u);
          T16 |= d << b;
        }
        if (lane == 0) mm->v0 = T16 ? ord_value(T16 << 16) : -INFINITY;
      }
      __syncthreads();
      if (mode == kCand) {
        // 6. keys that can still enter the top-K -> the selection buffer,
        //    position-strided over the window's list
        const float v0 = mm->v0;
        bool excl = false;
        for (int q0 = 0; q0 < n; q0 += kMThreads) {
          const int q = q0 + tid;
          const float x = q < n ? __uint_as_float(mm->val[q]) : -INFINITY;
          bool ok = x > -INFINITY && x >= v0;
          uint64_t key = 0;
          if (ok) {
            key = rankkey(x, mm->ids[q]);
            ok = key > tau;
          }
          excl |= x > -INFINITY && !ok;
          const unsigned bal = __ballot_sync(kFull, ok);
          if (bal) {
            int at = 0;
            if (lane == 0) at = atomicAdd(&mm->nsel, __popc(bal));
            at = __shfl_sync(kFull, at, 0) + __popc(bal & ((1u << lane) - 1u));
            if (ok && at < kSel) mm->sel[at] = key;
          }
        }
        if (__any_sync(kFull, excl) && lane == 0) mm->excluded = 1;
        __syncthreads();
        const int ns = mm->nsel;
        dropped |= mm->excluded != 0;
        if (ns <= kSel) {
          if (ncarry) {  // CTA-uniform: nothing is carried into the first window
            for (int i = tid; i < ncarry; i += kMThreads) mm->sel[ns + i] = mm->carry[i];
            __syncthreads();
          }
          const int tot = ns + ncarry;
          dropped |= tot > K;
          if (tot <= kMThreads) {
            // 7. rank by counting the larger keys (keys are unique); the K
            //    largest land sorted in the carry, with their Gumbel scores
            if (tid < tot) {
              const uint64_t kk = mm->sel[tid];
              int rank = 0;
#pragma unroll 4
              for (int j = 0; j < tot; ++j) rank += mm->sel[j] > kk;
              if (rank < K) {
                mm->carry[rank] = kk;
                if (last) mm->score[rank] = fadd(fmul(key_value(kk), inv_t), row_gumbel(a, row, key_index(kk)));
              }
            }
            // the last warp, idle while the ranking runs, computes the row's
            // log-sum-exp (the draw then only reads it)
            lse_early = last && needx && tot <= kMThreads - 32;  // CTA-uniform
            if (lse_early && wid == kMWarps - 1 && lane == 0) mm->lse = row_lse();
            ncarry = tot < K ? tot : K;
            __syncthreads();
          } else {
            ncarry = block_topk_sorted(mm->sel, tot, K, mm->carry, KC, mm->hist, mm->scal);
            __syncthreads();
            if (last) {
              for (int r = tid; r < ncarry; r += kMThreads)
                mm->score[r] = fadd(fmul(key_value(mm->carry[r]), inv_t), row_gumbel(a, row, key_index(mm->carry[r])));
              __syncthreads();
            }
          }
        } else {
          // more than kSel keys qualify: radix-select the K-th key over the
          // window (keys recomputed from the list) and the carry, keep the K
          dropped = true;
          uint64_t prefix = 0;
          int need = K;
          for (int shift = 56; shift >= 0; shift -= 8) {
            for (int i = tid; i < 256; i += kMThreads) mm->hist[i] = 0;
            __syncthreads();
            const int hs = shift + 8;
            for (int i = tid; i < n + ncarry; i += kMThreads) {
              uint64_t kk;
              if (i < n) {
                const float x = __uint_as_float(mm->val[i]);
                if (!(x > -INFINITY) || x < v0) continue;
                kk = rankkey(x, mm->ids[i]);
                if (kk <= tau) continue;
              } else {
                kk = mm->carry[i - n];
              }
              if (hs < 64 && (kk >> hs) != (prefix >> hs)) continue;
              atomicAdd(&mm->hist[(kk >> shift) & 255], 1u);
            }
            __syncthreads();
            if (wid == 0) {
              int above, in_bin;
              const int d = warp_find_digit(mm->hist, need, &above, &in_bin);
              if (lane == 0) { mm->scal[0] = d; mm->scal[1] = above; mm->scal[2] = in_bin; }
            }
            __syncthreads();
            need -= mm->scal[1];
            prefix |= (uint64_t)(mm->scal[0] & 255) << shift;
            const bool whole = mm->scal[2] == need;
            __syncthreads();
            if (whole) break;  // every key of the bin is in: keys >= prefix are exactly the top K
          }
          if (tid == 0) mm->nsel = 0;
          __syncthreads();
          for (int i = tid; i < n + ncarry; i += kMThreads) {
            uint64_t kk;
            if (i < n) {
              const float x = __uint_as_float(mm->val[i]);
              if (!(x > -INFINITY) || x < v0) continue;
              kk = rankkey(x, mm->ids[i]);
              if (kk <= tau) continue;
            } else {
              kk = mm->carry[i - n];
            }
            if (kk >= prefix) mm->sel[atomicAdd(&mm->nsel, 1)] = kk;
          }
          __syncthreads();
          int P = 1;
          while (P < K) P <<= 1;
          block_sort_desc(mm->sel, K, P);
          for (int i = tid; i < K; i += kMThreads) mm->carry[i] = mm->sel[i];
          ncarry = K;
          __syncthreads();
          if (last) {
            for (int r = tid; r < ncarry; r += kMThreads)
              mm->score[r] = fadd(fmul(key_value(mm->carry[r]), inv_t), row_gumbel(a, row, key_index(mm->carry[r])));
            __syncthreads();
          }
        }
        tau = ncarry == K ? mm->carry[K - 1] : 0ull;
      }
      lmax = 0;  // each window's bound comes from its own values
      t0 = t1;
    }
    // 8. the draw (warp 0)
    if (wid == 0) {
      float c = __int_as_float(0x7fc00000);
      if (needx) c = lse_early ? mm->lse : row_lse();
      int tok = 0, ns = 0;
      float x_tok = -INFINITY;
      if (mode == kGreedy) {
        if (best) {  // nothing finite at all: token 0, as the streaming pass
          tok = (int)key_index(best);
          x_tok = key_value(best);
        }
      } else if (mode == kCand) {
        tok = warp_filter_draw(a, p, row, mm->carry, ncarry, !dropped, c, &ns, mm->score, &x_tok);
        if (tok >= 0 && a.surv_ids && lane == 0) write_survivors(a, p, row, mm->carry, ns);
      } else {
        tok = warp_full_draw<T>(a, p, row, &x_tok);  // reads the y statistics this CTA wrote
      }
      if (lane == 0) write_row(a, row, mode, tok, x_tok, c, ns);
      if (lane == 0) {
        mm->alloc = 0;
        mm->overflow = 0;
        mm->rowmax = 0u;
      }
    }
    __syncthreads();
  }
}

}  // namespace pm

namespace {

template <typename T, int KC>
int launch_masked_t(const pm::SampleArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(pm::MaskedMem<KC>);
  static pmh::DeviceOnce once;
  once([&] {
    cudaFuncSetAttribute(pm::k_sample_masked<T, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  int64_t grid = a.rows;
  if (grid > (int64_t)pmh::num_sms() * 2) grid = (int64_t)pmh::num_sms() * 2;
  pm::k_sample_masked<T, KC><<<(unsigned)grid, pm::kMThreads, smem, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : pmh::cuda_fail(e);
}

}  // namespace

int pm_launch_masked(int dtype, int KC, const pm::SampleArgs& a, cudaStream_t st) {
  const bool bf = dtype == PM_DTYPE_BF16;
  if (KC == 64) return bf ? launch_masked_t<__nv_bfloat16, 64>(a, st) : launch_masked_t<float, 64>(a, st);
  return bf ? launch_masked_t<__nv_bfloat16, 256>(a, st) : launch_masked_t<float, 256>(a, st);
}
