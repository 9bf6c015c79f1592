// pm_masked.cuh -- the sampling pass for rows with an allowed-token mask,
// one CTA per row.
//
// A constrained-decoding mask usually allows a small part of the vocabulary
// (a grammar state, a forced token).  Every processed value of a disallowed
// token is -inf and contributes nothing to the row's log-sum-exp, candidates
// or draw, so this pass reads the row's mask words first and then fetches
// only the logits of allowed tokens: 4-byte loads cached in L2 only, many in
// flight per thread, into a shared-memory window compacted in ascending
// token order.  The HBM traffic is the mask plus the 32-byte sectors that
// hold an allowed token, instead of the whole row.
//
// Per row (8 warps, one CTA):
//   1. mask words -> shared memory (cut at the vocabulary), allowed count per
//      1024-token tile, their prefix (tile offsets in the row's list);
//   2. windows of whole tiles holding at most kWin allowed tokens: gather,
//      keys rankkey(x, id), processors on the few overridden ids, exact tile
//      statistics (the same 1024-token tiles as every other pass, so the
//      log-sum-exp is bit-identical), selection: the window's keys above the
//      running K-th key join the carried top-K, radix-selected back to K;
//   3. the draw by warp 0: greedy argmax, filters + Gumbel-max over the
//      sorted top-K, or the two-level inverse CDF over the y statistics.
// Results, tie rules and noise are those of the streaming pass.
#pragma once

namespace pm {

constexpr int kMThreads = 256;
constexpr int kMWarps = kMThreads / 32;
constexpr int kWin = 4096;                          // allowed tokens per window
constexpr int kMaxTiles = 32 * kMaxPer;             // tiles of the largest row (256)
constexpr int kMaxWords = kMaxTiles * 32;           // mask words of the largest row (8192)
constexpr int kSel = 1024;                          // keys the fast selection path holds
constexpr int kRun = kWin / kMThreads;              // positions a thread owns in a window (16)
static_assert(kMThreads == kMaxTiles && kMWarps == 8, "the row log-sum-exp gives one tile per thread, 8 warps");

template <int KC>
struct MaskedMem {
  uint32_t val[kWin];         // gathered raw words, then the processed fp32 values (bits), by position
  uint32_t ids[kWin];         // token id of each position
  uint32_t mw[kMaxWords];     // the row's mask words
  uint16_t wpre[kMaxWords];   // allowed tokens before each word inside its tile
  uint64_t sel[kSel + KC];    // selection buffer
  uint64_t carry[KC];         // the row's top-K so far, sorted descending
  uint32_t tmx[kMaxTiles];    // tile maxima of x as ordered keys (0: nothing finite)
  uint32_t tmy[kMaxTiles];    // tile maxima of y = x * inv_temperature
  uint64_t tsx[kMaxTiles];    // tile sums of q52(x - m_t)
  uint64_t tsy[kMaxTiles];
  uint32_t tsx3[kMaxTiles][3];  // the sums while they accumulate: 21-bit digits of each addend
  uint32_t tsy3[kMaxTiles][3];
  int toff[kMaxTiles + 1];    // allowed tokens before each tile
  unsigned hist[256];
  int scal[8];
  uint64_t wbest[kMWarps];
  uint32_t rmx[kMThreads];    // each thread's run maximum (ordered key; 0: nothing finite)
  double redd[kMWarps];       // per-warp subtrees of the log-sum-exp
  float redf[kMWarps];
  float score[KC];            // Gumbel scores of the carried keys
  int nsel;
  float v0;
};

__device__ __forceinline__ float ord_value(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

// Segmented reductions over lanes whose segment ids are contiguous runs
// (positions sorted by token, segments = tiles): the first lane of each run
// ends up with the run's total.
__device__ __forceinline__ uint32_t seg_max_u32(uint32_t v, int seg) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t ov = __shfl_down_sync(kFull, v, o);
    const int os = __shfl_down_sync(kFull, seg, o);
    if (lane + o < 32 && os == seg) v = max(v, ov);
  }
  return v;
}
__device__ __forceinline__ uint64_t seg_sum_u64(uint64_t v, int seg) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t ov = __shfl_down_sync(kFull, v, o);
    const int os = __shfl_down_sync(kFull, seg, o);
    if (lane + o < 32 && os == seg) v += ov;
  }
  return v;
}
__device__ __forceinline__ bool seg_head(int seg) {
  const int prev = __shfl_up_sync(kFull, seg, 1);
  return (threadIdx.x & 31) == 0 || prev != seg;
}

// A 64-bit sum accumulated in shared memory as three 32-bit counters, one
// per 21-bit digit of each addend (v < 2^63): three native atomic adds that
// return nothing, so no thread waits on them.  Exact while each counter
// stays below 2^32: fewer than 2^11 addends, as a tile has at most 1024
// values and each thread adds a tile's run once.
__device__ __forceinline__ void smem_add3(uint32_t* c, uint64_t v) {
  atomicAdd(&c[0], (uint32_t)(v & 0x1FFFFFu));
  atomicAdd(&c[1], (uint32_t)((v >> 21) & 0x1FFFFFu));
  atomicAdd(&c[2], (uint32_t)(v >> 42));
}
__device__ __forceinline__ uint64_t sum3(const uint32_t* c) {
  return ((uint64_t)c[2] << 42) + ((uint64_t)c[1] << 21) + (uint64_t)c[0];
}

// The processed logit of one token of a row (bias, penalties, mask): the
// single-token form of process_tile, for the rare paths.
__device__ float processed_value(const SampleArgs& a, int dtype, const pm_row_params& p, int64_t row, int tok) {
  float x;
  if (dtype == PM_DTYPE_F32) x = reinterpret_cast<const float*>(a.logits)[row * a.row_stride + tok];
  else x = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(a.logits)[row * a.row_stride + tok]);
  const int tile = tok / kTile;
  if (a.bias_off)
    for (int i = a.bias_off[tile]; i < a.bias_off[tile + 1]; ++i)
      if (a.bias_tok[i] == tok) x = fadd(x, a.bias_val[i]);
  if (a.ovr_off) {
    const int32_t* off = a.ovr_off + row * (int64_t)(a.n_tiles + 1) + tile;
    const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
    int lo = off[0];
    while (lo < off[1] && otok[lo] != tok) ++lo;  // a tile's entries are in no particular order
    if (lo < off[1]) {
      const uint32_t info = a.ovr_info[row * (int64_t)a.ovr_cap + lo];
      if (info & 1u) x = x < 0.0f ? fmul(x, p.repetition_penalty) : __fdiv_rn(x, p.repetition_penalty);
      if (info & 2u) x = fsub(x, p.presence_penalty);
      const uint32_t cnt = info >> 8;
      if (cnt) x = fsub(x, fmul(p.frequency_penalty, (float)cnt));
    }
  }
  if (a.mask && !((a.mask[row * a.mask_stride + (tok >> 5)] >> (tok & 31)) & 1u)) x = -INFINITY;
  return x;
}

// Position of token id in the window list that starts at `base`, or -1 when
// the mask disallows it.
template <int KC>
__device__ __forceinline__ int masked_pos(const MaskedMem<KC>* mm, int id, int base) {
  const int w = id >> 5, j = id & 31;
  const uint32_t word = mm->mw[w];
  if (!((word >> j) & 1u)) return -1;
  return mm->toff[id >> 10] - base + mm->wpre[w] + __popc(word & ((1u << j) - 1u));
}

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

template <typename T>
__device__ __forceinline__ float staged_value(uint32_t raw, int id) {
  if constexpr (sizeof(T) == 4) return __uint_as_float(raw);
  else return bf16_bits_to_f32((id & 1) ? (raw >> 16) : (raw & 0xffffu));
}

template <typename T, int KC>
__global__ void __launch_bounds__(kMThreads, 2) k_sample_masked(const __grid_constant__ SampleArgs a) {
  extern __shared__ __align__(128) unsigned char smem_masked[];
  MaskedMem<KC>* mm = reinterpret_cast<MaskedMem<KC>*>(smem_masked);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nt = a.n_tiles;
  const int nw = (int)((a.vocab + 31) >> 5);
  const int KW = (nt * 32 + kMThreads - 1) / kMThreads;  // mask-word rounds: word tid + 256 k is in tile 8 k + wid
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const pm_row_params p = row_params(a, row);
    const int mode = row_mode(p);
    const bool needx = needs_xstats(a, p, mode);
    const bool needy = mode == kFullDraw;
    const bool want_max = needx || needy || mode == kCand;
    const float inv_t = p.inv_temperature;
    const int K = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;
    // 1. mask words (cut at the vocabulary), in-tile word prefixes, tile counts;
    //    all loads first, then the scans
    const uint32_t* mrow = a.mask + row * a.mask_stride;
    uint32_t wr[kMaxPer * 4];
#pragma unroll
    for (int k = 0; k < kMaxPer * 4; ++k) {
      const int w = tid + k * kMThreads;
      wr[k] = (k < KW && w < nw) ? __ldcs(mrow + w) : 0u;
    }
    // groups of four rounds without a branch between them, so their warp
    // scans overlap; rounds past the row write zero counts into slots that
    // exist (kMaxWords words, kMaxTiles tiles) and nothing reads
#pragma unroll
    for (int k0 = 0; k0 < kMaxPer * 4; k0 += 4) {
      if (k0 >= KW) break;  // CTA-uniform
#pragma unroll
      for (int k = k0; k < k0 + 4; ++k) {
        const int w = tid + k * kMThreads;
        uint32_t word = wr[k];
        if (w == nw - 1 && (a.vocab & 31)) word &= (1u << (a.vocab & 31)) - 1u;
        mm->mw[w] = word;
        const int pc = __popc(word);
        const int incl = warp_incl_scan(pc);
        mm->wpre[w] = (uint16_t)(incl - pc);
        if (lane == 31) mm->toff[k * kMWarps + wid + 1] = incl;
      }
    }
    // tile statistics start at zero (each window fills its own tiles)
    mm->tmx[tid] = 0;
    mm->tmy[tid] = 0;
    mm->tsx[tid] = 0;
    mm->tsy[tid] = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      mm->tsx3[tid][j] = 0;
      mm->tsy3[tid][j] = 0;
    }
    __syncthreads();
    if (wid == 0) {
      int c[kMaxPer];
      int s = 0;
#pragma unroll
      for (int k = 0; k < kMaxPer; ++k) {
        const int t = lane * kMaxPer + k;
        c[k] = t < nt ? mm->toff[t + 1] : 0;
        s += c[k];
      }
      const int incl = warp_incl_scan(s);
      int run = incl - s;
#pragma unroll
      for (int k = 0; k < kMaxPer; ++k) {
        const int t = lane * kMaxPer + k;
        run += c[k];
        if (t < nt) mm->toff[t + 1] = run;
      }
      if (lane == 0) mm->toff[0] = 0;
    }
    __syncthreads();
    int ncarry = 0;
    bool dropped = false;  // a selection left keys out: the top-K may not hold every candidate
    uint64_t tau = 0;
    uint64_t best = 0;
    const T* rowp = reinterpret_cast<const T*>(a.logits) + row * a.row_stride;
    auto vf = [mm](int i) { return __uint_as_float(mm->val[i]); };
    // 2. windows of whole tiles
    for (int t0 = 0; t0 < nt;) {
      const int base = mm->toff[t0];
      int lo = t0 + 1, hi = nt;  // the last tile end whose window holds at most kWin tokens
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (mm->toff[mid] - base <= kWin) lo = mid; else hi = mid - 1;
      }
      const int t1 = lo;
      const int n = mm->toff[t1] - base;
      // the window's token ids in ascending order: lane per mask word, the
      // words and offsets of eight rounds loaded before their bit loops
#pragma unroll
      for (int k0 = 0; k0 < kMaxPer * 4; k0 += 8) {
        if (k0 >= KW) break;  // CTA-uniform
        uint32_t wv[8];
        int pv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int k = k0 + u;
          const int tile = k * kMWarps + wid;
          const bool in = k < KW && tile >= t0 && tile < t1;
          const int w = tid + k * kMThreads;
          wv[u] = in ? mm->mw[w] : 0u;
          pv[u] = in ? mm->toff[tile] - base + mm->wpre[w] : 0;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          uint32_t word = wv[u];
          int pos = pv[u];
          const int id0 = (tid + (k0 + u) * kMThreads) * 32;
          while (word) {
            mm->ids[pos++] = (uint32_t)(id0 + __ffs(word) - 1);
            word &= word - 1;
          }
        }
      }
      __syncthreads();
      // their logits: 4-byte loads cached in L2 only (one 32-byte sector
      // each; an L1-allocating load would fill the whole 128-byte line), all
      // kRun of a thread in flight before the shared-memory stores.  bf16
      // rows load the 32-bit word holding the value and widen it here.
      {
        uint32_t v[kRun];
#pragma unroll
        for (int r = 0; r < kRun; ++r) {
          const int i = tid + r * kMThreads;
          v[r] = 0u;
          if (i < n) {
            const uint32_t id = mm->ids[i];
            v[r] = __ldcg(reinterpret_cast<const unsigned int*>(rowp + (sizeof(T) == 4 ? id : (id & ~1u))));
          }
        }
#pragma unroll
        for (int r = 0; r < kRun; ++r) {
          const int i = tid + r * kMThreads;
          if (i < n) mm->val[i] = sizeof(T) == 4 ? v[r] : __float_as_uint(staged_value<T>(v[r], (int)mm->ids[i]));
        }
      }
      __syncthreads();
      // processors on the window's overridden ids (bias first, then penalties)
      if (a.bias_off) {
        for (int i = a.bias_off[t0] + tid; i < a.bias_off[t1]; i += kMThreads) {
          const int pos = masked_pos(mm, a.bias_tok[i], base);
          if (pos >= 0) mm->val[pos] = __float_as_uint(fadd(vf(pos), a.bias_val[i]));
        }
        __syncthreads();
      }
      if (a.ovr_off) {
        const int32_t* off = a.ovr_off + row * (int64_t)(nt + 1);
        const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
        const uint32_t* oinf = a.ovr_info + row * (int64_t)a.ovr_cap;
        for (int i = off[t0] + tid; i < off[t1]; i += kMThreads) {
          const int pos = masked_pos(mm, otok[i], base);
          if (pos < 0) continue;
          const uint32_t info = oinf[i];
          float x = vf(pos);
          if (info & 1u) x = x < 0.0f ? fmul(x, p.repetition_penalty) : __fdiv_rn(x, p.repetition_penalty);
          if (info & 2u) x = fsub(x, p.presence_penalty);
          const uint32_t cnt = info >> 8;
          if (cnt) x = fsub(x, fmul(p.frequency_penalty, (float)cnt));
          mm->val[pos] = __float_as_uint(x);
        }
        __syncthreads();
      }
      // each thread owns a contiguous run of at most kRun positions (tiles are
      // runs of positions), held in registers: values and token ids
      const int rl = (n + kMThreads - 1) / kMThreads;
      const int q0 = min(n, tid * rl);
      const int len = min(n, q0 + rl) - q0;
      float xv[kRun];
      uint32_t iv[kRun];
#pragma unroll
      for (int r = 0; r < kRun; ++r) {
        xv[r] = r < len ? vf(q0 + r) : -INFINITY;
        iv[r] = r < len ? mm->ids[q0 + r] : 0u;
      }
      // exact tile statistics: maxima, then q52 sums against them; a run's
      // tiles are flushed to shared memory when the tile changes
      if (want_max) {
        int cur = (int)(iv[0] >> 10);
        uint32_t mx = 0, my = 0, rmax = 0;
#pragma unroll
        for (int r = 0; r < kRun; ++r) {
          if (r < len) {
            const int seg = (int)(iv[r] >> 10);
            if (seg != cur) {
              if (mx) atomicMax(&mm->tmx[cur], mx);
              if (my) atomicMax(&mm->tmy[cur], my);
              cur = seg;
              mx = my = 0;
            }
            if (xv[r] > -INFINITY) {
              mx = max(mx, ordkey(xv[r]));
              rmax = max(rmax, ordkey(xv[r]));
              if (needy) my = max(my, ordkey(fmul(xv[r], inv_t)));
            }
          }
        }
        if (len > 0) {
          if (mx) atomicMax(&mm->tmx[cur], mx);
          if (my) atomicMax(&mm->tmy[cur], my);
        }
        mm->rmx[tid] = rmax;
        __syncthreads();
      }
      if (needx || needy) {
        // q52 of -inf or NaN is 0: positions past the run and tiles with
        // nothing finite add nothing
        auto tile_m = [](uint32_t o) { return o ? ord_value(o) : -INFINITY; };
        int cur = (int)(iv[0] >> 10);
        uint64_t sx = 0, sy = 0;
#pragma unroll
        for (int r = 0; r < kRun; r += 2) {
          uint64_t qx0 = 0, qx1 = 0, qy0 = 0, qy1 = 0;
          const uint32_t s0 = iv[r] >> 10, s1 = iv[r + 1] >> 10;
          if (needx) {
            const float d0 = r < len ? fsub(xv[r], tile_m(mm->tmx[s0])) : -INFINITY;
            const float d1 = r + 1 < len ? fsub(xv[r + 1], tile_m(mm->tmx[s1])) : -INFINITY;
            q52x2(d0, d1, qx0, qx1);
          }
          if (needy) {
            const float d0 = r < len && xv[r] > -INFINITY ? fsub(fmul(xv[r], inv_t), tile_m(mm->tmy[s0])) : -INFINITY;
            const float d1 = r + 1 < len && xv[r + 1] > -INFINITY
                                 ? fsub(fmul(xv[r + 1], inv_t), tile_m(mm->tmy[s1])) : -INFINITY;
            q52x2(d0, d1, qy0, qy1);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (r + h < len) {
              const int seg = (int)(h ? s1 : s0);
              if (seg != cur) {
                if (sx) smem_add3(mm->tsx3[cur], sx);
                if (sy) smem_add3(mm->tsy3[cur], sy);
                cur = seg;
                sx = sy = 0;
              }
              sx += h ? qx1 : qx0;
              sy += h ? qy1 : qy0;
            }
          }
        }
        if (len > 0) {
          if (sx) smem_add3(mm->tsx3[cur], sx);
          if (sy) smem_add3(mm->tsy3[cur], sy);
        }
        __syncthreads();
        for (int t = t0 + tid; t < t1; t += kMThreads) {
          TileStat st;
          st.pad = 0;
          if (needx) {
            st.m = mm->tmx[t] ? ord_value(mm->tmx[t]) : -INFINITY;
            st.s = sum3(mm->tsx3[t]);
            mm->tsx[t] = st.s;
            a.statx[row * nt + t] = st;
          }
          if (needy) {
            st.m = mm->tmy[t] ? ord_value(mm->tmy[t]) : -INFINITY;
            st.s = sum3(mm->tsy3[t]);
            mm->tsy[t] = st.s;
            a.staty[row * nt + t] = st;
          }
        }
      }
      // selection
      if (mode == kGreedy) {
        uint64_t b = 0;
#pragma unroll
        for (int r = 0; r < kRun; ++r) {
          const uint64_t k = rankkey(xv[r], iv[r]);
          if (r < len && xv[r] > -INFINITY && k > b) b = k;  // nothing finite at all: token 0, as the streaming pass
        }
        b = warp_max_u64(b);
        if (lane == 0) mm->wbest[wid] = b;
        __syncthreads();
#pragma unroll
        for (int w = 0; w < kMWarps; ++w) best = mm->wbest[w] > best ? mm->wbest[w] : best;
      } else if (mode == kCand) {
        // v0: the K-th largest of the threads' run maxima bounds the window's
        // top-K from below (K distinct tokens reach it); the K-th largest of
        // their upper 16 key bits, padded with zero bits, still does.  Warp 0
        // finds it two bits at a time: the largest T with at least K run
        // maxima >= T.
        if (wid == 0) {
          uint32_t rv[kMThreads / 32];
#pragma unroll
          for (int j = 0; j < kMThreads / 32; ++j) rv[j] = mm->rmx[lane + 32 * j] >> 16;
          uint32_t T = 0;
#pragma unroll
          for (int b = 14; b >= 0; b -= 2) {
            unsigned n1 = 0, n2 = 0, n3 = 0;
#pragma unroll
            for (int j = 0; j < kMThreads / 32; ++j) {
              n1 += rv[j] >= (T | (1u << b)) ? 1u : 0u;
              n2 += rv[j] >= (T | (2u << b)) ? 1u : 0u;
              n3 += rv[j] >= (T | (3u << b)) ? 1u : 0u;
            }
            const uint32_t d = ((int)__reduce_add_sync(kFull, n1) >= K ? 1u : 0u) +
                               ((int)__reduce_add_sync(kFull, n2) >= K ? 1u : 0u) +
                               ((int)__reduce_add_sync(kFull, n3) >= K ? 1u : 0u);
            T |= d << b;
          }
          if (lane == 0) {
            mm->v0 = T ? ord_value(T << 16) : -INFINITY;
            mm->nsel = 0;
          }
        }
        __syncthreads();
        const float v0 = mm->v0;
        // keys of the window that can still enter the top-K
        {
          uint32_t okm = 0;
#pragma unroll
          for (int r = 0; r < kRun; ++r)
            if (r < len && xv[r] > -INFINITY && xv[r] >= v0 && rankkey(xv[r], iv[r]) > tau) okm |= 1u << r;
          const int c = __popc(okm);
          const int incl = warp_incl_scan(c);
          int at = 0;
          if (lane == 31 && incl) at = atomicAdd(&mm->nsel, incl);
          at = __shfl_sync(kFull, at, 31) + incl - c;
#pragma unroll
          for (int r = 0; r < kRun; ++r)
            if ((okm >> r) & 1u) {
              if (at < kSel) mm->sel[at] = rankkey(xv[r], iv[r]);
              ++at;
            }
        }
        __syncthreads();
        const int ns = mm->nsel;
        if (ns <= kSel) {
          if (ncarry) {  // CTA-uniform: nothing carried into the first window
            for (int i = tid; i < ncarry; i += kMThreads) mm->sel[ns + i] = mm->carry[i];
            __syncthreads();
          }
          const int total = ns + ncarry;
          dropped |= total > K;
          if (total <= 512) {
            // rank by counting: the K largest land sorted in the carry
            for (int i = tid; i < total; i += kMThreads) {
              const uint64_t k = mm->sel[i];
              int rank = 0;
#pragma unroll 8
              for (int j = 0; j < total; ++j) rank += mm->sel[j] > k;
              if (rank < K) mm->carry[rank] = k;
            }
            ncarry = total < K ? total : K;
          } else {
            ncarry = block_topk_sorted(mm->sel, total, K, mm->carry, KC, mm->hist, mm->scal);
          }
        } else {
          // more than kSel keys qualify: radix-select the K-th key over the
          // window (keys recomputed on the fly) and the carry, then keep the K
          dropped = true;
          uint64_t prefix = 0;
          int need = K;
          for (int shift = 56; shift >= 0; shift -= 8) {
            for (int i = tid; i < 256; i += kMThreads) mm->hist[i] = 0;
            __syncthreads();
            const int hs = shift + 8;
            for (int i = tid; i < n + ncarry; i += kMThreads) {
              uint64_t k;
              if (i < n) {
                const float x = vf(i);
                if (!(x > -INFINITY) || x < v0) continue;
                k = rankkey(x, mm->ids[i]);
                if (k <= tau) continue;
              } else {
                k = mm->carry[i - n];
              }
              if (hs < 64 && (k >> hs) != (prefix >> hs)) continue;
              atomicAdd(&mm->hist[(k >> shift) & 255], 1u);
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
            uint64_t k;
            if (i < n) {
              const float x = vf(i);
              if (!(x > -INFINITY) || x < v0) continue;
              k = rankkey(x, mm->ids[i]);
              if (k <= tau) continue;
            } else {
              k = mm->carry[i - n];
            }
            if (k >= prefix) mm->sel[atomicAdd(&mm->nsel, 1)] = k;
          }
          __syncthreads();
          int P = 1;
          while (P < K) P <<= 1;
          block_sort_desc(mm->sel, K, P);
          for (int i = tid; i < K; i += kMThreads) mm->carry[i] = mm->sel[i];
          ncarry = K;
        }
        __syncthreads();
        tau = ncarry == K ? mm->carry[K - 1] : 0ull;
      }
      if (mode != kCand) __syncthreads();  // (candidate rows have just passed one)
      t0 = t1;
    }
    // 3. the draw.  Log-sum-exp by the whole CTA: thread t weighs tile t
    //    (kMThreads = kMaxTiles), each warp sums its 32 tiles pairwise, and
    //    the eight warp sums close the same zero-padded 256-leaf pairwise tree
    //    as the one-warp combine (every warp subtree is one of its subtrees),
    //    so the bits agree.  The carried keys' Gumbel scores meanwhile.
    float m_row = -INFINITY;
    if (needx) {
      const bool ok = tid < nt && mm->tmx[tid] != 0;
      const float mt = ok ? ord_value(mm->tmx[tid]) : -INFINITY;
      const uint64_t st = ok ? mm->tsx[tid] : 0ull;
      const float wmx = warp_max(mt);
      if (lane == 0) mm->redf[wid] = wmx;
      __syncthreads();
#pragma unroll
      for (int w = 0; w < kMWarps; ++w) m_row = fmaxf(m_row, mm->redf[w]);
      double v = m_row > -INFINITY ? tile_weight_of(mt, st, m_row) : 0.0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_down_sync(kFull, v, o);
        if ((lane & (2 * o - 1)) == 0) v = dadd(v, t);
      }
      if (lane == 0) mm->redd[wid] = v;
    }
    if (mode == kCand)
      for (int r = tid; r < ncarry; r += kMThreads)
        mm->score[r] = fadd(fmul(key_value(mm->carry[r]), inv_t), row_gumbel(a, row, key_index(mm->carry[r])));
    __syncthreads();
    if (wid == 0) {
      float c = __int_as_float(0x7fc00000);
      if (needx) {
        c = -INFINITY;
        if (m_row > -INFINITY) {
          const double z = dadd(dadd(dadd(mm->redd[0], mm->redd[1]), dadd(mm->redd[2], mm->redd[3])),
                                dadd(dadd(mm->redd[4], mm->redd[5]), dadd(mm->redd[6], mm->redd[7])));
          c = (float)dadd((double)m_row, det_log64(dmul(z, 0x1p-52)));
        }
      }
      int tok = 0, ns = 0;
      float x_tok = -INFINITY;
      if (mode == kGreedy) {
        if (best) {
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
    }
    __syncthreads();
  }
}

}  // namespace pm
