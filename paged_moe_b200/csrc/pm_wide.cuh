// pm_wide.cuh -- rows whose unbounded top-p / min-p survivors outrun the
// candidate buffers.
//
// The fused passes keep the 256 best keys of a row without top_k.  When
// top-p or min-p keeps more than that, the row is flagged (status bit 0) and
// this kernel finishes it exactly, one CTA per flagged row, by searches over
// the row instead of a sorted list:
//   n_p  = how many ranks top-p keeps: an MSD radix walk over the 64-bit
//          rank keys with q52 mass histograms finds the smallest key whose
//          mass above it is below 2^52 - Q (the keep rule of the filters);
//   n_m  = how many ranks min-p keeps: one counting pass (log-prob is
//          monotone in rank);
//   the cut = the n-th largest key (n from n_p, n_m, min_tokens_to_keep), by
//          a radix walk over counts;
//   the draw = Gumbel-max over the keys at or above the cut.
// Every pass re-reads the row (from L2 when it is still there) and applies
// the processors again.  Survivor lists are not produced for such rows
// (status bit 3 when they were asked for).
#pragma once

namespace pm {

constexpr int kWThreads = 256;
constexpr int kWWarps = kWThreads / 32;

struct WideMem {
  float wbuf[kWWarps][kTile];         // per-warp staging for the processors
  uint64_t wmass[kWWarps][256];       // per-warp histograms
  unsigned wcnt[kWWarps][256];
  uint64_t mass[256];
  unsigned cnt[256];
  unsigned long long red64[kWWarps];
  int red32[kWWarps];
  float redf[kWWarps];
  int sel[4];
  uint64_t sel64[4];
};

// One pass over the row: calls f(x, id) for every finite processed value.
template <typename T, typename F>
__device__ __forceinline__ void wide_pass(const SampleArgs& a, const pm_row_params& p, int64_t row, WideMem* wm,
                                          F&& f) {
  constexpr int VW = Lay<T>::VW;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int t = wid; t < a.n_tiles; t += kWWarps) {
    TileIn ti;
    load_tile<T>(a, row, t, ti);
    process_tile<VW>(a, p, row, t, ti, wm->wbuf[wid]);
    const int n_valid = tile_valid(a, t);
#pragma unroll
    for (int s = 0; s < 32; ++s) {
      const int e = slot_elem<VW>(s, lane);
      if (e < n_valid && ti.v[s] > -INFINITY) f(ti.v[s], (uint32_t)(t * kTile + e));
    }
  }
}

__device__ __forceinline__ void wide_clear(WideMem* wm) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int i = lane; i < 256; i += 32) { wm->wmass[wid][i] = 0; wm->wcnt[wid][i] = 0; }
  __syncwarp();
}

// Sum of the per-warp histograms into mass / cnt (all threads).
__device__ __forceinline__ void wide_merge(WideMem* wm) {
  __syncthreads();
  const int d = threadIdx.x;
  uint64_t m = 0;
  unsigned c = 0;
#pragma unroll
  for (int w = 0; w < kWWarps; ++w) { m += wm->wmass[w][d]; c += wm->wcnt[w][d]; }
  wm->mass[d] = m;
  wm->cnt[d] = c;
  __syncthreads();
}

// Lowest non-empty digit d whose keys above (above + mass of higher digits)
// weigh less than G; returns d, and the mass / count of the higher digits.
__device__ __forceinline__ int warp_find_mass_digit(const uint64_t* mass, const unsigned* cnt, uint64_t above,
                                                    uint64_t G, uint64_t* m_hi, unsigned* c_hi) {
  const int lane = threadIdx.x & 31;
  uint64_t ms[8];
  unsigned cs[8];
  uint64_t lm = 0;
  unsigned lc = 0;
#pragma unroll
  for (int b = 0; b < 8; ++b) { ms[b] = mass[lane * 8 + b]; cs[b] = cnt[lane * 8 + b]; lm += ms[b]; lc += cs[b]; }
  uint64_t sm = lm;   // suffix-inclusive over lanes >= lane
  unsigned sc = lc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t tm = __shfl_down_sync(kFull, sm, o);
    const unsigned tc = __shfl_down_sync(kFull, sc, o);
    if (lane + o < 32) { sm += tm; sc += tc; }
  }
  uint64_t hm = sm - lm;   // mass of digits above this lane's block
  unsigned hc = sc - lc;
  int found = 256;
  uint64_t fm = 0;
  unsigned fc = 0;
#pragma unroll
  for (int b = 7; b >= 0; --b) {
    if (cs[b] > 0 && above + hm < G) { found = lane * 8 + b; fm = hm; fc = hc; }
    hm += ms[b];
    hc += cs[b];
  }
  int best = found;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(kFull, best, o));
  const int src = best < 256 ? best / 8 : 0;
  *m_hi = __shfl_sync(kFull, fm, src);
  *c_hi = __shfl_sync(kFull, fc, src);
  return best;
}

template <typename T>
__global__ void __launch_bounds__(kWThreads) k_row_wide(const __grid_constant__ SampleArgs a) {
  extern __shared__ __align__(16) unsigned char smem_wide[];
  WideMem* wm = reinterpret_cast<WideMem*>(smem_wide);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    if (!(ld_cg(&a.status[row]) & 1)) continue;  // uniform across the CTA
    const pm_row_params p = row_params(a, row);
    float c, m;
    if (wid == 0) {
      c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &m);
      if (lane == 0) { wm->redf[0] = c; wm->redf[1] = m; }
    }
    __syncthreads();
    c = wm->redf[0];
    m = wm->redf[1];
    __syncthreads();
    // finite count and the min-p count (log-prob at or above the threshold)
    const bool minp = p.flags & PM_F_MIN_P;
    const float thr = fadd(fsub(m, c), p.log_min_p);
    int nf = 0, nm = 0;
    wide_pass<T>(a, p, row, wm, [&](float x, uint32_t) {
      ++nf;
      if (minp && !(fsub(x, c) < thr)) ++nm;
    });
    for (int o = 16; o > 0; o >>= 1) { nf += __shfl_xor_sync(kFull, nf, o); nm += __shfl_xor_sync(kFull, nm, o); }
    if (lane == 0) wm->red32[wid] = nf;
    __syncthreads();
    int n_fin = 0;
#pragma unroll
    for (int w = 0; w < kWWarps; ++w) n_fin += wm->red32[w];
    __syncthreads();
    if (lane == 0) wm->red32[wid] = nm;
    __syncthreads();
    int n_min = 0;
#pragma unroll
    for (int w = 0; w < kWWarps; ++w) n_min += wm->red32[w];
    __syncthreads();
    // top-p: ranks kept = keys whose mass above is below G
    int n_keep = n_fin;
    uint64_t cut = 0;
    bool have_cut = false;
    const uint64_t G = (1ull << 52) - __float2ull_rz(fmul(p.top_p_comp, 0x1p52f));
    if ((p.flags & PM_F_TOP_P) && G == 0) {
      n_keep = 1;  // nothing weighs less than zero: the top rank alone
    } else if (p.flags & PM_F_TOP_P) {
      uint64_t prefix = 0, above = 0;
      unsigned above_c = 0;
      for (int shift = 56; shift >= 0; shift -= 8) {
        wide_clear(wm);
        const int hs = shift + 8;
        wide_pass<T>(a, p, row, wm, [&](float x, uint32_t id) {
          const uint64_t k = rankkey(x, id);
          if (hs < 64 && (k >> hs) != (prefix >> hs)) return;
          const int d = (int)((k >> shift) & 255);
          atomicAdd(reinterpret_cast<unsigned long long*>(&wm->wmass[wid][d]), (unsigned long long)q52(fsub(x, c)));
          atomicAdd(&wm->wcnt[wid][d], 1u);
        });
        wide_merge(wm);
        if (wid == 0) {
          uint64_t mh;
          unsigned ch;
          const int d = warp_find_mass_digit(wm->mass, wm->cnt, above, G, &mh, &ch);
          if (lane == 0) { wm->sel[0] = d; wm->sel64[0] = mh; wm->sel[1] = (int)ch; }
        }
        __syncthreads();
        const int d = wm->sel[0];
        above += wm->sel64[0];
        above_c += (unsigned)wm->sel[1];
        prefix |= (uint64_t)(d & 255) << shift;
        __syncthreads();
      }
      n_keep = (int)above_c + 1;
      cut = prefix;
      have_cut = true;
    }
    // min-p on the top-p survivors (first min_tokens_to_keep ranks kept)
    int n = n_keep;
    if (minp) {
      const int first_drop = n_min > p.min_tokens_to_keep ? n_min : p.min_tokens_to_keep;
      if (first_drop < n) n = first_drop;
    }
    if (n < 1) n = 1;
    if (n != n_keep || !have_cut) {
      // the n-th largest key by counts
      uint64_t prefix = 0;
      int need = n;
      for (int shift = 56; shift >= 0; shift -= 8) {
        wide_clear(wm);
        const int hs = shift + 8;
        wide_pass<T>(a, p, row, wm, [&](float x, uint32_t id) {
          const uint64_t k = rankkey(x, id);
          if (hs < 64 && (k >> hs) != (prefix >> hs)) return;
          atomicAdd(&wm->wcnt[wid][(k >> shift) & 255], 1u);
        });
        wide_merge(wm);
        if (wid == 0) {
          int ab, ib;
          const int d = warp_find_digit(wm->cnt, need, &ab, &ib);
          if (lane == 0) { wm->sel[0] = d; wm->sel[1] = ab; }
        }
        __syncthreads();
        need -= wm->sel[1];
        prefix |= (uint64_t)(wm->sel[0] & 255) << shift;
        __syncthreads();
      }
      cut = prefix;
    }
    // Gumbel-max over the keys at or above the cut, ties to the lowest id
    float bs = -INFINITY;
    int bid = -1;
    float bx = -INFINITY;
    wide_pass<T>(a, p, row, wm, [&](float x, uint32_t id) {
      if (rankkey(x, id) < cut) return;
      const float sc = fadd(fmul(x, p.inv_temperature), row_gumbel(a, row, id));
      if (bid < 0 || sc > bs || (sc == bs && (int)id < bid)) { bs = sc; bid = (int)id; bx = x; }
    });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float os = __shfl_xor_sync(kFull, bs, o);
      const int oid = __shfl_xor_sync(kFull, bid, o);
      const float ox = __shfl_xor_sync(kFull, bx, o);
      if (oid >= 0 && (bid < 0 || os > bs || (os == bs && oid < bid))) { bs = os; bid = oid; bx = ox; }
    }
    if (lane == 0) { wm->redf[wid] = bs; wm->red32[wid] = bid; wm->red64[wid] = __float_as_uint(bx); }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kWWarps; ++w) {
        const float os = wm->redf[w];
        const int oid = wm->red32[w];
        if (oid >= 0 && (bid < 0 || os > bs || (os == bs && oid < bid))) {
          bs = os;
          bid = oid;
          bx = __uint_as_float((uint32_t)wm->red64[w]);
        }
      }
      const int32_t prev = a.status[row] & ~1;
      a.status[row] = prev | (a.surv_ids ? 8 : 0);
      a.tokens[row] = bid;
      if (a.tok_logprob) a.tok_logprob[row] = fsub(bx, c);
      if (a.n_surv) a.n_surv[row] = n;
    }
    __syncthreads();
  }
}

}  // namespace pm
