// pm_warp.cuh -- warp-level pieces of the streaming kernels: the candidate
// buffer behind a running threshold, the exact row log-sum-exp from tile
// statistics, the filters and the draws.  Each function is called by one
// full warp and uses only that warp's shared memory.
#pragma once

#include "pm_device.cuh"
#include "pm_select.cuh"
#include "pm_tile.cuh"

namespace pm {

// Candidate buffer state of one warp (identical in every lane).
struct Cand {
  int cnt;
  uint64_t tau;   // smallest key kept by the last compaction (0: none yet)
  float tau_x;    // its value, for the cheap pre-test
  bool trimmed;   // a compaction dropped keys
  uint64_t ctau;  // the last compaction's threshold (keys it dropped lie below)
};

// The threshold an empty merge buffer starts from so that it accepts every
// key at or above the row's shared bound rt.  A published bound is either a
// part's own K-th key (a real key, which that part's list holds, so the
// buffer must admit it: start one below) or a synthetic value threshold with
// zero low bits (a min-p floor, the first-tile estimate), which no real key
// equals.
__device__ __forceinline__ uint64_t merge_floor(uint64_t rt) { return (rt & 0xFFFFFFFFull) ? rt - 1 : rt; }

__device__ __forceinline__ void cand_reset(Cand& c) {
  c.cnt = 0;
  c.tau = 0;
  c.tau_x = -INFINITY;
  c.trimmed = false;
  c.ctau = 0;
}

// Keep the K largest of buf[0..cnt) (cnt > K); returns the smallest kept key.
// Out of line and by value, so the caller's buffer state stays in registers.
template <int CAP>
__device__ __noinline__ uint64_t compact_keys(uint64_t* buf, unsigned* hist, int cnt, int K) {
  return warp_select_topk<(CAP + 31) / 32>(buf, cnt, K, hist);
}

template <int CAP>
__device__ __forceinline__ void cand_compact(uint64_t* buf, unsigned* hist, Cand& c, int K) {
  c.tau = compact_keys<CAP>(buf, hist, c.cnt, K);
  c.tau_x = key_value(c.tau);
  c.cnt = K;
  c.trimmed = true;
  c.ctau = c.tau;
}

// Offer VW consecutive values per lane (tokens tok0 .. tok0+VW-1; lmax their
// maximum) to the buffer.  One vote per group in the common case; a group
// that passes writes its keys by one ballot per value position (no scan).
template <int VW, int CAP>
__device__ __forceinline__ bool cand_offer_vec(const float (&x)[VW], float lmax, uint32_t tok0, uint64_t* buf,
                                               unsigned* hist, Cand& c, int K) {
  const int lane = threadIdx.x & 31;
  if (!__any_sync(kFull, lmax > -INFINITY && lmax >= c.tau_x)) return false;
  // room for the 32 * VW keys this call may append: another offer routine
  // (one value per lane, or a narrower vector) can have left the buffer
  // fuller than this routine's own compaction bound
  bool compacted = false;
  if (c.cnt > CAP - 32 * VW) {
    cand_compact<CAP>(buf, hist, c, K);
    compacted = true;
  }
  const unsigned below = (1u << lane) - 1u;
  int base = c.cnt;
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    const uint64_t key = rankkey(x[i], tok0 + i);
    const bool ok = x[i] > -INFINITY && x[i] >= c.tau_x && key > c.tau;
    const unsigned bal = __ballot_sync(kFull, ok);
    if (ok) buf[base + __popc(bal & below)] = key;
    base += __popc(bal);
  }
  c.cnt = base;
  __syncwarp();
  // compactions come every 128 keys past K: a part's threshold then tracks
  // its running K-th key closely enough that few later values pass it
  if (c.cnt > min(CAP - 32 * VW, K + 128)) {
    cand_compact<CAP>(buf, hist, c, K);
    return true;
  }
  return compacted;
}

// Offer one value per lane (token tok) to the buffer: appended when its key
// beats the threshold.  The common case costs one compare and one vote.
template <int CAP>
__device__ __forceinline__ bool cand_offer_one(float x, uint32_t tok, uint64_t* buf, unsigned* hist, Cand& c,
                                               int K) {
  const int lane = threadIdx.x & 31;
  const bool pre = x > -INFINITY && x >= c.tau_x;
  if (!__any_sync(kFull, pre)) return false;
  const uint64_t key = rankkey(x, tok);
  const bool ok = pre && key > c.tau;
  const unsigned bal = __ballot_sync(kFull, ok);
  if (ok) buf[c.cnt + __popc(bal & ((1u << lane) - 1u))] = key;
  c.cnt += __popc(bal);
  __syncwarp();
  if (c.cnt > CAP - 32) {
    cand_compact<CAP>(buf, hist, c, K);
    return true;
  }
  return false;
}

// Offer one key per lane (0 = nothing).
template <int CAP>
__device__ __forceinline__ void cand_offer_key(uint64_t key, uint64_t* buf, unsigned* hist, Cand& c, int K) {
  const int lane = threadIdx.x & 31;
  const bool ok = key != 0ull && key > c.tau;
  const unsigned bal = __ballot_sync(kFull, ok);
  if (!bal) return;
  if (ok) buf[c.cnt + __popc(bal & ((1u << lane) - 1u))] = key;
  c.cnt += __popc(bal);
  __syncwarp();
  if (c.cnt > CAP - 32) cand_compact<CAP>(buf, hist, c, K);
}

// Bitonic sort of S[0..m) descending by one warp (P = power of two >= m, <= cap).
__device__ __forceinline__ void warp_sort_desc(uint64_t* S, int m) {
  const int lane = threadIdx.x & 31;
  int P = 1;
  while (P < m) P <<= 1;
  for (int i = m + lane; i < P; i += 32) S[i] = 0ull;
  __syncwarp();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < P; i += 32) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = S[i], y = S[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) { S[i] = y; S[ixj] = x; }
        }
      }
      __syncwarp();
    }
  }
}

// Bitonic sort of 32 E keys held in registers, descending: element i is
// k[i / 32] of lane i % 32.  Partners less than 32 apart are exchanged by
// shuffles, the others inside the lane.
template <int E>
__device__ __forceinline__ void warp_sort_regs_desc(uint64_t (&k)[E]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 2; kk <= 32 * E; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      uint64_t y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) y[e] = j < 32 ? __shfl_xor_sync(kFull, k[e], j) : k[e ^ (j >> 5)];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = e * 32 + lane;
        const bool want_max = ((i & j) == 0) == ((i & kk) == 0);
        k[e] = want_max ? (k[e] > y[e] ? k[e] : y[e]) : (k[e] < y[e] ? k[e] : y[e]);
      }
    }
  }
}

// The K largest of buf[0..n) (n <= 128, K <= n) sorted descending into
// buf[0..K), through registers.
__device__ __forceinline__ void warp_top_sorted_128(uint64_t* buf, int n, int K) {
  const int lane = threadIdx.x & 31;
  uint64_t k[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) k[e] = e * 32 + lane < n ? buf[e * 32 + lane] : 0ull;
  __syncwarp();
  warp_sort_regs_desc<4>(k);
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (e * 32 + lane < K) buf[e * 32 + lane] = k[e];
  __syncwarp();
}

// a_t = s_t e^(m_t - m) of tile t (0 for an empty tile).
__device__ __forceinline__ double tile_weight(const TileStat* st, int t, float m) {
  const uint64_t s = ld_cg(&st[t].s);
  if (!s) return 0.0;
  return dmul((double)s, det_exp64(dsub((double)ld_cg(&st[t].m), (double)m)));
}

// A lane's share of a row's tile statistics, loaded with all loads in flight
// at once: lane L holds tiles [L*per, L*per + per) of the row padded to
// P = 32 * per tiles (per = 1..kMaxPer; rows of up to 32 * kMaxPer tiles).
constexpr int kMaxPer = 8;  // rows of up to 256 tiles (262,144 tokens)

struct LaneTiles {
  int per;            // tiles per lane (a power of two)
  int nt;
  float m[kMaxPer];
  uint64_t s[kMaxPer];
};

__device__ __forceinline__ void load_lane_tiles(const TileStat* st, int nt, LaneTiles& lt) {
  const int lane = threadIdx.x & 31;
  int P = 32;
  while (P < nt) P <<= 1;
  lt.per = P >> 5;
  lt.nt = nt;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int t = lane * lt.per + i;
    const bool ok = i < lt.per && t < nt;
    lt.m[i] = ok ? ld_cg(&st[t].m) : -INFINITY;
    lt.s[i] = ok ? ld_cg(&st[t].s) : 0ull;
  }
}

__device__ __forceinline__ float lane_tiles_max(const LaneTiles& lt) {
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) m = fmaxf(m, lt.m[i]);
  return warp_max(m);
}

__device__ __forceinline__ double tile_weight_of(float mt, uint64_t s, float m) {
  if (!s) return 0.0;
  return dmul((double)s, det_exp64(dsub((double)mt, (double)m)));
}

// Row log-sum-exp from its tile statistics, one warp:
//   m = max_t m_t,  Z = pairwise sum over t of s_t e^(m_t - m)  (tiles padded
//   with zeros to a power of two; lane L sums its contiguous block of P/32
//   tiles as a complete subtree, then the lanes combine pairwise),
//   c = fl32(m + log(Z 2^-52)).  -inf when no tile has a finite value.
// kFullPer: lt.per is kMaxPer (no branch on it).
template <bool kFullPer = false>
__device__ __forceinline__ float combine_lane_tiles(const LaneTiles& lt, float m) {
  const int lane = threadIdx.x & 31;
  if (!(m > -INFINITY)) return -INFINITY;
  double stk[6];
  int sp = 0;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    if (kFullPer || i < lt.per) {
      double v = tile_weight_of(lt.m[i], lt.s[i], m);
      for (int c = i + 1; (c & 1) == 0; c >>= 1) v = dadd(stk[--sp], v);
      stk[sp++] = v;
    }
  }
  double acc = stk[0];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_down_sync(kFull, acc, o);
    if ((lane & (2 * o - 1)) == 0) acc = dadd(acc, t);
  }
  const double Z = __shfl_sync(kFull, acc, 0);
  return (float)dadd((double)m, det_log64(dmul(Z, 0x1p-52)));
}

// Every lane takes kMaxPer tiles: the zero-padded 256-leaf pairwise tree
// sums to the same bits as the tree over the row's own power of two (its
// right part is exactly zero), with no branch on the tile count.
__device__ __forceinline__ float warp_combine(const TileStat* st, int nt, float* m_out) {
  const int lane = threadIdx.x & 31;
  LaneTiles lt;
  lt.per = kMaxPer;
  lt.nt = nt;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int t = lane * kMaxPer + i;
    lt.m[i] = t < nt ? ld_cg(&st[t].m) : -INFINITY;
    lt.s[i] = t < nt ? ld_cg(&st[t].s) : 0ull;
  }
  const float m = lane_tiles_max(lt);
  *m_out = m;
  return combine_lane_tiles<true>(lt, m);
}

// Bracket [*c_lo, *c_hi] around the fp32 log-sum-exp that warp_combine
// returns from the row's exact statistics, computed from its parts'
// approximate statistics (ApproxStat, with their relative error bounds eps_p):
//   Z = sum_p s_p 2^(fl(mref_p L) - ML),  lse = ML ln2 + ln Z,
//   |ln(true sum) - lse| <= 1.0001 sum_p w_p eps_p / Z;
// the exact statistics differ from the true log-sum-exp by at most 1.3e-6
// before their final fp32 rounding (rounding of x - m_t, 14.02 2^-24 by the
// bound sum e^d |d| <= 14.02 sum e^d over a tile; two ulps of the fp32
// exponential; the floors).  The bracket is rounded outward and widened by
// one more ulp each side.  Returns false when a part's sum is not finite
// (the row takes the exact pass).
__device__ __forceinline__ bool warp_bracket(const SampleArgs& a, int64_t row, int n_parts, float* c_lo,
                                             float* c_hi) {
  const int lane = threadIdx.x & 31;
  const int64_t T = a.rows * a.n_tiles, base = row * a.n_tiles;
  const int64_t w0 = owner_warp(base, T, a.n_warps);
  const ApproxStat* st = reinterpret_cast<const ApproxStat*>(a.staty) + base;
  float ml = -INFINITY;
  bool bad = false;
  for (int p0 = 0; p0 < n_parts; p0 += 32) {
    const int p = p0 + lane;
    if (p < n_parts) {
      const int64_t g0 = (w0 + p) * T / a.n_warps;
      const int t0 = (int)(g0 > base ? g0 - base : 0);
      const float mr = ld_cg(&st[t0].mref);
      const double sv = ld_cg(&st[t0].s);
      bad |= !(sv == sv) || !(sv < 1e300) || !(mr == mr) || mr == INFINITY;
      if (mr > -INFINITY) ml = fmaxf(ml, fmul(mr, kLog2eF));
    }
  }
  ml = warp_max(ml);
  if (__any_sync(kFull, bad)) return false;
  if (ml == -INFINITY) {  // no finite value: the exact statistics give -inf
    *c_lo = *c_hi = -INFINITY;
    return true;
  }
  double z = 0.0, e = 0.0;
  for (int p0 = 0; p0 < n_parts; p0 += 32) {
    const int p = p0 + lane;
    if (p < n_parts) {
      const int64_t g0 = (w0 + p) * T / a.n_warps;
      const int t0 = (int)(g0 > base ? g0 - base : 0);
      const float mr = ld_cg(&st[t0].mref);
      if (mr > -INFINITY) {
        const double d = dsub((double)fmul(mr, kLog2eF), (double)ml);
        const double w = dmul(ld_cg(&st[t0].s), det_exp64(dmul(d, 0x1.62e42fefa39efp-1)));
        z = dadd(z, w);
        e = dfma(w, (double)ld_cg(&st[t0].eps), e);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    z = dadd(z, __shfl_xor_sync(kFull, z, o));
    e = dadd(e, __shfl_xor_sync(kFull, e, o));
  }
  if (!(z > 0.0) || !(z < 1e300)) return false;
  const double lse = dadd(dmul((double)ml, 0x1.62e42fefa39efp-1), det_log64(z));
  const double half = 1.0001 * (e / z) + 1.3e-6 + 1e-12 * fabs(lse);
  *c_lo = nextafterf(__double2float_rd(lse - half), -INFINITY);
  *c_hi = nextafterf(__double2float_ru(lse + half), INFINITY);
  return true;
}

__device__ __forceinline__ float row_gumbel(const SampleArgs& a, int64_t row, uint32_t token) {
  if (a.noise_mode == PM_NOISE_INJECTED) return a.gumbel[row * a.gumbel_stride + token];
  return philox_gumbel(a.seed, a.offset, a.row_base + (uint32_t)row, token);
}

__device__ __forceinline__ uint64_t row_u53(const SampleArgs& a, int64_t row, int stream) {
  if (a.noise_mode == PM_NOISE_INJECTED) return u53_from_double(a.uniform[row * 2 + stream]);
  return philox_u53(a.seed, a.offset, a.row_base + (uint32_t)row, (uint32_t)stream);
}

// The sampler's filters over the row's sorted top candidates S[0..m) and the
// Gumbel-max draw (mlx-lm make_sampler chain: top_k, top_p, min_p, then the
// categorical at temperature).
//   top_p: keep rank r while T - A_r > Q(1 - top_p), A_r the exclusive prefix
//          of q52(x - c) in rank order, T their sum when top_k is on, else 2^52;
//   min_p: drop ranks >= min_tokens_to_keep with fl32(x - c) <
//          fl32(fl32(x_0 - c) + log(min_p));
//   draw:  argmax over survivors of fl32(fl32(x * inv_temp) + g), ties to the
//          lowest id.
// Returns the token, or -1 when the survivors reach past the candidates (the
// row is then flagged; only possible when top_k is off).  *n_out = survivors;
// *x_out (when given) = the token's value, S's value at its rank.
// With c_hi given (not NaN), [c, c_hi] brackets the exact log-sum-exp (top-k
// rows, see warp_bracket): the cut is the one every value in the bracket
// gives, or the call returns -2 when the bracket does not decide it.
__device__ inline int warp_filter_draw(const SampleArgs& a, const pm_row_params& p, int64_t row, const uint64_t* S,
                                int m, bool complete, float c, int* n_out, const float* scores = nullptr,
                                float* x_out = nullptr, float c_hi = __builtin_nanf("")) {
  const int lane = threadIdx.x & 31;
  *n_out = 0;
  if (x_out) *x_out = -INFINITY;
  if (m == 0) return 0;
  const bool topk = p.top_k > 0;
  int cnt = (topk && p.top_k < m) ? p.top_k : m;
  bool determined = topk || complete;
  if ((p.flags & PM_F_TOP_P) && topk && c_hi == c_hi && c_hi != c) {
    // Tails T - A_r at c_hi bound the exact ones from below, at c from above
    // (the fp32 exponential is monotone up to two ulps, and each q52 floors:
    // margins of 2^-18 relative and 2 cnt + 2 absolute).  Rank r is kept
    // for sure when the lower bound clears the threshold, dropped for sure
    // when the upper one does not; the exact cut is then the first rank not
    // kept for sure, provided that rank is dropped for sure.
    const uint64_t qthr = __float2ull_rz(fmul(p.top_p_comp, 0x1p52f));
    const uint64_t slack = 2ull * (uint64_t)cnt + 2ull;
    uint64_t Th = 0, Tl = 0;
    for (int r = lane; r < cnt; r += 32) {
      const float x = key_value(S[r]);
      Th += q52(fsub(x, c_hi));
      Tl += q52(fsub(x, c));
    }
    Th = warp_sum_u64(Th);
    Tl = warp_sum_u64(Tl);
    uint64_t ch = 0, cl = 0;
    int k_keep = cnt, k_drop = cnt;
    bool f_keep = false, f_drop = false;
    for (int base = 0; base < cnt && !(f_keep && f_drop); base += 32) {
      const int r = base + lane;
      const float x = r < cnt ? key_value(S[r]) : 0.0f;
      const uint64_t qh = r < cnt ? q52(fsub(x, c_hi)) : 0ull;
      const uint64_t ql = r < cnt ? q52(fsub(x, c)) : 0ull;
      const uint64_t ih = warp_incl_scan_u64(qh), il = warp_incl_scan_u64(ql);
      const uint64_t tail_h = Th - (ch + ih - qh), tail_l = Tl - (cl + il - ql);
      uint64_t lower = tail_h - (tail_h >> 18);
      lower = lower > slack ? lower - slack : 0ull;
      const uint64_t upper = tail_l + (tail_l >> 18) + slack;
      const unsigned nk = __ballot_sync(kFull, r < cnt && !(lower > qthr));
      const unsigned nd = __ballot_sync(kFull, r < cnt && upper <= qthr);
      if (!f_keep && nk) { k_keep = base + __ffs(nk) - 1; f_keep = true; }
      if (!f_drop && nd) { k_drop = base + __ffs(nd) - 1; f_drop = true; }
      ch += __shfl_sync(kFull, ih, 31);
      cl += __shfl_sync(kFull, il, 31);
    }
    if (k_keep != k_drop) return -2;
    cnt = k_keep < 1 ? 1 : k_keep;
  } else if (p.flags & PM_F_TOP_P) {
    // q52 of the first 64 ranks once, kept for the cut search below
    const uint64_t qa = lane < cnt ? q52(fsub(key_value(S[lane]), c)) : 0ull;
    const uint64_t qb = lane + 32 < cnt ? q52(fsub(key_value(S[lane + 32]), c)) : 0ull;
    uint64_t T = qa + qb;
    for (int r = lane + 64; r < cnt; r += 32) T += q52(fsub(key_value(S[r]), c));
    T = warp_sum_u64(T);
    if (!topk) T = 1ull << 52;
    const uint64_t qthr = __float2ull_rz(fmul(p.top_p_comp, 0x1p52f));
    uint64_t carry = 0;
    int keep = cnt;
    bool found = false;
    for (int base = 0; base < cnt && !found; base += 32) {
      const int r = base + lane;
      const uint64_t q = base == 0 ? qa : base == 32 ? qb : r < cnt ? q52(fsub(key_value(S[r]), c)) : 0ull;
      const uint64_t incl = warp_incl_scan_u64(q);
      const uint64_t A = carry + incl - q;
      const bool ok = r < cnt && A < T && (T - A) > qthr;
      const unsigned fail = __ballot_sync(kFull, r < cnt && !ok);
      if (fail) { keep = base + __ffs(fail) - 1; found = true; }
      carry += __shfl_sync(kFull, incl, 31);
    }
    if (found) determined = true;
    cnt = keep < 1 ? 1 : keep;
  }
  if (p.flags & PM_F_MIN_P) {
    const float thr = fadd(fsub(key_value(S[0]), c), p.log_min_p);
    int keep = cnt;
    bool found = false;
    for (int base = 0; base < cnt && !found; base += 32) {
      const int r = base + lane;
      const bool drop = r < cnt && r >= p.min_tokens_to_keep && fsub(key_value(S[r]), c) < thr;
      const unsigned bal = __ballot_sync(kFull, drop);
      if (bal) { keep = base + __ffs(bal) - 1; found = true; }
    }
    if (found) determined = true;
    cnt = keep < 1 ? 1 : keep;
  }
  if (!determined) return -1;
  float bs = -INFINITY;
  int bid = -1, brank = -1;
  for (int r = lane; r < cnt; r += 32) {
    const uint32_t id = key_index(S[r]);
    const float sc = scores ? scores[r] : fadd(fmul(key_value(S[r]), p.inv_temperature), row_gumbel(a, row, id));
    if (bid < 0 || sc > bs || (sc == bs && (int)id < bid)) { bs = sc; bid = (int)id; brank = r; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float os = __shfl_xor_sync(kFull, bs, o);
    const int oid = __shfl_xor_sync(kFull, bid, o);
    const int ork = __shfl_xor_sync(kFull, brank, o);
    if (oid >= 0 && (bid < 0 || os > bs || (os == bs && oid < bid))) { bs = os; bid = oid; brank = ork; }
  }
  *n_out = cnt;
  if (x_out && brank >= 0) *x_out = key_value(S[brank]);
  return bid;
}

// Renormalised survivor probabilities at temperature (fp64, rank order,
// sequential sum) into the row's output slots.  Lane 0.
__device__ inline __noinline__ void write_survivors(const SampleArgs& a, const pm_row_params& p, int64_t row,
                                                const uint64_t* S, int cnt) {
  double ymax = -INFINITY;
  for (int r = 0; r < cnt; ++r) {
    const double yv = (double)fmul(key_value(S[r]), p.inv_temperature);
    ymax = yv > ymax ? yv : ymax;
  }
  double Z = 0.0;
  for (int r = 0; r < cnt; ++r) Z = dadd(Z, det_exp64(dsub((double)fmul(key_value(S[r]), p.inv_temperature), ymax)));
  int32_t* ids = a.surv_ids + row * a.surv_cap;
  float* prs = a.surv_probs + row * a.surv_cap;
  for (int r = 0; r < a.surv_cap; ++r) {
    if (r < cnt) {
      ids[r] = (int32_t)key_index(S[r]);
      prs[r] = (float)__ddiv_rn(det_exp64(dsub((double)fmul(key_value(S[r]), p.inv_temperature), ymax)), Z);
    } else {
      ids[r] = -1;
      prs[r] = 0.0f;
    }
  }
  a.n_surv[row] = cnt;
}

// Whole-vocabulary draw at temperature from the y-statistics (no filter on):
// tile weights w_t = floor(a_t 2^-sh), sh = ceil(log2 n_tiles) + 1; tile by
// the first uniform (first tile whose inclusive prefix of w exceeds
// floor(u1 W)), token inside it by the second (first whose inclusive prefix
// of q52(y - m_t) exceeds floor(u2 s_t)).  The warp re-reads that one tile.
// Processors on a tile held in registers without a staging buffer: each
// override is applied by the lane that owns its slot (rare path).
template <int VW>
__device__ __forceinline__ void process_tile_regs(const SampleArgs& a, const pm_row_params& p, int64_t row,
                                                  int tile, TileIn& ti) {
  const int lane = threadIdx.x & 31;
  const int64_t start = (int64_t)tile * kTile;
  for (int i = ti.bb; i < ti.be; ++i) {
    const int64_t e64 = a.bias_tok[i] - start;
    if (e64 < 0 || e64 >= kTile) continue;  // ids out of ascending order: skipped
    const int e = (int)e64;
    if ((e % (32 * VW)) / VW != lane) continue;
    const int sl = (e / (32 * VW)) * VW + e % VW;
    const float b = a.bias_val[i];
#pragma unroll
    for (int q = 0; q < 32; ++q)
      if (q == sl) ti.v[q] = fadd(ti.v[q], b);
  }
  const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
  const uint32_t* oinf = a.ovr_info + row * (int64_t)a.ovr_cap;
  for (int i = ti.ob; i < ti.oe; ++i) {
    const int e = (int)(otok[i] - start);
    if ((e % (32 * VW)) / VW != lane) continue;
    const int sl = (e / (32 * VW)) * VW + e % VW;
    const uint32_t info = oinf[i];
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      if (q != sl) continue;
      float x = ti.v[q];
      if (info & 1u) x = x < 0.0f ? fmul(x, p.repetition_penalty) : __fdiv_rn(x, p.repetition_penalty);
      if (info & 2u) x = fsub(x, p.presence_penalty);
      const uint32_t cnt = info >> 8;
      if (cnt) x = fsub(x, fmul(p.frequency_penalty, (float)cnt));
      ti.v[q] = x;
    }
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

// The tile of a whole-vocabulary draw: the first whose inclusive prefix of
// integer tile weights (over the row's y statistics) exceeds the row's first
// 53-bit uniform scaled to their sum, by one warp.  Returns the tile (-1: no
// finite value in the row) and, in every lane, the tile's maximum and the
// target of the token search inside it.
__device__ __forceinline__ int warp_full_pick(const SampleArgs& a, int64_t row, float* mt_out, uint64_t* t2_out) {
  const int lane = threadIdx.x & 31;
  const int nt = a.n_tiles;
  const TileStat* st = a.staty + row * (int64_t)nt;
  LaneTiles lt;
  load_lane_tiles(st, nt, lt);
  const float my = lane_tiles_max(lt);
  if (!(my > -INFINITY)) return -1;
  int sh = 1;
  while ((1 << (sh - 1)) < nt) ++sh;
  const double scale = __longlong_as_double((long long)(1023 - sh) << 52);  // 2^-sh
  // tile weights of this lane's contiguous block, their sum, and the warp's
  // exclusive prefix (lanes hold consecutive blocks, so block order = tile order)
  uint64_t w[kMaxPer];
  uint64_t lsum = 0;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    w[i] = i < lt.per ? __double2ull_rz(dmul(tile_weight_of(lt.m[i], lt.s[i], my), scale)) : 0ull;
    lsum += w[i];
  }
  const uint64_t incl = warp_incl_scan_u64(lsum);
  const uint64_t W = __shfl_sync(kFull, incl, 31);
  const uint64_t t1 = scale_u53(row_u53(a, row, 0), W);
  const unsigned hit = __ballot_sync(kFull, incl > t1);
  const int src = hit ? __ffs(hit) - 1 : 31;
  int tt = nt - 1;
  if (lane == src) {
    uint64_t run = incl - lsum;
    int found = -1;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      run += w[i];
      if (found < 0 && i < lt.per && run > t1) found = i;
    }
    tt = lane * lt.per + (found < 0 ? 0 : found);
  }
  tt = __shfl_sync(kFull, tt, src);
  if (tt >= nt) tt = nt - 1;
  *mt_out = ld_cg(&st[tt].m);
  *t2_out = scale_u53(row_u53(a, row, 1), ld_cg(&st[tt].s));
  return tt;
}

template <typename T>
__device__ __noinline__ int warp_full_draw(const SampleArgs& a, const pm_row_params& p, int64_t row, float* x_out) {
  constexpr int VW = Lay<T>::VW;
  const int lane = threadIdx.x & 31;
  *x_out = -INFINITY;
  float mt;
  uint64_t t2;
  const int tt = warp_full_pick(a, row, &mt, &t2);
  if (tt < 0) return 0;
  const int64_t start = (int64_t)tt * kTile;
  TileIn ti;
  load_tile<T>(a, row, tt, ti);
  process_tile_regs<VW>(a, p, row, tt, ti);
  uint64_t acc = 0;
  int tok = (int)start;
  float tx = -INFINITY;
  for (int j = 0; j < 32 / VW; ++j) {
    uint64_t q[VW];
    uint64_t ls = 0;
#pragma unroll
    for (int c = 0; c < VW; ++c) {
      const float x = ti.v[j * VW + c];
      const float y = x > -INFINITY ? fmul(x, p.inv_temperature) : -INFINITY;
      q[c] = q52(fsub(y, mt));
      ls += q[c];
    }
    const uint64_t incl = acc + warp_incl_scan_u64(ls);
    const unsigned hit = __ballot_sync(kFull, incl > t2);
    if (hit) {
      const int src = __ffs(hit) - 1;
      int found = -1;
      float fx = -INFINITY;
      if (lane == src) {
        uint64_t run = incl - ls;
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          run += q[c];
          if (found < 0 && run > t2) { found = c; fx = ti.v[j * VW + c]; }
        }
      }
      found = __shfl_sync(kFull, found, src);
      tx = __shfl_sync(kFull, fx, src);
      tok = (int)(start + j * 32 * VW + src * VW + found);
      break;
    }
    acc = __shfl_sync(kFull, incl, 31);
  }
  *x_out = tx;
  return tok;
}

// A part list's trimmed bit as a merge reads it.  On min-p floor rows a list
// whose compactions cut only at or below the row's shared floor rt still
// holds every survivor: its last compaction threshold (kept in the part's
// best slot, unused by such rows) decides.
__device__ __forceinline__ bool part_trimmed(const SampleArgs& a, int64_t row, int part, int raw, bool minp,
                                             uint64_t rt) {
  if (!((raw >> 30) & 1)) return false;
  return !(minp && rt && ld_cg(&a.best[row * a.max_parts + part]) <= rt);
}

// A row whose top-p cut the bracket left open: its sorted top candidates go
// to the row's first part slot and the row into the exact pass's queue.
template <int KC>
__device__ __forceinline__ void queue_exact(const SampleArgs& a, int64_t row, const uint64_t* S, int n) {
  const int lane = threadIdx.x & 31;
  uint64_t* dst = a.cand + row * a.max_parts * (int64_t)KC;
  for (int i = lane; i < n; i += 32) dst[i] = S[i];
  if (lane == 0) {
    a.cand_n[row * a.max_parts] = n;
    const int q = atomicAdd(&a.exact_q[0], 1);
    a.exact_q[1 + a.rows + q] = (int32_t)row;
  }
  __syncwarp();
}

// Row merge by the warp that completed the row: gathers the parts' results
// and draws the token.  Returns the token (-1 when flagged); *x_tok the
// chosen token's processed logit, *lse the row log-sum-exp (NaN if unused).
template <typename T, int KC, int CAP>
__device__ __noinline__ int warp_row_merge(const SampleArgs& a, int64_t row, int n_parts, uint64_t* cbuf,
                                           unsigned* hist, float* x_tok, float* lse_out, int* n_surv_out) {
  const int lane = threadIdx.x & 31;
  const pm_row_params p = row_params(a, row);
  const int mode = row_mode(p);
  float c = __int_as_float(0x7fc00000), c_hi = __int_as_float(0x7fc00000);
  float mx;
  bool bracket_ok = true;
  if (needs_xstats(a, p, mode)) c = warp_combine(a.statx + row * a.n_tiles, a.n_tiles, &mx);
  else if (needs_astats(a, p, mode))
    bracket_ok = warp_bracket(a, row, n_parts, &c, &c_hi);
  *lse_out = c_hi == c_hi ? __int_as_float(0x7fc00000) : c;
  *n_surv_out = 0;
  int tok = 0;
  *x_tok = -INFINITY;
  if (mode == kGreedy) {
    uint64_t bk = 0;
    for (int i = lane; i < n_parts; i += 32) {
      const uint64_t k = ld_cg(&a.best[row * a.max_parts + i]);
      bk = k > bk ? k : bk;
    }
    bk = warp_max_u64(bk);
    tok = (int)key_index(bk);
    *x_tok = key_value(bk);
  } else if (mode == kCand) {
    const int K = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;
    Cand cd;
    cand_reset(cd);
    // the row's shared threshold: the largest bound the parts published
    const bool minp = minp_floor_row(p);
    const uint64_t rt = ld_cg(&a.row_tau[row]);
    if (rt) {
      cd.tau = merge_floor(rt);
      cd.tau_x = key_value(rt);
      cd.trimmed = !minp;
    }
    // Parts in groups of 32: the counts in one round of loads (lane i: part
    // p0+i), then the group's keys in flattened order, eight independent
    // loads per lane per round; a key's part is found by a binary search
    // over the lanes' inclusive prefix counts.
    bool trimmed_any = false;
    for (int p0 = 0; p0 < n_parts; p0 += 32) {
      const int part = p0 + lane;
      const int raw = part < n_parts ? ld_cg(&a.cand_n[row * a.max_parts + part]) : 0;
      const int n = raw & 0x3fffffff;
      trimmed_any |= __any_sync(kFull, part_trimmed(a, row, part, raw, minp, rt)) != 0;
      const int incl = warp_incl_scan(n);
      const int tot = __shfl_sync(kFull, incl, 31);
      for (int f0 = 0; f0 < tot; f0 += 256) {
        uint64_t keys[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int f = f0 + u * 32 + lane;
          int q = 0;  // number of group parts whose inclusive prefix is <= f
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
            const uint64_t* src = a.cand + (row * a.max_parts + p0 + qi) * (int64_t)KC;
            keys[u] = ld_cg(&src[f - (iq - nq)]);
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) cand_offer_key<CAP>(keys[u], cbuf, hist, cd, K);
      }
    }
    if (cd.cnt <= 128) {
      // few keys (the usual case behind the row threshold): sort them in
      // registers and keep the first K
      if (cd.cnt > K) cd.trimmed = true;
      warp_top_sorted_128(cbuf, cd.cnt, K < cd.cnt ? K : cd.cnt);
      cd.cnt = K < cd.cnt ? K : cd.cnt;
    } else {
      cand_compact<CAP>(cbuf, hist, cd, K);
      if (cd.cnt <= 128) warp_top_sorted_128(cbuf, cd.cnt, cd.cnt);
      else warp_sort_desc(cbuf, cd.cnt);
    }
    int ns = 0;
    tok = bracket_ok ? warp_filter_draw(a, p, row, cbuf, cd.cnt, !(trimmed_any || cd.trimmed), c, &ns, nullptr,
                                        x_tok, c_hi)
                     : -2;
    *n_surv_out = ns;
    if (tok == -2) {
      queue_exact<KC>(a, row, cbuf, cd.cnt);
    } else if (tok >= 0) {
      if (a.surv_ids && lane == 0) write_survivors(a, p, row, cbuf, ns);
    }
  } else {
    tok = warp_full_draw<T>(a, p, row, x_tok);
  }
  return tok;
}

// Row outputs (lane 0).
__device__ __forceinline__ void write_row(const SampleArgs& a, int64_t row, int mode, int tok, float x_tok,
                                          float lse, int ns) {
  const int32_t prevs = a.status_live ? ld_cg(&a.status[row]) : 0;
  a.status[row] = prevs | (tok == -2 ? 64 : tok < 0 ? 1 : 0);
  a.tokens[row] = tok;
  if (a.lse_out) a.lse_out[row] = lse;
  if (a.row_lse) a.row_lse[row] = lse;
  if (a.tok_logprob) a.tok_logprob[row] = tok >= 0 ? fsub(x_tok, lse) : __int_as_float(0x7fc00000);
  if (a.n_surv && (mode != kCand || !a.surv_ids)) a.n_surv[row] = mode == kCand ? ns : 0;
}

// The processed logit of one token of a row (bias, penalties, mask): the
// single-token form of process_tile, for the rare paths.
__device__ inline __noinline__ float processed_value(const SampleArgs& a, int dtype, const pm_row_params& p, int64_t row, int tok) {
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

}  // namespace pm
