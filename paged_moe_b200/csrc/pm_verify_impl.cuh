// pm_verify_impl.cuh -- draft acceptance of a verify pass (included at the
// end of pm_sample.cu: it reuses that file's kernels and host planning).
//
// The target rows of every request go through the same fused streaming and
// merge kernels as plain sampling (their processors see history + [y] +
// drafts[:i] through the feed), writing each row's sample (and, in residual
// mode, its survivors) to the workspace.  Then:
//   match mode    (reference lookup_decode.py:363-369, verify_decode.py:915-921)
//                 a warp per request keeps the drafts while they equal the
//                 rows' own samples and emits samples[:accepted + 1];
//   residual mode (speculative sampling, Leviathan et al. 2023; not in the
//                 reference) a warp per request accepts draft i when
//                 u_i q_i(d_i) < p_i(d_i) (fp64) and, at the first rejection,
//                 draws from max(fl32(p - q), 0) by the exact fixed-point
//                 inverse CDF in ascending token order: over the survivors
//                 when the sampler filters, one-hot when greedy, and over the
//                 whole vocabulary (a CTA re-streams the row pair) otherwise.
#pragma once

namespace pm {

// What the acceptance test of one draft position needs, computed for every
// position at once (k_accept_probs) before the sequential walk.
struct AccProb {
  float pd;       // target probability of the draft token
  float qd;       // draft probability of the draft token
  float cy;       // whole-vocabulary rows: the row's log-sum-exp of y = x / temp
  int32_t wide;   // filtered rows whose survivors outrun the candidate lists
};
static_assert(sizeof(AccProb) == 16, "read as one 16-byte load");

struct VerifyK {
  int32_t mode;
  const int32_t* drafts;   // [B, k]
  int32_t k;
  const void* dlogits;     // [B*k, dstride] raw draft logits
  int32_t ddtype;
  int64_t dstride;
  float* dlse;             // [B*k] log-sum-exp of the draft rows (written by k_accept_probs)
  const TileStat* dstat;   // [B*k, n_tiles] tile statistics of the draft rows
  const double* u_accept;  // [B, k] or null (Philox stream 2)
  const double* u_residual;  // [B] or null (Philox stream 3)
  int32_t* tokens;         // [B, k+1], -1 padded
  int32_t* n_acc;          // [B]
  int32_t* row_tokens;     // optional [B*(k+1)] every row's own sample
  const int32_t* rtok;     // [B*(k+1)] the rows' samples (workspace)
  const int32_t* sids;     // [B*(k+1), scap] survivors in rank order
  const float* sprobs;
  const int32_t* ns;       // [B*(k+1)]
  int32_t scap;
  int32_t* pending;        // [B] row awaiting a whole-vocabulary residual draw, -1 if none
  float* ylse;             // [B] that row's log-sum-exp of y = x / temp
  uint64_t* rsum;          // [B, n_tiles] residual mass of each tile of that row
  AccProb* probs;          // [B, k] residual mode: every position's acceptance inputs
};

__device__ __forceinline__ float draft_value(const VerifyK& v, int64_t drow, int64_t tok) {
  if (v.ddtype == PM_DTYPE_F32) return reinterpret_cast<const float*>(v.dlogits)[drow * v.dstride + tok];
  return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(v.dlogits)[drow * v.dstride + tok]);
}

// q(tok) = expf(fl32(d - lse_d)) of a draft row.
__device__ __forceinline__ float draft_prob(const VerifyK& v, int64_t drow, int64_t tok, float cd) {
  return det_expf(fsub(draft_value(v, drow, tok), cd));
}

// floor(max(fl32(p - q), 0) 2^52); the scaling by 2^52 is exact.
__device__ __forceinline__ uint64_t residual_q52(float p, float q) {
  const float r = fsub(p, q);
  return r > 0.0f ? __float2ull_rz(fmul(r, 0x1p52f)) : 0ull;
}

__device__ __forceinline__ double accept_uniform(const SampleArgs& a, const VerifyK& v, int64_t b, int i,
                                                 int64_t row) {
  if (v.u_accept) return v.u_accept[b * v.k + i];
  return dmul((double)philox_u53(a.seed, a.offset, a.row_base + (uint32_t)row, 2), 0x1p-53);
}

__device__ __forceinline__ uint64_t residual_u53(const SampleArgs& a, const VerifyK& v, int64_t b, int64_t row) {
  if (v.u_residual) return u53_from_double(v.u_residual[b]);
  return philox_u53(a.seed, a.offset, a.row_base + (uint32_t)row, 3);
}

// Residual draw over a filtered row's survivors, ascending token order.
// Returns -1 when no survivor has a positive residual.
template <int KC>
__device__ int survivor_residual(const SampleArgs& a, const VerifyK& v, int64_t b, int64_t row, int64_t drow,
                                 float cd, uint64_t* key, uint64_t* q) {
  const int lane = threadIdx.x & 31;
  const int n = min(ld_cg(&v.ns[row]), v.scap);
  uint64_t R = 0;
  for (int r = lane; r < n; r += 32) {
    const int id = ld_cg(&v.sids[row * v.scap + r]);
    const uint64_t qq = residual_q52(ld_cg(&v.sprobs[row * v.scap + r]), draft_prob(v, drow, id, cd));
    key[r] = ((uint64_t)(0xFFFFFFFFu - (uint32_t)id) << 32) | (uint32_t)r;  // descending key = ascending id
    q[r] = qq;
    R += qq;
  }
  R = warp_sum_u64(R);
  __syncwarp();
  if (R == 0) return -1;
  warp_sort_desc(key, n);
  const uint64_t tgt = scale_u53(residual_u53(a, v, b, row), R);
  uint64_t carry = 0;
  for (int r0 = 0; r0 < n; r0 += 32) {
    const int r = r0 + lane;
    const uint64_t kk = r < n ? key[r] : 0ull;
    const uint64_t qq = r < n ? q[(uint32_t)kk] : 0ull;
    const uint64_t incl = carry + warp_incl_scan_u64(qq);
    const unsigned hit = __ballot_sync(kFull, r < n && incl > tgt);
    if (hit) {
      const uint64_t kh = __shfl_sync(kFull, kk, __ffs(hit) - 1);
      __syncwarp();
      return (int)(0xFFFFFFFFu - (uint32_t)(kh >> 32));
    }
    carry = __shfl_sync(kFull, incl, 31);
  }
  __syncwarp();
  return -1;
}

__device__ __forceinline__ AccProb ld_cg_accprob(const AccProb* p) {
  const float4 f = __ldcg(reinterpret_cast<const float4*>(p));
  AccProb r;
  r.pd = f.x;
  r.qd = f.y;
  r.cy = f.z;
  r.wide = __float_as_int(f.w);
  return r;
}

// Residual mode, before the acceptance walk: one warp per draft position
// (request b, position i) folds the draft row's tile statistics into its
// log-sum-exp (stored for the walk and the residual draw), then computes
// p(d_i), q(d_i) and, for whole-vocabulary rows, the row's log-sum-exp of y,
// with the same arithmetic the walk used to apply position by position.
__global__ void __launch_bounds__(256) k_accept_probs(const __grid_constant__ SampleArgs a, int dtype,
                                                      const __grid_constant__ VerifyK v) {
  const int lane = threadIdx.x & 31;
  const int K1 = v.k + 1;
  const int64_t D = (a.rows / K1) * v.k;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < D;
       w += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t b = w / v.k;
    const int i = (int)(w - b * v.k);
    const int64_t row = b * K1 + i;
    const pm_row_params p = row_params(a, row);
    const int mode = row_mode(p);
    const int d = v.drafts[w];
    float dm;
    const float cd = __shfl_sync(kFull, warp_combine(v.dstat + w * a.n_tiles, a.n_tiles, &dm), 0);
    if (lane == 0) v.dlse[w] = cd;
    AccProb r;
    r.qd = draft_prob(v, w, d, cd);
    r.cy = 0.0f;
    r.wide = 0;
    r.pd = 0.0f;
    if (mode == kGreedy) {
      r.pd = ld_cg(&v.rtok[row]) == d ? 1.0f : 0.0f;
    } else if (mode == kCand) {
      const int n = ld_cg(&v.ns[row]);
      if (n > v.scap) {
        r.wide = 1;
      } else {
        float f = 0.0f;
        for (int q = lane; q < n; q += 32)
          if (ld_cg(&v.sids[row * v.scap + q]) == d) f = ld_cg(&v.sprobs[row * v.scap + q]);
        r.pd = warp_max(f);
      }
    } else {
      float m;
      r.cy = warp_combine(a.staty + row * a.n_tiles, a.n_tiles, &m);
      const float x = processed_value(a, dtype, p, row, d);
      const float y = x > -INFINITY ? fmul(x, p.inv_temperature) : -INFINITY;
      r.pd = det_expf(fsub(y, r.cy));
    }
    if (lane == 0) v.probs[w] = r;
    __syncwarp();
  }
}

// Acceptance: one warp per request.
template <int KC>
__global__ void __launch_bounds__(256) k_verify_accept(const __grid_constant__ SampleArgs a, int dtype,
                                                       const __grid_constant__ VerifyK v) {
  struct AccMem {
    uint64_t key[KC];
    uint64_t q[KC];
  };
  extern __shared__ __align__(16) unsigned char smem_acc[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  AccMem* am = reinterpret_cast<AccMem*>(smem_acc) + wid;
  const int K1 = v.k + 1;
  const int64_t B = a.rows / K1;
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + wid; b < B;
       b += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t base = b * K1;
    int32_t* out = v.tokens + b * K1;
    if (v.row_tokens)
      for (int i = lane; i < K1; i += 32) v.row_tokens[base + i] = ld_cg(&v.rtok[base + i]);
    if (v.mode == PM_VERIFY_MATCH) {
      int emit = K1;
      for (int i0 = 0; i0 < K1; i0 += 32) {
        const int i = i0 + lane;
        bool stop = false;
        if (i < K1) stop = i == v.k || ld_cg(&v.rtok[base + i]) != v.drafts[b * v.k + i];
        const unsigned bal = __ballot_sync(kFull, stop);
        if (bal) { emit = i0 + __ffs(bal); break; }
      }
      for (int i = lane; i < K1; i += 32) out[i] = i < emit ? ld_cg(&v.rtok[base + i]) : -1;
      if (lane == 0) { v.n_acc[b] = emit - 1; v.pending[b] = -1; }
      __syncwarp();
      continue;
    }
    int i = 0;
    int final_tok = 0;
    bool pend = false;
    bool wide = false;
    for (; i < v.k; ++i) {
      const int64_t row = base + i;
      const int64_t drow = b * v.k + i;
      const pm_row_params p = row_params(a, row);
      const int mode = row_mode(p);
      const float cd = ld_cg(&v.dlse[drow]);
      const AccProb pr = ld_cg_accprob(&v.probs[drow]);
      if (pr.wide) {  // survivors beyond the candidate lists: this request cannot be judged exactly
        wide = true;
        break;
      }
      const float cy = pr.cy;
      if (dmul(accept_uniform(a, v, b, i, row), (double)pr.qd) < (double)pr.pd) continue;
      // first rejection at row i: a draw from max(p - q, 0)
      if (mode == kGreedy) {
        final_tok = ld_cg(&v.rtok[row]);  // the only token with a positive residual, or the row's own draw
      } else if (mode == kCand) {
        final_tok = survivor_residual<KC>(a, v, b, row, drow, cd, am->key, am->q);
        if (final_tok < 0) final_tok = ld_cg(&v.rtok[row]);
      } else {
        pend = true;  // whole vocabulary: k_residual_tiles and k_residual_draw draw it
        if (lane == 0) v.ylse[b] = cy;
      }
      break;
    }
    if (wide) {
      for (int r = lane; r < K1; r += 32) out[r] = -1;
      if (lane == 0) { v.n_acc[b] = -1; v.pending[b] = -1; }
      __syncwarp();
      continue;
    }
    if (i == v.k) final_tok = ld_cg(&v.rtok[base + v.k]);  // every draft accepted: the bonus token
    for (int r = lane; r < K1; r += 32)
      out[r] = r < i ? v.drafts[b * v.k + r] : (r == i && !pend ? final_tok : -1);
    if (lane == 0) { v.n_acc[b] = i; v.pending[b] = pend ? i : -1; }
    __syncwarp();
  }
}

// Whole-vocabulary residual draw, tile-parallel.  k_residual_tiles: one
// warp per (request, tile) of every request with a pending row: the tile's
// sum of floor(max(fl32(p - q), 0) 2^52), p = expf(fl32(y - c_y)),
// q = expf(fl32(d - c_d)).  k_residual_draw: one CTA per pending request:
// the tile whose inclusive prefix first exceeds floor(u R), then the token
// inside it the same way, the tile's 1,024 masses computed by all eight
// warps (no positive residual: the row's own draw).
template <typename T, typename TD>
__global__ void __launch_bounds__(256) k_residual_tiles(const __grid_constant__ SampleArgs a,
                                                        const __grid_constant__ SampleArgs da,
                                                        const __grid_constant__ VerifyK v) {
  constexpr int VW = Lay<T>::VW;
  constexpr bool same = Lay<T>::VW == Lay<TD>::VW;
  const int lane = threadIdx.x & 31;
  const int K1 = v.k + 1;
  const int64_t B = a.rows / K1;
  const int nt = a.n_tiles;
  const int64_t total = B * nt;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
       w += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t b = w / nt;
    const int t = (int)(w - b * nt);
    const int j = ld_cg(&v.pending[b]);
    if (j < 0) continue;  // warp-uniform
    const int64_t row = b * K1 + j;
    const int64_t drow = b * v.k + j;
    const pm_row_params p = row_params(a, row);
    const float cy = ld_cg(&v.ylse[b]);
    const float cd = ld_cg(&v.dlse[drow]);
    TileIn ti;
    load_tile<T>(a, row, t, ti);
    process_tile_regs<VW>(a, p, row, t, ti);
    TileIn td;
    if constexpr (same) load_tile<TD>(da, drow, t, td);
    const int64_t start = (int64_t)t * kTile;
    const int n_valid = tile_valid(a, t);
    uint64_t s = 0;
#pragma unroll
    for (int sl = 0; sl < 32; sl += 2) {
      float y2[2], d2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e = slot_elem<VW>(sl + h, lane);
        const float x = ti.v[sl + h];
        y2[h] = x > -INFINITY ? fmul(x, p.inv_temperature) : -INFINITY;
        if constexpr (same) d2[h] = td.v[sl + h];
        else d2[h] = e < n_valid ? draft_value(v, drow, start + e) : -INFINITY;
      }
      float p0, p1, q0, q1;
      det_expf_x2(fsub(y2[0], cy), fsub(y2[1], cy), p0, p1);
      det_expf_x2(fsub(d2[0], cd), fsub(d2[1], cd), q0, q1);
      if (slot_elem<VW>(sl, lane) < n_valid) s += residual_q52(p0, q0);
      if (slot_elem<VW>(sl + 1, lane) < n_valid) s += residual_q52(p1, q1);
    }
    s = warp_sum_u64(s);
    if (lane == 0) v.rsum[w] = s;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) k_residual_draw(const __grid_constant__ SampleArgs a,
                                                       const __grid_constant__ VerifyK v) {
  constexpr int VW = Lay<T>::VW;
  __shared__ uint64_t qbuf[kTile];  // the chosen tile's residual masses in token order
  __shared__ uint64_t wtot[8];
  __shared__ uint64_t s_t2;
  __shared__ int s_tt, s_tok;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int K1 = v.k + 1;
  const int64_t B = a.rows / K1;
  const int nt = a.n_tiles;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const int j = ld_cg(&v.pending[b]);
    if (j < 0) continue;  // uniform over the CTA
    const int64_t row = b * K1 + j;
    const int64_t drow = b * v.k + j;
    const pm_row_params p = row_params(a, row);
    const float cy = ld_cg(&v.ylse[b]);
    const float cd = ld_cg(&v.dlse[drow]);
    // warp 0: the tile whose inclusive prefix of the tile sums first exceeds
    // floor(u R), and the target left inside it
    if (wid == 0) {
      const uint64_t* rs = v.rsum + b * nt;
      uint64_t R = 0;
      for (int t = lane; t < nt; t += 32) R += ld_cg(&rs[t]);
      R = warp_sum_u64(R);
      int tt = -1;
      uint64_t t2 = 0;
      if (R > 0) {
        const uint64_t tgt = scale_u53(residual_u53(a, v, b, row), R);
        uint64_t carry = 0;
        for (int t0 = 0; t0 < nt; t0 += 32) {
          const int t = t0 + lane;
          const uint64_t wv = t < nt ? ld_cg(&rs[t]) : 0ull;
          const uint64_t incl = carry + warp_incl_scan_u64(wv);
          const unsigned hit = __ballot_sync(kFull, t < nt && incl > tgt);
          if (hit) {
            const int src = __ffs(hit) - 1;
            tt = t0 + src;
            t2 = tgt - (__shfl_sync(kFull, incl, src) - __shfl_sync(kFull, wv, src));
            break;
          }
          carry = __shfl_sync(kFull, incl, 31);
        }
      }
      if (lane == 0) {
        s_tt = tt;
        s_t2 = t2;
        s_tok = ld_cg(&v.rtok[row]);  // no positive residual: the row's own draw
      }
    }
    __syncthreads();
    const int tt = s_tt;
    if (tt >= 0) {
      // every warp loads and processes the tile; warp w computes the masses of
      // its four slots a lane (128 tokens), stored by token index
      TileIn ti;
      load_tile<T>(a, row, tt, ti);
      process_tile_regs<VW>(a, p, row, tt, ti);
      const int64_t start = (int64_t)tt * kTile;
      const int n_valid = tile_valid(a, tt);
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const int sl = wid * 4 + k4;
        const int e = slot_elem<VW>(sl, lane);
        uint64_t q = 0;
        if (e < n_valid) {
          const float x = ti.v[sl];
          const float y = x > -INFINITY ? fmul(x, p.inv_temperature) : -INFINITY;
          q = residual_q52(det_expf(fsub(y, cy)), draft_prob(v, drow, start + e, cd));
        }
        qbuf[e] = q;
      }
      __syncthreads();
      // the token whose inclusive prefix first exceeds t2: thread t scans
      // tokens [4 t, 4 t + 4) after a block scan of the four-token sums
      uint64_t loc = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) loc += qbuf[4 * tid + c];
      const uint64_t wincl = warp_incl_scan_u64(loc);
      if (lane == 31) wtot[wid] = wincl;
      __syncthreads();
      uint64_t base = 0;
      for (int w = 0; w < wid; ++w) base += wtot[w];
      const uint64_t excl = base + wincl - loc;
      const uint64_t t2 = s_t2;
      if (excl <= t2 && t2 < excl + loc) {
        uint64_t run = excl;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          run += qbuf[4 * tid + c];
          if (run > t2) {
            s_tok = (int)(start + 4 * tid + c);
            break;
          }
        }
      }
    }
    __syncthreads();
    if (tid == 0) v.tokens[b * K1 + j] = s_tok;
    __syncthreads();
  }
}

}  // namespace pm
