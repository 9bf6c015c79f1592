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
// The CTA that finishes a row's last chunk (self-resetting atomicInc
// counter, no spin-wait anywhere) merges the row: log-sum-exp from the tile
// statistics, the row's top-K candidates, top-p / min-p, and the draw.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "pm_device.cuh"
#include "pm_prep.cuh"
#include "pm_select.cuh"
#include "../../include/pm_sample.h"

namespace pm {

struct TileStat {
  float m;
  uint32_t pad;
  uint64_t s;
};

enum RowMode { kGreedy = 0, kCand = 1, kFullDraw = 2 };

// Everything one launch of the streaming kernel needs.
struct SampleArgs {
  const void* logits;
  int64_t rows, vocab, row_stride;
  bool vec_ok;
  const pm_row_params* params;
  int32_t params_per_row;
  // processors
  const int32_t* ovr_tok;
  const uint32_t* ovr_info;
  const int32_t* ovr_off;
  int32_t ovr_cap;
  const int32_t* bias_tok;
  const float* bias_val;
  const int32_t* bias_off;  // [n_tiles + 1]
  const uint32_t* mask;
  int64_t mask_stride;
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
  TileStat* statx;  // [rows, n_tiles]
  TileStat* staty;  // [rows, n_tiles]
  uint64_t* cand;   // [rows, n_chunks, KC]
  int32_t* cand_n;  // [rows, n_chunks]
  uint64_t* best;   // [rows, n_chunks]
  uint32_t* row_done;
  int32_t* status;
  float* row_lse;   // [rows]
  int32_t n_tiles, n_chunks, chunk_tiles;
  int64_t n_items;
};

template <typename T> struct Lay;
template <> struct Lay<float> { static constexpr int VW = 4; };
template <> struct Lay<__nv_bfloat16> { static constexpr int VW = 8; };

// Position inside the tile of value slot s (0..31) of `lane`.
template <int VW>
__device__ __forceinline__ int slot_elem(int s, int lane) {
  return (s / VW) * (32 * VW) + lane * VW + (s % VW);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// Raw values of one tile into v[32]; positions >= n_valid read as -inf.
template <typename T>
__device__ __forceinline__ void load_tile_raw(const T* rowp, int64_t start, int n_valid, bool vec_ok,
                                              float (&v)[32]) {
  constexpr int VW = Lay<T>::VW;
  const int lane = threadIdx.x & 31;
  if (vec_ok && n_valid == kTile) {
    if constexpr (sizeof(T) == 4) {
      const float4* p = reinterpret_cast<const float4*>(rowp + start);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 q = __ldcs(p + j * 32 + lane);
        v[4 * j] = q.x; v[4 * j + 1] = q.y; v[4 * j + 2] = q.z; v[4 * j + 3] = q.w;
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(rowp + start);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 q = __ldcs(p + j * 32 + lane);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[8 * j + 2 * h] = bf16_bits_to_f32(w[h] & 0xffffu);
          v[8 * j + 2 * h + 1] = bf16_bits_to_f32(w[h] >> 16);
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
      v[s] = x;
    }
  }
}

// Processors on one loaded tile: logit bias, penalties (through the warp's
// staging buffer, only when the tile holds an overridden id), then the mask.
// Order as mlx-lm's make_logits_processors list followed by the reference's
// mask processors (server.py:3045-3049 appends them last).
template <int VW>
__device__ __forceinline__ void process_tile(const SampleArgs& a, const pm_row_params& p, int64_t row,
                                             int tile, int n_valid, float (&v)[32], float* wbuf) {
  const int lane = threadIdx.x & 31;
  const int64_t start = (int64_t)tile * kTile;
  int ob = 0, oe = 0, bb = 0, be = 0;
  if (a.ovr_off) {
    const int32_t* off = a.ovr_off + row * (int64_t)(a.n_tiles + 1);
    ob = off[tile];
    oe = off[tile + 1];
  }
  if (a.bias_off) { bb = a.bias_off[tile]; be = a.bias_off[tile + 1]; }
  if (oe > ob || be > bb) {
#pragma unroll
    for (int s = 0; s < 32; ++s) wbuf[slot_elem<VW>(s, lane)] = v[s];
    __syncwarp();
    for (int i = bb + lane; i < be; i += 32) {
      const int e = (int)(a.bias_tok[i] - start);
      wbuf[e] = fadd(wbuf[e], a.bias_val[i]);
    }
    __syncwarp();
    const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
    const uint32_t* oinf = a.ovr_info + row * (int64_t)a.ovr_cap;
    for (int i = ob + lane; i < oe; i += 32) {
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
    for (int s = 0; s < 32; ++s) v[s] = wbuf[slot_elem<VW>(s, lane)];
    __syncwarp();
  }
  if (a.mask) {
    const uint32_t* mrow = a.mask + row * a.mask_stride + (start >> 5);
    const int nw = (n_valid + 31) >> 5;
    const uint32_t mw = lane < nw ? mrow[lane] : 0u;
#pragma unroll
    for (int j = 0; j < 32 / VW; ++j) {
      const uint32_t w = __shfl_sync(kFull, mw, j * VW + (lane * VW) / 32);
      const uint32_t bits = w >> ((lane * VW) & 31);
#pragma unroll
      for (int c = 0; c < VW; ++c)
        if (!((bits >> c) & 1u)) v[j * VW + c] = -INFINITY;
    }
  }
}

// Exact tile statistics of v (warp-uniform result).
__device__ __forceinline__ void tile_stats(const float (&v)[32], float* m_out, uint64_t* s_out) {
  float m = -INFINITY;
#pragma unroll
  for (int s = 0; s < 32; ++s) m = fmaxf(m, v[s]);
  m = warp_max(m);
  uint64_t sum = 0;
  if (m > -INFINITY) {
#pragma unroll
    for (int s = 0; s < 32; ++s) sum += q52(fsub(v[s], m));
  }
  *m_out = m;
  *s_out = warp_sum_u64(sum);
}

__device__ __forceinline__ const pm_row_params& row_params(const SampleArgs& a, int64_t row) {
  return a.params[a.params_per_row ? row : 0];
}

__device__ __forceinline__ int row_mode(const pm_row_params& p) {
  if (p.flags & PM_F_GREEDY) return kGreedy;
  if (p.top_k > 0 || (p.flags & (PM_F_TOP_P | PM_F_MIN_P))) return kCand;
  return kFullDraw;
}
__device__ __forceinline__ bool needs_xstats(const SampleArgs& a, const pm_row_params& p, int mode) {
  return a.want_lse || (mode == kCand && (p.flags & (PM_F_TOP_P | PM_F_MIN_P)));
}

// Shared-memory plan of the streaming kernel.
template <int KC, int VW>
struct Smem {
  static constexpr int CAP = KC + 32 * VW;          // per-warp candidate buffer
  static constexpr int kStage = kWarps * kTile * 4;  // staging floats / merge keys (bytes)
  static constexpr int kSort = KC * 8;
  static constexpr int kWarpBuf = kWarps * CAP * 8;
  static constexpr int kWarpHist = kWarps * 256 * 4;
  static constexpr int kBlockHist = 256 * 4;
  static constexpr int kTileVals = 1024 * 8;        // row-merge per-tile doubles
  static constexpr int kMisc = 256;
  static constexpr int bytes = kStage + kSort + kWarpBuf + kWarpHist + kBlockHist + kTileVals + kMisc;
};

struct MiscShared {
  int scal[8];
  int flag;
  int chunk_n;
  uint64_t warp_best[kWarps];
  double dscal[4];
  uint64_t u64s[4];
};

// --------------------------------------------------------------------------
// row-merge pieces
// --------------------------------------------------------------------------

// Log-sum-exp of a row from its tile statistics; also leaves
// a_t = s_t e^(m_t - m) in tv[0..n_tiles) and m in *m_out.  All threads.
__device__ float block_combine(const TileStat* st, int nt, double* tv, float* m_out, MiscShared* ms) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float m = -INFINITY;
  for (int t = tid; t < nt; t += blockDim.x) m = fmaxf(m, ld_cg(&st[t].m));
  m = warp_max(m);
  __shared__ float wm[kWarps];
  if (lane == 0) wm[wid] = m;
  __syncthreads();
  float mm = -INFINITY;
  for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, wm[w]);
  __syncthreads();
  *m_out = mm;
  if (!(mm > -INFINITY)) {
    for (int t = tid; t < nt; t += blockDim.x) tv[t] = 0.0;
    __syncthreads();
    return -INFINITY;
  }
  for (int t = tid; t < nt; t += blockDim.x) {
    const uint64_t s = ld_cg(&st[t].s);
    const float mt = ld_cg(&st[t].m);
    tv[t] = s ? dmul((double)s, det_exp64(dsub((double)mt, (double)mm))) : 0.0;
  }
  __syncthreads();
  // pairwise tree over P = next pow2 >= nt, zero padded.  Thread t reduces
  // its contiguous block of P/256 tiles, then a 256-wide tree.
  int P = 1;
  while (P < nt) P <<= 1;
  const int per = P > kThreads ? P / kThreads : 1;
  double acc = 0.0;
  {
    // local pairwise tree over [tid*per, tid*per+per)
    double loc[4];
    const int base = tid * per;
    if (per == 1) {
      acc = base < nt ? tv[base] : 0.0;
    } else {
      // per in {2, 4}: supported up to P = 1024 tiles
      for (int i = 0; i < per; ++i) loc[i] = (base + i < nt) ? tv[base + i] : 0.0;
      for (int w = per; w > 1; w >>= 1)
        for (int i = 0; i < w / 2; ++i) loc[i] = dadd(loc[2 * i], loc[2 * i + 1]);
      acc = loc[0];
    }
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_down_sync(kFull, acc, o);
    if ((lane & (2 * o - 1)) == 0) acc = dadd(acc, t);
  }
  __shared__ double wsum[kWarps];
  if (lane == 0) wsum[wid] = acc;
  __syncthreads();
  double Z;
  {
    double w[kWarps];
    for (int i = 0; i < kWarps; ++i) w[i] = wsum[i];
    for (int n = kWarps; n > 1; n >>= 1)
      for (int i = 0; i < n / 2; ++i) w[i] = dadd(w[2 * i], w[2 * i + 1]);
    Z = w[0];
  }
  __syncthreads();
  return (float)dadd((double)mm, det_log64(dmul(Z, 0x1p-52)));
}

__device__ __forceinline__ float row_gumbel(const SampleArgs& a, int64_t row, uint32_t token) {
  if (a.noise_mode == PM_NOISE_INJECTED) return a.gumbel[row * a.gumbel_stride + token];
  return philox_gumbel(a.seed, a.offset, a.row_base + (uint32_t)row, token);
}
__device__ __forceinline__ uint64_t row_u53(const SampleArgs& a, int64_t row, int stream) {
  if (a.noise_mode == PM_NOISE_INJECTED) return u53_from_double(a.uniform[row * 2 + stream]);
  return philox_u53(a.seed, a.offset, a.row_base + (uint32_t)row, (uint32_t)stream);
}

// Filters and Gumbel draw over the row's sorted top candidates S[0..m),
// one warp.  Returns the token (or -1 when the survivors cannot be decided
// from the candidates, which flags the row for the exact fallback).
__device__ int warp_filter_draw(const SampleArgs& a, const pm_row_params& p, int64_t row,
                                const uint64_t* S, int m, bool complete, float c) {
  const int lane = threadIdx.x & 31;
  if (m == 0) return 0;
  const bool topk = p.top_k > 0;
  int cnt = (topk && p.top_k < m) ? p.top_k : m;
  // With top_k on, the candidates hold the exact top-k prefix.  Otherwise
  // they are the exact top-KC prefix of the row (all of it when complete),
  // and the survivors are known once some filter cuts inside that prefix.
  bool determined = topk || complete;
  if (p.flags & PM_F_TOP_P) {
    uint64_t T = 0;
    for (int r = lane; r < cnt; r += 32) T += q52(fsub(key_value(S[r]), c));
    T = warp_sum_u64(T);
    if (!topk) T = 1ull << 52;
    const uint64_t qthr = __float2ull_rz(fmul(p.top_p_comp, 0x1p52f));
    uint64_t carry = 0;
    int keep = cnt;
    bool found = false;
    for (int base = 0; base < cnt && !found; base += 32) {
      const int r = base + lane;
      const uint64_t q = r < cnt ? q52(fsub(key_value(S[r]), c)) : 0ull;
      const uint64_t incl = warp_incl_scan_u64(q);
      const uint64_t A = carry + incl - q;  // exclusive prefix
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
  // Gumbel-max: argmax fl32(fl32(x * inv_temp) + g), ties to the lowest id
  float bs = -INFINITY;
  int bid = -1;
  for (int r = lane; r < cnt; r += 32) {
    const uint32_t id = key_index(S[r]);
    const float sc = fadd(fmul(key_value(S[r]), p.inv_temperature), row_gumbel(a, row, id));
    if (bid < 0 || sc > bs || (sc == bs && (int)id < bid)) { bs = sc; bid = (int)id; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float os = __shfl_xor_sync(kFull, bs, o);
    const int oid = __shfl_xor_sync(kFull, bid, o);
    if (oid >= 0 && (bid < 0 || os > bs || (os == bs && oid < bid))) { bs = os; bid = oid; }
  }
  if (a.surv_ids && lane == 0) {
    double ymax = -INFINITY;
    for (int r = 0; r < cnt; ++r) {
      const double yv = (double)fmul(key_value(S[r]), p.inv_temperature);
      ymax = yv > ymax ? yv : ymax;
    }
    double Z = 0.0;
    for (int r = 0; r < cnt; ++r) Z = dadd(Z, det_exp64(dsub((double)fmul(key_value(S[r]), p.inv_temperature), ymax)));
    for (int r = 0; r < cnt && r < a.surv_cap; ++r) {
      a.surv_ids[row * a.surv_cap + r] = (int32_t)key_index(S[r]);
      a.surv_probs[row * a.surv_cap + r] =
          (float)__ddiv_rn(det_exp64(dsub((double)fmul(key_value(S[r]), p.inv_temperature), ymax)), Z);
    }
    for (int r = cnt; r < a.surv_cap; ++r) { a.surv_ids[row * a.surv_cap + r] = -1; a.surv_probs[row * a.surv_cap + r] = 0.0f; }
    a.n_surv[row] = cnt;
  }
  return bid;
}

// Whole-vocabulary draw: tile by exact integer weights, then the id inside
// the tile by its integer masses (two uniforms).  Warp 0 re-reads the tile.
template <typename T>
__device__ int full_draw(const SampleArgs& a, const pm_row_params& p, int64_t row, const double* tv,
                         float my, float* wbuf) {
  constexpr int VW = Lay<T>::VW;
  const int lane = threadIdx.x & 31;
  const int nt = a.n_tiles;
  if (!(my > -INFINITY)) return 0;
  int sh = 1;
  while ((1 << (sh - 1)) < nt) ++sh;
  const double scale = __longlong_as_double((long long)(1023 - sh) << 52);  // 2^-sh
  uint64_t W = 0;
  for (int t = lane; t < nt; t += 32) W += __double2ull_rz(dmul(tv[t], scale));
  W = warp_sum_u64(W);
  const uint64_t t1 = scale_u53(row_u53(a, row, 0), W);
  int tt = nt - 1;
  uint64_t carry = 0;
  for (int base = 0; base < nt; base += 32) {
    const int t = base + lane;
    const uint64_t w = t < nt ? __double2ull_rz(dmul(tv[t], scale)) : 0ull;
    const uint64_t incl = carry + warp_incl_scan_u64(w);
    const unsigned hit = __ballot_sync(kFull, t < nt && incl > t1);
    if (hit) { tt = base + __ffs(hit) - 1; break; }
    carry = __shfl_sync(kFull, incl, 31);
  }
  const TileStat* st = a.staty + row * (int64_t)nt;
  const float mt = ld_cg(&st[tt].m);
  const uint64_t stt = ld_cg(&st[tt].s);
  const uint64_t t2 = scale_u53(row_u53(a, row, 1), stt);
  const int64_t start = (int64_t)tt * kTile;
  const int n_valid = (int)((a.vocab - start) < kTile ? (a.vocab - start) : kTile);
  float v[32];
  const T* rowp = reinterpret_cast<const T*>(a.logits) + row * a.row_stride;
  load_tile_raw<T>(rowp, start, n_valid, a.vec_ok, v);
  process_tile<VW>(a, p, row, tt, n_valid, v, wbuf);
  uint64_t acc = 0;
  int tok = (int)start;
  for (int j = 0; j < 32 / VW; ++j) {
    uint64_t q[VW];
    uint64_t ls = 0;
#pragma unroll
    for (int c = 0; c < VW; ++c) {
      const float x = v[j * VW + c];
      const float y = x > -INFINITY ? fmul(x, p.inv_temperature) : -INFINITY;
      q[c] = q52(fsub(y, mt));
      ls += q[c];
    }
    const uint64_t incl = acc + warp_incl_scan_u64(ls);
    const unsigned hit = __ballot_sync(kFull, incl > t2);
    if (hit) {
      const int src = __ffs(hit) - 1;
      int found = -1;
      if (lane == src) {
        uint64_t run = incl - ls;
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          run += q[c];
          if (found < 0 && run > t2) found = c;
        }
      }
      found = __shfl_sync(kFull, found, src);
      tok = (int)(start + j * 32 * VW + src * VW + found);
      break;
    }
    acc = __shfl_sync(kFull, incl, 31);
  }
  return tok;
}

// --------------------------------------------------------------------------
// the streaming kernel
// --------------------------------------------------------------------------
template <typename T, int KC>
__global__ void __launch_bounds__(kThreads) k_sample_stream(SampleArgs a) {
  constexpr int VW = Lay<T>::VW;
  using SM = Smem<KC, VW>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* stage = reinterpret_cast<float*>(smem_raw);
  uint64_t* U = reinterpret_cast<uint64_t*>(smem_raw);  // aliases stage after the tiles
  uint64_t* S = reinterpret_cast<uint64_t*>(smem_raw + SM::kStage);
  uint64_t* wcand = reinterpret_cast<uint64_t*>(smem_raw + SM::kStage + SM::kSort);
  unsigned* whist = reinterpret_cast<unsigned*>(smem_raw + SM::kStage + SM::kSort + SM::kWarpBuf);
  unsigned* bhist = whist + kWarps * 256;
  double* tv = reinterpret_cast<double*>(smem_raw + SM::kStage + SM::kSort + SM::kWarpBuf + SM::kWarpHist +
                                         SM::kBlockHist);
  MiscShared* ms = reinterpret_cast<MiscShared*>(smem_raw + SM::kStage + SM::kSort + SM::kWarpBuf +
                                                 SM::kWarpHist + SM::kBlockHist + SM::kTileVals);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float* wbuf = stage + wid * kTile;
  uint64_t* mybuf = wcand + wid * SM::CAP;
  unsigned* myhist = whist + wid * 256;

  for (int64_t item = blockIdx.x; item < a.n_items; item += gridDim.x) {
    const int64_t row = item / a.n_chunks;
    const int chunk = (int)(item % a.n_chunks);
    const pm_row_params p = row_params(a, row);
    const int mode = row_mode(p);
    const bool needx = needs_xstats(a, p, mode);
    const bool needy = mode == kFullDraw;
    const int t0 = chunk * a.chunk_tiles;
    const int t1 = min(t0 + a.chunk_tiles, a.n_tiles);
    const T* rowp = reinterpret_cast<const T*>(a.logits) + row * a.row_stride;
    // per-warp state
    float best_x = -INFINITY;
    int best_e = -1;
    int cnt = 0;
    uint64_t tau = 0;
    float tau_x = -INFINITY;
    const int kc_row = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;

    for (int t = t0 + wid; t < t1; t += kWarps) {
      const int64_t start = (int64_t)t * kTile;
      const int n_valid = (int)((a.vocab - start) < kTile ? (a.vocab - start) : kTile);
      float v[32];
      load_tile_raw<T>(rowp, start, n_valid, a.vec_ok, v);
      process_tile<VW>(a, p, row, t, n_valid, v, wbuf);
      if (needx) {
        float m;
        uint64_t s;
        tile_stats(v, &m, &s);
        if (lane == 0) { TileStat ts; ts.m = m; ts.pad = 0; ts.s = s; a.statx[row * a.n_tiles + t] = ts; }
      }
      if (needy) {
        float y[32];
#pragma unroll
        for (int s = 0; s < 32; ++s) y[s] = v[s] > -INFINITY ? fmul(v[s], p.inv_temperature) : -INFINITY;
        float m;
        uint64_t s;
        tile_stats(y, &m, &s);
        if (lane == 0) { TileStat ts; ts.m = m; ts.pad = 0; ts.s = s; a.staty[row * a.n_tiles + t] = ts; }
      }
      if (mode == kGreedy) {
#pragma unroll
        for (int s = 0; s < 32; ++s) {
          if (best_e < 0 || v[s] > best_x) {
            const int e = slot_elem<VW>(s, lane);
            if (e < n_valid) { best_x = v[s]; best_e = (int)(start + e); }
          }
        }
      } else if (mode == kCand) {
#pragma unroll
        for (int j = 0; j < 32 / VW; ++j) {
          unsigned pm = 0;
#pragma unroll
          for (int c = 0; c < VW; ++c) {
            const float x = v[j * VW + c];
            if (x > -INFINITY && x >= tau_x) pm |= 1u << c;
          }
          if (__any_sync(kFull, pm)) {
            uint64_t keys[VW];
            unsigned valid = 0;
#pragma unroll
            for (int c = 0; c < VW; ++c) {
              const int e = j * 32 * VW + lane * VW + c;
              keys[c] = rankkey(v[j * VW + c], (uint32_t)(start + e));
              if (((pm >> c) & 1u) && keys[c] > tau) valid |= 1u << c;
            }
            const int nv = __popc(valid);
            const int incl = warp_incl_scan(nv);
            int pos = cnt + incl - nv;
#pragma unroll
            for (int c = 0; c < VW; ++c)
              if ((valid >> c) & 1u) mybuf[pos++] = keys[c];
            cnt += __shfl_sync(kFull, incl, 31);
            __syncwarp();
            if (cnt > SM::CAP - 32 * VW) {
              tau = warp_select_topk<(SM::CAP + 31) / 32>(mybuf, cnt, kc_row, myhist);
              tau_x = key_value(tau);
              cnt = kc_row;
            }
          }
        }
      }
    }

    // ---- chunk end: combine the warps ----
    bool last = false;
    if (mode == kGreedy) {
      const uint64_t k = best_e >= 0 ? rankkey(best_x, (uint32_t)best_e) : 0ull;
      const uint64_t wk = warp_max_u64(k);
      if (lane == 0) ms->warp_best[wid] = wk;
      __syncthreads();
      if (tid == 0) {
        uint64_t bk = 0;
        for (int w = 0; w < kWarps; ++w) bk = ms->warp_best[w] > bk ? ms->warp_best[w] : bk;
        a.best[row * a.n_chunks + chunk] = bk;
      }
    } else if (mode == kCand) {
      if (cnt > kc_row) {
        warp_select_topk<(SM::CAP + 31) / 32>(mybuf, cnt, kc_row, myhist);
        cnt = kc_row;
      }
      if (tid == 0) ms->chunk_n = 0;
      __syncthreads();
      int base = 0;
      if (lane == 0) base = atomicAdd(&ms->chunk_n, cnt);
      base = __shfl_sync(kFull, base, 0);
      for (int i = lane; i < cnt; i += 32) U[base + i] = mybuf[i];
      __syncthreads();
      const int n = ms->chunk_n;
      __syncthreads();
      const int m = block_topk_sorted(U, n, kc_row, S, KC, bhist, ms->scal);
      uint64_t* dst = a.cand + (row * a.n_chunks + chunk) * (int64_t)KC;
      for (int i = tid; i < m; i += kThreads) dst[i] = S[i];
      if (tid == 0) a.cand_n[row * a.n_chunks + chunk] = m;
    }
    // publish, then count this chunk in; the CTA that completes the row merges it
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned prev = atomicInc(&a.row_done[row], (unsigned)(a.n_chunks - 1));
      ms->flag = (prev == (unsigned)(a.n_chunks - 1));
    }
    __syncthreads();
    last = ms->flag;
    __syncthreads();
    if (!last) continue;
    __threadfence();

    // ---- row merge ----
    float c = __int_as_float(0x7fc00000);
    float mx;
    if (needx) c = block_combine(a.statx + row * a.n_tiles, a.n_tiles, tv, &mx, ms);
    int tok = 0;
    float tok_x = -INFINITY;
    if (mode == kGreedy) {
      uint64_t bk = 0;
      for (int ch = tid; ch < a.n_chunks; ch += kThreads) {
        const uint64_t k = ld_cg(&a.best[row * a.n_chunks + ch]);
        bk = k > bk ? k : bk;
      }
      bk = warp_max_u64(bk);
      if (lane == 0) ms->warp_best[wid] = bk;
      __syncthreads();
      if (tid == 0) {
        uint64_t b2 = 0;
        for (int w = 0; w < kWarps; ++w) b2 = ms->warp_best[w] > b2 ? ms->warp_best[w] : b2;
        ms->u64s[0] = b2;
      }
      __syncthreads();
      const uint64_t b2 = ms->u64s[0];
      tok = (int)key_index(b2);
      tok_x = key_value(b2);
      __syncthreads();
    } else if (mode == kCand) {
      // gather the chunk lists
      if (tid == 0) {
        int off = 0, full = 0;
        for (int ch = 0; ch < a.n_chunks; ++ch) {
          const int n = ld_cg(&a.cand_n[row * a.n_chunks + ch]);
          full |= (n >= kc_row) ? 1 : 0;
          off += n;
        }
        ms->chunk_n = off;
        ms->scal[5] = full;
      }
      __syncthreads();
      {
        // copy lists (each thread walks the chunk table; lists are short)
        int off = 0;
        for (int ch = 0; ch < a.n_chunks; ++ch) {
          const int n = ld_cg(&a.cand_n[row * a.n_chunks + ch]);
          const uint64_t* src = a.cand + (row * a.n_chunks + ch) * (int64_t)KC;
          for (int i = tid; i < n; i += kThreads) U[off + i] = ld_cg(&src[i]);
          off += n;
        }
      }
      __syncthreads();
      const int n = ms->chunk_n;
      const bool complete = ms->scal[5] == 0;
      __syncthreads();
      const int m = block_topk_sorted(U, n, kc_row, S, KC, bhist, ms->scal);
      if (wid == 0) {
        const int r = warp_filter_draw(a, p, row, S, m, complete, c);
        if (lane == 0) ms->scal[6] = r;
      }
      __syncthreads();
      tok = ms->scal[6];
      if (tok < 0) {
        if (tid == 0) a.status[row] = 1;  // survivors beyond the candidates: exact fallback
        tok = -1;
      } else {
        for (int i = 0; i < m; ++i)
          if ((int)key_index(S[i]) == tok) { tok_x = key_value(S[i]); break; }
      }
      __syncthreads();
    } else {
      float my;
      block_combine(a.staty + row * a.n_tiles, a.n_tiles, tv, &my, ms);
      if (wid == 0) {
        const int r = full_draw<T>(a, p, row, tv, my, wbuf);
        if (lane == 0) ms->scal[6] = r;
      }
      __syncthreads();
      tok = ms->scal[6];
      __syncthreads();
      if (a.tok_logprob) {
        // processed logit of the chosen id
        if (wid == 0) {
          const int tt = tok / kTile;
          const int64_t start = (int64_t)tt * kTile;
          const int n_valid = (int)((a.vocab - start) < kTile ? (a.vocab - start) : kTile);
          float v[32];
          load_tile_raw<T>(rowp, start, n_valid, a.vec_ok, v);
          process_tile<VW>(a, p, row, tt, n_valid, v, wbuf);
#pragma unroll
          for (int s = 0; s < 32; ++s)
            if (start + slot_elem<VW>(s, lane) == tok) ms->dscal[0] = (double)v[s];
        }
        __syncthreads();
        tok_x = (float)ms->dscal[0];
        __syncthreads();
      }
    }
    if (tid == 0) {
      a.tokens[row] = tok;
      if (a.lse_out) a.lse_out[row] = c;
      if (a.row_lse) a.row_lse[row] = c;
      if (a.tok_logprob) a.tok_logprob[row] = (tok >= 0) ? fsub(tok_x, c) : __int_as_float(0x7fc00000);
      if (mode != kCand && a.n_surv) a.n_surv[row] = 0;
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------------------
// processors / logprobs: per-tile stats pass and a write pass
// --------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) k_process_rows(SampleArgs a, float* out, int64_t out_stride,
                                                           bool want_stats) {
  constexpr int VW = Lay<T>::VW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* wbuf = reinterpret_cast<float*>(smem_raw) + (threadIdx.x >> 5) * kTile;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t total = a.rows * a.n_tiles;
  for (int64_t w = gw; w < total; w += (int64_t)gridDim.x * kWarps) {
    const int64_t row = w / a.n_tiles;
    const int t = (int)(w % a.n_tiles);
    const pm_row_params p = row_params(a, row);
    const int64_t start = (int64_t)t * kTile;
    const int n_valid = (int)((a.vocab - start) < kTile ? (a.vocab - start) : kTile);
    const T* rowp = reinterpret_cast<const T*>(a.logits) + row * a.row_stride;
    float v[32];
    load_tile_raw<T>(rowp, start, n_valid, a.vec_ok, v);
    process_tile<VW>(a, p, row, t, n_valid, v, wbuf);
    if (want_stats) {
      float m;
      uint64_t s;
      tile_stats(v, &m, &s);
      if (lane == 0) { TileStat ts; ts.m = m; ts.pad = 0; ts.s = s; a.statx[row * a.n_tiles + t] = ts; }
    }
    if (out) {
      float* orow = out + row * out_stride + start;
#pragma unroll
      for (int s = 0; s < 32; ++s) {
        const int e = slot_elem<VW>(s, lane);
        if (e < n_valid) orow[e] = v[s];
      }
    }
  }
}

// row log-sum-exp from tile stats: one CTA per row
__global__ void __launch_bounds__(kThreads) k_row_lse(SampleArgs a, float* lse_out) {
  __shared__ double tv[1024];
  __shared__ MiscShared ms;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    float m;
    const float c = block_combine(a.statx + row * a.n_tiles, a.n_tiles, tv, &m, &ms);
    if (threadIdx.x == 0) { if (lse_out) lse_out[row] = c; a.row_lse[row] = c; }
    __syncthreads();
  }
}

// out[r, :] -= lse[r]   (log-softmax write pass)
__global__ void k_sub_lse(float* out, int64_t out_stride, int64_t rows, int64_t vocab, const float* lse) {
  const int64_t n = rows * vocab;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vocab, v = i % vocab;
    float* p = out + r * out_stride + v;
    *p = fsub(*p, lse[r]);
  }
}

}  // namespace pm

// ============================================================================
// host side
// ============================================================================
namespace {

thread_local int g_last_cuda = 0;

int cuda_fail(cudaError_t e) {
  g_last_cuda = (int)e;
  return PM_ERR_CUDA;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Layout {
  int n_tiles = 0, n_chunks = 0, chunk_tiles = 0, KC = 0, ovr_cap = 0;
  size_t row_done = 0, status = 0, statx = 0, staty = 0, cand = 0, cand_n = 0, best = 0, ovr_tok = 0,
         ovr_info = 0, ovr_off = 0, bias_off = 0, row_lse = 0, total = 0;
};

int pow2_at_least(int64_t x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

bool penalties_on(const pm_rows* r) {
  return r->hist && (r->flags_any & (PM_F_REP | PM_F_PRES | PM_F_FREQ));
}

int plan(const pm_rows* r, Layout* L) {
  if (!r || r->rows < 0 || r->vocab <= 0 || r->row_stride < r->vocab) return PM_ERR_ARG;
  if (r->vocab > (int64_t)1024 * pm::kTile) return PM_ERR_UNSUPPORTED;  // tile table bound
  L->n_tiles = (int)((r->vocab + pm::kTile - 1) / pm::kTile);
  int need = r->top_k_max > 0 ? r->top_k_max : 0;
  if (r->flags_any & PM_F_UNBOUNDED) need = need > 256 ? need : 256;
  if (need > 256) return PM_ERR_UNSUPPORTED;
  L->KC = need <= 64 ? 64 : 256;
  // merge keys must fit the staging area: n_chunks * KC <= 4096
  const int max_chunks = 4096 / L->KC;
  L->chunk_tiles = 16;
  while ((L->n_tiles + L->chunk_tiles - 1) / L->chunk_tiles > max_chunks) L->chunk_tiles *= 2;
  L->n_chunks = (L->n_tiles + L->chunk_tiles - 1) / L->chunk_tiles;
  L->ovr_cap = 0;
  if (penalties_on(r)) {
    int64_t w = r->hist_stride + (r->feed ? r->feed_group : 0);
    if (w > 8192) return PM_ERR_UNSUPPORTED;
    L->ovr_cap = pow2_at_least(w < 32 ? 32 : w);
  }
  const int64_t R = r->rows;
  size_t o = 0;
  auto take = [&](size_t bytes) { o = align_up(o, 256); const size_t at = o; o += bytes; return at; };
  L->row_done = take(sizeof(uint32_t) * R);
  L->status = take(sizeof(int32_t) * R);
  L->statx = take(sizeof(pm::TileStat) * R * L->n_tiles);
  L->staty = take(sizeof(pm::TileStat) * R * L->n_tiles);
  L->cand = take(sizeof(uint64_t) * R * L->n_chunks * L->KC);
  L->cand_n = take(sizeof(int32_t) * R * L->n_chunks);
  L->best = take(sizeof(uint64_t) * R * L->n_chunks);
  L->ovr_tok = take(sizeof(int32_t) * R * L->ovr_cap);
  L->ovr_info = take(sizeof(uint32_t) * R * L->ovr_cap);
  L->ovr_off = take(sizeof(int32_t) * R * (L->ovr_cap ? (L->n_tiles + 1) : 0));
  L->bias_off = take(sizeof(int32_t) * (L->n_tiles + 1));
  L->row_lse = take(sizeof(float) * R);
  L->total = align_up(o, 256);
  return PM_OK;
}

int num_sms() {
  static int sms = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  });
  return sms;
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

// prep kernels shared by every entry point; fills a.* processor fields
int launch_prep(const pm_rows* r, const Layout& L, unsigned char* ws, pm::SampleArgs& a, cudaStream_t st) {
  a.logits = r->logits;
  a.rows = r->rows;
  a.vocab = r->vocab;
  a.row_stride = r->row_stride;
  const size_t esz = r->dtype == PM_DTYPE_F32 ? 4 : 2;
  a.vec_ok = ((uintptr_t)r->logits % 16 == 0) && ((r->row_stride * esz) % 16 == 0);
  a.params = r->params;
  a.params_per_row = r->params_per_row;
  a.mask = r->mask;
  a.mask_stride = r->mask_stride;
  a.n_tiles = L.n_tiles;
  a.n_chunks = L.n_chunks;
  a.chunk_tiles = L.chunk_tiles;
  a.n_items = r->rows * (int64_t)L.n_chunks;
  a.statx = reinterpret_cast<pm::TileStat*>(ws + L.statx);
  a.staty = reinterpret_cast<pm::TileStat*>(ws + L.staty);
  a.cand = reinterpret_cast<uint64_t*>(ws + L.cand);
  a.cand_n = reinterpret_cast<int32_t*>(ws + L.cand_n);
  a.best = reinterpret_cast<uint64_t*>(ws + L.best);
  a.row_done = reinterpret_cast<uint32_t*>(ws + L.row_done);
  a.status = reinterpret_cast<int32_t*>(ws + L.status);
  a.row_lse = reinterpret_cast<float*>(ws + L.row_lse);
  a.ovr_tok = nullptr;
  a.ovr_info = nullptr;
  a.ovr_off = nullptr;
  a.ovr_cap = L.ovr_cap;
  a.bias_tok = nullptr;
  a.bias_val = nullptr;
  a.bias_off = nullptr;
  cudaError_t e = cudaMemsetAsync(ws + L.status, 0, sizeof(int32_t) * r->rows, st);
  if (e != cudaSuccess) return cuda_fail(e);
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
    pa.n_tiles = L.n_tiles;
    pa.cap = L.ovr_cap;
    pa.ovr_tok = reinterpret_cast<int32_t*>(ws + L.ovr_tok);
    pa.ovr_info = reinterpret_cast<uint32_t*>(ws + L.ovr_info);
    pa.ovr_off = reinterpret_cast<int32_t*>(ws + L.ovr_off);
    pa.status = a.status;
    const size_t smem = sizeof(uint64_t) * L.ovr_cap + 64 * sizeof(int);
    static std::once_flag once;
    std::call_once(once, [] {
      cudaFuncSetAttribute(pm::k_prep_overrides, cudaFuncAttributeMaxDynamicSharedMemorySize, 8192 * 8 + 256);
    });
    pm::k_prep_overrides<<<(unsigned)r->rows, 1024, smem, st>>>(pa);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    a.ovr_tok = pa.ovr_tok;
    a.ovr_info = pa.ovr_info;
    a.ovr_off = pa.ovr_off;
  }
  if (r->n_bias > 0) {
    // per-tile offsets of the (ascending) shared bias list, computed on the host
    // is not possible without reading device memory; a tiny kernel does it.
    a.bias_tok = r->bias_tokens;
    a.bias_val = r->bias_values;
    a.bias_off = reinterpret_cast<int32_t*>(ws + L.bias_off);
  }
  return PM_OK;
}

}  // namespace

namespace pm {
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

namespace {

int launch_bias(const pm_rows* r, const Layout& L, pm::SampleArgs& a, cudaStream_t st) {
  if (r->n_bias <= 0) return PM_OK;
  pm::k_bias_offsets<<<(L.n_tiles + 256) / 256, 256, 0, st>>>(r->bias_tokens, r->n_bias, L.n_tiles,
                                                              const_cast<int32_t*>(a.bias_off));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

template <typename T, int KC>
int launch_stream(const pm::SampleArgs& a, cudaStream_t st) {
  using SM = pm::Smem<KC, pm::Lay<T>::VW>;
  static std::once_flag once;
  static int occ = 1;
  std::call_once(once, [] {
    cudaFuncSetAttribute(pm::k_sample_stream<T, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::bytes);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, pm::k_sample_stream<T, KC>, pm::kThreads, SM::bytes);
    if (occ < 1) occ = 1;
  });
  if (a.n_items == 0) return PM_OK;
  int64_t grid = (int64_t)num_sms() * occ;
  if (grid > a.n_items) grid = a.n_items;
  pm::k_sample_stream<T, KC><<<(unsigned)grid, pm::kThreads, SM::bytes, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

}  // namespace

extern "C" {

int pm_last_cuda_error(void) { return g_last_cuda; }

const char* pm_version(void) { return "pm_sample 0.1 sm_100a"; }

size_t pm_sample_workspace_bytes(const pm_rows* rows) {
  Layout L;
  if (plan(rows, &L) != PM_OK) return 0;
  return L.total;
}

int pm_sample_rows(const pm_rows* rows, const pm_noise* noise, const pm_sample_out* out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int rc = check_rows(rows);
  if (rc) return rc;
  if (!noise || !out || !out->tokens || !workspace) return PM_ERR_ARG;
  if (noise->mode != PM_NOISE_PHILOX && noise->mode != PM_NOISE_INJECTED) return PM_ERR_ARG;
  if (noise->mode == PM_NOISE_INJECTED) {
    const bool cand = rows->top_k_max > 0 || (rows->flags_any & (PM_F_TOP_P | PM_F_MIN_P));
    if (cand && (!noise->gumbel || noise->gumbel_stride < rows->vocab)) return PM_ERR_ARG;
    if ((rows->flags_any & PM_F_FULL) && !noise->uniform) return PM_ERR_ARG;
  }
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
  rc = launch_bias(rows, L, a, st);
  if (rc) return rc;
  a.noise_mode = noise->mode;
  a.seed = noise->seed;
  a.offset = noise->offset;
  a.row_base = noise->row_base;
  a.gumbel = noise->gumbel;
  a.gumbel_stride = noise->gumbel_stride;
  a.uniform = noise->uniform;
  a.tokens = out->tokens;
  a.lse_out = out->lse;
  a.tok_logprob = out->token_logprob;
  a.surv_ids = out->surv_ids;
  a.surv_probs = out->surv_probs;
  a.n_surv = out->n_surv;
  a.surv_cap = out->surv_cap;
  a.want_lse = out->lse != nullptr || out->token_logprob != nullptr;
  const bool bf = rows->dtype == PM_DTYPE_BF16;
  if (L.KC == 64) rc = bf ? launch_stream<__nv_bfloat16, 64>(a, st) : launch_stream<float, 64>(a, st);
  else rc = bf ? launch_stream<__nv_bfloat16, 256>(a, st) : launch_stream<float, 256>(a, st);
  return rc;
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
  rc = launch_bias(rows, L, a, st);
  if (rc) return rc;
  const size_t smem = pm::kWarps * pm::kTile * 4;
  const int64_t work = rows->rows * (int64_t)L.n_tiles;
  int64_t grid = (work + pm::kWarps - 1) / pm::kWarps;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (grid > cap) grid = cap;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(pm::k_process_rows<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768);
    cudaFuncSetAttribute(pm::k_process_rows<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768);
  });
  if (rows->dtype == PM_DTYPE_BF16)
    pm::k_process_rows<__nv_bfloat16><<<(unsigned)grid, pm::kThreads, smem, st>>>(a, out, out_stride, logprobs);
  else
    pm::k_process_rows<float><<<(unsigned)grid, pm::kThreads, smem, st>>>(a, out, out_stride, logprobs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  if (logprobs) {
    int64_t g2 = rows->rows < (int64_t)num_sms() * 4 ? rows->rows : (int64_t)num_sms() * 4;
    pm::k_row_lse<<<(unsigned)g2, pm::kThreads, 0, st>>>(a, lse_out);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    const int64_t n = rows->rows * rows->vocab;
    int64_t g3 = (n + 255) / 256;
    if (g3 > (int64_t)num_sms() * 16) g3 = (int64_t)num_sms() * 16;
    pm::k_sub_lse<<<(unsigned)g3, 256, 0, st>>>(out, out_stride, rows->rows, rows->vocab, a.row_lse);
    e = cudaGetLastError();
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

}  // extern "C"
