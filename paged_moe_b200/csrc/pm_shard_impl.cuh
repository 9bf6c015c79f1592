// pm_shard_impl.cuh -- vocabulary-sharded sampling (included at the end of
// pm_sample.cu: it reuses that file's streaming pass and host planning).
//
// When a tensor-parallel LM head leaves every GPU with a contiguous slice of
// each row's logits, each shard runs the ordinary streaming pass over its
// slice and packs a fixed-size record per row: its best greedy key, its top-K
// candidate keys and its tile statistics (ids made global).  One all-gather
// of the records (NCCL, by the caller) and a merge per row give exactly the
// unsharded result when every shard but the last is a whole number of
// 1024-token tiles: the row's tile list is the shards' lists end to end, the
// top-K of the row is inside the union of the shards' top-K, and a
// whole-vocabulary draw picks a tile by the global tile weights, then takes
// the token that tile's shard already drew inside it with the same uniform.
#pragma once

namespace pm {

// Byte layout of one row's record.
struct ShardLayout {
  int cand_k = 0;     // keys per record
  int nts = 0;        // tiles of a full shard
  bool full = false;  // records carry y statistics and per-tile draws
  size_t keys = 0, xst = 0, yst = 0, ttok = 0, tx = 0, row_bytes = 0;
};

struct ShardK {
  unsigned char* rec;   // this shard's records [rows][row_bytes]
  int64_t row_bytes;
  int64_t keys, xst, yst, ttok, tx;
  int32_t cand_k;
  uint32_t id_base;     // global id of this shard's first token
  bool full;
};

// Pack the streaming pass's per-part results of each row into its record:
// one warp per row, launched after the streaming kernel (programmatic
// dependent launch, like the row merge).
template <typename T, int KC>
__global__ void __launch_bounds__(256) k_shard_pack(const __grid_constant__ SampleArgs a,
                                                    const __grid_constant__ ShardK sk) {
  constexpr int CAP = StreamMem<KC>::CAP;
  struct PackMem {
    uint64_t cand[CAP];
    unsigned hist[256];
  };
  extern __shared__ __align__(128) unsigned char smem_pack[];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  PackMem* pm_ = reinterpret_cast<PackMem*>(smem_pack) + wid;
  const int64_t total = a.rows * a.n_tiles;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + wid; row < a.rows;
       row += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    unsigned char* rec = sk.rec + row * sk.row_bytes;
    const int n_parts = (int)(owner_warp((row + 1) * a.n_tiles - 1, total, a.n_warps) -
                              owner_warp(row * a.n_tiles, total, a.n_warps) + 1);
    const pm_row_params p = row_params(a, row);
    const int mode = row_mode(p);
    uint64_t* keys = reinterpret_cast<uint64_t*>(rec + sk.keys);
    uint64_t best = 0;
    int cnt = 0;
    bool trimmed = false;
    if (mode == kGreedy) {
      for (int i = lane; i < n_parts; i += 32) {
        const uint64_t k = ld_cg(&a.best[row * a.max_parts + i]);
        best = k > best ? k : best;
      }
      best = warp_max_u64(best);
      best -= sk.id_base;  // index word 0xFFFFFFFF - id: the global id is id_base larger
    } else if (mode == kCand) {
      const int K = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;
      Cand cd;
      cand_reset(cd);
      const bool minp = minp_floor_row(p);
      const uint64_t rt = minp ? ld_cg(&a.row_tau[row]) : 0ull;
      for (int part = 0; part < n_parts; ++part) {
        const int raw = ld_cg(&a.cand_n[row * a.max_parts + part]);
        trimmed |= part_trimmed(a, row, part, raw, minp, rt);
        const int n = raw & 0x3fffffff;
        const uint64_t* src = a.cand + (row * a.max_parts + part) * (int64_t)KC;
        for (int i0 = 0; i0 < n; i0 += 32)
          cand_offer_key<CAP>(i0 + lane < n ? ld_cg(&src[i0 + lane]) : 0ull, pm_->cand, pm_->hist, cd, K);
      }
      if (cd.cnt > K) cand_compact<CAP>(pm_->cand, pm_->hist, cd, K);
      trimmed |= cd.trimmed;
      cnt = cd.cnt;
      for (int i = lane; i < sk.cand_k; i += 32) keys[i] = i < cnt ? pm_->cand[i] - sk.id_base : 0ull;
    }
    // tile statistics (the row's x statistics were written by the streaming pass when its filters or the
    // caller need them; y statistics for whole-vocabulary draws)
    TileStat* xs = reinterpret_cast<TileStat*>(rec + sk.xst);
    for (int t = lane; t < a.n_tiles; t += 32) {
      TileStat st;
      st.m = -INFINITY;
      st.pad = 0;
      st.s = 0;
      if (needs_xstats(a, p, mode)) st = a.statx[row * a.n_tiles + t];
      xs[t] = st;
    }
    if (sk.full) {
      TileStat* ys = reinterpret_cast<TileStat*>(rec + sk.yst);
      for (int t = lane; t < a.n_tiles; t += 32) {
        TileStat st;
        st.m = -INFINITY;
        st.pad = 0;
        st.s = 0;
        if (mode == kFullDraw) st = a.staty[row * a.n_tiles + t];
        ys[t] = st;
      }
    }
    if (lane == 0) {
      *reinterpret_cast<uint64_t*>(rec) = best;
      *reinterpret_cast<uint32_t*>(rec + 8) = (uint32_t)cnt | (trimmed ? 0x80000000u : 0u);
      *reinterpret_cast<uint32_t*>(rec + 12) = 0u;
    }
    __syncwarp();
  }
}

// Per-tile draws of the whole-vocabulary rows: for every tile of the shard,
// the token the tile would give to the row's second uniform (the first
// token whose inclusive prefix of q52(y - m_t) exceeds floor(u2 s_t)), and
// its processed logit.  One warp per (row, tile).
template <typename T>
__global__ void __launch_bounds__(256) k_shard_tiles(const __grid_constant__ SampleArgs a,
                                                     const __grid_constant__ ShardK sk) {
  constexpr int VW = Lay<T>::VW;
  const int lane = threadIdx.x & 31;
  const int64_t total = a.rows * a.n_tiles;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
       w += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t row = w / a.n_tiles;
    const int t = (int)(w % a.n_tiles);
    const pm_row_params p = row_params(a, row);
    if (row_mode(p) != kFullDraw) continue;
    unsigned char* rec = sk.rec + row * sk.row_bytes;
    const TileStat st = a.staty[row * a.n_tiles + t];
    int tok = t * kTile;
    float tx = -INFINITY;
    if (st.s) {
      const uint64_t t2 = scale_u53(row_u53(a, row, 1), st.s);
      TileIn ti;
      load_tile<T>(a, row, t, ti);
      process_tile_regs<VW>(a, p, row, t, ti);
      const int n_valid = tile_valid(a, t);
      uint64_t acc = 0;
      for (int j = 0; j < 32 / VW; ++j) {
        uint64_t q[VW];
        uint64_t ls = 0;
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          const int e = j * 32 * VW + lane * VW + c;
          const float x = ti.v[j * VW + c];
          const float y = (e < n_valid && x > -INFINITY) ? fmul(x, p.inv_temperature) : -INFINITY;
          q[c] = q52(fsub(y, st.m));
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
          tok = t * kTile + j * 32 * VW + src * VW + found;
          break;
        }
        acc = __shfl_sync(kFull, incl, 31);
      }
    }
    if (lane == 0) {
      reinterpret_cast<int32_t*>(rec + sk.ttok)[t] = tok + (int32_t)sk.id_base;
      reinterpret_cast<float*>(rec + sk.tx)[t] = tx;
    }
  }
}

struct MergeK {
  const unsigned char* recs;  // [n_shards][rows][row_bytes]
  int64_t shard_bytes;        // rows * row_bytes
  int64_t row_bytes;
  int64_t keys, xst, yst, ttok, tx;
  int32_t n_shards;
  int32_t nts;                // tiles of a full shard
  int32_t nt;                 // tiles of the whole row
  int32_t cand_k;
};

__device__ __forceinline__ const TileStat* merge_tile(const MergeK& m, int64_t row, int t, int64_t off) {
  const int s = min(t / m.nts, m.n_shards - 1);
  const int tl = t - s * m.nts;
  return reinterpret_cast<const TileStat*>(m.recs + s * m.shard_bytes + row * m.row_bytes + off) + tl;
}

__device__ __forceinline__ void merge_lane_tiles(const MergeK& m, int64_t row, int64_t off, LaneTiles& lt) {
  const int lane = threadIdx.x & 31;
  int P = 32;
  while (P < m.nt) P <<= 1;
  lt.per = P >> 5;
  lt.nt = m.nt;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int t = lane * lt.per + i;
    const bool ok = i < lt.per && t < m.nt;
    lt.m[i] = -INFINITY;
    lt.s[i] = 0;
    if (ok) {
      const TileStat* st = merge_tile(m, row, t, off);
      lt.m[i] = ld_cg(&st->m);
      lt.s[i] = ld_cg(&st->s);
    }
  }
}

// The merge: one CTA per row over the gathered records of every shard.
// Filtered rows: every shard's keys copied into shared memory by the whole
// CTA and one block radix select of the row's top K (sorted); warp 0 then
// computes the log-sum-exp and filters and draws as for the other modes.
template <int KC>
__global__ void __launch_bounds__(256) k_shard_merge(const __grid_constant__ SampleArgs a,
                                                     const __grid_constant__ MergeK m) {
  extern __shared__ __align__(128) unsigned char smem_smerge[];
  uint64_t* U = reinterpret_cast<uint64_t*>(smem_smerge);   // [n_shards * cand_k] gathered keys
  uint64_t* carry = U + (int64_t)m.n_shards * m.cand_k;     // [KC] the row's top K, sorted
  unsigned* mhist = reinterpret_cast<unsigned*>(carry + KC);  // [256]
  int* scal = reinterpret_cast<int*>(mhist + 256);          // [8]
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const pm_row_params p = row_params(a, row);
    const int mode = row_mode(p);
    int ncarry = 0;
    bool trimmed = false;
    // warp 0: the row's log-sum-exp from the shards' tile statistics, while
    // warps 1..7 gather the shards' keys
    float c = __int_as_float(0x7fc00000);
    if (wid == 0) {
      if (needs_xstats(a, p, mode)) {
        LaneTiles lt;
        merge_lane_tiles(m, row, m.xst, lt);
        c = combine_lane_tiles(lt, lane_tiles_max(lt));
      }
    }
    if (mode == kCand) {
      const int K = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;
      int off = 0;
      for (int s = 0; s < m.n_shards; ++s) {
        const unsigned char* rec = m.recs + s * m.shard_bytes + row * m.row_bytes;
        const uint32_t hdr = ld_cg(reinterpret_cast<const uint32_t*>(rec + 8));
        trimmed |= (hdr >> 31) != 0;
        const int n = (int)(hdr & 0x7fffffffu);
        const uint64_t* keys = reinterpret_cast<const uint64_t*>(rec + m.keys);
        if (wid > 0)
          for (int i = tid - 32; i < n; i += blockDim.x - 32) U[off + i] = ld_cg(&keys[i]);
        off += n;
      }
      __syncthreads();
      ncarry = block_topk_sorted(U, off, K, carry, KC, mhist, scal);
      trimmed = trimmed || off > K;
      __syncthreads();
    }
    if (wid == 0) {
      int tok = 0, ns = 0;
      float x_tok = -INFINITY;
      if (mode == kGreedy) {
        uint64_t b = 0;
        for (int s = lane; s < m.n_shards; s += 32) {
          const uint64_t k = ld_cg(reinterpret_cast<const uint64_t*>(m.recs + s * m.shard_bytes + row * m.row_bytes));
          b = k > b ? k : b;
        }
        b = warp_max_u64(b);
        tok = (int)key_index(b);
        x_tok = key_value(b);
      } else if (mode == kCand) {
        tok = warp_filter_draw(a, p, row, carry, ncarry, !trimmed, c, &ns);
        if (tok >= 0) {
          float fx = -INFINITY;
          for (int r = lane; r < ncarry; r += 32)
            if ((int)key_index(carry[r]) == tok) fx = key_value(carry[r]);
          x_tok = warp_max(fx);
          if (a.surv_ids && lane == 0) write_survivors(a, p, row, carry, ns);
        }
      } else {
        // tile by the first uniform over the global tile weights, token from
        // the tile's own draw
        LaneTiles lt;
        merge_lane_tiles(m, row, m.yst, lt);
        const float my = lane_tiles_max(lt);
        if (my > -INFINITY) {
          int sh = 1;
          while ((1 << (sh - 1)) < m.nt) ++sh;
          const double scale = __longlong_as_double((long long)(1023 - sh) << 52);  // 2^-sh
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
          int tt = m.nt - 1;
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
          if (tt >= m.nt) tt = m.nt - 1;
          const int s = min(tt / m.nts, m.n_shards - 1);
          const int tl = tt - s * m.nts;
          const unsigned char* rec = m.recs + s * m.shard_bytes + row * m.row_bytes;
          tok = ld_cg(reinterpret_cast<const int32_t*>(rec + m.ttok) + tl);
          x_tok = ld_cg(reinterpret_cast<const float*>(rec + m.tx) + tl);
        }
      }
      if (lane == 0) {
        a.status[row] = tok < 0 ? 1 : 0;
        a.tokens[row] = tok;
        if (a.lse_out) a.lse_out[row] = c;
        if (a.tok_logprob) a.tok_logprob[row] = tok >= 0 ? fsub(x_tok, c) : __int_as_float(0x7fc00000);
        if (a.n_surv && (mode != kCand || !a.surv_ids)) a.n_surv[row] = mode == kCand ? ns : 0;
      }
      __syncwarp();
    }
    __syncthreads();
  }
}

}  // namespace pm
