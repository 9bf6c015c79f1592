// pm_lmhead.cu -- the LM head on the tensor cores, with the sampler's tile
// statistics and candidates computed in the GEMM's epilogue.
//
// The reference's decode step produces logits = lm_head(final_norm(h)) for
// every row (pagedmoe/verify_decode.py:821, :824 for a plain step, :887 for a
// verify pass), then runs the processors, the log-sum-exp and the sampler
// over those [rows, vocab] logits (:828-839).  Unfused, the logits make a
// round trip through HBM (written by the GEMM, read back by the sampling
// pass).  Here the GEMM's accumulators never leave the SM: the epilogue
// reads them from tensor memory and writes only what the row merge consumes.
//
// Tile of one CTA: 128 rows (tokens, the MMA's M = TMEM lanes) x 256
// vocabulary ids (N = 256 fp32 TMEM columns) over the whole hidden size,
// bf16 operands staged by TMA (128-byte swizzle, 64 hidden values a stage),
// tcgen05.mma issued by one thread, fp32 accumulation in TMEM.  Four CTAs of
// a cluster cover one 1024-id statistics tile, so the tile's exact
// statistics (max, integer sum of floor(e^(x - max) 2^52)) come out of one
// exchange of row maxima and one of partial sums through distributed shared
// memory -- the same bits as the streaming pass over the written logits.
//
// Epilogue, eight warps: warp w reads TMEM lane quarter w % 4 (32 rows) and
// column half w / 4, so each thread owns one row's 128 consecutive ids (a
// "half slice"), read in chunks of 32 columns:
//   pass A: the mask, the half's maximum, its best key (greedy rows);
//   half maxima -> slice maxima -> cluster exchange -> the tile maximum m;
//   pass B: sum of q52(x - m); cluster exchange; rank 0 writes the tile's
//           statistics;
//   candidates (filtered rows): every finite key of the half when it holds
//           at most KC; otherwise the keys at or above the row's shared
//           threshold (when at most KC), or those within the value bin of
//           the half's K-th largest value (a 64-bin histogram of quarter
//           units below the half's maximum), or, when that bin is too full,
//           exactly the half's top K by a radix select over the keys; the
//           last two raise the row's shared threshold.
// Each half slice is one part of its row for the merge
// (SampleArgs::fixed_parts = 8 x tiles), which then runs unchanged.
//
// No multicast loads: every CTA loads its own operand tiles.  Every wait on
// an mbarrier is bounded; the cluster barriers are reached by every thread
// of every CTA on every path.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "pm_device.cuh"
#include "pm_host.h"
#include "pm_tile.cuh"
#include "pm_tma.cuh"

namespace pm {

constexpr int kLM = 128;        // rows of a CTA tile (MMA M, TMEM lanes)
constexpr int kLN = 256;        // vocabulary ids of a CTA tile (MMA N, TMEM columns)
constexpr int kLK = 64;         // hidden values per stage (128 bytes of bf16: the swizzle span)
constexpr int kLStages = 2;
constexpr int kLThreads = 256;  // eight warps: warp w reads TMEM lane quarter w % 4, column half w / 4
constexpr int kLHalf = kLN / 2;  // columns (ids) of one epilogue thread
constexpr int kLParts = kTile / kLHalf;  // row parts per statistics tile (8)
constexpr int kLCluster = kTile / kLN;  // CTAs per statistics tile (4)
constexpr uint32_t kLABytes = kLM * kLK * 2;    // 16 KB
constexpr uint32_t kLBBytes = kLN * kLK * 2;    // 32 KB
constexpr uint32_t kLStageBytes = kLABytes + kLBBytes;
constexpr int kLBins = 64;       // value histogram of the candidate pass: quarter-unit bins below the maximum
static_assert(kLCluster * kLN == kTile, "a cluster covers one statistics tile");
static_assert(256 * kLThreads <= kLStages * kLStageBytes, "radix histograms (8-bit counts) fit the stage buffers");

// Status bit of a row whose logits were not all finite or -inf (a NaN or +inf
// accumulator): the row's results are not defined.
constexpr int32_t kStatusNonFinite = 128;
// Status bit of a tile pipeline wait that ran out (same as the streaming
// pass's copy timeout).
constexpr int32_t kStatusTimeout = 4;

struct LmShared {
  uint64_t full[kLStages];
  uint64_t empty[kLStages];
  uint64_t done;
  uint32_t tmem;
  int32_t consumed;   // stages the MMA thread consumed (for the drain on a timeout)
  int32_t err;
  float hmax[2][kLM];             // this CTA's half maxima of each row
  float xmax[kLCluster][kLM];     // the cluster's slice maxima of each row
  uint64_t xsum[2 * kLCluster][kLM];  // the cluster's partial sums by (rank, half) (rank 0's copy is read)
};

// ---------------------------------------------------------------------------
// tcgen05 / TMA / cluster primitives
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] x B[smem]^T, bf16 in, fp32 accumulate (kind::f16).
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive fp32 columns back into this thread's TMEM lane (the
// store is complete when this returns).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The shared::cluster address of `p` (this CTA's shared memory) in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void st_cluster_u64(uint32_t addr, uint64_t v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}

// Shared-memory matrix descriptor of a K-major bf16 tile whose rows are 128
// bytes (64 values), 128-byte swizzled as TMA writes it, 8-row groups 1024
// bytes apart; the tile starts on a 1024-byte boundary.  Bits: start address
// >> 4 [0,14), leading byte offset >> 4 [16,30) (unused for this layout),
// stride byte offset >> 4 [32,46), version 1 [46,48), swizzle mode 2
// (128-byte) [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator [4,6) = 1, A and B
// bf16 [7,10) = [10,13) = 1, both K-major, N >> 3 at [17,23), M >> 4 at [24,29).
constexpr uint32_t lm_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kLN >> 3) << 17) | ((uint32_t)(kLM >> 4) << 24);
}

}  // namespace pm

namespace pm {

// The processors' entries of one 32-id chunk (ids c0id ..), in the order of
// the other passes: logit bias, then the row's repetition, presence and
// frequency overrides (the mask comes later, as the chunk is read).
__device__ __forceinline__ void lm_processors(const SampleArgs& a, int64_t row, int64_t c0id, int ob, int oe, int bb,
                                              int be, float (&v)[32]) {
  for (int i = bb; i < be; ++i) {
    const int64_t jj = a.bias_tok[i] - c0id;
    if (jj >= 0 && jj < 32) {
      const float bv = a.bias_val[i];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j == jj) v[j] = fadd(v[j], bv);
    }
  }
  if (oe > ob) {
    const pm_row_params& pp = row_params(a, row);
    const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
    const uint32_t* oinf = a.ovr_info + row * (int64_t)a.ovr_cap;
    for (int i = ob; i < oe; ++i) {
      const int64_t jj = otok[i] - c0id;
      if (jj >= 0 && jj < 32) {
        const uint32_t info = oinf[i];
        float x = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j == jj) x = v[j];
        if (info & 1u) x = x < 0.0f ? fmul(x, pp.repetition_penalty) : __fdiv_rn(x, pp.repetition_penalty);
        if (info & 2u) x = fsub(x, pp.presence_penalty);
        const uint32_t cnt = info >> 8;
        if (cnt) x = fsub(x, fmul(pp.frequency_penalty, (float)cnt));
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j == jj) v[j] = x;
      }
    }
  }
}

// Quarter-unit cells of the value axis: qcell(x) = floor(4 x), exact (4 x is
// exact in fp32), clamped to +-2^22 so that every cell edge c / 4 is an exact
// fp32 value.  x >= c / 4 exactly when qcell(x) >= c (for c > -2^22).  The
// candidate histograms count values by cell below the tile maximum's cell.
constexpr int kCellLim = 1 << 22;
__device__ __forceinline__ int qcell(float x) {
  return (int)floorf(fminf(fmaxf(fmul(x, 4.0f), -(float)kCellLim), (float)kCellLim));
}
__device__ __forceinline__ float cell_edge(int c) { return (float)c * 0.25f; }
__device__ __forceinline__ int cell_bin(float x, int cm) {
  const int b = cm - qcell(x);
  return b < kLBins - 1 ? b : kLBins - 1;
}

struct LmParams {
  int64_t n_tok;         // rows (tokens) of the hidden states
  int64_t vocab;
  int32_t k_slabs;       // stages over the hidden size (ceil(hidden / 64))
  int32_t n_groups;      // row groups of 128
  float* logits;         // plain mode: [n_tok, logits_stride] fp32 out
  int64_t logits_stride;
  // fused mode, zeroed before the launch: each row's histogram of candidate
  // values by quarter-unit cell below its reference cell, and that cell
  // (+ 2^22 + 1; 0: not set yet)
  uint32_t* row_hist;    // [n_tok, 64]
  uint32_t* row_cell;    // [n_tok]
};

// One CTA: rows [g 128, g 128 + 128) x ids [v0, v0 + 256), v0 = tile 1024 +
// rank 256.  Clusters are ordered row group fastest, so the row groups of a
// vocabulary tile run side by side and share its weight rows through L2.
template <bool kFused, int KC>
__global__ void __cluster_dims__(kLCluster, 1, 1) __launch_bounds__(kLThreads, 2)
    k_lmhead(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
             const __grid_constant__ SampleArgs a, const __grid_constant__ LmParams lp) {
  extern __shared__ __align__(1024) unsigned char lm_raw[];
  const uint32_t pad = (1024u - (smem_u32(lm_raw) & 1023u)) & 1023u;
  unsigned char* stages = lm_raw + pad;
  LmShared* sh = reinterpret_cast<LmShared*>(stages + kLStages * kLStageBytes);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const uint32_t rank = cluster_rank();
  const int64_t cl = blockIdx.x / kLCluster;
  const int g = (int)(cl % lp.n_groups);
  const int64_t tile = cl / lp.n_groups;
  const int64_t v0 = tile * kTile + (int64_t)rank * kLN;
  const bool active = v0 < lp.vocab;
  const int ncols = active ? (int)(lp.vocab - v0 < kLN ? lp.vocab - v0 : kLN) : 0;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kLStages; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    mbar_init(&sh->done, 1);
    sh->consumed = 0;
    sh->err = 0;
    fence_proxy_async_smem();
  }
  if (wid == 0) tmem_alloc(&sh->tmem, kLN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem;
  // every CTA of the cluster has started before any distributed shared memory access
  cluster_sync_all();

  // ---- mainloop: TMA producer (warp 0) and MMA issuer (warp 1), one thread each
  int issued = 0;
  int err = 0;
  if (active && wid == 0 && lane == 0) {
    for (int s = 0; s < lp.k_slabs; ++s) {
      const int st = s % kLStages;
      if (s >= kLStages && !mbar_wait(&sh->empty[st], ((s / kLStages) - 1) & 1)) {
        err = 1;
        break;
      }
      unsigned char* sa = stages + st * kLStageBytes;
      mbar_arrive_expect_tx(&sh->full[st], kLStageBytes);
      tma_load_2d(sa, &map_h, s * kLK, g * kLM, &sh->full[st]);
      tma_load_2d(sa + kLABytes, &map_w, s * kLK, (int)v0, &sh->full[st]);
      ++issued;
    }
  } else if (active && wid == 1 && lane == 0) {
    int s = 0;
    for (; s < lp.k_slabs; ++s) {
      const int st = s % kLStages;
      if (!mbar_wait(&sh->full[st], (s / kLStages) & 1)) {
        err = 1;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(stages + st * kLStageBytes);
      const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sa + kLABytes);
#pragma unroll
      for (int k = 0; k < kLK / 16; ++k)  // 16 values (32 bytes) per MMA along the swizzled row
        tc_mma(tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), lm_idesc(), (uint32_t)(s | k));
      tc_commit(&sh->empty[st]);
    }
    sh->consumed = s;
    tc_commit(&sh->done);
  }
  __syncwarp();
  if (active && !mbar_wait(&sh->done, 0)) err = 1;
  tc_fence_after();
  if (err) atomicOr(&sh->err, 1);

  const int quarter = wid & 3, half = wid >> 2;
  const int r_local = quarter * 32 + lane;
  const int64_t row = (int64_t)g * kLM + r_local;
  const bool vrow = row < lp.n_tok;
  const int c0 = half * kLHalf;  // this thread's first column of the CTA tile
  const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
  // columns of this thread's half that hold ids of the vocabulary (uniform over the warp)
  const int hcols = ncols - c0 < 0 ? 0 : (ncols - c0 < kLHalf ? ncols - c0 : kLHalf);
  const int nch = (hcols + 31) >> 5;

  if constexpr (!kFused) {
    // plain logits: each thread writes its row's 128 values, 128 bytes a chunk
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      float v[32];
      tmem_ld32(tl + c * 32, v);
      if (vrow) {
        float* o = lp.logits + row * lp.logits_stride + v0 + c0 + c * 32;
        const int rem = hcols - c * 32;
        if (rem >= 32) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < rem) o[j] = v[j];
        }
      }
    }
    cluster_sync_all();
    cluster_sync_all();
  } else {
    const pm_row_params& p = row_params(a, vrow ? row : 0);
    const int mode = vrow ? row_mode(p) : kGreedy;
    const int part = (int)((tile * kLCluster + rank) * 2 + half);
    const uint32_t id0 = (uint32_t)(v0 + c0);  // id of this thread's column 0
    // chunk c of the row's processed values: ids past the vocabulary and
    // disallowed ids (bit j of the row's mask word (id0 >> 5) + c) are -inf
    const uint32_t* mrow = (a.mask && vrow) ? a.mask + row * a.mask_stride + (id0 >> 5) : nullptr;
    // the processors' entries of this tile: logit bias (shared by the rows)
    // and the row's penalty overrides, applied to the chunk that holds them
    // in the order of the other passes (bias, repetition, presence,
    // frequency, then the mask)
    int ob = 0, oe = 0, bb = 0, be = 0;
    if (a.ovr_off && vrow) {
      ob = a.ovr_off[row * (int64_t)(a.n_tiles + 1) + tile];
      oe = a.ovr_off[row * (int64_t)(a.n_tiles + 1) + tile + 1];
    }
    if (a.bias_off) {
      bb = a.bias_off[tile];
      be = a.bias_off[tile + 1];
    }
    // once per tile, before the passes: the processed values replace the
    // raw ones in TMEM (chunks of warps where some row has an entry)
    {
      const bool has = oe > ob || be > bb;
      if (__any_sync(kFull, has)) {
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          float v[32];
          tmem_ld32(tl + c * 32, v);
          if (has) lm_processors(a, row, (int64_t)id0 + c * 32, ob, oe, bb, be, v);
          tmem_st32(tl + c * 32, v);
        }
      }
    }
    const bool plain = a.mask == nullptr;  // uniform: no mask words to apply
    auto chunk = [&](int c, float (&v)[32]) {
      const uint32_t w = mrow ? __ldg(mrow + c) : 0xFFFFFFFFu;
      tmem_ld32(tl + c * 32, v);
      if (plain && c * 32 + 32 <= hcols) return;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (!((w >> j) & 1u) || c * 32 + j >= hcols) v[j] = -INFINITY;
    };

    // pass A: the half's maximum, finite count, best key
    float mh = -INFINITY;
    uint64_t bk = 0;
    int nfin = 0;
    bool bad = false;
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      float v[32];
      chunk(c, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x = v[j];
        bad |= !(x == x) || x == INFINITY;
        if (x > -INFINITY) {
          ++nfin;
          mh = fmaxf(mh, x);
        }
      }
      if (mode == kGreedy) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const uint64_t k = v[j] > -INFINITY ? rankkey(v[j], id0 + (uint32_t)(c * 32 + j)) : 0ull;
          bk = k > bk ? k : bk;
        }
      }
    }
    // the slice maximum (two halves), then the tile maximum over the cluster
    sh->hmax[half][r_local] = mh;
    __syncthreads();
    if (half == 0) {
      const float ms = fmaxf(sh->hmax[0][r_local], sh->hmax[1][r_local]);
#pragma unroll
      for (uint32_t q = 0; q < (uint32_t)kLCluster; ++q) st_cluster_f32(cluster_addr(&sh->xmax[rank][r_local], q), ms);
    }
    cluster_sync_all();
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < kLCluster; ++q) m = fmaxf(m, sh->xmax[q][r_local]);

    // pass B: integer sum of q52(x - m) over the half and, for filtered
    // rows, a 64-bin histogram of the values by the tile's exact edges
    // e_b = m - (b + 1) / 4 (bin(x) <= b exactly when x >= e_b)
    const bool candrow = vrow && mode == kCand;
    const int K = (p.top_k > 0 && p.top_k < KC) ? p.top_k : KC;
    uint32_t* hist = reinterpret_cast<uint32_t*>(stages);  // [bin / 4][thread], 8-bit counts (<= 128)
    const bool binned = candrow && nfin > KC;
    // values below the row's shared threshold cannot move the tile's bound
    // above it, so only the values at or above it are binned
    float bfloor = INFINITY;
    if (binned) {
      const uint64_t rt = ld_cg(&a.row_tau[row]);
      bfloor = rt ? key_value(rt) : -INFINITY;
    }
    const int cm = m > -INFINITY ? qcell(m) : 0;  // the tile maximum's cell
    if (binned)
      for (int b4 = 0; b4 < kLBins / 4; ++b4) hist[b4 * kLThreads + tid] = 0;
    uint64_t s = 0;
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      float v[32];
      chunk(c, v);
      if (m > -INFINITY) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          uint64_t q0, q1;
          q52x2(fsub(v[j], m), fsub(v[j + 1], m), q0, q1);
          s += q0 + q1;
        }
      }
      if (binned) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (v[j] > -INFINITY && v[j] >= bfloor) {
            const int b = cell_bin(v[j], cm);
            hist[(b >> 2) * kLThreads + tid] += 1u << ((b & 3) * 8);
          }
      }
    }
    // partial sums and histograms to rank 0 ([rank * 2 + half][bin / 4][row]
    // words in its stage buffers past the local histograms)
    st_cluster_u64(cluster_addr(&sh->xsum[rank * 2 + half][r_local], 0), s);
    uint32_t* hx = reinterpret_cast<uint32_t*>(stages + 16384);
    const int hi = (int)rank * 2 + half;
#pragma unroll
    for (int b4 = 0; b4 < kLBins / 4; ++b4)
      st_cluster_u32(cluster_addr(&hx[(hi * (kLBins / 4) + b4) * kLM + r_local], 0), binned ? hist[b4 * kLThreads + tid] : 0u);
    cluster_sync_all();
    // rank 0, per row: the tile's statistics; for filtered rows the tile's
    // histogram (the eight halves summed) goes into the row's global
    // histogram, whose cells are counted from the cell of the first tile that
    // reached the row (so every tile adds by an integer shift); the bound is
    // the higher of two lower edges -- of the first cell where the tile's own
    // count reaches K and of the first where the row's count so far does --
    // as a synthetic key (low bits 0: at least K keys lie at or above it),
    // raised into the row's shared threshold and sent to every CTA of the
    // cluster with its bin in this tile (bl: the halves' count there bounds
    // what they emit)
    uint64_t* tb = reinterpret_cast<uint64_t*>(stages + 16384 + 65536);  // [row]: the bound
    int32_t* bs = reinterpret_cast<int32_t*>(tb + kLM);                   // [row]: its bin in this tile
    if (rank == 0 && half == 0) {
      if (vrow) {
        uint64_t tot = 0;
#pragma unroll
        for (int q = 0; q < 2 * kLCluster; ++q) tot += sh->xsum[q][r_local];
        TileStat t;
        t.m = m;
        t.pad = 0;
        t.s = m > -INFINITY ? tot : 0ull;
        a.statx[row * a.n_tiles + tile] = t;
      }
      uint64_t tkey = 0;
      int bl = kLBins;  // none
      if (candrow && m > -INFINITY) {
        uint32_t* gh = lp.row_hist + row * kLBins;
        unsigned cr = atomicCAS(lp.row_cell + row, 0u, (unsigned)(cm + kCellLim + 1));
        const int cref = cr ? (int)cr - kCellLim - 1 : cm;  // the row's reference cell
        const int shift = cref - cm;                         // tile bin b is row bin b + shift
        int cum = 0, bt = kLBins;
        for (int b4 = 0; b4 < kLBins / 4; ++b4) {
          uint32_t lo = 0, hi2 = 0;  // bins b4*4 + {0, 2} and {1, 3} in 16-bit lanes
#pragma unroll
          for (int q = 0; q < 2 * kLCluster; ++q) {
            const uint32_t w = hx[(q * (kLBins / 4) + b4) * kLM + r_local];
            lo += w & 0x00FF00FFu;
            hi2 += (w >> 8) & 0x00FF00FFu;
          }
          const int cnt4[4] = {(int)(lo & 0xFFFF), (int)(hi2 & 0xFFFF), (int)(lo >> 16), (int)(hi2 >> 16)};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int b = b4 * 4 + e;
            if (b < kLBins - 1 && cnt4[e]) {
              if (bt == kLBins) {
                cum += cnt4[e];
                if (cum >= K) bt = b;
              }
              const int gb = b + shift;
              if (gb < kLBins - 1) atomicAdd(gh + (gb > 0 ? gb : 0), (unsigned)cnt4[e]);
            }
          }
        }
        int bc = bt < kLBins - 1 ? cm - bt : -kCellLim;  // the bound's cell
        int gcum = 0;
        for (int gb = 0; gb < kLBins - 1; ++gb) {
          gcum += (int)ld_cg(gh + gb);
          if (gcum >= K) {
            bc = cref - gb > bc ? cref - gb : bc;
            break;
          }
        }
        if (bc > -kCellLim + 1) {
          tkey = (uint64_t)ordkey(cell_edge(bc)) << 32;
          atomicMax(reinterpret_cast<unsigned long long*>(&a.row_tau[row]), (unsigned long long)tkey);
          bl = cm - bc;  // < 0: no value of this tile reaches it
        }
      }
#pragma unroll
      for (uint32_t q = 0; q < (uint32_t)kLCluster; ++q) {
        st_cluster_u64(cluster_addr(&tb[r_local], q), tkey);
        st_cluster_u32(cluster_addr(&bs[r_local], q), (uint32_t)bl);
      }
    }
    cluster_sync_all();
    if (vrow && mode == kGreedy) a.best[row * a.max_parts + part] = bk;

    // candidates of filtered rows, one list per half slice (a row part): the
    // keys at or above teff = max(bound, row threshold); at most KC of them
    // when every finite key fits, or when the half's count at or above the
    // bound fits; else a threshold the half proves itself -- the row's
    // threshold when the keys above it fit, or exactly the half's top K by a
    // radix select over its keys
    const uint64_t tkey = tb[r_local];
    const int bl = (int)bs[r_local];
    uint64_t teff = 0;
    int path = 0;  // 1 keys >= teff fit; 2 count the keys >= teff first; 4 the half's own top K
    if (candrow) {
      const uint64_t rt = ld_cg(&a.row_tau[row]);
      teff = tkey > rt ? tkey : rt;
      if (nfin <= KC) {
        path = 1;
      } else if (tkey && bl <= kLBins - 2) {
        int le = 0;  // the half's binned values at or above the bound (all it may emit)
        if (bl >= 0) {
          for (int b4 = 0; b4 <= bl / 4; ++b4) {
            const uint32_t w = hist[b4 * kLThreads + tid];
#pragma unroll
            for (int e = 0; e < 4; ++e) le += (b4 * 4 + e <= bl) ? (int)((w >> (8 * e)) & 255u) : 0;
          }
        }
        path = le <= KC ? 1 : (teff > tkey ? 2 : 4);
      } else {
        path = teff ? 2 : 4;
      }
    }
    __syncthreads();  // every thread has read its bin counts before the radix histograms reuse them
    if (__any_sync(kFull, path == 2)) {
      const bool below = path == 2 && ordkey(mh) < (uint32_t)(teff >> 32);
      int over = 0;
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        float v[32];
        chunk(c, v);
        if (path == 2 && !below) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            over += v[j] > -INFINITY && rankkey(v[j], id0 + (uint32_t)(c * 32 + j)) >= teff;
        }
      }
      if (path == 2) path = over <= KC ? 1 : 4;
    }
    uint32_t pre = 0;
    int need = K;
    if (__any_sync(kFull, path == 4)) {
      uint8_t* h8 = reinterpret_cast<uint8_t*>(stages);  // [digit][thread] (the bin histograms are no longer read)
      uint32_t pmask = 0;
#pragma unroll 1
      for (int shf = 24; shf >= 0; shf -= 8) {
        if (path == 4)
          for (int b = 0; b < 256; ++b) h8[b * kLThreads + tid] = 0;
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          float v[32];
          chunk(c, v);
          if (path == 4) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint32_t ok = ordkey(v[j]);
              if (v[j] > -INFINITY && (ok & pmask) == pre) h8[((ok >> shf) & 255u) * kLThreads + tid] += 1;
            }
          }
        }
        if (path == 4) {
          int cum = 0, b = 255;
          for (; b > 0; --b) {
            const int h = h8[b * kLThreads + tid];
            if (cum + h >= need) break;
            cum += h;
          }
          need -= cum;
          pre |= (uint32_t)b << shf;
          pmask |= 0xFFu << shf;
        }
      }
    }
    if (__any_sync(kFull, path != 0)) {
      // path 4 also needs every value at or above its K-th to count ties
      const float tv = (path == 4 || !teff) ? -INFINITY : key_value(teff);
      uint64_t* dst = a.cand + (row * a.max_parts + part) * (int64_t)KC;
      int cnt = 0, ties = 0;
      uint64_t theta = 0;
      // a half whose maximum lies below the threshold's value emits nothing:
      // when no lane of the warp can emit, the sweep is skipped
      const bool idle = path == 0 || !(mh >= tv);
      const int nsweep = __all_sync(kFull, idle) ? 0 : nch;
#pragma unroll 1
      for (int c = 0; c < nsweep; ++c) {
        float v[32];
        chunk(c, v);
        if (path != 0) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const bool fin = v[j] > -INFINITY;
            if (!(fin && v[j] >= tv)) continue;  // below the threshold's value: never taken
            const uint64_t k = rankkey(v[j], id0 + (uint32_t)(c * 32 + j));
            const uint32_t ok = (uint32_t)(k >> 32);
            bool take = k >= teff;
            if (path == 4) {
              const bool tie = fin && ok == pre;
              const bool top = fin && (ok > pre || (tie && ties < need));
              if (tie && top && ++ties == need) theta = k;
              take = take && top;
            }
            if (take && cnt < KC) dst[cnt++] = k;
          }
        }
      }
      if (path != 0) {
        a.cand_n[row * a.max_parts + part] = cnt | (cnt < nfin ? (1 << 30) : 0);
        if (path == 4 && theta > teff)
          atomicMax(reinterpret_cast<unsigned long long*>(&a.row_tau[row]), (unsigned long long)theta);
      }
    }
    if (vrow && bad) atomicOr(&a.status[row], kStatusNonFinite);
  }

  // ---- teardown: a timed-out pipeline first waits (bounded) for its copies
  // in flight, then the TMEM columns are released
  __syncthreads();
  const bool failed = sh->err != 0;
  if (failed && tid == 0 && active) {
    for (int s = sh->consumed; s < issued; ++s) mbar_wait(&sh->full[s % kLStages], (s / kLStages) & 1);
  }
  if (failed && vrow && kFused) atomicOr(&a.status[row], kStatusTimeout);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (wid == 0) tmem_dealloc(tmem, kLN);
}

}  // namespace pm

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

using pmh::cuda_fail;
using pmh::DeviceOnce;
using pmh::num_sms;

// cuTensorMapEncodeTiled, found through the runtime (no link to libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static DeviceOnce once;
  once([&] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

// A 2-D bf16 tensor map over [rows, cols] (cols contiguous, row pitch
// `stride` elements) with boxes of box_rows x 64 values, 128-byte swizzled;
// out-of-range boxes read zeros.
int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t stride, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return PM_ERR_UNSUPPORTED;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  const cuuint32_t box[2] = {(cuuint32_t)pm::kLK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PM_OK : PM_ERR_ARG;
}

int check_lmhead(const pm_lmhead* h, int64_t vocab) {
  if (!h || !h->hidden || !h->weight || h->n_tokens < 0 || h->hidden_size <= 0 || vocab <= 0) return PM_ERR_ARG;
  if (h->hidden_stride < h->hidden_size || h->weight_stride < h->hidden_size) return PM_ERR_ARG;
  // TMA: 16-byte aligned bases and row pitches
  if ((uintptr_t)h->hidden % 16 || (uintptr_t)h->weight % 16 || h->hidden_stride % 8 || h->weight_stride % 8)
    return PM_ERR_ARG;
  if (vocab > (int64_t)1 << 30 || h->n_tokens > (int64_t)1 << 30 || h->hidden_size > (int64_t)1 << 20)
    return PM_ERR_UNSUPPORTED;
  return PM_OK;
}

constexpr size_t lm_smem_bytes() { return pm::kLStages * pm::kLStageBytes + sizeof(pm::LmShared) + 1024; }

template <bool kFused, int KC>
int launch_lmhead(const pm_lmhead* h, int64_t vocab, const pm::SampleArgs& a, const pm::LmParams& lp,
                  cudaStream_t st) {
  CUtensorMap mh, mw;
  int rc = make_map(&mh, h->hidden, h->n_tokens, h->hidden_size, h->hidden_stride, pm::kLM);
  if (rc) return rc;
  rc = make_map(&mw, h->weight, vocab, h->hidden_size, h->weight_stride, pm::kLN);
  if (rc) return rc;
  static DeviceOnce once;
  once([&] {
    cudaFuncSetAttribute(pm::k_lmhead<kFused, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lm_smem_bytes());
  });
  const int64_t n_tiles = (vocab + pm::kTile - 1) / pm::kTile;
  const int64_t grid = n_tiles * lp.n_groups * pm::kLCluster;
  if (grid > 0x7fffffff) return PM_ERR_UNSUPPORTED;
  pm::k_lmhead<kFused, KC><<<(unsigned)grid, pm::kLThreads, lm_smem_bytes(), st>>>(mh, mw, a, lp);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e);
}

pm::LmParams lm_params(const pm_lmhead* h, int64_t vocab) {
  pm::LmParams lp;
  memset(&lp, 0, sizeof(lp));
  lp.n_tok = h->n_tokens;
  lp.vocab = vocab;
  lp.k_slabs = (int32_t)((h->hidden_size + pm::kLK - 1) / pm::kLK);
  lp.n_groups = (int32_t)((h->n_tokens + pm::kLM - 1) / pm::kLM);
  return lp;
}

// Workspace of the fused call.
struct LmLayout {
  int n_tiles = 0, KC = 0, max_parts = 0;
  size_t status = 0, row_tau = 0, row_hist = 0, row_cell = 0, statx = 0, cand = 0, cand_n = 0, best = 0, row_lse = 0,
         prep = 0, total = 0;
};

size_t align256(size_t o) { return (o + 255) & ~(size_t)255; }

int plan_lm(const pm_lmhead* h, const pm_rows* r, LmLayout* L) {
  if (!r || !r->params || r->rows != h->n_tokens || r->vocab <= 0) return PM_ERR_ARG;
  if (r->mask && r->mask_stride < (r->vocab + 31) / 32) return PM_ERR_ARG;
  // the fused pass finishes greedy rows and rows whose filters keep at most
  // top_k <= 256 tokens; processors other than the mask need the history
  // prep, and whole-vocabulary draws or unbounded filters need the row
  if (r->feed || r->forced) return PM_ERR_UNSUPPORTED;
  if (r->flags_any & (PM_F_UNBOUNDED | PM_F_FULL)) return PM_ERR_UNSUPPORTED;
  if (r->hist && r->hist_stride <= 0) return PM_ERR_ARG;
  if (r->n_bias < 0 || (r->n_bias > 0 && (!r->bias_tokens || !r->bias_values))) return PM_ERR_ARG;
  if (r->top_k_max > 256) return PM_ERR_UNSUPPORTED;
  L->n_tiles = (int)((r->vocab + pm::kTile - 1) / pm::kTile);
  if (L->n_tiles > 32 * 8) return PM_ERR_UNSUPPORTED;  // the merge's log-sum-exp tree: 256 tiles at most
  L->KC = r->top_k_max <= 64 ? 64 : 256;
  L->max_parts = L->n_tiles * pm::kLParts;
  const int64_t R = r->rows;
  size_t o = 0;
  auto take = [&](size_t bytes) { o = align256(o); const size_t at = o; o += bytes; return at; };
  L->status = take(sizeof(int32_t) * R);
  L->row_tau = take(sizeof(uint64_t) * R);
  L->row_hist = take(sizeof(uint32_t) * R * pm::kLBins);
  L->row_cell = take(sizeof(uint32_t) * R);
  L->statx = take(sizeof(pm::TileStat) * R * L->n_tiles);
  L->cand = take(sizeof(uint64_t) * R * L->max_parts * L->KC);
  L->cand_n = take(sizeof(int32_t) * R * L->max_parts);
  L->best = take(sizeof(uint64_t) * R * L->max_parts);
  L->row_lse = take(sizeof(float) * R);
  const size_t pb = pm_prep_bytes(r, L->n_tiles);
  if (!pb) return PM_ERR_UNSUPPORTED;  // a penalty window beyond the build's history cap
  L->prep = take(pb);
  L->total = align256(o);
  return PM_OK;
}

}  // namespace

extern "C" {

int pm_lmhead_logits(const pm_lmhead* h, int64_t vocab, float* logits, int64_t logits_stride, void* stream) {
  int rc = check_lmhead(h, vocab);
  if (rc) return rc;
  if (!logits || logits_stride < vocab || logits_stride % 4 || (uintptr_t)logits % 16) return PM_ERR_ARG;
  if (h->n_tokens == 0) return PM_OK;
  pm::SampleArgs a;
  memset(&a, 0, sizeof(a));
  pm::LmParams lp = lm_params(h, vocab);
  lp.logits = logits;
  lp.logits_stride = logits_stride;
  return launch_lmhead<false, 64>(h, vocab, a, lp, reinterpret_cast<cudaStream_t>(stream));
}

size_t pm_lmhead_sample_workspace_bytes(const pm_lmhead* h, const pm_rows* rows) {
  LmLayout L;
  if (!h || plan_lm(h, rows, &L) != PM_OK) return 0;
  return L.total;
}

int pm_lmhead_sample(const pm_lmhead* h, const pm_rows* rows, const pm_noise* noise, const pm_sample_out* out,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (!rows) return PM_ERR_ARG;
  int rc = check_lmhead(h, rows->vocab);
  if (rc) return rc;
  if (!out || !out->tokens || !workspace || !noise) return PM_ERR_ARG;
  if (noise->mode != PM_NOISE_PHILOX && noise->mode != PM_NOISE_INJECTED) return PM_ERR_ARG;
  if (noise->mode == PM_NOISE_INJECTED && rows->top_k_max > 0 &&
      (!noise->gumbel || noise->gumbel_stride < rows->vocab))
    return PM_ERR_ARG;
  if (out->surv_ids && (!out->surv_probs || !out->n_surv || out->surv_cap <= 0)) return PM_ERR_ARG;
  LmLayout L;
  rc = plan_lm(h, rows, &L);
  if (rc) return rc;
  if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
  if (rows->rows == 0) return PM_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  pm::SampleArgs a;
  memset(&a, 0, sizeof(a));
  a.rows = rows->rows;
  a.vocab = rows->vocab;
  a.row_stride = rows->vocab;
  a.params = rows->params;
  a.params_per_row = rows->params_per_row;
  a.mask = rows->mask;
  a.mask_stride = rows->mask_stride;
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
  a.status = reinterpret_cast<int32_t*>(ws + L.status);
  a.row_tau = reinterpret_cast<uint64_t*>(ws + L.row_tau);
  a.statx = reinterpret_cast<pm::TileStat*>(ws + L.statx);
  a.cand = reinterpret_cast<uint64_t*>(ws + L.cand);
  a.cand_n = reinterpret_cast<int32_t*>(ws + L.cand_n);
  a.best = reinterpret_cast<uint64_t*>(ws + L.best);
  a.row_lse = reinterpret_cast<float*>(ws + L.row_lse);
  a.status_live = true;
  a.n_tiles = L.n_tiles;
  a.max_parts = L.max_parts;
  a.fixed_parts = L.max_parts;
  a.n_warps = rows->rows * (int64_t)L.n_tiles;
  // row status, shared thresholds and the rows' candidate histograms start
  // at zero (the plan lays them out one after the other: one memset)
  cudaError_t e = cudaMemsetAsync(ws + L.status, 0, L.statx - L.status, st);
  if (e != cudaSuccess) return cuda_fail(e);
  // the processors' lists: penalty overrides by tile, logit-bias offsets
  rc = pm_prep_launch(rows, L.n_tiles, ws + L.prep, a, st);
  if (rc) return rc;
  pm::LmParams lp = lm_params(h, rows->vocab);
  lp.row_hist = reinterpret_cast<uint32_t*>(ws + L.row_hist);
  lp.row_cell = reinterpret_cast<uint32_t*>(ws + L.row_cell);
  rc = L.KC == 64 ? launch_lmhead<true, 64>(h, rows->vocab, a, lp, st) : launch_lmhead<true, 256>(h, rows->vocab, a, lp, st);
  if (rc) return rc;
  return pm_launch_merges(L.KC, a, st);
}

}  // extern "C"
