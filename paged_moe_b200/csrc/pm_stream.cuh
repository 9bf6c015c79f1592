// pm_stream.cuh -- the warp's view of its streamed tiles in shared memory.
//
// Each warp owns a ring of kStages tile buffers.  Lane 0 fills a buffer with
// one bulk copy (TMA) of the tile's logits plus one of its 128-byte slice of
// the allowed-token bitmask, both completing on the buffer's mbarrier; the
// warp then reads the tile from shared memory in compact loops, so the next
// tiles are always in flight while the current one is processed.
//
// Element layout inside a tile buffer is the natural one (token t of the tile
// at index t).  A lane reads 16 bytes per step: VW = 4 fp32 or 8 bf16 values,
// tokens j*32*VW + lane*VW + c, c < VW.
#pragma once

#include "pm_device.cuh"
#include "pm_tile.cuh"
#include "pm_tma.cuh"

namespace pm {

constexpr int kStages = 2;

// Per-warp shared memory of the streaming kernels.
template <int KC>
struct alignas(128) StreamMem {
  // KC kept + room for the pushes between compactions (every 128 keys past
  // K); with two stages a 4-warp CTA of KC = 64 takes 52 KB, four per SM
  static constexpr int CAP = KC + 384;
  float tile[kStages][kTile];           // fp32 tile, or a bf16 tile in the first half
  uint32_t mask[kStages][32];
  uint64_t bar[kStages];
  uint64_t cand[CAP];
  unsigned hist[256];
};

template <typename T> struct Vec;
template <> struct Vec<float> { static constexpr int VW = 4; };
template <> struct Vec<__nv_bfloat16> { static constexpr int VW = 8; };

// VW values of step j of this lane from a tile buffer holding elements of type T.
template <typename T>
__device__ __forceinline__ void read_step(const float* buf, int j, int lane, float (&x)[Vec<T>::VW]) {
  if constexpr (sizeof(T) == 4) {
    const float4 q = reinterpret_cast<const float4*>(buf)[j * 32 + lane];
    x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
  } else {
    const uint4 q = reinterpret_cast<const uint4*>(buf)[j * 32 + lane];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      x[2 * h] = bf16_bits_to_f32(w[h] & 0xffffu);
      x[2 * h + 1] = bf16_bits_to_f32(w[h] >> 16);
    }
  }
}

template <typename T>
__device__ __forceinline__ float read_elem(const float* buf, int e) {
  if constexpr (sizeof(T) == 4) return buf[e];
  else return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(buf)[e]);
}

// This lane's 32-slot allowed mask (slot s = j*VW + c) from the tile's 32 mask words.
template <int VW>
__device__ __forceinline__ uint32_t slot_mask(const uint32_t* mw_smem) {
  const int lane = threadIdx.x & 31;
  const uint32_t mw = mw_smem[lane];
  uint32_t sm = 0;
#pragma unroll
  for (int j = 0; j < 32 / VW; ++j) {
    const uint32_t w = __shfl_sync(kFull, mw, j * VW + (lane * VW) / 32);
    const uint32_t bits = (w >> ((lane * VW) & 31)) & ((1u << VW) - 1u);
    sm |= bits << (j * VW);
  }
  return sm;
}

template <int VW>
__device__ __forceinline__ int slot_to_elem(int s, int lane) {
  return (s / VW) * (32 * VW) + lane * VW + (s % VW);
}

// Convert a bf16 tile (first 2 KB of buf) to fp32 in place, top chunk first
// so no value is overwritten before it has been read.
__device__ __forceinline__ void expand_bf16_in_place(float* buf) {
  const int lane = threadIdx.x & 31;
  const uint16_t* h = reinterpret_cast<const uint16_t*>(buf);
  for (int base = kTile - 256; base >= 0; base -= 256) {
    float x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = bf16_bits_to_f32(h[base + k * 32 + lane]);
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; ++k) buf[base + k * 32 + lane] = x[k];
    __syncwarp();
  }
}

// Logit bias and penalties of a tile, in place on its fp32 buffer.
__device__ __forceinline__ void apply_overrides_smem(const SampleArgs& a, const pm_row_params& p, int64_t row,
                                                     int tile, int ob, int oe, int bb, int be, float* buf) {
  const int lane = threadIdx.x & 31;
  const int64_t start = (int64_t)tile * kTile;
  for (int i = bb + lane; i < be; i += 32) {
    const int64_t e = a.bias_tok[i] - start;
    if (e >= 0 && e < kTile) buf[e] = fadd(buf[e], a.bias_val[i]);  // ids out of ascending order: skipped
  }
  __syncwarp();
  const int32_t* otok = a.ovr_tok + row * (int64_t)a.ovr_cap;
  const uint32_t* oinf = a.ovr_info + row * (int64_t)a.ovr_cap;
  for (int i = ob + lane; i < oe; i += 32) {
    const int e = (int)(otok[i] - start);
    const uint32_t info = oinf[i];
    float x = buf[e];
    if (info & 1u) x = x < 0.0f ? fmul(x, p.repetition_penalty) : __fdiv_rn(x, p.repetition_penalty);
    if (info & 2u) x = fsub(x, p.presence_penalty);
    const uint32_t cnt = info >> 8;
    if (cnt) x = fsub(x, fmul(p.frequency_penalty, (float)cnt));
    buf[e] = x;
  }
  __syncwarp();
}

}  // namespace pm
