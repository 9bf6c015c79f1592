// pm_select.cuh -- top-K selection over 64-bit rank keys in shared memory.
//
// Keys are unique (the low word carries the token id), so "the K largest
// keys" is a well-defined set.  Selection is an MSD radix select with 8-bit
// digits over shared-memory histograms: each pass histograms the keys that
// match the digits fixed so far, a warp scans the 256 bins from the top to
// find the digit holding the K-th key, and the search stops as soon as that
// bin is taken whole.  The survivors are then sorted by a bitonic network.
#pragma once

#include "pm_device.cuh"

namespace pm {

// Digit search over a 256-bin histogram by one full warp: the digit d with
// (keys in bins above d) < need <= (keys in bins >= d).  Returns d; *above
// receives the count in bins above d, *in_bin the count in bin d.
__device__ __forceinline__ int warp_find_digit(const unsigned* hist, int need, int* above, int* in_bin) {
  const int lane = threadIdx.x & 31;
  unsigned c[8];
  unsigned tot = 0;
#pragma unroll
  for (int b = 0; b < 8; ++b) { c[b] = hist[lane * 8 + b]; tot += c[b]; }
  unsigned incl = tot;  // suffix-inclusive over lanes >= lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_down_sync(kFull, incl, o);
    if (lane + o < 32) incl += t;
  }
  unsigned run = incl - tot;  // keys in bins of higher lanes
  int found = -1, fa = 0, fb = 0;
#pragma unroll
  for (int b = 7; b >= 0; --b) {
    if (found < 0 && (int)run < need && need <= (int)(run + c[b])) { found = lane * 8 + b; fa = (int)run; fb = (int)c[b]; }
    run += c[b];
  }
  const unsigned bal = __ballot_sync(kFull, found >= 0);
  const int src = bal ? __ffs(bal) - 1 : 0;
  const int d = __shfl_sync(kFull, found, src);
  *above = __shfl_sync(kFull, fa, src);
  *in_bin = __shfl_sync(kFull, fb, src);
  return d;
}

// Warp-level: compact buf[0..cnt) to its K largest keys (in any order) and
// return the smallest kept key.  Requires cnt > K >= 1.  hist: 256 words of
// this warp's shared memory.  Every lane gets the result.
template <int MAXPER>
__device__ uint64_t warp_select_topk(uint64_t* buf, int cnt, int K, unsigned* hist) {
  const int lane = threadIdx.x & 31;
  // Skip the leading bits every key shares: the first digit starts at the
  // highest bit where the smallest and largest key differ, so the first
  // histogram spreads over the bins instead of piling into one.
  uint64_t kmin = ~0ull, kmax = 0ull;
  for (int i = lane; i < cnt; i += 32) {
    const uint64_t k = buf[i];
    kmin = k < kmin ? k : kmin;
    kmax = k > kmax ? k : kmax;
  }
  kmin = warp_min_u64(kmin);
  kmax = warp_max_u64(kmax);
  // bits at and above `hi` are common to every key still in play
  int hi = 64 - __clzll(kmin ^ kmax);  // keys are unique, so kmin != kmax
  uint64_t prefix = hi >= 64 ? 0ull : (kmax >> hi) << hi;
  int need = K;
  for (;;) {
    const int w = hi < 8 ? hi : 8;
    const int shift = hi - w;
    for (int i = lane; i < 256; i += 32) hist[i] = 0;
    __syncwarp();
    for (int i = lane; i < cnt; i += 32) {
      const uint64_t k = buf[i];
      const bool match = hi >= 64 || ((k ^ prefix) >> hi) == 0;
      if (match) atomicAdd(&hist[(k >> shift) & ((1u << w) - 1u)], 1u);
    }
    __syncwarp();
    int above, in_bin;
    const int d = warp_find_digit(hist, need, &above, &in_bin);
    __syncwarp();
    need -= above;
    prefix |= (uint64_t)d << shift;
    if (in_bin == need || shift == 0) break;
    hi = shift;
  }
  // keep keys >= prefix (low bits of prefix below `shift` are zero), in
  // place: a round's keys are read before any of its writes, and the writes
  // land below the next round's keys
  uint64_t kept_min = ~0ull;
  int base = 0;
  for (int r0 = 0; r0 < cnt; r0 += 32) {
    const int i = r0 + lane;
    const uint64_t k = i < cnt ? buf[i] : 0ull;
    const bool keep = i < cnt && k >= prefix;
    const unsigned bal = __ballot_sync(kFull, keep);
    if (keep) {
      buf[base + __popc(bal & ((1u << lane) - 1u))] = k;
      kept_min = k < kept_min ? k : kept_min;
    }
    base += __popc(bal);
    __syncwarp();
  }
  return warp_min_u64(kept_min);
}

// Block-level: the K largest of U[0..n) sorted descending into S[0..m),
// m = min(n, K), returned to every thread.  U may be clobbered.  hist is a
// 256-word shared array, scal 4 shared ints.  Call with all threads.
__device__ inline int block_topk_sorted(uint64_t* U, int n, int K, uint64_t* S, int S_cap, unsigned* hist,
                                 int* scal) {
  const int tid = threadIdx.x, nth = blockDim.x;
  int m;
  if (n <= K) {
    for (int i = tid; i < n; i += nth) S[i] = U[i];
    m = n;
  } else {
    uint64_t prefix = 0;
    int need = K;
    int shift = 56;
    for (;;) {
      for (int i = tid; i < 256; i += nth) hist[i] = 0;
      __syncthreads();
      for (int i = tid; i < n; i += nth) {
        const uint64_t k = U[i];
        const bool match = (shift == 56) || (((k ^ prefix) >> (shift + 8)) == 0);
        if (match) atomicAdd(&hist[(k >> shift) & 255], 1u);
      }
      __syncthreads();
      if (tid < 32) {
        int above, in_bin;
        const int d = warp_find_digit(hist, need, &above, &in_bin);
        if (tid == 0) { scal[0] = d; scal[1] = above; scal[2] = in_bin; }
      }
      __syncthreads();
      const int d = scal[0], above = scal[1], in_bin = scal[2];
      __syncthreads();
      need -= above;
      prefix |= (uint64_t)d << shift;
      if (in_bin == need || shift == 0) break;
      shift -= 8;
    }
    if (tid == 0) scal[3] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += nth) {
      const uint64_t k = U[i];
      if (k >= prefix) S[atomicAdd(&scal[3], 1)] = k;
    }
    __syncthreads();
    m = K;
  }
  // bitonic sort S[0..P) descending, P = next power of two >= m
  int P = 1;
  while (P < m) P <<= 1;
  if (P > S_cap) P = S_cap;  // callers size S_cap to a power of two >= K
  for (int i = m + tid; i < P; i += nth) S[i] = 0ull;
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < P; i += nth) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = S[i], b = S[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) { S[i] = b; S[ixj] = a; }
        }
      }
      __syncthreads();
    }
  }
  return m;
}

}  // namespace pm
