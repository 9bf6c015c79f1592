// pm_device.cuh -- device-side building blocks of the token-selection kernels.
//
// Everything here is deterministic: the same inputs give the same bits on
// every run and every launch configuration.  The elementary functions are
// this project's own (Cody & Waite 1980 range reduction with Taylor / atanh
// series, explicit fused multiply-adds only); every other floating-point
// operation is written with a rounding intrinsic so the compiler cannot fuse
// or reorder it.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace pm {

constexpr int kTile = 1024;       // tokens per statistics tile
constexpr int kWarps = 8;         // warps per CTA of the streaming kernels
constexpr int kThreads = kWarps * 32;
constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// fp32 / fp64 arithmetic that the compiler may not contract
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dfma(double a, double b, double c) { return __fma_rn(a, b, c); }

// e^d in fp32 for d <= ~0: d = k ln2 + r (ln2 as a 16-bit head plus tail),
// degree-7 Taylor polynomial of e^r, exact scaling by 2^k.  d < -87 or NaN -> 0.
__device__ __forceinline__ float det_expf(float d) {
  if (!(d >= -87.0f)) return 0.0f;
  const float t = fmul(d, 0x1.715476p+0f);
  const float kf = fsub(fadd(t, 12582912.0f), 12582912.0f);
  float r = ffma(-kf, 0x1.62e4p-1f, d);
  r = ffma(-kf, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = ffma(p, r, 0x1.6c16c2p-10f);
  p = ffma(p, r, 0x1.111112p-7f);
  p = ffma(p, r, 0x1.555556p-5f);
  p = ffma(p, r, 0x1.555556p-3f);
  p = ffma(p, r, 0x1.0p-1f);
  p = ffma(p, r, 1.0f);
  p = ffma(p, r, 1.0f);
  // p in [0.70, 1.42] and k in [-126, 0]: scale through the exponent field.
  const int k = (int)kf;
  return __int_as_float(__float_as_int(p) + (k << 23));
}

// floor(e * 2^52) of a positive normal fp32 e below 2^7, from its bits:
// adding 52 to the exponent field gives e * 2^52 exactly (a float below 2^59),
// and the truncating conversion to a 64-bit integer is then exact.
__device__ __forceinline__ uint64_t q52_from_bits(uint32_t be) {
  return __float2ull_rz(__uint_as_float(be + (52u << 23)));
}

// floor(e^d * 2^52) with e^d = det_expf(d); 0 for d < -38, -inf or NaN.
// Clamping d to -38 gives the same value as cutting there: det_expf(-38)
// * 2^52 < 1.  Branch-free, and the conversion is an exact integer shift.
__device__ __forceinline__ uint64_t q52(float d) {
  d = fmaxf(d, -38.0f);  // NaN -> -38
  const float t = fmul(d, 0x1.715476p+0f);
  const float tm = fadd(t, 12582912.0f);
  const float kf = fsub(tm, 12582912.0f);
  float r = ffma(-kf, 0x1.62e4p-1f, d);
  r = ffma(-kf, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = ffma(p, r, 0x1.6c16c2p-10f);
  p = ffma(p, r, 0x1.111112p-7f);
  p = ffma(p, r, 0x1.555556p-5f);
  p = ffma(p, r, 0x1.555556p-3f);
  p = ffma(p, r, 0x1.0p-1f);
  p = ffma(p, r, 1.0f);
  p = ffma(p, r, 1.0f);
  const int k = (int)(__float_as_uint(tm) - 0x4B400000u);  // tm = 1.5 * 2^23 + k exactly
  return q52_from_bits(__float_as_uint(p) + ((uint32_t)k << 23));
}

// Packed pairs of fp32 (Blackwell f32x2 arithmetic): each half is an
// independent IEEE fp32 operation with round-to-nearest.
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// fl32(log2 e): the multiplier of every base-2 exponent argument here.
constexpr float kLog2eF = 0x1.715476p+0f;

// The hardware 2^a (MUFU ex2, flush-to-zero).  Its bits are not specified,
// so it serves only the bracketed statistics, whose error budget covers it
// (relative error 2^-20; the GPU tests measure it).
__device__ __forceinline__ float ex2_approx(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// q52 of two values at once; bit-identical to two q52 calls.
__device__ __forceinline__ void q52x2(float d0, float d1, uint64_t& q0, uint64_t& q1) {
  const uint64_t D = pk(fmaxf(d0, -38.0f), fmaxf(d1, -38.0f));
  const uint64_t T = mul2(D, pk(0x1.715476p+0f, 0x1.715476p+0f));
  const uint64_t TM = add2(T, pk(12582912.0f, 12582912.0f));
  const uint64_t KF = add2(TM, pk(-12582912.0f, -12582912.0f));
  uint64_t R = fma2(KF, pk(-0x1.62e4p-1f, -0x1.62e4p-1f), D);
  R = fma2(KF, pk(-0x1.7f7d1cp-20f, -0x1.7f7d1cp-20f), R);
  uint64_t P = pk(0x1.a01a02p-13f, 0x1.a01a02p-13f);
  P = fma2(P, R, pk(0x1.6c16c2p-10f, 0x1.6c16c2p-10f));
  P = fma2(P, R, pk(0x1.111112p-7f, 0x1.111112p-7f));
  P = fma2(P, R, pk(0x1.555556p-5f, 0x1.555556p-5f));
  P = fma2(P, R, pk(0x1.555556p-3f, 0x1.555556p-3f));
  P = fma2(P, R, pk(0x1.0p-1f, 0x1.0p-1f));
  P = fma2(P, R, pk(1.0f, 1.0f));
  P = fma2(P, R, pk(1.0f, 1.0f));
  const uint32_t k0 = (uint32_t)TM - 0x4B400000u, k1 = (uint32_t)(TM >> 32) - 0x4B400000u;
  q0 = q52_from_bits((uint32_t)P + (k0 << 23));
  q1 = q52_from_bits((uint32_t)(P >> 32) + (k1 << 23));
}

// det_expf of two values at once (packed f32x2: each half is the same IEEE
// fp32 sequence as det_expf); bit-identical to two det_expf calls.
__device__ __forceinline__ void det_expf_x2(float d0, float d1, float& e0, float& e1) {
  const bool z0 = !(d0 >= -87.0f), z1 = !(d1 >= -87.0f);
  const uint64_t D = pk(z0 ? 0.0f : d0, z1 ? 0.0f : d1);
  const uint64_t T = mul2(D, pk(0x1.715476p+0f, 0x1.715476p+0f));
  const uint64_t TM = add2(T, pk(12582912.0f, 12582912.0f));
  const uint64_t KF = add2(TM, pk(-12582912.0f, -12582912.0f));
  uint64_t R = fma2(KF, pk(-0x1.62e4p-1f, -0x1.62e4p-1f), D);
  R = fma2(KF, pk(-0x1.7f7d1cp-20f, -0x1.7f7d1cp-20f), R);
  uint64_t P = pk(0x1.a01a02p-13f, 0x1.a01a02p-13f);
  P = fma2(P, R, pk(0x1.6c16c2p-10f, 0x1.6c16c2p-10f));
  P = fma2(P, R, pk(0x1.111112p-7f, 0x1.111112p-7f));
  P = fma2(P, R, pk(0x1.555556p-5f, 0x1.555556p-5f));
  P = fma2(P, R, pk(0x1.555556p-3f, 0x1.555556p-3f));
  P = fma2(P, R, pk(0x1.0p-1f, 0x1.0p-1f));
  P = fma2(P, R, pk(1.0f, 1.0f));
  P = fma2(P, R, pk(1.0f, 1.0f));
  const uint32_t k0 = (uint32_t)TM - 0x4B400000u, k1 = (uint32_t)(TM >> 32) - 0x4B400000u;
  e0 = z0 ? 0.0f : __uint_as_float((uint32_t)P + (k0 << 23));
  e1 = z1 ? 0.0f : __uint_as_float((uint32_t)(P >> 32) + (k1 << 23));
}

// e^d in fp64 for d <= ~0; d < -700 or NaN -> 0.
__device__ __forceinline__ double det_exp64(double d) {
  if (!(d >= -700.0)) return 0.0;
  const double kd = rint(dmul(d, 0x1.71547652b82fep+0));
  double r = dfma(-kd, 0x1.62e42fefa3800p-1, d);
  r = dfma(-kd, 0x1.ef35793c76730p-45, r);
  double p = 0x1.6124613a86d09p-33;
  p = dfma(p, r, 0x1.1eed8eff8d898p-29);
  p = dfma(p, r, 0x1.ae64567f544e4p-26);
  p = dfma(p, r, 0x1.27e4fb7789f5cp-22);
  p = dfma(p, r, 0x1.71de3a556c734p-19);
  p = dfma(p, r, 0x1.a01a01a01a01ap-16);
  p = dfma(p, r, 0x1.a01a01a01a01ap-13);
  p = dfma(p, r, 0x1.6c16c16c16c17p-10);
  p = dfma(p, r, 0x1.1111111111111p-7);
  p = dfma(p, r, 0x1.5555555555555p-5);
  p = dfma(p, r, 0x1.5555555555555p-3);
  p = dfma(p, r, 0x1.0p-1);
  p = dfma(p, r, 1.0);
  p = dfma(p, r, 1.0);
  // p in [0.70, 1.42], k in [-1010, 1]: scale through the exponent field.
  const long long k = (long long)kd;
  return __longlong_as_double(__double_as_longlong(p) + (k << 52));
}

// natural log in fp64 of a positive normal z: z = f 2^e, f in [sqrt(1/2), sqrt(2)),
// log f = 2 atanh((f-1)/(f+1)) by its odd series to s^23.
__device__ __forceinline__ double det_log64(double z) {
  long long b = __double_as_longlong(z);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  b = (b & 0x000fffffffffffffll) | 0x3ff0000000000000ll;
  double f = __longlong_as_double(b);
  if (f > 0x1.6a09e667f3bcdp+0) { f = dmul(f, 0.5); e += 1; }
  const double s = __ddiv_rn(dsub(f, 1.0), dadd(f, 1.0));
  const double s2 = dmul(s, s);
  double t = 0x1.642c8590b2164p-4;
  t = dfma(t, s2, 0x1.8618618618618p-4);
  t = dfma(t, s2, 0x1.af286bca1af28p-4);
  t = dfma(t, s2, 0x1.e1e1e1e1e1e1ep-4);
  t = dfma(t, s2, 0x1.1111111111111p-3);
  t = dfma(t, s2, 0x1.3b13b13b13b14p-3);
  t = dfma(t, s2, 0x1.745d1745d1746p-3);
  t = dfma(t, s2, 0x1.c71c71c71c71cp-3);
  t = dfma(t, s2, 0x1.2492492492492p-2);
  t = dfma(t, s2, 0x1.999999999999ap-2);
  t = dfma(t, s2, 0x1.5555555555555p-1);
  t = dfma(t, s2, 0x1.0p+1);
  const double lf = dmul(s, t);
  return dfma((double)e, 0x1.62e42fefa39efp-1, lf);
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC'11) and the noise derived from it
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// Gumbel value for (row, token): counter {token/4, row, off_lo, off_hi},
// key {seed_lo, seed_hi}, word token%4 -> u = (w + 1/2) 2^-32 -> -log(-log u).
__device__ __forceinline__ float philox_gumbel(uint64_t seed, uint64_t offset, uint32_t row,
                                               uint32_t token) {
  const uint4 o = philox4x32_10(make_uint4(token >> 2, row, (uint32_t)offset, (uint32_t)(offset >> 32)),
                                make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
  const uint32_t w = (token & 3) == 0 ? o.x : (token & 3) == 1 ? o.y : (token & 3) == 2 ? o.z : o.w;
  const double u = dmul(dadd((double)w, 0.5), 0x1p-32);
  return (float)(-det_log64(-det_log64(u)));
}

// 53-bit uniform integer for (row, stream): counter {~0, row, off_lo, off_hi},
// key {seed_lo, seed_hi ^ stream}, top 53 bits of (w0 << 32 | w1).
__device__ __forceinline__ uint64_t philox_u53(uint64_t seed, uint64_t offset, uint32_t row,
                                               uint32_t stream) {
  const uint4 o = philox4x32_10(make_uint4(0xFFFFFFFFu, row, (uint32_t)offset, (uint32_t)(offset >> 32)),
                                make_uint2((uint32_t)seed, (uint32_t)(seed >> 32) ^ stream));
  return ((((uint64_t)o.x) << 32) | o.y) >> 11;
}

// A uniform in [0,1) given in fp64 -> floor(u 2^53).
__device__ __forceinline__ uint64_t u53_from_double(double u) {
  if (!(u > 0.0)) return 0ull;
  if (u >= 1.0) return (1ull << 53) - 1;
  return __double2ull_rz(dmul(u, 0x1p53));
}

// floor(u53 * w / 2^53).
__device__ __forceinline__ uint64_t scale_u53(uint64_t u53, uint64_t w) {
  return __umul64hi(u53 << 11, w);
}

// ---------------------------------------------------------------------------
// Rank keys: (logit desc, token asc) as one unsigned 64-bit key
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ordkey(float x) {
  const uint32_t u = __float_as_uint(fadd(x, 0.0f));  // folds -0 into +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint64_t rankkey(float x, uint32_t idx) {
  return ((uint64_t)ordkey(x) << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ float key_value(uint64_t key) {
  const uint32_t o = (uint32_t)(key >> 32);
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return __uint_as_float(u);
}
__device__ __forceinline__ uint32_t key_index(uint64_t key) { return 0xFFFFFFFFu - (uint32_t)key; }

// ---------------------------------------------------------------------------
// warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}
__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(kFull, v, o);
    v = w > v ? w : v;
  }
  return v;
}
__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(kFull, v, o);
    v = w < v ? w : v;
  }
  return v;
}
__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += t;
  }
  return v;
}
__device__ __forceinline__ uint64_t warp_incl_scan_u64(uint64_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t t = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Loads that bypass L1: workspace written by other CTAs of the same launch.
template <typename T>
__device__ __forceinline__ T ld_cg(const T* p) { return __ldcg(p); }

}  // namespace pm
