// sv_common.cuh -- device arithmetic shared by the decode-sampling kernels.
//
// The arithmetic here is the specification the kernels implement.  It reproduces
// the reference's sampling chain (ComfyUI-StarVector-GGUF runtime_shared.py:170-237)
// with decisions made in exact integer arithmetic:
//   * sv_exp: Cody-Waite reduction x = n ln2 + r, degree-7 Taylor polynomial of e^r
//     (coefficients 1/k!) in Horner form with fused multiply-add, scaling by 2^n in
//     two steps below 2^-126 so subnormal results round once (max error < 1 ulp);
//   * weights W = trunc(w * 2^44) summed in 64-bit integers: sums are exact and
//     independent of reduction order, so a parallel reduction gives the same bits
//     as a sequential one;
//   * floor(a * f) for a float f in [0,1) is exact (128-bit product);
//   * ln of a fixed-point sum in double precision (atanh series), rounded to float.
// Every float operation that matters is spelled with an explicit rounding intrinsic
// so the compiler cannot contract or reorder it.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace sv {

// Row status codes (also returned per row through out_status).
enum Status : int32_t {
  ST_OK = 0,
  ST_NAN = 1,         // a NaN logit
  ST_POSINF = 2,      // +inf after penalty / temperature (the reference's softmax gives NaN)
  ST_ALLNEGINF = 3,   // no finite logit in the row
  ST_HISTORY = 4,     // a history id outside [0, V)
  ST_TIMEOUT = 5,     // a bounded wait on an asynchronous copy ran out
  ST_SHARD_OVERFLOW = 6,  // vocab-sharded merge: a slice's kept list exceeded its capacity
};

__device__ __forceinline__ uint32_t ord_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// NaN-propagating maximum (max.NaN.f32): a NaN anywhere reaches the reductions.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float sv_exp(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -104.0f) return 0.0f;
  float j = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  int n = (int)j;
  // ln 2 split in two floats, as SLEEF's single-precision L2Uf / L2Lf (Cody-Waite):
  // the high part has few mantissa bits, so j times it is exact over the j used here.
  float r = __fmaf_rn(-j, 0.693145751953125f, x);
  r = __fmaf_rn(-j, 1.428606765330187045e-06f, r);
  float p = 1.98412698412698412698e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  if (n > 127) { p = __fmul_rn(p, 2.0f); n -= 1; }
  if (n >= -126) return __fmul_rn(p, __uint_as_float((uint32_t)(n + 127) << 23));
  return __fmul_rn(__fmul_rn(p, __uint_as_float((uint32_t)(n + 127 + 64) << 23)),
                   __uint_as_float((uint32_t)(127 - 64) << 23));
}

// trunc(w * 2^44) for w in [0, 1].
__device__ __forceinline__ uint64_t fixw(float w) {
  return __float2ull_rz(__fmul_rn(w, 17592186044416.0f));
}

// (float)total * 2^-44: the fixed-point sum as a float (total >= 2^44 in use).
__device__ __forceinline__ float fix_to_float(uint64_t total) {
  return __fmul_rn(__ull2float_rn(total), 5.684341886080801487e-14f);
}

// floor(a * f) for f in [0,1) exactly; f <= 0 or NaN gives 0, f >= 1 is clamped.
__device__ __forceinline__ uint64_t mulfloor(uint64_t a, float f) {
  if (!(f > 0.0f)) return 0;
  if (f >= 1.0f) f = __uint_as_float(0x3f7fffffu);
  uint32_t b = __float_as_uint(f);
  int ex = (int)((b >> 23) & 0xffu);
  uint64_t mant = b & 0x7fffffu;
  int sh;
  if (ex == 0) sh = 149;
  else { mant |= 0x800000u; sh = 150 - ex; }
  uint64_t lo = a * mant;
  uint64_t hi = __umul64hi(a, mant);
  if (sh >= 128) return 0;
  if (sh >= 64) return hi >> (sh - 64);
  return (lo >> sh) | (hi << (64 - sh));  // sh >= 24 here, so 64 - sh < 64
}

// ln(sw * 2^-44) rounded to float (sw >= 1): sw = m 2^e, m in [sqrt(1/2), sqrt(2)),
// ln m = 2 atanh(z), z = (m-1)/(m+1), series through z^23, all in double.
__device__ __forceinline__ float log_fixed(uint64_t sw) {
  double d = __ull2double_rn(sw);
  int e;
  double m = frexp(d, &e);
  if (m < 0.70710678118654752440) { m = __dmul_rn(m, 2.0); e -= 1; }
  double z = __ddiv_rn(__dadd_rn(m, -1.0), __dadd_rn(m, 1.0));
  double z2 = __dmul_rn(z, z);
  double p = 1.0 / 23.0;
  p = __fma_rn(p, z2, 1.0 / 21.0);
  p = __fma_rn(p, z2, 1.0 / 19.0);
  p = __fma_rn(p, z2, 1.0 / 17.0);
  p = __fma_rn(p, z2, 1.0 / 15.0);
  p = __fma_rn(p, z2, 1.0 / 13.0);
  p = __fma_rn(p, z2, 1.0 / 11.0);
  p = __fma_rn(p, z2, 1.0 / 9.0);
  p = __fma_rn(p, z2, 1.0 / 7.0);
  p = __fma_rn(p, z2, 1.0 / 5.0);
  p = __fma_rn(p, z2, 1.0 / 3.0);
  p = __fma_rn(p, z2, 1.0);
  double lm = __dmul_rn(__dadd_rn(z, z), p);
  double r = __fma_rn((double)(e - 44), 0.69314718055994530942, lm);
  return __double2float_rn(r);
}

// Repetition penalty of one score (runtime_shared.py:172): s<0 ? s*p : s/p.
__device__ __forceinline__ float penalize(float s, float rp) {
  return (s < 0.0f) ? __fmul_rn(s, rp) : __fdiv_rn(s, rp);
}

// Temperature (runtime_shared.py:178-179) followed by canonicalising -0 to +0, so
// float comparisons and the ordered-key comparisons agree (torch treats -0 == +0).
__device__ __forceinline__ float temper(float s, float T) {
  return __fadd_rn(__fdiv_rn(s, T), 0.0f);
}

template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kSize = 4;
  __device__ static float load(const float* p) { return __ldg(p); }
  __device__ static float to_f(float v) { return v; }
  __device__ static float neg_inf() { return __int_as_float(0xff800000); }
};
template <> struct Elem<__half> {
  static constexpr int kSize = 2;
  __device__ static float load(const __half* p) { return __half2float(__ldg(p)); }
  __device__ static float to_f(__half v) { return __half2float(v); }
  __device__ static __half neg_inf() { return __ushort_as_half((unsigned short)0xfc00u); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kSize = 2;
  __device__ static float load(const __nv_bfloat16* p) { return __bfloat162float(__ldg(p)); }
  __device__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __nv_bfloat16 neg_inf() { return __ushort_as_bfloat16((unsigned short)0xff80u); }
};

// Nanoseconds from the global timer, for bounded waits.
__device__ __forceinline__ uint64_t gtimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace sv
