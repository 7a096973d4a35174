// Shared device/host helpers of the HeadStartLSTM B200 library.
#pragma once

#include <cuda_runtime.h>
#include <atomic>
#include <stdint.h>
#include <stdio.h>

#include "../../include/headstartlstm_b200.h"

#define HS_DEV __device__ __forceinline__

namespace hs {

// ---------------------------------------------------------------- host side
// Records a message for hs_last_error_message() and returns `code`.
int fail(int code, const char *fmt, ...);
int check_launch(const char *what);

// Upper bound on every device-side wait (flag of another CTA); past it the
// waiting CTA records HS_ERR_DEVICE_TIMEOUT in the status word and returns.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------- math
// Power-of-two scale of the 3 x fp16 split: 2^(14 - floor(log2 m)) for
// m = the float with bits absmax_bits, so that |x| <= m maps into [0, 2^15);
// 1 for zero, infinite or NaN m.
HS_DEV float pow2_scale(unsigned absmax_bits) {
  const float m = __uint_as_float(absmax_bits);
  if (!(m > 0.f) || !(m < 3.0e38f)) return 1.0f;
  int e;
  (void)frexpf(m, &e);  // m = f 2^e, f in [0.5, 1): floor(log2 m) = e - 1
  const int k = max(e - 1, -100);
  return ldexpf(1.0f, 14 - k);
}

// Logistic sigmoid from expf; 1/(1+inf) = 0 keeps the large-negative tail exact.
HS_DEV float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }
#ifndef HS_SIGF_NR
#define HS_SIGF_NR 1
#endif
#ifndef HS_TANH_POLY
#define HS_TANH_POLY 1
#endif
// Reciprocal of d >= 1: the hardware approximation refined by one
// Newton-Raphson step, r' = r + r (1 - d r) (the classical iteration for 1/d,
// which squares the relative error of the seed).  One step brings the ~1 ulp
// seed to within rounding of the correctly rounded result, for three
// instructions instead of the IEEE-rounded reciprocal's longer sequence.
// d = +inf gives 0 (the step itself would form inf*0); a NaN stays NaN.
HS_DEV float rcp_nr(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  const float n = fmaf(r, fmaf(-d, r, 1.0f), r);
  return d == __int_as_float(0x7f800000) ? 0.0f : n;
}
// Scan-path sigmoid: hardware exp and a reciprocal rounded to (nearly) the
// correctly rounded value.  The rounding of the reciprocal matters: an
// approximate divide biases every forget gate by about an ulp, which the
// product of thousands of gates turns into a 1e-5 error of c at T = 2048.
HS_DEV float sigf(float x) {
#if HS_SIGF_NR
  return rcp_nr(1.0f + __expf(-x));
#else
  return __frcp_rn(1.0f + __expf(-x));
#endif
}
// tanh for c >= 0 (the scan's cell state is positive): (1 - e^-2c)/(1 + e^-2c)
// from the hardware exp.  Below 0.25 that form loses relative accuracy to
// cancellation, so small arguments use the odd Taylor series of tanh,
//   c - c^3/3 + 2c^5/15 - 17c^7/315 + 62c^9/2835,
// whose first omitted term (1382/155925 c^11) is below 1e-8 relative there.
HS_DEV float tanh_pos(float c) {
#if HS_TANH_POLY
  // both forms, one selected: no divergence where lanes straddle 0.25
  const float u = c * c;
  float p = fmaf(u, 62.0f / 2835.0f, -17.0f / 315.0f);
  p = fmaf(p, u, 2.0f / 15.0f);
  p = fmaf(p, u, -1.0f / 3.0f);
  const float tp = fmaf(p * u, c, c);
  const float e = __expf(-2.0f * c);
  const float te = __fdividef(1.0f - e, 1.0f + e);
  return c < 0.25f ? tp : te;
#else
  if (c < 0.25f) return tanhf(c);
  const float e = __expf(-2.0f * c);
  return __fdividef(1.0f - e, 1.0f + e);
#endif
}

// tanh of either sign: tanh_pos of |c| with c's sign.
HS_DEV float tanh_any(float c) { return copysignf(tanh_pos(fabsf(c)), c); }

// The hardware reciprocal alone (about 1 ulp; +inf gives 0).  Enough where
// a value's rounding does not compound over time steps: the input and output
// gates and i*g enter each cell state once, while the forget gate multiplies
// every later state and keeps the refined reciprocal (sigf).
HS_DEV float rcp_fast(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return r;
}
HS_DEV float sig_fast(float x) { return rcp_fast(1.0f + __expf(-x)); }

// sigma(x) * sigma(y) with one reciprocal: 1 / ((1 + e^-x)(1 + e^-y)).  An
// infinite denominator gives 0, a NaN stays NaN.
HS_DEV float sig2(float x, float y) { return rcp_fast((1.0f + __expf(-x)) * (1.0f + __expf(-y))); }

// sigma(z) * tanh(c) for c >= 0 from eo = e^-z, with one reciprocal:
// poly(c) / (1 + eo) below 0.25 (odd Taylor series of tanh, as tanh_pos) and
// (1 - e^-2c) / ((1 + e^-2c)(1 + eo)) above.
HS_DEV float sig_tanh_pos(float eo, float c) {
  // both forms, one selected (no divergence where lanes straddle 0.25)
  const float u = c * c;
  float p = fmaf(u, 62.0f / 2835.0f, -17.0f / 315.0f);
  p = fmaf(p, u, 2.0f / 15.0f);
  p = fmaf(p, u, -1.0f / 3.0f);
  const float tp = fmaf(p * u, c, c);
  const float e = __expf(-2.0f * c);
  const bool small = c < 0.25f;
  const float num = small ? tp : 1.0f - e;
  const float den = small ? 1.0f + eo : (1.0f + e) * (1.0f + eo);
  return num * rcp_fast(den);
}

// ---------------------------------------------------------------- memory model
HS_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
HS_DEV unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
HS_DEV void st_release(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
HS_DEV int ld_status(const int *p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
HS_DEV void set_status(int *p, int code) { atomicCAS(p, 0, code); }

// Spin until *flag != 0, bounded by kWaitLimitNs and by the sticky status
// word (another CTA that already gave up makes every waiter leave at once).
// Returns the flag value, or 0 if the wait was abandoned.
HS_DEV unsigned wait_flag(const unsigned *flag, int *status, uint64_t limit_ns = kWaitLimitNs) {
  unsigned v = ld_acquire(flag);
  if (v) return v;
  const uint64_t t0 = globaltimer();
  unsigned ns = 32;
  while (true) {
    __nanosleep(ns);
    if (ns < 1024) ns <<= 1;
    v = ld_acquire(flag);
    if (v) return v;
    if (ld_status(status) != 0) return 0;
    if (globaltimer() - t0 > limit_ns) {
      set_status(status, HS_ERR_DEVICE_TIMEOUT);
      return 0;
    }
  }
}

// ---------------------------------------------------------------- vectors
template <int VEC> struct Vec;
template <> struct Vec<1> {
  float v[1];
  HS_DEV void load(const float *p) { v[0] = *p; }
  HS_DEV void load_cg(const float *p) { v[0] = __ldcg(p); }
  HS_DEV void load_cs(const float *p) { v[0] = __ldcs(p); }
  HS_DEV void store(float *p) const { *p = v[0]; }
  HS_DEV void store_cg(float *p) const { __stcg(p, v[0]); }
  HS_DEV void store_cs(float *p) const { __stcs(p, v[0]); }
};
template <> struct Vec<2> {
  float v[2];
  HS_DEV void load(const float *p) { float2 t = *reinterpret_cast<const float2 *>(p); v[0] = t.x; v[1] = t.y; }
  HS_DEV void load_cg(const float *p) { float2 t = __ldcg(reinterpret_cast<const float2 *>(p)); v[0] = t.x; v[1] = t.y; }
  HS_DEV void load_cs(const float *p) { float2 t = __ldcs(reinterpret_cast<const float2 *>(p)); v[0] = t.x; v[1] = t.y; }
  HS_DEV void store(float *p) const { *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]); }
  HS_DEV void store_cg(float *p) const { __stcg(reinterpret_cast<float2 *>(p), make_float2(v[0], v[1])); }
  HS_DEV void store_cs(float *p) const { __stcs(reinterpret_cast<float2 *>(p), make_float2(v[0], v[1])); }
};
template <> struct Vec<4> {
  float v[4];
  HS_DEV void load(const float *p) { float4 t = *reinterpret_cast<const float4 *>(p); v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w; }
  HS_DEV void load_cg(const float *p) { float4 t = __ldcg(reinterpret_cast<const float4 *>(p)); v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w; }
  HS_DEV void load_cs(const float *p) { float4 t = __ldcs(reinterpret_cast<const float4 *>(p)); v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w; }
  HS_DEV void store(float *p) const { *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]); }
  HS_DEV void store_cg(float *p) const { __stcg(reinterpret_cast<float4 *>(p), make_float4(v[0], v[1], v[2], v[3])); }
  HS_DEV void store_cs(float *p) const { __stcs(reinterpret_cast<float4 *>(p), make_float4(v[0], v[1], v[2], v[3])); }
};

// Raises a kernel's dynamic shared-memory limit to `bytes`, once per device
// (the attribute belongs to the device's context); `done` is the kernel's
// bit mask of devices already set.
inline int allow_dynamic_smem(const void *fn, size_t bytes, std::atomic<unsigned long long> *done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
  const unsigned long long bit = 1ull << (dev & 63);
  if (done->load(std::memory_order_relaxed) & bit) return HS_OK;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  done->fetch_or(bit);
  return HS_OK;
}

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace hs
