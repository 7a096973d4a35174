// Shared device/host helpers of the HeadStartLSTM B200 library.
#pragma once

#include <cuda_runtime.h>
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
// Logistic sigmoid from expf; 1/(1+inf) = 0 keeps the large-negative tail exact.
HS_DEV float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

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

// Look-back state shared by the scan kernels (scan.cu, scan_tma.cu).
struct ScanTmaWs {
  unsigned *ticket;
  unsigned *flags;  // per tile slot: 0 empty, 1 aggregate ready, 2 inclusive ready
  float *agg_a, *agg_c, *incl;
  float *db_part;   // bias-gradient partial rows (backward)
};

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace hs
