// Persistent, TMA-fed versions of the parallel-mode scan kernels (scan.cu
// holds the recurrence, layouts and the look-back protocol they share; these
// kernels take every shape with H % 4 == 0, scan.cu's per-tile kernels the
// rest).
//
// Why: a one-tile-per-CTA kernel has bytes in flight only while it issues
// its loads, then idles at its look-back.  Here each CTA (one per SM) holds
// up to three tiles: the current one and the next two, whose inputs a single
// thread streams into a 3-stage shared-memory ring with TMA
// (cp.async.bulk.tensor, no multicast) while the CTA computes, publishes and
// looks back.  Tickets are still taken in time-major order and each CTA
// processes its tickets in increasing order, so the smallest unfinished
// ticket is always some CTA's current tile, whose predecessors are done: the
// look-back cannot deadlock.
//
// Transcendentals use the hardware exp2 (__expf) and a correctly rounded
// reciprocal so the kernels stay memory-bound; tanh of the (positive) cell state is
// (1 - e^{-2c}) / (1 + e^{-2c}), with tanhf below 0.25 where that quotient
// would cancel.  Both are checked against tanhf/expf-based float64 oracles by
// the parity tests (normwise 1e-5).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "hs_common.cuh"

namespace hs {

namespace {

#ifndef HS_TMA_FWD_S
#define HS_TMA_FWD_S 4
#endif
#ifndef HS_TMA_BWD_S
#define HS_TMA_BWD_S 2
#endif
#ifndef HS_TMA_MINB
#define HS_TMA_MINB 1
#endif
constexpr int NW = 8, NT = NW * 32, VEC = 4, HW = 128, STAGES = 3;

// The reciprocal is the correctly rounded one: products of forget gates run
// over thousands of steps, where an approximate (biased) reciprocal's error
// accumulates; __expf's error is damped by 1/(1+e) where f is near 1.
HS_DEV float sigf(float x) { return __frcp_rn(1.0f + __expf(-x)); }
HS_DEV float tanh_pos(float c) {
  if (c < 0.25f) return tanhf(c);
  const float e = __expf(-2.0f * c);
  return __fdividef(1.0f - e, 1.0f + e);
}

HS_DEV uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
HS_DEV void mbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
HS_DEV void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
HS_DEV bool mbar_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
HS_DEV bool mbar_wait(uint64_t *b, uint32_t parity, int *status) {
  if (mbar_try(b, parity)) return true;
  const uint64_t t0 = globaltimer();
  unsigned n = 0;
  while (!mbar_try(b, parity)) {
    if ((++n & 63u) == 0) {
      if (ld_status(status) != 0) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        set_status(status, HS_ERR_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}
// Bounded wait that records nothing (used when draining on an abort path).
HS_DEV void mbar_drain(uint64_t *b, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try(b, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) return;
  }
}
HS_DEV void tma_3d(void *dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(su32(dst)),
      "l"(tm), "r"(c0), "r"(c1), "r"(c2), "r"(su32(bar))
      : "memory");
}

struct Geo {
  int64_t T, B, H;
  int nchunk, nhb;
  unsigned ntiles;
};

// Warp 0: publish this tile's summary (TA, TC per lane x VEC) in `slot` and
// obtain the carry entering it from its predecessors in scan order
// (k-1, k-2, ...).  `first` = the tile is first in scan order; its carry is
// `cin` as given.  Returns false if a wait gave up.
HS_DEV bool publish_and_look_back(const ScanTmaWs &ws, const Geo &g, int k, int64_t b, int hb,
                                  const float (&TA)[VEC], const float (&TC)[VEC], float (&cin)[VEC],
                                  int lane, int *status) {
  const int64_t slot = ((int64_t)k * g.B + b) * g.nhb + hb;
  bool ok = true;
  if (k > 0) {
    Vec<VEC> va, vc;
#pragma unroll
    for (int v = 0; v < VEC; ++v) { va.v[v] = TA[v]; vc.v[v] = TC[v]; }
    va.store_cg(ws.agg_a + slot * HW + lane * VEC);
    vc.store_cg(ws.agg_c + slot * HW + lane * VEC);
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release(ws.flags + slot, 1u);
    float ra[VEC], rc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) { ra[v] = 1.f; rc[v] = 0.f; }
    for (int kk = k - 1; kk >= 0; --kk) {
      const int64_t ks = ((int64_t)kk * g.B + b) * g.nhb + hb;
      const unsigned f = wait_flag(ws.flags + ks, status);
      if (f == 0) { ok = false; break; }
      if (f == 2u) {
        Vec<VEC> p;
        p.load_cg(ws.incl + ks * HW + lane * VEC);
#pragma unroll
        for (int v = 0; v < VEC; ++v) cin[v] = fmaf(ra[v], p.v[v], rc[v]);
        break;
      }
      Vec<VEC> ka, kc;
      ka.load_cg(ws.agg_a + ks * HW + lane * VEC);
      kc.load_cg(ws.agg_c + ks * HW + lane * VEC);
#pragma unroll
      for (int v = 0; v < VEC; ++v) { rc[v] = fmaf(ra[v], kc.v[v], rc[v]); ra[v] *= ka.v[v]; }
    }
  }
  if (ok) {
    Vec<VEC> p;
#pragma unroll
    for (int v = 0; v < VEC; ++v) p.v[v] = fmaf(TA[v], cin[v], TC[v]);
    p.store_cg(ws.incl + slot * HW + lane * VEC);
    __threadfence();
  }
  __syncwarp();
  const bool all_ok = __all_sync(0xffffffffu, ok);
  if (all_ok && lane == 0) st_release(ws.flags + slot, 2u);
  return all_ok;
}

// ============================================================== forward
template <int S>
__global__ void __launch_bounds__(NT, HS_TMA_MINB)
scan_fwd_tma_kernel(const __grid_constant__ CUtensorMap tmZ, const float *__restrict__ c0,
                    float *__restrict__ out, float *__restrict__ cbuf, float *__restrict__ h_n,
                    float *__restrict__ c_n, Geo g, float eps, ScanTmaWs ws, int *status) {
  constexpr int L = S * NW;
  constexpr int GATE_FL = L * HW;               // floats per gate block of a tile
  constexpr uint32_t TILE_BYTES = 4 * GATE_FL * 4;
  extern __shared__ __align__(128) float sm[];
  float *stage = sm;                             // [STAGES][4][L][HW]
  float *sA = stage + STAGES * 4 * GATE_FL;      // [NW][HW]
  float *sC = sA + NW * HW;
  float *s_carry = sC + NW * HW;                 // [HW]
  uint64_t *full = reinterpret_cast<uint64_t *>(s_carry + HW);
  unsigned *s_ticket = reinterpret_cast<unsigned *>(full + STAGES);
  int *s_abort = reinterpret_cast<int *>(s_ticket + STAGES);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t T = g.T, B = g.B, H = g.H;
  const unsigned per_chunk = (unsigned)(B * g.nhb);

  auto issue = [&](unsigned tk, int st) {
    const int j = tk / per_chunk;
    const unsigned r = tk - j * per_chunk;
    const int b = (int)(r / g.nhb);
    const int hb = (int)(r % g.nhb);
    float *dst = stage + st * 4 * GATE_FL;
    mbar_expect_tx(&full[st], TILE_BYTES);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      tma_3d(dst + q * GATE_FL, &tmZ, &full[st], (int)(q * H + hb * HW), b, j * L);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *s_abort = ld_status(status) != 0;
    for (int s = 0; s < STAGES - 1; ++s) {
      // an aborted launch takes no tiles, so nothing is ever in flight
      const unsigned tk = *s_abort ? 0xFFFFFFFFu : atomicAdd(ws.ticket, 1u);
      s_ticket[s] = tk;
      if (tk < g.ntiles) issue(tk, s);
    }
  }
  __syncthreads();
  int it = 0;
  int issued_last = 0;  // thread 0: the load for iteration it+2 was issued
  for (;; ++it) {
    const int st = it % STAGES;
    issued_last = 0;
    const unsigned cur = s_ticket[st];
    if (cur >= g.ntiles || *s_abort) break;
    if (threadIdx.x == 0) {
      const int ns = (it + STAGES - 1) % STAGES;
      const unsigned nxt = atomicAdd(ws.ticket, 1u);
      s_ticket[ns] = nxt;
      issued_last = nxt < g.ntiles;
      if (issued_last) issue(nxt, ns);
    }
    // the wait's outcome is made uniform before anyone leaves the loop
    const bool got = mbar_wait(&full[st], (it / STAGES) & 1, status);
    if (!__syncthreads_and(got)) {
      if (threadIdx.x == 0) *s_abort = 1;
      break;
    }
    const int j = cur / per_chunk;
    const unsigned r = cur - j * per_chunk;
    const int64_t b = r / g.nhb;
    const int hb = (int)(r % g.nhb);
    const int64_t h = (int64_t)hb * HW + lane * VEC;
    const bool hv = h < H;
    const int64_t t0 = (int64_t)j * L + warp * S;
    const float *tile = stage + st * 4 * GATE_FL;

    float fp[S][VEC], bp[S][VEC], og[S][VEC];
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int row = warp * S + s;
      const float4 zi = *reinterpret_cast<const float4 *>(tile + 0 * GATE_FL + row * HW + lane * VEC);
      const float4 zf = *reinterpret_cast<const float4 *>(tile + 1 * GATE_FL + row * HW + lane * VEC);
      const float4 zg = *reinterpret_cast<const float4 *>(tile + 2 * GATE_FL + row * HW + lane * VEC);
      const float4 zo = *reinterpret_cast<const float4 *>(tile + 3 * GATE_FL + row * HW + lane * VEC);
      const float ai[4] = {zi.x, zi.y, zi.z, zi.w}, af[4] = {zf.x, zf.y, zf.z, zf.w};
      const float ag[4] = {zg.x, zg.y, zg.z, zg.w}, ao[4] = {zo.x, zo.y, zo.z, zo.w};
      const bool tv = hv && (t0 + s) < T;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        if (tv) {
          fp[s][v] = fmaxf(sigf(af[v]), eps);
          bp[s][v] = fmaxf(sigf(ai[v]) * sigf(ag[v]), eps);
          og[s][v] = sigf(ao[v]);
        } else {
          fp[s][v] = 1.f; bp[s][v] = 0.f; og[s][v] = 0.f;
        }
      }
    }
    float A[VEC], C[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) { A[v] = 1.f; C[v] = 0.f; }
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
      for (int v = 0; v < VEC; ++v) { C[v] = fmaf(fp[s][v], C[v], bp[s][v]); A[v] *= fp[s][v]; }
#pragma unroll
    for (int v = 0; v < VEC; ++v) { sA[warp * HW + lane * VEC + v] = A[v]; sC[warp * HW + lane * VEC + v] = C[v]; }
    __syncthreads();  // also: every thread is done reading stage st

    if (warp == 0) {
      float TA[VEC], TC[VEC], cin[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) { TA[v] = 1.f; TC[v] = 0.f; }
#pragma unroll
      for (int w = 0; w < NW; ++w)
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const float a = sA[w * HW + lane * VEC + v];
          TC[v] = fmaf(a, TC[v], sC[w * HW + lane * VEC + v]);
          TA[v] *= a;
        }
#pragma unroll
      for (int v = 0; v < VEC; ++v) cin[v] = fmaxf((j == 0 && c0 && hv) ? c0[b * H + h + v] : 0.f, eps);
      const bool ok = publish_and_look_back(ws, g, j, b, hb, TA, TC, cin, lane, status);
      if (lane == 0 && !ok) *s_abort = 1;
#pragma unroll
      for (int v = 0; v < VEC; ++v) s_carry[lane * VEC + v] = cin[v];
    }
    __syncthreads();
    if (*s_abort) break;

    float c[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) c[v] = s_carry[lane * VEC + v];
    for (int w = 0; w < warp; ++w)
#pragma unroll
      for (int v = 0; v < VEC; ++v) c[v] = fmaf(sA[w * HW + lane * VEC + v], c[v], sC[w * HW + lane * VEC + v]);
    if (hv) {
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const int64_t t = t0 + s;
        if (t >= T) break;
        Vec<VEC> vc, vo;
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          c[v] = fmaf(fp[s][v], c[v], bp[s][v]);
          vc.v[v] = c[v];
          vo.v[v] = og[s][v] * tanh_pos(c[v]);
        }
        const int64_t o = (t * B + b) * H + h;
        vc.store(cbuf + o);
        vo.store(out + o);
        if (t == T - 1) {
          if (c_n) vc.store(c_n + b * H + h);
          if (h_n) vo.store(h_n + b * H + h);
        }
      }
    }
    __syncthreads();  // sA/sC/s_carry reuse
  }
  // Leave no TMA copy in flight into this CTA's shared memory.
  // Leave no TMA copy in flight into this CTA's shared memory: on an abort,
  // wait (bounded) for every stage whose load was issued and not consumed.
  __syncthreads();
  if (threadIdx.x == 0 && *s_abort) {
    for (int k = 0; k < STAGES; ++k) {
      const int i2 = it + k;  // iterations it .. it+2 own the three stages
      const int st = i2 % STAGES;
      const bool issued = (k < STAGES - 1) ? (s_ticket[st] < g.ntiles) : (issued_last != 0);
      if (issued) {
        mbar_drain(&full[st], (i2 / STAGES) & 1);
      }
    }
  }
}

// ============================================================== backward
template <int S>
__global__ void __launch_bounds__(NT, HS_TMA_MINB)
scan_bwd_tma_kernel(const __grid_constant__ CUtensorMap tmZ, const __grid_constant__ CUtensorMap tmC,
                    const __grid_constant__ CUtensorMap tmD, const float *cbuf,
                    const float *__restrict__ c0, const float *__restrict__ dh_n,
                    const float *__restrict__ dc_n, float *dz, float *__restrict__ dc0, Geo g, float eps,
                    ScanTmaWs ws, int *status) {
  constexpr int L = S * NW;
  constexpr int BLK = L * HW;                         // floats per [L][HW] block
  constexpr int STAGE_FL = 6 * BLK;                   // z (4 gates), c, dout
  constexpr uint32_t TILE_BYTES = STAGE_FL * 4;
  extern __shared__ __align__(128) float sm[];
  float *stage = sm;                                  // [STAGES][6][L][HW]
  float *sA = stage + STAGES * STAGE_FL;              // [NW][HW]
  float *sC = sA + NW * HW;
  float *s_carry = sC + NW * HW;                      // [HW]
  float *s_db = s_carry + HW;                         // [4][Hp]
  const int Hp = g.nhb * HW;
  uint64_t *full = reinterpret_cast<uint64_t *>(s_db + 4 * Hp);
  unsigned *s_ticket = reinterpret_cast<unsigned *>(full + STAGES);
  int *s_abort = reinterpret_cast<int *>(s_ticket + STAGES);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t T = g.T, B = g.B, H = g.H;
  const unsigned per_chunk = (unsigned)(B * g.nhb);

  for (int i = threadIdx.x; i < 4 * Hp; i += NT) s_db[i] = 0.f;

  auto issue = [&](unsigned tk, int st) {
    const int q = tk / per_chunk;
    const int j = g.nchunk - 1 - q;
    const unsigned r = tk - q * per_chunk;
    const int b = (int)(r / g.nhb);
    const int hb = (int)(r % g.nhb);
    float *dst = stage + st * STAGE_FL;
    mbar_expect_tx(&full[st], TILE_BYTES);
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) tma_3d(dst + gg * BLK, &tmZ, &full[st], (int)(gg * H + hb * HW), b, j * L);
    tma_3d(dst + 4 * BLK, &tmC, &full[st], hb * HW, b, j * L);
    tma_3d(dst + 5 * BLK, &tmD, &full[st], hb * HW, b, j * L);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *s_abort = ld_status(status) != 0;
    for (int s = 0; s < STAGES - 1; ++s) {
      // an aborted launch takes no tiles, so nothing is ever in flight
      const unsigned tk = *s_abort ? 0xFFFFFFFFu : atomicAdd(ws.ticket, 1u);
      s_ticket[s] = tk;
      if (tk < g.ntiles) issue(tk, s);
    }
  }
  __syncthreads();
  int it = 0;
  int issued_last = 0;  // thread 0: the load for iteration it+2 was issued
  for (;; ++it) {
    const int st = it % STAGES;
    issued_last = 0;
    const unsigned cur = s_ticket[st];
    if (cur >= g.ntiles || *s_abort) break;
    if (threadIdx.x == 0) {
      const int ns = (it + STAGES - 1) % STAGES;
      const unsigned nxt = atomicAdd(ws.ticket, 1u);
      s_ticket[ns] = nxt;
      issued_last = nxt < g.ntiles;
      if (issued_last) issue(nxt, ns);
    }
    // the wait's outcome is made uniform before anyone leaves the loop
    const bool got = mbar_wait(&full[st], (it / STAGES) & 1, status);
    if (!__syncthreads_and(got)) {
      if (threadIdx.x == 0) *s_abort = 1;
      break;
    }
    const int q = cur / per_chunk;
    const int j = g.nchunk - 1 - q;
    const unsigned r = cur - q * per_chunk;
    const int64_t b = r / g.nhb;
    const int hb = (int)(r % g.nhb);
    const int64_t h = (int64_t)hb * HW + lane * VEC;
    const bool hv = h < H;
    const int64_t t0 = (int64_t)j * L + warp * S;
    const float *tile = stage + st * STAGE_FL;

    float FP[S][VEC], DCD[S][VEC], KI[S][VEC], KF[S][VEC], KG[S][VEC];
    float acc[4][VEC];
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2)
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[q2][v] = 0.f;
    float cprev[VEC];
    if (warp > 0) {
      const float4 cp = *reinterpret_cast<const float4 *>(tile + 4 * BLK + (warp * S - 1) * HW + lane * VEC);
      cprev[0] = cp.x; cprev[1] = cp.y; cprev[2] = cp.z; cprev[3] = cp.w;
    } else if (t0 == 0) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) cprev[v] = fmaxf((c0 && hv) ? c0[b * H + h + v] : 0.f, eps);
    } else if (hv && t0 - 1 < T) {
      Vec<VEC> tv;
      tv.load(cbuf + ((t0 - 1) * B + b) * H + h);
#pragma unroll
      for (int v = 0; v < VEC; ++v) cprev[v] = tv.v[v];
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) cprev[v] = 0.f;
    }
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int64_t t = t0 + s;
      const int row = warp * S + s;
      const bool tv = hv && t < T;
      const float4 zi = *reinterpret_cast<const float4 *>(tile + 0 * BLK + row * HW + lane * VEC);
      const float4 zf = *reinterpret_cast<const float4 *>(tile + 1 * BLK + row * HW + lane * VEC);
      const float4 zg = *reinterpret_cast<const float4 *>(tile + 2 * BLK + row * HW + lane * VEC);
      const float4 zo = *reinterpret_cast<const float4 *>(tile + 3 * BLK + row * HW + lane * VEC);
      const float4 cc = *reinterpret_cast<const float4 *>(tile + 4 * BLK + row * HW + lane * VEC);
      const float4 dd = *reinterpret_cast<const float4 *>(tile + 5 * BLK + row * HW + lane * VEC);
      const float ai[4] = {zi.x, zi.y, zi.z, zi.w}, af[4] = {zf.x, zf.y, zf.z, zf.w};
      const float ag[4] = {zg.x, zg.y, zg.z, zg.w}, ao[4] = {zo.x, zo.y, zo.z, zo.w};
      const float ac[4] = {cc.x, cc.y, cc.z, cc.w};
      float ad[4] = {dd.x, dd.y, dd.z, dd.w};
      if (tv && t == T - 1 && dh_n) {
        const float4 e = *reinterpret_cast<const float4 *>(dh_n + b * H + h);
        ad[0] += e.x; ad[1] += e.y; ad[2] += e.z; ad[3] += e.w;
      }
      Vec<VEC> dzo;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        if (tv) {
          const float i = sigf(ai[v]), f = sigf(af[v]), gg = sigf(ag[v]), o = sigf(ao[v]);
          const float th = tanh_pos(ac[v]);
          const float mb = (i * gg >= eps) ? 1.f : 0.f;
          const float mf = (f >= eps) ? 1.f : 0.f;
          FP[s][v] = fmaxf(f, eps);
          DCD[s][v] = ad[v] * o * (1.f - th * th);
          KI[s][v] = gg * i * (1.f - i) * mb;
          KF[s][v] = cprev[v] * f * (1.f - f) * mf;
          KG[s][v] = i * gg * (1.f - gg) * mb;
          dzo.v[v] = ad[v] * th * o * (1.f - o);
          acc[3][v] += dzo.v[v];
          cprev[v] = ac[v];
        } else {
          FP[s][v] = 1.f; DCD[s][v] = 0.f; KI[s][v] = KF[s][v] = KG[s][v] = 0.f; dzo.v[v] = 0.f;
        }
      }
      if (tv) {
        if (t == T - 1 && dc_n) {
          const float4 e = *reinterpret_cast<const float4 *>(dc_n + b * H + h);
          DCD[s][0] += e.x; DCD[s][1] += e.y; DCD[s][2] += e.z; DCD[s][3] += e.w;
        }
        dzo.store_cs(dz + (t * B + b) * 4 * H + 3 * H + h);
      }
    }
    float A[VEC], C[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) { A[v] = 1.f; C[v] = 0.f; }
#pragma unroll
    for (int s = S - 1; s >= 0; --s)
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        C[v] = FP[s][v] * (C[v] + DCD[s][v]);
        A[v] *= FP[s][v];
      }
#pragma unroll
    for (int v = 0; v < VEC; ++v) { sA[warp * HW + lane * VEC + v] = A[v]; sC[warp * HW + lane * VEC + v] = C[v]; }
    __syncthreads();  // also: every thread is done reading stage st

    if (warp == 0) {
      float TA[VEC], TC[VEC], cin[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) { TA[v] = 1.f; TC[v] = 0.f; cin[v] = 0.f; }
#pragma unroll
      for (int w = NW - 1; w >= 0; --w)
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const float a = sA[w * HW + lane * VEC + v];
          TC[v] = fmaf(a, TC[v], sC[w * HW + lane * VEC + v]);
          TA[v] *= a;
        }
      const bool ok = publish_and_look_back(ws, g, q, b, hb, TA, TC, cin, lane, status);
      if (lane == 0 && !ok) *s_abort = 1;
#pragma unroll
      for (int v = 0; v < VEC; ++v) s_carry[lane * VEC + v] = cin[v];
    }
    __syncthreads();
    if (*s_abort) break;

    float e[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) e[v] = s_carry[lane * VEC + v];
    for (int w = NW - 1; w > warp; --w)
#pragma unroll
      for (int v = 0; v < VEC; ++v) e[v] = fmaf(sA[w * HW + lane * VEC + v], e[v], sC[w * HW + lane * VEC + v]);
    if (hv) {
#pragma unroll
      for (int s = S - 1; s >= 0; --s) {
        const int64_t t = t0 + s;
        if (t >= T) continue;
        Vec<VEC> di, df, dg;
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const float dc = DCD[s][v] + e[v];
          e[v] = FP[s][v] * dc;
          di.v[v] = dc * KI[s][v];
          df.v[v] = dc * KF[s][v];
          dg.v[v] = dc * KG[s][v];
          acc[0][v] += di.v[v];
          acc[1][v] += df.v[v];
          acc[2][v] += dg.v[v];
        }
        const int64_t zo = (t * B + b) * 4 * H + h;
        di.store_cs(dz + zo);
        df.store_cs(dz + zo + H);
        dg.store_cs(dz + zo + 2 * H);
        if (t == 0 && dc0) {
          Vec<VEC> d;
#pragma unroll
          for (int v = 0; v < VEC; ++v) d.v[v] = (c0 && c0[b * H + h + v] >= eps) ? e[v] : 0.f;
          d.store(dc0 + b * H + h);
        }
      }
    }
    // bias-gradient sums of this tile, added into the CTA's running sums
    if (ws.db_part) {
      __syncthreads();
#pragma unroll
      for (int q2 = 0; q2 < 4; ++q2) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) sA[warp * HW + lane * VEC + v] = acc[q2][v];
        __syncthreads();
        if (warp == 0 && hv) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) {
            float a = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) a += sA[w * HW + lane * VEC + v];
            s_db[q2 * Hp + h + v] += a;
          }
        }
        __syncthreads();
      }
    } else {
      __syncthreads();
    }
  }
  // Leave no TMA copy in flight into this CTA's shared memory: on an abort,
  // wait (bounded) for every stage whose load was issued and not consumed.
  __syncthreads();
  if (threadIdx.x == 0 && *s_abort) {
    for (int k = 0; k < STAGES; ++k) {
      const int i2 = it + k;  // iterations it .. it+2 own the three stages
      const int st = i2 % STAGES;
      const bool issued = (k < STAGES - 1) ? (s_ticket[st] < g.ntiles) : (issued_last != 0);
      if (issued) {
        mbar_drain(&full[st], (i2 / STAGES) & 1);
      }
    }
  }
  if (ws.db_part) {
    __syncthreads();
    float *row = ws.db_part + (int64_t)blockIdx.x * 4 * H;
    for (int i = threadIdx.x; i < 4 * H; i += NT) row[i] = s_db[(i / H) * Hp + (i % H)];
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [T][B][W] fp32 tensor, boxes of 128 x 1 x L.
bool map3(CUtensorMap *tm, const float *ptr, int64_t W, int64_t B, int64_t T, int L) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)W, (cuuint64_t)B, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)(W * 4), (cuuint64_t)(W * B * 4)};
  cuuint32_t box[3] = {(cuuint32_t)HW, 1, (cuuint32_t)L};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)ptr, dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

}  // namespace

constexpr int kTmaFwdS = HS_TMA_FWD_S, kTmaBwdS = HS_TMA_BWD_S;
int scan_tma_fwd_chunk() { return kTmaFwdS * NW; }
int scan_tma_bwd_chunk() { return kTmaBwdS * NW; }
int scan_tma_grid(unsigned ntiles) {
  return (int)std::min<unsigned>(ntiles, (unsigned)(sms() * HS_TMA_MINB));
}

size_t scan_tma_bwd_smem(int64_t H) {
  const int L = kTmaBwdS * NW;
  const int Hp = (int)((H + HW - 1) / HW) * HW;
  return (size_t)(STAGES * 6 * L * HW + 2 * NW * HW + HW + 4 * Hp) * 4 + STAGES * 8 + STAGES * 4 + 4 + 64;
}

// Launch the TMA forward kernel; *done = false if this shape/pointer set
// is not taken (then the caller runs the per-tile kernel).
int scan_fwd_tma_launch(const float *z, const float *c0, float *out, float *c, float *h_n, float *c_n,
                        int64_t T, int64_t B, int64_t H, float eps, const ScanTmaWs &ws, int nchunk, int nhb,
                        int *status, cudaStream_t st, bool *done) {
  *done = false;
  constexpr int S = kTmaFwdS, L = S * NW;
  if (H % 4 || !aligned(z, 16) || T >= (1ll << 31) || B >= (1ll << 31) || 4 * H >= (1ll << 31)) return HS_OK;
  CUtensorMap tz;
  if (!map3(&tz, z, 4 * H, B, T, L)) return HS_OK;
  Geo g{T, B, H, nchunk, nhb, (unsigned)((int64_t)nchunk * B * nhb)};
  const size_t smem = (size_t)(STAGES * 4 * L * HW + 2 * NW * HW + HW) * 4 + STAGES * 8 + STAGES * 4 + 4 + 64;
  static std::once_flag once;
  std::call_once(once, [&] {
    cudaFuncSetAttribute((const void *)scan_fwd_tma_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  });
  scan_fwd_tma_kernel<S><<<scan_tma_grid(g.ntiles), NT, smem, st>>>(tz, c0, out, c, h_n, c_n, g, eps, ws, status);
  if (int e = check_launch("scan_fwd_tma_kernel")) return e;
  *done = true;
  return HS_OK;
}

int scan_bwd_tma_launch(const float *z, const float *c, const float *c0, const float *dout,
                        const float *dh_n, const float *dc_n, float *dz, float *dc0, int64_t T, int64_t B,
                        int64_t H, float eps, const ScanTmaWs &ws, int nchunk, int nhb, int *status,
                        cudaStream_t st, bool *done) {
  *done = false;
  constexpr int S = kTmaBwdS, L = S * NW;
  if (H % 4 || !aligned(z, 16) || !aligned(c, 16) || !aligned(dout, 16) || (dh_n && !aligned(dh_n, 16)) ||
      (dc_n && !aligned(dc_n, 16)) || (dz && !aligned(dz, 16)) || (dc0 && !aligned(dc0, 16)))
    return HS_OK;
  if (T >= (1ll << 31) || B >= (1ll << 31) || 4 * H >= (1ll << 31)) return HS_OK;
  const size_t smem = scan_tma_bwd_smem(H);
  if (smem > 220 * 1024) return HS_OK;
  CUtensorMap tz, tc, td;
  if (!map3(&tz, z, 4 * H, B, T, L) || !map3(&tc, c, H, B, T, L) || !map3(&td, dout, H, B, T, L)) return HS_OK;
  Geo g{T, B, H, nchunk, nhb, (unsigned)((int64_t)nchunk * B * nhb)};
  static size_t set_for = 0;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (smem > set_for) {
      cudaFuncSetAttribute((const void *)scan_bwd_tma_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)std::max<size_t>(smem, 160 * 1024));
      set_for = std::max<size_t>(smem, 160 * 1024);
    }
  }
  scan_bwd_tma_kernel<S><<<scan_tma_grid(g.ntiles), NT, smem, st>>>(tz, tc, td, c, c0, dh_n, dc_n, dz, dc0, g, eps,
                                                                    ws, status);
  if (int e = check_launch("scan_bwd_tma_kernel")) return e;
  *done = true;
  return HS_OK;
}

}  // namespace hs
