// Parallel-mode (Heinsen) scan of HeadStartLSTM, forward and backward.
//
// Reference: src/headstartlstm/_parallel.py:21-74 computes
//   c = exp(cumsum(log f') + logcumsumexp(cat[log c0', log b' - cumsum(log f')]))
// with f' = max(sigmoid(z_f), eps), b' = max(sigmoid(z_i) sigmoid(z_g), eps),
// c0' = max(c0, eps), then out = sigmoid(z_o) tanh(c).  That expression is the
// solution of the positive linear recurrence c_t = f'_t c_{t-1} + b'_t,
// c_{-1} = c0'.  These kernels evaluate the recurrence directly: a chunk of
// time steps is summarised by the affine map c_out = A c_in + C
// (A = prod f', C = the chunk's scan from 0), maps compose associatively,
// (A1,C1) then (A2,C2) = (A1 A2, A2 C1 + C2), and the carry into each chunk
// comes from a single-pass decoupled look-back over the chunks before it.
// Every quantity is positive, so nothing cancels: the float32 result tracks
// float64 at any T, where the reference's float32 log-domain form drifts.
//
// The backward is the same construction run from T-1 down to 0 on
// e_t = f'_t (dcd_t + e_{t+1}), the gradient reaching c_{t-1}; the autograd
// backward of _parallel.py:21-74 computes the same quantities through ATen.
//
// Layout: z [T,B,4H] (gate order i,f,g,o), c/out/dout [T,B,H].  A warp owns
// 32*VEC consecutive hidden units (float4 when H%4==0), a thread owns S
// consecutive time steps, a CTA stacks NW warps along time: a tile is
// (L = NW*S steps) x (one sequence b) x (32*VEC units).  Tiles are handed out
// in time-major order by an atomic ticket, so a tile's predecessor has always
// started before it (the look-back can never wait on an unscheduled CTA).
#include <mutex>

#include "hs_common.cuh"

namespace hs {

int scan_tma_fwd_chunk();
int scan_tma_bwd_chunk();
int scan_tma_grid(unsigned ntiles);
int scan_fwd_tma_launch(const float *z, const float *c0, float *out, float *c, float *h_n, float *c_n,
                        int64_t T, int64_t B, int64_t H, float eps, const ScanTmaWs &ws, int nchunk, int nhb,
                        int *status, cudaStream_t st, bool *done);
int scan_bwd_tma_launch(const float *z, const float *c, const float *c0, const float *dout,
                        const float *dh_n, const float *dc_n, float *dz, float *dc0, int64_t T, int64_t B,
                        int64_t H, float eps, const ScanTmaWs &ws, int nchunk, int nhb, int *status,
                        cudaStream_t st, bool *done);

namespace {

struct ScanWs {
  unsigned *ticket;
  unsigned *flags;   // [nslot]: 0 empty, 1 aggregate ready, 2 inclusive ready
  float *agg_a;      // [nslot][HW]
  float *agg_c;      // [nslot][HW]
  float *incl;       // [nslot][HW]
  float *db_part;    // [nchunk*B][4H] (backward only)
};

struct ScanShape {
  int64_t T, B, H;
  int nchunk, nhb;
};

// Tile geometry of the per-tile kernels (compile-time; the defaults are the
// measured best on B200 for the benchmark shapes).
#ifndef HS_SCAN_FWD_S
#define HS_SCAN_FWD_S 4
#endif
#ifndef HS_SCAN_FWD_NW
#define HS_SCAN_FWD_NW 8
#endif
#ifndef HS_SCAN_BWD_S
#define HS_SCAN_BWD_S 4
#endif
#ifndef HS_SCAN_BWD_NW
#define HS_SCAN_BWD_NW 8
#endif
#ifndef HS_SCAN_USE_TMA
#define HS_SCAN_USE_TMA 1
#endif
constexpr int kFwdS = HS_SCAN_FWD_S, kFwdNW = HS_SCAN_FWD_NW;
constexpr int kBwdS = HS_SCAN_BWD_S, kBwdNW = HS_SCAN_BWD_NW;

template <int VEC> __host__ __device__ constexpr int hw() { return 32 * VEC; }

size_t ws_layout(const ScanShape &s, int HW, bool with_db, ScanWs *out, void *base) {
  const int64_t nslot = (int64_t)s.nchunk * s.B * s.nhb;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = round_up(off + bytes, 256);
    return o;
  };
  size_t o_ticket = take(sizeof(unsigned));
  size_t o_flags = take(sizeof(unsigned) * nslot);
  size_t o_a = take(sizeof(float) * nslot * HW);
  size_t o_c = take(sizeof(float) * nslot * HW);
  size_t o_i = take(sizeof(float) * nslot * HW);
  // bias partial rows: one per (chunk, sequence) for the per-tile kernel, one
  // per CTA (<= 256) for the persistent kernel
  const size_t db_rows = std::max<int64_t>((int64_t)s.nchunk * s.B, 256);
  size_t o_db = with_db ? take(sizeof(float) * db_rows * 4 * s.H) : off;
  if (out) {
    char *b = static_cast<char *>(base);
    out->ticket = reinterpret_cast<unsigned *>(b + o_ticket);
    out->flags = reinterpret_cast<unsigned *>(b + o_flags);
    out->agg_a = reinterpret_cast<float *>(b + o_a);
    out->agg_c = reinterpret_cast<float *>(b + o_c);
    out->incl = reinterpret_cast<float *>(b + o_i);
    out->db_part = with_db ? reinterpret_cast<float *>(b + o_db) : nullptr;
  }
  (void)o_db;
  return off;
}

// Bytes of the part of the workspace that must be zero at launch (ticket+flags).
size_t ws_zero_bytes(const ScanShape &s) {
  const int64_t nslot = (int64_t)s.nchunk * s.B * s.nhb;
  return round_up(sizeof(unsigned), 256) + sizeof(unsigned) * nslot;
}

#ifndef HS_SCAN_FAST_SIG
#define HS_SCAN_FAST_SIG 0
#endif
#if HS_SCAN_FAST_SIG
// hardware exp2 with a correctly rounded reciprocal (see scan_tma.cu)
#define sigm(x) __frcp_rn(1.0f + __expf(-(x)))
#endif

// ============================================================== forward
template <int VEC, int S, int NW>
__global__ void __launch_bounds__(NW * 32)
scan_fwd_kernel(const float *__restrict__ z, const float *__restrict__ c0,
                float *__restrict__ out, float *__restrict__ cbuf,
                float *__restrict__ h_n, float *__restrict__ c_n,
                ScanShape sh, float eps, ScanWs ws, int *status) {
  constexpr int HW = hw<VEC>();
  constexpr int L = S * NW;
  __shared__ float sA[NW][HW];
  __shared__ float sC[NW][HW];
  __shared__ float s_carry[HW];
  __shared__ unsigned s_tile;
  __shared__ int s_abort;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    s_tile = atomicAdd(ws.ticket, 1u);
    s_abort = ld_status(status) != 0;
  }
  __syncthreads();
  if (s_abort) return;
  const unsigned tile = s_tile;
  const int64_t T = sh.T, B = sh.B, H = sh.H;
  const unsigned per_chunk = (unsigned)(B * sh.nhb);
  const int j = tile / per_chunk;
  const unsigned r = tile - j * per_chunk;
  const int64_t b = r / sh.nhb;
  const int hb = r - b * sh.nhb;
  const int64_t h = (int64_t)hb * HW + lane * VEC;
  const bool hv = h < H;
  const int64_t t0 = (int64_t)j * L + warp * S;

  // Pass 1: activations and this thread's summary over its S steps.
  float fp[S][VEC], bp[S][VEC], og[S][VEC];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int64_t t = t0 + s;
    if (hv && t < T) {
      const float *zr = z + (t * B + b) * 4 * H + h;
      Vec<VEC> zi, zf, zg, zo;
      zi.load_cs(zr);
      zf.load_cs(zr + H);
      zg.load_cs(zr + 2 * H);
      zo.load_cs(zr + 3 * H);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float ig = sigm(zi.v[v]) * sigm(zg.v[v]);
        fp[s][v] = fmaxf(sigm(zf.v[v]), eps);
        bp[s][v] = fmaxf(ig, eps);
        og[s][v] = sigm(zo.v[v]);
      }
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) { fp[s][v] = 1.f; bp[s][v] = 0.f; og[s][v] = 0.f; }
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
  for (int v = 0; v < VEC; ++v) { sA[warp][lane * VEC + v] = A[v]; sC[warp][lane * VEC + v] = C[v]; }
  __syncthreads();

  // Tile summary, publication and look-back (warp 0; each lane is an
  // independent chain for its VEC hidden units).
  if (warp == 0) {
    float TA[VEC], TC[VEC], cin[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) { TA[v] = 1.f; TC[v] = 0.f; }
#pragma unroll
    for (int w = 0; w < NW; ++w)
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float a = sA[w][lane * VEC + v];
        TC[v] = fmaf(a, TC[v], sC[w][lane * VEC + v]);
        TA[v] *= a;
      }
    const int64_t slot = ((int64_t)j * B + b) * sh.nhb + hb;
    float *my_incl = ws.incl + slot * HW + lane * VEC;
    bool ok = true;
    if (j == 0) {
#pragma unroll
      for (int v = 0; v < VEC; ++v)
        cin[v] = fmaxf((c0 && hv) ? c0[b * H + h + v] : 0.f, eps);
    } else {
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
      for (int k = j - 1; k >= 0; --k) {
        const int64_t ks = ((int64_t)k * B + b) * sh.nhb + hb;
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
      p.store_cg(my_incl);
      __threadfence();
    }
    __syncwarp();
    const bool all_ok = __all_sync(0xffffffffu, ok);
    if (all_ok && lane == 0) st_release(ws.flags + slot, 2u);
    if (lane == 0) s_abort = !all_ok;
#pragma unroll
    for (int v = 0; v < VEC; ++v) s_carry[lane * VEC + v] = cin[v];
  }
  __syncthreads();
  if (s_abort) return;

  // Pass 2: carry into this warp's steps, then the exact recurrence.
  float c[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) c[v] = s_carry[lane * VEC + v];
  for (int w = 0; w < warp; ++w)
#pragma unroll
    for (int v = 0; v < VEC; ++v) c[v] = fmaf(sA[w][lane * VEC + v], c[v], sC[w][lane * VEC + v]);
  if (!hv) return;
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int64_t t = t0 + s;
    if (t >= T) break;
    Vec<VEC> vc, vo;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      c[v] = fmaf(fp[s][v], c[v], bp[s][v]);
      vc.v[v] = c[v];
      vo.v[v] = og[s][v] * tanhf(c[v]);
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

// ============================================================== backward
template <int VEC, int S, int NW>
__global__ void __launch_bounds__(NW * 32)
scan_bwd_kernel(const float *z, const float *__restrict__ cbuf,
                const float *__restrict__ c0, const float *__restrict__ dout,
                const float *__restrict__ dh_n, const float *__restrict__ dc_n,
                float *dz, float *__restrict__ dc0, ScanShape sh, float eps,
                ScanWs ws, int *status) {
  constexpr int HW = hw<VEC>();
  constexpr int L = S * NW;
  __shared__ float sA[NW][HW];
  __shared__ float sC[NW][HW];
  __shared__ float s_carry[HW];
  __shared__ unsigned s_tile;
  __shared__ int s_abort;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    s_tile = atomicAdd(ws.ticket, 1u);
    s_abort = ld_status(status) != 0;
  }
  __syncthreads();
  if (s_abort) return;
  const unsigned tile = s_tile;
  const int64_t T = sh.T, B = sh.B, H = sh.H;
  const unsigned per_chunk = (unsigned)(B * sh.nhb);
  const int q = tile / per_chunk;           // 0 = last chunk in time
  const int j = sh.nchunk - 1 - q;
  const unsigned r = tile - q * per_chunk;
  const int64_t b = r / sh.nhb;
  const int hb = r - b * sh.nhb;
  const int64_t h = (int64_t)hb * HW + lane * VEC;
  const bool hv = h < H;
  const int64_t t0 = (int64_t)j * L + warp * S;

  // Pass 1 (reverse time): per-step coefficients, the o-gate gradient (final
  // already), and this thread's summary of e over its steps.
  float FP[S][VEC], DCD[S][VEC], KI[S][VEC], KF[S][VEC], KG[S][VEC];
  float acc[4][VEC];
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[g][v] = 0.f;
  float cprev[VEC];
  if (hv && t0 < T) {
    if (t0 == 0) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) cprev[v] = fmaxf(c0 ? c0[b * H + h + v] : 0.f, eps);
    } else {
      Vec<VEC> t;
      t.load(cbuf + ((t0 - 1) * B + b) * H + h);
#pragma unroll
      for (int v = 0; v < VEC; ++v) cprev[v] = t.v[v];
    }
  }
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int64_t t = t0 + s;
    if (hv && t < T) {
      const int64_t zo = (t * B + b) * 4 * H + h;
      const int64_t so = (t * B + b) * H + h;
      Vec<VEC> zi, zf, zg, zz, vc, vd;
      zi.load_cs(z + zo);
      zf.load_cs(z + zo + H);
      zg.load_cs(z + zo + 2 * H);
      zz.load_cs(z + zo + 3 * H);
      vc.load(cbuf + so);
      vd.load_cs(dout + so);
      if (t == T - 1 && dh_n) {
        Vec<VEC> e;
        e.load(dh_n + b * H + h);
#pragma unroll
        for (int v = 0; v < VEC; ++v) vd.v[v] += e.v[v];
      }
      Vec<VEC> dzo;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float i = sigm(zi.v[v]), f = sigm(zf.v[v]), g = sigm(zg.v[v]), o = sigm(zz.v[v]);
        const float th = tanhf(vc.v[v]);
        const float mb = (i * g >= eps) ? 1.f : 0.f;
        const float mf = (f >= eps) ? 1.f : 0.f;
        FP[s][v] = fmaxf(f, eps);
        DCD[s][v] = vd.v[v] * o * (1.f - th * th);
        KI[s][v] = g * i * (1.f - i) * mb;
        KF[s][v] = cprev[v] * f * (1.f - f) * mf;
        KG[s][v] = i * g * (1.f - g) * mb;
        dzo.v[v] = vd.v[v] * th * o * (1.f - o);
        acc[3][v] += dzo.v[v];
        cprev[v] = vc.v[v];
      }
      if (t == T - 1 && dc_n) {
        Vec<VEC> e;
        e.load(dc_n + b * H + h);
#pragma unroll
        for (int v = 0; v < VEC; ++v) DCD[s][v] += e.v[v];
      }
      dzo.store_cs(dz + zo + 3 * H);
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) { FP[s][v] = 1.f; DCD[s][v] = 0.f; KI[s][v] = KF[s][v] = KG[s][v] = 0.f; }
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
  for (int v = 0; v < VEC; ++v) { sA[warp][lane * VEC + v] = A[v]; sC[warp][lane * VEC + v] = C[v]; }
  __syncthreads();

  if (warp == 0) {
    float TA[VEC], TC[VEC], cin[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) { TA[v] = 1.f; TC[v] = 0.f; cin[v] = 0.f; }
#pragma unroll
    for (int w = NW - 1; w >= 0; --w)
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float a = sA[w][lane * VEC + v];
        TC[v] = fmaf(a, TC[v], sC[w][lane * VEC + v]);
        TA[v] *= a;
      }
    const int64_t slot = ((int64_t)q * B + b) * sh.nhb + hb;
    bool ok = true;
    if (q > 0) {
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
      for (int k = q - 1; k >= 0; --k) {
        const int64_t ks = ((int64_t)k * B + b) * sh.nhb + hb;
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
    if (lane == 0) s_abort = !all_ok;
#pragma unroll
    for (int v = 0; v < VEC; ++v) s_carry[lane * VEC + v] = cin[v];
  }
  __syncthreads();
  if (s_abort) return;

  // Pass 2: e entering this warp's last step, then the exact reverse recurrence.
  float e[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) e[v] = s_carry[lane * VEC + v];
  for (int w = NW - 1; w > warp; --w)
#pragma unroll
    for (int v = 0; v < VEC; ++v) e[v] = fmaf(sA[w][lane * VEC + v], e[v], sC[w][lane * VEC + v]);
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

  // Per-chunk column sums of dz for the bias gradient (deterministic order).
  if (ws.db_part) {
    __syncthreads();
    float *red = &sA[0][0];  // reuse: NW x HW floats per gate
#pragma unroll
    for (int g = 0; g < 4; ++g) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) red[warp * HW + lane * VEC + v] = acc[g][v];
      __syncthreads();
      if (warp == 0 && hv) {
        Vec<VEC> sum;
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          float a = 0.f;
          for (int w = 0; w < NW; ++w) a += red[w * HW + lane * VEC + v];
          sum.v[v] = a;
        }
        sum.store(ws.db_part + ((int64_t)j * B + b) * 4 * H + g * H + h);
      }
      __syncthreads();
    }
  }
}

// db[n] = beta*db[n] + sum_r part[r][n], fixed summation order.
__global__ void rowsum_kernel(const float *__restrict__ part, float *__restrict__ db,
                              int64_t R, int64_t N, int beta) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int64_t r = 0;
  for (; r + 4 <= R; r += 4) {
    s0 += part[(r + 0) * N + n];
    s1 += part[(r + 1) * N + n];
    s2 += part[(r + 2) * N + n];
    s3 += part[(r + 3) * N + n];
  }
  for (; r < R; ++r) s0 += part[r * N + n];
  const float s = (s0 + s1) + (s2 + s3);
  db[n] = beta ? db[n] + s : s;
}

int pick_vec(int64_t H, std::initializer_list<const void *> ptrs) {
  if (H % 4 == 0) {
    bool ok = true;
    for (const void *p : ptrs) ok = ok && (p == nullptr || aligned(p, 16));
    if (ok) return 4;
  }
  return 1;
}

ScanShape make_shape(int64_t T, int64_t B, int64_t H, int L, int HW) {
  ScanShape s;
  s.T = T;
  s.B = B;
  s.H = H;
  s.nchunk = (int)((T + L - 1) / L);
  s.nhb = (int)((H + HW - 1) / HW);
  return s;
}

size_t scan_ws_bytes(int64_t T, int64_t B, int64_t H) {
  size_t m = 0;
  for (int HW : {32, 128}) {
    for (int L : {kFwdS * kFwdNW, kBwdS * kBwdNW, scan_tma_fwd_chunk(), scan_tma_bwd_chunk()}) {
      ScanShape f = make_shape(T, B, H, L, HW);
      m = std::max(m, ws_layout(f, HW, false, nullptr, nullptr));
      m = std::max(m, ws_layout(f, HW, true, nullptr, nullptr));
    }
  }
  return m;
}

int check_scan_args(int64_t T, int64_t B, int64_t H) {
  if (T <= 0 || B <= 0 || H <= 0) return fail(HS_ERR_INVALID_ARG, "T, B, H must be positive (got %lld, %lld, %lld)", (long long)T, (long long)B, (long long)H);
  if ((T + 31) / 32 * B * ((H + 31) / 32) >= (1ll << 31)) return fail(HS_ERR_UNSUPPORTED, "scan grid too large");
  if (B * 4 * H >= (1ll << 40)) return fail(HS_ERR_UNSUPPORTED, "B*4H too large");
  return HS_OK;
}

}  // namespace

size_t scan_workspace(int64_t T, int64_t B, int64_t H) { return scan_ws_bytes(T, B, H); }

// ------------------------------------------------------------------ host API
int scan_forward(const float *z, const float *c0, float *out, float *c, float *h_n,
                 float *c_n, int64_t T, int64_t B, int64_t H, float eps, void *ws_base,
                 size_t ws_bytes, int *status, cudaStream_t st) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !out || !c || !status) return fail(HS_ERR_INVALID_ARG, "scan_forward: null z/out/c/status");
  const int VEC = pick_vec(H, {z, c0, out, c, h_n, c_n});
  const int HW = 32 * VEC;
  if (!ws_base || !aligned(ws_base, 256)) return fail(HS_ERR_INVALID_ARG, "workspace must be non-null and 256-byte aligned");
  if (VEC == 4 && HS_SCAN_USE_TMA) {  // persistent TMA kernel
    ScanShape sh = make_shape(T, B, H, scan_tma_fwd_chunk(), HW);
    ScanWs w;
    const size_t need = ws_layout(sh, HW, false, &w, ws_base);
    if (ws_bytes < need) return fail(HS_ERR_WORKSPACE, "scan_forward: workspace %zu < %zu bytes", ws_bytes, need);
    if (cudaMemsetAsync(ws_base, 0, ws_zero_bytes(sh), st) != cudaSuccess) return check_launch("scan_forward memset");
    ScanTmaWs tw{w.ticket, w.flags, w.agg_a, w.agg_c, w.incl, nullptr};
    bool done = false;
    if (int e = scan_fwd_tma_launch(z, c0, out, c, h_n, c_n, T, B, H, eps, tw, sh.nchunk, sh.nhb, status, st, &done)) return e;
    if (done) return HS_OK;
  }
  ScanShape sh = make_shape(T, B, H, kFwdS * kFwdNW, HW);
  ScanWs ws;
  const size_t need = ws_layout(sh, HW, false, &ws, ws_base);
  if (ws_bytes < need) return fail(HS_ERR_WORKSPACE, "scan_forward: workspace %zu < %zu bytes", ws_bytes, need);
  if (cudaMemsetAsync(ws_base, 0, ws_zero_bytes(sh), st) != cudaSuccess) return check_launch("scan_forward memset");
  const unsigned ntile = (unsigned)((int64_t)sh.nchunk * B * sh.nhb);
  if (VEC == 4)
    scan_fwd_kernel<4, kFwdS, kFwdNW><<<ntile, kFwdNW * 32, 0, st>>>(z, c0, out, c, h_n, c_n, sh, eps, ws, status);
  else
    scan_fwd_kernel<1, kFwdS, kFwdNW><<<ntile, kFwdNW * 32, 0, st>>>(z, c0, out, c, h_n, c_n, sh, eps, ws, status);
  return check_launch("scan_fwd_kernel");
}

int scan_backward(const float *z, const float *c, const float *c0, const float *dout,
                  const float *dh_n, const float *dc_n, float *dz, float *dc0, float *db,
                  int64_t T, int64_t B, int64_t H, float eps, void *ws_base, size_t ws_bytes,
                  int *status, cudaStream_t st) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !c || !dout || !dz || !status) return fail(HS_ERR_INVALID_ARG, "scan_backward: null z/c/dout/dz/status");
  const int VEC = pick_vec(H, {z, c, c0, dout, dh_n, dc_n, dz, dc0});
  const int HW = 32 * VEC;
  if (!ws_base || !aligned(ws_base, 256)) return fail(HS_ERR_INVALID_ARG, "workspace must be non-null and 256-byte aligned");
  if (VEC == 4 && HS_SCAN_USE_TMA) {  // persistent TMA kernel
    ScanShape sh = make_shape(T, B, H, scan_tma_bwd_chunk(), HW);
    ScanWs w;
    const size_t need = ws_layout(sh, HW, db != nullptr, &w, ws_base);
    if (ws_bytes < need) return fail(HS_ERR_WORKSPACE, "scan_backward: workspace %zu < %zu bytes", ws_bytes, need);
    if (cudaMemsetAsync(ws_base, 0, ws_zero_bytes(sh), st) != cudaSuccess) return check_launch("scan_backward memset");
    ScanTmaWs tw{w.ticket, w.flags, w.agg_a, w.agg_c, w.incl, w.db_part};
    bool done = false;
    if (int e = scan_bwd_tma_launch(z, c, c0, dout, dh_n, dc_n, dz, dc0, T, B, H, eps, tw, sh.nchunk, sh.nhb, status,
                                    st, &done))
      return e;
    if (done) {
      if (db) {
        const int64_t N = 4 * H;
        const int64_t R = scan_tma_grid((unsigned)((int64_t)sh.nchunk * B * sh.nhb));
        rowsum_kernel<<<(unsigned)((N + 255) / 256), 256, 0, st>>>(w.db_part, db, R, N, 0);
        return check_launch("rowsum_kernel");
      }
      return HS_OK;
    }
  }
  ScanShape sh = make_shape(T, B, H, kBwdS * kBwdNW, HW);
  ScanWs ws;
  const size_t need = ws_layout(sh, HW, db != nullptr, &ws, ws_base);
  if (ws_bytes < need) return fail(HS_ERR_WORKSPACE, "scan_backward: workspace %zu < %zu bytes", ws_bytes, need);
  if (cudaMemsetAsync(ws_base, 0, ws_zero_bytes(sh), st) != cudaSuccess) return check_launch("scan_backward memset");
  const unsigned ntile = (unsigned)((int64_t)sh.nchunk * B * sh.nhb);
  if (VEC == 4)
    scan_bwd_kernel<4, kBwdS, kBwdNW><<<ntile, kBwdNW * 32, 0, st>>>(z, c, c0, dout, dh_n, dc_n, dz, dc0, sh, eps, ws, status);
  else
    scan_bwd_kernel<1, kBwdS, kBwdNW><<<ntile, kBwdNW * 32, 0, st>>>(z, c, c0, dout, dh_n, dc_n, dz, dc0, sh, eps, ws, status);
  if (int e = check_launch("scan_bwd_kernel")) return e;
  if (db) {
    const int64_t N = 4 * H, R = (int64_t)sh.nchunk * B;
    rowsum_kernel<<<(unsigned)((N + 255) / 256), 256, 0, st>>>(ws.db_part, db, R, N, 0);
    return check_launch("rowsum_kernel");
  }
  return HS_OK;
}

// ------------------------------------------------------------------ no-allocation variant
// Some callers cannot allocate device memory at all: a host framework that
// hands this library only its input and output buffers (no device allocator
// of its own), or a latency-critical path where cudaMalloc's implicit device
// synchronisation is not acceptable.  hs_scan_forward_noalloc serves them:
// its look-back scratch lives in this fixed, file-scope device array instead
// of a caller workspace.  Every GPU that loads the library holds the array
// until the process exits.
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int g_noalloc_status;

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices];
int *g_noalloc_status_ptr[kMaxDevices];

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, once per device with that device current.
int noalloc_scratch(void **scratch, int **status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(HS_ERR_CUDA, "hs_scan_forward_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    int *q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(HS_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    e = cudaGetSymbolAddress((void **)&q, g_noalloc_status);
    if (e != cudaSuccess)
      return fail(HS_ERR_CUDA, "cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
    g_noalloc_status_ptr[dev] = q;
  }
  *scratch = g_noalloc_ptr[dev];
  *status = g_noalloc_status_ptr[dev];
  return HS_OK;
}
}  // namespace

int scan_forward_noalloc(const float *z, const float *c0, float *out, float *c, float *h_n,
                         float *c_n, int64_t T, int64_t B, int64_t H, float eps,
                         int *dev_status, cudaStream_t st) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !out || !c) return fail(HS_ERR_INVALID_ARG, "scan_forward_noalloc: null z/out/c");
  const int VEC = pick_vec(H, {z, c0, out, c, h_n, c_n});
  const int HW = 32 * VEC;
  const size_t need = ws_layout(make_shape(T, B, H, kFwdS * kFwdNW, HW), HW, false, nullptr, nullptr);
  if (need > kNoAllocScratchBytes)
    return fail(HS_ERR_UNSUPPORTED,
                "hs_scan_forward_noalloc: T=%lld B=%lld H=%lld needs %zu bytes of scratch, above "
                "the fixed %zu-byte array; use hs_scan_forward with a caller workspace",
                (long long)T, (long long)B, (long long)H, need, kNoAllocScratchBytes);
  void *scratch = nullptr;
  int *own_status = nullptr;
  if (int e = noalloc_scratch(&scratch, &own_status)) return e;
  // scan_forward clears the ticket and flags (all that must start at zero)
  // with a stream-ordered memset before its launch.
  return scan_forward(z, c0, out, c, h_n, c_n, T, B, H, eps, scratch, kNoAllocScratchBytes,
                      dev_status ? dev_status : own_status, st);
}

}  // namespace hs

extern "C" {

size_t hs_scan_workspace_bytes(int64_t T, int64_t B, int64_t H) {
  if (T <= 0 || B <= 0 || H <= 0) return 0;
  return hs::scan_ws_bytes(T, B, H);
}

int hs_scan_forward(const float *z, const float *c0, float *out, float *c, float *h_n,
                    float *c_n, int64_t T, int64_t B, int64_t H, float eps,
                    void *workspace, size_t workspace_bytes, int *dev_status,
                    hs_stream_t stream) {
  return hs::scan_forward(z, c0, out, c, h_n, c_n, T, B, H, eps, workspace, workspace_bytes,
                          dev_status, (cudaStream_t)stream);
}

int hs_scan_backward(const float *z, const float *c, const float *c0, const float *dout,
                     const float *dh_n, const float *dc_n, float *dz, float *dc0, float *db,
                     int64_t T, int64_t B, int64_t H, float eps, void *workspace,
                     size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::scan_backward(z, c, c0, dout, dh_n, dc_n, dz, dc0, db, T, B, H, eps, workspace,
                           workspace_bytes, dev_status, (cudaStream_t)stream);
}

int hs_scan_forward_noalloc(const float *z, const float *c0, float *out, float *c, float *h_n,
                            float *c_n, int64_t T, int64_t B, int64_t H, float eps,
                            int *dev_status, hs_stream_t stream) {
  return hs::scan_forward_noalloc(z, c0, out, c, h_n, c_n, T, B, H, eps, dev_status,
                                  (cudaStream_t)stream);
}

}  // extern "C"
