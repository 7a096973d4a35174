// Recurrent-mode HeadStartLSTM: one persistent kernel per direction.
//
// Reference: HeadStartLSTMTorchFn (src/headstartlstm/_torch.py:86-170) and
// HeadStartLSTMTritonFn (src/headstartlstm/_triton.py:331-465) run a host loop
// of T steps, each a cuBLAS GEMM h.(a*W_hh)^T plus a fused cell launch, and a
// reverse loop of cell-backward launches and dgates.(a*W_hh) GEMMs.  Here each
// direction is ONE cooperative launch that keeps every CTA resident for all T
// steps:
//   * CTA c owns U consecutive hidden units and therefore the 4U rows
//     {g*H+u} of W_hh; its slice of a*W_hh (forward: [H][4U], k-major;
//     backward: [4H][U]) stays in shared memory for the whole launch when it
//     fits, and is streamed from L2 in K-chunks otherwise.
//   * Per step the CTA computes its [4U x B] block of gates (backward:
//     [U x B] block of dh) with FFMA: the K axis is split across the 8 warps
//     and across KSL lanes of each warp, each lane accumulates a 4-row x
//     4-batch register tile, then shuffles and shared memory reduce.
//   * The per-step state that crosses CTAs (h_t forward, dgates_t backward)
//     goes through a small double-buffered, k-major exchange buffer in global
//     memory (L2-resident), copied into shared memory with cp.async.cg
//     (L2 only, never a stale L1 line), and one grid barrier per step.
//   * Gate scaling by a, the sigmoid-g cell, the c/h update and the stores of
//     h, c and the activations (forward), and the cell backward with the
//     dgates store (backward) are fused into the step's epilogue.
// Every wait is bounded (kWaitLimitNs); a CTA that gives up records
// HS_ERR_DEVICE_TIMEOUT in the caller's status word and leaves.
#include <cooperative_groups.h>

#include <algorithm>

#include "hs_common.cuh"

namespace hs {

int linear_forward(const float *x, const float *w, const float *bias, float *y, int64_t M,
                   int64_t N, int64_t K, void *ws, size_t ws_bytes, int *status, cudaStream_t st);
int linear_dgrad(const float *dy, const float *w, float *dx, int64_t M, int64_t N, int64_t K,
                 void *ws, size_t ws_bytes, int *status, cudaStream_t st);
int linear_wgrad(const float *dy, const float *x, float *dw, int64_t M, int64_t N, int64_t K,
                 int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st);
size_t linear_ws_bytes(int64_t M, int64_t N, int64_t K);
size_t linear_backward_ws(int64_t M, int64_t N, int64_t K, int64_t K2);
int linear_backward_ex(const float *dy, const float *w, float *dx, const float *x, float *dw, const float *x2,
                       float *dw2, int64_t M, int64_t N, int64_t K, int64_t K2, int beta, void *ws, size_t ws_bytes,
                       int *status, cudaStream_t st, const unsigned *dy_absmax);
int colsum(const float *x, float *out, int64_t M, int64_t N, int beta, cudaStream_t st, void *ws = nullptr,
           size_t ws_bytes = 0);
bool rec_tc_wanted(int dir, int64_t B, int64_t H, bool bf = false);
bool rec_cluster_wanted(int64_t B, int64_t H);
size_t rec_cluster_ws_bytes(int64_t H);
bool rec_wide_wanted(int64_t B, int64_t H);
size_t rec_wide_ws_bytes(int64_t H);
int rec_wide_forward(const float *h0, const float *c0, const float *w_hh, const float *b_hh, const float *a,
                     float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t H, void *ws,
                     size_t ws_bytes, int *status, cudaStream_t st);
int rec_wide_backward(const float *w_hh, const float *a, const float *c_save, float *acts, const float *dout,
                      const float *dh_n, const float *dc_n, int64_t T, int64_t B, int64_t H, void *ws,
                      size_t ws_bytes, int *status, cudaStream_t st);
int rec_cluster_forward(const float *h0, const float *c0, const float *w_hh, const float *b_hh, const float *a,
                        float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t H, void *ws,
                        size_t ws_bytes, int *status, cudaStream_t st);
int rec_cluster_backward(const float *w_hh, const float *a, const float *c_save, float *acts, const float *dout,
                         const float *dh_n, const float *dc_n, int64_t T, int64_t B, int64_t H, void *ws,
                         size_t ws_bytes, int *status, cudaStream_t st);
size_t rec_tc_ws_bytes(int64_t B, int64_t H);
int rec_tc_forward(const float *h0, const float *c0, const float *w_hh, const float *b_hh, const float *a,
                   float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t H, void *ws,
                   size_t ws_bytes, int *status, cudaStream_t st, bool bf);
int rec_tc_backward(const float *w_hh, const float *a, const float *c_save, float *acts, const float *dout,
                    const float *dh_n, const float *dc_n, int64_t T, int64_t B, int64_t H, void *ws, size_t ws_bytes,
                    int *status, cudaStream_t st, bool bf);

namespace {

#ifndef HS_REC_KUNROLL
#define HS_REC_KUNROLL 8
#endif
constexpr int kKUnroll = HS_REC_KUNROLL;  // k-loop unroll of the step matvec
#ifndef HS_REC_NW
#define HS_REC_NW 8
#endif
constexpr int NW = HS_REC_NW;  // warps per CTA
constexpr int NT = NW * 32;
constexpr int kMaxPairs = 4;   // (unit, batch) pairs per thread in the epilogue
constexpr int kMaxBatch = 32;  // batch rows per launch (larger B: several launches)
constexpr size_t kSmemBudget = 216 * 1024;
// Chunk buffers of the step matvec: chunks c+1 .. c+kStages-1 are in flight
// (cp.async) while chunk c is multiplied, hiding the L2 latency of the
// streamed operands (exchange rows, and weights when not resident).
constexpr int kStages = 4;

// ------------------------------------------------------------------ plan
struct Dir {
  int RG, NRT, rows_pad, KSL, KC;
  int64_t K, K_pad;
  bool resident;
  size_t smem;
};
struct Plan {
  int BP, BG, U, ncta;
  Dir fwd, bwd;
  // workspace offsets (bytes)
  size_t o_bar, o_wf, o_bf, o_wb, o_xf, o_xb, total;
};

int pow2ceil(int x) { int p = 1; while (p < x) p <<= 1; return p; }

bool plan_dir(Dir &d, int rows, int BG, int64_t K) {
  const int rg_max = std::min(8, 32 / BG);
  d.RG = std::min(rg_max, pow2ceil((rows + 3) / 4));
  d.NRT = (rows + 4 * d.RG - 1) / (4 * d.RG);
  if (d.NRT > 4) return false;
  d.rows_pad = d.NRT * 4 * d.RG;
  d.KSL = 32 / (BG * d.RG);
  d.K = K;
  return true;
}

// Largest chunk of the step matvec's k range (smaller chunks start the
// multiply sooner after the step's exchange rows begin to arrive).
#ifndef HS_REC_KC_MAX
#define HS_REC_KC_MAX 256
#endif

void size_dir(Dir &d, int BP) {
  const size_t red = (size_t)NW * d.rows_pad * BP * 4;
  for (int kc : {256, 128, 64, 32}) {
    if (kc > HS_REC_KC_MAX) continue;
    d.KC = kc;
    d.K_pad = (d.K + kc - 1) / kc * kc;
    const size_t xbuf = (size_t)kStages * kc * BP * 4;
    const size_t wres = (size_t)d.K_pad * d.rows_pad * 4;
    if (wres + xbuf + red <= kSmemBudget) { d.resident = true; d.smem = wres + xbuf + red; return; }
  }
  d.resident = false;
  for (int kc : {128, 64, 32}) {
    if (kc > HS_REC_KC_MAX && kc > 32) continue;
    d.KC = kc;
    d.K_pad = (d.K + kc - 1) / kc * kc;
    d.smem = (size_t)kStages * kc * (BP + d.rows_pad) * 4 + red;
    if (d.smem <= kSmemBudget) return;
  }
}

bool make_plan(Plan &p, int64_t B, int64_t H, int nsm) {
  const int Bc = (int)std::min<int64_t>(B, kMaxBatch);
  p.BP = Bc <= 4 ? 4 : Bc <= 8 ? 8 : Bc <= 16 ? 16 : 32;
  p.BG = p.BP / 4;
  const int rg_max = std::min(8, 32 / p.BG);
  int U = (int)((H + nsm - 1) / nsm);
  U = std::max(U, rg_max);
  U = (U + rg_max - 1) / rg_max * rg_max;
  U = (int)std::min<int64_t>(U, H);
  p.U = U;
  p.ncta = (int)((H + U - 1) / U);
  if (p.ncta > nsm) return false;
  if ((int64_t)U * p.BP > (int64_t)kMaxPairs * NT) return false;
  if (!plan_dir(p.fwd, 4 * U, p.BG, H)) return false;
  if (!plan_dir(p.bwd, U, p.BG, 4 * H)) return false;
  size_dir(p.fwd, p.BP);
  size_dir(p.bwd, p.BP);
  if (p.fwd.smem > kSmemBudget || p.bwd.smem > kSmemBudget) return false;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = round_up(off + bytes, 256); return o; };
  p.o_bar = take(256);
  p.o_wf = take((size_t)p.ncta * p.fwd.K_pad * p.fwd.rows_pad * 4);
  p.o_bf = take((size_t)p.ncta * p.fwd.rows_pad * 4);
  p.o_wb = take((size_t)p.ncta * p.bwd.K_pad * p.bwd.rows_pad * 4);
  p.o_xf = take(2ull * p.fwd.K_pad * p.BP * 4);
  p.o_xb = take(2ull * p.bwd.K_pad * p.BP * 4);
  p.total = off;
  return true;
}

// ------------------------------------------------------------------ prologue
// Wf[c][k][ri] = a[g] W_hh[g*H+u][k], ri = ul*4+g, u = c*U+ul   (forward slice)
// bf[c][ri]    = a[g] b_hh[g*H+u]
// Wb[c][r][ul] = a[g(r)] W_hh[r][c*U+ul]                          (backward slice)
// wf/bf are built when wf != null (forward), wb when wb != null (backward).
__global__ void rec_prep_kernel(const float *__restrict__ w_hh, const float *__restrict__ b_hh,
                                const float *__restrict__ a, float *__restrict__ wf,
                                float *__restrict__ bf, float *__restrict__ wb, int64_t H, int U,
                                int ncta, int rpf, int64_t kpf, int rpb, int64_t kpb) {
  const int64_t nf = wf ? (int64_t)ncta * kpf * rpf : 0;
  const int64_t nb = wb ? (int64_t)ncta * kpb * rpb : 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nbias = wf ? (int64_t)ncta * rpf : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nf + nb + nbias; i += stride) {
    if (i < nf) {
      const int ri = (int)(i % rpf);
      const int64_t k = (i / rpf) % kpf;
      const int c = (int)(i / ((int64_t)rpf * kpf));
      const int ul = ri / 4, g = ri % 4;
      const int64_t u = (int64_t)c * U + ul;
      float v = 0.f;
      if (ul < U && u < H && k < H) v = a[g] * w_hh[(g * H + u) * H + k];
      wf[i] = v;
    } else if (i < nf + nb) {
      const int64_t j = i - nf;
      const int ul = (int)(j % rpb);
      const int64_t r = (j / rpb) % kpb;
      const int c = (int)(j / ((int64_t)rpb * kpb));
      const int64_t u = (int64_t)c * U + ul;
      float v = 0.f;
      if (ul < U && u < H && r < 4 * H) v = a[r / H] * w_hh[r * H + u];
      wb[j] = v;
    } else {
      const int64_t j = i - nf - nb;
      const int ri = (int)(j % rpf);
      const int c = (int)(j / rpf);
      const int ul = ri / 4, g = ri % 4;
      const int64_t u = (int64_t)c * U + ul;
      bf[j] = (ul < U && u < H) ? a[g] * b_hh[g * H + u] : 0.f;
    }
  }
}

// Forward slices as a tiled transpose: block (c, k-tile) reads the CTA's
// weight rows {g*H + u} for 32 consecutive k (coalesced along k) into shared
// memory and writes wf[c][k][ri] for those k (coalesced along ri).  Rows of
// the slice beyond 4U, units beyond H and k beyond H are written as zero.
__global__ void __launch_bounds__(256) rec_prep_fwd_kernel(const float *__restrict__ w_hh,
                                                           const float *__restrict__ b_hh,
                                                           const float *__restrict__ a, float *__restrict__ wf,
                                                           float *__restrict__ bf, int64_t H, int U, int rpf,
                                                           int64_t kpf) {
  __shared__ float tile[256][33];  // [ri][k] (rpf <= 256)
  const int c = blockIdx.y;
  const int64_t k0 = (int64_t)blockIdx.x * 32;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int ri = w; ri < rpf; ri += 8) {
    const int ul = ri / 4, g = ri % 4;
    const int64_t u = (int64_t)c * U + ul, k = k0 + lane;
    float v = 0.f;
    if (ul < U && u < H && k < H) v = a[g] * w_hh[(g * H + u) * H + k];
    tile[ri][lane] = v;
  }
  __syncthreads();
  float *dst = wf + ((int64_t)c * kpf + k0) * rpf;
  for (int i = threadIdx.x; i < 32 * rpf; i += 256) {
    const int kk = i / rpf, ri = i - kk * rpf;
    if (k0 + kk < kpf) dst[(int64_t)kk * rpf + ri] = tile[ri][kk];
  }
  if (blockIdx.x == 0) {
    for (int ri = threadIdx.x; ri < rpf; ri += 256) {
      const int ul = ri / 4, g = ri % 4;
      const int64_t u = (int64_t)c * U + ul;
      bf[(int64_t)c * rpf + ri] = (ul < U && u < H) ? a[g] * b_hh[g * H + u] : 0.f;
    }
  }
}

// ------------------------------------------------------------------ device pieces
HS_DEV void cp_async16(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
HS_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> HS_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

HS_DEV void copy_chunk(float *dst, const float *src, int nfloat) {
  for (int i = threadIdx.x; i < nfloat / 4; i += NT) cp_async16(dst + 4 * i, src + 4 * i);
}

// Grid barrier on a monotonically increasing counter.  Returns false (and the
// status word is set) if the wait gave up.
HS_DEV bool grid_barrier(unsigned *bar, unsigned target, int *status) {
  __syncthreads();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    __threadfence();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    int ok = 1;
    unsigned v = ld_acquire(bar);
    if (v < target) {
      const uint64_t t0 = globaltimer();
      unsigned polls = 0;
      while ((v = ld_acquire(bar)) < target) {
        if ((++polls & 255u) == 0) {
          if (ld_status(status) != 0) { ok = 0; break; }
          if (globaltimer() - t0 > kWaitLimitNs) { set_status(status, HS_ERR_DEVICE_TIMEOUT); ok = 0; break; }
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// K-split FFMA matvec of one step: out[rows_pad][BP] += W[K][rows_pad]^T-contract X[K][BP].
// W: resident smem (wres != null) or streamed from global wsrc; X streamed from xsrc.
// Leaves the per-warp partials in red[NW][rows_pad][BP].
// NR: row tiles per thread the kernel is compiled for (d.NRT <= NR); the
// accumulators take NR x 16 registers, so small row counts get small kernels.
template <int BG, int RG, int NR>
HS_DEV void step_matvec(const float *wres, const float *wsrc, const float *xsrc, float *xbuf,
                        float *wbuf, float *red, const Dir &d, int BP) {
  constexpr int KSL = 32 / (BG * RG);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ks = lane % KSL;
  const int bg = (lane / KSL) % BG;
  const int rg = lane / (KSL * BG);
  const int q = warp * KSL + ks;  // k-lane index within a chunk
  const int QN = NW * KSL;
  const int rp = d.rows_pad;
  float acc[NR][4][4];
#pragma unroll
  for (int rt = 0; rt < NR; ++rt)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[rt][i][j] = 0.f;

  const int nchunk = (int)(d.K_pad / d.KC);
  const int xfl = d.KC * BP, wfl = d.KC * rp;
  // prologue: chunks 0 .. kStages-2 (one commit group each, empty past the end)
#pragma unroll
  for (int c = 0; c < kStages - 1; ++c) {
    if (c < nchunk) {
      copy_chunk(xbuf + c * xfl, xsrc + (int64_t)c * xfl, xfl);
      if (!wres) copy_chunk(wbuf + c * wfl, wsrc + (int64_t)c * wfl, wfl);
    }
    cp_async_commit();
  }
  for (int c = 0; c < nchunk; ++c) {
    const int cur = c % kStages;
    // refill the buffer that chunk c-1 used (every thread left it at the
    // barrier closing iteration c-1) with chunk c + kStages - 1
    const int nxt = c + kStages - 1;
    if (nxt < nchunk) {
      const int b = nxt % kStages;
      copy_chunk(xbuf + b * xfl, xsrc + (int64_t)nxt * xfl, xfl);
      if (!wres) copy_chunk(wbuf + b * wfl, wsrc + (int64_t)nxt * wfl, wfl);
    }
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // chunk c has landed
    __syncthreads();
    const float *X = xbuf + cur * xfl;
    const float *W = wres ? wres + (int64_t)c * wfl : wbuf + cur * wfl;
#pragma unroll kKUnroll
    for (int k = q; k < d.KC; k += QN) {
      const float4 xv = *reinterpret_cast<const float4 *>(X + k * BP + bg * 4);
#pragma unroll
      for (int rt = 0; rt < NR; ++rt) {
        if (rt < d.NRT) {
          const float4 wv = *reinterpret_cast<const float4 *>(W + k * rp + rt * RG * 4 + rg * 4);
          const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
          const float x4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[rt][i][j] = fmaf(w4[i], x4[j], acc[rt][i][j]);
        }
      }
    }
    __syncthreads();
  }
  // reduce over the KSL lanes of the warp that share (rg, bg)
#pragma unroll
  for (int off = 1; off < KSL; off <<= 1)
#pragma unroll
    for (int rt = 0; rt < NR; ++rt)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[rt][i][j] += __shfl_xor_sync(0xffffffffu, acc[rt][i][j], off);
  if (ks == 0) {
#pragma unroll
    for (int rt = 0; rt < NR; ++rt) {
      if (rt < d.NRT) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float *dst = red + ((int64_t)warp * rp + rt * RG * 4 + rg * 4 + i) * BP + bg * 4;
          *reinterpret_cast<float4 *>(dst) = make_float4(acc[rt][i][0], acc[rt][i][1], acc[rt][i][2], acc[rt][i][3]);
        }
      }
    }
  }
  __syncthreads();
}

HS_DEV float red_sum(const float *red, int rp, int BP, int row, int b) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) s += red[((int64_t)w * rp + row) * BP + b];
  return s;
}

struct RecArgs {
  float *zacts;          // [T,Bt,4H] in: Z, out: activations (fwd) / in: acts, out: dG (bwd)
  const float *h0, *c0;  // [Bt,H] or null
  float *h_save, *c_save;  // [T+1,Bt,H]
  const float *dout, *dh_n, *dc_n;
  const float *wf, *bf, *wb;
  float *xf, *xb;        // exchange buffers [2][K_pad][BP]
  unsigned *bar;
  int *status;
  int64_t T, Bt, H;
  int b_off, Bc, U, ncta;
  Dir d;
  int BP;
};

// ------------------------------------------------------------------ forward
template <int BG, int RG, int NR>
__global__ void __launch_bounds__(NT, 1) rec_fwd_kernel(RecArgs p) {
  extern __shared__ __align__(16) float smem[];
  const Dir &d = p.d;
  const int BP = p.BP, rp = d.rows_pad;
  const int cta = blockIdx.x;
  float *wres = d.resident ? smem : nullptr;
  float *xbuf = smem + (d.resident ? d.K_pad * rp : 0);
  float *wbuf = xbuf + kStages * d.KC * BP;
  float *red = wbuf + (d.resident ? 0 : kStages * d.KC * rp);
  const float *wsrc = p.wf + (int64_t)cta * d.K_pad * rp;
  const int64_t H = p.H, Bt = p.Bt;
  const int u0 = cta * p.U;
  const int Uc = (int)min((int64_t)p.U, H - u0);

  if (wres) {
    for (int i = threadIdx.x; i < d.K_pad * rp / 4; i += NT)
      reinterpret_cast<float4 *>(wres)[i] = reinterpret_cast<const float4 *>(wsrc)[i];
  }
  // Epilogue pairs (ul, b) owned by this thread for the whole launch.
  const int npairs = Uc * p.Bc;
  float cst[kMaxPairs];
#pragma unroll
  for (int e = 0; e < kMaxPairs; ++e) {
    const int pi = threadIdx.x + e * NT;
    cst[e] = 0.f;
    if (pi < npairs) {
      const int ul = pi / p.Bc, bl = pi % p.Bc;
      const int64_t u = u0 + ul, b = p.b_off + bl;
      const float h = p.h0 ? p.h0[b * H + u] : 0.f;
      const float c = p.c0 ? p.c0[b * H + u] : 0.f;
      cst[e] = c;
      p.h_save[b * H + u] = h;
      p.c_save[b * H + u] = c;
      __stcg(p.xf + (int64_t)u * BP + bl, h);
    }
  }
  unsigned epoch = 1;
  if (!grid_barrier(p.bar, epoch * p.ncta, p.status)) return;
  const float *bf = p.bf + (int64_t)cta * rp;

  for (int64_t t = 0; t < p.T; ++t) {
    // prefetch this step's input-projection gates for the owned pairs
    float zg[kMaxPairs][4];
#pragma unroll
    for (int e = 0; e < kMaxPairs; ++e) {
      const int pi = threadIdx.x + e * NT;
      if (pi < npairs) {
        const int ul = pi / p.Bc, bl = pi % p.Bc;
        const float *zr = p.zacts + (t * Bt + p.b_off + bl) * 4 * H + u0 + ul;
#pragma unroll
        for (int g = 0; g < 4; ++g) zg[e][g] = zr[g * H];
      }
    }
    const float *xsrc = p.xf + (int64_t)(t & 1) * d.K_pad * BP;
    step_matvec<BG, RG, NR>(wres, wsrc, xsrc, xbuf, wbuf, red, d, BP);
    float *xdst = p.xf + (int64_t)((t + 1) & 1) * d.K_pad * BP;
#pragma unroll
    for (int e = 0; e < kMaxPairs; ++e) {
      const int pi = threadIdx.x + e * NT;
      if (pi < npairs) {
        const int ul = pi / p.Bc, bl = pi % p.Bc;
        float act[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int ri = ul * 4 + g;
          act[g] = sigm(zg[e][g] + red_sum(red, rp, BP, ri, bl) + bf[ri]);
        }
        const float c = fmaf(act[1], cst[e], act[0] * act[2]);
        const float h = act[3] * tanhf(c);
        cst[e] = c;
        const int64_t b = p.b_off + bl, u = u0 + ul;
        float *ar = p.zacts + (t * Bt + b) * 4 * H + u;
#pragma unroll
        for (int g = 0; g < 4; ++g) ar[g * H] = act[g];
        p.h_save[((t + 1) * Bt + b) * H + u] = h;
        p.c_save[((t + 1) * Bt + b) * H + u] = c;
        __stcg(xdst + u * BP + bl, h);
      }
    }
    if (t + 1 < p.T) {
      ++epoch;
      if (!grid_barrier(p.bar, epoch * p.ncta, p.status)) return;
    }
  }
}

// ------------------------------------------------------------------ backward
template <int BG, int RG, int NR>
__global__ void __launch_bounds__(NT, 1) rec_bwd_kernel(RecArgs p) {
  extern __shared__ __align__(16) float smem[];
  const Dir &d = p.d;
  const int BP = p.BP, rp = d.rows_pad;
  const int cta = blockIdx.x;
  float *wres = d.resident ? smem : nullptr;
  float *xbuf = smem + (d.resident ? d.K_pad * rp : 0);
  float *wbuf = xbuf + kStages * d.KC * BP;
  float *red = wbuf + (d.resident ? 0 : kStages * d.KC * rp);
  const float *wsrc = p.wb + (int64_t)cta * d.K_pad * rp;
  const int64_t H = p.H, Bt = p.Bt;
  const int u0 = cta * p.U;
  const int Uc = (int)min((int64_t)p.U, H - u0);

  if (wres) {
    for (int i = threadIdx.x; i < d.K_pad * rp / 4; i += NT)
      reinterpret_cast<float4 *>(wres)[i] = reinterpret_cast<const float4 *>(wsrc)[i];
  }
  const int npairs = Uc * p.Bc;
  float dcst[kMaxPairs];
#pragma unroll
  for (int e = 0; e < kMaxPairs; ++e) {
    const int pi = threadIdx.x + e * NT;
    dcst[e] = 0.f;
    if (pi < npairs && p.dc_n) {
      const int ul = pi / p.Bc, bl = pi % p.Bc;
      dcst[e] = p.dc_n[(p.b_off + bl) * H + u0 + ul];
    }
  }
  __syncthreads();
  unsigned epoch = 0;
  for (int64_t t = p.T - 1; t >= 0; --t) {
    // prefetch per-pair operands of this step
    float act[kMaxPairs][4], ct[kMaxPairs], cp[kMaxPairs], dh[kMaxPairs];
#pragma unroll
    for (int e = 0; e < kMaxPairs; ++e) {
      const int pi = threadIdx.x + e * NT;
      if (pi < npairs) {
        const int ul = pi / p.Bc, bl = pi % p.Bc;
        const int64_t b = p.b_off + bl, u = u0 + ul;
        const float *ar = p.zacts + (t * Bt + b) * 4 * H + u;
#pragma unroll
        for (int g = 0; g < 4; ++g) act[e][g] = ar[g * H];
        ct[e] = p.c_save[((t + 1) * Bt + b) * H + u];
        cp[e] = p.c_save[(t * Bt + b) * H + u];
        dh[e] = p.dout[(t * Bt + b) * H + u];
        if (t == p.T - 1 && p.dh_n) dh[e] += p.dh_n[b * H + u];
      }
    }
    if (t < p.T - 1) {
      const float *xsrc = p.xb + (int64_t)((t + 1) & 1) * d.K_pad * BP;
      step_matvec<BG, RG, NR>(wres, wsrc, xsrc, xbuf, wbuf, red, d, BP);
    }
    float *xdst = p.xb + (int64_t)(t & 1) * d.K_pad * BP;
#pragma unroll
    for (int e = 0; e < kMaxPairs; ++e) {
      const int pi = threadIdx.x + e * NT;
      if (pi < npairs) {
        const int ul = pi / p.Bc, bl = pi % p.Bc;
        const int64_t b = p.b_off + bl, u = u0 + ul;
        float dhv = dh[e];
        if (t < p.T - 1) dhv += red_sum(red, rp, BP, ul, bl);
        const float i = act[e][0], f = act[e][1], g = act[e][2], o = act[e][3];
        const float th = tanhf(ct[e]);
        const float dct = dcst[e] + dhv * o * (1.f - th * th);
        float dg[4];
        dg[0] = dct * g * i * (1.f - i);
        dg[1] = dct * cp[e] * f * (1.f - f);
        dg[2] = dct * i * g * (1.f - g);
        dg[3] = dhv * th * o * (1.f - o);
        dcst[e] = dct * f;
        float *ar = p.zacts + (t * Bt + b) * 4 * H + u;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          ar[q * H] = dg[q];
          __stcg(xdst + (q * H + u) * BP + bl, dg[q]);
        }
      }
    }
    if (t > 0) {
      ++epoch;
      if (!grid_barrier(p.bar, epoch * p.ncta, p.status)) return;
    }
  }
}

// a-unscaling (_torch.py:165-168): dW_hh = a_exp*dW_hh_s (in place),
// db_hh = a_exp*db, da[g] = sum_{r in g} (sum_k W_hh*dW_hh_s + b_hh*db).
// Pass 1: grid (kUnscaleParts, 4 gates); part j of gate g takes rows
// [j*H/P, (j+1)*H/P) of that gate, scales them and writes its partial sum.
// Pass 2: one warp per gate adds the partials in a fixed order.
constexpr int kUnscaleParts = 128;

__global__ void __launch_bounds__(256) rec_unscale_kernel(const float *__restrict__ w_hh,
                                                          const float *__restrict__ b_hh,
                                                          const float *__restrict__ a,
                                                          float *__restrict__ dw_hh,
                                                          const float *__restrict__ db,
                                                          float *__restrict__ db_hh,
                                                          float *__restrict__ part, int64_t H) {
  const int g = blockIdx.y, j = blockIdx.x;
  const float ag = a[g];
  const int64_t r0 = H * j / kUnscaleParts, r1 = H * (j + 1) / kUnscaleParts;
  float s = 0.f;
  for (int64_t i = (int64_t)g * H * H + r0 * H + threadIdx.x; i < (int64_t)g * H * H + r1 * H; i += 256) {
    const float dws = dw_hh[i];
    s = fmaf(w_hh[i], dws, s);
    dw_hh[i] = ag * dws;
  }
  for (int64_t r = r0 + threadIdx.x; r < r1; r += 256) {
    const int64_t idx = (int64_t)g * H + r;
    s = fmaf(b_hh[idx], db[idx], s);
    db_hh[idx] = ag * db[idx];
  }
  __shared__ float red[256];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[g * kUnscaleParts + j] = red[0];
}

__global__ void rec_da_kernel(const float *__restrict__ part, float *__restrict__ da) {
  const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float s = 0.f;
  for (int j = lane; j < kUnscaleParts; j += 32) s += part[g * kUnscaleParts + j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) da[g] = s;
}

using KernelFn = void (*)(RecArgs);

// NR = 1, 2 or 4 (a plan with 3 row tiles takes the 4-tile kernel).
#define HS_CASES(K)                                                                        \
  HS_CASE(K, 1, 1) HS_CASE(K, 1, 2) HS_CASE(K, 1, 4) HS_CASE(K, 1, 8)                       \
  HS_CASE(K, 2, 1) HS_CASE(K, 2, 2) HS_CASE(K, 2, 4) HS_CASE(K, 2, 8)                       \
  HS_CASE(K, 4, 1) HS_CASE(K, 4, 2) HS_CASE(K, 4, 4) HS_CASE(K, 4, 8)                       \
  HS_CASE(K, 8, 1) HS_CASE(K, 8, 2) HS_CASE(K, 8, 4)
#define HS_CASE(K, bg, rg)                                                                 \
  if (BG == bg && RG == rg)                                                                \
    return NRT <= 1 ? K<bg, rg, 1> : NRT <= 2 ? K<bg, rg, 2> : K<bg, rg, 4>;
KernelFn pick_fwd(int BG, int RG, int NRT) {
  HS_CASES(rec_fwd_kernel)
  return nullptr;
}
KernelFn pick_bwd(int BG, int RG, int NRT) {
  HS_CASES(rec_bwd_kernel)
  return nullptr;
}
#undef HS_CASE
#undef HS_CASES

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

int launch_persistent(KernelFn fn, const Plan &pl, const Dir &d, RecArgs &args, cudaStream_t st) {
  const size_t smem = d.smem;
  if (cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(rec)");
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, (const void *)fn, NT, smem) != cudaSuccess)
    return check_launch("occupancy(rec)");
  if (per_sm < 1) return fail(HS_ERR_UNSUPPORTED, "recurrent kernel does not fit on an SM (smem %zu)", smem);
  void *kargs[] = {&args};
  if (cudaLaunchCooperativeKernel((const void *)fn, dim3(pl.ncta), dim3(NT), kargs, smem, st) != cudaSuccess)
    return check_launch("cudaLaunchCooperativeKernel(rec)");
  return HS_OK;
}

int check_rec_args(int64_t T, int64_t B, int64_t D, int64_t H) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0)
    return fail(HS_ERR_INVALID_ARG, "T, B, D, H must be positive (got %lld, %lld, %lld, %lld)", (long long)T, (long long)B, (long long)D, (long long)H);
  return HS_OK;
}

}  // namespace

size_t rec_ws_bytes(int64_t T, int64_t B, int64_t D, int64_t H) {
  Plan p;
  const int nsm = num_sms();
  if (!make_plan(p, B, H, nsm > 0 ? nsm : 148)) return 0;
  // the GEMMs run before the persistent kernels (forward) or after them
  // (backward), so they reuse the same scratch
  return std::max<size_t>({p.total, rec_tc_ws_bytes(B, H), rec_cluster_ws_bytes(H), rec_wide_ws_bytes(H), linear_ws_bytes(T * B, 4 * H, D),
                           linear_ws_bytes(T * B, 4 * H, H), linear_backward_ws(T * B, 4 * H, D, H)});
}

// bf: a bfloat16 module's step product (bf16 weights and state, one product
// per instruction) where the step runs on the tensor cores; the FFMA kernels
// compute in float32 on the same (bf16-valued) inputs either way.
int rec_forward(const float *x, const float *h0, const float *c0, const float *w_ih,
                const float *w_hh, const float *b_ih, const float *b_hh, const float *a,
                float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t D,
                int64_t H, void *ws, size_t ws_bytes, int *status, cudaStream_t st, bool bf = false) {
  if (int e = check_rec_args(T, B, D, H)) return e;
  if (!x || !w_ih || !w_hh || !b_ih || !b_hh || !a || !h_save || !c_save || !acts || !status)
    return fail(HS_ERR_INVALID_ARG, "recurrent_forward: null required pointer");
  Plan pl;
  const int nsm = num_sms();
  if (nsm <= 0) return fail(HS_ERR_CUDA, "no CUDA device");
  if (!make_plan(pl, B, H, nsm)) return fail(HS_ERR_UNSUPPORTED, "recurrent: no tiling for B=%lld H=%lld on %d SMs", (long long)B, (long long)H, nsm);
  if (!ws || ws_bytes < pl.total) return fail(HS_ERR_WORKSPACE, "recurrent_forward: workspace %zu < %zu bytes", ws_bytes, pl.total);
  if (!aligned(ws, 256)) return fail(HS_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  char *w = static_cast<char *>(ws);
  // Z = x W_ih^T + b_ih, written into acts (_torch.py:96)
  if (int e = linear_forward(x, w_ih, b_ih, acts, T * B, 4 * H, D, ws, ws_bytes, status, st)) return e;
  // small H: the whole recurrence of a batch group on one cluster
  if (rec_cluster_wanted(B, H))
    return rec_cluster_forward(h0, c0, w_hh, b_hh, a, h_save, c_save, acts, T, B, H, ws, ws_bytes, status, st);
  // H = 512: clusters of 16 with a few sequences each, the state exchanged in
  // distributed shared memory
  if (rec_wide_wanted(B, H))
    return rec_wide_forward(h0, c0, w_hh, b_hh, a, h_save, c_save, acts, T, B, H, ws, ws_bytes, status, st);
  // the step product on the tensor cores where the shape allows
  if (rec_tc_wanted(0, B, H, bf))
    return rec_tc_forward(h0, c0, w_hh, b_hh, a, h_save, c_save, acts, T, B, H, ws, ws_bytes, status, st, bf);
  if (pl.fwd.rows_pad > 256) return fail(HS_ERR_UNSUPPORTED, "recurrent: slice of %d rows", pl.fwd.rows_pad);
  rec_prep_fwd_kernel<<<dim3((unsigned)((pl.fwd.K_pad + 31) / 32), (unsigned)pl.ncta), 256, 0, st>>>(
      w_hh, b_hh, a, (float *)(w + pl.o_wf), (float *)(w + pl.o_bf), H, pl.U, pl.fwd.rows_pad, pl.fwd.K_pad);
  if (int e = check_launch("rec_prep_fwd_kernel")) return e;
  KernelFn fn = pick_fwd(pl.BG, pl.fwd.RG, pl.fwd.NRT);
  if (!fn) return fail(HS_ERR_UNSUPPORTED, "recurrent_forward: no kernel for BG=%d RG=%d", pl.BG, pl.fwd.RG);
  for (int64_t b0 = 0; b0 < B; b0 += kMaxBatch) {
    if (cudaMemsetAsync(w + pl.o_bar, 0, 256, st) != cudaSuccess) return check_launch("memset(bar)");
    if (cudaMemsetAsync(w + pl.o_xf, 0, 2ull * pl.fwd.K_pad * pl.BP * 4, st) != cudaSuccess) return check_launch("memset(xf)");
    RecArgs args{};
    args.zacts = acts;
    args.h0 = h0;
    args.c0 = c0;
    args.h_save = h_save;
    args.c_save = c_save;
    args.wf = (const float *)(w + pl.o_wf);
    args.bf = (const float *)(w + pl.o_bf);
    args.xf = (float *)(w + pl.o_xf);
    args.bar = (unsigned *)(w + pl.o_bar);
    args.status = status;
    args.T = T;
    args.Bt = B;
    args.H = H;
    args.b_off = (int)b0;
    args.Bc = (int)std::min<int64_t>(kMaxBatch, B - b0);
    args.U = pl.U;
    args.ncta = pl.ncta;
    args.d = pl.fwd;
    args.BP = pl.BP;
    if (int e = launch_persistent(fn, pl, pl.fwd, args, st)) return e;
  }
  return HS_OK;
}

int rec_backward(const float *x, const float *w_ih, const float *w_hh, const float *b_hh,
                 const float *a, const float *h_save, const float *c_save, float *acts,
                 const float *dout, const float *dh_n, const float *dc_n, float *dx,
                 float *dw_ih, float *dw_hh, float *db_ih, float *db_hh, float *da, int64_t T,
                 int64_t B, int64_t D, int64_t H, void *ws, size_t ws_bytes, int *status,
                 cudaStream_t st, bool bf = false) {
  if (int e = check_rec_args(T, B, D, H)) return e;
  if (!x || !w_ih || !w_hh || !b_hh || !a || !h_save || !c_save || !acts || !dout || !dw_ih ||
      !dw_hh || !db_ih || !db_hh || !da || !status)
    return fail(HS_ERR_INVALID_ARG, "recurrent_backward: null required pointer");
  Plan pl;
  const int nsm = num_sms();
  if (nsm <= 0) return fail(HS_ERR_CUDA, "no CUDA device");
  if (!make_plan(pl, B, H, nsm)) return fail(HS_ERR_UNSUPPORTED, "recurrent: no tiling for B=%lld H=%lld on %d SMs", (long long)B, (long long)H, nsm);
  if (!ws || ws_bytes < pl.total) return fail(HS_ERR_WORKSPACE, "recurrent_backward: workspace %zu < %zu bytes", ws_bytes, pl.total);
  char *w = static_cast<char *>(ws);
  if (rec_cluster_wanted(B, H)) {
    if (int e = rec_cluster_backward(w_hh, a, c_save, acts, dout, dh_n, dc_n, T, B, H, ws, ws_bytes, status, st))
      return e;
  } else if (rec_wide_wanted(B, H)) {
    if (int e = rec_wide_backward(w_hh, a, c_save, acts, dout, dh_n, dc_n, T, B, H, ws, ws_bytes, status, st))
      return e;
  } else if (rec_tc_wanted(1, B, H, bf)) {
    // the step product on the tensor cores
    if (int e = rec_tc_backward(w_hh, a, c_save, acts, dout, dh_n, dc_n, T, B, H, ws, ws_bytes, status, st, bf))
      return e;
  } else {
  // The scaled backward slices are built here so a backward never depends
  // on workspace contents left by its forward.
  rec_prep_kernel<<<4 * nsm, 256, 0, st>>>(w_hh, b_hh, a, nullptr, nullptr, (float *)(w + pl.o_wb), H,
                                           pl.U, pl.ncta, pl.fwd.rows_pad, pl.fwd.K_pad, pl.bwd.rows_pad,
                                           pl.bwd.K_pad);
  if (int e = check_launch("rec_prep_kernel")) return e;
  KernelFn fn = pick_bwd(pl.BG, pl.bwd.RG, pl.bwd.NRT);
  if (!fn) return fail(HS_ERR_UNSUPPORTED, "recurrent_backward: no kernel for BG=%d RG=%d", pl.BG, pl.bwd.RG);
  for (int64_t b0 = 0; b0 < B; b0 += kMaxBatch) {
    if (cudaMemsetAsync(w + pl.o_bar, 0, 256, st) != cudaSuccess) return check_launch("memset(bar)");
    if (cudaMemsetAsync(w + pl.o_xb, 0, 2ull * pl.bwd.K_pad * pl.BP * 4, st) != cudaSuccess) return check_launch("memset(xb)");
    RecArgs args{};
    args.zacts = acts;
    args.c_save = const_cast<float *>(c_save);
    args.dout = dout;
    args.dh_n = dh_n;
    args.dc_n = dc_n;
    args.wb = (const float *)(w + pl.o_wb);
    args.xb = (float *)(w + pl.o_xb);
    args.bar = (unsigned *)(w + pl.o_bar);
    args.status = status;
    args.T = T;
    args.Bt = B;
    args.H = H;
    args.b_off = (int)b0;
    args.Bc = (int)std::min<int64_t>(kMaxBatch, B - b0);
    args.U = pl.U;
    args.ncta = pl.ncta;
    args.d = pl.bwd;
    args.BP = pl.BP;
    if (int e = launch_persistent(fn, pl, pl.bwd, args, st)) return e;
  }
  }
  // Batched parameter gradients (_torch.py:153-162); acts now holds dgates.
  // dX = dG.W_ih, dW_ih = dG^T.x and dW_hh_s = dG^T.h_{t-1} share one
  // conversion of dG (h_save rows 0..T-1 are the h_{t-1} of steps 0..T-1).
  const int64_t M = T * B, N = 4 * H;
  if (int e = linear_backward_ex(acts, w_ih, dx, x, dw_ih, h_save, dw_hh, M, N, D, H, 0, ws, ws_bytes, status, st,
                                  nullptr))
    return e;
  if (int e = colsum(acts, db_ih, M, N, 0, st, ws, ws_bytes)) return e;
  // partial sums of da in the (now free) workspace
  float *part = reinterpret_cast<float *>(w);
  rec_unscale_kernel<<<dim3(kUnscaleParts, 4), 256, 0, st>>>(w_hh, b_hh, a, dw_hh, db_ih, db_hh, part, H);
  if (int e = check_launch("rec_unscale_kernel")) return e;
  rec_da_kernel<<<1, 128, 0, st>>>(part, da);
  return check_launch("rec_da_kernel");
}

}  // namespace hs

extern "C" {

int hs_recurrent_uses_tensor_cores(int64_t B, int64_t H, int backward) {
  if (B <= 0 || H <= 0 || hs::rec_cluster_wanted(B, H) || hs::rec_wide_wanted(B, H)) return 0;
  return hs::rec_tc_wanted(backward ? 1 : 0, B, H) ? 1 : 0;
}

int hs_recurrent_path(int64_t B, int64_t H, int backward) {
  if (B <= 0 || H <= 0) return -1;
  if (hs::rec_cluster_wanted(B, H) || hs::rec_wide_wanted(B, H)) return 2;
  return hs::rec_tc_wanted(backward ? 1 : 0, B, H) ? 1 : 0;
}

size_t hs_recurrent_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return 0;
  return hs::rec_ws_bytes(T, B, D, H);
}

int hs_recurrent_forward(const float *x, const float *h0, const float *c0, const float *w_ih,
                         const float *w_hh, const float *b_ih, const float *b_hh, const float *a,
                         float *h_save, float *c_save, float *acts, int64_t T, int64_t B,
                         int64_t D, int64_t H, void *workspace, size_t workspace_bytes,
                         int *dev_status, hs_stream_t stream) {
  return hs::rec_forward(x, h0, c0, w_ih, w_hh, b_ih, b_hh, a, h_save, c_save, acts, T, B, D, H,
                         workspace, workspace_bytes, dev_status, (cudaStream_t)stream);
}

int hs_recurrent_backward(const float *x, const float *w_ih, const float *w_hh,
                          const float *b_hh, const float *a, const float *h_save,
                          const float *c_save, float *acts, const float *dout,
                          const float *dh_n, const float *dc_n, float *dx, float *dw_ih,
                          float *dw_hh, float *db_ih, float *db_hh, float *da, int64_t T,
                          int64_t B, int64_t D, int64_t H, void *workspace,
                          size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::rec_backward(x, w_ih, w_hh, b_hh, a, h_save, c_save, acts, dout, dh_n, dc_n, dx,
                          dw_ih, dw_hh, db_ih, db_hh, da, T, B, D, H, workspace, workspace_bytes,
                          dev_status, (cudaStream_t)stream);
}

int hs_recurrent_forward_bf16(const float *x, const float *h0, const float *c0, const float *w_ih,
                              const float *w_hh, const float *b_ih, const float *b_hh, const float *a,
                              float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t D, int64_t H,
                              void *workspace, size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::rec_forward(x, h0, c0, w_ih, w_hh, b_ih, b_hh, a, h_save, c_save, acts, T, B, D, H, workspace,
                         workspace_bytes, dev_status, (cudaStream_t)stream, true);
}

int hs_recurrent_backward_bf16(const float *x, const float *w_ih, const float *w_hh, const float *b_hh,
                               const float *a, const float *h_save, const float *c_save, float *acts,
                               const float *dout, const float *dh_n, const float *dc_n, float *dx, float *dw_ih,
                               float *dw_hh, float *db_ih, float *db_hh, float *da, int64_t T, int64_t B, int64_t D,
                               int64_t H, void *workspace, size_t workspace_bytes, int *dev_status,
                               hs_stream_t stream) {
  return hs::rec_backward(x, w_ih, w_hh, b_hh, a, h_save, c_save, acts, dout, dh_n, dc_n, dx, dw_ih, dw_hh, db_ih,
                          db_hh, da, T, B, D, H, workspace, workspace_bytes, dev_status, (cudaStream_t)stream, true);
}

}  // extern "C"
