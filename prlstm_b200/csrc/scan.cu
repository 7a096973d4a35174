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
// Layout: z [T,B,4H] (gate order i,f,g,o), c/out/dout [T,B,H].
//
// Work split: a warp tile is L consecutive time steps x 32 consecutive hidden
// units of one sequence; lane l owns unit h0+l and walks the L steps itself.
// The warp stages its tile into shared memory with cp.async (16-byte copies
// when H%4 == 0, so in-flight data holds no registers and many tiles per SM
// are in flight), computes its summary, runs its own look-back (one 64-bit
// word per lane, no block barrier), and writes its outputs.  A CTA stacks WPC
// warps on WPC consecutive chunks of the same 32-unit column; the backward
// adds the CTA's bias-gradient sums in a fixed order into one partial row.
//
// Ordering: blockIdx.x runs over tiles in scan order (chunk-group major), so
// every predecessor of a tile sits in a lower-indexed block, or in a lower
// warp of the same block, and is dispatched no later than the tile itself;
// every wait is also bounded in time and reports HS_ERR_DEVICE_TIMEOUT
// instead of hanging.
//
// When the columns (sequence x 32 units) alone fill the GPU, the one-CTA-per-
// column kernels of scan_chain.cu run instead (see scan_chain_wanted): they
// pass the carry between the warps of a CTA through shared memory and need
// no look-back scratch.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "hs_common.cuh"

namespace hs {

bool scan_chain_wanted(int64_t T, int64_t B, int64_t H);
int64_t scan_wave_sequences(int64_t H);
int scan_fwd_chain_launch(const float *z, const float *c0, float *out, float *c, float *h_n, float *c_n,
                          int64_t T, int64_t B, int64_t H, float eps, unsigned *kf_max, int *status,
                          cudaStream_t st);
int scan_bwd_chain_launch(const float *z, const float *c, const float *c0, const float *dout,
                          const float *dh_n, const float *dc_n, float *dz, float *dc0, float *db_part,
                          int64_t T, int64_t B, int64_t H, float eps, unsigned *dz_absmax, int *status,
                          cudaStream_t st, __half *dzh = nullptr, __half *dzl = nullptr,
                          const unsigned *dz_bound = nullptr, const int *gate = nullptr);
int h3_split_known(const float *x, int64_t rows, int64_t cols, int64_t ld, const unsigned *absmax, void *dst,
                   cudaStream_t st, const int *gate);
size_t h3_split_bytes(int64_t rows, int64_t cols);

namespace {

// Look-back state.  One 64-bit word per (tile, hidden unit), stored
// complemented so that the all-zero word means "not published yet" and the
// workspace is cleared with a plain zero memset:
//   hi == kInclusive : lo holds the tile's inclusive value (the carry out)
//   otherwise        : the tile's aggregate, hi = bits of A, lo = bits of C.
// A = prod f' lies in [0, 1] (never a NaN pattern) and hi == kInclusive is a
// NaN pattern, so the three states cannot be confused.  Flag and payload
// travel in one single-copy-atomic store: a reader that sees the word sees
// its value, with no fence between them.
struct ScanWs {
  unsigned long long *words;  // [nchunk][B*ncol][32]
  float *db_part;             // [ngroup*B][4H] (backward only)
};

struct ScanShape {
  int64_t T, B, H;
  int nchunk;  // ceil(T / L)
  int ncol;    // ceil(H / 32)
  int ngroup;  // ceil(nchunk / WPC): CTAs along time per column
};

// Tile geometry (compile-time; the defaults are the measured best on B200
// for the benchmark shapes).  L = steps per warp tile, WPC = warps per CTA.
#ifndef HS_SCAN_FWD_L
#define HS_SCAN_FWD_L 8
#endif
#ifndef HS_SCAN_FWD_WPC
#define HS_SCAN_FWD_WPC 4
#endif
#ifndef HS_SCAN_BWD_L
#define HS_SCAN_BWD_L 8
#endif
#ifndef HS_SCAN_BWD_WPC
#define HS_SCAN_BWD_WPC 8
#endif
constexpr int kFwdL = HS_SCAN_FWD_L, kFwdWPC = HS_SCAN_FWD_WPC;
constexpr int kBwdL = HS_SCAN_BWD_L, kBwdWPC = HS_SCAN_BWD_WPC;
constexpr unsigned kInclusive = 0xFFFFFFFEu;
constexpr int kFwdRow = 4 * 32;  // staged floats per forward step: z_i, z_f, z_g, z_o
constexpr int kBwdRow = 6 * 32;  // backward: z_i, z_f, z_g, z_o, c, dout
constexpr size_t kFwdSmem = sizeof(float) * kFwdWPC * kFwdL * kFwdRow;
constexpr size_t kBwdSmem = sizeof(float) * kBwdWPC * (kBwdL * kBwdRow + 32);

ScanShape make_shape(int64_t T, int64_t B, int64_t H, int L, int WPC) {
  ScanShape s;
  s.T = T;
  s.B = B;
  s.H = H;
  s.nchunk = (int)((T + L - 1) / L);
  s.ncol = (int)((H + 31) / 32);
  s.ngroup = (s.nchunk + WPC - 1) / WPC;
  return s;
}

size_t ws_words_bytes(const ScanShape &s) {
  return round_up(sizeof(unsigned long long) * (size_t)s.nchunk * s.B * s.ncol * 32, 256);
}

size_t ws_layout(const ScanShape &s, bool with_db, ScanWs *out, void *base) {
  size_t off = ws_words_bytes(s);
  const size_t o_db = off;
  if (with_db) off += round_up(sizeof(float) * (size_t)s.ngroup * s.B * 4 * s.H, 256);
  if (out) {
    char *b = static_cast<char *>(base);
    out->words = reinterpret_cast<unsigned long long *>(b);
    out->db_part = with_db ? reinterpret_cast<float *>(b + o_db) : nullptr;
  }
  return off;
}

// ------------------------------------------------------------------ device helpers
HS_DEV void cp_async16(float *dst, const float *src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
HS_DEV void cp_async4(float *dst, const float *src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
HS_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

HS_DEV unsigned long long pack(unsigned hi, float lo) {
  return ~(((unsigned long long)hi << 32) | __float_as_uint(lo));
}
HS_DEV void st_word(unsigned long long *p, unsigned long long w) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
HS_DEV unsigned long long ld_word(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Decoupled look-back of one lane's unit.  (TA, TC) is the tile's own map
// c_out = TA c_in + TC; k is the tile's position in scan order along its
// chain, and the predecessors' words sit at my - m*stride.  On entry cin
// holds the chain's initial carry (used when k == 0); on return it holds the
// carry into this tile, and this tile's inclusive value is published.
//
// The aggregate is published first, so that successors can pass over this
// tile while it looks back; then the predecessors are composed nearest first
// (an aggregate extends the map, an inclusive value ends the look-back).
// Reading several predecessors per round trip measured slower on B200 than
// this one-at-a-time walk: the predecessors are mostly published already and
// the extra polling loads cost more than the round trips they save.  Every
// wait is bounded by kWaitLimitNs and by the sticky status word (a waiter
// that already gave up makes every other waiter leave).
HS_DEV bool look_back(unsigned long long *my, int64_t stride, int k, float TA, float TC, float &cin,
                      int *status) {
  if (k > 0) {
    st_word(my, pack(__float_as_uint(TA), TC));
    float ra = 1.f, rc = 0.f;
    const unsigned long long *p = my - stride;
    uint64_t t0 = 0;
    for (unsigned n = 0;; ++n) {
      const unsigned long long v = ld_word(p);
      if (v != 0ull) {
        const unsigned long long x = ~v;
        const unsigned hi = (unsigned)(x >> 32);
        const float lo = __uint_as_float((unsigned)x);
        if (hi == kInclusive) {
          cin = fmaf(ra, lo, rc);
          break;
        }
        rc = fmaf(ra, lo, rc);
        ra *= __uint_as_float(hi);
        p -= stride;  // tile 0 publishes only an inclusive value: p stays in range
        continue;
      }
      if (n >= 2) {  // the nearest unread predecessor is not published yet
        __nanosleep(64);
        if ((n & 15) == 0) {
          if (t0 == 0) t0 = globaltimer();
          if (ld_status(status) != 0) return false;
          if (globaltimer() - t0 > kWaitLimitNs) {
            set_status(status, HS_ERR_DEVICE_TIMEOUT);
            return false;
          }
        }
      }
    }
  }
  st_word(my, pack(kInclusive, fmaf(TA, cin, TC)));
  return true;
}

// ============================================================== forward
template <bool V16>
__global__ void __launch_bounds__(kFwdWPC * 32)
scan_fwd_kernel(const float *__restrict__ z, const float *__restrict__ c0, float *__restrict__ out,
                float *__restrict__ cbuf, float *__restrict__ h_n, float *__restrict__ c_n, ScanShape sh,
                float eps, ScanWs ws, int *status) {
  constexpr int L = kFwdL;
  extern __shared__ float4 smem_f4[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *zs = reinterpret_cast<float *>(smem_f4) + warp * (L * kFwdRow);
  const int64_t T = sh.T, B = sh.B, H = sh.H;
  const int64_t per_chunk = B * sh.ncol;
  const int64_t grp = blockIdx.x / per_chunk;
  const int64_t col = blockIdx.x - grp * per_chunk;
  const int j = (int)(grp * kFwdWPC + warp);
  if (j >= sh.nchunk) return;  // no block barrier in this kernel
  if (ld_status(status) != 0) return;
  const int64_t b = col / sh.ncol;
  const int64_t h0 = (col - b * sh.ncol) * 32;
  const int64_t h = h0 + lane;
  const bool hv = h < H;
  const int64_t t0 = (int64_t)j * L;
  const int nst = (int)min((int64_t)L, T - t0);
  const int64_t zstep = B * 4 * H;

  // Stage z[t0 .. t0+nst) for units h0 .. h0+31 (4 gate rows per step).
  if (V16) {
    const int g = lane >> 3, k = (lane & 7) * 4;
    if (h0 + k < H) {
      const float *src = z + (t0 * B + b) * 4 * H + g * H + h0 + k;
      float *dst = zs + g * 32 + k;
#pragma unroll 4
      for (int s = 0; s < nst; ++s) cp_async16(dst + s * kFwdRow, src + s * zstep);
    }
  } else if (hv) {
    const float *src = z + (t0 * B + b) * 4 * H + h;
    for (int s = 0; s < nst; ++s)
#pragma unroll
      for (int g = 0; g < 4; ++g) cp_async4(zs + s * kFwdRow + g * 32 + lane, src + s * zstep + g * H);
  }
  cp_async_wait_all();
  __syncwarp();

  // Pass 1: activations (kept in place: slot i <- b', f <- f', o <- e^-z_o)
  // and the tile's map.
  float A = 1.f, C = 0.f;
  if (hv) {
#pragma unroll
    for (int s = 0; s < L; ++s) {
      if (s < nst) {
        float *r = zs + s * kFwdRow + lane;
        const float fp = fmaxf(sigf(r[32]), eps);
        const float bp = fmaxf(sig2(r[0], r[64]), eps);
        r[0] = bp;
        r[32] = fp;
        r[96] = __expf(-r[96]);  // e^-z_o; sigma(z_o) is folded into pass 2
        C = fmaf(fp, C, bp);
        A *= fp;
      }
    }
  }
  float cin = fmaxf((j == 0 && c0 && hv) ? c0[b * H + h] : 0.f, eps);
  if (!look_back(ws.words + ((int64_t)j * per_chunk + col) * 32 + lane, per_chunk * 32, j, A, C, cin, status))
    return;
  if (!hv) return;

  // Pass 2: the exact recurrence from the carry.
  float c = cin;
  const int64_t os = B * H;
  float *ob = out + (t0 * B + b) * H + h;
  float *cb = cbuf + (t0 * B + b) * H + h;
#pragma unroll
  for (int s = 0; s < L; ++s) {
    if (s < nst) {
      const float *r = zs + s * kFwdRow + lane;
      c = fmaf(r[32], c, r[0]);
      const float o = sig_tanh_pos(r[96], c);
      __stcs(cb + s * os, c);
      __stcs(ob + s * os, o);
      if (t0 + s == T - 1) {
        if (c_n) c_n[b * H + h] = c;
        if (h_n) h_n[b * H + h] = o;
      }
    }
  }
}

// ============================================================== backward
template <bool V16>
__global__ void __launch_bounds__(kBwdWPC * 32)
scan_bwd_kernel(const float *z, const float *__restrict__ cbuf, const float *__restrict__ c0,
                const float *__restrict__ dout, const float *__restrict__ dh_n, const float *__restrict__ dc_n,
                float *dz, float *__restrict__ dc0, ScanShape sh, float eps, ScanWs ws, unsigned *dz_absmax,
                int *status) {
  constexpr int L = kBwdL;
  extern __shared__ float4 smem_f4[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *bs = reinterpret_cast<float *>(smem_f4) + warp * (L * kBwdRow + 32);
  float *cprev_row = bs + L * kBwdRow;
  const int64_t T = sh.T, B = sh.B, H = sh.H;
  const int64_t per_chunk = B * sh.ncol;
  const int64_t grp = blockIdx.x / per_chunk;
  const int64_t col = blockIdx.x - grp * per_chunk;
  const int q = (int)(grp * kBwdWPC + warp);  // scan order: 0 = last chunk in time
  bool active = q < sh.nchunk && ld_status(status) == 0;
  const int j = sh.nchunk - 1 - q;
  const int64_t b = col / sh.ncol;
  const int64_t h0 = (col - b * sh.ncol) * 32;
  const int64_t h = h0 + lane;
  const bool hv = h < H;
  const int64_t t0 = (int64_t)j * L;
  const int nst = active ? (int)min((int64_t)L, T - t0) : 0;
  const int64_t zstep = B * 4 * H, sstep = B * H;
  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  float amax = 0.f;  // max |dz| of this lane (NaN ignored), if dz_absmax is wanted

  if (active) {
    // Stage z (4 rows), c and dout of each step, and c_{t0-1}.
    if (V16) {
      const int g = lane >> 3, k = (lane & 7) * 4;
      if (h0 + k < H) {
        const float *zsrc = z + (t0 * B + b) * 4 * H + g * H + h0 + k;
        const float *ssrc = (g == 0 ? cbuf : dout) + (t0 * B + b) * H + h0 + k;
        float *dst = bs + g * 32 + k;
#pragma unroll 4
        for (int s = 0; s < nst; ++s) {
          cp_async16(dst + s * kBwdRow, zsrc + s * zstep);
          if (g < 2) cp_async16(dst + s * kBwdRow + 128, ssrc + s * sstep);
        }
        if (g == 0 && t0 > 0) cp_async16(cprev_row + k, cbuf + ((t0 - 1) * B + b) * H + h0 + k);
      }
    } else if (hv) {
      const float *zsrc = z + (t0 * B + b) * 4 * H + h;
      const float *csrc = cbuf + (t0 * B + b) * H + h;
      const float *dsrc = dout + (t0 * B + b) * H + h;
      for (int s = 0; s < nst; ++s) {
#pragma unroll
        for (int g = 0; g < 4; ++g) cp_async4(bs + s * kBwdRow + g * 32 + lane, zsrc + s * zstep + g * H);
        cp_async4(bs + s * kBwdRow + 128 + lane, csrc + s * sstep);
        cp_async4(bs + s * kBwdRow + 160 + lane, dsrc + s * sstep);
      }
      if (t0 > 0) cp_async4(cprev_row + lane, cbuf + ((t0 - 1) * B + b) * H + h);
    }
    cp_async_wait_all();
    __syncwarp();

    // Pass 1 (reverse time): per-step coefficients kept in place
    // (slot i <- KI, f <- KF, g <- KG, o <- f', dout <- dcd; the c slot stays,
    // it is the next step's c_{t-1}), the o-gate gradient (already final),
    // and the tile's map of e.
    float A = 1.f, C = 0.f;
    if (hv) {
      const float c_init = (t0 > 0) ? cprev_row[lane] : fmaxf(c0 ? c0[b * H + h] : 0.f, eps);
#pragma unroll
      for (int s = L - 1; s >= 0; --s) {
        if (s < nst) {
          float *r = bs + s * kBwdRow + lane;
          const int64_t t = t0 + s;
          float d = r[160];
          if (t == T - 1 && dh_n) d += dh_n[b * H + h];
          const float cp = s > 0 ? r[128 - kBwdRow] : c_init;
          const float i = sig_fast(r[0]), f = sigf(r[32]), g = sig_fast(r[64]), o = sig_fast(r[96]);
          const float th = tanh_pos(r[128]);
          const float mb = (i * g >= eps) ? 1.f : 0.f;
          const float mf = (f >= eps) ? 1.f : 0.f;
          const float fp = fmaxf(f, eps);
          float dcd = d * o * (1.f - th * th);
          if (t == T - 1 && dc_n) dcd += dc_n[b * H + h];
          const float dzo = d * th * o * (1.f - o);
          __stcs(dz + (t * B + b) * 4 * H + 3 * H + h, dzo);
          acc3 += dzo;
          amax = fmaxf(amax, fabsf(dzo));
          r[0] = g * i * (1.f - i) * mb;
          r[32] = cp * f * (1.f - f) * mf;
          r[64] = i * g * (1.f - g) * mb;
          r[96] = fp;
          r[160] = dcd;
          C = fp * (C + dcd);
          A *= fp;
        }
      }
    }
    float e = 0.f;
    active = look_back(ws.words + ((int64_t)q * per_chunk + col) * 32 + lane, per_chunk * 32, q, A, C, e, status);

    // Pass 2: e entering this tile's last step, then the exact reverse recurrence.
    if (active && hv) {
#pragma unroll
      for (int s = L - 1; s >= 0; --s) {
        if (s < nst) {
          const float *r = bs + s * kBwdRow + lane;
          const int64_t t = t0 + s;
          const float dc = r[160] + e;
          e = r[96] * dc;
          const float di = dc * r[0], df = dc * r[32], dg = dc * r[64];
          float *dzr = dz + (t * B + b) * 4 * H + h;
          __stcs(dzr, di);
          __stcs(dzr + H, df);
          __stcs(dzr + 2 * H, dg);
          acc0 += di;
          acc1 += df;
          acc2 += dg;
          amax = fmaxf(amax, fmaxf(fabsf(di), fmaxf(fabsf(df), fabsf(dg))));
        }
      }
      if (t0 == 0 && dc0) dc0[b * H + h] = (c0 && c0[b * H + h] >= eps) ? e : 0.f;
    }
  }
  if (dz_absmax) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) atomicMax(dz_absmax, __float_as_uint(amax));
  }

  // Bias-gradient sums of this CTA's WPC tiles, added in a fixed order.
  if (ws.db_part) {
    __syncthreads();  // every warp is done with its staging area
    float *red = reinterpret_cast<float *>(smem_f4);  // [WPC][4][32]
    red[(warp * 4 + 0) * 32 + lane] = acc0;
    red[(warp * 4 + 1) * 32 + lane] = acc1;
    red[(warp * 4 + 2) * 32 + lane] = acc2;
    red[(warp * 4 + 3) * 32 + lane] = acc3;
    __syncthreads();
    if (hv) {
      for (int g = warp; g < 4; g += kBwdWPC) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kBwdWPC; ++w) s += red[(w * 4 + g) * 32 + lane];
        ws.db_part[(grp * B + b) * 4 * H + g * H + h] = s;
      }
    }
  }
}

// db[n] = beta*db[n] + sum_r part[r][n]: 32 columns per CTA, 8 warps over
// rows, partials added in a fixed order.
__global__ void __launch_bounds__(256) rowsum_kernel(const float *__restrict__ part, float *__restrict__ db,
                                                     int64_t R, int64_t N, int beta) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t n = (int64_t)blockIdx.x * 32 + lane;
  float s0 = 0.f, s1 = 0.f;
  if (n < N) {
    int64_t r = w;
    for (; r + 8 < R; r += 16) {
      s0 += part[r * N + n];
      s1 += part[(r + 8) * N + n];
    }
    for (; r < R; r += 8) s0 += part[r * N + n];
  }
  red[w][lane] = s0 + s1;
  __syncthreads();
  if (w == 0 && n < N) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i][lane];
    db[n] = beta ? db[n] + s : s;
  }
}

// *out = max over (t, b, h) of c_{t-1} f'_t (1 - f'_t) (c_{-1} = max(c0, eps),
// f' = max(sigma(z_f), eps)) as float bits, for the look-back forward (the
// per-column forward folds it in).
__global__ void kf_max_kernel(const float *__restrict__ z, const float *__restrict__ c,
                              const float *__restrict__ c0, int64_t T, int64_t B, int64_t H, float eps,
                              unsigned *out) {
  float m = 0.f;
  const int64_t n = T * B * H, BH = B * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / BH, r = i - t * BH, b = r / H, h = r - b * H;
    const float cp = t > 0 ? c[i - BH] : fmaxf(c0 ? c0[r] : 0.f, eps);
    const float f = fmaxf(sigf(z[(t * B + b) * 4 * H + H + h]), eps);
    m = fmaxf(m, cp * f * (1.f - f));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

bool all_aligned16(std::initializer_list<const void *> ptrs) {
  for (const void *p : ptrs)
    if (p && !aligned(p, 16)) return false;
  return true;
}

size_t scan_ws_bytes(int64_t T, int64_t B, int64_t H) {
  const size_t f = ws_layout(make_shape(T, B, H, kFwdL, kFwdWPC), false, nullptr, nullptr);
  const size_t g = ws_layout(make_shape(T, B, H, kBwdL, kBwdWPC), true, nullptr, nullptr);
  return std::max(f, g);
}

int check_scan_args(int64_t T, int64_t B, int64_t H) {
  if (T <= 0 || B <= 0 || H <= 0)
    return fail(HS_ERR_INVALID_ARG, "T, B, H must be positive (got %lld, %lld, %lld)", (long long)T, (long long)B,
                (long long)H);
  const int Lmin = std::min(kFwdL, kBwdL);
  const int Wmin = std::min(kFwdWPC, kBwdWPC);
  if ((T + (int64_t)Lmin * Wmin - 1) / ((int64_t)Lmin * Wmin) * B * ((H + 31) / 32) >= (1ll << 31))
    return fail(HS_ERR_UNSUPPORTED, "scan grid too large");
  if ((T + Lmin - 1) / Lmin >= (1ll << 30)) return fail(HS_ERR_UNSUPPORTED, "T too large");
  return HS_OK;
}

std::atomic<unsigned long long> g_fwd_smem_set[2], g_bwd_smem_set[2];

}  // namespace

size_t scan_workspace(int64_t T, int64_t B, int64_t H) { return scan_ws_bytes(T, B, H); }

// ------------------------------------------------------------------ host API
int scan_forward(const float *z, const float *c0, float *out, float *c, float *h_n, float *c_n, int64_t T,
                 int64_t B, int64_t H, float eps, void *ws_base, size_t ws_bytes, int *status, cudaStream_t st,
                 unsigned *kf_max = nullptr) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !out || !c || !status) return fail(HS_ERR_INVALID_ARG, "scan_forward: null z/out/c/status");
  if (kf_max && cudaMemsetAsync(kf_max, 0, 4, st) != cudaSuccess) return check_launch("kf_max memset");
  if (scan_chain_wanted(T, B, H))  // one CTA per column, no scratch
    return scan_fwd_chain_launch(z, c0, out, c, h_n, c_n, T, B, H, eps, kf_max, status, st);
  if (!ws_base || !aligned(ws_base, 256))
    return fail(HS_ERR_INVALID_ARG, "workspace must be non-null and 256-byte aligned");
  const ScanShape sh = make_shape(T, B, H, kFwdL, kFwdWPC);
  ScanWs ws;
  const size_t need = ws_layout(sh, false, &ws, ws_base);
  if (ws_bytes < need) return fail(HS_ERR_WORKSPACE, "scan_forward: workspace %zu < %zu bytes", ws_bytes, need);
  if (cudaMemsetAsync(ws.words, 0, ws_words_bytes(sh), st) != cudaSuccess) return check_launch("scan memset");
  const bool v16 = H % 4 == 0 && aligned(z, 16);
  const void *fn = v16 ? (const void *)scan_fwd_kernel<true> : (const void *)scan_fwd_kernel<false>;
  if (int e = allow_dynamic_smem(fn, kFwdSmem, &g_fwd_smem_set[v16])) return e;
  const unsigned grid = (unsigned)((int64_t)sh.ngroup * B * sh.ncol);
  if (v16)
    scan_fwd_kernel<true><<<grid, kFwdWPC * 32, kFwdSmem, st>>>(z, c0, out, c, h_n, c_n, sh, eps, ws, status);
  else
    scan_fwd_kernel<false><<<grid, kFwdWPC * 32, kFwdSmem, st>>>(z, c0, out, c, h_n, c_n, sh, eps, ws, status);
  if (int e = check_launch("scan_fwd_kernel")) return e;
  if (!kf_max) return HS_OK;
  const int64_t n = T * B * H;
  kf_max_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 8 * 1024), 256, 0, st>>>(z, c, c0, T, B, H, eps, kf_max);
  return check_launch("kf_max_kernel");
}

int scan_backward(const float *z, const float *c, const float *c0, const float *dout, const float *dh_n,
                  const float *dc_n, float *dz, float *dc0, float *db, int64_t T, int64_t B, int64_t H, float eps,
                  void *ws_base, size_t ws_bytes, int *status, cudaStream_t st, unsigned *dz_absmax) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !c || !dout || !dz || !status) return fail(HS_ERR_INVALID_ARG, "scan_backward: null z/c/dout/dz/status");
  if (!ws_base || !aligned(ws_base, 256))
    return fail(HS_ERR_INVALID_ARG, "workspace must be non-null and 256-byte aligned");
  const ScanShape sh = make_shape(T, B, H, kBwdL, kBwdWPC);
  ScanWs ws;
  const size_t need = ws_layout(sh, db != nullptr, &ws, ws_base);
  if (ws_bytes < need) return fail(HS_ERR_WORKSPACE, "scan_backward: workspace %zu < %zu bytes", ws_bytes, need);
  const int64_t N = 4 * H;
  const bool v16 = H % 4 == 0 && all_aligned16({z, c, dout});
  if (scan_chain_wanted(T, B, H)) {
    // one CTA per column; bias sums per sequence
    if (int e = scan_bwd_chain_launch(z, c, c0, dout, dh_n, dc_n, dz, dc0, db ? ws.db_part : nullptr, T, B, H, eps,
                                      dz_absmax, status, st))
      return e;
    if (db) {
      rowsum_kernel<<<(unsigned)((N + 31) / 32), 256, 0, st>>>(ws.db_part, db, B, N, 0);
      return check_launch("rowsum_kernel");
    }
    return HS_OK;
  }
  if (cudaMemsetAsync(ws.words, 0, ws_words_bytes(sh), st) != cudaSuccess) return check_launch("scan memset");
  const void *fn = v16 ? (const void *)scan_bwd_kernel<true> : (const void *)scan_bwd_kernel<false>;
  if (int e = allow_dynamic_smem(fn, kBwdSmem, &g_bwd_smem_set[v16])) return e;
  const unsigned grid = (unsigned)((int64_t)sh.ngroup * B * sh.ncol);
  if (v16)
    scan_bwd_kernel<true><<<grid, kBwdWPC * 32, kBwdSmem, st>>>(z, c, c0, dout, dh_n, dc_n, dz, dc0, sh, eps, ws,
                                                                dz_absmax, status);
  else
    scan_bwd_kernel<false><<<grid, kBwdWPC * 32, kBwdSmem, st>>>(z, c, c0, dout, dh_n, dc_n, dz, dc0, sh, eps, ws,
                                                                 dz_absmax, status);
  if (int e = check_launch("scan_bwd_kernel")) return e;
  if (db) {
    rowsum_kernel<<<(unsigned)((N + 31) / 32), 256, 0, st>>>(ws.db_part, db, (int64_t)sh.ngroup * B, N, 0);
    return check_launch("rowsum_kernel");
  }
  return HS_OK;
}

// ------------------------------------------------------------------ backward into the fp16 split
// The gradient GEMMs after the scan take dZ as its 3 x fp16 split, scaled by
// a power of two chosen from max |dZ|.  Writing the split from the scan
// itself (instead of float32 dZ and a split pass reading it back) needs the
// scale before the first element, so it comes from an upper bound:
//   e_t = sum_{s>=t} (prod f') d_s o_s (1 - tanh^2 c_s)  + (prod f') dc_n,
// with f' <= 1, so |e_t| <= D = max over columns of sum_t |dout| + |dh_n| +
// |dc_n|.  The o, i and g components are at most D/4 (sigmoid derivatives
// are <= 1/4, gates <= 1) and the forget component e c_{t-1} f'(1 - f') at
// most D Kf, Kf being the forward's maximum of c_{t-1} f'(1 - f') (the cell
// state is large only where f' is near 1, which that product accounts for).
// After the scan the exact max |dZ| it
// folded in is compared with the bound: if the bound was more than 2^16 too
// large (the small elements would lose bits in fp16's subnormal range), or
// anything is not finite, the scan runs again into float32 dZ (in place of
// Z) and the split is made from the exact maximum.  Both re-run kernels
// return at once when the flag says they are not needed.
namespace {
constexpr int kBoundSteps = 256;

// part[j][i] = sum of |dout[t][i]| over steps t of block j (i = b*H + h).
// V4: four columns per thread with 16-byte loads (BH % 4 == 0, aligned);
// four steps in flight per thread either way.
template <bool V4>
__global__ void dout_colsum_kernel(const float *__restrict__ dout, int64_t T, int64_t BH, float *__restrict__ part) {
  constexpr int W = V4 ? 4 : 1;
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * W;
  if (i >= BH) return;
  const int64_t t0 = (int64_t)blockIdx.y * kBoundSteps, t1 = min(T, t0 + kBoundSteps);
  const float *p = dout + t0 * BH + i;
  float acc[4][W];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int k = 0; k < W; ++k) acc[u][k] = 0.f;
  auto add = [&](int u, const float *q) {
    if constexpr (V4) {
      const float4 v = __ldcs(reinterpret_cast<const float4 *>(q));
      acc[u][0] += fabsf(v.x);
      acc[u][1] += fabsf(v.y);
      acc[u][2] += fabsf(v.z);
      acc[u][3] += fabsf(v.w);
    } else {
      acc[u][0] += fabsf(__ldcs(q));
    }
  };
  int64_t t = t0;
  for (; t + 3 < t1; t += 4, p += 4 * BH) {
#pragma unroll
    for (int u = 0; u < 4; ++u) add(u, p + u * BH);
  }
  for (; t < t1; ++t, p += BH) add(0, p);
#pragma unroll
  for (int k = 0; k < W; ++k)
    part[(int64_t)blockIdx.y * BH + i + k] = (acc[0][k] + acc[1][k]) + (acc[2][k] + acc[3][k]);
}

// words[1] = max over columns of the summed |dout| (+ |dh_n| + |dc_n|) as
// float bits by atomicMax (zeroed before).  Sums over the step blocks in a
// fixed order.
__global__ void dout_bound_kernel(const float *__restrict__ part, int64_t nj, int64_t BH,
                                  const float *__restrict__ dh_n, const float *__restrict__ dc_n, unsigned *words) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float d = 0.f;
  if (i < BH) {
    for (int64_t j = 0; j < nj; ++j) d += part[j * BH + i];
    if (dh_n) d += fabsf(dh_n[i]);
    if (dc_n) d += fabsf(dc_n[i]);
  }
  // NaN stays visible: fmaxf would drop it, so it is mapped to +inf first
  if (d != d) d = __int_as_float(0x7f800000);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) d = fmaxf(d, __shfl_xor_sync(0xffffffffu, d, o));
  if ((threadIdx.x & 31) == 0) atomicMax(&words[1], __float_as_uint(d));
}

// words[0] = the bound D x max(1/4, Kf), Kf = the forward's max of
// c_{t-1} f' (1 - f').
__global__ void dz_bound_final_kernel(unsigned *words, const unsigned *kf_max) {
  const float D = __uint_as_float(words[1]);
  words[0] = __float_as_uint(D * fmaxf(__uint_as_float(*kf_max), 0.25f));
}

// After the split scan: words[3] = exact max |dZ|.  Sets words[5] (re-run
// flag) and words[4] (the scale word the GEMMs read: the bound, or the exact
// maximum when re-running).
__global__ void dz_check_kernel(unsigned *words) {
  const float y = __uint_as_float(words[3]) * pow2_scale(words[0]);
  const bool ok = y >= 0.25f && y < 32768.0f;  // bound at most 2^16 above the maximum, and above it
  reinterpret_cast<int *>(words)[5] = ok ? 0 : 1;
  words[4] = ok ? words[0] : words[3];
}
}  // namespace

size_t scan_split_ws_bytes(int64_t T, int64_t B, int64_t H) {
  const int64_t nj = (T + kBoundSteps - 1) / kBoundSteps;
  return 256 + round_up(scan_ws_bytes(T, B, H), 256) + round_up((size_t)nj * B * H * 4, 256);
}

// dZ of the scan backward as its fp16 split (hi then lo, [T*B][4H] each) in
// dz_split, the scale's float bits in *dz_scale; z may be overwritten (the
// re-run).  kf_max: the forward's max of c_{t-1} f'(1 - f')
// (hs_scan_forward_kf).
int scan_backward_split(float *z, const float *c, const float *c0, const float *dout, const float *dh_n,
                        const float *dc_n, const unsigned *kf_max, void *dz_split, unsigned *dz_scale, float *dc0,
                        float *db, int64_t T, int64_t B, int64_t H, float eps, void *ws_base, size_t ws_bytes,
                        int *status, cudaStream_t st) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !c || !dout || !dz_split || !dz_scale || !status)
    return fail(HS_ERR_INVALID_ARG, "scan_backward_split: null z/c/dout/dz_split/dz_scale/status");
  if (!ws_base || !aligned(ws_base, 256) || !aligned(dz_split, 16))
    return fail(HS_ERR_INVALID_ARG, "workspace must be 256-byte and dz_split 16-byte aligned");
  if (ws_bytes < scan_split_ws_bytes(T, B, H))
    return fail(HS_ERR_WORKSPACE, "scan_backward_split: workspace %zu < %zu bytes", ws_bytes,
                scan_split_ws_bytes(T, B, H));
  unsigned *words = static_cast<unsigned *>(ws_base);
  char *sws = static_cast<char *>(ws_base) + 256;
  const size_t sws_bytes = round_up(scan_ws_bytes(T, B, H), 256);
  float *part = reinterpret_cast<float *>(sws + sws_bytes);
  const int64_t M = T * B, N = 4 * H, BH = B * H;
  const bool fused = kf_max && scan_chain_wanted(T, B, H) && H % 4 == 0 && all_aligned16({z, c, dout});
  if (!fused) {  // float32 dZ in place, then the split from its exact maximum
    if (cudaMemsetAsync(dz_scale, 0, 4, st) != cudaSuccess) return check_launch("dz_scale memset");
    if (int e = scan_backward(z, c, c0, dout, dh_n, dc_n, z, dc0, db, T, B, H, eps, sws, sws_bytes, status, st,
                              dz_scale))
      return e;
    return h3_split_known(z, M, N, N, dz_scale, dz_split, st, nullptr);
  }
  if (cudaMemsetAsync(words, 0, 256, st) != cudaSuccess) return check_launch("scan split memset");
  const int64_t nj = (T + kBoundSteps - 1) / kBoundSteps;
  if (BH % 4 == 0)  // dout is 16-byte aligned on this path
    dout_colsum_kernel<true><<<dim3((unsigned)((BH / 4 + 255) / 256), (unsigned)nj), 256, 0, st>>>(dout, T, BH, part);
  else
    dout_colsum_kernel<false><<<dim3((unsigned)((BH + 255) / 256), (unsigned)nj), 256, 0, st>>>(dout, T, BH, part);
  if (int e = check_launch("dout_colsum_kernel")) return e;
  dout_bound_kernel<<<(unsigned)((BH + 255) / 256), 256, 0, st>>>(part, nj, BH, dh_n, dc_n, words);
  if (int e = check_launch("dout_bound_kernel")) return e;
  dz_bound_final_kernel<<<1, 1, 0, st>>>(words, kf_max);
  if (int e = check_launch("dz_bound_final_kernel")) return e;
  const ScanShape sh = make_shape(T, B, H, kBwdL, kBwdWPC);
  ScanWs ws;
  (void)ws_layout(sh, true, &ws, sws);
  __half *hi = static_cast<__half *>(dz_split);
  __half *lo = hi + M * N;
  if (int e = scan_bwd_chain_launch(z, c, c0, dout, dh_n, dc_n, z, dc0, db ? ws.db_part : nullptr, T, B, H, eps,
                                    &words[3], status, st, hi, lo, &words[0], nullptr))
    return e;
  if (db) {
    rowsum_kernel<<<(unsigned)((N + 31) / 32), 256, 0, st>>>(ws.db_part, db, B, N, 0);
    if (int e = check_launch("rowsum_kernel")) return e;
  }
  dz_check_kernel<<<1, 1, 0, st>>>(words);
  if (int e = check_launch("dz_check_kernel")) return e;
  const int *redo = reinterpret_cast<const int *>(&words[5]);
  if (int e = scan_bwd_chain_launch(z, c, c0, dout, dh_n, dc_n, z, dc0, nullptr, T, B, H, eps, nullptr, status, st,
                                    nullptr, nullptr, nullptr, redo))
    return e;
  if (int e = h3_split_known(z, M, N, N, &words[4], dz_split, st, redo)) return e;
  if (cudaMemcpyAsync(dz_scale, &words[4], 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return check_launch("dz_scale copy");
  return HS_OK;
}

// ------------------------------------------------------------------ bf16 storage
// A bf16 module's scans: Z, c, out and dout stored in bf16 (half the bytes of
// the saved activations), dZ written in bf16 for the bf16 gradient GEMMs;
// the arithmetic and the carried state stay float32.  Per-column kernels
// only (every 8-unit bf16 copy inside one column): shapes they do not take
// are refused, and the caller widens to float32 instead.
int scan_fwd_chain_launch_bf16(const void *z, const float *c0, void *out, void *c, float *h_n, float *c_n, int64_t T,
                               int64_t B, int64_t H, float eps, int *status, cudaStream_t st);
int scan_bwd_chain_launch_bf16(const void *z, const void *c, const float *c0, const void *dout, const float *dh_n,
                               const float *dc_n, void *dz, float *dc0, float *db_part, int64_t T, int64_t B,
                               int64_t H, float eps, int *status, cudaStream_t st);

bool scan_bf16_ok(int64_t T, int64_t B, int64_t H) {
  return T > 0 && B > 0 && H > 0 && H % 8 == 0 && scan_chain_wanted(T, B, H);
}
size_t scan_bf16_ws_bytes(int64_t B, int64_t H) { return round_up((size_t)B * 4 * H * 4, 256); }

int scan_forward_bf16(const void *z, const float *c0, void *out, void *c, float *h_n, float *c_n, int64_t T, int64_t B,
                      int64_t H, float eps, int *status, cudaStream_t st) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !out || !c || !status) return fail(HS_ERR_INVALID_ARG, "scan_forward_bf16: null z/out/c/status");
  if (!scan_bf16_ok(T, B, H))
    return fail(HS_ERR_UNSUPPORTED, "bf16 scan: needs H %% 8 == 0 and a shape the per-column kernels take");
  return scan_fwd_chain_launch_bf16(z, c0, out, c, h_n, c_n, T, B, H, eps, status, st);
}

int scan_backward_bf16(const void *z, const void *c, const float *c0, const void *dout, const float *dh_n,
                       const float *dc_n, void *dz, float *dc0, float *db, int64_t T, int64_t B, int64_t H, float eps,
                       void *ws, size_t ws_bytes, int *status, cudaStream_t st) {
  if (int e = check_scan_args(T, B, H)) return e;
  if (!z || !c || !dout || !dz || !status) return fail(HS_ERR_INVALID_ARG, "scan_backward_bf16: null z/c/dout/dz/status");
  if (!scan_bf16_ok(T, B, H))
    return fail(HS_ERR_UNSUPPORTED, "bf16 scan: needs H %% 8 == 0 and a shape the per-column kernels take");
  const int64_t N = 4 * H;
  float *part = nullptr;
  if (db) {
    if (!ws || !aligned(ws, 256) || ws_bytes < scan_bf16_ws_bytes(B, H))
      return fail(HS_ERR_WORKSPACE, "scan_backward_bf16: workspace %zu < %zu bytes", ws_bytes, scan_bf16_ws_bytes(B, H));
    part = static_cast<float *>(ws);
  }
  if (int e = scan_bwd_chain_launch_bf16(z, c, c0, dout, dh_n, dc_n, dz, dc0, part, T, B, H, eps, status, st))
    return e;
  if (db) {
    rowsum_kernel<<<(unsigned)((N + 31) / 32), 256, 0, st>>>(part, db, B, N, 0);
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
  // Shapes that scan_forward sends to the one-CTA-per-column chain kernels
  // use no scratch at all; only the look-back path is limited by the array.
  if (!scan_chain_wanted(T, B, H)) {
    const size_t need = ws_layout(make_shape(T, B, H, kFwdL, kFwdWPC), false, nullptr, nullptr);
    if (need > kNoAllocScratchBytes)
      return fail(HS_ERR_UNSUPPORTED,
                  "hs_scan_forward_noalloc: T=%lld B=%lld H=%lld needs %zu bytes of scratch, above "
                  "the fixed %zu-byte array; use hs_scan_forward with a caller workspace",
                  (long long)T, (long long)B, (long long)H, need, kNoAllocScratchBytes);
  }
  void *scratch = nullptr;
  int *own_status = nullptr;
  if (int e = noalloc_scratch(&scratch, &own_status)) return e;
  if (!dev_status) {
    // The library's own status word reports this call only: cleared in
    // stream order first, so a wait that gave up in an earlier call does not
    // make this one's kernels return at entry.  hs_scan_noalloc_status reads
    // and clears it.
    if (cudaMemsetAsync(own_status, 0, sizeof(int), st) != cudaSuccess)
      return check_launch("hs_scan_forward_noalloc status memset");
  }
  // scan_forward zeroes the look-back words (all that must start at zero)
  // with a stream-ordered memset before its launch; the chain kernels it may
  // pick instead use no scratch.
  return scan_forward(z, c0, out, c, h_n, c_n, T, B, H, eps, scratch, kNoAllocScratchBytes,
                      dev_status ? dev_status : own_status, st);
}

int noalloc_status_word(int **word) {
  void *scratch = nullptr;
  return noalloc_scratch(&scratch, word);
}

int scan_noalloc_status(int *host_status, cudaStream_t st) {
  if (!host_status) return fail(HS_ERR_INVALID_ARG, "hs_scan_noalloc_status: null host_status");
  void *scratch = nullptr;
  int *own_status = nullptr;
  if (int e = noalloc_scratch(&scratch, &own_status)) return e;
  if (cudaMemcpyAsync(host_status, own_status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return check_launch("hs_scan_noalloc_status read");
  if (cudaMemsetAsync(own_status, 0, sizeof(int), st) != cudaSuccess)
    return check_launch("hs_scan_noalloc_status clear");
  if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("hs_scan_noalloc_status sync");
  return HS_OK;
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
                           workspace_bytes, dev_status, (cudaStream_t)stream, nullptr);
}

int hs_scan_backward_absmax(const float *z, const float *c, const float *c0, const float *dout,
                            const float *dh_n, const float *dc_n, float *dz, float *dc0, float *db, int64_t T,
                            int64_t B, int64_t H, float eps, void *workspace, size_t workspace_bytes,
                            unsigned *dz_absmax, int *dev_status, hs_stream_t stream) {
  if (!dz_absmax || !hs::aligned(dz_absmax, 4))
    return hs::fail(HS_ERR_INVALID_ARG, "hs_scan_backward_absmax: null or misaligned dz_absmax");
  if (cudaMemsetAsync(dz_absmax, 0, 4, (cudaStream_t)stream) != cudaSuccess)
    return hs::check_launch("hs_scan_backward_absmax memset");
  return hs::scan_backward(z, c, c0, dout, dh_n, dc_n, dz, dc0, db, T, B, H, eps, workspace, workspace_bytes,
                           dev_status, (cudaStream_t)stream, dz_absmax);
}

int hs_scan_forward_bf16(const void *z, const float *c0, void *out, void *c, float *h_n, float *c_n, int64_t T,
                         int64_t B, int64_t H, float eps, int *dev_status, hs_stream_t stream) {
  return hs::scan_forward_bf16(z, c0, out, c, h_n, c_n, T, B, H, eps, dev_status, (cudaStream_t)stream);
}

size_t hs_scan_bf16_workspace_bytes(int64_t T, int64_t B, int64_t H) {
  return (T > 0 && B > 0 && H > 0) ? hs::scan_bf16_ws_bytes(B, H) : 0;
}

int hs_scan_backward_bf16(const void *z, const void *c, const float *c0, const void *dout, const float *dh_n,
                          const float *dc_n, void *dz, float *dc0, float *db, int64_t T, int64_t B, int64_t H,
                          float eps, void *workspace, size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::scan_backward_bf16(z, c, c0, dout, dh_n, dc_n, dz, dc0, db, T, B, H, eps, workspace, workspace_bytes,
                                dev_status, (cudaStream_t)stream);
}

int hs_scan_uses_column_kernels(int64_t T, int64_t B, int64_t H) {
  return (T > 0 && B > 0 && H > 0 && hs::scan_chain_wanted(T, B, H)) ? 1 : 0;
}

int64_t hs_scan_wave_sequences(int64_t H) { return hs::scan_wave_sequences(H); }

size_t hs_scan_split_workspace_bytes(int64_t T, int64_t B, int64_t H) {
  return (T > 0 && B > 0 && H > 0) ? hs::scan_split_ws_bytes(T, B, H) : 0;
}

int hs_scan_forward_kf(const float *z, const float *c0, float *out, float *c, float *h_n, float *c_n, int64_t T,
                           int64_t B, int64_t H, float eps, void *workspace, size_t workspace_bytes,
                           unsigned *kf_max, int *dev_status, hs_stream_t stream) {
  if (!kf_max || !hs::aligned(kf_max, 4))
    return hs::fail(HS_ERR_INVALID_ARG, "hs_scan_forward_kf: null or misaligned kf_max");
  return hs::scan_forward(z, c0, out, c, h_n, c_n, T, B, H, eps, workspace, workspace_bytes, dev_status,
                          (cudaStream_t)stream, kf_max);
}

int hs_scan_backward_split(float *z, const float *c, const float *c0, const float *dout, const float *dh_n,
                           const float *dc_n, const unsigned *kf_max, void *dz_split, unsigned *dz_scale,
                           float *dc0, float *db, int64_t T, int64_t B, int64_t H, float eps, void *workspace,
                           size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::scan_backward_split(z, c, c0, dout, dh_n, dc_n, kf_max, dz_split, dz_scale, dc0, db, T, B, H, eps,
                                 workspace, workspace_bytes, dev_status, (cudaStream_t)stream);
}

int hs_scan_forward_noalloc(const float *z, const float *c0, float *out, float *c, float *h_n,
                            float *c_n, int64_t T, int64_t B, int64_t H, float eps,
                            int *dev_status, hs_stream_t stream) {
  return hs::scan_forward_noalloc(z, c0, out, c, h_n, c_n, T, B, H, eps, dev_status,
                                  (cudaStream_t)stream);
}

int hs_scan_noalloc_status(int *host_status, hs_stream_t stream) {
  return hs::scan_noalloc_status(host_status, (cudaStream_t)stream);
}

}  // extern "C"
