// Parallel-mode scan, one CTA per column: the path for shapes with many
// independent columns (a column = one sequence x 32 consecutive hidden units)
// and long T, such as the configs[4] training step (B x H/32 = 1024 columns of
// 16384 steps per 32-sequence micro-batch).
//
// The recurrence is the one of scan.cu (c_t = max(f,eps) c_{t-1} +
// max(i g,eps); reference src/headstartlstm/_parallel.py:21-74), split over
// time inside the CTA instead of across CTAs: time is cut into chunks of L
// steps and warp w takes chunks w, w+NW, w+2NW, ... of the CTA's column, lane
// l owning hidden unit h0+l.  For each chunk the warp computes the gate
// activations and the chunk's affine map (A, C) while it waits for nothing,
// then takes the carry into the chunk from a shared-memory slot written by the
// warp of the previous chunk, hands A*carry + C on to the next warp at once,
// and only then writes the chunk's outputs.  The carry therefore moves
// through the CTA at shared-memory latency (one slot write per chunk) while
// every warp's loads, math and stores overlap; no other CTA and no global
// scratch is involved, so nothing has to be cleared between calls.
//
// Inputs stream into a per-warp double buffer with 16-byte cp.async copies
// (L2 -> shared, no L1 allocation) issued two chunks ahead.  Rows of 32
// floats are 128-byte aligned segments: every warp access is one full line.
// Per (t,b,h) element the forward moves its 24 algorithmic bytes and the
// backward its 40, plus one c row per backward chunk (c_{t0-1}).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "hs_common.cuh"

namespace hs {
namespace {

// Chunk length L and warps per CTA NW (compile-time; the defaults are the
// measured best on B200 for the benchmark shapes).  The shared memory per
// CTA is sized so that seven CTAs fit on an SM: 1036 resident CTAs on 148
// SMs hold all 1024 columns of a 32-sequence, H=1024 micro-batch at once.
#ifndef HS_CHAIN_FWD_L
#define HS_CHAIN_FWD_L 6
#endif
#ifndef HS_CHAIN_FWD_NW
#define HS_CHAIN_FWD_NW 4
#endif
#ifndef HS_CHAIN_BWD_L
#define HS_CHAIN_BWD_L 4
#endif
#ifndef HS_CHAIN_BWD_NW
#define HS_CHAIN_BWD_NW 4
#endif
#ifndef HS_CHAIN_MIN_CTAS
#define HS_CHAIN_MIN_CTAS 7
#endif
// Resident CTAs per SM the register budget allows on the 16-byte path; the
// 4-byte path (H % 4 != 0 or unaligned inputs) needs more registers and
// takes two fewer.
constexpr int kMinCtas = HS_CHAIN_MIN_CTAS;
constexpr int kFL = HS_CHAIN_FWD_L, kFNW = HS_CHAIN_FWD_NW;
constexpr int kBL = HS_CHAIN_BWD_L, kBNW = HS_CHAIN_BWD_NW;
constexpr int kFRow = 4 * 32;              // staged floats per forward step: z_i, z_f, z_g, z_o
constexpr int kBRow = 6 * 32;              // backward: z_i, z_f, z_g, z_o, c, dout
constexpr int kFBuf = kFL * kFRow;         // floats per forward chunk buffer
constexpr int kBBuf = kBL * kBRow + 32;    // backward, + the c_{t0-1} row
constexpr size_t kFSmem = sizeof(float) * kFNW * 2 * kFBuf + sizeof(unsigned long long) * kFNW * 32;
constexpr size_t kBSmem = sizeof(float) * kBNW * 2 * kBBuf + sizeof(unsigned long long) * kBNW * 32;
static_assert(kBNW * 2 * kBBuf >= kBNW * 4 * 32, "db reduction area");

// 16- and 4-byte copies global -> shared; .cg bypasses L1, so in-flight lines
// do not compete with the shared-memory carve-out.
// Destinations are shared-window addresses (see sa()).
HS_DEV void cp16(unsigned dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
HS_DEV void cp4(unsigned dst, const float *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
HS_DEV unsigned sa(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
HS_DEV void commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> HS_DEV void wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Storage of Z, c, out and dout: float32, or bf16 (a bf16 module's path,
// whose saved activations are half the bytes).  Staged rows keep the float32
// layout's element positions (32 units per gate row), at 2 bytes each.
template <typename TS> HS_DEV float lds(const float *buf, int i) {
  if constexpr (std::is_same<TS, float>::value) return buf[i];
  else return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(buf)[i]);
}
template <typename TS> HS_DEV void st_cs(TS *p, float v) {
  if constexpr (std::is_same<TS, float>::value) __stcs(p, v);
  else __stcs(reinterpret_cast<unsigned short *>(p), __bfloat16_as_ushort(__float2bfloat16_rn(v)));
}

// Carry slots: one 64-bit shared word per (consumer warp, lane), holding
// (chunk index << 32) | float bits.  The consumer of chunk c (c >= 1) waits for
// tag c, so the initial zero is never mistaken for a carry.  A slot is written
// again (tag c+NW) only after its consumer has read tag c: the producer's next
// carry depends, around the ring of warps, on the consumer's own next carry.
HS_DEV void slot_put(unsigned long long *s, unsigned tag, float v) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.volatile.shared.u64 [%0], %1;" ::"r"((unsigned)__cvta_generic_to_shared(s)), "l"(w) : "memory");
}
HS_DEV unsigned long long slot_get(const unsigned long long *s) {
  unsigned long long w;
  asm volatile("ld.volatile.shared.u64 %0, [%1];" : "=l"(w) : "r"((unsigned)__cvta_generic_to_shared(s)) : "memory");
  return w;
}
// Waits for tag in *s; bounded by kWaitLimitNs and by the sticky status word.
HS_DEV bool slot_wait(const unsigned long long *s, unsigned tag, float *v, int *status) {
  uint64_t t0 = 0;
  for (unsigned n = 0;; ++n) {
    const unsigned long long w = slot_get(s);
    if ((unsigned)(w >> 32) == tag) {
      *v = __uint_as_float((unsigned)w);
      return true;
    }
    if (n >= 32) {
      __nanosleep(32);
      if ((n & 63) == 0) {
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

// ------------------------------------------------------------------ forward
// TS = __nv_bfloat16: z, out and c in bf16 (needs V16: H % 8 == 0, 16-byte
// aligned), c0, h_n, c_n float32.
template <bool V16, typename TS = float>
__global__ void __launch_bounds__(kFNW * 32, V16 ? kMinCtas : kMinCtas - 2)
scan_fwd_col_kernel(const TS *__restrict__ z, const float *__restrict__ c0, TS *__restrict__ out,
                    TS *__restrict__ cbuf, float *__restrict__ h_n, float *__restrict__ c_n, int64_t T,
                    int64_t B, int64_t H, float eps, unsigned *kf_max, int *status) {
  constexpr bool BF = !std::is_same<TS, float>::value;
  static_assert(!BF || V16, "bf16 storage takes the 16-byte copies");
  extern __shared__ float4 smem_f4[];
  float *sm = reinterpret_cast<float *>(smem_f4);
  unsigned long long *slots = reinterpret_cast<unsigned long long *>(sm + kFNW * 2 * kFBuf);  // [NW][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t ncol = (H + 31) / 32;
  const int64_t b = blockIdx.x / ncol;
  const int64_t h0 = (blockIdx.x - b * ncol) * 32;
  const int64_t h = h0 + lane;
  const bool hv = h < H;
  const int64_t nchunk = (T + kFL - 1) / kFL;
  const int64_t zstep = B * 4 * H, ostep = B * H;
  const TS *zb = z + b * 4 * H;
  float *buf0 = sm + warp * 2 * kFBuf;
  slots[warp * 32 + lane] = 0ull;
  __syncthreads();

  // Copies of one chunk into a buffer: pointers advance by one step per copy
  // (no per-step index products).
  auto stage = [&](int64_t c, float *dst) {
    const int64_t t0 = c * kFL;
    const int n = (int)min((int64_t)kFL, T - t0);
    if constexpr (BF) {
      // a step row is 4 gates x 32 units x 2 bytes = 16 copies of 8 units:
      // lanes 0-15 take the chunk's even steps, 16-31 the odd ones
      const int g = (lane & 15) >> 2, k = (lane & 3) * 8, s0 = lane >> 4;
      if (h0 + k < H) {
        const TS *src = zb + (t0 + s0) * zstep + g * H + h0 + k;
        unsigned d = sa(dst) + (unsigned)((s0 * kFRow + g * 32 + k) * 2);
        for (int s = s0; s < n; s += 2, src += 2 * zstep, d += 2 * kFRow * 2) cp16(d, src);
      }
    } else if (V16) {
      const int g = lane >> 3, k = (lane & 7) * 4;
      if (h0 + k < H) {
        const float *src = zb + t0 * zstep + g * H + h0 + k;
        unsigned d = sa(dst + g * 32 + k);
        for (int s = 0; s < n; ++s, src += zstep, d += kFRow * 4) cp16(d, src);
      }
    } else if (hv) {
      const float *src = zb + t0 * zstep + h;
      unsigned d = sa(dst + lane);
#pragma unroll 1
      for (int s = 0; s < n; ++s, src += zstep, d += kFRow * 4)
#pragma unroll
        for (int g = 0; g < 4; ++g) cp4(d + g * 128, src + g * H);
    }
  };

  // max over this lane's steps of c_{t-1} f'_t (1 - f'_t), the forget-gate
  // factor of the backward's bound on |dZ| (if kf_max is wanted)
  float kmax = 0.f;
  int64_t c = warp;
  if (c < nchunk) stage(c, buf0);
  commit();
  if (c + kFNW < nchunk) stage(c + kFNW, buf0 + kFBuf);
  commit();
  for (int i = 0; c < nchunk; c += kFNW, ++i) {
    float *buf = buf0 + (i & 1) * kFBuf;
    wait_group<1>();  // this chunk's copies are done (the next chunk's may still fly)
    __syncwarp();
    const int64_t t0 = c * kFL;
    const int n = (int)min((int64_t)kFL, T - t0);
    float fp[kFL], bp[kFL], eo[kFL];  // f', b', e^-z_o
    float A = 1.f, C = 0.f;
    // Full chunks (all but a sequence's last one, every lane valid) take a
    // copy of the step loops without per-step conditions.
    const bool full = n == kFL && hv;
    auto coeffs = [&](auto full_tag) {
#pragma unroll
      for (int s = 0; s < kFL; ++s) {
        if (decltype(full_tag)::value || (s < n && hv)) {
          const int r = s * kFRow + lane;
          fp[s] = fmaxf(sigf(lds<TS>(buf, r + 32)), eps);
          bp[s] = fmaxf(sig2(lds<TS>(buf, r), lds<TS>(buf, r + 64)), eps);
          eo[s] = __expf(-lds<TS>(buf, r + 96));
          C = fmaf(fp[s], C, bp[s]);
          A *= fp[s];
        } else {
          fp[s] = 1.f;
          bp[s] = 0.f;
          eo[s] = 0.f;
        }
      }
    };
    if (full) coeffs(std::true_type{});
    else coeffs(std::false_type{});
    __syncwarp();  // every lane has read the buffer before it is refilled
    if (c + 2 * kFNW < nchunk) stage(c + 2 * kFNW, buf);
    commit();
    float cin = fmaxf((c == 0 && c0 && hv) ? c0[b * H + h] : 0.f, eps);
    const bool ok = c == 0 || slot_wait(&slots[warp * 32 + lane], (unsigned)c, &cin, status);
    if (!__all_sync(0xffffffffu, ok)) break;
    if (c + 1 < nchunk) slot_put(&slots[((warp + 1) % kFNW) * 32 + lane], (unsigned)(c + 1), fmaf(A, cin, C));
    if (hv) {
      float cc = cin, o = 0.f;
      TS *ob = out + (t0 * B + b) * H + h;
      TS *cb = cbuf + (t0 * B + b) * H + h;
      auto emit = [&](auto full_tag) {
#pragma unroll
        for (int s = 0; s < kFL; ++s) {
          if (decltype(full_tag)::value || s < n) {
            kmax = fmaxf(kmax, cc * fp[s] * (1.f - fp[s]));
            cc = fmaf(fp[s], cc, bp[s]);
            o = sig_tanh_pos(eo[s], cc);
            st_cs(cb + s * ostep, cc);
            st_cs(ob + s * ostep, o);
          }
        }
      };
      if (full) emit(std::true_type{});
      else emit(std::false_type{});
      if (t0 + n == T) {  // the chunk that ends the sequence
        if (c_n) c_n[b * H + h] = cc;
        if (h_n) h_n[b * H + h] = o;
      }
    }
  }
  wait_group<0>();  // no copy is left in flight at exit
  if (kf_max) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    if (lane == 0) atomicMax(kf_max, __float_as_uint(kmax));
  }
}

// ------------------------------------------------------------------ backward
// Scan order q = 0, 1, ... runs over chunks from the last in time (j =
// nchunk-1-q); the carry is e, the gradient reaching c_{t0-1} of the chunk
// after in time.  Bias sums are kept per lane over all of a warp's chunks and
// added over the CTA's warps in a fixed order at the end: one partial row per
// sequence.
// OUT selects how dZ is written: kDzF32 float32 into dz; kDzSplit its
// 3 x fp16 split (hi, lo [T*B][4H] fp16, scaled by pow2_scale(*dz_bound),
// *dz_bound being an upper bound of max |dZ|); kDzBf16 bf16 into dzb (the
// bf16 gradient GEMMs' operand: bf16 keeps float32's exponent range, so no
// scale).  gate (may be null): the kernel does nothing unless *gate != 0 (a
// conditional re-run).
// TS = __nv_bfloat16: z, c and dout in bf16 (needs V16 and OUT = kDzBf16).
constexpr int kDzF32 = 0, kDzSplit = 1, kDzBf16 = 2;
template <bool V16, int OUT, typename TS = float>
__global__ void __launch_bounds__(kBNW * 32, V16 ? kMinCtas : kMinCtas - 2)
scan_bwd_col_kernel(const TS *z, const TS *__restrict__ cbuf, const float *__restrict__ c0,
                    const TS *__restrict__ dout, const float *__restrict__ dh_n, const float *__restrict__ dc_n,
                    float *dz, float *__restrict__ dc0, float *__restrict__ db_part, int64_t T, int64_t B,
                    int64_t H, float eps, unsigned *dz_absmax, __half *__restrict__ dzh, __half *__restrict__ dzl,
                    const unsigned *__restrict__ dz_bound, __nv_bfloat16 *__restrict__ dzb, const int *gate,
                    int *status) {
  constexpr bool BF = !std::is_same<TS, float>::value;
  static_assert(!BF || (V16 && OUT == kDzBf16), "bf16 storage: 16-byte copies, bf16 dZ");
  if (gate && *gate == 0) return;
  extern __shared__ float4 smem_f4[];
  float *sm = reinterpret_cast<float *>(smem_f4);
  unsigned long long *slots = reinterpret_cast<unsigned long long *>(sm + kBNW * 2 * kBBuf);  // [NW][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t ncol = (H + 31) / 32;
  const int64_t b = blockIdx.x / ncol;
  const int64_t h0 = (blockIdx.x - b * ncol) * 32;
  const int64_t h = h0 + lane;
  const bool hv = h < H;
  const int64_t nchunk = (T + kBL - 1) / kBL;
  const int64_t zstep = B * 4 * H, sstep = B * H;
  float *buf0 = sm + warp * 2 * kBBuf;
  slots[warp * 32 + lane] = 0ull;
  __syncthreads();
  const float c0p = fmaxf((c0 && hv) ? c0[b * H + h] : 0.f, eps);

  auto stage = [&](int64_t q, float *dst) {
    const int64_t t0 = (nchunk - 1 - q) * kBL;
    const int n = (int)min((int64_t)kBL, T - t0);
    if constexpr (BF) {
      // a step row is 6 rows (z_i, z_f, z_g, z_o, c, dout) x 32 units x 2
      // bytes = 24 copies of 8 units, one per lane 0-23; lanes 24-27 copy
      // the c_{t0-1} row
      const int rr = lane >> 2, k = (lane & 3) * 8;
      if (h0 + k < H) {
        if (rr < 6) {
          const TS *src = rr < 4 ? z + (t0 * B + b) * 4 * H + rr * H + h0 + k
                                 : (rr == 4 ? cbuf : dout) + (t0 * B + b) * H + h0 + k;
          const int64_t step = rr < 4 ? zstep : sstep;
          unsigned d = sa(dst) + (unsigned)((rr * 32 + k) * 2);
          for (int s = 0; s < n; ++s, src += step, d += kBRow * 2) cp16(d, src);
        } else if (rr == 6 && t0 > 0) {
          cp16(sa(dst) + (unsigned)((kBL * kBRow + k) * 2), cbuf + ((t0 - 1) * B + b) * H + h0 + k);
        }
      }
    } else if (V16) {
      const int g = lane >> 3, k = (lane & 7) * 4;
      if (h0 + k < H) {
        const float *zsrc = z + (t0 * B + b) * 4 * H + g * H + h0 + k;
        const float *ssrc = (g == 0 ? cbuf : dout) + (t0 * B + b) * H + h0 + k;
        unsigned d = sa(dst + g * 32 + k);
        for (int s = 0; s < n; ++s, zsrc += zstep, ssrc += sstep, d += kBRow * 4) {
          cp16(d, zsrc);
          if (g < 2) cp16(d + 512, ssrc);
        }
        if (g == 0 && t0 > 0) cp16(sa(dst + kBL * kBRow + k), cbuf + ((t0 - 1) * B + b) * H + h0 + k);
      }
    } else if (hv) {
      const float *zsrc = z + (t0 * B + b) * 4 * H + h;
      const float *csrc = cbuf + (t0 * B + b) * H + h;
      const float *dsrc = dout + (t0 * B + b) * H + h;
      unsigned d = sa(dst + lane);
#pragma unroll 1
      for (int s = 0; s < n; ++s, zsrc += zstep, csrc += sstep, dsrc += sstep, d += kBRow * 4) {
#pragma unroll
        for (int g = 0; g < 4; ++g) cp4(d + g * 128, zsrc + g * H);
        cp4(d + 512, csrc);
        cp4(d + 640, dsrc);
      }
      if (t0 > 0) cp4(sa(dst + kBL * kBRow + lane), cbuf + ((t0 - 1) * B + b) * H + h);
    }
  };

  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  float amax = 0.f;  // max |dz| of this lane (NaN ignored), if dz_absmax is wanted
  const float sc = OUT == kDzSplit ? pow2_scale(*dz_bound) : 1.f;
  // One dZ element at offset i of the [T*B][4H] layout.
  auto put = [&](int64_t i, float v) {
    if (OUT == kDzSplit) {
      const float y = v * sc;
      const __half hv = __float2half_rn(y);
      __stcs(dzh + i, hv);
      __stcs(dzl + i, __float2half_rn(y - __half2float(hv)));
    } else if (OUT == kDzBf16) {
      __stcs(reinterpret_cast<unsigned short *>(dzb) + i, __bfloat16_as_ushort(__float2bfloat16_rn(v)));
    } else {
      __stcs(dz + i, v);
    }
  };
  int64_t q = warp;
  if (q < nchunk) stage(q, buf0);
  commit();
  if (q + kBNW < nchunk) stage(q + kBNW, buf0 + kBBuf);
  commit();
  for (int i = 0; q < nchunk; q += kBNW, ++i) {
    float *buf = buf0 + (i & 1) * kBBuf;
    wait_group<1>();
    __syncwarp();
    const int64_t t0 = (nchunk - 1 - q) * kBL;
    const int n = (int)min((int64_t)kBL, T - t0);
    // dh_n joins dout of the sequence's last step; dc_n is the initial
    // carry of the reverse scan (below).
    const float dhn = (q == 0 && dh_n && hv) ? dh_n[b * H + h] : 0.f;
    // Pass 1 (reverse time): per-step coefficients, the o-gate gradient
    // (final already) and the chunk's map of e.
    float FP[kBL], DCD[kBL], KI[kBL], KF[kBL], KG[kBL];
    float A = 1.f, C = 0.f;
    const int64_t dzs = (t0 * B + b) * 4 * H + h;  // dZ offset of step t0, unit h
    // (A condition-free copy of the step loops for full chunks, as in the
    // forward, measured slower here.)
#pragma unroll
    for (int s = kBL - 1; s >= 0; --s) {
      FP[s] = 1.f;
      DCD[s] = KI[s] = KF[s] = KG[s] = 0.f;
      if (s < n && hv) {
        const int r = s * kBRow + lane;
        const float d = lds<TS>(buf, r + 160) + (s == n - 1 ? dhn : 0.f);
        const float cp = s > 0 ? lds<TS>(buf, r + 128 - kBRow) : (t0 > 0 ? lds<TS>(buf, kBL * kBRow + lane) : c0p);
        const float ig = sig_fast(lds<TS>(buf, r)), f = sigf(lds<TS>(buf, r + 32)), g = sig_fast(lds<TS>(buf, r + 64)),
                    o = sig_fast(lds<TS>(buf, r + 96));
        const float th = tanh_pos(lds<TS>(buf, r + 128));
        const float mb = (ig * g >= eps) ? 1.f : 0.f;
        const float mf = (f >= eps) ? 1.f : 0.f;
        const float dcd = d * o * (1.f - th * th);
        const float dzo = d * th * o * (1.f - o);
        put(dzs + s * zstep + 3 * H, dzo);
        acc3 += dzo;
        amax = fmaxf(amax, fabsf(dzo));
        FP[s] = fmaxf(f, eps);
        DCD[s] = dcd;
        KI[s] = g * ig * (1.f - ig) * mb;
        KF[s] = cp * f * (1.f - f) * mf;
        KG[s] = ig * g * (1.f - g) * mb;
        C = FP[s] * (C + dcd);
        A *= FP[s];
      }
    }
    __syncwarp();
    if (q + 2 * kBNW < nchunk) stage(q + 2 * kBNW, buf);
    commit();
    float e = (q == 0 && dc_n && hv) ? dc_n[b * H + h] : 0.f;
    const bool ok = q == 0 || slot_wait(&slots[warp * 32 + lane], (unsigned)q, &e, status);
    if (!__all_sync(0xffffffffu, ok)) break;
    if (q + 1 < nchunk) slot_put(&slots[((warp + 1) % kBNW) * 32 + lane], (unsigned)(q + 1), fmaf(A, e, C));
    if (hv) {
#pragma unroll
      for (int s = kBL - 1; s >= 0; --s) {
        if (s < n) {
          const float dc = DCD[s] + e;
          e = FP[s] * dc;
          const float di = dc * KI[s], df = dc * KF[s], dg = dc * KG[s];
          const int64_t dzr = dzs + s * zstep;
          put(dzr, di);
          put(dzr + H, df);
          put(dzr + 2 * H, dg);
          acc0 += di;
          acc1 += df;
          acc2 += dg;
          amax = fmaxf(amax, fmaxf(fabsf(di), fmaxf(fabsf(df), fabsf(dg))));
        }
      }
      if (t0 == 0 && dc0) dc0[b * H + h] = (c0 && c0[b * H + h] >= eps) ? e : 0.f;
    }
  }
  wait_group<0>();
  if (dz_absmax) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) atomicMax(dz_absmax, __float_as_uint(amax));
  }
  if (db_part) {
    __syncthreads();  // every warp is done with its buffers
    float *red = sm;  // [NW][4][32]
    red[(warp * 4 + 0) * 32 + lane] = acc0;
    red[(warp * 4 + 1) * 32 + lane] = acc1;
    red[(warp * 4 + 2) * 32 + lane] = acc2;
    red[(warp * 4 + 3) * 32 + lane] = acc3;
    __syncthreads();
    if (hv) {
      for (int g = warp; g < 4; g += kBNW) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kBNW; ++w) s += red[(w * 4 + g) * 32 + lane];
        db_part[b * 4 * H + g * H + h] = s;
      }
    }
  }
}

// ------------------------------------------------------------------ two units per lane
// The same scans with lane l owning the adjacent units h0+2l and h0+2l+1 of a
// 64-unit column: staged rows are read as float2 (or bf16x2) pairs and the
// outputs stored as pairs, so the loads, stores, address and loop work of a
// step are shared by two elements (the scans are issue-bound).  Each unit
// keeps its own carry slot ([warp][unit of the pair][lane], conflict-free)
// and its own arithmetic, identical to the one-unit kernels: results are the
// same bit for bit.  Needs H even (both units of a pair valid or neither);
// the 16-byte copies need H % 4 == 0 (float32) or H % 8 == 0 (bf16).
// Half the CTAs of the one-unit kernels, each with twice the shared memory:
// four CTAs per SM hold the 512 columns of a 32-sequence, H=1024 micro-batch
// at once.
constexpr int kMinCtas2 = 4;
constexpr int kF2Row = 4 * 64;              // staged floats per forward step
constexpr int kB2Row = 6 * 64;              // backward: z_i, z_f, z_g, z_o, c, dout
constexpr int kF2Buf = kFL * kF2Row;
constexpr int kB2Buf = kBL * kB2Row + 64;   // + the c_{t0-1} row
constexpr size_t kF2Smem = sizeof(float) * kFNW * 2 * kF2Buf + sizeof(unsigned long long) * kFNW * 64;
constexpr size_t kB2Smem = sizeof(float) * kBNW * 2 * kB2Buf + sizeof(unsigned long long) * kBNW * 64;
static_assert(kBNW * 2 * kB2Buf >= kBNW * 4 * 64, "db reduction area");

// Staged pair at float position i (even) of a buffer holding TS elements.
template <typename TS> HS_DEV float2 lds2(const float *buf, int i) {
  if constexpr (std::is_same<TS, float>::value) return *reinterpret_cast<const float2 *>(buf + i);
  else return __bfloat1622float2(reinterpret_cast<const __nv_bfloat162 *>(buf)[i >> 1]);
}
template <typename TS> HS_DEV void st2_cs(TS *p, float a, float b) {
  if constexpr (std::is_same<TS, float>::value) {
    __stcs(reinterpret_cast<float2 *>(p), make_float2(a, b));
  } else {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    __stcs(reinterpret_cast<unsigned *>(p), *reinterpret_cast<const unsigned *>(&v));
  }
}

template <typename TS>
__global__ void __launch_bounds__(kFNW * 32, kMinCtas2)
scan_fwd_col2_kernel(const TS *__restrict__ z, const float *__restrict__ c0, TS *__restrict__ out,
                     TS *__restrict__ cbuf, float *__restrict__ h_n, float *__restrict__ c_n, int64_t T, int64_t B,
                     int64_t H, float eps, unsigned *kf_max, int *status) {
  constexpr bool BF = !std::is_same<TS, float>::value;
  extern __shared__ float4 smem_f4[];
  float *sm = reinterpret_cast<float *>(smem_f4);
  unsigned long long *slots = reinterpret_cast<unsigned long long *>(sm + kFNW * 2 * kF2Buf);  // [NW][2][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t ncol = (H + 63) / 64;
  const int64_t b = blockIdx.x / ncol;
  const int64_t h0 = (blockIdx.x - b * ncol) * 64;
  const int64_t h = h0 + 2 * lane;
  const bool hv = h < H;
  const int64_t nchunk = (T + kFL - 1) / kFL;
  const int64_t zstep = B * 4 * H, ostep = B * H;
  const TS *zb = z + b * 4 * H;
  float *buf0 = sm + warp * 2 * kF2Buf;
  slots[warp * 64 + lane] = 0ull;
  slots[warp * 64 + 32 + lane] = 0ull;
  __syncthreads();

  // a step row: 4 gates x 64 units, in 16-byte copies of 4 floats (two per
  // lane) or 8 bf16 (one per lane)
  auto stage = [&](int64_t c, float *dst) {
    const int64_t t0 = c * kFL;
    const int n = (int)min((int64_t)kFL, T - t0);
    constexpr int EB = BF ? 2 : 4, PER = BF ? 8 : 4;
#pragma unroll
    for (int j0 = 0; j0 < 256 / PER; j0 += 32) {
      const int j = j0 + lane, g = j / (64 / PER), k = (j % (64 / PER)) * PER;
      if (h0 + k < H) {
        const TS *src = zb + t0 * zstep + g * H + h0 + k;
        unsigned d = sa(dst) + (unsigned)((g * 64 + k) * EB);
        for (int s = 0; s < n; ++s, src += zstep, d += kF2Row * EB) cp16(d, src);
      }
    }
  };

  float kmax = 0.f;
  int64_t c = warp;
  if (c < nchunk) stage(c, buf0);
  commit();
  if (c + kFNW < nchunk) stage(c + kFNW, buf0 + kF2Buf);
  commit();
  for (int i = 0; c < nchunk; c += kFNW, ++i) {
    float *buf = buf0 + (i & 1) * kF2Buf;
    wait_group<1>();
    __syncwarp();
    const int64_t t0 = c * kFL;
    const int n = (int)min((int64_t)kFL, T - t0);
    float fp[kFL][2], bp[kFL][2], eo[kFL][2];
    float A0 = 1.f, A1 = 1.f, C0 = 0.f, C1 = 0.f;
    const bool full = n == kFL && hv;
    auto coeffs = [&](auto full_tag) {
#pragma unroll
      for (int s = 0; s < kFL; ++s) {
        if (decltype(full_tag)::value || (s < n && hv)) {
          const int r = s * kF2Row + 2 * lane;
          const float2 zi = lds2<TS>(buf, r), zf = lds2<TS>(buf, r + 64), zg = lds2<TS>(buf, r + 128),
                       zo = lds2<TS>(buf, r + 192);
          fp[s][0] = fmaxf(sigf(zf.x), eps);
          fp[s][1] = fmaxf(sigf(zf.y), eps);
          bp[s][0] = fmaxf(sig2(zi.x, zg.x), eps);
          bp[s][1] = fmaxf(sig2(zi.y, zg.y), eps);
          eo[s][0] = __expf(-zo.x);
          eo[s][1] = __expf(-zo.y);
          C0 = fmaf(fp[s][0], C0, bp[s][0]);
          C1 = fmaf(fp[s][1], C1, bp[s][1]);
          A0 *= fp[s][0];
          A1 *= fp[s][1];
        } else {
          fp[s][0] = fp[s][1] = 1.f;
          bp[s][0] = bp[s][1] = 0.f;
          eo[s][0] = eo[s][1] = 0.f;
        }
      }
    };
    if (full) coeffs(std::true_type{});
    else coeffs(std::false_type{});
    __syncwarp();
    if (c + 2 * kFNW < nchunk) stage(c + 2 * kFNW, buf);
    commit();
    float cin0 = fmaxf((c == 0 && c0 && hv) ? c0[b * H + h] : 0.f, eps);
    float cin1 = fmaxf((c == 0 && c0 && hv) ? c0[b * H + h + 1] : 0.f, eps);
    const bool ok = c == 0 || (slot_wait(&slots[warp * 64 + lane], (unsigned)c, &cin0, status) &&
                               slot_wait(&slots[warp * 64 + 32 + lane], (unsigned)c, &cin1, status));
    if (!__all_sync(0xffffffffu, ok)) break;
    if (c + 1 < nchunk) {
      const int nw = ((warp + 1) % kFNW) * 64;
      slot_put(&slots[nw + lane], (unsigned)(c + 1), fmaf(A0, cin0, C0));
      slot_put(&slots[nw + 32 + lane], (unsigned)(c + 1), fmaf(A1, cin1, C1));
    }
    if (hv) {
      float cc0 = cin0, cc1 = cin1, o0 = 0.f, o1 = 0.f;
      TS *ob = out + (t0 * B + b) * H + h;
      TS *cb = cbuf + (t0 * B + b) * H + h;
      auto emit = [&](auto full_tag) {
#pragma unroll
        for (int s = 0; s < kFL; ++s) {
          if (decltype(full_tag)::value || s < n) {
            kmax = fmaxf(kmax, fmaxf(cc0 * fp[s][0] * (1.f - fp[s][0]), cc1 * fp[s][1] * (1.f - fp[s][1])));
            cc0 = fmaf(fp[s][0], cc0, bp[s][0]);
            cc1 = fmaf(fp[s][1], cc1, bp[s][1]);
            o0 = sig_tanh_pos(eo[s][0], cc0);
            o1 = sig_tanh_pos(eo[s][1], cc1);
            st2_cs(cb + s * ostep, cc0, cc1);
            st2_cs(ob + s * ostep, o0, o1);
          }
        }
      };
      if (full) emit(std::true_type{});
      else emit(std::false_type{});
      if (t0 + n == T) {
        if (c_n) {
          c_n[b * H + h] = cc0;
          c_n[b * H + h + 1] = cc1;
        }
        if (h_n) {
          h_n[b * H + h] = o0;
          h_n[b * H + h + 1] = o1;
        }
      }
    }
  }
  wait_group<0>();
  if (kf_max) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    if (lane == 0) atomicMax(kf_max, __float_as_uint(kmax));
  }
}

template <int OUT, typename TS>
__global__ void __launch_bounds__(kBNW * 32, kMinCtas2)
scan_bwd_col2_kernel(const TS *z, const TS *__restrict__ cbuf, const float *__restrict__ c0,
                     const TS *__restrict__ dout, const float *__restrict__ dh_n, const float *__restrict__ dc_n,
                     float *dz, float *__restrict__ dc0, float *__restrict__ db_part, int64_t T, int64_t B,
                     int64_t H, float eps, unsigned *dz_absmax, __half *__restrict__ dzh, __half *__restrict__ dzl,
                     const unsigned *__restrict__ dz_bound, __nv_bfloat16 *__restrict__ dzb, const int *gate,
                     int *status) {
  constexpr bool BF = !std::is_same<TS, float>::value;
  static_assert(!BF || OUT == kDzBf16, "bf16 storage writes bf16 dZ");
  if (gate && *gate == 0) return;
  extern __shared__ float4 smem_f4[];
  float *sm = reinterpret_cast<float *>(smem_f4);
  unsigned long long *slots = reinterpret_cast<unsigned long long *>(sm + kBNW * 2 * kB2Buf);  // [NW][2][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t ncol = (H + 63) / 64;
  const int64_t b = blockIdx.x / ncol;
  const int64_t h0 = (blockIdx.x - b * ncol) * 64;
  const int64_t h = h0 + 2 * lane;
  const bool hv = h < H;
  const int64_t nchunk = (T + kBL - 1) / kBL;
  const int64_t zstep = B * 4 * H, sstep = B * H;
  float *buf0 = sm + warp * 2 * kB2Buf;
  slots[warp * 64 + lane] = 0ull;
  slots[warp * 64 + 32 + lane] = 0ull;
  __syncthreads();
  const float c0p0 = fmaxf((c0 && hv) ? c0[b * H + h] : 0.f, eps);
  const float c0p1 = fmaxf((c0 && hv) ? c0[b * H + h + 1] : 0.f, eps);

  // a step row: z_i, z_f, z_g, z_o, c, dout x 64 units in 16-byte copies
  // (three per lane for float32, one or two for bf16), then the c_{t0-1} row
  auto stage = [&](int64_t q, float *dst) {
    const int64_t t0 = (nchunk - 1 - q) * kBL;
    const int n = (int)min((int64_t)kBL, T - t0);
    constexpr int EB = BF ? 2 : 4, PER = BF ? 8 : 4, RC = 64 / PER;  // copies per row
#pragma unroll
    for (int j0 = 0; j0 < 6 * RC; j0 += 32) {
      const int j = j0 + lane, rr = j / RC, k = (j % RC) * PER;
      if (j < 6 * RC && h0 + k < H) {
        const TS *src = rr < 4 ? z + (t0 * B + b) * 4 * H + rr * H + h0 + k
                               : (rr == 4 ? cbuf : dout) + (t0 * B + b) * H + h0 + k;
        const int64_t step = rr < 4 ? zstep : sstep;
        unsigned d = sa(dst) + (unsigned)((rr * 64 + k) * EB);
        for (int s = 0; s < n; ++s, src += step, d += kB2Row * EB) cp16(d, src);
      }
    }
    if (lane < RC && t0 > 0 && h0 + lane * PER < H)
      cp16(sa(dst) + (unsigned)((kBL * kB2Row + lane * PER) * EB), cbuf + ((t0 - 1) * B + b) * H + h0 + lane * PER);
  };

  float acc[4][2] = {};
  float amax = 0.f;
  const float sc = OUT == kDzSplit ? pow2_scale(*dz_bound) : 1.f;
  // the dZ pair at element offset i (even) of the [T*B][4H] layout
  auto put2 = [&](int64_t i, float v0, float v1) {
    if (OUT == kDzSplit) {
      const __half2 hi = __floats2half2_rn(v0 * sc, v1 * sc);
      const float2 hf = __half22float2(hi);
      const __half2 lo = __floats2half2_rn(v0 * sc - hf.x, v1 * sc - hf.y);
      __stcs(reinterpret_cast<unsigned *>(dzh + i), *reinterpret_cast<const unsigned *>(&hi));
      __stcs(reinterpret_cast<unsigned *>(dzl + i), *reinterpret_cast<const unsigned *>(&lo));
    } else if (OUT == kDzBf16) {
      const __nv_bfloat162 v = __floats2bfloat162_rn(v0, v1);
      __stcs(reinterpret_cast<unsigned *>(dzb + i), *reinterpret_cast<const unsigned *>(&v));
    } else {
      __stcs(reinterpret_cast<float2 *>(dz + i), make_float2(v0, v1));
    }
  };
  int64_t q = warp;
  if (q < nchunk) stage(q, buf0);
  commit();
  if (q + kBNW < nchunk) stage(q + kBNW, buf0 + kB2Buf);
  commit();
  for (int i = 0; q < nchunk; q += kBNW, ++i) {
    float *buf = buf0 + (i & 1) * kB2Buf;
    wait_group<1>();
    __syncwarp();
    const int64_t t0 = (nchunk - 1 - q) * kBL;
    const int n = (int)min((int64_t)kBL, T - t0);
    float dhn0 = 0.f, dhn1 = 0.f;
    if (q == 0 && dh_n && hv) {
      dhn0 = dh_n[b * H + h];
      dhn1 = dh_n[b * H + h + 1];
    }
    float FP[kBL][2], DCD[kBL][2], KI[kBL][2], KF[kBL][2], KG[kBL][2];
    float A[2] = {1.f, 1.f}, C[2] = {0.f, 0.f};
    const int64_t dzs = (t0 * B + b) * 4 * H + h;
#pragma unroll
    for (int s = kBL - 1; s >= 0; --s) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        FP[s][u] = 1.f;
        DCD[s][u] = KI[s][u] = KF[s][u] = KG[s][u] = 0.f;
      }
      if (s < n && hv) {
        const int r = s * kB2Row + 2 * lane;
        const float2 zi = lds2<TS>(buf, r), zf = lds2<TS>(buf, r + 64), zg = lds2<TS>(buf, r + 128),
                     zo = lds2<TS>(buf, r + 192), cs = lds2<TS>(buf, r + 256), dd = lds2<TS>(buf, r + 320);
        const float2 cpv = s > 0 ? lds2<TS>(buf, r + 256 - kB2Row)
                                 : (t0 > 0 ? lds2<TS>(buf, kBL * kB2Row + 2 * lane) : make_float2(c0p0, c0p1));
        const float dv[2] = {dd.x + (s == n - 1 ? dhn0 : 0.f), dd.y + (s == n - 1 ? dhn1 : 0.f)};
        const float zis[2] = {zi.x, zi.y}, zfs[2] = {zf.x, zf.y}, zgs[2] = {zg.x, zg.y}, zos[2] = {zo.x, zo.y};
        const float css[2] = {cs.x, cs.y}, cps[2] = {cpv.x, cpv.y};
        float dzo[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float ig = sig_fast(zis[u]), f = sigf(zfs[u]), g = sig_fast(zgs[u]), o = sig_fast(zos[u]);
          const float th = tanh_pos(css[u]);
          const float mb = (ig * g >= eps) ? 1.f : 0.f;
          const float mf = (f >= eps) ? 1.f : 0.f;
          const float d = dv[u];
          const float dcd = d * o * (1.f - th * th);
          dzo[u] = d * th * o * (1.f - o);
          acc[3][u] += dzo[u];
          amax = fmaxf(amax, fabsf(dzo[u]));
          FP[s][u] = fmaxf(f, eps);
          DCD[s][u] = dcd;
          KI[s][u] = g * ig * (1.f - ig) * mb;
          KF[s][u] = cps[u] * f * (1.f - f) * mf;
          KG[s][u] = ig * g * (1.f - g) * mb;
          C[u] = FP[s][u] * (C[u] + dcd);
          A[u] *= FP[s][u];
        }
        put2(dzs + s * zstep + 3 * H, dzo[0], dzo[1]);
      }
    }
    __syncwarp();
    if (q + 2 * kBNW < nchunk) stage(q + 2 * kBNW, buf);
    commit();
    float e0 = (q == 0 && dc_n && hv) ? dc_n[b * H + h] : 0.f;
    float e1 = (q == 0 && dc_n && hv) ? dc_n[b * H + h + 1] : 0.f;
    const bool ok = q == 0 || (slot_wait(&slots[warp * 64 + lane], (unsigned)q, &e0, status) &&
                               slot_wait(&slots[warp * 64 + 32 + lane], (unsigned)q, &e1, status));
    if (!__all_sync(0xffffffffu, ok)) break;
    if (q + 1 < nchunk) {
      const int nw = ((warp + 1) % kBNW) * 64;
      slot_put(&slots[nw + lane], (unsigned)(q + 1), fmaf(A[0], e0, C[0]));
      slot_put(&slots[nw + 32 + lane], (unsigned)(q + 1), fmaf(A[1], e1, C[1]));
    }
    if (hv) {
      float e[2] = {e0, e1};
#pragma unroll
      for (int s = kBL - 1; s >= 0; --s) {
        if (s < n) {
          float di[2], df[2], dg[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float dc = DCD[s][u] + e[u];
            e[u] = FP[s][u] * dc;
            di[u] = dc * KI[s][u];
            df[u] = dc * KF[s][u];
            dg[u] = dc * KG[s][u];
            acc[0][u] += di[u];
            acc[1][u] += df[u];
            acc[2][u] += dg[u];
            amax = fmaxf(amax, fmaxf(fabsf(di[u]), fmaxf(fabsf(df[u]), fabsf(dg[u]))));
          }
          const int64_t dzr = dzs + s * zstep;
          put2(dzr, di[0], di[1]);
          put2(dzr + H, df[0], df[1]);
          put2(dzr + 2 * H, dg[0], dg[1]);
        }
      }
      if (t0 == 0 && dc0) {
        dc0[b * H + h] = (c0 && c0[b * H + h] >= eps) ? e[0] : 0.f;
        dc0[b * H + h + 1] = (c0 && c0[b * H + h + 1] >= eps) ? e[1] : 0.f;
      }
    }
  }
  wait_group<0>();
  if (dz_absmax) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) atomicMax(dz_absmax, __float_as_uint(amax));
  }
  if (db_part) {
    __syncthreads();  // every warp is done with its buffers
    float *red = sm;  // [NW][4][64]
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      red[(warp * 4 + g) * 64 + 2 * lane] = acc[g][0];
      red[(warp * 4 + g) * 64 + 2 * lane + 1] = acc[g][1];
    }
    __syncthreads();
    if (hv) {
      for (int g = warp; g < 4; g += kBNW) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int w = 0; w < kBNW; ++w) {
          s0 += red[(w * 4 + g) * 64 + 2 * lane];
          s1 += red[(w * 4 + g) * 64 + 2 * lane + 1];
        }
        db_part[b * 4 * H + g * H + h] = s0;
        db_part[b * 4 * H + g * H + h + 1] = s1;
      }
    }
  }
}

// Units per lane of the per-column kernels: 2 where the 16-byte copies apply
// (HS_SCAN_UNITS=1 keeps one, for comparison).
bool two_units() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("HS_SCAN_UNITS");
    v = (e && e[0] == '1') ? 1 : 2;
  }
  return v == 2;
}

// Path choice: HS_SCAN_PATH=chain|lookback forces one (tests); otherwise the
// per-column kernels whenever the columns alone fill the GPU.
int path_override() {
  const char *e = getenv("HS_SCAN_PATH");
  if (!e) return 0;
  if (e[0] == 'c') return 1;
  if (e[0] == 'l') return 2;
  return 0;
}

int sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

std::atomic<unsigned long long> g_fwd_attr[3], g_bwd_attr[5], g_fwd2_attr[2], g_bwd2_attr[3];

}  // namespace

#ifndef HS_CHAIN_MIN_COLS_PER_SM
#define HS_CHAIN_MIN_COLS_PER_SM 4
#endif

bool scan_chain_wanted(int64_t T, int64_t B, int64_t H) {
  const int o = path_override();
  if (o) return o == 1;
  const int64_t ncol = B * ((H + 31) / 32);
  return T >= 64 && ncol >= (int64_t)HS_CHAIN_MIN_COLS_PER_SM * sm_count();
}

// Sequences whose per-column scan CTAs (two units per lane, 64-unit columns)
// are all resident at once on the current device, in both directions: the
// batch per call at which one wave of columns fills the SMs.  0 if the
// occupancy cannot be queried.
int64_t scan_wave_sequences(int64_t H) {
  if (H <= 0) return 0;
  const void *f = (const void *)scan_fwd_col2_kernel<float>;
  const void *b = (const void *)scan_bwd_col2_kernel<kDzSplit, float>;
  if (allow_dynamic_smem(f, kF2Smem, &g_fwd2_attr[0]) || allow_dynamic_smem(b, kB2Smem, &g_bwd2_attr[1])) {
    (void)cudaGetLastError();
    return 0;
  }
  int nf = 0, nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nf, f, kFNW * 32, kF2Smem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, b, kBNW * 32, kB2Smem) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return (int64_t)std::min(nf, nb) * sm_count() / ((H + 63) / 64);
}

int scan_fwd_chain_launch(const float *z, const float *c0, float *out, float *c, float *h_n, float *c_n,
                          int64_t T, int64_t B, int64_t H, float eps, unsigned *kf_max, int *status,
                          cudaStream_t st) {
  const int64_t grid = B * ((H + 31) / 32);
  if (grid >= (1ll << 31)) return fail(HS_ERR_UNSUPPORTED, "scan: too many columns");
  if ((T + kFL - 1) / kFL >= (1ll << 32)) return fail(HS_ERR_UNSUPPORTED, "scan: T too large");
  const bool v16 = H % 4 == 0 && aligned(z, 16);
  if (v16 && two_units() && aligned(out, 16) && aligned(c, 16)) {
    const void *fn2 = (const void *)scan_fwd_col2_kernel<float>;
    if (int e = allow_dynamic_smem(fn2, kF2Smem, &g_fwd2_attr[0])) return e;
    scan_fwd_col2_kernel<float><<<(unsigned)(B * ((H + 63) / 64)), kFNW * 32, kF2Smem, st>>>(
        z, c0, out, c, h_n, c_n, T, B, H, eps, kf_max, status);
    return check_launch("scan_fwd_col2_kernel");
  }
  const void *fn = v16 ? (const void *)scan_fwd_col_kernel<true> : (const void *)scan_fwd_col_kernel<false>;
  if (int e = allow_dynamic_smem(fn, kFSmem, &g_fwd_attr[v16])) return e;
  if (v16)
    scan_fwd_col_kernel<true><<<(unsigned)grid, kFNW * 32, kFSmem, st>>>(z, c0, out, c, h_n, c_n, T, B, H, eps,
                                                                       kf_max, status);
  else
    scan_fwd_col_kernel<false><<<(unsigned)grid, kFNW * 32, kFSmem, st>>>(z, c0, out, c, h_n, c_n, T, B, H, eps,
                                                                        kf_max, status);
  return check_launch("scan_fwd_col_kernel");
}

// dZ goes to dz (float32), or to its fp16 split (dzh, dzl, dz_bound).
int scan_bwd_chain_launch(const float *z, const float *c, const float *c0, const float *dout, const float *dh_n,
                          const float *dc_n, float *dz, float *dc0, float *db_part, int64_t T, int64_t B, int64_t H,
                          float eps, unsigned *dz_absmax, int *status, cudaStream_t st, __half *dzh, __half *dzl,
                          const unsigned *dz_bound, const int *gate) {
  const int64_t grid = B * ((H + 31) / 32);
  if (grid >= (1ll << 31)) return fail(HS_ERR_UNSUPPORTED, "scan: too many columns");
  if ((T + kBL - 1) / kBL >= (1ll << 32)) return fail(HS_ERR_UNSUPPORTED, "scan: T too large");
  const bool v16 = H % 4 == 0 && aligned(z, 16) && aligned(c, 16) && aligned(dout, 16);
  const bool split = dzh != nullptr;
  if (split && (!v16 || !dzl || !dz_bound)) return fail(HS_ERR_INVALID_ARG, "scan split: needs H % 4 == 0, aligned inputs");
  if (v16 && two_units() && (split ? (aligned(dzh, 4) && aligned(dzl, 4)) : aligned(dz, 8))) {
    const unsigned grid2 = (unsigned)(B * ((H + 63) / 64));
    const void *fn2 = split ? (const void *)scan_bwd_col2_kernel<kDzSplit, float>
                            : (const void *)scan_bwd_col2_kernel<kDzF32, float>;
    if (int e = allow_dynamic_smem(fn2, kB2Smem, &g_bwd2_attr[split ? 1 : 0])) return e;
    if (split)
      scan_bwd_col2_kernel<kDzSplit, float><<<grid2, kBNW * 32, kB2Smem, st>>>(
          z, c, c0, dout, dh_n, dc_n, dz, dc0, db_part, T, B, H, eps, dz_absmax, dzh, dzl, dz_bound, nullptr, gate,
          status);
    else
      scan_bwd_col2_kernel<kDzF32, float><<<grid2, kBNW * 32, kB2Smem, st>>>(
          z, c, c0, dout, dh_n, dc_n, dz, dc0, db_part, T, B, H, eps, dz_absmax, nullptr, nullptr, nullptr, nullptr,
          gate, status);
    return check_launch("scan_bwd_col2_kernel");
  }
  const void *fn = split ? (const void *)scan_bwd_col_kernel<true, kDzSplit>
                         : v16 ? (const void *)scan_bwd_col_kernel<true, kDzF32>
                               : (const void *)scan_bwd_col_kernel<false, kDzF32>;
  if (int e = allow_dynamic_smem(fn, kBSmem, &g_bwd_attr[split ? 2 : (int)v16])) return e;
  if (split)
    scan_bwd_col_kernel<true, kDzSplit><<<(unsigned)grid, kBNW * 32, kBSmem, st>>>(
        z, c, c0, dout, dh_n, dc_n, dz, dc0, db_part, T, B, H, eps, dz_absmax, dzh, dzl, dz_bound, nullptr, gate,
        status);
  else if (v16)
    scan_bwd_col_kernel<true, kDzF32><<<(unsigned)grid, kBNW * 32, kBSmem, st>>>(
        z, c, c0, dout, dh_n, dc_n, dz, dc0, db_part, T, B, H, eps, dz_absmax, nullptr, nullptr, nullptr, nullptr,
        gate, status);
  else
    scan_bwd_col_kernel<false, kDzF32><<<(unsigned)grid, kBNW * 32, kBSmem, st>>>(
        z, c, c0, dout, dh_n, dc_n, dz, dc0, db_part, T, B, H, eps, dz_absmax, nullptr, nullptr, nullptr, nullptr,
        gate, status);
  return check_launch("scan_bwd_col_kernel");
}

// bf16 storage (a bf16 module's path): z, out, c (forward) and z, c, dout
// (backward) in bf16, dZ written as bf16.  Needs H % 8 == 0 and 16-byte
// aligned tensors (every 8-unit copy then lies inside one column).
bool scan_chain_bf16_ok(int64_t H, std::initializer_list<const void *> ptrs) {
  if (H % 8) return false;
  for (const void *p : ptrs)
    if (!aligned(p, 16)) return false;
  return true;
}

int scan_fwd_chain_launch_bf16(const void *z, const float *c0, void *out, void *c, float *h_n, float *c_n, int64_t T,
                               int64_t B, int64_t H, float eps, int *status, cudaStream_t st) {
  const int64_t grid = B * ((H + 31) / 32);
  if (grid >= (1ll << 31)) return fail(HS_ERR_UNSUPPORTED, "scan: too many columns");
  if ((T + kFL - 1) / kFL >= (1ll << 32)) return fail(HS_ERR_UNSUPPORTED, "scan: T too large");
  if (!scan_chain_bf16_ok(H, {z, out, c})) return fail(HS_ERR_UNSUPPORTED, "bf16 scan: needs H % 8 == 0, 16-byte aligned z/out/c");
  using K = __nv_bfloat16;
  if (two_units()) {
    const void *fn2 = (const void *)scan_fwd_col2_kernel<K>;
    if (int e = allow_dynamic_smem(fn2, kF2Smem, &g_fwd2_attr[1])) return e;
    scan_fwd_col2_kernel<K><<<(unsigned)(B * ((H + 63) / 64)), kFNW * 32, kF2Smem, st>>>(
        static_cast<const K *>(z), c0, static_cast<K *>(out), static_cast<K *>(c), h_n, c_n, T, B, H, eps, nullptr,
        status);
    return check_launch("scan_fwd_col2_kernel<bf16>");
  }
  const void *fn = (const void *)scan_fwd_col_kernel<true, K>;
  if (int e = allow_dynamic_smem(fn, kFSmem, &g_fwd_attr[2])) return e;
  scan_fwd_col_kernel<true, K><<<(unsigned)grid, kFNW * 32, kFSmem, st>>>(
      static_cast<const K *>(z), c0, static_cast<K *>(out), static_cast<K *>(c), h_n, c_n, T, B, H, eps, nullptr,
      status);
  return check_launch("scan_fwd_col_kernel<bf16>");
}

int scan_bwd_chain_launch_bf16(const void *z, const void *c, const float *c0, const void *dout, const float *dh_n,
                               const float *dc_n, void *dz, float *dc0, float *db_part, int64_t T, int64_t B,
                               int64_t H, float eps, int *status, cudaStream_t st) {
  const int64_t grid = B * ((H + 31) / 32);
  if (grid >= (1ll << 31)) return fail(HS_ERR_UNSUPPORTED, "scan: too many columns");
  if ((T + kBL - 1) / kBL >= (1ll << 32)) return fail(HS_ERR_UNSUPPORTED, "scan: T too large");
  if (!scan_chain_bf16_ok(H, {z, c, dout, dz}))
    return fail(HS_ERR_UNSUPPORTED, "bf16 scan: needs H % 8 == 0, 16-byte aligned z/c/dout/dz");
  using K = __nv_bfloat16;
  if (two_units()) {
    const void *fn2 = (const void *)scan_bwd_col2_kernel<kDzBf16, K>;
    if (int e = allow_dynamic_smem(fn2, kB2Smem, &g_bwd2_attr[2])) return e;
    scan_bwd_col2_kernel<kDzBf16, K><<<(unsigned)(B * ((H + 63) / 64)), kBNW * 32, kB2Smem, st>>>(
        static_cast<const K *>(z), static_cast<const K *>(c), c0, static_cast<const K *>(dout), dh_n, dc_n, nullptr,
        dc0, db_part, T, B, H, eps, nullptr, nullptr, nullptr, nullptr, static_cast<K *>(dz), nullptr, status);
    return check_launch("scan_bwd_col2_kernel<bf16>");
  }
  const void *fn = (const void *)scan_bwd_col_kernel<true, kDzBf16, K>;
  if (int e = allow_dynamic_smem(fn, kBSmem, &g_bwd_attr[4])) return e;
  scan_bwd_col_kernel<true, kDzBf16, K><<<(unsigned)grid, kBNW * 32, kBSmem, st>>>(
      static_cast<const K *>(z), static_cast<const K *>(c), c0, static_cast<const K *>(dout), dh_n, dc_n, nullptr,
      dc0, db_part, T, B, H, eps, nullptr, nullptr, nullptr, nullptr, static_cast<K *>(dz), nullptr, status);
  return check_launch("scan_bwd_col_kernel<bf16>");
}

}  // namespace hs
