// Recurrent-mode HeadStartLSTM with the per-step product on the tensor cores.
//
// Reference: HeadStartLSTMTorchFn (src/headstartlstm/_torch.py:86-170) and
// HeadStartLSTMTritonFn (src/headstartlstm/_triton.py:331-465): per step the
// gates are Z[t] + h_{t-1} (a*W_hh)^T + a*b_hh (_torch.py:111-120), and the
// backward's dh = dgates (a*W_hh) (_torch.py:150).  Here each direction is
// one cooperative persistent launch of thread-block clusters; every step's
// product runs as tcgen05 MMAs with fp32 accumulators in tensor memory.
//
// Shape of the product.  A tcgen05.mma costs the issuing SM about the same
// time whatever its N (measured: ~150 cycles for M = 128, K = 16 and any N
// from 16 to 256), so the step is laid out to need as few instructions as
// possible: the batch state is the M = 128 operand (rows 0-31 its fp16 hi
// part, rows 32-63 its lo part, rows 64-127 unused) and the weights the N =
// 256 operand (128 weight rows as fp16 hi, the same 128 rows as lo).  One
// instruction then yields, for 128 weight rows x 32 sequences x 16 k, the
// three products Wh.hh + Wl.hh + Wh.hl (the lo.lo term, 2^-22 relative, is
// not used) of a float32-accurate split; the weights carry a power-of-two
// scale (from max |a W_hh|), h a fixed 2^14 (|h| < 1), dgates a power-of-two
// scale per producing CTA and step.
//
// Split over k.  The reduction axis (forward: H units; backward: 4H gate rows)
// is cut into KS slices, one per CTA of a cluster of KS CTAs that share the
// same 128 weight rows (forward: 32 units x 4 gates; backward: 128 units).
// Each CTA reduces its slice, then the clusters' partial sums meet in
// distributed shared memory: CTA j of the cluster receives, by bulk copies
// between the CTAs' shared memories, every CTA's partial for the units it owns
// (32/KS or 128/KS of them), adds them in a fixed order and runs the cell for
// those units: forward the a-scaled bias, sigmoids, c/h update and the stores
// of h, c and the activations; backward the cell's backward, the dgates store
// and the split of dgates for the next step.
//
// Exchange between clusters.  The state of the next step crosses clusters
// through a double-buffered exchange buffer in global memory (L2) in the
// operand layout, published with release/acquire on a step counter per batch
// group: one grid-wide barrier per step.  The loading warp fetches its k slice
// with bulk copies as soon as the counter is complete.
//
// Operands use the K-major layout without swizzle (8 x 16-byte core matrices;
// LBO = the distance between core matrices along k, SBO = 128 bytes between
// 8-row groups), so a CTA's k slice of the state is one contiguous block of
// the exchange buffer.  The weight slice stays in shared memory for the whole
// launch when it fits (H = 128 and 512, both directions), and is streamed
// from L2 through a ring of bulk copies otherwise (H = 2048: 512 KB per CTA
// per step), fetched before the step's state is ready.
//
// Warp roles: warp 0 loads, warp 1 issues the MMAs, warps 2-9 drain the
// accumulators (two per step slot, so the MMAs of one group overlap the drain
// of the previous), reduce across the cluster and run the cell.  Batch groups
// of 32 sequences run side by side on disjoint clusters.
// Every wait on another CTA is bounded (kWaitLimitNs); a CTA that gives up
// records HS_ERR_DEVICE_TIMEOUT in the caller's status word, waits (bounded)
// for its own copies and MMAs in flight, frees its tensor memory and returns.
// bf16 mode (a bfloat16 module): the weights a*W_hh rounded to bf16 and the
// state (h forward, dgates backward) rounded to bf16 each step, one product
// per instruction with bf16 operands and float32 accumulation: the weight
// operand is the N = UB rows themselves (half the bytes, no lo part), the
// state occupies rows 0-31 only (rows 32-63 of the exchange buffer stay zero),
// no operand scales.  Blocks, clusters, the exchange and the cell are the
// same as in the float32 mode.
// No cluster multicast.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "hs_common.cuh"

namespace hs {

namespace {

constexpr int kThreads = 320;    // warp 0 loads, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpi = 256;        // epilogue threads
constexpr int KCH = 64;          // k per chunk: 8 core-matrix columns
constexpr uint32_t kTmemCols = 512;
constexpr size_t kSmemMax = 227 * 1024;
constexpr int kMaxBar = 96;      // mbarriers in shared memory

HS_DEV uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

HS_DEV void mbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
// Raise the transaction count of the current phase without arriving.
HS_DEV void mbar_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
HS_DEV void mbar_arrive_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
HS_DEV void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
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
// Bounded wait on a phase: false (status set) after kWaitLimitNs, or as soon
// as the status word shows another CTA gave up.
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
// Bounded wait that records nothing (draining on the way out).
HS_DEV void mbar_drain(uint64_t *b, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try(b, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) return;
  }
}
// Contiguous global -> shared copy by the bulk-copy engine.
HS_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
      "l"(src), "r"(bytes), "r"(su32(bar))
      : "memory");
}
// Shared-memory operand descriptor: K-major, no swizzle (layout type 0).
HS_DEV uint64_t kdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}
// Instruction descriptor: D f32, A and B f16, both K-major, N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
HS_DEV void mma_f16(uint32_t dt, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dt),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
HS_DEV void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}
HS_DEV void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
HS_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
HS_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
HS_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Named barrier of the 256 epilogue threads, returning whether any of them
// passed `fail` (so that all of them leave their loop at the same point).
HS_DEV bool epi_sync_any(bool fail) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)fail)
      : "memory");
  return r != 0;
}
HS_DEV void epi_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Wait until the batch group's step counter reaches `target` (every CTA of
// the group has published its slice of the state).  Bounded.
HS_DEV bool wait_counter(const unsigned *bar, unsigned target, int *status) {
  if (ld_acquire(bar) >= target) return true;
  const uint64_t t0 = globaltimer();
  unsigned n = 0;
  while (ld_acquire(bar) < target) {
    if ((++n & 31u) == 0) {
      if (ld_status(status) != 0) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        set_status(status, HS_ERR_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}
// Publish this CTA's part of a step: a release at GPU scope (cumulative:
// it covers the writes of the CTA's other threads, ordered before it by the
// barrier that precedes the call).
HS_DEV void arrive_counter(unsigned *bar) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

// A load that stays where it is written: issued before the waits that
// follow it (volatile asm is not reordered across the barrier waits), read
// through L2 only.
HS_DEV float ld_early(const float *p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// fp16 split of x*s into hi + lo; returns hi's bits in the low half of .x
// and lo's in .y.
HS_DEV void split_h2(float y, __half &hi, __half &lo) {
  hi = __float2half_rn(y);
  lo = __float2half_rn(y - __half2float(hi));
}

// Byte offset of element (row, k) in a K-major no-swizzle operand tile whose
// core-matrix columns (8 k) are kstr bytes apart.
HS_DEV uint32_t koff(int row, int64_t k, uint32_t kstr) {
  return (uint32_t)((k >> 3) * kstr) + (uint32_t)((row >> 3) << 7) + (uint32_t)((row & 7) << 4) +
         (uint32_t)((k & 7) << 1);
}

// Cluster helpers: rank of this CTA, address of a peer's shared variable,
// and the cluster-wide barrier (start and end of the launch only).
HS_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HS_DEV uint32_t peer_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(su32(p)), "r"(rank));
  return r;
}
HS_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared -> shared copy into a CTA of the cluster (possibly this one); the
// bytes complete on that CTA's barrier at cluster address bar.
HS_DEV void bulk_s2c(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "r"(su32(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// ------------------------------------------------------------------ staging
// max |a[g] W_hh[r][k]| as float bits into *out (zeroed by the caller): the
// max |W_hh| of gate block blockIdx.y (float4 loads, H % 4 == 0) times
// |a[g]|; rounding is monotone, so this is the max of the rounded products.
// vec: w_hh is 16-byte aligned (else scalar loads).
__global__ void rtc_absmax_kernel(const float *__restrict__ w_hh, const float *__restrict__ a, int64_t H,
                                  unsigned *out, int vec) {
  const int g = blockIdx.y;
  const float *blk = w_hh + (int64_t)g * H * H;
  float m = 0.f;
  if (vec) {
    const int64_t n4 = H * H / 4;
    const float4 *src = reinterpret_cast<const float4 *>(blk);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
      const float4 v = __ldg(src + i);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < H * H; i += (int64_t)gridDim.x * blockDim.x)
      m = fmaxf(m, fabsf(blk[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(fabsf(a[g]) * m));
}

// Weight tiles, one per CTA: the N = 2 UB operand [UB rows hi | the same UB
// rows lo] over the CTA's k slice, K-major without swizzle (core-matrix
// columns of 8 k are 2 UB x 16 bytes apart), scaled by the power of two of
// max |a W_hh|.  One thread writes 8 consecutive k of one row (16 bytes).
//   forward  (UB = 128) CTA (rb, s): row n % 128 = g * 32 + ul is
//            a[g] W_hh[g H + 32 rb + ul][k], k in [s Ks, (s + 1) Ks) (a unit index);
//   backward (UB = 128 or 64 units) CTA (ub, s): row n % UB = ul is
//            a[g] W_hh[g H + u'][UB ub + ul] for the gate row (g, u') at position
//            k of the permuted order in which each producing CTA's 4 x UCP rows
//            are contiguous: k = (P 4 + g) UCP + l, u' = (P / KS) UB + (P % KS) UCP + l.
// bf != 0: the N = UB operand of the rows themselves in bf16, unscaled.
__global__ void rtc_prep_kernel(const float *__restrict__ w_hh, const float *__restrict__ a,
                                const unsigned *__restrict__ absmax, unsigned char *__restrict__ wg, int dir,
                                int64_t H, int KS, int UCP, int UB, int64_t Ks, int NC, int bf, int vec) {
  const float s = bf ? 1.0f : pow2_scale(*absmax);
  const int NW = bf ? UB : 2 * UB;
  // 32-bit index arithmetic: NC * Ks/8 * NW < 2^31 for every plan (H <= 2^14)
  const int nkc = (int)(Ks / 8);
  const int total = NC * nkc * NW;
  const size_t tile = (size_t)Ks * NW * 2;
  const int Hi = (int)H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int n = i % NW;
    const int kc = (i / NW) % nkc;
    const int cta = i / (NW * nkc);
    const int blk = cta / KS, sp = cta % KS;
    const int r = n % UB;
    const bool lo = n >= UB;
    float wv[8];
    const int k0 = sp * (int)Ks + kc * 8;
    if (dir == 0) {
      // 8 consecutive k of one row: two 16-byte loads (k0 is a multiple of 8)
      const int g = r / 32, ul = r % 32;
      const float ag = a[g];
      const float *row = w_hh + ((int64_t)g * Hi + blk * 32 + ul) * Hi + k0;
      if (vec) {
        const float4 v0 = __ldg(reinterpret_cast<const float4 *>(row)), v1 = __ldg(reinterpret_cast<const float4 *>(row) + 1);
        wv[0] = ag * v0.x; wv[1] = ag * v0.y; wv[2] = ag * v0.z; wv[3] = ag * v0.w;
        wv[4] = ag * v1.x; wv[5] = ag * v1.y; wv[6] = ag * v1.z; wv[7] = ag * v1.w;
      } else {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) wv[kk] = ag * row[kk];
      }
    } else {
      // UCP is a multiple of 8 (UB / KS with UB in {64, 128}, KS <= 8), so
      // the 8 consecutive k share one producer block P and gate g
      const int P = k0 / (4 * UCP);
      const int g = (k0 / UCP) % 4, l0 = k0 % UCP;
      const int up0 = (P / KS) * UB + (P % KS) * UCP + l0;
      const float ag = a[g];
      const float *col = w_hh + ((int64_t)g * Hi + up0) * Hi + blk * UB + r;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) wv[kk] = ag * col[(int64_t)kk * Hi];
    }
    __align__(16) __half v[8];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const float w = wv[kk];
      if (bf) {
        v[kk] = __ushort_as_half(__bfloat16_as_ushort(__float2bfloat16_rn(w)));
      } else {
        __half hi, lh;
        split_h2(w * s, hi, lh);
        v[kk] = lo ? lh : hi;
      }
    }
    *reinterpret_cast<uint4 *>(wg + (size_t)cta * tile + koff(n, kc * 8, (uint32_t)NW * 16)) =
        *reinterpret_cast<const uint4 *>(v);
  }
}

// ------------------------------------------------------------------ kernel
struct RtcArgs {
  const unsigned char *wg;  // weight tiles, Ks * 512 bytes per CTA
  unsigned char *xg;        // exchange buffers [ngrp][2 parities][xbytes]
  float *xscale;            // backward: inverse scales of the producers' dgates blocks [ngrp][2][NC]
  const unsigned *w_absmax; // max |a W_hh| (float bits)
  unsigned *bar;            // step counters, one per batch group, 32 words apart
  int *status;
  float *zacts;             // forward: Z in, activations out; backward: activations in, dgates out
  const float *h0, *c0;     // forward initial state [Bt,H] or null
  float *h_save, *c_save;   // [T+1,Bt,H]
  const float *dout, *dh_n, *dc_n;
  const float *b_hh, *a;
  int64_t T, Bt, H;
  int bf;                   // bf16 mode (see the top of the file)
  int64_t Ks;               // k per CTA (slice of the reduction axis)
  size_t xbytes;            // one exchange buffer: K / 8 core columns x 1 KB
  int b0;                   // first sequence of batch group 0 of this launch
  int NC, KS, UCP, UB, nchunk, gch, stages, resident;
};

// Shared-memory carve-up (1024-aligned base):
//   resident: [W (Ks/8 x NW x 16 B) | state (Ks/8 x 1 KB) | 1 KB]
//   streaming: stages of [W chunk (8 x NW x 16 B) | state chunk 8 KB], then 1 KB
//   (NW = 2 UB weight rows: 256, or 128 for 64-unit backward blocks)
//   then the outgoing partials pout [128][32] f32, the incoming [4096]
//   f32, 8 floats, the mbarriers and the TMEM address.
// The 1 KB after the state keeps in bounds the reads of the unused rows
// 64-127 of the M = 128 operand.
struct Layout {
  size_t w, h, ring, stage, pout, pin, red, bars, holder, total;
};
__host__ __device__ inline Layout make_layout(int64_t Ks, int stages, bool resident, int NW) {
  Layout L{};
  size_t off = 0;
  const size_t kstr = (size_t)NW * 16;
  if (resident) {
    L.w = 0;
    off = (size_t)Ks / 8 * kstr;
    L.h = off;
    off += (size_t)Ks / 8 * 1024 + 1024;
  } else {
    L.ring = 0;
    L.stage = 8 * kstr + 8192;
    off = (size_t)stages * L.stage + 1024;
  }
  L.pout = off;
  off += 4096 * 4;
  L.pin = off;
  off += 4096 * 4;
  L.red = off;
  off += 64;
  L.bars = off;
  off += (size_t)kMaxBar * 8;
  L.holder = off;
  off += 16;
  L.total = off + 1024;  // alignment slack of the dynamic base
  return L;
}

// Barrier slots: [0, 32) full (ring stages, or the resident state chunks),
// [32, 40) empty, [40, 44) slot_full, [44, 48) slot_free, 48 weights loaded,
// 49 MMA drain, 50 partial sums in.
constexpr int B_FULL = 0, B_EMPTY = 32, B_SFULL = 40, B_SFREE = 44, B_W = 48, B_DONE = 49, B_PIN = 50;

// NCELL: cells (unit x sequence) per epilogue thread, UCP * 32 / 256 (1, 2
// or 4), a compile-time constant so that the per-cell state stays in
// registers.
template <int DIR, int NCELL>
__global__ void __launch_bounds__(kThreads, 1) rtc_kernel(RtcArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool bf = p.bf != 0;
  const int NC = p.NC, KS = p.KS, UCP = p.UCP, UB = p.UB, NW = bf ? p.UB : 2 * p.UB;
  const bool resident = p.resident != 0;
  const Layout L = make_layout(p.Ks, p.stages, resident, NW);
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L.bars);
  uint32_t *holder = reinterpret_cast<uint32_t *>(sm + L.holder);
  float *pout = reinterpret_cast<float *>(sm + L.pout);
  float *pin = reinterpret_cast<float *>(sm + L.pin);
  float *red = reinterpret_cast<float *>(sm + L.red);
  const int grp = blockIdx.x / NC, cta = blockIdx.x % NC;
  const int blk = cta / KS;                 // weight-row block
  const int sp = (int)cluster_rank();        // k slice = rank in the cluster (== cta % KS)
  const int64_t H = p.H, Bt = p.Bt, T = p.T;
  const int bg0 = p.b0 + grp * 32;           // first sequence of this group
  const int Bc = (int)min((int64_t)32, Bt - bg0);
  unsigned *bar = p.bar + grp * 32;
  unsigned char *xg = p.xg + (size_t)grp * 2 * p.xbytes;
  float *xscale = p.xscale ? p.xscale + (size_t)grp * 2 * NC : nullptr;
  const int S = p.stages, nchunk = p.nchunk, gch = p.gch;
  // two accumulator slots of NW columns: the MMAs of one group overlap the
  // drain of the previous one (four slots for 128-row blocks measured slower)
  const int NS = 2;
  const int ngroups = (nchunk + gch - 1) / gch;
  const int slot_f = DIR == 0 ? 4 * UCP * 32 : UCP * 32;  // floats of one CTA's partial for one owner
  const uint32_t kstrW = (uint32_t)NW * 16;
  const uint32_t wchunk = 8 * kstrW, hchunk = 8192;
  const size_t xoff = (size_t)sp * p.Ks / 8 * 1024;       // this CTA's k slice in the exchange buffer
  const int64_t nsteps = DIR == 0 ? T : T - 1;            // steps that run a product

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < 32; ++i) mbar_init(&bars[B_FULL + i], 1);
    for (int i = 0; i < 8; ++i) mbar_init(&bars[B_EMPTY + i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&bars[B_SFULL + i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&bars[B_SFREE + i], bf ? 2 : 4);  // the draining warps
    mbar_init(&bars[B_W], 1);
    mbar_init(&bars[B_DONE], 1);
    mbar_init(&bars[B_PIN], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every CTA's barriers exist before a peer copies into it
  tc_fence_after();
  const uint32_t tmem = *holder;

  if (warp == 0) {
    // ------------------------------------------------------------ loads
    if (lane == 0) {
      const unsigned char *wsrc = p.wg + (size_t)cta * p.Ks * NW * 2;
      bool ok = true;
      int64_t fills = 0;
      if (resident && nsteps > 0) {
        const size_t wb = (size_t)p.Ks * NW * 2;
        mbar_arrive_expect(&bars[B_W], (uint32_t)wb);
        for (size_t off = 0; off < wb; off += 32768)
          bulk_g2s(sm + L.w + off, wsrc + off, (uint32_t)min((size_t)32768, wb - off), &bars[B_W]);
      }
      for (int64_t s = 0; s < nsteps && ok; ++s) {
        const int64_t t = DIR == 0 ? s : T - 2 - s;
        const unsigned target = (unsigned)((s + 1) * NC);
        const int par = (int)((DIR == 0 ? t : t + 1) & 1);
        const unsigned char *xsrc = xg + (size_t)par * p.xbytes + xoff;
        if (resident) {
          if (!wait_counter(bar, target, p.status)) { ok = false; break; }
          asm volatile("fence.proxy.async.global;" ::: "memory");
          for (int j = 0; j < nchunk; ++j) {
            mbar_arrive_expect(&bars[B_FULL + j], hchunk);
            bulk_g2s(sm + L.h + (size_t)j * hchunk, xsrc + (size_t)j * hchunk, hchunk, &bars[B_FULL + j]);
          }
        } else {
          const int pre = min(S, nchunk);
          int armed = 0;
          for (int j = 0; j < pre; ++j) {
            const int64_t f = fills + j;
            const int st = (int)(f % S);
            if (f >= S && !mbar_wait(&bars[B_EMPTY + st], (uint32_t)((f / S - 1) & 1), p.status)) { ok = false; break; }
            mbar_expect(&bars[B_FULL + st], wchunk);
            bulk_g2s(sm + L.ring + (size_t)st * L.stage, wsrc + (size_t)j * wchunk, wchunk, &bars[B_FULL + st]);
            ++armed;
          }
          if (ok && !wait_counter(bar, target, p.status)) ok = false;
          if (!ok) {
            for (int j = 0; j < armed; ++j) mbar_arrive(&bars[B_FULL + (int)((fills + j) % S)]);
            fills += armed;
            break;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");
          for (int j = 0; j < pre; ++j) {
            const int st = (int)((fills + j) % S);
            mbar_arrive_expect(&bars[B_FULL + st], hchunk);
            bulk_g2s(sm + L.ring + (size_t)st * L.stage + wchunk, xsrc + (size_t)j * hchunk, hchunk,
                     &bars[B_FULL + st]);
          }
          for (int j = pre; j < nchunk; ++j) {
            const int64_t f = fills + j;
            const int st = (int)(f % S);
            if (!mbar_wait(&bars[B_EMPTY + st], (uint32_t)((f / S - 1) & 1), p.status)) {
              ok = false;
              fills = f;
              break;
            }
            unsigned char *dst = sm + L.ring + (size_t)st * L.stage;
            mbar_arrive_expect(&bars[B_FULL + st], wchunk + hchunk);
            bulk_g2s(dst, wsrc + (size_t)j * wchunk, wchunk, &bars[B_FULL + st]);
            bulk_g2s(dst + wchunk, xsrc + (size_t)j * hchunk, hchunk, &bars[B_FULL + st]);
          }
          if (ok) fills += nchunk;
        }
      }
      if (resident) {
        if (nsteps > 0) mbar_drain(&bars[B_W], 0);
      } else {
        for (int64_t f = max((int64_t)0, fills - S); f < fills; ++f)
          mbar_drain(&bars[B_FULL + (int)(f % S)], (uint32_t)((f / S) & 1));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, NW) | (bf ? ((1u << 7) | (1u << 10)) : 0u);  // bf16 A and B
      bool ok = true;
      if (resident && nsteps > 0) ok = mbar_wait(&bars[B_W], 0, p.status);
      int64_t chunks = 0, groups = 0;
      for (int64_t s = 0; s < nsteps && ok; ++s) {
        int slot = 0;
        for (int j = 0; j < nchunk && ok; ++j) {
          if (j % gch == 0) {
            slot = (int)(groups % NS);
            if (groups >= NS && !mbar_wait(&bars[B_SFREE + slot], (uint32_t)((groups / NS - 1) & 1), p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const unsigned char *wa, *hb;
          if (resident) {
            if (!mbar_wait(&bars[B_FULL + j], (uint32_t)(s & 1), p.status)) { ok = false; break; }
            wa = sm + L.w + (size_t)j * wchunk;
            hb = sm + L.h + (size_t)j * hchunk;
          } else {
            const int st = (int)(chunks % S);
            if (!mbar_wait(&bars[B_FULL + st], (uint32_t)((chunks / S) & 1), p.status)) { ok = false; break; }
            wa = sm + L.ring + (size_t)st * L.stage;
            hb = wa + wchunk;
          }
          tc_fence_after();
          const uint32_t dt = tmem + (uint32_t)(slot * NW);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t ad = kdesc(su32(hb + 2 * ks * 1024), 1024, 128);  // state rows (M)
            const uint64_t bd = kdesc(su32(wa + 2 * ks * kstrW), kstrW, 128);  // weight rows (N)
            mma_f16(dt, ad, bd, idesc, (j % gch != 0 || ks > 0) ? 1u : 0u);
          }
          if (!resident) mma_commit(&bars[B_EMPTY + (int)(chunks % S)]);
          ++chunks;
          if (j % gch == gch - 1 || j == nchunk - 1) {
            mma_commit(&bars[B_SFULL + slot]);
            ++groups;
          }
        }
      }
      mma_commit(&bars[B_DONE]);
      mbar_drain(&bars[B_DONE], 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2, q = warp & 3, half = ew >> 2;
    const int e = ew * 32 + lane;  // 0..255
    // TMEM lanes 0-31 (hi state rows) and 32-63 (lo state rows; none in bf16 mode)
    const bool drains = bf ? q == 0 : q < 2;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
    const float inv_w = bf ? 1.0f : 1.0f / pow2_scale(*p.w_absmax);
    int64_t groups = 0;
    bool fail = false;
    int64_t pin_armed = 0, pin_seen = 0;  // phases of the partial-sums barrier

    // One step's drain of the accumulator groups into acc[64] (weight rows
    // 64 half + i), the cluster exchange of the partial sums, and the wait
    // for every CTA's partials of this CTA's units.
    auto reduce_step = [&](int64_t s_idx, int par) -> bool {
      float acc[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0.f;
      if (e == 0) mbar_arrive_expect(&bars[B_PIN], (uint32_t)(KS * slot_f * 4));
      ++pin_armed;
      // Only the draining warps wait on a slot: their release of it gates the
      // MMA's next use, so they never fall two phases behind (a warp that
      // waited without gating could miss a phase and wait on the next one).
      for (int gi = 0; gi < ngroups; ++gi) {
        const int slot = (int)(groups % NS);
        if (drains && !fail && !mbar_wait(&bars[B_SFULL + slot], (uint32_t)((groups / NS) & 1), p.status)) fail = true;
        if (!fail) {
          tc_fence_after();
          if (drains && 64 * half < UB) {
            float sc = 1.0f;
            if (DIR == 1 && !bf) sc = __ldcg(&xscale[par * NC + (int)(sp * ngroups + gi)]) * inv_w;
            const uint32_t base = tl + (uint32_t)(slot * NW) + (uint32_t)(64 * half);
            // four quarters of 16 weight rows, the loads of a quarter in
            // flight together (registers: the 64 sums + 32 loaded values)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t v[16], w[16];
              tmem_ld16_nowait(base + 16 * c, v);
              if (q == 0 && !bf) tmem_ld16_nowait(base + UB + 16 * c, w);
              tmem_wait_ld();
              if (q == 0 && !bf) {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                  acc[16 * c + i] = fmaf(__uint_as_float(v[i]) + __uint_as_float(w[i]), sc, acc[16 * c + i]);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[16 * c + i] = fmaf(__uint_as_float(v[i]), sc, acc[16 * c + i]);
              }
            }
          }
          if (drains) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_SFREE + slot]);
          }
        }
        ++groups;
      }
      // The partial sums of the weight rows r (forward: r = gate x 32 + unit;
      // backward: r = unit) for sequence b, pout[r][b]: the lo-state rows'
      // sums first, then the hi-state rows add theirs.
      if (q == (bf ? 0 : 1) && !fail && 64 * half < UB) {
#pragma unroll
        for (int i = 0; i < 64; ++i) pout[(64 * half + i) * 32 + lane] = acc[i];
      }
      // pout is free again: the previous step's copies out of it landed in
      // every CTA of the cluster before those CTAs published the state this
      // step's MMAs consumed
      if (epi_sync_any(fail)) return false;
      if (q == 0 && !bf && 64 * half < UB) {
#pragma unroll
        for (int i = 0; i < 64; ++i) pout[(64 * half + i) * 32 + lane] += acc[i];
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      epi_sync();
      // CTA j of the cluster owns units [j UCP, (j+1) UCP) of the block: it
      // receives their rows (forward: of each gate) into its slot for this
      // CTA's k slice, pin[sp][g][ul][b] (backward pin[sp][ul][b]).
      if (e == 0) {
        const uint32_t part = (uint32_t)UCP * 32 * 4;  // bytes of one gate's rows of one owner
        for (int j = 0; j < KS; ++j) {
          const uint32_t bar_j = peer_addr(&bars[B_PIN], (uint32_t)j);
          if (DIR == 0) {
            for (int g = 0; g < 4; ++g)
              bulk_s2c(peer_addr(pin + ((sp * 4 + g) * UCP) * 32, (uint32_t)j), pout + (g * 32 + j * UCP) * 32, part,
                       bar_j);
          } else {
            bulk_s2c(peer_addr(pin + sp * UCP * 32, (uint32_t)j), pout + j * UCP * 32, part, bar_j);
          }
        }
      }
      const bool ok = mbar_wait(&bars[B_PIN], (uint32_t)(s_idx & 1), p.status);
      if (ok) ++pin_seen;
      return !epi_sync_any(!ok);
    };

    if (DIR == 0) {
      // ---------------- forward: this CTA's units u = 32 blk + UCP sp + ul
      float cst[NCELL] = {};
      // prologue: h0 into exchange parity 0, h_save[0], c_save[0]
      _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
        const int ci = e + kEpi * m;
        const int b = ci % 32, ul = ci / 32;
        if (ul >= UCP || b >= Bc) continue;
        const int64_t u = (int64_t)blk * 32 + sp * UCP + ul, bb = bg0 + b;
        const float h = p.h0 ? p.h0[bb * H + u] : 0.f;
        const float c = p.c0 ? p.c0[bb * H + u] : 0.f;
        cst[m] = c;
        p.h_save[bb * H + u] = h;
        p.c_save[bb * H + u] = c;
        if (bf) {
          *reinterpret_cast<__nv_bfloat16 *>(xg + koff(b, u, 1024)) = __float2bfloat16_rn(h);
        } else {
          __half hi, lo;
          split_h2(h * 16384.0f, hi, lo);
          *reinterpret_cast<__half *>(xg + koff(b, u, 1024)) = hi;
          *reinterpret_cast<__half *>(xg + koff(32 + b, u, 1024)) = lo;
        }
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
      epi_sync();
      if (e == 0) arrive_counter(bar);
      const float inv = bf ? 1.0f : inv_w * (1.0f / 16384.0f);
      float bias[NCELL][4];  // a-scaled b_hh of the thread's cells (_torch.py:93)
      _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
        const int ul = (e + kEpi * m) >> 5;
        const int64_t u = (int64_t)blk * 32 + sp * UCP + min(ul, UCP - 1);
#pragma unroll
        for (int g = 0; g < 4; ++g) bias[m][g] = p.a[g] * p.b_hh[g * H + u];
      }
      for (int64_t t = 0; t < T; ++t) {
        // this step's input projection and bias for the thread's cells
        float zb[NCELL][4];
        _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
          const int ci = e + kEpi * m;
          const int b = ci & 31, ul = ci >> 5;
          const int64_t u = (int64_t)blk * 32 + sp * UCP + ul;
#pragma unroll
          for (int g = 0; g < 4; ++g)
            zb[m][g] = (ul < UCP && b < Bc) ? ld_early(&p.zacts[(t * Bt + bg0 + b) * 4 * H + g * H + u]) : 0.f;
        }
        if (!reduce_step(t, 0)) { fail = true; break; }
        unsigned char *xdst = xg + (size_t)((t + 1) & 1) * p.xbytes;
        float act[NCELL][4], hv[NCELL];
        _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
          const int ci = e + kEpi * m;
          const int b = ci & 31, ul = ci >> 5;
          if (ul >= UCP || b >= Bc) continue;
          const int64_t u = (int64_t)blk * 32 + sp * UCP + ul;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            float sum = 0.f;
            for (int s2 = 0; s2 < KS; ++s2) sum += pin[s2 * slot_f + (g * UCP + ul) * 32 + b];
            act[m][g] = sigf(fmaf(sum, inv, zb[m][g] + bias[m][g]));
          }
          const float c = fmaf(act[m][1], cst[m], act[m][0] * act[m][2]);
          hv[m] = act[m][3] * tanh_any(c);
          cst[m] = c;
          if (t + 1 < T) {
            if (bf) {
              *reinterpret_cast<__nv_bfloat16 *>(xdst + koff(b, u, 1024)) = __float2bfloat16_rn(hv[m]);
            } else {
              __half hi, lo;
              split_h2(hv[m] * 16384.0f, hi, lo);
              *reinterpret_cast<__half *>(xdst + koff(b, u, 1024)) = hi;
              *reinterpret_cast<__half *>(xdst + koff(32 + b, u, 1024)) = lo;
            }
          }
        }
        // publish the exchange slice first; the step's outputs, which no
        // other CTA reads, are stored after the release
        asm volatile("fence.proxy.async.global;" ::: "memory");
        if (epi_sync_any(fail)) { fail = true; break; }
        if (e == 0 && t + 1 < T) arrive_counter(bar);
        _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
          const int ci = e + kEpi * m;
          const int b = ci & 31, ul = ci >> 5;
          if (ul >= UCP || b >= Bc) continue;
          const int64_t u = (int64_t)blk * 32 + sp * UCP + ul, bb = bg0 + b;
#pragma unroll
          for (int g = 0; g < 4; ++g) p.zacts[(t * Bt + bb) * 4 * H + g * H + u] = act[m][g];
          p.h_save[((t + 1) * Bt + bb) * H + u] = hv[m];
          p.c_save[((t + 1) * Bt + bb) * H + u] = cst[m];
        }
      }
    } else {
      // ---------------- backward: this CTA's units u = 128 blk + UCP sp + ul
      float dc[NCELL] = {};
      _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
        const int ci = e + kEpi * m;
        const int b = ci & 31, ul = ci >> 5;
        if (ul < UCP && b < Bc && p.dc_n) dc[m] = p.dc_n[(int64_t)(bg0 + b) * H + (int64_t)blk * UB + sp * UCP + ul];
      }
      for (int64_t t = T - 1; t >= 0; --t) {
        float ld[NCELL][7];  // i, f, g, o, c_t, c_{t-1}, dh
        _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
          const int ci = e + kEpi * m;
          const int b = ci % 32, ul = ci / 32;
          const bool v = ul < UCP && b < Bc;
          const int64_t u = (int64_t)blk * UB + sp * UCP + ul, bb = bg0 + b;
          const float *ar = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
          for (int g = 0; g < 4; ++g) ld[m][g] = v ? ld_early(ar + g * H) : 0.f;
          ld[m][4] = v ? ld_early(p.c_save + ((t + 1) * Bt + bb) * H + u) : 0.f;
          ld[m][5] = v ? ld_early(p.c_save + (t * Bt + bb) * H + u) : 0.f;
          ld[m][6] = v ? ld_early(p.dout + (t * Bt + bb) * H + u) + ((t == T - 1 && p.dh_n) ? p.dh_n[bb * H + u] : 0.f)
                       : 0.f;
        }
        if (t < T - 1) {
          if (!reduce_step(T - 2 - t, (int)((t + 1) & 1))) { fail = true; break; }
        }
        float mx = 0.f;
        float dg[NCELL][4];
        _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
          const int ci = e + kEpi * m;
          const int b = ci % 32, ul = ci / 32;
          dg[m][0] = dg[m][1] = dg[m][2] = dg[m][3] = 0.f;
          if (ul >= UCP || b >= Bc) continue;
          float dh = ld[m][6];
          if (t < T - 1)
            for (int s2 = 0; s2 < KS; ++s2) dh += pin[s2 * slot_f + ul * 32 + b];
          const float i = ld[m][0], f = ld[m][1], g = ld[m][2], o = ld[m][3];
          const float th = tanh_any(ld[m][4]);
          const float dct = fmaf(dh * o, 1.f - th * th, dc[m]);
          dg[m][0] = dct * g * i * (1.f - i);
          dg[m][1] = dct * ld[m][5] * f * (1.f - f);
          dg[m][2] = dct * i * g * (1.f - g);
          dg[m][3] = dh * th * o * (1.f - o);
          dc[m] = dct * f;
#pragma unroll
          for (int q2 = 0; q2 < 4; ++q2) mx = fmaxf(mx, fabsf(dg[m][q2]));
        }
        // dgates of this step into acts (no other CTA reads them)
        auto store_dg = [&]() {
          _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
            const int ci = e + kEpi * m;
            const int b = ci & 31, ul = ci >> 5;
            if (ul >= UCP || b >= Bc) continue;
            const int64_t u = (int64_t)blk * UB + sp * UCP + ul, bb = bg0 + b;
            float *ar = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) ar[q2 * H] = dg[m][q2];
          }
        };
        if (t == 0) {
          store_dg();
          break;
        }
        // power-of-two scale of this CTA's dgates block (max over the CTA)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[ew] = mx;
        if (epi_sync_any(fail)) { fail = true; break; }
        float m8 = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) m8 = fmaxf(m8, red[w]);
        const float scl = pow2_scale(__float_as_uint(m8));
        unsigned char *xdst = xg + (size_t)(t & 1) * p.xbytes;
        _Pragma("unroll") for (int m = 0; m < NCELL; ++m) {
          const int ci = e + kEpi * m;
          const int b = ci % 32, ul = ci / 32;
          if (ul >= UCP || b >= Bc) continue;
#pragma unroll
          for (int q2 = 0; q2 < 4; ++q2) {
            const int64_t k = ((int64_t)cta * 4 + q2) * UCP + ul;  // producer-major gate-row order
            if (bf) {
              *reinterpret_cast<__nv_bfloat16 *>(xdst + koff(b, k, 1024)) = __float2bfloat16_rn(dg[m][q2]);
            } else {
              __half hi, lo;
              split_h2(dg[m][q2] * scl, hi, lo);
              *reinterpret_cast<__half *>(xdst + koff(b, k, 1024)) = hi;
              *reinterpret_cast<__half *>(xdst + koff(32 + b, k, 1024)) = lo;
            }
          }
        }
        if (e == 0 && !bf) __stcg(&xscale[(t & 1) * NC + cta], 1.0f / scl);
        asm volatile("fence.proxy.async.global;" ::: "memory");
        if (epi_sync_any(fail)) { fail = true; break; }
        if (e == 0) arrive_counter(bar);
        store_dg();
      }
    }
    // On the way out after a failure: partial sums of a phase this CTA
    // armed but did not see complete may still be landing; let them (bounded)
    // before the CTA may leave.
    if (e == 0 && pin_armed > pin_seen) mbar_drain(&bars[B_PIN], (uint32_t)((pin_armed - 1) & 1));
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every CTA of the cluster has seen its last partial sums land
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// ------------------------------------------------------------------ host
struct RtcPlan {
  int dir, KS, UCP, UB, NBLK, NC, ngrp, nchunk, gch, stages;
  bool resident, bf;
  int64_t K, Ks;
  size_t xbytes, smem;
  size_t o_bar, o_absmax, o_w, o_x, o_xs, total;
};

std::atomic<unsigned long long> g_attr[6];

// The kernel instance for a direction and k split (cells per epilogue
// thread = units per CTA x 32 / 256).
int ncell_of(int dir, int ks, int ub) { return (dir == 0 ? 32 : ub) / ks * 32 / kEpi; }
int attr_index(int dir, int ks, int ub) {
  const int n = ncell_of(dir, ks, ub);
  return dir * 3 + (n <= 1 ? 0 : n == 2 ? 1 : 2);
}
const void *rtc_fn(int dir, int ks, int ub) {
  const int n = ncell_of(dir, ks, ub);
  if (dir == 0) {
    if (n <= 1) return (const void *)rtc_kernel<0, 1>;
    if (n == 2) return (const void *)rtc_kernel<0, 2>;
    if (n == 4) return (const void *)rtc_kernel<0, 4>;
  } else {
    if (n <= 1) return (const void *)rtc_kernel<1, 1>;
    if (n == 2) return (const void *)rtc_kernel<1, 2>;
    if (n == 4) return (const void *)rtc_kernel<1, 4>;
  }
  return nullptr;
}

// Clusters of ks CTAs of the direction's kernel with `smem` bytes each that
// can be resident at once on the current device (0 if the query fails),
// cached per (device, direction, ks, smem).
int max_clusters(int dir, int ks, int ub, size_t smem) {
  struct Entry { int dev, dir, ks, ub; size_t smem; int n; };
  static std::mutex mu;
  static Entry cache[64];
  static int ncache = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < ncache; ++i)
    if (cache[i].dev == dev && cache[i].dir == dir && cache[i].ks == ks && cache[i].ub == ub && cache[i].smem == smem)
      return cache[i].n;
  const void *fn = rtc_fn(dir, ks, ub);
  if (!fn || allow_dynamic_smem(fn, kSmemMax, &g_attr[attr_index(dir, ks, ub)]) != HS_OK) return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)ks);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)ks;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  if (ncache < 64) cache[ncache++] = Entry{dev, dir, ks, ub, smem, n};
  return n;
}

bool make_rtc_plan(RtcPlan &p, int dir, int64_t B, int64_t H, int nsm, bool bf = false) {
  p = RtcPlan{};
  p.dir = dir;
  p.bf = bf;
  if (H <= 0 || B <= 0) return false;
  if (dir == 0 ? (H % 64 != 0) : (H % 64 != 0)) return false;
  p.K = dir == 0 ? H : 4 * H;
  // Weight blocks: forward 32 units x 4 gates = 128 rows; backward 128 or 64
  // units.  Among the k splits whose clusters all fit on the GPU at once (at
  // most 4 cells of 32 sequences per epilogue thread, whole 64-k chunks, a
  // backward producer block of whole chunks), take the one with the most
  // CTAs (each CTA streams or holds less of the weights and issues fewer
  // MMAs per step), then the larger block.
  bool found = false;
  RtcPlan best{};
  int best_fit = 0;
  for (int ub : {128, 64}) {
    if (dir == 0 && ub != 128) continue;
    const int unit_block = dir == 0 ? 32 : ub;
    if (H % unit_block) continue;
    for (int ks : {8, 4, 2, 1}) {
      RtcPlan c = p;
      c.UB = ub;
      c.NBLK = (int)(H / unit_block);
      const int64_t Ks = c.K / ks;
      if (c.K % ks || Ks % KCH || unit_block % ks || unit_block / ks > 32) continue;
      if ((int64_t)c.NBLK * ks > nsm) continue;
      c.KS = ks;
      c.Ks = Ks;
      c.UCP = unit_block / ks;
      if (dir == 1 && c.UCP % 8) continue;  // the backward tile prep reads 8 k of one block
      c.nchunk = (int)(Ks / KCH);
      // accumulator groups: forward every 256 k; backward one producer block
      // (4 x UCP k of one scale)
      const int64_t gk = dir == 0 ? std::min<int64_t>(256, Ks) : 4 * c.UCP;
      if (gk % KCH) continue;
      c.gch = (int)(gk / KCH);
      const int NW = bf ? ub : 2 * ub;
      const Layout Lr = make_layout(Ks, 0, true, NW);
      if (Lr.total <= kSmemMax && c.nchunk <= 32) {
        c.resident = true;
        c.stages = 0;
        c.smem = Lr.total;
      } else {
        c.resident = false;
        int S = 0;
        for (int st = 8; st >= 2; --st)
          if (make_layout(Ks, st, false, NW).total <= kSmemMax) { S = st; break; }
        if (!S) continue;
        c.stages = S;
        c.smem = make_layout(Ks, S, false, NW).total;
      }
      const int fit = max_clusters(dir, ks, ub, c.smem);
      if (fit < c.NBLK) continue;
      if (!found || c.NBLK * c.KS > best.NBLK * best.KS) {
        best = c;
        best_fit = fit;
        found = true;
      }
      break;  // smaller splits of this block size only have fewer CTAs
    }
  }
  if (!found) return false;
  p = best;
  const int fit = best_fit;
  p.NC = p.NBLK * p.KS;
  p.ngrp = (int)std::max<int64_t>(1, std::min<int64_t>((B + 31) / 32, fit / p.NBLK));
  p.xbytes = (size_t)p.K / 8 * 1024;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = round_up(off + bytes, 256); return o; };
  p.o_bar = take((size_t)p.ngrp * 128);
  p.o_absmax = take(16);
  p.o_w = take((size_t)p.NC * p.Ks * 4 * p.UB);
  p.o_x = take((size_t)p.ngrp * 2 * p.xbytes);
  p.o_xs = take((size_t)p.ngrp * 2 * p.NC * 4);
  p.total = off;
  return true;
}

int rtc_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

// Path choice: HS_REC_PATH=ffma|tc forces one (tests); otherwise the
// tensor-core kernels wherever their plan exists.
int rtc_override() {
  const char *e = getenv("HS_REC_PATH");
  if (!e) return 0;
  if (e[0] == 'f') return 1;
  if (e[0] == 't') return 2;
  return 0;
}

// Launch of one batch-group window: clusters of KS CTAs, cooperative (all
// clusters co-resident, which the step counter relies on).
int rtc_launch(const void *fn, const RtcPlan &pl, int ngrp, RtcArgs &args, cudaStream_t st) {
  const unsigned grid = (unsigned)(pl.NC * ngrp);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)pl.KS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeCooperative;
  at[1].val.cooperative = 1;
  cfg.attrs = at;
  // HS_REC_COOP=0 leaves out the cooperative attribute (for profilers that
  // cannot launch cooperative cluster kernels); every cluster still fits on
  // the GPU at once (checked below), and every wait on another CTA is bounded.
  const char *coop = getenv("HS_REC_COOP");
  cfg.numAttrs = (coop && coop[0] == '0') ? 1 : 2;
  int nclusters = 0;
  cudaLaunchConfig_t q = cfg;
  q.numAttrs = 1;
  if (cudaOccupancyMaxActiveClusters(&nclusters, fn, &q) != cudaSuccess)
    return check_launch("cudaOccupancyMaxActiveClusters(rtc)");
  if ((int64_t)nclusters * pl.KS < (int64_t)grid)
    return fail(HS_ERR_UNSUPPORTED, "recurrent (tensor cores): %u CTAs in clusters of %d, %d clusters fit", grid,
                pl.KS, nclusters);
  void *kargs[] = {&args};
  if (cudaLaunchKernelExC(&cfg, fn, kargs) != cudaSuccess) return check_launch("cudaLaunchKernelEx(rtc)");
  return HS_OK;
}

}  // namespace

// Default choice between the two recurrent implementations, per direction,
// from their per-step times measured on B200 at B = 32 (forward / backward,
// microseconds): H = 128 FFMA 5.3 / 10.9, tensor cores 8.4 / 13.7; H = 512
// FFMA 7.0 / 14.8, tensor cores 7.4 / 12.0; H = 2048 FFMA 63.7 / 76.5, tensor
// cores 26.5 / 48.4.  At small H both are bound by the cross-CTA exchange of
// the state (about 2.5 us per step) and the FFMA kernels' shorter epilogue
// wins; the tensor cores take over from H = 512 in the backward (four times
// the product of the forward per step) and from H = 1024 in the forward.
constexpr int64_t kTcMinH[2] = {1024, 512};

bool rec_tc_wanted(int dir, int64_t B, int64_t H, bool bf) {
  const int o = rtc_override();
  if (o == 1) return false;
  if (o == 0 && H < kTcMinH[dir]) return false;
  RtcPlan p;
  const int n = rtc_sms();
  return make_rtc_plan(p, dir, B, H, n > 0 ? n : 148, bf);
}

size_t rec_tc_ws_bytes(int64_t B, int64_t H) {
  const int n = rtc_sms() > 0 ? rtc_sms() : 148;
  size_t m = 0;
  for (int dir = 0; dir < 2; ++dir)
    for (bool bf : {false, true}) {
      RtcPlan pl;
      if (make_rtc_plan(pl, dir, B, H, n, bf)) m = std::max(m, pl.total);
    }
  return m;
}

namespace {
int rtc_prepare(const RtcPlan &pl, const float *w_hh, const float *a, int64_t H, char *w, int nsm, cudaStream_t st) {
  unsigned *absmax = reinterpret_cast<unsigned *>(w + pl.o_absmax);
  if (!pl.bf) {  // the fp16 split's weight scale (bf16 needs none)
    if (cudaMemsetAsync(absmax, 0, 4, st) != cudaSuccess) return check_launch("memset(absmax)");
    const int vec = aligned(w_hh, 16) ? 1 : 0;  // H is a multiple of 64
    rtc_absmax_kernel<<<dim3((unsigned)std::max(1, nsm / 2), 4), 256, 0, st>>>(w_hh, a, H, absmax, vec);
    if (int e = check_launch("rtc_absmax_kernel")) return e;
  }
  const int64_t n = (int64_t)pl.NC * (pl.Ks / 8) * (pl.bf ? 1 : 2) * pl.UB;
  rtc_prep_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 16 * nsm), 256, 0, st>>>(
      w_hh, a, absmax, reinterpret_cast<unsigned char *>(w + pl.o_w), pl.dir, H, pl.KS, pl.UCP, pl.UB, pl.Ks, pl.NC,
      pl.bf ? 1 : 0, aligned(w_hh, 16) ? 1 : 0);
  return check_launch("rtc_prep_kernel");
}

void fill_args(RtcArgs &args, const RtcPlan &pl, char *w, int *status, int64_t T, int64_t B, int64_t H, int64_t b0) {
  args.wg = reinterpret_cast<const unsigned char *>(w + pl.o_w);
  args.xg = reinterpret_cast<unsigned char *>(w + pl.o_x);
  args.xscale = reinterpret_cast<float *>(w + pl.o_xs);
  args.w_absmax = reinterpret_cast<const unsigned *>(w + pl.o_absmax);
  args.bar = reinterpret_cast<unsigned *>(w + pl.o_bar);
  args.status = status;
  args.T = T;
  args.Bt = B;
  args.H = H;
  args.bf = pl.bf ? 1 : 0;
  args.Ks = pl.Ks;
  args.xbytes = pl.xbytes;
  args.b0 = (int)b0;
  args.NC = pl.NC;
  args.KS = pl.KS;
  args.UCP = pl.UCP;
  args.UB = pl.UB;
  args.nchunk = pl.nchunk;
  args.gch = pl.gch;
  args.stages = pl.stages;
  args.resident = pl.resident ? 1 : 0;
}
}  // namespace

// Forward recurrence on the tensor cores; acts holds Z on entry (the input
// projection) and the gate activations on return.
// bf: bf16 mode (see the top of the file).
int rec_tc_forward(const float *h0, const float *c0, const float *w_hh, const float *b_hh, const float *a,
                   float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t H, void *ws,
                   size_t ws_bytes, int *status, cudaStream_t st, bool bf) {
  RtcPlan pl;
  const int nsm = rtc_sms();
  if (nsm <= 0) return fail(HS_ERR_CUDA, "no CUDA device");
  if (!make_rtc_plan(pl, 0, B, H, nsm, bf))
    return fail(HS_ERR_UNSUPPORTED, "recurrent (tensor cores): no plan for B=%lld H=%lld", (long long)B, (long long)H);
  if (!ws || ws_bytes < pl.total || !aligned(ws, 256))
    return fail(HS_ERR_WORKSPACE, "recurrent (tensor cores): workspace %zu < %zu bytes", ws_bytes, pl.total);
  char *w = static_cast<char *>(ws);
  if (int e = rtc_prepare(pl, w_hh, a, H, w, nsm, st)) return e;
  const void *fn = rtc_fn(0, pl.KS, pl.UB);
  if (!fn) return fail(HS_ERR_UNSUPPORTED, "recurrent (tensor cores): no kernel for KS=%d", pl.KS);
  if (int e = allow_dynamic_smem(fn, kSmemMax, &g_attr[attr_index(0, pl.KS, pl.UB)])) return e;
  for (int64_t b0 = 0; b0 < B; b0 += 32 * pl.ngrp) {
    const int ngrp = (int)std::min<int64_t>(pl.ngrp, (B - b0 + 31) / 32);
    if (cudaMemsetAsync(w + pl.o_bar, 0, (size_t)ngrp * 128, st) != cudaSuccess) return check_launch("memset(bar)");
    if (cudaMemsetAsync(w + pl.o_x, 0, (size_t)ngrp * 2 * pl.xbytes, st) != cudaSuccess)
      return check_launch("memset(xbuf)");
    RtcArgs args{};
    fill_args(args, pl, w, status, T, B, H, b0);
    args.xscale = nullptr;
    args.zacts = acts;
    args.h0 = h0;
    args.c0 = c0;
    args.h_save = h_save;
    args.c_save = c_save;
    args.b_hh = b_hh;
    args.a = a;
    if (int e = rtc_launch(fn, pl, ngrp, args, st)) return e;
  }
  return HS_OK;
}

// Backward recurrence on the tensor cores; acts holds the forward's gate
// activations on entry and dgates on return.
int rec_tc_backward(const float *w_hh, const float *a, const float *c_save, float *acts, const float *dout,
                    const float *dh_n, const float *dc_n, int64_t T, int64_t B, int64_t H, void *ws, size_t ws_bytes,
                    int *status, cudaStream_t st, bool bf) {
  RtcPlan pl;
  const int nsm = rtc_sms();
  if (nsm <= 0) return fail(HS_ERR_CUDA, "no CUDA device");
  if (!make_rtc_plan(pl, 1, B, H, nsm, bf))
    return fail(HS_ERR_UNSUPPORTED, "recurrent backward (tensor cores): no plan for B=%lld H=%lld", (long long)B,
                (long long)H);
  if (!ws || ws_bytes < pl.total || !aligned(ws, 256))
    return fail(HS_ERR_WORKSPACE, "recurrent backward (tensor cores): workspace %zu < %zu bytes", ws_bytes, pl.total);
  char *w = static_cast<char *>(ws);
  if (int e = rtc_prepare(pl, w_hh, a, H, w, nsm, st)) return e;
  const void *fn = rtc_fn(1, pl.KS, pl.UB);
  if (!fn) return fail(HS_ERR_UNSUPPORTED, "recurrent backward (tensor cores): no kernel for KS=%d", pl.KS);
  if (int e = allow_dynamic_smem(fn, kSmemMax, &g_attr[attr_index(1, pl.KS, pl.UB)])) return e;
  for (int64_t b0 = 0; b0 < B; b0 += 32 * pl.ngrp) {
    const int ngrp = (int)std::min<int64_t>(pl.ngrp, (B - b0 + 31) / 32);
    if (cudaMemsetAsync(w + pl.o_bar, 0, (size_t)ngrp * 128, st) != cudaSuccess) return check_launch("memset(bar)");
    if (cudaMemsetAsync(w + pl.o_x, 0, (size_t)ngrp * 2 * pl.xbytes, st) != cudaSuccess)
      return check_launch("memset(xbuf)");
    RtcArgs args{};
    fill_args(args, pl, w, status, T, B, H, b0);
    args.zacts = acts;
    args.c_save = const_cast<float *>(c_save);
    args.dout = dout;
    args.dh_n = dh_n;
    args.dc_n = dc_n;
    args.a = a;
    if (int e = rtc_launch(fn, pl, ngrp, args, st)) return e;
  }
  return HS_OK;
}

}  // namespace hs
