// tcgen05 / TMEM / TMA GEMM with float32 accuracy (3xTF32) for the
// linear-layer products of HeadStartLSTM (input projection x.W_ih^T + b_ih,
// input gradient dZ.W_ih, weight gradients dZ^T.x and dG^T.h).
//
// fp32 parity on tensor cores.  kind::tf32 reads fp32 words from shared
// memory and uses their top 19 bits (the low 13 mantissa bits are dropped).
// Each operand x is split as x = hi + lo with hi = x itself (the tensor core
// drops the low bits) and lo = x - trunc19(x) (exact in fp32), and
//     A.B ~= A.B_hi-part + A.B_lo + A_lo.B      (three MMAs per k-step)
// which leaves only the lo*lo product and the tf32 rounding of lo (~2^-21
// of |a||b| per term; measured ~7e-7 normwise, the level of an FFMA GEMM).
//
// Accumulation.  The tensor core adds each MMA's products into the fp32 TMEM
// accumulator with truncation (measured here: a bias toward zero of ~1e-6
// per 32-deep k-block, growing linearly with K).  Two measures keep the
// result at fp32 accuracy for any K:
//   * the big A.B product goes to its own accumulator (1 MMA per k-step);
//     the two small correction products (2^-11 of it) go to a second one;
//   * every PROMOTE k-blocks both accumulators are folded into fp32 register
//     totals (round-to-nearest adds) by the epilogue warps and restarted.
//     The accumulator pairs are double-buffered (4 x 128 of the 512 TMEM
//     columns) so the MMAs of the next group run while one is folded.
//
// Kernel structure (one 128 x 128 output tile per CTA, 1 CTA per SM):
//   warp 0      TMA producer: raw A/B k-blocks (32 fp32 = one 128-byte
//               swizzle row) into a ring of HS_TC_RAW_STAGES stages;
//   warp 1      allocates 512 TMEM columns; one lane issues tcgen05.mma and
//               commits raw stages back to the producer, lo slots back to
//               the transform and finished groups to the epilogue warps;
//   warps 2..5  compute lo for every k-block into a ring of HS_TC_LO_SLOTS
//               slots in shared memory (elementwise, so the swizzled layout
//               is kept);
//   warps 6..9  fold finished groups into their row's register totals (one
//               TMEM lane quadrant each) and finally store the tile (bias,
//               beta) or a split-K partial.  Folding in separate warps keeps
//               the transform running ahead of the tensor core.
// No cluster multicast anywhere.  Every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "hs_common.cuh"
#include "tc_dev.cuh"

namespace hs {

namespace {

// Raw operand stages (TMA targets) and lo slots (transform outputs) are
// separate rings: a raw stage is busy from its TMA issue until its MMAs
// complete, a lo slot only from the transform until the same MMAs, so a deep
// raw ring (load latency) and a short lo ring fit in shared memory together.
#ifndef HS_TC_RAW_STAGES
#define HS_TC_RAW_STAGES 3
#endif
#ifndef HS_TC_LO_SLOTS
#define HS_TC_LO_SLOTS 3
#endif
constexpr int BM = 128, BN = 128, BK = 32, PROMOTE = 4;
constexpr int STAGES = HS_TC_RAW_STAGES, LOS = HS_TC_LO_SLOTS;
constexpr int NTHREADS = 320;  // producer, MMA, 4 transform, 4 fold/epilogue warps
constexpr int A_BYTES = BM * BK * 4;                 // 16 KB
constexpr int B_BYTES = BN * BK * 4;                 // 16 KB
constexpr int RAW_BYTES = A_BYTES + B_BYTES;         // 32 KB
constexpr int LO_OFF = STAGES * RAW_BYTES;           // lo slots follow the raw stages
constexpr int SMEM_BYTES = (STAGES + LOS) * RAW_BYTES + 1024 /*align*/ + 256 /*barriers*/;
static_assert(SMEM_BYTES <= 232448, "shared memory per block");
static_assert((STAGES + LOS) * RAW_BYTES >= BM * BN * 4, "epilogue staging area");
constexpr uint32_t TMEM_COLS = 512;                  // 2 buffers x (main, correction) x 128


// lo = x - (x with its low 13 mantissa bits cleared), exact in fp32, then
// rounded to the nearest tf32 value so the tensor core's own truncation of
// it is exact (no bias toward zero).
HS_DEV float lo_part(float x) {
  const float r = x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  return __uint_as_float((__float_as_uint(r) + 0x1000u) & 0xFFFFE000u);
}


HS_DEV void tma_2d(void *dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(su32(dst)),
      "l"(tm), "r"(c0), "r"(c1), "r"(su32(bar))
      : "memory");
}



// Instruction descriptor: D f32, A/B tf32, majors, N>>3, M>>4.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

HS_DEV void mma_tf32(uint32_t dt, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(dt),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
HS_DEV void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}


struct TcArgs {
  float *C;
  const float *bias;
  float *partial;  // split-K partials [splits][M][N] or null
  int64_t M, N, K;
  int64_t ldc;
  int beta;
  int kb_per_split;
  int nkb;
  int *status;
  int out_bf16 = 0;  // pair kernel, bf16 operands: the output is bf16 (no split-K, no beta)
};

// Epilogue of the fold warps (128 threads, thread = tile row q*32+lane):
// stage the tile in shared memory (free: every MMA and load has completed) as
// four 128-row x 32-column boxes with the 128-byte swizzle (conflict-free
// row-per-thread writes), then write it with TMA bulk stores (reduce-add
// when beta = 1), or store a split-K partial.
HS_DEV void store_tile(const float (&tot)[BN], unsigned char *smem, const CUtensorMap *tmC_, const TcArgs &p,
                       int q, int lane, int t, int64_t m0, int64_t n0) {
  const CUtensorMap &tmC = *tmC_;
  const int r = q * 32 + lane;
  const bool direct = p.partial == nullptr;
  float *box0 = reinterpret_cast<float *>(smem);
#pragma unroll
  for (int c = 0; c < BN / 32; ++c) {
    float *boxc = box0 + c * (BM * 32);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 o = make_float4(tot[c * 32 + 4 * j], tot[c * 32 + 4 * j + 1], tot[c * 32 + 4 * j + 2],
                             tot[c * 32 + 4 * j + 3]);
      if (direct && p.bias) {
        const int64_t n = n0 + c * 32 + 4 * j;
        if (n + 3 < p.N) {
          const float4 bb = *reinterpret_cast<const float4 *>(p.bias + n);
          o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
        } else {
          if (n < p.N) o.x += p.bias[n];
          if (n + 1 < p.N) o.y += p.bias[n + 1];
          if (n + 2 < p.N) o.z += p.bias[n + 2];
        }
      }
      *reinterpret_cast<float4 *>(boxc + r * 32 + ((j ^ (r & 7)) * 4)) = o;
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (t == 0) {
    const int zc = p.partial ? (int)blockIdx.z : 0;
#pragma unroll
    for (int c = 0; c < BN / 32; ++c) {
      if (direct && p.beta) tma_reduce_add_3d(&tmC, box0 + c * (BM * 32), (int)n0 + 32 * c, (int)m0, zc);
      else tma_store_3d(&tmC, box0 + c * (BM * 32), (int)n0 + 32 * c, (int)m0, zc);
    }
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NTHREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, TcArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (STAGES + LOS) * RAW_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *xformed = empty + STAGES;  // [LOS] lo slot written
  uint64_t *lofree = xformed + LOS;    // [LOS] lo slot consumed by its MMAs
  uint64_t *pfull = lofree + LOS;     // [2] group finished in accumulator pair b
  uint64_t *pempty = pfull + 2;       // [2] accumulator pair b folded, reusable
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(pempty + 2);
  int *abort_flag = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(p.nkb, kb0 + p.kb_per_split);
  const int nk = kb1 - kb0;
  const int ngroups = (nk + PROMOTE - 1) / PROMOTE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int l = 0; l < LOS; ++l) {
      mbar_init(&xformed[l], 4);
      mbar_init(&lofree[l], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 4);
    }
    *abort_flag = ld_status(p.status) != 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  const bool skip = *abort_flag != 0 || nk <= 0;

  if (!skip && warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, p.status)) break;
        ++issued;
        unsigned char *st = smem + s * RAW_BYTES;
        mbar_expect_tx(&full[s], RAW_BYTES);
        const int k0 = (kb0 + i) * BK;
        // M/N-major operands arrive as 32 x 32 boxes (128-byte rows of 32
        // M/N elements, 32 k rows), one 4 KB block per 32 rows of M/N.
        if (A_MN) {
#pragma unroll
          for (int j = 0; j < BM / 32; ++j) tma_2d(st + j * 4096, &tmA, &full[s], (int)m0 + 32 * j, k0);
        } else {
          tma_2d(st, &tmA, &full[s], k0, (int)m0);
        }
        if (B_MN) {
#pragma unroll
          for (int j = 0; j < BN / 32; ++j) tma_2d(st + A_BYTES + j * 4096, &tmB, &full[s], (int)n0 + 32 * j, k0);
        } else {
          tma_2d(st + A_BYTES, &tmB, &full[s], k0, (int)n0);
        }
      }
      // Never leave while a copy into this CTA's shared memory is in flight:
      // wait (bounded) for the last load issued into each stage.
      for (int i = std::max(0, issued - STAGES); i < issued; ++i) {
        if (ld_status(p.status)) mbar_drain(&full[i % STAGES], (i / STAGES) & 1);
        else (void)mbar_wait(&full[i % STAGES], (i / STAGES) & 1, p.status);
      }
    }
  } else if (!skip && warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        const int l = i % LOS;
        const uint32_t lph = (i / LOS) & 1;
        const int g = i / PROMOTE, b = g & 1;
        const bool gstart = (i % PROMOTE) == 0;
        if (gstart && !mbar_wait(&pempty[b], ((g >> 1) & 1) ^ 1, p.status)) break;
        if (!mbar_wait(&xformed[l], lph, p.status)) break;  // implies full[s] of this k-block
        (void)ph;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_raw = su32(smem + s * RAW_BYTES);
        const uint32_t b_raw = a_raw + A_BYTES;
        const uint32_t a_lo = su32(smem + LO_OFF + l * RAW_BYTES);
        const uint32_t b_lo = a_lo + A_BYTES;
        const uint32_t t_main = tmem + (uint32_t)(b * 2 * BN);
        const uint32_t t_corr = t_main + BN;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          // K-major (layout 2): the 8 k of this step are 32 bytes into each
          // 128-byte row; 8-row groups are 1 KB apart (SBO).
          // M/N-major (layout 1): the 8 k are the next 8 rows of 128 bytes
          // (two 512-byte atoms of 4 rows, SBO = 512); the 32-wide M/N blocks
          // are 4 KB apart (LBO).
          const uint32_t ao = A_MN ? kk * 1024 : kk * 32;
          const uint32_t bo = B_MN ? kk * 1024 : kk * 32;
          const uint32_t la = A_MN ? 1u : 2u, lb = B_MN ? 1u : 2u;
          const uint32_t albo = A_MN ? 4096 : 16, asbo = A_MN ? 512 : 1024;
          const uint32_t blbo = B_MN ? 4096 : 16, bsbo = B_MN ? 512 : 1024;
          const uint64_t dA = sdesc(a_raw + ao, albo, asbo, la), dAl = sdesc(a_lo + ao, albo, asbo, la);
          const uint64_t dB = sdesc(b_raw + bo, blbo, bsbo, lb), dBl = sdesc(b_lo + bo, blbo, bsbo, lb);
          const uint32_t acc = (gstart && kk == 0) ? 0u : 1u;
          mma_tf32(t_main, dA, dB, idesc, acc);
          mma_tf32(t_corr, dA, dBl, idesc, acc);
          mma_tf32(t_corr, dAl, dB, idesc, 1u);
        }
        mma_commit(&empty[s]);
        mma_commit(&lofree[l]);
        if ((i % PROMOTE) == PROMOTE - 1 || i == nk - 1) mma_commit(&pfull[b]);
      }
    }
  } else if (!skip && warp < 6) {
    // ---------------- transform: lo parts of every k-block
    const int t = threadIdx.x - 64;  // 0..127
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1;
      const int l = i % LOS;
      const uint32_t lph = (i / LOS) & 1;
      if (!mbar_wait(&lofree[l], lph ^ 1, p.status)) break;
      if (!mbar_wait(&full[s], ph, p.status)) break;
      const float4 *raw = reinterpret_cast<const float4 *>(smem + s * RAW_BYTES);
      float4 *lo = reinterpret_cast<float4 *>(smem + LO_OFF + l * RAW_BYTES);
#pragma unroll 4
      for (int j = t; j < RAW_BYTES / 16; j += 128) {
        const float4 v = raw[j];
        lo[j] = make_float4(lo_part(v.x), lo_part(v.y), lo_part(v.z), lo_part(v.w));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&xformed[l]);
    }
  } else if (!skip) {
    // ---------------- fold finished groups into register totals, epilogue
    const int t = threadIdx.x - 192;  // 0..127
    const int q = warp & 3;           // TMEM lane quadrant of this warp
    float tot[BN];
#pragma unroll
    for (int j = 0; j < BN; ++j) tot[j] = 0.f;
    bool ok = true;
    for (int g = 0; g < ngroups; ++g) {
      const int b = g & 1;
      if (!mbar_wait(&pfull[b], (g >> 1) & 1, p.status)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 2 * BN);
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld32(base + BN + c, v);  // correction first: tot += (corr + main)
#pragma unroll
        for (int j = 0; j < 32; ++j) tot[c + j] += v[j];
        tmem_ld32(base + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) tot[c + j] += v[j];
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[b]);
    }
    if (ok) {
      // Stage the tile in shared memory (stage 0 is free: every MMA has
      // completed) as four 128-row x 32-column boxes with the 128-byte
      // swizzle (conflict-free row-per-thread writes), then write it with
      // TMA bulk stores (reduce-add when beta = 1).
      store_tile(tot, smem, &tmC, p, q, lane, t, m0, n0);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}


// ---------------------------------------------------------------- operand A in TMEM
// Variant for K-major A (the projection x.W_ih^T and the input gradient
// dZ.W_ih).  Shared memory is the bound of the kernel above: per 32-deep
// k-block the three MMAs read 96 KB of operands, the TMA writes 32 KB and the
// lo transform reads 32 KB and writes 32 KB, against 128 B/clk per SM.  Here
// the transform warps copy each k-block's A rows into tensor memory, both the
// raw words and their lo parts (tcgen05.st, one row per thread), and the MMAs
// take A from TMEM ("TS" form): per k-block shared memory then carries the
// TMA's 32 KB, the transform's 32 KB of reads and 16 KB of B_lo writes, and
// the MMAs' 48 KB of B reads.
//
// TMEM columns: [0,128) and [128,256) are two accumulators (one per group,
// double-buffered as above, but each holds the main product and both
// corrections); [256 + 64 l, +32) and [+32, +64) hold A raw / A lo of lo-slot
// l.  With every product in one accumulator each MMA adds into a value of the
// group's magnitude, so groups are kept short (TA_PROMOTE k-blocks) and
// folded into float32 register totals by the fold warps.
#ifndef HS_TA_STAGES
#define HS_TA_STAGES 4
#endif
#ifndef HS_TA_LOS
#define HS_TA_LOS 3
#endif
#ifndef HS_TA_PROMOTE
#define HS_TA_PROMOTE 2
#endif
constexpr int TA_STAGES = HS_TA_STAGES, TA_LOS = HS_TA_LOS, TA_PROMOTE = HS_TA_PROMOTE;
constexpr int TA_BLO_OFF = TA_STAGES * RAW_BYTES;                 // B_lo slots after the raw stages
constexpr int TA_SMEM_BYTES = TA_STAGES * RAW_BYTES + TA_LOS * B_BYTES + 1024 + 256;
constexpr uint32_t TA_ACOL = 2 * BN;                              // first A-slot column
static_assert(TA_ACOL + TA_LOS * 64 <= TMEM_COLS, "TMEM columns");
static_assert(TA_SMEM_BYTES <= 232448, "shared memory per block");
static_assert(TA_STAGES * RAW_BYTES + TA_LOS * B_BYTES >= BM * BN * 4, "epilogue staging area");

HS_DEV void mma_tf32_ts(uint32_t dt, uint32_t at, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(dt),
      "r"(at), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

HS_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

template <bool B_MN>
__global__ void __launch_bounds__(NTHREADS, 1)
gemm_ta_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, TcArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + TA_STAGES * RAW_BYTES + TA_LOS * B_BYTES);
  uint64_t *empty = full + TA_STAGES;
  uint64_t *xformed = empty + TA_STAGES;  // [TA_LOS] A slot + B_lo slot written
  uint64_t *lofree = xformed + TA_LOS;    // [TA_LOS] consumed by their MMAs
  uint64_t *pfull = lofree + TA_LOS;      // [2] group finished in accumulator b
  uint64_t *pempty = pfull + 2;           // [2] accumulator b folded, reusable
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(pempty + 2);
  int *abort_flag = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(p.nkb, kb0 + p.kb_per_split);
  const int nk = kb1 - kb0;
  const int ngroups = (nk + TA_PROMOTE - 1) / TA_PROMOTE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TA_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int l = 0; l < TA_LOS; ++l) {
      mbar_init(&xformed[l], 4);
      mbar_init(&lofree[l], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 4);
    }
    *abort_flag = ld_status(p.status) != 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  const bool skip = *abort_flag != 0 || nk <= 0;

  if (!skip && warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % TA_STAGES;
        const uint32_t ph = (i / TA_STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, p.status)) break;
        ++issued;
        unsigned char *st = smem + s * RAW_BYTES;
        mbar_expect_tx(&full[s], RAW_BYTES);
        const int k0 = (kb0 + i) * BK;
        tma_2d(st, &tmA, &full[s], k0, (int)m0);
        if (B_MN) {
#pragma unroll
          for (int j = 0; j < BN / 32; ++j) tma_2d(st + A_BYTES + j * 4096, &tmB, &full[s], (int)n0 + 32 * j, k0);
        } else {
          tma_2d(st + A_BYTES, &tmB, &full[s], k0, (int)n0);
        }
      }
      for (int i = std::max(0, issued - TA_STAGES); i < issued; ++i) {
        if (ld_status(p.status)) mbar_drain(&full[i % TA_STAGES], (i / TA_STAGES) & 1);
        else (void)mbar_wait(&full[i % TA_STAGES], (i / TA_STAGES) & 1, p.status);
      }
    }
  } else if (!skip && warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(BM, BN, false, B_MN);
      for (int i = 0; i < nk; ++i) {
        const int s = i % TA_STAGES;
        const int l = i % TA_LOS;
        const uint32_t lph = (i / TA_LOS) & 1;
        const int g = i / TA_PROMOTE, b = g & 1;
        const bool gstart = (i % TA_PROMOTE) == 0;
        if (gstart && !mbar_wait(&pempty[b], ((g >> 1) & 1) ^ 1, p.status)) break;
        if (!mbar_wait(&xformed[l], lph, p.status)) break;  // implies full[s] of this k-block
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t b_raw = su32(smem + s * RAW_BYTES) + A_BYTES;
        const uint32_t b_lo = su32(smem + TA_BLO_OFF + l * B_BYTES);
        const uint32_t t_acc = tmem + (uint32_t)(b * BN);
        const uint32_t a_raw = tmem + TA_ACOL + (uint32_t)(l * 64);
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint32_t bo = B_MN ? kk * 1024 : kk * 32;
          const uint32_t lb = B_MN ? 1u : 2u;
          const uint32_t blbo = B_MN ? 4096 : 16, bsbo = B_MN ? 512 : 1024;
          const uint64_t dB = sdesc(b_raw + bo, blbo, bsbo, lb), dBl = sdesc(b_lo + bo, blbo, bsbo, lb);
          const uint32_t acc = (gstart && kk == 0) ? 0u : 1u;
          mma_tf32_ts(t_acc, a_raw + kk * 8, dB, idesc, acc);
          mma_tf32_ts(t_acc, a_raw + kk * 8, dBl, idesc, 1u);
          mma_tf32_ts(t_acc, a_raw + 32 + kk * 8, dB, idesc, 1u);
        }
        mma_commit(&empty[s]);
        mma_commit(&lofree[l]);
        if ((i % TA_PROMOTE) == TA_PROMOTE - 1 || i == nk - 1) mma_commit(&pfull[b]);
      }
    }
  } else if (!skip && warp < 6) {
    // ---------------- transform: A rows -> TMEM (raw, lo), B -> B_lo in smem
    const int t = threadIdx.x - 64;  // 0..127
    const int q = warp & 3;          // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;     // A row (TMEM lane) of this thread
    for (int i = 0; i < nk; ++i) {
      const int s = i % TA_STAGES;
      const uint32_t ph = (i / TA_STAGES) & 1;
      const int l = i % TA_LOS;
      const uint32_t lph = (i / TA_LOS) & 1;
      if (!mbar_wait(&lofree[l], lph ^ 1, p.status)) break;
      if (!mbar_wait(&full[s], ph, p.status)) break;
      // A: row r of the K-major 128-byte-swizzled tile; 16-byte chunk c of
      // the row (k = 4c..4c+3) sits at chunk position c ^ (r % 8).
      const unsigned char *arow = smem + s * RAW_BYTES + r * 128;
      uint32_t hi[32], lo[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 v = *reinterpret_cast<const float4 *>(arow + ((c ^ (r & 7)) << 4));
        hi[4 * c + 0] = __float_as_uint(v.x);
        hi[4 * c + 1] = __float_as_uint(v.y);
        hi[4 * c + 2] = __float_as_uint(v.z);
        hi[4 * c + 3] = __float_as_uint(v.w);
        lo[4 * c + 0] = __float_as_uint(lo_part(v.x));
        lo[4 * c + 1] = __float_as_uint(lo_part(v.y));
        lo[4 * c + 2] = __float_as_uint(lo_part(v.z));
        lo[4 * c + 3] = __float_as_uint(lo_part(v.w));
      }
      const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + TA_ACOL + (uint32_t)(l * 64);
      tmem_st32(ta, hi);
      tmem_st32(ta + 32, lo);
      // B: elementwise lo parts (the swizzled layout is kept)
      const float4 *braw = reinterpret_cast<const float4 *>(smem + s * RAW_BYTES + A_BYTES);
      float4 *blo = reinterpret_cast<float4 *>(smem + TA_BLO_OFF + l * B_BYTES);
#pragma unroll 4
      for (int j = t; j < B_BYTES / 16; j += 128) {
        const float4 v = braw[j];
        blo[j] = make_float4(lo_part(v.x), lo_part(v.y), lo_part(v.z), lo_part(v.w));
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&xformed[l]);
    }
  } else if (!skip) {
    // ---------------- fold finished groups into register totals, epilogue
    const int t = threadIdx.x - 192;  // 0..127
    const int q = warp & 3;
    float tot[BN];
#pragma unroll
    for (int j = 0; j < BN; ++j) tot[j] = 0.f;
    bool ok = true;
    for (int g = 0; g < ngroups; ++g) {
      const int b = g & 1;
      if (!mbar_wait(&pfull[b], (g >> 1) & 1, p.status)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN);
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld32(base + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) tot[c + j] += v[j];
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[b]);
    }
    if (ok) store_tile(tot, smem, &tmC, p, q, lane, t, m0, n0);
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}


// ---------------------------------------------------------------- 3 x fp16 split
// K-major products (the projection x.W_ih^T) on the f16 tensor-core kind,
// which runs at twice the tf32 rate and reads half the operand bytes.  Each
// operand is scaled by a power of two s (so that max|x s| lies in
// [2^14, 2^15)) and split into two fp16 words,
//     hi = fp16(x s),   lo = fp16(x s - hi),
// which keep 22 significand bits together (as tf32 hi + lo do), and
//     A.B ~= [Ah.Bh + Ah.Bl + Al.Bh] / (s_A s_B)
// in three MMAs per k-step; the tensor core's float32 sums run over a few
// k-blocks at a time and are then added in float32 registers (promotion),
// as in the tf32 kernel.  Elements far below the tensor's maximum lose
// relative precision in fp16's subnormal range (lo below 2^-14, i.e.
// |x s| < 2^-4); their absolute error stays below 2^-25 in scaled units,
// 2^-39 of the largest element, far under the float32 result's own rounding.
// The split runs as a separate pass over each operand (absmax, then split),
// into caller workspace.
// (pow2_scale: hs_common.cuh)

// Rows are taken one warp at a time (warps of the whole grid round-robin),
// lanes stride over the columns: coalesced, no per-element index division.
__global__ void absmax_kernel(const float *__restrict__ x, int64_t rows, int64_t cols, int64_t ld,
                              unsigned *out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarp = ((int64_t)gridDim.x * blockDim.x) >> 5;
  float m = 0.f;
  for (int64_t r = warp; r < rows; r += nwarp) {
    const float *row = x + r * ld;
    for (int64_t c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(row[c]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) atomicMax(out, __float_as_uint(m));
}

// hi/lo [rows][ldo] fp16, ldo = cols rounded up to 8 (zero padding).  Lanes
// take 4 consecutive columns (one float4 load when the row allows it, one
// 8-byte store per part).
__global__ void split_h2_kernel(const float *__restrict__ x, int64_t rows, int64_t cols, int64_t ld,
                                const unsigned *__restrict__ absmax, __half *__restrict__ hi,
                                __half *__restrict__ lo, int64_t ldo, const int *gate = nullptr) {
  if (gate && *gate == 0) return;  // a conditional split that is not needed this time
  const float s = pow2_scale(*absmax);
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarp = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const bool vec = (cols % 4 == 0) && (ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  for (int64_t r = warp; r < rows; r += nwarp) {
    const float *row = x + r * ld;
    __half *hr = hi + r * ldo, *lr = lo + r * ldo;
    for (int64_t c = 4 * lane; c < ldo; c += 128) {  // ldo is a multiple of 8, so c+3 < ldo
      float v[4];
      if (vec && c + 3 < cols) {
        const float4 q = *reinterpret_cast<const float4 *>(row + c);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = c + j < cols ? row[c + j] : 0.f;
      }
      __half h[4], l[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float y = v[j] * s;
        h[j] = __float2half_rn(y);
        l[j] = __float2half_rn(y - __half2float(h[j]));
      }
      *reinterpret_cast<uint2 *>(hr + c) = *reinterpret_cast<const uint2 *>(h);
      *reinterpret_cast<uint2 *>(lr + c) = *reinterpret_cast<const uint2 *>(l);
    }
  }
}

HS_DEV void mma_f16(uint32_t dt, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dt),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

constexpr int H3_BK = 64;                        // fp16 k per block: one 128-byte row
constexpr int H3_TILE = 128 * H3_BK * 2;         // 16 KB per operand part
constexpr int H3_STAGE = 4 * H3_TILE;            // Ah, Al, Bh, Bl
constexpr int H3_STAGES = 3;
#ifndef HS_H3_PROMOTE
#define HS_H3_PROMOTE 4
#endif
constexpr int H3_PROMOTE = HS_H3_PROMOTE;         // k-blocks per accumulator group
// 1: Ah.Bh and Ah.Bl as one N = 256 MMA (Bh and Bl are adjacent in shared
// memory, main and correction accumulators adjacent in TMEM), so A_hi is
// read once per k-step for both; 0: three N = 128 MMAs.
#ifndef HS_H3_WIDE
#define HS_H3_WIDE 1
#endif
constexpr int H3_THREADS = 192;                  // producer, MMA, 4 fold/epilogue warps
constexpr int H3_SMEM_BYTES = H3_STAGES * H3_STAGE + 1024 + 256;
static_assert(H3_SMEM_BYTES <= 232448, "shared memory per block");

// An operand part in shared memory is 16 KB either way: K-major, 128 rows of
// 64 k (one 128-byte swizzled row each); MN-major, two 8 KB blocks of 64 M/N
// elements x 64 k rows (canonical SW128 MN-major layout: 8-row atoms 1 KB
// apart, blocks 8 KB apart).
//
// Persistent: one CTA per SM walks the output tiles (n fastest, then m,
// then the split), the load ring and the accumulator groups continuing from
// tile to tile, so the MMAs of the next tile run while the fold warps finish
// the last groups and the epilogue of the previous one.  The epilogue stages
// one 128 x 32 box at a time in its own 16 KB buffer (the operand stages
// belong to the next tile's loads by then).
constexpr int H3_EPI = BM * 32 * 4;              // 16 KB staging box
constexpr int H3_SMEM_P = H3_STAGES * H3_STAGE + H3_EPI + 1024 + 256;
static_assert(H3_SMEM_P <= 232448, "shared memory per block");


// bar_id: the named barrier of these 128 threads (1 unless several groups
// store at once).
HS_DEV void store_tile_boxes(const float (&tot)[BN], float *box, const CUtensorMap *tmC_, const TcArgs &p, int q,
                             int lane, int t, int64_t m0, int64_t n0, int zc, int bar_id = 1) {
  const CUtensorMap &tmC = *tmC_;
  const int r = q * 32 + lane;
  const bool direct = p.partial == nullptr;
#pragma unroll
  for (int c = 0; c < BN / 32; ++c) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 o = make_float4(tot[c * 32 + 4 * j], tot[c * 32 + 4 * j + 1], tot[c * 32 + 4 * j + 2],
                             tot[c * 32 + 4 * j + 3]);
      if (direct && p.bias) {
        const int64_t n = n0 + c * 32 + 4 * j;
        if (n + 3 < p.N) {
          const float4 bb = *reinterpret_cast<const float4 *>(p.bias + n);
          o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
        } else {
          if (n < p.N) o.x += p.bias[n];
          if (n + 1 < p.N) o.y += p.bias[n + 1];
          if (n + 2 < p.N) o.z += p.bias[n + 2];
        }
      }
      *reinterpret_cast<float4 *>(box + r * 32 + ((j ^ (r & 7)) * 4)) = o;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_sync(bar_id);
    if (t == 0) {
      if (direct && p.beta) tma_reduce_add_3d(&tmC, box, (int)n0 + 32 * c, (int)m0, zc);
      else tma_store_3d(&tmC, box, (int)n0 + 32 * c, (int)m0, zc);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // box free again
    }
    named_sync(bar_id);
  }
}

// The same epilogue writing bf16 (a bf16 module's Z or dX): 128-row x
// 64-column bf16 boxes (128-byte rows, the same swizzle), bias added in
// float32 before the rounding.  No split-K partials, no beta.
HS_DEV uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&v);
}
HS_DEV void store_tile_boxes_bf16(const float (&tot)[BN], float *boxf, const CUtensorMap *tmC_, const TcArgs &p,
                                  int q, int lane, int t, int64_t m0, int64_t n0, int bar_id) {
  const CUtensorMap &tmC = *tmC_;
  const int r = q * 32 + lane;
  uint4 *box = reinterpret_cast<uint4 *>(boxf);
#pragma unroll
  for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int64_t n = n0 + c * 64 + 8 * j + e;
        v[e] = tot[c * 64 + 8 * j + e] + ((p.bias && n < p.N) ? p.bias[n] : 0.f);
      }
      box[r * 8 + (j ^ (r & 7))] =
          make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_sync(bar_id);
    if (t == 0) {
      tma_store_3d(&tmC, box, (int)n0 + 64 * c, (int)m0, 0);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // box free again
    }
    named_sync(bar_id);
  }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(H3_THREADS, 1)
gemm_h3_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
               const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
               const __grid_constant__ CUtensorMap tmC, TcArgs p, const unsigned *absmax_a,
               const unsigned *absmax_b, int mtiles, int ntiles, int ntiles_total) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *epi = reinterpret_cast<float *>(smem + H3_STAGES * H3_STAGE);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + H3_STAGES * H3_STAGE + H3_EPI);
  uint64_t *empty = full + H3_STAGES;
  uint64_t *pfull = empty + H3_STAGES;
  uint64_t *pempty = pfull + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(pempty + 2);
  int *abort_flag = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto tile_of = [&](int tl, int64_t &m0, int64_t &n0, int &z, int &nk) {
    const int per = mtiles * ntiles;
    z = tl / per;
    const int rem = tl - z * per;
    m0 = (int64_t)(rem / ntiles) * BM;
    n0 = (int64_t)(rem % ntiles) * BN;
    const int kb0 = z * p.kb_per_split;
    nk = min(p.nkb, kb0 + p.kb_per_split) - kb0;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < H3_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 4);
    }
    *abort_flag = ld_status(p.status) != 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  const bool skip = *abort_flag != 0;

  if (!skip && warp == 0) {
    // ---------------- TMA producer: the k-blocks of every tile of this CTA
    if (lane == 0) {
      int it = 0, issued = 0;
      bool ok = true;
      for (int tl = blockIdx.x; tl < ntiles_total && ok; tl += gridDim.x) {
        int64_t m0, n0;
        int z, nk;
        tile_of(tl, m0, n0, z, nk);
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % H3_STAGES;
          const uint32_t ph = (it / H3_STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status)) { ok = false; break; }
          ++issued;
          unsigned char *st = smem + s * H3_STAGE;
          mbar_expect_tx(&full[s], H3_STAGE);
          const int k0 = (z * p.kb_per_split + i) * H3_BK;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              tma_2d(st + j * 8192, &tmAh, &full[s], (int)m0 + 64 * j, k0);
              tma_2d(st + H3_TILE + j * 8192, &tmAl, &full[s], (int)m0 + 64 * j, k0);
            }
          } else {
            tma_2d(st, &tmAh, &full[s], k0, (int)m0);
            tma_2d(st + H3_TILE, &tmAl, &full[s], k0, (int)m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              tma_2d(st + 2 * H3_TILE + j * 8192, &tmBh, &full[s], (int)n0 + 64 * j, k0);
              tma_2d(st + 3 * H3_TILE + j * 8192, &tmBl, &full[s], (int)n0 + 64 * j, k0);
            }
          } else {
            tma_2d(st + 2 * H3_TILE, &tmBh, &full[s], k0, (int)n0);
            tma_2d(st + 3 * H3_TILE, &tmBl, &full[s], k0, (int)n0);
          }
        }
      }
      // never leave while a copy into this CTA's shared memory is in flight
      for (int j = std::max(0, issued - H3_STAGES); j < issued; ++j) {
        if (ld_status(p.status)) mbar_drain(&full[j % H3_STAGES], (j / H3_STAGES) & 1);
        else (void)mbar_wait(&full[j % H3_STAGES], (j / H3_STAGES) & 1, p.status);
      }
    }
  } else if (!skip && warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t majors = ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16);
      constexpr uint32_t idesc = idesc_f16(BM, BN) | majors;
      constexpr uint32_t idesc2 = idesc_f16(BM, 2 * BN) | majors;
      (void)idesc2;
      int it = 0, gg = 0;
      bool ok = true;
      for (int tl = blockIdx.x; tl < ntiles_total && ok; tl += gridDim.x) {
        int64_t m0, n0;
        int z, nk;
        tile_of(tl, m0, n0, z, nk);
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % H3_STAGES;
          const uint32_t ph = (it / H3_STAGES) & 1;
          const bool gstart = (i % H3_PROMOTE) == 0;
          const int b = gg & 1;
          if (gstart && !mbar_wait(&pempty[b], ((gg >> 1) & 1) ^ 1, p.status)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, p.status)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t ah = su32(smem + s * H3_STAGE);
          const uint32_t al = ah + H3_TILE, bh = ah + 2 * H3_TILE, bl = ah + 3 * H3_TILE;
          const uint32_t t_main = tmem + (uint32_t)(b * 2 * BN);
          const uint32_t t_corr = t_main + BN;
#pragma unroll
          for (int kk = 0; kk < H3_BK / 16; ++kk) {
            // K-major: 16 fp16 = 32 bytes into each 128-byte row; MN-major: the
            // next 16 k rows (2 KB), LBO = 8 KB between 64-element blocks.
            const uint32_t oa = A_MN ? kk * 2048 : kk * 32, ob = B_MN ? kk * 2048 : kk * 32;
            const uint32_t la = A_MN ? 8192 : 16, lb = B_MN ? 8192 : 16;
            const uint64_t dAh = sdesc(ah + oa, la, 1024, 2), dAl = sdesc(al + oa, la, 1024, 2);
            const uint64_t dBh = sdesc(bh + ob, lb, 1024, 2), dBl = sdesc(bl + ob, lb, 1024, 2);
            const uint32_t acc = (gstart && kk == 0) ? 0u : 1u;
#if HS_H3_WIDE
            (void)dBl;
            mma_f16(t_main, dAh, dBh, idesc2, acc);  // [main | corr] = Ah.[Bh | Bl]
#else
            mma_f16(t_main, dAh, dBh, idesc, acc);
            mma_f16(t_corr, dAh, dBl, idesc, acc);
#endif
            mma_f16(t_corr, dAl, dBh, idesc, 1u);
          }
          mma_commit(&empty[s]);
          if ((i % H3_PROMOTE) == H3_PROMOTE - 1 || i == nk - 1) {
            mma_commit(&pfull[b]);
            ++gg;
          }
        }
      }
    }
  } else if (!skip) {
    // ---------------- fold finished groups, epilogue per tile
    const int t = threadIdx.x - 64;  // 0..127
    const int q = warp & 3;
    // Undo the two operand scales one at a time: each inverse is an exact
    // power of two within float range, their product may not be (tiny
    // operands get scales up to 2^114 each).
    const float inv_a = 1.0f / pow2_scale(*absmax_a), inv_b = 1.0f / pow2_scale(*absmax_b);
    int gg = 0;
    bool ok = true;
    for (int tl = blockIdx.x; tl < ntiles_total && ok; tl += gridDim.x) {
      int64_t m0, n0;
      int z, nk;
      tile_of(tl, m0, n0, z, nk);
      const int ngroups = (nk + H3_PROMOTE - 1) / H3_PROMOTE;
      float tot[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) tot[j] = 0.f;
      for (int g = 0; g < ngroups; ++g, ++gg) {
        const int b = gg & 1;
        if (!mbar_wait(&pfull[b], (gg >> 1) & 1, p.status)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 2 * BN);
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
          float v[32], w[32];
          tmem_ld32(base + BN + c, w);
          tmem_ld32(base + c, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) tot[c + j] += w[j] + v[j];
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[b]);
      }
      if (!ok) break;
#pragma unroll
      for (int j = 0; j < BN; ++j) tot[j] = (tot[j] * inv_a) * inv_b;
      store_tile_boxes(tot, epi, &tmC, p, q, lane, t, m0, n0, p.partial ? z : 0);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- 2-SM pairs
// The same 3 x fp16 product with the pair MMA (tcgen05 cta_group::2): a
// cluster of two CTAs on two SMs computes a 256 x 256 output tile, each CTA
// holding 128 rows of A and 128 rows (N) of B per stage in its own shared
// memory, and the MMA reads both halves of B across the pair.  Per SM and
// k-step of 16 this reads 4 KB of A and 4 KB of B per product (half what a
// one-SM 128 x 256 tile reads for the same work), which keeps the three
// products per k-step below the shared-memory bandwidth.  The three products
// go into ONE accumulator (lo parts are unscaled), 256 TMEM columns, so two
// accumulator buffers fit the 512 columns.
//
// Roles: warp 0 loads (both CTAs, each its own rows; the completion bytes of
// both land on the first CTA's barrier), warp 1 of the first CTA issues the
// MMAs, warps 2-9 of both CTAs fold the groups and store the tile (two
// groups of four warps, one per 128-column half, thread = row).
//
// Cross-CTA signals without multicast: the first CTA's producer, having seen
// a stage freed by the MMAs (one commit covers both CTAs' operands), passes
// the release on to the second CTA's barrier; the first CTA's fold thread
// passes on "accumulator ready" likewise; every fold warp of both CTAs
// arrives on the first CTA's "accumulator free" barrier.  Every wait is
// bounded.
// k-block depth: 64 fp16 (128-byte rows, 128-byte swizzle, 3 stages) or 32
// (64-byte rows and swizzle, 6 stages: the same ring bytes in finer steps).
#ifndef HS_P_BK
#define HS_P_BK 64
#endif
constexpr int P_BK = HS_P_BK;
static_assert(P_BK == 64 || P_BK == 32, "pair k-block depth");
constexpr int P_ROWB = P_BK * 2;                     // bytes per operand row (K-major)
constexpr int P_TILE = 128 * P_BK * 2;               // bytes per operand part per CTA
constexpr int P_STAGE = 4 * P_TILE;                  // Ah, Al, Bh, Bl
constexpr int P_STAGES = P_BK == 64 ? 3 : 6;
constexpr int P_PROMOTE = H3_PROMOTE * 64 / P_BK;    // same k per accumulator group
constexpr uint32_t P_LAYOUT = P_BK == 64 ? 2u : 4u;  // descriptor swizzle: 128 B or 64 B
constexpr uint32_t P_SBO = 8 * P_ROWB;               // 8-row core-matrix groups
// MN-major parts: boxes of P_BK M/N elements (one swizzle row) x P_BK k rows,
// 128 / P_BK of them side by side.
constexpr int P_MN_BOX = P_BK * P_BK * 2;
constexpr int P_MN_NBOX = 128 / P_BK;
constexpr int P_THREADS = 320;                       // producer, MMA, 8 fold/epilogue warps
constexpr int P_SMEM = P_STAGES * P_STAGE + 2 * H3_EPI + 1024 + 256;
static_assert(P_SMEM <= 232448, "shared memory per block");
constexpr int P_BM = 256, P_BN = 256;                // pair tile
constexpr uint32_t P_ACC_COLS = 256;                 // one accumulator buffer
// bf16 variant (BF): the operands are bf16 themselves, whose products are
// exact in one kind::f16 MMA with bf16 inputs, so a stage holds A and B only
// (twice the stages in the same ring), one MMA per k-step, no operand
// scales; accumulator groups of 8 k-blocks (512 k) bound the tensor core's
// truncating accumulation to ~2e-5 relative per group before the fp32 fold.
constexpr int P_PROMOTE_BF = 8 * 64 / P_BK;
static_assert(2 * P_STAGES * 2 * P_TILE == P_STAGES * P_STAGE, "bf16 ring reuses the split ring's bytes");


// BF: bf16 operands in tmAh / tmBh (tmAl, tmBl unused), one product.
template <bool A_MN, bool B_MN, bool BF = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
gemm_h3_pair_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                    const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                    const __grid_constant__ CUtensorMap tmC, TcArgs p, const unsigned *absmax_a,
                    const unsigned *absmax_b, int mtiles, int ntiles, int ntiles_total) {
  constexpr int NSTG = BF ? 2 * P_STAGES : P_STAGES;     // ring stages
  constexpr int SBYTES = BF ? 2 * P_TILE : P_STAGE;      // bytes per stage per CTA
  constexpr int PROM = BF ? P_PROMOTE_BF : P_PROMOTE;    // k-blocks per accumulator group
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *epi = reinterpret_cast<float *>(smem + NSTG * SBYTES);  // two 16 KB boxes
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + NSTG * SBYTES + 2 * H3_EPI);
  uint64_t *empty = full + NSTG;
  uint64_t *pfull = empty + NSTG;
  uint64_t *pempty = pfull + 2;
  uint64_t *mdone = pempty + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(mdone + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  auto tile_of = [&](int tl, int64_t &m0, int64_t &n0, int &z, int &nk) {
    const int per = mtiles * ntiles;
    z = tl / per;
    const int rem = tl - z * per;
    m0 = (int64_t)(rem / ntiles) * P_BM;
    n0 = (int64_t)(rem % ntiles) * P_BN;
    const int kb0 = z * p.kb_per_split;
    nk = min(p.nkb, kb0 + p.kb_per_split) - kb0;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTG; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 16);  // 8 fold warps x 2 CTAs (used in the first CTA)
    }
    mbar_init(mdone, 1);
    *abort_flag = ld_status(p.status) != 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // barriers and TMEM of both CTAs ready before any cross-CTA use
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  const bool skip = *abort_flag != 0;

  if (!skip && warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (lane == 0) {
      int it = 0, issued = 0;
      bool ok = true;
      for (int tl = pair; tl < ntiles_total && ok; tl += npairs) {
        int64_t m0, n0;
        int z, nk;
        tile_of(tl, m0, n0, z, nk);
        const int mr = (int)m0 + 128 * (int)rank, nr = (int)n0 + 128 * (int)rank;
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % NSTG;
          const uint32_t ph = (it / NSTG) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status)) { ok = false; break; }
          // pass a real release (not the first use of a stage) on to the
          // second CTA first, so that its loads start with this CTA's
          if (rank == 0 && it >= NSTG) mbar_arrive_cluster(cluster_addr(&empty[s], 1));
          const uint32_t fb = cluster_addr(&full[s], 0);
          unsigned char *st = smem + s * SBYTES;
          if (rank == 0) mbar_expect_tx(&full[s], 2 * SBYTES);  // both CTAs' bytes
          const int k0 = (z * p.kb_per_split + i) * P_BK;
          if (BF) {
            // A then B, one part each
            if (A_MN) {
#pragma unroll
              for (int j = 0; j < P_MN_NBOX; ++j) tma_2d_pair(st + j * P_MN_BOX, &tmAh, fb, mr + P_BK * j, k0);
            } else {
              tma_2d_pair(st, &tmAh, fb, k0, mr);
            }
            if (B_MN) {
#pragma unroll
              for (int j = 0; j < P_MN_NBOX; ++j)
                tma_2d_pair(st + P_TILE + j * P_MN_BOX, &tmBh, fb, nr + P_BK * j, k0);
            } else {
              tma_2d_pair(st + P_TILE, &tmBh, fb, k0, nr);
            }
            ++issued;
            continue;
          }
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < P_MN_NBOX; ++j) {
              tma_2d_pair(st + j * P_MN_BOX, &tmAh, fb, mr + P_BK * j, k0);
              tma_2d_pair(st + P_TILE + j * P_MN_BOX, &tmAl, fb, mr + P_BK * j, k0);
            }
          } else {
            tma_2d_pair(st, &tmAh, fb, k0, mr);
            tma_2d_pair(st + P_TILE, &tmAl, fb, k0, mr);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < P_MN_NBOX; ++j) {
              tma_2d_pair(st + 2 * P_TILE + j * P_MN_BOX, &tmBh, fb, nr + P_BK * j, k0);
              tma_2d_pair(st + 3 * P_TILE + j * P_MN_BOX, &tmBl, fb, nr + P_BK * j, k0);
            }
          } else {
            tma_2d_pair(st + 2 * P_TILE, &tmBh, fb, k0, nr);
            tma_2d_pair(st + 3 * P_TILE, &tmBl, fb, k0, nr);
          }
          ++issued;
        }
      }
      // The first CTA's barrier counts both CTAs' bytes: never leave while a
      // copy into either CTA's shared memory is in flight.
      if (rank == 0) {
        for (int j = std::max(0, issued - NSTG); j < issued; ++j) {
          if (ld_status(p.status)) mbar_drain(&full[j % NSTG], (j / NSTG) & 1);
          else (void)mbar_wait(&full[j % NSTG], (j / NSTG) & 1, p.status);
        }
      }
    }
  } else if (!skip && warp == 1) {
    // ---------------- MMA issuer (first CTA only)
    if (rank == 0 && lane == 0) {
      // bf16: A and B format fields (bits 7-9, 10-12) = 1; fp16 is 0
      constexpr uint32_t idesc = idesc_f16(P_BM, P_BN) | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16) |
                                 (BF ? ((1u << 7) | (1u << 10)) : 0u);
      int it = 0, gg = 0;
      bool ok = true;
      for (int tl = pair; tl < ntiles_total && ok; tl += npairs) {
        int64_t m0, n0;
        int z, nk;
        tile_of(tl, m0, n0, z, nk);
        for (int i = 0; i < nk; ++i, ++it) {
          const int s = it % NSTG;
          const uint32_t ph = (it / NSTG) & 1;
          const bool gstart = (i % PROM) == 0;
          const int b = gg & 1;
          if (gstart && !mbar_wait(&pempty[b], ((gg >> 1) & 1) ^ 1, p.status)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, p.status)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t ah = su32(smem + s * SBYTES);
          const uint32_t al = ah + P_TILE, bh = ah + (BF ? 1 : 2) * P_TILE, bl = ah + 3 * P_TILE;
          const uint32_t t_acc = tmem + (uint32_t)(b * P_ACC_COLS);
#pragma unroll
          for (int kk = 0; kk < P_BK / 16; ++kk) {
            // K-major: 16 fp16 = 32 bytes into each row; MN-major: the next 16
            // k rows; LBO = one box between M/N blocks.
            const uint32_t oa = A_MN ? kk * 16 * P_ROWB : kk * 32, ob = B_MN ? kk * 16 * P_ROWB : kk * 32;
            const uint32_t la = A_MN ? P_MN_BOX : 16, lb = B_MN ? P_MN_BOX : 16;
            const uint64_t dAh = sdesc(ah + oa, la, P_SBO, P_LAYOUT), dAl = sdesc(al + oa, la, P_SBO, P_LAYOUT);
            const uint64_t dBh = sdesc(bh + ob, lb, P_SBO, P_LAYOUT), dBl = sdesc(bl + ob, lb, P_SBO, P_LAYOUT);
            const uint32_t acc = (gstart && kk == 0) ? 0u : 1u;
            mma_f16_pair(t_acc, dAh, dBh, idesc, acc);
            if (!BF) {
              mma_f16_pair(t_acc, dAh, dBl, idesc, 1u);
              mma_f16_pair(t_acc, dAl, dBh, idesc, 1u);
            }
          }
          mma_commit_pair(&empty[s]);
          if ((i % PROM) == PROM - 1 || i == nk - 1) {
            mma_commit_pair(&pfull[b]);
            ++gg;
          }
        }
      }
      // all issued MMAs complete before the CTAs may leave
      mma_commit_pair(mdone);
      if (ld_status(p.status)) mbar_drain(mdone, 0);
      else (void)mbar_wait(mdone, 0, p.status);
    }
  } else if (!skip) {
    // ---------------- fold finished groups, epilogue per tile (both CTAs)
    const int e = warp - 2;            // 0..7
    const int half = e >> 2;           // 128-column half of the tile
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int t = (e & 3) * 32 + lane;  // 0..127 within the half's group
    // Undo the two operand scales one at a time: each inverse is an exact
    // power of two within float range, their product may not be (tiny
    // operands get scales up to 2^114 each).
    const float inv_a = BF ? 1.f : 1.0f / pow2_scale(*absmax_a), inv_b = BF ? 1.f : 1.0f / pow2_scale(*absmax_b);
    const uint32_t pe0 = cluster_addr(&pempty[0], 0), pe1 = cluster_addr(&pempty[1], 0);
    const uint32_t pf0 = cluster_addr(&pfull[0], 1), pf1 = cluster_addr(&pfull[1], 1);
    int gg = 0;
    bool ok = true;
    for (int tl = pair; tl < ntiles_total && ok; tl += npairs) {
      int64_t m0, n0;
      int z, nk;
      tile_of(tl, m0, n0, z, nk);
      const int ngroups = (nk + PROM - 1) / PROM;
      float tot[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) tot[j] = 0.f;
      for (int g = 0; g < ngroups; ++g, ++gg) {
        const int b = gg & 1;
        if (!mbar_wait(&pfull[b], (gg >> 1) & 1, p.status)) { ok = false; break; }
        if (rank == 0 && e == 0 && lane == 0) mbar_arrive_cluster(b ? pf1 : pf0);  // tell the second CTA
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t base =
            tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * P_ACC_COLS) + (uint32_t)(half * BN);
#pragma unroll
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(base + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) tot[c + j] += v[j];
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(b ? pe1 : pe0);
      }
      if (!ok) break;
#pragma unroll
      for (int j = 0; j < BN; ++j) tot[j] = (tot[j] * inv_a) * inv_b;
      if (BF && p.out_bf16)
        store_tile_boxes_bf16(tot, epi + half * (H3_EPI / 4), &tmC, p, q, lane, t, m0 + 128 * (int64_t)rank,
                              n0 + (int64_t)half * BN, 1 + half);
      else
        store_tile_boxes(tot, epi + half * (H3_EPI / 4), &tmC, p, q, lane, t, m0 + 128 * (int64_t)rank,
                         n0 + (int64_t)half * BN, p.partial ? z : 0, 1 + half);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  __syncthreads();
  cluster_sync_all();  // neither CTA frees TMEM or leaves while the pair's work may touch it
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// C[m,n] = beta*C + sum_z partial[z][m][n] (+ bias[n]); fixed order over z.
__global__ void splitk_reduce_kernel(const float *__restrict__ part, float *__restrict__ C,
                                     const float *__restrict__ bias, int64_t M, int64_t N,
                                     int64_t ldc, int splits, int beta) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= M * N) return;
  const int64_t m = idx / N, n = idx % N;
  float s = 0.f;
  for (int z = 0; z < splits; ++z) s += part[(int64_t)z * M * N + idx];
  if (bias) s += bias[n];
  float *c = C + m * ldc + n;
  *c = beta ? *c + s : s;
}

// ---------------------------------------------------------------- host side

// Output map: C [splits][M][N] fp32 with row stride ld; 32-column x 128-row
// boxes, 128-byte swizzle (matches the epilogue's shared-memory staging).
// bf16 output [M][ld]: 3D {N, M, 1}, box {64, 128, 1} (128-byte rows).
bool make_out_map_bf16(CUtensorMap *tm, void *ptr, int64_t M, int64_t N, int64_t ld) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, 1};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(ld * M * 2)};
  cuuint32_t box[3] = {64, (cuuint32_t)BM, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ptr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_out_map(CUtensorMap *tm, float *ptr, int64_t splits, int64_t M, int64_t N, int64_t ld) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)splits};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(ld * M * 4)};
  cuuint32_t box[3] = {32, (cuuint32_t)BM, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)ptr, dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Operand view: element (r, k) of an R x K operand (R = M for A, N for B).
//   K-major:  ptr[r*ld + k]   -> 2D map {K, R}, box {32, rows}
//   MN-major: ptr[k*ld + r]   -> 2D map {R, K}, box {32, 32}
bool make_map(CUtensorMap *tm, const float *ptr, int64_t R, int64_t K, int64_t ld, bool mn, int rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  CUresult r;
  if (!mn) {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)R};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)rows};
    cuuint32_t es[2] = {1, 1};
    r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)ptr, dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    (void)rows;
    cuuint64_t dims[2] = {(cuuint64_t)R, (cuuint64_t)K};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t es[2] = {1, 1};
    r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)ptr, dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r == CUDA_SUCCESS;
}

// HS_TC_TMEM_A=0 runs K-major-A products on the shared-memory-A kernel
// (cross-checks of the two tensor-core kernels).
bool tmem_a_enabled() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("HS_TC_TMEM_A");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

int g_disable = -1;  // HS_DISABLE_TC=1 forces the FFMA path (cross-checks)

bool tc_enabled() {
  if (g_disable < 0) {
    const char *e = getenv("HS_DISABLE_TC");
    g_disable = (e && e[0] == '1') ? 1 : 0;
  }
  return g_disable == 0;
}

// Smallest M*N*K the tensor-core path takes (HS_TC_MIN_MNK overrides, for
// exercising the tensor-core path on small shapes in tests).
double tc_min_mnk() {
  static double v = -1;
  if (v < 0) {
    const char *e = getenv("HS_TC_MIN_MNK");
    v = e ? atof(e) : 3.3e7;
  }
  return v;
}

int device_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

struct TcPlan {
  bool ok = false;
  int splits = 1;
  int nkb = 0;
  int kbps = 0;
  size_t ws = 0;
};

int split_count(int64_t M, int64_t N, int nkb, int nsm) {
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  int splits = 1;
  if (tiles < nsm / 2 && nkb >= 16) splits = (int)std::max<int64_t>(1, std::min<int64_t>(nsm / tiles, nkb / 8));
  const int kbps = (nkb + splits - 1) / splits;
  return (nkb + kbps - 1) / kbps;
}

TcPlan plan_tc(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, int64_t lda,
               int64_t ldb, int64_t ldc, bool a_kc, bool b_kc) {
  TcPlan pl;
  if (!tc_enabled()) return pl;
  if ((double)M * N * K < tc_min_mnk()) return pl;  // small products: FFMA path
  auto al = [](const void *p) { return aligned(p, 16); };
  if (!al(A) || !al(B) || !al(C) || lda % 4 || ldb % 4 || ldc % 4 || N % 4) return pl;
  if (a_kc ? (K % 4) : (M % 4)) return pl;
  if (b_kc ? (K % 4) : (N % 4)) return pl;
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return pl;
  pl.nkb = (int)((K + BK - 1) / BK);
  pl.splits = split_count(M, N, pl.nkb, device_sms());
  pl.kbps = (pl.nkb + pl.splits - 1) / pl.splits;  // every split gets >= 1 k-block
  pl.ws = pl.splits > 1 ? (size_t)pl.splits * M * N * 4 : 0;
  pl.ok = true;
  return pl;
}

// ---------------------------------------------------------------- 3 x fp16 host side
bool h3_enabled() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("HS_TC_F16");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}
int64_t round8(int64_t x) { return (x + 7) / 8 * 8; }
// absmax words (256 B), then Ah, Al [M][K8] and Bh, Bl [N][K8] fp16
size_t h3_scratch(int64_t M, int64_t N, int64_t K) {
  return 256 + round_up((size_t)2 * M * round8(K) * 2, 256) + round_up((size_t)2 * N * round8(K) * 2, 256);
}
int h3_splits(int64_t M, int64_t N, int64_t K, int nsm) {
  return split_count(M, N, (int)((round8(K) + H3_BK - 1) / H3_BK), nsm);
}
// 2-SM pair path (HS_H3_PAIR=0 turns it off).
bool h3_pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("HS_H3_PAIR");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}
constexpr int kPairMaxSplits = 16;
// Split-K count for pair tiles: none when the tiles fill the pairs; else the
// smallest count whose work units fill whole waves of the pairs to >= 90%
// (the best one if none does), each split keeping >= 8 k-blocks.
int pair_split_count(int64_t tiles, int nkb, int npairs) {
  if (tiles >= npairs || nkb < 16) return 1;
  const int smax = std::max(1, std::min(kPairMaxSplits, nkb / 8));
  int best = 1;
  double best_eff = 0.0;
  for (int sp = 1; sp <= smax; ++sp) {
    const int64_t units = tiles * sp;
    const int64_t waves = (units + npairs - 1) / npairs;
    const double eff = (double)units / (double)(waves * npairs);
    if (eff >= 0.9) { best = sp; break; }
    if (eff > best_eff + 1e-9) { best_eff = eff; best = sp; }
  }
  const int kbps = (nkb + best - 1) / best;
  return (nkb + kbps - 1) / kbps;
}
size_t h3_partial_bound(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int sp = h3_splits(M, N, K, 256);
  size_t b = sp > 1 ? (size_t)sp * M * N * 4 : 0;
  const int nkb = (int)((round8(K) + P_BK - 1) / P_BK);
  const int64_t ptiles = ((M + P_BM - 1) / P_BM) * ((N + P_BN - 1) / P_BN);
  if (ptiles < 128 && nkb >= 16)  // any pair count up to 128 (256 SMs)
    b = std::max(b, (size_t)std::min(kPairMaxSplits, std::max(1, nkb / 8)) * M * N * 4);
  return b;
}
// Map of a split operand stored [rows][ld] fp16.  K-major use (rows = M or
// N, columns = K): box {64 k, 128 rows}.  MN-major use (rows = K, columns =
// M or N): box {64 columns, 64 k rows}.
bool make_map_f16(CUtensorMap *tm, const __half *ptr, int64_t rows, int64_t ld, bool mn) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {H3_BK, mn ? 64u : (cuuint32_t)BM};
  cuuint32_t es[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)ptr, dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The pair kernel's maps: K-major box {P_BK k, 128 rows}, MN-major box
// {P_BK columns, P_BK k rows}, swizzled to the row width (128 or 64 bytes);
// fp16 elements, or bf16 (bf).
bool make_map_f16_pair(CUtensorMap *tm, const void *ptr, int64_t rows, int64_t ld, bool mn, bool bf = false) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)P_BK, mn ? (cuuint32_t)P_BK : 128u};
  cuuint32_t es[2] = {1, 1};
  return enc(tm, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)ptr, dims,
             strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, P_BK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t h3_split_bytes(int64_t rows, int64_t cols) { return round_up((size_t)4 * rows * round8(cols), 256); }

// hi/lo fp16 [rows][round8(cols)] of a float32 [rows][ld] matrix, scaled by
// the power of two its absmax selects; *absmax (in device memory) is written.
int h3_split(const float *x, int64_t rows, int64_t cols, int64_t ld, unsigned *absmax, void *dst,
             cudaStream_t st) {
  const int nsm = device_sms();
  const int64_t ldo = round8(cols);
  __half *hi = static_cast<__half *>(dst);
  __half *lo = hi + rows * ldo;
  if (cudaMemsetAsync(absmax, 0, 4, st) != cudaSuccess) return check_launch("h3 memset");
  const int grid = (int)std::min<int64_t>(8 * nsm, (rows + 7) / 8);
  absmax_kernel<<<grid, 256, 0, st>>>(x, rows, cols, ld, absmax);
  if (int e = check_launch("absmax_kernel")) return e;
  split_h2_kernel<<<grid, 256, 0, st>>>(x, rows, cols, ld, absmax, hi, lo, ldo);
  return check_launch("split_h2_kernel");
}

// The same split with *absmax already known: an upper bound of max |x| as
// float bits (the exact maximum keeps the most precision; anything below it
// overflows fp16).
// gate (device memory, may be null): the split runs only if *gate != 0.
int h3_split_known(const float *x, int64_t rows, int64_t cols, int64_t ld, const unsigned *absmax, void *dst,
                   cudaStream_t st, const int *gate) {
  const int nsm = device_sms();
  const int64_t ldo = round8(cols);
  __half *hi = static_cast<__half *>(dst);
  __half *lo = hi + rows * ldo;
  const int grid = (int)std::min<int64_t>(8 * nsm, (rows + 7) / 8);
  split_h2_kernel<<<grid, 256, 0, st>>>(x, rows, cols, ld, absmax, hi, lo, ldo, gate);
  return check_launch("split_h2_kernel");
}

// *out = max |x| over a [rows][cols] float32 matrix with row stride ld, as
// float bits (NaN ignored).
int absmax_rows(const float *x, int64_t rows, int64_t cols, int64_t ld, unsigned *out, cudaStream_t st) {
  if (cudaMemsetAsync(out, 0, 4, st) != cudaSuccess) return check_launch("absmax memset");
  const int grid = (int)std::min<int64_t>(8 * device_sms(), (rows + 7) / 8);
  absmax_kernel<<<grid, 256, 0, st>>>(x, rows, cols, ld, out);
  return check_launch("absmax_kernel");
}

// Largest number of pairs (clusters of two CTAs) of this kernel variant
// resident at once on the current device; 0 if none.
int pair_capacity(const void *fn, int variant) {
  static std::atomic<int> cached[64][8];
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int> &c = cached[dev & 63][variant & 7];
  int v = c.load(std::memory_order_relaxed);
  if (v > 0) return v - 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)device_sms(), 1, 1);
  cfg.blockDim = dim3(P_THREADS, 1, 1);
  cfg.dynamicSmemBytes = P_SMEM;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  c.store(n + 1, std::memory_order_relaxed);
  return n;
}

using PairFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                       const CUtensorMap, TcArgs, const unsigned *, const unsigned *, int, int, int);

template <bool BF>
PairFn pair_fn(bool a_mn, bool b_mn) {
  if (a_mn) return b_mn ? gemm_h3_pair_kernel<true, true, BF> : gemm_h3_pair_kernel<true, false, BF>;
  return b_mn ? gemm_h3_pair_kernel<false, true, BF> : gemm_h3_pair_kernel<false, false, BF>;
}

// The pair kernel on encoded operand maps (tal, tbl unused when bf); *done =
// false if it does not apply (no pair fits, or a split-K partial would not
// fit ws).
// c_bf16 (bf operands only): C is bf16, written without split-K or beta.
static int pair_run(bool bf, const CUtensorMap &tah, const CUtensorMap &tal, const CUtensorMap &tbh, const CUtensorMap &tbl,
             bool a_mn, bool b_mn, const unsigned *a_absmax, const unsigned *b_absmax, void *Cv, const float *bias,
             int64_t M, int64_t N, int64_t K, int64_t ldc, int beta, void *ws, size_t ws_bytes, int *status,
             cudaStream_t st, bool *done, bool c_bf16 = false) {
  *done = false;
  if (c_bf16 && (!bf || beta)) return HS_OK;
  float *C = static_cast<float *>(Cv);
  const PairFn fn = bf ? pair_fn<true>(a_mn, b_mn) : pair_fn<false>(a_mn, b_mn);
  const int variant = (bf ? 4 : 0) + (a_mn ? 2 : 0) + (b_mn ? 1 : 0);
  static std::atomic<unsigned long long> attr_set[8];
  if (int e = allow_dynamic_smem((const void *)fn, P_SMEM, &attr_set[variant])) return e;
  const int npairs = pair_capacity((const void *)fn, variant);
  if (npairs < 1) return HS_OK;
  const int nkb = (int)((round8(K) + P_BK - 1) / P_BK);
  const int64_t mt = (M + P_BM - 1) / P_BM, nt = (N + P_BN - 1) / P_BN;
  int splits = c_bf16 ? 1 : pair_split_count(mt * nt, nkb, npairs);
  if (splits > 1 && (!ws || !aligned(ws, 256) || ws_bytes < (size_t)splits * M * N * 4)) splits = 1;
  const int kbps = (nkb + splits - 1) / splits;
  splits = (nkb + kbps - 1) / kbps;
  float *partial = splits > 1 ? static_cast<float *>(ws) : nullptr;
  CUtensorMap tc;
  if (c_bf16 ? !make_out_map_bf16(&tc, Cv, M, N, ldc)
             : !make_out_map(&tc, splits > 1 ? partial : C, splits, M, N, splits > 1 ? N : ldc))
    return HS_OK;
  const int64_t ntot = mt * nt * splits;
  if (ntot >= (1ll << 30)) return HS_OK;
  const unsigned grid = 2u * (unsigned)std::min<int64_t>(ntot, npairs);
  TcArgs args;
  args.out_bf16 = c_bf16 ? 1 : 0;
  args.C = C;
  args.bias = bias;
  args.partial = partial;
  args.M = M;
  args.N = N;
  args.K = K;
  args.ldc = ldc;
  args.beta = beta;
  args.kb_per_split = kbps;
  args.nkb = nkb;
  args.status = status;
  fn<<<grid, P_THREADS, P_SMEM, st>>>(tah, tal, tbh, tbl, tc, args, a_absmax, b_absmax, (int)mt, (int)nt, (int)ntot);
  if (int e = check_launch("gemm_h3_pair_kernel")) return e;
  if (splits > 1) {
    const int64_t n = M * N;
    splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(partial, C, bias, M, N, ldc, splits, beta);
    if (int e = check_launch("splitk_reduce_kernel")) return e;
  }
  *done = true;
  return HS_OK;
}

// The pair kernel on the fp16 split operands.
int gemm_h3_pair(const __half *ah, const __half *al, int64_t a_rows, int64_t a_ld, bool a_mn, const __half *bh,
                 const __half *bl, int64_t b_rows, int64_t b_ld, bool b_mn, const unsigned *a_absmax,
                 const unsigned *b_absmax, float *C, const float *bias, int64_t M, int64_t N, int64_t K, int64_t ldc,
                 int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st, bool *done) {
  *done = false;
  CUtensorMap tah, tal, tbh, tbl;
  if (!make_map_f16_pair(&tah, ah, a_rows, a_ld, a_mn) || !make_map_f16_pair(&tal, al, a_rows, a_ld, a_mn) ||
      !make_map_f16_pair(&tbh, bh, b_rows, b_ld, b_mn) || !make_map_f16_pair(&tbl, bl, b_rows, b_ld, b_mn))
    return HS_OK;
  return pair_run(false, tah, tal, tbh, tbl, a_mn, b_mn, a_absmax, b_absmax, C, bias, M, N, K, ldc, beta, ws,
                  ws_bytes, status, st, done);
}

// C[M,N] = A.B^T over K (+bias, beta) from split operands.  A is stored
// [M][.] (a_mn false, K-major) or [K][.] (a_mn true); B likewise with N.
// Scratch (split-K partials, if any) from ws; *done = false if the shape or
// the scratch does not suit (the caller then takes another path).
int gemm_h3_presplit(const void *a_split, const unsigned *a_absmax, bool a_mn, const void *b_split,
                     const unsigned *b_absmax, bool b_mn, float *C, const float *bias, int64_t M, int64_t N,
                     int64_t K, int64_t ldc, int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st,
                     bool *done) {
  *done = false;
  if (!status || M <= 0 || N <= 0 || K <= 0) return HS_OK;
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return HS_OK;
  if (!aligned(C, 16) || ldc % 4 || N % 4) return HS_OK;
  const int nsm = device_sms();
  const int64_t K8 = round8(K), M8 = round8(M), N8 = round8(N);
  int splits = split_count(M, N, (int)((K8 + H3_BK - 1) / H3_BK), nsm);
  if (splits > 1 && (!ws || !aligned(ws, 256) || ws_bytes < (size_t)splits * M * N * 4)) splits = 1;
  const __half *ah = static_cast<const __half *>(a_split);
  const __half *bh = static_cast<const __half *>(b_split);
  const int64_t a_rows = a_mn ? K : M, a_ld = a_mn ? M8 : K8;
  const int64_t b_rows = b_mn ? K : N, b_ld = b_mn ? N8 : K8;
  const __half *al = ah + a_rows * a_ld;
  const __half *bl = bh + b_rows * b_ld;
  CUtensorMap tah, tal, tbh, tbl, tc;
  if (!make_map_f16(&tah, ah, a_rows, a_ld, a_mn) || !make_map_f16(&tal, al, a_rows, a_ld, a_mn) ||
      !make_map_f16(&tbh, bh, b_rows, b_ld, b_mn) || !make_map_f16(&tbl, bl, b_rows, b_ld, b_mn))
    return HS_OK;
  if (h3_pair_enabled()) {
    bool pdone = false;
    if (int e = gemm_h3_pair(ah, al, a_rows, a_ld, a_mn, bh, bl, b_rows, b_ld, b_mn, a_absmax, b_absmax, C, bias, M,
                             N, K, ldc, beta, ws, ws_bytes, status, st, &pdone))
      return e;
    if (pdone) {
      *done = true;
      return HS_OK;
    }
  }
  float *partial = splits > 1 ? static_cast<float *>(ws) : nullptr;
  if (!make_out_map(&tc, splits > 1 ? partial : C, splits, M, N, splits > 1 ? N : ldc)) return HS_OK;
  const int nkb = (int)((K8 + H3_BK - 1) / H3_BK);
  const int kbps = (nkb + splits - 1) / splits;
  splits = (nkb + kbps - 1) / kbps;
  const int64_t mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
  const int64_t ntot = mt * nt * splits;
  if (ntot >= (1ll << 31)) return HS_OK;
  const unsigned grid = (unsigned)std::min<int64_t>(ntot, nsm);
  TcArgs args;
  args.C = C;
  args.bias = bias;
  args.partial = partial;
  args.M = M;
  args.N = N;
  args.K = K;
  args.ldc = ldc;
  args.beta = beta;
  args.kb_per_split = kbps;
  args.nkb = nkb;
  args.status = status;
  void (*fn)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, TcArgs,
             const unsigned *, const unsigned *, int, int, int);
  if (a_mn) fn = b_mn ? gemm_h3_kernel<true, true> : gemm_h3_kernel<true, false>;
  else fn = b_mn ? gemm_h3_kernel<false, true> : gemm_h3_kernel<false, false>;
  static std::atomic<unsigned long long> attr_set[4];
  if (int e = allow_dynamic_smem((const void *)fn, H3_SMEM_P, &attr_set[(a_mn ? 2 : 0) + (b_mn ? 1 : 0)])) return e;
  fn<<<grid, H3_THREADS, H3_SMEM_P, st>>>(tah, tal, tbh, tbl, tc, args, a_absmax, b_absmax, (int)mt, (int)nt,
                                           (int)ntot);
  if (int e = check_launch("gemm_h3_kernel")) return e;
  if (splits > 1) {
    const int64_t n = M * N;
    splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(partial, C, bias, M, N, ldc, splits, beta);
    if (int e = check_launch("splitk_reduce_kernel")) return e;
  }
  *done = true;
  return HS_OK;
}

// C[M,N] = A.B^T over K (+bias, beta) from bf16 operands, one bf16 MMA per
// k-step on SM pairs.  A is stored [M][a_ld] (a_mn false, K-major) or
// [K][a_ld] (a_mn true, M-major); B likewise with N.  Leading dimensions
// must be multiples of 8 elements (16-byte TMA strides) and the operands
// 16-byte aligned; *done = false if the shape, the alignment or the scratch
// (split-K partials) does not suit.
// c_bf16: C is bf16 [M][ldc] (ldc, N multiples of 8; beta 0), else float32.
int gemm_bf16(const void *a, int64_t a_ld, bool a_mn, const void *b, int64_t b_ld, bool b_mn, void *C,
              const float *bias, int64_t M, int64_t N, int64_t K, int64_t ldc, int beta, void *ws, size_t ws_bytes,
              int *status, cudaStream_t st, bool *done, bool c_bf16) {
  *done = false;
  if (!tc_enabled() || !status || M <= 0 || N <= 0 || K <= 0) return HS_OK;
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return HS_OK;
  if (!aligned(C, 16) || ldc % 4 || N % 4 || !aligned(a, 16) || !aligned(b, 16) || a_ld % 8 || b_ld % 8) return HS_OK;
  if (c_bf16 && (ldc % 8 || N % 8 || beta)) return HS_OK;
  if (a_ld < (a_mn ? M : K) || b_ld < (b_mn ? N : K)) return HS_OK;
  CUtensorMap ta, tb;
  if (!make_map_f16_pair(&ta, a, a_mn ? K : M, a_ld, a_mn, true) ||
      !make_map_f16_pair(&tb, b, b_mn ? K : N, b_ld, b_mn, true))
    return HS_OK;
  return pair_run(true, ta, ta, tb, tb, a_mn, b_mn, nullptr, nullptr, C, bias, M, N, K, ldc, beta, ws, ws_bytes,
                  status, st, done, c_bf16);
}

// Split-K partial scratch the bf16 pair GEMM may use for an M x N product over K.
size_t gemm_bf16_partial_bound(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int nkb = (int)((round8(K) + P_BK - 1) / P_BK);
  const int64_t ptiles = ((M + P_BM - 1) / P_BM) * ((N + P_BN - 1) / P_BN);
  if (ptiles >= 128 || nkb < 16) return 0;
  return (size_t)std::min(kPairMaxSplits, std::max(1, nkb / 8)) * M * N * 4;
}

namespace {

// K-major product from float32 operands: split both into ws, then multiply.
int gemm_h3_try(const float *A, const float *B, float *C, const float *bias, int64_t M, int64_t N, int64_t K,
                int64_t lda, int64_t ldb, int64_t ldc, int beta, void *ws, size_t ws_bytes, int *status,
                cudaStream_t st, bool *done) {
  *done = false;
  const size_t scratch = h3_scratch(M, N, K);
  if (!ws || !aligned(ws, 256) || ws_bytes < scratch) return HS_OK;
  char *w = static_cast<char *>(ws);
  unsigned *absmax = reinterpret_cast<unsigned *>(w);
  void *as = w + 256;
  void *bs = w + 256 + h3_split_bytes(M, K);
  if (int e = h3_split(A, M, K, lda, absmax, as, st)) return e;
  if (int e = h3_split(B, N, K, ldb, absmax + 1, bs, st)) return e;
  return gemm_h3_presplit(as, absmax, false, bs, absmax + 1, false, C, bias, M, N, K, ldc, beta, w + scratch,
                          ws_bytes - scratch, status, st, done);
}

}  // namespace

bool gemm_h3_enabled() { return tc_enabled() && h3_enabled(); }
bool gemm_tc_size_ok(int64_t M, int64_t N, int64_t K) { return (double)M * N * K >= tc_min_mnk(); }
size_t gemm_h3_partial_bound(int64_t M, int64_t N, int64_t K) { return h3_partial_bound(M, N, K); }

size_t gemm_tc_workspace(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K,
                         int64_t lda, int64_t ldb, int64_t ldc, bool a_kc, bool b_kc) {
  TcPlan pl = plan_tc(A, B, C, M, N, K, lda, ldb, ldc, a_kc, b_kc);
  return pl.ok ? pl.ws : 0;
}

// Upper bound of the scratch of one M x N x K product on any device with up
// to 256 SMs (the split count only grows with the SM count): split-K
// partials, and for products with both operands K-major the fp16 split.
size_t gemm_tc_workspace_bound(int64_t M, int64_t N, int64_t K, bool kmajor_both) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int splits = split_count(M, N, (int)((K + BK - 1) / BK), 256);
  const size_t partial = splits > 1 ? (size_t)splits * M * N * 4 : 0;
  if (!kmajor_both) return partial;
  return std::max(partial, h3_scratch(M, N, K) + h3_partial_bound(M, N, K));
}

int gemm_tc_try(const float *A, const float *B, float *C, const float *bias, int64_t M, int64_t N,
                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, bool a_kc, bool b_kc, int beta,
                void *ws, size_t ws_bytes, int *status, cudaStream_t st, bool *done) {
  if (!status) return HS_OK;  // the tensor-core path needs a status word for its bounded waits
  *done = false;
  TcPlan pl = plan_tc(A, B, C, M, N, K, lda, ldb, ldc, a_kc, b_kc);
  if (!pl.ok) return HS_OK;
  if (a_kc && b_kc && h3_enabled()) {
    if (int e = gemm_h3_try(A, B, C, bias, M, N, K, lda, ldb, ldc, beta, ws, ws_bytes, status, st, done)) return e;
    if (*done) return HS_OK;
  }
  if (pl.splits > 1 && (!ws || ws_bytes < pl.ws || !aligned(ws, 16))) {
    // not enough scratch for split-K: run unsplit (fewer CTAs, still exact)
    pl.splits = 1;
    pl.kbps = pl.nkb;
    pl.ws = 0;
  }
  CUtensorMap ta, tb, tc;
  if (!make_map(&ta, A, M, K, lda, !a_kc, BM)) return HS_OK;
  if (!make_map(&tb, B, N, K, ldb, !b_kc, BN)) return HS_OK;
  float *cdst = pl.splits > 1 ? static_cast<float *>(ws) : C;
  if (!make_out_map(&tc, cdst, pl.splits, M, N, pl.splits > 1 ? N : ldc)) return HS_OK;
  TcArgs args;
  args.C = C;
  args.bias = bias;
  args.partial = pl.splits > 1 ? static_cast<float *>(ws) : nullptr;
  args.M = M;
  args.N = N;
  args.K = K;
  args.ldc = ldc;
  args.beta = beta;
  args.kb_per_split = pl.kbps;
  args.nkb = pl.nkb;
  args.status = status;
  const dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM), (unsigned)pl.splits);
  void (*fn)(const CUtensorMap, const CUtensorMap, const CUtensorMap, TcArgs);
  const bool tmem_a = a_kc && tmem_a_enabled();
  if (tmem_a) fn = b_kc ? gemm_ta_kernel<false> : gemm_ta_kernel<true>;
  else if (!a_kc && !b_kc) fn = gemm_tc_kernel<true, true>;
  else if (!a_kc) fn = gemm_tc_kernel<true, false>;
  else if (!b_kc) fn = gemm_tc_kernel<false, true>;
  else fn = gemm_tc_kernel<false, false>;
  const int smem_bytes = tmem_a ? TA_SMEM_BYTES : SMEM_BYTES;
  static std::atomic<unsigned long long> attr_set[6];
  const int which = tmem_a ? 4 + (b_kc ? 0 : 1) : (a_kc ? 0 : 2) + (b_kc ? 0 : 1);
  if (int e = allow_dynamic_smem((const void *)fn, smem_bytes, &attr_set[which])) return e;
  if (grid.y > 65535) return HS_OK;
  fn<<<grid, NTHREADS, smem_bytes, st>>>(ta, tb, tc, args);
  if (int e = check_launch("gemm_tc_kernel")) return e;
  if (pl.splits > 1) {
    const int64_t n = M * N;
    splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<float *>(ws), C, bias, M, N,
                                                                      ldc, pl.splits, beta);
    if (int e = check_launch("splitk_reduce_kernel")) return e;
  }
  *done = true;
  return HS_OK;
}

}  // namespace hs
