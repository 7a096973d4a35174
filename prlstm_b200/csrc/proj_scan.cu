// The input projection with the parallel-mode scan forward in its epilogue:
// one persistent kernel computes Z = x.W_ih^T + b_ih on the tensor cores
// (3 x fp16 split, 2-SM pairs, as the projection GEMM), and, per output
// tile, the gates, the cell-state recurrence c_t = f'_t c_{t-1} + (i g)'_t,
// out_t = o_t tanh(c_t), h_n, c_n and the backward's bound max c_{t-1}
// f'(1-f').  Z is still written once (the backward reads it), but it is
// never read back for the forward.
//
// Reference: the projection `linear(x, W_ih, b_ih)` followed by the gate
// activations and the Heinsen scan, src/headstartlstm/_parallel.py:38-74
// (log-domain scan restated as the clamped affine recurrence it computes,
// _parallel.py:21-35).
//
// Tiles.  A tile is one pair of CTAs: each CTA takes 128 consecutive time
// steps of ONE sequence (its TMA box runs along t with the sequence fixed:
// x is [T, B, D], the box {64 k, 1 b, 128 t}), the two CTAs of a pair take
// two sequences over the same steps, and both take the same block of 32
// hidden units: the 128 output columns are gates i, f (the first CTA's half
// of W_ih's rows) and g, o (the second's) of those units.  So every thread
// of the epilogue holds all four gates of its units for one time step: four
// quads of four warps split the block's 32 units, 8 per thread (32 values
// in registers, four warps per scheduler to hide each other's latency).
// Four TMEM accumulators of 128 columns let the MMAs run up to two tiles
// ahead of the epilogue.
//
// Chains.  (sequence pair, unit block) is a chain; its time tiles follow
// one another.  Tiles are numbered time-major, tile = tt * chains + chain,
// and dealt round-robin to the resident pairs, which keeps every pair busy
// (no chain is pinned to a pair).  A tile's carry-in (c just before its
// first step) comes from the chain's previous tile through global memory:
// per (sequence, unit) one 64-bit word holds the carry and the number of the
// tile it is for.  The tile it waits for has a smaller number, and
// every pair takes its tiles in increasing order, so the smallest unfinished
// tile can always proceed (the grid never exceeds the resident pairs).
// With chains >= pairs the tile waited for finished rounds earlier.
//
// The scan inside a tile: the epilogue threads (thread = time step) write
// each unit's f' and (i g)' into the staging buffers that the next store
// will use, unit-major; then a thread per (unit, segment of 8 steps) walks
// its 8 steps in order (the segment's map c -> A c + C), a 16-lane shuffle
// scan combines the unit's 16 segments, the last segment's thread hands the
// chain's carry in and out, every walker then produces c at its 8 steps
// (and the backward's bound), and the step threads read c back.  Every
// product of maps is of nonnegative terms (no cancellation).
//
// Every wait is bounded; a failed wait is made uniform across the 128
// threads of an epilogue quad by a reducing named barrier.  No cluster
// multicast.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>

#include "hs_common.cuh"
#include "tc_dev.cuh"

namespace hs {

// from gemm_tc.cu / capi.cu
size_t h3_split_bytes(int64_t rows, int64_t cols);
int h3_split(const float *x, int64_t rows, int64_t cols, int64_t ld, unsigned *absmax, void *dst, cudaStream_t st);
bool gemm_h3_enabled();
bool gemm_tc_size_ok(int64_t M, int64_t N, int64_t K);

namespace {

constexpr int PS_BK = 64;                        // fp16 k per block: one 128-byte row
constexpr int PS_TT = 128;                       // time steps per CTA tile (TMEM lanes)
constexpr int PS_UB = 32;                        // hidden units per chain
constexpr int PS_N = 4 * PS_UB;                  // output columns per pair tile (4 gates)
constexpr int PS_ATILE = PS_TT * PS_BK * 2;      // 16 KB: one A part (x hi or lo) per CTA
constexpr int PS_BGATE = PS_UB * PS_BK * 2;      // 4 KB: one gate's rows of one B part
constexpr int PS_BTILE = 2 * PS_BGATE;           // 8 KB: a CTA's half of one B part
constexpr int PS_STAGE = 2 * PS_ATILE + 2 * PS_BTILE;  // 48 KB: Ah, Al, Bh, Bl
constexpr int PS_STAGES = 3;
constexpr int PS_PROM = 4;                       // k-blocks per accumulator group
constexpr int PS_NACC = 4;                       // accumulator buffers (PS_N TMEM columns each)
constexpr int PS_NQ = 4;                         // epilogue quads (4 warps each)
constexpr int PS_QU = PS_UB / PS_NQ;             // units per quad
constexpr int PS_THREADS = 64 + PS_NQ * 128;     // producer, MMA, 16 epilogue warps
constexpr int PS_BOX = PS_TT * PS_QU * 4;        // 4 KB staging box (32-byte rows)
constexpr int PS_NBUF = 4;                       // staging boxes per quad
constexpr int PS_SMEM = PS_STAGES * PS_STAGE + PS_NQ * PS_NBUF * PS_BOX + 1024 + 256;
static_assert(PS_SMEM <= 232448, "shared memory per block");
static_assert(PS_QU == 8, "the epilogue's boxes and TMEM loads are 8 columns wide");
constexpr uint32_t PS_TMEM_COLS = PS_NACC * PS_N;  // 512
constexpr uint32_t PS_SBO = 8 * PS_BK * 2;       // 8-row core-matrix groups (1 KB)

struct PsArgs {
  const float *bias;            // b_ih [4H] or null
  const float *c0;              // [B][H] or null
  float *h_n, *c_n;             // [B][H] or null
  unsigned long long *slots;    // [B][H] chain carries: (tile tag << 32) | float bits (zeroed per call)
  unsigned *kf;                 // max c_{t-1} f'(1-f') as float bits, or null
  const unsigned *absmax_a;     // x's split scale word
  const unsigned *absmax_b;     // W_ih's split scale word
  int *status;
  int T, B, H;
  int nkb;                      // k-blocks over D
  int nub;                      // unit blocks, H / 32
  int nch;                      // chains, ceil(B / 2) * nub
  int ntt;                      // time tiles, ceil(T / 128)
  int ntiles;                   // ntt * nch
  float eps;
};

HS_DEV void tma_3d_pair(void *dst, const CUtensorMap *tm, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(su32(dst)),
      "l"(tm), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// Named barrier of the 128 threads of one epilogue quad that also ANDs a
// predicate over them: every thread leaves with the same answer.
HS_DEV bool named_and(int id, bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.s32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 128, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v), "r"(id)
      : "memory");
  return r != 0;
}

// Eight TMEM columns of this warp's 32 lanes, no wait: the registers are
// valid only after tmem_wait_ld below, which takes them as operands so that
// no use is scheduled ahead of it.
HS_DEV void tmem_ld8_nowait(uint32_t taddr, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
HS_DEV void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// A chain's carry: one 64-bit word per (sequence, unit) holding the value
// and the number of the time tile that follows it, written and read whole
// (single-copy atomic), so the value needs no fence or flag of its own.
HS_DEV void gslot_put(unsigned long long *s, unsigned tag, float v) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(s), "l"(w) : "memory");
}
// Waits (bounded) for tag in *s and returns its value in *v.
HS_DEV bool gslot_wait(const unsigned long long *s, unsigned tag, float *v, int *status) {
  uint64_t t0 = 0;
  for (unsigned n = 0;; ++n) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(s) : "memory");
    if ((unsigned)(w >> 32) == tag) {
      *v = __uint_as_float((unsigned)w);
      return true;
    }
    if ((n & 63u) == 63u) {
      if (t0 == 0) t0 = globaltimer();
      if (ld_status(status) != 0) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        set_status(status, HS_ERR_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
}

// Stage two 128-row x 8-column float boxes of this thread's row (v[OFF0 ..
// OFF0 + 7] and v[OFF1 .. OFF1 + 7]) in one of the quad's two pairs of
// staging buffers and store them with TMA at (n0, b, t0) and (n1, b, t0),
// one bulk group.  The pairs alternate (sp counts the quad's staged pairs):
// this pair is free on entry, and before the barrier that releases this
// pair's stores the issuer waits for the OTHER pair's stores (issued one
// stage of work earlier) to have read it, so the next call finds its pair
// free without waiting on the stores just issued.  32-byte rows with the
// 32-byte swizzle: the 16-byte chunk c of row r sits at chunk c ^ ((r >> 2)
// & 1).
template <int OFF0, int OFF1>
HS_DEV void store_two(const float (&v)[4 * PS_QU], float *stg, int &sp, const CUtensorMap *tm0,
                      const CUtensorMap *tm1, int r, bool issuer, int bar, int n0, int n1, int b, int t0) {
  float *b0 = stg + (sp & 1) * 2 * (PS_BOX / 4), *b1 = b0 + PS_BOX / 4;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int o = r * PS_QU + ((c ^ ((r >> 2) & 1)) * 4);
    *reinterpret_cast<float4 *>(b0 + o) =
        make_float4(v[OFF0 + 4 * c], v[OFF0 + 4 * c + 1], v[OFF0 + 4 * c + 2], v[OFF0 + 4 * c + 3]);
    *reinterpret_cast<float4 *>(b1 + o) =
        make_float4(v[OFF1 + 4 * c], v[OFF1 + 4 * c + 1], v[OFF1 + 4 * c + 2], v[OFF1 + 4 * c + 3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the other pair is read
  named_sync(bar);
  if (issuer) {
    tma_store_3d(tm0, b0, n0, b, t0);
    tma_store_3d(tm1, b1, n1, b, t0);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  ++sp;
}

// Roles as in the projection's pair GEMM: warp 0 loads (both CTAs, each its
// own rows; the bytes of both land on the first CTA's barrier), warp 1 of
// the first CTA issues the MMAs, warps 2-17 of both CTAs fold the
// accumulator groups and run the epilogue (four quads of four warps, one
// per 8 units, thread = time step).
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PS_THREADS, 1)
proj_scan_pair_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                      const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                      const __grid_constant__ CUtensorMap tmZ, const __grid_constant__ CUtensorMap tmO,
                      const __grid_constant__ CUtensorMap tmC, const PsArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *epi = reinterpret_cast<float *>(smem + PS_STAGES * PS_STAGE);  // 4 quads x PS_NBUF staging boxes
  uint64_t *full = reinterpret_cast<uint64_t *>(epi + PS_NQ * PS_NBUF * (PS_BOX / 4));
  uint64_t *empty = full + PS_STAGES;
  uint64_t *pfull = empty + PS_STAGES;
  uint64_t *pempty = pfull + PS_NACC;
  uint64_t *mdone = pempty + PS_NACC;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(mdone + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PS_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < PS_NACC; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 2 * PS_NQ * 4);  // 16 epilogue warps x 2 CTAs (used in the first CTA)
    }
    mbar_init(mdone, 1);
    *abort_flag = ld_status(p.status) != 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_holder)),
                 "r"(PS_TMEM_COLS)
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
      const int g0 = 2 * (int)rank;  // gates i, f (first CTA) or g, o (second)
      for (int tl = pair; tl < p.ntiles && ok; tl += npairs) {
        const int tt = tl / p.nch, ch = tl - tt * p.nch;
        const int bq = 2 * (ch / p.nub) + (int)rank;  // this CTA's sequence
        const int u0 = (ch % p.nub) * PS_UB;
        const int t0 = tt * PS_TT;
        for (int i = 0; i < p.nkb; ++i, ++it) {
          const int s = it % PS_STAGES;
          const uint32_t ph = (it / PS_STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status)) { ok = false; break; }
          // pass a real release (not the first use of a stage) on to the
          // second CTA first, so that its loads start with this CTA's
          if (rank == 0 && it >= PS_STAGES) mbar_arrive_cluster(cluster_addr(&empty[s], 1));
          const uint32_t fb = cluster_addr(&full[s], 0);
          unsigned char *st = smem + s * PS_STAGE;
          if (rank == 0) mbar_expect_tx(&full[s], 2 * PS_STAGE);  // both CTAs' bytes
          const int k0 = i * PS_BK;
          tma_3d_pair(st, &tmAh, fb, k0, bq, t0);
          tma_3d_pair(st + PS_ATILE, &tmAl, fb, k0, bq, t0);
          // B: two PS_UB-row boxes per part, gate g0's rows then gate g0+1's
          unsigned char *sb = st + 2 * PS_ATILE;
          tma_2d_pair(sb, &tmBh, fb, k0, g0 * p.H + u0);
          tma_2d_pair(sb + PS_BGATE, &tmBh, fb, k0, (g0 + 1) * p.H + u0);
          tma_2d_pair(sb + PS_BTILE, &tmBl, fb, k0, g0 * p.H + u0);
          tma_2d_pair(sb + PS_BTILE + PS_BGATE, &tmBl, fb, k0, (g0 + 1) * p.H + u0);
          ++issued;
        }
      }
      // The first CTA's barrier counts both CTAs' bytes: never leave while a
      // copy into either CTA's shared memory is in flight.
      if (rank == 0) {
        for (int j = std::max(0, issued - PS_STAGES); j < issued; ++j) {
          if (ld_status(p.status)) mbar_drain(&full[j % PS_STAGES], (j / PS_STAGES) & 1);
          else (void)mbar_wait(&full[j % PS_STAGES], (j / PS_STAGES) & 1, p.status);
        }
      }
    }
  } else if (!skip && warp == 1) {
    // ---------------- MMA issuer (first CTA only): three fp16 products per
    // k-step into one accumulator, groups of PS_PROM k-blocks, PS_NACC
    // accumulator buffers in turn
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_f16(256, PS_N);
      int it = 0, gg = 0;
      bool ok = true;
      for (int tl = pair; tl < p.ntiles && ok; tl += npairs) {
        for (int i = 0; i < p.nkb; ++i, ++it) {
          const int s = it % PS_STAGES;
          const uint32_t ph = (it / PS_STAGES) & 1;
          const bool gstart = (i % PS_PROM) == 0;
          const int b = gg % PS_NACC;
          if (gstart && !mbar_wait(&pempty[b], ((gg / PS_NACC) & 1) ^ 1, p.status)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, p.status)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t ah = su32(smem + s * PS_STAGE);
          const uint32_t al = ah + PS_ATILE, bh = ah + 2 * PS_ATILE, bl = bh + PS_BTILE;
          const uint32_t t_acc = tmem + (uint32_t)(b * PS_N);
#pragma unroll
          for (int kk = 0; kk < PS_BK / 16; ++kk) {
            const uint32_t o = kk * 32;  // 16 fp16 = 32 bytes into each row
            const uint64_t dAh = sdesc(ah + o, 16, PS_SBO, 2), dAl = sdesc(al + o, 16, PS_SBO, 2);
            const uint64_t dBh = sdesc(bh + o, 16, PS_SBO, 2), dBl = sdesc(bl + o, 16, PS_SBO, 2);
            mma_f16_pair(t_acc, dAh, dBh, idesc, (gstart && kk == 0) ? 0u : 1u);
            mma_f16_pair(t_acc, dAh, dBl, idesc, 1u);
            mma_f16_pair(t_acc, dAl, dBh, idesc, 1u);
          }
          mma_commit_pair(&empty[s]);
          if ((i % PS_PROM) == PS_PROM - 1 || i == p.nkb - 1) {
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
    // ---------------- epilogue (both CTAs): four quads of four warps, quad
    // w takes units 8 w .. 8 w + 7 of the chain's block, thread = step.
    // Per tile, five barriers of the quad: after the fold, after the staged
    // Z of gates i and f, after the step maps and the Z of g and o, after
    // the carry, after the staged c and out.  The staged pairs alternate
    // between two pairs of buffers (store_two), so no wait for a store's
    // read follows right behind that store.
    const int e = warp - 2;           // 0..15
    const int quad = e >> 2;
    const int q = warp & 3;           // TMEM lane quarter: tile rows 32q .. 32q + 31
    const int r = q * 32 + lane;      // tile row = time step t0 + r
    const int bar = 1 + quad;
    const bool lead = (e & 3) == 0;   // the quad's carry warp; its lane 0 issues the stores
    const bool issuer = lead && lane == 0;
    float *stg = epi + quad * PS_NBUF * (PS_BOX / 4);
    int sp = 0;  // staged pairs so far (alternating buffer pairs)
    // Undo the two operand scales one at a time (each inverse is an exact
    // power of two within float range, their product may not be).
    const float inv_a = 1.0f / pow2_scale(*p.absmax_a), inv_b = 1.0f / pow2_scale(*p.absmax_b);
    const int ngroups = (p.nkb + PS_PROM - 1) / PS_PROM;
    const int H = p.H;
    const float eps = p.eps;
    float kmax = 0.f;
    int gg = 0;
    for (int tl = pair; tl < p.ntiles; tl += npairs) {
      const int tt = tl / p.nch, ch = tl - tt * p.nch;
      const int bq = 2 * (ch / p.nub) + (int)rank;
      const int ub = ch % p.nub;
      const int u0 = ub * PS_UB + PS_QU * quad;
      const int t0 = tt * PS_TT;
      const bool bvalid = bq < p.B;
      // the bias of this tile's units, loaded before the accumulator wait
      float4 bias4[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        bias4[k] = p.bias ? *reinterpret_cast<const float4 *>(p.bias + (k >> 1) * H + u0 + 4 * (k & 1))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      // v[8 gate + j]: gate (i, f, g, o) of unit u0 + j at step t0 + r
      float v[4 * PS_QU];
#pragma unroll
      for (int j = 0; j < 4 * PS_QU; ++j) v[j] = 0.f;
      bool ok = true;
      for (int g = 0; g < ngroups; ++g, ++gg) {
        const int b = gg % PS_NACC;
        if (!mbar_wait(&pfull[b], (gg / PS_NACC) & 1, p.status)) { ok = false; break; }
        if (rank == 0 && e == 0 && lane == 0) mbar_arrive_cluster(cluster_addr(&pfull[b], 1));  // tell the second CTA
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * PS_N) + (uint32_t)(PS_QU * quad);
        uint32_t w[32];
#pragma unroll
        for (int gate = 0; gate < 4; ++gate) tmem_ld8_nowait(base + (uint32_t)(gate * PS_UB), w + 8 * gate);
        tmem_wait_ld(w);
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] += __uint_as_float(w[k]);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&pempty[b], 0));
      }
      if (!named_and(bar, ok && ld_status(p.status) == 0)) break;

      // Z = acc / (s_A s_B) + b_ih, stored for the backward
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int o = 4 * k;
        v[o] = (v[o] * inv_a) * inv_b + bias4[k].x;
        v[o + 1] = (v[o + 1] * inv_a) * inv_b + bias4[k].y;
        v[o + 2] = (v[o + 2] * inv_a) * inv_b + bias4[k].z;
        v[o + 3] = (v[o + 3] * inv_a) * inv_b + bias4[k].w;
      }
      store_two<0, PS_QU>(v, stg, sp, &tmZ, &tmZ, r, issuer, bar, u0, H + u0, bq, t0);

      // Gates (z_i, z_f are staged; z_g, z_o stay until their boxes): f'
      // and (i g)' go to the staging pair the next store_two will use (free
      // until then), unit-major, for the walk; e^-o stays in registers.
      float *fpS = stg + (sp & 1) * 2 * (PS_BOX / 4), *bpS = fpS + PS_BOX / 4;  // [8 units][128 steps]
      float eo[PS_QU];
#pragma unroll
      for (int j = 0; j < PS_QU; ++j) {
        fpS[j * PS_TT + r] = fmaxf(sigf(v[PS_QU + j]), eps);
        bpS[j * PS_TT + r] = fmaxf(sig2(v[j], v[2 * PS_QU + j]), eps);
        eo[j] = __expf(-v[3 * PS_QU + j]);
      }
      named_sync(bar);

      // The walk: thread (unit u, segment sg) takes steps 8 sg .. 8 sg + 7 of
      // unit u in order.  Its segment's map c -> A c + C, the 16 segments of
      // the unit combined by a 16-lane shuffle scan, the chain's carry in and
      // out by the last segment's thread, then c at every step of the
      // segment (written over (i g)') and the backward's bound.
      bool good = true;
      {
        const int tq = (e & 3) * 32 + lane, u = tq >> 4, sg = tq & 15;
        const float4 f0 = *reinterpret_cast<const float4 *>(fpS + u * PS_TT + 8 * sg);
        const float4 f1 = *reinterpret_cast<const float4 *>(fpS + u * PS_TT + 8 * sg + 4);
        const float4 b0 = *reinterpret_cast<const float4 *>(bpS + u * PS_TT + 8 * sg);
        const float4 b1 = *reinterpret_cast<const float4 *>(bpS + u * PS_TT + 8 * sg + 4);
        const float fw[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
        const float bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float A = 1.f, C = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          C = fmaf(fw[i], C, bw[i]);
          A *= fw[i];
        }
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) {
          const float Ap = __shfl_up_sync(0xffffffffu, A, off, 16), Cp = __shfl_up_sync(0xffffffffu, C, off, 16);
          if (sg >= off) {
            C = fmaf(A, Cp, C);
            A *= Ap;
          }
        }
        // the map of the segments before this one (identity for the first)
        float Ae = __shfl_up_sync(0xffffffffu, A, 1, 16), Ce = __shfl_up_sync(0xffffffffu, C, 1, 16);
        if (sg == 0) {
          Ae = 1.f;
          Ce = 0.f;
        }
        float cin = eps;
        if (sg == 15 && bvalid) {
          unsigned long long *slot = p.slots + (int64_t)bq * H + u0 + u;
          if (tt == 0) cin = fmaxf(p.c0 ? p.c0[(int64_t)bq * H + u0 + u] : 0.f, eps);
          else good = gslot_wait(slot, (unsigned)tt, &cin, p.status);
          if (good && tt + 1 < p.ntt) gslot_put(slot, (unsigned)(tt + 1), fmaf(A, cin, C));
        }
        cin = __shfl_sync(0xffffffffu, cin, (lane & 16) | 15);
        float c = fmaf(Ae, cin, Ce);  // c just before this segment's first step
        float cs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (bvalid && t0 + 8 * sg + i < p.T) kmax = fmaxf(kmax, c * fw[i] * (1.f - fw[i]));
          c = fmaf(fw[i], c, bw[i]);
          cs[i] = c;
        }
        *reinterpret_cast<float4 *>(bpS + u * PS_TT + 8 * sg) = make_float4(cs[0], cs[1], cs[2], cs[3]);
        *reinterpret_cast<float4 *>(bpS + u * PS_TT + 8 * sg + 4) = make_float4(cs[4], cs[5], cs[6], cs[7]);
      }
      if (!named_and(bar, good && ld_status(p.status) == 0)) break;

      // c and out at this thread's step
      float cc[PS_QU], oo[PS_QU];
#pragma unroll
      for (int j = 0; j < PS_QU; ++j) {
        cc[j] = bpS[j * PS_TT + r];
        oo[j] = sig_tanh_pos(eo[j], cc[j]);
      }
      named_sync(bar);  // the walk's buffers are read before the Z of g and o goes there
      store_two<2 * PS_QU, 3 * PS_QU>(v, stg, sp, &tmZ, &tmZ, r, issuer, bar, 2 * H + u0, 3 * H + u0, bq, t0);
#pragma unroll
      for (int j = 0; j < PS_QU; ++j) {
        v[2 * PS_QU + j] = cc[j];
        v[3 * PS_QU + j] = oo[j];
      }
      store_two<2 * PS_QU, 3 * PS_QU>(v, stg, sp, &tmC, &tmO, r, issuer, bar, u0, u0, bq, t0);
      if (bvalid && t0 + r == p.T - 1) {
        const int64_t ci = (int64_t)bq * H + u0;
#pragma unroll
        for (int j = 0; j < PS_QU; ++j) {
          if (p.h_n) p.h_n[ci + j] = oo[j];
          if (p.c_n) p.c_n[ci + j] = cc[j];
        }
      }
    }
    // every store has read its staging buffer before the CTA may leave
    if (issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    if (p.kf) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
      if (lane == 0) atomicMax(p.kf, __float_as_uint(kmax));
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  __syncthreads();
  cluster_sync_all();  // neither CTA frees TMEM or leaves while the pair's work may touch it
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PS_TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- host side
// x split [T*B][ld] fp16 as the 3D tensor {ld, B, T}: box {64 k, 1 b, 128 t}.
bool make_map_x(CUtensorMap *tm, const __half *ptr, int64_t T, int64_t B, int64_t ld) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)B, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(B * ld * 2)};
  cuuint32_t box[3] = {(cuuint32_t)PS_BK, 1, (cuuint32_t)PS_TT};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void *)ptr, dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// W_ih split [4H][ld] fp16: box {64 k, 32 rows} (one gate's rows of a chain).
bool make_map_w(CUtensorMap *tm, const __half *ptr, int64_t rows, int64_t ld) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)PS_BK, (cuuint32_t)PS_UB};
  cuuint32_t es[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)ptr, dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// [T][B][N] float32 output as {N, B, T}: box {8 columns, 1 b, 128 t},
// 32-byte swizzle (the epilogue's staging layout).
bool make_map_tbn(CUtensorMap *tm, float *ptr, int64_t T, int64_t B, int64_t N) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)B, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)N * 4, (cuuint64_t)(B * N * 4)};
  cuuint32_t box[3] = {(cuuint32_t)PS_QU, 1, (cuuint32_t)PS_TT};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)ptr, dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::atomic<unsigned long long> g_ps_attr{0};
char g_ps_cap_msg[256] = "";

// Pairs of this kernel resident at once on the current device (0: none,
// g_ps_cap_msg says why).
int ps_capacity() {
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int> &c = cached[dev & 63];
  int v = c.load(std::memory_order_relaxed);
  if (v > 0) return v - 1;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (allow_dynamic_smem((const void *)proj_scan_pair_kernel, PS_SMEM, &g_ps_attr) != HS_OK) {
    snprintf(g_ps_cap_msg, sizeof(g_ps_cap_msg), "setting %d bytes of dynamic shared memory failed", PS_SMEM);
    (void)cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)std::max(sms, 2), 1, 1);
  cfg.blockDim = dim3(PS_THREADS, 1, 1);
  cfg.dynamicSmemBytes = PS_SMEM;
  int n = 0;
  const cudaError_t err = cudaOccupancyMaxActiveClusters(&n, (const void *)proj_scan_pair_kernel, &cfg);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  if (n < 1) {
    cudaFuncAttributes fa = {};
    (void)cudaFuncGetAttributes(&fa, (const void *)proj_scan_pair_kernel);
    (void)cudaGetLastError();
    snprintf(g_ps_cap_msg, sizeof(g_ps_cap_msg),
             "cluster occupancy %d (%s); kernel: %d registers, %zu static + %d dynamic smem bytes, max %d threads",
             n, cudaGetErrorString(err), fa.numRegs, fa.sharedSizeBytes, PS_SMEM, fa.maxThreadsPerBlock);
  }
  c.store(n + 1, std::memory_order_relaxed);
  return n;
}

// HS_PROJ_SCAN: 0 never takes the fused kernel, 1 takes it for every shape
// it can run; unset, it is taken when the sequence fills most of one time
// tile (112 <= T <= 128: no carries between tiles, at most 1/8 of the
// tile's rows padding).  Measured on B200 (configs[4]'s 32-sequence
// micro-batch, T = 4096, one box): run alone, 1.78 ms fused against
// 1.83-1.89 ms for the projection GEMM (N = 256 tiles) and the column scan;
// inside the power-capped training step, where tensor and SIMT work at once
// draw more power, 10.7 ms against 9.4 ms per 37-sequence micro-batch; at
// T = 128 the fused step is 22% faster.
int ps_mode() {
  static int v = -2;
  if (v == -2) {
    const char *e = getenv("HS_PROJ_SCAN");
    v = (e && e[0] == '0') ? 0 : (e && e[0] == '1') ? 1 : -1;
  }
  return v;
}

int64_t ps_round8(int64_t x) { return (x + 7) / 8 * 8; }

}  // namespace

size_t proj_scan_ws(int64_t T, int64_t B, int64_t D, int64_t H) {
  (void)T;
  if (B <= 0 || D <= 0 || H <= 0) return 0;
  return 256 + h3_split_bytes(4 * H, D) + round_up((size_t)B * H * 8, 256);
}

// Shapes the fused kernel can run: 32-unit chain blocks, int32 tile and
// coordinate arithmetic, the fp16-split tensor-core GEMMs enabled.
bool proj_scan_shape_ok(int64_t T, int64_t B, int64_t D, int64_t H) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0 || H % PS_UB) return false;
  if (T >= (1ll << 30) || B >= (1ll << 30) || 4 * H >= (1ll << 30) || T * B >= (1ll << 31)) return false;
  const int64_t ntt = (T + PS_TT - 1) / PS_TT, nch = (B + 1) / 2 * (H / PS_UB);
  if (ntt * nch >= (1ll << 31) || D >= (1ll << 30)) return false;
  return gemm_h3_enabled() && gemm_tc_size_ok(T * B, 4 * H, D);
}

bool proj_scan_wanted(int64_t T, int64_t B, int64_t D, int64_t H) {
  const int mode = ps_mode();
  if (mode == 0 || !proj_scan_shape_ok(T, B, D, H)) return false;
  const int npairs = ps_capacity();
  if (npairs < 1) return false;
  if (mode == 1) return true;
  // one time tile, mostly filled: a tile always spans PS_TT steps, so at
  // small T most of its MMA rows would be padding
  return T <= PS_TT && 8 * T >= 7 * PS_TT;
}

// Z, out, c [T][B][4H | H | H], h_n, c_n and *kf (max c_{t-1} f'(1-f')) from
// x's fp16 split (hs_split layout, with its scale word) and float32 W_ih,
// b_ih, c0.  *took = false (nothing launched, *why says which condition) if
// the shape, the alignment or the scratch does not suit; the caller then
// runs the GEMM and the scan.
int proj_scan_forward(const void *x_split, const unsigned *x_scale, const float *w, const float *bias,
                      const float *c0, float *z, float *out, float *c, float *h_n, float *c_n, int64_t T, int64_t B,
                      int64_t D, int64_t H, float eps, void *ws, size_t ws_bytes, unsigned *kf, int *status,
                      cudaStream_t st, bool *took, const char **why) {
  *took = false;
  const char *dummy = nullptr;
  if (!why) why = &dummy;
  *why = "shape or null argument";
  if (!proj_scan_shape_ok(T, B, D, H) || !status || !x_split || !x_scale || !w || !z || !out || !c) return HS_OK;
  *why = "x_split, z, out, c or b_ih not 16-byte aligned";
  if (!aligned(x_split, 16) || !aligned(z, 16) || !aligned(out, 16) || !aligned(c, 16) ||
      (bias && !aligned(bias, 16)) || (kf && !aligned(kf, 4)))
    return HS_OK;
  *why = "workspace missing, not 256-byte aligned or too small";
  if (!ws || !aligned(ws, 256) || ws_bytes < proj_scan_ws(T, B, D, H)) return HS_OK;
  const int npairs = ps_capacity();
  *why = g_ps_cap_msg;
  if (npairs < 1) return HS_OK;
  const int64_t D8 = ps_round8(D), N = 4 * H;
  char *w8 = static_cast<char *>(ws);
  unsigned *w_scale = reinterpret_cast<unsigned *>(w8);
  __half *wh = reinterpret_cast<__half *>(w8 + 256);
  const __half *wl = wh + N * D8;
  unsigned long long *slots = reinterpret_cast<unsigned long long *>(w8 + 256 + h3_split_bytes(N, D));
  const __half *xh = static_cast<const __half *>(x_split);
  const __half *xl = xh + T * B * D8;
  CUtensorMap tah, tal, tbh, tbl, tz, to, tc;
  if (!make_map_x(&tah, xh, T, B, D8) || !make_map_x(&tal, xl, T, B, D8) || !make_map_w(&tbh, wh, N, D8) ||
      !make_map_w(&tbl, wl, N, D8) || !make_map_tbn(&tz, z, T, B, N) || !make_map_tbn(&to, out, T, B, H) ||
      !make_map_tbn(&tc, c, T, B, H)) {
    *why = "tensor-map encoding failed";
    return HS_OK;
  }
  if (int e = h3_split(w, N, D, D, w_scale, wh, st)) return e;
  if (cudaMemsetAsync(slots, 0, (size_t)B * H * 8, st) != cudaSuccess) return check_launch("proj_scan slots memset");
  if (kf && cudaMemsetAsync(kf, 0, 4, st) != cudaSuccess) return check_launch("proj_scan kf memset");
  PsArgs a;
  a.bias = bias;
  a.c0 = c0;
  a.h_n = h_n;
  a.c_n = c_n;
  a.slots = slots;
  a.kf = kf;
  a.absmax_a = x_scale;
  a.absmax_b = w_scale;
  a.status = status;
  a.T = (int)T;
  a.B = (int)B;
  a.H = (int)H;
  a.nkb = (int)((D8 + PS_BK - 1) / PS_BK);
  a.nub = (int)(H / PS_UB);
  a.nch = (int)((B + 1) / 2 * a.nub);
  a.ntt = (int)((T + PS_TT - 1) / PS_TT);
  a.ntiles = a.ntt * a.nch;
  a.eps = eps;
  if (int e = allow_dynamic_smem((const void *)proj_scan_pair_kernel, PS_SMEM, &g_ps_attr)) return e;
  const unsigned grid = 2u * (unsigned)std::min<int64_t>(a.ntiles, npairs);
  proj_scan_pair_kernel<<<grid, PS_THREADS, PS_SMEM, st>>>(tah, tal, tbh, tbl, tz, to, tc, a);
  if (int e = check_launch("proj_scan_pair_kernel")) return e;
  *took = true;
  return HS_OK;
}

}  // namespace hs
