// Recurrent-mode HeadStartLSTM for small H on one thread-block cluster per
// batch group of up to 32 sequences.
//
// Reference: HeadStartLSTMTorchFn (src/headstartlstm/_torch.py:86-170): per
// step gates = Z[t] + h_{t-1} (a*W_hh)^T + a*b_hh (_torch.py:111-120), and in
// the backward dh = dgates (a*W_hh) (_torch.py:150).
//
// When a*W_hh (4H x H float32) fits in the shared memory of one cluster, the
// whole recurrence of a batch group stays on that cluster: CTA j of the C
// CTAs owns UC = H / C hidden units and keeps its slice of the weights
// resident for the launch (forward: its 4 UC gate rows over all k; backward:
// all 4H gate rows for its UC units).  Each step it
//   1. multiplies its slice by the state of the previous step held in its
//      own shared memory (float32 FFMA in 4 x 4 register blocks, k split over
//      groups of threads, partial sums added in a fixed order);
//   2. runs the cell for its units (forward: sigmoids, c, h; backward: the
//      cell's backward, dgates);
//   3. sends the new state block (forward: h of its units, 1 KB; backward:
//      dgates of its units' 4 gate rows, 4 KB) to every CTA of the cluster by
//      bulk copies between the CTAs' shared memories, which complete on the
//      receiver's mbarrier.
// The state never leaves the cluster: no global exchange buffer and no wait
// on another cluster, so batch groups run independently and the launch needs
// no co-residency beyond the cluster itself.
//
// Buffers: the receive buffers and the outgoing staging blocks are double
// buffered by step parity.  A receive buffer is written for step t+1 only by
// CTAs that have finished step t, which needed this CTA's state of step t,
// sent after this CTA finished reading the buffer; a staging block is reused
// two steps later, after every receiver has sent a state that needed it.
// Every wait is bounded (kWaitLimitNs); a CTA that gives up records
// HS_ERR_DEVICE_TIMEOUT, stops, lets the copies it expects land (bounded) and
// meets the others at the final cluster barrier.  No cluster multicast.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "hs_common.cuh"

namespace hs {

namespace {

constexpr int kCT = 256;  // threads per CTA
constexpr int kBC = 32;   // sequences per cluster (one batch group), padded

HS_DEV uint32_t csu32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
HS_DEV void cmbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(csu32(b)), "r"(count) : "memory");
}
HS_DEV void cmbar_arrive_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(csu32(b)), "r"(bytes) : "memory");
}
HS_DEV bool cmbar_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(csu32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false (status set) after kWaitLimitNs or once another CTA
// has recorded a failure.
HS_DEV bool cmbar_wait(uint64_t *b, uint32_t parity, int *status) {
  if (cmbar_try(b, parity)) return true;
  const uint64_t t0 = globaltimer();
  unsigned n = 0;
  while (!cmbar_try(b, parity)) {
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
// Bounded wait that records nothing (on the way out after a failure).
HS_DEV void cmbar_drain(uint64_t *b, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!cmbar_try(b, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) return;
  }
}
HS_DEV uint32_t crank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HS_DEV uint32_t cpeer(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(csu32(p)), "r"(rank));
  return r;
}
HS_DEV void ccluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
HS_DEV void cbulk_s2c(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "r"(csu32(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Sequence blocks of 4 per row block: the fewest that cover Bc sequences for
// which the thread count splits k evenly (kCT / (rows * nbq) groups dividing
// K), at most 8.
HS_DEV int seq_blocks(int Bc, int rows, int K, int lo) {
  int nbq = lo;
  while (nbq < 8 && (4 * nbq < Bc || kCT % (rows * nbq) != 0 || kCT / (rows * nbq) > K ||
                     K % (kCT / (rows * nbq)) != 0))
    nbq *= 2;
  return nbq;
}

struct RclArgs {
  const float *w;      // forward: [C][H][4UC] (k-major, row ul*4+g); backward: [C][4H][UC] (row u*4+g)
  const float *bias;   // forward: [C][4UC], a*b_hh
  float *zacts;        // forward: Z in, activations out; backward: activations in, dgates out
  const float *h0, *c0;
  float *h_save, *c_save;
  const float *dout, *dh_n, *dc_n;
  int *status;
  int64_t T, Bt, H;
  int C, UC;
};

// Shared-memory carve-up in floats (16-byte aligned pieces), for R rows of
// the step product (forward 4 UC, backward UC), K (forward H, backward 4H),
// KG k-groups, and a state block of SB floats per CTA (forward UC x 32,
// backward 4 UC x 32).
struct CLayout {
  int w, bias, rx, stage, red, bars, total;  // offsets in floats; total bytes in total
};
__host__ __device__ inline CLayout clayout(int R, int K, int KG, int SB, int C) {
  CLayout L{};
  int off = 0;
  auto take = [&](int n) { int o = off; off += (n + 3) & ~3; return o; };
  L.w = take(K * R);
  L.bias = take(R);
  L.rx = take(2 * C * SB);     // receive buffers [2][K rows of the state][32]
  L.stage = take(2 * SB);      // outgoing blocks [2][SB]
  L.red = take(KG * R * kBC);  // partial sums [KG][R][32]
  L.bars = take(4);            // 2 mbarriers (8 bytes each)
  L.total = off * 4;
  return L;
}

// ------------------------------------------------------------------ forward
__global__ void __launch_bounds__(kCT, 1) rcl_fwd_kernel(RclArgs p) {
  extern __shared__ __align__(16) float smc[];
  const int C = p.C, UC = p.UC, R = 4 * UC;
  const int64_t H = p.H, Bt = p.Bt, T = p.T;
  const int K = (int)H;
  const int SB = UC * kBC;
  const CLayout L = clayout(R, K, kCT / (UC * 8), SB, C);
  float *W = smc + L.w, *bias = smc + L.bias, *rx = smc + L.rx, *stage = smc + L.stage, *red = smc + L.red;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smc + L.bars);
  const uint32_t j = crank();
  const int grp = blockIdx.x / C;
  const int b0 = grp * kBC;
  const int Bc = (int)min((int64_t)kBC, Bt - b0);
  const int tid = threadIdx.x;
  const uint32_t sbytes = (uint32_t)SB * 4;
  // 4 x 4 blocks of (rows, sequences) over this group's BP = 4 nbq padded
  // sequences; the threads left over split k into KG groups (partial sums
  // [KG][R][BP]: 4096 floats whatever nbq)
  const int nbq = seq_blocks(Bc, UC, K, 1);
  const int BP = 4 * nbq, nblk = UC * nbq, KG = kCT / nblk, KL = K / KG;

  // weights and bias of this CTA, resident for the launch
  const float4 *wsrc = reinterpret_cast<const float4 *>(p.w + (size_t)j * K * R);
  for (int i = tid; i < K * R / 4; i += kCT) reinterpret_cast<float4 *>(W)[i] = wsrc[i];
  for (int i = tid; i < R; i += kCT) bias[i] = p.bias[(size_t)j * R + i];
  if (tid == 0) {
    cmbar_init(&bars[0], 1);
    cmbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    cmbar_arrive_expect(&bars[0], (uint32_t)C * sbytes);  // h0 blocks
    cmbar_arrive_expect(&bars[1], (uint32_t)C * sbytes);  // step 0's blocks
  }
  __syncthreads();
  ccluster_sync();  // every CTA's barriers armed before any copy targets them

  // cells of this thread: (ul, b), b fastest
  constexpr int kMaxCells = 4;
  float cst[kMaxCells];
  const int ncell = UC * kBC;
  // prologue: h0 of this CTA's units into staging block 1 (block 0 is step
  // 0's; block 1 is next written at step 1, after every CTA has sent h_0,
  // which needed this block's copy), then to every CTA
  float *stg0 = stage + SB;
#pragma unroll
  for (int m = 0; m < kMaxCells; ++m) {
    const int ci = tid + kCT * m;
    cst[m] = 0.f;
    if (ci >= ncell) continue;
    const int ul = ci / kBC, b = ci % kBC;
    const int64_t u = (int64_t)j * UC + ul, bb = b0 + b;
    float h = 0.f, c = 0.f;
    if (b < Bc) {
      h = p.h0 ? p.h0[bb * H + u] : 0.f;
      c = p.c0 ? p.c0[bb * H + u] : 0.f;
      p.h_save[bb * H + u] = h;
      p.c_save[bb * H + u] = c;
    }
    cst[m] = c;
    stg0[ul * kBC + b] = h;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  if (tid < C)  // one copy per peer, issued by thread r for rank r
    cbulk_s2c(cpeer(rx + j * SB, (uint32_t)tid), stg0, sbytes, cpeer(&bars[0], (uint32_t)tid));

  __shared__ int s_fail;
  int64_t waited = 0;  // uses of the receive barriers completed by this CTA
  bool fail = false;
  const int kg = tid / nblk, blk = tid % nblk, rb = blk / nbq, bq = blk % nbq;
  for (int64_t t = 0; t < T && !fail; ++t) {
    const int par = (int)(t & 1);
    // this step's input projection for the thread's cells (before the wait)
    float zg[kMaxCells][4];
#pragma unroll
    for (int m = 0; m < kMaxCells; ++m) {
      const int ci = tid + kCT * m;
      const int ul = ci / kBC, b = ci % kBC;
#pragma unroll
      for (int g = 0; g < 4; ++g)
        zg[m][g] = (ci < ncell && b < Bc) ? p.zacts[(t * Bt + b0 + b) * 4 * H + g * H + (int64_t)j * UC + ul] : 0.f;
    }
    if (tid == 0) {
      s_fail = !cmbar_wait(&bars[par], (uint32_t)((t >> 1) & 1), p.status);
      if (!s_fail) {
        ++waited;
        // next use of this barrier: the blocks of step t+1 (h_{t+1}), read at t+2
        if (t + 2 < T) cmbar_arrive_expect(&bars[par], (uint32_t)C * sbytes);
      }
    }
    __syncthreads();
    if (s_fail) { fail = true; break; }
    // gates = h_{t-1} W^T over this thread's k group: 4 rows x 4 sequences
    const float *X = rx + par * C * SB;  // [K][32]
    float acc[4][4] = {};
#pragma unroll 4
    for (int k = kg * KL; k < (kg + 1) * KL; ++k) {
      const float4 wv = *reinterpret_cast<const float4 *>(W + k * R + 4 * rb);
      const float4 xv = *reinterpret_cast<const float4 *>(X + k * kBC + 4 * bq);
      const float w4[4] = {wv.x, wv.y, wv.z, wv.w}, x4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(w4[i], x4[q], acc[i][q]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<float4 *>(red + (kg * R + 4 * rb + i) * BP + 4 * bq) =
          make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    __syncthreads();
    // cells; h_t into staging block par (the outputs no other CTA reads are
    // stored after the send)
    float *stg = stage + par * SB;
    float act[kMaxCells][4], hv[kMaxCells];
#pragma unroll
    for (int m = 0; m < kMaxCells; ++m) {
      const int ci = tid + kCT * m;
      if (ci >= ncell) continue;
      const int ul = ci / kBC, b = ci % kBC;
      if (b >= BP) {  // beyond the computed sequences: zero state
        stg[ul * kBC + b] = 0.f;
        continue;
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int row = ul * 4 + g;
        float s = 0.f;
        for (int q = 0; q < KG; ++q) s += red[(q * R + row) * BP + b];
        act[m][g] = sigf(zg[m][g] + s + bias[row]);
      }
      const float c = fmaf(act[m][1], cst[m], act[m][0] * act[m][2]);
      hv[m] = act[m][3] * tanh_any(c);
      cst[m] = c;
      stg[ul * kBC + b] = b < Bc ? hv[m] : 0.f;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid < C && t + 1 < T)
      cbulk_s2c(cpeer(rx + (par ^ 1) * C * SB + j * SB, (uint32_t)tid), stg, sbytes,
                cpeer(&bars[par ^ 1], (uint32_t)tid));
#pragma unroll
    for (int m = 0; m < kMaxCells; ++m) {
      const int ci = tid + kCT * m;
      const int ul = ci / kBC, b = ci % kBC;
      if (ci >= ncell || b >= Bc) continue;
      const int64_t bb = b0 + b, u = (int64_t)j * UC + ul;
      float *ar = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
      for (int g = 0; g < 4; ++g) ar[g * H] = act[m][g];
      p.h_save[((t + 1) * Bt + bb) * H + u] = hv[m];
      p.c_save[((t + 1) * Bt + bb) * H + u] = cst[m];
    }
  }
  // On the way out after a failure: the blocks of the armed uses may still be
  // landing; let them (bounded) before meeting the cluster.
  if (tid == 0 && fail) {
    for (int64_t u2 = waited; u2 < std::min<int64_t>(T, waited + 2); ++u2)
      cmbar_drain(&bars[u2 & 1], (uint32_t)((u2 >> 1) & 1));
  }
  __syncthreads();
  ccluster_sync();
}

// ------------------------------------------------------------------ backward
__global__ void __launch_bounds__(kCT, 1) rcl_bwd_kernel(RclArgs p) {
  extern __shared__ __align__(16) float smc[];
  const int C = p.C, UC = p.UC;
  const int64_t H = p.H, Bt = p.Bt, T = p.T;
  const int K = (int)(4 * H), R = UC;
  const int SB = 4 * UC * kBC;
  const CLayout L = clayout(R, K, kCT / ((UC / 2) * 8), SB, C);
  float *W = smc + L.w, *rx = smc + L.rx, *stage = smc + L.stage, *red = smc + L.red;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smc + L.bars);
  const uint32_t j = crank();
  const int grp = blockIdx.x / C;
  const int b0 = grp * kBC;
  const int Bc = (int)min((int64_t)kBC, Bt - b0);
  const int tid = threadIdx.x;
  const uint32_t sbytes = (uint32_t)SB * 4;
  // 2 x 4 blocks of (units, sequences), the rest of the threads split k
  const int nbq = seq_blocks(Bc, UC / 2, K, 1);
  const int BP = 4 * nbq, nblk = (UC / 2) * nbq, KG = kCT / nblk, KL = K / KG;

  const float4 *wsrc = reinterpret_cast<const float4 *>(p.w + (size_t)j * K * R);
  for (int i = tid; i < K * R / 4; i += kCT) reinterpret_cast<float4 *>(W)[i] = wsrc[i];
  if (tid == 0) {
    cmbar_init(&bars[0], 1);
    cmbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // step T-1 sends into parity (T-1)&1, read by step T-2; one use each to start
    cmbar_arrive_expect(&bars[0], (uint32_t)C * sbytes);
    cmbar_arrive_expect(&bars[1], (uint32_t)C * sbytes);
  }
  __syncthreads();
  ccluster_sync();

  constexpr int kMaxCells = 4;
  const int ncell = UC * kBC;
  float dcst[kMaxCells];
#pragma unroll
  for (int m = 0; m < kMaxCells; ++m) {
    const int ci = tid + kCT * m;
    const int ul = ci / kBC, b = ci % kBC;
    dcst[m] = (ci < ncell && b < Bc && p.dc_n) ? p.dc_n[(int64_t)(b0 + b) * H + (int64_t)j * UC + ul] : 0.f;
  }
  __shared__ int s_fail;
  int64_t waited = 0;
  bool fail = false;
  const int kg = tid / nblk, blk = tid % nblk, ub = blk / nbq, bq = blk % nbq;
  for (int64_t t = T - 1; t >= 0 && !fail; --t) {
    const int par = (int)(t & 1);  // dgates of step t+1 arrived in rx[par]
    float ld[kMaxCells][7];        // i, f, g, o, c_t, c_{t-1}, dh
#pragma unroll
    for (int m = 0; m < kMaxCells; ++m) {
      const int ci = tid + kCT * m;
      const int ul = ci / kBC, b = ci % kBC;
      const bool v = ci < ncell && b < Bc;
      const int64_t u = (int64_t)j * UC + ul, bb = b0 + b;
      const float *ar = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
      for (int g = 0; g < 4; ++g) ld[m][g] = v ? ar[g * H] : 0.f;
      ld[m][4] = v ? p.c_save[((t + 1) * Bt + bb) * H + u] : 0.f;
      ld[m][5] = v ? p.c_save[(t * Bt + bb) * H + u] : 0.f;
      ld[m][6] = v ? p.dout[(t * Bt + bb) * H + u] + ((t == T - 1 && p.dh_n) ? p.dh_n[bb * H + u] : 0.f) : 0.f;
    }
    if (t < T - 1) {
      // use index of barrier par: steps T-2, T-4, ... (parity of T-2) or T-3, ...
      const int64_t use = (T - 2 - t) >> 1;
      if (tid == 0) {
        s_fail = !cmbar_wait(&bars[par], (uint32_t)(use & 1), p.status);
        if (!s_fail) {
          ++waited;
          if (t - 2 >= 0) cmbar_arrive_expect(&bars[par], (uint32_t)C * sbytes);
        }
      }
      __syncthreads();
      if (s_fail) { fail = true; break; }
      // dh = dgates_{t+1} (a W_hh) over this thread's k group: 2 units x 4 sequences
      const float *X = rx + par * C * SB;  // [4H][32], row u*4+g
      float acc[2][4] = {};
#pragma unroll 4
      for (int k = kg * KL; k < (kg + 1) * KL; ++k) {
        const float2 wv = *reinterpret_cast<const float2 *>(W + k * R + 2 * ub);
        const float4 xv = *reinterpret_cast<const float4 *>(X + k * kBC + 4 * bq);
        const float w2[2] = {wv.x, wv.y}, x4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(w2[i], x4[q], acc[i][q]);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i)
        *reinterpret_cast<float4 *>(red + (kg * R + 2 * ub + i) * BP + 4 * bq) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      __syncthreads();
    }
    float *stg = stage + par * SB;  // dgates of step t, rows ul*4+g
    float dgs[kMaxCells][4];        // stored to acts after the send
#pragma unroll
    for (int m = 0; m < kMaxCells; ++m) {
      const int ci = tid + kCT * m;
      if (ci >= ncell) continue;
      const int ul = ci / kBC, b = ci % kBC;
      float dh = ld[m][6];
      if (t < T - 1 && b < BP)
        for (int q = 0; q < KG; ++q) dh += red[(q * R + ul) * BP + b];
      const float i = ld[m][0], f = ld[m][1], g = ld[m][2], o = ld[m][3];
      const float th = tanh_any(ld[m][4]);
      const float dct = dcst[m] + dh * o * (1.f - th * th);
      float dg[4];
      dg[0] = dct * g * i * (1.f - i);
      dg[1] = dct * ld[m][5] * f * (1.f - f);
      dg[2] = dct * i * g * (1.f - g);
      dg[3] = dh * th * o * (1.f - o);
      dcst[m] = dct * f;
      const bool v = b < Bc;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        stg[(ul * 4 + q) * kBC + b] = v ? dg[q] : 0.f;
        dgs[m][q] = dg[q];
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    // dgates of step t, read by step t-1 from rx[(t-1)&1]
    if (tid < C && t > 0)
      cbulk_s2c(cpeer(rx + (par ^ 1) * C * SB + j * SB, (uint32_t)tid), stg, sbytes,
                cpeer(&bars[par ^ 1], (uint32_t)tid));
#pragma unroll
    for (int m = 0; m < kMaxCells; ++m) {
      const int ci = tid + kCT * m;
      const int ul = ci / kBC, b = ci % kBC;
      if (ci >= ncell || b >= Bc) continue;
      float *ar = p.zacts + (t * Bt + b0 + b) * 4 * H + (int64_t)j * UC + ul;
#pragma unroll
      for (int q = 0; q < 4; ++q) ar[q * H] = dgs[m][q];
    }
  }
  if (tid == 0 && fail) {
    for (int64_t u2 = waited; u2 < std::min<int64_t>(T - 1, waited + 2); ++u2) {
      const int64_t t2 = T - 2 - u2;  // the step that reads the use-u2 blocks
      cmbar_drain(&bars[t2 & 1], (uint32_t)(((T - 2 - t2) >> 1) & 1));
    }
  }
  __syncthreads();
  ccluster_sync();
}

// ------------------------------------------------------------ H = 512 (wide)
//
// The same recurrence at H = 512 on clusters of 16 CTAs with S
// <= 8 sequences per cluster, the batch spread over as many clusters as the
// device runs at once.  CTA j owns units 32j..32j+31, i.e. the 128 gate rows
// ul*4+g of a*W_hh (256 KB of float32, more than one CTA's shared memory):
// each thread keeps the first KR of its 32 k values of the slice in
// registers, the rest of the slice stays in shared memory.
//   forward:  gates[128 rows][S] = Z + (a W)_j h_{t-1} over the 512 units;
//             h_{t-1} [512][S] is all-gathered (every CTA sends its units'
//             block to every CTA, as in the kernels above);
//   backward: the CTA's share of dh[512][S] = (a W)_j^T dgates_j over its 128
//             rows is reduce-scattered: warp w computes the units of CTA w
//             and sends that block to CTA w, which adds the 16 blocks it
//             receives (in rank order) before its cells run.
// Product layout, 512 threads: a lane holds a block of 4 outputs (rows
// forward, units backward) x S sequences for one of 4 k subsets; the warp's
// 4 k subsets are added by shuffles (forward: then the 4 warps of a row group
// through shared memory).  Barriers, double buffering and bounded waits
// follow the kernels above.
constexpr int kWC = 16;               // CTAs per cluster
constexpr int kWUC = 32;              // units per CTA
constexpr int kWH = kWC * kWUC;       // H
constexpr int kWR = 4 * kWUC;         // gate rows per CTA
constexpr int kWT = 512;              // threads per CTA
constexpr int kWMaxS = 8;             // sequences per cluster

// Shared-memory carve-ups in floats (16-byte aligned pieces).
template <int S>
struct WideFwd {
  static constexpr int XS = S <= 4 ? 4 : 8;  // floats per state row
  static constexpr int KR = S <= 6 ? 16 : 12;  // k values per thread in registers (no spills)
  static constexpr int KS = kWH - 16 * KR;   // k rows of the slice in shared memory
  static constexpr int o_w = 0;
  static constexpr int o_bias = o_w + KS * kWR;
  static constexpr int o_rx = o_bias + kWR;           // [2][512][XS]
  static constexpr int o_stage = o_rx + 2 * kWH * XS;  // [2][32][XS]
  static constexpr int o_red = o_stage + 2 * kWUC * XS;  // [4 k groups][4 gates][S][32 units]
  static constexpr int o_bars = o_red + ((4 * 4 * S * kWUC + 3) & ~3);
  static constexpr int bytes = (o_bars + 4) * 4;
};
template <int S>
struct WideBwd {
  static constexpr int XS = S <= 4 ? 4 : 8;
  static constexpr int KR = S <= 4 ? 12 : 14;  // rows per thread in registers
  static constexpr int KS = kWR - 4 * KR;      // rows of the slice in shared memory
  static constexpr int o_w = 0;
  static constexpr int o_rx = o_w + KS * kWH;                // [2][16 senders][S][32 units]
  static constexpr int o_stage = o_rx + 2 * kWC * S * kWUC;  // [2][16 receivers][S][32 units]
  static constexpr int o_dg = o_stage + 2 * kWC * S * kWUC;  // [128 rows g*32+ul][XS]
  static constexpr int o_bars = o_dg + kWR * XS;
  static constexpr int bytes = (o_bars + 4) * 4;
};

struct RwArgs {
  const float *w;     // forward [16][512 k][128 rows ul*4+g]; backward [16][128 rows g*32+ul][512 units]
  const float *bias;  // forward [16][128]
  float *zacts;       // forward: Z in, activations out; backward: activations in, dgates out
  const float *h0, *c0;
  float *h_save, *c_save;
  const float *dout, *dh_n, *dc_n;
  int *status;
  int64_t T, Bt;
};

template <int S, int XS>
HS_DEV void wide_ldx(const float *p, float (&v)[S]) {
  const float4 a = *reinterpret_cast<const float4 *>(p);
  float t[8] = {a.x, a.y, a.z, a.w, 0.f, 0.f, 0.f, 0.f};
  if constexpr (S > 4) {
    const float4 b = *reinterpret_cast<const float4 *>(p + 4);
    t[4] = b.x; t[5] = b.y; t[6] = b.z; t[7] = b.w;
  }
#pragma unroll
  for (int s = 0; s < S; ++s) v[s] = t[s];
}
// Sum of the 4 k subsets of a warp (lanes l, l^8, l^16, l^24), halving the
// values at each exchange: afterwards lane l holds output 4-block element
// (l >> 3) for its S sequences.
template <int S>
HS_DEV void wide_reduce4(const float (&acc)[4][S], int lane, float (&v)[S]) {
  const bool hi2 = (lane & 16) != 0, hi1 = (lane & 8) != 0;
  float b2[2][S];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const float send = hi2 ? acc[r][s] : acc[r + 2][s];
      const float keep = hi2 ? acc[r + 2][s] : acc[r][s];
      b2[r][s] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const float send = hi1 ? b2[0][s] : b2[1][s];
    const float keep = hi1 ? b2[1][s] : b2[0][s];
    v[s] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
}

template <int S>
__global__ void __launch_bounds__(kWT, 1) rcw_fwd_kernel(RwArgs p) {
  using L = WideFwd<S>;
  constexpr int XS = L::XS, KR = L::KR;
  constexpr int64_t H = kWH;
  constexpr uint32_t sbytes = kWUC * XS * 4;  // one CTA's state block
  extern __shared__ __align__(16) float smw[];
  float *Ws = smw + L::o_w, *bias = smw + L::o_bias, *rx = smw + L::o_rx, *stage = smw + L::o_stage,
        *red = smw + L::o_red;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smw + L::o_bars);
  const uint32_t j = crank();
  const int64_t T = p.T, Bt = p.Bt;
  const int64_t b0 = (int64_t)(blockIdx.x / kWC) * S;
  const int Bc = (int)min((int64_t)S, Bt - b0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // product: rows r0..r0+3 (row group warp & 3), k = 16 i + q, i < 32
  const int kgw = warp >> 2, ks = lane >> 3;
  const int r0 = 32 * (warp & 3) + 4 * (lane & 7), q = kgw * 4 + ks;
  const float *wj = p.w + (size_t)j * kWH * kWR;  // [k][128 rows]
  {
    const float4 *src = reinterpret_cast<const float4 *>(wj + 16 * KR * kWR);
    for (int i = tid; i < L::KS * kWR / 4; i += kWT) reinterpret_cast<float4 *>(Ws)[i] = src[i];
  }
  float wr[4][KR];
#pragma unroll
  for (int i = 0; i < KR; ++i) {
    const float4 v = *reinterpret_cast<const float4 *>(wj + (size_t)(16 * i + q) * kWR + r0);
    wr[0][i] = v.x;
    wr[1][i] = v.y;
    wr[2][i] = v.z;
    wr[3][i] = v.w;
  }
  for (int i = tid; i < kWR; i += kWT) bias[i] = p.bias[(size_t)j * kWR + i];
  if (tid == 0) {
    cmbar_init(&bars[0], 1);
    cmbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    cmbar_arrive_expect(&bars[0], kWC * sbytes);  // h0 blocks
    cmbar_arrive_expect(&bars[1], kWC * sbytes);  // step 0's blocks
  }
  __syncthreads();
  ccluster_sync();

  // the cell of this thread (tid < 32 S): unit ul, sequence s
  const bool is_cell = tid < kWUC * S;
  const int ul = tid & 31, s = tid >> 5;
  const bool valid = is_cell && s < Bc;
  const int64_t u = (int64_t)j * kWUC + ul, bb = b0 + s;
  float cst = 0.f;
  float *stg0 = stage + kWUC * XS;  // block 1 carries h0 (block 0 is step 0's)
  if (is_cell) {
    float h = 0.f, c = 0.f;
    if (valid) {
      h = p.h0 ? p.h0[bb * H + u] : 0.f;
      c = p.c0 ? p.c0[bb * H + u] : 0.f;
      p.h_save[bb * H + u] = h;
      p.c_save[bb * H + u] = c;
    }
    cst = c;
    stg0[ul * XS + s] = h;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  if (tid < kWC) cbulk_s2c(cpeer(rx + j * kWUC * XS, (uint32_t)tid), stg0, sbytes, cpeer(&bars[0], (uint32_t)tid));

  __shared__ int s_fail;
  int64_t waited = 0;
  bool fail = false;
  for (int64_t t = 0; t < T && !fail; ++t) {
    const int par = (int)(t & 1);
    float zg[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
      const float *zr = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
      for (int g = 0; g < 4; ++g) zg[g] = zr[g * H];
    }
    if (tid == 0) {
      s_fail = !cmbar_wait(&bars[par], (uint32_t)((t >> 1) & 1), p.status);
      if (!s_fail) {
        ++waited;
        if (t + 2 < T) cmbar_arrive_expect(&bars[par], kWC * sbytes);
      }
    }
    __syncthreads();
    if (s_fail) { fail = true; break; }
    const float *X = rx + par * kWH * XS;  // h_{t-1} [512][XS]
    float acc[4][S];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int b = 0; b < S; ++b) acc[r][b] = 0.f;
#pragma unroll
    for (int i = 0; i < KR; ++i) {
      float xv[S];
      wide_ldx<S, XS>(X + (16 * i + q) * XS, xv);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int b = 0; b < S; ++b) acc[r][b] = fmaf(wr[r][i], xv[b], acc[r][b]);
    }
#pragma unroll 4
    for (int i = KR; i < 32; ++i) {
      const int k = 16 * i + q;
      const float4 wv = *reinterpret_cast<const float4 *>(Ws + (k - 16 * KR) * kWR + r0);
      const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
      float xv[S];
      wide_ldx<S, XS>(X + k * XS, xv);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int b = 0; b < S; ++b) acc[r][b] = fmaf(w4[r], xv[b], acc[r][b]);
    }
    float v[S];
    wide_reduce4<S>(acc, lane, v);
    {  // row r0 + ks = unit 8 (warp & 3) + (lane & 7), gate ks: unit-contiguous for the cells' reads
      float *dst = red + (kgw * 4 + ks) * S * kWUC + 8 * (warp & 3) + (lane & 7);
#pragma unroll
      for (int b = 0; b < S; ++b) dst[b * kWUC] = v[b];
    }
    __syncthreads();
    // cells; h_t into staging block par (outputs no other CTA reads are
    // stored after the send)
    float *stg = stage + par * kWUC * XS;
    float act[4] = {0.f, 0.f, 0.f, 0.f}, hv = 0.f;
    if (is_cell) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float sum = 0.f;
#pragma unroll
        for (int kq = 0; kq < 4; ++kq) sum += red[((kq * 4 + g) * S + s) * kWUC + ul];
        act[g] = sigf(zg[g] + sum + bias[ul * 4 + g]);
      }
      const float c = fmaf(act[1], cst, act[0] * act[2]);
      hv = act[3] * tanh_any(c);
      cst = c;
      stg[ul * XS + s] = valid ? hv : 0.f;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid < kWC && t + 1 < T)
      cbulk_s2c(cpeer(rx + (par ^ 1) * kWH * XS + j * kWUC * XS, (uint32_t)tid), stg, sbytes,
                cpeer(&bars[par ^ 1], (uint32_t)tid));
    if (valid) {
      float *ar = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
      for (int g = 0; g < 4; ++g) ar[g * H] = act[g];
      p.h_save[((t + 1) * Bt + bb) * H + u] = hv;
      p.c_save[((t + 1) * Bt + bb) * H + u] = cst;
    }
  }
  if (tid == 0 && fail) {
    for (int64_t u2 = waited; u2 < std::min<int64_t>(T, waited + 2); ++u2)
      cmbar_drain(&bars[u2 & 1], (uint32_t)((u2 >> 1) & 1));
  }
  __syncthreads();
  ccluster_sync();
}

template <int S>
__global__ void __launch_bounds__(kWT, 1) rcw_bwd_kernel(RwArgs p) {
  using L = WideBwd<S>;
  constexpr int XS = L::XS, KR = L::KR;
  constexpr int64_t H = kWH;
  constexpr uint32_t bbytes = S * kWUC * 4;  // one block: S sequences x 32 units
  extern __shared__ __align__(16) float smw[];
  float *Ws = smw + L::o_w, *rx = smw + L::o_rx, *stage = smw + L::o_stage, *DG = smw + L::o_dg;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smw + L::o_bars);
  const uint32_t j = crank();
  const int64_t T = p.T, Bt = p.Bt;
  const int64_t b0 = (int64_t)(blockIdx.x / kWC) * S;
  const int Bc = (int)min((int64_t)S, Bt - b0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // product: units u0..u0+3 (CTA warp's units), rows k = 4 i + ks, i < 32
  const int ks = lane >> 3, u0 = 32 * warp + 4 * (lane & 7);
  const float *wj = p.w + (size_t)j * kWR * kWH;  // [128 rows][512 units]
  {
    const float4 *src = reinterpret_cast<const float4 *>(wj + 4 * KR * kWH);
    for (int i = tid; i < L::KS * kWH / 4; i += kWT) reinterpret_cast<float4 *>(Ws)[i] = src[i];
  }
  float wr[4][KR];
#pragma unroll
  for (int i = 0; i < KR; ++i) {
    const float4 v = *reinterpret_cast<const float4 *>(wj + (size_t)(4 * i + ks) * kWH + u0);
    wr[0][i] = v.x;
    wr[1][i] = v.y;
    wr[2][i] = v.z;
    wr[3][i] = v.w;
  }
  if (tid == 0) {
    cmbar_init(&bars[0], 1);
    cmbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // step T-1 sends into parity (T-2)&1, read by step T-2; one use each to start
    cmbar_arrive_expect(&bars[0], kWC * bbytes);
    cmbar_arrive_expect(&bars[1], kWC * bbytes);
  }
  __syncthreads();
  ccluster_sync();

  const bool is_cell = tid < kWUC * S;
  const int ul = tid & 31, s = tid >> 5;
  const bool valid = is_cell && s < Bc;
  const int64_t u = (int64_t)j * kWUC + ul, bb = b0 + s;
  float dcst = (valid && p.dc_n) ? p.dc_n[bb * H + u] : 0.f;
  __shared__ int s_fail;
  int64_t waited = 0;
  bool fail = false;
  for (int64_t t = T - 1; t >= 0 && !fail; --t) {
    const int par = (int)(t & 1);  // the blocks for step t arrived in rx[par]
    float ld[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // i, f, g, o, c_t, c_{t-1}, dh
    if (valid) {
      const float *ar = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
      for (int g = 0; g < 4; ++g) ld[g] = ar[g * H];
      ld[4] = p.c_save[((t + 1) * Bt + bb) * H + u];
      ld[5] = p.c_save[(t * Bt + bb) * H + u];
      ld[6] = p.dout[(t * Bt + bb) * H + u] + ((t == T - 1 && p.dh_n) ? p.dh_n[bb * H + u] : 0.f);
    }
    if (t < T - 1) {
      const int64_t use = (T - 2 - t) >> 1;
      if (tid == 0) {
        s_fail = !cmbar_wait(&bars[par], (uint32_t)(use & 1), p.status);
        if (!s_fail) {
          ++waited;
          if (t - 2 >= 0) cmbar_arrive_expect(&bars[par], kWC * bbytes);
        }
      }
      __syncthreads();
      if (s_fail) { fail = true; break; }
    }
    float dg[4] = {0.f, 0.f, 0.f, 0.f};
    if (is_cell) {
      float dh = ld[6];
      if (t < T - 1) {
        const float *R = rx + (par * kWC * S + s) * kWUC + ul;
#pragma unroll
        for (int src = 0; src < kWC; ++src) dh += R[src * S * kWUC];
      }
      const float i = ld[0], f = ld[1], g = ld[2], o = ld[3];
      const float th = tanh_any(ld[4]);
      const float dct = dcst + dh * o * (1.f - th * th);
      dg[0] = dct * g * i * (1.f - i);
      dg[1] = dct * ld[5] * f * (1.f - f);
      dg[2] = dct * i * g * (1.f - g);
      dg[3] = dh * th * o * (1.f - o);
      dcst = dct * f;
#pragma unroll
      for (int q = 0; q < 4; ++q) DG[(q * kWUC + ul) * XS + s] = valid ? dg[q] : 0.f;
    }
    __syncthreads();
    if (t > 0) {
      // this CTA's rows' share of dh_{t-1} for the units of CTA warp
      float acc[4][S];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int b = 0; b < S; ++b) acc[r][b] = 0.f;
#pragma unroll
      for (int i = 0; i < KR; ++i) {
        float xv[S];
        wide_ldx<S, XS>(DG + (4 * i + ks) * XS, xv);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int b = 0; b < S; ++b) acc[r][b] = fmaf(wr[r][i], xv[b], acc[r][b]);
      }
#pragma unroll 4
      for (int i = KR; i < 32; ++i) {
        const int k = 4 * i + ks;
        const float4 wv = *reinterpret_cast<const float4 *>(Ws + (k - 4 * KR) * kWH + u0);
        const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
        float xv[S];
        wide_ldx<S, XS>(DG + k * XS, xv);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int b = 0; b < S; ++b) acc[r][b] = fmaf(w4[r], xv[b], acc[r][b]);
      }
      float v[S];
      wide_reduce4<S>(acc, lane, v);
      // staging block par of receiver warp (reused two steps later, after
      // that receiver has sent blocks that needed this one)
      float *blk = stage + (par * kWC + warp) * S * kWUC;
#pragma unroll
      for (int b = 0; b < S; ++b) blk[b * kWUC + 4 * (lane & 7) + ks] = v[b];
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0)
        cbulk_s2c(cpeer(rx + ((par ^ 1) * kWC + j) * S * kWUC, (uint32_t)warp), blk, bbytes,
                  cpeer(&bars[par ^ 1], (uint32_t)warp));
    }
    if (valid) {
      float *ar = p.zacts + (t * Bt + bb) * 4 * H + u;
#pragma unroll
      for (int q = 0; q < 4; ++q) ar[q * H] = dg[q];
    }
  }
  if (tid == 0 && fail) {
    for (int64_t u2 = waited; u2 < std::min<int64_t>(T - 1, waited + 2); ++u2) {
      const int64_t t2 = T - 2 - u2;  // the step that reads the use-u2 blocks
      cmbar_drain(&bars[t2 & 1], (uint32_t)(((T - 2 - t2) >> 1) & 1));
    }
  }
  __syncthreads();
  ccluster_sync();
}

// Backward weights of the wide kernels: [16][128 rows][512 units], row
// g*32+ul of CTA jc = a[g] W_hh[g H + 32 jc + ul][u].
__global__ void rcw_prep_bwd_kernel(const float *__restrict__ w_hh, const float *__restrict__ a,
                                    float *__restrict__ wb) {
  const int64_t n = (int64_t)4 * kWH * kWH;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t uu = i % kWH;
    const int row = (int)((i / kWH) % kWR);
    const int64_t jc = i / ((int64_t)kWH * kWR);
    const int g = row / kWUC, ul = row % kWUC;
    wb[i] = a[g] * w_hh[((int64_t)g * kWH + jc * kWUC + ul) * kWH + uu];
  }
}

// Weights of the cluster kernels: forward [C][H][4UC], row ul*4+g =
// a[g] W_hh[g H + j UC + ul][k]; backward [C][4H][UC], row u*4+g =
// a[g] W_hh[g H + u][j UC + ul]; bias [C][4UC] = a[g] b_hh[g H + j UC + ul].
__global__ void rcl_prep_kernel(const float *__restrict__ w_hh, const float *__restrict__ b_hh,
                                const float *__restrict__ a, float *__restrict__ wf, float *__restrict__ bias,
                                float *__restrict__ wb, int64_t H, int C, int UC) {
  const int64_t n = 4 * H * H;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (wf) {  // forward: i = (jc, k, row)
      const int R = 4 * UC;
      const int row = (int)(i % R);
      const int64_t k = (i / R) % H;
      const int jc = (int)(i / (R * H));
      const int ul = row / 4, g = row % 4;
      wf[i] = a[g] * w_hh[(g * H + (int64_t)jc * UC + ul) * H + k];
    }
    if (wb) {  // backward: i = (jc, row, ul)
      const int ul = (int)(i % UC);
      const int64_t row = (i / UC) % (4 * H);
      const int jc = (int)(i / (UC * 4 * H));
      const int64_t u = row / 4;
      const int g = (int)(row % 4);
      wb[i] = a[g] * w_hh[(g * H + u) * H + (int64_t)jc * UC + ul];
    }
  }
  if (bias) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < 4 * H; i += stride) {
      const int R = 4 * UC;
      const int row = (int)(i % R), jc = (int)(i / R);
      bias[i] = a[row % 4] * b_hh[(row % 4) * H + (int64_t)jc * UC + row / 4];
    }
  }
}

struct RclPlan {
  int C, UC;
  size_t smem_f, smem_b;
  size_t o_wf, o_bias, o_wb, total;
};

std::atomic<unsigned long long> g_rcl_attr[2];

// Clusters of 16 CTAs (non-portable; half the product per CTA) where the
// device runs them with this shared memory, else 8: H = C UC with UC even,
// the thread blocks and k groups dividing the product evenly.
// HS_RCL_CLUSTER=8 forces 8.
int rcl_clusters_fit(int C, size_t smem_f, size_t smem_b);

bool make_rcl_plan(RclPlan &pl, int64_t H, bool check_fit = true) {
  if (H <= 0 || H > 128) return false;
  const char *force = getenv("HS_RCL_CLUSTER");
  for (int C : {16, 8}) {
    if (force && force[0] == '8' && C != 8) continue;
    if (H % C) continue;
    const int UC = (int)(H / C);
    if (UC < 2 || UC % 2 || UC * kBC > 4 * kCT) continue;
    const int nf = UC * 8, nb = (UC / 2) * 8;
    if (kCT % nf || kCT % nb) continue;
    const int KGf = kCT / nf, KGb = kCT / nb;
    if (H % KGf || (4 * H) % KGb) continue;
    const CLayout Lf = clayout(4 * UC, (int)H, KGf, UC * kBC, C);
    const CLayout Lb = clayout(UC, (int)(4 * H), KGb, 4 * UC * kBC, C);
    if ((size_t)Lf.total > 200 * 1024 || (size_t)Lb.total > 200 * 1024) continue;
    if (check_fit && !rcl_clusters_fit(C, Lf.total, Lb.total)) continue;
    pl.C = C;
    pl.UC = UC;
    pl.smem_f = Lf.total;
    pl.smem_b = Lb.total;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = round_up(off + bytes, 256); return o; };
    pl.o_wf = take((size_t)4 * H * H * 4);
    pl.o_bias = take((size_t)4 * H * 4);
    pl.o_wb = take((size_t)4 * H * H * 4);
    pl.total = off;
    return true;
  }
  return false;
}

// Kernel attributes for a cluster size: dynamic shared memory up to what the
// kernel may need, non-portable cluster sizes allowed.
// Set once per device (bit dev of *attr for the shared memory, of
// g_rcl_np for the cluster size), so that launches inside a stream capture
// make no attribute calls.
std::atomic<unsigned long long> g_rcl_np[2];
int rcl_prepare_fn(const void *fn, std::atomic<unsigned long long> *attr) {
  if (int e = allow_dynamic_smem(fn, 200 * 1024, attr)) return e;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
  std::atomic<unsigned long long> &np = g_rcl_np[attr == &g_rcl_attr[0] ? 0 : 1];
  const unsigned long long bit = 1ull << (dev & 63);
  if (np.load(std::memory_order_acquire) & bit) return HS_OK;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(non-portable cluster)");
  np.fetch_or(bit, std::memory_order_acq_rel);
  return HS_OK;
}

// Whether one cluster of C CTAs of each direction's kernel fits on the
// current device with these shared-memory sizes (cached per device and size).
int rcl_clusters_fit(int C, size_t smem_f, size_t smem_b) {
  struct Entry { int dev, C; size_t f, b; int ok; };
  static std::mutex mu;
  static Entry cache[32];
  static int n = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (cache[i].dev == dev && cache[i].C == C && cache[i].f == smem_f && cache[i].b == smem_b) return cache[i].ok;
  int ok = 1;
  const void *fns[2] = {(const void *)rcl_fwd_kernel, (const void *)rcl_bwd_kernel};
  const size_t sm[2] = {smem_f, smem_b};
  for (int d = 0; d < 2 && ok; ++d) {
    if (rcl_prepare_fn(fns[d], &g_rcl_attr[d]) != HS_OK) { (void)cudaGetLastError(); ok = 0; break; }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)C);
    cfg.blockDim = dim3(kCT);
    cfg.dynamicSmemBytes = sm[d];
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)C;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, fns[d], &cfg) != cudaSuccess || nc < 1) {
      (void)cudaGetLastError();
      ok = 0;
    }
  }
  if (n < 32) cache[n++] = Entry{dev, C, smem_f, smem_b, ok};
  return ok;
}

int rcl_launch(const void *fn, int C, int ngrp, size_t smem, std::atomic<unsigned long long> *attr, RclArgs &args,
               cudaStream_t st) {
  if (int e = rcl_prepare_fn(fn, attr)) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(C * ngrp));
  cfg.blockDim = dim3(kCT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)C;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  void *kargs[] = {&args};
  if (cudaLaunchKernelExC(&cfg, fn, kargs) != cudaSuccess) return check_launch("cudaLaunchKernelEx(rcl)");
  return HS_OK;
}

// HS_REC_PATH=cluster forces this path where it applies, =ffma|tc excludes it.
int rcl_override() {
  const char *e = getenv("HS_REC_PATH");
  if (!e) return 0;
  if (e[0] == 'c') return 1;
  return 2;
}

// ------------------------------------------------------------ wide: host side
const void *rcw_fn(int dir, int S) {
#define HS_RCW_CASE(n) \
  case n:              \
    return dir ? (const void *)rcw_bwd_kernel<n> : (const void *)rcw_fwd_kernel<n>;
  switch (S) {
    HS_RCW_CASE(1) HS_RCW_CASE(2) HS_RCW_CASE(3) HS_RCW_CASE(4)
    HS_RCW_CASE(5) HS_RCW_CASE(6) HS_RCW_CASE(7) HS_RCW_CASE(8)
    default: return nullptr;
  }
#undef HS_RCW_CASE
}
size_t rcw_smem(int dir, int S) {
#define HS_RCW_CASE(n) \
  case n:              \
    return dir ? (size_t)WideBwd<n>::bytes : (size_t)WideFwd<n>::bytes;
  switch (S) {
    HS_RCW_CASE(1) HS_RCW_CASE(2) HS_RCW_CASE(3) HS_RCW_CASE(4)
    HS_RCW_CASE(5) HS_RCW_CASE(6) HS_RCW_CASE(7) HS_RCW_CASE(8)
    default: return 0;
  }
#undef HS_RCW_CASE
}

// Attributes of one wide kernel (its shared memory, clusters of 16), set once
// per device so that launches inside a stream capture make no attribute calls.
std::atomic<unsigned long long> g_rcw_attr[2][kWMaxS + 1];
int rcw_prepare(int dir, int S) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
  std::atomic<unsigned long long> &done = g_rcw_attr[dir][S];
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return HS_OK;
  const void *fn = rcw_fn(dir, S);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rcw_smem(dir, S)) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(wide recurrent shared memory)");
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(non-portable cluster)");
  done.fetch_or(bit, std::memory_order_acq_rel);
  return HS_OK;
}

cudaLaunchConfig_t rcw_config(int dir, int S, int ngrp, cudaStream_t st, cudaLaunchAttribute *at) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(kWC * ngrp));
  cfg.blockDim = dim3(kWT);
  cfg.dynamicSmemBytes = rcw_smem(dir, S);
  cfg.stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)kWC;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cfg;
}

// Clusters of 16 that the device runs at once with the wide kernels (both
// directions, the largest shared-memory variant; every variant runs one CTA
// per SM), cached per device; 0 where they do not run.
int rcw_max_clusters() {
  static std::mutex mu;
  static int cache[64];
  static bool have[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { (void)cudaGetLastError(); return 0; }
  std::lock_guard<std::mutex> lock(mu);
  if (have[dev & 63]) return cache[dev & 63];
  int best = 1 << 30;
  for (int d = 0; d < 2; ++d) {
    int nc = 0;
    cudaLaunchAttribute at[1];
    cudaLaunchConfig_t cfg = rcw_config(d, kWMaxS, 1, nullptr, at);
    if (rcw_prepare(d, kWMaxS) != HS_OK ||
        cudaOccupancyMaxActiveClusters(&nc, rcw_fn(d, kWMaxS), &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      nc = 0;
    }
    best = std::min(best, nc);
  }
  cache[dev & 63] = best;
  have[dev & 63] = true;
  return best;
}

// Sequences per cluster: the batch over every cluster that runs at once, at
// most kWMaxS per cluster.  A larger batch would run as further waves of
// clusters (independent of one another: a cluster waits only on its own
// CTAs); by default it goes to the other kernels instead (at B = 64 the two
// measured level, 3.25 against 3.23 M tokens/s), HS_REC_PATH=cluster takes
// the waves.
bool rcw_plan(int64_t B, int64_t H, int &S, int &ngrp) {
  if (H != kWH || B <= 0) return false;
  const int ncl = rcw_max_clusters();
  if (ncl < 1) return false;
  const int64_t s = (B + ncl - 1) / ncl;
  if (s > kWMaxS && rcl_override() != 1) return false;
  S = (int)std::min<int64_t>(s, kWMaxS);
  ngrp = (int)((B + S - 1) / S);
  return true;
}

size_t rcw_o_bias() { return round_up((size_t)4 * kWH * kWH * 4, 256); }
size_t rcw_o_wb() { return rcw_o_bias() + round_up((size_t)4 * kWH * 4, 256); }

int rcw_launch(int dir, int S, int ngrp, RwArgs &args, cudaStream_t st) {
  if (int e = rcw_prepare(dir, S)) return e;
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t cfg = rcw_config(dir, S, ngrp, st, at);
  void *kargs[] = {&args};
  if (cudaLaunchKernelExC(&cfg, rcw_fn(dir, S), kargs) != cudaSuccess)
    return check_launch("cudaLaunchKernelEx(wide recurrent)");
  return HS_OK;
}

}  // namespace

bool rec_cluster_wanted(int64_t B, int64_t H) {
  (void)B;
  if (rcl_override() == 2) return false;
  RclPlan pl;
  return make_rcl_plan(pl, H);
}

size_t rec_cluster_ws_bytes(int64_t H) {
  RclPlan pl;
  return make_rcl_plan(pl, H) ? pl.total : 0;
}

// acts holds Z on entry (the input projection) and the gate activations on return.
int rec_cluster_forward(const float *h0, const float *c0, const float *w_hh, const float *b_hh, const float *a,
                        float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t H, void *ws,
                        size_t ws_bytes, int *status, cudaStream_t st) {
  RclPlan pl;
  if (!make_rcl_plan(pl, H)) return fail(HS_ERR_UNSUPPORTED, "recurrent (cluster): H=%lld", (long long)H);
  if (!ws || ws_bytes < pl.total || !aligned(ws, 256))
    return fail(HS_ERR_WORKSPACE, "recurrent (cluster): workspace %zu < %zu bytes", ws_bytes, pl.total);
  char *w = static_cast<char *>(ws);
  float *wf = reinterpret_cast<float *>(w + pl.o_wf), *bias = reinterpret_cast<float *>(w + pl.o_bias);
  rcl_prep_kernel<<<(unsigned)std::min<int64_t>((4 * H * H + 255) / 256, 1024), 256, 0, st>>>(w_hh, b_hh, a, wf, bias,
                                                                                          nullptr, H, pl.C, pl.UC);
  if (int e = check_launch("rcl_prep_kernel")) return e;
  RclArgs args{};
  args.w = wf;
  args.bias = bias;
  args.zacts = acts;
  args.h0 = h0;
  args.c0 = c0;
  args.h_save = h_save;
  args.c_save = c_save;
  args.status = status;
  args.T = T;
  args.Bt = B;
  args.H = H;
  args.C = pl.C;
  args.UC = pl.UC;
  const int ngrp = (int)((B + kBC - 1) / kBC);
  return rcl_launch((const void *)rcl_fwd_kernel, pl.C, ngrp, pl.smem_f, &g_rcl_attr[0], args, st);
}

// acts holds the forward's gate activations on entry and dgates on return.
int rec_cluster_backward(const float *w_hh, const float *a, const float *c_save, float *acts, const float *dout,
                         const float *dh_n, const float *dc_n, int64_t T, int64_t B, int64_t H, void *ws,
                         size_t ws_bytes, int *status, cudaStream_t st) {
  RclPlan pl;
  if (!make_rcl_plan(pl, H)) return fail(HS_ERR_UNSUPPORTED, "recurrent backward (cluster): H=%lld", (long long)H);
  if (!ws || ws_bytes < pl.total || !aligned(ws, 256))
    return fail(HS_ERR_WORKSPACE, "recurrent backward (cluster): workspace %zu < %zu bytes", ws_bytes, pl.total);
  char *w = static_cast<char *>(ws);
  float *wb = reinterpret_cast<float *>(w + pl.o_wb);
  rcl_prep_kernel<<<(unsigned)std::min<int64_t>((4 * H * H + 255) / 256, 1024), 256, 0, st>>>(
      w_hh, nullptr, a, nullptr, nullptr, wb, H, pl.C, pl.UC);
  if (int e = check_launch("rcl_prep_kernel")) return e;
  RclArgs args{};
  args.w = wb;
  args.zacts = acts;
  args.c_save = const_cast<float *>(c_save);
  args.dout = dout;
  args.dh_n = dh_n;
  args.dc_n = dc_n;
  args.status = status;
  args.T = T;
  args.Bt = B;
  args.H = H;
  args.C = pl.C;
  args.UC = pl.UC;
  const int ngrp = (int)((B + kBC - 1) / kBC);
  return rcl_launch((const void *)rcl_bwd_kernel, pl.C, ngrp, pl.smem_b, &g_rcl_attr[1], args, st);
}


// H = 512 on clusters of 16 with a few sequences per cluster (rcw_* kernels).
bool rec_wide_wanted(int64_t B, int64_t H) {
  if (H != kWH || rcl_override() == 2) return false;
  int S = 0, ngrp = 0;
  return rcw_plan(B, H, S, ngrp);
}

size_t rec_wide_ws_bytes(int64_t H) {
  return H == kWH ? rcw_o_wb() + round_up((size_t)4 * kWH * kWH * 4, 256) : 0;
}

// acts holds Z on entry (the input projection) and the gate activations on return.
int rec_wide_forward(const float *h0, const float *c0, const float *w_hh, const float *b_hh, const float *a,
                     float *h_save, float *c_save, float *acts, int64_t T, int64_t B, int64_t H, void *ws,
                     size_t ws_bytes, int *status, cudaStream_t st) {
  int S = 0, ngrp = 0;
  if (!rcw_plan(B, H, S, ngrp))
    return fail(HS_ERR_UNSUPPORTED, "recurrent (wide cluster): B=%lld H=%lld", (long long)B, (long long)H);
  const size_t need = rec_wide_ws_bytes(H);
  if (!ws || ws_bytes < need || !aligned(ws, 256))
    return fail(HS_ERR_WORKSPACE, "recurrent (wide cluster): workspace %zu < %zu bytes", ws_bytes, need);
  char *w = static_cast<char *>(ws);
  float *wf = reinterpret_cast<float *>(w), *bias = reinterpret_cast<float *>(w + rcw_o_bias());
  rcl_prep_kernel<<<1024, 256, 0, st>>>(w_hh, b_hh, a, wf, bias, nullptr, H, kWC, kWUC);
  if (int e = check_launch("rcl_prep_kernel")) return e;
  RwArgs args{};
  args.w = wf;
  args.bias = bias;
  args.zacts = acts;
  args.h0 = h0;
  args.c0 = c0;
  args.h_save = h_save;
  args.c_save = c_save;
  args.status = status;
  args.T = T;
  args.Bt = B;
  return rcw_launch(0, S, ngrp, args, st);
}

// acts holds the forward's gate activations on entry and dgates on return.
int rec_wide_backward(const float *w_hh, const float *a, const float *c_save, float *acts, const float *dout,
                      const float *dh_n, const float *dc_n, int64_t T, int64_t B, int64_t H, void *ws,
                      size_t ws_bytes, int *status, cudaStream_t st) {
  int S = 0, ngrp = 0;
  if (!rcw_plan(B, H, S, ngrp))
    return fail(HS_ERR_UNSUPPORTED, "recurrent backward (wide cluster): B=%lld H=%lld", (long long)B, (long long)H);
  const size_t need = rec_wide_ws_bytes(H);
  if (!ws || ws_bytes < need || !aligned(ws, 256))
    return fail(HS_ERR_WORKSPACE, "recurrent backward (wide cluster): workspace %zu < %zu bytes", ws_bytes, need);
  float *wb = reinterpret_cast<float *>(static_cast<char *>(ws) + rcw_o_wb());
  rcw_prep_bwd_kernel<<<1024, 256, 0, st>>>(w_hh, a, wb);
  if (int e = check_launch("rcw_prep_bwd_kernel")) return e;
  RwArgs args{};
  args.w = wb;
  args.zacts = acts;
  args.c_save = const_cast<float *>(c_save);
  args.dout = dout;
  args.dh_n = dh_n;
  args.dc_n = dc_n;
  args.status = status;
  args.T = T;
  args.Bt = B;
  return rcw_launch(1, S, ngrp, args, st);
}

}  // namespace hs
