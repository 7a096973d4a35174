// Device helpers of the tcgen05 / TMA kernels (shared memory barriers,
// tensor-map copies, shared-memory matrix descriptors, TMEM loads, 2-SM
// cluster signals) and the host's tensor-map encoder.  Every TMA copy here
// targets this GPU's own memory; none uses cluster multicast.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "hs_common.cuh"

namespace hs {
namespace {

HS_DEV uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

HS_DEV void mbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
HS_DEV void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
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
// Bounded wait on a phase; gives up (status set) after kWaitLimitNs or as
// soon as another CTA has recorded a failure.
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

// Output maps are 3D {N, M, splits}: a split-K partial is clipped to its own
// M rows, and the unsplit output is the splits = 1 case.
HS_DEV void tma_store_3d(const CUtensorMap *tm, const void *src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(tm),
               "r"(c0), "r"(c1), "r"(c2), "r"(su32(src))
               : "memory");
}
HS_DEV void tma_reduce_add_3d(const CUtensorMap *tm, const void *src, int c0, int c1, int c2) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(tm),
      "r"(c0), "r"(c1), "r"(c2), "r"(su32(src))
      : "memory");
}

// Shared-memory matrix descriptor (sm100 version bits).  Layout type 2 is
// the 128-byte swizzle of K-major tiles (16-byte chunks XOR row%8); layout
// type 1 is the 128-byte swizzle with 32-byte atoms (32-byte chunks XOR
// row%4), the only layout tf32 accepts for M/N-major operands.
HS_DEV uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

HS_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

HS_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

HS_DEV void named_sync(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

HS_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HS_DEV uint32_t cluster_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(su32(p)), "r"(rank));
  return r;
}
// Arrive on a barrier of either CTA of the cluster (default semantics:
// release at CTA scope, no cluster-wide fence).
HS_DEV void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
HS_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Load into this CTA's shared memory; completion bytes counted on the
// barrier at cluster address bar (the first CTA's).
HS_DEV void tma_2d_pair(void *dst, const CUtensorMap *tm, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(su32(dst)),
      "l"(tm), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
HS_DEV void mma_f16_pair(uint32_t dt, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dt),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
HS_DEV void mma_commit_pair(uint64_t *b) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
               : "memory");
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

}  // namespace
}  // namespace hs
