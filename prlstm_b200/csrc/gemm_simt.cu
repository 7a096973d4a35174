// fp32 FFMA GEMM for the linear-layer products of HeadStartLSTM.
//
// Used for every shape the tensor-core path (gemm_tc.cu) does not take:
// small or ragged M/N/K (the reference's own test shapes have D=8, H=12),
// and as the exact-fp32 cross-check of that path.
//
// C[M,N] = sum_k A(m,k) B(k,n), with each operand either K-contiguous or
// M/N-contiguous, covering the three products of a linear layer:
//   forward  y  = x  w^T    A = x  [M,K] K-contig, B = w [N,K] K-contig
//   dgrad    dx = dy w      A = dy [M,N] K-contig, B = w [N,K] N-contig
//   wgrad    dw = dy^T x    A = dy [M,N] M-contig, B = x [M,K] N-contig
// 128x128 output tile per 256-thread CTA, 8x8 outputs per thread, k-step 8,
// register-prefetched double buffering of the shared-memory tiles.  Shapes
// with few output tiles and a long K (the gradient products of a short
// recurrent sequence: N = D or H, K = T*B) split K over blockIdx.z into
// partial tiles in caller scratch, added in a fixed order by a second pass.
#include <algorithm>

#include "hs_common.cuh"

namespace hs {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, NT = 256;

struct GemmArgs {
  const float *A, *B;
  float *C;
  const float *bias;   // [N] or null
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
  int a_kcontig, b_kcontig;
  int beta;            // 0 or 1: C = beta*C + A.B (+bias)
  float *partial;      // split-K: [splits][M][N], or null
  int64_t kps;         // k per split (multiple of BK)
};

__device__ __forceinline__ float ldA(const GemmArgs &g, int64_t m, int64_t k) {
  if (m >= g.M || k >= g.K) return 0.f;
  return g.a_kcontig ? g.A[m * g.lda + k] : g.A[k * g.lda + m];
}
__device__ __forceinline__ float ldB(const GemmArgs &g, int64_t k, int64_t n) {
  if (n >= g.N || k >= g.K) return 0.f;
  return g.b_kcontig ? g.B[n * g.ldb + k] : g.B[k * g.ldb + n];
}

__global__ void __launch_bounds__(NT) gemm_simt_kernel(GemmArgs g) {
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t kbeg = (int64_t)blockIdx.z * g.kps, kend = min(g.K, kbeg + g.kps);

  // Load mapping: 1024 elements per operand tile, 4 per thread.  For a
  // K-contiguous operand consecutive threads walk k first; otherwise m/n.
  float ra[4], rb[4];
  auto gload = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * NT;
      int mm, kk;
      if (g.a_kcontig) { mm = e / BK; kk = e % BK; } else { mm = e % BM; kk = e / BM; }
      ra[i] = (k0 + kk < kend) ? ldA(g, m0 + mm, k0 + kk) : 0.f;
      int nn, kb;
      if (g.b_kcontig) { nn = e / BK; kb = e % BK; } else { nn = e % BN; kb = e / BN; }
      rb[i] = (k0 + kb < kend) ? ldB(g, k0 + kb, n0 + nn) : 0.f;
    }
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * NT;
      int mm, kk;
      if (g.a_kcontig) { mm = e / BK; kk = e % BK; } else { mm = e % BM; kk = e / BM; }
      As[buf][kk][mm] = ra[i];
      int nn, kb;
      if (g.b_kcontig) { nn = e / BK; kb = e % BK; } else { nn = e % BN; kb = e / BN; }
      Bs[buf][kb][nn] = rb[i];
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int64_t nk = (kend - kbeg + BK - 1) / BK;
  gload(kbeg);
  sstore(0);
  __syncthreads();
  for (int64_t kt = 0; kt < nk; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nk) gload(kbeg + (kt + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][k][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][k][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) sstore(buf ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (n >= g.N) continue;
      float v = acc[i][j];
      if (g.partial) {
        g.partial[((int64_t)blockIdx.z * g.M + m) * g.N + n] = v;
        continue;
      }
      if (g.bias) v += g.bias[n];
      float *cp = g.C + m * g.ldc + n;
      if (g.beta) v += *cp;
      *cp = v;
    }
  }
}

// C = beta*C + sum over splits (in order) + bias.
__global__ void simt_splitk_reduce_kernel(const float *__restrict__ part, float *__restrict__ C,
                                          const float *__restrict__ bias, int64_t M, int64_t N, int64_t ldc,
                                          int splits, int beta) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * N; i += stride) {
    float v = 0.f;
    for (int z = 0; z < splits; ++z) v += part[(int64_t)z * M * N + i];
    const int64_t m = i / N, n = i - m * N;
    if (bias) v += bias[n];
    float *cp = C + m * ldc + n;
    if (beta) v += *cp;
    *cp = v;
  }
}

// Column sums in one pass with a fixed summation order: a CTA owns 32
// columns, warp w sums rows w, w+8, ... (coalesced 128-byte rows), and the 8
// warp partials are added in order.
// out[n] = beta*out[n] + sum_m x[m][n]: 32 columns per CTA, 32 warps over
// rows with four independent accumulators each (enough loads in flight to
// stream from HBM), warp partials added in a fixed order.
// With gridDim.y = S > 1 the rows are cut into S slices (slice y: rows
// [y*rps, (y+1)*rps)) whose sums go to part_out[y][n], added in order by
// colsum_parts_kernel.
__global__ void __launch_bounds__(1024) colsum_kernel(const float *__restrict__ x, float *__restrict__ out,
                                                      int64_t M, int64_t N, int beta, float *__restrict__ part_out,
                                                      int64_t rps) {
  __shared__ float part[32][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t n = (int64_t)blockIdx.x * 32 + lane;
  const int64_t r0 = (int64_t)blockIdx.y * rps, r1 = min(M, r0 + rps);
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (n < N) {
    int64_t r = r0 + w;
    for (; r + 96 < r1; r += 128) {
      s0 += x[r * N + n];
      s1 += x[(r + 32) * N + n];
      s2 += x[(r + 64) * N + n];
      s3 += x[(r + 96) * N + n];
    }
    for (; r < r1; r += 32) s0 += x[r * N + n];
  }
  part[w][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (w == 0 && n < N) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) s += part[i][lane];
    if (part_out) part_out[(int64_t)blockIdx.y * N + n] = s;
    else out[n] = beta ? out[n] + s : s;
  }
}

__global__ void colsum_parts_kernel(const float *__restrict__ part, float *__restrict__ out, int64_t N, int S,
                                    int beta) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float s = 0.f;
  for (int y = 0; y < S; ++y) s += part[(int64_t)y * N + n];
  out[n] = beta ? out[n] + s : s;
}

}  // namespace

// ws (may be null): scratch for split-K partials; without enough of it the
// product runs unsplit.
int gemm_simt(const float *A, const float *B, float *C, const float *bias, int64_t M, int64_t N,
              int64_t K, int64_t lda, int64_t ldb, int64_t ldc, bool a_kcontig, bool b_kcontig,
              int beta, cudaStream_t st, void *ws, size_t ws_bytes) {
  if (M == 0 || N == 0) return HS_OK;
  GemmArgs g{A, B, C, bias, M, N, K, lda, ldb, ldc, a_kcontig ? 1 : 0, b_kcontig ? 1 : 0, beta, nullptr, 0};
  const int64_t gy = (M + BM - 1) / BM, gx = (N + BN - 1) / BN;
  if (gy > 65535) return fail(HS_ERR_UNSUPPORTED, "gemm: M=%lld too large for the FFMA path", (long long)M);
  // split K while the tiles fill fewer than ~148 CTAs and every split keeps
  // at least 32 k (4 k-steps)
  const int64_t nkb = (K + BK - 1) / BK;
  int64_t splits = 1;
  while (gx * gy * splits * 2 <= 160 && nkb / (splits * 2) >= 4) splits *= 2;
  while (splits > 1 && (!ws || !aligned(ws, 16) || ws_bytes < (size_t)splits * M * N * 4)) splits /= 2;
  const int64_t kps = (nkb + splits - 1) / splits * BK;
  splits = (K + kps - 1) / kps;
  g.kps = splits > 1 ? kps : K;
  if (splits > 1) g.partial = static_cast<float *>(ws);
  gemm_simt_kernel<<<dim3((unsigned)gx, (unsigned)gy, (unsigned)std::max<int64_t>(1, splits)), NT, 0, st>>>(g);
  if (int e = check_launch("gemm_simt_kernel")) return e;
  if (splits > 1) {
    const int64_t n = M * N;
    simt_splitk_reduce_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1024), 256, 0, st>>>(
        g.partial, C, bias, M, N, ldc, (int)splits, beta);
    return check_launch("simt_splitk_reduce_kernel");
  }
  return HS_OK;
}

// Scratch the split-K partials of an M x N product may use (zero for
// products with enough tiles not to split).
size_t gemm_simt_ws_bound(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  int64_t splits = 1;
  while (tiles * splits * 2 <= 160) splits *= 2;
  return splits > 1 ? (size_t)splits * M * N * 4 : 0;
}

// ws (may be null): with room for S x N floats, the rows are split into S
// slices so that the column blocks and slices fill the GPU.
int colsum(const float *x, float *out, int64_t M, int64_t N, int beta, cudaStream_t st, void *ws,
           size_t ws_bytes) {
  if (N == 0) return HS_OK;
  const int64_t nb = (N + 31) / 32;
  int64_t S = 1;
  while (nb * S * 2 <= 296 && M / (S * 2) >= 512) S *= 2;
  while (S > 1 && (!ws || !aligned(ws, 16) || ws_bytes < (size_t)S * N * 4)) S /= 2;
  const int64_t rps = (M + S - 1) / S;
  float *part = S > 1 ? static_cast<float *>(ws) : nullptr;
  colsum_kernel<<<dim3((unsigned)nb, (unsigned)S), 1024, 0, st>>>(x, out, M, N, beta, part, S > 1 ? rps : M);
  if (int e = check_launch("colsum_kernel")) return e;
  if (S > 1) {
    colsum_parts_kernel<<<(unsigned)((N + 255) / 256), 256, 0, st>>>(part, out, N, (int)S, beta);
    return check_launch("colsum_parts_kernel");
  }
  return HS_OK;
}

}  // namespace hs
