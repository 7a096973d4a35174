// Chunk maps of the parallel-mode scan, for a sequence split over time
// across GPUs (each rank scans its own chunk of T).
//
// The scan (reference src/headstartlstm/_parallel.py:21-35, evaluated here as
// the clamped linear recurrence c_t = f'_t c_{t-1} + b'_t with f' = max(f,eps),
// b' = max(i g, eps)) is affine in its carry, so a chunk of steps acts on the
// state entering it as c -> A c + C, with A the product of the chunk's f' and
// C the chunk's last state from a zero carry.  Its backward acts on the
// gradient arriving at the chunk's last state as e -> A e + D, with D the
// gradient the chunk passes to the state before it from a zero incoming
// gradient (the same A).  One thread per column (sequence, hidden unit), a
// sequential loop over the chunk's steps with coalesced rows.  The carries
// between chunks then follow from all ranks' maps; each rank runs the
// ordinary scan with its carry as c0 (forward) or dc_n (backward).
#include "hs_common.cuh"

namespace hs {
namespace {

__global__ void __launch_bounds__(256) chunk_maps_kernel(const float *__restrict__ z, const float *__restrict__ c,
                                                         const float *__restrict__ dout,
                                                         const float *__restrict__ dh_last, int64_t T, int64_t B,
                                                         int64_t H, float eps, float *__restrict__ A,
                                                         float *__restrict__ CD, int backward) {
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= B * H) return;
  const int64_t b = col / H, h = col - b * H;
  const int64_t zs = B * 4 * H, ss = B * H;
  const float *zr = z + b * 4 * H + h;
  float a = 1.f, v = 0.f;
  if (!backward) {
#pragma unroll 8
    for (int64_t t = 0; t < T; ++t) {
      const float *r = zr + t * zs;
      const float f = fmaxf(sigf(r[H]), eps);
      const float bb = fmaxf(sig_fast(r[0]) * sig_fast(r[2 * H]), eps);
      v = fmaf(f, v, bb);
      a *= f;
    }
  } else {
    const float *cr = c + b * H + h;
    const float *dr = dout + b * H + h;
    const float dhl = dh_last ? dh_last[b * H + h] : 0.f;
#pragma unroll 8
    for (int64_t t = T - 1; t >= 0; --t) {
      const float *r = zr + t * zs;
      const float f = fmaxf(sigf(r[H]), eps);
      const float o = sig_fast(r[3 * H]);
      const float th = tanh_pos(cr[t * ss]);
      const float d = dr[t * ss] + (t == T - 1 ? dhl : 0.f);
      v = f * fmaf(d * o, 1.f - th * th, v);  // e_{t} = f'_t (dcd_t + e_{t+1})
      a *= f;
    }
  }
  A[col] = a;
  CD[col] = v;
}

}  // namespace
}  // namespace hs

extern "C" int hs_scan_chunk_maps(const float *z, const float *c, const float *dout, const float *dh_last, int64_t T,
                                  int64_t B, int64_t H, float eps, float *A, float *CD, int backward,
                                  hs_stream_t stream) {
  if (T <= 0 || B <= 0 || H <= 0)
    return hs::fail(HS_ERR_INVALID_ARG, "hs_scan_chunk_maps: T, B, H must be positive");
  if (!z || !A || !CD || (backward && (!c || !dout)))
    return hs::fail(HS_ERR_INVALID_ARG, "hs_scan_chunk_maps: null required pointer");
  const int64_t n = B * H;
  hs::chunk_maps_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(z, c, dout, dh_last, T, B, H,
                                                                                     eps, A, CD, backward);
  return hs::check_launch("chunk_maps_kernel");
}
