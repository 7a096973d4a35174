// C ABI of the library: argument checks, status handling, the linear-layer
// GEMM entry points and the whole-path parallel-mode calls.
// (Declarations and reference citations: include/headstartlstm_b200.h.)
#include <stdarg.h>
#include <string.h>

#include <algorithm>

#include "hs_common.cuh"

namespace hs {

namespace {
thread_local char g_msg[512] = "";
}

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return HS_OK;
  return fail(HS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int gemm_simt(const float *A, const float *B, float *C, const float *bias, int64_t M, int64_t N,
              int64_t K, int64_t lda, int64_t ldb, int64_t ldc, bool a_kcontig, bool b_kcontig,
              int beta, cudaStream_t st, void *ws, size_t ws_bytes);
size_t gemm_simt_ws_bound(int64_t M, int64_t N);
int gemm_tc_try(const float *A, const float *B, float *C, const float *bias, int64_t M, int64_t N,
                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, bool a_kc, bool b_kc, int beta,
                void *ws, size_t ws_bytes, int *status, cudaStream_t st, bool *done);
size_t gemm_tc_workspace_bound(int64_t M, int64_t N, int64_t K, bool kmajor_both);
bool gemm_h3_enabled();
bool gemm_tc_size_ok(int64_t M, int64_t N, int64_t K);
size_t gemm_h3_partial_bound(int64_t M, int64_t N, int64_t K);
size_t h3_split_bytes(int64_t rows, int64_t cols);
int h3_split(const float *x, int64_t rows, int64_t cols, int64_t ld, unsigned *absmax, void *dst,
             cudaStream_t st);
int h3_split_known(const float *x, int64_t rows, int64_t cols, int64_t ld, const unsigned *absmax, void *dst,
                   cudaStream_t st, const int *gate = nullptr);
int gemm_h3_presplit(const void *a_split, const unsigned *a_absmax, bool a_mn, const void *b_split,
                     const unsigned *b_absmax, bool b_mn, float *C, const float *bias, int64_t M, int64_t N,
                     int64_t K, int64_t ldc, int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st,
                     bool *done);
size_t scan_workspace(int64_t T, int64_t B, int64_t H);
int noalloc_status_word(int **word);
int colsum(const float *x, float *out, int64_t M, int64_t N, int beta, cudaStream_t st, void *ws = nullptr,
           size_t ws_bytes = 0);
int scan_forward(const float *z, const float *c0, float *out, float *c, float *h_n, float *c_n,
                 int64_t T, int64_t B, int64_t H, float eps, void *ws, size_t ws_bytes,
                 int *status, cudaStream_t st, unsigned *kf_max = nullptr);
size_t scan_split_ws_bytes(int64_t T, int64_t B, int64_t H);
size_t proj_scan_ws(int64_t T, int64_t B, int64_t D, int64_t H);
bool proj_scan_shape_ok(int64_t T, int64_t B, int64_t D, int64_t H);
bool proj_scan_wanted(int64_t T, int64_t B, int64_t D, int64_t H);
int proj_scan_forward(const void *x_split, const unsigned *x_scale, const float *w, const float *bias,
                      const float *c0, float *z, float *out, float *c, float *h_n, float *c_n, int64_t T, int64_t B,
                      int64_t D, int64_t H, float eps, void *ws, size_t ws_bytes, unsigned *kf, int *status,
                      cudaStream_t st, bool *took, const char **why = nullptr);
int scan_backward_split(float *z, const float *c, const float *c0, const float *dout, const float *dh_n,
                        const float *dc_n, const unsigned *kf_max, void *dz_split, unsigned *dz_scale, float *dc0,
                        float *db, int64_t T, int64_t B, int64_t H, float eps, void *ws_base, size_t ws_bytes,
                        int *status, cudaStream_t st);
int scan_backward(const float *z, const float *c, const float *c0, const float *dout,
                  const float *dh_n, const float *dc_n, float *dz, float *dc0, float *db,
                  int64_t T, int64_t B, int64_t H, float eps, void *ws, size_t ws_bytes,
                  int *status, cudaStream_t st, unsigned *dz_absmax);

// One GEMM: tensor-core path when it takes the shape, FFMA path otherwise.
static int gemm(const float *A, const float *B, float *C, const float *bias, int64_t M, int64_t N,
                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, bool a_kc, bool b_kc, int beta,
                void *ws, size_t ws_bytes, int *status, cudaStream_t st) {
  bool done = false;
  if (int e = gemm_tc_try(A, B, C, bias, M, N, K, lda, ldb, ldc, a_kc, b_kc, beta, ws, ws_bytes, status,
                          st, &done))
    return e;
  if (done) return HS_OK;
  return gemm_simt(A, B, C, bias, M, N, K, lda, ldb, ldc, a_kc, b_kc, beta, st, ws, ws_bytes);
}

// Scratch any of the three linear-layer products of these extents may use.
size_t linear_backward_ws(int64_t M, int64_t N, int64_t K, int64_t K2);

size_t linear_ws_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return std::max({gemm_tc_workspace_bound(M, N, K, true), gemm_tc_workspace_bound(M, K, N, false),
                   gemm_tc_workspace_bound(N, K, M, false),
                   linear_backward_ws(M, N, K, 0), gemm_simt_ws_bound(M, N), gemm_simt_ws_bound(M, K),
                   gemm_simt_ws_bound(N, K)});
}

static int check_gemm(const void *a, const void *b, const void *c, int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) return fail(HS_ERR_INVALID_ARG, "negative GEMM extent");
  if ((M && N && K) && (!a || !b)) return fail(HS_ERR_INVALID_ARG, "null GEMM operand");
  if (M && N && !c) return fail(HS_ERR_INVALID_ARG, "null GEMM output");
  return HS_OK;
}

int linear_forward(const float *x, const float *w, const float *bias, float *y, int64_t M,
                   int64_t N, int64_t K, void *ws, size_t ws_bytes, int *status, cudaStream_t st) {
  if (int e = check_gemm(x, w, y, M, N, K)) return e;
  return gemm(x, w, y, bias, M, N, K, K, K, N, true, true, 0, ws, ws_bytes, status, st);
}
int linear_dgrad(const float *dy, const float *w, float *dx, int64_t M, int64_t N, int64_t K,
                 void *ws, size_t ws_bytes, int *status, cudaStream_t st) {
  if (int e = check_gemm(dy, w, dx, M, N, K)) return e;
  // dx[M,K] = dy[M,N] . w[N,K]: reduction over N; w is K-contiguous = output-contiguous
  return gemm(dy, w, dx, nullptr, M, K, N, N, K, K, true, false, 0, ws, ws_bytes, status, st);
}
int linear_wgrad(const float *dy, const float *x, float *dw, int64_t M, int64_t N, int64_t K,
                 int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st) {
  if (int e = check_gemm(dy, x, dw, M, N, K)) return e;
  // dw[N,K] = dy[M,N]^T . x[M,K]: reduction over M; both operands output-contiguous
  return gemm(dy, x, dw, nullptr, N, K, M, N, K, K, false, false, beta, ws, ws_bytes, status, st);
}

// Gradient products of y = x.w^T (+ x2.w2^T): dx[M,K] = dy.w (dx may be
// null), dw[N,K] = beta*dw + dy^T.x and, if x2 is given, dw2[N,K2] =
// beta*dw2 + dy^T.x2.  Through the fp16 split, dy is split once and shared
// by all products (K-major for dx, M/N-major for the weight gradients);
// otherwise each product runs on its own.  dy_absmax (device memory, may be
// null) holds an upper bound of max |dy| as float bits, computed by the
// producer of dy; the split then skips its own pass over dy.
size_t linear_backward_ws(int64_t M, int64_t N, int64_t K, int64_t K2) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  size_t sc = 256 + h3_split_bytes(M, N) + h3_split_bytes(M, K) + h3_split_bytes(N, K);
  size_t part = std::max(gemm_h3_partial_bound(M, K, N), gemm_h3_partial_bound(N, K, M));
  if (K2 > 0) {
    sc += h3_split_bytes(M, K2);
    part = std::max(part, gemm_h3_partial_bound(N, K2, M));
  }
  return sc + part;
}

int linear_backward_ex(const float *dy, const float *w, float *dx, const float *x, float *dw, const float *x2,
                       float *dw2, int64_t M, int64_t N, int64_t K, int64_t K2, int beta, void *ws, size_t ws_bytes,
                       int *status, cudaStream_t st, const unsigned *dy_absmax) {
  if (int e = check_gemm(dy, x, dw, N, K, M)) return e;
  if (x2)
    if (int e = check_gemm(dy, x2, dw2, N, K2, M)) return e;
  bool ddx = dx == nullptr, ddw = false, ddw2 = x2 == nullptr;
  size_t sc = 256 + h3_split_bytes(M, N) + h3_split_bytes(M, K) + h3_split_bytes(N, K);
  if (x2) sc += h3_split_bytes(M, K2);
  if (gemm_h3_enabled() && status && gemm_tc_size_ok(M, N, K) && ws && aligned(ws, 256) && ws_bytes >= sc &&
      aligned(dw, 16) && K % 4 == 0 && (!dx || aligned(dx, 16)) && (!x2 || (aligned(dw2, 16) && K2 % 4 == 0))) {
    char *w8 = static_cast<char *>(ws);
    unsigned *am = reinterpret_cast<unsigned *>(w8);
    char *dys = w8 + 256;
    char *xs = dys + h3_split_bytes(M, N);
    char *wsp = xs + h3_split_bytes(M, K);
    char *x2s = wsp + h3_split_bytes(N, K);
    char *tail = w8 + sc;
    const size_t tb = ws_bytes - sc;
    const unsigned *dam = dy_absmax ? dy_absmax : am;
    if (dy_absmax) {
      if (int e = h3_split_known(dy, M, N, N, dy_absmax, dys, st)) return e;
    } else if (int e = h3_split(dy, M, N, N, am, dys, st)) {
      return e;
    }
    if (dx) {
      if (int e = h3_split(w, N, K, K, am + 2, wsp, st)) return e;
      if (int e = gemm_h3_presplit(dys, dam, false, wsp, am + 2, true, dx, nullptr, M, K, N, K, 0, tail, tb, status,
                                   st, &ddx))
        return e;
    }
    if (int e = h3_split(x, M, K, K, am + 1, xs, st)) return e;
    if (int e = gemm_h3_presplit(dys, dam, true, xs, am + 1, true, dw, nullptr, N, K, M, K, beta, tail, tb, status,
                                 st, &ddw))
      return e;
    if (x2) {
      if (int e = h3_split(x2, M, K2, K2, am + 3, x2s, st)) return e;
      if (int e = gemm_h3_presplit(dys, dam, true, x2s, am + 3, true, dw2, nullptr, N, K2, M, K2, beta, tail, tb,
                                   status, st, &ddw2))
        return e;
    }
  }
  if (!ddx)
    if (int e = linear_dgrad(dy, w, dx, M, N, K, ws, ws_bytes, status, st)) return e;
  if (!ddw)
    if (int e = linear_wgrad(dy, x, dw, M, N, K, beta, ws, ws_bytes, status, st)) return e;
  if (!ddw2)
    if (int e = linear_wgrad(dy, x2, dw2, M, N, K2, beta, ws, ws_bytes, status, st)) return e;
  return HS_OK;
}

// dx = dy.w and dw = beta*dw + dy^T.x from dy given only as its fp16 split
// (hi, lo [M][N], N % 8 == 0, scale word dy_scale); *took = false if the
// tensor-core path does not take the shape or the workspace (nothing can be
// done without float32 dy).
// x may instead be given as its split (x_split, x_scale; x may then be null).
int linear_backward_split_only(const void *dy_split, const unsigned *dy_scale, const float *x, const void *x_split,
                               const unsigned *x_scale, const float *w, float *dx, float *dw, int64_t M, int64_t N,
                               int64_t K, int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st,
                               bool *took) {
  *took = false;
  if (M <= 0 || N <= 0 || K <= 0 || !(x || (x_split && x_scale)) || !w || !dw || !status)
    return fail(HS_ERR_INVALID_ARG, "linear backward: bad arguments");
  const size_t sc = 256 + h3_split_bytes(M, K) + h3_split_bytes(N, K);
  if (!ws || !aligned(ws, 256) || ws_bytes < sc || !aligned(dw, 16) || K % 4 || (dx && !aligned(dx, 16))) return HS_OK;
  char *w8 = static_cast<char *>(ws);
  unsigned *am = reinterpret_cast<unsigned *>(w8);
  char *xs = w8 + 256;
  char *wsp = xs + h3_split_bytes(M, K);
  char *tail = w8 + sc;
  const size_t tb = ws_bytes - sc;
  bool ddx = dx == nullptr, ddw = false;
  if (dx) {
    if (int e = h3_split(w, N, K, K, am + 2, wsp, st)) return e;
    if (int e = gemm_h3_presplit(dy_split, dy_scale, false, wsp, am + 2, true, dx, nullptr, M, K, N, K, 0, tail, tb,
                                 status, st, &ddx))
      return e;
  }
  if (!x_split) {
    if (int e = h3_split(x, M, K, K, am + 1, xs, st)) return e;
    x_split = xs;
    x_scale = am + 1;
  }
  if (int e = gemm_h3_presplit(dy_split, dy_scale, true, x_split, x_scale, true, dw, nullptr, N, K, M, K, beta, tail,
                               tb, status, st, &ddw))
    return e;
  *took = ddx && ddw;
  return HS_OK;
}

// y = x.w^T (+ bias) from x given as its split; *took = false if the
// tensor-core path does not take it.
int linear_forward_split_only(const void *x_split, const unsigned *x_scale, const float *w, const float *bias,
                              float *y, int64_t M, int64_t N, int64_t K, void *ws, size_t ws_bytes, int *status,
                              cudaStream_t st, bool *took) {
  *took = false;
  if (M <= 0 || N <= 0 || K <= 0 || !x_split || !x_scale || !w || !y || !status)
    return fail(HS_ERR_INVALID_ARG, "linear forward: bad arguments");
  const size_t sc = 256 + h3_split_bytes(N, K);
  if (!ws || !aligned(ws, 256) || ws_bytes < sc || !aligned(y, 16) || N % 4) return HS_OK;
  char *w8 = static_cast<char *>(ws);
  unsigned *am = reinterpret_cast<unsigned *>(w8);
  if (int e = h3_split(w, N, K, K, am, w8 + 256, st)) return e;
  return gemm_h3_presplit(x_split, x_scale, false, w8 + 256, am, false, y, bias, M, N, K, N, 0, w8 + sc,
                          ws_bytes - sc, status, st, took);
}

size_t linear_backward_split_ws(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return 256 + h3_split_bytes(M, K) + h3_split_bytes(N, K) +
         std::max(gemm_h3_partial_bound(M, K, N), gemm_h3_partial_bound(N, K, M));
}

int linear_backward(const float *dy, const float *x, const float *w, float *dx, float *dw, int64_t M, int64_t N,
                    int64_t K, int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st) {
  return linear_backward_ex(dy, w, dx, x, dw, nullptr, nullptr, M, N, K, 0, beta, ws, ws_bytes, status, st,
                            nullptr);
}

// Scratch of the backward that takes dZ to the GEMMs as its fp16 split:
// [dZ split][256 B: scale word][max(scan split scratch, GEMM scratch)].
size_t parallel_fused_ws(int64_t T, int64_t B, int64_t D, int64_t H) {
  const int64_t M = T * B, N = 4 * H;
  return round_up(h3_split_bytes(M, N), 256) + 256 +
         std::max(scan_split_ws_bytes(T, B, H), linear_backward_split_ws(M, N, D));
}

// The scan's and the linear layer's scratch overlap (they run one after the
// other); the last 256 bytes hold max |dz|, which the scan backward writes
// and the gradient GEMMs' split reads.  The split-handoff backward's layout
// (parallel_fused_ws) is covered as well.
// The forward that runs the projection and the scan as one kernel needs
// x's fp16 split and its scale word ahead of the kernel's own scratch.
size_t proj_scan_fwd_ws(int64_t T, int64_t B, int64_t D, int64_t H) {
  return round_up(h3_split_bytes(T * B, D), 256) + 256 + proj_scan_ws(T, B, D, H);
}

size_t parallel_ws_bytes(int64_t T, int64_t B, int64_t D, int64_t H) {
  size_t b = std::max(std::max(scan_workspace(T, B, H), linear_ws_bytes(T * B, 4 * H, D)) + 256,
                      parallel_fused_ws(T, B, D, H));
  if (proj_scan_shape_ok(T, B, D, H)) b = std::max(b, proj_scan_fwd_ws(T, B, D, H));
  return b;
}

// kf (device word, may be null): receives the forward's max of
// c_{t-1} f'(1 - f') for the backward's dZ split (parallel_backward).
int parallel_forward(const float *x, const float *c0, const float *w_ih, const float *b_ih,
                     float *z, float *out, float *c, float *h_n, float *c_n, int64_t T, int64_t B,
                     int64_t D, int64_t H, float eps, void *ws, size_t ws_bytes, int *status,
                     cudaStream_t st, unsigned *kf = nullptr) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return fail(HS_ERR_INVALID_ARG, "T, B, D, H must be positive");
  if (!x || !w_ih || !z) return fail(HS_ERR_INVALID_ARG, "parallel_forward: null x/w_ih/z");
  // The projection with the scan in its epilogue (one kernel, Z written for
  // the backward but not read back), where the shape fills the GPU with it.
  if (out && c && aligned(x, 16) && ws && aligned(ws, 256) && ws_bytes >= proj_scan_fwd_ws(T, B, D, H) &&
      proj_scan_wanted(T, B, D, H)) {
    char *w8 = static_cast<char *>(ws);
    const size_t xb = round_up(h3_split_bytes(T * B, D), 256);
    unsigned *x_scale = reinterpret_cast<unsigned *>(w8 + xb);
    if (int e = h3_split(x, T * B, D, D, x_scale, w8, st)) return e;
    bool took = false;
    if (int e = proj_scan_forward(w8, x_scale, w_ih, b_ih, c0, z, out, c, h_n, c_n, T, B, D, H, eps, w8 + xb + 256,
                                  ws_bytes - xb - 256, kf, status, st, &took))
      return e;
    if (took) return HS_OK;
  }
  if (int e = linear_forward(x, w_ih, b_ih, z, T * B, 4 * H, D, ws, ws_bytes, status, st)) return e;
  return scan_forward(z, c0, out, c, h_n, c_n, T, B, H, eps, ws, ws_bytes, status, st, kf);
}

int parallel_backward(const float *x, const float *w_ih, float *z, const float *c,
                      const float *c0, const float *dout, const float *dh_n, const float *dc_n,
                      float *dx, float *dw_ih, float *db_ih, float *dc0, int64_t T, int64_t B,
                      int64_t D, int64_t H, float eps, void *ws, size_t ws_bytes, int *status,
                      cudaStream_t st, const unsigned *kf = nullptr) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return fail(HS_ERR_INVALID_ARG, "T, B, D, H must be positive");
  if (!x || !w_ih || !z || !dw_ih || !db_ih) return fail(HS_ERR_INVALID_ARG, "parallel_backward: null x/w_ih/z/dw_ih/db_ih");
  // With the forward's kf, room for it and a shape the tensor-core GEMMs
  // take, dZ goes from the scan to the GEMMs as its fp16 split (never stored
  // in float32); every condition the GEMMs check is checked here first, as
  // there is no float32 dZ to fall back on afterwards.
  const int64_t M = T * B, N = 4 * H;
  if (kf && ws && aligned(ws, 256) && ws_bytes >= parallel_fused_ws(T, B, D, H) && N % 8 == 0 && D % 4 == 0 &&
      M < (1ll << 31) && gemm_h3_enabled() && gemm_tc_size_ok(M, N, D) && gemm_tc_size_ok(N, D, M) &&
      aligned(dw_ih, 16) && (!dx || aligned(dx, 16)) && aligned(x, 16) && aligned(w_ih, 16)) {
    char *w8 = static_cast<char *>(ws);
    const size_t sb = round_up(h3_split_bytes(M, N), 256);
    unsigned *scale = reinterpret_cast<unsigned *>(w8 + sb);
    char *rest = w8 + sb + 256;
    const size_t rb = ws_bytes - sb - 256;
    if (int e = scan_backward_split(z, c, c0, dout, dh_n, dc_n, kf, w8, scale, dc0, db_ih, T, B, H, eps, rest, rb,
                                    status, st))
      return e;
    bool took = false;
    if (int e = linear_backward_split_only(w8, scale, x, nullptr, nullptr, w_ih, dx, dw_ih, M, N, D, 0, rest, rb,
                                           status, st, &took))
      return e;
    return took ? HS_OK : fail(HS_ERR_UNSUPPORTED, "parallel_backward: the split GEMMs declined the shape");
  }
  // With room for it, max |dz| comes out of the scan (the split then reads dz once, not twice).
  unsigned *dz_absmax = nullptr;
  size_t wsb = ws_bytes & ~(size_t)255;
  if (ws && aligned(ws, 256) && wsb >= scan_workspace(T, B, H) + 256) {
    wsb -= 256;
    dz_absmax = reinterpret_cast<unsigned *>(static_cast<char *>(ws) + wsb);
    if (cudaMemsetAsync(dz_absmax, 0, 4, st) != cudaSuccess) return check_launch("parallel_backward memset");
  } else {
    wsb = ws_bytes;
  }
  if (int e = scan_backward(z, c, c0, dout, dh_n, dc_n, z, dc0, db_ih, T, B, H, eps, ws, wsb, status, st, dz_absmax))
    return e;
  return linear_backward_ex(z, w_ih, dx, x, dw_ih, nullptr, nullptr, T * B, 4 * H, D, 0, 0, ws, wsb, status, st,
                            dz_absmax);
}

// ---------------------------------------------------------------- bf16 operands
// A bfloat16 module's linear-layer products: bf16 x bf16 products are exact
// in one kind::f16 tensor-core MMA with bf16 inputs (no fp16 split, no
// operand scale), accumulated in float32.
int gemm_bf16(const void *a, int64_t a_ld, bool a_mn, const void *b, int64_t b_ld, bool b_mn, void *C,
              const float *bias, int64_t M, int64_t N, int64_t K, int64_t ldc, int beta, void *ws, size_t ws_bytes,
              int *status, cudaStream_t st, bool *done, bool c_bf16);
size_t gemm_bf16_partial_bound(int64_t M, int64_t N, int64_t K);
bool scan_bf16_ok(int64_t T, int64_t B, int64_t H);
size_t scan_bf16_ws_bytes(int64_t B, int64_t H);
int scan_forward_bf16(const void *z, const float *c0, void *out, void *c, float *h_n, float *c_n, int64_t T, int64_t B,
                      int64_t H, float eps, int *status, cudaStream_t st);
int scan_backward_bf16(const void *z, const void *c, const float *c0, const void *dout, const float *dh_n,
                       const float *dc_n, void *dz, float *dc0, float *db, int64_t T, int64_t B, int64_t H, float eps,
                       void *ws, size_t ws_bytes, int *status, cudaStream_t st);

size_t linear_bf16_ws(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return std::max({gemm_bf16_partial_bound(M, N, K), gemm_bf16_partial_bound(M, K, N),
                   gemm_bf16_partial_bound(N, K, M), (size_t)256});
}

static int bf16_declined(const char *what) {
  return fail(HS_ERR_UNSUPPORTED, "%s: the bf16 tensor-core GEMM declined (operands must be 16-byte aligned, "
              "the tensor cores enabled)", what);
}

// y[M,N] = x[M,K].w[N,K]^T (+ bias): x, w bf16; bias float32; y float32, or
// bf16 if y_bf16.
int linear_forward_bf16(const void *x, const void *w, const float *bias, void *y, int64_t M, int64_t N, int64_t K,
                        void *ws, size_t ws_bytes, int *status, cudaStream_t st, bool y_bf16 = false) {
  if (int e = check_gemm(x, w, y, M, N, K)) return e;
  if (!status) return fail(HS_ERR_INVALID_ARG, "bf16 linear: null status");
  if (K % 8 || N % (y_bf16 ? 8 : 4)) return fail(HS_ERR_UNSUPPORTED, "bf16 linear: K must be a multiple of 8, N of 4 (8 for bf16 y)");
  if (!M || !N) return HS_OK;
  bool done = false;
  if (int e = gemm_bf16(x, K, false, w, K, false, y, bias, M, N, K, N, 0, ws, ws_bytes, status, st, &done, y_bf16))
    return e;
  return done ? HS_OK : bf16_declined("bf16 linear forward");
}

// dx[M,K] = dy[M,N].w[N,K] (dx may be null; float32, or bf16 if dx_bf16) and
// dw[N,K] = beta*dw + dy^T.x (float32): dy, x, w bf16.
int linear_backward_bf16(const void *dy, const void *x, const void *w, void *dx, float *dw, int64_t M, int64_t N,
                         int64_t K, int beta, void *ws, size_t ws_bytes, int *status, cudaStream_t st,
                         bool dx_bf16 = false) {
  if (int e = check_gemm(dy, x, dw, N, K, M)) return e;
  if (dx && !w) return fail(HS_ERR_INVALID_ARG, "bf16 linear backward: dx wanted without w");
  if (!status) return fail(HS_ERR_INVALID_ARG, "bf16 linear backward: null status");
  if (K % 8 || N % 8) return fail(HS_ERR_UNSUPPORTED, "bf16 linear backward: N and K must be multiples of 8");
  if (!M || !N || !K) return HS_OK;
  bool done = false;
  if (dx) {
    if (int e = gemm_bf16(dy, N, false, w, K, true, dx, nullptr, M, K, N, K, 0, ws, ws_bytes, status, st, &done,
                          dx_bf16))
      return e;
    if (!done) return bf16_declined("bf16 linear dgrad");
  }
  if (int e = gemm_bf16(dy, N, true, x, K, true, dw, nullptr, N, K, M, K, beta, ws, ws_bytes, status, st, &done,
                        false))
    return e;
  return done ? HS_OK : bf16_declined("bf16 linear wgrad");
}

// The whole parallel path of a bf16 module with bf16 saved activations:
// x, w_ih, z, out, c, dout, dx bf16; c0, b_ih, h_n, c_n, dh_n, dc_n, dw_ih,
// db_ih, dc0 float32.
bool parallel_bf16_ok(int64_t T, int64_t B, int64_t D, int64_t H) {
  return D > 0 && D % 8 == 0 && scan_bf16_ok(T, B, H) && T * B < (1ll << 31);
}

// [dZ bf16 [T*B][4H]][max(scan scratch, GEMM scratch)]
size_t parallel_bf16_ws(int64_t T, int64_t B, int64_t D, int64_t H) {
  const int64_t M = T * B, N = 4 * H;
  return round_up((size_t)M * N * 2, 256) + std::max(scan_bf16_ws_bytes(B, H), linear_bf16_ws(M, N, D));
}

int parallel_forward_bf16(const void *x, const float *c0, const void *w_ih, const float *b_ih, void *z, void *out,
                          void *c, float *h_n, float *c_n, int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                          void *ws, size_t ws_bytes, int *status, cudaStream_t st) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return fail(HS_ERR_INVALID_ARG, "T, B, D, H must be positive");
  if (!x || !w_ih || !z) return fail(HS_ERR_INVALID_ARG, "parallel_forward_bf16: null x/w_ih/z");
  if (!parallel_bf16_ok(T, B, D, H))
    return fail(HS_ERR_UNSUPPORTED, "bf16 parallel path: needs D, H multiples of 8 and a shape the per-column scan takes");
  if (int e = linear_forward_bf16(x, w_ih, b_ih, z, T * B, 4 * H, D, ws, ws_bytes, status, st, true)) return e;
  return scan_forward_bf16(z, c0, out, c, h_n, c_n, T, B, H, eps, status, st);
}

int parallel_backward_bf16(const void *x, const void *w_ih, const void *z, const void *c, const float *c0,
                           const void *dout, const float *dh_n, const float *dc_n, void *dx, float *dw_ih, float *db_ih,
                           float *dc0, int64_t T, int64_t B, int64_t D, int64_t H, float eps, void *ws, size_t ws_bytes,
                           int *status, cudaStream_t st) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return fail(HS_ERR_INVALID_ARG, "T, B, D, H must be positive");
  if (!x || !w_ih || !z || !dw_ih || !db_ih)
    return fail(HS_ERR_INVALID_ARG, "parallel_backward_bf16: null x/w_ih/z/dw_ih/db_ih");
  if (!parallel_bf16_ok(T, B, D, H))
    return fail(HS_ERR_UNSUPPORTED, "bf16 parallel path: needs D, H multiples of 8 and a shape the per-column scan takes");
  if (!ws || !aligned(ws, 256)) return fail(HS_ERR_INVALID_ARG, "workspace must be non-null and 256-byte aligned");
  if (ws_bytes < parallel_bf16_ws(T, B, D, H))
    return fail(HS_ERR_WORKSPACE, "parallel_backward_bf16: workspace %zu < %zu bytes", ws_bytes,
                parallel_bf16_ws(T, B, D, H));
  const int64_t M = T * B, N = 4 * H;
  const size_t sb = round_up((size_t)M * N * 2, 256);
  char *rest = static_cast<char *>(ws) + sb;
  const size_t rb = ws_bytes - sb;
  if (int e = scan_backward_bf16(z, c, c0, dout, dh_n, dc_n, ws, dc0, db_ih, T, B, H, eps, rest, rb, status, st))
    return e;
  return linear_backward_bf16(ws, x, w_ih, dx, dw_ih, M, N, D, 0, rest, rb, status, st, true);
}

namespace {
__global__ void selftest_wait_kernel(const unsigned *flag, int *status, uint64_t limit_ns) {
  if (threadIdx.x == 0) (void)wait_flag(flag, status, limit_ns);
}

// Relative errors of the scan's activations against double precision:
// sigf over x in [-lim, lim] and tanh_pos over c in (0, lim], n points each
// (uniform in x, plus the small-argument range of tanh_pos densely), folded
// into out[0] (sigmoid) and out[1] (tanh) as max |rel err| by atomicMax on
// the float bits (valid for non-negative floats).
__global__ void selftest_activation_kernel(float *out, int n, float lim) {
  float es = 0.f, et = 0.f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float u = (i + 0.5f) / n;
    const float x = -lim + 2.f * lim * u;
    const double sd = 1.0 / (1.0 + exp(-(double)x));
    const float sg = sigf(x);
    if (sd > 1e-30) es = fmaxf(es, (float)(fabs((double)sg - sd) / sd));
    const float c = i & 1 ? lim * u : 0.25f * u;  // odd points: (0, lim]; even: (0, 0.25)
    const double td = tanh((double)c);
    et = fmaxf(et, (float)(fabs((double)tanh_pos(c) - td) / td));
  }
  atomicMax(reinterpret_cast<unsigned *>(out), __float_as_uint(es));
  atomicMax(reinterpret_cast<unsigned *>(out + 1), __float_as_uint(et));
}
}  // namespace

}  // namespace hs

extern "C" {

int hs_abi_version(void) { return 1; }

const char *hs_status_string(int status) {
  switch (status) {
    case HS_OK: return "ok";
    case HS_ERR_INVALID_ARG: return "invalid argument";
    case HS_ERR_WORKSPACE: return "workspace missing or too small";
    case HS_ERR_UNSUPPORTED: return "unsupported shape";
    case HS_ERR_CUDA: return "CUDA error";
    case HS_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

const char *hs_last_error_message(void) { return hs::g_msg; }

int hs_read_status(const int *dev_status, int *host_status, hs_stream_t stream) {
  if (!dev_status || !host_status) return hs::fail(HS_ERR_INVALID_ARG, "null status pointer");
  if (cudaMemcpyAsync(host_status, dev_status, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream) != cudaSuccess)
    return hs::check_launch("hs_read_status");
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return hs::check_launch("hs_read_status sync");
  return HS_OK;
}

int hs_clear_status(int *dev_status, hs_stream_t stream) {
  if (!dev_status) return hs::fail(HS_ERR_INVALID_ARG, "null status pointer");
  if (cudaMemsetAsync(dev_status, 0, sizeof(int), (cudaStream_t)stream) != cudaSuccess)
    return hs::check_launch("hs_clear_status");
  return HS_OK;
}

int hs_selftest_bounded_wait(const unsigned *flag, int *dev_status, uint64_t limit_ns,
                             hs_stream_t stream) {
  if (!flag) return hs::fail(HS_ERR_INVALID_ARG, "null flag");
  if (limit_ns > hs::kWaitLimitNs) return hs::fail(HS_ERR_INVALID_ARG, "limit above the library's wait bound");
  if (!dev_status) {
    // NULL: the library's own word that NULL-status hs_scan_forward_noalloc
    // calls report into (so a test can plant a timeout there)
    if (int e = hs::noalloc_status_word(&dev_status)) return e;
  }
  hs::selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flag, dev_status, limit_ns);
  return hs::check_launch("selftest_wait_kernel");
}

int hs_selftest_activations(float *max_rel_err, int n, float lim, hs_stream_t stream) {
  if (!max_rel_err || n <= 0 || !(lim > 0.f)) return hs::fail(HS_ERR_INVALID_ARG, "selftest_activations: bad args");
  if (cudaMemsetAsync(max_rel_err, 0, 2 * sizeof(float), (cudaStream_t)stream) != cudaSuccess)
    return hs::check_launch("selftest_activations memset");
  hs::selftest_activation_kernel<<<148, 256, 0, (cudaStream_t)stream>>>(max_rel_err, n, lim);
  return hs::check_launch("selftest_activation_kernel");
}

size_t hs_linear_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  return hs::linear_ws_bytes(M, N, K);
}
size_t hs_parallel_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return 0;
  return hs::parallel_ws_bytes(T, B, D, H);
}
int hs_linear_forward(const float *x, const float *w, const float *bias, float *y, int64_t M,
                      int64_t N, int64_t K, void *workspace, size_t workspace_bytes, int *dev_status,
                      hs_stream_t stream) {
  return hs::linear_forward(x, w, bias, y, M, N, K, workspace, workspace_bytes, dev_status,
                            (cudaStream_t)stream);
}
int hs_linear_dgrad(const float *dy, const float *w, float *dx, int64_t M, int64_t N, int64_t K,
                    void *workspace, size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::linear_dgrad(dy, w, dx, M, N, K, workspace, workspace_bytes, dev_status,
                          (cudaStream_t)stream);
}
int hs_linear_backward(const float *dy, const float *x, const float *w, float *dx, float *dw, int64_t M,
                       int64_t N, int64_t K, int beta, void *workspace, size_t workspace_bytes, int *dev_status,
                       hs_stream_t stream) {
  return hs::linear_backward(dy, x, w, dx, dw, M, N, K, beta, workspace, workspace_bytes, dev_status,
                             (cudaStream_t)stream);
}

int hs_linear_backward_absmax(const float *dy, const float *x, const float *w, float *dx, float *dw, int64_t M,
                              int64_t N, int64_t K, int beta, const unsigned *dy_absmax, void *workspace,
                              size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  if (!dy_absmax || !hs::aligned(dy_absmax, 4))
    return hs::fail(HS_ERR_INVALID_ARG, "hs_linear_backward_absmax: null or misaligned dy_absmax");
  return hs::linear_backward_ex(dy, w, dx, x, dw, nullptr, nullptr, M, N, K, 0, beta, workspace, workspace_bytes,
                                dev_status, (cudaStream_t)stream, dy_absmax);
}

int hs_split(const float *x, int64_t rows, int64_t cols, void *dst, unsigned *scale, hs_stream_t stream) {
  if (rows <= 0 || cols <= 0 || !x || !dst || !scale || !hs::aligned(dst, 16) || !hs::aligned(scale, 4))
    return hs::fail(HS_ERR_INVALID_ARG, "hs_split: bad arguments");
  return hs::h3_split(x, rows, cols, cols, scale, dst, (cudaStream_t)stream);
}

int hs_linear_forward_presplit(const void *x_split, const unsigned *x_scale, const float *w, const float *bias,
                               float *y, int64_t M, int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                               int *dev_status, hs_stream_t stream) {
  if (!hs::gemm_h3_enabled() || !hs::gemm_tc_size_ok(M, N, K))
    return hs::fail(HS_ERR_UNSUPPORTED, "hs_linear_forward_presplit: the fp16-split GEMMs do not take this shape");
  bool took = false;
  if (int e = hs::linear_forward_split_only(x_split, x_scale, w, bias, y, M, N, K, workspace, workspace_bytes,
                                            dev_status, (cudaStream_t)stream, &took))
    return e;
  return took ? HS_OK
              : hs::fail(HS_ERR_WORKSPACE, "hs_linear_forward_presplit: workspace too small or operands unaligned");
}

size_t hs_projection_scan_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H) {
  return (T > 0 && B > 0 && D > 0 && H > 0) ? hs::proj_scan_ws(T, B, D, H) : 0;
}

int hs_projection_scan_supported(int64_t T, int64_t B, int64_t D, int64_t H) {
  return hs::proj_scan_wanted(T, B, D, H) ? 1 : 0;
}

int hs_projection_scan_forward(const void *x_split, const unsigned *x_scale, const float *w_ih, const float *b_ih,
                               const float *c0, float *z, float *out, float *c, float *h_n, float *c_n, int64_t T,
                               int64_t B, int64_t D, int64_t H, float eps, void *workspace, size_t workspace_bytes,
                               unsigned *kf, int *dev_status, hs_stream_t stream) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return hs::fail(HS_ERR_INVALID_ARG, "T, B, D, H must be positive");
  if (!x_split || !x_scale || !w_ih || !z || !out || !c || !dev_status)
    return hs::fail(HS_ERR_INVALID_ARG, "hs_projection_scan_forward: null argument");
  if (!hs::proj_scan_shape_ok(T, B, D, H))
    return hs::fail(HS_ERR_UNSUPPORTED,
                    "hs_projection_scan_forward: needs H %% 32 == 0 and a shape the fp16-split GEMMs take");
  bool took = false;
  const char *why = "";
  if (int e = hs::proj_scan_forward(x_split, x_scale, w_ih, b_ih, c0, z, out, c, h_n, c_n, T, B, D, H, eps, workspace,
                                    workspace_bytes, kf, dev_status, (cudaStream_t)stream, &took, &why))
    return e;
  return took ? HS_OK : hs::fail(HS_ERR_WORKSPACE, "hs_projection_scan_forward: %s", why);
}

int hs_linear_backward_presplit(const void *dy_split, const unsigned *dy_scale, const float *x, const void *x_split,
                                const unsigned *x_scale, const float *w, float *dx, float *dw, int64_t M, int64_t N,
                                int64_t K, int beta, void *workspace, size_t workspace_bytes, int *dev_status,
                                hs_stream_t stream) {
  if (!dy_split || !dy_scale || !hs::aligned(dy_split, 16) || !hs::aligned(dy_scale, 4))
    return hs::fail(HS_ERR_INVALID_ARG, "hs_linear_backward_presplit: null or misaligned dy_split/dy_scale");
  if (N % 8) return hs::fail(HS_ERR_UNSUPPORTED, "hs_linear_backward_presplit: N must be a multiple of 8");
  if (!hs::gemm_h3_enabled() || !hs::gemm_tc_size_ok(M, N, K))
    return hs::fail(HS_ERR_UNSUPPORTED, "hs_linear_backward_presplit: the fp16-split GEMMs do not take this shape");
  bool took = false;
  if (int e = hs::linear_backward_split_only(dy_split, dy_scale, x, x_split, x_scale, w, dx, dw, M, N, K, beta,
                                             workspace, workspace_bytes, dev_status, (cudaStream_t)stream, &took))
    return e;
  return took ? HS_OK
              : hs::fail(HS_ERR_WORKSPACE, "hs_linear_backward_presplit: workspace too small or operands unaligned");
}

size_t hs_linear_presplit_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  return hs::linear_backward_split_ws(M, N, K);
}

size_t hs_split_bytes(int64_t rows, int64_t cols) {
  return (rows > 0 && cols > 0) ? hs::h3_split_bytes(rows, cols) : 0;
}

int hs_linear_wgrad(const float *dy, const float *x, float *dw, int64_t M, int64_t N, int64_t K,
                    int beta, void *workspace, size_t workspace_bytes, int *dev_status,
                    hs_stream_t stream) {
  return hs::linear_wgrad(dy, x, dw, M, N, K, beta, workspace, workspace_bytes, dev_status,
                          (cudaStream_t)stream);
}
int hs_colsum(const float *dy, float *db, int64_t M, int64_t N, int beta, hs_stream_t stream) {
  if (M < 0 || N < 0 || (N && !db) || (M && N && !dy)) return hs::fail(HS_ERR_INVALID_ARG, "hs_colsum: bad arguments");
  return hs::colsum(dy, db, M, N, beta, (cudaStream_t)stream);
}

int hs_parallel_forward(const float *x, const float *c0, const float *w_ih, const float *b_ih,
                        float *z, float *out, float *c, float *h_n, float *c_n, int64_t T,
                        int64_t B, int64_t D, int64_t H, float eps, void *workspace,
                        size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::parallel_forward(x, c0, w_ih, b_ih, z, out, c, h_n, c_n, T, B, D, H, eps, workspace,
                              workspace_bytes, dev_status, (cudaStream_t)stream);
}

int hs_parallel_forward_kf(const float *x, const float *c0, const float *w_ih, const float *b_ih, float *z,
                           float *out, float *c, float *h_n, float *c_n, int64_t T, int64_t B, int64_t D, int64_t H,
                           float eps, void *workspace, size_t workspace_bytes, unsigned *kf, int *dev_status,
                           hs_stream_t stream) {
  if (!kf || !hs::aligned(kf, 4)) return hs::fail(HS_ERR_INVALID_ARG, "hs_parallel_forward_kf: null or misaligned kf");
  return hs::parallel_forward(x, c0, w_ih, b_ih, z, out, c, h_n, c_n, T, B, D, H, eps, workspace, workspace_bytes,
                              dev_status, (cudaStream_t)stream, kf);
}

int hs_parallel_backward_kf(const float *x, const float *w_ih, float *z, const float *c, const float *c0,
                            const float *dout, const float *dh_n, const float *dc_n, float *dx, float *dw_ih,
                            float *db_ih, float *dc0, int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                            void *workspace, size_t workspace_bytes, const unsigned *kf, int *dev_status,
                            hs_stream_t stream) {
  return hs::parallel_backward(x, w_ih, z, c, c0, dout, dh_n, dc_n, dx, dw_ih, db_ih, dc0, T, B, D, H, eps,
                               workspace, workspace_bytes, dev_status, (cudaStream_t)stream, kf);
}

int hs_parallel_backward(const float *x, const float *w_ih, float *z, const float *c,
                         const float *c0, const float *dout, const float *dh_n,
                         const float *dc_n, float *dx, float *dw_ih, float *db_ih, float *dc0,
                         int64_t T, int64_t B, int64_t D, int64_t H, float eps, void *workspace,
                         size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::parallel_backward(x, w_ih, z, c, c0, dout, dh_n, dc_n, dx, dw_ih, db_ih, dc0, T, B,
                               D, H, eps, workspace, workspace_bytes, dev_status,
                               (cudaStream_t)stream);
}

size_t hs_linear_bf16_workspace_bytes(int64_t M, int64_t N, int64_t K) { return hs::linear_bf16_ws(M, N, K); }

int hs_linear_forward_bf16(const void *x, const void *w, const float *bias, float *y, int64_t M, int64_t N, int64_t K,
                           void *workspace, size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::linear_forward_bf16(x, w, bias, y, M, N, K, workspace, workspace_bytes, dev_status,
                                 (cudaStream_t)stream);
}

int hs_linear_backward_bf16(const void *dy, const void *x, const void *w, float *dx, float *dw, int64_t M, int64_t N,
                            int64_t K, int beta, void *workspace, size_t workspace_bytes, int *dev_status,
                            hs_stream_t stream) {
  return hs::linear_backward_bf16(dy, x, w, dx, dw, M, N, K, beta, workspace, workspace_bytes, dev_status,
                                  (cudaStream_t)stream);
}

int hs_parallel_bf16_supported(int64_t T, int64_t B, int64_t D, int64_t H) {
  return (T > 0 && B > 0 && H > 0 && hs::parallel_bf16_ok(T, B, D, H)) ? 1 : 0;
}

size_t hs_parallel_bf16_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H) {
  if (T <= 0 || B <= 0 || D <= 0 || H <= 0) return 0;
  return hs::parallel_bf16_ws(T, B, D, H);
}

int hs_parallel_forward_bf16(const void *x, const float *c0, const void *w_ih, const float *b_ih, void *z, void *out,
                             void *c, float *h_n, float *c_n, int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                             void *workspace, size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::parallel_forward_bf16(x, c0, w_ih, b_ih, z, out, c, h_n, c_n, T, B, D, H, eps, workspace,
                                   workspace_bytes, dev_status, (cudaStream_t)stream);
}

int hs_parallel_backward_bf16(const void *x, const void *w_ih, const void *z, const void *c, const float *c0,
                              const void *dout, const float *dh_n, const float *dc_n, void *dx, float *dw_ih,
                              float *db_ih, float *dc0, int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                              void *workspace, size_t workspace_bytes, int *dev_status, hs_stream_t stream) {
  return hs::parallel_backward_bf16(x, w_ih, z, c, c0, dout, dh_n, dc_n, dx, dw_ih, db_ih, dc0, T, B, D, H, eps,
                                    workspace, workspace_bytes, dev_status, (cudaStream_t)stream);
}

}  // extern "C"
