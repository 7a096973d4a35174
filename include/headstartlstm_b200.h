/*
 * headstartlstm_b200.h -- C ABI of the B200 (sm_100a) HeadStartLSTM library.
 *
 * The library implements the two hot paths of HeadStartLSTM
 * (m-j-tilley/prLSTM, package `headstartlstm`):
 *   - the recurrent cell: input projection, per-step a-scaled W_hh.h
 *     recurrence with the sigmoid-g cell, and its BPTT backward;
 *   - the parallel=True Heinsen scan over time, forward and backward.
 *
 * Conventions
 *   - Every pointer is a DEVICE pointer to contiguous row-major fp32 data
 *     unless stated otherwise.  Shapes use T (time), B (batch), D (input
 *     features), H (hidden units); the gate axis has 4H entries in the order
 *     [i, f, g, o] (nn.LSTM order).
 *   - Ownership: the caller allocates every tensor and every workspace.  The
 *     library never allocates or frees device memory.
 *   - Streams: every call is asynchronous and stream-ordered on `stream`
 *     (a cudaStream_t; NULL means the legacy default stream).
 *   - Status: 0 (HS_OK) on success, else an HS_ERR_* code.  Argument checks
 *     run on the host before any launch; a call that fails them launches
 *     nothing.  Device-side failures (a bounded wait that gave up) are
 *     recorded in the caller's `dev_status` word (a device int, sticky: the
 *     first nonzero code stays until the caller clears it) and can be read
 *     with hs_read_status().
 *   - Workspace: calls that need scratch take (`workspace`, `workspace_bytes`);
 *     the matching *_workspace_bytes() query returns the size to allocate.
 *     Calls that overlap on the GPU must not share a workspace.
 */
#ifndef HEADSTARTLSTM_B200_H
#define HEADSTARTLSTM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *hs_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define HS_API __attribute__((visibility("default")))
#else
#define HS_API
#endif

enum {
  HS_OK = 0,
  HS_ERR_INVALID_ARG = 1,   /* bad shape, null pointer or misaligned buffer   */
  HS_ERR_WORKSPACE = 2,     /* workspace missing or smaller than required     */
  HS_ERR_UNSUPPORTED = 3,   /* shape outside what the kernels implement       */
  HS_ERR_CUDA = 4,          /* a CUDA runtime call or launch failed           */
  HS_ERR_DEVICE_TIMEOUT = 5 /* a device-side bounded wait gave up             */
};

/* Library identity and diagnostics. */
HS_API int hs_abi_version(void);
HS_API const char *hs_status_string(int status);
/* Text of the last host-side error on the calling thread (never NULL). */
HS_API const char *hs_last_error_message(void);
/* Copy the device status word to *host_status (synchronises `stream`). */
HS_API int hs_read_status(const int *dev_status, int *host_status, hs_stream_t stream);
/* Reset the device status word to HS_OK (stream-ordered). */
HS_API int hs_clear_status(int *dev_status, hs_stream_t stream);
/* Failure-detection self test: launches one CTA that waits on *flag (a
 * device word nothing sets) with the library's bounded wait, shortened to
 * limit_ns.  The wait gives up, records HS_ERR_DEVICE_TIMEOUT in *dev_status
 * and the kernel returns; the context stays usable.  dev_status NULL targets
 * the library's own word of NULL-status hs_scan_forward_noalloc calls on the
 * current device (read it with hs_scan_noalloc_status).  No reference
 * counterpart (the reference has no device-side waits). */
HS_API int hs_selftest_bounded_wait(const unsigned *flag, int *dev_status, uint64_t limit_ns,
                                    hs_stream_t stream);
/* Accuracy self test of the scan kernels' activation functions: evaluates
 * the logistic sigmoid on n points of [-lim, lim] and tanh on n points of
 * (0, lim] (half of them in (0, 0.25)) and writes the largest relative errors
 * against double precision to max_rel_err[0] (sigmoid) and [1] (tanh), a
 * device array of two floats.  No reference counterpart (the reference calls
 * ATen's sigmoid and tanh). */
HS_API int hs_selftest_activations(float *max_rel_err, int n, float lim, hs_stream_t stream);

/* ------------------------------------------------------------------------
 * Linear-layer GEMMs (fp32 in, fp32 out, fp32-accurate).
 * Replace the cuBLAS/ATen calls of the reference:
 *   forward projection  F.linear(x, W_ih, b_ih)   _torch.py:96, _parallel.py:56,
 *                                                  _triton.py:345
 *   input gradient      dgates_flat @ W_ih         _torch.py:162, _triton.py:456
 *   weight gradients    dgates_flat.t() @ h / x    _torch.py:157-158, _triton.py:451-452
 *   bias gradient       dgates_flat.sum(dim=0)     _torch.py:159, _triton.py:453
 * ---------------------------------------------------------------------- */
/* Scratch (bytes) any of the products below may use on these extents (split-K
 * partials, fp16 operand splits); pass at least this much, or NULL/0 (then
 * the products take slower paths with the same accuracy). */
HS_API size_t hs_linear_workspace_bytes(int64_t M, int64_t N, int64_t K);
/* y[M,N] = x[M,K] . w[N,K]^T (+ bias[N] if bias != NULL) */
HS_API int hs_linear_forward(const float *x, const float *w, const float *bias, float *y,
                             int64_t M, int64_t N, int64_t K, void *workspace,
                             size_t workspace_bytes, int *dev_status, hs_stream_t stream);
/* dx[M,K] = dy[M,N] . w[N,K] */
HS_API int hs_linear_dgrad(const float *dy, const float *w, float *dx, int64_t M, int64_t N,
                           int64_t K, void *workspace, size_t workspace_bytes, int *dev_status,
                           hs_stream_t stream);
/* dw[N,K] = beta * dw + dy[M,N]^T . x[M,K]   (beta is 0 or 1) */
HS_API int hs_linear_wgrad(const float *dy, const float *x, float *dw, int64_t M, int64_t N,
                           int64_t K, int beta, void *workspace, size_t workspace_bytes,
                           int *dev_status, hs_stream_t stream);
/* Both gradient products of y = x.w^T + b in one call: dx[M,K] = dy . w
 * (skipped if dx is NULL) and dw[N,K] = beta * dw + dy^T . x.  Replaces the
 * pair of products of the reference's backward (_torch.py:157-162,
 * _triton.py:451-456); with enough workspace dy, x and w are converted once
 * and shared by both products. */
HS_API int hs_linear_backward(const float *dy, const float *x, const float *w, float *dx, float *dw,
                              int64_t M, int64_t N, int64_t K, int beta, void *workspace,
                              size_t workspace_bytes, int *dev_status, hs_stream_t stream);
/* hs_linear_backward with max |dy| already known: *dy_absmax (device
 * memory) is an upper bound of max |dy| as float32 bits, for example the
 * word hs_scan_backward_absmax writes for its dz.  The fp16 split of dy then
 * skips its own pass over dy.  A bound below the true maximum overflows the
 * split; the exact maximum keeps the most precision.  Same replacement as
 * hs_linear_backward (_torch.py:157-162, _triton.py:451-456). */
HS_API int hs_linear_backward_absmax(const float *dy, const float *x, const float *w, float *dx,
                                     float *dw, int64_t M, int64_t N, int64_t K, int beta,
                                     const unsigned *dy_absmax, void *workspace,
                                     size_t workspace_bytes, int *dev_status, hs_stream_t stream);
/* Bytes of an fp16 split buffer of a [rows][cols] float32 matrix: hi then
 * lo, each [rows][cols rounded up to 8] fp16. */
HS_API size_t hs_split_bytes(int64_t rows, int64_t cols);
/* The fp16 split of a contiguous float32 [rows][cols] matrix into dst
 * (16-byte aligned, hs_split_bytes(rows, cols) bytes), its scale word (the
 * float32 bits of max |x|) into *scale, for the _presplit entry points. */
HS_API int hs_split(const float *x, int64_t rows, int64_t cols, void *dst, unsigned *scale,
                    hs_stream_t stream);
/* hs_linear_forward from x given as its split (x_split, x_scale from
 * hs_split of x [M][K]): the same split then serves the weight gradient in
 * hs_linear_backward_presplit.  Same replacement as hs_linear_forward. */
HS_API int hs_linear_forward_presplit(const void *x_split, const unsigned *x_scale, const float *w,
                                      const float *bias, float *y, int64_t M, int64_t N, int64_t K,
                                      void *workspace, size_t workspace_bytes, int *dev_status,
                                      hs_stream_t stream);
/* hs_linear_backward with dy given only as its fp16 split (dy_split, as
 * hs_scan_backward_split writes it; N % 8 == 0) and its scale word dy_scale
 * (float32 bits of an upper bound of max |dy|); x either as float32 (x) or
 * as its split (x_split, x_scale; x may then be NULL).  No float32 dy is
 * read, so there is no fallback: shapes the tensor-core path does not take,
 * or a workspace below hs_linear_presplit_workspace_bytes(M, N, K), return an
 * error.  Same replacement as hs_linear_backward (_torch.py:157-162). */
HS_API size_t hs_linear_presplit_workspace_bytes(int64_t M, int64_t N, int64_t K);
HS_API int hs_linear_backward_presplit(const void *dy_split, const unsigned *dy_scale, const float *x,
                                       const void *x_split, const unsigned *x_scale, const float *w,
                                       float *dx, float *dw, int64_t M, int64_t N, int64_t K, int beta,
                                       void *workspace, size_t workspace_bytes, int *dev_status,
                                       hs_stream_t stream);
/* db[N] = beta * db + sum_m dy[m, N]   (beta is 0 or 1) */
HS_API int hs_colsum(const float *dy, float *db, int64_t M, int64_t N, int beta,
              hs_stream_t stream);

/* ------------------------------------------------------------------------
 * Parallel (Heinsen) path.  Replaces headstartlstm_parallel and
 * _log_parallel_scan (_parallel.py:21-74) and the autograd backward the
 * reference traces through them.  c_t = max(f_t,eps) c_{t-1} + max(i_t g_t,eps)
 * with c_{-1} = max(c0, eps), out_t = o_t tanh(c_t).
 * ---------------------------------------------------------------------- */
HS_API size_t hs_scan_workspace_bytes(int64_t T, int64_t B, int64_t H);
/* Workspace of hs_parallel_forward / hs_parallel_backward (scan + GEMMs). */
HS_API size_t hs_parallel_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H);

/* Fused gate activations + chunked scan over T (single pass, decoupled
 * look-back).  z [T,B,4H] gate pre-activations (x W_ih^T + b_ih);
 * c0 [B,H] (NULL = zeros).  Writes out [T,B,H], c [T,B,H] (kept for the
 * backward), h_n [B,H], c_n [B,H] (either may be NULL). */
HS_API int hs_scan_forward(const float *z, const float *c0, float *out, float *c, float *h_n,
                    float *c_n, int64_t T, int64_t B, int64_t H, float eps,
                    void *workspace, size_t workspace_bytes, int *dev_status,
                    hs_stream_t stream);

/* Reverse-time scan of the gradient.  dout [T,B,H] = dL/dout; dh_n, dc_n
 * [B,H] (NULL = zeros) are the gradients of h_n and c_n.  Writes dz [T,B,4H]
 * (may alias z: each element is read before it is overwritten by the same
 * thread), dc0 [B,H] (NULL = not wanted) and db [4H] = sum over (t,b) of dz
 * (NULL = not wanted; reduced deterministically from per-chunk sums). */
HS_API int hs_scan_backward(const float *z, const float *c, const float *c0, const float *dout,
                     const float *dh_n, const float *dc_n, float *dz, float *dc0,
                     float *db, int64_t T, int64_t B, int64_t H, float eps,
                     void *workspace, size_t workspace_bytes, int *dev_status,
                     hs_stream_t stream);
/* hs_scan_backward that also writes *dz_absmax (device memory, 4-byte
 * aligned) = max |dz| over all written elements as float32 bits (NaN
 * ignored), for hs_linear_backward_absmax: the gradient GEMMs that follow
 * the scan in the reference's backward (_parallel.py:38-74 traced by
 * autograd) then read dz once.  The word is zeroed by this call. */
HS_API int hs_scan_backward_absmax(const float *z, const float *c, const float *c0,
                                   const float *dout, const float *dh_n, const float *dc_n,
                                   float *dz, float *dc0, float *db, int64_t T, int64_t B,
                                   int64_t H, float eps, void *workspace, size_t workspace_bytes,
                                   unsigned *dz_absmax, int *dev_status, hs_stream_t stream);

/* hs_scan_forward that also writes *kf_max (device memory) = the maximum
 * over all steps of c_{t-1} f'_t (1 - f'_t) (c_{-1} = max(c0, eps),
 * f' = max(sigmoid(z_f), eps)) as float32 bits: the forget-gate factor of
 * the bound on |dZ| that hs_scan_backward_split uses.  Same replacement as
 * hs_scan_forward. */
HS_API int hs_scan_forward_kf(const float *z, const float *c0, float *out, float *c, float *h_n,
                              float *c_n, int64_t T, int64_t B, int64_t H, float eps,
                              void *workspace, size_t workspace_bytes, unsigned *kf_max,
                              int *dev_status, hs_stream_t stream);
/* The projection and the scan forward as ONE kernel: z = x W_ih^T + b_ih
 * (x given as its fp16 split, x_split and x_scale from hs_split of x
 * [T*B][D]) on the tensor cores, with the gates, the scan, out, c, h_n, c_n
 * and *kf (as hs_scan_forward_kf; may be NULL) computed in the GEMM's
 * epilogue.  z [T,B,4H] is written for the backward but never read back.
 * Needs H % 32 == 0, 16-byte aligned z, out, c, x_split (and b_ih if given)
 * and dev_status; workspace >= hs_projection_scan_workspace_bytes (256-byte
 * aligned).  hs_projection_scan_supported says whether the library's own
 * forward (hs_parallel_forward*) takes this kernel for a shape by default
 * (it does for 112 <= T <= 128, one mostly filled time tile of 128 steps,
 * where it is faster than the GEMM and the scan as two calls; a tile
 * always spans 128 steps, so much shorter sequences would pad it, and at
 * longer T the two calls win inside a power-capped training step);
 * HS_PROJ_SCAN=0 / 1 turns that off / on for every shape it can run.  Replaces, with hs_split, the projection `linear` and the scan of
 * headstartlstm_parallel (_parallel.py:38-74, _parallel.py:21-35). */
HS_API size_t hs_projection_scan_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H);
HS_API int hs_projection_scan_supported(int64_t T, int64_t B, int64_t D, int64_t H);
HS_API int hs_projection_scan_forward(const void *x_split, const unsigned *x_scale, const float *w_ih,
                                      const float *b_ih, const float *c0, float *z, float *out, float *c,
                                      float *h_n, float *c_n, int64_t T, int64_t B, int64_t D, int64_t H,
                                      float eps, void *workspace, size_t workspace_bytes, unsigned *kf,
                                      int *dev_status, hs_stream_t stream);
/* The scan backward with dZ delivered as its fp16 split for the gradient
 * GEMMs (hs_linear_backward_presplit) instead of float32: dz_split (16-byte
 * aligned, hs_split_bytes(T*B, 4H) bytes) receives hi then lo, *dz_scale the
 * scale word.  The scale is chosen before the scan from an upper bound of
 * max |dZ|: D x max(1/4, Kf), D the largest column sum of |dout| (with
 * |dh_n| + |dc_n|) and Kf the forward's kf_max; the scan writes the split
 * directly, so dZ is never stored in float32.  If the bound turns out more
 * than 2^16 above the exact maximum (or anything is not finite), the scan
 * runs again into float32 dZ in place of z and the split is made from the
 * exact maximum (z is overwritten then).
 * Replaces, with the GEMMs after it, the autograd backward of
 * headstartlstm_parallel (_parallel.py:38-74). */
/* Diagnostic: 1 if the scans of this T, B, H run on the per-column kernels
 * (one CTA per sequence x 32 units, a fixed order of operations, so results
 * are the same bit for bit from run to run), 0 if on the look-back kernels
 * (the carry into a tile is composed from whichever predecessors have
 * published: float32 results may differ in the last bits between runs).
 * HS_SCAN_PATH=chain|lookback forces one. */
HS_API int hs_scan_uses_column_kernels(int64_t T, int64_t B, int64_t H);
/* Sizing hint for callers that split a batch into several calls (micro-
 * batches): the number of sequences whose per-column scan CTAs (one per
 * sequence x 64 units) are all resident at once on the current device, in
 * the forward and the backward; calls of about this many sequences fill the
 * SMs with one wave of columns (0 if it cannot be queried).  No reference
 * counterpart (the reference runs its batch as one call). */
HS_API int64_t hs_scan_wave_sequences(int64_t H);
HS_API size_t hs_scan_split_workspace_bytes(int64_t T, int64_t B, int64_t H);
HS_API int hs_scan_backward_split(float *z, const float *c, const float *c0, const float *dout,
                                  const float *dh_n, const float *dc_n, const unsigned *kf_max,
                                  void *dz_split, unsigned *dz_scale, float *dc0, float *db, int64_t T,
                                  int64_t B, int64_t H, float eps, void *workspace,
                                  size_t workspace_bytes, int *dev_status, hs_stream_t stream);

/* hs_scan_forward without a workspace argument, for callers that cannot
 * allocate device memory (for example a host framework that passes the
 * library only its input and output buffers, or a latency-critical path that
 * must not pay cudaMalloc's implicit synchronisation).  No counterpart in the
 * reference, which allocates through PyTorch.  The look-back scratch is a
 * fixed 8 MiB device array inside the library (held by every GPU that loads
 * it, until exit); shapes whose scratch exceeds it are rejected with
 * HS_ERR_UNSUPPORTED before any launch: the scratch is ceil(T/8) * B *
 * ceil(H/32) * 256 bytes, so roughly T*B*H <= 8M elements.
 * The first call on each device looks up the array's device address, so
 * make that first call before any stream capture.  All calls share the
 * array: calls that overlap on the GPU (other streams, other threads) race
 * and must be serialised by the caller.  Allocates nothing.
 * dev_status may be NULL: the call then reports into a status word inside the
 * library (one per device), which it first clears in stream order, so that
 * word describes the most recent NULL-status call on that device only; read
 * it with hs_scan_noalloc_status before the next such call.  Shapes that take
 * the one-CTA-per-column chain kernels (many columns, B * ceil(H/32) filling
 * the GPU) use no scratch and have no size limit. */
HS_API int hs_scan_forward_noalloc(const float *z, const float *c0, float *out, float *c,
                                   float *h_n, float *c_n, int64_t T, int64_t B, int64_t H,
                                   float eps, int *dev_status, hs_stream_t stream);
/* Outcome of the most recent hs_scan_forward_noalloc call made with
 * dev_status == NULL on the current device: synchronises `stream`, writes
 * the library's status word (HS_OK, or HS_ERR_DEVICE_TIMEOUT if a bounded
 * wait gave up and out/c were not fully written) to *host_status and clears
 * it.  No counterpart in the reference (its calls allocate through PyTorch
 * and have no device-side waits).  Allocates nothing. */
HS_API int hs_scan_noalloc_status(int *host_status, hs_stream_t stream);

/* Affine maps of one chunk of time steps of the scan, for a sequence split
 * over time across GPUs (each rank scans its own chunk; the state crossing a
 * chunk boundary is the only dependency).  z [T,B,4H] is the chunk's gate
 * pre-activations.  backward = 0: the chunk maps the state entering it to its
 * last state as c -> A c + C; writes A = prod_t max(f_t, eps) and CD = C (the
 * chunk's last state from a zero carry), both [B,H].  backward = 1: the chunk
 * maps the gradient arriving at its last state to the gradient it passes to
 * the state before it as e -> A e + D; needs c [T,B,H] (the chunk's states),
 * dout [T,B,H] and dh_last [B,H] (gradient of the chunk's last output, NULL =
 * zeros); writes A and CD = D.  The carries then follow from all chunks' maps
 * in order; each rank runs hs_scan_forward with its incoming state as c0 and
 * hs_scan_backward with its incoming gradient as dc_n.  Sequence-sharded form
 * of _log_parallel_scan (_parallel.py:21-35), which the reference runs on one
 * device only. */
HS_API int hs_scan_chunk_maps(const float *z, const float *c, const float *dout, const float *dh_last,
                              int64_t T, int64_t B, int64_t H, float eps, float *A, float *CD, int backward,
                              hs_stream_t stream);

/* Whole parallel-mode forward: z = x W_ih^T + b_ih (z is caller-owned
 * [T,B,4H] scratch kept for the backward), then hs_scan_forward. */
HS_API int hs_parallel_forward(const float *x, const float *c0, const float *w_ih,
                        const float *b_ih, float *z, float *out, float *c, float *h_n,
                        float *c_n, int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                        void *workspace, size_t workspace_bytes, int *dev_status,
                        hs_stream_t stream);

/* Whole parallel-mode backward.  z is overwritten with dz.  Outputs:
 * dx [T,B,D] (NULL = not wanted), dw_ih [4H,D], db_ih [4H], dc0 [B,H] (NULL =
 * not wanted).  The reference returns no gradient for W_hh, b_hh, a and h0
 * in this mode (_parallel.py:41-43); neither does this call. */
HS_API int hs_parallel_backward(const float *x, const float *w_ih, float *z, const float *c,
                         const float *c0, const float *dout, const float *dh_n,
                         const float *dc_n, float *dx, float *dw_ih, float *db_ih,
                         float *dc0, int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                         void *workspace, size_t workspace_bytes, int *dev_status,
                         hs_stream_t stream);

/* hs_parallel_forward that also writes *kf (device word) for
 * hs_parallel_backward_kf: with it the backward hands dZ from the scan to
 * the gradient GEMMs as its fp16 split (hs_scan_backward_split ->
 * hs_linear_backward_presplit) when the shape, alignment and workspace
 * (hs_parallel_workspace_bytes covers it) allow, and otherwise takes the
 * path of hs_parallel_backward.  Same replacements as the two calls above. */
HS_API int hs_parallel_forward_kf(const float *x, const float *c0, const float *w_ih,
                                  const float *b_ih, float *z, float *out, float *c, float *h_n,
                                  float *c_n, int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                                  void *workspace, size_t workspace_bytes, unsigned *kf,
                                  int *dev_status, hs_stream_t stream);
HS_API int hs_parallel_backward_kf(const float *x, const float *w_ih, float *z, const float *c,
                                   const float *c0, const float *dout, const float *dh_n,
                                   const float *dc_n, float *dx, float *dw_ih, float *db_ih,
                                   float *dc0, int64_t T, int64_t B, int64_t D, int64_t H,
                                   float eps, void *workspace, size_t workspace_bytes,
                                   const unsigned *kf, int *dev_status, hs_stream_t stream);

/* ------------------------------------------------------------------------
 * bfloat16 module path.  The reference runs the same module with bf16
 * parameters and data (tests/test_parallel.py:24, tests/test_triton.py:22).
 * Here a bf16 x bf16 product is exact in one tensor-core MMA with bf16
 * inputs, accumulated in float32; the scan's arithmetic and carried state
 * are float32; the saved activations (Z, c) and out, dout, dZ, dx are stored
 * in bf16 (half the bytes).  bf16 arguments are `void *` (uint16 storage),
 * 16-byte aligned, with row lengths (D, 4H, H) multiples of 8.
 * HS_ERR_UNSUPPORTED when the shape or alignment does not suit (the caller
 * then widens to float32 and takes the calls above).
 * ---------------------------------------------------------------------- */
HS_API size_t hs_linear_bf16_workspace_bytes(int64_t M, int64_t N, int64_t K);
/* y[M,N] = x[M,K].w[N,K]^T (+ bias[N]), x and w bf16, bias and y float32.
 * Replaces F.linear on bf16 tensors (_torch.py:96, _parallel.py:56). */
HS_API int hs_linear_forward_bf16(const void *x, const void *w, const float *bias, float *y, int64_t M,
                                  int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                                  int *dev_status, hs_stream_t stream);
/* dx[M,K] = dy[M,N].w[N,K] (dx may be NULL) and dw[N,K] = beta*dw + dy^T.x;
 * dy, x, w bf16, dx and dw float32.  Replaces the gradient products of
 * F.linear on bf16 tensors (_torch.py:157-162). */
HS_API int hs_linear_backward_bf16(const void *dy, const void *x, const void *w, float *dx, float *dw,
                                   int64_t M, int64_t N, int64_t K, int beta, void *workspace,
                                   size_t workspace_bytes, int *dev_status, hs_stream_t stream);
/* The scan forward with z [T*B][4H], out and c [T][B][H] in bf16 (c0, h_n,
 * c_n float32).  No workspace.  Shapes the per-column kernels take
 * (hs_scan_uses_column_kernels) with H % 8 == 0.  Replaces
 * _log_parallel_scan with the activations (_parallel.py:21-35, :56-74) on
 * bf16 tensors. */
HS_API int hs_scan_forward_bf16(const void *z, const float *c0, void *out, void *c, float *h_n,
                                float *c_n, int64_t T, int64_t B, int64_t H, float eps, int *dev_status,
                                hs_stream_t stream);
/* Its backward: z, c, dout bf16 in, dz [T*B][4H] bf16 out (the operand of
 * hs_linear_backward_bf16); dh_n, dc_n, dc0, db float32.  Workspace (for db):
 * hs_scan_bf16_workspace_bytes. */
HS_API size_t hs_scan_bf16_workspace_bytes(int64_t T, int64_t B, int64_t H);
HS_API int hs_scan_backward_bf16(const void *z, const void *c, const float *c0, const void *dout,
                                 const float *dh_n, const float *dc_n, void *dz, float *dc0, float *db,
                                 int64_t T, int64_t B, int64_t H, float eps, void *workspace,
                                 size_t workspace_bytes, int *dev_status, hs_stream_t stream);
/* hs_parallel_forward / hs_parallel_backward for a bf16 module: x, w_ih,
 * z, out, c, dout and dx bf16; c0, b_ih, h_n, c_n, dh_n, dc_n, dw_ih, db_ih,
 * dc0 float32.  hs_parallel_bf16_supported says whether the shape is taken;
 * one workspace size covers both calls.  Replaces headstartlstm_parallel +
 * its autograd (_parallel.py:38-74) on bf16 tensors. */
HS_API int hs_parallel_bf16_supported(int64_t T, int64_t B, int64_t D, int64_t H);
HS_API size_t hs_parallel_bf16_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H);
HS_API int hs_parallel_forward_bf16(const void *x, const float *c0, const void *w_ih, const float *b_ih,
                                    void *z, void *out, void *c, float *h_n, float *c_n, int64_t T,
                                    int64_t B, int64_t D, int64_t H, float eps, void *workspace,
                                    size_t workspace_bytes, int *dev_status, hs_stream_t stream);
HS_API int hs_parallel_backward_bf16(const void *x, const void *w_ih, const void *z, const void *c,
                                     const float *c0, const void *dout, const float *dh_n,
                                     const float *dc_n, void *dx, float *dw_ih, float *db_ih, float *dc0,
                                     int64_t T, int64_t B, int64_t D, int64_t H, float eps,
                                     void *workspace, size_t workspace_bytes, int *dev_status,
                                     hs_stream_t stream);

/* ------------------------------------------------------------------------
 * Recurrent path.  Replaces HeadStartLSTMTorchFn / HeadStartLSTMTritonFn
 * (_torch.py:78-176, _triton.py:327-470) and the C++ headstartlstm_forward
 * (_csrc/lstm_cell.cpp:28-78).
 * ---------------------------------------------------------------------- */
HS_API size_t hs_recurrent_workspace_bytes(int64_t T, int64_t B, int64_t D, int64_t H);
/* 1 if hs_recurrent_forward (backward = 0) or hs_recurrent_backward
 * (backward = 1) runs the per-step product on the tensor cores for this B
 * and H on the current device, 0 if on the FFMA kernels (shapes the tensor-core
 * kernels do not cover, or where the FFMA kernels measured faster).  A
 * diagnostic with no reference counterpart; the environment variable
 * HS_REC_PATH=tc|ffma forces one implementation. */
HS_API int hs_recurrent_uses_tensor_cores(int64_t B, int64_t H, int backward);
/* Diagnostic: which kernels run the recurrence of this B, H on the current
 * device: 0 FFMA kernels over the whole GPU (one grid barrier per step),
 * 1 tensor-core kernels, 2 thread-block clusters with the weights resident
 * and the state exchanged in distributed shared memory: one cluster per
 * batch group of 32 sequences for H <= 128, and for H = 512 clusters of 16
 * CTAs with up to 8 sequences each, the batch spread over the clusters the
 * device runs at once (B up to 8 times that count; HS_REC_PATH=cluster also
 * runs larger batches, as further waves of clusters); -1 for bad arguments.
 * HS_REC_PATH=ffma|tc|cluster forces one where it applies. */
HS_API int hs_recurrent_path(int64_t B, int64_t H, int backward);

/* Whole recurrent forward.  Inputs x [T,B,D], h0/c0 [B,H] (NULL = zeros),
 * w_ih [4H,D], w_hh [4H,H], b_ih/b_hh [4H], a [4].  Outputs:
 *   h_save [T+1,B,H]  (h_save[0]=h0; out = h_save[1:], h_n = h_save[T])
 *   c_save [T+1,B,H]  (c_n = c_save[T])
 *   acts   [T,B,4H]   gate activations i,f,g,o kept for the backward. */
HS_API int hs_recurrent_forward(const float *x, const float *h0, const float *c0,
                         const float *w_ih, const float *w_hh, const float *b_ih,
                         const float *b_hh, const float *a, float *h_save, float *c_save,
                         float *acts, int64_t T, int64_t B, int64_t D, int64_t H,
                         void *workspace, size_t workspace_bytes, int *dev_status,
                         hs_stream_t stream);

/* Whole recurrent backward (hand-written BPTT, _torch.py:133-170).
 * acts is overwritten with dgates.  dout [T,B,H]; dh_n, dc_n [B,H] (NULL =
 * zeros).  Outputs dx [T,B,D] (NULL = not wanted), dw_ih [4H,D], dw_hh [4H,H],
 * db_ih [4H], db_hh [4H], da [4].  Like the reference, no gradient for h0/c0. */
HS_API int hs_recurrent_backward(const float *x, const float *w_ih, const float *w_hh,
                          const float *b_hh, const float *a, const float *h_save,
                          const float *c_save, float *acts, const float *dout,
                          const float *dh_n, const float *dc_n, float *dx, float *dw_ih,
                          float *dw_hh, float *db_ih, float *db_hh, float *da,
                          int64_t T, int64_t B, int64_t D, int64_t H,
                          void *workspace, size_t workspace_bytes, int *dev_status,
                          hs_stream_t stream);
/* The same two calls for a bfloat16 module (inputs and parameters
 * bf16-valued, passed widened to float32): where the per-step product runs
 * on the tensor cores (hs_recurrent_uses_tensor_cores), a*W_hh and the state
 * carried between steps (h forward, dgates backward) are rounded to bf16 and
 * multiplied in one bf16 product per instruction with float32 accumulation,
 * as the reference's bf16 module computes its per-step GEMM in bf16
 * (_torch.py:111-120, :150; _triton.py:230, :299); elsewhere float32 on the
 * bf16 values.  Same workspace size. */
HS_API int hs_recurrent_forward_bf16(const float *x, const float *h0, const float *c0, const float *w_ih,
                                     const float *w_hh, const float *b_ih, const float *b_hh, const float *a,
                                     float *h_save, float *c_save, float *acts, int64_t T, int64_t B,
                                     int64_t D, int64_t H, void *workspace, size_t workspace_bytes,
                                     int *dev_status, hs_stream_t stream);
HS_API int hs_recurrent_backward_bf16(const float *x, const float *w_ih, const float *w_hh,
                                      const float *b_hh, const float *a, const float *h_save,
                                      const float *c_save, float *acts, const float *dout,
                                      const float *dh_n, const float *dc_n, float *dx, float *dw_ih,
                                      float *dw_hh, float *db_ih, float *db_hh, float *da, int64_t T,
                                      int64_t B, int64_t D, int64_t H, void *workspace,
                                      size_t workspace_bytes, int *dev_status, hs_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HEADSTARTLSTM_B200_H */
