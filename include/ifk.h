/*
 * ifk.h — C ABI of the B200 (sm_100a) IFKFAC curvature library (libifk.so).
 *
 * The library replaces the linear algebra under the reference's Python front
 * end (Gsend/ifkfac): the streaming TSQR that folds captured activations X and
 * back-propagated gradients delta into upper-triangular factors R_X / R_G, the
 * damping fold, the four triangular solves that give the natural gradient,
 * and the momentum / lr update of fp32 master weights.
 *
 * Conventions
 *  - All matrices are device pointers, row-major, with an explicit leading
 *    dimension in elements.  The caller owns every buffer and passes the
 *    scratch each call needs as a workspace; the library never allocates
 *    device memory on these paths and never frees caller memory.  One
 *    exception: ifk_natgrad_noalloc takes no workspace and uses a fixed 2 MiB
 *    device array inside the library (present on every GPU that loads it).
 *  - R factors are n x n fp32 (or bf16 where stated), upper triangular, with a
 *    non-negative diagonal (the reference's positive-diagonal convention,
 *    ifkfac/triangular.py:230-239).  A running factor that has seen fewer
 *    than n rows is trapezoidal: only its first rows_R rows are meaningful and
 *    the remaining rows are zero.
 *  - Every call is asynchronous on `stream` (a cudaStream_t) and returns an
 *    ifk status code.  Host-side argument errors are reported before any GPU
 *    work is queued.  Errors found on the device (non-finite factors, a timed
 *    out wait) are written to a caller-provided device int, which stays 0 on
 *    success.
 *  - Calls are reentrant: no hidden global state other than the per-device
 *    kernel attributes set on first use, and the fixed scratch array of
 *    ifk_natgrad_noalloc (shared by all of its calls, which must therefore be
 *    ordered by the caller).  Calls that share a workspace must be ordered on
 *    one stream.
 *  - Precision: IFK_PREC_BF16 runs the GEMM-shaped work on tcgen05 tensor
 *    cores with bf16 operands and fp32 accumulation (fp32 panels, norms,
 *    divides and storage); IFK_PREC_FP32 runs everything in fp32 on the CUDA
 *    cores.  IFK_PREC_AUTO picks BF16 for a bf16 chunk and FP32 otherwise.
 *
 * Reference citations are path:line inside the reference project.
 */
#ifndef IFK_H_
#define IFK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define IFK_OK             0
#define IFK_ERR_RANK       1  /* factor still trapezoidal: fewer rows than columns seen */
#define IFK_ERR_NONFINITE  2  /* a factor has a NaN or Inf entry */
#define IFK_ERR_SHAPE      3  /* inconsistent sizes or leading dimensions */
#define IFK_ERR_TIMEOUT    4  /* a bounded device-side wait gave up */
#define IFK_ERR_CUDA       5  /* a CUDA runtime call failed */
#define IFK_ERR_WORKSPACE  6  /* workspace missing, too small or misaligned */
#define IFK_ERR_DTYPE      7  /* unsupported element type */
#define IFK_ERR_ARG        8  /* other invalid argument (null pointer, bad flag) */
#define IFK_ERR_DEVICE     9  /* current device is not an sm_100 part */
#define IFK_ERR_LIMIT     10  /* size above the fixed scratch of ifk_natgrad_noalloc */

/* ---- element types ---------------------------------------------------- */
#define IFK_F32   0
#define IFK_BF16  1

/* ---- precision modes -------------------------------------------------- */
#define IFK_PREC_AUTO  0
#define IFK_PREC_FP32  1
#define IFK_PREC_BF16  2

/* ---- fold flags ------------------------------------------------------- */
#define IFK_FOLD_TRAPEZOIDAL_CHUNK 1  /* chunk row i is zero left of column i (an R factor) */
/* Tests of the failure path only (ifk_tsqr_fold, IFK_PREC_BF16): the first
 * panel of the fold is never published and the cross-CTA waits give up after
 * a few milliseconds instead of seconds, so every task that needs that panel
 * times out; the call then leaves IFK_ERR_TIMEOUT in *d_status, R is not a
 * valid factor, and the device stays usable for the next call. */
#define IFK_FOLD_DEBUG_WITHHOLD 256

typedef void* ifk_stream_t;  /* a cudaStream_t */

#if defined(__GNUC__)
#define IFK_API __attribute__((visibility("default")))
#else
#define IFK_API
#endif

/* Library version string and a message for a status code. */
IFK_API const char* ifk_version(void);
IFK_API const char* ifk_status_string(int status);

/* IFK_OK when the current CUDA device is compute capability 10.0 (B200). */
IFK_API int ifk_device_check(void);

/* ---- streaming TSQR ---------------------------------------------------- */

/* Workspace bytes for ifk_tsqr_fold on a chunk of `rows` rows and n columns. */
IFK_API size_t ifk_tsqr_fold_workspace(int64_t rows, int64_t n);

/*
 * Fold `rows` rows of `chunk` (rows x n, element type chunk_dtype, leading
 * dimension ld_chunk) into the running factor R (n x n fp32, in place).
 * R holds rows_R meaningful rows (0 for an empty factor: R must then be all
 * zero); afterwards it holds min(n, rows_R + rows) rows, upper triangular
 * with a non-negative diagonal, such that R'^T R' = R^T R + chunk^T chunk.
 * flags: IFK_FOLD_TRAPEZOIDAL_CHUNK when the chunk is itself an R factor
 * (zero left of its diagonal), which skips the known-zero work.
 *
 * Replaces streaming_tsqr_update (ifkfac/triangular.py:246-307), i.e. the
 * leaf QR + merge QR + _positive_diagonal_R (:230-239) that the forward and
 * backward hooks call (ifkfac/activation_hooks.py:579,642).  Also the merge
 * step of the tile/tree TSQR (ifkfac/triangular.py:207-220) when the chunk
 * is another R factor.  *d_status (device int, may be NULL) receives
 * IFK_ERR_TIMEOUT if a bounded device-side wait gave up.
 */
IFK_API int ifk_tsqr_fold(float* R, int64_t ldR, int64_t rows_R,
                  const void* chunk, int64_t ld_chunk, int64_t rows, int64_t n,
                  int chunk_dtype, int prec, int flags, int* d_status,
                  void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/* Workspace bytes for ifk_tsqr_fold_batched. */
IFK_API size_t ifk_tsqr_fold_batched_workspace(int nfolds, const int64_t* rows, const int64_t* n);

/*
 * nfolds independent folds in one wave schedule: fold f absorbs rows[f] rows
 * of chunk[f] (n[f] columns, leading dimension ld_chunk[f]) into R[f]
 * (n[f] x n[f], leading dimension ldR[f], rows_R[f] meaningful rows), with
 * the semantics of ifk_tsqr_fold.  The R[f] must not overlap.  Host arrays of
 * length nfolds; folds of zero rows are skipped.
 *
 * Replaces batched_streaming_tsqr_update (ifkfac/triangular.py:331-379) and
 * the bucketed flush of the hooks (ifkfac/activation_hooks.py:370-457),
 * without the zero padding: every fold keeps its own row count.  Also used to
 * fold X and delta of one layer together.
 */
IFK_API int ifk_tsqr_fold_batched(int nfolds, float* const* R, const int64_t* ldR,
                          const int64_t* rows_R, const void* const* chunk,
                          const int64_t* ld_chunk, const int64_t* rows, const int64_t* n,
                          int chunk_dtype, int prec, int flags, int* d_status,
                          void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/*
 * One segment of rows for ifk_tsqr_fold_segments.  Row i of the segment
 * (i < rows) is row row_index[i] of `chunk` when row_index (a device array of
 * `rows` int64) is given, else row i: the reference's random row subsample
 * (x[randperm(rows)[:k]], ifkfac/activation_hooks.py:531-538) is read in
 * place instead of copied.  The chunk holds `cols` columns with leading
 * dimension `ld` (elements); cols is the factor's n, or n - 1, in which case a
 * column of ones is appended (the augmented-bias column of
 * ifkfac/activation_hooks.py:541-543).  src_rows is the chunk's row count: an
 * index outside [0, src_rows) reads as a zero row and sets IFK_ERR_ARG in the
 * status word.  dtype (IFK_F32 or IFK_BF16) is the chunk's element type when
 * the call's chunk_dtype is IFK_PER_SEGMENT_DTYPE, and is ignored otherwise.
 */
typedef struct ifk_conv2d ifk_conv2d;
typedef struct ifk_segment {
  const void* chunk;
  int64_t ld;
  int64_t rows;
  const int64_t* row_index;
  int64_t src_rows;
  int64_t cols;
  int32_t dtype;
  int32_t reserved;
  const ifk_conv2d* conv;  /* NULL, or the chunk is an image read through im2col (below) */
} ifk_segment;

/*
 * An ifk_segment whose `conv` is set reads its rows from a contiguous
 * N x C x H x W image `chunk` through im2col, the rows of the reference's
 * F.unfold (ifkfac/activation_hooks.py:489-499): image row
 * b * Ho * Wo + oh * Wo + ow, column (c * kernel_h + ki) * kernel_w + kj, holds
 * chunk[b, c, oh * stride_h - pad_h + ki * dilation_h,
 *       ow * stride_w - pad_w + kj * dilation_w] (zero outside the image), with
 * Ho, Wo the output size of the convolution.  cols must be C * kernel_h *
 * kernel_w and src_rows N * Ho * Wo; row_index (optional) picks image rows, the
 * conv-row subsample of :522-530; `ld` is ignored.  The fold reads the elements
 * in place: the im2col matrix is never formed.  The geometry is read during
 * the call (host memory).
 */
struct ifk_conv2d {
  int64_t batch, channels, height, width;
  int32_t kernel_h, kernel_w, stride_h, stride_w;
  int32_t pad_h, pad_w, dilation_h, dilation_w;
};

/* chunk_dtype of ifk_tsqr_fold_segments: each segment gives its own (needs an
 * explicit IFK_PREC_FP32 or IFK_PREC_BF16). */
#define IFK_PER_SEGMENT_DTYPE (-1)

/* Workspace bytes for ifk_tsqr_fold_segments (same arguments). */
IFK_API size_t ifk_tsqr_fold_segments_workspace(int nfolds, const int64_t* n, const int* nseg,
                                                const ifk_segment* segs, const double* ident_tail);

/* Workspace bytes with which ifk_tsqr_fold_segments in fp32 mode (IFK_PREC_FP32)
 * folds every fold's segments through one wave schedule together (same
 * arguments; at least ifk_tsqr_fold_segments_workspace).  The segments of a fold
 * are copied one after another into the workspace, so the schedule has T + K - 1
 * waves for the fold's T sub-tiles and K panels instead of one schedule per
 * segment; the sub-tile sequence, and so the result, is that of one fold per
 * segment in turn.  This applies when every segment of a fold but its last holds
 * a multiple of 256 rows and at most 16 folds are given; otherwise, or with the
 * smaller workspace, the segments are folded one after another.  The same
 * operation as the reference's streaming update per chunk
 * (ifkfac/triangular.py:246-307) followed by finalize_R (:386-421). */
IFK_API size_t ifk_tsqr_fold_segments_fp32_workspace(int nfolds, const int64_t* n, const int* nseg,
                                                     const ifk_segment* segs, const double* ident_tail);

/*
 * Fold a sequence of segments of rows into each of nfolds factors, in order,
 * in one persistent launch where they fit (IFK_PREC_BF16): the result is that
 * of one ifk_tsqr_fold per segment in turn, with the same reflector sequence
 * (one sub-tile of rows after another), while the fold of segment s + 1
 * overlaps that of segment s.  Fold f has nseg[f] segments; `segs` is flat,
 * fold after fold.  The segments need not be adjacent in memory; all have
 * element type chunk_dtype, or each its own (IFK_PER_SEGMENT_DTYPE, with an
 * explicit precision).  Folds of one call share launches (up to 64 folds and
 * 256 segments per launch).  When ident_tail is not NULL and
 * ident_tail[f] > 0, n[f] more rows ident_tail[f] * I follow the segments
 * (the damping rows of ifk_finalize at the caller's scale: a caller that then
 * runs ifk_finalize with damping 0 and rows_total p gets the damped factor of
 * lambda = ident_tail^2 / p).  R[f], ldR[f], rows_R[f] are as in
 * ifk_tsqr_fold.
 *
 * Replaces the deferred drain of the hooks, which concatenates the buffered
 * chunks and folds them with one streaming_tsqr_update
 * (ifkfac/activation_hooks.py:347-364, 560-570, 627-635), without the
 * concatenation; a run of streaming_tsqr_update calls over row tiles that are
 * all resident (ifkfac/triangular.py:246-307); and the hooks' row subsample
 * and bias column (ifkfac/activation_hooks.py:519-548) without the copies.
 */
IFK_API int ifk_tsqr_fold_segments(int nfolds, float* const* R, const int64_t* ldR,
                                   const int64_t* rows_R, const int64_t* n, const int* nseg,
                                   const ifk_segment* segs, int chunk_dtype,
                                   const double* ident_tail, int prec, int* d_status,
                                   void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/* ---- R-tree merge --------------------------------------------------------- */

/* Workspace bytes for ifk_rtree_merge of nfactors factors of order n. */
IFK_API size_t ifk_rtree_merge_workspace(int nfactors, int64_t n);

/*
 * Merge nfactors running factors held by this process (R[i]: n x n fp32,
 * leading dimension ldR[i], rows[i] meaningful rows; for instance the local
 * factors of all data-parallel ranks after a gather) into R[0], in the order
 * of the reference's tile/tree TSQR (ifkfac/triangular.py:207-220): round by
 * round, adjacent pairs [R_a; R_b] are merged into R_a (a fold of R_b as a
 * trapezoidal chunk, positive diagonal) and the odd one out is carried
 * forward.  The merges of one round share one persistent launch.  prec is
 * IFK_PREC_FP32 or IFK_PREC_BF16.  *rows_out (host) receives the merged
 * factor's meaningful rows, min(n, sum of rows).  The other R[i] are left in
 * intermediate states.  Replaces the merge tree of tsqr (the batched leaf
 * QRs before it are ifk_tsqr_fold_batched).
 */
IFK_API int ifk_rtree_merge(int nfactors, float* const* R, const int64_t* ldR, const int64_t* rows,
                            int64_t n, int prec, int64_t* rows_out, int* d_status,
                            void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/* ---- damping fold ------------------------------------------------------ */

/* Workspace bytes for ifk_finalize on an n x n factor. */
IFK_API size_t ifk_finalize_workspace(int64_t n);

/*
 * R_out = the positive-diagonal R factor of [R_in / sqrt(rows_total);
 * sqrt(damping) I_n], so that R_out^T R_out = R_in^T R_in / rows_total +
 * damping I.  R_in (n x n fp32) must be square (rows_R == n), otherwise
 * IFK_ERR_RANK is returned and nothing is queued, matching the reference's
 * skip of a non-square factor.  R_out has element type out_dtype (fp32, or
 * bf16 for use_true_bf16) and may not alias R_in.  *d_status (device int,
 * may be NULL) receives IFK_ERR_NONFINITE if any entry of the result is not
 * finite (or IFK_ERR_TIMEOUT if a bounded device-side wait gave up); it is
 * not cleared on success.
 *
 * Replaces the factor half of RawActivationHooks.get_factors
 * (ifkfac/activation_hooks.py:328-332), finalize_R
 * (ifkfac/triangular.py:386-421), and the finite check and bf16 cast of
 * IFKFAC._update_factors (ifkfac/ifkfac.py:231-237, 292-294).
 */
IFK_API int ifk_finalize(const float* R_in, int64_t ldR, int64_t rows_R, int64_t n,
                 double rows_total, double damping,
                 void* R_out, int64_t ld_out, int out_dtype, int prec,
                 int* d_status, void* workspace, size_t workspace_bytes,
                 ifk_stream_t stream);

/* Workspace bytes for ifk_finalize_batched. */
IFK_API size_t ifk_finalize_batched_workspace(int nfactors, const int64_t* n);

/*
 * ifk_finalize on nfactors factors in one wave schedule (host arrays of
 * length nfactors; every factor must be square; the damping folds of up to 16
 * factors share a launch).  Used to refresh R_X and R_G of a layer together.
 */
IFK_API int ifk_finalize_batched(int nfactors, const float* const* R_in, const int64_t* ldR,
                         const int64_t* rows_R, const int64_t* n, const double* rows_total,
                         double damping, void* const* R_out, const int64_t* ld_out,
                         int out_dtype, int prec, int* d_status, void* workspace,
                         size_t workspace_bytes, ifk_stream_t stream);

/*
 * ifk_finalize_batched with a status word per factor: d_status is a host array
 * of nfactors device pointers (entries may be NULL), and factor f's finite
 * check writes to d_status[f] only, so a caller that refreshes many layers at
 * once can still skip just the layers whose factors are not finite, as the
 * reference does per layer (ifkfac/ifkfac.py:231-237).  A timed-out wait of a
 * shared launch is reported to the word of the first factor of its group of
 * 16.  Same workspace as ifk_finalize_batched.
 */
IFK_API int ifk_finalize_many(int nfactors, const float* const* R_in, const int64_t* ldR,
                              const int64_t* rows_R, const int64_t* n, const double* rows_total,
                              double damping, void* const* R_out, const int64_t* ld_out,
                              int out_dtype, int prec, int* const* d_status, void* workspace,
                              size_t workspace_bytes, ifk_stream_t stream);

/* ---- natural gradient ---------------------------------------------------- */

/* Workspace bytes for ifk_natgrad on an n_out x n_in gradient. */
IFK_API size_t ifk_natgrad_workspace(int64_t n_out, int64_t n_in);

/*
 * nat = R_G^-1 R_G^-T grad_W R_X^-1 R_X^-T (n_out x n_in fp32), by four
 * blocked triangular solves.  R_X (n_in x n_in) and R_G (n_out x n_out) have
 * element type r_dtype (fp32, or bf16 for bf16-stored factors); grad_W and
 * nat are fp32 and may alias.
 *
 * Replaces apply_vered (ifkfac/triangular.py:551-656), including the
 * bf16-stored dispatch (:607-628), and the per-layer loop of
 * apply_vered_batched / _apply_vered_batched_impl (:430-451, :506-544).
 * *d_status (device int, may be NULL) receives IFK_ERR_TIMEOUT if a bounded
 * device-side wait gave up.
 */
IFK_API int ifk_natgrad(const float* grad_W, int64_t ld_g,
                const void* R_X, int64_t ld_rx, const void* R_G, int64_t ld_rg,
                int r_dtype, float* nat, int64_t ld_nat,
                int64_t n_out, int64_t n_in, int prec, int* d_status,
                void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/* Workspace bytes for ifk_natgrad_update. */
IFK_API size_t ifk_natgrad_update_workspace(int64_t n_out, int64_t n_in);

/*
 * The natural gradient of ifk_natgrad followed by the update of ifk_update
 * without clipping, in one call: with nat = R_G^-1 R_G^-T grad_W R_X^-1 R_X^-T,
 *   buf = momentum * buf + nat (buf read as zero when buf_is_new; no buffer
 *   when momentum == 0, buf may then be NULL), W *= 1 - lr * weight_decay
 *   (weight_decay > 0), W -= lr * buf (or lr * nat without momentum).
 * W and buf are contiguous n_out x n_in fp32; grad_W is not modified.  The
 * natural gradient goes to the workspace and one elementwise pass applies the
 * update; the result is bit for bit that of ifk_natgrad followed by ifk_update
 * with grad_clip <= 0.  A caller that clips (a norm over all of nat) uses the
 * two calls.
 *
 * Replaces apply_vered (ifkfac/triangular.py:551-656) together with the
 * per-layer epilogue of the bucketed fast path (ifkfac/ifkfac.py:394-413).
 */
IFK_API int ifk_natgrad_update(const float* grad_W, int64_t ld_g,
                               const void* R_X, int64_t ld_rx, const void* R_G, int64_t ld_rg,
                               int r_dtype, float* W, float* buf, int64_t n_out, int64_t n_in,
                               double lr, double momentum, double weight_decay, int buf_is_new,
                               int prec, int* d_status, void* workspace, size_t workspace_bytes,
                               ifk_stream_t stream);

/* ---- K-FAC Laplace posterior draw ---------------------------------------- */

/* Workspace bytes for ifk_posterior_sample (that of ifk_natgrad). */
IFK_API size_t ifk_posterior_sample_workspace(int64_t n_out, int64_t n_in);

/*
 * out = C_G^-1 xi C_A^-T (n_out x n_in fp32; xi and out may alias), by two
 * blocked triangular solves: a draw of a layer's weight perturbation from the
 * K-FAC Laplace posterior when xi holds iid N(0, 1) entries and C_A, C_G are
 * the upper-triangular factors of the per-side posterior precisions,
 *   C_A^T C_A = sqrt(N) A + sqrt(lambda) I,   C_G^T C_G = sqrt(N) G + sqrt(lambda) I,
 * i.e. ifk_finalize of R_A (R_A^T R_A = A) with rows_total = N^-1/2 and
 * damping = sqrt(lambda).  out then has covariance
 * (C_A^T C_A)^-1 (x) (C_G^T C_G)^-1, the posterior of LaplacePosterior
 * (ifkfac/laplace.py:58-109, drawn at :127-149 as
 * U_G diag((sqrt(N) d_G + sqrt(lambda))^-1/2) xi diag(..) U_A^T from
 * eigendecompositions): the same distribution from the triangular square
 * root, with no eigensolver.  Arguments and status as ifk_natgrad.
 */
IFK_API int ifk_posterior_sample(const float* xi, int64_t ld_xi,
                         const void* C_A, int64_t ld_ca, const void* C_G, int64_t ld_cg,
                         int c_dtype, float* out, int64_t ld_out,
                         int64_t n_out, int64_t n_in, int prec, int* d_status,
                         void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/* Largest factor order ifk_natgrad_noalloc accepts. */
#define IFK_NOALLOC_MAX_N 4096

/*
 * ifk_natgrad for callers that cannot allocate device memory where they call
 * it (a step run inside another framework's operator whose memory belongs to
 * that framework's pool, or a host runtime that only works with buffers it was
 * given up front).  It takes no workspace: the scratch of the tensor-core
 * solves is a fixed 2 MiB array inside the library, held on every GPU that
 * loads the library until the process exits.  Same arguments and results as
 * ifk_natgrad; n_out and n_in above IFK_NOALLOC_MAX_N give IFK_ERR_LIMIT
 * before anything is queued.  The first call on a device looks up that
 * device's address of the array (make it before any stream capture).  All
 * calls share the one array, so calls that overlap on the GPU (different
 * streams, or different host threads on one device) race and must be ordered
 * by the caller.  No cudaMalloc or cudaFree is made.
 * This entry point has no counterpart in the reference.
 */
IFK_API int ifk_natgrad_noalloc(const float* grad_W, int64_t ld_g,
                        const void* R_X, int64_t ld_rx, const void* R_G, int64_t ld_rg,
                        int r_dtype, float* nat, int64_t ld_nat,
                        int64_t n_out, int64_t n_in, int prec, int* d_status,
                        ifk_stream_t stream);

/* Workspace bytes for ifk_natgrad_batched: per layer, ifk_natgrad_workspace and
 * the scratch of its bias solve. */
IFK_API size_t ifk_natgrad_batched_workspace(int nlayers, const int64_t* n_out, const int64_t* n_in);

/*
 * ifk_natgrad for nlayers layers at once (host arrays of length nlayers).
 * Layers on the persistent bf16 path (bf16 factors, IFK_PREC_BF16, orders
 * that 16-byte copies address) share their launches: one launch of the
 * diagonal-block inverses of every factor, then for each of the four solves
 * one launch that packs the operand tiles of every layer and one that solves
 * every layer, the CTAs dealt across the layers' column groups.  Other layers
 * run one by one.  Each layer's result is the one ifk_natgrad gives.
 * grad_b / nat_b (both NULL, or arrays with an entry per layer, NULL for a layer
 * without bias): nat_b = R_G^-1 R_G^-T grad_b (n_out fp32, may alias), the
 * layer's bias as one more right-hand side of its left solves (the persistent
 * path) or ifk_natgrad_bias (the other layers).
 *
 * Replaces apply_vered_batched / _apply_vered_batched_impl and the graphed
 * bucketed apply of the reference (ifkfac/triangular.py:430-544,
 * ifkfac/ifkfac.py:315-423), with apply_vered_bias
 * (ifkfac/triangular.py:659-705) for the biases.
 */
IFK_API int ifk_natgrad_batched(int nlayers, const float* const* grad_W, const int64_t* ld_g,
                                const void* const* R_X, const int64_t* ld_rx, const void* const* R_G,
                                const int64_t* ld_rg, int r_dtype, float* const* nat,
                                const int64_t* ld_nat, const int64_t* n_out, const int64_t* n_in,
                                const float* const* grad_b, float* const* nat_b, int prec,
                                int* d_status, void* workspace, size_t workspace_bytes,
                                ifk_stream_t stream);

/*
 * nat_b = R_G^-1 R_G^-T grad_b (vectors of n_out fp32; may alias).
 * Replaces apply_vered_bias (ifkfac/triangular.py:659-705).
 */
IFK_API int ifk_natgrad_bias(const float* grad_b, const void* R_G, int64_t ld_rg, int r_dtype,
                     float* nat_b, int64_t n_out, int prec,
                     void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/* ---- update epilogue ------------------------------------------------------ */

/*
 * Per-layer update of the bucketed fast path (ifkfac/ifkfac.py:394-413):
 *   g = nat, scaled by grad_clip/||nat|| when grad_clip > 0 and ||nat|| > grad_clip;
 *   if momentum > 0: buf = momentum*buf + g (buf is read as zero when
 *   buf_is_new != 0, the reference's zero-initialised buffer), g = buf;
 *   if weight_decay > 0: W *= 1 - lr*weight_decay;  W -= lr*g.
 * W, buf and nat are `count` contiguous fp32 values; buf may be NULL when
 * momentum == 0.  grad_clip <= 0 disables clipping.  workspace holds the
 * norm reduction (ifk_update_workspace bytes) and may be NULL when clipping
 * is off.
 */
IFK_API size_t ifk_update_workspace(int64_t count);
IFK_API int ifk_update(float* W, float* buf, const float* nat, int64_t count,
               double lr, double momentum, double weight_decay, double grad_clip,
               int buf_is_new, void* workspace, size_t workspace_bytes, ifk_stream_t stream);

/*
 * Bias update (ifkfac/ifkfac.py:415-423): b *= 1 - lr*wd (wd > 0), b -= lr*nat_b.
 */
IFK_API int ifk_update_bias(float* b, const float* nat_b, int64_t count, double lr,
                    double weight_decay, ifk_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* IFK_H_ */
