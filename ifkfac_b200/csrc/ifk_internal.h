// Host-side launchers shared between the kernel files and the C ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace ifk {

// Working state of one fold: R (n x n fp32, in place) absorbs the rows of X
// (rows x n fp32 working copy, overwritten with Householder vectors).
struct FoldArgs {
  float* R;
  int64_t ldR;
  float* X;
  int64_t ldX;
  float* Tb;       // one NB x NB compact-WY T per sub-tile (column-major)
  int64_t n;
  int64_t rows;
  int64_t rows_R;  // meaningful rows of R before the fold
  int tiles;       // ceil(rows / SUB)
  int K;           // ceil(n / NB)
  int tri;         // chunk row i is zero left of column i
  int* err;        // device status word for bounded-wait timeouts (may be null)
};

// Up to MAX_FOLDS independent folds share one wave schedule (blockIdx.z selects the fold).
constexpr int MAX_FOLDS = 16;
struct FoldBatch {
  FoldArgs f[MAX_FOLDS];
  int nf;
};

size_t fold_tbuf_bytes(int64_t rows);
size_t xw_bytes(int64_t rows, int64_t n);
int64_t xw_ld(int64_t n);

// One fold of the persistent tensor-core path (fold_engine.cu).  Its rows come
// in up to MAX_SEGS segments that are folded in order, with the result of
// folding them one after another: a chunk read in place (fp32 or bf16), or
// ident * I (n rows, the damping rows).  Only the last segment may be
// trapezoidal (row i zero left of column i).
constexpr int MAX_SEGS = 12;
// One persistent launch takes up to PFOLD_MAX_FOLDS folds with PFOLD_MAX_BATCH_SEGS
// segments between them (the launch parameters hold both tables).
constexpr int PFOLD_MAX_FOLDS = 64;
constexpr int PFOLD_MAX_BATCH_SEGS = 256;
constexpr int PFOLD_MAX_CONV = 8;  // im2col segments per launch (their geometry is in the launch parameters)
// im2col geometry of a contiguous N x C x H x W tensor (the rows of F.unfold,
// transposed): row b * Ho * Wo + oh * Wo + ow, column (c * kh + ki) * kw + kj holds
// x[b, c, oh * sh - ph + ki * dh, ow * sw - pw + kj * dw], zero outside the image.
struct ConvGeo {
  int64_t B, C, H, W;
  int kh, kw, sh, sw, ph, pw, dh, dw, Ho, Wo;
};
// Value of im2col row si, column col (si < B * Ho * Wo, col < C * kh * kw): its
// offset in x, or -1 for the zero padding.
__host__ __device__ inline int64_t conv_offset(const ConvGeo& g, int64_t si, int64_t col) {
  const int64_t L = (int64_t)g.Ho * g.Wo;
  const int64_t b = si / L, l = si - b * L;
  const int oh = (int)(l / g.Wo), ow = (int)(l - (int64_t)oh * g.Wo);
  const int kk = g.kh * g.kw;
  const int64_t c = col / kk;
  const int rr = (int)(col - c * kk), ki = rr / g.kw, kj = rr - ki * g.kw;
  const int y = oh * g.sh - g.ph + ki * g.dh, x = ow * g.sw - g.pw + kj * g.dw;
  if (y < 0 || y >= g.H || x < 0 || x >= g.W) return -1;
  return ((b * g.C + c) * g.H + y) * g.W + x;
}

struct PFoldSeg {
  const void* X;
  int64_t ldX;
  int64_t rows;
  int xkind;     // 0 fp32, 1 bf16, 2 ident * I (X unused)
  float ident;
  int tri;
  const int64_t* ridx = nullptr;  // device row indices into X (rows of them), or null: rows 0 .. rows-1
  int64_t src_rows = 0;           // rows of X (bound for ridx)
  int64_t cols = -1;              // columns of X read (n, or n - 1 with a column of ones after them); < 0: n
  const ConvGeo* conv = nullptr;  // X is an NCHW image read through im2col (host pointer; src_rows = B Ho Wo)
};
struct PFoldDesc {
  float* R;
  int64_t ldR;
  int64_t n, rows_R;
  int nseg;
  PFoldSeg seg[MAX_SEGS];
};
inline PFoldDesc pfold_desc(float* R, int64_t ldR, int64_t n, int64_t rows_R) {
  PFoldDesc d{};
  d.R = R;
  d.ldR = ldR;
  d.n = n;
  d.rows_R = rows_R;
  return d;
}
inline void pfold_add(PFoldDesc& d, const void* X, int64_t ldX, int64_t rows, int xkind, float ident, int tri) {
  PFoldSeg g;
  g.X = X;
  g.ldX = ldX;
  g.rows = rows;
  g.xkind = xkind;
  g.ident = ident;
  g.tri = tri;
  d.seg[d.nseg++] = g;
}
// sub-tiles of a fold (sum over its segments)
int64_t pfold_subtiles(const PFoldDesc& d);
// most sub-tiles one launch takes for a fold of n columns
int64_t pfold_max_subtiles(int64_t n);
// workspace of one launch over folds of the given sub-tile counts and widths
size_t pfold_workspace(int nf, const int64_t* subtiles, const int64_t* n);
// one launch; every fold must have at most pfold_max_subtiles sub-tiles.  debug:
// PFOLD_DEBUG_WITHHOLD (tests only) withholds the first panel of the first fold and
// shortens the cross-CTA waits, so the launch ends with IFK_ERR_TIMEOUT.
constexpr int PFOLD_DEBUG_WITHHOLD = 1;
int pfold_run(int nf, const PFoldDesc* d, void* ws, int* status, cudaStream_t s, int debug = 0);

// chunk (bf16 or fp32, rows x n) -> X fp32.  With ridx, row i is chunk row ridx[i]
// (an index outside [0, src_rows) gives a zero row and IFK_ERR_ARG in *status);
// with cols = n - 1, column n - 1 is ones.
int copy_chunk(float* X, int64_t ldX, const void* chunk, int64_t ld_chunk, int64_t rows,
               int64_t n, int dtype, cudaStream_t s, const int64_t* ridx = nullptr, int64_t src_rows = 0,
               int64_t cols = -1, int* status = nullptr, const ConvGeo* conv = nullptr);
// X = sqrt(damping) I (n x n)
int fill_scaled_identity(float* X, int64_t ldX, int64_t n, float v, cudaStream_t s);
// Rout = upper(Rin) * scale (n x n fp32)
int scale_upper(float* Rout, int64_t ldo, const float* Rin, int64_t ldi, int64_t n, float scale,
                cudaStream_t s);
// Run the fold waves.  prec: IFK_PREC_FP32 or IFK_PREC_BF16.
int fold_run(const FoldArgs& a, int prec, cudaStream_t s);
int fold_run_batch(const FoldBatch& b, int prec, cudaStream_t s);
// Cast an n x n fp32 factor to the output type and flag non-finite entries; with
// scale > 0 the output is upper(R) / scale (scale_upper and the cast in one pass).
int finish_factor(void* out, int64_t ldo, int out_dtype, const float* R, int64_t ldR, int64_t n,
                  int* d_status, cudaStream_t s, float scale = 0.f);

// In-place triangular solve op(A) X = B on a strided view of B (n x N).
// A is an n x n upper-triangular factor (fp32 or bf16); trans != 0 solves
// with A^T (lower, forward order), trans == 0 with A (upper, backward).
// ws: trsm_tc_workspace(n) bytes for the tensor-core path (one launch per block
// row; inverses of the diagonal blocks); err: device status word for
// bounded-wait timeouts.
int trsm_run(const void* A, int64_t ldA, int a_dtype, int trans, float* B, int64_t rs,
             int64_t cs, int64_t n, int64_t N, int prec, void* ws, int* err, cudaStream_t s);
size_t trsm_tc_workspace(int64_t n);
// Persistent tensor-core solve (bf16 A that 16-byte copies can address: trsm_persist_ok).
// trsm_persist_prepare writes the diagonal-block inverses of one or two factors
// (trsm_persist_inverse_bytes(n) each, both operand layouts) in one launch;
// trsm_persist_run then needs trsm_persist_workspace(n, N) bytes of scratch.
bool trsm_persist_ok(const void* A, int64_t ldA, int64_t n);
size_t trsm_persist_inverse_bytes(int64_t n);
size_t trsm_persist_workspace(int64_t n, int64_t N);
int trsm_persist_prepare(const __nv_bfloat16* A0, int64_t ld0, int64_t n0, void* inv0, const __nv_bfloat16* A1,
                         int64_t ld1, int64_t n1, void* inv1, cudaStream_t s);
int trsm_persist_run(const __nv_bfloat16* A, int64_t ldA, int trans, float* B, int64_t rs, int64_t cs,
                     int64_t n, int64_t N, const void* inv, void* ws, int* err, cudaStream_t s);
// Several solves with the same op in one pack launch and one solve launch (groups
// of TRSM_MAX_PROBLEMS); each problem has its own trsm_persist_workspace scratch.
constexpr int TRSM_MAX_PROBLEMS = 64;
struct TrsmProblem {
  const __nv_bfloat16* A;
  int64_t ldA;
  float* B;
  int64_t rs, cs, n, N;
  const void* inv;
  void* ws;
};
int trsm_persist_run_many(int np, const TrsmProblem* p, int trans, int* err, cudaStream_t s);
// diagonal-block inverses of nm factors in one launch (groups of 2 TRSM_MAX_PROBLEMS)
int trsm_persist_prepare_many(int nm, const __nv_bfloat16* const* A, const int64_t* ld, const int64_t* n,
                              void* const* inv, cudaStream_t s);

int update_run(float* W, float* buf, const float* nat, int64_t count, double lr, double mom,
               double wd, double clip, int buf_is_new, double* norm_ws, cudaStream_t s);
int update_bias_run(float* b, const float* nat, int64_t count, double lr, double wd,
                    cudaStream_t s);

}  // namespace ifk
