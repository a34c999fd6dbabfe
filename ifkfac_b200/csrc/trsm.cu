// Blocked multi-right-hand-side triangular solves.
//
// op(A) X = B is solved in place on a strided view of B (n x N), with A an
// upper-triangular factor (fp32 or bf16 storage) and op(A) = A (upper,
// back substitution) or A^T (lower, forward substitution).  Block rows of NS
// rows are visited in solve order; at each step the diagonal block is solved
// for every right-hand-side tile (one thread per column, substitution with
// fp32 FMAs), then the solved block is eliminated from every later block row
// by a GEMM tile update B_j -= op(A)_{j,s} X_s.
//
// The four solves of the natural gradient (ifkfac/triangular.py:630-656)
// are two calls on grad_W (R_G^T then R_G) and two on its transpose view
// (R_X^T then R_X).
#include "ifk_common.cuh"
#include "ifk_internal.h"

namespace ifk {

namespace {

constexpr int LDS_ = NRHS + 1;

// op(A)[i][j] for block-local reads.
template <typename TA>
__device__ __forceinline__ float opA(const TA* A, int64_t ldA, int trans, int64_t i, int64_t j) {
  return trans ? ld_elem(A, j * ldA + i) : ld_elem(A, i * ldA + j);
}

// DIAG_TPB threads load the tiles (DIAG_LD loads in flight per thread); the
// first NRHS of them then solve one column each.
constexpr int DIAG_TPB = 256;
constexpr int DIAG_LD = NS * NS / DIAG_TPB;  // 16
static_assert(NS * NRHS == NS * NS, "square tiles");

template <typename TA>
__global__ void __launch_bounds__(DIAG_TPB) trsm_diag_kernel(const TA* A, int64_t ldA, int trans,
                                                             float* B, int64_t rs, int64_t cs,
                                                             int64_t n, int64_t N, int64_t b0) {
  __shared__ float Ad[NS][NS + 1];
  __shared__ float Bs[NS][LDS_];
  const int tid = threadIdx.x;
  const int64_t c0 = (int64_t)blockIdx.x * NRHS;
  const int nb = (int)mn<int64_t>(NS, n - b0);
  const int nc = (int)mn<int64_t>(NRHS, N - c0);
  // A's contiguous index fastest across threads: j for op = A, i for op = A^T.
  // B's contiguous index too: the columns of a row-major view, the rows of a
  // transposed one (rs == 1).  All loads of a thread are issued before its stores.
  const bool tv = rs == 1 && cs != 1;
  {
    float va[DIAG_LD], vb[DIAG_LD];
#pragma unroll
    for (int u = 0; u < DIAG_LD; ++u) {
      const int idx = tid + u * DIAG_TPB;
      const int i = trans ? idx % NS : idx / NS, j = trans ? idx / NS : idx % NS;
      va[u] = (i < nb && j < nb) ? opA(A, ldA, trans, b0 + i, b0 + j) : (i == j ? 1.f : 0.f);
      const int bi = tv ? idx % NS : idx / NRHS, bj = tv ? idx / NS : idx % NRHS;
      vb[u] = (bi < nb && bj < nc) ? B[(b0 + bi) * rs + (c0 + bj) * cs] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < DIAG_LD; ++u) {
      const int idx = tid + u * DIAG_TPB;
      const int i = trans ? idx % NS : idx / NS, j = trans ? idx / NS : idx % NS;
      Ad[i][j] = va[u];
      const int bi = tv ? idx % NS : idx / NRHS, bj = tv ? idx / NS : idx % NRHS;
      Bs[bi][bj] = vb[u];
    }
  }
  __syncthreads();
  // Column c by column-oriented substitution: its residues stay in registers; once
  // x_r = res_r / op(A)[r][r] is known it is folded into the rows still to come
  // with independent FMAs (op(A)[l][r] is the same for every column: a broadcast).
  // Rows past nb are the identity pad and come out zero.
  const int c = tid;
  if (c < NRHS) {
    float res[NS];
#pragma unroll
    for (int i = 0; i < NS; ++i) res[i] = Bs[i][c];
    if (trans) {  // lower: forward
#pragma unroll
      for (int r = 0; r < NS; ++r) {
        const float x = res[r] / Ad[r][r];
        res[r] = x;
#pragma unroll
        for (int l = r + 1; l < NS; ++l) res[l] = fmaf(-Ad[l][r], x, res[l]);
      }
    } else {  // upper: backward
#pragma unroll
      for (int r = NS - 1; r >= 0; --r) {
        const float x = res[r] / Ad[r][r];
        res[r] = x;
#pragma unroll
        for (int l = 0; l < r; ++l) res[l] = fmaf(-Ad[l][r], x, res[l]);
      }
    }
#pragma unroll
    for (int i = 0; i < NS; ++i) Bs[i][c] = res[i];
  }
  __syncthreads();
  for (int idx = tid; idx < NS * NRHS; idx += DIAG_TPB) {
    const int i = tv ? idx % NS : idx / NRHS, j = tv ? idx / NS : idx % NRHS;
    if (i < nb && j < nc) B[(b0 + i) * rs + (c0 + j) * cs] = Bs[i][j];
  }
}

// B_j -= op(A)[j block, s block] X_s for every block row j after s in solve order.
template <typename TA>
__global__ void __launch_bounds__(256) trsm_update_kernel(const TA* A, int64_t ldA, int trans,
                                                          float* B, int64_t rs, int64_t cs,
                                                          int64_t n, int64_t N, int64_t s0) {
  // op(A)'s tile transposed (AsT[l][i]) and X's tile, rows 16-byte aligned: the
  // product loop reads one float4 of each per step
  __shared__ __align__(16) float AsT[NS][NS + 4];
  __shared__ __align__(16) float Xs[NS][NRHS + 4];
  const int tid = threadIdx.x;
  // trans (forward): targets are the blocks after s; otherwise the blocks before s.
  const int64_t jb = trans ? (s0 / NS + 1 + blockIdx.x) : blockIdx.x;
  const int64_t j0 = jb * NS;
  if (trans ? (j0 >= n) : (j0 >= s0)) return;
  const int64_t c0 = (int64_t)blockIdx.y * NRHS;
  const int nj = (int)mn<int64_t>(NS, n - j0);
  const int ns = (int)mn<int64_t>(NS, n - s0);
  const int nc = (int)mn<int64_t>(NRHS, N - c0);
  // A's contiguous index fastest across threads (l for op = A, i for op = A^T), and
  // B's (see trsm_diag_kernel): the tile loads and the read-modify-writes of the
  // result coalesce.  All loads of a thread are issued before its stores.
  const bool tv = rs == 1 && cs != 1;
  {
    constexpr int LD = NS * NS / 256;
    float va[LD], vx[LD];
#pragma unroll
    for (int u = 0; u < LD; ++u) {
      const int idx = tid + u * 256;
      const int i = trans ? idx % NS : idx / NS, l = trans ? idx / NS : idx % NS;
      va[u] = (i < nj && l < ns) ? opA(A, ldA, trans, j0 + i, s0 + l) : 0.f;
      const int xl = tv ? idx % NS : idx / NRHS, xc = tv ? idx / NS : idx % NRHS;
      vx[u] = (xl < ns && xc < nc) ? B[(s0 + xl) * rs + (c0 + xc) * cs] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < LD; ++u) {
      const int idx = tid + u * 256;
      const int i = trans ? idx % NS : idx / NS, l = trans ? idx / NS : idx % NS;
      AsT[l][i] = va[u];
      const int xl = tv ? idx % NS : idx / NRHS, xc = tv ? idx / NS : idx % NRHS;
      Xs[xl][xc] = vx[u];
    }
  }
  __syncthreads();
  // thread tile: rows ri .. ri + 3, columns ci .. ci + 3 of the result, the
  // contiguous one taken from the lane index
  const int ty = tid / 16, tx = tid % 16;
  const int ri = (tv ? tx : ty) * 4, ci = (tv ? ty : tx) * 4;
  float acc[4][4] = {};
#pragma unroll 8
  for (int l = 0; l < NS; ++l) {
    const float4 a4 = *reinterpret_cast<const float4*>(&AsT[l][ri]);
    const float4 b4 = *reinterpret_cast<const float4*>(&Xs[l][ci]);
    const float av[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[r][q] += av[r] * bv[q];
  }
  // the result's four contiguous elements (the columns of a row-major view, the
  // rows of a transposed one) by one 16-byte read-modify-write where aligned
  const int64_t cstride = tv ? rs : cs;  // stride of the contiguous index (1)
  const bool vec = cstride == 1 && (((uintptr_t)B) & 15) == 0 && ((tv ? cs : rs) & 3) == 0 &&
                   (((tv ? j0 : c0) & 3) == 0);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    // u runs over the non-contiguous index of the thread tile
    const int i0 = tv ? ri : ri + u, cc0 = tv ? ci + u : ci;
    float* p = B + (j0 + i0) * rs + (c0 + cc0) * cs;
    const int left = tv ? nj - ri : nc - ci;  // valid contiguous elements from the tile's start
    const bool inb = tv ? (cc0 < nc) : (i0 < nj);
    if (!inb) continue;
    if (vec && left >= 4) {
      float4 v = *reinterpret_cast<float4*>(p);
      v.x -= tv ? acc[0][u] : acc[u][0];
      v.y -= tv ? acc[1][u] : acc[u][1];
      v.z -= tv ? acc[2][u] : acc[u][2];
      v.w -= tv ? acc[3][u] : acc[u][3];
      *reinterpret_cast<float4*>(p) = v;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (e < left) {
          float* pe = p + (tv ? (int64_t)e * rs : (int64_t)e * cs);
          *pe -= tv ? acc[e][u] : acc[u][e];
        }
      }
    }
  }
}

template <typename TA>
int trsm_simt(const TA* A, int64_t ldA, int trans, float* B, int64_t rs, int64_t cs, int64_t n,
              int64_t N, cudaStream_t s) {
  const int64_t nblk = cdiv(n, NS);
  const unsigned ctiles = (unsigned)cdiv(N, NRHS);
  for (int64_t step = 0; step < nblk; ++step) {
    const int64_t sb = trans ? step : (nblk - 1 - step);
    const int64_t s0 = sb * NS;
    trsm_diag_kernel<TA><<<ctiles, DIAG_TPB, 0, s>>>(A, ldA, trans, B, rs, cs, n, N, s0);
    const int64_t rem = trans ? (nblk - 1 - sb) : sb;
    if (rem > 0) {
      trsm_update_kernel<TA><<<dim3((unsigned)rem, ctiles), 256, 0, s>>>(A, ldA, trans, B, rs, cs,
                                                                         n, N, s0);
    }
  }
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

}  // namespace

int trsm_tc_run(const void* A, int64_t ldA, int a_dtype, int trans, float* B, int64_t rs,
                int64_t cs, int64_t n, int64_t N, void* ws, int* err, cudaStream_t s);

int trsm_run(const void* A, int64_t ldA, int a_dtype, int trans, float* B, int64_t rs, int64_t cs,
             int64_t n, int64_t N, int prec, void* ws, int* err, cudaStream_t s) {
  if (n == 0 || N == 0) return IFK_OK;
  if (prec == IFK_PREC_BF16) return trsm_tc_run(A, ldA, a_dtype, trans, B, rs, cs, n, N, ws, err, s);
  if (a_dtype == IFK_BF16)
    return trsm_simt((const __nv_bfloat16*)A, ldA, trans, B, rs, cs, n, N, s);
  return trsm_simt((const float*)A, ldA, trans, B, rs, cs, n, N, s);
}

}  // namespace ifk
