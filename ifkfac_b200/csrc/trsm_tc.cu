// Tensor-core (tcgen05) blocked triangular solve, op(A) X = B in place.
//
// Block rows of NB2 = 128 rows are solved in order, one launch per block row
// j; each CTA owns NT right-hand-side columns.  Left-looking:
//   D   = sum_{s solved} op(A)_{j,s} X_s        tcgen05, bf16 operands, fp32 TMEM
//   Y   = B_j - D                               fp32
//   X_j = inv(op(A)_{j,j}) Y                    tcgen05, 3-term bf16 split
// inv(A_bb) of every diagonal block is computed first by column-parallel
// substitution in fp32 (one thread per column), so the diagonal solve is a
// product: the inverse of op(A)_jj = A_jj^T is the transpose of inv(A_jj).
// op(A) = A^T (trans) is lower triangular and solved forward; op(A) = A is
// upper and solved backward.  B is a strided view: the left solves of the
// natural gradient run on grad_W, the right solves on its transpose.
#include "ifk_common.cuh"
#include "ifk_internal.h"
#include "tc.cuh"

namespace ifk {

namespace {

constexpr int NB2 = 128;   // diagonal block
constexpr int NT = 32;     // right-hand-side columns per CTA
constexpr int TPB = 128;

constexpr uint32_t SZ_A = NB2 * NB2 * 2;  // op(A)_{j,s}, 32 KB
constexpr uint32_t SZ_X = NB2 * NT * 2;   // X_s / Y tile, 8 KB
constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_X = OFF_A + SZ_A;
constexpr uint32_t OFF_IH = OFF_X + SZ_X;
constexpr uint32_t OFF_IL = OFF_IH + SZ_A;
constexpr uint32_t OFF_YH = OFF_IL + SZ_A;
constexpr uint32_t OFF_YL = OFF_YH + SZ_X;
constexpr uint32_t OFF_BAR = OFF_YL + SZ_X;
constexpr uint32_t SMEM = OFF_BAR + 64;   // ~120 KB: one CTA per SM, so TMEM never contends

// A-operand tiles (128 x 128): mn-stride 128 B, k-stride 16 * 128 B
constexpr uint32_t A_MN = 128, A_K = (NB2 / 8) * 128;
// B-operand tiles (K = 128 rows q, N = NT columns c)
constexpr uint32_t X_N = 128, X_K = (NT / 8) * 128;
constexpr uint32_t TM_D = 0, TM_X = NT, TM_COLS = 64;
constexpr size_t INV_SMEM = 2 * sizeof(float) * NB2 * (NB2 + 1);

template <typename TA>
__device__ __forceinline__ float ldA(const TA* A, int64_t ldA_, int64_t i, int64_t j) {
  return ld_elem(A, i * ldA_ + j);
}

// inv(A_bb) of upper-triangular diagonal blocks, fp32, written as bf16 hi / lo
// (row-major 128 x 128 per block; a ragged last block is padded with identity).
template <typename TA>
__global__ void __launch_bounds__(NB2) diag_inverse_kernel(const TA* A, int64_t ldA_, int64_t n,
                                                           __nv_bfloat16* inv_hi, __nv_bfloat16* inv_lo) {
  extern __shared__ float dsm[];
  float (*U)[NB2 + 1] = reinterpret_cast<float (*)[NB2 + 1]>(dsm);
  float (*Xs)[NB2 + 1] = reinterpret_cast<float (*)[NB2 + 1]>(dsm + NB2 * (NB2 + 1));
  const int b = blockIdx.x, q = threadIdx.x;
  const int64_t b0 = (int64_t)b * NB2;
  const int nb = (int)mn<int64_t>(NB2, n - b0);
  for (int idx = q; idx < NB2 * NB2; idx += NB2) {
    const int r = idx / NB2, l = idx % NB2;
    float v = (r == l) ? 1.f : 0.f;
    if (r < nb && l < nb) v = (l >= r) ? ldA(A, ldA_, b0 + r, b0 + l) : 0.f;
    U[r][l] = v;
    Xs[r][l] = 0.f;
  }
  __syncthreads();
  // column q of U^-1: back substitution, rows r from the bottom
  for (int r = NB2 - 1; r >= 0; --r) {
    float s = (r == q) ? 1.f : 0.f;
    for (int l = r + 1; l < NB2; ++l) s -= U[r][l] * Xs[l][q];
    Xs[r][q] = s / U[r][r];
  }
  __syncthreads();
  __nv_bfloat16* oh = inv_hi + (size_t)b * NB2 * NB2;
  __nv_bfloat16* ol = inv_lo + (size_t)b * NB2 * NB2;
  for (int idx = q; idx < NB2 * NB2; idx += NB2) {
    const int r = idx / NB2, l = idx % NB2;
    float hi, lo;
    tc::split_bf16(Xs[r][l], hi, lo);
    oh[idx] = __float2bfloat16_rn(hi);
    ol[idx] = __float2bfloat16_rn(lo);
  }
}

__device__ __forceinline__ void st16(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void store8(uint32_t addr, const float (&v)[8]) {
  st16(addr, make_uint4(tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]), tc::pack_bf16(v[4], v[5]),
                        tc::pack_bf16(v[6], v[7])));
}

// One block row j for NT right-hand-side columns per CTA.
template <typename TA>
__global__ void __launch_bounds__(TPB, 1) trsm_row_tc_kernel(const TA* A, int64_t ldA_, int trans,
                                                            float* B, int64_t rs, int64_t cs, int64_t n,
                                                            int64_t N, int64_t jb,
                                                            const __nv_bfloat16* inv_hi,
                                                            const __nv_bfloat16* inv_lo, int* err) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  const uint32_t sb = tc::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nblk = cdiv(n, NB2);
  const int64_t j0 = jb * NB2;
  const int nj = (int)mn<int64_t>(NB2, n - j0);
  const int64_t c0 = (int64_t)blockIdx.x * NT;
  const int nc = (int)mn<int64_t>(NT, N - c0);

  if (warp == 0) tc::tmem_alloc(tslot, TM_COLS);
  if (tid == 0) tc::mbar_init(bar, 1);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = *tslot;
  uint32_t phase = 0;
  bool ok = true;

  // solved blocks: s < jb (forward) or s > jb (backward)
  const int64_t s_first = trans ? 0 : jb + 1;
  const int64_t s_last = trans ? jb : nblk;  // exclusive
  bool any = false;
#pragma unroll 1
  for (int64_t sblk = s_first; sblk < s_last; ++sblk) {
    const int64_t s0 = sblk * NB2;
    const int ns = (int)mn<int64_t>(NB2, n - s0);
    // op(A)_{j,s}[r][q]: upper -> A[j0+r][s0+q] (K-major rows); lower -> A[s0+q][j0+r] (MN-major)
    for (int it = tid; it < NB2 * (NB2 / 8); it += TPB) {
      float v[8];
      if (!trans) {
        const int r = (it & 7) + 8 * (it >> 7), q8 = (it >> 3) & 15;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int q = q8 * 8 + e;
          v[e] = (r < nj && q < ns) ? ldA(A, ldA_, j0 + r, s0 + q) : 0.f;
        }
        store8(sb + OFF_A + tc::cm_off<true>(r, q8 * 8, A_MN, A_K), v);
      } else {
        const int q = (it & 7) + 8 * (it >> 7), r8 = (it >> 3) & 15;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int r = r8 * 8 + e;
          v[e] = (r < nj && q < ns) ? ldA(A, ldA_, s0 + q, j0 + r) : 0.f;
        }
        store8(sb + OFF_A + tc::cm_off<false>(r8 * 8, q, A_MN, A_K), v);
      }
    }
    // X_s[q][c] as B (K = q, N = c), MN-major (8 consecutive columns per 16 B)
    for (int it = tid; it < NB2 * (NT / 8); it += TPB) {
      const int q = it / (NT / 8), c8 = it % (NT / 8);
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = c8 * 8 + e;
        v[e] = (q < ns && c < nc) ? B[(s0 + q) * rs + (c0 + c) * cs] : 0.f;
      }
      store8(sb + OFF_X + tc::cm_off<false>(c8 * 8, q, X_N, X_K), v);
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (tid == 0) {
      const uint32_t id = trans ? tc::idesc_bf16(128, NT, true, true) : tc::idesc_bf16(128, NT, false, true);
#pragma unroll 1
      for (int k = 0; k < NB2 / 16; ++k) {
        const uint64_t ad = tc::sdesc(sb + OFF_A + k * 2 * A_K, A_K, A_MN);
        const uint64_t bd = tc::sdesc(sb + OFF_X + k * 2 * X_K, X_K, X_N);
        tc::mma_bf16(tm + TM_D, ad, bd, id, (any || k > 0) ? 1u : 0u);
      }
      tc::commit(bar);
    }
    any = true;
    ok = tc::mbar_wait(bar, phase) && ok;
    phase ^= 1;
    tc::fence_after();
  }

  // ---- Y = B_j - D, split hi/lo as B operand (MN-major); stage inv(op(A)_jj) hi/lo ----
  const int r = warp * 32 + lane;  // row of block j == TMEM lane
  const uint32_t lane_base = tm + ((uint32_t)(warp * 32) << 16);
  {
    float d[32];
    if (any) {
      tc::tmem_ld32(lane_base + TM_D, d);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) d[e] = 0.f;
    }
#pragma unroll
    for (int g = 0; g < NT / 8; ++g) {
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = g * 8 + e;
        const float bv = (r < nj && c < nc) ? B[(j0 + r) * rs + (c0 + c) * cs] : 0.f;
        tc::split_bf16(bv - d[c], hi[e], lo[e]);
      }
      const uint32_t off = tc::cm_off<false>(g * 8, r, X_N, X_K);
      store8(sb + OFF_YH + off, hi);
      store8(sb + OFF_YL + off, lo);
    }
  }
  {
    const uint4* ih = reinterpret_cast<const uint4*>(inv_hi + (size_t)jb * NB2 * NB2);
    const uint4* il = reinterpret_cast<const uint4*>(inv_lo + (size_t)jb * NB2 * NB2);
    // inv(U_jj) row-major: 16 B = 8 consecutive columns l of row m.
    // upper: operand (r = m, q = l) K-major; lower: inverse is the transpose, (r = l, q = m) MN-major
    for (int it = tid; it < NB2 * (NB2 / 8); it += TPB) {
      const int m = it >> 4, l8 = it & 15;
      const uint32_t off = trans ? tc::cm_off<false>(l8 * 8, m, A_MN, A_K) : tc::cm_off<true>(m, l8 * 8, A_MN, A_K);
      st16(sb + OFF_IH + off, ih[it]);
      st16(sb + OFF_IL + off, il[it]);
    }
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (tid == 0) {
    const uint32_t id = tc::idesc_bf16(128, NT, trans != 0, true);
#pragma unroll 1
    for (int k = 0; k < NB2 / 16; ++k) {
      const uint64_t ah = tc::sdesc(sb + OFF_IH + k * 2 * A_K, A_K, A_MN);
      const uint64_t al = tc::sdesc(sb + OFF_IL + k * 2 * A_K, A_K, A_MN);
      const uint64_t bh = tc::sdesc(sb + OFF_YH + k * 2 * X_K, X_K, X_N);
      const uint64_t bl = tc::sdesc(sb + OFF_YL + k * 2 * X_K, X_K, X_N);
      tc::mma_bf16(tm + TM_X, ah, bh, id, k > 0);
      tc::mma_bf16(tm + TM_X, ah, bl, id, 1);
      tc::mma_bf16(tm + TM_X, al, bh, id, 1);
    }
    tc::commit(bar);
  }
  ok = tc::mbar_wait(bar, phase) && ok;
  tc::fence_after();
  {
    float x[32];
    tc::tmem_ld32(lane_base + TM_X, x);
    if (r < nj) {
#pragma unroll
      for (int c = 0; c < NT; ++c)
        if (c < nc) B[(j0 + r) * rs + (c0 + c) * cs] = x[c];
    }
  }
  if (!ok && err) atomicExch(err, IFK_ERR_TIMEOUT);
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(tm, TM_COLS);
  }
}

template <typename TA>
bool attr_once() {
  static thread_local int done_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (done_dev == dev) return true;
  if (cudaFuncSetAttribute(trsm_row_tc_kernel<TA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)SMEM) != cudaSuccess)
    return false;
  if (cudaFuncSetAttribute(diag_inverse_kernel<TA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)INV_SMEM) != cudaSuccess)
    return false;
  done_dev = dev;
  return true;
}

template <typename TA>
int run(const TA* A, int64_t ldA_, int trans, float* B, int64_t rs, int64_t cs, int64_t n, int64_t N,
        __nv_bfloat16* inv, int* err, cudaStream_t s) {
  if (!attr_once<TA>()) return IFK_ERR_CUDA;
  const int64_t nblk = cdiv(n, NB2);
  __nv_bfloat16* ih = inv;
  __nv_bfloat16* il = inv + (size_t)nblk * NB2 * NB2;
  diag_inverse_kernel<TA><<<(unsigned)nblk, NB2, INV_SMEM, s>>>(A, ldA_, n, ih, il);
  const unsigned grid = (unsigned)cdiv(N, NT);
  for (int64_t step = 0; step < nblk; ++step) {
    const int64_t jb = trans ? step : nblk - 1 - step;
    trsm_row_tc_kernel<TA><<<grid, TPB, SMEM, s>>>(A, ldA_, trans, B, rs, cs, n, N, jb, ih, il, err);
  }
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

}  // namespace

size_t trsm_tc_workspace(int64_t n) { return (size_t)cdiv(n, NB2) * NB2 * NB2 * 2 * sizeof(__nv_bfloat16); }

int trsm_tc_run(const void* A, int64_t ldA_, int a_dtype, int trans, float* B, int64_t rs, int64_t cs,
                int64_t n, int64_t N, void* ws, int* err, cudaStream_t s) {
  if (a_dtype == IFK_BF16)
    return run((const __nv_bfloat16*)A, ldA_, trans, B, rs, cs, n, N, (__nv_bfloat16*)ws, err, s);
  return run((const float*)A, ldA_, trans, B, rs, cs, n, N, (__nv_bfloat16*)ws, err, s);
}

}  // namespace ifk
