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
constexpr uint32_t OFF_A = 0;                 // two buffers
constexpr uint32_t OFF_X = OFF_A + 2 * SZ_A;  // two buffers
constexpr uint32_t OFF_IH = OFF_X + 2 * SZ_X;
constexpr uint32_t OFF_IL = OFF_IH + SZ_A;
constexpr uint32_t OFF_YH = OFF_IL + SZ_A;
constexpr uint32_t OFF_YL = OFF_YH + SZ_X;
constexpr uint32_t OFF_BAR = OFF_YL + SZ_X;
constexpr uint32_t SMEM = OFF_BAR + 64;   // ~160 KB: one CTA per SM, so TMEM never contends

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

// 8 consecutive elements of op(A) as 8 bf16 (16 bytes); vectorised when in bounds.
__device__ __forceinline__ uint4 ld8_bf16(const __nv_bfloat16* p, int valid, bool vec) {
  if (vec && valid >= 8) return *reinterpret_cast<const uint4*>(p);
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = e < valid ? __bfloat162float(p[e]) : 0.f;
  return make_uint4(tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]), tc::pack_bf16(v[4], v[5]),
                    tc::pack_bf16(v[6], v[7]));
}
__device__ __forceinline__ uint4 ld8_bf16(const float* p, int valid, bool vec) {
  float4 a, b;
  if (vec) {
    a = ld4(p, valid);
    b = ld4(p + 4, valid - 4);
  } else {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = e < valid ? p[e] : 0.f;
    a = make_float4(v[0], v[1], v[2], v[3]);
    b = make_float4(v[4], v[5], v[6], v[7]);
  }
  return make_uint4(tc::pack_bf16(a.x, a.y), tc::pack_bf16(a.z, a.w), tc::pack_bf16(b.x, b.y),
                    tc::pack_bf16(b.z, b.w));
}

// One block row j for NT right-hand-side columns per CTA.  BKM: the right-hand
// sides are a transposed view (rs == 1), so solved blocks X_s are staged as a
// K-major B operand (8 consecutive rows q per 16 bytes, contiguous in memory);
// otherwise MN-major (8 consecutive columns c).  VA / VB: 16-byte loads allowed.
template <typename TA, bool BKM>
__global__ void __launch_bounds__(TPB, 1) trsm_row_tc_kernel(const TA* A, int64_t ldA_, int trans,
                                                            float* B, int64_t rs, int64_t cs, int64_t n,
                                                            int64_t N, int64_t jb,
                                                            const __nv_bfloat16* inv_hi,
                                                            const __nv_bfloat16* inv_lo, int* err,
                                                            int va, int vb) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);  // [0],[1]: K-loop buffers, [2]: diagonal
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 32);
  const uint32_t sb = tc::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nblk = cdiv(n, NB2);
  const int64_t j0 = jb * NB2;
  const int nj = (int)mn<int64_t>(NB2, n - j0);
  const int64_t c0 = (int64_t)blockIdx.x * NT;
  const int nc = (int)mn<int64_t>(NT, N - c0);

  if (warp == 0) tc::tmem_alloc(tslot, TM_COLS);
  if (tid == 0) {
    tc::mbar_init(&bar[0], 1);
    tc::mbar_init(&bar[1], 1);
    tc::mbar_init(&bar[2], 1);
  }
  // inv(op(A)_jj) hi/lo; inv(U_jj) row-major, 16 B = 8 consecutive columns l of row m.
  // upper: operand (r = m, q = l) K-major; lower: the transpose, (r = l, q = m) MN-major
  {
    const uint4* ih = reinterpret_cast<const uint4*>(inv_hi + (size_t)jb * NB2 * NB2);
    const uint4* il = reinterpret_cast<const uint4*>(inv_lo + (size_t)jb * NB2 * NB2);
    for (int it = tid; it < NB2 * (NB2 / 8); it += TPB) {
      const int m = it >> 4, l8 = it & 15;
      const uint32_t off = trans ? tc::cm_off<false>(l8 * 8, m, A_MN, A_K) : tc::cm_off<true>(m, l8 * 8, A_MN, A_K);
      st16(sb + OFF_IH + off, ih[it]);
      st16(sb + OFF_IL + off, il[it]);
    }
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = *tslot;
  bool ok = true;

  // solved blocks: s < jb (forward) or s > jb (backward)
  const int64_t s_first = trans ? 0 : jb + 1;
  const int64_t s_last = trans ? jb : nblk;  // exclusive
  const int nsteps = (int)(s_last - s_first);
  const uint32_t idK = tc::idesc_bf16(128, NT, trans != 0, !BKM);
#pragma unroll 1
  for (int it = 0; it < nsteps; ++it) {
    const int bsel = it & 1;
    if (it >= 2) ok = tc::mbar_wait(&bar[bsel], ((it >> 1) - 1) & 1) && ok;  // MMAs of it-2 done
    const uint32_t offA = OFF_A + bsel * SZ_A, offX = OFF_X + bsel * SZ_X;
    const int64_t s0 = (s_first + it) * NB2;
    const int ns = (int)mn<int64_t>(NB2, n - s0);
    // op(A)_{j,s}[r][q]: upper -> A[j0+r][s0+q] (K-major rows); lower -> A[s0+q][j0+r] (MN-major)
    for (int i0 = tid; i0 < NB2 * (NB2 / 8); i0 += 4 * TPB) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * TPB;
        if (!trans) {
          const int r = (i & 7) + 8 * (i >> 7), q8 = (i >> 3) & 15;
          v[u] = r < nj ? ld8_bf16(A + (j0 + r) * ldA_ + s0 + q8 * 8, ns - q8 * 8, va) : make_uint4(0, 0, 0, 0);
        } else {
          const int q = (i & 7) + 8 * (i >> 7), r8 = (i >> 3) & 15;
          v[u] = q < ns ? ld8_bf16(A + (s0 + q) * ldA_ + j0 + r8 * 8, nj - r8 * 8, va) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * TPB;
        uint32_t off;
        if (!trans) {
          const int r = (i & 7) + 8 * (i >> 7), q8 = (i >> 3) & 15;
          off = tc::cm_off<true>(r, q8 * 8, A_MN, A_K);
        } else {
          const int q = (i & 7) + 8 * (i >> 7), r8 = (i >> 3) & 15;
          off = tc::cm_off<false>(r8 * 8, q, A_MN, A_K);
        }
        st16(sb + offA + off, v[u]);
      }
    }
    // X_s[q][c] as B (K = q, N = c)
    for (int i = tid; i < NB2 * (NT / 8); i += TPB) {
      if (!BKM) {  // MN-major: 8 consecutive columns c of row q
        const int q = i / (NT / 8), c8 = i % (NT / 8);
        const uint4 v = q < ns ? ld8_bf16(B + (s0 + q) * rs + (c0 + c8 * 8) * cs, nc - c8 * 8, vb)
                               : make_uint4(0, 0, 0, 0);
        st16(sb + offX + tc::cm_off<false>(c8 * 8, q, X_N, X_K), v);
      } else {     // K-major: 8 consecutive rows q of column c (contiguous in the transposed view)
        const int c = i % NT, q8 = i / NT;
        const uint4 v = c < nc ? ld8_bf16(B + (s0 + q8 * 8) * rs + (c0 + c) * cs, ns - q8 * 8, vb)
                               : make_uint4(0, 0, 0, 0);
        st16(sb + offX + tc::cm_off<true>(c, q8 * 8, X_N, X_K), v);
      }
    }
    tc::fence_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (tid == 0) {
#pragma unroll 1
      for (int k = 0; k < NB2 / 16; ++k) {
        const uint64_t ad = tc::sdesc(sb + offA + k * 2 * A_K, A_K, A_MN);
        const uint64_t bd = tc::sdesc(sb + offX + k * 2 * X_K, X_K, X_N);
        tc::mma_bf16(tm + TM_D, ad, bd, idK, (it > 0 || k > 0) ? 1u : 0u);
      }
      tc::commit(&bar[bsel]);
    }
  }
  if (nsteps > 0) {
    const int last = nsteps - 1;
    ok = tc::mbar_wait(&bar[last & 1], (last >> 1) & 1) && ok;  // in-order completion: all K-loop MMAs
    tc::fence_after();
  }

  // ---- Y = B_j - D, split hi/lo as B operand (MN-major) ----
  const int r = warp * 32 + lane;  // row of block j == TMEM lane
  const uint32_t lane_base = tm + ((uint32_t)(warp * 32) << 16);
  {
    float d[32];
    if (nsteps > 0) {
      tc::tmem_ld32(lane_base + TM_D, d);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) d[e] = 0.f;
    }
    float bv[NT];
    if (cs == 1 && vb) {
#pragma unroll
      for (int g = 0; g < NT / 4; ++g) {
        const float4 x = r < nj ? ld4(B + (j0 + r) * rs + c0 + 4 * g, nc - 4 * g) : make_float4(0.f, 0.f, 0.f, 0.f);
        bv[4 * g] = x.x; bv[4 * g + 1] = x.y; bv[4 * g + 2] = x.z; bv[4 * g + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < NT; ++c) bv[c] = (r < nj && c < nc) ? B[(j0 + r) * rs + (c0 + c) * cs] : 0.f;
    }
#pragma unroll
    for (int g = 0; g < NT / 8; ++g) {
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) tc::split_bf16(bv[g * 8 + e] - d[g * 8 + e], hi[e], lo[e]);
      const uint32_t off = tc::cm_off<false>(g * 8, r, X_N, X_K);
      store8(sb + OFF_YH + off, hi);
      store8(sb + OFF_YL + off, lo);
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
    tc::commit(&bar[2]);
  }
  ok = tc::mbar_wait(&bar[2], 0) && ok;
  tc::fence_after();
  {
    float x[32];
    tc::tmem_ld32(lane_base + TM_X, x);
    if (r < nj) {
      if (cs == 1 && vb) {
#pragma unroll
        for (int g = 0; g < NT / 4; ++g)
          st4(B + (j0 + r) * rs + c0 + 4 * g, make_float4(x[4 * g], x[4 * g + 1], x[4 * g + 2], x[4 * g + 3]),
              nc - 4 * g);
      } else {
#pragma unroll
        for (int c = 0; c < NT; ++c)
          if (c < nc) B[(j0 + r) * rs + (c0 + c) * cs] = x[c];
      }
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
  if (cudaFuncSetAttribute(trsm_row_tc_kernel<TA, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)SMEM) != cudaSuccess)
    return false;
  if (cudaFuncSetAttribute(trsm_row_tc_kernel<TA, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  // 16-byte vector loads need 16-byte aligned rows
  const int va = (((uintptr_t)A % 16) == 0 && (ldA_ * (int64_t)sizeof(TA)) % 16 == 0) ? 1 : 0;
  const int vb = (((uintptr_t)B % 16) == 0 && ((rs == 1 ? cs : rs) * 4) % 16 == 0) ? 1 : 0;
  const unsigned grid = (unsigned)cdiv(N, NT);
  for (int64_t step = 0; step < nblk; ++step) {
    const int64_t jb = trans ? step : nblk - 1 - step;
    if (rs == 1 && cs != 1)
      trsm_row_tc_kernel<TA, true><<<grid, TPB, SMEM, s>>>(A, ldA_, trans, B, rs, cs, n, N, jb, ih, il, err, va, vb);
    else
      trsm_row_tc_kernel<TA, false><<<grid, TPB, SMEM, s>>>(A, ldA_, trans, B, rs, cs, n, N, jb, ih, il, err, va, vb);
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
