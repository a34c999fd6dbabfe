// Householder panel factorisation of the streaming TSQR fold (device code shared
// by the wave scheduler in tsqr.cu and the persistent fold in fold_engine.cu).
#pragma once

#include "ifk_common.cuh"

namespace ifk {
namespace panel {

#ifdef IFK_TRACE
// Diagnostic build only: time spent in each phase of panel_factor (ns, summed over panels).
__device__ unsigned long long g_panel_phase[16];
__device__ __forceinline__ long long ptime() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define PH_MARK(i)                                                                      \
  do {                                                                                  \
    if (threadIdx.x == 0) {                                                             \
      const long long t_ = ptime();                                                     \
      atomicAdd(&g_panel_phase[i], (unsigned long long)(t_ - ph_last));                  \
      ph_last = t_;                                                                     \
    }                                                                                   \
  } while (0)
#else
#define PH_MARK(i) do { } while (0)
#endif

constexpr int LDP = NB + 1;   // row stride of the small NB x NB blocks
constexpr int SP = SUB + 4;    // column stride of the panel: column-major, 16-byte aligned columns
constexpr int LDW2 = 52;       // row stride of the inner-update W (16-byte aligned rows)

// ---- panel factorisation ----------------------------------------------------
// 256 threads; thread t owns row t of the sub-tile.  The NB = 64 panel columns
// are processed in 4 leaves of 16: a leaf's row lives in 16 registers per
// thread and each column step needs one reduction of 16 dot products
// (x_j . x_c for every leaf column c: c == j gives the squared norm, c > j the
// inputs of w, c < j the entries of Y^T Y for T) and one __syncthreads.  The
// reduction is a warp butterfly that halves the payload each round
// (8+4+2+1+1 shuffles), then 8 warp partials from shared memory.  After a
// leaf, its compact-WY block reflector is applied to the remaining panel
// columns with register-tiled micro-GEMMs on the column-major panel; after the
// panel, T is assembled from the leaf T's by T_AB = -T_A (Y_A^T Y_B) T_B.
constexpr int PT2 = 256;
constexpr int NWARP = PT2 / 32;
constexpr int LEAF = 16;
constexpr int NLEAF = NB / LEAF;
static_assert(SUB == PT2, "the panel maps one row to each thread");

struct PanelSmem {
  float P[NB * SP];          // X_t[:, panel] -> Y, column-major: element (i, c) at P[c * SP + i]
  float Rk[NB * LDP];        // diagonal block of R
  float G[NB * LDP];         // strict upper part of Y^T Y
  float Tm[NB * LDP];        // T, row-major
  float Tmp[NB * LDP];       // scratch: inner-update Z, G partial sums, T assembly
  float Rl[LEAF * (LEAF + 1)];
  float Wb[LEAF * LDW2];     // W of the inner update (row-major)
  float part[2][NWARP][LEAF];
  float tau[NB];
};

__device__ __forceinline__ void reflector(float aj, float xn2, float& tj, float& beta, float& inv_v0) {
  if (xn2 == 0.f) {
    // nothing to annihilate; flip the row if its diagonal is negative
    tj = aj >= 0.f ? 0.f : 2.f;
    beta = fabsf(aj);
    inv_v0 = 0.f;
  } else {
    const float nrm = __fsqrt_rn(aj * aj + xn2);
    const float v0 = aj > 0.f ? -xn2 * __frcp_rn(aj + nrm) : aj - nrm;
    beta = nrm;
    tj = -v0 * __frcp_rn(nrm);
    inv_v0 = __frcp_rn(v0);
  }
}

// Butterfly reduce-scatter of 16 values over a warp: returns the warp total of
// value index ((lane>>4)&1)*8 + ((lane>>3)&1)*4 + ((lane>>2)&1)*2 + ((lane>>1)&1).
__device__ __forceinline__ float warp_reduce16(float (&v)[16], int lane) {
  const unsigned F = 0xffffffffu;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const bool hi = lane & 16;
    const float send = hi ? v[k] : v[k + 8];
    const float keep = hi ? v[k + 8] : v[k];
    v[k] = keep + __shfl_xor_sync(F, send, 16);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bool hi = lane & 8;
    const float send = hi ? v[k] : v[k + 4];
    const float keep = hi ? v[k + 4] : v[k];
    v[k] = keep + __shfl_xor_sync(F, send, 8);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool hi = lane & 4;
    const float send = hi ? v[k] : v[k + 2];
    const float keep = hi ? v[k + 2] : v[k];
    v[k] = keep + __shfl_xor_sync(F, send, 4);
  }
  {
    const bool hi = lane & 2;
    const float send = hi ? v[0] : v[1];
    const float keep = hi ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(F, send, 2);
  }
  return v[0] + __shfl_xor_sync(F, v[0], 1);
}

// dst block (m x n at dr, dc) = (neg ? -1 : 1) * A (m x k at ar, ac) * M (k x n at mr, mc),
// row-major LDP-stride blocks in shared memory; all PT2 threads.  Used for T assembly.
__device__ __forceinline__ void matmul(float* dst, int dr, int dc, const float* A, int ar, int ac,
                                       const float* M, int mr, int mc, int m, int k, int n, int tid, bool neg) {
  for (int o = tid; o < m * n; o += PT2) {
    const int i = o / n, j = o % n;
    float s = 0.f;
    for (int l = 0; l < k; ++l) s += A[(ar + i) * LDP + ac + l] * M[(mr + l) * LDP + mc + j];
    dst[(dr + i) * LDP + dc + j] = neg ? -s : s;
  }
}

// Factor the panel in S.P (SUB x NB fp32, column-major; rows beyond the
// sub-tile are zero) under the R diagonal block S.Rk.  nbk panel columns exist,
// the first nact carry reflectors (the rest lie beyond the rank bound and get
// identity reflectors).  On return S.P holds Y, S.Rk the new R block
// (non-negative diagonal), S.Tm the compact-WY T (row-major) and S.tau the
// tau's.  All PT2 threads call it; it begins and ends with a __syncthreads.
static __device__ __noinline__ void panel_factor(PanelSmem& S, const int nbk, const int nact) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
#ifdef IFK_TRACE
  long long ph_last = ptime();
#endif
  for (int idx = tid; idx < NB * LDP; idx += PT2) {
    S.G[idx] = 0.f;
    S.Tm[idx] = 0.f;
  }
  if (tid < NB) S.tau[tid] = 0.f;
  __syncthreads();
  const int r = tid;
  const int vidx = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
  int buf = 0;
#pragma unroll 1
  for (int s = 0; s < NLEAF; ++s) {
    const int L0 = s * LEAF;
    if (L0 >= nbk) break;
    float a[LEAF];
#pragma unroll
    for (int c = 0; c < LEAF; ++c) a[c] = S.P[(L0 + c) * SP + r];
#pragma unroll
    for (int jj = 0; jj < LEAF; ++jj) {
      const int j = L0 + jj;
      if (j < nact) {
        float v[LEAF];
#pragma unroll
        for (int c = 0; c < LEAF; ++c) v[c] = a[jj] * a[c];
        const float part = warp_reduce16(v, lane);
        if ((lane & 1) == 0) S.part[buf][warp][vidx] = part;
        __syncthreads();
        float tl = 0.f;
        if (lane < LEAF) {
#pragma unroll
          for (int w = 0; w < NWARP; ++w) tl += S.part[buf][w][lane];
        }
        float tot[LEAF];
#pragma unroll
        for (int c = 0; c < LEAF; ++c) tot[c] = __shfl_sync(0xffffffffu, tl, c);
        buf ^= 1;
        float tj, beta, inv_v0;
        reflector(S.Rk[j * LDP + j], tot[jj], tj, beta, inv_v0);
        float wv[LEAF];
#pragma unroll
        for (int c = jj + 1; c < LEAF; ++c) {
          const float rr = S.Rk[j * LDP + L0 + c];
          wv[c] = rr + tot[c] * inv_v0;
          if (tid == 0) S.Rl[jj * (LEAF + 1) + c] = rr - tj * wv[c];
        }
        if (tid == 0) {
          S.Rl[jj * (LEAF + 1) + jj] = beta;
          S.tau[j] = tj;
#pragma unroll
          for (int c = 0; c < jj; ++c) S.G[(L0 + c) * LDP + j] = tot[c] * inv_v0;
        }
        const float y = a[jj] * inv_v0;
        a[jj] = y;
        const float ty = tj * y;
#pragma unroll
        for (int c = jj + 1; c < LEAF; ++c) a[c] -= ty * wv[c];
      } else {
        // beyond the rank bound: identity reflector, zero Householder vector
        a[jj] = 0.f;
        if (tid == 0) {
#pragma unroll
          for (int c = jj; c < LEAF; ++c) S.Rl[jj * (LEAF + 1) + c] = S.Rk[j * LDP + L0 + c];
        }
      }
    }
#pragma unroll
    for (int c = 0; c < LEAF; ++c) S.P[(L0 + c) * SP + r] = a[c];
    __syncthreads();
    PH_MARK(0);
    // leaf R block back into Rk; leaf T by the column recursion, one row per lane of warp 1
    if (tid < LEAF) {
#pragma unroll
      for (int c = 0; c < LEAF; ++c)
        if (c >= tid && L0 + c < nbk) S.Rk[(L0 + tid) * LDP + L0 + c] = S.Rl[tid * (LEAF + 1) + c];
    } else if (tid >= 32 && tid < 32 + LEAF) {
      const int i = tid - 32;
      float Tr[LEAF];
#pragma unroll
      for (int jj = 0; jj < LEAF; ++jj) {
        const float tj = S.tau[L0 + jj];
        float acc = 0.f;
#pragma unroll
        for (int l = 0; l < jj; ++l) acc += Tr[l] * S.G[(L0 + l) * LDP + L0 + jj];
        Tr[jj] = (i == jj) ? tj : (i < jj ? -tj * acc : 0.f);
      }
#pragma unroll
      for (int jj = 0; jj < LEAF; ++jj) S.Tm[(L0 + i) * LDP + L0 + jj] = Tr[jj];
    }
    __syncthreads();
    PH_MARK(1);
    // apply the leaf's block reflector to the remaining panel columns
    const int C0 = L0 + LEAF;
    const int wcI = nbk - C0;
    if (wcI > 0 && L0 < nact) {
      // Z = Rk[leaf rows, C] + Y_leaf^T P[:, C] -> Tmp[0..15][C]; 1 x 4 register tiles,
      // 16-byte loads of 4 consecutive rows of a column
      const int nq = (wcI + 3) / 4;
      for (int o = tid; o < LEAF * nq; o += PT2) {
        const int jj = o / nq, cq = o % nq;
        const int j0 = L0 + jj, cc0 = C0 + 4 * cq;
        float z[4] = {};
        const float* yp = S.P + j0 * SP;
        const float* pc[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pc[e] = S.P + (cc0 + e < nbk ? cc0 + e : cc0) * SP;
#pragma unroll 4
        for (int i = 0; i < SUB; i += 4) {
          const float4 ya = *reinterpret_cast<const float4*>(yp + i);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 x = *reinterpret_cast<const float4*>(pc[e] + i);
            z[e] += ya.x * x.x + ya.y * x.y + ya.z * x.z + ya.w * x.w;
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = cc0 + e;
          if (c < nbk) S.Tmp[jj * LDP + c] = z[e] + S.Rk[j0 * LDP + c];
        }
      }
      __syncthreads();
      PH_MARK(2);
      // W = T_leaf^T Z -> Wb (columns relative to C0) ; Rk[leaf rows, C] -= W
      for (int o = tid; o < LEAF * wcI; o += PT2) {
        const int jj = o % LEAF, cr = o / LEAF, c = C0 + cr;
        float w = 0.f;
#pragma unroll
        for (int l = 0; l < LEAF; ++l) w += S.Tm[(L0 + l) * LDP + L0 + jj] * S.Tmp[l * LDP + c];
        S.Wb[jj * LDW2 + cr] = w;
        S.Rk[(L0 + jj) * LDP + c] -= w;
      }
      for (int o = tid; o < LEAF * 4; o += PT2) {  // zero the padding columns of the last quad
        const int jj = o / 4, cr = wcI + o % 4;
        if (cr < nq * 4) S.Wb[jj * LDW2 + cr] = 0.f;
      }
      __syncthreads();
      PH_MARK(3);
      // P[:, C] -= Y_leaf W; this thread's Y_leaf row is still in a[]
#pragma unroll 1
      for (int cq = 0; cq < nq; ++cq) {
        float d[4] = {};
#pragma unroll
        for (int l = 0; l < LEAF; ++l) {
          const float4 w = *reinterpret_cast<const float4*>(S.Wb + l * LDW2 + 4 * cq);
          d[0] += a[l] * w.x; d[1] += a[l] * w.y; d[2] += a[l] * w.z; d[3] += a[l] * w.w;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = C0 + 4 * cq + e;
          if (c < nbk) S.P[c * SP + r] -= d[e];
        }
      }
      __syncthreads();
      PH_MARK(4);
    }
  }

  // off-diagonal leaf blocks of G = Y^T Y: 6 blocks of 16 x 16 as 96 tiles of 4 x 4;
  // threads 0..95 sum rows 0..127, threads 128..223 rows 128..255
  {
    const int half = tid >> 7, tt = tid & 127;
    const bool act = tt < 96;
    const int blk = tt >> 4, tile = tt & 15;
    const int la = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
    const int lb = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
    const int a0c = la * LEAF + 4 * (tile >> 2), b0c = lb * LEAF + 4 * (tile & 3);
    float g[4][4] = {};
    if (act) {
#pragma unroll 2
      for (int i = half * (SUB / 2); i < (half + 1) * (SUB / 2); i += 4) {
        float4 ya[4], yb[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          ya[e] = *reinterpret_cast<const float4*>(S.P + (a0c + e) * SP + i);
          yb[e] = *reinterpret_cast<const float4*>(S.P + (b0c + e) * SP + i);
        }
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            g[p][q] += ya[p].x * yb[q].x + ya[p].y * yb[q].y + ya[p].z * yb[q].z + ya[p].w * yb[q].w;
      }
      if (half == 1) {
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int q = 0; q < 4; ++q) S.Tmp[tt * 16 + p * 4 + q] = g[p][q];
      }
    }
    __syncthreads();
    if (act && half == 0) {
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) S.G[(a0c + p) * LDP + b0c + q] = g[p][q] + S.Tmp[tt * 16 + p * 4 + q];
    }
  }
  __syncthreads();
  PH_MARK(5);
  // T assembly: T_{01} = -T_0 G_{01} T_1, T_{23} likewise, then the 32 x 32 coupling
  matmul(S.Tmp, 0, 0, S.Tm, 0, 0, S.G, 0, 16, 16, 16, 16, tid, false);     // T0 G01
  matmul(S.Tmp, 16, 32, S.Tm, 32, 32, S.G, 32, 48, 16, 16, 16, tid, false); // T2 G23
  __syncthreads();
  matmul(S.Tm, 0, 16, S.Tmp, 0, 0, S.Tm, 16, 16, 16, 16, 16, tid, true);    // T01
  matmul(S.Tm, 32, 48, S.Tmp, 16, 32, S.Tm, 48, 48, 16, 16, 16, tid, true); // T23
  __syncthreads();
  matmul(S.Tmp, 0, 0, S.Tm, 0, 0, S.G, 0, 32, 32, 32, 32, tid, false);   // T_A G_AB (32 x 32)
  __syncthreads();
  matmul(S.Tm, 0, 32, S.Tmp, 0, 0, S.Tm, 32, 32, 32, 32, 32, tid, true);  // T_AB
  __syncthreads();
  PH_MARK(6);
}

}  // namespace panel
}  // namespace ifk
