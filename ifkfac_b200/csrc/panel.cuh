// Householder panel factorisation of the streaming TSQR fold (device code shared
// by the wave scheduler in tsqr.cu and the persistent fold in fold_engine.cu).
#pragma once

#include "ifk_common.cuh"

namespace ifk {
namespace panel {

#ifdef IFK_TRACE
// Diagnostic build only: slot for per-phase panel times (filled when
// IFK_TRACE_PANEL is also defined; the phase marks slow the Gram steps down
// severely, so task-level traces leave them out); slots 9 and 10 count Gram
// runs and leaves.
__device__ unsigned long long g_panel_phase[16];
#endif
#ifdef IFK_TRACE_PANEL
// Time spent in each phase of panel_factor (SM cycles, summed over panels; slot 8
// counts panels).
// SM cycle counter (cheap to read; thread 0 only, so deltas are on one SM)
__device__ __forceinline__ long long ptime() { return clock64(); }
#define PH_DECL long long ph_last = ptime();
#define PH_MARK(i)                                                          \
  do {                                                                      \
    if (threadIdx.x == 0) {                                                 \
      const long long t_ = ptime();                                         \
      atomicAdd(&g_panel_phase[i], (unsigned long long)(t_ - ph_last));     \
      ph_last = t_;                                                         \
    }                                                                       \
  } while (0)
#define PH_FLUSH()                                   \
  if (threadIdx.x == 0) atomicAdd(&g_panel_phase[8], 1ull);
#else
#define PH_DECL
#define PH_MARK(i) do { } while (0)
#define PH_FLUSH()
#endif

constexpr int LDP = NB + 1;   // row stride of the small NB x NB blocks
// The panel has ROWS rows (256 for the wave scheduler, 128 for the persistent
// fold) and runs on threads 0 .. ROWS-1, thread = row.
template <int ROWS>
struct Geo {
  static constexpr int SP = ROWS + 4;  // column stride of the panel (column-major; 16-byte aligned
                                       // columns, column c starts at bank 4c mod 32)
  static constexpr int NW = ROWS / 32;
  static_assert(ROWS == 128 || ROWS == 256, "panels of 128 or 256 rows");
};
constexpr int SP = Geo<SUB>::SP;  // the wave scheduler's panels (SUB rows)
constexpr int PT2 = SUB;
constexpr int LEAF = 16;
constexpr int NLEAF = NB / LEAF;
constexpr int ZST = 20;       // stride per output column of the block-product partials (bank-conflict free)
constexpr int LDW = NB;       // row stride of W

// A column's squared norm may shrink to this fraction of its value at the last
// Gram evaluation before the Gram matrix is evaluated again from the data.
constexpr float GRAM_KEEP = 0.5f;

// ---- method --------------------------------------------------------------------
// ROWS threads; thread t owns row t of the sub-tile.  The NB = 64 panel columns
// are factored in 4 leaves of 16 Householder reflectors (TPQRT: reflector j acts
// on row j of the R block and on the sub-tile rows).
//  * Leaf: the Gram matrix M = X_leaf^T X_leaf of the leaf's current columns is
//    formed once (block product over the rows).  One warp then computes the
//    16 reflectors in sequence from M and the leaf's R rows: reflector j needs
//    |x_j|^2 = M[j][j] and the dot products M[j][c]; applying it updates M by a
//    rank-2 term and row j of R.  No block-wide reduction is needed per column.
//    If a column's squared norm falls below GRAM_KEEP of its value at the last
//    evaluation (cancellation in the update), the warp stops, the reflectors so
//    far are applied to the data and M is evaluated again.  Each thread then
//    applies the reflectors to its row, which yields Y_leaf.
//  * Y_leaf^T P[:, 0:nbk] (one block product) gives the leaf's blocks of Y^T Y
//    and Z = Y_leaf^T P[:, trailing]; W = T_leaf^T (R + Z) by forward
//    substitution with T^-T = diag(1/tau) + strict_lower(Y^T Y); then
//    R[leaf rows, trailing] -= W and P[:, trailing] -= Y_leaf W.
//  * T is assembled from the leaf T's by T_AB = -T_A (Y_A^T Y_B) T_B.
template <int ROWS>
struct PanelSmemT {
  float P[NB * Geo<ROWS>::SP];  // X_t[:, panel] -> Y, column-major: element (i, c) at P[c * SP + i]
  float Rk[NB * LDP];        // diagonal block of R
  float G[NB * LDP];         // strict upper part of Y^T Y
  float Tm[NB * LDP];        // T, row-major
  float Zp[4 * NB * ZST];    // block-product partials [row quarter][column][16]; T assembly scratch
  float Wb[LEAF * LDW];      // Z, then W, of the leaf update (row-major)
  float Wr[LEAF * LEAF];     // tau_j w_jc of the leaf's reflectors (row j)
  float ivv[LEAF];           // 1 / v0_j of the leaf's reflectors
  float tau[NB];
  int jend;
};
using PanelSmem = PanelSmemT<SUB>;
static_assert(4 * NB * ZST >= NB * LDP, "T assembly scratch fits the partials block");

// Barrier of the panel's threads (id 2; the panel may run on part of a CTA)
template <int ROWS>
__device__ __forceinline__ void psync() {
  asm volatile("bar.sync 2, %0;" ::"n"(ROWS) : "memory");
}

// Reflector of xLARFGP form (beta >= 0) for the column (aj; x) with |x|^2 = xn2:
// H = I - tj v v^T, v = (1; x / v0), v0 = aj - beta formed without cancellation.
// With u = aj + beta (aj > 0) or u = v0 (aj <= 0), one reciprocal of u depends on
// beta; 1/xn2 is taken alongside the square root:
//   aj > 0:  v0 = -xn2 / u, 1/v0 = -u / xn2, tj = -v0 / beta = xn2 / (u beta)
//   aj <= 0: 1/v0 = 1/u, tj = -u / beta.
// A residual with |x| below the fp32 resolution of the diagonal (|x| < 2^-24 |aj|:
// beta rounds to |aj|) or |x|^2 below XN2_MIN is dropped, and the reflector reduces
// to the sign flip.  Leaving x in place perturbs column j by at most 2^-24 |aj| (or
// 1e-15), inside Householder's backward error; without the cut, an exactly dependent
// column (duplicate or constant activations: its residual cancels to a denormal)
// makes 1/xn2 and (1/beta)^2 leave the fp32 range and the panel turns NaN.  A NaN
// xn2 fails both tests and still propagates to the finite check.
constexpr float XN2_MIN = 1e-30f;
__device__ __forceinline__ void reflector(float aj, float xn2, float& tj, float& beta, float& inv_v0) {
  const float s = fmaf(aj, aj, xn2);
  const float rs = rsqrtf(s);
  const float rx = __fdividef(1.f, xn2);
  const float nrm = s * rs;
  const bool pos = aj > 0.f;
  const float u = pos ? aj + nrm : aj - nrm;
  const float ru = __fdividef(1.f, u);
  const float ea = aj * 0x1p-24f;
  if (xn2 < XN2_MIN || xn2 < ea * ea) {
    // nothing to annihilate at fp32 resolution; flip the row if its diagonal is negative
    tj = aj >= 0.f ? 0.f : 2.f;
    beta = fabsf(aj);
    inv_v0 = 0.f;
  } else {
    beta = nrm;
    tj = pos ? (xn2 * rs) * ru : -u * rs;
    inv_v0 = pos ? -u * rx : ru;
  }
}

__device__ __forceinline__ float dot4(const float4 a, const float4 b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

// Block product partials: for the 16 panel columns a0.. and the nb (1..64)
// columns b0.., Zp[(q * NB + c) * ZST + i] = sum over the rows of quarter q
// of P[r][a0 + i] * P[r][b0 + c].  Warp w takes row quarter w % 4; with 8 warps,
// warps w and w + 4 split the output columns.  Lane (i4 = lane & 3, g = lane >> 2)
// accumulates rows i4 + 4u of A against columns g + 8e of B, so every 16-byte
// load of a warp touches distinct banks or broadcasts.  E = output-column groups of 8 (even).
template <int ROWS, int E>
__device__ __forceinline__ void block_product(PanelSmemT<ROWS>& S, int a0, int b0, int nb) {
  constexpr int SP = Geo<ROWS>::SP;
  constexpr int EH = E * 4 / Geo<ROWS>::NW;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i4 = lane & 3, g = lane >> 2;
  const int rq = warp & 3, oh = warp >> 2;
  const float* pa[4];
  const float* pb[EH];
#pragma unroll
  for (int u = 0; u < 4; ++u) pa[u] = S.P + (a0 + i4 + 4 * u) * SP + rq * (ROWS / 4);
#pragma unroll
  for (int e = 0; e < EH; ++e) {
    const int c = g + 8 * (oh * EH + e);
    pb[e] = S.P + (b0 + (c < nb ? c : nb - 1)) * SP + rq * (ROWS / 4);
  }
  float acc[4][EH];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int e = 0; e < EH; ++e) acc[u][e] = 0.f;
#pragma unroll 4
  for (int i = 0; i < ROWS / 4; i += 4) {
    float4 ya[4], pv[EH];
#pragma unroll
    for (int u = 0; u < 4; ++u) ya[u] = *reinterpret_cast<const float4*>(pa[u] + i);
#pragma unroll
    for (int e = 0; e < EH; ++e) pv[e] = *reinterpret_cast<const float4*>(pb[e] + i);
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int e = 0; e < EH; ++e) acc[u][e] = dot4(ya[u], pv[e], acc[u][e]);
  }
#pragma unroll
  for (int e = 0; e < EH; ++e) {
    const int c = g + 8 * (oh * EH + e);
    if (c < nb) {
#pragma unroll
      for (int u = 0; u < 4; ++u) S.Zp[(rq * NB + c) * ZST + i4 + 4 * u] = acc[u][e];
    }
  }
}

// Sum of the four row-quarter partials of output (i, c)
template <int ROWS>
__device__ __forceinline__ float zsum(const PanelSmemT<ROWS>& S, int i, int c) {
  const float* z = S.Zp + c * ZST + i;
  return (z[0] + z[NB * ZST]) + (z[2 * NB * ZST] + z[3 * NB * ZST]);
}

// dst block (M x N at dr, dc) = (NEG ? -1 : 1) * A (M x K at ar, ac) * B (K x N at br, bc),
// row-major LDP-stride blocks in shared memory; all PT threads.  Used for T assembly.
template <int PT, int M, int K, int N, bool NEG>
__device__ __forceinline__ void matmul(float* dst, int dr, int dc, const float* A, int ar, int ac, const float* B,
                                       int br, int bc, int tid) {
#pragma unroll
  for (int o = tid; o < M * N; o += PT) {
    const int i = o / N, j = o % N;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int l = 0; l < K; l += 2) {
      s0 = fmaf(A[(ar + i) * LDP + ac + l], B[(br + l) * LDP + bc + j], s0);
      s1 = fmaf(A[(ar + i) * LDP + ac + l + 1], B[(br + l + 1) * LDP + bc + j], s1);
    }
    dst[(dr + i) * LDP + dc + j] = NEG ? -(s0 + s1) : (s0 + s1);
  }
}

// Warp 0: reflectors jl .. of the leaf at L0 from the Gram matrix in Zp (columns
// L0..L0+15 against themselves) and the leaf's R rows in Rk, up to nl or until a
// column's norm has shrunk past GRAM_KEEP.  Writes the R rows, tau, 1/v0 and
// tau_j w_jc, and the end of the run to S.jend.
// Lanes c and c + 16 own column c of the leaf and split its row of M by the
// parity of the column index (lane c + 16h keeps M[c][d] for d = h mod 2), so a
// step costs each lane half the shuffles and updates of a whole row.  The
// diagonal M[c][c] follows its own recurrence in both lanes, and the next pivot
// |x_j|^2 is read from it, off the shuffles of the row update.
template <int ROWS>
__device__ __forceinline__ void gram_steps(PanelSmemT<ROWS>& S, int L0, int jl, int nl, int nbk) {
  const unsigned F = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int c = lane & 15, h = lane >> 4;
  constexpr int HALF = LEAF / 2;
  float Mh[HALF], Rc[LEAF];
#pragma unroll
  for (int k = 0; k < HALF; ++k) Mh[k] = zsum(S, c, 2 * k + h);
#pragma unroll
  for (int j = 0; j < LEAF; ++j) Rc[j] = S.Rk[(L0 + j) * LDP + L0 + c];
  float dc = zsum(S, c, c);  // M[c][c], kept by its own recurrence
  const float m0 = GRAM_KEEP * dc;
  // Steps run to nl; a step whose update shrank a norm past GRAM_KEEP ends the
  // run after it (steps computed beyond that point are discarded).
  unsigned badmask = 0u;
  // software pipelined: each step ends its critical chain (reflector, w, own
  // diagonal) by fetching the next pivot, then does its row update
  float xn2_next = __shfl_sync(F, dc, jl & 15);
#pragma unroll
  for (int j = 0; j < LEAF; ++j) {
    if (j >= jl && j < nl) {
      const float xn2 = xn2_next;
      const float al = __shfl_sync(F, Rc[j], j);
      // M[c][j]: in this lane when j has its parity, else in the partner lane
      const float other = __shfl_xor_sync(F, Mh[j >> 1], 16);
      const float mcj = (h == (j & 1)) ? Mh[j >> 1] : other;
      float tj, beta, iv;
      reflector(al, xn2, tj, beta, iv);
      const float w = fmaf(mcj, iv, Rc[j]);
      const float p = tj * iv;
      const float qw = p * p * xn2 * w;
      // own diagonal M[c][c] (c > j): -2 p w M[c][j] + p^2 xn2 w^2; next pivot
      dc = fmaf(qw, w, fmaf(-2.f * p * w, mcj, dc));
      if (j + 1 < LEAF) xn2_next = __shfl_sync(F, dc, j + 1);
      // row j of M, this lane's parity: lane j + 16h holds it
      float Mj[HALF];
#pragma unroll
      for (int k = 0; k < HALF; ++k)
        if (2 * k + 1 > j) Mj[k] = __shfl_sync(F, Mh[k], j + 16 * h);
      // rows of finished columns (c <= j) are dead: update every lane's row
#pragma unroll
      for (int k = 0; k < HALF; ++k) {
        if (2 * k + 1 > j) {
          const float wd = __shfl_sync(F, w, 2 * k + h);  // w of column d = 2k + h
          const float upd = fmaf(qw, wd, fmaf(-p, fmaf(w, Mj[k], wd * mcj), Mh[k]));
          Mh[k] = (2 * k + h > j) ? upd : Mh[k];
        }
      }
      Rc[j] = (c == j) ? beta : fmaf(-tj, w, Rc[j]);
      if (c > j && h == 0) S.Wr[j * LEAF + c] = tj * w;
      if (lane == j) {
        S.ivv[j] = iv;
        S.tau[L0 + j] = tj;
      }
      const bool bad = c > j && c < nl && !(dc >= m0);
      badmask |= __ballot_sync(F, bad) ? (1u << j) : 0u;
    }
  }
  const int jend = badmask ? __ffs(badmask) : nl;  // last good step + 1
  // rows jl .. jend-1 of the leaf's R block (upper part, columns inside the block)
  if (lane < LEAF && L0 + c < nbk) {
#pragma unroll
    for (int j = 0; j < LEAF; ++j)
      if (j >= jl && j < jend && j <= c) S.Rk[(L0 + j) * LDP + L0 + c] = Rc[j];
  }
  if (lane == 0) S.jend = jend;
}

// Leaf hooks of panel_factor.  Rows L0 .. L0 + 15 of the R diagonal block are
// read and written by leaf L0 / 16 only, so a caller may load them just before
// that leaf (before_leaf, which ends with a barrier of the panel's threads and
// returns false to abandon the panel) and store them as soon as they are final:
// rows_final, called after the barrier that follows the leaf's W (only the update
// of the panel's trailing columns comes after it; not called for a leaf without
// reflectors or trailing columns), else after_leaf, called after the leaf's last
// barrier.  NoLeafHook: the caller loads and stores the whole block around the call.
struct NoLeafHook {
  template <class SM>
  __device__ __forceinline__ bool before_leaf(SM&, int) { return true; }
  template <class SM>
  __device__ __forceinline__ void rows_final(SM&, int) {}
  template <class SM>
  __device__ __forceinline__ void after_leaf(SM&, int) {}
};

// Factor the panel in S.P (ROWS x NB fp32, column-major; rows beyond the
// sub-tile are zero) under the R diagonal block S.Rk.  nbk panel columns exist,
// the first nact carry reflectors (the rest lie beyond the rank bound and get
// identity reflectors).  On return S.P holds Y, S.Rk the new R block
// (non-negative diagonal), S.Tm the compact-WY T (row-major) and S.tau the
// tau's.  Threads 0 .. ROWS-1 call it; it begins and ends with a barrier of them.
// Returns false when a hook abandoned the panel (every thread returns together).
template <int ROWS, class Hook = NoLeafHook>
static __device__ __noinline__ bool panel_factor(PanelSmemT<ROWS>& S, const int nbk, const int nact,
                                                 Hook hook = Hook()) {
  constexpr int SP = Geo<ROWS>::SP;
  constexpr int PT = ROWS;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  PH_DECL
  for (int idx = tid; idx < NB * LDP; idx += PT) {
    S.G[idx] = 0.f;
    S.Tm[idx] = 0.f;
  }
  if (tid < NB) S.tau[tid] = 0.f;
  const int r = tid;
  for (int c = nbk; c < NB; ++c) S.P[c * SP + r] = 0.f;  // columns past the block: zero
  psync<ROWS>();
#pragma unroll 1
  for (int s = 0; s < NLEAF; ++s) {
    const int L0 = s * LEAF;
    if (L0 >= nbk) break;
    if (!hook.before_leaf(S, s)) return false;
    // the leaf; every exit from it ('continue') follows a barrier of the panel's threads
    do {
    const int nl = nact - L0 < LEAF ? nact - L0 : LEAF;  // reflectors of this leaf (may be <= 0)
    float a[LEAF];
#pragma unroll
    for (int c = 0; c < LEAF; ++c) a[c] = S.P[(L0 + c) * SP + r];
    // ---- leaf: Gram runs ----
    int jl = 0;
#pragma unroll 1
#ifdef IFK_TRACE
    if (tid == 0 && nl > 0) atomicAdd(&g_panel_phase[10], 1ull);
#endif
    while (jl < nl) {
#ifdef IFK_TRACE
      if (tid == 0) atomicAdd(&g_panel_phase[9], 1ull);
#endif
      block_product<ROWS, 2>(S, L0, L0, LEAF);
      psync<ROWS>();
      PH_MARK(0);
      if (warp == 0) gram_steps<ROWS>(S, L0, jl, nl, nbk);
      psync<ROWS>();
      PH_MARK(1);
      const int jend = S.jend;
      // apply reflectors jl .. jend-1 to this thread's row
#pragma unroll
      for (int j = 0; j < LEAF; ++j) {
        if (j >= jl && j < jend) {
          const float y = a[j] * S.ivv[j];
          a[j] = y;
          const float4* wr = reinterpret_cast<const float4*>(S.Wr + j * LEAF);
#pragma unroll
          for (int c4 = 0; c4 < LEAF / 4; ++c4) {
            if (4 * c4 + 3 <= j) continue;
            const float4 t = wr[c4];
            if (4 * c4 + 0 > j) a[4 * c4 + 0] = fmaf(-y, t.x, a[4 * c4 + 0]);
            if (4 * c4 + 1 > j) a[4 * c4 + 1] = fmaf(-y, t.y, a[4 * c4 + 1]);
            if (4 * c4 + 2 > j) a[4 * c4 + 2] = fmaf(-y, t.z, a[4 * c4 + 2]);
            if (4 * c4 + 3 > j) a[4 * c4 + 3] = fmaf(-y, t.w, a[4 * c4 + 3]);
          }
        }
      }
      jl = jend;
      if (jl < nl) {
#pragma unroll
        for (int c = 0; c < LEAF; ++c) S.P[(L0 + c) * SP + r] = a[c];
      }
      psync<ROWS>();  // Wr / ivv / jend are rewritten by the next run
      PH_MARK(2);
    }
    // columns beyond the rank bound carry no reflector
#pragma unroll
    for (int c = 0; c < LEAF; ++c) {
      if (L0 + c >= nact) a[c] = 0.f;
      S.P[(L0 + c) * SP + r] = a[c];
    }
    psync<ROWS>();
    if (L0 >= nact) continue;  // no reflectors: R rows, T and trailing columns unchanged
    // ---- Y_leaf^T P[:, 0:nbk]: leaf blocks of Y^T Y and Z ----
    block_product<ROWS, 8>(S, L0, 0, nbk);
    psync<ROWS>();
    PH_MARK(3);
    const int C0 = L0 + LEAF;
    const int wcI = nbk - C0;
    for (int o = tid; o < LEAF * nbk; o += PT) {
      const int i = o & 15, c = o >> 4;
      const float v = zsum(S, i, c);
      if (c < L0) S.G[c * LDP + L0 + i] = v;                    // (Y_c-leaf)^T Y_leaf
      else if (c < C0) { if (c > L0 + i) S.G[(L0 + i) * LDP + c] = v; }  // strict upper of the leaf block
      else S.Wb[i * LDW + (c - C0)] = v + S.Rk[(L0 + i) * LDP + c];     // Z + R rows
    }
    psync<ROWS>();
    PH_MARK(4);
    // W = T_leaf^T Z by forward substitution; leaf T by the column recursion (warp 7)
    if (tid < wcI) {
      const int c = tid;
      float wv[LEAF];
#pragma unroll
      for (int j = 0; j < LEAF; ++j) {
        float acc0 = S.Wb[j * LDW + c], acc1 = 0.f;
#pragma unroll
        for (int l = 0; l < j; l += 2) {
          acc0 = fmaf(-S.G[(L0 + l) * LDP + L0 + j], wv[l], acc0);
          if (l + 1 < j) acc1 = fmaf(-S.G[(L0 + l + 1) * LDP + L0 + j], wv[l + 1], acc1);
        }
        wv[j] = S.tau[L0 + j] * (acc0 + acc1);
      }
#pragma unroll
      for (int j = 0; j < LEAF; ++j) {
        S.Wb[j * LDW + c] = wv[j];
        S.Rk[(L0 + j) * LDP + C0 + c] -= wv[j];
      }
    } else if (tid < ((wcI + 3) & ~3)) {
#pragma unroll
      for (int j = 0; j < LEAF; ++j) S.Wb[j * LDW + tid] = 0.f;
    }
    if (warp == Geo<ROWS>::NW - 1 && (tid & 31) < LEAF) {
      const int i = tid & 31;
      float Tr[LEAF];
#pragma unroll
      for (int jj = 0; jj < LEAF; ++jj) {
        const float tj = S.tau[L0 + jj];
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int l = 0; l < jj; l += 2) {
          acc0 = fmaf(Tr[l], S.G[(L0 + l) * LDP + L0 + jj], acc0);
          if (l + 1 < jj) acc1 = fmaf(Tr[l + 1], S.G[(L0 + l + 1) * LDP + L0 + jj], acc1);
        }
        Tr[jj] = (i == jj) ? tj : (i < jj ? -tj * (acc0 + acc1) : 0.f);
      }
#pragma unroll
      for (int jj = 0; jj < LEAF; ++jj) S.Tm[(L0 + i) * LDP + L0 + jj] = Tr[jj];
    }
    if (wcI <= 0) {
      psync<ROWS>();
      continue;
    }
    psync<ROWS>();
    PH_MARK(5);
    // the leaf's R rows are final here (the trailing update below touches P only)
    hook.rows_final(S, s);
    // P[:, C] -= Y_leaf W; this thread's Y_leaf row is still in a[]
    const int nq = (wcI + 3) / 4;
#pragma unroll 1
    for (int cq = 0; cq < nq; ++cq) {
      float d[4] = {};
#pragma unroll
      for (int l = 0; l < LEAF; ++l) {
        const float4 w = *reinterpret_cast<const float4*>(S.Wb + l * LDW + 4 * cq);
        d[0] = fmaf(a[l], w.x, d[0]);
        d[1] = fmaf(a[l], w.y, d[1]);
        d[2] = fmaf(a[l], w.z, d[2]);
        d[3] = fmaf(a[l], w.w, d[3]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = C0 + 4 * cq + e;
        if (c < nbk) S.P[c * SP + r] -= d[e];
      }
    }
    psync<ROWS>();
    PH_MARK(6);
    } while (0);
    hook.after_leaf(S, s);
  }
  // T assembly: T_{01} = -T_0 G_{01} T_1, T_{23} likewise, then the 32 x 32 coupling
  float* Tmp = S.Zp;
  matmul<PT, 16, 16, 16, false>(Tmp, 0, 0, S.Tm, 0, 0, S.G, 0, 16, tid);     // T0 G01
  matmul<PT, 16, 16, 16, false>(Tmp, 16, 32, S.Tm, 32, 32, S.G, 32, 48, tid); // T2 G23
  psync<ROWS>();
  matmul<PT, 16, 16, 16, true>(S.Tm, 0, 16, Tmp, 0, 0, S.Tm, 16, 16, tid);    // T01
  matmul<PT, 16, 16, 16, true>(S.Tm, 32, 48, Tmp, 16, 32, S.Tm, 48, 48, tid); // T23
  psync<ROWS>();
  matmul<PT, 32, 32, 32, false>(Tmp, 0, 0, S.Tm, 0, 0, S.G, 0, 32, tid);      // T_A G_AB (32 x 32)
  psync<ROWS>();
  matmul<PT, 32, 32, 32, true>(S.Tm, 0, 32, Tmp, 0, 0, S.Tm, 32, 32, tid);    // T_AB
  psync<ROWS>();
  PH_MARK(7);
  PH_FLUSH()
  return true;
}

}  // namespace panel
}  // namespace ifk
