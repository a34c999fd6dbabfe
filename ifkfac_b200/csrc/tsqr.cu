// Streaming TSQR fold: R <- qr([R; X]).R with a non-negative diagonal.
//
// Algorithm (restated from LAPACK's triangular-pentagonal QR, xTPQRT, and
// matching the result of the reference's leaf + merge QR,
// ifkfac/triangular.py:246-307): the chunk is cut into sub-tiles of SUB rows
// that are folded one after another.  Folding a sub-tile is a blocked
// Householder QR of the stack [R; X_t] in which panel k (NB columns) only
// touches rows k*NB.. of R and the rows of X_t: reflector j maps
// [R[j,j]; X_t[:, j]] to [beta; 0] with beta >= 0 (the reflector form of
// LAPACK's xLARFGP, computed without cancellation), so no sign pass is
// needed afterwards.  The panel's reflectors are aggregated in compact-WY
// form V = [I; Y], Q = I - V T V^T, and applied to the trailing columns as
//   W = T^T (R[k rows, c] + Y^T X_t[:, c]);  R[k rows, c] -= W;  X_t[:, c] -= Y W.
// T comes from T^-1 = strict_upper(Y^T Y) + diag(1/tau) (Puglisi's identity).
//
// Scheduling: task (t, k) = panel k of sub-tile t.  It depends on (t-1, k)
// (R rows of block k) and on (t, k-1) (X_t columns of block k), so all tasks
// with t + k = d form wave d and waves run in order: one panel launch and one
// trailing-update launch per wave.
#include "ifk_common.cuh"
#include "ifk_internal.h"
#include "panel.cuh"

namespace ifk {

namespace {

constexpr int PT = 256;  // threads of the panel and SIMT update kernels
static_assert(SUB == PT, "panel kernel maps one thread to one row");
constexpr int LDP = NB + 1;

// Task (t, k) of the wave schedule.  Every sub-tile factors every panel (no
// rank bound): while R is trapezoidal, a sub-tile past the rows folded so far
// holds only rounding residuals in exact arithmetic, but an exactly or
// numerically dependent column (duplicated or constant activations) spends a
// reflector on rounding noise and leaves a true row direction there, which a
// bound at rows_R + rows would drop.  This is the fp32 path, so it keeps them.
// (The persistent bf16 fold keeps the bound; its own rounding is coarser than
// that loss.)  Only the zero block of a trapezoidal chunk is skipped.
__device__ __forceinline__ bool task_active(const FoldArgs& a, int t, int k) {
  if (t < 0 || t >= a.tiles || k < 0 || k >= a.K) return false;
  return !(a.tri && (int64_t)k * NB + NB <= (int64_t)t * SUB);  // sub-tile is zero left of its diagonal
}

// ---- panel factorisation: see panel.cuh -----------------------------------------
using panel::PT2;
using panel::PanelSmem;
constexpr size_t panel_smem_bytes() { return sizeof(PanelSmem); }

// One panel factorisation per block: block t handles task (t, wave - t).
__global__ void __launch_bounds__(PT2) fold_panel_kernel(FoldBatch fb, int wave) {
  const FoldArgs& a = fb.f[blockIdx.z];
  const int t = blockIdx.x;
  const int k = wave - t;
  if (!task_active(a, t, k)) return;

  extern __shared__ __align__(1024) float smraw[];
  PanelSmem& S = *reinterpret_cast<PanelSmem*>(smraw);
  const int tid = threadIdx.x;

  const int64_t row0 = (int64_t)t * SUB;
  const int h = (int)mn<int64_t>(SUB, a.rows - row0);
  const int64_t c0 = (int64_t)k * NB;
  const int nbk = (int)mn<int64_t>(NB, a.n - c0);
  const int nact = nbk;

  // X_t panel -> P: 16-byte loads, 8 in flight per thread
  for (int q0 = tid; q0 < SUB * NB / 4; q0 += 8 * PT2) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = q0 + u * PT2, i = q / (NB / 4), j4 = (q % (NB / 4)) * 4;
      v[u] = (i < h) ? ld4(a.X + (row0 + i) * a.ldX + c0 + j4, nbk - j4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = q0 + u * PT2, i = q / (NB / 4), j4 = (q % (NB / 4)) * 4;
      S.P[(j4 + 0) * panel::SP + i] = v[u].x;
      S.P[(j4 + 1) * panel::SP + i] = v[u].y;
      S.P[(j4 + 2) * panel::SP + i] = v[u].z;
      S.P[(j4 + 3) * panel::SP + i] = v[u].w;
    }
  }
  for (int q0 = tid; q0 < NB * NB; q0 += 8 * PT2) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = q0 + u * PT2, i = idx / NB, j = idx % NB;
      v[u] = (i < nbk && j < nbk && j >= i) ? a.R[(c0 + i) * a.ldR + c0 + j] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = q0 + u * PT2, i = idx / NB, j = idx % NB;
      S.Rk[i * LDP + j] = v[u];
    }
  }

  panel::panel_factor<SUB>(S, nbk, nact);

  // T stored column-major (Tb[j*NB + i] = T[i][j]) for the trailing update
  float* Tb = a.Tb + (size_t)t * NB * NB;
  for (int idx = tid; idx < NB * NB; idx += PT2) Tb[idx] = S.Tm[(idx % NB) * LDP + idx / NB];
  for (int q = tid; q < SUB * NB / 4; q += PT2) {
    const int i = q / (NB / 4), j4 = (q % (NB / 4)) * 4;
    if (i < h) {
      const float* sp = S.P + i;
      st4(a.X + (row0 + i) * a.ldX + c0 + j4,
          make_float4(sp[(j4 + 0) * panel::SP], sp[(j4 + 1) * panel::SP], sp[(j4 + 2) * panel::SP],
                      sp[(j4 + 3) * panel::SP]),
          nbk - j4);
    }
  }
  for (int idx = tid; idx < NB * NB; idx += PT2) {
    const int i = idx / NB, j = idx % NB;
    if (i < nbk && j < nbk && j >= i) a.R[(c0 + i) * a.ldR + c0 + j] = S.Rk[i * LDP + j];
  }
}

// Shared-memory row strides of the fp32 trailing update: 16-byte aligned rows, so
// that the tiles arrive by 16-byte cp.async copies and are read as float4.
// Every read pattern of the update touches at most four distinct rows of a Y
// chunk or of Ts per warp (broadcasts) or one contiguous row of an X chunk or
// of W, so the padding only has to keep the rows aligned.
constexpr int LDS = NB + 4;   // rows of Y chunks and Ts
constexpr int LDWS = WC + 4;  // rows of X chunks and W
static_assert(NB == 64 && WC == 64 && SUB == 256 && PT == 256, "the update's thread tiles");
constexpr int CR = 64;            // rows of a chunk of the sub-tile
constexpr int NCH = SUB / CR;     // chunks
constexpr int STAGE = CR * LDS + CR * LDWS;  // floats of one stage: a Y chunk and an X chunk
constexpr size_t upd_smem_bytes() {
  return sizeof(float) * ((size_t)2 * STAGE + (size_t)NB * LDWS + (size_t)NB * LDS);
}

// 16 bytes global -> shared, the bytes past `valid` floats zero-filled (valid 0..4)
__device__ __forceinline__ void cp16(float* dst, const float* src, int valid, const float* dummy) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(valid > 0 ? src : dummy),
               "r"(valid * 4)
               : "memory");
}

// Rows m*CR .. of Y (panel columns c0 ..) and of the sub-tile's columns cs .. into
// a stage, as one cp.async group (rows past h and columns past the blocks zero).
__device__ __forceinline__ void load_chunk(float* st, const FoldArgs& a, int64_t row0, int h, int64_t c0,
                                           int nbk, int64_t cs, int wc, int m) {
  float* Yc = st;
  float* Xc = st + CR * LDS;
  for (int q = threadIdx.x; q < CR * (NB / 4); q += PT) {
    const int i = q >> 4, j4 = (q & 15) * 4, gi = m * CR + i;
    const int vy = gi < h ? mx<int>(0, mn<int>(4, nbk - j4)) : 0;
    const int vx = gi < h ? mx<int>(0, mn<int>(4, wc - j4)) : 0;
    const float* rowp = a.X + (row0 + gi) * a.ldX;
    cp16(Yc + i * LDS + j4, rowp + c0 + j4, vy, a.X);
    cp16(Xc + i * LDWS + j4, rowp + cs + j4, vx, a.X);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// fp32 trailing update of one (sub-tile, panel, column block) per block:
//   W = Y^T X_t[:, cols] + R[k rows, cols];  W2 = T^T W;  R[k rows, cols] -= W2;
//   X_t[:, cols] -= Y W2.
// The sub-tile's rows stream through two stages of CR-row chunks by cp.async
// (the next chunk's copy runs under the current chunk's products), once for the
// first product and once for the last, so a block holds ~104 KB of shared memory
// and two blocks share an SM.  All shared reads are float4.
__global__ void __launch_bounds__(PT, 2) fold_update_simt_kernel(FoldBatch fb, int wave) {
  const FoldArgs& a = fb.f[blockIdx.z];
  const int t = blockIdx.x;
  const int k = wave - t;
  if (!task_active(a, t, k)) return;
  const int64_t c0 = (int64_t)k * NB;
  const int64_t cs = (int64_t)blockIdx.y * WC;
  if (cs < c0 + NB || cs >= a.n) return;

  extern __shared__ __align__(16) float sm[];
  // chunk stages sm and sm + STAGE: a Y chunk (CR x LDS), then an X chunk (CR x LDWS)
  auto stage = [&](int idx) { return idx ? sm + STAGE : sm; };
  float* W = sm + 2 * STAGE;          // NB x LDWS
  float* Ts = W + NB * LDWS;          // NB x LDS: Ts[i][l] = T[l][i]

  const int tid = threadIdx.x;
  const int64_t row0 = (int64_t)t * SUB;
  const int h = (int)mn<int64_t>(SUB, a.rows - row0);
  const int nbk = (int)mn<int64_t>(NB, a.n - c0);
  const int wc = (int)mn<int64_t>(WC, a.n - cs);
  const float* Tb = a.Tb + (size_t)t * NB * NB;  // column-major: Tb[i*NB + l] = T[l][i]
  const int nch = (h + CR - 1) / CR;              // chunks holding rows of the sub-tile

  // T with chunk 0's group, chunk 1 in the other stage
  for (int q = tid; q < NB * NB / 4; q += PT) {
    const int i = q >> 4, l4 = (q & 15) * 4;
    cp16(Ts + i * LDS + l4, Tb + i * NB + l4, 4, Tb);
  }
  load_chunk(stage(0), a, row0, h, c0, nbk, cs, wc, 0);
  load_chunk(stage(1), a, row0, h, c0, nbk, cs, wc, 1);

  const int ty = tid >> 4, tx = tid & 15;
  // ---- W = Y^T X (+ R rows): thread (ty, tx) owns W[ty*4 .. +3][tx*4 .. +3] ----
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[r][q] = 0.f;
#pragma unroll 1
  for (int m = 0; m < NCH; ++m) {
    // groups in flight: chunks m and m + 1 (the last chunk: m only)
    if (m + 1 < NCH) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const float* Yc = stage(m & 1);
    const float* Xc = Yc + CR * LDS;
    const int kend = mn<int>(CR, h - m * CR);
#pragma unroll 4
    for (int kk = 0; kk < kend; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(Yc + kk * LDS + ty * 4);
      const float4 bv = *reinterpret_cast<const float4*>(Xc + kk * LDWS + tx * 4);
      const float ar[4] = {av.x, av.y, av.z, av.w}, bq[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[r][q] = fmaf(ar[r], bq[q], acc[r][q]);
    }
    __syncthreads();  // every thread is done with this stage
    // refill it: chunk m + 2 for this product; for the last product, the chunks
    // not resident at its start (it takes the two resident ones first)
    if (m + 2 < NCH) load_chunk(stage(m & 1), a, row0, h, c0, nbk, cs, wc, m + 2);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = ty * 4 + r;
    float o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = tx * 4 + q;
      const float rv = (i < nbk && c < wc) ? a.R[(c0 + i) * a.ldR + cs + c] : 0.f;
      o[q] = acc[r][q] + rv;
    }
    *reinterpret_cast<float4*>(W + i * LDWS + tx * 4) = make_float4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  // ---- W2 = T^T W; R rows -= W2 ----
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[r][q] = 0.f;
#pragma unroll 2
  for (int l = 0; l < NB; l += 4) {
    float4 bw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) bw[u] = *reinterpret_cast<const float4*>(W + (l + u) * LDWS + tx * 4);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float4 tv = *reinterpret_cast<const float4*>(Ts + (ty * 4 + r) * LDS + l);
      const float tl[4] = {tv.x, tv.y, tv.z, tv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc[r][0] = fmaf(tl[u], bw[u].x, acc[r][0]);
        acc[r][1] = fmaf(tl[u], bw[u].y, acc[r][1]);
        acc[r][2] = fmaf(tl[u], bw[u].z, acc[r][2]);
        acc[r][3] = fmaf(tl[u], bw[u].w, acc[r][3]);
      }
    }
  }
  __syncthreads();  // every thread has read W
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = ty * 4 + r;
    *reinterpret_cast<float4*>(W + i * LDWS + tx * 4) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = tx * 4 + q;
      if (i < nbk && c < wc) a.R[(c0 + i) * a.ldR + cs + c] -= acc[r][q];
    }
  }
  __syncthreads();
  // ---- X_t[:, cols] -= Y W2, chunk by chunk: the two resident chunks (NCH - 2,
  // NCH - 1) first, the others copied in again behind them; thread (ty, tx): rows
  // ty*4 .. +3 of a chunk, columns tx*4 .. +3 ----
  const bool full = tx * 4 + 4 <= wc;
#pragma unroll 1
  for (int step = 0; step < NCH; ++step) {
    const int m = step < 2 ? NCH - 2 + step : step - 2;  // chunk of this step
    const int sidx = m & 1;                               // its stage
    if (step >= 2) {
      // chunk m was copied in after step - 2 finished with its stage
      if (step + 1 < NCH) asm volatile("cp.async.wait_group 1;" ::: "memory");
      else asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncthreads();
    }
    if (m * CR < h) {
      const float* Yc = stage(sidx);
      const float* Xc = Yc + CR * LDS;
      float a3[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) a3[r][q] = 0.f;
#pragma unroll 4
      for (int l = 0; l < NB; l += 4) {
        float4 bw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) bw[u] = *reinterpret_cast<const float4*>(W + (l + u) * LDWS + tx * 4);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float4 yv = *reinterpret_cast<const float4*>(Yc + (ty * 4 + r) * LDS + l);
          const float yl[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            a3[r][0] = fmaf(yl[u], bw[u].x, a3[r][0]);
            a3[r][1] = fmaf(yl[u], bw[u].y, a3[r][1]);
            a3[r][2] = fmaf(yl[u], bw[u].z, a3[r][2]);
            a3[r][3] = fmaf(yl[u], bw[u].w, a3[r][3]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = m * CR + ty * 4 + r;
        if (i >= h) continue;
        const float4 xv = *reinterpret_cast<const float4*>(Xc + (ty * 4 + r) * LDWS + tx * 4);
        const float o[4] = {xv.x - a3[r][0], xv.y - a3[r][1], xv.z - a3[r][2], xv.w - a3[r][3]};
        float* dst = a.X + (row0 + i) * a.ldX + cs + tx * 4;
        if (full) {
          *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (tx * 4 + q < wc) dst[q] = o[q];
        }
      }
    }
    if (step < 2) {
      // this stage is free once every thread is done: copy in chunk step again
      __syncthreads();
      load_chunk(stage(sidx), a, row0, h, c0, nbk, cs, wc, step);
    }
  }
}
template <typename Tin>
__global__ void copy_chunk_kernel(float* X, int64_t ldX, const Tin* src, int64_t lds, int64_t rows,
                                  int64_t n, const int64_t* ridx, int64_t src_rows, int64_t cols,
                                  int* status) {
  const int64_t total = rows * n;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = idx / n, j = idx % n;
    int64_t si = i;
    if (ridx) {
      si = ridx[i];
      if (si < 0 || si >= src_rows) {
        if (status && j == 0) atomicExch(status, IFK_ERR_ARG);
        X[i * ldX + j] = 0.f;
        continue;
      }
    }
    X[i * ldX + j] = j < cols ? ld_elem(src, si * lds + j) : 1.f;
  }
}

// im2col rows of an NCHW image (ConvGeo), optionally gathered by ridx
template <typename Tin>
__global__ void copy_conv_kernel(float* X, int64_t ldX, const Tin* src, ConvGeo g, int64_t rows, int64_t n,
                                 const int64_t* ridx, int64_t src_rows, int64_t cols, int* status) {
  const int64_t total = rows * n;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = idx / n, j = idx % n;
    int64_t si = i;
    if (ridx) {
      si = ridx[i];
      if (si < 0 || si >= src_rows) {
        if (status && j == 0) atomicExch(status, IFK_ERR_ARG);
        X[i * ldX + j] = 0.f;
        continue;
      }
    }
    float v = 1.f;
    if (j < cols) {
      const int64_t off = conv_offset(g, si, j);
      v = off >= 0 ? ld_elem(src, off) : 0.f;
    }
    X[i * ldX + j] = v;
  }
}

__global__ void fill_identity_kernel(float* X, int64_t ldX, int64_t n, float v) {
  const int64_t total = n * n;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = idx / n, j = idx % n;
    X[i * ldX + j] = (i == j) ? v : 0.f;
  }
}

// Row-per-block elementwise passes over an n x n factor: blockIdx.y (and further
// rows by stride) picks the row, the threads take its columns 4 at a time.
__device__ __forceinline__ bool aligned16(const void* p, int64_t ld, int bytes) {
  return ((uintptr_t)p % 16) == 0 && (ld * bytes) % 16 == 0;
}

__global__ void scale_upper_kernel(float* Ro, int64_t ldo, const float* Ri, int64_t ldi, int64_t n,
                                   float scale) {
  const bool vec = aligned16(Ro, ldo, 4) && aligned16(Ri, ldi, 4);
  for (int64_t i = blockIdx.y; i < n; i += gridDim.y) {
    const float* src = Ri + i * ldi;
    float* dst = Ro + i * ldo;
    for (int64_t j0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; j0 < n;
         j0 += (int64_t)gridDim.x * blockDim.x * 4) {
      if (vec && j0 + 4 <= n) {
        const float4 v = *reinterpret_cast<const float4*>(src + j0);
        float4 o;
        o.x = j0 >= i ? v.x / scale : 0.f;
        o.y = j0 + 1 >= i ? v.y / scale : 0.f;
        o.z = j0 + 2 >= i ? v.z / scale : 0.f;
        o.w = j0 + 3 >= i ? v.w / scale : 0.f;
        *reinterpret_cast<float4*>(dst + j0) = o;
      } else {
        for (int64_t j = j0; j < j0 + 4 && j < n; ++j) dst[j] = (j >= i) ? src[j] / scale : 0.f;
      }
    }
  }
}

// out = upper(R) / scale (scale 1: a copy) in out's element type; any non-finite
// value sets IFK_ERR_NONFINITE.  With scale != 1 this is the damping-free finalize
// in one pass: the same division and cast as scale_upper followed by the cast.
template <typename Tout>
__global__ void finish_factor_kernel(Tout* out, int64_t ldo, const float* R, int64_t ldR, int64_t n,
                                     int* status, float scale, int apply_scale) {
  bool bad = false;
  const bool vec = aligned16(R, ldR, 4) && aligned16(out, ldo, sizeof(Tout) == 2 ? 2 : 4) &&
                   (sizeof(Tout) == 4 || ((uintptr_t)out % 8) == 0);
  for (int64_t i = blockIdx.y; i < n; i += gridDim.y) {
    const float* src = R + i * ldR;
    Tout* dst = out + i * ldo;
    for (int64_t j0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; j0 < n;
         j0 += (int64_t)gridDim.x * blockDim.x * 4) {
      float v[4];
      const bool full = vec && j0 + 4 <= n;
      if (full) {
        const float4 x = *reinterpret_cast<const float4*>(src + j0);
        v[0] = x.x;
        v[1] = x.y;
        v[2] = x.z;
        v[3] = x.w;
      } else {
        for (int e = 0; e < 4; ++e) v[e] = j0 + e < n ? src[j0 + e] : 0.f;
      }
      if (apply_scale) {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (j0 + e >= i) ? v[e] / scale : 0.f;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) bad |= (j0 + e < n) && !isfinite(v[e]);
      if constexpr (sizeof(Tout) == 2) {
        if (full) {
          __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
          uint2 u;
          u.x = *reinterpret_cast<uint32_t*>(&a);
          u.y = *reinterpret_cast<uint32_t*>(&b);
          *reinterpret_cast<uint2*>(dst + j0) = u;
        } else {
          for (int e = 0; e < 4; ++e)
            if (j0 + e < n) dst[j0 + e] = __float2bfloat16_rn(v[e]);
        }
      } else {
        if (apply_scale || (const void*)out != (const void*)R || ldo != ldR) {
          if (full) {
            *reinterpret_cast<float4*>(dst + j0) = make_float4(v[0], v[1], v[2], v[3]);
          } else {
            for (int e = 0; e < 4; ++e)
              if (j0 + e < n) dst[j0 + e] = v[e];
          }
        }
      }
    }
  }
  if (bad && status) atomicExch(status, IFK_ERR_NONFINITE);
}

dim3 rows_grid(int64_t n) {
  const int64_t x = cdiv(cdiv(n, 4), 256);
  const int64_t y = n < 2048 ? n : 2048;
  return dim3((unsigned)(x < 1 ? 1 : x), (unsigned)(y < 1 ? 1 : y));
}

int grid_for(int64_t total) {
  int64_t g = cdiv(total, 256);
  if (g > 148 * 16) g = 148 * 16;
  return (int)(g < 1 ? 1 : g);
}

bool set_smem_attr_once() {
  static thread_local int done_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (done_dev == dev) return true;
  if (cudaFuncSetAttribute(fold_panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)panel_smem_bytes()) != cudaSuccess)
    return false;
  if (cudaFuncSetAttribute(fold_update_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)upd_smem_bytes()) != cudaSuccess)
    return false;
  done_dev = dev;
  return true;
}

}  // namespace

// Defined in tsqr_tc.cu: tensor-core trailing update of one wave.
int fold_update_tc_launch(const FoldBatch& b, int tiles, int64_t ncols, int wave, cudaStream_t s);

int64_t xw_ld(int64_t n) { return cdiv(n, 4) * 4; }
size_t xw_bytes(int64_t rows, int64_t n) { return (size_t)rows * xw_ld(n) * sizeof(float); }
size_t fold_tbuf_bytes(int64_t rows) { return (size_t)cdiv(rows, SUB) * NB * NB * sizeof(float); }

int copy_chunk(float* X, int64_t ldX, const void* chunk, int64_t ld_chunk, int64_t rows, int64_t n,
               int dtype, cudaStream_t s, const int64_t* ridx, int64_t src_rows, int64_t cols, int* status,
               const ConvGeo* conv) {
  if (rows == 0) return IFK_OK;
  if (cols < 0) cols = n;
  if (conv) {
    if (dtype == IFK_BF16)
      copy_conv_kernel<<<grid_for(rows * n), 256, 0, s>>>(X, ldX, (const __nv_bfloat16*)chunk, *conv, rows, n, ridx,
                                                          src_rows, cols, status);
    else
      copy_conv_kernel<<<grid_for(rows * n), 256, 0, s>>>(X, ldX, (const float*)chunk, *conv, rows, n, ridx,
                                                          src_rows, cols, status);
    IFK_CUDA_TRY(cudaGetLastError());
    return IFK_OK;
  }
  if (dtype == IFK_BF16)
    copy_chunk_kernel<<<grid_for(rows * n), 256, 0, s>>>(
        X, ldX, (const __nv_bfloat16*)chunk, ld_chunk, rows, n, ridx, src_rows, cols, status);
  else
    copy_chunk_kernel<<<grid_for(rows * n), 256, 0, s>>>(X, ldX, (const float*)chunk, ld_chunk,
                                                         rows, n, ridx, src_rows, cols, status);
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

int fill_scaled_identity(float* X, int64_t ldX, int64_t n, float v, cudaStream_t s) {
  fill_identity_kernel<<<grid_for(n * n), 256, 0, s>>>(X, ldX, n, v);
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

int scale_upper(float* Rout, int64_t ldo, const float* Rin, int64_t ldi, int64_t n, float scale,
                cudaStream_t s) {
  scale_upper_kernel<<<rows_grid(n), 256, 0, s>>>(Rout, ldo, Rin, ldi, n, scale);
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

int finish_factor(void* out, int64_t ldo, int out_dtype, const float* R, int64_t ldR, int64_t n,
                  int* d_status, cudaStream_t s, float scale) {
  const int apply = scale > 0.f ? 1 : 0;
  if (out_dtype == IFK_BF16)
    finish_factor_kernel<<<rows_grid(n), 256, 0, s>>>((__nv_bfloat16*)out, ldo, R, ldR, n, d_status, scale, apply);
  else
    finish_factor_kernel<<<rows_grid(n), 256, 0, s>>>((float*)out, ldo, R, ldR, n, d_status, scale, apply);
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

int fold_run_batch(const FoldBatch& b, int prec, cudaStream_t s) {
  if (b.nf <= 0) return IFK_OK;
  if (!set_smem_attr_once()) return IFK_ERR_CUDA;
  int waves = 0, tiles = 0;
  int64_t ncols = 0;
  for (int f = 0; f < b.nf; ++f) {
    if (b.f[f].rows == 0) continue;
    waves = (int)mx<int64_t>(waves, b.f[f].tiles + b.f[f].K - 1);
    tiles = (int)mx<int64_t>(tiles, b.f[f].tiles);
    ncols = mx<int64_t>(ncols, b.f[f].n);
  }
  if (waves == 0) return IFK_OK;
  const dim3 pgrid(tiles, 1, b.nf);
  const dim3 ugrid(tiles, (unsigned)cdiv(ncols, WC), b.nf);
  for (int w = 0; w < waves; ++w) {
    fold_panel_kernel<<<pgrid, PT2, panel_smem_bytes(), s>>>(b, w);
    if (prec == IFK_PREC_BF16) {
      const int rc = fold_update_tc_launch(b, tiles, ncols, w, s);
      if (rc != IFK_OK) return rc;
    } else {
      fold_update_simt_kernel<<<ugrid, PT, upd_smem_bytes(), s>>>(b, w);
    }
  }
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

int fold_run(const FoldArgs& a, int prec, cudaStream_t s) {
  FoldBatch b;
  b.f[0] = a;
  b.nf = 1;
  return fold_run_batch(b, prec, s);
}

}  // namespace ifk
