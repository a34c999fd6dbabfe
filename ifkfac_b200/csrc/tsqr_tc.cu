// Tensor-core (tcgen05) trailing update of the streaming TSQR fold.
//
// One CTA applies the compact-WY block reflector of panel k of sub-tile t to
// one block of WT = 128 trailing columns:
//   GEMM1  D1 = X_t^T Y          (128 x 64,  K = SUB)      bf16 operands
//   W^T    = D1 + R[k rows, c]^T                               fp32
//   GEMM2  D2 = W^T T            (128 x 64,  K = NB)       3-term bf16 split
//   R[k rows, c] -= D2^T                                       fp32
//   GEMM3  D3 = Y W2             (256 x 128, K = NB)       bf16 operands
//   X_t[:, c] -= D3                                            fp32
// Accumulators live in TMEM (D1 64 cols, D2 64, D3 2 x 128).  The fp32
// working copy X_t and R stay fp32 in global memory; operands are rounded to
// bf16 only when staged into shared memory.  GEMM2 multiplies by T, whose
// entries are not small integers, so W and T are each split into bf16 hi+lo
// and three products (hi.hi + hi.lo + lo.hi) keep ~16 significant bits.
#include "ifk_common.cuh"
#include "ifk_internal.h"
#include "tc.cuh"

namespace ifk {

namespace {

constexpr int WT = 128;   // trailing columns per CTA
constexpr int TPB = 128;  // 4 warps: warp w owns TMEM lanes 32w..32w+31

// shared-memory map (bytes)
constexpr uint32_t SZ_A1 = WT * SUB * 2;   // X_t^T, MN-major (mn = column c, k = row i)
constexpr uint32_t SZ_Y = SUB * NB * 2;    // Y: B of GEMM1 (MN-major) and A of GEMM3 (K-major)
constexpr uint32_t SZ_A2 = WT * NB * 2;    // W^T hi / lo, K-major (mn = c, k = j)
constexpr uint32_t SZ_B2 = NB * NB * 2;    // T hi / lo, K-major (mn = j, k = l)
constexpr uint32_t OFF_A1 = 0;
constexpr uint32_t OFF_Y = OFF_A1 + SZ_A1;
constexpr uint32_t OFF_A2H = OFF_Y + SZ_Y;
constexpr uint32_t OFF_A2L = OFF_A2H + SZ_A2;
constexpr uint32_t OFF_B2H = OFF_A2L + SZ_A2;
constexpr uint32_t OFF_B2L = OFF_B2H + SZ_B2;
constexpr uint32_t OFF_B3 = OFF_B2L + SZ_B2;  // W2, K-major (mn = c, k = j)
constexpr uint32_t OFF_BAR = OFF_B3 + SZ_A2;
constexpr uint32_t SMEM = OFF_BAR + 64;

// core-matrix strides
constexpr uint32_t A1_MN = 128, A1_K = (WT / 8) * 128;   // 128, 2048
constexpr uint32_t Y_I = 1024, Y_J = 128;                // i-stride, j-stride
constexpr uint32_t A2_MN = 128, A2_K = (WT / 8) * 128;   // 128, 2048
constexpr uint32_t B2_MN = 128, B2_K = (NB / 8) * 128;   // 128, 1024

constexpr uint32_t TM_D1 = 0, TM_D2 = 64, TM_D3 = 128, TM_COLS = 512;

// Task (t, k) of the wave schedule (every panel is factored: see tsqr.cu).
__device__ __forceinline__ bool task_active_tc(const FoldArgs& a, int t, int k) {
  if (t < 0 || t >= a.tiles || k < 0 || k >= a.K) return false;
  return !(a.tri && (int64_t)k * NB + NB <= (int64_t)t * SUB);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ void store8(uint32_t addr, const float (&v)[8]) {
  st_shared_v4(addr, tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]), tc::pack_bf16(v[4], v[5]),
               tc::pack_bf16(v[6], v[7]));
}

__global__ void __launch_bounds__(TPB, 1) fold_update_tc_kernel(FoldBatch fb, int wave) {
  const FoldArgs& a = fb.f[blockIdx.z];
  const int t = blockIdx.x;
  const int k = wave - t;
  if (!task_active_tc(a, t, k)) return;
  const int64_t c0 = (int64_t)k * NB;
  const int64_t cs = c0 + NB + (int64_t)blockIdx.y * WT;
  if (cs >= a.n) return;

  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  const uint32_t sbase = tc::smem_u32(sm);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row0 = (int64_t)t * SUB;
  const int h = (int)mn<int64_t>(SUB, a.rows - row0);
  const int nbk = (int)mn<int64_t>(NB, a.n - c0);
  const int wc = (int)mn<int64_t>(WT, a.n - cs);
  const float* Tb = a.Tb + (size_t)t * NB * NB;
  const float* Xt = a.X + row0 * a.ldX;

  if (warp == 0) tc::tmem_alloc(tslot, TM_COLS);
  if (tid == 0) tc::mbar_init(bar, 1);

  // ---- stage operands: X_t^T (A1), Y, T hi/lo ----
  constexpr int UN = 4;  // items in flight per thread (2 x 16-byte loads each)
  for (int q0 = tid; q0 < SUB * (WT / 8); q0 += UN * TPB) {  // item: row i, 8 columns
    float4 v[UN][2];
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const int q = q0 + u * TPB, i = (q & 7) + 8 * (q >> 7), c8 = (q >> 3) & 15;
      const float* src = Xt + (int64_t)i * a.ldX + cs + c8 * 8;
      const bool in = i < h;
      v[u][0] = in ? ld4(src, wc - c8 * 8) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[u][1] = in ? ld4(src + 4, wc - c8 * 8 - 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const int q = q0 + u * TPB, i = (q & 7) + 8 * (q >> 7), c8 = (q >> 3) & 15;
      const float e8[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                           v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
      store8(sbase + OFF_A1 + tc::cm_off<false>(c8 * 8, i, A1_MN, A1_K), e8);
    }
  }
  for (int q0 = tid; q0 < SUB * (NB / 8); q0 += UN * TPB) {  // item: row i, 8 panel columns
    float4 v[UN][2];
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const int q = q0 + u * TPB, i = (q & 7) + 8 * (q >> 6), j8 = (q >> 3) & 7;
      const float* src = Xt + (int64_t)i * a.ldX + c0 + j8 * 8;
      const bool in = i < h;
      v[u][0] = in ? ld4(src, nbk - j8 * 8) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[u][1] = in ? ld4(src + 4, nbk - j8 * 8 - 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const int q = q0 + u * TPB, i = (q & 7) + 8 * (q >> 6), j8 = (q >> 3) & 7;
      const float e8[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                           v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
      store8(sbase + OFF_Y + tc::cm_off<true>(i, j8 * 8, Y_I, Y_J), e8);
    }
  }
  for (int q = tid; q < NB * (NB / 8); q += TPB) {  // item: column j of T, 8 rows l
    const int j = (q & 7) + 8 * (q >> 6), l8 = (q >> 3) & 7;
    const float4 t0 = *reinterpret_cast<const float4*>(Tb + j * NB + l8 * 8);
    const float4 t1 = *reinterpret_cast<const float4*>(Tb + j * NB + l8 * 8 + 4);
    const float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
    float hi[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) tc::split_bf16(tv[e], hi[e], lo[e]);
    const uint32_t off = tc::cm_off<true>(j, l8 * 8, B2_MN, B2_K);
    store8(sbase + OFF_B2H + off, hi);
    store8(sbase + OFF_B2L + off, lo);
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = *tslot;

  // ---- GEMM1: D1 (c x j) = X_t^T Y, K = SUB ----
  if (tid == 0) {
    constexpr uint32_t id1 = tc::idesc_bf16(128, NB, true, true);
#pragma unroll 1
    for (int s = 0; s < SUB / 16; ++s) {
      const uint64_t ad = tc::sdesc(sbase + OFF_A1 + s * 2 * A1_K, A1_K, A1_MN);
      const uint64_t bd = tc::sdesc(sbase + OFF_Y + s * 2 * Y_I, Y_I, Y_J);
      tc::mma_bf16(tm + TM_D1, ad, bd, id1, s > 0);
    }
    tc::commit(bar);
  }
  bool ok = tc::mbar_wait(bar, 0);
  tc::fence_after();

  // ---- W^T = D1 + R^T ; split into A2 hi / lo ----
  const int c = warp * 32 + lane;  // this thread's trailing column (TMEM lane)
  const uint32_t lane_base = tm + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float w[32];
    tc::tmem_ld32(lane_base + TM_D1 + half * 32, w);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = half * 32 + g * 8 + e;
        const float r = (j < nbk && c < wc) ? a.R[(c0 + j) * a.ldR + cs + c] : 0.f;
        tc::split_bf16(w[g * 8 + e] + r, hi[e], lo[e]);
      }
      const uint32_t off = tc::cm_off<true>(c, half * 32 + g * 8, A2_MN, A2_K);
      store8(sbase + OFF_A2H + off, hi);
      store8(sbase + OFF_A2L + off, lo);
    }
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  // ---- GEMM2: D2 = W^T T (hi.hi + hi.lo + lo.hi), K = NB ----
  if (tid == 0) {
    constexpr uint32_t id2 = tc::idesc_bf16(128, NB, false, false);
#pragma unroll 1
    for (int s = 0; s < NB / 16; ++s) {
      const uint64_t ah = tc::sdesc(sbase + OFF_A2H + s * 2 * A2_K, A2_K, A2_MN);
      const uint64_t al = tc::sdesc(sbase + OFF_A2L + s * 2 * A2_K, A2_K, A2_MN);
      const uint64_t bh = tc::sdesc(sbase + OFF_B2H + s * 2 * B2_K, B2_K, B2_MN);
      const uint64_t bl = tc::sdesc(sbase + OFF_B2L + s * 2 * B2_K, B2_K, B2_MN);
      tc::mma_bf16(tm + TM_D2, ah, bh, id2, s > 0);
      tc::mma_bf16(tm + TM_D2, ah, bl, id2, 1);
      tc::mma_bf16(tm + TM_D2, al, bh, id2, 1);
    }
    tc::commit(bar);
  }
  ok = tc::mbar_wait(bar, 1) && ok;
  tc::fence_after();

  // ---- R[k rows, c] -= W2^T ; W2 -> B3 (bf16) ----
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float w[32];
    tc::tmem_ld32(lane_base + TM_D2 + half * 32, w);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = half * 32 + g * 8 + e;
        v[e] = w[g * 8 + e];
        if (j < nbk && c < wc) a.R[(c0 + j) * a.ldR + cs + c] -= v[e];
      }
      store8(sbase + OFF_B3 + tc::cm_off<true>(c, half * 32 + g * 8, A2_MN, A2_K), v);
    }
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  // ---- GEMM3: D3 (i x c) = Y W2, two M = 128 halves, K = NB ----
  if (tid == 0) {
    constexpr uint32_t id3 = tc::idesc_bf16(128, WT, false, false);
#pragma unroll 1
    for (int mh = 0; mh < 2; ++mh) {
#pragma unroll 1
      for (int s = 0; s < NB / 16; ++s) {
        const uint64_t ad = tc::sdesc(sbase + OFF_Y + mh * 16 * Y_I + s * 2 * Y_J, Y_J, Y_I);
        const uint64_t bd = tc::sdesc(sbase + OFF_B3 + s * 2 * A2_K, A2_K, A2_MN);
        tc::mma_bf16(tm + TM_D3 + mh * WT, ad, bd, id3, s > 0);
      }
    }
    tc::commit(bar);
  }
  ok = tc::mbar_wait(bar, 0) && ok;
  tc::fence_after();

  // ---- X_t[:, c] -= D3 ----
#pragma unroll 1
  for (int mh = 0; mh < 2; ++mh) {
    const int i = mh * 128 + warp * 32 + lane;
    float* xrow = a.X + (row0 + i) * a.ldX + cs;
#pragma unroll 1
    for (int q = 0; q < WT / 32; ++q) {
      float d[32];
      tc::tmem_ld32(lane_base + TM_D3 + mh * WT + q * 32, d);
      if (i < h) {
        float4 x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = ld4(xrow + q * 32 + 4 * e, wc - q * 32 - 4 * e);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          x[e].x -= d[4 * e];
          x[e].y -= d[4 * e + 1];
          x[e].z -= d[4 * e + 2];
          x[e].w -= d[4 * e + 3];
          st4(xrow + q * 32 + 4 * e, x[e], wc - q * 32 - 4 * e);
        }
      }
    }
  }
  if (!ok && a.err) atomicExch(a.err, IFK_ERR_TIMEOUT);
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(tm, TM_COLS);
  }
}

bool tc_attr_once() {
  static thread_local int done_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (done_dev == dev) return true;
  if (cudaFuncSetAttribute(fold_update_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)SMEM) != cudaSuccess)
    return false;
  done_dev = dev;
  return true;
}

}  // namespace

int fold_update_tc_launch(const FoldBatch& b, int tiles, int64_t ncols, int wave, cudaStream_t s) {
  if (!tc_attr_once()) return IFK_ERR_CUDA;
  // trailing blocks of WT columns start right after the panel of task (t, wave - t);
  // the widest case is panel 0
  const unsigned gy = (unsigned)cdiv(mx<int64_t>(0, ncols - NB), WT);
  if (gy == 0) return IFK_OK;
  fold_update_tc_kernel<<<dim3(tiles, gy, b.nf), TPB, SMEM, s>>>(b, wave);
  return IFK_OK;
}

}  // namespace ifk
