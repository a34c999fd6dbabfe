// Shared definitions of the IFKFAC sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/ifk.h"

namespace ifk {

// Blocking of the streaming TSQR (TPQRT: triangle on top of a row tile).
// A chunk is folded in sub-tiles of SUB rows; each sub-tile is a blocked
// Householder fold with panels of NB columns and compact-WY trailing updates
// on column blocks of WC columns.
constexpr int NB = 64;
constexpr int SUB = 256;
constexpr int WC = 64;

// Blocking of the triangular solves: NS rows per diagonal block, NRHS
// right-hand-side columns per tile.
constexpr int NS = 64;
constexpr int NRHS = 64;

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
template <typename T>
__host__ __device__ __forceinline__ T mn(T a, T b) { return a < b ? a : b; }
template <typename T>
__host__ __device__ __forceinline__ T mx(T a, T b) { return a < b ? b : a; }

__device__ __forceinline__ float ld_elem(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float ld_elem(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// A strided read-only matrix view: element (i, j) at base[i*rs + j*cs].
// Transposed factors and transposed right-hand sides are views, not copies.
template <typename T>
struct View {
  const T* base;
  int64_t rs, cs;
  __device__ __forceinline__ float operator()(int64_t i, int64_t j) const {
    return ld_elem(base, i * rs + j * cs);
  }
};

struct MutView {
  float* base;
  int64_t rs, cs;
  __device__ __forceinline__ float& operator()(int64_t i, int64_t j) const {
    return base[i * rs + j * cs];
  }
};

// 4 consecutive floats from a 16-byte aligned address; elements at index >= valid read as 0.
__device__ __forceinline__ float4 ld4(const float* p, int valid) {
  if (valid >= 4) return *reinterpret_cast<const float4*>(p);
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (valid > 0) r.x = p[0];
  if (valid > 1) r.y = p[1];
  if (valid > 2) r.z = p[2];
  return r;
}
__device__ __forceinline__ void st4(float* p, float4 v, int valid) {
  if (valid >= 4) {
    *reinterpret_cast<float4*>(p) = v;
    return;
  }
  if (valid > 0) p[0] = v.x;
  if (valid > 1) p[1] = v.y;
  if (valid > 2) p[2] = v.z;
}

// One element of the momentum / lr update on fp32 master weights
// (ifkfac/ifkfac.py:394-413; a clip factor, when any, is already applied to g):
//   buf = mom * buf + g (buf read as zero when buf_new), g = buf;  W *= decay;  W -= lr * g.
struct UpdCoef {
  float lr, mom, decay;
  int use_mom, use_decay, buf_new;
};
// The rounding steps are spelled out (fused multiply-adds, no compiler
// contraction), so every kernel that applies the update gives the same bits.
__device__ __forceinline__ float upd_elem(float w, float& b, float g, const UpdCoef& p) {
  if (p.use_mom) {
    b = __fmaf_rn(p.buf_new ? 0.f : b, p.mom, g);
    g = b;
  }
  if (p.use_decay) w = __fmul_rn(w, p.decay);
  return __fmaf_rn(-p.lr, g, w);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace ifk

#define IFK_CUDA_TRY(expr)                                  \
  do {                                                      \
    cudaError_t e_ = (expr);                                \
    if (e_ != cudaSuccess) return IFK_ERR_CUDA;             \
  } while (0)
