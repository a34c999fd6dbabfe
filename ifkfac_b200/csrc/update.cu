// Weight update epilogue (ifkfac/ifkfac.py:394-423): optional norm clip of
// the natural gradient, momentum, decoupled weight decay, lr step on fp32
// master weights.  HBM-bound elementwise work: one pass reads nat, buf, W
// and writes buf, W (20 bytes per element), vectorised by 4.
#include "ifk_common.cuh"
#include "ifk_internal.h"

namespace ifk {

namespace {

__global__ void sumsq_kernel(const float* x, int64_t count, double* out) {
  double s = 0.0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const double v = x[i];
    s += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ double part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) atomicAdd(out, s);
  }
}

struct UpdParams {
  float lr, mom, decay, clip;
  int use_mom, use_decay, use_clip, buf_new;
};

__device__ __forceinline__ float upd_one(float w, float* bufp, float g, const UpdParams& p, float gs) {
  // the element arithmetic is shared with the fused epilogue of the last solve
  UpdCoef c;
  c.lr = p.lr;
  c.mom = p.mom;
  c.decay = p.decay;
  c.use_mom = p.use_mom;
  c.use_decay = p.use_decay;
  c.buf_new = p.buf_new;
  return upd_elem(w, *bufp, __fmul_rn(g, gs), c);
}

__global__ void update_kernel(float* W, float* buf, const float* nat, int64_t count, UpdParams p,
                              const double* sumsq) {
  float gs = 1.f;
  if (p.use_clip) {
    const float gn = (float)sqrt(*sumsq);
    if (gn > p.clip) gs = p.clip / gn;
  }
  const int64_t n4 = count / 4;
  const bool vec = ((((uintptr_t)W) | ((uintptr_t)nat) | (p.use_mom ? (uintptr_t)buf : 0)) & 15) == 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t tail0 = 0;
  if (vec) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 w = reinterpret_cast<float4*>(W)[i];
      const float4 g = reinterpret_cast<const float4*>(nat)[i];
      float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p.use_mom && !p.buf_new) b = reinterpret_cast<float4*>(buf)[i];
      float bb[4] = {b.x, b.y, b.z, b.w};
      const float gg[4] = {g.x, g.y, g.z, g.w};
      float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) ww[q] = upd_one(ww[q], &bb[q], gg[q], p, gs);
      if (p.use_mom) reinterpret_cast<float4*>(buf)[i] = make_float4(bb[0], bb[1], bb[2], bb[3]);
      reinterpret_cast<float4*>(W)[i] = make_float4(ww[0], ww[1], ww[2], ww[3]);
    }
    tail0 = n4 * 4;
  }
  for (int64_t i = tail0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += stride) {
    float bv = 0.f;
    if (p.use_mom && !p.buf_new) bv = buf[i];
    W[i] = upd_one(W[i], &bv, nat[i], p, gs);
    if (p.use_mom) buf[i] = bv;
  }
}

__global__ void update_bias_kernel(float* b, const float* nat, int64_t count, float lr, float decay,
                                   int use_decay) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = b[i];
    if (use_decay) v *= decay;
    b[i] = v - lr * nat[i];
  }
}

int grid_elems(int64_t count) {
  int64_t g = cdiv(cdiv(count, 4), 256);
  if (g > 148 * 8) g = 148 * 8;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

int update_run(float* W, float* buf, const float* nat, int64_t count, double lr, double mom,
               double wd, double clip, int buf_is_new, double* norm_ws, cudaStream_t s) {
  if (count == 0) return IFK_OK;
  UpdParams p;
  p.lr = (float)lr;
  p.mom = (float)mom;
  p.decay = (float)(1.0 - lr * wd);
  p.clip = (float)clip;
  p.use_mom = mom > 0;
  p.use_decay = wd > 0;
  p.use_clip = clip > 0;
  p.buf_new = buf_is_new ? 1 : 0;
  if (p.use_clip) {
    IFK_CUDA_TRY(cudaMemsetAsync(norm_ws, 0, sizeof(double), s));
    sumsq_kernel<<<grid_elems(count), 256, 0, s>>>(nat, count, norm_ws);
  }
  update_kernel<<<grid_elems(count), 256, 0, s>>>(W, buf, nat, count, p, norm_ws);
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

int update_bias_run(float* b, const float* nat, int64_t count, double lr, double wd,
                    cudaStream_t s) {
  if (count == 0) return IFK_OK;
  update_bias_kernel<<<grid_elems(count), 256, 0, s>>>(b, nat, count, (float)lr,
                                                       (float)(1.0 - lr * wd), wd > 0);
  IFK_CUDA_TRY(cudaGetLastError());
  return IFK_OK;
}

}  // namespace ifk
