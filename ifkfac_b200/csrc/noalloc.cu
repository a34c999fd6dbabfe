// ifk_natgrad_noalloc: the natural gradient without any device allocation.
//
// Some callers cannot allocate device memory at the point where they need
// the natural gradient: for example an optimizer step issued from inside
// another framework's operator whose memory is owned by that framework's own
// pool (so a call into the CUDA allocator, or a second pool, is not allowed
// there), or a host runtime that works only with buffers it was handed up
// front.  For them this entry point takes no workspace: the scratch the
// tensor-core solves need (the bf16 hi/lo inverses of the 128 x 128 diagonal
// blocks of one factor) lives in a fixed file-scope device array sized for
// factors of order up to IFK_NOALLOC_MAX_N.  Every GPU that loads the library
// holds that array until the process exits.
#include "ifk_common.cuh"
#include "ifk_internal.h"

namespace {

constexpr int64_t kMaxN = IFK_NOALLOC_MAX_N;
constexpr size_t kScratchBytes = 2ull << 20;  // trsm_tc_workspace(IFK_NOALLOC_MAX_N), checked per call

// Shared by every call on a device; it keeps the last call's contents.
static __device__ __align__(256) unsigned char g_natgrad_scratch[kScratchBytes];

// Device address of g_natgrad_scratch in the current context.  In host code the
// symbol itself is only a host-side handle, never a device address, so kernels
// are always given the address looked up here, with the calling device
// current.  It is looked up on every call (cheap once the module is loaded)
// rather than cached per device, so a context destroyed and created again
// (cudaDeviceReset) never leaves a stale address behind.  The first call on a
// device loads the module there; make it before any stream capture.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return IFK_ERR_CUDA;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_natgrad_scratch) != cudaSuccess || !p) return IFK_ERR_CUDA;
  *out = p;
  return IFK_OK;
}

}  // namespace

extern "C" int ifk_natgrad_noalloc(const float* grad_W, int64_t ld_g, const void* R_X, int64_t ld_rx,
                                   const void* R_G, int64_t ld_rg, int r_dtype, float* nat,
                                   int64_t ld_nat, int64_t n_out, int64_t n_in, int prec,
                                   int* d_status, ifk_stream_t stream) {
  if (!grad_W || !R_X || !R_G || !nat) return IFK_ERR_ARG;
  if (n_out <= 0 || n_in <= 0 || ld_g < n_in || ld_nat < n_in || ld_rx < n_in || ld_rg < n_out)
    return IFK_ERR_SHAPE;
  if (n_out > kMaxN || n_in > kMaxN) return IFK_ERR_LIMIT;
  // the scratch layout of the per-block-row solves must fit the fixed array
  if (ifk::trsm_tc_workspace(n_out > n_in ? n_out : n_in) > kScratchBytes) return IFK_ERR_LIMIT;
  if (r_dtype != IFK_F32 && r_dtype != IFK_BF16) return IFK_ERR_DTYPE;
  if (prec != IFK_PREC_AUTO && prec != IFK_PREC_FP32 && prec != IFK_PREC_BF16) return IFK_ERR_ARG;
  if (prec == IFK_PREC_AUTO) prec = r_dtype == IFK_BF16 ? IFK_PREC_BF16 : IFK_PREC_FP32;
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != IFK_OK) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (nat != grad_W || ld_nat != ld_g) {
    IFK_CUDA_TRY(cudaMemcpy2DAsync(nat, ld_nat * sizeof(float), grad_W, ld_g * sizeof(float),
                                   n_in * sizeof(float), n_out, cudaMemcpyDeviceToDevice, s));
  }
  // the four solves of ifk_natgrad; each writes the scratch inverses before reading them
  rc = ifk::trsm_run(R_G, ld_rg, r_dtype, 1, nat, ld_nat, 1, n_out, n_in, prec, scratch, d_status, s);
  if (rc != IFK_OK) return rc;
  rc = ifk::trsm_run(R_G, ld_rg, r_dtype, 0, nat, ld_nat, 1, n_out, n_in, prec, scratch, d_status, s);
  if (rc != IFK_OK) return rc;
  rc = ifk::trsm_run(R_X, ld_rx, r_dtype, 1, nat, 1, ld_nat, n_in, n_out, prec, scratch, d_status, s);
  if (rc != IFK_OK) return rc;
  return ifk::trsm_run(R_X, ld_rx, r_dtype, 0, nat, 1, ld_nat, n_in, n_out, prec, scratch, d_status, s);
}
