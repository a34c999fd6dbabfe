// Temporary: the tensor-core triangular solve is not built yet.
#include "ifk_common.cuh"
#include "ifk_internal.h"
namespace ifk {
int trsm_tc_run(const void*, int64_t, int, int, float*, int64_t, int64_t, int64_t, int64_t, cudaStream_t) { return IFK_ERR_ARG; }
}
