// Placeholder for the tcgen05 path: declines every problem so callers use the
// CUDA-core kernel.
#include "kernels.h"

namespace sb {

size_t gemm_tcgen05_workspace(const GemmArgs&, bool) { return 0; }

cudaError_t gemm_tcgen05(const GemmArgs&, bool, void*, size_t, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace sb
