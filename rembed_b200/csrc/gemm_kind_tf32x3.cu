// gemm_kind_tf32x3.cu - instantiations of the GEMM for operand kind tf32x3.
#include "gemm_impl.cuh"

namespace rg {
template cudaError_t dispatch_kind<4>(int, int, const GemmMaps&, const GemmArgs&, int, cudaStream_t);
}  // namespace rg
