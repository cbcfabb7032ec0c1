// gemm_kind_bf16.cu - instantiations of the GEMM for operand kind bf16.
#include "gemm_impl.cuh"

namespace rg {
template cudaError_t dispatch_kind<0>(int, int, const GemmMaps&, const GemmArgs&, int, cudaStream_t);
}  // namespace rg
