// gemm_kind_f16.cu - instantiations of the GEMM for operand kind f16.
#include "gemm_impl.cuh"

namespace rg {
template cudaError_t dispatch_kind<2>(int, int, const GemmMaps&, const GemmArgs&, int, cudaStream_t);
}  // namespace rg
