// gemm_kind_s8.cu - instantiations of the GEMM for operand kind s8.
#include "gemm_impl.cuh"

namespace rg {
template cudaError_t dispatch_kind<1>(int, int, const GemmMaps&, const GemmArgs&, int, cudaStream_t);
}  // namespace rg
