// gemm_kind_w8.cu - instantiations of the GEMM for operand kind w8.
#include "gemm_impl.cuh"

namespace rg {
template cudaError_t dispatch_kind<3>(int, int, const GemmMaps&, const GemmArgs&, int, cudaStream_t);
}  // namespace rg
