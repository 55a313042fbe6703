// Instantiations of the tcgen05 GEMM kernel for bf16 operands, implicit 3x3 convolution A.
#include "gemm_tc_kernel.cuh"

namespace dav2cuda {
namespace gemm_impl {
int dispatch_bf16_conv(int bn, const CUtensorMap& ma, const CUtensorMap& mb, const EpiMaps& em, const GemmParamsDev& p,
                 uint32_t staging, int max_ctas, cudaStream_t st, bool epi8) {
    return dispatch_bn<kElemBF16, kAModeConv3x3>(bn, ma, mb, em, p, staging, max_ctas, st, epi8);
}
}  // namespace gemm_impl
}  // namespace dav2cuda
