// Tensor-core GEMM kernels for __nv_bfloat16, A M-contiguous, B K-contiguous:
// one of the eight instantiation units of bio_gemm_tc.cuh (split so that the
// kernels compile in parallel).
#include "bio_gemm_tc.cuh"

namespace bio_gemm_tc {
BIO_GEMM_TC_DECL(, true, false, __nv_bfloat16)
}  // namespace bio_gemm_tc
