// Tensor-core GEMM kernels for __nv_bfloat16, A M-contiguous, B N-contiguous:
// one of the eight instantiation units of bio_gemm_tc.cuh (split so that the
// kernels compile in parallel).
#include "bio_gemm_tc.cuh"

namespace bio_gemm_tc {
BIO_GEMM_TC_DECL(, true, true, __nv_bfloat16)
}  // namespace bio_gemm_tc
