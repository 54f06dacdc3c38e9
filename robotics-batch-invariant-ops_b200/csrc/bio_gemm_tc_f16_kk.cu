// Tensor-core GEMM kernels for __half, A K-contiguous, B K-contiguous:
// one of the eight instantiation units of bio_gemm_tc.cuh (split so that the
// kernels compile in parallel).
#include "bio_gemm_tc.cuh"

namespace bio_gemm_tc {
BIO_GEMM_TC_DECL(, false, false, __half)
}  // namespace bio_gemm_tc
