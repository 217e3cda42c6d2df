// Dense GEMV kernels for IQ4_NL, IQ4_XS, BF16, Q2_0 (instantiation unit).
#include "fn_gemv_impl.cuh"

namespace fn {
FN_GEMV_INST(T_IQ4_NL)
FN_GEMV_INST(T_IQ4_XS)
FN_GEMV_INST(T_BF16)
FN_GEMV_INST(T_Q2_0)
}  // namespace fn
