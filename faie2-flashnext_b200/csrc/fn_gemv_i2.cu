// Dense GEMV kernels for IQ2_XXS, IQ2_XS, IQ2_S, IQ3_XXS, IQ3_S (instantiation unit).
#include "fn_gemv_impl.cuh"

namespace fn {
FN_GEMV_INST(T_IQ2_XXS)
FN_GEMV_INST(T_IQ2_XS)
FN_GEMV_INST(T_IQ2_S)
FN_GEMV_INST(T_IQ3_XXS)
FN_GEMV_INST(T_IQ3_S)
}  // namespace fn
