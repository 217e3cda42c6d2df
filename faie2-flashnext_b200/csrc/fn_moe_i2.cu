// Routed-expert kernels for IQ2_XXS, IQ2_XS, IQ2_S, IQ3_XXS, IQ3_S (instantiation unit).
#include "fn_moe_impl.cuh"

namespace fn {
FN_MOE_INST(T_IQ2_XXS)
FN_MOE_INST(T_IQ2_XS)
FN_MOE_INST(T_IQ2_S)
FN_MOE_INST(T_IQ3_XXS)
FN_MOE_INST(T_IQ3_S)
}  // namespace fn
