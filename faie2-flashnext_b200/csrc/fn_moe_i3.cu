// Routed-expert kernels for IQ4_NL, IQ4_XS, BF16, Q2_0 (instantiation unit).
#include "fn_moe_impl.cuh"

namespace fn {
FN_MOE_INST(T_IQ4_NL)
FN_MOE_INST(T_IQ4_XS)
FN_MOE_INST(T_BF16)
FN_MOE_INST(T_Q2_0)
}  // namespace fn
