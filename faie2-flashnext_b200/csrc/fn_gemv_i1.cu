// Dense GEMV kernels for Q2_K, Q3_K, Q4_K, Q5_K, Q6_K (instantiation unit).
#include "fn_gemv_impl.cuh"

namespace fn {
FN_GEMV_INST(T_Q2_K)
FN_GEMV_INST(T_Q3_K)
FN_GEMV_INST(T_Q4_K)
FN_GEMV_INST(T_Q5_K)
FN_GEMV_INST(T_Q6_K)
}  // namespace fn
