// Dense GEMV kernels for Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 (instantiation unit).
#include "fn_gemv_impl.cuh"

namespace fn {
FN_GEMV_INST(T_Q4_0)
FN_GEMV_INST(T_Q4_1)
FN_GEMV_INST(T_Q5_0)
FN_GEMV_INST(T_Q5_1)
FN_GEMV_INST(T_Q8_0)
}  // namespace fn
