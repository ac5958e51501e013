// Instantiations of the GEMV launcher (fp4x_launch.cuh) compiled in their own translation unit.
#include "fp4x_launch.cuh"

namespace fp4x {
template int launch_nt<FMT_BF16, EPI_STORE>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
template int launch_nt<FMT_INT2, EPI_HEAD>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
}  // namespace fp4x
