// tcgen05 tensor-core MLP (placeholder until the tensor-core kernels land).
#include "sc_internal.h"

namespace sc {

bool mlp_tc_supported(const sc_model *) { return false; }
void mlp_tc_prepare(sc_model *) {}
void mlp_tc(sc_model *m, const int16_t *windows, int64_t rows, int8_t *logits, cudaStream_t s)
{
    mlp_simple(m, windows, rows, logits, s);
}

}  // namespace sc
