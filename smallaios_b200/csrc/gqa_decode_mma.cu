// Fast decode kernel for the common shapes (placeholder until the tensor-core
// path lands): reports "not handled" so the generic kernel runs.
#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

int launch_gqa_decode_fast(const AttendArgs &a, cudaStream_t stream, bool *handled) {
    (void)a;
    (void)stream;
    *handled = false;
    return SA_OK;
}

}  // namespace sa
