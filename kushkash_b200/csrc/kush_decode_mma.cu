// Tensor-core decode kernel (placeholder until the mma kernel lands): no configuration selects it yet.
#include "kush_common.cuh"

namespace kush {

int decode_mma_supported(int, int, int, int, int) { return 0; }

int launch_decode_mma(int, int, int, int, int, const void*, void*, const void*, int64_t, int64_t, const void*,
                      const int32_t*, const int32_t*, const int32_t*, int64_t, int32_t, float, int32_t, float*, float*,
                      int32_t, cudaStream_t) {
    return set_error(KUSH_ERR_UNSUPPORTED, "tensor-core decode not built");
}

}  // namespace kush
