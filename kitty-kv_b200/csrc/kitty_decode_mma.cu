// Tensor-core decode variant (placeholder until the mma path lands).
#include "kitty_decode.cuh"

namespace kitty {

bool mma_supports(const KittyDecodeArgs&) { return false; }
int mma_ctas_per_sm() { return 2; }
int launch_decode_mma(const KittyDecodeArgs&, const DecodePlan&, cudaStream_t) {
  return fail(KITTY_ERR_UNSUPPORTED, "tensor-core decode not built");
}

}  // namespace kitty
