// Internal interface between the decode dispatcher and the decode kernels.
#pragma once

#include "kitty_common.cuh"

namespace kitty {

// How one kitty_paged_decode call is split over the GPU.  Split s of a
// sequence covers its pages [s*pages_per_split, (s+1)*pages_per_split); split 0
// also covers the fp16 sinks and tail.  With num_splits == 1 the decode kernel
// writes the final output itself and no workspace is used.
struct DecodePlan {
  int num_splits;
  int pages_per_split;
  int variant;        // 0 = CUDA-core (any shape), 1 = tensor-core (D = G = 128)
  float* ws_m;        // [B][H][S][g] running max per split
  float* ws_l;        // [B][H][S][g] running sum per split
  float* ws_o;        // [B][H][S][g][D] unnormalised accumulator per split
};

int launch_decode_simt(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
int launch_decode_mma(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
int launch_decode_merge(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
bool simt_supports(const KittyDecodeArgs& a);
bool mma_supports(const KittyDecodeArgs& a);
int mma_ctas_per_sm();
int read_decode_error(uint32_t* flags, int clear);

}  // namespace kitty
