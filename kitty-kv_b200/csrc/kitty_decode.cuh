// Internal interface between the decode dispatcher and the decode kernels.
#pragma once

#include "kitty_common.cuh"

namespace kitty {

// How one kitty_paged_decode call is split over the GPU.  Split s of a
// sequence covers its pages [s*pages_per_split, (s+1)*pages_per_split); split 0
// also covers the fp16 sinks and tail.  With num_splits == 1 the decode kernel
// writes the final output itself and no workspace is used.
//
// The tensor-core variants use the fields differently: every warp walks a
// contiguous slice of the (sequence, KV head, item) space and writes one
// partial per (sequence, KV head) it touches; num_splits is then the number of
// partial slots per (sequence, KV head), pages_per_split the minimum slice
// length, grid the persistent grid size, and ws_count[b][h] receives the number
// of slots written.
struct DecodePlan {
  int num_splits;
  int pages_per_split;
  int variant;        // 0 = CUDA-core (any shape), 2 = integer mma.sync (D = G = 128, g <= 8),
                      // 3 = integer tcgen05 / tensor memory (D = G = 128, g <= 8, pages only)
  int grid;           // tensor-core variant: CTAs of the persistent grid
  int qh_base;        // integer mma.sync variant in passes: first query head (of each KV head's
  int g_pass;         //   group) this launch covers, and how many (0: all g = Hq / H)
  float* ws_m;        // [B][H][S][g] running max per split (natural log units)
  float* ws_l;        // [B][H][S][g] running sum per split
  float* ws_o;        // [B][H][S][g][D] unnormalised accumulator per split
  int* ws_count;      // [B][H] slots written (tensor-core variant), else nullptr
};

// Most partial slots the merge kernel combines per (sequence, KV head).
constexpr int kMaxDecodeSlots = 1024;

int launch_decode_simt(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
int launch_decode_merge(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
bool simt_supports(const KittyDecodeArgs& a);
int launch_decode_i8(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
bool i8_supports(const KittyDecodeArgs& a);
int i8_ctas_per_sm();
void i8_plan(const KittyDecodeArgs& a, int sm_count, DecodePlan* plan);
// query heads per KV head one integer-kernel launch handles (more run in passes)
constexpr int kI8MaxHeadsPerPass = 8;
int read_decode_error_i8(uint32_t* flags, int clear);
int launch_decode_tc(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream);
bool tc_supports(const KittyDecodeArgs& a);
void tc_plan(const KittyDecodeArgs& a, int sm_count, DecodePlan* plan);
int read_decode_error_tc(uint32_t* flags, int clear);

}  // namespace kitty
