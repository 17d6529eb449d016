// Device helpers shared by the tensor-core decode kernels: inline PTX
// (byte permutes, fp16x2 arithmetic, mbarriers, 1-D bulk async copies) and the
// walk over the (sequence, KV head, item) space that both kernels split into
// contiguous per-warp slices.
#pragma once

#include "kitty_common.cuh"

namespace kitty {
namespace dev {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t pack_f32x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// Packed fp32 pairs (two lanes of work per instruction, IEEE round-to-nearest
// like the scalar forms).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~2^22 polls (seconds), never spins forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ uint32_t pack16(uint32_t lo, uint32_t hi) { return lo | (hi << 16); }

// ---- segment walk -----------------------------------------------------------
//
// Segment (b, h) has L_b = num_pages[b] + 1 items: item 0 is the fp16 region
// (sinks then tail), items 1..n are the quantised pages in block-table order.

struct SegmentScan {
  int64_t total;     // items over all segments
  int64_t seg_begin; // for the located item: start of its segment
  int b, h, p;       // located item: sequence, KV head, item index in the segment
};

// Warp-cooperative: total item count and the (b, h, p) of item f (when f < total).
// Segment (b, h) has L_b = num_pages[b] + 1 items; sequence b's segments start at
// H * sum_{b' < b} L_b'.
__device__ inline SegmentScan scan_segments(const int32_t* num_pages, int B, int H, int64_t f, int lane) {
  SegmentScan r;
  r.b = -1; r.h = 0; r.p = 0; r.seg_begin = 0;
  int64_t run = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int64_t seq_items = (b < B) ? int64_t(H) * (int64_t(max(num_pages[b], 0)) + 1) : 0;
    int64_t incl = seq_items;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int64_t start = run + incl - seq_items;
    const bool hit = (b < B) && (f >= start) && (f < start + seq_items);
    const uint32_t bal = __ballot_sync(0xffffffffu, hit);
    if (bal != 0u && r.b < 0) {
      const int src = __ffs(bal) - 1;
      const int64_t st = __shfl_sync(0xffffffffu, start, src);
      const int bb = b0 + src;
      const int64_t L = int64_t(max(num_pages[bb], 0)) + 1;
      r.b = bb;
      r.h = int((f - st) / L);
      r.p = int((f - st) - int64_t(r.h) * L);
      r.seg_begin = st + int64_t(r.h) * L;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  r.total = run;
  return r;
}

// Producer cursor over the real pages of a warp's slice.
struct Cursor {
  int64_t f;   // item index
  int b, h, p; // sequence, KV head, item in segment (p >= 1: page p - 1)
};

__device__ __forceinline__ void cursor_step(Cursor& c, const int32_t* num_pages, int H) {
  ++c.f; ++c.p;
  if (c.p >= num_pages[c.b] + 1) { c.p = 0; if (++c.h == H) { c.h = 0; ++c.b; } }
}

// advance to the next real page in [c.f, end); false if none
__device__ __forceinline__ bool cursor_to_page(Cursor& c, const int32_t* num_pages, int H, int64_t end) {
  while (c.f < end) {
    if (c.p >= 1) return true;
    cursor_step(c, num_pages, H);
  }
  return false;
}

}  // namespace dev
}  // namespace kitty
