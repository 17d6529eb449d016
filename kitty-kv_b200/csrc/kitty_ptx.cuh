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
// 2^x for the softmax weights (x <= 0).  The .ftz form is a single instruction; results
// below 2^-126 become 0, far below anything a weight contributes next to the row maximum.
__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// approximate 1/x (x a normal float), single instruction
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
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

// Fetch the 128-byte line holding p into L1 (plain load-path prefetch).
__device__ __forceinline__ void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" :: "l"(p)); }

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ uint32_t pack16(uint32_t lo, uint32_t hi) { return lo | (hi << 16); }

// ---- segment walk -----------------------------------------------------------
//
// Segment (b, h) has n16_b + num_pages[row of b] items: items 0 .. n16_b - 1 are
// chunks of its fp16 region (sinks then tail, at most kMaxFp16Items chunks of
// about the same length, at least one item even when the region is empty), items
// n16_b .. are the quantised pages in block-table order.  Splitting the fp16 region
// lets several warps share it.
//
// Warps split the walk by cost units, not items: a page is one unit and an fp16
// chunk w16 units (w16 = 1 makes units and items the same).  A chunk item costs a
// warp several pages' time (row loads from the fp16 buffers, one round trip per
// 16-token tile), so counting it as one unit would leave the warps whose slice
// holds segment starts running well after the others.  Item p of a segment starts
// at unit w16 * p (p < n16) or w16 * n16 + (p - n16); a warp takes the items whose
// first unit lies in its slice of the unit range.

constexpr int kFp16ChunkTokens = 32;   // a chunk item covers at least this many tokens
constexpr int kMaxFp16Items = 4;

// cache row of batch row b (KittyDecodeArgs::seq_map)
__device__ __forceinline__ int cache_row(const KittyDecodeArgs& a, int b) { return a.seq_map ? a.seq_map[b] : b; }

// fp16 tokens (sinks + tail) of cache row s
__device__ __forceinline__ int fp16_tokens(const KittyDecodeArgs& a, int s) {
  return max(a.sink_len ? a.sink_len[s] : a.sink_len_all, 0) + max(a.tail_len ? a.tail_len[s] : a.tail_len_all, 0);
}
__device__ __forceinline__ int fp16_items(int tokens) {
  return tokens <= kFp16ChunkTokens ? 1 : min(kMaxFp16Items, (tokens + kFp16ChunkTokens - 1) / kFp16ChunkTokens);
}
// items of the segments of cache row s; n16 receives its fp16 items
__device__ __forceinline__ int seg_items(const KittyDecodeArgs& a, int s, int& n16) {
  n16 = fp16_items(fp16_tokens(a, s));
  return n16 + max(a.num_pages[s], 0);
}
// units of a segment with `items` items of which n16 are fp16 chunks
__device__ __forceinline__ int seg_units(int items, int n16, int w16) { return items + (w16 - 1) * n16; }
// tokens [t0, t1) of fp16 chunk c of a region of `tokens` tokens split into n16 chunks
__device__ __forceinline__ void fp16_chunk(int tokens, int n16, int c, int& t0, int& t1) {
  const int len = (tokens + n16 - 1) / n16;
  t0 = min(tokens, c * len);
  t1 = min(tokens, t0 + len);
}

struct SegmentScan {
  int64_t total;     // units over all segments
  int64_t seg_begin; // for the located unit: first unit of its segment
  int b, h;          // located unit: sequence, KV head
  int u;             // unit offset inside the segment
};

// Warp-cooperative: total unit count and the segment (b, h) holding unit f (when
// f < total).  Sequence b's segments start at H * sum_{b' < b} U_b'.
__device__ inline SegmentScan scan_segments(const KittyDecodeArgs& a, int B, int H, int64_t f, int lane, int w16 = 1) {
  SegmentScan r;
  r.b = -1; r.h = 0; r.u = 0; r.seg_begin = 0;
  int64_t run = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    int n16 = 0;
    const int64_t L = (b < B) ? seg_units(seg_items(a, cache_row(a, b), n16), n16, w16) : 0;
    const int64_t seq_units = int64_t(H) * L;
    int64_t incl = seq_units;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int64_t start = run + incl - seq_units;
    const bool hit = (b < B) && (f >= start) && (f < start + seq_units);
    const uint32_t bal = __ballot_sync(0xffffffffu, hit);
    if (bal != 0u && r.b < 0) {
      const int src = __ffs(bal) - 1;
      const int64_t st = __shfl_sync(0xffffffffu, start, src);
      const int64_t Ls = __shfl_sync(0xffffffffu, L, src);
      r.b = b0 + src;
      r.h = int((f - st) / Ls);
      r.u = int((f - st) - int64_t(r.h) * Ls);
      r.seg_begin = st + int64_t(r.h) * Ls;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  r.total = run;
  return r;
}

// Walk over a warp's slice (items, segments); used for the consumer position and for
// the producer cursor that runs ahead over the real pages.
struct Cursor {
  int64_t f;      // first unit of the current item
  int b, h, p;    // sequence (batch row), KV head, item in segment
  int s;          // cache row of b
  int n16, items; // fp16 items and all items of the current segment
};

// units the current item spans
__device__ __forceinline__ int cursor_width(const Cursor& c, int w16) { return c.p < c.n16 ? w16 : 1; }

// first item of the next segment (f already at that segment's first unit); false past
// the last segment
__device__ __forceinline__ bool cursor_next_segment(Cursor& c, const KittyDecodeArgs& a) {
  c.p = 0;
  if (++c.h == a.num_kv_heads) {
    c.h = 0;
    if (++c.b >= a.batch) return false;
    c.s = cache_row(a, c.b);
  }
  c.items = seg_items(a, c.s, c.n16);
  return true;
}

// Cursor at the first item of segment (b, h) whose first unit is >= seg_begin + u
// (the next segment's first item if none); false if there is none at all.
__device__ __forceinline__ bool make_cursor(Cursor& c, const KittyDecodeArgs& a, int64_t seg_begin, int b, int h,
                                            int u, int w16 = 1) {
  c.b = b; c.h = h;
  c.s = cache_row(a, b);
  c.items = seg_items(a, c.s, c.n16);
  const int fp = w16 * c.n16;
  c.p = u <= fp ? (u + w16 - 1) / w16 : c.n16 + (u - fp);
  c.f = seg_begin + (c.p <= c.n16 ? int64_t(w16) * c.p : int64_t(fp) + (c.p - c.n16));
  if (c.p < c.items) return true;
  c.f = seg_begin + seg_units(c.items, c.n16, w16);
  return cursor_next_segment(c, a);
}

// next item; false past the last segment
__device__ __forceinline__ bool cursor_step(Cursor& c, const KittyDecodeArgs& a, int w16 = 1) {
  c.f += cursor_width(c, w16);
  if (++c.p >= c.items) return cursor_next_segment(c, a);
  return true;
}

// advance to the next real page starting in [c.f, end); false if none
__device__ __forceinline__ bool cursor_to_page(Cursor& c, const KittyDecodeArgs& a, int64_t end, int w16 = 1) {
  while (c.f < end) {
    if (c.p >= c.n16) return true;
    if (!cursor_step(c, a, w16)) return false;
  }
  return false;
}

}  // namespace dev
}  // namespace kitty
