// Paged GQA decode attention with integer tensor-core contractions
// (head_dim = group = 128; up to 8 query heads per KV head per launch, more in
// passes of 8 that share the workspace).
//
// Work decomposition: segments (sequence, KV head) of items (the fp16 sinks + tail
// in up to four chunk items, then the quantised pages), one contiguous slice of
// cost units per warp, one partial result per touched segment, per-warp key and
// value buffers filled by 1-D bulk async copies on bounded mbarrier waits.
//
// Arithmetic of a page-head.  The 2-bit codes stay
// integers: one AND per register extracts four codes into the bytes of an
// 8-bit MMA operand (mma.sync.m16n8k32, u8 x u8 -> s32), and the other operand
// carries the folded scales in fixed point:
//
//   keys    w[qh][c] = q[qh][c] * scale_k[c]           (exact in fp32)
//           x[qh][c] = rint(w * R),  R = (2^22 - 4) / max_c |w|
//           x is split into bytes: x = 65536 (b2 - 64) + 256 b1 + b0 (b0, b1, b2
//           unsigned), so  sum_c code * x = 65536 (S[b2] - 64 S[1]) + 256 S[b1] + S[b0]
//           where S[d] is the MMA sum against digit plane d and S[1] the code sum
//           (an all-ones operand).  Scores = (sum_c code * x) / R - sum_c zp_k w,
//           i.e. 23 significant bits per product (16 bits moved the logits by up
//           to ~1e-3, too much next to the value outliers).
//   values  P'[qh][t] = p[qh][t] * scale_v[t]           (fp32)
//           y[qh][t] = rint(P' * Rv), Rv = 65535 / max_t P'   (two unsigned digits)
//           O[c][qh] += (sum_t code_v * y - sum_t zp_v * y) / Rv
//           (the zero-point sum uses the same rounded y, so (code - zp) is
//           weighted consistently).
//
// Per MMA the 8 columns are 4 query heads x 2 digits (hi, lo), so one lane holds
// both digits of the same (token, query head) and combines them with one
// integer multiply-add: no exchange between lanes, and after the key
// contraction lane (g_, q_) owns the 16 scores of query head q_ for the tokens
// 32 k + 4 g_ + i (k, i = 0..3; the same 16 channels of the value accumulator).
// With 8 query heads (two groups of 4 per lane: q_ and q_ + 4) the top key digit
// is stored signed, b2 - 64 (u8 x s8 MMA), which makes the all-ones column
// unnecessary: one MMA per code plane then holds the b2 sums of both groups, its
// column g_ carrying query head (g_ >> 1) + 4 (g_ & 1) so that a lane receives
// those of its own two heads (3 key MMAs per plane and half instead of 4).
//
// Operand layout.  Both planes are stored with the packed dimension along a row
// (key row = channel, 4 tokens per byte; value row = token, 4 channels per byte)
// while the contraction runs along the rows, so a k-step loads 32 rows as two
// transposed 16 x 16 byte matrices per half (ldmatrix .trans .b8): each lane gets,
// for two row-bytes j, the bytes of 4 consecutive rows, and masking bit pair i of
// every byte gives the A operand of element 4 j + i of those rows, scaled by 4^i.
// The scale is removed per tile in the fp32 epilogue.  Keys use the factors
// (1, 4, 16, 16) for i = 0..3 (i = 3 shifted down by two bits) so that the
// boosted high plane can reuse the same accumulators with its factor 4 built into
// the masks ((4, 16, 64, 64) * high code).  The fixed-point digit tables are
// stored in natural K order with row and plane strides that keep their lane
// loads on distinct banks.
//
// Reference semantics: (code - zp) * scale from kitty/kernels/dequantize_key.py:89-95
// and kitty/kernels/quantize_value.py:121-133; softmax over [sinks ; pages ;
// tail] as in kitty/kernels/attention.py:172-189.

#include <algorithm>

#include "kitty_decode.cuh"
#include "kitty_ptx.cuh"

namespace kitty {

__device__ unsigned int g_decode_error_i8 = 0;  // bit 0: a bulk-copy wait timed out

namespace {

using namespace dev;

// Resident warps per SM: 12 (<= 170 registers), as one CTA: warps of one CTA share a
// scheduling age, while with three CTAs of four the oldest CTA's warps won the issue
// slots and finished well before the youngest, which then set the kernel's end (4 query
// heads per KV head, config 2: 1.5 % slower; 8 heads, config 4: 1.5 % slower, and two
// CTAs of six 3 % slower).  With 8 query heads the 168-register cap costs a few spills
// but 12 warps still beat 8 warps at 245 registers by 5 %.  A CTA whose warps' shared
// memory exceeds the per-CTA limit (8 heads with many boosted channels) is launched
// with fewer warps (the kernel reads its warp count from blockDim).
#ifndef KITTY_I8_W1
#define KITTY_I8_W1 12
#endif
#ifndef KITTY_I8_W2
#define KITTY_I8_W2 12
#endif
#ifndef KITTY_I8_C2
#define KITTY_I8_C2 1
#endif
template <int kQG>
__host__ __device__ constexpr int warps_per_cta() { return kQG == 1 ? KITTY_I8_W1 : KITTY_I8_W2; }
template <int kQG>
__host__ __device__ constexpr int ctas_per_sm() { return kQG == 1 ? 1 : KITTY_I8_C2; }
constexpr int kD = 128, kG = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kSlotsTarget = 16;
// cost units of one fp16 chunk item in the warps' slicing of the walk (a page is one
// unit); chunk items cost a warp a few pages' time
constexpr int kFp16Weight = 2;
constexpr float kKeyRange = 4194300.0f;     // 2^22 - 4: |x| < 2^22 even with an approximate reciprocal
constexpr float kValRange = 65535.0f;
constexpr float kMagicKey = 12582912.0f;    // 1.5 * 2^23: fma(w, R, magic) has bits 0x4B400000 + rint(w R)
constexpr float kMagicVal = 8388608.0f;     // 2^23: fma(P', Rv, magic) has bits 0x4B000000 + rint(P' Rv)
constexpr int kRow = 160;                   // digit table: query-head row stride (bytes; 40 words = 8 mod 32)
// digit table plane stride for 4 (8) query-head rows: 164 (324) words = 4 mod 32 banks
__host__ __device__ constexpr int plane_bytes(int qg) { return qg == 1 ? 656 : 1296; }
constexpr int kPhRow = 136;                 // fp16 P staging (fp16 region): row stride in halves

// per-warp shared memory (bytes)
struct Layout {
  int kbuf, vbuf, dtab, ptab, ent, qs, bars, size, plane;
};
// qg = groups of four query heads per KV head (1: g <= 4, 2: g <= 8)
__host__ __device__ inline Layout i8_layout(int K, int qg) {
  Layout L;
  L.plane = plane_bytes(qg);
  int o = 0;
  L.kbuf = o; o += (4096 + 512 + K * 32 + 32 + 127) & ~127;  // low plane, scale/zero rows, high plane, zero row
  L.vbuf = o; o += 4096 + 512;                               // codes, (scale, zero) per token
  L.dtab = o; o += 3 * L.plane;                              // key digits b0, b1, b2 [qh][channel]
  L.ptab = o; o += 2 * L.plane;                              // P' digits y0, y1 [qh][token] / fp16 P (fp16 region)
  L.ent = o;  o += 128 * 4;                                  // boosted entries (row offset | position << 16)
  L.qs = o;   o += 1024 * qg;                                // q of the prep lanes [qg][half][lane] (16 B each)
  L.bars = o; o += 16;
  L.size = (o + 127) & ~127;
  return L;
}

// ---- integer MMA and operand helpers -----------------------------------------

__device__ __forceinline__ void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// first k-step of an accumulation: C = 0 (no accumulator initialisation)
__device__ __forceinline__ void mma_k32_z(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
template <bool kFirst>
__device__ __forceinline__ void mma_k32_acc(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  if (kFirst) mma_k32_z(c, a0, a1, a2, a3, b0, b1);
  else mma_k32(c, a0, a1, a2, a3, b0, b1);
}
__device__ __forceinline__ void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}
// A unsigned, B signed (the signed top key digit)
template <bool kFirst>
__device__ __forceinline__ void mma_k32s(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if (kFirst)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_k16s(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <bool kBf16>
__device__ __forceinline__ void mma_h16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  if (kBf16) mma_bf16(c, a0, a1, a2, a3, b0, b1);
  else mma_f16(c, a0, a1, a2, a3, b0, b1);
}
// exact product of two 16-bit floats in fp32 (11- or 8-bit significands)
template <bool kBf16>
__device__ __forceinline__ float mul_h16_f32(uint16_t a, uint16_t b) {
  if (kBf16) return Half16<true>::to_f(a) * Half16<true>::to_f(b);
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(0.0f));
  return d;
}
// Two transposed 16 x 16 byte matrices (rows from the addresses of lanes 0-15 and
// 16-31): r[0] / r[1] = bytes 4 q_ .. 4 q_ + 3 of column g_ / g_ + 8 of the first
// matrix, r[2] / r[3] the same of the second, i.e. the A operand of an m16n8k32
// MMA whose K index is the matrix row.  The rows are written by bulk copies that
// completed on an mbarrier wait (volatile keeps the load after it).
__device__ __forceinline__ void ldsm_t_x2(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// code i of every byte of t, times the row factor (see the header comment)
template <int i>
__device__ __forceinline__ uint32_t high_code(uint32_t t) {   // 4 * key_code factor
  return i < 3 ? ((t << 2) & (0x0C0C0C0Cu << (2 * i))) : (t & 0xC0C0C0C0u);
}
// the same with the code index as an argument (a constant after unrolling)
__device__ __forceinline__ uint32_t high_code_of(int i, uint32_t t) {
  return i < 3 ? ((t << 2) & (0x0C0C0C0Cu << (2 * i))) : (t & 0xC0C0C0C0u);
}
// bytes k of v0..v3 packed into one word
__device__ __forceinline__ void bytes01(uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3, uint32_t& w0,
                                        uint32_t& w1) {
  const uint32_t a = prmt(v0, v1, 0x5140u), b = prmt(v2, v3, 0x5140u);
  w0 = prmt(a, b, 0x5410u);
  w1 = prmt(a, b, 0x7632u);
}
__device__ __forceinline__ uint32_t byte2(uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3) {
  return prmt(prmt(v0, v1, 0x0062u), prmt(v2, v3, 0x0062u), 0x5410u);
}

// Top key digits b2 in [0, 128) (offset binary: the digit value is b2 - 64) as signed
// bytes b2 - 64: flip bit 6 and copy the flipped bit 6 into bit 7, byte by byte.
__device__ __forceinline__ uint32_t signed_top_digits(uint32_t b2) {
  const uint32_t t = b2 ^ 0x40404040u;
  return t | ((t & 0x40404040u) << 1);
}

// One 32-channel k-step of the key baseline plane (K index = channel 32 ks + k) into
// the 8 token tiles: tile 4 half + i, row r <-> token byte 16 half + r, code i, i.e.
// token 64 half + 4 r + i.  lane_row = smem address of row 32 ks + lane of the plane.
template <bool kFirst>
__device__ __forceinline__ void key_kstep(int (&acc1)[8][4], int (&acc2)[8][4], uint32_t lane_row,
                                          const uint8_t* kb1, const uint8_t* kb2, bool ones, int ks, int q_) {
  const uint32_t b10 = lds32(kb1 + 32 * ks + 4 * q_), b11 = lds32(kb1 + 32 * ks + 16 + 4 * q_);
  const uint32_t b20 = ones ? 0x01010101u : lds32(kb2 + 32 * ks + 4 * q_);
  const uint32_t b21 = ones ? 0x01010101u : lds32(kb2 + 32 * ks + 16 + 4 * q_);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t r[4];
    ldsm_t_x2(lane_row + 16 * half, r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // code i scaled by (1, 4, 16, 16)
      const uint32_t m = i < 3 ? (0x03030303u << (2 * i)) : 0x30303030u;
      const int sh = i < 3 ? 0 : 2;
      const uint32_t c0 = (r[0] >> sh) & m, c1 = (r[1] >> sh) & m, c2 = (r[2] >> sh) & m, c3 = (r[3] >> sh) & m;
      mma_k32_acc<kFirst>(acc1[4 * half + i], c0, c1, c2, c3, b10, b11);
      mma_k32_acc<kFirst>(acc2[4 * half + i], c0, c1, c2, c3, b20, b21);
    }
  }
}

// One 32-token k-step of the value plane (K index = token 32 ks + k) into the 8 channel
// tiles: tile 4 half + i, row r <-> channel 64 half + 4 r + i.
template <bool kFirst>
__device__ __forceinline__ void val_kstep(int (&acc)[8][4], uint32_t lane_row, const uint8_t* vb, int ks, int q_) {
  const uint32_t b0 = lds32(vb + 32 * ks + 4 * q_), b1 = lds32(vb + 32 * ks + 16 + 4 * q_);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t r[4];
    ldsm_t_x2(lane_row + 16 * half, r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t m = 0x03030303u << (2 * i);
      mma_k32_acc<kFirst>(acc[4 * half + i], r[0] & m, r[1] & m, r[2] & m, r[3] & m, b0, b1);
    }
  }
}

struct State {
  float o[16];   // unnormalised accumulator, channels 16 g_ + v, query head q_
  float m;       // running max (log2 domain)
  float l;       // running sum over this lane's tokens
  float zs;      // value zero-point sums over this lane's tokens (already divided by Rv)
};

__device__ __forceinline__ void reset_state(State& st) {
#pragma unroll
  for (int v = 0; v < 16; ++v) st.o[v] = 0.f;
  st.m = -INFINITY;
  st.l = 0.f;
  st.zs = 0.f;
}

// Online-softmax step over the lane's 16 scores (log2 domain; -inf = masked).
// Returns p in s.
// three-input maximum (sm_100 form of max.f32)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float max16(const float (&x)[16], float init) {
  return fmax3(fmax3(fmax3(x[0], x[1], x[2]), fmax3(x[3], x[4], x[5]), fmax3(x[6], x[7], x[8])),
               fmax3(x[9], x[10], x[11]), fmax3(fmax3(x[12], x[13], x[14]), x[15], init));
}
__device__ __forceinline__ void softmax_step(State& st, float (&s)[16]) {
  float mx = max16(s, -INFINITY);
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
  const float mn = fmaxf(st.m, mx);
  const bool moved = mn > st.m;   // false while the running max holds (and for -inf == -inf)
  const float alpha = (st.m == -INFINITY) ? 0.f : ex2(st.m - mn);
  // a fully masked chunk before any real token keeps everything at zero
  const float base = (mn == -INFINITY) ? 0.f : mn;
  st.m = mn;
  float2 sum = make_float2(0.f, 0.f);
#pragma unroll
  for (int v = 0; v < 16; v += 2) {
    const float2 d = add2(make_float2(s[v], s[v + 1]), make_float2(-base, -base));
    s[v] = ex2(d.x);
    s[v + 1] = ex2(d.y);
    sum = add2(sum, make_float2(s[v], s[v + 1]));
  }
  // once the running maxima settle, no lane rescales: skip the accumulator update
  if (__any_sync(0xffffffffu, moved)) {
    st.l *= alpha;
    st.zs *= alpha;
#pragma unroll
    for (int v = 0; v < 16; v += 2) {
      const float2 o = mul2(make_float2(st.o[v], st.o[v + 1]), make_float2(alpha, alpha));
      st.o[v] = o.x;
      st.o[v + 1] = o.y;
    }
  }
  st.l += sum.x + sum.y;
}

// Per-segment setup: q of the prep lane's (query heads pq + 4 qg, 16 channels), kept in
// shared memory rather than registers (read once per page by the digit step), and the
// boosted-entry table.  Returns the number of boosted entries.
template <int kQG>
__device__ int setup_segment(const KittyDecodeArgs& a, int b, int h, int g, int g_all, int qb, uint8_t* wsm,
                             const Layout& L, int lane) {
  const int pq = lane >> 3, cb = lane & 7;
#pragma unroll
  for (int qg = 0; qg < kQG; ++qg) {
    uint4 x0 = make_uint4(0u, 0u, 0u, 0u), x1 = x0;
    if (pq + 4 * qg < g) {
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.q) + b * a.q_s_seq +
                                                        int64_t(h * g_all + qb + pq + 4 * qg) * a.q_s_head + 16 * cb);
      x0 = src[0];
      x1 = src[1];
    }
    uint4* qs = reinterpret_cast<uint4*>(wsm + L.qs + 1024 * qg);
    qs[lane] = x0;
    qs[32 + lane] = x1;
  }
  uint32_t* ent = reinterpret_cast<uint32_t*>(wsm + L.ent);
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  const uint32_t zero_row = uint32_t(a.d_boost) * 32u;
  int nb = 0;
  for (int c0 = 0; c0 < kD; c0 += 32) {
    const int c = c0 + lane;
    const int r = bidx[c];
    const bool boosted = r < a.d_boost;
    const uint32_t bal = __ballot_sync(0xffffffffu, boosted);
    if (boosted) ent[nb + __popc(bal & ((1u << lane) - 1u))] = uint32_t(r) * 32u | (uint32_t(c) << 16);
    nb += __popc(bal);
  }
  // pad to a multiple of 16 entries with the zero row
  const int padded = (nb + 15) & ~15;
  if (nb + lane < padded) ent[nb + lane] = zero_row;
  __syncwarp();
  return nb;
}

// Query heads qoff .. qoff + 3, tokens [t_begin, t_end) of the fp16 region of (b, h) (sinks then tail; one chunk
// item of the segment walk), at most 128 per pass (fp16 MMAs; 16-token tiles without
// real tokens are skipped).  Scores: token 16 m + g_ + 8 hh <-> row g_ + 8 hh of M tile
// m; values: channel 32 (m >> 1) + 4 g_ + 2 (m & 1) + hh <-> row g_ + 8 hh of M tile m
// (the channels of st.o[2 m + hh], as on the page path).
template <bool kBf16>
__device__ void process_fp16_region(const KittyDecodeArgs& a, int b, int h, int g, int qoff, State& st,
                                    uint8_t* wsm, const Layout& L, float qk_scale, int lane, int t_begin,
                                    int t_end) {
  const int cr = cache_row(a, b);   // cache row (sinks, tail, lengths)
  const int g_ = lane >> 2, q_ = lane & 3;
  const int sink_len = a.sink_len ? a.sink_len[cr] : a.sink_len_all;
  const int tail_len = a.tail_len ? a.tail_len[cr] : a.tail_len_all;
  if (t_end <= t_begin || sink_len + tail_len <= 0) return;
  __half* ph = reinterpret_cast<__half*>(wsm + L.ptab);
  // q of query head g_ >> 1 (B column g_), channels 32 q_ .. 32 q_ + 31: the K
  // index (2q_, 2q_+1, 2q_+8, 2q_+9) of k-step s <-> channel 32 q_ + 4 s + (0..3)
  // from the segment's q copy in shared memory (setup_segment: [group][half][prep lane], prep
  // lane 8 head + channel block; zeros past the last query head)
  uint32_t qw[16];
  {
    const uint4* qs = reinterpret_cast<const uint4*>(wsm + L.qs + 1024 * (qoff >> 2));
    const int l0 = 8 * (g_ >> 1) + 2 * q_;   // channels 32 q_ .. 32 q_ + 15 (block 2 q_), then block 2 q_ + 1
    const uint4 x0 = qs[l0], x1 = qs[32 + l0], x2 = qs[l0 + 1], x3 = qs[32 + l0 + 1];
    const uint4 xs[4] = {x0, x1, x2, x3};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      qw[4 * i] = xs[i].x; qw[4 * i + 1] = xs[i].y; qw[4 * i + 2] = xs[i].z; qw[4 * i + 3] = xs[i].w;
    }
  }
  for (int f0 = t_begin; f0 < t_end; f0 += kG) {
    const int ntok = min(kG, t_end - f0);
    const int tiles = (ntok + 15) >> 4;   // 16-token tiles holding real tokens (warp-uniform)
    auto row = [&](bool key, int t) -> const uint16_t* {   // row of chunk token t (t < ntok)
      const int ft = f0 + t;
      if (ft < sink_len) {
        return key ? reinterpret_cast<const uint16_t*>(a.sink_k) + cr * a.sk_s_seq + h * a.sk_s_head + ft * a.sk_s_tok
                   : reinterpret_cast<const uint16_t*>(a.sink_v) + cr * a.sv_s_seq + h * a.sv_s_head + ft * a.sv_s_tok;
      }
      const int tt = ft - sink_len;
      return key ? reinterpret_cast<const uint16_t*>(a.tail_k) + cr * a.tk_s_seq + h * a.tk_s_head + tt * a.tk_s_tok
                 : reinterpret_cast<const uint16_t*>(a.tail_v) + cr * a.tv_s_seq + h * a.tv_s_head + tt * a.tv_s_tok;
    };
    // every key and value row of this pass into L1 first (two 128-byte lines per row, one
    // line per lane and request): the tile loads below then wait on one round trip, not one
    // per tile
    for (int i = lane; i < 2 * ntok; i += 32) {
      prefetch_l1(row(true, i >> 1) + 64 * (i & 1));
      prefetch_l1(row(false, i >> 1) + 64 * (i & 1));
    }
    // scores: tile m rows g_ / g_ + 8 <-> tokens 16 m + g_ / 16 m + g_ + 8 (s[2 m], s[2 m + 1])
    float s[16];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      s[2 * m] = s[2 * m + 1] = -INFINITY;
      if (m < tiles) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int ta = 16 * m + g_, tb = ta + 8;
        uint4 ka[4], kb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) { ka[i] = make_uint4(0, 0, 0, 0); kb[i] = ka[i]; }
        if (ta < ntok) {
          const uint4* r = reinterpret_cast<const uint4*>(row(true, ta) + 32 * q_);
#pragma unroll
          for (int i = 0; i < 4; ++i) ka[i] = r[i];
        }
        if (tb < ntok) {
          const uint4* r = reinterpret_cast<const uint4*>(row(true, tb) + 32 * q_);
#pragma unroll
          for (int i = 0; i < 4; ++i) kb[i] = r[i];
        }
        const uint32_t* wa = reinterpret_cast<const uint32_t*>(ka);
        const uint32_t* wb = reinterpret_cast<const uint32_t*>(kb);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_h16<kBf16>(acc, wa[2 * k], wb[2 * k], wa[2 * k + 1], wb[2 * k + 1], qw[2 * k], qw[2 * k + 1]);
        if (ta < ntok) s[2 * m] = acc[0] * qk_scale;
        if (tb < ntok) s[2 * m + 1] = acc[2] * qk_scale;
      }
    }
    softmax_step(st, s);
    // P (scale 1) as fp16 [query head q_][token]; tokens past ntok hold zeros.  For bf16
    // values P is carried as two bf16 parts (hi + lo, 16 significant bits), the lo part in
    // the key digit table (unused on this path)
    {
      uint16_t* prow = reinterpret_cast<uint16_t*>(ph) + q_ * kPhRow;
      uint16_t* plo = reinterpret_cast<uint16_t*>(wsm + L.dtab) + q_ * kPhRow;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const int t = 16 * (m >> 1) + g_ + 8 * (m & 1);
        const float p = s[m];
        if (kBf16) {
          const __nv_bfloat16 hi = __float2bfloat16_rn(p);
          prow[t] = __bfloat16_as_ushort(hi);
          plo[t] = __bfloat16_as_ushort(__float2bfloat16_rn(p - __bfloat162float(hi)));
        } else {
          prow[t] = __half_as_ushort(__float2half_rn(p));
        }
      }
    }
    __syncwarp();
    // values: M = channel pairs (word m of the lane's 8 words), K = tokens 16 k + (2q_,
    // 2q_+1, 2q_+8, 2q_+9)
    float oacc[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m) oacc[m][0] = oacc[m][1] = oacc[m][2] = oacc[m][3] = 0.f;
    const __half* pb = ph + (g_ >> 1) * kPhRow;
    const __half* pbl = reinterpret_cast<const __half*>(wsm + L.dtab) + (g_ >> 1) * kPhRow;
#pragma unroll 1
    for (int k = 0; k < tiles; ++k) {
      uint2 v[4][4];   // token e, channels 32 j + 4 g_ .. + 3
      const int t0 = 16 * k + 2 * q_;
      const int ts[4] = {t0, t0 + 1, t0 + 8, t0 + 9};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (ts[e] < ntok) {
          const uint16_t* r = row(false, ts[e]) + 4 * g_;
#pragma unroll
          for (int j = 0; j < 4; ++j) v[e][j] = *reinterpret_cast<const uint2*>(r + 32 * j);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) v[e][j] = make_uint2(0, 0);
        }
      }
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(pb + t0);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(pb + t0 + 8);
      const uint32_t b0l = kBf16 ? *reinterpret_cast<const uint32_t*>(pbl + t0) : 0u;
      const uint32_t b1l = kBf16 ? *reinterpret_cast<const uint32_t*>(pbl + t0 + 8) : 0u;
      const uint32_t* w0 = reinterpret_cast<const uint32_t*>(v[0]);
      const uint32_t* w1 = reinterpret_cast<const uint32_t*>(v[1]);
      const uint32_t* w2 = reinterpret_cast<const uint32_t*>(v[2]);
      const uint32_t* w3 = reinterpret_cast<const uint32_t*>(v[3]);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const uint32_t a0 = prmt(w0[m], w1[m], 0x5410u), a1 = prmt(w0[m], w1[m], 0x7632u);
        const uint32_t a2 = prmt(w2[m], w3[m], 0x5410u), a3 = prmt(w2[m], w3[m], 0x7632u);
        mma_h16<kBf16>(oacc[m], a0, a1, a2, a3, b0, b1);
        if (kBf16) mma_bf16(oacc[m], a0, a1, a2, a3, b0l, b1l);
      }
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      st.o[2 * m] += oacc[m][0];
      st.o[2 * m + 1] += oacc[m][2];
    }
    __syncwarp();
  }
}

// kQG groups of four query heads per KV head share each page-head's unpacked
// operands: with kQG = 2 the key contraction runs one 64-token half at a time
// (three accumulator sets: the two groups' bytes 1 | 0 and both groups' signed byte 2)
// and the value contraction one 64-channel half at a time.
template <bool kBf16, int kQG>
__global__ void __launch_bounds__(32 * warps_per_cta<kQG>(), ctas_per_sm<kQG>())
decode_i8_kernel(const KittyDecodeArgs a, DecodePlan plan) {
  using T = Half16<kBf16>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.d_boost, H = a.num_kv_heads, B = a.batch;
  // this launch's query heads: qb .. qb + g - 1 of every KV head's group of g_all
  const int g_all = a.num_q_heads / H;
  const int g = plan.g_pass > 0 ? plan.g_pass : g_all, qb = plan.qh_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g_ = lane >> 2, q_ = lane & 3;
  const int pq = lane >> 3, cb = lane & 7;
  const Layout L = i8_layout(K, kQG);
  const int kPlane = L.plane;
  uint8_t* wsm = smem + warp * L.size;
  uint8_t* kbuf = wsm + L.kbuf;
  uint8_t* vbuf = wsm + L.vbuf;
  uint8_t* dtab = wsm + L.dtab;
  uint8_t* ptab = wsm + L.ptab;
  const uint32_t* ent = reinterpret_cast<const uint32_t*>(wsm + L.ent);
  const uint32_t bar_k = smem_u32(wsm + L.bars), bar_v = bar_k + 8;

  // ---- this warp's slice of the item space
  // slice index: warp-major over the CTAs, so a small job spreads over many SMs
  const int64_t gw = int64_t(warp) * gridDim.x + blockIdx.x;
  const int64_t n_warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  // (units: pages count 1, fp16 chunk items kFp16Weight)
  SegmentScan sc = scan_segments(a, B, H, 0, lane, kFp16Weight);
  const int64_t total = sc.total;
  int64_t F = (total + n_warps - 1) / n_warps;
  if (F < plan.pages_per_split) F = plan.pages_per_split;
  const int64_t f0 = gw * F;
  if (f0 >= total) return;
  const int64_t f1 = min(total, f0 + F);
  sc = scan_segments(a, B, H, f0, lane, kFp16Weight);
  Cursor pos;   // the item being processed: the first one starting in [f0, f1)
  if (!make_cursor(pos, a, sc.seg_begin, sc.b, sc.h, sc.u, kFp16Weight) || pos.f >= f1) {
    // No item starts in the slice: it lies inside the span of an fp16 chunk item that
    // an earlier warp processes.  Its slot of that segment gets a neutral partial (the
    // merge reads every slot below the segment's count).
    const int64_t base = ((int64_t(sc.b) * H + sc.h) * plan.num_splits + int(gw - sc.seg_begin / F)) * g;
    for (int i = lane; i < g; i += 32) {
      plan.ws_m[base + i] = -INFINITY;
      plan.ws_l[base + i] = 0.f;
    }
    for (int i = lane; i < g * kD; i += 32) plan.ws_o[base * kD + i] = 0.f;
    return;
  }
  const int64_t pos_unit = pos.p <= pos.n16 ? int64_t(kFp16Weight) * pos.p
                                            : int64_t(kFp16Weight) * pos.n16 + (pos.p - pos.n16);
  int slot = int(gw - (pos.f - pos_unit) / F);

  if (lane == 0) {
    mbar_init(bar_k, 1);
    mbar_init(bar_v, 1);
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  // constant table: the zero row after the high plane
  if (lane < 8) reinterpret_cast<uint32_t*>(kbuf + 4608 + K * 32)[lane] = 0u;
  __syncwarp();

  const float qk_scale = a.sm_scale * kLog2e;
  const int64_t ph_low = int64_t(kD) * (kG / 4), ph_high = int64_t(K) * (kG / 4);
  const uint32_t bytes_high = uint32_t(ph_high);
  const uint32_t k_tx = 4096u + 512u + bytes_high, v_tx = 4096u + 512u;
  uint32_t k_phase = 0, v_phase = 0;
  bool failed = false;

  // Block-table window: lane l holds the physical page of page index bt_base + l of
  // cache row bt_row, so the page of the next copy is a register shuffle instead of a
  // dependent global load on the copy-issue path (reloaded once per 32 pages or at a
  // segment change).  Warp-uniform.
  int bt_row = -1, bt_base = 0, bt_val = 0;
  auto page_of = [&](const Cursor& c) -> int {
    const int idx = c.p - c.n16;
    if (c.s != bt_row || idx < bt_base || idx >= bt_base + 32) {
      bt_row = c.s;
      bt_base = idx;
      const int e = idx + lane;
      bt_val = e < c.items - c.n16 ? a.block_table[int64_t(c.s) * a.bt_s_seq + e] : -1;
    }
    return __shfl_sync(0xffffffffu, bt_val, idx - bt_base);
  };
  auto issue_k = [&](const Cursor& c, int page) {
    if (page < 0 || page >= a.pool_pages) page = 0;
    const int64_t phh = int64_t(page) * H + c.h;
    mbar_arrive_expect_tx(bar_k, k_tx);
    bulk_g2s(smem_u32(kbuf), a.key_low + phh * ph_low, 4096u, bar_k);
    bulk_g2s(smem_u32(kbuf + 4096), reinterpret_cast<const uint8_t*>(a.key_meta) + phh * (2 * kD * 2), 512u, bar_k);
    if (bytes_high) bulk_g2s(smem_u32(kbuf + 4608), a.key_high + phh * ph_high, bytes_high, bar_k);
  };
  auto issue_v = [&](const Cursor& c, int page) {
    if (page < 0 || page >= a.pool_pages) page = 0;
    const int64_t phh = int64_t(page) * H + c.h;
    mbar_arrive_expect_tx(bar_v, v_tx);
    bulk_g2s(smem_u32(vbuf), a.val_codes + phh * ph_low, 4096u, bar_v);
    bulk_g2s(smem_u32(vbuf + 4096), reinterpret_cast<const uint8_t*>(a.val_meta) + phh * (2 * kG * 2), 512u, bar_v);
  };

  Cursor cur = pos;
  bool have_next = cursor_to_page(cur, a, f1, kFp16Weight);
  int cur_page = have_next ? page_of(cur) : -1;   // physical page of cur (the copies in flight)
  if (lane == 0 && have_next) { issue_k(cur, cur_page); issue_v(cur, cur_page); }
  __syncwarp();
  // the key (value) buffer has been read by every lane: request the next page's keys
  // (values) at once, before the epilogue that only needs registers
  auto next_keys = [&]() {
    __syncwarp();
    have_next = cursor_step(cur, a, kFp16Weight) && cursor_to_page(cur, a, f1, kFp16Weight);
    cur_page = have_next ? page_of(cur) : -1;
    if (lane == 0 && have_next) issue_k(cur, cur_page);
  };
  auto next_values = [&]() {
    __syncwarp();
    if (lane == 0 && have_next) issue_v(cur, cur_page);
  };

  State st[kQG];
#pragma unroll
  for (int qg = 0; qg < kQG; ++qg) reset_state(st[qg]);
  int nb = setup_segment<kQG>(a, pos.b, pos.h, g, g_all, qb, wsm, L, lane);

  // ldmatrix row addresses: row `lane` of a 32-row k-step of the key / value plane
  const uint32_t k_row = smem_u32(kbuf) + 32u * lane, v_row = smem_u32(vbuf) + 32u * lane;
  // B operand bases: column g_ of an MMA = query head g_ >> 1, digit (g_ & 1 ? lo : hi)
  const uint8_t* kb1 = dtab + ((g_ & 1) ? 0 : 1) * kPlane + (g_ >> 1) * kRow;   // b1 | b0
  const uint8_t* kb2 = dtab + 2 * kPlane + (g_ >> 1) * kRow;                     // b2 (even columns)
  const bool ones_col = (g_ & 1) != 0;                                          // odd columns: all-ones plane
  const uint8_t* vb = ptab + ((g_ & 1) ? 0 : 1) * kPlane + (g_ >> 1) * kRow;    // y1 | y0

  for (;;) {   // the items starting in [f0, f1)
    const int b = pos.b, h = pos.h;
    if (pos.p < pos.n16) {
      int t0, t1;
      fp16_chunk(fp16_tokens(a, pos.s), pos.n16, pos.p, t0, t1);
#pragma unroll
      for (int qg = 0; qg < kQG; ++qg)
        process_fp16_region<kBf16>(a, b, h, g, 4 * qg, st[qg], wsm, L, qk_scale, lane, t0, t1);
    } else {
      const bool valid = cur_page >= 0 && cur_page < a.pool_pages;   // cur is this page
      if (!mbar_wait(bar_k, k_phase)) { failed = true; break; }
      k_phase ^= 1u;
      const uint8_t* km = kbuf + 4096;   // scale[128] fp16, zero[128] fp16
      const uint8_t* kh = kbuf + 4608;   // high plane rows, then the zero row

      // ---- key digits: prep lane (query heads pq + 4 qg, channels 16 cb .. 16 cb + 15)
      float zsum[kQG];
      float delta[kQG];
      const uint4* sp = reinterpret_cast<const uint4*>(km + 32 * cb);
      const uint4* zp = reinterpret_cast<const uint4*>(km + 256 + 32 * cb);
      const uint4 s0 = sp[0], s1 = sp[1], z0 = zp[0], z1 = zp[1];
      const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      const uint32_t zw[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
#pragma unroll
      for (int qg = 0; qg < kQG; ++qg) {
        const uint4* qs = reinterpret_cast<const uint4*>(wsm + L.qs + 1024 * qg);
        const uint4 q0 = qs[lane], q1 = qs[32 + lane];
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float w[16];
        float mx = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          w[2 * j] = mul_h16_f32<kBf16>(uint16_t(qw[j] & 0xffffu), uint16_t(sw[j] & 0xffffu));
          w[2 * j + 1] = mul_h16_f32<kBf16>(uint16_t(qw[j] >> 16), uint16_t(sw[j] >> 16));
          mx = fmaxf(mx, fmaxf(fabsf(w[2 * j]), fabsf(w[2 * j + 1])));
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float R = mx > 0.f ? kKeyRange * rcp_approx(mx) : 0.f;   // mx is 0 or >= 2^-48 (fp16 x fp16)
        delta[qg] = mx * (1.0f / kKeyRange);
        uint32_t fb[16];
        float2 zs2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 wj = make_float2(w[2 * j], w[2 * j + 1]);
          const float2 f = fma2(wj, make_float2(R, R), make_float2(kMagicKey, kMagicKey));
          fb[2 * j] = __float_as_uint(f.x);
          fb[2 * j + 1] = __float_as_uint(f.y);
          zs2 = fma2(T::to_f2(zw[j]), wj, zs2);
        }
        float zsm = zs2.x + zs2.y;
        zsm += __shfl_xor_sync(0xffffffffu, zsm, 1);
        zsm += __shfl_xor_sync(0xffffffffu, zsm, 2);
        zsm += __shfl_xor_sync(0xffffffffu, zsm, 4);
        zsum[qg] = zsm;
        // word qq <-> channels 16 cb + 4 qq .. 16 cb + 4 qq + 3
        uint32_t d0[4], d1[4], d2[4];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          bytes01(fb[4 * qq], fb[4 * qq + 1], fb[4 * qq + 2], fb[4 * qq + 3], d0[qq], d1[qq]);
          d2[qq] = byte2(fb[4 * qq], fb[4 * qq + 1], fb[4 * qq + 2], fb[4 * qq + 3]);
          if constexpr (kQG == 2) d2[qq] = signed_top_digits(d2[qq]);
        }
        uint8_t* row = dtab + (pq + 4 * qg) * kRow + 16 * cb;
        *reinterpret_cast<uint4*>(row) = make_uint4(d0[0], d0[1], d0[2], d0[3]);
        *reinterpret_cast<uint4*>(row + kPlane) = make_uint4(d1[0], d1[1], d1[2], d1[3]);
        *reinterpret_cast<uint4*>(row + 2 * kPlane) = make_uint4(d2[0], d2[1], d2[2], d2[3]);
      }
      __syncwarp();
      // this lane's query heads q_ + 4 qg: zero-point term and digit step, from prep lane 8 q_
      float zqg[kQG], cqg[kQG];
#pragma unroll
      for (int qg = 0; qg < kQG; ++qg) {
        zqg[qg] = __shfl_sync(0xffffffffu, zsum[qg], 8 * q_) * qk_scale;
        cqg[qg] = __shfl_sync(0xffffffffu, delta[qg], 8 * q_) * qk_scale;
      }
      // ---- scores (log2 domain): s[qg][4 k + i] <-> token 32 k + 4 g_ + i; tile 4 half + i
      // holds tokens 64 half + 4 g_ + i (row g_, k = 2 half) and + 32 (row g_ + 8)
      float s[kQG][16];
      if constexpr (kQG == 1) {
      const float zq = zqg[0], cq = cqg[0];
      int acc1[8][4], acc2[8][4];
      // ---- baseline plane
      key_kstep<true>(acc1, acc2, k_row, kb1, kb2, ones_col, 0, q_);
#pragma unroll
      for (int ks = 1; ks < 4; ++ks) key_kstep<false>(acc1, acc2, k_row + 1024u * ks, kb1, kb2, ones_col, ks, q_);
      // ---- boosted high plane: K = entries 16 bs + k (row of entry k from lane k,
      // token bytes 0-15 / 16-31 as the two matrices of one transposed load)
      for (int bs = 0; bs < nb; bs += 16) {
        const uint4 e4 = *reinterpret_cast<const uint4*>(ent + bs + 4 * q_);
        const uint32_t es[4] = {e4.x, e4.y, e4.z, e4.w};
        uint32_t r[4], bb1 = 0u, bb2 = 0u;
        ldsm_t_x2(smem_u32(kh) + (ent[bs + (lane & 15)] & 0xffffu) + 16u * (lane >> 4), r);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t pos = es[kk] >> 16;
          bb1 |= uint32_t(kb1[pos]) << (8 * kk);
          bb2 |= uint32_t(kb2[pos]) << (8 * kk);
        }
        if (ones_col) bb2 = 0x01010101u;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t x0 = r[2 * half], x1 = r[2 * half + 1];
          mma_k16(acc1[4 * half + 0], high_code<0>(x0), high_code<0>(x1), bb1);
          mma_k16(acc2[4 * half + 0], high_code<0>(x0), high_code<0>(x1), bb2);
          mma_k16(acc1[4 * half + 1], high_code<1>(x0), high_code<1>(x1), bb1);
          mma_k16(acc2[4 * half + 1], high_code<1>(x0), high_code<1>(x1), bb2);
          mma_k16(acc1[4 * half + 2], high_code<2>(x0), high_code<2>(x1), bb1);
          mma_k16(acc2[4 * half + 2], high_code<2>(x0), high_code<2>(x1), bb2);
          mma_k16(acc1[4 * half + 3], high_code<3>(x0), high_code<3>(x1), bb1);
          mma_k16(acc2[4 * half + 3], high_code<3>(x0), high_code<3>(x1), bb2);
        }
      }
      next_keys();
      {
        // row factors 1, 4, 16, 16 of code i
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int i = mt & 3, half = mt >> 2;
          const float f = cq * (i == 0 ? 1.0f : i == 1 ? 0.25f : 0.0625f);
          const float2 fl = make_float2(f, f), fh = make_float2(f * 65536.0f, f * 65536.0f);
          const int lo0 = 256 * acc1[mt][0] + acc1[mt][1], lo1 = 256 * acc1[mt][2] + acc1[mt][3];
          const int hi0 = acc2[mt][0] - 64 * acc2[mt][1], hi1 = acc2[mt][2] - 64 * acc2[mt][3];
          const float2 t = fma2(make_float2(float(lo0), float(lo1)), fl, make_float2(-zq, -zq));
          const float2 r = fma2(make_float2(float(hi0), float(hi1)), fh, t);
          s[0][8 * half + i] = r.x;
          s[0][8 * half + 4 + i] = r.y;
        }
      }
      } else {
        // 8 query heads: this lane's heads q_ (group 0) and q_ + 4 (group 1).  Digits b1 | b0
        // of a group in one MMA per code plane (column g_: head (g_ >> 1) + 4 qg, digit hi /
        // lo, as for 4 heads); the signed top digits b2 - 64 of both groups in one more
        // (column g_: head (g_ >> 1) + 4 (g_ & 1)), so C columns 2 q_ / 2 q_ + 1 of a thread
        // hold the b2 sums of its heads q_ / q_ + 4 and no all-ones column is needed.
        // (Splitting the four code planes of a half into two passes, for fewer live
        // accumulators, re-reads the digits and was 7 % slower.)
        const uint8_t* kb2s = dtab + 2 * kPlane + ((g_ >> 1) + 4 * (g_ & 1)) * kRow;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          int a1[2][4][4], a2[4][4];
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t b10 = lds32(kb1 + 32 * ks + 4 * q_), b11 = lds32(kb1 + 32 * ks + 16 + 4 * q_);
            const uint32_t b12 = lds32(kb1 + 4 * kRow + 32 * ks + 4 * q_);
            const uint32_t b13 = lds32(kb1 + 4 * kRow + 32 * ks + 16 + 4 * q_);
            const uint32_t b20 = lds32(kb2s + 32 * ks + 4 * q_), b21 = lds32(kb2s + 32 * ks + 16 + 4 * q_);
            uint32_t r[4];
            ldsm_t_x2(k_row + 1024u * ks + 16u * half, r);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t m = i < 3 ? (0x03030303u << (2 * i)) : 0x30303030u;
              const int sh = i < 3 ? 0 : 2;
              const uint32_t c0 = (r[0] >> sh) & m, c1 = (r[1] >> sh) & m, c2 = (r[2] >> sh) & m,
                             c3 = (r[3] >> sh) & m;
              if (ks == 0) {
                mma_k32_z(a1[0][i], c0, c1, c2, c3, b10, b11);
                mma_k32_z(a1[1][i], c0, c1, c2, c3, b12, b13);
                mma_k32s<true>(a2[i], c0, c1, c2, c3, b20, b21);
              } else {
                mma_k32(a1[0][i], c0, c1, c2, c3, b10, b11);
                mma_k32(a1[1][i], c0, c1, c2, c3, b12, b13);
                mma_k32s<false>(a2[i], c0, c1, c2, c3, b20, b21);
              }
            }
          }
          for (int bs = 0; bs < nb; bs += 16) {
            const uint4 e4 = *reinterpret_cast<const uint4*>(ent + bs + 4 * q_);
            const uint32_t es[4] = {e4.x, e4.y, e4.z, e4.w};
            uint32_t r[4], bb10 = 0u, bb11 = 0u, bb2 = 0u;
            ldsm_t_x2(smem_u32(kh) + (ent[bs + (lane & 15)] & 0xffffu) + 16u * (lane >> 4), r);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t pos = es[kk] >> 16;
              bb10 |= uint32_t(kb1[pos]) << (8 * kk);
              bb11 |= uint32_t(kb1[4 * kRow + pos]) << (8 * kk);
              bb2 |= uint32_t(kb2s[pos]) << (8 * kk);
            }
            const uint32_t x0 = r[2 * half], x1 = r[2 * half + 1];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t h0 = high_code_of(i, x0), h1 = high_code_of(i, x1);
              mma_k16(a1[0][i], h0, h1, bb10);
              mma_k16(a1[1][i], h0, h1, bb11);
              mma_k16s(a2[i], h0, h1, bb2);
            }
          }
#pragma unroll
          for (int qg = 0; qg < 2; ++qg)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float f = cqg[qg] * (i == 0 ? 1.0f : i == 1 ? 0.25f : 0.0625f);
              const float2 fl = make_float2(f, f), fh = make_float2(f * 65536.0f, f * 65536.0f);
              const int lo0 = 256 * a1[qg][i][0] + a1[qg][i][1], lo1 = 256 * a1[qg][i][2] + a1[qg][i][3];
              const int hi0 = a2[i][qg], hi1 = a2[i][2 + qg];
              const float2 t = fma2(make_float2(float(lo0), float(lo1)), fl, make_float2(-zqg[qg], -zqg[qg]));
              const float2 rr = fma2(make_float2(float(hi0), float(hi1)), fh, t);
              s[qg][8 * half + i] = rr.x;
              s[qg][8 * half + 4 + i] = rr.y;
            }
        }
      }
      if constexpr (kQG != 1) next_keys();

      if (!mbar_wait(bar_v, v_phase)) { failed = true; break; }
      v_phase ^= 1u;
      bool v_requested = false;
      if (valid) {
        // ---- P' = p * scale_v as 16-bit fixed point, tokens 32 k + 4 g_ + i (v = 4 k + i)
        float dvg[kQG];
#pragma unroll
        for (int qg = 0; qg < kQG; ++qg) {
        // (scale, zero) of this lane's tokens, read again for every query group
        uint32_t sz[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 x = *reinterpret_cast<const uint4*>(vbuf + 4096 + 4 * (32 * k + 4 * g_));
          sz[4 * k] = x.x; sz[4 * k + 1] = x.y; sz[4 * k + 2] = x.z; sz[4 * k + 3] = x.w;
        }
        softmax_step(st[qg], s[qg]);   // s -> p
        float pp[16];
#pragma unroll
        for (int v = 0; v < 16; v += 2) {
          // (scale, zero) of tokens v and v + 1 -> (scale_v, scale_v+1)
          const float2 sc = make_float2(T::lo_f(sz[v]), T::lo_f(sz[v + 1]));
          const float2 pr = mul2(make_float2(s[qg][v], s[qg][v + 1]), sc);
          pp[v] = pr.x;
          pp[v + 1] = pr.y;
        }
        float mp = max16(pp, 0.f);
        mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 4));
        mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 8));
        mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 16));
        // a page whose largest weighted probability is below 1e-30 adds nothing next to the
        // row maximum (weight 1): its digits are left at zero
        const float Rv = mp > 1e-30f ? kValRange * rcp_approx(mp) : 0.f;
        const float dv = mp * (1.0f / kValRange);
        dvg[qg] = dv;
        uint32_t yb[16];
        float2 zv2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int v = 0; v < 16; v += 2) {
          const float2 fy = fma2(make_float2(pp[v], pp[v + 1]), make_float2(Rv, Rv), make_float2(kMagicVal, kMagicVal));
          yb[v] = __float_as_uint(fy.x);
          yb[v + 1] = __float_as_uint(fy.y);
          const float2 y = add2(fy, make_float2(-kMagicVal, -kMagicVal));
          // zero-points of tokens v, v + 1
          zv2 = fma2(make_float2(T::hi_f(sz[v]), T::hi_f(sz[v + 1])), y, zv2);
        }
        const float zv = zv2.x + zv2.y;
        st[qg].zs = __fmaf_rn(zv, dv, st[qg].zs);
        uint8_t* prow = ptab + (q_ + 4 * qg) * kRow + 4 * g_;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint32_t y0, y1;
          bytes01(yb[4 * k], yb[4 * k + 1], yb[4 * k + 2], yb[4 * k + 3], y0, y1);
          *reinterpret_cast<uint32_t*>(prow + 32 * k) = y0;
          *reinterpret_cast<uint32_t*>(prow + kPlane + 32 * k) = y1;
        }
        }
        __syncwarp();
        if constexpr (kQG == 1) {
        const float dv = dvg[0];
        State& sto = st[0];
        // ---- values: M = channels, K = tokens 32 ks + k
        int acc[8][4];
        val_kstep<true>(acc, v_row, vb, 0, q_);
#pragma unroll
        for (int ks = 1; ks < 4; ++ks) val_kstep<false>(acc, v_row + 1024u * ks, vb, ks, q_);
        next_values();
        v_requested = true;
        // ---- accumulate: tile 4 half + i holds channels 64 half + 4 g_ + i (row g_) and
        // + 32 (row g_ + 8), i.e. st.o[8 half + i] and st.o[8 half + 4 + i]; row factor 4^i
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int i = mt & 3, half = mt >> 2;
          const float f = dv * (i == 0 ? 1.0f : i == 1 ? 0.25f : i == 2 ? 0.0625f : 0.015625f);
          const int c0 = 256 * acc[mt][0] + acc[mt][1], c1 = 256 * acc[mt][2] + acc[mt][3];
          const float2 o = fma2(make_float2(float(c0), float(c1)), make_float2(f, f),
                                make_float2(sto.o[8 * half + i], sto.o[8 * half + 4 + i]));
          sto.o[8 * half + i] = o.x;
          sto.o[8 * half + 4 + i] = o.y;
        }
        } else {
          const uint8_t* vbg[kQG];
#pragma unroll
          for (int qg = 0; qg < kQG; ++qg) vbg[qg] = vb + 4 * qg * kRow;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            int acc[kQG][4][4];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              uint32_t bv[kQG][2];
#pragma unroll
              for (int qg = 0; qg < kQG; ++qg) {
                bv[qg][0] = lds32(vbg[qg] + 32 * ks + 4 * q_);
                bv[qg][1] = lds32(vbg[qg] + 32 * ks + 16 + 4 * q_);
              }
              uint32_t r[4];
              ldsm_t_x2(v_row + 1024u * ks + 16u * half, r);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t m = 0x03030303u << (2 * i);
#pragma unroll
                for (int qg = 0; qg < kQG; ++qg) {
                  if (ks == 0) mma_k32_z(acc[qg][i], r[0] & m, r[1] & m, r[2] & m, r[3] & m, bv[qg][0], bv[qg][1]);
                  else mma_k32(acc[qg][i], r[0] & m, r[1] & m, r[2] & m, r[3] & m, bv[qg][0], bv[qg][1]);
                }
              }
            }
            if (half == 1) {   // the value buffer has been read: request the next page's values
              next_values();
              v_requested = true;
            }
#pragma unroll
            for (int qg = 0; qg < kQG; ++qg)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float f = dvg[qg] * (i == 0 ? 1.0f : i == 1 ? 0.25f : i == 2 ? 0.0625f : 0.015625f);
                const int c0 = 256 * acc[qg][i][0] + acc[qg][i][1], c1 = 256 * acc[qg][i][2] + acc[qg][i][3];
                const float2 o = fma2(make_float2(float(c0), float(c1)), make_float2(f, f),
                                      make_float2(st[qg].o[8 * half + i], st[qg].o[8 * half + 4 + i]));
                st[qg].o[8 * half + i] = o.x;
                st[qg].o[8 * half + 4 + i] = o.y;
              }
          }
        }
      }
      if (!v_requested) next_values();
    }

    // ---- advance; write the partial at a segment end or at the end of the slice
    const bool seg_end = pos.p + 1 >= pos.items;
    const bool last = pos.f + cursor_width(pos, kFp16Weight) >= f1;   // no item of the slice follows
    if (seg_end || last) {
      const int64_t base = ((int64_t(b) * H + h) * plan.num_splits + slot) * g;
#pragma unroll
      for (int qg = 0; qg < kQG; ++qg) {
        State& sq = st[qg];
        float l = sq.l, zs = sq.zs;
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        zs += __shfl_xor_sync(0xffffffffu, zs, 4);
        zs += __shfl_xor_sync(0xffffffffu, zs, 8);
        zs += __shfl_xor_sync(0xffffffffu, zs, 16);
        const int qh = q_ + 4 * qg;
        if (qh < g) {
          // o[4 k + i] <-> channel 32 k + 4 g_ + i
          float* o = plan.ws_o + (base + qh) * kD + 4 * g_;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            *reinterpret_cast<float4*>(o + 32 * k) =
                make_float4(sq.o[4 * k] - zs, sq.o[4 * k + 1] - zs, sq.o[4 * k + 2] - zs, sq.o[4 * k + 3] - zs);
          if (g_ == 0) {
            plan.ws_m[base + qh] = sq.m == -INFINITY ? -INFINITY : sq.m * kLn2;
            plan.ws_l[base + qh] = l;
          }
        }
        reset_state(sq);
      }
      if (seg_end && lane == 0) plan.ws_count[int64_t(b) * H + h] = slot + 1;
    }
    if (last) break;
    cursor_step(pos, a, kFp16Weight);
    if (seg_end) {
      slot = 0;
      __syncwarp();
      nb = setup_segment<kQG>(a, pos.b, pos.h, g, g_all, qb, wsm, L, lane);
    }
  }
  if (failed) {
    if (lane == 0) atomicOr(&g_decode_error_i8, 1u);
    // copies still in flight must land before the CTA's shared memory is released
    mbar_wait(bar_k, k_phase);
    mbar_wait(bar_v, v_phase);
  }
}

}  // namespace

bool i8_supports(const KittyDecodeArgs& a) {
  const int g = a.num_q_heads / a.num_kv_heads;
  auto region_ok = [](const void* p, int64_t s_seq, int64_t s_head, int64_t s_tok) {
    return p == nullptr || (aligned(p, 16) && s_seq % 8 == 0 && s_head % 8 == 0 && s_tok % 8 == 0);
  };
  return a.head_dim == kD && a.group == kG && g >= 1 && a.d_boost <= 128 &&
         aligned(a.q, 16) && a.q_s_seq % 8 == 0 && a.q_s_head % 8 == 0 &&
         region_ok(a.sink_k, a.sk_s_seq, a.sk_s_head, a.sk_s_tok) &&
         region_ok(a.sink_v, a.sv_s_seq, a.sv_s_head, a.sv_s_tok) &&
         region_ok(a.tail_k, a.tk_s_seq, a.tk_s_head, a.tk_s_tok) &&
         region_ok(a.tail_v, a.tv_s_seq, a.tv_s_head, a.tv_s_tok) &&
         (a.max_pages_per_seq == 0 ||
          (aligned(a.key_low, 16) && aligned(a.key_meta, 16) && aligned(a.val_codes, 16) &&
           aligned(a.val_meta, 16) && (a.d_boost == 0 || aligned(a.key_high, 16))));
}

int i8_ctas_per_sm() { return 1; }

namespace {
// groups of four query heads per launch (a launch covers at most kI8MaxHeadsPerPass)
int i8_pass_heads(const KittyDecodeArgs& a, const DecodePlan& plan) {
  return plan.g_pass > 0 ? plan.g_pass : std::min(a.num_q_heads / a.num_kv_heads, kI8MaxHeadsPerPass);
}
int i8_groups(const KittyDecodeArgs& a, const DecodePlan& plan) { return i8_pass_heads(a, plan) > 4 ? 2 : 1; }
// warps of one CTA: the compile-time count, fewer when their shared memory would pass
// the per-CTA limit of the current device
int i8_warps(int qg, int d_boost) {
  static int optin = 0;
  if (optin == 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0) {
      cudaGetLastError();
      v = 227 * 1024;
    }
    optin = v;
  }
  const int w = qg == 1 ? warps_per_cta<1>() : warps_per_cta<2>();
  return std::max(1, std::min(w, optin / i8_layout(d_boost, qg).size));
}
int i8_ctas(int qg) { return qg == 1 ? ctas_per_sm<1>() : ctas_per_sm<2>(); }
}  // namespace

// Slots per segment S = num_splits (default kSlotsTarget, more when there are fewer
// segment cost units than warps need for a full grid): every warp takes at least
// F_min = ceil(units_max / S) units, so a segment spans at most ceil(units_max / F_min)
// + 1 warps, which is the slot count the merge reads.
void i8_plan(const KittyDecodeArgs& a, int sm_count, DecodePlan* plan) {
  // cost units of the longest segment: pages + weighted fp16 chunk items
  const int items_max = a.max_pages_per_seq + kFp16Weight * dev::kMaxFp16Items;
  // few segments (small batch, few KV heads per GPU): more slots per segment so that
  // every warp of the persistent grid gets a slice
  const int qg = i8_groups(a, *plan);
  const int64_t warps = int64_t(sm_count) * i8_ctas(qg) * i8_warps(qg, a.d_boost);
  const int64_t per_warp = std::max<int64_t>(1, int64_t(a.batch) * a.num_kv_heads * items_max / warps);
  const int auto_target = int(std::max<int64_t>(kSlotsTarget, (items_max + per_warp - 1) / per_warp));
  int target = a.num_splits > 0 ? a.num_splits : auto_target;
  target = std::max(1, std::min({target, items_max, kMaxDecodeSlots - 1}));
  const int f_min = (items_max + target - 1) / target;
  plan->pages_per_split = f_min;
  plan->num_splits = (items_max + f_min - 1) / f_min + 1;
  const int64_t total_max = int64_t(a.batch) * a.num_kv_heads * items_max;
  const int64_t warps_needed = (total_max + f_min - 1) / f_min;
  // slices are interleaved over the CTAs, so fewer slices than CTA slots need only as
  // many CTAs as slices
  plan->grid = int(std::max<int64_t>(1, std::min<int64_t>(warps_needed, int64_t(sm_count) * i8_ctas(qg))));
}

namespace {
// shared-memory attribute and resident CTAs per SM of one instantiation, set up once
// per shared-memory size
template <bool kBf16, int kQG>
int prepare_i8(int threads, int smem, int* blocks) {
  static int configured_bytes = 0;
  if (configured_bytes < smem) {
    cudaError_t e =
        cudaFuncSetAttribute(decode_i8_kernel<kBf16, kQG>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("decode_i8 smem attribute: ") + cudaGetErrorString(e));
    configured_bytes = smem;
  }
  // persistent grid: no more CTAs than fit on the GPU at once (shared memory grows with d_boost)
  static int occ_smem = -1, occ_blocks = 1;
  if (occ_smem != smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_i8_kernel<kBf16, kQG>, threads, smem) != cudaSuccess ||
        n <= 0) {
      cudaGetLastError();
      n = 1;
    }
    occ_blocks = std::min(n, ctas_per_sm<kQG>());
    occ_smem = smem;
  }
  *blocks = occ_blocks;
  return KITTY_OK;
}
}  // namespace

int launch_decode_i8(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  const int qg = i8_groups(a, plan);
  const Layout L = i8_layout(a.d_boost, qg);
  const int warps = i8_warps(qg, a.d_boost);
  const int smem = warps * L.size;
  const bool bf16 = a.dtype == KITTY_DTYPE_BF16;
  int occ_blocks = 1;
  const int th = 32 * warps;
  const int rc = qg == 1 ? (bf16 ? prepare_i8<true, 1>(th, smem, &occ_blocks) : prepare_i8<false, 1>(th, smem, &occ_blocks))
                         : (bf16 ? prepare_i8<true, 2>(th, smem, &occ_blocks) : prepare_i8<false, 2>(th, smem, &occ_blocks));
  if (rc != KITTY_OK) return rc;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms = 148;
  }
  const int grid = std::max(1, std::min(plan.grid, sms * occ_blocks));
  if (qg == 1) {
    if (bf16) decode_i8_kernel<true, 1><<<grid, 32 * warps, smem, stream>>>(a, plan);
    else decode_i8_kernel<false, 1><<<grid, 32 * warps, smem, stream>>>(a, plan);
  } else {
    if (bf16) decode_i8_kernel<true, 2><<<grid, 32 * warps, smem, stream>>>(a, plan);
    else decode_i8_kernel<false, 2><<<grid, 32 * warps, smem, stream>>>(a, plan);
  }
  return check_launch("decode_i8_kernel");
}

int read_decode_error_i8(uint32_t* flags, int clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_decode_error_i8, sizeof(v));
  if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("read error flags: ") + cudaGetErrorString(e));
  if (clear && v) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_decode_error_i8, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("clear error flags: ") + cudaGetErrorString(e));
  }
  *flags = v;
  return KITTY_OK;
}

}  // namespace kitty
