// Paged GQA decode attention on the tensor cores (head_dim = group = 128,
// up to 8 query heads per KV head).
//
// Work decomposition.  Each (sequence b, KV head h) is a *segment* of items:
// item 0 is the fp16 region (sinks then tail), items 1..n are its quantised
// pages.  All segments are laid end to end (a warp-level prefix scan of the
// page counts gives every segment's start), and every warp of the persistent
// grid takes one contiguous slice of F items.  A warp keeps an online softmax
// while it walks its slice and writes one partial result (max, sum,
// unnormalised accumulator) for every segment it touches; the merge kernel
// combines the partials of a segment.  No CTA-wide barrier sits on the data
// path, so warps never wait for one another, and long and short sequences are
// spread over the warps to within one item.
//
// Data movement.  Each warp owns a key buffer (low plane, metadata, high
// plane of one page-head) and a value buffer (codes, metadata), filled by
// 1-D bulk async copies (cp.async.bulk, no multicast) that complete on one
// mbarrier each.  The next page's keys are requested as soon as the current
// scores are done, and its values as soon as the current value contraction is
// done.  Waits are bounded: a wait that gives up sets a device error bit and
// the warp stops.
//
// Contraction (per page-head):
//   scores  S[t][qh] = sum_c (q[qh][c] * scale_k[c]) * code_k[c][t]
//                    + 4 * sum_{boosted c} (q[qh][c] * scale_k[c]) * high[row(c)][t]
//                    - sum_c (q[qh][c] * scale_k[c]) * zp_k[c]
//   values  O[c][qh] = sum_t (p[qh][t] * scale_v[t]) * code_v[t][c] - sum_t (p * scale_v)[t] * zp_v[t]
// i.e. (code - zp) * scale from kitty/kernels/dequantize_key.py:89-95 and
// kitty/kernels/quantize_value.py:121-133 with the scales folded into the
// small operand.  Both contractions run as mma.sync.m16n8k16 (fp16 inputs,
// fp32 accumulation) with the 2-bit codes as the A operand (tokens or
// channels as M = 16 rows, the query heads as N = 8 columns); each
// zero-point sum is one extra M tile whose first row holds the zero-points.
// q * scale_k is carried as two fp16 parts (hi + lo, two MMAs per key tile):
// with outlier channels scale_k is large and one fp16 rounding of the
// product moves the logits by ~1e-2, outside the fp16 output tolerance.
//
// 2-bit -> fp16 unpack: a byte permute pairs the same byte of two rows into
// the low bytes of the two 16-bit halves, a 3-input logic op keeps code k of
// each byte and ORs in the exponent of 1024.0 (value 1024 + code * 4^k,
// exact), and one fp16x2 FMA with (4^-k, -1024 * 4^-k) yields the code
// exactly.  Rows are assigned to lanes so that every 32-bit shared-memory
// word load of a warp hits 32 distinct banks.

#include <algorithm>

#include "kitty_decode.cuh"
#include "kitty_ptx.cuh"

namespace kitty {

__device__ unsigned int g_decode_error = 0;  // bit 0: a bulk-copy wait timed out

namespace {

using namespace dev;

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kCtasPerSm = 3;
constexpr int kD = 128, kG = 128;
constexpr int kPRow = 136;          // fp16 elements per row of the P staging tile (16-byte aligned rows)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kSlotsTarget = 16;    // partial slots per segment when the library chooses

// per-warp shared memory (bytes)
struct WarpLayout {
  int kbuf, vbuf, ps, qfrag, qnat, blist, bars, size;
};
__host__ __device__ inline WarpLayout warp_layout(int K) {
  WarpLayout L;
  int o = 0;
  L.kbuf = o;  o += (4096 + 512 + K * 32 + 127) & ~127;   // low plane, scale/zero rows, high plane
  L.vbuf = o;  o += 4096 + 512;                            // codes, (scale, zero) per token
  L.ps = o;    o += 8 * kPRow * 2;                          // P' staging [qh][token]
  L.qfrag = o; o += 8 * 32 * 8;                             // q in B-fragment order [kstep][lane][2]
  L.qnat = o;  o += 8 * kD * 2;                             // q [qh][channel]
  L.blist = o; o += 128 * 2 + 16;                           // boosted channels (c | row << 8)
  L.bars = o;  o += 16;                                     // key / value mbarriers
  L.size = (o + 127) & ~127;
  return L;
}

// ---- PTX helpers (fp16 path) ---------------------------------------------

template <uint32_t kMask>
__device__ __forceinline__ uint32_t mask_or_magic(uint32_t a) {  // (a & mask) | 1024.0h in both halves
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(a), "n"(kMask), "n"(0x64006400u));
  return r;
}
// x * y as an unevaluated fp16 pair hi + lo: hi = RN(x*y), lo = RN(x*y - hi) (the
// fused multiply-add sees the exact product), so hi + lo carries ~22 bits.
__device__ __forceinline__ void hmul2_split(uint32_t x, uint32_t y, uint32_t& hi, uint32_t& lo) {
  hi = hmul2_u32(x, y);
  lo = hfma2_u32(x, y, hi ^ 0x80008000u);
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// code (0..3) of byte-slot k of both 16-bit halves of u, as exact fp16x2
template <int k>
__device__ __forceinline__ uint32_t code2(uint32_t u) {
  constexpr uint32_t mask = 0x00030003u << (2 * k);
  constexpr uint32_t scale = k == 0 ? 0x3C003C00u : k == 1 ? 0x34003400u : k == 2 ? 0x2C002C00u : 0x24002400u;
  constexpr uint32_t bias = k == 0 ? 0xE400E400u : k == 1 ? 0xDC00DC00u : k == 2 ? 0xD400D400u : 0xCC00CC00u;
  return hfma2_u32(mask_or_magic<mask>(u), scale, bias);
}

// One 16-wide k-step of a [row][32-byte] 2-bit plane into 8 M tiles.  w0..w3 are
// word g_ of rows r0, r0+4, r0+8, r0+12 (the thread's K indices 2q_, 2q_+1, 2q_+8,
// 2q_+9); each word holds the 16 M-index values 16*g_ .. 16*g_+15.  M tile m:
// row g_ <-> value m, row g_ + 8 <-> value m + 8.  With kSplit the B operand is
// (b0, b1) + (c0, c1).
template <bool kSplit>
__device__ __forceinline__ void plane_kstep(float (&acc)[8][4], uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                            uint32_t b0, uint32_t b1, uint32_t c0 = 0u, uint32_t c1 = 0u) {
  uint32_t ulo[4], uhi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sel = uint32_t(j) | (uint32_t(j) << 4) | (uint32_t(4 + j) << 8) | (uint32_t(4 + j) << 12);
    ulo[j] = prmt(w0, w1, sel);
    uhi[j] = prmt(w2, w3, sel);
  }
#define KITTY_MTILE(m, k)                                                                          \
  {                                                                                                \
    const uint32_t x0 = code2<k>(ulo[(m) >> 2]), x1 = code2<k>(ulo[((m) >> 2) + 2]);              \
    const uint32_t x2 = code2<k>(uhi[(m) >> 2]), x3 = code2<k>(uhi[((m) >> 2) + 2]);              \
    mma16816(acc[m], x0, x1, x2, x3, b0, b1);                                                      \
    if (kSplit) mma16816(acc[m], x0, x1, x2, x3, c0, c1);                                          \
  }
  KITTY_MTILE(0, 0) KITTY_MTILE(1, 1) KITTY_MTILE(2, 2) KITTY_MTILE(3, 3)
  KITTY_MTILE(4, 0) KITTY_MTILE(5, 1) KITTY_MTILE(6, 2) KITTY_MTILE(7, 3)
#undef KITTY_MTILE
}

struct WarpState {
  float o[8][4];     // O^T C fragments: channel rows, query-head columns 2*q_, 2*q_+1
  float zv[4];       // value zero-point sums (meaningful in lanes 0..3, row 0)
  float m[2];        // running max (log2 domain) for the thread's two query-head columns
  float l[2];        // running sum over this thread's tokens
};

__device__ __forceinline__ void reset_state(WarpState& st) {
#pragma unroll
  for (int m = 0; m < 8; ++m) st.o[m][0] = st.o[m][1] = st.o[m][2] = st.o[m][3] = 0.f;
  st.zv[0] = st.zv[1] = st.zv[2] = st.zv[3] = 0.f;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
}

// Online-softmax update with the scores in `s` (log2 domain, masked = -inf), then
// P' = p * scale_v staged as fp16 in Ps[qh][16*g_ + kappa] (kappa order: token pairs
// (tau, tau+4)).  `svw[tau]` holds (scale, zp) fp16 of the thread's token 16*g_+tau.
__device__ __forceinline__ void softmax_and_stage(WarpState& st, float (&s)[8][4], const uint32_t (&svw)[16],
                                                  __half* ps, int g_, int q_) {
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    mx0 = fmaxf(mx0, fmaxf(s[m][0], s[m][2]));
    mx1 = fmaxf(mx1, fmaxf(s[m][1], s[m][3]));
  }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  const float mn0 = fmaxf(st.m[0], mx0), mn1 = fmaxf(st.m[1], mx1);
  const float a0 = (st.m[0] == -INFINITY) ? 0.f : ex2(st.m[0] - mn0);
  const float a1 = (st.m[1] == -INFINITY) ? 0.f : ex2(st.m[1] - mn1);
  st.m[0] = mn0; st.m[1] = mn1;
  float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    s[m][0] = ex2(s[m][0] - mn0); s[m][1] = ex2(s[m][1] - mn1);
    s[m][2] = ex2(s[m][2] - mn0); s[m][3] = ex2(s[m][3] - mn1);
    sum0 += s[m][0] + s[m][2];
    sum1 += s[m][1] + s[m][3];
    st.o[m][0] *= a0; st.o[m][1] *= a1; st.o[m][2] *= a0; st.o[m][3] *= a1;
  }
  st.l[0] = st.l[0] * a0 + sum0;
  st.l[1] = st.l[1] * a1 + sum1;
  st.zv[0] *= a0; st.zv[1] *= a1; st.zv[2] *= a0; st.zv[3] *= a1;
#pragma unroll
  for (int col = 0; col < 2; ++col) {
    uint32_t w[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t sv_a = prmt(svw[t], svw[t + 4], 0x5410);
      const uint32_t sv_b = prmt(svw[t + 8], svw[t + 12], 0x5410);
      w[t] = hmul2_u32(pack_f32x2(s[t][col], s[t + 4][col]), sv_a);
      w[t + 4] = hmul2_u32(pack_f32x2(s[t][col + 2], s[t + 4][col + 2]), sv_b);
    }
    __half* row = ps + (2 * q_ + col) * kPRow + 16 * g_;
    *reinterpret_cast<uint4*>(row) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(row + 8) = make_uint4(w[4], w[5], w[6], w[7]);
  }
  __syncwarp();
}

// B fragment of P' for value k-step s (tokens 16s .. 16s+15).
__device__ __forceinline__ void load_pfrag(uint32_t& b0, uint32_t& b1, const __half* ps, int s, int lane) {
  const int mi = (lane >> 3) & 1, n = lane & 7;
  ldmatrix_x2(b0, b1, smem_u32(ps + n * kPRow + 16 * s + 8 * mi));
}

// Query rows of (b, h) and the boosted-channel list of head h into the warp's
// shared memory, plus q in B-fragment order (channels 16s + q_ + 4e, head g_).
// Returns the number of boosted channels.
__device__ int setup_segment(const KittyDecodeArgs& a, int b, int h, int g, uint8_t* wsm, const WarpLayout& L,
                             int lane) {
  __half* qnat = reinterpret_cast<__half*>(wsm + L.qnat);
  const uint16_t* qg = reinterpret_cast<const uint16_t*>(a.q) + b * a.q_s_seq + int64_t(h * g) * a.q_s_head;
  {  // lane -> query head lane >> 2, channels (lane & 3) * 32 .. +31
    const int qh = lane >> 2, c0 = (lane & 3) * 32;
    uint4* dst = reinterpret_cast<uint4*>(qnat + qh * kD + c0);
    if (qh < g) {
      const uint4* src = reinterpret_cast<const uint4*>(qg + qh * a.q_s_head + c0);
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = src[i];
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
  uint16_t* blist = reinterpret_cast<uint16_t*>(wsm + L.blist);
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  int base = 0;
  for (int c0 = 0; c0 < kD; c0 += 32) {
    const int c = c0 + lane;
    const int r = bidx[c];
    const bool boosted = r < a.d_boost;
    const uint32_t bal = __ballot_sync(0xffffffffu, boosted);
    if (boosted) blist[base + __popc(bal & ((1u << lane) - 1u))] = uint16_t(c | (r << 8));
    base += __popc(bal);
  }
  __syncwarp();
  const int g_ = lane >> 2, q_ = lane & 3;
  const uint16_t* qr = reinterpret_cast<const uint16_t*>(qnat) + g_ * kD + q_;
  uint2* qf = reinterpret_cast<uint2*>(wsm + L.qfrag);
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    qf[s * 32 + lane] = make_uint2(pack16(qr[16 * s], qr[16 * s + 4]), pack16(qr[16 * s + 8], qr[16 * s + 12]));
  }
  __syncwarp();
  return base;
}

// fp16 region of (b, h): sinks then tail, 128 tokens per chunk, read straight
// from global memory with 16-byte loads.
__device__ void process_fp16_region(const KittyDecodeArgs& a, int b, int h, WarpState& st, uint8_t* wsm,
                                    const WarpLayout& L, float qk_scale, int lane, int t_begin, int t_end) {
  const int cr = cache_row(a, b);   // cache row (sinks, tail, lengths)
  const int g_ = lane >> 2, q_ = lane & 3;
  const int sink_len = a.sink_len ? a.sink_len[cr] : a.sink_len_all;
  const int tail_len = a.tail_len ? a.tail_len[cr] : a.tail_len_all;
  (void)tail_len;
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(wsm + L.qnat);   // [8][64] words
  __half* ps = reinterpret_cast<__half*>(wsm + L.ps);
  for (int f0 = t_begin; f0 < t_end; f0 += kG) {
    const int ntok = min(kG, t_end - f0);
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
    // scores: rows = tokens 16 g_ + m / m + 8; k-step s, K indices (2q_, 2q_+1, 2q_+8, 2q_+9)
    // <-> channels 32 q_ + 4 s + (0, 1, 2, 3): the thread reads 64 contiguous bytes per token
    float sacc[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      sacc[m][0] = sacc[m][1] = sacc[m][2] = sacc[m][3] = 0.f;
      const int ta = 16 * g_ + m, tb = ta + 8;
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
      for (int s = 0; s < 8; ++s) {
        const uint32_t b0 = qw[g_ * 64 + 16 * q_ + 2 * s], b1 = qw[g_ * 64 + 16 * q_ + 2 * s + 1];
        mma16816(sacc[m], wa[2 * s], wb[2 * s], wa[2 * s + 1], wb[2 * s + 1], b0, b1);
      }
      const bool va = ta < ntok, vb = tb < ntok;
      sacc[m][0] = va ? sacc[m][0] * qk_scale : -INFINITY;
      sacc[m][1] = va ? sacc[m][1] * qk_scale : -INFINITY;
      sacc[m][2] = vb ? sacc[m][2] * qk_scale : -INFINITY;
      sacc[m][3] = vb ? sacc[m][3] * qk_scale : -INFINITY;
    }
    uint32_t svw[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) svw[t] = 0x3C00u;  // scale 1.0, zero-point 0
    softmax_and_stage(st, sacc, svw, ps, g_, q_);
    // values: rows = channels 16 g_ + m / m + 8, k-step s: tokens 16 s + q_ + 4 e
#pragma unroll 1
    for (int s = 0; s < 8; ++s) {
      uint4 v[4][2];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = 16 * s + q_ + 4 * e;
        if (t < ntok) {
          const uint4* r = reinterpret_cast<const uint4*>(row(false, t) + 16 * g_);
          v[e][0] = r[0]; v[e][1] = r[1];
        } else {
          v[e][0] = v[e][1] = make_uint4(0, 0, 0, 0);
        }
      }
      uint32_t b0, b1;
      load_pfrag(b0, b1, ps, s, lane);
      const uint32_t* w0 = reinterpret_cast<const uint32_t*>(v[0]);
      const uint32_t* w1 = reinterpret_cast<const uint32_t*>(v[1]);
      const uint32_t* w2 = reinterpret_cast<const uint32_t*>(v[2]);
      const uint32_t* w3 = reinterpret_cast<const uint32_t*>(v[3]);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        // channel m (and m + 8) of the 16-channel slice: word m / 2, half m & 1
        const uint32_t sel = (m & 1) ? 0x7632u : 0x5410u;
        mma16816(st.o[m], prmt(w0[m >> 1], w1[m >> 1], sel), prmt(w0[(m + 8) >> 1], w1[(m + 8) >> 1], sel),
                 prmt(w2[m >> 1], w3[m >> 1], sel), prmt(w2[(m + 8) >> 1], w3[(m + 8) >> 1], sel), b0, b1);
      }
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
decode_mma_kernel(const KittyDecodeArgs a, DecodePlan plan) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.d_boost, H = a.num_kv_heads, B = a.batch;
  const int g = a.num_q_heads / H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g_ = lane >> 2, q_ = lane & 3;
  const WarpLayout L = warp_layout(K);
  uint8_t* wsm = smem + warp * L.size;
  uint8_t* kbuf = wsm + L.kbuf;
  uint8_t* vbuf = wsm + L.vbuf;
  __half* ps = reinterpret_cast<__half*>(wsm + L.ps);
  const uint16_t* blist = reinterpret_cast<const uint16_t*>(wsm + L.blist);
  const __half* qnat = reinterpret_cast<const __half*>(wsm + L.qnat);
  const uint2* qfrag = reinterpret_cast<const uint2*>(wsm + L.qfrag);
  const uint32_t bar_k = smem_u32(wsm + L.bars), bar_v = bar_k + 8;

  // ---- this warp's slice of the item space
  const int64_t gw = int64_t(blockIdx.x) * kWarps + warp;
  const int64_t n_warps = int64_t(gridDim.x) * kWarps;
  SegmentScan sc = scan_segments(a, B, H, 0, lane);
  const int64_t total = sc.total;
  int64_t F = (total + n_warps - 1) / n_warps;
  if (F < plan.pages_per_split) F = plan.pages_per_split;
  const int64_t f0 = gw * F;
  if (f0 >= total) return;
  const int64_t f1 = min(total, f0 + F);
  sc = scan_segments(a, B, H, f0, lane);
  Cursor pos;   // the item being processed
  make_cursor(pos, a, sc.seg_begin, sc.b, sc.h, sc.u);
  int slot = int(gw - sc.seg_begin / F);

  if (lane == 0) {
    mbar_init(bar_k, 1);
    mbar_init(bar_v, 1);
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncwarp();

  const float qk_scale = a.sm_scale * kLog2e;
  const int64_t ph_low = int64_t(kD) * (kG / 4), ph_high = int64_t(K) * (kG / 4);
  const uint32_t bytes_high = uint32_t(ph_high);
  const uint32_t k_tx = 4096u + 512u + bytes_high, v_tx = 4096u + 512u;
  uint32_t k_phase = 0, v_phase = 0;
  bool failed = false;

  // physical page of page item pp (>= n16) of sequence bb; out-of-range entries fetch page 0 and are skipped
  auto phys = [&](int bb, int pp, int n16) -> int64_t { return a.block_table[bb * a.bt_s_seq + (pp - n16)]; };
  auto issue_k = [&](const Cursor& c) {
    int64_t page = phys(c.s, c.p, c.n16);
    if (page < 0 || page >= a.pool_pages) page = 0;
    const int64_t phh = page * H + c.h;
    mbar_arrive_expect_tx(bar_k, k_tx);
    bulk_g2s(smem_u32(kbuf), a.key_low + phh * ph_low, 4096u, bar_k);
    bulk_g2s(smem_u32(kbuf + 4096), reinterpret_cast<const uint8_t*>(a.key_meta) + phh * (2 * kD * 2), 512u, bar_k);
    if (bytes_high) bulk_g2s(smem_u32(kbuf + 4608), a.key_high + phh * ph_high, bytes_high, bar_k);
  };
  auto issue_v = [&](const Cursor& c) {
    int64_t page = phys(c.s, c.p, c.n16);
    if (page < 0 || page >= a.pool_pages) page = 0;
    const int64_t phh = page * H + c.h;
    mbar_arrive_expect_tx(bar_v, v_tx);
    bulk_g2s(smem_u32(vbuf), a.val_codes + phh * ph_low, 4096u, bar_v);
    bulk_g2s(smem_u32(vbuf + 4096), reinterpret_cast<const uint8_t*>(a.val_meta) + phh * (2 * kG * 2), 512u, bar_v);
  };

  Cursor cur = pos;
  bool have_next = cursor_to_page(cur, a, f1);
  if (lane == 0 && have_next) { issue_k(cur); issue_v(cur); }
  __syncwarp();

  WarpState st;
  reset_state(st);
  int nb = setup_segment(a, pos.b, pos.h, g, wsm, L, lane);

  for (int64_t f = f0; f < f1; ++f) {
    const int b = pos.b, h = pos.h;
    if (pos.p < pos.n16) {
      int t0, t1;
      fp16_chunk(fp16_tokens(a, pos.s), pos.n16, pos.p, t0, t1);
      process_fp16_region(a, b, h, st, wsm, L, qk_scale, lane, t0, t1);
    } else {
      // this page is the producer cursor's current page
      const int64_t page = phys(pos.s, pos.p, pos.n16);
      const bool valid = page >= 0 && page < a.pool_pages;
      if (!mbar_wait(bar_k, k_phase)) { failed = true; break; }
      k_phase ^= 1u;
      const uint8_t* km = kbuf + 4096;   // scale[128] fp16, zero[128] fp16
      const uint8_t* kh = kbuf + 4608;
      float sacc[8][4];
#pragma unroll
      for (int m = 0; m < 8; ++m) sacc[m][0] = sacc[m][1] = sacc[m][2] = sacc[m][3] = 0.f;
      float zk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int s = 0; s < 8; ++s) {
        const int c0 = 16 * s + q_;
        const uint32_t sk_lo = pack16(lds16(km + 2 * c0), lds16(km + 2 * (c0 + 4)));
        const uint32_t sk_hi = pack16(lds16(km + 2 * (c0 + 8)), lds16(km + 2 * (c0 + 12)));
        const uint2 qq = qfrag[s * 32 + lane];
        uint32_t b0, b1, c0l, c1l;
        hmul2_split(qq.x, sk_lo, b0, c0l);
        hmul2_split(qq.y, sk_hi, b1, c1l);
        const uint8_t* rowp = kbuf + c0 * 32 + g_ * 4;
        plane_kstep<true>(sacc, lds32(rowp), lds32(rowp + 4 * 32), lds32(rowp + 8 * 32), lds32(rowp + 12 * 32),
                          b0, b1, c0l, c1l);
        uint32_t z0 = 0u, z2 = 0u;
        if (g_ == 0) {
          const uint8_t* zr = km + 256;
          z0 = pack16(lds16(zr + 2 * c0), lds16(zr + 2 * (c0 + 4)));
          z2 = pack16(lds16(zr + 2 * (c0 + 8)), lds16(zr + 2 * (c0 + 12)));
        }
        mma16816(zk, z0, 0u, z2, 0u, b0, b1);
        mma16816(zk, z0, 0u, z2, 0u, c0l, c1l);
      }
      for (int hs = 0; hs < (nb + 15) >> 4; ++hs) {
        uint32_t w[4], qv[4], sv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int vi = 16 * hs + q_ + 4 * e;
          w[e] = 0u; qv[e] = 0u; sv[e] = 0u;
          if (vi < nb) {
            const uint32_t ent = blist[vi];
            const int c = ent & 0xff, r = ent >> 8;
            w[e] = lds32(kh + r * 32 + g_ * 4);
            qv[e] = reinterpret_cast<const uint16_t*>(qnat)[g_ * kD + c];
            sv[e] = lds16(km + 2 * c);
          }
        }
        uint32_t b0, b1, c0l, c1l;   // 4 * q * scale as hi + lo (scaling by 4 is exact)
        hmul2_split(pack16(qv[0], qv[1]), pack16(sv[0], sv[1]), b0, c0l);
        hmul2_split(pack16(qv[2], qv[3]), pack16(sv[2], sv[3]), b1, c1l);
        b0 = hmul2_u32(b0, 0x44004400u); c0l = hmul2_u32(c0l, 0x44004400u);
        b1 = hmul2_u32(b1, 0x44004400u); c1l = hmul2_u32(c1l, 0x44004400u);
        plane_kstep<true>(sacc, w[0], w[1], w[2], w[3], b0, b1, c0l, c1l);
      }
      __syncwarp();
      // keys consumed: request the next page's keys
      have_next = cursor_step(cur, a) && cursor_to_page(cur, a, f1);
      if (lane == 0 && have_next) issue_k(cur);

      const float zk0 = __shfl_sync(0xffffffffu, zk[0], q_);
      const float zk1 = __shfl_sync(0xffffffffu, zk[1], q_);
      const float off0 = -zk0 * qk_scale, off1 = -zk1 * qk_scale;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        sacc[m][0] = fmaf(sacc[m][0], qk_scale, off0);
        sacc[m][1] = fmaf(sacc[m][1], qk_scale, off1);
        sacc[m][2] = fmaf(sacc[m][2], qk_scale, off0);
        sacc[m][3] = fmaf(sacc[m][3], qk_scale, off1);
      }
      if (!mbar_wait(bar_v, v_phase)) { failed = true; break; }
      v_phase ^= 1u;
      const uint8_t* vm = vbuf + 4096;   // [t](scale, zero) fp16
      if (valid) {
        uint32_t svw[16];
        const uint4* v4 = reinterpret_cast<const uint4*>(vm + 16 * g_ * 4);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint4 x = v4[t];
          svw[4 * t] = x.x; svw[4 * t + 1] = x.y; svw[4 * t + 2] = x.z; svw[4 * t + 3] = x.w;
        }
        softmax_and_stage(st, sacc, svw, ps, g_, q_);
#pragma unroll 1
        for (int s = 0; s < 8; ++s) {
          const int t0 = 16 * s + q_;
          uint32_t b0, b1;
          load_pfrag(b0, b1, ps, s, lane);
          const uint8_t* rowp = vbuf + t0 * 32 + g_ * 4;
          plane_kstep<false>(st.o, lds32(rowp), lds32(rowp + 4 * 32), lds32(rowp + 8 * 32), lds32(rowp + 12 * 32),
                             b0, b1);
          uint32_t z0 = 0u, z2 = 0u;
          if (g_ == 0) {
            z0 = pack16(lds16(vm + 4 * t0 + 2), lds16(vm + 4 * (t0 + 4) + 2));
            z2 = pack16(lds16(vm + 4 * (t0 + 8) + 2), lds16(vm + 4 * (t0 + 12) + 2));
          }
          mma16816(st.zv, z0, 0u, z2, 0u, b0, b1);
        }
      }
      __syncwarp();
      // values consumed: request the next page's values
      if (lane == 0 && have_next) issue_v(cur);
    }

    // ---- advance; write the partial at a segment end or at the end of the slice
    const bool seg_end = pos.p + 1 >= pos.items;
    if (seg_end || f + 1 == f1) {
      float l0 = st.l[0], l1 = st.l[1];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
      }
      const float zv0 = __shfl_sync(0xffffffffu, st.zv[0], q_);
      const float zv1 = __shfl_sync(0xffffffffu, st.zv[1], q_);
      const int64_t base = ((int64_t(b) * H + h) * plan.num_splits + slot) * g;
      const int qa = 2 * q_, qb = 2 * q_ + 1;
      if (qa < g) {
        float* o = plan.ws_o + (base + qa) * kD + 16 * g_;
#pragma unroll
        for (int m = 0; m < 8; ++m) { o[m] = st.o[m][0] - zv0; o[m + 8] = st.o[m][2] - zv0; }
        if (g_ == 0) {
          plan.ws_m[base + qa] = st.m[0] == -INFINITY ? -INFINITY : st.m[0] * kLn2;
          plan.ws_l[base + qa] = l0;
        }
      }
      if (qb < g) {
        float* o = plan.ws_o + (base + qb) * kD + 16 * g_;
#pragma unroll
        for (int m = 0; m < 8; ++m) { o[m] = st.o[m][1] - zv1; o[m + 8] = st.o[m][3] - zv1; }
        if (g_ == 0) {
          plan.ws_m[base + qb] = st.m[1] == -INFINITY ? -INFINITY : st.m[1] * kLn2;
          plan.ws_l[base + qb] = l1;
        }
      }
      if (seg_end && lane == 0) plan.ws_count[int64_t(b) * H + h] = slot + 1;
      reset_state(st);
    }
    if (f + 1 < f1) {
      cursor_step(pos, a);
      if (seg_end) {
        slot = 0;
        __syncwarp();
        nb = setup_segment(a, pos.b, pos.h, g, wsm, L, lane);
      }
    }
  }
  if (failed) {
    if (lane == 0) atomicOr(&g_decode_error, 1u);
    // copies still in flight must land before the CTA's shared memory is released
    mbar_wait(bar_k, k_phase);
    mbar_wait(bar_v, v_phase);
  }
}

}  // namespace

bool mma_supports(const KittyDecodeArgs& a) {
  if (a.dtype != KITTY_DTYPE_F16) return false;   // fp16 operands only
  const int g = a.num_q_heads / a.num_kv_heads;
  auto region_ok = [](const void* p, int64_t s_seq, int64_t s_head, int64_t s_tok) {
    return p == nullptr || (aligned(p, 16) && s_seq % 8 == 0 && s_head % 8 == 0 && s_tok % 8 == 0);
  };
  return a.head_dim == kD && a.group == kG && g >= 1 && g <= 8 && a.d_boost <= 128 &&
         aligned(a.q, 16) && a.q_s_seq % 8 == 0 && a.q_s_head % 8 == 0 &&
         region_ok(a.sink_k, a.sk_s_seq, a.sk_s_head, a.sk_s_tok) &&
         region_ok(a.sink_v, a.sv_s_seq, a.sv_s_head, a.sv_s_tok) &&
         region_ok(a.tail_k, a.tk_s_seq, a.tk_s_head, a.tk_s_tok) &&
         region_ok(a.tail_v, a.tv_s_seq, a.tv_s_head, a.tv_s_tok) &&
         (a.max_pages_per_seq == 0 ||
          (aligned(a.key_low, 16) && aligned(a.key_meta, 16) && aligned(a.val_codes, 16) &&
           aligned(a.val_meta, 16) && (a.d_boost == 0 || aligned(a.key_high, 16))));
}

int mma_ctas_per_sm() { return kCtasPerSm; }

// Slots per segment S = num_splits (default kSlotsTarget, more when there are fewer
// segment items than warps need for a full grid): every warp takes at least
// F_min = ceil(items_max / S) items, so a segment spans at most ceil(items_max / F_min)
// + 1 warps, which is the slot count the merge reads.
void mma_plan(const KittyDecodeArgs& a, int sm_count, DecodePlan* plan) {
  const int items_max = a.max_pages_per_seq + dev::kMaxFp16Items;   // pages + fp16 chunk items
  // few segments (small batch, few KV heads per GPU): more slots per segment so that
  // every warp of the persistent grid gets a slice
  const int64_t warps = int64_t(sm_count) * kCtasPerSm * kWarps;
  const int64_t per_warp = std::max<int64_t>(1, int64_t(a.batch) * a.num_kv_heads * items_max / warps);
  const int auto_target = int(std::max<int64_t>(kSlotsTarget, (items_max + per_warp - 1) / per_warp));
  int target = a.num_splits > 0 ? a.num_splits : auto_target;
  target = std::max(1, std::min({target, items_max, kMaxDecodeSlots - 1}));
  const int f_min = (items_max + target - 1) / target;
  plan->pages_per_split = f_min;
  plan->num_splits = (items_max + f_min - 1) / f_min + 1;
  const int64_t total_max = int64_t(a.batch) * a.num_kv_heads * items_max;
  const int64_t warps_needed = (total_max + f_min - 1) / f_min;
  const int64_t ctas = std::min<int64_t>((warps_needed + kWarps - 1) / kWarps, int64_t(sm_count) * kCtasPerSm);
  plan->grid = int(std::max<int64_t>(1, ctas));
}

int launch_decode_mma(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  const WarpLayout L = warp_layout(a.d_boost);
  const int smem = kWarps * L.size;
  static int configured_bytes = 0;
  if (configured_bytes < smem) {
    cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("decode_mma smem attribute: ") + cudaGetErrorString(e));
    configured_bytes = smem;
  }
  decode_mma_kernel<<<plan.grid, kThreads, smem, stream>>>(a, plan);
  return check_launch("decode_mma_kernel");
}

int read_decode_error(uint32_t* flags, int clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_decode_error, sizeof(v));
  if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("read error flags: ") + cudaGetErrorString(e));
  if (clear && v) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_decode_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("clear error flags: ") + cudaGetErrorString(e));
  }
  *flags = v;
  return KITTY_OK;
}

}  // namespace kitty
