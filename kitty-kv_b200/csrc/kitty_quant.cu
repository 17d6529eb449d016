// Page quantise/pack kernels (key: per channel, dense-sparse INT2/INT4;
// value: per token INT2) and key page dequantisation.
//
// Arithmetic follows the reference's PyTorch path operation by operation in
// IEEE float32 (kitty/kernels/quantize_key.py:69-124,
// kitty/kernels/quantize_value.py:50-90): divisions are correctly rounded
// (__fdiv_rn), rounding is half-to-even (rintf), and the stored scale is the
// float32 scale rounded to fp16 (then to bf16 for a bfloat16 cache, as the
// reference's copy into bf16 pool views does).  The packed planes are therefore
// bit-exact.  Every kernel is instantiated for fp16 and bf16 sources (Half16).
//
// One CTA handles one page-head.  The general kernels stage the G x D fp16
// block in shared memory, reduce per channel (keys) or per token (values),
// then quantise and pack four 2-bit codes per byte into the pool slice; the
// D = G = 128 kernels keep the block in registers (see below).

#include "kitty_common.cuh"
#include "kitty_ptx.cuh"

namespace kitty {
namespace {

using dev::fma2;
using dev::prmt;

#ifndef KITTY_Q_MINB
#define KITTY_Q_MINB 4    // resident CTAs of the D = G = 128 quantisers the register budget is set for
#endif
#ifndef KITTY_Q_PAIRS
#define KITTY_Q_PAIRS 1   // the fixed-point rounding on packed fp32 pairs (0: scalar FMAs)
#endif

constexpr int kQuantThreads = 256;

// Stage the (G tokens x D channels) fp16 block of job j / head h into
// shared memory as tile[t * D + c].
__device__ __forceinline__ void stage_block(uint16_t* tile, const uint16_t* src, int64_t s_tok,
                                            int64_t s_ch, int G, int D, int n_valid) {
  const int tid = threadIdx.x;
  const bool vec = (s_ch == 1) && (D % 8 == 0) && ((s_tok % 8) == 0) &&
                   ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
  if (vec) {
    const int chunks_per_row = D / 8;
    const int total = G * chunks_per_row;
    for (int i = tid; i < total; i += blockDim.x) {
      const int t = i / chunks_per_row;
      const int c8 = (i - t * chunks_per_row) * 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (t < n_valid) v = *reinterpret_cast<const uint4*>(src + t * s_tok + c8);
      *reinterpret_cast<uint4*>(tile + t * D + c8) = v;
    }
  } else {
    const int total = G * D;
    for (int i = tid; i < total; i += blockDim.x) {
      const int t = i / D;
      const int c = i - t * D;
      tile[i] = (t < n_valid) ? src[t * s_tok + c * s_ch] : uint16_t(0);
    }
  }
}

template <bool kBf16, bool kMetaBf16>
__global__ void __launch_bounds__(kQuantThreads)
quantize_key_kernel(const KittyKeyQuantArgs a) {
  using T = Half16<kBf16>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int D = a.head_dim, G = a.group, K = a.d_boost;
  const int job = blockIdx.x / a.num_heads;
  const int h = blockIdx.x - job * a.num_heads;
  const int G4 = G / 4;

  uint16_t* tile = reinterpret_cast<uint16_t*>(smem);                        // G*D fp16
  float* s_scale = reinterpret_cast<float*>(smem + ((size_t(G) * D * 2 + 15) & ~size_t(15)));
  float* s_zp = s_scale + D;
  float* s_maxq = s_zp + D;
  int* s_row = reinterpret_cast<int*>(s_maxq + D);                          // high row or -1
  uint32_t* s_high = reinterpret_cast<uint32_t*>(s_row + D);                // K*G4 bytes as words

  const uint16_t* src = reinterpret_cast<const uint16_t*>(a.key) + a.key_off[job] + h * a.key_s_head;
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  const int64_t page = a.dst_page[job];
  if (page < 0) return;   // skipped job (a batched append flushes only full buffers)

  stage_block(tile, src, a.key_s_tok, a.key_s_ch, G, D, G);
  const int high_words = (K * G4 + 3) / 4;
  for (int i = threadIdx.x; i < high_words; i += blockDim.x) s_high[i] = 0u;
  __syncthreads();

  uint16_t* out_scale = reinterpret_cast<uint16_t*>(a.key_scale) + page * a.meta_s_page + h * a.meta_s_head;
  uint16_t* out_zero = reinterpret_cast<uint16_t*>(a.key_zero) + page * a.meta_s_page + h * a.meta_s_head;

  // Per-channel statistics (quantize_key.py:73-87).
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float mn = T::to_f(tile[c]), mx = mn;
    for (int t = 1; t < G; ++t) {
      const float x = T::to_f(tile[t * D + c]);
      mn = tmin(mn, x);
      mx = tmax(mx, x);
    }
    const int b = bidx[c];
    const bool boosted = b < a.sentinel;
    const float maxq = boosted ? 15.0f : 3.0f;
    const float range = clamp_min(mx - mn, 1e-8f);
    const float scale = __fdiv_rn(range, maxq);
    float zp = rintf(__fdiv_rn(-mn, scale));
    zp = tmin(tmax(zp, 0.0f), maxq);
    s_scale[c] = scale;
    s_zp[c] = zp;
    s_maxq[c] = maxq;
    s_row[c] = (boosted && b < K) ? b : -1;
    out_scale[c] = Half16<kMetaBf16>::meta(scale);
    out_zero[c] = Half16<kMetaBf16>::meta(zp);
  }
  __syncthreads();

  // Quantise and pack: byte (c, j) holds tokens 4j..4j+3 (quantize_key.py:95-119).
  uint8_t* out_low = a.key_low + page * a.low_s_page + h * a.low_s_head;
  for (int i = threadIdx.x; i < D * G4; i += blockDim.x) {
    const int c = i / G4;
    const int j = i - c * G4;
    const float scale = s_scale[c], zp = s_zp[c], maxq = s_maxq[c];
    uint32_t low = 0u, high = 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = T::to_f(tile[(4 * j + k) * D + c]);
      float q = rintf(__fdiv_rn(x, scale)) + zp;
      q = tmin(tmax(q, 0.0f), maxq);
      const uint32_t code = to_code(q);
      low |= (code & 3u) << (2 * k);
      high |= ((code >> 2) & 3u) << (2 * k);
    }
    out_low[i] = static_cast<uint8_t>(low);
    const int r = s_row[c];
    if (r >= 0 && high != 0u) {
      const int byte = r * G4 + j;
      atomicOr(&s_high[byte >> 2], high << (8 * (byte & 3)));
    }
  }
  __syncthreads();

  uint8_t* out_high = a.key_high + page * a.high_s_page + h * a.high_s_head;
  const uint8_t* sh = reinterpret_cast<const uint8_t*>(s_high);
  for (int i = threadIdx.x; i < K * G4; i += blockDim.x) out_high[i] = sh[i];
}

template <bool kBf16, bool kMetaBf16>
__global__ void __launch_bounds__(kQuantThreads)
quantize_value_kernel(const KittyValueQuantArgs a) {
  using T = Half16<kBf16>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int D = a.head_dim, G = a.group;
  const int job = blockIdx.x / a.num_heads;
  const int h = blockIdx.x - job * a.num_heads;
  const int D4 = D / 4;

  uint16_t* tile = reinterpret_cast<uint16_t*>(smem);
  float* s_scale = reinterpret_cast<float*>(smem + ((size_t(G) * D * 2 + 15) & ~size_t(15)));
  float* s_zp = s_scale + G;

  const uint16_t* src = reinterpret_cast<const uint16_t*>(a.value) + a.value_off[job] + h * a.val_s_head;
  const int n_valid = a.n_valid ? a.n_valid[job] : G;
  const int64_t page = a.dst_page[job];
  if (page < 0) return;   // skipped job (a batched append flushes only full buffers)
  stage_block(tile, src, a.val_s_tok, a.val_s_ch, G, D, n_valid);
  __syncthreads();

  uint16_t* out_scale = reinterpret_cast<uint16_t*>(a.val_scale) + page * a.meta_s_page + h * a.meta_s_head;
  uint16_t* out_zero = reinterpret_cast<uint16_t*>(a.val_zero) + page * a.meta_s_page + h * a.meta_s_head;

  // Per-token statistics (quantize_value.py:62-72): a warp per token, lanes over channels.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int t = warp; t < G; t += nwarps) {
    float mn = T::to_f(tile[t * D + (lane < D ? lane : 0)]), mx = mn;
    for (int c = lane + 32; c < D; c += 32) {
      const float x = T::to_f(tile[t * D + c]);
      mn = tmin(mn, x);
      mx = tmax(mx, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = tmin(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = tmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) {
      const float range = clamp_min(mx - mn, 1e-8f);
      const float scale = __fdiv_rn(range, 3.0f);
      float zp = rintf(__fdiv_rn(-mn, scale));
      zp = tmin(tmax(zp, 0.0f), 3.0f);
      s_scale[t] = scale;
      s_zp[t] = zp;
      out_scale[t * a.meta_s_tok] = Half16<kMetaBf16>::meta(scale);
      out_zero[t * a.meta_s_tok] = Half16<kMetaBf16>::meta(zp);
    }
  }
  __syncthreads();

  // Quantise and pack: byte (t, j) holds channels 4j..4j+3 (quantize_value.py:77-86).
  uint8_t* out = a.val_codes + page * a.codes_s_page + h * a.codes_s_head;
  for (int i = threadIdx.x; i < G * D4; i += blockDim.x) {
    const int t = i / D4;
    const int j = i - t * D4;
    const float scale = s_scale[t], zp = s_zp[t];
    uint32_t byte = 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = T::to_f(tile[t * D + 4 * j + k]);
      float q = rintf(__fdiv_rn(x, scale)) + zp;
      q = tmin(tmax(q, 0.0f), 3.0f);
      byte |= (to_code(q) & 3u) << (2 * k);
    }
    out[i] = static_cast<uint8_t>(byte);
  }
}

// Element store of the dequantisers: the metadata's 16-bit type, or float32.
template <bool kBf16, bool kF32Out>
__device__ __forceinline__ void store_dq(void* out, int64_t idx, float x) {
  if constexpr (kF32Out) reinterpret_cast<float*>(out)[idx] = x;
  else reinterpret_cast<uint16_t*>(out)[idx] = Half16<kBf16>::from_f(x);
}

template <bool kBf16, bool kF32Out>
__global__ void dequantize_key_kernel(const KittyKeyDequantArgs a) {
  using T = Half16<kBf16>;
  const int D = a.head_dim, G = a.group, K = a.d_boost, G4 = G / 4;
  const int job = blockIdx.x;
  const int64_t page = a.src_page[job];
  const int h = a.head[job];
  const uint8_t* low = a.key_low + page * a.low_s_page + h * a.low_s_head;
  const uint8_t* high = a.key_high + page * a.high_s_page + h * a.high_s_head;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(a.key_scale) + page * a.meta_s_page + h * a.meta_s_head;
  const uint16_t* zr = reinterpret_cast<const uint16_t*>(a.key_zero) + page * a.meta_s_page + h * a.meta_s_head;
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  const int64_t base = a.out_off[job];
  // dequantize_key.py:69-97: code = low | (high << 2) when boost_idx < d_boost.
  for (int i = threadIdx.x; i < D * G4; i += blockDim.x) {
    const int c = i / G4;
    const int j = i - c * G4;
    const int b = bidx[c];
    const uint32_t lo = low[i];
    const uint32_t hi = (b < K) ? high[b * G4 + j] : 0u;
    const float s = T::to_f(sc[c]), z = T::to_f(zr[c]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t code = ((lo >> (2 * k)) & 3u) | (((hi >> (2 * k)) & 3u) << 2);
      const float x = __fmul_rn(__fsub_rn(static_cast<float>(code), z), s);
      store_dq<kBf16, kF32Out>(a.out, base + c * a.out_s_ch + (4 * j + k) * a.out_s_tok, x);
    }
  }
}

// quantize_value.py:122-133: codes unpacked per token (byte j of token t holds
// channels 4j..4j+3 at bits 0,2,4,6), x = (code - zp_t) * scale_t in float32.
template <bool kBf16, bool kF32Out>
__global__ void dequantize_value_kernel(const KittyValueDequantArgs a) {
  using T = Half16<kBf16>;
  const int D4 = a.head_dim / 4, G = a.group;
  const int job = blockIdx.x;
  const int64_t page = a.src_page[job];
  const int h = a.head[job];
  const uint8_t* codes = a.val_codes + page * a.codes_s_page + h * a.codes_s_head;
  const int64_t m0 = page * a.meta_s_page + h * a.meta_s_head;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(a.val_scale) + m0;
  const uint16_t* zr = reinterpret_cast<const uint16_t*>(a.val_zero) + m0;
  const int64_t base = a.out_off[job];
  for (int i = threadIdx.x; i < G * D4; i += blockDim.x) {
    const int t = i / D4;
    const int j = i - t * D4;
    const uint32_t byte = codes[i];
    const float s = T::to_f(sc[int64_t(t) * a.meta_s_tok]), z = T::to_f(zr[int64_t(t) * a.meta_s_tok]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = __fmul_rn(__fsub_rn(static_cast<float>((byte >> (2 * k)) & 3u), z), s);
      store_dq<kBf16, kF32Out>(a.out, base + t * a.out_s_tok + (4 * j + k) * a.out_s_ch, x);
    }
  }
}

// ---------------------------------------------------------------------------
// D = G = 128 fast paths.  256 threads: thread (tg = tid >> 4, cg = tid & 15)
// holds tokens 8*tg .. 8*tg+7 x channels 8*cg .. 8*cg+7 of the page-head in
// registers (eight 16-byte loads, coalesced: a half-warp reads one 256-byte
// token row).  Min / max are taken on packed halves (exact, NaN-propagating),
// the statistics follow the reference's float32 sequence, and the packed
// planes are staged in shared memory so every global store is 16 bytes wide.
// ---------------------------------------------------------------------------

constexpr int kFastThreads = 256;
constexpr float kMagic = 12582912.0f;          // 1.5 * 2^23: fma(x, r, kMagic + zp) = kMagic + zp + rint(x r)
constexpr float kNearHalf = 0.49996948f;       // 0.5 - 2^-15

struct Tile8x8 {
  uint4 row[8];  // row[i] = 8 channels (fp16) of token 8*tg + i
};

// The job offset comes from device memory, so 16-byte alignment of the rows is
// checked here (uniform per CTA); unaligned sources take 16-bit loads.
__device__ __forceinline__ void load_tile(Tile8x8& t, const uint16_t* src, int64_t s_tok, int tg, int cg,
                                          int n_valid) {
  const bool vec = ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int tok = 8 * tg + i;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (tok < n_valid) {
      const uint16_t* p = src + tok * s_tok + 8 * cg;
      if (vec) {
        v = *reinterpret_cast<const uint4*>(p);
      } else {
        v.x = uint32_t(p[0]) | (uint32_t(p[1]) << 16); v.y = uint32_t(p[2]) | (uint32_t(p[3]) << 16);
        v.z = uint32_t(p[4]) | (uint32_t(p[5]) << 16); v.w = uint32_t(p[6]) | (uint32_t(p[7]) << 16);
      }
    }
    t.row[i] = v;
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int w) {
  return w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
}

// code of x (fp32 of an fp16) with the reference's arithmetic, exact IEEE division;
// handles non-finite statistics (NaN codes become 0)
__device__ __forceinline__ uint32_t quant_code(float x, float scale, float zp, float maxq) {
  float q = rintf(__fdiv_rn(x, scale)) + zp;
  q = tmin(tmax(q, 0.0f), maxq);
  return to_code(q);
}

// Fast codes of an fp16 pair.  fma(x, r, kMagic + zp) with r = __frcp_rn(scale) holds
// kMagic + zp + rint(x r) (one rounding of the exact product); x r is within
// 2^-23 |x / scale| of the correctly rounded quotient, so rint agrees with the
// reference's rintf(x / scale) unless x r is within 2^-15 of a half-integer (for
// |x / scale| < 64; beyond that every rounding clamps to the same code).  Such
// elements - in practice quotients that are exact half-integers, ~1e-4 of the
// elements - set their bit in the near-tie masks (bits b0, b1) and are recomputed
// with the exact division by the caller.  The clamp to [0, maxq] is taken on the
// biased floats, so the low byte of each result is the code.  Statistics must be
// finite.
template <bool kBf16>
__device__ __forceinline__ void fast_pair(uint32_t hx, float2 r, float2 mz, float2 top, uint32_t& mask, uint32_t b0,
                                          uint32_t b1, uint32_t& c0, uint32_t& c1) {
  const float2 x = Half16<kBf16>::to_f2(hx);
  const float f0 = __fmaf_rn(x.x, r.x, mz.x), f1 = __fmaf_rn(x.y, r.y, mz.y);
  const float e0 = __fmaf_rn(x.x, r.x, mz.x - f0), e1 = __fmaf_rn(x.y, r.y, mz.y - f1);   // x r - rint(x r)
  if (fabsf(e0) > kNearHalf) mask |= b0;
  if (fabsf(e1) > kNearHalf) mask |= b1;
  c0 = __float_as_uint(fminf(fmaxf(f0, kMagic), top.x));
  c1 = __float_as_uint(fminf(fmaxf(f1, kMagic), top.y));
}

// Fast codes of an fp16 pair in one word: lane k (16 bits) = code of element k, clamped
// to [0, maxq] as signed 16-bit integers.  Same rounding as fast_pair (fma(x, r, kMagic +
// zp) = kMagic + zp + rint(x r), on fp32 pairs), one near-tie test for the pair (the
// larger rounding distance; both elements are recomputed exactly when it is near a
// half-integer).  Valid while |zp + rint(x r)| < 2^15: the caller routes channels whose
// |x| / scale can reach 16000 (near-constant channels far from zero) to fast_pair.
template <bool kBf16>
__device__ __forceinline__ uint32_t fast_pair16(uint32_t hx, float2 r, float2 mz, uint32_t lim, bool& tie) {
  const float2 x = Half16<kBf16>::to_f2(hx);
#if KITTY_Q_PAIRS
  const float2 f = fma2(x, r, mz);                               // kMagic + zp + rint(x r)
  const float2 t = fma2(f, make_float2(-1.0f, -1.0f), mz);       // -rint(x r), exact
  const float2 e = fma2(x, r, t);                                // x r - rint(x r)
#else
  const float2 f = make_float2(__fmaf_rn(x.x, r.x, mz.x), __fmaf_rn(x.y, r.y, mz.y));   // kMagic + zp + rint(x r)
  const float2 e = make_float2(__fmaf_rn(x.x, r.x, mz.x - f.x), __fmaf_rn(x.y, r.y, mz.y - f.y));   // x r - rint(x r)
#endif
  tie |= fmaxf(fabsf(e.x), fabsf(e.y)) > kNearHalf;
  uint32_t w, v;
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(w) : "r"(__float_as_uint(f.x)), "r"(__float_as_uint(f.y)));
  asm("max.s16x2 %0, %1, %2;" : "=r"(v) : "r"(w), "r"(0u));
  asm("min.s16x2 %0, %1, %2;" : "=r"(w) : "r"(v), "r"(lim));
  return w;
}

// Exact codes of the flagged elements of one 8-element row (bit j of `flags` =
// element j; element j's fp16 value at src[j * stride]); patches the 2-bit fields
// of lo (bits 0-1 of each code) and hi (bits 2-3).  Rare: kept out of line.
template <bool kBf16>
__device__ __noinline__ uint2 patch_row(uint32_t flags, const uint16_t* src, int64_t stride, float scale, float zp,
                                        float maxq, uint32_t lo, uint32_t hi) {
  for (int j = 0; j < 8; ++j) {
    if (!((flags >> j) & 1u)) continue;
    const uint32_t code = quant_code(Half16<kBf16>::to_f(src[j * stride]), scale, zp, maxq);
    lo = (lo & ~(3u << (2 * j))) | ((code & 3u) << (2 * j));
    hi = (hi & ~(3u << (2 * j))) | (((code >> 2) & 3u) << (2 * j));
  }
  return make_uint2(lo, hi);
}

// low plane byte of channel c, token word j (tokens 4j..4j+3) in the swizzled
// shared staging: 32-bit word (j / 4) ^ (c >> 3 & 7) of row c
__device__ __forceinline__ int low_swz(int c, int byte) {
  return c * 32 + ((((byte >> 2) ^ (c >> 3)) & 7) << 2) + (byte & 3);
}

template <bool kBf16, bool kMetaBf16>
__global__ void __launch_bounds__(kFastThreads, KITTY_Q_MINB)
quantize_key_d128_kernel(const KittyKeyQuantArgs a) {
  using T = Half16<kBf16>;
  constexpr int D = 128, G = 128, G4 = 32;
  __shared__ __align__(16) uint32_t s_red[8][64][2];   // per warp, per channel pair: (min, max) half2
  __shared__ float s_scale[D], s_zp[D], s_maxq[D], s_r[D];
  __shared__ int s_row[D];
  __shared__ int s_wide[D];   // |x| / scale can reach 16000: the 16-bit lane path does not apply
  __shared__ int s_nonfinite;
  __shared__ __align__(16) uint8_t s_low[D * G4];
  __shared__ __align__(16) uint32_t s_high[128 * G4 / 4];
  const int K = a.d_boost;
  const int job = blockIdx.x / a.num_heads;
  const int h = blockIdx.x - job * a.num_heads;
  const int tid = threadIdx.x, tg = tid >> 4, cg = tid & 15, warp = tid >> 5, lane = tid & 31;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(a.key) + a.key_off[job] + h * a.key_s_head;
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  const int64_t page = a.dst_page[job];
  if (page < 0) return;   // skipped job (a batched append flushes only full buffers)

  Tile8x8 t;
  load_tile(t, src, a.key_s_tok, tg, cg, G);
  for (int i = tid; i < K * G4 / 4; i += kFastThreads) s_high[i] = 0u;
  if (tid == 0) s_nonfinite = 0;

  // per channel-pair min / max over this thread's 8 tokens
  uint32_t mn[4], mx[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) mn[w] = mx[w] = word_of(t.row[0], w);
#pragma unroll
  for (int i = 1; i < 8; ++i)
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t v = word_of(t.row[i], w);
      mn[w] = T::min2(mn[w], v);
      mx[w] = T::max2(mx[w], v);
    }
  // lanes l and l^16 hold the other token group of the same channels
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    mn[w] = T::min2(mn[w], __shfl_xor_sync(0xffffffffu, mn[w], 16));
    mx[w] = T::max2(mx[w], __shfl_xor_sync(0xffffffffu, mx[w], 16));
  }
  if (lane < 16) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      s_red[warp][4 * cg + w][0] = mn[w];
      s_red[warp][4 * cg + w][1] = mx[w];
    }
  }
  __syncthreads();
  if (tid < D) {  // channel tid (one per thread: the divisions below run 128-wide, not 64)
    const int c = tid, pr = c >> 1;
    uint32_t a2 = s_red[0][pr][0], b2 = s_red[0][pr][1];
#pragma unroll
    for (int w = 1; w < 8; ++w) {
      a2 = T::min2(a2, s_red[w][pr][0]);
      b2 = T::max2(b2, s_red[w][pr][1]);
    }
    const float mnf = (c & 1) ? T::hi_f(a2) : T::lo_f(a2);
    const float mxf = (c & 1) ? T::hi_f(b2) : T::lo_f(b2);
    uint16_t* out_scale = reinterpret_cast<uint16_t*>(a.key_scale) + page * a.meta_s_page + h * a.meta_s_head;
    uint16_t* out_zero = reinterpret_cast<uint16_t*>(a.key_zero) + page * a.meta_s_page + h * a.meta_s_head;
    const int r = bidx[c];
    const bool boosted = r < a.sentinel;
    const float maxq = boosted ? 15.0f : 3.0f;
    const float scale = __fdiv_rn(clamp_min(mxf - mnf, 1e-8f), maxq);
    float zp = rintf(__fdiv_rn(-mnf, scale));
    zp = tmin(tmax(zp, 0.0f), maxq);
    s_scale[c] = scale; s_zp[c] = zp; s_maxq[c] = maxq; s_r[c] = __frcp_rn(scale);
    s_row[c] = (boosted && r < K) ? r : -1;
    s_wide[c] = !(fmaxf(fabsf(mnf), fabsf(mxf)) * __frcp_rn(scale) < 16000.0f);
    out_scale[c] = Half16<kMetaBf16>::meta(scale);
    out_zero[c] = Half16<kMetaBf16>::meta(zp);
    if (!(isfinite(mnf) && isfinite(mxf) && isfinite(scale))) s_nonfinite = 1;
  }
  __syncthreads();

  // quantise: channel c = 8 cg + k; this thread's 8 tokens -> 16 bits of its low / high rows
  auto store = [&](int c, uint32_t lo, uint32_t hi) {
    *reinterpret_cast<uint16_t*>(s_low + low_swz(c, 2 * tg)) = uint16_t(lo);
    const int r = s_row[c];
    if (r >= 0 && hi != 0u) {
      const int byte = r * G4 + 2 * tg;   // 2-byte aligned: never straddles a word
      atomicOr(&s_high[byte >> 2], hi << (8 * (byte & 3)));
    }
  };
  const uint16_t* my_src = src + (8 * tg) * a.key_s_tok + 8 * cg;   // this thread's tile (token-major)
  if (s_nonfinite == 0) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int c = 8 * cg + 2 * w;
      const float2 r = make_float2(s_r[c], s_r[c + 1]);
      const float2 mz = make_float2(kMagic + s_zp[c], kMagic + s_zp[c + 1]);
      // code words of channels c, c + 1 (16-bit lanes) for tokens 8 tg + i, folded as they come
      // into the low-plane (bits 0-1) and high-plane (bits 2-3) fields of tokens 0-3 / 4-7
      uint32_t l03 = 0u, l47 = 0u, h03 = 0u, h47 = 0u;
      uint32_t tie = 0u;
      auto fold = [&](int i, uint32_t wv) {
        const int sh = 2 * (i & 3);
        const uint32_t lo = (wv & 0x00030003u) << sh, hi = ((wv >> 2) & 0x00030003u) << sh;
        if (i < 4) { l03 += lo; h03 += hi; } else { l47 += lo; h47 += hi; }
      };
      if (!(s_wide[c] | s_wide[c + 1])) {
        const uint32_t lim = uint32_t(s_maxq[c]) | (uint32_t(s_maxq[c + 1]) << 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          bool ti = false;
          fold(i, fast_pair16<kBf16>(word_of(t.row[i], w), r, mz, lim, ti));
          tie |= uint32_t(ti) << i;
        }
      } else {   // codes of channels far beyond 16 bits: the fp32 clamp
        const float2 top = make_float2(kMagic + s_maxq[c], kMagic + s_maxq[c + 1]);
        uint32_t m = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint32_t ca, cb;
          fast_pair<kBf16>(word_of(t.row[i], w), r, mz, top, m, 1u << i, 1u << (8 + i), ca, cb);
          fold(i, prmt(ca, cb, 0x5410u));
        }
        tie = (m | (m >> 8)) & 0xffu;
      }
      uint32_t lo_a = prmt(l03, l47, 0x0040u) & 0xffffu, lo_b = prmt(l03, l47, 0x0062u) & 0xffffu;
      uint32_t hi_a = prmt(h03, h47, 0x0040u) & 0xffffu, hi_b = prmt(h03, h47, 0x0062u) & 0xffffu;
      if (tie) {
        uint2 p = patch_row<kBf16>(tie, my_src + 2 * w, a.key_s_tok, s_scale[c], s_zp[c], s_maxq[c], lo_a, hi_a);
        lo_a = p.x; hi_a = p.y;
        p = patch_row<kBf16>(tie, my_src + 2 * w + 1, a.key_s_tok, s_scale[c + 1], s_zp[c + 1], s_maxq[c + 1], lo_b,
                             hi_b);
        lo_b = p.x; hi_b = p.y;
      }
      store(c, lo_a, hi_a);
      store(c + 1, lo_b, hi_b);
    }
  } else {   // non-finite statistics somewhere in the page-head: the exact path throughout
#pragma unroll 1
    for (int k = 0; k < 8; ++k) {
      const int c = 8 * cg + k;
      const uint2 p = patch_row<kBf16>(0xffu, my_src + k, a.key_s_tok, s_scale[c], s_zp[c], s_maxq[c], 0u, 0u);
      store(c, p.x, p.y);
    }
  }
  __syncthreads();
  {  // row c = tid / 2, bytes 16 (tid & 1) .. +15: four swizzled words
    const int c = tid >> 1, b0 = 16 * (tid & 1);
    const uint32_t* srow = reinterpret_cast<const uint32_t*>(s_low);
    uint4 v;
    v.x = srow[low_swz(c, b0) >> 2]; v.y = srow[low_swz(c, b0 + 4) >> 2];
    v.z = srow[low_swz(c, b0 + 8) >> 2]; v.w = srow[low_swz(c, b0 + 12) >> 2];
    uint8_t* out_low = a.key_low + page * a.low_s_page + h * a.low_s_head;
    reinterpret_cast<uint4*>(out_low)[tid] = v;
  }
  uint8_t* out_high = a.key_high + page * a.high_s_page + h * a.high_s_head;
  for (int i = tid; i < K * G4 / 16; i += kFastThreads)
    reinterpret_cast<uint4*>(out_high)[i] = reinterpret_cast<const uint4*>(s_high)[i];
}

// The 8 packed bytes of 32 channels of one token (byte j = channels 4 j .. 4 j + 3 at
// bits 0,2,4,6) from their code words (lane k = code of channel 2 w + k of word w)
__device__ __forceinline__ uint2 value_bytes(const uint32_t (&wv)[16]) {
  uint32_t y[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t x = wv[2 * j] + (wv[2 * j + 1] << 4);   // (c0 + 16 c2, c1 + 16 c3) in the lanes
    y[j] = x + (x >> 14);                                  // byte 0: c0 + 4 c1 + 16 c2 + 64 c3
  }
  return make_uint2(prmt(prmt(y[0], y[1], 0x0040u), prmt(y[2], y[3], 0x0040u), 0x5410u),
                    prmt(prmt(y[4], y[5], 0x0040u), prmt(y[6], y[7], 0x0040u), 0x5410u));
}

// One token's 32 channels with per-pair near-tie flags and clamped codes: the path for
// tokens with a near-tie or a code outside 0..3 somewhere (rare), out of line.  Returns
// the packed bytes and the tie bits (bit c = channel c of the 32).
template <bool kBf16>
__device__ __noinline__ uint3 value_token_slow(uint4 a0, uint4 a1, uint4 a2, uint4 a3, float rcp, float zp,
                                               int wide) {
  const uint4 v[4] = {a0, a1, a2, a3};
  const float2 r2 = make_float2(rcp, rcp);
  const float2 mz = make_float2(kMagic + zp, kMagic + zp);
  uint32_t wv[16];
  uint32_t tie = 0u;
  if (!wide) {
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      bool ti = false;
      wv[w] = fast_pair16<kBf16>(word_of(v[w >> 2], w & 3), r2, mz, 0x00030003u, ti);
      tie |= ti ? (3u << (2 * w)) : 0u;
    }
  } else {
    const float2 top = make_float2(kMagic + 3.0f, kMagic + 3.0f);
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      uint32_t c0, c1;
      fast_pair<kBf16>(word_of(v[w >> 2], w & 3), r2, mz, top, tie, 1u << (2 * w), 1u << (2 * w + 1), c0, c1);
      wv[w] = prmt(c0, c1, 0x5410u);
    }
  }
  const uint2 o = value_bytes(wv);
  return make_uint3(o.x, o.y, tie);
}

// Value pages, D = G = 128: 256 threads per page-head; thread (tp = tid >> 2, cq = tid & 3)
// holds tokens 2 tp and 2 tp + 1, channels 32 cq .. 32 cq + 31 (four 16-byte loads per
// token).  The four lanes of a token reduce its min / max with two shuffles and each
// computes the token's statistics (same values in all four), so no statistic is
// broadcast and no shared memory or barrier is needed; each thread packs its 32
// channels of a token into 8 bytes (byte j = channels 4 j .. 4 j + 3 at bits 0,2,4,6)
// and stores them directly (the four lanes of a token write its 32-byte row).
template <bool kBf16, bool kMetaBf16>
__global__ void __launch_bounds__(kFastThreads, KITTY_Q_MINB)
quantize_value_d128_kernel(const KittyValueQuantArgs a) {
  using T = Half16<kBf16>;
  const int job = blockIdx.x / a.num_heads;
  const int h = blockIdx.x - job * a.num_heads;
  const int tid = threadIdx.x, cq = tid & 3, tp = tid >> 2;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(a.value) + a.value_off[job] + h * a.val_s_head;
  const int n_valid = a.n_valid ? a.n_valid[job] : 128;
  const int64_t page = a.dst_page[job];
  if (page < 0) return;   // skipped job (a batched append flushes only full buffers)
  uint16_t* out_scale = reinterpret_cast<uint16_t*>(a.val_scale) + page * a.meta_s_page + h * a.meta_s_head;
  uint16_t* out_zero = reinterpret_cast<uint16_t*>(a.val_zero) + page * a.meta_s_page + h * a.meta_s_head;
  uint8_t* out_codes = a.val_codes + page * a.codes_s_page + h * a.codes_s_head;
  const bool vec = ((reinterpret_cast<uintptr_t>(src) & 15) == 0);

  uint4 v[2][4];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int tok = 2 * tp + k;
#pragma unroll
    for (int j = 0; j < 4; ++j) v[k][j] = make_uint4(0u, 0u, 0u, 0u);
    if (tok < n_valid) {
      const uint16_t* p = src + tok * a.val_s_tok + 32 * cq;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (vec) {
          v[k][j] = reinterpret_cast<const uint4*>(p)[j];
        } else {
          const uint16_t* q = p + 8 * j;
          v[k][j] = make_uint4(uint32_t(q[0]) | (uint32_t(q[1]) << 16), uint32_t(q[2]) | (uint32_t(q[3]) << 16),
                               uint32_t(q[4]) | (uint32_t(q[5]) << 16), uint32_t(q[6]) | (uint32_t(q[7]) << 16));
        }
      }
    }
  }
  // per-token statistics in the reference's float32 sequence (quantize_value.py:62-81):
  // min / max of both tokens over the four lanes, then lanes with cq even compute token
  // 2 tp and lanes with cq odd token 2 tp + 1 (the divisions once per token and lane
  // pair); the partner lane's values come by one shuffle each
  float mnk[2], mxk[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    uint32_t lo = T::min2(T::min2(v[k][0].x, v[k][0].y), T::min2(v[k][0].z, v[k][0].w));
    uint32_t hi = T::max2(T::max2(v[k][0].x, v[k][0].y), T::max2(v[k][0].z, v[k][0].w));
#pragma unroll
    for (int j = 1; j < 4; ++j) {
      lo = T::min2(lo, T::min2(T::min2(v[k][j].x, v[k][j].y), T::min2(v[k][j].z, v[k][j].w)));
      hi = T::max2(hi, T::max2(T::max2(v[k][j].x, v[k][j].y), T::max2(v[k][j].z, v[k][j].w)));
    }
    lo = T::min2(lo, __funnelshift_l(lo, lo, 16));   // both halves: min of the pair
    hi = T::max2(hi, __funnelshift_l(hi, hi, 16));
    // (min, -max) in one pair: the sign flip of the high half negates it (NaN stays NaN)
    uint32_t mm = (lo & 0x0000ffffu) | ((hi ^ 0x80000000u) & 0xffff0000u);
    mm = T::min2(mm, __shfl_xor_sync(0xffffffffu, mm, 1));
    mm = T::min2(mm, __shfl_xor_sync(0xffffffffu, mm, 2));
    const float2 mmf = T::to_f2(mm);
    mnk[k] = mmf.x;
    mxk[k] = -mmf.y;
  }
  const int mine = cq & 1;
  const float mn = mine ? mnk[1] : mnk[0], mx = mine ? mxk[1] : mxk[0];
  const float scale_m = __fdiv_rn(clamp_min(mx - mn, 1e-8f), 3.0f);
  const float zp_m = tmin(tmax(rintf(__fdiv_rn(-mn, scale_m)), 0.0f), 3.0f);
  const float rcp_m = __frcp_rn(scale_m);
  // |x| / scale can reach 16000: that token's codes take the fp32 clamp
  const int wide_m = !(fmaxf(fabsf(mn), fabsf(mx)) * rcp_m < 16000.0f);
  if (cq < 2) {
    out_scale[(2 * tp + mine) * a.meta_s_tok] = Half16<kMetaBf16>::meta(scale_m);
    out_zero[(2 * tp + mine) * a.meta_s_tok] = Half16<kMetaBf16>::meta(zp_m);
  }
  const float scale_o = __shfl_xor_sync(0xffffffffu, scale_m, 1), zp_o = __shfl_xor_sync(0xffffffffu, zp_m, 1);
  const float rcp_o = __shfl_xor_sync(0xffffffffu, rcp_m, 1);
  const int wide_o = __shfl_xor_sync(0xffffffffu, wide_m, 1);
  const float scale[2] = {mine ? scale_o : scale_m, mine ? scale_m : scale_o};
  const float zp[2] = {mine ? zp_o : zp_m, mine ? zp_m : zp_o};
  const float rcp[2] = {mine ? rcp_o : rcp_m, mine ? rcp_m : rcp_o};
  const int wide[2] = {mine ? wide_o : wide_m, mine ? wide_m : wide_o};
  bool finite = isfinite(mnk[0]) && isfinite(mxk[0]) && isfinite(mnk[1]) && isfinite(mxk[1]);
  finite = __all_sync(0xffffffffu, finite);   // warp-uniform: the warp takes one path
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int tok = 2 * tp + k;
    const uint16_t* my_src = src + tok * a.val_s_tok + 32 * cq;
    uint32_t out0, out1;
    if (finite) {
      const float2 r2 = make_float2(rcp[k], rcp[k]);
      const float2 mz = make_float2(kMagic + zp[k], kMagic + zp[k]);
      // fast: rint(x r) + zp in 16-bit lanes, one running maximum of the rounding distance
      // and one OR of the code bits outside 0..3 for the whole token
      uint32_t tie = 0u;
      bool slow = wide[k] != 0;
      if (!slow) {
        float emax = 0.f;
        uint32_t bad = 0u;
        uint32_t wv[16];
#pragma unroll
        for (int w = 0; w < 16; ++w) {
          const float2 x = T::to_f2(word_of(v[k][w >> 2], w & 3));
          const float2 f = fma2(x, r2, mz);
          const float2 e = fma2(x, r2, fma2(f, make_float2(-1.0f, -1.0f), mz));
          asm("max.f32 %0, %1, %2, %3;" : "=f"(emax) : "f"(emax), "f"(fabsf(e.x)), "f"(fabsf(e.y)));
          wv[w] = prmt(__float_as_uint(f.x), __float_as_uint(f.y), 0x5410u);
          bad |= wv[w];
        }
        const uint2 o = value_bytes(wv);
        out0 = o.x;
        out1 = o.y;
        slow = emax > kNearHalf || (bad & 0xfffcfffcu) != 0u;
      }
      if (slow) {   // a near-tie or a code outside 0..3 in this token: per-pair flags and clamps
        const uint3 r = value_token_slow<kBf16>(v[k][0], v[k][1], v[k][2], v[k][3], rcp[k], zp[k], wide[k]);
        out0 = r.x;
        out1 = r.y;
        tie = r.z;
      }
      if (tie && tok < n_valid) {   // near-ties: exact codes of the flagged channels (8 per call)
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t f = (tie >> (8 * g)) & 0xffu;
          if (f) {
            uint32_t& o = g < 2 ? out0 : out1;
            const int sh = 16 * (g & 1);
            const uint32_t b = patch_row<kBf16>(f, my_src + 8 * g, 1, scale[k], zp[k], 3.0f, (o >> sh) & 0xffffu, 0u).x;
            o = (o & ~(0xffffu << sh)) | ((b & 0xffffu) << sh);
          }
        }
      }
    } else {   // non-finite statistics in this warp: the exact path (tokens beyond n_valid read as zeros)
      uint32_t g16[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        g16[g] = tok < n_valid ? patch_row<kBf16>(0xffu, my_src + 8 * g, 1, scale[k], zp[k], 3.0f, 0u, 0u).x
                               : (quant_code(0.0f, scale[k], zp[k], 3.0f) & 3u) * 0x5555u;
      }
      out0 = (g16[0] & 0xffffu) | (g16[1] << 16);
      out1 = (g16[2] & 0xffffu) | (g16[3] << 16);
    }
    *reinterpret_cast<uint2*>(out_codes + tok * 32 + 8 * cq) = make_uint2(out0, out1);
  }
}

bool fast_source_ok(const void* base, const int64_t s_tok, const int64_t s_ch) {
  return s_ch == 1 && (s_tok % 8) == 0 && aligned(base, 16);
}

size_t key_smem_bytes(int D, int G, int K) {
  return ((size_t(G) * D * 2 + 15) & ~size_t(15)) + size_t(D) * 16 + ((size_t(K) * (G / 4) + 3) / 4) * 4;
}
size_t value_smem_bytes(int D, int G) {
  return ((size_t(G) * D * 2 + 15) & ~size_t(15)) + size_t(G) * 8;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

int quantize_key_pages_impl(const KittyKeyQuantArgs* a, void* stream) {
  if (!a) return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: args is NULL");
  if (a->n_jobs == 0 || a->num_heads == 0) return KITTY_OK;
  if (a->n_jobs < 0 || a->num_heads < 0 || a->head_dim <= 0 || a->group <= 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: negative or zero size");
  if (a->group % 4 != 0 || a->head_dim % 4 != 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: head_dim and group must be multiples of 4");
  if (a->d_boost < 0 || a->d_boost > 255 || a->sentinel < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: d_boost must be in [0,255], sentinel >= 0");
  if (a->dtype != KITTY_DTYPE_F16 && a->dtype != KITTY_DTYPE_BF16 && a->dtype != KITTY_DTYPE_BF16_F16META)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: unknown dtype");
  const int dt = a->dtype;
  if (!a->key || !a->key_off || !a->boost_idx || !a->dst_page || !a->key_low || !a->key_scale || !a->key_zero ||
      (a->d_boost > 0 && !a->key_high))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: NULL pointer");
  const size_t smem = key_smem_bytes(a->head_dim, a->group, a->d_boost);
  if (smem > 200 * 1024)
    return fail(KITTY_ERR_UNSUPPORTED, "quantize_key_pages: head_dim*group too large for one CTA");
  if (int64_t(a->n_jobs) * a->num_heads > 0x7fffffffLL)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: too many page-heads");
  // fast path: D = G = 128, token-major 16-byte aligned rows, 16-byte aligned pool slices
  // (offsets are element offsets: the kernel adds key_off[j]; callers pass multiples of 8)
  if (a->head_dim == 128 && a->group == 128 && a->d_boost <= 128 &&
      fast_source_ok(a->key, a->key_s_tok, a->key_s_ch) && (a->key_s_head % 8) == 0 &&
      aligned(a->key_low, 16) && (a->low_s_page % 16) == 0 && (a->low_s_head % 16) == 0 &&
      (a->d_boost == 0 || (aligned(a->key_high, 16) && (a->high_s_page % 16) == 0 && (a->high_s_head % 16) == 0))) {
    auto fast = dt == KITTY_DTYPE_BF16 ? quantize_key_d128_kernel<true, true>
                : dt == KITTY_DTYPE_BF16_F16META ? quantize_key_d128_kernel<true, false>
                                                 : quantize_key_d128_kernel<false, false>;
    fast<<<a->n_jobs * a->num_heads, kFastThreads, 0, as_stream(stream)>>>(*a);
    return check_launch("quantize_key_d128_kernel");
  }
  auto kern = dt == KITTY_DTYPE_BF16 ? quantize_key_kernel<true, true>
              : dt == KITTY_DTYPE_BF16_F16META ? quantize_key_kernel<true, false>
                                               : quantize_key_kernel<false, false>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  kern<<<a->n_jobs * a->num_heads, kQuantThreads, smem, as_stream(stream)>>>(*a);
  return check_launch("quantize_key_kernel");
}

int quantize_value_pages_impl(const KittyValueQuantArgs* a, void* stream) {
  if (!a) return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_value_pages: args is NULL");
  if (a->n_jobs == 0 || a->num_heads == 0) return KITTY_OK;
  if (a->n_jobs < 0 || a->num_heads < 0 || a->head_dim <= 0 || a->group <= 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_value_pages: negative or zero size");
  if (a->group % 4 != 0 || a->head_dim % 4 != 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_value_pages: head_dim and group must be multiples of 4");
  if (!a->value || !a->value_off || !a->dst_page || !a->val_codes || !a->val_scale || !a->val_zero)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_value_pages: NULL pointer");
  if (a->dtype != KITTY_DTYPE_F16 && a->dtype != KITTY_DTYPE_BF16 && a->dtype != KITTY_DTYPE_BF16_F16META)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_value_pages: unknown dtype");
  const int dt = a->dtype;
  const size_t smem = value_smem_bytes(a->head_dim, a->group);
  if (smem > 200 * 1024)
    return fail(KITTY_ERR_UNSUPPORTED, "quantize_value_pages: head_dim*group too large for one CTA");
  if (int64_t(a->n_jobs) * a->num_heads > 0x7fffffffLL)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_value_pages: too many page-heads");
  if (a->head_dim == 128 && a->group == 128 && fast_source_ok(a->value, a->val_s_tok, a->val_s_ch) &&
      (a->val_s_head % 8) == 0 && aligned(a->val_codes, 16) && (a->codes_s_page % 16) == 0 &&
      (a->codes_s_head % 16) == 0) {
    auto fast = dt == KITTY_DTYPE_BF16 ? quantize_value_d128_kernel<true, true>
                : dt == KITTY_DTYPE_BF16_F16META ? quantize_value_d128_kernel<true, false>
                                                 : quantize_value_d128_kernel<false, false>;
    fast<<<a->n_jobs * a->num_heads, kFastThreads, 0, as_stream(stream)>>>(*a);
    return check_launch("quantize_value_d128_kernel");
  }
  auto kern = dt == KITTY_DTYPE_BF16 ? quantize_value_kernel<true, true>
              : dt == KITTY_DTYPE_BF16_F16META ? quantize_value_kernel<true, false>
                                               : quantize_value_kernel<false, false>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  kern<<<a->n_jobs * a->num_heads, kQuantThreads, smem, as_stream(stream)>>>(*a);
  return check_launch("quantize_value_kernel");
}

namespace {
// metadata type and output type of a dequantiser call: (bf16 metadata, float32 out)
bool dequant_types(int32_t dt, bool* bf16, bool* f32) {
  *bf16 = dt == KITTY_DTYPE_BF16 || dt == KITTY_DTYPE_BF16_F32OUT;
  *f32 = dt == KITTY_DTYPE_F16_F32OUT || dt == KITTY_DTYPE_BF16_F32OUT;
  return dt == KITTY_DTYPE_F16 || dt == KITTY_DTYPE_BF16 || *f32;
}
}  // namespace

int dequantize_key_pages_impl(const KittyKeyDequantArgs* a, void* stream) {
  if (!a) return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_key_pages: args is NULL");
  if (a->n_jobs == 0) return KITTY_OK;
  if (a->n_jobs < 0 || a->head_dim <= 0 || a->group <= 0 || a->group % 4 != 0 || a->d_boost < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_key_pages: bad sizes");
  if (!a->key_low || !a->key_scale || !a->key_zero || !a->src_page || !a->head || !a->boost_idx || !a->out ||
      !a->out_off || (a->d_boost > 0 && !a->key_high))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_key_pages: NULL pointer");
  bool bf16 = false, f32 = false;
  if (!dequant_types(a->dtype, &bf16, &f32))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_key_pages: dtype must be KITTY_DTYPE_F16, BF16, "
                                            "F16_F32OUT or BF16_F32OUT");
  auto kern = bf16 ? (f32 ? dequantize_key_kernel<true, true> : dequantize_key_kernel<true, false>)
                   : (f32 ? dequantize_key_kernel<false, true> : dequantize_key_kernel<false, false>);
  kern<<<a->n_jobs, 256, 0, as_stream(stream)>>>(*a);
  return check_launch("dequantize_key_kernel");
}

int dequantize_value_pages_impl(const KittyValueDequantArgs* a, void* stream) {
  if (!a) return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_value_pages: args is NULL");
  if (a->n_jobs == 0) return KITTY_OK;
  if (a->n_jobs < 0 || a->head_dim <= 0 || a->head_dim % 4 != 0 || a->group <= 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_value_pages: bad sizes");
  if (!a->val_codes || !a->val_scale || !a->val_zero || !a->src_page || !a->head || !a->out || !a->out_off)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_value_pages: NULL pointer");
  bool bf16 = false, f32 = false;
  if (!dequant_types(a->dtype, &bf16, &f32))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_value_pages: dtype must be KITTY_DTYPE_F16, BF16, "
                                            "F16_F32OUT or BF16_F32OUT");
  auto kern = bf16 ? (f32 ? dequantize_value_kernel<true, true> : dequantize_value_kernel<true, false>)
                   : (f32 ? dequantize_value_kernel<false, true> : dequantize_value_kernel<false, false>);
  kern<<<a->n_jobs, 256, 0, as_stream(stream)>>>(*a);
  return check_launch("dequantize_value_kernel");
}

}  // namespace kitty
