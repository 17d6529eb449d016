// Page quantise/pack kernels (key: per channel, dense-sparse INT2/INT4;
// value: per token INT2) and key page dequantisation.
//
// Arithmetic follows the reference's PyTorch path operation by operation in
// IEEE float32 (kitty/kernels/quantize_key.py:69-124,
// kitty/kernels/quantize_value.py:50-90): divisions are correctly rounded
// (__fdiv_rn), rounding is half-to-even (rintf), and the stored scale is the
// float32 scale rounded to fp16.  The packed planes are therefore bit-exact.
//
// One CTA handles one page-head: it stages the G x D fp16 block in shared
// memory with coalesced 16-byte loads (the block is 32 KB at D = G = 128),
// reduces per channel (keys) or per token (values), then quantises and packs
// four 2-bit codes per byte straight into the pool slice.

#include "kitty_common.cuh"

namespace kitty {
namespace {

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

__global__ void __launch_bounds__(kQuantThreads)
quantize_key_kernel(const KittyKeyQuantArgs a) {
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

  stage_block(tile, src, a.key_s_tok, a.key_s_ch, G, D, G);
  const int high_words = (K * G4 + 3) / 4;
  for (int i = threadIdx.x; i < high_words; i += blockDim.x) s_high[i] = 0u;
  __syncthreads();

  uint16_t* out_scale = reinterpret_cast<uint16_t*>(a.key_scale) + page * a.meta_s_page + h * a.meta_s_head;
  uint16_t* out_zero = reinterpret_cast<uint16_t*>(a.key_zero) + page * a.meta_s_page + h * a.meta_s_head;

  // Per-channel statistics (quantize_key.py:73-87).
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float mn = h2f(tile[c]), mx = mn;
    for (int t = 1; t < G; ++t) {
      const float x = h2f(tile[t * D + c]);
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
    out_scale[c] = f2h(scale);
    out_zero[c] = f2h(zp);
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
      const float x = h2f(tile[(4 * j + k) * D + c]);
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

__global__ void __launch_bounds__(kQuantThreads)
quantize_value_kernel(const KittyValueQuantArgs a) {
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
  stage_block(tile, src, a.val_s_tok, a.val_s_ch, G, D, n_valid);
  __syncthreads();

  uint16_t* out_scale = reinterpret_cast<uint16_t*>(a.val_scale) + page * a.meta_s_page + h * a.meta_s_head;
  uint16_t* out_zero = reinterpret_cast<uint16_t*>(a.val_zero) + page * a.meta_s_page + h * a.meta_s_head;

  // Per-token statistics (quantize_value.py:62-72): a warp per token, lanes over channels.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int t = warp; t < G; t += nwarps) {
    float mn = h2f(tile[t * D + (lane < D ? lane : 0)]), mx = mn;
    for (int c = lane + 32; c < D; c += 32) {
      const float x = h2f(tile[t * D + c]);
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
      out_scale[t * a.meta_s_tok] = f2h(scale);
      out_zero[t * a.meta_s_tok] = f2h(zp);
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
      const float x = h2f(tile[t * D + 4 * j + k]);
      float q = rintf(__fdiv_rn(x, scale)) + zp;
      q = tmin(tmax(q, 0.0f), 3.0f);
      byte |= (to_code(q) & 3u) << (2 * k);
    }
    out[i] = static_cast<uint8_t>(byte);
  }
}

__global__ void dequantize_key_kernel(const KittyKeyDequantArgs a) {
  const int D = a.head_dim, G = a.group, K = a.d_boost, G4 = G / 4;
  const int job = blockIdx.x;
  const int64_t page = a.src_page[job];
  const int h = a.head[job];
  const uint8_t* low = a.key_low + page * a.low_s_page + h * a.low_s_head;
  const uint8_t* high = a.key_high + page * a.high_s_page + h * a.high_s_head;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(a.key_scale) + page * a.meta_s_page + h * a.meta_s_head;
  const uint16_t* zr = reinterpret_cast<const uint16_t*>(a.key_zero) + page * a.meta_s_page + h * a.meta_s_head;
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  uint16_t* out = reinterpret_cast<uint16_t*>(a.out) + a.out_off[job];
  // dequantize_key.py:69-97: code = low | (high << 2) when boost_idx < d_boost.
  for (int i = threadIdx.x; i < D * G4; i += blockDim.x) {
    const int c = i / G4;
    const int j = i - c * G4;
    const int b = bidx[c];
    const uint32_t lo = low[i];
    const uint32_t hi = (b < K) ? high[b * G4 + j] : 0u;
    const float s = h2f(sc[c]), z = h2f(zr[c]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t code = ((lo >> (2 * k)) & 3u) | (((hi >> (2 * k)) & 3u) << 2);
      const float x = (static_cast<float>(code) - z) * s;
      out[c * a.out_s_ch + (4 * j + k) * a.out_s_tok] = f2h(x);
    }
  }
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
  if (!a->key || !a->key_off || !a->boost_idx || !a->dst_page || !a->key_low || !a->key_scale || !a->key_zero ||
      (a->d_boost > 0 && !a->key_high))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: NULL pointer");
  const size_t smem = key_smem_bytes(a->head_dim, a->group, a->d_boost);
  if (smem > 200 * 1024)
    return fail(KITTY_ERR_UNSUPPORTED, "quantize_key_pages: head_dim*group too large for one CTA");
  if (int64_t(a->n_jobs) * a->num_heads > 0x7fffffffLL)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_key_pages: too many page-heads");
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(quantize_key_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  }
  quantize_key_kernel<<<a->n_jobs * a->num_heads, kQuantThreads, smem, as_stream(stream)>>>(*a);
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
  const size_t smem = value_smem_bytes(a->head_dim, a->group);
  if (smem > 200 * 1024)
    return fail(KITTY_ERR_UNSUPPORTED, "quantize_value_pages: head_dim*group too large for one CTA");
  if (int64_t(a->n_jobs) * a->num_heads > 0x7fffffffLL)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "quantize_value_pages: too many page-heads");
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(quantize_value_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  }
  quantize_value_kernel<<<a->n_jobs * a->num_heads, kQuantThreads, smem, as_stream(stream)>>>(*a);
  return check_launch("quantize_value_kernel");
}

int dequantize_key_pages_impl(const KittyKeyDequantArgs* a, void* stream) {
  if (!a) return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_key_pages: args is NULL");
  if (a->n_jobs == 0) return KITTY_OK;
  if (a->n_jobs < 0 || a->head_dim <= 0 || a->group <= 0 || a->group % 4 != 0 || a->d_boost < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_key_pages: bad sizes");
  if (!a->key_low || !a->key_scale || !a->key_zero || !a->src_page || !a->head || !a->boost_idx || !a->out ||
      !a->out_off || (a->d_boost > 0 && !a->key_high))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "dequantize_key_pages: NULL pointer");
  dequantize_key_kernel<<<a->n_jobs, 256, 0, as_stream(stream)>>>(*a);
  return check_launch("dequantize_key_kernel");
}

}  // namespace kitty
