// Paged GQA decode attention, CUDA-core (FMA) variant for any shape, and the
// split-K merge kernel shared by every decode variant.
//
// One CTA handles one (split, KV head, sequence).  It walks its chunk of the
// key/value sequence - the fp16 sinks and tail (split 0 only) and the pages
// block_table[b][split range] - keeping an online softmax (running max m,
// running sum l, accumulator o) for each of the g = Hq/H query heads that
// share the KV head.  Keys are dequantised exactly as the reference does,
// (code - zp) * scale in fp32 (kitty/kernels/dequantize_key.py:89-95); values
// likewise (kitty/kernels/quantize_value.py:121-133).  Scores are
// (q . k) * sm_scale (kitty/kernels/attention.py:172-187).
//
// Per page the phases are: stage the 5 pool slices in shared memory, score
// (thread <-> token), softmax update, accumulate (thread <-> channel).

#include "kitty_decode.cuh"

namespace kitty {
namespace {

constexpr int kSimtThreads = 128;
constexpr int kMaxGroupSimt = 16;  // query heads per KV head

struct SimtSmem {
  // offsets into dynamic shared memory (bytes)
  size_t q, kl, kh, vc, ks, kz, vs, vz, p, row, red, stats, total;
};

__host__ __device__ inline SimtSmem simt_layout(int D, int G, int K, int g) {
  SimtSmem s;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t r = o; o = (o + bytes + 15) & ~size_t(15); return r; };
  s.q = take(size_t(g) * D * 4);
  s.kl = take(size_t(D) * (G / 4));
  s.kh = take(size_t(K) * (G / 4) + 4);
  s.vc = take(size_t(G) * (D / 4));
  s.ks = take(size_t(D) * 4);   // key scale / zero-point per channel, float
  s.kz = take(size_t(D) * 4);
  s.vs = take(size_t(G) * 4);   // value scale / zero-point per token, float
  s.vz = take(size_t(G) * 4);
  const int chunk = G > kSimtThreads ? G : kSimtThreads;
  s.p = take(size_t(g) * chunk * 4);
  s.row = take(size_t(D) * 4);
  s.red = take(size_t(kSimtThreads / 32) * g * 4);
  s.stats = take(size_t(3) * g * 4);
  s.total = o;
  return s;
}

// bytes [0, n) of src into dst: 16-byte copies when both ends allow it
__device__ __forceinline__ void stage_bytes(uint8_t* dst, const uint8_t* src, int n, int tid) {
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0 && (n & 15) == 0) {
    for (int i = tid; i < n / 16; i += kSimtThreads)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int i = tid; i < n; i += kSimtThreads) dst[i] = src[i];
  }
}

// kGT: query heads per KV head rounded up to a power of two (loops over heads have a
// constant trip count; heads g .. kGT-1 are predicated off).  Channels and tokens of
// the inner loops go four at a time: q, probabilities and metadata as 16-byte loads.
template <bool kBf16, int kGT>
__global__ void __launch_bounds__(kSimtThreads)
decode_simt_kernel(const KittyDecodeArgs a, DecodePlan plan) {
  using T = Half16<kBf16>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int D = a.head_dim, G = a.group, K = a.d_boost, H = a.num_kv_heads;
  const int g = a.num_q_heads / H;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = kSimtThreads / 32;
  const SimtSmem L = simt_layout(D, G, K, g);

  float* q_s = reinterpret_cast<float*>(smem + L.q);
  uint8_t* kl_s = smem + L.kl;
  uint8_t* kh_s = smem + L.kh;
  uint8_t* vc_s = smem + L.vc;
  float* ks_s = reinterpret_cast<float*>(smem + L.ks);
  float* kz_s = reinterpret_cast<float*>(smem + L.kz);
  float* vs_s = reinterpret_cast<float*>(smem + L.vs);
  float* vz_s = reinterpret_cast<float*>(smem + L.vz);
  float* p_s = reinterpret_cast<float*>(smem + L.p);
  int* row_s = reinterpret_cast<int*>(smem + L.row);
  float* red_s = reinterpret_cast<float*>(smem + L.red);
  float* m_s = reinterpret_cast<float*>(smem + L.stats);
  float* l_s = m_s + g;
  float* alpha_s = l_s + g;
  const int chunk_cap = G > kSimtThreads ? G : kSimtThreads;

  const uint16_t* qg = reinterpret_cast<const uint16_t*>(a.q) + b * a.q_s_seq + (h * g) * a.q_s_head;
  for (int i = tid; i < g * D; i += kSimtThreads) {
    const int qh = i / D, c = i - qh * D;
    q_s[i] = T::to_f(qg[qh * a.q_s_head + c]);
  }
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  for (int c = tid; c < D; c += kSimtThreads) {
    const int r = bidx[c];
    row_s[c] = r < K ? r : -1;
  }
  if (tid < g) { m_s[tid] = -INFINITY; l_s[tid] = 0.f; alpha_s[tid] = 1.f; }

  // per-thread accumulators: channel c = tid + j*128 for j < ceil(D/128)
  constexpr int kMaxChanPerThread = 2;  // D <= 256
  float o_acc[kMaxChanPerThread][kGT];
#pragma unroll
  for (int j = 0; j < kMaxChanPerThread; ++j)
#pragma unroll
    for (int qh = 0; qh < kGT; ++qh) o_acc[j][qh] = 0.f;

  const int cr = a.seq_map ? a.seq_map[b] : b;   // cache row of batch row b
  const int npages = a.num_pages[cr];
  const int p_begin = split * plan.pages_per_split;
  const int p_end = min(npages, p_begin + plan.pages_per_split);
  const int sink_len = a.sink_len ? a.sink_len[cr] : a.sink_len_all;
  const int tail_len = a.tail_len ? a.tail_len[cr] : a.tail_len_all;
  const int fp16_tokens = (split == 0) ? (sink_len + tail_len) : 0;
  const int fp16_chunks = (fp16_tokens + chunk_cap - 1) / chunk_cap;
  const int n_items = fp16_chunks + max(0, p_end - p_begin);
  __syncthreads();

  for (int item = 0; item < n_items; ++item) {
    const bool is_page = item >= fp16_chunks;
    int ntok;
    int64_t page = 0;
    int f0 = 0;  // first fp16 token of this chunk (sinks first, then tail)
    if (is_page) {
      page = a.block_table[cr * a.bt_s_seq + p_begin + (item - fp16_chunks)];
      if (page < 0 || page >= a.pool_pages) continue;  // out-of-range entries are skipped
      ntok = G;
      // stage the code planes; metadata straight to float
      const int64_t ph = page * H + h;
      stage_bytes(kl_s, a.key_low + ph * (int64_t(D) * (G / 4)), D * (G / 4), tid);
      stage_bytes(kh_s, a.key_high + ph * (int64_t(K) * (G / 4)), K * (G / 4), tid);
      stage_bytes(vc_s, a.val_codes + ph * (int64_t(G) * (D / 4)), G * (D / 4), tid);
      const uint16_t* km = reinterpret_cast<const uint16_t*>(a.key_meta) + ph * (2 * int64_t(D));
      const uint16_t* vm = reinterpret_cast<const uint16_t*>(a.val_meta) + ph * (2 * int64_t(G));
      for (int c = tid; c < D; c += kSimtThreads) { ks_s[c] = T::to_f(km[c]); kz_s[c] = T::to_f(km[D + c]); }
      for (int t = tid; t < G; t += kSimtThreads) { vs_s[t] = T::to_f(vm[2 * t]); vz_s[t] = T::to_f(vm[2 * t + 1]); }
    } else {
      f0 = item * chunk_cap;
      ntok = min(chunk_cap, fp16_tokens - f0);
    }
    __syncthreads();

    // ---- scores: thread <-> token, channels four at a time
    for (int t = tid; t < chunk_cap; t += kSimtThreads) {
      float acc[kGT];
#pragma unroll
      for (int qh = 0; qh < kGT; ++qh) acc[qh] = 0.f;
      if (t < ntok) {
        const int G4 = G / 4, j = t >> 2, sh = 2 * (t & 3);
        const uint16_t* kp = nullptr;
        if (!is_page) {
          const int ft = f0 + t;
          kp = (ft < sink_len)
              ? reinterpret_cast<const uint16_t*>(a.sink_k) + cr * a.sk_s_seq + h * a.sk_s_head + ft * a.sk_s_tok
              : reinterpret_cast<const uint16_t*>(a.tail_k) + cr * a.tk_s_seq + h * a.tk_s_head + (ft - sink_len) * a.tk_s_tok;
        }
        for (int c = 0; c < D; c += 4) {
          float kv[4];
          if (is_page) {
            const int4 r4 = *reinterpret_cast<const int4*>(row_s + c);
            const float4 s4 = *reinterpret_cast<const float4*>(ks_s + c);
            const float4 z4 = *reinterpret_cast<const float4*>(kz_s + c);
            const int rr[4] = {r4.x, r4.y, r4.z, r4.w};
            const float ss[4] = {s4.x, s4.y, s4.z, s4.w}, zz[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t code = (kl_s[(c + i) * G4 + j] >> sh) & 3u;
              if (rr[i] >= 0) code |= ((kh_s[rr[i] * G4 + j] >> sh) & 3u) << 2;
              kv[i] = (static_cast<float>(code) - zz[i]) * ss[i];
            }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) kv[i] = T::to_f(kp[c + i]);
          }
#pragma unroll
          for (int qh = 0; qh < kGT; ++qh) {
            if (qh < g) {
              const float4 qv = *reinterpret_cast<const float4*>(q_s + qh * D + c);
              acc[qh] = fmaf(qv.x, kv[0], acc[qh]);
              acc[qh] = fmaf(qv.y, kv[1], acc[qh]);
              acc[qh] = fmaf(qv.z, kv[2], acc[qh]);
              acc[qh] = fmaf(qv.w, kv[3], acc[qh]);
            }
          }
        }
      }
#pragma unroll
      for (int qh = 0; qh < kGT; ++qh)
        if (qh < g) p_s[qh * chunk_cap + t] = (t < ntok) ? acc[qh] * a.sm_scale : -INFINITY;
    }
    __syncthreads();

    // ---- online softmax update
    for (int qh = 0; qh < g; ++qh) {
      float mx = -INFINITY;
      for (int t = tid; t < chunk_cap; t += kSimtThreads) mx = fmaxf(mx, p_s[qh * chunk_cap + t]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) red_s[warp * g + qh] = mx;
    }
    __syncthreads();
    if (tid < g) {
      float mx = m_s[tid];
      for (int w = 0; w < nwarps; ++w) mx = fmaxf(mx, red_s[w * g + tid]);
      alpha_s[tid] = (m_s[tid] == -INFINITY) ? 0.f : __expf(m_s[tid] - mx);
      m_s[tid] = mx;
    }
    __syncthreads();
    for (int qh = 0; qh < g; ++qh) {
      const float mx = m_s[qh];
      float sum = 0.f;
      for (int t = tid; t < chunk_cap; t += kSimtThreads) {
        const float s = p_s[qh * chunk_cap + t];
        const float p = (s == -INFINITY) ? 0.f : __expf(s - mx);
        p_s[qh * chunk_cap + t] = p;
        sum += p;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) red_s[warp * g + qh] = sum;
    }
    __syncthreads();
    if (tid < g) {
      float sum = 0.f;
      for (int w = 0; w < nwarps; ++w) sum += red_s[w * g + tid];
      l_s[tid] = l_s[tid] * alpha_s[tid] + sum;
    }

    // ---- accumulate: thread <-> channel; page tokens four at a time
#pragma unroll
    for (int j = 0; j < kMaxChanPerThread; ++j) {
      const int c = tid + j * kSimtThreads;
      if (c >= D) break;
      float acc[kGT];
#pragma unroll
      for (int qh = 0; qh < kGT; ++qh) acc[qh] = o_acc[j][qh] * (qh < g ? alpha_s[qh] : 0.f);
      if (is_page) {
        const int D4 = D / 4, jj = c >> 2, sh = 2 * (c & 3);
        for (int t = 0; t < ntok; t += 4) {
          const float4 s4 = *reinterpret_cast<const float4*>(vs_s + t);
          const float4 z4 = *reinterpret_cast<const float4*>(vz_s + t);
          const float vv[4] = {(static_cast<float>((vc_s[t * D4 + jj] >> sh) & 3u) - z4.x) * s4.x,
                               (static_cast<float>((vc_s[(t + 1) * D4 + jj] >> sh) & 3u) - z4.y) * s4.y,
                               (static_cast<float>((vc_s[(t + 2) * D4 + jj] >> sh) & 3u) - z4.z) * s4.z,
                               (static_cast<float>((vc_s[(t + 3) * D4 + jj] >> sh) & 3u) - z4.w) * s4.w};
#pragma unroll
          for (int qh = 0; qh < kGT; ++qh) {
            if (qh < g) {
              const float4 pv = *reinterpret_cast<const float4*>(p_s + qh * chunk_cap + t);
              acc[qh] = fmaf(pv.x, vv[0], acc[qh]);
              acc[qh] = fmaf(pv.y, vv[1], acc[qh]);
              acc[qh] = fmaf(pv.z, vv[2], acc[qh]);
              acc[qh] = fmaf(pv.w, vv[3], acc[qh]);
            }
          }
        }
      } else {
        for (int t = 0; t < ntok; ++t) {
          const int ft = f0 + t;
          const uint16_t* vp = (ft < sink_len)
              ? reinterpret_cast<const uint16_t*>(a.sink_v) + cr * a.sv_s_seq + h * a.sv_s_head + ft * a.sv_s_tok
              : reinterpret_cast<const uint16_t*>(a.tail_v) + cr * a.tv_s_seq + h * a.tv_s_head + (ft - sink_len) * a.tv_s_tok;
          const float vv = T::to_f(vp[c]);
#pragma unroll
          for (int qh = 0; qh < kGT; ++qh)
            if (qh < g) acc[qh] = fmaf(p_s[qh * chunk_cap + t], vv, acc[qh]);
        }
      }
#pragma unroll
      for (int qh = 0; qh < kGT; ++qh) o_acc[j][qh] = acc[qh];
    }
    __syncthreads();
  }

  // ---- write the partial (or final, when unsplit) result
#pragma unroll
  for (int j = 0; j < kMaxChanPerThread; ++j) {
    const int c = tid + j * kSimtThreads;
    if (c >= D) break;
#pragma unroll
    for (int qh = 0; qh < kGT; ++qh) {
      if (qh >= g) break;
      if (plan.num_splits == 1) {
        const float l = l_s[qh];
        uint16_t* out = reinterpret_cast<uint16_t*>(a.out) + b * a.out_s_seq + (h * g + qh) * a.out_s_head;
        out[c] = f2h(l > 0.f ? o_acc[j][qh] / l : 0.f);
      } else {
        float* o = plan.ws_o + (((int64_t(b) * H + h) * plan.num_splits + split) * g + qh) * D;
        o[c] = o_acc[j][qh];
      }
    }
  }
  if (plan.num_splits > 1 && tid < g) {
    const int64_t idx = ((int64_t(b) * H + h) * plan.num_splits + split) * g + tid;
    plan.ws_m[idx] = m_s[tid];
    plan.ws_l[idx] = l_s[tid];
  }
}

}  // namespace

// Merge the per-split partials: out = sum_s e^{m_s-M} o_s / sum_s e^{m_s-M} l_s.
// Combines the split partials of one (sequence, query head): max M over the slots,
// weights w_s = exp(m_s - M), L = sum_s w_s l_s, out = sum_s w_s o_s / L.  Up to 32
// slots (the usual case) each warp computes the weights itself, one lane per slot, and
// broadcasts them by shuffles; with more slots the weights are computed once per block
// and kept in shared memory, and the accumulation issues its loads in groups of eight,
// so a call with many slots costs a few memory latencies instead of one per slot.
constexpr int kMergeThreads = 128;
constexpr int kMergeMaxSlots = kMaxDecodeSlots;

__global__ void __launch_bounds__(kMergeThreads)
decode_merge_kernel(const KittyDecodeArgs a, DecodePlan plan) {
  __shared__ float s_w[kMergeMaxSlots];
  __shared__ float s_red[kMergeThreads / 32];
  __shared__ float s_M, s_L;
  // blockIdx.x = query head within the launch's heads: g of every KV head's group of g_all,
  // starting at plan.qh_base (all of them unless the integer kernel ran in passes)
  const int b = blockIdx.y;
  const int H = a.num_kv_heads, g_all = a.num_q_heads / H, D = a.head_dim;
  const int g = plan.g_pass > 0 ? plan.g_pass : g_all;
  const int h = blockIdx.x / g, qh = blockIdx.x - h * g;
  const int qhg = h * g_all + plan.qh_base + qh;   // global query head
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t base = (int64_t(b) * H + h) * plan.num_splits;
  // slots written for this (sequence, head): all of them, or the recorded count
  const int nsl = min(plan.ws_count ? min(max(plan.ws_count[int64_t(b) * H + h], 0), plan.num_splits)
                                    : plan.num_splits, kMergeMaxSlots);
  uint16_t* out = reinterpret_cast<uint16_t*>(a.out) + b * a.out_s_seq + qhg * a.out_s_head;
  const float* o = plan.ws_o + ((base) * g + qh) * int64_t(D);
  const int64_t slot_stride = int64_t(g) * D;
  if (nsl <= 32) {
    // few slots (the usual case): every warp derives the slot weights itself, lane s for
    // slot s, and broadcasts them by shuffles - no block-wide reduction or barrier
    const float ms = lane < nsl ? plan.ws_m[(base + lane) * g + qh] : -INFINITY;
    float M = ms;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, d));
    const float ws = (ms == -INFINITY) ? 0.f : __expf(ms - M);
    float L = lane < nsl ? ws * plan.ws_l[(base + lane) * g + qh] : 0.f;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) L += __shfl_xor_sync(0xffffffffu, L, d);
    // whole warps walk the channels (the shuffles need every lane), loads guarded by c < D
    for (int c0 = warp * 32; c0 < D; c0 += kMergeThreads) {
      const int c = c0 + lane;
      const bool in = c < D;
      float acc = 0.f;
      int s = 0;
      for (; s + 4 <= nsl; s += 4) {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = in ? o[(s + k) * slot_stride + c] : 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) acc += __shfl_sync(0xffffffffu, ws, s + k) * v[k];
      }
      for (; s < nsl; ++s) {
        const float v = in ? o[s * slot_stride + c] : 0.f;
        acc += __shfl_sync(0xffffffffu, ws, s) * v;
      }
      if (in) out[c] = f2h(L > 0.f ? acc / L : 0.f);
    }
    return;
  }
  float mx = -INFINITY;
  for (int s = tid; s < nsl; s += kMergeThreads) mx = fmaxf(mx, plan.ws_m[(base + s) * g + qh]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float M = s_red[0];
    for (int w = 1; w < kMergeThreads / 32; ++w) M = fmaxf(M, s_red[w]);
    s_M = M;
  }
  __syncthreads();
  const float M = s_M;
  float part = 0.f;
  for (int s = tid; s < nsl; s += kMergeThreads) {
    const float m = plan.ws_m[(base + s) * g + qh];
    const float w = (m == -INFINITY) ? 0.f : __expf(m - M);
    s_w[s] = w;
    part += w * plan.ws_l[(base + s) * g + qh];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  __syncthreads();
  if (lane == 0) s_red[warp] = part;
  __syncthreads();
  if (tid == 0) {
    float L = 0.f;
    for (int w = 0; w < kMergeThreads / 32; ++w) L += s_red[w];
    s_L = L;
  }
  __syncthreads();
  const float L = s_L;
  for (int c = tid; c < D; c += kMergeThreads) {
    float acc = 0.f;
    int s = 0;
    for (; s + 8 <= nsl; s += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = o[(s + k) * slot_stride + c];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += s_w[s + k] * v[k];
    }
    for (; s < nsl; ++s) acc += s_w[s] * o[s * slot_stride + c];
    out[c] = f2h(L > 0.f ? acc / L : 0.f);
  }
}

namespace {
template <bool kBf16, int kGT>
void launch_simt_t(const KittyDecodeArgs& a, const DecodePlan& plan, size_t smem, cudaStream_t stream) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(decode_simt_kernel<kBf16, kGT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  dim3 grid(plan.num_splits, a.num_kv_heads, a.batch);
  decode_simt_kernel<kBf16, kGT><<<grid, kSimtThreads, smem, stream>>>(a, plan);
}
template <bool kBf16>
void launch_simt_g(const KittyDecodeArgs& a, const DecodePlan& plan, size_t smem, int g, cudaStream_t stream) {
  if (g <= 1) launch_simt_t<kBf16, 1>(a, plan, smem, stream);
  else if (g <= 2) launch_simt_t<kBf16, 2>(a, plan, smem, stream);
  else if (g <= 4) launch_simt_t<kBf16, 4>(a, plan, smem, stream);
  else if (g <= 8) launch_simt_t<kBf16, 8>(a, plan, smem, stream);
  else launch_simt_t<kBf16, 16>(a, plan, smem, stream);
}
}  // namespace

int launch_decode_simt(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  const int g = a.num_q_heads / a.num_kv_heads;
  const SimtSmem L = simt_layout(a.head_dim, a.group, a.d_boost, g);
  if (L.total > 200 * 1024) return fail(KITTY_ERR_UNSUPPORTED, "paged_decode: shape needs too much shared memory");
  if (a.dtype == KITTY_DTYPE_BF16) launch_simt_g<true>(a, plan, L.total, g, stream);
  else launch_simt_g<false>(a, plan, L.total, g, stream);
  return check_launch("decode_simt_kernel");
}

int launch_decode_merge(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  const int g = plan.g_pass > 0 ? plan.g_pass : a.num_q_heads / a.num_kv_heads;
  dim3 grid(a.num_kv_heads * g, a.batch);
  if (plan.num_splits > kMergeMaxSlots)
    return fail(KITTY_ERR_UNSUPPORTED, "paged_decode: more than 1024 partial slots per sequence and head");
  decode_merge_kernel<<<grid, kMergeThreads, 0, stream>>>(a, plan);
  return check_launch("decode_merge_kernel");
}

bool simt_supports(const KittyDecodeArgs& a) {
  const int g = a.num_q_heads / a.num_kv_heads;
  return a.head_dim <= 256 && a.head_dim % 4 == 0 && a.group % 4 == 0 && g <= kMaxGroupSimt;
}

}  // namespace kitty
