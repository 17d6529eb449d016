// Paged GQA decode attention on the tensor cores (head_dim = group = 128,
// up to 8 query heads per KV head).
//
// Work: one CTA per (split, KV head, sequence); each of its 4 warps streams
// every 4th page of the split through its own 2-stage shared-memory ring
// filled by bulk async copies (cp.async.bulk + mbarrier, five copies per
// page-head: the two key planes, key metadata, value codes, value metadata;
// no multicast).  Each warp keeps an online softmax for the g query heads;
// the warps are merged in shared memory at the end and the CTA writes either
// the final fp16 output (one split) or a partial for the merge kernel.
//
// Contraction (per page-head, per warp):
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
// exactly.  Row / column assignment is chosen so that every 32-bit shared
// memory word load of a warp hits 32 distinct banks.

#include "kitty_decode.cuh"

namespace kitty {

__device__ unsigned int g_decode_error = 0;  // bit 0: a bulk-copy wait timed out

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 2;
constexpr int kD = 128, kG = 128;
constexpr int kPRow = 136;          // fp16 elements per row of the P staging tile (16-byte aligned rows)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct MmaLayout {
  int stage_bytes;   // 9216 + K*32, rounded to 128
  int stages_off, p_off, qnat_off, blist_off, bars_off, total;
};

__host__ __device__ inline MmaLayout mma_layout(int K) {
  MmaLayout L;
  L.stage_bytes = (9216 + K * 32 + 127) & ~127;
  int o = 0;
  L.stages_off = o; o += kWarps * kStages * L.stage_bytes;
  L.p_off = o;      o += kWarps * 8 * kPRow * 2;
  L.qnat_off = o;   o += 8 * kD * 2;
  L.blist_off = o;  o += 128 * 2 + 16;
  L.bars_off = o;   o += kWarps * kStages * 8;
  // the end-of-kernel warp merge reuses the stage area: 4 warps x (128 x 8 + 32) floats
  L.total = (o + 127) & ~127;
  return L;
}

// ---- PTX helpers ----------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// (a & mask) | 1024.0h in both halves
template <uint32_t kMask>
__device__ __forceinline__ uint32_t mask_or_magic(uint32_t a) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(a), "n"(kMask), "n"(0x64006400u));
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
// x * y as an unevaluated fp16 pair hi + lo: hi = RN(x*y), lo = RN(x*y - hi) (the
// fused multiply-add sees the exact product), so hi + lo carries ~22 bits.
__device__ __forceinline__ void hmul2_split(uint32_t x, uint32_t y, uint32_t& hi, uint32_t& lo) {
  hi = hmul2_u32(x, y);
  lo = hfma2_u32(x, y, hi ^ 0x80008000u);
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
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                            uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
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

// code (0..3) of byte-slot k of both 16-bit halves of u, as exact fp16x2
template <int k>
__device__ __forceinline__ uint32_t code2(uint32_t u) {
  constexpr uint32_t mask = 0x00030003u << (2 * k);
  // 4^-k and -1024 * 4^-k as fp16x2
  constexpr uint32_t scale = k == 0 ? 0x3C003C00u : k == 1 ? 0x34003400u : k == 2 ? 0x2C002C00u : 0x24002400u;
  constexpr uint32_t bias = k == 0 ? 0xE400E400u : k == 1 ? 0xDC00DC00u : k == 2 ? 0xD400D400u : 0xCC00CC00u;
  return hfma2_u32(mask_or_magic<mask>(u), scale, bias);
}

// Contract one 16-wide k-step of a [row][32-byte] 2-bit plane into 8 M tiles.
// Rows (K index) of this thread: r0 + {0, 4, 8, 12}; word g_ of each row holds
// its 16 M-index values (tokens or channels 16*g_ .. 16*g_+15).
template <bool kSplit>
__device__ __forceinline__ void plane_kstep(float (&acc)[8][4], uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                            uint32_t b0, uint32_t b1, uint32_t c0 = 0u, uint32_t c1 = 0u) {
  // u?[j]: byte j of the two rows in the low byte of each 16-bit half
  uint32_t ulo[4], uhi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sel = uint32_t(j) | (uint32_t(j) << 4) | (uint32_t(4 + j) << 8) | (uint32_t(4 + j) << 12);
    ulo[j] = prmt(w0, w1, sel);
    uhi[j] = prmt(w2, w3, sel);
  }
  // M tile m: row g_ <-> index 4*(m>>2) + (m&3) = m, row g_+8 <-> m + 8.
  // With kSplit the B operand is the fp16 pair (b0, b1) + (c0, c1) (hi + lo parts).
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

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ uint32_t pack16(uint32_t lo, uint32_t hi) { return lo | (hi << 16); }

struct WarpState {
  float o[8][4];     // O^T C fragments: channel rows, query-head columns 2*q_, 2*q_+1
  float zv[4];       // value zero-point sums (valid in lanes 0..3, row 0)
  float m[2];        // running max (log2 domain) for the thread's two query-head columns
  float l[2];        // running sum over this thread's tokens
};

// Softmax update + P' staging + returns nothing; scores in `s` (log2 domain, masked = -inf).
// `sv` words: (scale, zp) fp16 per token for this thread's 16 tokens in token order
// (pass 0x3C00 scale for fp16 regions).
__device__ __forceinline__ void softmax_and_stage(WarpState& st, float (&s)[8][4], const uint32_t (&svw)[16],
                                                  __half* ps_warp, int g_, int q_) {
  // tile max per column pair
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

  // P' = p * scale_v, fp16, staged as Ps[qh][16*g_ + kappa] with kappa order
  // (tau, tau+4) pairs: words (0,4) (1,5) (2,6) (3,7) (8,12) (9,13) (10,14) (11,15)
  // token tau = m (C rows 0/1) or m + 8 (C rows 2/3).
#pragma unroll
  for (int col = 0; col < 2; ++col) {
    uint32_t w[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      // tokens t and t+4 (rows g_), then t+8 and t+12 (rows g_+8)
      const uint32_t sv_a = prmt(svw[t], svw[t + 4], 0x5410);
      const uint32_t sv_b = prmt(svw[t + 8], svw[t + 12], 0x5410);
      w[t] = hmul2_u32(pack_f32x2(s[t][col], s[t + 4][col]), sv_a);
      w[t + 4] = hmul2_u32(pack_f32x2(s[t][col + 2], s[t + 4][col + 2]), sv_b);
    }
    __half* row = ps_warp + (2 * q_ + col) * kPRow + 16 * g_;
    *reinterpret_cast<uint4*>(row) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(row + 8) = make_uint4(w[4], w[5], w[6], w[7]);
  }
  __syncwarp();
}

// B fragments of P' for the 8 token k-steps of the value contraction.
__device__ __forceinline__ void load_pfrags(uint32_t (&pb)[8][2], const __half* ps_warp, int lane) {
  const int mi = lane >> 3, n = lane & 7;
#pragma unroll
  for (int s = 0; s < 8; s += 2) {
    const __half* p = ps_warp + n * kPRow + 16 * (s + (mi >> 1)) + 8 * (mi & 1);
    ldmatrix_x4(pb[s][0], pb[s][1], pb[s + 1][0], pb[s + 1][1], smem_u32(p));
  }
}

__global__ void __launch_bounds__(kThreads, 2)
decode_mma_kernel(const KittyDecodeArgs a, DecodePlan plan) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.d_boost, H = a.num_kv_heads;
  const int g = a.num_q_heads / H;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g_ = lane >> 2, q_ = lane & 3;
  const MmaLayout L = mma_layout(K);

  __half* qnat = reinterpret_cast<__half*>(smem + L.qnat_off);                  // [8][128]
  uint16_t* blist = reinterpret_cast<uint16_t*>(smem + L.blist_off);           // boosted (channel | row << 8)
  int* nb_s = reinterpret_cast<int*>(smem + L.blist_off + 256);
  __half* ps_warp = reinterpret_cast<__half*>(smem + L.p_off) + warp * 8 * kPRow;
  uint8_t* stage0 = smem + L.stages_off + warp * kStages * L.stage_bytes;
  const uint32_t bar0 = smem_u32(smem + L.bars_off) + warp * kStages * 8;

  // ---- per-CTA setup
  const uint16_t* qg = reinterpret_cast<const uint16_t*>(a.q) + b * a.q_s_seq + int64_t(h * g) * a.q_s_head;
  for (int i = tid; i < 8 * kD; i += kThreads) {
    const int qh = i >> 7, c = i & 127;
    qnat[i] = (qh < g) ? __ushort_as_half(qg[qh * a.q_s_head + c]) : __float2half(0.f);
  }
  const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
  if (warp == 0) {
    int base = 0;
    for (int c0 = 0; c0 < kD; c0 += 32) {
      const int c = c0 + lane;
      const int r = bidx[c];
      const bool boosted = r < K;
      const uint32_t bal = __ballot_sync(0xffffffffu, boosted);
      if (boosted) blist[base + __popc(bal & ((1u << lane) - 1u))] = uint16_t(c | (r << 8));
      base += __popc(bal);
    }
    if (lane == 0) *nb_s = base;
  }
  if (tid < kWarps * kStages) mbar_init(smem_u32(smem + L.bars_off) + tid * 8, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();
  const int nb = *nb_s;
  const int n_high_ksteps = (nb + 15) >> 4;

  // q in page order for this thread: channels 16s + q_ + 4e, query head g_
  uint32_t qreg[8][2];
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const uint16_t* qr = reinterpret_cast<const uint16_t*>(qnat) + g_ * kD + 16 * s + q_;
    qreg[s][0] = pack16(qr[0], qr[4]);
    qreg[s][1] = pack16(qr[8], qr[12]);
  }

  WarpState st;
#pragma unroll
  for (int m = 0; m < 8; ++m) st.o[m][0] = st.o[m][1] = st.o[m][2] = st.o[m][3] = 0.f;
  st.zv[0] = st.zv[1] = st.zv[2] = st.zv[3] = 0.f;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;

  const float qk_scale = a.sm_scale * kLog2e;
  const int npages = a.num_pages[b];
  const int p_begin = split * plan.pages_per_split;
  const int p_end = min(npages, p_begin + plan.pages_per_split);
  const int n_split_pages = max(0, p_end - p_begin);
  const int n_my = n_split_pages > warp ? (n_split_pages - warp + kWarps - 1) / kWarps : 0;
  const int32_t* bt = a.block_table + b * a.bt_s_seq;
  const int64_t ph_low = int64_t(kD) * (kG / 4), ph_high = int64_t(K) * (kG / 4);
  const uint32_t bytes_high = uint32_t(ph_high);
  const uint32_t stage_tx = 4096u + 4096u + 512u + 512u + bytes_high;
  bool failed = false;

  auto issue = [&](int i) {  // lane 0 only
    const int stage = i % kStages;
    const uint32_t bar = bar0 + stage * 8;
    const int64_t page = bt[p_begin + warp + i * kWarps];
    uint8_t* dst = stage0 + stage * L.stage_bytes;
    if (page < 0 || page >= a.pool_pages) {  // out-of-range entries are skipped
      mbar_arrive(bar);
      return;
    }
    const int64_t ph = page * H + h;
    mbar_arrive_expect_tx(bar, stage_tx);
    bulk_g2s(smem_u32(dst), a.key_low + ph * ph_low, 4096u, bar);
    bulk_g2s(smem_u32(dst + 4096), a.val_codes + ph * ph_low, 4096u, bar);
    bulk_g2s(smem_u32(dst + 8192), reinterpret_cast<const uint8_t*>(a.key_meta) + ph * (2 * kD * 2), 512u, bar);
    bulk_g2s(smem_u32(dst + 8704), reinterpret_cast<const uint8_t*>(a.val_meta) + ph * (2 * kG * 2), 512u, bar);
    if (bytes_high) bulk_g2s(smem_u32(dst + 9216), a.key_high + ph * ph_high, bytes_high, bar);
  };

  if (lane == 0) {
    for (int i = 0; i < kStages && i < n_my; ++i) issue(i);
  }
  __syncwarp();

  int done = 0;  // pages whose copies have landed
  for (int i = 0; i < n_my; ++i) {
    const int stage = i % kStages;
    if (!mbar_wait(bar0 + stage * 8, (i / kStages) & 1)) {
      failed = true;
      break;
    }
    done = i + 1;
    const int64_t page = bt[p_begin + warp + i * kWarps];
    if (page >= 0 && page < a.pool_pages) {
      const uint8_t* kl = stage0 + stage * L.stage_bytes;
      const uint8_t* vc = kl + 4096;
      const uint8_t* km = kl + 8192;   // scale[128] fp16, zero[128] fp16
      const uint8_t* vm = kl + 8704;   // [t](scale, zero) fp16
      const uint8_t* kh = kl + 9216;

      // ---------------- scores
      float sacc[8][4];
#pragma unroll
      for (int m = 0; m < 8; ++m) sacc[m][0] = sacc[m][1] = sacc[m][2] = sacc[m][3] = 0.f;
      float zk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int c0 = 16 * s + q_;
        const uint32_t sk_lo = pack16(lds16(km + 2 * c0), lds16(km + 2 * (c0 + 4)));
        const uint32_t sk_hi = pack16(lds16(km + 2 * (c0 + 8)), lds16(km + 2 * (c0 + 12)));
        // q * scale as hi + lo fp16 parts: a single fp16 rounding of q * scale loses too much
        // on the large-scale (outlier) channels
        uint32_t b0, b1, c0l, c1l;
        hmul2_split(qreg[s][0], sk_lo, b0, c0l);
        hmul2_split(qreg[s][1], sk_hi, b1, c1l);
        const uint8_t* rowp = kl + c0 * 32 + g_ * 4;
        plane_kstep<true>(sacc, lds32(rowp), lds32(rowp + 4 * 32), lds32(rowp + 8 * 32), lds32(rowp + 12 * 32),
                          b0, b1, c0l, c1l);
        // zero-point tile: row 0 of the A tile holds zp_k (lanes 0..3), other rows 0
        uint32_t z0 = 0u, z2 = 0u;
        if (g_ == 0) {
          const uint8_t* zr = km + 256;
          z0 = pack16(lds16(zr + 2 * c0), lds16(zr + 2 * (c0 + 4)));
          z2 = pack16(lds16(zr + 2 * (c0 + 8)), lds16(zr + 2 * (c0 + 12)));
        }
        mma16816(zk, z0, 0u, z2, 0u, b0, b1);
        mma16816(zk, z0, 0u, z2, 0u, c0l, c1l);
      }
      // high plane: virtual row i = boosted channel #i (row = its boost index)
      for (int hs = 0; hs < n_high_ksteps; ++hs) {
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
        // 4 * q * scale (the high bits weigh 4; scaling by 4 is exact), as hi + lo parts
        uint32_t b0, b1, c0l, c1l;
        hmul2_split(pack16(qv[0], qv[1]), pack16(sv[0], sv[1]), b0, c0l);
        hmul2_split(pack16(qv[2], qv[3]), pack16(sv[2], sv[3]), b1, c1l);
        b0 = hmul2_u32(b0, 0x44004400u); c0l = hmul2_u32(c0l, 0x44004400u);
        b1 = hmul2_u32(b1, 0x44004400u); c1l = hmul2_u32(c1l, 0x44004400u);
        plane_kstep<true>(sacc, w[0], w[1], w[2], w[3], b0, b1, c0l, c1l);
      }
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
      // ---------------- softmax and P'
      uint32_t svw[16];
      {
        const uint4* v4 = reinterpret_cast<const uint4*>(vm + 16 * g_ * 4);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint4 x = v4[t];
          svw[4 * t] = x.x; svw[4 * t + 1] = x.y; svw[4 * t + 2] = x.z; svw[4 * t + 3] = x.w;
        }
      }
      softmax_and_stage(st, sacc, svw, ps_warp, g_, q_);
      uint32_t pb[8][2];
      load_pfrags(pb, ps_warp, lane);
      // ---------------- values
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int t0 = 16 * s + q_;
        const uint8_t* rowp = vc + t0 * 32 + g_ * 4;
        plane_kstep<false>(st.o, lds32(rowp), lds32(rowp + 4 * 32), lds32(rowp + 8 * 32), lds32(rowp + 12 * 32),
                           pb[s][0], pb[s][1]);
        uint32_t z0 = 0u, z2 = 0u;
        if (g_ == 0) {
          z0 = pack16(lds16(vm + 4 * t0 + 2), lds16(vm + 4 * (t0 + 4) + 2));
          z2 = pack16(lds16(vm + 4 * (t0 + 8) + 2), lds16(vm + 4 * (t0 + 12) + 2));
        }
        mma16816(st.zv, z0, 0u, z2, 0u, pb[s][0], pb[s][1]);
      }
    }
    __syncwarp();
    if (lane == 0 && i + kStages < n_my) issue(i + kStages);
    __syncwarp();
  }
  if (failed) {
    if (lane == 0) atomicOr(&g_decode_error, 1u);
    // give copies still in flight (pages done .. issued-1) a bounded chance to land
    // before the shared memory is reused
    const int issued = min(n_my, done + kStages);
    for (int i = done + 1; i < issued; ++i) mbar_wait(bar0 + (i % kStages) * 8, (i / kStages) & 1);
  }

  // ---------------- fp16 regions (split 0): sinks then tail, 128 tokens per chunk
  if (split == 0) {
    const int sink_len = a.sink_len ? a.sink_len[b] : a.sink_len_all;
    const int tail_len = a.tail_len ? a.tail_len[b] : a.tail_len_all;
    const int total = sink_len + tail_len;
    const int nchunks = (total + kG - 1) / kG;
    for (int ch = 0; ch < nchunks; ++ch) {
      if (warp != kWarps - 1 - (ch % kWarps)) continue;
      const int f0 = ch * kG;
      auto krow = [&](int t) -> const uint16_t* {  // fp16 key row of chunk token t (t valid)
        const int ft = f0 + t;
        return ft < sink_len
            ? reinterpret_cast<const uint16_t*>(a.sink_k) + b * a.sk_s_seq + h * a.sk_s_head + ft * a.sk_s_tok
            : reinterpret_cast<const uint16_t*>(a.tail_k) + b * a.tk_s_seq + h * a.tk_s_head +
                  (ft - sink_len) * a.tk_s_tok;
      };
      auto vrow = [&](int t) -> const uint16_t* {
        const int ft = f0 + t;
        return ft < sink_len
            ? reinterpret_cast<const uint16_t*>(a.sink_v) + b * a.sv_s_seq + h * a.sv_s_head + ft * a.sv_s_tok
            : reinterpret_cast<const uint16_t*>(a.tail_v) + b * a.tv_s_seq + h * a.tv_s_head +
                  (ft - sink_len) * a.tv_s_tok;
      };
      const int ntok = min(kG, total - f0);
      float sacc[8][4];
#pragma unroll
      for (int m = 0; m < 8; ++m) sacc[m][0] = sacc[m][1] = sacc[m][2] = sacc[m][3] = 0.f;
      // scores: A rows = tokens 16 g_ + m / m + 8, columns = adjacent channel pairs
      for (int s = 0; s < 8; ++s) {
        const uint16_t* qr = reinterpret_cast<const uint16_t*>(qnat) + g_ * kD + 16 * s + 2 * q_;
        const uint32_t b0 = pack16(qr[0], qr[1]), b1 = pack16(qr[8], qr[9]);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int t_a = 16 * g_ + m, t_b = t_a + 8;
          uint32_t a0 = 0u, a1 = 0u, a2 = 0u, a3 = 0u;
          const int c = 16 * s + 2 * q_;
          if (t_a < ntok) { const uint16_t* r = krow(t_a); a0 = pack16(r[c], r[c + 1]); a2 = pack16(r[c + 8], r[c + 9]); }
          if (t_b < ntok) { const uint16_t* r = krow(t_b); a1 = pack16(r[c], r[c + 1]); a3 = pack16(r[c + 8], r[c + 9]); }
          mma16816(sacc[m], a0, a1, a2, a3, b0, b1);
        }
      }
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const bool va = 16 * g_ + m < ntok, vb = 16 * g_ + m + 8 < ntok;
        sacc[m][0] = va ? sacc[m][0] * qk_scale : -INFINITY;
        sacc[m][1] = va ? sacc[m][1] * qk_scale : -INFINITY;
        sacc[m][2] = vb ? sacc[m][2] * qk_scale : -INFINITY;
        sacc[m][3] = vb ? sacc[m][3] * qk_scale : -INFINITY;
      }
      uint32_t svw[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) svw[t] = 0x3C00u;  // scale 1.0
      softmax_and_stage(st, sacc, svw, ps_warp, g_, q_);
      uint32_t pb[8][2];
      load_pfrags(pb, ps_warp, lane);
      // values: A rows = channels 16 g_ + m / m + 8, columns = tokens 16s + q_ + 4e
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        int tt[4];
        uint32_t ok[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) { tt[e] = 16 * s + q_ + 4 * e; ok[e] = tt[e] < ntok; }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int ca = 16 * g_ + m, cb = ca + 8;
          uint32_t v[4][2];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (ok[e]) { const uint16_t* r = vrow(tt[e]); v[e][0] = r[ca]; v[e][1] = r[cb]; }
            else { v[e][0] = v[e][1] = 0u; }
          }
          mma16816(st.o[m], pack16(v[0][0], v[1][0]), pack16(v[0][1], v[1][1]), pack16(v[2][0], v[3][0]),
                   pack16(v[2][1], v[3][1]), pb[s][0], pb[s][1]);
        }
      }
      __syncwarp();
    }
  }

  // ---------------- finish this warp: reduce l over the token lanes, subtract zero-point sums
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    st.l[0] += __shfl_xor_sync(0xffffffffu, st.l[0], o);
    st.l[1] += __shfl_xor_sync(0xffffffffu, st.l[1], o);
  }
  const float zv0 = __shfl_sync(0xffffffffu, st.zv[0], q_);
  const float zv1 = __shfl_sync(0xffffffffu, st.zv[1], q_);

  // ---------------- merge the 4 warps in shared memory (stage area reused)
  __syncthreads();
  float* mo = reinterpret_cast<float*>(smem + L.stages_off);          // [warp][qh 8][c 128]
  float* mml = mo + kWarps * 8 * kD;                                   // [warp][2][8] (m, l)
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int ca = 16 * g_ + m, cb = ca + 8;
    const int q0 = 2 * q_, q1 = 2 * q_ + 1;
    mo[(warp * 8 + q0) * kD + ca] = st.o[m][0] - zv0;
    mo[(warp * 8 + q1) * kD + ca] = st.o[m][1] - zv1;
    mo[(warp * 8 + q0) * kD + cb] = st.o[m][2] - zv0;
    mo[(warp * 8 + q1) * kD + cb] = st.o[m][3] - zv1;
  }
  if (g_ == 0) {
    mml[(warp * 2 + 0) * 8 + 2 * q_] = st.m[0];
    mml[(warp * 2 + 0) * 8 + 2 * q_ + 1] = st.m[1];
    mml[(warp * 2 + 1) * 8 + 2 * q_] = st.l[0];
    mml[(warp * 2 + 1) * 8 + 2 * q_ + 1] = st.l[1];
  }
  __syncthreads();
  // thread -> (qh, channel block): 8 query heads x 128 channels over 128 threads
  for (int idx = tid; idx < g * kD; idx += kThreads) {
    const int qh = idx >> 7, c = idx & 127;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mml[(w * 2) * 8 + qh]);
    float l = 0.f, o = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = mml[(w * 2) * 8 + qh];
        if (mw != -INFINITY) {
          const float f = ex2(mw - M);
          l += f * mml[(w * 2 + 1) * 8 + qh];
          o += f * mo[(w * 8 + qh) * kD + c];
        }
      }
    }
    if (plan.num_splits == 1) {
      uint16_t* out = reinterpret_cast<uint16_t*>(a.out) + b * a.out_s_seq + int64_t(h * g + qh) * a.out_s_head;
      out[c] = f2h(l > 0.f ? o / l : 0.f);
    } else {
      const int64_t base = ((int64_t(b) * H + h) * plan.num_splits + split) * g + qh;
      plan.ws_o[base * kD + c] = o;
      if (c == 0) {
        plan.ws_m[base] = (M == -INFINITY) ? -INFINITY : M * kLn2;   // natural-log units for the merge
        plan.ws_l[base] = l;
      }
    }
  }
}

}  // namespace

bool mma_supports(const KittyDecodeArgs& a) {
  const int g = a.num_q_heads / a.num_kv_heads;
  return a.head_dim == kD && a.group == kG && g >= 1 && g <= 8 && a.d_boost <= 128 &&
         (a.max_pages_per_seq == 0 ||
          (aligned(a.key_low, 16) && aligned(a.key_meta, 16) && aligned(a.val_codes, 16) &&
           aligned(a.val_meta, 16) && (a.d_boost == 0 || aligned(a.key_high, 16))));
}

int mma_ctas_per_sm() { return 2; }

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

int launch_decode_mma(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  const MmaLayout L = mma_layout(a.d_boost);
  const int merge_bytes = kWarps * 8 * kD * 4 + kWarps * 2 * 8 * 4;
  if (merge_bytes > kWarps * kStages * L.stage_bytes)
    return fail(KITTY_ERR_UNSUPPORTED, "decode_mma: merge scratch does not fit");
  static int configured_bytes = 0;
  if (configured_bytes < L.total) {
    cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
    if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("decode_mma smem attribute: ") + cudaGetErrorString(e));
    configured_bytes = L.total;
  }
  dim3 grid(plan.num_splits, a.num_kv_heads, a.batch);
  decode_mma_kernel<<<grid, kThreads, L.total, stream>>>(a, plan);
  return check_launch("decode_mma_kernel");
}

}  // namespace kitty
