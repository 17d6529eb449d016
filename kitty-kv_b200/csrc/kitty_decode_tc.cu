// Paged GQA decode attention on the fifth-generation tensor cores (tcgen05,
// accumulators in tensor memory), head_dim = group = 128, up to 8 query heads
// per KV head.
//
// One CTA of four warps works on one page-head at a time; its persistent grid
// (four CTAs per SM) splits the walk over (sequence, KV head, page) into equal
// contiguous slices, one partial result per touched segment and slice, merged by
// decode_merge_kernel.  Per page-head:
//
//   keys    The 2-bit codes are unpacked in registers (ldmatrix .trans of the
//           channel-major plane, one AND per code position: code i of every byte
//           scaled by 4^i, code 3 shifted down to 16) and stored into tensor
//           memory as the A operand of a K-major integer MMA: lane = token,
//           4 channels per 32-bit column.  Warp w writes the 32 tokens of its lane
//           quarter.  The boosted channels' high planes follow as one more
//           32-entry K step (4 x high code, same per-token factor).  The B operand
//           is the fixed-point digit table of q * scale_k (three unsigned bytes per
//           (query head, channel) plus an all-ones column per head, as in the
//           integer mma.sync kernel) written to shared memory in the canonical
//           K-major layout.  One thread issues tcgen05.mma.kind::i8 (M = 128 tokens,
//           N = 16 or 32 digit columns, K = 128 + 32), the scores land in tensor
//           memory and each thread reads back 4 consecutive tokens x its query heads.
//   softmax CTA-wide running maximum per query head (one exchange through shared
//           memory per page); every thread keeps its own partial sums.
//   values  P' = p * scale_v as 16-bit fixed point (two digit columns per query
//           head, step from exp2(page max - running max) x max_t scale_v), the
//           value codes unpacked into tensor memory as A (lane = channel, 4 tokens
//           per column), one more MMA (M = 128 channels, N = 16, K = 128 tokens),
//           read back 4 channels x query heads per thread and accumulated in fp32.
//
// Data movement: 1-D bulk async copies (cp.async.bulk, no tensor map, no
// multicast) of the five pieces of the next page-head into the other of two
// shared-memory stages; every wait is bounded and a timeout ends the CTA's walk at
// the next barrier with a device error bit set.
//
// This form runs the quantised pages only: calls whose sequences have fp16 sink
// or tail tokens use the integer mma.sync kernel.
//
// Reference semantics: (code - zp) * scale from kitty/kernels/dequantize_key.py:89-95
// and kitty/kernels/quantize_value.py:121-133; softmax over [sinks ; pages ; tail]
// as in kitty/kernels/attention.py:172-189.

#include <algorithm>

#include "kitty_decode.cuh"
#include "kitty_ptx.cuh"

namespace kitty {

__device__ unsigned int g_decode_error_tc = 0;  // bit 0: a bulk-copy or MMA wait timed out

namespace {

using namespace dev;

constexpr int kD = 128, kG = 128;
constexpr int kThreads = 128;
constexpr int kCtasPerSm = 4;
constexpr int kMaxBoost = 32;
constexpr int kSlotsTarget = 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kKeyRange = 4194300.0f;   // 2^22 - 4
constexpr float kValRange = 65535.0f;
constexpr float kMagicKey = 12582912.0f;  // 1.5 * 2^23
constexpr float kMagicVal = 8388608.0f;   // 2^23

// tensor-memory columns of one CTA's allocation (32-bit columns, 128 lanes)
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kColDk = 0;    // key sums: [token][digit column], 16 or 32 columns
constexpr uint32_t kColDv = 32;   // value sums: [channel][digit column], 16 columns
constexpr uint32_t kColAk = 48;   // key codes: [token][channel byte], 40 columns
constexpr uint32_t kColAv = 88;   // value codes: [channel][token byte], 32 columns
constexpr int kNv = 16;           // value digit columns (8 used with up to 4 query heads)
// digit tables: one block of [column][16 bytes] per (k step, 16-byte K chunk), blocks 16
// bytes apart beyond their size so that the digit-step stores of a warp spread over the banks
__host__ __device__ constexpr int bk_block(int nk) { return nk * 16 + 16; }
constexpr int kBvBlock = kNv * 16 + 16;

// shared memory of one CTA (bytes)
struct TcLayout {
  int kbuf, vbuf, bk, bv, ent, entof, dq, red, reds, red2, pid, flag, bars, size;
};
__host__ __device__ constexpr int tc_kbuf_bytes() { return (4096 + 512 + kMaxBoost * 32 + 32 + 127) & ~127; }
__host__ __device__ constexpr TcLayout tc_layout(int nk) {
  TcLayout L{};
  int o = 0;
  L.kbuf = o; o += 2 * tc_kbuf_bytes();     // two stages: low plane, scale/zero rows, high plane, zero row
  L.vbuf = o; o += 2 * 4608;                // two stages: codes, (scale, zero) per token
  L.bk = o;   o += 5 * 2 * bk_block(nk);    // key digits [k step][16-byte K chunk][column][16 bytes]
  L.bv = o;   o += 4 * 2 * kBvBlock;        // value digits, same layout
  L.ent = o;  o += 4 * 32 * 4;              // per warp: boosted entries (high-plane row offset)
  L.entof = o; o += 4 * 128;                // per warp: entry of each channel (-1: not boosted)
  L.dq = o;   o += 8 * 2 * 4;               // per query head: key digit step, zero-point term
  L.red = o;  o += 4 * 8 * 4;               // per warp and query head: page maximum
  L.reds = o; o += 4 * 4;                   // per warp: largest value scale of the page
  L.red2 = o; o += 4 * 8 * 2 * 4;           // per warp and query head: partial sum, zero-point sum
  L.pid = o;  o += 2 * 4;                   // physical page of each stage (-1: invalid)
  L.flag = o; o += 16;                      // [0]: abort, [1]: tensor-memory base address
  L.bars = o; o += 6 * 8;                   // key copy x2, value copy x2, key MMA, value MMA
  L.size = (o + 127) & ~127;
  return L;
}

// ---- tcgen05 ---------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(slot), "r"(cols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// generic-proxy shared-memory writes made visible to the tensor cores (async proxy)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 lanes x 256 bits: thread (g_, q_) <-> lanes g_ and g_ + 8, columns 2 q_ and 2 q_ + 1
// of every 8-column repetition; registers [4 r .. 4 r + 3] = (g_, 2q_), (g_, 2q_+1),
// (g_+8, 2q_), (g_+8, 2q_+1) of repetition r.
__device__ __forceinline__ void tmem_st_x1(uint32_t t, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1, %2, %3, %4};"
               :: "r"(t), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]) : "memory");
}
__device__ __forceinline__ void tmem_st_x4(uint32_t t, const uint32_t (&v)[16]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
               "%13, %14, %15, %16};"
               :: "r"(t), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
                  "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
               : "memory");
}
__device__ __forceinline__ void tmem_ld_x1(uint32_t t, uint32_t (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(t) : "memory");
}
__device__ __forceinline__ void tmem_ld_x2(uint32_t t, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(t) : "memory");
}
__device__ __forceinline__ void tmem_ld_x4(uint32_t t, uint32_t (&v)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
               "%13, %14, %15}, [%16];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
               : "r"(t) : "memory");
}
// D[tmem] (+)= A[tmem] x B[smem], u8 x u8 -> s32, one elected thread
__device__ __forceinline__ void umma_i8(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n}\n"
      :: "r"(d), "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u) : "memory");
}
// arrive on an mbarrier once every MMA this thread issued has completed
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
}
// shared-memory matrix descriptor: K-major, no swizzle; core matrices of 8 rows x 16
// bytes, lbo = byte distance of the two 16-byte K chunks, sbo = of 8-row groups
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
// instruction descriptor: s32 accumulator, u8 x u8, both K-major, M = 128
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (uint32_t(n >> 3) << 17) | (uint32_t(128 >> 4) << 24);
}

// Bounded wait that suspends the thread until the phase completes (up to 1 ms per try)
// instead of polling: the waits on MMA completion would otherwise take issue slots from
// the other warps.  Gives up after ~2 s.
__device__ __forceinline__ bool mbar_sleep_wait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < 2000; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(bar), "r"(parity), "r"(1000000u) : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ void ldsm_t_x2(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// high code i of every byte, times 4 x its token's factor (1, 4, 16, 16)
template <int i>
__device__ __forceinline__ uint32_t high_code(uint32_t t) {
  return i < 3 ? ((t << 2) & (0x0C0C0C0Cu << (2 * i))) : (t & 0xC0C0C0C0u);
}
__device__ __forceinline__ void bytes01(uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3, uint32_t& w0,
                                        uint32_t& w1) {
  const uint32_t a = prmt(v0, v1, 0x5140u), b = prmt(v2, v3, 0x5140u);
  w0 = prmt(a, b, 0x5410u);
  w1 = prmt(a, b, 0x7632u);
}
__device__ __forceinline__ uint32_t byte2(uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3) {
  return prmt(prmt(v0, v1, 0x0062u), prmt(v2, v3, 0x0062u), 0x5410u);
}
template <bool kBf16>
__device__ __forceinline__ float mul_h16_f32(uint16_t a, uint16_t b) {
  if (kBf16) return Half16<true>::to_f(a) * Half16<true>::to_f(b);
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(0.0f));
  return d;
}

// ---- page walk ---------------------------------------------------------------
// Segments (b, h) in batch-major order, each of num_pages[row of b] pages; the CTAs
// split the concatenated page sequence into equal contiguous slices.

struct PageCur {
  int b, h, p, n, s;   // batch row, KV head, page in segment, pages of the segment, cache row
};

struct PageScan {
  int64_t total, seg_begin;
  int b, h, p;
};

__device__ __forceinline__ int seg_pages(const KittyDecodeArgs& a, int s) { return max(a.num_pages[s], 0); }

// Warp-cooperative: total page count and the segment holding page f (f < total).
__device__ PageScan scan_pages(const KittyDecodeArgs& a, int64_t f, int lane) {
  PageScan r;
  r.b = -1; r.h = 0; r.p = 0; r.seg_begin = 0;
  const int B = a.batch, H = a.num_kv_heads;
  int64_t run = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int64_t n = (b < B) ? seg_pages(a, cache_row(a, b)) : 0;
    const int64_t seq = int64_t(H) * n;
    int64_t incl = seq;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int64_t start = run + incl - seq;
    const bool hit = (b < B) && f >= start && f < start + seq;
    const uint32_t bal = __ballot_sync(0xffffffffu, hit);
    if (bal != 0u && r.b < 0) {
      const int src = __ffs(bal) - 1;
      const int64_t st = __shfl_sync(0xffffffffu, start, src);
      const int64_t ns = __shfl_sync(0xffffffffu, n, src);
      r.b = b0 + src;
      r.h = int((f - st) / ns);
      r.p = int((f - st) - int64_t(r.h) * ns);
      r.seg_begin = st + int64_t(r.h) * ns;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  r.total = run;
  return r;
}

// next page; false past the last one (segments without pages are skipped)
__device__ __forceinline__ bool page_step(PageCur& c, const KittyDecodeArgs& a) {
  if (++c.p < c.n) return true;
  c.p = 0;
  for (;;) {
    if (++c.h == a.num_kv_heads) {
      c.h = 0;
      if (++c.b >= a.batch) return false;
      c.s = cache_row(a, c.b);
      c.n = seg_pages(a, c.s);
    }
    if (c.n > 0) return true;
    c.h = a.num_kv_heads - 1;   // no pages in this sequence: move on to the next one
  }
}

// column of digit plane pl (0: b0, 1: b1, 2: b2, 3: all ones) of query head hq in the
// key sums: thread q_ reads heads q_ and q_ + 4, (b0, b1) from one 8-column repetition
// and (b2, ones) from the next
__device__ __forceinline__ int key_col(int hq, int pl) {
  return 8 * (2 * (hq >> 2) + (pl >> 1)) + 2 * (hq & 3) + (pl & 1);
}

template <bool kBf16, bool kH8>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
decode_tc_kernel(const KittyDecodeArgs a, DecodePlan plan) {
  using T = Half16<kBf16>;
  constexpr int kNk = kH8 ? 32 : 16;   // key digit columns
  constexpr int kHL = kH8 ? 2 : 1;     // query heads per thread (q_ and q_ + 4)
  constexpr int kCpt = kH8 ? 8 : 4;    // digit step: channels per thread
  constexpr int kTph = 128 / kCpt;     // digit step: threads per query head
  constexpr TcLayout L = tc_layout(kNk);
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g_ = lane >> 2, q_ = lane & 3;
  const int H = a.num_kv_heads, K = a.d_boost;
  const int g = a.num_q_heads / H;

  // ---- this CTA's slice of the page sequence
  PageScan sc = scan_pages(a, 0, lane);
  const int64_t total = sc.total;
  int64_t F = (total + gridDim.x - 1) / gridDim.x;
  if (F < plan.pages_per_split) F = plan.pages_per_split;
  const int64_t f0 = int64_t(blockIdx.x) * F;
  if (f0 >= total) return;   // the same for every thread of the CTA, before any allocation
  const int64_t f1 = min(total, f0 + F);
  sc = scan_pages(a, f0, lane);
  int slot = int(int64_t(blockIdx.x) - sc.seg_begin / F);

  uint8_t* kbuf0 = smem + L.kbuf;
  uint8_t* vbuf0 = smem + L.vbuf;
  uint8_t* bk = smem + L.bk;
  uint8_t* bv = smem + L.bv;
  uint32_t* ent = reinterpret_cast<uint32_t*>(smem + L.ent) + 32 * warp;
  int8_t* entof = reinterpret_cast<int8_t*>(smem + L.entof) + 128 * warp;
  float* dq = reinterpret_cast<float*>(smem + L.dq);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* reds = reinterpret_cast<float*>(smem + L.reds);
  float* red2 = reinterpret_cast<float*>(smem + L.red2);
  int* pid = reinterpret_cast<int*>(smem + L.pid);
  volatile int* flag = reinterpret_cast<volatile int*>(smem + L.flag);
  const uint32_t bars = smem_u32(smem + L.bars);
  auto bar_kc = [&](int s) { return bars + 8u * s; };
  auto bar_vc = [&](int s) { return bars + 16u + 8u * s; };
  const uint32_t bar_mk = bars + 32u, bar_mv = bars + 40u;
  auto kbuf = [&](int s) { return kbuf0 + s * tc_kbuf_bytes(); };
  auto vbuf = [&](int s) { return vbuf0 + s * 4608; };

  // ---- set-up: barriers, constant digit columns, zero rows, tensor memory
  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(bars + 8u * i, 1);
    flag[0] = 0;
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  for (int i = tid; i < 5 * 2 * kNk * 4; i += kThreads) {   // words of the key digit table
    const int blk = i / (kNk * 4), n = (i >> 2) % kNk;
    const bool ones = (n & 8) != 0 && (n & 1) != 0;          // plane 3 columns (key_col(hq, 3))
    reinterpret_cast<uint32_t*>(bk + blk * bk_block(kNk))[i - blk * kNk * 4] = ones ? 0x01010101u : 0u;
  }
  for (int i = tid; i < 2 * 8; i += kThreads)
    reinterpret_cast<uint32_t*>(kbuf(i >> 3) + 4608 + K * 32)[i & 7] = 0u;   // zero row after the high plane
  if (warp == 0) {
    tmem_alloc(smem_u32(smem + L.flag + 4), kTmemCols);
    tmem_relinquish();
  }
  fence_async_smem();
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  const uint32_t tbase = flag[1];
  const uint32_t t_lane0 = tbase + (uint32_t(32 * warp) << 16);   // this warp's lane quarter
  const uint32_t t_lane16 = t_lane0 + (16u << 16);

  const float qk_scale = a.sm_scale * kLog2e;
  const uint32_t bytes_high = uint32_t(K) * 32u;
  uint32_t kph[2] = {0u, 0u}, vph[2] = {0u, 0u}, mkph = 0u, mvph = 0u;

  // ---- producer (warp 1): copies of the next page-heads, block-table window in its lanes;
  // the MMAs are issued by thread 0, so the two single-thread roles sit in different warps
  constexpr int kProducer = 1;
  PageCur pc{sc.b, sc.h, sc.p, seg_pages(a, cache_row(a, sc.b)), cache_row(a, sc.b)};
  int64_t pf = f0;
  uint32_t pend_k = 0u, pend_v = 0u;   // producer warp: stages with copies not yet waited for
  int bt_row = -1, bt_base = 0, bt_val = 0;
  auto issue = [&](int stage) {   // producer warp, converged
    const int idx = pc.p;
    if (pc.s != bt_row || idx < bt_base || idx >= bt_base + 32) {
      bt_row = pc.s;
      bt_base = idx;
      const int e = idx + lane;
      bt_val = e < pc.n ? a.block_table[int64_t(pc.s) * a.bt_s_seq + e] : -1;
    }
    const int page = __shfl_sync(0xffffffffu, bt_val, idx - bt_base);
    const bool ok = page >= 0 && page < a.pool_pages;
    if (lane == 0) {
      pid[stage] = ok ? page : -1;
      const int64_t phh = int64_t(ok ? page : 0) * H + pc.h;
      uint8_t* kb = kbuf(stage);
      uint8_t* vb = vbuf(stage);
      mbar_arrive_expect_tx(bar_kc(stage), 4608u + bytes_high);
      bulk_g2s(smem_u32(kb), a.key_low + phh * 4096, 4096u, bar_kc(stage));
      bulk_g2s(smem_u32(kb + 4096), reinterpret_cast<const uint8_t*>(a.key_meta) + phh * 512, 512u, bar_kc(stage));
      if (bytes_high) bulk_g2s(smem_u32(kb + 4608), a.key_high + phh * bytes_high, bytes_high, bar_kc(stage));
      mbar_arrive_expect_tx(bar_vc(stage), 4608u);
      bulk_g2s(smem_u32(vb), a.val_codes + phh * 4096, 4096u, bar_vc(stage));
      bulk_g2s(smem_u32(vb + 4096), reinterpret_cast<const uint8_t*>(a.val_meta) + phh * 512, 512u, bar_vc(stage));
    }
    pend_k |= 1u << stage;
    pend_v |= 1u << stage;
    page_step(pc, a);
    ++pf;
  };
  if (warp == kProducer) {
    if (pf < f1) issue(0);
    if (pf < f1) issue(1);
  }

  // ---- consumer state: query heads q_ + 4 j, channels 32 warp + 4 g_ + t
  PageCur pos{sc.b, sc.h, sc.p, seg_pages(a, cache_row(a, sc.b)), cache_row(a, sc.b)};
  float o[kHL][4], m[kHL], l[kHL], zs[kHL];
  auto reset = [&]() {
#pragma unroll
    for (int j = 0; j < kHL; ++j) {
      m[j] = -INFINITY; l[j] = 0.f; zs[j] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[j][i] = 0.f;
    }
  };
  reset();
  // the page whose value MMA is in flight: its softmax factors and where its result goes
  float alpha_p[kHL], dv_p[kHL];
#pragma unroll
  for (int j = 0; j < kHL; ++j) alpha_p[j] = dv_p[j] = 0.f;
  bool pend_val = false, p_seg_end = false, p_last = false;
  int p_b = 0, p_h = 0, p_slot = 0;
  // digit-step role: query head dh, channels dc .. dc + kCpt - 1
  const int dh = tid / kTph, dc = kCpt * (tid % kTph);
  uint32_t qv[kCpt / 2];
  int nb = 0;
  bool bad = false;
  const int sel = warp & 1;                                  // ldmatrix column half of this warp's bytes
  const uint32_t krow_off = 32u * lane + 16u * (warp >> 1);  // ldmatrix row address offset

  // value sums of the pending page into the fp32 accumulators
  auto value_epilogue = [&]() {
    if (!mbar_sleep_wait(bar_mv, mvph)) bad = true;
    mvph ^= 1u;
    tc_after_sync();
    uint32_t v0[4 * kHL], v1[4 * kHL];
    if constexpr (kH8) {
      tmem_ld_x2(t_lane0 + kColDv, v0);
      tmem_ld_x2(t_lane16 + kColDv, v1);
    } else {
      tmem_ld_x1(t_lane0 + kColDv, v0);
      tmem_ld_x1(t_lane16 + kColDv, v1);
    }
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < kHL; ++j)
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t* v = t < 2 ? v0 : v1;
        const int e = t & 1;
        const int c = 256 * int(v[4 * j + 2 * e + 1]) + int(v[4 * j + 2 * e]);
        const float fct = dv_p[j] * (t == 0 ? 1.0f : t == 1 ? 0.25f : t == 2 ? 0.0625f : 0.015625f);
        o[j][t] = __fmaf_rn(float(c), fct, o[j][t] * alpha_p[j]);
      }
  };
  // partial result of segment (b, h) over this slice into workspace slot `slot`
  auto write_partial = [&](int b, int h, int slot, bool seg_end) {
#pragma unroll
    for (int j = 0; j < kHL; ++j) {
      float lt = l[j], zt = zs[j];
      lt += __shfl_xor_sync(0xffffffffu, lt, 4);
      lt += __shfl_xor_sync(0xffffffffu, lt, 8);
      lt += __shfl_xor_sync(0xffffffffu, lt, 16);
      zt += __shfl_xor_sync(0xffffffffu, zt, 4);
      zt += __shfl_xor_sync(0xffffffffu, zt, 8);
      zt += __shfl_xor_sync(0xffffffffu, zt, 16);
      if (g_ == 0) {
        red2[2 * (8 * warp + q_ + 4 * j)] = lt;
        red2[2 * (8 * warp + q_ + 4 * j) + 1] = zt;
      }
    }
    __syncthreads();
    const int64_t base = ((int64_t(b) * H + h) * plan.num_splits + slot) * g;
#pragma unroll
    for (int j = 0; j < kHL; ++j) {
      const int hq = q_ + 4 * j;
      float Lh = 0.f, Zh = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < 4; ++w2) {
        Lh += red2[2 * (8 * w2 + hq)];
        Zh += red2[2 * (8 * w2 + hq) + 1];
      }
      if (hq < g) {
        *reinterpret_cast<float4*>(plan.ws_o + (base + hq) * kD + 32 * warp + 4 * g_) =
            make_float4(o[j][0] - Zh, o[j][1] - Zh, o[j][2] - Zh, o[j][3] - Zh);
        if (warp == 0 && g_ == 0) {
          plan.ws_m[base + hq] = m[j] == -INFINITY ? -INFINITY : m[j] * kLn2;
          plan.ws_l[base + hq] = Lh;
        }
      }
    }
    if (seg_end && tid == 0) plan.ws_count[int64_t(b) * H + h] = slot + 1;
    reset();
  };

  bool aborted = false;
  for (int64_t f = f0; f < f1; ++f) {
    const int s = int(f - f0) & 1;
    const int b = pos.b, h = pos.h;
    if (pos.p == 0 || f == f0) {
      // segment set-up: boosted entries of KV head h (per warp), this thread's q
      const uint8_t* bidx = a.boost_idx + h * a.bidx_s_head;
      nb = 0;
      for (int c0 = 0; c0 < kD; c0 += 32) {
        const int c = c0 + lane;
        const int r = bidx[c];
        const bool boosted = r < K;
        const uint32_t bal = __ballot_sync(0xffffffffu, boosted);
        const int e = nb + __popc(bal & ((1u << lane) - 1u));
        if (boosted && e < kMaxBoost) ent[e] = uint32_t(r) * 32u;
        entof[c] = int8_t(boosted && e < kMaxBoost ? e : -1);
        nb += __popc(bal);
      }
      if (nb > kMaxBoost) nb = kMaxBoost;   // never reached: the host routes d_boost > 32 elsewhere
      if (lane >= nb) ent[lane] = uint32_t(K) * 32u;   // zero row
      __syncwarp();
      const int qh = h * g + dh;
      const uint16_t* qsrc = reinterpret_cast<const uint16_t*>(a.q) + b * a.q_s_seq + int64_t(qh) * a.q_s_head + dc;
      if constexpr (kCpt == 8) {
        const uint4 x = dh < g ? *reinterpret_cast<const uint4*>(qsrc) : make_uint4(0u, 0u, 0u, 0u);
        qv[0] = x.x; qv[1] = x.y; qv[2] = x.z; qv[3] = x.w;
      } else {
        const uint2 x = dh < g ? *reinterpret_cast<const uint2*>(qsrc) : make_uint2(0u, 0u);
        qv[0] = x.x; qv[1] = x.y;
      }
    }

    // ---- 1. keys of this page: codes into tensor memory, digits into shared memory
    if (!mbar_sleep_wait(bar_kc(s), kph[s])) bad = true;
    kph[s] ^= 1u;
    pend_k &= ~(1u << s);
    const uint8_t* kb = kbuf(s);
    {
      uint32_t a0[16], a1[16];
      const uint32_t krow = smem_u32(kb) + krow_off;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t r[4];
        ldsm_t_x2(krow + 1024u * ks, r);
        const uint32_t x0 = sel ? r[1] : r[0], x1 = sel ? r[3] : r[2];
        a0[4 * ks + 0] = x0 & 0x03030303u;          // code 0 (lane row g_)
        a0[4 * ks + 1] = x1 & 0x03030303u;
        a0[4 * ks + 2] = x0 & 0x0C0C0C0Cu;          // code 1 x 4 (lane row g_ + 8)
        a0[4 * ks + 3] = x1 & 0x0C0C0C0Cu;
        a1[4 * ks + 0] = x0 & 0x30303030u;          // code 2 x 16 (second 16-lane block)
        a1[4 * ks + 1] = x1 & 0x30303030u;
        a1[4 * ks + 2] = (x0 >> 2) & 0x30303030u;   // code 3 x 16
        a1[4 * ks + 3] = (x1 >> 2) & 0x30303030u;
      }
      tmem_st_x4(t_lane0 + kColAk, a0);
      tmem_st_x4(t_lane16 + kColAk, a1);
      if (nb > 0) {
        uint32_t r[4];
        ldsm_t_x2(smem_u32(kb + 4608) + ent[lane] + 16u * (warp >> 1), r);
        const uint32_t x0 = sel ? r[1] : r[0], x1 = sel ? r[3] : r[2];
        const uint32_t h0[4] = {high_code<0>(x0), high_code<0>(x1), high_code<1>(x0), high_code<1>(x1)};
        const uint32_t h1[4] = {high_code<2>(x0), high_code<2>(x1), high_code<3>(x0), high_code<3>(x1)};
        tmem_st_x1(t_lane0 + kColAk + 32, h0);
        tmem_st_x1(t_lane16 + kColAk + 32, h1);
      }
    }
    {
      // digit step: w = q * scale_k exact in fp32, x = rint(w R) in three bytes
      const uint16_t* sc16 = reinterpret_cast<const uint16_t*>(kb + 4096) + dc;
      const uint16_t* zp16 = reinterpret_cast<const uint16_t*>(kb + 4096 + 256) + dc;
      uint32_t sw[kCpt / 2], zw[kCpt / 2];
      if constexpr (kCpt == 8) {
        const uint4 x = *reinterpret_cast<const uint4*>(sc16), y = *reinterpret_cast<const uint4*>(zp16);
        sw[0] = x.x; sw[1] = x.y; sw[2] = x.z; sw[3] = x.w;
        zw[0] = y.x; zw[1] = y.y; zw[2] = y.z; zw[3] = y.w;
      } else {
        const uint2 x = *reinterpret_cast<const uint2*>(sc16), y = *reinterpret_cast<const uint2*>(zp16);
        sw[0] = x.x; sw[1] = x.y; zw[0] = y.x; zw[1] = y.y;
      }
      float w[kCpt];
      float mx = 0.f;
#pragma unroll
      for (int j = 0; j < kCpt / 2; ++j) {
        w[2 * j] = mul_h16_f32<kBf16>(uint16_t(qv[j] & 0xffffu), uint16_t(sw[j] & 0xffffu));
        w[2 * j + 1] = mul_h16_f32<kBf16>(uint16_t(qv[j] >> 16), uint16_t(sw[j] >> 16));
        mx = fmaxf(mx, fmaxf(fabsf(w[2 * j]), fabsf(w[2 * j + 1])));
      }
#pragma unroll
      for (int o2 = 1; o2 < kTph && o2 < 32; o2 <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
      const float R = mx > 0.f ? kKeyRange * rcp_approx(mx) : 0.f;
      uint32_t fb[kCpt];
      float2 zs2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kCpt / 2; ++j) {
        const float2 wj = make_float2(w[2 * j], w[2 * j + 1]);
        const float2 fr = fma2(wj, make_float2(R, R), make_float2(kMagicKey, kMagicKey));
        fb[2 * j] = __float_as_uint(fr.x);
        fb[2 * j + 1] = __float_as_uint(fr.y);
        zs2 = fma2(T::to_f2(zw[j]), wj, zs2);
      }
      float zsum = zs2.x + zs2.y;
#pragma unroll
      for (int o2 = 1; o2 < kTph && o2 < 32; o2 <<= 1) zsum += __shfl_xor_sync(0xffffffffu, zsum, o2);
      if (tid % kTph == 0) {
        dq[2 * dh] = mx * (1.0f / kKeyRange) * qk_scale;
        dq[2 * dh + 1] = zsum * qk_scale;
      }
      // four consecutive channels c0 .. c0 + 3 <-> K bytes of column 2 q + e' of k step ks,
      // where c0 = 32 ks + 16 e' + 4 q
#pragma unroll
      for (int grp = 0; grp < kCpt / 4; ++grp) {
        const int c0 = dc + 4 * grp;
        const int ks = c0 >> 5, e1 = (c0 >> 4) & 1, qq = (c0 >> 2) & 3;
        const int kc = 2 * qq + e1;
        uint8_t* dst = bk + (ks * 2 + (kc >> 2)) * bk_block(kNk) + 4 * (kc & 3);
        uint32_t d0, d1;
        bytes01(fb[4 * grp], fb[4 * grp + 1], fb[4 * grp + 2], fb[4 * grp + 3], d0, d1);
        const uint32_t d2 = byte2(fb[4 * grp], fb[4 * grp + 1], fb[4 * grp + 2], fb[4 * grp + 3]);
        *reinterpret_cast<uint32_t*>(dst + key_col(dh, 0) * 16) = d0;
        *reinterpret_cast<uint32_t*>(dst + key_col(dh, 1) * 16) = d1;
        *reinterpret_cast<uint32_t*>(dst + key_col(dh, 2) * 16) = d2;
      }
      // boosted channels: the same digits in their entry's row of the extra K step
#pragma unroll
      for (int j = 0; j < kCpt; ++j) {
        const int e = entof[dc + j];
        if (e >= 0) {
          // entry e = 16 e' + 4 q + j sits in K column 2 q + e' of the extra step, byte j
          const int kc = 2 * ((e >> 2) & 3) + (e >> 4);
          uint8_t* dst = bk + (4 * 2 + (kc >> 2)) * bk_block(kNk) + 4 * (kc & 3) + (e & 3);
          dst[key_col(dh, 0) * 16] = uint8_t(fb[j]);
          dst[key_col(dh, 1) * 16] = uint8_t(fb[j] >> 8);
          dst[key_col(dh, 2) * 16] = uint8_t(fb[j] >> 16);
        }
      }
    }

    // ---- 2. the previous page's value sums (its MMA ran behind this page's key work)
    if (pend_val) {
      value_epilogue();
      pend_val = false;
      if (p_seg_end || p_last) write_partial(p_b, p_h, p_slot, p_seg_end);
    }

    if (bad) flag[0] = 1;
    tmem_wait_st();
    fence_async_smem();
    tc_before_sync();
    __syncthreads();   // ---- A: key operands ready
    tc_after_sync();
    if (flag[0]) { aborted = true; break; }
    if (tid == 0) {
      const uint32_t idk = idesc_i8(kNk);
      const uint32_t lbo = bk_block(kNk), sbo = 128;
      const int ksteps = nb > 0 ? 5 : 4;
      for (int ks = 0; ks < ksteps; ++ks)
        umma_i8(tbase + kColDk, tbase + kColAk + 8u * ks,
                smem_desc(smem_u32(bk + ks * 2 * bk_block(kNk)), lbo, sbo), idk, ks > 0 ? 1u : 0u);
      umma_commit(bar_mk);
    }

    // ---- 3. values of this page: codes into tensor memory, scales into registers
    if (!mbar_sleep_wait(bar_vc(s), vph[s])) bad = true;
    vph[s] ^= 1u;
    pend_v &= ~(1u << s);
    const uint8_t* vbp = vbuf(s);
    {
      uint32_t a0[16], a1[16];
      const uint32_t vrow = smem_u32(vbp) + krow_off;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t r[4];
        ldsm_t_x2(vrow + 1024u * ks, r);
        const uint32_t x0 = sel ? r[1] : r[0], x1 = sel ? r[3] : r[2];
        a0[4 * ks + 0] = x0 & 0x03030303u;
        a0[4 * ks + 1] = x1 & 0x03030303u;
        a0[4 * ks + 2] = x0 & 0x0C0C0C0Cu;
        a0[4 * ks + 3] = x1 & 0x0C0C0C0Cu;
        a1[4 * ks + 0] = x0 & 0x30303030u;
        a1[4 * ks + 1] = x1 & 0x30303030u;
        a1[4 * ks + 2] = x0 & 0xC0C0C0C0u;
        a1[4 * ks + 3] = x1 & 0xC0C0C0C0u;
      }
      tmem_st_x4(t_lane0 + kColAv, a0);
      tmem_st_x4(t_lane16 + kColAv, a1);
    }
    // (scale, zero) of this thread's tokens 32 warp + 4 g_ + 0..3
    const uint4 szv = *reinterpret_cast<const uint4*>(vbp + 4096 + 4 * (32 * warp + 4 * g_));
    const uint32_t sz[4] = {szv.x, szv.y, szv.z, szv.w};
    float smax = fmaxf(fmaxf(T::lo_f(sz[0]), T::lo_f(sz[1])), fmaxf(T::lo_f(sz[2]), T::lo_f(sz[3])));
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o2));

    // ---- 4. scores: thread tokens 32 warp + 4 g_ + t (t = 2 block + row), heads q_ + 4 j
    if (!mbar_sleep_wait(bar_mk, mkph)) bad = true;
    mkph ^= 1u;
    tc_after_sync();
    const bool valid = pid[s] >= 0;
    float sco[kHL][4];
    {
      uint32_t d0[kNk / 2], d1[kNk / 2];
      if constexpr (kH8) {
        tmem_ld_x4(t_lane0 + kColDk, d0);
        tmem_ld_x4(t_lane16 + kColDk, d1);
      } else {
        tmem_ld_x2(t_lane0 + kColDk, d0);
        tmem_ld_x2(t_lane16 + kColDk, d1);
      }
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < kHL; ++j) {
        const float cq = dq[2 * (q_ + 4 * j)], zq = dq[2 * (q_ + 4 * j) + 1];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t* d = t < 2 ? d0 : d1;
          const int e = t & 1;
          const int b0v = int(d[8 * j + 2 * e]), b1v = int(d[8 * j + 2 * e + 1]);
          const int b2v = int(d[8 * j + 4 + 2 * e]), onev = int(d[8 * j + 4 + 2 * e + 1]);
          const float fct = cq * (t == 0 ? 1.0f : t == 1 ? 0.25f : 0.0625f);
          const int lo = 256 * b1v + b0v, hi = b2v - 64 * onev;
          sco[j][t] = valid ? __fmaf_rn(float(hi), fct * 65536.0f, __fmaf_rn(float(lo), fct, -zq)) : -INFINITY;
        }
        float mx = fmaxf(fmaxf(sco[j][0], sco[j][1]), fmaxf(sco[j][2], sco[j][3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        if (g_ == 0) red[8 * warp + q_ + 4 * j] = mx;
      }
    }
    if (lane == 0) reds[warp] = smax;
    if (bad) flag[0] = 1;
    tc_before_sync();
    __syncthreads();   // ---- B: page maxima exchanged
    tc_after_sync();
    if (flag[0]) { aborted = true; break; }

    // ---- 5. softmax step, P' digits into shared memory
    {
      const float vmax = fmaxf(fmaxf(reds[0], reds[1]), fmaxf(reds[2], reds[3]));
      const int kc = 2 * (g_ & 3) + (g_ >> 2);   // K column of tokens 4 g_ .. 4 g_ + 3 in k step `warp`
      uint8_t* dst = bv + (warp * 2 + (kc >> 2)) * kBvBlock + 4 * (kc & 3);
#pragma unroll
      for (int j = 0; j < kHL; ++j) {
        const int hq = q_ + 4 * j;
        const float pm = fmaxf(fmaxf(red[hq], red[8 + hq]), fmaxf(red[16 + hq], red[24 + hq]));
        const float mn = fmaxf(m[j], pm);
        const float alpha = (m[j] == -INFINITY) ? 0.f : ex2(m[j] - mn);
        const float base = (mn == -INFINITY) ? 0.f : mn;
        m[j] = mn;
        float p[4], psum = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          p[t] = ex2(sco[j][t] - base);
          psum += p[t];
        }
        l[j] = __fmaf_rn(l[j], alpha, psum);
        // P' <= exp2(page max - running max) * max_t scale_v: the digit step of this page
        const float bound = (pm == -INFINITY) ? 0.f : ex2(pm - base) * vmax;
        const float Rv = bound > 1e-30f ? kValRange * rcp_approx(bound) : 0.f;
        const float dvj = bound * (1.0f / kValRange);
        uint32_t yb[4];
        float zv = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float pp = p[t] * T::lo_f(sz[t]);
          const float fy = __fmaf_rn(pp, Rv, kMagicVal);
          yb[t] = __float_as_uint(fy);
          zv = __fmaf_rn(T::hi_f(sz[t]), fy - kMagicVal, zv);
        }
        zs[j] = __fmaf_rn(zv, dvj, zs[j] * alpha);
        alpha_p[j] = alpha;
        dv_p[j] = dvj;
        uint32_t y0, y1;
        bytes01(yb[0], yb[1], yb[2], yb[3], y0, y1);
        *reinterpret_cast<uint32_t*>(dst + (8 * j + 2 * q_) * 16) = y0;
        *reinterpret_cast<uint32_t*>(dst + (8 * j + 2 * q_ + 1) * 16) = y1;
      }
    }
    tmem_wait_st();
    fence_async_smem();
    tc_before_sync();
    __syncthreads();   // ---- C: value operands ready; stage s free
    tc_after_sync();
    if (flag[0]) { aborted = true; break; }
    if (tid == 0) {
      const uint32_t idv = idesc_i8(kNv);
      for (int ks = 0; ks < 4; ++ks)
        umma_i8(tbase + kColDv, tbase + kColAv + 8u * ks, smem_desc(smem_u32(bv + ks * 2 * kBvBlock), kBvBlock, 128),
                idv, ks > 0 ? 1u : 0u);
      umma_commit(bar_mv);
    }
    if (warp == kProducer && pf < f1) issue(s);

    // ---- 6. this page's value sums are read at the next page (or after the walk)
    pend_val = true;
    p_b = b; p_h = h; p_slot = slot;
    p_seg_end = pos.p + 1 >= pos.n;
    p_last = f + 1 >= f1;
    if (p_seg_end) slot = 0;
    page_step(pos, a);
  }
  if (pend_val && !aborted) {
    value_epilogue();
    write_partial(p_b, p_h, p_slot, p_seg_end);
  }

  // ---- end: drain copies still in flight (a walk that ended early), free tensor memory
  if (tid == 0 && (flag[0] || bad)) atomicOr(&g_decode_error_tc, 1u);
  tc_before_sync();
  __syncthreads();
  if (warp == kProducer && lane == 0) {
    // copies issued but not consumed: let them land (bounded waits) before the CTA's
    // shared memory is released
    for (int st = 0; st < 2; ++st) {
      if (pend_k & (1u << st)) mbar_sleep_wait(bar_kc(st), kph[st]);
      if (pend_v & (1u << st)) mbar_sleep_wait(bar_vc(st), vph[st]);
    }
  }
  __syncthreads();
  tc_after_sync();
  if (warp == 0) tmem_dealloc(tbase, kTmemCols);
}

}  // namespace

bool tc_supports(const KittyDecodeArgs& a) {
  const int g = a.num_q_heads / a.num_kv_heads;
  const bool no_fp16 = !a.sink_len && a.sink_len_all == 0 && !a.tail_len && a.tail_len_all == 0;
  return no_fp16 && a.head_dim == kD && a.group == kG && g >= 1 && g <= 8 && a.d_boost <= kMaxBoost &&
         a.max_pages_per_seq > 0 && aligned(a.q, 16) && a.q_s_seq % 8 == 0 && a.q_s_head % 8 == 0 &&
         aligned(a.key_low, 16) && aligned(a.key_meta, 16) && aligned(a.val_codes, 16) && aligned(a.val_meta, 16) &&
         (a.d_boost == 0 || aligned(a.key_high, 16));
}

void tc_plan(const KittyDecodeArgs& a, int sm_count, DecodePlan* plan) {
  const int maxp = std::max(1, a.max_pages_per_seq);
  const int target = a.num_splits > 0 ? std::min(a.num_splits, kMaxDecodeSlots - 1) : kSlotsTarget;
  const int f_min = (maxp + target - 1) / target;
  plan->pages_per_split = f_min;
  plan->num_splits = (maxp + f_min - 1) / f_min + 1;
  const int64_t total_max = int64_t(a.batch) * a.num_kv_heads * maxp;
  plan->grid = int(std::max<int64_t>(1, std::min<int64_t>((total_max + f_min - 1) / f_min,
                                                          int64_t(sm_count) * kCtasPerSm)));
}

int launch_decode_tc(const KittyDecodeArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  const int g = a.num_q_heads / a.num_kv_heads;
  const bool h8 = g > 4, bf16 = a.dtype == KITTY_DTYPE_BF16;
  // at least 48 KB per CTA, so that no more than four CTAs (4 x 128 tensor-memory
  // columns = all 512) are ever resident on an SM and no allocation has to wait
  const int smem = std::max(tc_layout(h8 ? 32 : 16).size, 48 * 1024);
  auto kern = h8 ? (bf16 ? decode_tc_kernel<true, true> : decode_tc_kernel<false, true>)
                 : (bf16 ? decode_tc_kernel<true, false> : decode_tc_kernel<false, false>);
  static int configured = 0;   // bit per instantiation
  const int bit = (h8 ? 2 : 1) << (bf16 ? 2 : 0);
  if (!(configured & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("decode_tc smem attribute: ") + cudaGetErrorString(e));
    configured |= bit;
  }
  kern<<<plan.grid, kThreads, smem, stream>>>(a, plan);
  return check_launch("decode_tc_kernel");
}

int read_decode_error_tc(uint32_t* flags, int clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_decode_error_tc, sizeof(v));
  if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("read error flags: ") + cudaGetErrorString(e));
  if (clear && v) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_decode_error_tc, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("clear error flags: ") + cudaGetErrorString(e));
  }
  *flags = v;
  return KITTY_OK;
}

}  // namespace kitty
