// Device-resident cache state: batched append with in-step page flushes, bulk
// append (prefill), release and reset (kitty_cache_* in the C ABI).
//
// A decode step of n sequences runs four launches and no host synchronisation:
//   1. append_plan_kernel (one CTA): per token, the sequence's next slot (a sink
//      position or a buffer position); sequences whose G-token buffer fills pop a
//      page from the free stack, in token order (a block-wide prefix sum, so the
//      page assignment is deterministic), and record a quantisation job;
//   2. append_copy_kernel: the fp16 key / value rows into their slots (16-byte
//      vectors), and the duplicate-detection claims cleared;
//   3. + 4. the page quantisers over the recorded jobs (jobs without a page skip).
// A prefill (many tokens per sequence) plans every sequence at once in the same
// way and quantises all full G-token groups straight from the source rows.
// The state machine per sequence is the reference pipeline's push_token
// (kitty/pipeline.py:115-181: sinks first, then the Key Q-buffer, a flush when it
// holds G tokens) with the values of the same tokens in a parallel buffer, and
// the allocator is a stack in place of PageCentricKVLayoutManager's free mask
// (kitty/layout.py:161-220).
#include <cuda_runtime.h>

#include <algorithm>

#include "kitty_common.cuh"

namespace kitty {

int quantize_key_pages_impl(const KittyKeyQuantArgs* a, void* stream);
int quantize_value_pages_impl(const KittyValueQuantArgs* a, void* stream);

__device__ unsigned int g_cache_error = 0;

namespace {

constexpr uint32_t kErrNoPage = 1u << 1;      // free stack empty
constexpr uint32_t kErrTableFull = 1u << 2;   // block table row full
constexpr uint32_t kErrBadSeq = 1u << 3;      // id out of range or repeated in one batch
constexpr uint32_t kErrOverflow = 1u << 4;    // release would overflow the stack
constexpr uint32_t kErrBudget = 1u << 5;      // prefill: more source pages than max_pages

constexpr int kPlanThreads = 1024;
constexpr int32_t kTailSlot = 1 << 30;        // job_slot: kTailSlot | pos = buffer slot, pos = sink slot

// Block-wide exclusive prefix sum of v (blockDim.x == kPlanThreads); *total gets the sum.
__device__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    s_warp[lane] = wi - w;          // exclusive prefix of the warp totals
    if (lane == 31) s_warp[32] = wi;
  }
  __syncthreads();
  const int r = s_warp[warp] + incl - v;
  *total = s_warp[32];
  __syncthreads();                  // s_warp is reused by the next call
  return r;
}

__global__ void __launch_bounds__(kPlanThreads) append_plan_kernel(KittyCacheState st, int n,
                                                                   const int32_t* __restrict__ seq_ids) {
  __shared__ int s_warp[33];
  __shared__ int s_top;
  if (threadIdx.x == 0) s_top = *st.free_top;
  __syncthreads();
  const int S = st.sink_size, G = st.group;
  const int64_t buf_elems = int64_t(st.num_heads) * G * st.head_dim;
  uint32_t err = 0;
  for (int base = 0; base < n; base += kPlanThreads) {
    const int i = base + threadIdx.x;
    int s = -1, slot = -1, need = 0, np = 0;
    if (i < n) {
      s = seq_ids[i];
      if (s < 0 || s >= st.max_seqs) {
        err |= kErrBadSeq; s = -1;
      } else if (atomicExch(st.claim + s, 1) != 0) {
        err |= kErrBadSeq; s = -1;       // second occurrence in this batch: dropped
      }
      if (s >= 0) {
        const int sl = st.sink_len[s];
        if (sl < S) {
          slot = sl;
          st.sink_len[s] = sl + 1;
        } else {
          const int tl = st.tail_len[s];
          if (tl < G - 1) {
            slot = kTailSlot | tl;
            st.tail_len[s] = tl + 1;
          } else {
            np = st.num_pages[s];
            if (np < st.max_pages_per_seq) need = 1;
            else err |= kErrTableFull;   // token dropped, sequence unchanged
          }
        }
      }
    }
    int total = 0;
    const int rank = block_exclusive_scan(need, s_warp, &total);
    const int top = s_top;
    int page = -1;
    if (need) {
      const int idx = top - 1 - rank;
      if (idx >= 0) {
        page = st.free_pages[idx];
        st.block_table[int64_t(s) * st.max_pages_per_seq + np] = page;
        st.num_pages[s] = np + 1;
        st.tail_len[s] = 0;              // the buffer becomes the new page
        slot = kTailSlot | (G - 1);
      } else {
        err |= kErrNoPage;               // token dropped, sequence unchanged
      }
    }
    if (i < n) {
      st.job_slot[i] = slot;
      st.job_page[i] = page;
      st.job_off[i] = (s >= 0 ? int64_t(s) : 0) * buf_elems;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_top = max(top - total, 0);
    __syncthreads();
  }
  if (threadIdx.x == 0) *st.free_top = s_top;
  if (err) atomicOr(&g_cache_error, err);
}

// One thread per 16-byte vector: (token, head, key|value, vector).
__global__ void append_copy_kernel(KittyCacheState st, int n, const int32_t* __restrict__ seq_ids,
                                   const uint16_t* __restrict__ key, int64_t k_s_tok, int64_t k_s_head,
                                   const uint16_t* __restrict__ value, int64_t v_s_tok, int64_t v_s_head) {
  const int H = st.num_heads, D = st.head_dim, S = st.sink_size, G = st.group;
  const int vecs = D / 8;
  const int64_t per_tok = int64_t(H) * 2 * vecs;
  const int64_t units = int64_t(n) * per_tok;
  for (int64_t u = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += int64_t(gridDim.x) * blockDim.x) {
    const int i = int(u / per_tok);
    int r = int(u - int64_t(i) * per_tok);
    const int which = r / (H * vecs);       // 0 key, 1 value
    r -= which * H * vecs;
    const int h = r / vecs, v = r - h * vecs;
    const int s = seq_ids[i];
    if (which == 0 && h == 0 && v == 0 && s >= 0 && s < st.max_seqs) st.claim[s] = 0;
    const int slot = st.job_slot[i];
    if (slot < 0) continue;
    const uint16_t* src = which == 0 ? key + i * k_s_tok + h * k_s_head : value + i * v_s_tok + h * v_s_head;
    uint16_t* dst;
    if (slot & kTailSlot) {
      const int pos = slot & (kTailSlot - 1);
      uint16_t* base = static_cast<uint16_t*>(which == 0 ? st.tail_k : st.tail_v);
      dst = base + ((int64_t(s) * H + h) * G + pos) * D;
    } else {
      uint16_t* base = static_cast<uint16_t*>(which == 0 ? st.sink_k : st.sink_v);
      dst = base + ((int64_t(s) * H + h) * S + slot) * D;
    }
    reinterpret_cast<uint4*>(dst)[v] = __ldg(reinterpret_cast<const uint4*>(src) + v);
  }
}

// ---- bulk append (prefill) ---------------------------------------------------
//
// Per sequence (one thread): a = tokens to the sinks, pre = tokens completing a
// partly filled buffer (flush = it becomes full), m = full G-token groups quantised
// straight from the source rows, rem = tokens left in the (then empty) buffer.
// Pages: the flushed buffer's first, then the m source pages, all from the free
// stack in sequence order; job slots of the source pages by prefix sum.
constexpr int kPlanInts = 6;   // seq_plan: sink_len, a, tail_len, pre, rem, m

__global__ void __launch_bounds__(kPlanThreads) prefill_plan_kernel(KittyCacheState st, KittyPrefillArgs p) {
  __shared__ int s_warp[33];
  __shared__ int s_top, s_jobs;
  if (threadIdx.x == 0) { s_top = *st.free_top; s_jobs = 0; }
  for (int j = threadIdx.x; j < p.max_pages; j += kPlanThreads) p.page_dst[j] = -1;
  __syncthreads();
  const int S = st.sink_size, G = st.group;
  const int64_t buf_elems = int64_t(st.num_heads) * G * st.head_dim;
  uint32_t err = 0;
  for (int base = 0; base < p.n; base += kPlanThreads) {
    const int i = base + threadIdx.x;
    int s = -1, sl = 0, tl = 0, np = 0, a = 0, pre = 0, flush = 0, m = 0, rem = 0, need = 0;
    if (i < p.n) {
      s = p.seq_ids[i];
      const int T = p.lengths[i];
      if (s < 0 || s >= st.max_seqs || T < 0) {
        err |= kErrBadSeq; s = -1;
      } else if (atomicExch(st.claim + s, 1) != 0) {
        err |= kErrBadSeq; s = -1;
      }
      if (s >= 0) {
        sl = st.sink_len[s]; tl = st.tail_len[s]; np = st.num_pages[s];
        a = min(max(S - sl, 0), T);
        int r = T - a;
        if (r > 0 && tl > 0) { pre = min(G - tl, r); r -= pre; flush = (tl + pre == G) ? 1 : 0; }
        if (r > 0) { m = r / G; rem = r - m * G; }
        need = flush + m;
        if (np + need > st.max_pages_per_seq) { err |= kErrTableFull; s = -1; need = 0; m = 0; }
      }
    }
    int total = 0;
    const int rank_need = block_exclusive_scan(need, s_warp, &total);
    const int rank_m = block_exclusive_scan(m, s_warp, &total);
    const int top = s_top, jobs = s_jobs;
    bool ok = s >= 0;
    if (ok && need > 0 && top - rank_need - need < 0) { ok = false; err |= kErrNoPage; }
    if (ok && m > 0 && int64_t(jobs) + rank_m + m > p.max_pages) { ok = false; err |= kErrBudget; }
    int total_need = 0, total_m = 0;
    const int r2 = block_exclusive_scan(ok ? need : 0, s_warp, &total_need);
    const int rm2 = block_exclusive_scan(ok ? m : 0, s_warp, &total_m);
    if (i < p.n) {
      int* plan = p.seq_plan + int64_t(kPlanInts) * i;
      st.job_page[i] = -1;
      st.job_off[i] = 0;
      if (ok) {
        int32_t* row = st.block_table + int64_t(s) * st.max_pages_per_seq + np;
        int k = 0;
        if (flush) {
          const int page = st.free_pages[top - 1 - r2];
          row[0] = page;
          st.job_page[i] = page;
          st.job_off[i] = int64_t(s) * buf_elems;
          k = 1;
        }
        const int64_t first = p.row_start[i] + a + pre;
        for (int j = 0; j < m; ++j) {
          const int page = st.free_pages[top - 1 - r2 - k - j];
          row[k + j] = page;
          p.page_dst[jobs + rm2 + j] = page;
          p.page_off[jobs + rm2 + j] = (first + int64_t(j) * G) * p.s_tok;
        }
        st.sink_len[s] = sl + a;
        st.num_pages[s] = np + need;
        st.tail_len[s] = flush ? rem : tl + pre + rem;
        plan[0] = sl; plan[1] = a; plan[2] = tl; plan[3] = pre; plan[4] = rem; plan[5] = m;
      } else {
        plan[0] = plan[1] = plan[2] = plan[3] = plan[4] = plan[5] = 0;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) { s_top = top - total_need; s_jobs = jobs + total_m; }
    __syncthreads();
  }
  if (threadIdx.x == 0) *st.free_top = s_top;
  if (err) atomicOr(&g_cache_error, err);
}

// One CTA per sequence.  Phase 0: the sink tokens and the tokens completing the
// buffer; phase 1 (after the buffer was quantised): the remaining tokens into the
// emptied buffer, and the claims cleared.
__global__ void prefill_copy_kernel(KittyCacheState st, KittyPrefillArgs p, int phase) {
  const int i = blockIdx.x;
  const int s = p.seq_ids[i];
  if (s < 0 || s >= st.max_seqs) return;
  const int* plan = p.seq_plan + int64_t(kPlanInts) * i;
  const int sl = plan[0], a = plan[1], tl = plan[2], pre = plan[3], rem = plan[4], m = plan[5];
  const int H = st.num_heads, D = st.head_dim, S = st.sink_size, G = st.group;
  const int vecs = D / 8;
  const int64_t r0 = p.row_start[i];
  const int count = phase == 0 ? a + pre : rem;
  const int64_t per_tok = int64_t(H) * 2 * vecs;
  for (int64_t u = threadIdx.x; u < int64_t(count) * per_tok; u += blockDim.x) {
    const int t = int(u / per_tok);
    int r = int(u - int64_t(t) * per_tok);
    const int which = r / (H * vecs);
    r -= which * H * vecs;
    const int h = r / vecs, v = r - h * vecs;
    int64_t src_row;
    uint16_t* dst;
    if (phase == 0 && t < a) {
      src_row = r0 + t;
      uint16_t* b = static_cast<uint16_t*>(which == 0 ? st.sink_k : st.sink_v);
      dst = b + ((int64_t(s) * H + h) * S + sl + t) * D;
    } else {
      const int pos = phase == 0 ? tl + (t - a) : t;
      src_row = phase == 0 ? r0 + t : r0 + a + pre + int64_t(m) * G + t;
      uint16_t* b = static_cast<uint16_t*>(which == 0 ? st.tail_k : st.tail_v);
      dst = b + ((int64_t(s) * H + h) * G + pos) * D;
    }
    const uint16_t* src = static_cast<const uint16_t*>(which == 0 ? p.key : p.value) + src_row * p.s_tok +
                          h * p.s_head;
    reinterpret_cast<uint4*>(dst)[v] = __ldg(reinterpret_cast<const uint4*>(src) + v);
  }
  if (phase == 1 && threadIdx.x == 0) st.claim[s] = 0;
}

// One CTA: pages of the released sequences pushed in token order (prefix sum of
// the page counts), counters zeroed.  num_pages is taken with atomicExch, so an id
// repeated in the batch pushes its pages once.  A chunk whose pages would overflow
// the stack (only possible when pages were pushed twice by the caller) is refused
// whole and its sequences keep their pages.
__global__ void __launch_bounds__(kPlanThreads) release_kernel(KittyCacheState st, int n,
                                                               const int32_t* __restrict__ seq_ids) {
  __shared__ int s_warp[33];
  __shared__ int s_top;
  if (threadIdx.x == 0) s_top = *st.free_top;
  __syncthreads();
  uint32_t err = 0;
  for (int base = 0; base < n; base += kPlanThreads) {
    const int i = base + threadIdx.x;
    int s = -1, np = 0;
    if (i < n) {
      s = seq_ids[i];
      if (s < 0 || s >= st.max_seqs) { err |= kErrBadSeq; s = -1; }
      else np = max(atomicExch(st.num_pages + s, 0), 0);
    }
    int total = 0;
    const int rank = block_exclusive_scan(np, s_warp, &total);
    const int top = s_top;
    const bool fits = int64_t(top) + total <= st.pool_pages;
    if (s >= 0) {
      if (fits) {
        const int32_t* row = st.block_table + int64_t(s) * st.max_pages_per_seq;
        for (int k = 0; k < np; ++k) st.free_pages[top + rank + k] = row[k];
        st.sink_len[s] = 0;
        st.tail_len[s] = 0;
      } else {
        err |= kErrOverflow;
        if (np > 0) st.num_pages[s] = np;   // keep the pages
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && fits) s_top = top + total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *st.free_top = s_top;
  if (err) atomicOr(&g_cache_error, err);
}

__global__ void reset_kernel(KittyCacheState st) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t t0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t j = t0; j < st.pool_pages; j += stride) st.free_pages[j] = int32_t(st.pool_pages - 1 - j);
  for (int64_t j = t0; j < st.max_seqs; j += stride) {
    st.sink_len[j] = 0; st.tail_len[j] = 0; st.num_pages[j] = 0; st.claim[j] = 0;
  }
  if (t0 == 0) *st.free_top = int32_t(st.pool_pages);
}

int validate_state(const KittyCacheState* st, const char* what) {
  const std::string w(what);
  if (!st) return fail(KITTY_ERR_INVALID_ARGUMENT, w + ": state is NULL");
  if (st->max_seqs <= 0 || st->num_heads <= 0 || st->head_dim <= 0 || st->group <= 0 || st->sink_size < 0 ||
      st->max_pages_per_seq < 0 || st->pool_pages < 0 || st->d_boost < 0 || st->sentinel < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, w + ": negative or zero size");
  if (st->dtype != KITTY_DTYPE_F16 && st->dtype != KITTY_DTYPE_BF16)
    return fail(KITTY_ERR_INVALID_ARGUMENT, w + ": dtype must be KITTY_DTYPE_F16 or KITTY_DTYPE_BF16");
  if (st->pool_pages > 0x7fffffffLL)
    return fail(KITTY_ERR_INVALID_ARGUMENT, w + ": pool_pages must fit int32 page numbers");
  if (st->head_dim % 8 != 0 || st->group % 4 != 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, w + ": head_dim must be a multiple of 8 and group of 4");
  if (!st->sink_len || !st->tail_len || !st->num_pages || !st->claim || !st->free_pages || !st->free_top ||
      !st->tail_k || !st->tail_v || (st->sink_size > 0 && (!st->sink_k || !st->sink_v)) ||
      (st->max_pages_per_seq > 0 && !st->block_table) || !st->job_off || !st->job_page || !st->job_slot ||
      !st->boost_idx || !st->key_low || !st->key_meta || !st->val_codes || !st->val_meta ||
      (st->d_boost > 0 && !st->key_high))
    return fail(KITTY_ERR_INVALID_ARGUMENT, w + ": NULL array in the state");
  const void* vecs[] = {st->tail_k, st->tail_v, st->sink_k, st->sink_v};
  for (const void* p : vecs)
    if (p && !aligned(p, 16)) return fail(KITTY_ERR_INVALID_ARGUMENT, w + ": fp16 buffers must be 16-byte aligned");
  return KITTY_OK;
}

int grid_for(int64_t units, int threads) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  const int64_t want = (units + threads - 1) / threads;
  return int(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(sms) * 8)));
}

}  // namespace

int read_cache_error(uint32_t* flags, int clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_cache_error, sizeof(v));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_cache_error, &zero, sizeof(zero));
  }
  if (e != cudaSuccess) return fail(KITTY_ERR_CUDA, std::string("device_error_flags: ") + cudaGetErrorString(e));
  *flags = v;
  return KITTY_OK;
}

// Key and value quantisation of n_jobs page jobs: source element (t, h, c) of job j
// at base + off[j] + h*s_head + t*s_tok + c, destination page dst[j] (< 0 skips).
int quantize_pages(const KittyCacheState& st, int n_jobs, const void* key, const void* value, const int64_t* off,
                   const int32_t* dst, int64_t s_head, int64_t s_tok, void* stream) {
  if (n_jobs == 0) return KITTY_OK;
  const int H = st.num_heads, D = st.head_dim, G = st.group, K = st.d_boost;
  KittyKeyQuantArgs ka{};
  ka.key = key; ka.key_off = off;
  ka.key_s_head = s_head; ka.key_s_tok = s_tok; ka.key_s_ch = 1;
  ka.boost_idx = st.boost_idx; ka.bidx_s_head = st.bidx_s_head;
  ka.dst_page = dst;
  ka.key_low = st.key_low; ka.key_high = st.key_high;
  ka.key_scale = st.key_meta;
  ka.key_zero = static_cast<uint16_t*>(st.key_meta) + D;
  ka.low_s_page = int64_t(H) * D * (G / 4); ka.low_s_head = int64_t(D) * (G / 4);
  ka.high_s_page = int64_t(H) * K * (G / 4); ka.high_s_head = int64_t(K) * (G / 4);
  ka.meta_s_page = int64_t(H) * 2 * D; ka.meta_s_head = 2 * D;
  ka.n_jobs = n_jobs; ka.num_heads = H; ka.head_dim = D; ka.group = G; ka.d_boost = K; ka.sentinel = st.sentinel;
  ka.dtype = st.dtype;
  int rc = quantize_key_pages_impl(&ka, stream);
  if (rc != KITTY_OK) return rc;
  KittyValueQuantArgs va{};
  va.value = value; va.value_off = off;
  va.val_s_head = s_head; va.val_s_tok = s_tok; va.val_s_ch = 1;
  va.n_valid = nullptr; va.dst_page = dst;
  va.val_codes = st.val_codes;
  va.val_scale = st.val_meta;
  va.val_zero = static_cast<uint16_t*>(st.val_meta) + 1;
  va.codes_s_page = int64_t(H) * G * (D / 4); va.codes_s_head = int64_t(G) * (D / 4);
  va.meta_s_page = int64_t(H) * G * 2; va.meta_s_head = int64_t(G) * 2; va.meta_s_tok = 2;
  va.n_jobs = n_jobs; va.num_heads = H; va.head_dim = D; va.group = G;
  va.dtype = st.dtype;
  return quantize_value_pages_impl(&va, stream);
}

int cache_reset_impl(const KittyCacheState* st, void* stream) {
  int rc = validate_state(st, "cache_reset");
  if (rc != KITTY_OK) return rc;
  const int64_t units = std::max<int64_t>(st->pool_pages, st->max_seqs);
  reset_kernel<<<grid_for(units, 256), 256, 0, as_stream(stream)>>>(*st);
  return check_launch("cache_reset");
}

int cache_append_impl(const KittyCacheState* st, int32_t n, const int32_t* seq_ids, const void* key,
                      int64_t k_s_tok, int64_t k_s_head, const void* value, int64_t v_s_tok, int64_t v_s_head,
                      void* stream) {
  int rc = validate_state(st, "cache_append");
  if (rc != KITTY_OK) return rc;
  if (n < 0 || n > st->max_seqs)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_append: n must be in [0, max_seqs]");
  if (n == 0) return KITTY_OK;
  if (!seq_ids || !key || !value) return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_append: NULL seq_ids/key/value");
  if (!aligned(key, 16) || !aligned(value, 16) || k_s_tok % 8 || k_s_head % 8 || v_s_tok % 8 || v_s_head % 8 ||
      k_s_tok < 0 || k_s_head < 0 || v_s_tok < 0 || v_s_head < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT,
                "cache_append: key/value rows must be 16-byte aligned (strides multiples of 8 elements)");
  cudaStream_t s = as_stream(stream);
  append_plan_kernel<<<1, kPlanThreads, 0, s>>>(*st, n, seq_ids);
  rc = check_launch("cache_append (plan)");
  if (rc != KITTY_OK) return rc;
  const int64_t units = int64_t(n) * st->num_heads * 2 * (st->head_dim / 8);
  append_copy_kernel<<<grid_for(units, 256), 256, 0, s>>>(
      *st, n, seq_ids, static_cast<const uint16_t*>(key), k_s_tok, k_s_head, static_cast<const uint16_t*>(value),
      v_s_tok, v_s_head);
  rc = check_launch("cache_append (copy)");
  if (rc != KITTY_OK) return rc;

  return quantize_pages(*st, n, st->tail_k, st->tail_v, st->job_off, st->job_page,
                        int64_t(st->group) * st->head_dim, st->head_dim, stream);
}

int cache_prefill_impl(const KittyCacheState* st, const KittyPrefillArgs* p, void* stream) {
  int rc = validate_state(st, "cache_prefill");
  if (rc != KITTY_OK) return rc;
  if (!p) return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_prefill: args is NULL");
  if (p->n < 0 || p->n > st->max_seqs)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_prefill: n must be in [0, max_seqs]");
  if (p->max_pages < 0) return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_prefill: negative max_pages");
  if (p->n == 0) return KITTY_OK;
  if (!p->seq_ids || !p->lengths || !p->row_start || !p->key || !p->value || !p->seq_plan ||
      (p->max_pages > 0 && (!p->page_off || !p->page_dst)))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_prefill: NULL pointer");
  if (!aligned(p->key, 16) || !aligned(p->value, 16) || p->s_tok % 8 || p->s_head % 8 || p->s_tok < 0 ||
      p->s_head < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT,
                "cache_prefill: key/value rows must be 16-byte aligned (strides multiples of 8 elements)");
  cudaStream_t s = as_stream(stream);
  prefill_plan_kernel<<<1, kPlanThreads, 0, s>>>(*st, *p);
  rc = check_launch("cache_prefill (plan)");
  if (rc != KITTY_OK) return rc;
  prefill_copy_kernel<<<p->n, 256, 0, s>>>(*st, *p, 0);
  rc = check_launch("cache_prefill (copy)");
  if (rc != KITTY_OK) return rc;
  // buffers that filled, then the full groups straight from the source rows
  rc = quantize_pages(*st, p->n, st->tail_k, st->tail_v, st->job_off, st->job_page,
                      int64_t(st->group) * st->head_dim, st->head_dim, stream);
  if (rc != KITTY_OK) return rc;
  rc = quantize_pages(*st, p->max_pages, p->key, p->value, p->page_off, p->page_dst, p->s_head, p->s_tok, stream);
  if (rc != KITTY_OK) return rc;
  prefill_copy_kernel<<<p->n, 256, 0, s>>>(*st, *p, 1);
  return check_launch("cache_prefill (copy)");
}

int cache_release_impl(const KittyCacheState* st, int32_t n, const int32_t* seq_ids, void* stream) {
  int rc = validate_state(st, "cache_release");
  if (rc != KITTY_OK) return rc;
  if (n < 0) return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_release: negative n");
  if (n == 0) return KITTY_OK;
  if (!seq_ids) return fail(KITTY_ERR_INVALID_ARGUMENT, "cache_release: NULL seq_ids");
  release_kernel<<<1, kPlanThreads, 0, as_stream(stream)>>>(*st, n, seq_ids);
  return check_launch("cache_release");
}

}  // namespace kitty

extern "C" {

int kitty_cache_reset(const KittyCacheState* state, void* stream) {
  kitty::clear_error();
  return kitty::cache_reset_impl(state, stream);
}

int kitty_cache_append(const KittyCacheState* state, int32_t n, const int32_t* seq_ids, const void* key,
                       int64_t k_s_tok, int64_t k_s_head, const void* value, int64_t v_s_tok, int64_t v_s_head,
                       void* stream) {
  kitty::clear_error();
  return kitty::cache_append_impl(state, n, seq_ids, key, k_s_tok, k_s_head, value, v_s_tok, v_s_head, stream);
}

int kitty_cache_prefill(const KittyCacheState* state, const KittyPrefillArgs* args, void* stream) {
  kitty::clear_error();
  return kitty::cache_prefill_impl(state, args, stream);
}

int kitty_cache_release(const KittyCacheState* state, int32_t n, const int32_t* seq_ids, void* stream) {
  kitty::clear_error();
  return kitty::cache_release_impl(state, n, seq_ids, stream);
}

}  // extern "C"
