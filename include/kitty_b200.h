/*
 * kitty_b200.h - C ABI of the B200 (sm_100a) kernels for Kitty's quantized KV cache.
 *
 * Plain C: pointers, sizes and element strides only.  Every entry point
 *   - returns KITTY_OK (0) or a KITTY_ERR_* code, with a message available
 *     from kitty_last_error() (thread-local);
 *   - launches asynchronously on the given CUDA stream (cudaStream_t passed as
 *     void*, NULL = legacy default stream) and never allocates device memory;
 *   - validates its arguments on the host before launching anything.
 *
 * Data layout (the reference's page pools, kitty/layout.py:128-147 in
 * bitxwolf/kitty-kv).  P = pages, H = KV heads, D = head_dim, G = group (page)
 * size, K = d_boost.  A "page-head" is one (page, head) slice:
 *   key_low   [P][H][D][G/4]  u8   2-bit low plane, byte j of channel c holds
 *                                   tokens 4j..4j+3 at bits 0,2,4,6
 *   key_high  [P][H][K][G/4]  u8   high 2 bits of the boosted channels, row r
 *                                   belongs to the channel with boost_idx == r
 *   key_meta  [P][H][2][D]    f16  row 0 per-channel scale, row 1 zero-point
 *   val_codes [P][H][G][D/4]  u8   2-bit value codes, byte j of token t holds
 *                                   channels 4j..4j+3
 *   val_meta  [P][H][G][2]    f16  per-token (scale, zero-point)
 * fp16 (or bf16, see KITTY_DTYPE_*) tensors are passed as their 16-bit
 * patterns (uint16_t / void*); "f16" above means the call's 16-bit type.
 */
#ifndef KITTY_B200_H_
#define KITTY_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KITTY_OK 0
#define KITTY_ERR_INVALID_ARGUMENT 1 /* shape, stride, alignment or range problem */
#define KITTY_ERR_UNSUPPORTED 2      /* valid but not implemented (e.g. head_dim not 128) */
#define KITTY_ERR_CUDA 3             /* a CUDA runtime call failed */
#define KITTY_ERR_WORKSPACE 4        /* workspace missing or too small */

#define KITTY_ABI_VERSION 5

/* 16-bit floating-point type of the fp16 tensors of a call (the `dtype` field
 * of the argument structs; 0 = the zero-initialised default).  With bf16 the
 * sources, buffers and metadata are bfloat16; quantisation keeps the
 * reference's float32 arithmetic and stores scale and zero-point the way it
 * does for a bfloat16 cache: rounded to fp16, then to bf16 (kitty/kernels/
 * quantize_key.py:121-124 returns fp16 that the launcher copies into the bf16
 * pool views, :261-269).  Decode outputs are fp16 in both cases (the
 * reference's paged attention returns float16, kitty/kernels/attention.py:189). */
#define KITTY_DTYPE_F16 0
#define KITTY_DTYPE_BF16 1
/* quantisers only: bf16 source, fp16 scale / zero-point (what the reference's
 * functional quantize_*_page_torch returns for a bf16 input) */
#define KITTY_DTYPE_BF16_F16META 3
/* dequantisers only: fp16 (4) or bf16 (5) scale / zero-point and a float32
 * output, as the reference's functional dequantize_*_page_torch return */
#define KITTY_DTYPE_F16_F32OUT 4
#define KITTY_DTYPE_BF16_F32OUT 5

/* ABI version compiled into the library (KITTY_ABI_VERSION). */
int kitty_abi_version(void);

/* Message describing the last error returned on the calling thread ("" if none). */
const char* kitty_last_error(void);

/* sizeof() of the argument structs below, so a foreign-function binding can
 * check its mirror of them: kind 0 = KittyKeyQuantArgs, 1 = KittyValueQuantArgs,
 * 2 = KittyKeyDequantArgs, 3 = KittyDecodeArgs, 4 = KittyCacheState,
 * 5 = KittyPrefillArgs, 6 = KittyValueDequantArgs, 7 = KittyTpGatherArgs; 0 for an
 * unknown kind. */
size_t kitty_args_size(int kind);

/* ---------------------------------------------------------------------------
 * Key page quantisation (per channel over a G-token group; INT4 for channels
 * with boost_idx < sentinel, INT2 otherwise; dense low plane + sparse high plane).
 *
 * Replaces quantize_key_page / quantize_key_page_torch
 * (kitty/kernels/quantize_key.py:217-269 and :38-124) and the per-head loop of
 * KittyInferencePipeline._trigger_quantization (kitty/pipeline.py:199-230).
 * Bit-exact with the reference: scale = max(max-min, 1e-8f)/(2^b-1) in IEEE
 * fp32, zp = clamp(rint(-min/scale), 0, 2^b-1), code = clamp(rint(x/scale)+zp),
 * scale stored as fp16 (RN).  High-plane row boost_idx[c] receives channel c's
 * high bits when boost_idx[c] < d_boost (rows nobody writes are zeroed; rows
 * shared by several channels receive the OR of their bits).
 *
 * Job j, head h: the source element (token t, channel c) is at
 *   key + key_off[j] + h*key_s_head + t*key_s_tok + c*key_s_ch   (fp16 elements)
 * and the outputs go to page-head (dst_page[j], h) of the pools, whose page /
 * head strides are given in elements (the slice itself is contiguous).  Jobs
 * with dst_page[j] < 0 are skipped (same for the value quantiser).
 * ------------------------------------------------------------------------- */
typedef struct KittyKeyQuantArgs {
  const void* key;            /* fp16 source */
  const int64_t* key_off;     /* [n_jobs] element offsets (device memory) */
  int64_t key_s_head, key_s_tok, key_s_ch;
  const uint8_t* boost_idx;   /* [H][D], unit channel stride (device memory) */
  int64_t bidx_s_head;
  const int32_t* dst_page;    /* [n_jobs] destination pages (device memory) */
  uint8_t* key_low;           /* pool bases (device memory) */
  uint8_t* key_high;
  void* key_scale;            /* fp16; usually key_meta */
  void* key_zero;             /* fp16; usually key_meta + D */
  int64_t low_s_page, low_s_head;
  int64_t high_s_page, high_s_head;
  int64_t meta_s_page, meta_s_head;
  int32_t n_jobs, num_heads, head_dim, group, d_boost, sentinel;
  int32_t dtype;              /* KITTY_DTYPE_*: key source and key_scale / key_zero (BF16_F16META allowed) */
} KittyKeyQuantArgs;

int kitty_quantize_key_pages(const KittyKeyQuantArgs* args, void* stream);

/* ---------------------------------------------------------------------------
 * Value page quantisation (per token INT2 over D channels).
 *
 * Replaces quantize_value_page / quantize_value_page_torch
 * (kitty/kernels/quantize_value.py:197-227 and :38-90) and the per-head loop of
 * _trigger_quantization (kitty/pipeline.py:232-250), including the zero padding
 * of a partial Value Q-buffer: tokens t >= n_valid[j] are quantised as +0.0.
 * Scale and zero-point of token t go to val_scale/val_zero + t*meta_s_tok
 * (meta_s_tok = 2 for the interleaved val_meta pool).
 * ------------------------------------------------------------------------- */
typedef struct KittyValueQuantArgs {
  const void* value;          /* fp16 source */
  const int64_t* value_off;   /* [n_jobs] element offsets (device memory) */
  int64_t val_s_head, val_s_tok, val_s_ch;
  const int32_t* n_valid;     /* [n_jobs] or NULL (= group) (device memory) */
  const int32_t* dst_page;    /* [n_jobs] (device memory) */
  uint8_t* val_codes;
  void* val_scale;            /* fp16; usually val_meta */
  void* val_zero;             /* fp16; usually val_meta + 1 */
  int64_t codes_s_page, codes_s_head;
  int64_t meta_s_page, meta_s_head, meta_s_tok;
  int32_t n_jobs, num_heads, head_dim, group;
  int32_t dtype;              /* KITTY_DTYPE_*: value source and val_scale / val_zero (BF16_F16META allowed) */
} KittyValueQuantArgs;

int kitty_quantize_value_pages(const KittyValueQuantArgs* args, void* stream);

/* ---------------------------------------------------------------------------
 * Key page dequantisation to fp16 (D, G) blocks: x = (code - zp) * scale in fp32,
 * code = low | (high << 2) for channels with boost_idx < d_boost.
 * Replaces dequantize_key_page (kitty/kernels/dequantize_key.py:169-228) and,
 * with dtype KITTY_DTYPE_F16_F32OUT / BF16_F32OUT (float32 out),
 * dequantize_key_page_torch (kitty/kernels/dequantize_key.py:35-97).
 * Job j's output element (c, t) is at out + out_off[j] + c*out_s_ch + t*out_s_tok.
 * Source page-head: (src_page[j], head[j]).
 * ------------------------------------------------------------------------- */
typedef struct KittyKeyDequantArgs {
  const uint8_t* key_low;
  const uint8_t* key_high;
  const void* key_scale;
  const void* key_zero;
  int64_t low_s_page, low_s_head, high_s_page, high_s_head, meta_s_page, meta_s_head;
  const int32_t* src_page;    /* [n_jobs] */
  const int32_t* head;        /* [n_jobs] */
  const uint8_t* boost_idx;   /* [H][D] */
  int64_t bidx_s_head;
  void* out;                  /* fp16 */
  const int64_t* out_off;     /* [n_jobs] */
  int64_t out_s_ch, out_s_tok;
  int32_t n_jobs, num_heads, head_dim, group, d_boost;
  int32_t dtype;              /* KITTY_DTYPE_*: key_scale / key_zero and out (F32OUT: float32 out) */
} KittyKeyDequantArgs;

int kitty_dequantize_key_pages(const KittyKeyDequantArgs* args, void* stream);

/* ---------------------------------------------------------------------------
 * Value page dequantisation: x = (code - zp_t) * scale_t in fp32 for every
 * token t and channel c of a (G, D/4) packed page-head.
 * Replaces dequantize_value_page_torch (kitty/kernels/quantize_value.py:97-133):
 * dtype KITTY_DTYPE_F16_F32OUT / BF16_F32OUT give its float32 (G, D) block;
 * KITTY_DTYPE_F16 / BF16 round the result to the metadata's 16-bit type.
 * Job j reads page-head (src_page[j], head[j]); the scale and zero-point of
 * token t are at val_scale / val_zero + src_page*meta_s_page + head*meta_s_head
 * + t*meta_s_tok (meta_s_tok = 2 for the interleaved value_metadata pool).
 * Output element (t, c) is at out + out_off[j] + t*out_s_tok + c*out_s_ch.
 * ------------------------------------------------------------------------- */
typedef struct KittyValueDequantArgs {
  const uint8_t* val_codes;
  const void* val_scale;      /* usually value_metadata */
  const void* val_zero;       /* usually value_metadata + 1 element */
  int64_t codes_s_page, codes_s_head;
  int64_t meta_s_page, meta_s_head, meta_s_tok;
  const int32_t* src_page;    /* [n_jobs] (device memory) */
  const int32_t* head;        /* [n_jobs] (device memory) */
  void* out;
  const int64_t* out_off;     /* [n_jobs] (device memory) */
  int64_t out_s_tok, out_s_ch;
  int32_t n_jobs, head_dim, group;
  int32_t dtype;              /* KITTY_DTYPE_F16 / BF16 / F16_F32OUT / BF16_F32OUT */
} KittyValueDequantArgs;

int kitty_dequantize_value_pages(const KittyValueDequantArgs* args, void* stream);

/* ---------------------------------------------------------------------------
 * Fused paged GQA decode attention over the quantised pools plus the fp16
 * regions.  For sequence b and query head qh (KV head h = qh / (Hq/H)) the keys
 * are [sink_k (sink_len) ; pages block_table[b][0..num_pages[b]) ; tail_k
 * (tail_len)] and the values are [sink_v ; value pages ; tail_v] in the same
 * order; out = softmax(q.k * sm_scale) . v in fp32, stored as fp16.
 *
 * Replaces paged_attention / paged_attention_reference
 * (kitty/kernels/attention.py:292-341 and :46-189, batch 1 there) with a
 * batched form.  Key and value tails have one common length (the reference's
 * qbuf_k / qbuf_v must be equally long, attention.py:163-165).
 *
 * Pools use the layout above with P = pool_pages (contiguous).  Work is split
 * over pages ("split-K"); partial (max, sum, acc) go to the workspace and a
 * second kernel merges them, both launched on `stream` by this call.
 * num_splits = 0 lets the library choose.  The workspace must hold
 * kitty_paged_decode_workspace_size() bytes for the same (batch, heads,
 * num_splits) and be 16-byte aligned.  Concurrent calls must not share it.
 * ------------------------------------------------------------------------- */
typedef struct KittyDecodeArgs {
  int32_t batch, num_q_heads, num_kv_heads, head_dim, group, d_boost;
  float sm_scale;                     /* usually 1/sqrt(head_dim) */
  const void* q;                      /* fp16 [B][Hq][D] (unit channel stride) */
  int64_t q_s_seq, q_s_head;
  void* out;                          /* fp16 [B][Hq][D] */
  int64_t out_s_seq, out_s_head;
  const int32_t* block_table;         /* [B][*] physical pages */
  int64_t bt_s_seq;
  const int32_t* num_pages;           /* [B] */
  int64_t pool_pages;                 /* P (pages must be < P) */
  const uint8_t* key_low;
  const uint8_t* key_high;
  const void* key_meta;
  const uint8_t* val_codes;
  const void* val_meta;
  const uint8_t* boost_idx;           /* [H][D] */
  int64_t bidx_s_head;
  const void* sink_k;                 /* fp16, element (b,h,t,c) at b*s_seq+h*s_head+t*s_tok+c */
  int64_t sk_s_seq, sk_s_head, sk_s_tok;
  const void* sink_v;
  int64_t sv_s_seq, sv_s_head, sv_s_tok;
  const int32_t* sink_len;            /* [B] or NULL -> sink_len_all */
  int32_t sink_len_all;
  const void* tail_k;
  int64_t tk_s_seq, tk_s_head, tk_s_tok;
  const void* tail_v;
  int64_t tv_s_seq, tv_s_head, tv_s_tok;
  const int32_t* tail_len;            /* [B] or NULL -> tail_len_all */
  int32_t tail_len_all;
  int32_t max_pages_per_seq;          /* upper bound of num_pages[b] (host-known) */
  int32_t num_splits;                 /* 0 = choose */
  void* workspace;
  size_t workspace_bytes;
  /* Row b of q / out reads the cache row seq_map[b] of num_pages, sink_len,
   * tail_len, block_table and the sink / tail tensors (for a decode over a
   * subset of a KittyCacheState's sequences, in any order).  NULL = b.  Values
   * must be valid rows of those arrays. */
  const int32_t* seq_map;
  int32_t dtype;                      /* KITTY_DTYPE_*: q, key_meta, val_meta, sinks, tail (out is fp16) */
} KittyDecodeArgs;

/* Bytes of workspace kitty_paged_decode needs; writes the split count it will
 * use for these arguments to *num_splits_out (may be NULL). */
int kitty_paged_decode_workspace_size(const KittyDecodeArgs* args, size_t* bytes, int32_t* num_splits_out);

int kitty_paged_decode(const KittyDecodeArgs* args, void* stream);

/* Paged decode for callers that cannot allocate device memory (an engine whose
 * memory arena forbids allocation on the decode path, or a thin FFI host with
 * no device allocator).  No counterpart in the reference: it runs the same
 * kernels as kitty_paged_decode but ignores args->workspace and keeps the
 * split partial results in a static 8 MiB device array inside the library
 * (held on every GPU that loads the library until exit).  The first call on a
 * device looks the array up (make it before any stream capture) and caches
 * the address for the life of the process, so do not call it after
 * cudaDeviceReset; all calls share the array, so calls that overlap on the
 * GPU race.  With num_splits == 0 the split count is lowered to the largest
 * that fits; an explicit num_splits that does not fit returns
 * KITTY_ERR_WORKSPACE.  Allocates nothing. */
int kitty_paged_decode_noalloc(const KittyDecodeArgs* args, void* stream);

/* ---------------------------------------------------------------------------
 * Device-resident cache state: per-sequence fp16 buffers, counters, block
 * tables and a free-page stack, all in device memory, so that a decode step of
 * many sequences appends its tokens (and flushes the buffers that fill into
 * new pages) without a host round trip.
 *
 * Replaces, for one layer and a batch of sequences at once,
 * KittyInferencePipeline.push_token / _trigger_quantization / reset_sequence
 * (kitty/pipeline.py:115-181, 183-258, 286-313) and the page allocator of
 * PageCentricKVLayoutManager (allocate_page / free_sequence,
 * kitty/layout.py:161-220).  Same state machine per sequence: the first S
 * tokens go to the fp16 sinks, later tokens to a G-token fp16 buffer; when
 * that buffer fills, its keys and values are quantised into a newly allocated
 * page (the values of the same G tokens, like the pipeline's aligned-values
 * mode; the reference's separate value window is not kept here).
 *
 * Arrays (all device memory, contiguous):
 *   sink_k, sink_v   fp16 [max_seqs][H][S][D]
 *   tail_k, tail_v   fp16 [max_seqs][H][G][D]
 *   sink_len, tail_len, num_pages, claim   int32 [max_seqs]
 *   block_table      int32 [max_seqs][max_pages_per_seq]
 *   free_pages       int32 [pool_pages]  (stack: entries [0, *free_top))
 *   free_top         int32 [1]
 *   job_off int64, job_page int32, job_slot int32   [max_seqs] scratch
 *   pools            the page layout at the top of this file, P = pool_pages
 * Several states (one per layer) may share the pools, free_pages and free_top;
 * their launches must then be ordered (one stream).  The state can be passed
 * straight to kitty_paged_decode: block_table / num_pages / sink_len /
 * tail_len / sink_* / tail_* with row strides of the layouts above, and
 * seq_map = the step's sequence ids.
 * ------------------------------------------------------------------------- */
typedef struct KittyCacheState {
  int32_t max_seqs, num_heads, head_dim, group, sink_size, d_boost, sentinel;
  int32_t max_pages_per_seq;
  int64_t pool_pages;
  const uint8_t* boost_idx;           /* [H][D] */
  int64_t bidx_s_head;
  void* sink_k;
  void* sink_v;
  void* tail_k;
  void* tail_v;
  int32_t* sink_len;
  int32_t* tail_len;
  int32_t* num_pages;
  int32_t* claim;                     /* zero between calls */
  int32_t* block_table;
  int32_t* free_pages;
  int32_t* free_top;
  uint8_t* key_low;
  uint8_t* key_high;
  void* key_meta;
  uint8_t* val_codes;
  void* val_meta;
  int64_t* job_off;
  int32_t* job_page;
  int32_t* job_slot;
  int32_t dtype;                      /* KITTY_DTYPE_*: buffers, appended rows and metadata */
} KittyCacheState;

/* Empty every sequence and put all pool pages on the free stack (pages are
 * handed out in increasing order until some are released).  Use it once on a
 * new state; states sharing a stack need it once. */
int kitty_cache_reset(const KittyCacheState* state, void* stream);

/* Append one token to each of n distinct sequences: seq_ids[i] (device memory)
 * receives key / value row i, fp16, element (i, h, c) at
 * key + i*k_s_tok + h*k_s_head + c (16-byte aligned rows: pointer and strides
 * multiples of 8 elements).  A sequence whose G-token buffer fills is flushed
 * in the same call: a page is popped from the free stack, appended to its
 * block table, and the buffer quantised into it (bit-exact with
 * kitty_quantize_key_pages / kitty_quantize_value_pages on the same tokens).
 * Four launches on `stream` (plan, copy, key and value quantisation), no host
 * synchronisation, n <= max_seqs.  Failures found on the device drop that
 * token, leave its sequence unchanged and set a sticky error bit
 * (kitty_device_error_flags): bit 1 no free page, bit 2 block table full,
 * bit 3 sequence id out of range or repeated in the batch. */
int kitty_cache_append(const KittyCacheState* state, int32_t n, const int32_t* seq_ids,
                       const void* key, int64_t k_s_tok, int64_t k_s_head,
                       const void* value, int64_t v_s_tok, int64_t v_s_head, void* stream);

/* Bulk append of many tokens per sequence (a prefill, or a chunk of one).
 *
 * Replaces KittyPagedAttention._prefill's per-token push loop
 * (kitty/attention.py:153-191, kitty/pipeline.py:115-181).  Sequence
 * seq_ids[i] receives lengths[i] tokens: source rows row_start[i] ..
 * row_start[i] + lengths[i] - 1, row r / head h at key + r*s_tok + h*s_head
 * (value likewise, same strides; 16-byte aligned rows).  The result equals
 * appending those tokens one by one with kitty_cache_append: sinks first, then
 * the G-token buffer; a buffer that fills is quantised into a new page, and
 * every further full group of G tokens is quantised straight from the source
 * rows into its own page (bit-exact with the page quantisers).  Seven launches,
 * no host synchronisation.
 *
 * max_pages bounds the pages quantised straight from the source in this call
 * (sum over i of lengths[i] / G is always enough); page_off / page_dst are
 * scratch of max_pages entries and seq_plan of 6 n entries (device memory).
 * Sequences are served in order; a sequence whose pages do not fit (free stack,
 * its block table, or max_pages) is left unchanged and sets error bit 1, 2 or
 * 5 — once one has failed for want of pages, the later ones that need pages
 * fail too.  Ids out of range or repeated set bit 3. */
typedef struct KittyPrefillArgs {
  int32_t n;
  const int32_t* seq_ids;     /* [n] */
  const int32_t* lengths;     /* [n] tokens per sequence (>= 0) */
  const int64_t* row_start;   /* [n] first source row of each sequence */
  const void* key;            /* fp16 */
  const void* value;          /* fp16 */
  int64_t s_tok, s_head;      /* element strides of a row / a head in key and value */
  int32_t max_pages;
  int64_t* page_off;          /* [max_pages] scratch */
  int32_t* page_dst;          /* [max_pages] scratch */
  int32_t* seq_plan;          /* [6 n] scratch */
} KittyPrefillArgs;

int kitty_cache_prefill(const KittyCacheState* state, const KittyPrefillArgs* args, void* stream);

/* Empty the n sequences seq_ids[i] (device memory) and push their pages back on
 * the free stack (in block-table order, sequence after sequence).  Releasing an
 * empty sequence is a no-op; ids out of range set error bit 3; a stack that
 * would overflow pool_pages sets bit 4 and keeps the pages of that sequence. */
int kitty_cache_release(const KittyCacheState* state, int32_t n, const int32_t* seq_ids, void* stream);

/* Sticky error bits set by device code on the current device (bit 0: a decode
 * kernel gave up waiting for a bulk copy after its bounded wait and returned
 * without a valid result; bits 1-5: kitty_cache_append / _prefill / _release,
 * above; bit 6: kitty_tp_allgather gave up waiting for another rank).
 * Synchronises with the device; clear != 0 resets the bits after reading them. */
int kitty_device_error_flags(uint32_t* flags, int clear);

/* ---------------------------------------------------------------------------
 * Tensor-parallel output exchange over peer memory (no counterpart in the
 * reference, which is single-GPU).  When the decode is sharded by KV head, rank r
 * holds the head-major outputs of its query heads, (Hq_local, B, D) fp16, and
 * every rank needs all of them, (Hq, B, D).  Instead of a library all-gather,
 * each rank's exchange region (one cudaMalloc, mapped into the other ranks'
 * processes by CUDA IPC) receives the slices by direct NVLink stores:
 *
 *   region = [buffer 0: data_bytes][buffer 1: data_bytes][arrival counters:
 *             KITTY_TP_MAX_RANKS x u32][epoch u32][done u32]   (see
 *             kitty_tp_region_bytes)
 *
 * kitty_tp_allgather launches two kernels on `stream`: the first stores this
 * rank's slice (src_bytes at src) at byte offset dst_offset of buffer (e & 1)
 * of every rank (e = the call's epoch, counted on the device, so CUDA-graph
 * replays stay in step) and then adds to that rank's arrival counter for this
 * rank (system-scope fence first); the second waits until every rank's counter
 * has reached this epoch (bounded wait: after about a second it sets error bit 6
 * and returns), copies buffer (e & 1) into dst (data_bytes, the assembled
 * output) and advances the epoch.  Two buffers alternate so a rank that runs
 * ahead never overwrites the data another rank may still be reading.  Every rank
 * must make the same sequence of calls with the same sizes; src_bytes,
 * dst_offset and data_bytes are multiples of 16 and src / dst 16-byte aligned.
 * Plain peer stores and atomics only: no multicast objects. */
#define KITTY_TP_MAX_RANKS 8
typedef struct {
  int32_t world;                       /* ranks taking part, 1..KITTY_TP_MAX_RANKS */
  int32_t rank;                        /* this rank */
  void* region[KITTY_TP_MAX_RANKS];    /* every rank's region as mapped in this process (own included) */
  uint64_t data_bytes;                 /* bytes of one assembled output (one buffer) */
  const void* src;                     /* this rank's slice (device memory) */
  uint64_t src_bytes;
  uint64_t dst_offset;                 /* where the slice goes in the assembled output */
  void* dst;                           /* the assembled output of this call (data_bytes) */
} KittyTpGatherArgs;

/* Bytes of an exchange region for data_bytes of assembled output. */
size_t kitty_tp_region_bytes(uint64_t data_bytes);
/* cudaMalloc a zeroed exchange region of kitty_tp_region_bytes(data_bytes) on the
 * current device. */
int kitty_tp_region_alloc(uint64_t data_bytes, void** region);
int kitty_tp_region_free(void* region);
/* CUDA IPC handle (64 bytes into handle) of a region of this process, and the
 * mapping of another process's region into this one (and its release). */
int kitty_tp_ipc_handle(void* region, void* handle);
int kitty_tp_ipc_open(const void* handle, void** region);
int kitty_tp_ipc_close(void* region);
int kitty_tp_allgather(const KittyTpGatherArgs* args, void* stream);

/* Test and benchmark hook, no counterpart in the reference: pin the decode
 * kernel family used by later kitty_paged_decode / _workspace_size / _noalloc
 * calls of this process (-1 = library choice, 0 = CUDA-core, 2 = integer
 * mma.sync tensor-core, 3 = integer tcgen05 with tensor-memory accumulators,
 * which takes calls without fp16 sink / tail tokens only; 1 is not a family).
 * A pinned family that does not support a call's shape falls back to the
 * library choice.  The previous setting is stored in *previous when it is not
 * NULL. */
int kitty_decode_force_variant(int variant, int* previous);

#ifdef __cplusplus
}
#endif

#endif /* KITTY_B200_H_ */
