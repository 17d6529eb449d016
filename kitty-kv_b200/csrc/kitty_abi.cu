// C ABI entry points: argument validation, split planning, dispatch.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "kitty_decode.cuh"

namespace kitty {

int quantize_key_pages_impl(const KittyKeyQuantArgs* a, void* stream);
int quantize_value_pages_impl(const KittyValueQuantArgs* a, void* stream);
int dequantize_key_pages_impl(const KittyKeyDequantArgs* a, void* stream);
int dequantize_value_pages_impl(const KittyValueDequantArgs* a, void* stream);
int read_cache_error(uint32_t* flags, int clear);
int read_tp_error(uint32_t* flags, int clear);

namespace {
thread_local std::string g_last_error;
std::atomic<int> g_forced_variant{-1};   // -1: the library chooses

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return 148; }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return 148;
  }
  return sms;
}

int validate_decode(const KittyDecodeArgs* a) {
  if (!a) return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: args is NULL");
  if (a->batch < 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->head_dim <= 0 || a->group <= 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: non-positive size");
  if (a->num_q_heads % a->num_kv_heads != 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: num_q_heads must be a multiple of num_kv_heads");
  if (a->head_dim % 4 != 0 || a->group % 4 != 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: head_dim and group must be multiples of 4");
  if (a->d_boost < 0 || a->max_pages_per_seq < 0 || a->pool_pages < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: negative d_boost / page counts");
  if (a->batch == 0) return KITTY_OK;
  if (!a->q || !a->out || !a->num_pages || !a->boost_idx)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: NULL q/out/num_pages/boost_idx");
  if (a->max_pages_per_seq > 0 && (!a->block_table || !a->key_low || !a->key_meta || !a->val_codes ||
                                   !a->val_meta || (a->d_boost > 0 && !a->key_high)))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: NULL pool or block table");
  if ((a->sink_len || a->sink_len_all > 0) && (!a->sink_k || !a->sink_v))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: sink length given without sink tensors");
  if ((a->tail_len || a->tail_len_all > 0) && (!a->tail_k || !a->tail_v))
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: tail length given without tail tensors");
  if (a->dtype != KITTY_DTYPE_F16 && a->dtype != KITTY_DTYPE_BF16)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: dtype must be KITTY_DTYPE_F16 or KITTY_DTYPE_BF16");
  if (a->sink_len_all < 0 || a->tail_len_all < 0)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode: negative region length");
  if (!simt_supports(*a) && !i8_supports(*a))
    return fail(KITTY_ERR_UNSUPPORTED,
                "paged_decode: no kernel for this shape (the CUDA-core kernel takes head_dim <= 256 and at most 16 "
                "query heads per KV head; the integer kernel head_dim = group = 128 with 16-byte aligned tensors)");
  return KITTY_OK;
}

// Fill plan.num_splits / pages_per_split / variant / grid (no workspace pointers).
int choose_variant(const KittyDecodeArgs* a) {
  const int forced = g_forced_variant.load();
  if (forced == 3 && tc_supports(*a)) return 3;
  if (forced == 2 && i8_supports(*a)) return 2;
  if (forced == 0 && simt_supports(*a)) return 0;
  if (i8_supports(*a)) return 2;
  return 0;
}

void make_plan(const KittyDecodeArgs* a, DecodePlan* plan) {
  plan->variant = choose_variant(a);
  plan->grid = 0;
  plan->qh_base = 0;
  plan->g_pass = 0;
  plan->ws_m = plan->ws_l = plan->ws_o = nullptr;
  plan->ws_count = nullptr;
  if (plan->variant == 3) {
    tc_plan(*a, device_sm_count(), plan);
    return;
  }
  if (plan->variant == 2) {
    // more than kI8MaxHeadsPerPass query heads per KV head run in passes of that many
    const int g = a->num_q_heads / a->num_kv_heads;
    if (g > kI8MaxHeadsPerPass) plan->g_pass = kI8MaxHeadsPerPass;
    i8_plan(*a, device_sm_count(), plan);
    return;
  }
  const int maxp = std::max(0, a->max_pages_per_seq);
  const int64_t units = int64_t(a->batch) * a->num_kv_heads;
  int splits;
  if (a->num_splits > 0) {
    splits = a->num_splits;
  } else {
    const int64_t target = int64_t(device_sm_count()) * 4 * 2;
    splits = int(std::max<int64_t>(1, (target + units - 1) / std::max<int64_t>(units, 1)));
  }
  splits = std::max(1, std::min({splits, std::max(1, maxp), kMaxDecodeSlots}));
  const int pps = maxp > 0 ? (maxp + splits - 1) / splits : 1;
  plan->pages_per_split = pps;
  plan->num_splits = maxp > 0 ? (maxp + pps - 1) / pps : 1;
  plan->ws_m = plan->ws_l = plan->ws_o = nullptr;
}

size_t workspace_bytes(const KittyDecodeArgs* a, const DecodePlan& plan) {
  if (plan.variant == 0 && plan.num_splits <= 1) return 0;
  const size_t g = size_t(a->num_q_heads / a->num_kv_heads);
  const size_t n = size_t(a->batch) * a->num_kv_heads * plan.num_splits * g;
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t counts = plan.variant >= 1 ? up(size_t(a->batch) * a->num_kv_heads * 4) : 0;
  return up(n * 4) * 2 + up(n * a->head_dim * 4) + counts;
}

}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }
const char* last_error() { return g_last_error.c_str(); }

}  // namespace kitty

using namespace kitty;

extern "C" {

int kitty_abi_version(void) { return KITTY_ABI_VERSION; }

const char* kitty_last_error(void) { return kitty::last_error(); }

size_t kitty_args_size(int kind) {
  switch (kind) {
    case 0: return sizeof(KittyKeyQuantArgs);
    case 1: return sizeof(KittyValueQuantArgs);
    case 2: return sizeof(KittyKeyDequantArgs);
    case 3: return sizeof(KittyDecodeArgs);
    case 4: return sizeof(KittyCacheState);
    case 5: return sizeof(KittyPrefillArgs);
    case 6: return sizeof(KittyValueDequantArgs);
    case 7: return sizeof(KittyTpGatherArgs);
    default: return 0;
  }
}

int kitty_quantize_key_pages(const KittyKeyQuantArgs* args, void* stream) {
  clear_error();
  return quantize_key_pages_impl(args, stream);
}

int kitty_quantize_value_pages(const KittyValueQuantArgs* args, void* stream) {
  clear_error();
  return quantize_value_pages_impl(args, stream);
}

int kitty_dequantize_key_pages(const KittyKeyDequantArgs* args, void* stream) {
  clear_error();
  return dequantize_key_pages_impl(args, stream);
}

int kitty_dequantize_value_pages(const KittyValueDequantArgs* args, void* stream) {
  clear_error();
  return dequantize_value_pages_impl(args, stream);
}

int kitty_device_error_flags(uint32_t* flags, int clear) {
  clear_error();
  if (!flags) return fail(KITTY_ERR_INVALID_ARGUMENT, "device_error_flags: flags is NULL");
  uint32_t b = 0, c = 0, d = 0, t = 0;
  int rc = read_decode_error_i8(&b, clear);
  if (rc != KITTY_OK) return rc;
  rc = read_decode_error_tc(&d, clear);
  if (rc != KITTY_OK) return rc;
  rc = read_cache_error(&c, clear);
  if (rc != KITTY_OK) return rc;
  rc = read_tp_error(&t, clear);
  if (rc != KITTY_OK) return rc;
  *flags = b | c | d | t;
  return KITTY_OK;
}

int kitty_decode_force_variant(int variant, int* previous) {
  clear_error();
  if (variant < -1 || variant > 3 || variant == 1)
    return fail(KITTY_ERR_INVALID_ARGUMENT, "decode_force_variant: variant must be -1, 0, 2 or 3");
  const int old = g_forced_variant.exchange(variant);
  if (previous) *previous = old;
  return KITTY_OK;
}

int kitty_paged_decode_workspace_size(const KittyDecodeArgs* args, size_t* bytes, int32_t* num_splits_out) {
  clear_error();
  int rc = validate_decode(args);
  if (rc != KITTY_OK) return rc;
  if (!bytes) return fail(KITTY_ERR_INVALID_ARGUMENT, "paged_decode_workspace_size: bytes is NULL");
  DecodePlan plan;
  make_plan(args, &plan);
  *bytes = args->batch == 0 ? 0 : workspace_bytes(args, plan);
  if (num_splits_out) *num_splits_out = plan.num_splits;
  return KITTY_OK;
}

int kitty_paged_decode(const KittyDecodeArgs* args, void* stream) {
  clear_error();
  int rc = validate_decode(args);
  if (rc != KITTY_OK) return rc;
  if (args->batch == 0) return KITTY_OK;
  DecodePlan plan;
  make_plan(args, &plan);
  const size_t need = workspace_bytes(args, plan);
  if (need > 0) {
    if (!args->workspace || args->workspace_bytes < need)
      return fail(KITTY_ERR_WORKSPACE, "paged_decode: workspace missing or smaller than "
                                       "kitty_paged_decode_workspace_size()");
    if (!aligned(args->workspace, 16))
      return fail(KITTY_ERR_WORKSPACE, "paged_decode: workspace must be 16-byte aligned");
    const size_t g = size_t(args->num_q_heads / args->num_kv_heads);
    const size_t n = size_t(args->batch) * args->num_kv_heads * plan.num_splits * g;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    uint8_t* w = static_cast<uint8_t*>(args->workspace);
    plan.ws_m = reinterpret_cast<float*>(w);
    plan.ws_l = reinterpret_cast<float*>(w + up(n * 4));
    plan.ws_o = reinterpret_cast<float*>(w + 2 * up(n * 4));
    if (plan.variant >= 1) plan.ws_count = reinterpret_cast<int*>(w + 2 * up(n * 4) + up(n * args->head_dim * 4));
  }
  cudaStream_t s = as_stream(stream);
  if (plan.variant == 2 && plan.g_pass > 0) {
    // the integer kernel in passes over the query heads of each KV head (the workspace,
    // sized for all heads, is reused pass after pass on the same stream)
    const int g = args->num_q_heads / args->num_kv_heads;
    for (int qb = 0; qb < g; qb += kI8MaxHeadsPerPass) {
      DecodePlan pp = plan;
      pp.qh_base = qb;
      pp.g_pass = std::min(kI8MaxHeadsPerPass, g - qb);
      rc = launch_decode_i8(*args, pp, s);
      if (rc != KITTY_OK) return rc;
      rc = launch_decode_merge(*args, pp, s);
      if (rc != KITTY_OK) return rc;
    }
    return KITTY_OK;
  }
  rc = plan.variant == 3   ? launch_decode_tc(*args, plan, s)
       : plan.variant == 2 ? launch_decode_i8(*args, plan, s)
                           : launch_decode_simt(*args, plan, s);
  if (rc != KITTY_OK) return rc;
  if (plan.variant >= 1 || plan.num_splits > 1) rc = launch_decode_merge(*args, plan, s);
  return rc;
}

}  // extern "C"
