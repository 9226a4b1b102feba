// C ABI of libtfattn (include/tfattn.h): argument validation, device selection and dispatch.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <string>

#include "launch.h"
#include "tfattn.h"

namespace tf {
namespace {

thread_local std::string g_last_error;

tf_status fail(tf_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

tf_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TF_OK;
  if (e == cudaErrorNotSupported)
    return fail(TF_ERR_UNSUPPORTED, "%s: dimension combination not compiled", what);
  return fail(TF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Runs the launch on the stream's device, restoring the caller's current device afterwards.
class DeviceGuard {
 public:
  // A stream being captured into a CUDA graph belongs to the capturing thread's current device,
  // and cudaStreamGetDevice on it invalidates the capture: query it only when not capturing.
  explicit DeviceGuard(cudaStream_t s) {
    ok_ = cudaGetDevice(&prev_) == cudaSuccess;
    int dev = prev_;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (ok_ && s != nullptr && cudaStreamIsCapturing(s, &cap) == cudaSuccess &&
        cap == cudaStreamCaptureStatusNone && cudaStreamGetDevice(s, &dev) == cudaSuccess &&
        dev != prev_) {
      ok_ = cudaSetDevice(dev) == cudaSuccess;
      switched_ = ok_;
    }
  }
  ~DeviceGuard() {
    if (switched_) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = 0;
  bool ok_ = false, switched_ = false;
};

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];

bool dtype_ok(int d) { return d == TF_DTYPE_F32 || d == TF_DTYPE_BF16 || d == TF_DTYPE_F16; }

}  // namespace

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  g_sm_count[dev].store(n, std::memory_order_relaxed);
  return n;
}

static tf_status check_paged(const tf_paged_attn_args* a, bool decode) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->batch_size < 0 || a->num_tokens < 0)
    return fail(TF_ERR_INVALID_ARG, "negative batch_size (%d) or num_tokens (%d)", a->batch_size,
                a->num_tokens);
  if (a->batch_size == 0 || a->num_tokens == 0) return TF_OK;
  if (!a->q || !a->k_buffer || !a->v_buffer || !a->req_to_token || !a->req_pool_indices ||
      !a->seq_lens || !a->out)
    return fail(TF_ERR_INVALID_ARG, "a required tensor pointer is NULL");
  if (a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->num_q_heads % a->num_kv_heads != 0)
    return fail(TF_ERR_INVALID_ARG, "num_q_heads %d is not a multiple of num_kv_heads %d",
                a->num_q_heads, a->num_kv_heads);
  if (a->num_q_heads / a->num_kv_heads > 64)
    return fail(TF_ERR_UNSUPPORTED, "more than 64 query heads per kv head");
  if (a->head_dim <= 0 || a->head_dim > 256)
    return fail(TF_ERR_UNSUPPORTED, "head_dim %d outside [1, 256]", a->head_dim);
  if (!dtype_ok(a->dtype)) return fail(TF_ERR_INVALID_ARG, "unknown dtype %d", a->dtype);
  if (a->gate_mode < TF_GATE_NONE || a->gate_mode > TF_GATE_SIGMOID)
    return fail(TF_ERR_INVALID_ARG, "unknown gate_mode %d", a->gate_mode);
  if (a->gate_mode != TF_GATE_NONE && a->gate == nullptr)
    return fail(TF_ERR_INVALID_ARG, "gate_mode %d needs a gate tensor", a->gate_mode);
  if (a->slot_mode != TF_SLOT_CLAMP && a->slot_mode != TF_SLOT_WRAP)
    return fail(TF_ERR_INVALID_ARG, "unknown slot_mode %d", a->slot_mode);
  if (a->num_slots <= 0 || a->r2t_rows <= 0 || a->r2t_cols <= 0)
    return fail(TF_ERR_INVALID_ARG, "empty pool or req_to_token table");
  if (a->max_seq_len > a->r2t_cols)
    return fail(TF_ERR_INVALID_ARG, "max_seq_len %d exceeds req_to_token columns %lld",
                a->max_seq_len, (long long)a->r2t_cols);
  if (decode && a->num_tokens != a->batch_size)
    return fail(TF_ERR_INVALID_ARG, "decode batch needs num_tokens == batch_size (%d vs %d)",
                a->num_tokens, a->batch_size);
  if (!decode && a->extend_lens == nullptr && a->num_tokens != a->batch_size)
    return fail(TF_ERR_INVALID_ARG, "extend batch needs extend_lens");
  return TF_OK;
}

static tf_status check_gdn(const tf_gdn_args* a, bool decode) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->batch_size < 0 || a->num_tokens < 0) return fail(TF_ERR_INVALID_ARG, "negative sizes");
  if (a->batch_size == 0 || a->num_tokens == 0) return TF_OK;
  if (!a->qkv || !a->b || !a->a || !a->conv_weight || !a->A_log || !a->dt_bias || !a->conv_state ||
      !a->ssm_state || !a->req_pool_indices || !a->out)
    return fail(TF_ERR_INVALID_ARG, "a required tensor pointer is NULL");
  if (!dtype_ok(a->dtype)) return fail(TF_ERR_INVALID_ARG, "unknown dtype %d", a->dtype);
  if (a->num_k_heads <= 0 || a->num_v_heads <= 0 || a->num_v_heads % a->num_k_heads != 0)
    return fail(TF_ERR_INVALID_ARG, "num_v_heads %d is not a multiple of num_k_heads %d",
                a->num_v_heads, a->num_k_heads);
  if (!gdn_dims_supported(a->head_k_dim, a->head_v_dim))
    return fail(TF_ERR_UNSUPPORTED, "head dims dk=%d dv=%d not compiled (16/32/64/128, dk == dv)",
                a->head_k_dim, a->head_v_dim);
  if (a->conv_kernel < 2 || a->conv_kernel > 9)
    return fail(TF_ERR_UNSUPPORTED, "conv_kernel %d outside [2, 9]", a->conv_kernel);
  const int64_t conv_dim = 2LL * a->num_k_heads * a->head_k_dim + (int64_t)a->num_v_heads * a->head_v_dim;
  if (a->conv_stride_slot < conv_dim * (a->conv_kernel - 1))
    return fail(TF_ERR_INVALID_ARG, "conv_stride_slot %lld smaller than conv_dim*(K-1)",
                (long long)a->conv_stride_slot);
  if (a->ssm_stride_slot < (int64_t)a->num_v_heads * a->head_k_dim * a->head_v_dim)
    return fail(TF_ERR_INVALID_ARG, "ssm_stride_slot %lld smaller than Hv*dk*dv",
                (long long)a->ssm_stride_slot);
  if ((reinterpret_cast<uintptr_t>(a->ssm_state) & 15) != 0 || (a->ssm_stride_slot & 3) != 0)
    return fail(TF_ERR_ALIGNMENT, "ssm_state must be 16-byte aligned with a stride multiple of 4");
  if (a->qkv_stride_tok < conv_dim)
    return fail(TF_ERR_INVALID_ARG, "qkv_stride_tok smaller than conv_dim");
  if (a->z != nullptr &&
      (a->norm_weight == nullptr ||
       (a->norm_weight_len != a->head_v_dim && a->norm_weight_len != a->num_v_heads * a->head_v_dim)))
    return fail(TF_ERR_INVALID_ARG, "fused norm needs norm_weight of length dv or Hv*dv");
  if (a->num_slots <= 0) return fail(TF_ERR_INVALID_ARG, "empty state pool");
  if (decode && a->num_tokens != a->batch_size)
    return fail(TF_ERR_INVALID_ARG, "decode batch needs num_tokens == batch_size");
  if (!decode && a->extend_lens == nullptr)
    return fail(TF_ERR_INVALID_ARG, "extend batch needs extend_lens");
  return TF_OK;
}

}  // namespace tf

using namespace tf;

// One pool of tf_state_copy_args: each (layer, slot) block of `elems` elements must be disjoint
// from every other, which holds for the layer-major and the slot-major layouts.
static const char* state_pool_problem(const void* base, int64_t stride_layer, int64_t stride_slot,
                                      int64_t elems, int32_t dtype, int32_t layers, int64_t slots) {
  if (!base) return nullptr;
  if (!dtype_ok(dtype)) return "unknown dtype";
  if (elems <= 0 || stride_layer <= 0 || stride_slot <= 0) return "non-positive extent or stride";
  if (stride_slot < elems || stride_layer < elems) return "a stride is smaller than a slot's rows";
  const bool layer_major = stride_layer >= slots * stride_slot;
  const bool slot_major = stride_slot >= (int64_t)layers * stride_layer;
  if (layers > 1 && slots > 1 && !layer_major && !slot_major) return "slot rows overlap";
  return nullptr;
}

extern "C" {

int tf_abi_version(void) { return TFATTN_ABI_VERSION; }

const char* tf_status_string(tf_status s) {
  switch (s) {
    case TF_OK: return "ok";
    case TF_ERR_INVALID_ARG: return "invalid argument";
    case TF_ERR_UNSUPPORTED: return "unsupported configuration";
    case TF_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case TF_ERR_WORKSPACE: return "workspace missing or too small";
    case TF_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* tf_last_error(void) { return g_last_error.c_str(); }

tf_status tf_kv_store(const tf_kv_store_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->num_tokens < 0 || a->num_kv_heads < 0 || a->head_dim < 0)
    return fail(TF_ERR_INVALID_ARG, "negative sizes");
  if (a->num_tokens == 0) return TF_OK;
  if (!a->k_buffer || !a->v_buffer || !a->k || !a->v || !a->out_cache_loc)
    return fail(TF_ERR_INVALID_ARG, "a required tensor pointer is NULL");
  if (!dtype_ok(a->dtype)) return fail(TF_ERR_INVALID_ARG, "unknown dtype %d", a->dtype);
  if (a->num_slots <= 0) return fail(TF_ERR_INVALID_ARG, "empty pool");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_kv_store(*a, s), "tf_kv_store");
}

tf_status tf_attn_prologue(const tf_attn_prologue_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->num_tokens < 0 || a->num_q_heads < 0 || a->num_kv_heads < 0 || a->head_dim < 0)
    return fail(TF_ERR_INVALID_ARG, "negative sizes");
  if (a->num_tokens == 0) return TF_OK;
  if (a->num_tokens > 0x7fffffff) return fail(TF_ERR_INVALID_ARG, "too many tokens for one launch");
  if (!a->q || !a->k || !a->v || !a->q_out || !a->k_buffer || !a->v_buffer || !a->out_cache_loc ||
      !a->q_norm_weight || !a->k_norm_weight || !a->positions || !a->inv_freq)
    return fail(TF_ERR_INVALID_ARG, "a required tensor pointer is NULL");
  if (!dtype_ok(a->dtype)) return fail(TF_ERR_INVALID_ARG, "unknown dtype %d", a->dtype);
  if (a->norm_weight_dtype != a->dtype && a->norm_weight_dtype != TF_DTYPE_F32)
    return fail(TF_ERR_INVALID_ARG, "norm weights must be float32 or of the activation dtype");
  if (a->num_q_heads <= 0 || a->num_kv_heads <= 0) return fail(TF_ERR_INVALID_ARG, "no heads");
  if (a->num_slots <= 0) return fail(TF_ERR_INVALID_ARG, "empty pool");
  if (a->pos_rows != 1 && a->pos_rows != 3)
    return fail(TF_ERR_INVALID_ARG, "positions must have 1 or 3 rows, got %d", a->pos_rows);
  if (a->pos_rows == 3) {
    const int32_t* m = a->mrope_section;
    if (m[0] < 0 || m[1] < 0 || m[2] < 0 || m[0] + m[1] + m[2] != a->rotary_dim / 2)
      return fail(TF_ERR_INVALID_ARG, "mrope_section must sum to rotary_dim / 2");
  }
  if (!attn_prologue_supported(*a))
    return fail(TF_ERR_UNSUPPORTED,
                "prologue: head_dim %d with rotary_dim %d is not built (head_dim 64/128/256; "
                "rotary_dim/2 a multiple of 32 or a power of two below 32)",
                a->head_dim, a->rotary_dim);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_attn_prologue(*a, s), "tf_attn_prologue");
}

size_t tf_paged_decode_workspace_size(const tf_paged_attn_args* a) {
  if (a == nullptr || a->batch_size <= 0) return 0;
  if (!paged_decode_mma_supported(*a)) return 0;
  return paged_decode_mma_workspace(*a, device_sm_count());
}

tf_status tf_paged_decode_attn(const tf_paged_attn_args* a, void* ws, size_t ws_bytes,
                               void* stream) {
  tf_status st = check_paged(a, true);
  if (st != TF_OK || a->batch_size == 0) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  if (paged_decode_mma_supported(*a)) {
    const int nsm = device_sm_count();
    const size_t need = paged_decode_mma_workspace(*a, nsm);
    if (ws == nullptr || ws_bytes < need)
      return fail(TF_ERR_WORKSPACE, "decode workspace of %zu bytes needed, %zu given", need,
                  ws_bytes);
    if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
      return fail(TF_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
    return cuda_status(launch_paged_decode_mma(*a, ws, ws_bytes, nsm, s), "tf_paged_decode_attn");
  }
  tf_paged_attn_args d = *a;
  d.extend_lens = nullptr;
  return cuda_status(launch_paged_attn_simt(d, s), "tf_paged_decode_attn");
}

tf_status tf_paged_decode_attn_noalloc(const tf_paged_attn_args* a, void* stream) {
  tf_status st = check_paged(a, true);
  if (st != TF_OK || a->batch_size == 0) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // one stated bound for every dtype and head_dim, checked before anything is launched
  if (a->batch_size > kDecodeMmaMaxBatch)
    return fail(TF_ERR_WORKSPACE,
                "tf_paged_decode_attn_noalloc: the built-in scratch serves batches of up to %d "
                "requests, this one has %d; use tf_paged_decode_attn with a caller workspace",
                kDecodeMmaMaxBatch, a->batch_size);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  if (!paged_decode_mma_supported(*a)) {  // the CUDA-core path needs no scratch at all
    tf_paged_attn_args d = *a;
    d.extend_lens = nullptr;
    return cuda_status(launch_paged_attn_simt(d, s), "tf_paged_decode_attn_noalloc");
  }
  const int nsm = device_sm_count();
  const size_t need = paged_decode_mma_workspace(*a, nsm);
  if (need > kNoAllocScratchBytes)
    return fail(TF_ERR_WORKSPACE,
                "tf_paged_decode_attn_noalloc: the built-in scratch holds %zu bytes; this batch "
                "(batch_size %d, head_dim %d, %d SMs) needs %zu; use tf_paged_decode_attn with a "
                "caller workspace",
                kNoAllocScratchBytes, a->batch_size, a->head_dim, nsm, need);
  const cudaError_t e = launch_paged_decode_mma_noalloc(*a, nsm, s);
  if (e == cudaErrorStreamCaptureUnsupported)
    return fail(TF_ERR_CUDA,
                "tf_paged_decode_attn_noalloc: the first call on a device must be made outside "
                "stream capture (it resolves the device address of the built-in scratch)");
  return cuda_status(e, "tf_paged_decode_attn_noalloc");
}

size_t tf_paged_extend_workspace_size(const tf_paged_attn_args* a) {
  (void)a;
  return 0;
}

tf_status tf_paged_extend_attn(const tf_paged_attn_args* a, void* ws, size_t ws_bytes,
                               void* stream) {
  (void)ws;
  (void)ws_bytes;
  tf_status st = check_paged(a, false);
  if (st != TF_OK || a->batch_size == 0 || a->num_tokens == 0) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  if (paged_extend_tc_supported(*a))
    return cuda_status(launch_paged_extend_tc(*a, s), "tf_paged_extend_attn");
  return cuda_status(launch_paged_attn_simt(*a, s), "tf_paged_extend_attn");
}

tf_status tf_gdn_decode(const tf_gdn_args* a, void* stream) {
  tf_status st = check_gdn(a, true);
  if (st != TF_OK || a->batch_size == 0) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_gdn_decode(*a, s), "tf_gdn_decode");
}

size_t tf_gdn_extend_workspace_size(const tf_gdn_args* a) {
  if (a == nullptr || a->batch_size <= 0 || a->num_tokens <= 0) return 0;
  return gdn_extend_workspace(*a);
}

tf_status tf_gdn_extend(const tf_gdn_args* a, void* ws, size_t ws_bytes, void* stream) {
  tf_status st = check_gdn(a, false);
  if (st != TF_OK || a->batch_size == 0 || a->num_tokens == 0) return st;
  const size_t need = gdn_extend_workspace(*a);
  if (ws == nullptr || ws_bytes < need)
    return fail(TF_ERR_WORKSPACE, "extend workspace of %zu bytes needed, %zu given", need, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(TF_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_gdn_extend(*a, ws, ws_bytes, s), "tf_gdn_extend");
}

tf_status tf_gated_rmsnorm(const tf_gated_rmsnorm_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->num_tokens < 0 || a->num_heads < 0 || a->head_dim < 0)
    return fail(TF_ERR_INVALID_ARG, "negative sizes");
  if (a->num_tokens == 0 || a->num_heads == 0) return TF_OK;
  if (!a->x || !a->z || !a->weight || !a->out)
    return fail(TF_ERR_INVALID_ARG, "a required tensor pointer is NULL");
  if (a->weight_len != a->head_dim && a->weight_len != a->num_heads * a->head_dim)
    return fail(TF_ERR_INVALID_ARG, "weight length %d is neither head_dim nor heads*head_dim",
                a->weight_len);
  if (!dtype_ok(a->dtype)) return fail(TF_ERR_INVALID_ARG, "unknown dtype %d", a->dtype);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_gated_rmsnorm(*a, s), "tf_gated_rmsnorm");
}

tf_status tf_state_slots_copy(const tf_state_copy_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->num_ops < 0 || a->num_layers < 0 || a->num_slots < 0)
    return fail(TF_ERR_INVALID_ARG, "negative sizes");
  if (a->num_ops == 0 || a->num_layers == 0 || (!a->conv_state && !a->ssm_state)) return TF_OK;
  if (!a->src_slots || !a->dst_slots) return fail(TF_ERR_INVALID_ARG, "slot lists are NULL");
  if (a->num_slots == 0) return fail(TF_ERR_INVALID_ARG, "empty pool");
  if (const char* e = state_pool_problem(a->conv_state, a->conv_stride_layer, a->conv_stride_slot,
                                         a->conv_slot_elems, a->conv_dtype, a->num_layers,
                                         a->num_slots))
    return fail(TF_ERR_INVALID_ARG, "conv_state: %s", e);
  if (const char* e = state_pool_problem(a->ssm_state, a->ssm_stride_layer, a->ssm_stride_slot,
                                         a->ssm_slot_elems, a->ssm_dtype, a->num_layers,
                                         a->num_slots))
    return fail(TF_ERR_INVALID_ARG, "ssm_state: %s", e);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_state_slots_copy(*a, s), "tf_state_slots_copy");
}

tf_status tf_req_to_token_sync(const tf_r2t_sync_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->num_segments < 0 || a->num_values < 0) return fail(TF_ERR_INVALID_ARG, "negative sizes");
  if (a->num_segments == 0) return TF_OK;
  if (!a->req_to_token || !a->segments || (a->num_values > 0 && !a->values))
    return fail(TF_ERR_INVALID_ARG, "a required tensor pointer is NULL");
  if (a->r2t_rows <= 0 || a->r2t_cols <= 0 || a->r2t_stride < a->r2t_cols)
    return fail(TF_ERR_INVALID_ARG, "bad req_to_token shape or stride");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_req_to_token_sync(*a, s), "tf_req_to_token_sync");
}

tf_status tf_sample_tokens(const tf_sample_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->batch_size < 0) return fail(TF_ERR_INVALID_ARG, "negative batch size");
  if (a->batch_size == 0) return TF_OK;
  if (a->vocab_size <= 0 || a->logits_stride < a->vocab_size)
    return fail(TF_ERR_INVALID_ARG, "bad vocab size or row stride");
  if (!a->logits || !a->temperature || !a->out)
    return fail(TF_ERR_INVALID_ARG, "a required tensor pointer is NULL");
  if (!dtype_ok(a->dtype)) return fail(TF_ERR_INVALID_ARG, "unknown dtype %d", a->dtype);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_sample_tokens(*a, s), "tf_sample_tokens");
}

tf_status tf_fp8_quantize(const tf_fp8_quant_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->M < 0 || a->K < 0) return fail(TF_ERR_INVALID_ARG, "negative sizes");
  if (a->M == 0 || a->K == 0) return TF_OK;
  if (!a->x || !a->q || !a->x_scale || !a->workspace)
    return fail(TF_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!dtype_ok(a->dtype)) return fail(TF_ERR_INVALID_ARG, "unknown dtype %d", a->dtype);
  if (a->K % 16 != 0 || a->x_stride < a->K)
    return fail(TF_ERR_UNSUPPORTED, "K must be a multiple of 16 and x_stride >= K");
  const int eb = a->dtype == TF_DTYPE_F32 ? 4 : 2;
  if (((reinterpret_cast<uintptr_t>(a->x) | (uintptr_t)(a->x_stride * eb)) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 3) != 0 || (reinterpret_cast<uintptr_t>(a->q) & 15) != 0)
    return fail(TF_ERR_ALIGNMENT, "x rows and q must be 16-byte aligned, workspace 4-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_fp8_quantize(*a, s), "tf_fp8_quantize");
}

tf_status tf_fp8_block_gemm(const tf_fp8_gemm_args* a, void* stream) {
  if (a == nullptr) return fail(TF_ERR_INVALID_ARG, "args is NULL");
  if (a->M < 0 || a->N < 0 || a->K <= 0) return fail(TF_ERR_INVALID_ARG, "bad sizes");
  if (a->M == 0 || a->N == 0) return TF_OK;
  if (a->M > (int64_t)65535 * 128) return fail(TF_ERR_INVALID_ARG, "M too large for one launch");
  if (!a->q || !a->w || !a->x_scale || !a->out)
    return fail(TF_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!dtype_ok(a->out_dtype) || (a->bias && !dtype_ok(a->bias_dtype)))
    return fail(TF_ERR_INVALID_ARG, "unknown dtype");
  if (a->K % 16 != 0) return fail(TF_ERR_UNSUPPORTED, "K must be a multiple of 16, got %d", a->K);
  if (a->w_scale && (a->block_h <= 0 || a->block_w <= 0 || a->block_h % 128 || a->block_w % 128))
    return fail(TF_ERR_UNSUPPORTED, "block_h and block_w must be multiples of 128 (got %d, %d)",
                a->block_h, a->block_w);
  if (a->q_stride < a->K || a->w_stride < a->K || a->out_stride < a->N)
    return fail(TF_ERR_INVALID_ARG, "a row stride is shorter than its row");
  if (((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->w) |
        (uintptr_t)a->q_stride | (uintptr_t)a->w_stride) & 15) != 0)
    return fail(TF_ERR_ALIGNMENT, "q, w and their row strides must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceGuard g(s);
  if (!g.ok()) return fail(TF_ERR_CUDA, "cannot select the stream's device");
  return cuda_status(launch_fp8_block_gemm(*a, s), "tf_fp8_block_gemm");
}

}  // extern "C"
