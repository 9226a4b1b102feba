// tokenfactory_b200._C: the PyTorch front end of libtfattn's C ABI (include/tfattn.h).
//
// Each function takes torch tensors in the reference's layouts, checks dtypes, shapes and strides,
// fills the POD argument structure of one tf_* entry point with data pointers and element strides,
// and launches on the current PyTorch stream of the tensors' device.  Argument problems raise
// ValueError / TypeError, a non-zero tf_status raises tokenfactory_b200._capi.TFAttnError with the
// library's message: the error behaviour of the Python front end (ops.py) it serves.  Nothing here
// computes; there is no CPU path.  Scratch for the entry points that take a workspace is a
// per-(device, stream) byte tensor grown on demand and reused in stream order.
#include <torch/extension.h>
#include <pybind11/stl.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "tfattn.h"

namespace py = pybind11;

namespace {

py::object& err_class() {
  static py::object cls;  // tokenfactory_b200._capi.TFAttnError, set at import
  return cls;
}

[[noreturn]] void raise_status(const char* fn, tf_status st) {
  std::string msg = tf_last_error();
  if (msg.empty()) msg = tf_status_string(st);
  py::object e = err_class()(fn, (int)st, msg);
  PyErr_SetObject(err_class().ptr(), e.ptr());
  throw py::error_already_set();
}

inline void check(const char* fn, tf_status st) {
  if (st != TF_OK) raise_status(fn, st);
}

[[noreturn]] void value_error(const std::string& m) { throw py::value_error(m); }
[[noreturn]] void type_error(const std::string& m) { throw py::type_error(m); }

using OptT = c10::optional<at::Tensor>;

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return TF_DTYPE_F32;
    case at::kBFloat16: return TF_DTYPE_BF16;
    case at::kHalf: return TF_DTYPE_F16;
    default: type_error(std::string("unsupported dtype ") + c10::toString(t.scalar_type()));
  }
}

std::string shape(const at::Tensor& t) {
  std::string s = "(";
  for (int64_t i = 0; i < t.dim(); ++i) s += (i ? ", " : "") + std::to_string(t.size(i));
  return s + (t.dim() == 1 ? ",)" : ")");
}

// Every given tensor is a CUDA tensor on one device; returns that device.
c10::Device need_cuda(std::initializer_list<const at::Tensor*> ts) {
  c10::optional<c10::Device> dev;
  for (const at::Tensor* t : ts) {
    if (t == nullptr || !t->defined()) continue;
    if (!t->is_cuda()) value_error("tokenfactory_b200 kernels need CUDA tensors (no CPU fallback)");
    if (!dev) {
      dev = t->device();
    } else if (t->device() != *dev) {
      value_error("tensors on different devices: " + dev->str() + " and " + t->device().str());
    }
  }
  if (!dev) value_error("tokenfactory_b200 kernels need CUDA tensors (no CPU fallback)");
  return *dev;
}

const at::Tensor* opt(const OptT& t) { return t.has_value() ? &*t : nullptr; }
void* optp(const OptT& t) { return t.has_value() ? t->data_ptr() : nullptr; }
int32_t* errp(const OptT& e) { return e.has_value() ? (int32_t*)e->data_ptr() : nullptr; }

at::Tensor i64(const at::Tensor& t, const char* name) {
  if (t.scalar_type() != at::kLong)
    type_error(std::string(name) + " must be int64 (got " + c10::toString(t.scalar_type()) + ")");
  return t.is_contiguous() ? t : t.contiguous();
}

void* stream_of(const c10::Device& d) {
  return (void*)at::cuda::getCurrentCUDAStream(d.index()).stream();
}

// A 256-byte aligned scratch tensor of at least `nbytes` for the current stream of `d`.
void* workspace(const c10::Device& d, size_t nbytes) {
  static std::mutex mu;
  static std::map<std::pair<int, void*>, at::Tensor> bufs;
  void* s = stream_of(d);
  std::lock_guard<std::mutex> lock(mu);
  at::Tensor& b = bufs[{d.index(), s}];
  if (!b.defined() || (size_t)b.numel() < nbytes) {
    b = at::empty({(int64_t)std::max<size_t>(nbytes, 1 << 20)},
                  at::TensorOptions().dtype(at::kByte).device(d));
  }
  return b.data_ptr();
}

// ---------------------------------------------------------------------------------------------
// a1 KV store, f1 prologue
// ---------------------------------------------------------------------------------------------
void kv_store(const at::Tensor& k_buffer, const at::Tensor& v_buffer, const at::Tensor& loc_in,
              const at::Tensor& k, const at::Tensor& v, const OptT& err) {
  const c10::Device dev = need_cuda({&k_buffer, &v_buffer, &loc_in, &k, &v, opt(err)});
  if (k.dim() != 3 || !k.sizes().equals(v.sizes()) || !k_buffer.sizes().equals(v_buffer.sizes()))
    value_error("kv_store shapes: k " + shape(k) + " v " + shape(v) + " pool " + shape(k_buffer) +
                " / " + shape(v_buffer));
  if (!k_buffer.strides().equals(v_buffer.strides()) || k_buffer.stride(2) != 1 ||
      k.stride(2) != 1 || v.stride(2) != 1)
    value_error("kv_store needs unit stride on head_dim and equal pool strides");
  if (k_buffer.dim() != 3 || k.size(1) != k_buffer.size(1) || k.size(2) != k_buffer.size(2) ||
      k.scalar_type() != k_buffer.scalar_type() || v.scalar_type() != k.scalar_type())
    value_error("kv_store: k/v rows must match the pool's [Hkv, D] and dtype");
  const at::Tensor loc = i64(loc_in, "out_cache_loc");
  if (loc.numel() != k.size(0)) value_error("out_cache_loc must have one entry per token");
  tf_kv_store_args a{};
  a.k_buffer = k_buffer.data_ptr();
  a.v_buffer = v_buffer.data_ptr();
  a.buf_stride_slot = k_buffer.stride(0);
  a.buf_stride_head = k_buffer.stride(1);
  a.num_slots = k_buffer.size(0);
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.k_stride_tok = k.stride(0);
  a.k_stride_head = k.stride(1);
  a.v_stride_tok = v.stride(0);
  a.v_stride_head = v.stride(1);
  a.out_cache_loc = loc.data_ptr<int64_t>();
  a.num_tokens = k.size(0);
  a.num_kv_heads = (int32_t)k.size(1);
  a.head_dim = (int32_t)k.size(2);
  a.dtype = dtype_code(k);
  a.err = errp(err);
  c10::cuda::CUDAGuard g(dev);
  check("tf_kv_store", tf_kv_store(&a, stream_of(dev)));
}

at::Tensor attn_prologue(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                         const at::Tensor& q_norm_weight, const at::Tensor& k_norm_weight,
                         const at::Tensor& positions, const at::Tensor& inv_freq,
                         const at::Tensor& k_buffer, const at::Tensor& v_buffer,
                         const at::Tensor& out_cache_loc, double eps,
                         std::vector<int64_t> mrope_section, bool mrope_interleaved, OptT q_out,
                         const OptT& err) {
  const c10::Device dev = need_cuda({&q, &k, &v, &q_norm_weight, &k_norm_weight, &positions,
                                     &inv_freq, &k_buffer, &v_buffer, &out_cache_loc,
                                     opt(q_out), opt(err)});
  if (q.dim() != 3 || k.dim() != 3 || !k.sizes().equals(v.sizes()) ||
      !k_buffer.sizes().equals(v_buffer.sizes()) || k_buffer.dim() != 3)
    value_error("attn_prologue shapes: q " + shape(q) + " k " + shape(k) + " v " + shape(v) +
                " pool " + shape(k_buffer));
  const int64_t t = q.size(0), hq = q.size(1), d = q.size(2);
  if (k.size(0) != t || k.size(2) != d || k.size(1) != k_buffer.size(1) ||
      k.size(2) != k_buffer.size(2))
    value_error("attn_prologue: k/v rows must be [T, Hkv, D] matching the pool");
  if (q.stride(2) != 1 || k.stride(2) != 1 || v.stride(2) != 1 || k_buffer.stride(2) != 1 ||
      !k_buffer.strides().equals(v_buffer.strides()))
    value_error("attn_prologue needs unit stride on head_dim and equal pool strides");
  const auto dt = q.scalar_type();
  if (k.scalar_type() != dt || v.scalar_type() != dt || k_buffer.scalar_type() != dt ||
      v_buffer.scalar_type() != dt)
    type_error("attn_prologue: q, k, v and the pools share a dtype");
  if (q_norm_weight.scalar_type() != k_norm_weight.scalar_type() ||
      (q_norm_weight.scalar_type() != dt && q_norm_weight.scalar_type() != at::kFloat))
    type_error("attn_prologue: norm weights are float32 or of the activation dtype");
  if (q_norm_weight.numel() != d || k_norm_weight.numel() != d)
    value_error("norm weights must have head_dim entries");
  if (inv_freq.scalar_type() != at::kFloat || inv_freq.dim() != 1 || !inv_freq.is_contiguous())
    type_error("inv_freq must be a contiguous float32 vector");
  at::Tensor pos = i64(positions, "positions");
  int32_t rows = 1;
  int64_t pstride = 0;
  if (pos.dim() == 1) {
    if (pos.size(0) != t) value_error("positions must have one entry per token");
  } else if (pos.dim() == 2 && pos.size(0) == 3 && pos.size(1) == t) {
    rows = 3;
    pstride = pos.stride(0);
  } else {
    value_error("positions must be [T] or [3, T], got " + shape(pos));
  }
  const at::Tensor loc = i64(out_cache_loc, "out_cache_loc");
  if (loc.numel() != t) value_error("out_cache_loc must have one entry per token");
  if (mrope_section.size() != 3) value_error("mrope_section must have three entries");
  at::Tensor qo = q_out.has_value() ? *q_out : at::empty({t, hq, d}, q.options());
  const at::Tensor qw = q_norm_weight.contiguous(), kw = k_norm_weight.contiguous();
  tf_attn_prologue_args a{};
  a.q = q.data_ptr();
  a.q_stride_tok = q.stride(0);
  a.q_stride_head = q.stride(1);
  a.k = k.data_ptr();
  a.k_stride_tok = k.stride(0);
  a.k_stride_head = k.stride(1);
  a.v = v.data_ptr();
  a.v_stride_tok = v.stride(0);
  a.v_stride_head = v.stride(1);
  a.q_norm_weight = qw.data_ptr();
  a.k_norm_weight = kw.data_ptr();
  a.positions = pos.data_ptr<int64_t>();
  a.pos_stride = pstride;
  a.inv_freq = inv_freq.data_ptr<float>();
  a.q_out = qo.data_ptr();
  a.q_out_stride_tok = qo.stride(0);
  a.q_out_stride_head = qo.stride(1);
  a.k_buffer = k_buffer.data_ptr();
  a.v_buffer = v_buffer.data_ptr();
  a.buf_stride_slot = k_buffer.stride(0);
  a.buf_stride_head = k_buffer.stride(1);
  a.num_slots = k_buffer.size(0);
  a.out_cache_loc = loc.data_ptr<int64_t>();
  a.num_tokens = t;
  a.eps = (float)eps;
  a.pos_rows = rows;
  for (int i = 0; i < 3; ++i) a.mrope_section[i] = (int32_t)mrope_section[i];
  a.mrope_interleaved = mrope_interleaved ? 1 : 0;
  a.rotary_dim = (int32_t)(2 * inv_freq.numel());
  a.num_q_heads = (int32_t)hq;
  a.num_kv_heads = (int32_t)k.size(1);
  a.head_dim = (int32_t)d;
  a.dtype = dtype_code(q);
  a.norm_weight_dtype = dtype_code(qw);
  a.err = errp(err);
  c10::cuda::CUDAGuard g(dev);
  check("tf_attn_prologue", tf_attn_prologue(&a, stream_of(dev)));
  return qo;
}

// ---------------------------------------------------------------------------------------------
// a2-a4 paged attention
// ---------------------------------------------------------------------------------------------
struct PagedKeep {
  at::Tensor rpi, sl, el;
};

tf_paged_attn_args paged_args(const at::Tensor& q, const at::Tensor& k_buffer,
                              const at::Tensor& v_buffer, const at::Tensor& r2t,
                              const at::Tensor& req_pool_indices, const at::Tensor& seq_lens,
                              const OptT& extend_lens, double scale, const OptT& gate,
                              int64_t gate_mode, const at::Tensor& out, int64_t max_seq_len,
                              int64_t max_extend_len, int64_t slot_mode, const OptT& err,
                              PagedKeep& keep) {
  if (q.dim() != 3 || k_buffer.dim() != 3 || !k_buffer.sizes().equals(v_buffer.sizes()))
    value_error("paged attention shapes: q " + shape(q) + ", pool " + shape(k_buffer));
  const int64_t t = q.size(0), hq = q.size(1), d = q.size(2);
  if (k_buffer.size(2) != d || hq % k_buffer.size(1) != 0)
    value_error("q heads must be a multiple of kv heads and head dims must agree");
  if (out.dim() != 3 || q.stride(2) != 1 || k_buffer.stride(2) != 1 || out.stride(2) != 1 ||
      !k_buffer.strides().equals(v_buffer.strides()))
    value_error("paged attention needs unit stride on head_dim");
  if (q.scalar_type() != k_buffer.scalar_type() || v_buffer.scalar_type() != q.scalar_type() ||
      out.scalar_type() != q.scalar_type())
    type_error("q, pools and out must share a dtype");
  if (gate.has_value()) {
    if (!gate->sizes().equals(q.sizes()) || gate->stride(2) != 1 ||
        gate->scalar_type() != q.scalar_type())
      value_error("gate must be a [T, Hq, D] view with unit stride on D");
  }
  if (r2t.scalar_type() != at::kLong || r2t.dim() != 2 || r2t.stride(1) != 1)
    value_error("req_to_token must be a row-major int64 [rows, cols] table");
  keep.rpi = i64(req_pool_indices, "req_pool_indices");
  keep.sl = i64(seq_lens, "seq_lens");
  if (extend_lens.has_value()) keep.el = i64(*extend_lens, "extend_lens");
  tf_paged_attn_args a{};
  a.q = q.data_ptr();
  a.q_stride_tok = q.stride(0);
  a.q_stride_head = q.stride(1);
  a.k_buffer = k_buffer.data_ptr();
  a.v_buffer = v_buffer.data_ptr();
  a.kv_stride_slot = k_buffer.stride(0);
  a.kv_stride_head = k_buffer.stride(1);
  a.num_slots = k_buffer.size(0);
  a.req_to_token = r2t.data_ptr<int64_t>();
  a.r2t_stride = r2t.stride(0);
  a.r2t_rows = r2t.size(0);
  a.r2t_cols = r2t.size(1);
  a.req_pool_indices = keep.rpi.data_ptr<int64_t>();
  a.seq_lens = keep.sl.data_ptr<int64_t>();
  a.extend_lens = keep.el.defined() ? keep.el.data_ptr<int64_t>() : nullptr;
  a.gate = optp(gate);
  a.gate_stride_tok = gate.has_value() ? gate->stride(0) : 0;
  a.gate_stride_head = gate.has_value() ? gate->stride(1) : 0;
  a.out = out.data_ptr();
  a.out_stride_tok = out.stride(0);
  a.out_stride_head = out.stride(1);
  a.batch_size = (int32_t)keep.rpi.numel();
  a.num_tokens = (int32_t)t;
  a.num_q_heads = (int32_t)hq;
  a.num_kv_heads = (int32_t)k_buffer.size(1);
  a.head_dim = (int32_t)d;
  a.max_seq_len = (int32_t)max_seq_len;
  a.max_extend_len = (int32_t)max_extend_len;
  a.scale = (float)scale;
  a.dtype = dtype_code(q);
  a.gate_mode = (int32_t)gate_mode;
  a.slot_mode = (int32_t)slot_mode;
  a.err = errp(err);
  return a;
}

at::Tensor paged_decode(const at::Tensor& q, const at::Tensor& k_buffer, const at::Tensor& v_buffer,
                        const at::Tensor& req_to_token, const at::Tensor& req_pool_indices,
                        const at::Tensor& seq_lens, double scale, int64_t max_seq_len,
                        const OptT& gate, int64_t gate_mode, OptT out, int64_t slot_mode,
                        const OptT& err) {
  const c10::Device dev = need_cuda({&q, &k_buffer, &v_buffer, &req_to_token, &req_pool_indices,
                                     &seq_lens, opt(gate), opt(out), opt(err)});
  at::Tensor o = out.has_value() ? *out : at::empty_like(q);
  PagedKeep keep;
  tf_paged_attn_args a = paged_args(q, k_buffer, v_buffer, req_to_token, req_pool_indices,
                                    seq_lens, c10::nullopt, scale, gate, gate_mode, o, max_seq_len,
                                    1, slot_mode, err, keep);
  c10::cuda::CUDAGuard g(dev);
  const size_t nbytes = tf_paged_decode_workspace_size(&a);
  void* ws = nbytes ? workspace(dev, nbytes) : nullptr;
  check("tf_paged_decode_attn", tf_paged_decode_attn(&a, ws, nbytes, stream_of(dev)));
  return o;
}

at::Tensor paged_extend(const at::Tensor& q, const at::Tensor& k_buffer, const at::Tensor& v_buffer,
                        const at::Tensor& req_to_token, const at::Tensor& req_pool_indices,
                        const at::Tensor& seq_lens, const at::Tensor& extend_lens, double scale,
                        int64_t max_seq_len, int64_t max_extend_len, const OptT& gate,
                        int64_t gate_mode, OptT out, int64_t slot_mode, const OptT& err) {
  const c10::Device dev = need_cuda({&q, &k_buffer, &v_buffer, &req_to_token, &req_pool_indices,
                                     &seq_lens, &extend_lens, opt(gate), opt(out), opt(err)});
  at::Tensor o = out.has_value() ? *out : at::empty_like(q);
  PagedKeep keep;
  tf_paged_attn_args a = paged_args(q, k_buffer, v_buffer, req_to_token, req_pool_indices,
                                    seq_lens, extend_lens, scale, gate, gate_mode, o, max_seq_len,
                                    max_extend_len, slot_mode, err, keep);
  c10::cuda::CUDAGuard g(dev);
  const size_t nbytes = tf_paged_extend_workspace_size(&a);
  void* ws = nbytes ? workspace(dev, nbytes) : nullptr;
  check("tf_paged_extend_attn", tf_paged_extend_attn(&a, ws, nbytes, stream_of(dev)));
  return o;
}

// ---------------------------------------------------------------------------------------------
// a5-a9 Gated DeltaNet
// ---------------------------------------------------------------------------------------------
struct GdnKeep {
  at::Tensor cw, rpi, el, A_log, dt_bias, nw, bias;
};

tf_gdn_args gdn_args(const at::Tensor& qkv, const at::Tensor& b, const at::Tensor& a_in,
                     const at::Tensor& conv_weight, const OptT& conv_bias, const at::Tensor& A_log,
                     const at::Tensor& dt_bias, const at::Tensor& conv_state,
                     const at::Tensor& ssm_state, const at::Tensor& req_pool_indices,
                     const OptT& extend_lens, const OptT& z, const OptT& norm_weight,
                     double norm_eps, const at::Tensor& out, int64_t num_k_heads,
                     int64_t head_k_dim, int64_t head_v_dim, int64_t max_extend_len,
                     const OptT& err, GdnKeep& keep) {
  if (qkv.dim() != 2 || b.dim() != 2) value_error("qkv and b must be [T, ...] matrices");
  const int64_t t = qkv.size(0), conv_dim = qkv.size(1), hv = b.size(1);
  const int64_t kc = conv_weight.size(-1);
  if (conv_dim != 2 * num_k_heads * head_k_dim + hv * head_v_dim)
    value_error("qkv width " + std::to_string(conv_dim) + " != 2*Hk*dk + Hv*dv");
  if (conv_state.dim() != 3 || conv_state.size(1) != conv_dim || conv_state.size(2) != kc - 1 ||
      conv_state.stride(2) != 1 || conv_state.stride(1) != kc - 1)
    value_error("conv_state must be a [slots, " + std::to_string(conv_dim) + ", " +
                std::to_string(kc - 1) + "] view, channel-major");
  if (ssm_state.dim() != 4 || ssm_state.size(1) != hv || ssm_state.size(2) != head_k_dim ||
      ssm_state.size(3) != head_v_dim || ssm_state.scalar_type() != at::kFloat ||
      ssm_state.stride(1) != head_k_dim * head_v_dim || ssm_state.stride(2) != head_v_dim ||
      ssm_state.stride(3) != 1)
    value_error("ssm_state must be a float32 [slots, Hv, dk, dv] view, contiguous per slot");
  if (conv_state.size(0) != ssm_state.size(0))
    value_error("conv_state and ssm_state must have the same slots");
  if (qkv.stride(-1) != 1) value_error("qkv needs unit stride on its last dim");
  if (b.stride(-1) != 1) value_error("b needs unit stride on its last dim");
  if (a_in.stride(-1) != 1) value_error("a needs unit stride on its last dim");
  if (out.stride(-1) != 1) value_error("out needs unit stride on its last dim");
  if (z.has_value() && z->stride(-1) != 1) value_error("z needs unit stride on its last dim");
  keep.cw = conv_weight.reshape({conv_dim, kc});
  if (!keep.cw.is_contiguous()) keep.cw = keep.cw.contiguous();
  const auto dt = qkv.scalar_type();
  const std::pair<const char*, const at::Tensor*> same[] = {
      {"b", &b}, {"a", &a_in}, {"conv_weight", &keep.cw}, {"A_log", &A_log},
      {"dt_bias", &dt_bias}, {"conv_state", &conv_state}, {"out", &out}};
  for (const auto& p : same)
    if (p.second->scalar_type() != dt)
      type_error(std::string(p.first) + " has dtype " + c10::toString(p.second->scalar_type()) +
                 ", expected " + c10::toString(dt) + " (one model dtype)");
  keep.rpi = i64(req_pool_indices, "req_pool_indices");
  if (extend_lens.has_value()) keep.el = i64(*extend_lens, "extend_lens");
  keep.A_log = A_log.contiguous();
  keep.dt_bias = dt_bias.contiguous();
  if (norm_weight.has_value()) keep.nw = norm_weight->contiguous();
  if (conv_bias.has_value()) keep.bias = conv_bias->contiguous();
  tf_gdn_args g{};
  g.qkv = qkv.data_ptr();
  g.qkv_stride_tok = qkv.stride(0);
  g.b = b.data_ptr();
  g.b_stride_tok = b.stride(0);
  g.a = a_in.data_ptr();
  g.a_stride_tok = a_in.stride(0);
  g.conv_weight = keep.cw.data_ptr();
  g.conv_bias = keep.bias.defined() ? keep.bias.data_ptr() : nullptr;
  g.A_log = keep.A_log.data_ptr();
  g.dt_bias = keep.dt_bias.data_ptr();
  g.conv_state = conv_state.data_ptr();
  g.conv_stride_slot = conv_state.stride(0);
  g.ssm_state = ssm_state.data_ptr<float>();
  g.ssm_stride_slot = ssm_state.stride(0);
  g.num_slots = ssm_state.size(0);
  g.req_pool_indices = keep.rpi.data_ptr<int64_t>();
  g.extend_lens = keep.el.defined() ? keep.el.data_ptr<int64_t>() : nullptr;
  g.z = optp(z);
  g.z_stride_tok = z.has_value() ? z->stride(0) : 0;
  g.norm_weight = keep.nw.defined() ? keep.nw.data_ptr() : nullptr;
  g.norm_weight_len = keep.nw.defined() ? (int32_t)keep.nw.numel() : 0;
  g.norm_eps = (float)norm_eps;
  g.out = out.data_ptr();
  g.out_stride_tok = out.stride(0);
  g.batch_size = (int32_t)keep.rpi.numel();
  g.num_tokens = (int32_t)t;
  g.max_extend_len = (int32_t)max_extend_len;
  g.num_k_heads = (int32_t)num_k_heads;
  g.num_v_heads = (int32_t)hv;
  g.head_k_dim = (int32_t)head_k_dim;
  g.head_v_dim = (int32_t)head_v_dim;
  g.conv_kernel = (int32_t)kc;
  g.dtype = dtype_code(qkv);
  g.err = errp(err);
  return g;
}

at::Tensor gdn_decode(const at::Tensor& qkv, const at::Tensor& b, const at::Tensor& a,
                      const at::Tensor& conv_weight, const at::Tensor& A_log,
                      const at::Tensor& dt_bias, const at::Tensor& conv_state,
                      const at::Tensor& ssm_state, const at::Tensor& req_pool_indices,
                      int64_t num_k_heads, int64_t head_k_dim, int64_t head_v_dim,
                      const OptT& conv_bias, const OptT& z, const OptT& norm_weight,
                      double norm_eps, OptT out, const OptT& err) {
  const c10::Device dev = need_cuda({&qkv, &b, &a, &conv_weight, &A_log, &dt_bias, &conv_state,
                                     &ssm_state, &req_pool_indices, opt(z), opt(norm_weight),
                                     opt(conv_bias), opt(out), opt(err)});
  if (b.dim() != 2) value_error("b must be [T, Hv]");
  at::Tensor o = out.has_value() ? *out
                                 : at::empty({qkv.size(0), b.size(1) * head_v_dim}, qkv.options());
  GdnKeep keep;
  tf_gdn_args g = gdn_args(qkv, b, a, conv_weight, conv_bias, A_log, dt_bias, conv_state,
                           ssm_state, req_pool_indices, c10::nullopt, z, norm_weight, norm_eps, o,
                           num_k_heads, head_k_dim, head_v_dim, 1, err, keep);
  c10::cuda::CUDAGuard guard(dev);
  check("tf_gdn_decode", tf_gdn_decode(&g, stream_of(dev)));
  return o;
}

at::Tensor gdn_extend(const at::Tensor& qkv, const at::Tensor& b, const at::Tensor& a,
                      const at::Tensor& conv_weight, const at::Tensor& A_log,
                      const at::Tensor& dt_bias, const at::Tensor& conv_state,
                      const at::Tensor& ssm_state, const at::Tensor& req_pool_indices,
                      const at::Tensor& extend_lens, int64_t num_k_heads, int64_t head_k_dim,
                      int64_t head_v_dim, int64_t max_extend_len, const OptT& conv_bias,
                      const OptT& z, const OptT& norm_weight, double norm_eps, OptT out,
                      const OptT& err) {
  const c10::Device dev = need_cuda({&qkv, &b, &a, &conv_weight, &A_log, &dt_bias, &conv_state,
                                     &ssm_state, &req_pool_indices, &extend_lens, opt(z),
                                     opt(norm_weight), opt(conv_bias), opt(out), opt(err)});
  if (b.dim() != 2) value_error("b must be [T, Hv]");
  at::Tensor o = out.has_value() ? *out
                                 : at::empty({qkv.size(0), b.size(1) * head_v_dim}, qkv.options());
  GdnKeep keep;
  tf_gdn_args g = gdn_args(qkv, b, a, conv_weight, conv_bias, A_log, dt_bias, conv_state,
                           ssm_state, req_pool_indices, extend_lens, z, norm_weight, norm_eps, o,
                           num_k_heads, head_k_dim, head_v_dim, max_extend_len, err, keep);
  c10::cuda::CUDAGuard guard(dev);
  const size_t nbytes = tf_gdn_extend_workspace_size(&g);
  void* ws = nbytes ? workspace(dev, nbytes) : nullptr;
  check("tf_gdn_extend", tf_gdn_extend(&g, ws, nbytes, stream_of(dev)));
  return o;
}

at::Tensor gated_rmsnorm(const at::Tensor& x, const at::Tensor& z, const at::Tensor& weight,
                         int64_t head_dim, double eps, OptT out) {
  const c10::Device dev = need_cuda({&x, &z, &weight, opt(out)});
  at::Tensor o = out.has_value() ? *out : at::empty_like(x);
  if (x.dim() != 2 || !x.sizes().equals(z.sizes()) || x.stride(-1) != 1 || z.stride(-1) != 1 ||
      head_dim <= 0 || x.size(1) % head_dim)
    value_error("gated_rmsnorm: x and z must be [T, H*head_dim] with unit inner stride");
  const at::Tensor w = weight.contiguous();
  tf_gated_rmsnorm_args a{};
  a.x = x.data_ptr();
  a.x_stride_tok = x.stride(0);
  a.z = z.data_ptr();
  a.z_stride_tok = z.stride(0);
  a.weight = w.data_ptr();
  a.weight_len = (int32_t)w.numel();
  a.out = o.data_ptr();
  a.out_stride_tok = o.stride(0);
  a.num_tokens = (int32_t)x.size(0);
  a.num_heads = (int32_t)(x.size(1) / head_dim);
  a.head_dim = (int32_t)head_dim;
  a.eps = (float)eps;
  a.dtype = dtype_code(x);
  c10::cuda::CUDAGuard g(dev);
  check("tf_gated_rmsnorm", tf_gated_rmsnorm(&a, stream_of(dev)));
  return o;
}

// ---------------------------------------------------------------------------------------------
// f3 state-slot copies, f2 runtime
// ---------------------------------------------------------------------------------------------
struct SlotRows {
  void* ptr = nullptr;
  int64_t layer = 0, slot = 0, elems = 0;
  int32_t dtype = TF_DTYPE_F32;
};

SlotRows slot_rows(const OptT& pool, const char* name) {
  SlotRows r;
  if (!pool.has_value()) return r;
  const at::Tensor& p = *pool;
  if (p.dim() < 2) value_error(std::string(name) + " must be [layers, slots, ...], got " + shape(p));
  if (p.numel() && !p[0][0].is_contiguous())
    value_error(std::string(name) + ": the rows of one slot in one layer must be contiguous");
  int64_t elems = 1;
  for (int64_t i = 2; i < p.dim(); ++i) elems *= p.size(i);
  r.ptr = p.data_ptr();
  r.layer = p.stride(0);
  r.slot = p.stride(1);
  r.elems = elems;
  r.dtype = dtype_code(p);
  return r;
}

void state_slots_copy(const OptT& conv_state, const OptT& ssm_state, const at::Tensor& src_in,
                      const at::Tensor& dst_in, const OptT& err) {
  if (!conv_state.has_value() && !ssm_state.has_value()) return;
  const c10::Device dev = need_cuda({opt(conv_state), opt(ssm_state), &src_in, &dst_in, opt(err)});
  const at::Tensor& p0 = conv_state.has_value() ? *conv_state : *ssm_state;
  const int64_t L = p0.size(0), S = p0.size(1);
  if (conv_state.has_value() && ssm_state.has_value() &&
      (ssm_state->size(0) != L || ssm_state->size(1) != S))
    value_error("conv_state and ssm_state disagree on layers or slots");
  const at::Tensor src = i64(src_in, "src_slots"), dst = i64(dst_in, "dst_slots");
  if (src.numel() != dst.numel()) value_error("src_slots and dst_slots differ in length");
  if (dst.numel() == 0) return;
  const SlotRows c = slot_rows(conv_state, "conv_state"), s = slot_rows(ssm_state, "ssm_state");
  tf_state_copy_args a{};
  a.conv_state = c.ptr;
  a.conv_stride_layer = c.layer;
  a.conv_stride_slot = c.slot;
  a.conv_slot_elems = c.elems;
  a.conv_dtype = c.dtype;
  a.ssm_state = s.ptr;
  a.ssm_stride_layer = s.layer;
  a.ssm_stride_slot = s.slot;
  a.ssm_slot_elems = s.elems;
  a.ssm_dtype = s.dtype;
  a.num_layers = (int32_t)L;
  a.num_slots = S;
  a.src_slots = src.data_ptr<int64_t>();
  a.dst_slots = dst.data_ptr<int64_t>();
  a.num_ops = (int32_t)dst.numel();
  a.err = errp(err);
  c10::cuda::CUDAGuard g(dev);
  check("tf_state_slots_copy", tf_state_slots_copy(&a, stream_of(dev)));
}

void req_to_token_sync(const at::Tensor& r2t, const at::Tensor& segments_in,
                       const at::Tensor& values_in, const OptT& err) {
  const c10::Device dev = need_cuda({&r2t, &segments_in, &values_in, opt(err)});
  if (r2t.scalar_type() != at::kLong || r2t.dim() != 2 || r2t.stride(1) != 1)
    value_error("req_to_token must be a row-major [rows, cols] int64 tensor");
  const at::Tensor seg = i64(segments_in, "segments"), val = i64(values_in, "values");
  if (seg.dim() != 2 || seg.size(1) != 4) value_error("segments must be [n, 4] (row, col, len, src)");
  tf_r2t_sync_args a{};
  a.req_to_token = r2t.data_ptr<int64_t>();
  a.r2t_stride = r2t.stride(0);
  a.r2t_rows = r2t.size(0);
  a.r2t_cols = r2t.size(1);
  a.segments = seg.data_ptr<int64_t>();
  a.num_segments = (int32_t)seg.size(0);
  a.values = val.data_ptr<int64_t>();
  a.num_values = val.numel();
  a.err = errp(err);
  c10::cuda::CUDAGuard g(dev);
  check("tf_req_to_token_sync", tf_req_to_token_sync(&a, stream_of(dev)));
}

at::Tensor sample_tokens(const at::Tensor& logits, const at::Tensor& temperature,
                         const OptT& uniform, OptT out) {
  const c10::Device dev = need_cuda({&logits, &temperature, opt(uniform), opt(out)});
  if (logits.dim() != 2 || logits.stride(1) != 1)
    value_error("logits must be [B, V] with contiguous rows");
  const int64_t B = logits.size(0), V = logits.size(1);
  if (temperature.scalar_type() != at::kFloat || temperature.numel() != B)
    value_error("temperature must be float32 [B]");
  if (uniform.has_value() && (uniform->scalar_type() != at::kFloat || uniform->numel() != B))
    value_error("uniform must be float32 [B]");
  at::Tensor o = out.has_value() ? *out
                                 : at::empty({B}, logits.options().dtype(at::kLong));
  const at::Tensor temp = temperature.contiguous();
  tf_sample_args a{};
  a.logits = logits.data_ptr();
  a.logits_stride = logits.stride(0);
  a.batch_size = (int32_t)B;
  a.vocab_size = (int32_t)V;
  a.dtype = dtype_code(logits);
  a.temperature = temp.data_ptr<float>();
  a.uniform = uniform.has_value() ? uniform->data_ptr<float>() : nullptr;
  a.out = o.data_ptr<int64_t>();
  c10::cuda::CUDAGuard g(dev);
  check("tf_sample_tokens", tf_sample_tokens(&a, stream_of(dev)));
  return o;
}

// ---------------------------------------------------------------------------------------------
// f4 block-FP8 linear
// ---------------------------------------------------------------------------------------------
std::tuple<at::Tensor, at::Tensor> fp8_quantize(const at::Tensor& x2d) {
  const c10::Device dev = need_cuda({&x2d});
  if (x2d.dim() != 2 || x2d.stride(1) != 1)
    value_error("fp8_quantize takes [M, K] with contiguous rows");
  const int64_t M = x2d.size(0), K = x2d.size(1);
  at::Tensor q = at::empty({M, K}, x2d.options().dtype(at::ScalarType::Float8_e4m3fn));
  at::Tensor scale = at::empty({1}, x2d.options().dtype(at::kFloat));
  at::Tensor scratch = at::empty({4}, x2d.options().dtype(at::kInt));
  tf_fp8_quant_args a{};
  a.x = x2d.data_ptr();
  a.x_stride = x2d.stride(0);
  a.M = M;
  a.K = (int32_t)K;
  a.dtype = dtype_code(x2d);
  a.q = (uint8_t*)q.data_ptr();
  a.x_scale = scale.data_ptr<float>();
  a.workspace = scratch.data_ptr();
  c10::cuda::CUDAGuard g(dev);
  check("tf_fp8_quantize", tf_fp8_quantize(&a, stream_of(dev)));
  return {q, scale};
}

at::Tensor fp8_block_gemm(const at::Tensor& q, const at::Tensor& x_scale, const at::Tensor& weight,
                          const OptT& weight_scale_inv, const OptT& bias, int64_t out_dtype_code,
                          int64_t block_h, int64_t block_w, OptT out) {
  const c10::Device dev =
      need_cuda({&q, &x_scale, &weight, opt(weight_scale_inv), opt(bias), opt(out)});
  if (q.dim() != 2 || weight.dim() != 2) value_error("q [M, K] and weight [N, K] must be matrices");
  const int64_t M = q.size(0), K = q.size(1), N = weight.size(0);
  if (weight.size(1) != K || weight.stride(1) != 1 || q.stride(1) != 1)
    value_error("q [M, K] and weight [N, K] need contiguous rows of the same K");
  const at::ScalarType out_dtype = out_dtype_code == TF_DTYPE_F32    ? at::kFloat
                                   : out_dtype_code == TF_DTYPE_BF16 ? at::kBFloat16
                                   : out_dtype_code == TF_DTYPE_F16  ? at::kHalf
                                                                     : at::kByte;
  if (out_dtype == at::kByte) type_error("fp8_block_gemm: unsupported output dtype");
  at::Tensor o = out.has_value() ? *out : at::empty({M, N}, q.options().dtype(out_dtype));
  at::Tensor ws;
  if (weight_scale_inv.has_value())
    ws = weight_scale_inv->scalar_type() == at::kFloat ? *weight_scale_inv
                                                        : weight_scale_inv->to(at::kFloat);
  tf_fp8_gemm_args a{};
  a.q = (const uint8_t*)q.data_ptr();
  a.q_stride = q.stride(0);
  a.x_scale = x_scale.data_ptr<float>();
  a.w = (const uint8_t*)weight.data_ptr();
  a.w_stride = weight.stride(0);
  a.w_scale = ws.defined() ? ws.data_ptr<float>() : nullptr;
  a.ws_stride_n = ws.defined() ? ws.stride(0) : 0;
  a.ws_stride_k = ws.defined() ? ws.stride(1) : 0;
  a.block_h = (int32_t)block_h;
  a.block_w = (int32_t)block_w;
  a.bias = optp(bias);
  a.bias_dtype = bias.has_value() ? dtype_code(*bias) : 0;
  a.out = o.data_ptr();
  a.out_stride = o.stride(0);
  a.out_dtype = dtype_code(o);
  a.M = M;
  a.N = (int32_t)N;
  a.K = (int32_t)K;
  c10::cuda::CUDAGuard g(dev);
  check("tf_fp8_block_gemm", tf_fp8_block_gemm(&a, stream_of(dev)));
  return o;
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "PyTorch front end of libtfattn (include/tfattn.h)";
  err_class() = py::module_::import("tokenfactory_b200._capi").attr("TFAttnError");
  m.attr("ABI_VERSION") = tf_abi_version();
  const auto none = py::none();
  m.def("kv_store", &kv_store, py::arg("k_buffer"), py::arg("v_buffer"), py::arg("out_cache_loc"),
        py::arg("k"), py::arg("v"), py::arg("err") = none);
  m.def("attn_prologue", &attn_prologue);
  m.def("paged_decode", &paged_decode);
  m.def("paged_extend", &paged_extend);
  m.def("gdn_decode", &gdn_decode);
  m.def("gdn_extend", &gdn_extend);
  m.def("gated_rmsnorm", &gated_rmsnorm);
  m.def("state_slots_copy", &state_slots_copy);
  m.def("req_to_token_sync", &req_to_token_sync);
  m.def("sample_tokens", &sample_tokens);
  m.def("fp8_quantize", &fp8_quantize);
  m.def("fp8_block_gemm", &fp8_block_gemm);
}
