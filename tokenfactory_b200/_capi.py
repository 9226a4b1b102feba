"""ctypes binding of libtfattn.so, the C ABI declared in include/tfattn.h.

The structures below mirror the header field by field (tests/test_capi_abi.py compiles the header
with the host C compiler and checks every size and offset).  Loading fails loudly: there is no CPU
fallback for the hot path.
"""

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtfattn.so")

ABI_VERSION = 1

TF_OK, TF_ERR_INVALID_ARG, TF_ERR_UNSUPPORTED, TF_ERR_ALIGNMENT, TF_ERR_WORKSPACE, TF_ERR_CUDA = range(6)
TF_DTYPE_F32, TF_DTYPE_BF16, TF_DTYPE_F16 = 0, 1, 2
TF_GATE_NONE, TF_GATE_SILU, TF_GATE_SIGMOID = 0, 1, 2
TF_SLOT_CLAMP, TF_SLOT_WRAP = 0, 1
TF_KERR_NONE, TF_KERR_SLOT_RANGE, TF_KERR_REQ_RANGE, TF_KERR_TIMEOUT = 0, 1, 2, 3

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float


class KVStoreArgs(ctypes.Structure):
    _fields_ = [
        ("k_buffer", _vp), ("v_buffer", _vp),
        ("buf_stride_slot", _i64), ("buf_stride_head", _i64), ("num_slots", _i64),
        ("k", _vp), ("v", _vp),
        ("k_stride_tok", _i64), ("k_stride_head", _i64),
        ("v_stride_tok", _i64), ("v_stride_head", _i64),
        ("out_cache_loc", _vp), ("num_tokens", _i64),
        ("num_kv_heads", _i32), ("head_dim", _i32), ("dtype", _i32),
        ("err", _vp),
    ]


class AttnPrologueArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("q_stride_tok", _i64), ("q_stride_head", _i64),
        ("k", _vp), ("k_stride_tok", _i64), ("k_stride_head", _i64),
        ("v", _vp), ("v_stride_tok", _i64), ("v_stride_head", _i64),
        ("q_norm_weight", _vp), ("k_norm_weight", _vp),
        ("positions", _vp), ("pos_stride", _i64), ("inv_freq", _vp),
        ("q_out", _vp), ("q_out_stride_tok", _i64), ("q_out_stride_head", _i64),
        ("k_buffer", _vp), ("v_buffer", _vp),
        ("buf_stride_slot", _i64), ("buf_stride_head", _i64), ("num_slots", _i64),
        ("out_cache_loc", _vp), ("num_tokens", _i64),
        ("eps", ctypes.c_float), ("pos_rows", _i32), ("mrope_section", _i32 * 3),
        ("mrope_interleaved", _i32), ("rotary_dim", _i32),
        ("num_q_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32), ("dtype", _i32),
        ("norm_weight_dtype", _i32), ("err", _vp),
    ]


class PagedAttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("q_stride_tok", _i64), ("q_stride_head", _i64),
        ("k_buffer", _vp), ("v_buffer", _vp),
        ("kv_stride_slot", _i64), ("kv_stride_head", _i64), ("num_slots", _i64),
        ("req_to_token", _vp), ("r2t_stride", _i64), ("r2t_rows", _i64), ("r2t_cols", _i64),
        ("req_pool_indices", _vp), ("seq_lens", _vp), ("extend_lens", _vp),
        ("gate", _vp), ("gate_stride_tok", _i64), ("gate_stride_head", _i64),
        ("out", _vp), ("out_stride_tok", _i64), ("out_stride_head", _i64),
        ("batch_size", _i32), ("num_tokens", _i32),
        ("num_q_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("max_seq_len", _i32), ("max_extend_len", _i32),
        ("scale", _f32), ("dtype", _i32), ("gate_mode", _i32), ("slot_mode", _i32),
        ("err", _vp),
    ]


class GdnArgs(ctypes.Structure):
    _fields_ = [
        ("qkv", _vp), ("qkv_stride_tok", _i64),
        ("b", _vp), ("b_stride_tok", _i64),
        ("a", _vp), ("a_stride_tok", _i64),
        ("conv_weight", _vp), ("conv_bias", _vp), ("A_log", _vp), ("dt_bias", _vp),
        ("conv_state", _vp), ("conv_stride_slot", _i64),
        ("ssm_state", _vp), ("ssm_stride_slot", _i64), ("num_slots", _i64),
        ("req_pool_indices", _vp), ("extend_lens", _vp),
        ("z", _vp), ("z_stride_tok", _i64),
        ("norm_weight", _vp), ("norm_weight_len", _i32), ("norm_eps", _f32),
        ("out", _vp), ("out_stride_tok", _i64),
        ("batch_size", _i32), ("num_tokens", _i32), ("max_extend_len", _i32),
        ("num_k_heads", _i32), ("num_v_heads", _i32), ("head_k_dim", _i32), ("head_v_dim", _i32),
        ("conv_kernel", _i32), ("dtype", _i32),
        ("err", _vp),
    ]


class GatedRMSNormArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("x_stride_tok", _i64),
        ("z", _vp), ("z_stride_tok", _i64),
        ("weight", _vp), ("weight_len", _i32),
        ("out", _vp), ("out_stride_tok", _i64),
        ("num_tokens", _i32), ("num_heads", _i32), ("head_dim", _i32),
        ("eps", _f32), ("dtype", _i32),
    ]


class StateCopyArgs(ctypes.Structure):
    _fields_ = [
        ("conv_state", _vp), ("conv_stride_layer", _i64), ("conv_stride_slot", _i64),
        ("conv_slot_elems", _i64), ("conv_dtype", _i32),
        ("ssm_state", _vp), ("ssm_stride_layer", _i64), ("ssm_stride_slot", _i64),
        ("ssm_slot_elems", _i64), ("ssm_dtype", _i32),
        ("num_layers", _i32), ("num_slots", _i64),
        ("src_slots", _vp), ("dst_slots", _vp), ("num_ops", _i32),
        ("err", _vp),
    ]


class R2TSyncArgs(ctypes.Structure):
    _fields_ = [
        ("req_to_token", _vp), ("r2t_stride", _i64), ("r2t_rows", _i64), ("r2t_cols", _i64),
        ("segments", _vp), ("num_segments", _i32),
        ("values", _vp), ("num_values", _i64),
        ("err", _vp),
    ]


class SampleArgs(ctypes.Structure):
    _fields_ = [
        ("logits", _vp), ("logits_stride", _i64),
        ("batch_size", _i32), ("vocab_size", _i32), ("dtype", _i32),
        ("temperature", _vp), ("uniform", _vp), ("out", _vp),
    ]


class FP8QuantArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("x_stride", _i64), ("M", _i64), ("K", _i32), ("dtype", _i32),
        ("q", _vp), ("x_scale", _vp), ("workspace", _vp),
    ]


class FP8GemmArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("q_stride", _i64), ("x_scale", _vp),
        ("w", _vp), ("w_stride", _i64),
        ("w_scale", _vp), ("ws_stride_n", _i64), ("ws_stride_k", _i64),
        ("block_h", _i32), ("block_w", _i32),
        ("bias", _vp), ("bias_dtype", _i32),
        ("out", _vp), ("out_stride", _i64), ("out_dtype", _i32),
        ("M", _i64), ("N", _i32), ("K", _i32),
        ("err", _vp),
    ]


# (name, restype, argtypes) of every exported entry point, in header order
SIGNATURES = [
    ("tf_abi_version", ctypes.c_int, []),
    ("tf_status_string", ctypes.c_char_p, [_i32]),
    ("tf_last_error", ctypes.c_char_p, []),
    ("tf_kv_store", _i32, [ctypes.POINTER(KVStoreArgs), _vp]),
    ("tf_attn_prologue", _i32, [ctypes.POINTER(AttnPrologueArgs), _vp]),
    ("tf_paged_decode_workspace_size", ctypes.c_size_t, [ctypes.POINTER(PagedAttnArgs)]),
    ("tf_paged_decode_attn", _i32, [ctypes.POINTER(PagedAttnArgs), _vp, ctypes.c_size_t, _vp]),
    ("tf_paged_decode_attn_noalloc", _i32, [ctypes.POINTER(PagedAttnArgs), _vp]),
    ("tf_paged_extend_workspace_size", ctypes.c_size_t, [ctypes.POINTER(PagedAttnArgs)]),
    ("tf_paged_extend_attn", _i32, [ctypes.POINTER(PagedAttnArgs), _vp, ctypes.c_size_t, _vp]),
    ("tf_gdn_decode", _i32, [ctypes.POINTER(GdnArgs), _vp]),
    ("tf_gdn_extend_workspace_size", ctypes.c_size_t, [ctypes.POINTER(GdnArgs)]),
    ("tf_gdn_extend", _i32, [ctypes.POINTER(GdnArgs), _vp, ctypes.c_size_t, _vp]),
    ("tf_gated_rmsnorm", _i32, [ctypes.POINTER(GatedRMSNormArgs), _vp]),
    ("tf_state_slots_copy", _i32, [ctypes.POINTER(StateCopyArgs), _vp]),
    ("tf_req_to_token_sync", _i32, [ctypes.POINTER(R2TSyncArgs), _vp]),
    ("tf_sample_tokens", _i32, [ctypes.POINTER(SampleArgs), _vp]),
    ("tf_fp8_quantize", _i32, [ctypes.POINTER(FP8QuantArgs), _vp]),
    ("tf_fp8_block_gemm", _i32, [ctypes.POINTER(FP8GemmArgs), _vp]),
]

_lib = None
_lock = threading.Lock()


class TFAttnError(RuntimeError):
    """A libtfattn entry point returned a non-zero tf_status."""

    def __init__(self, fn: str, status: int, message: str):
        self.status = status
        super().__init__(f"{fn} failed ({status}): {message}")


def load() -> ctypes.CDLL:
    """Load libtfattn.so once (thread-safe); raises if it is missing or of another ABI."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m tokenfactory_b200.build` "
                "(the hot path has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.tf_abi_version() != ABI_VERSION:
            raise ImportError(f"{LIB_PATH} has ABI {lib.tf_abi_version()}, expected {ABI_VERSION}")
        _lib = lib
    return _lib


def check(fn: str, status: int) -> None:
    if status != TF_OK:
        lib = load()
        msg = lib.tf_last_error().decode(errors="replace") or lib.tf_status_string(status).decode()
        raise TFAttnError(fn, status, msg)
