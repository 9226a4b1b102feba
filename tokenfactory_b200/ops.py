"""torch-tensor front end of the C ABI (libtfattn.so).

Each function takes torch CUDA tensors in the reference's layouts and hands them to the PyTorch
C++ extension `tokenfactory_b200._C` (csrc/torch_ext.cpp), which checks shapes, dtypes and strides,
fills the C argument structure with data pointers and strides, and launches on the current torch
stream of the tensors' device; scratch memory comes from a per-(device, stream) workspace grown on
demand and reused in stream order.  Argument errors raise ValueError / TypeError, a failing entry
point raises _capi.TFAttnError.  Nothing here computes on the CPU, and importing this module fails
loudly when the extension or the library has not been built.
"""

import ctypes
from typing import Optional, Tuple

import torch

from . import _capi as C

try:
    from . import _C
except ImportError as e:  # no fallback: the hot path exists only as CUDA kernels
    raise ImportError("tokenfactory_b200._C is not built (python -m tokenfactory_b200.build): "
                      f"{e}") from e

_DTYPES = {torch.float32: C.TF_DTYPE_F32, torch.bfloat16: C.TF_DTYPE_BF16,
           torch.float16: C.TF_DTYPE_F16}
GATE_MODES = {"none": C.TF_GATE_NONE, "silu": C.TF_GATE_SILU, "sigmoid": C.TF_GATE_SIGMOID}
SLOT_MODES = {"clamp": C.TF_SLOT_CLAMP, "wrap": C.TF_SLOT_WRAP}


def _dtype(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("tokenfactory_b200 kernels need CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _i64(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int64:
        raise TypeError(f"{name} must be int64 (got {t.dtype})")
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------------------------
# a1. KV store
# ---------------------------------------------------------------------------------------------
def kv_store(k_buffer: torch.Tensor, v_buffer: torch.Tensor, out_cache_loc: torch.Tensor,
             k: torch.Tensor, v: torch.Tensor, err: Optional[torch.Tensor] = None) -> None:
    """k_buffer[out_cache_loc] = k; v_buffer[out_cache_loc] = v (qwen3_8/full_attention.py:147-149).

    k_buffer/v_buffer: layer views [num_slots, Hkv, D]; k, v: [T, Hkv, D]; out_cache_loc [T] int64.
    """
    _C.kv_store(k_buffer, v_buffer, out_cache_loc, k, v, err)

def attn_prologue(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm_weight: torch.Tensor,
                  k_norm_weight: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
                  k_buffer: torch.Tensor, v_buffer: torch.Tensor, out_cache_loc: torch.Tensor,
                  eps: float = 1e-6, mrope_section=(11, 11, 10), mrope_interleaved: bool = True,
                  q_out: Optional[torch.Tensor] = None,
                  err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused q/k RMSNorm + partial (M-)RoPE + KV-pool store of Qwen3_8FullAttention.forward
    (qwen3_8/full_attention.py:142-149, qwen3_8/rms_norm.py:19-24,
    qwen3_8/rotary_embedding.py:46-95).  q [T, Hq, D], k/v [T, Hkv, D] (strided views allowed),
    positions [T] or [3, T] int64, inv_freq the rotary module's fp32 buffer [rotary_dim/2].
    Writes k/v into k_buffer/v_buffer at out_cache_loc and returns the rotated q [T, Hq, D]."""
    if positions.dim() == 2 and positions.stride(-1) != 1:
        positions = positions.contiguous()
    return _C.attn_prologue(q, k, v, q_norm_weight, k_norm_weight, positions, inv_freq, k_buffer,
                            v_buffer, out_cache_loc, float(eps), list(mrope_section),
                            bool(mrope_interleaved), q_out, err)

# ---------------------------------------------------------------------------------------------
# a2-a4. paged attention
# ---------------------------------------------------------------------------------------------
def _paged_args(q, k_buffer, v_buffer, req_to_token, req_pool_indices, seq_lens, extend_lens,
                scale, gate, gate_mode, out, max_seq_len, max_extend_len, slot_mode, err):
    if q.dim() != 3 or k_buffer.dim() != 3 or k_buffer.shape != v_buffer.shape:
        raise ValueError(f"paged attention shapes: q {tuple(q.shape)}, pool {tuple(k_buffer.shape)}")
    t, hq, d = q.shape
    if k_buffer.shape[2] != d or hq % k_buffer.shape[1] != 0:
        raise ValueError("q heads must be a multiple of kv heads and head dims must agree")
    if q.stride(2) != 1 or k_buffer.stride(2) != 1 or out.stride(2) != 1 or \
            k_buffer.stride() != v_buffer.stride():
        raise ValueError("paged attention needs unit stride on head_dim")
    if q.dtype != k_buffer.dtype or v_buffer.dtype != q.dtype or out.dtype != q.dtype:
        raise TypeError("q, pools and out must share a dtype")
    if gate is not None:
        if gate.shape != q.shape or gate.stride(2) != 1 or gate.dtype != q.dtype:
            raise ValueError("gate must be a [T, Hq, D] view with unit stride on D")
    r2t = req_to_token
    if r2t.dtype != torch.int64 or r2t.dim() != 2 or r2t.stride(1) != 1:
        raise ValueError("req_to_token must be a row-major int64 [rows, cols] table")
    rpi = _i64(req_pool_indices, "req_pool_indices")
    sl = _i64(seq_lens, "seq_lens")
    el = None if extend_lens is None else _i64(extend_lens, "extend_lens")
    return C.PagedAttnArgs(
        q=q.data_ptr(), q_stride_tok=q.stride(0), q_stride_head=q.stride(1),
        k_buffer=k_buffer.data_ptr(), v_buffer=v_buffer.data_ptr(),
        kv_stride_slot=k_buffer.stride(0), kv_stride_head=k_buffer.stride(1),
        num_slots=k_buffer.shape[0],
        req_to_token=r2t.data_ptr(), r2t_stride=r2t.stride(0), r2t_rows=r2t.shape[0],
        r2t_cols=r2t.shape[1],
        req_pool_indices=rpi.data_ptr(), seq_lens=sl.data_ptr(),
        extend_lens=None if el is None else el.data_ptr(),
        gate=_ptr(gate), gate_stride_tok=0 if gate is None else gate.stride(0),
        gate_stride_head=0 if gate is None else gate.stride(1),
        out=out.data_ptr(), out_stride_tok=out.stride(0), out_stride_head=out.stride(1),
        batch_size=rpi.numel(), num_tokens=t, num_q_heads=hq, num_kv_heads=k_buffer.shape[1],
        head_dim=d, max_seq_len=int(max_seq_len), max_extend_len=int(max_extend_len),
        scale=float(scale), dtype=_dtype(q), gate_mode=GATE_MODES[gate_mode],
        slot_mode=SLOT_MODES[slot_mode], err=_ptr(err)), (rpi, sl, el)


def paged_decode(q: torch.Tensor, k_buffer: torch.Tensor, v_buffer: torch.Tensor,
                 req_to_token: torch.Tensor, req_pool_indices: torch.Tensor,
                 seq_lens: torch.Tensor, scale: float, max_seq_len: int,
                 gate: Optional[torch.Tensor] = None, gate_mode: str = "none",
                 out: Optional[torch.Tensor] = None, slot_mode: str = "clamp",
                 err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode step of paged GQA attention, one query token per request
    (qwen3_8/full_attention.py:215-242), with the output gate fused (:157-158).  Returns
    out [B, Hq, D]."""
    return _C.paged_decode(q, k_buffer, v_buffer, req_to_token, req_pool_indices, seq_lens,
                           float(scale), int(max_seq_len), gate, GATE_MODES[gate_mode], out,
                           SLOT_MODES[slot_mode], err)

def paged_extend(q: torch.Tensor, k_buffer: torch.Tensor, v_buffer: torch.Tensor,
                 req_to_token: torch.Tensor, req_pool_indices: torch.Tensor,
                 seq_lens: torch.Tensor, extend_lens: torch.Tensor, scale: float,
                 max_seq_len: int, max_extend_len: int, gate: Optional[torch.Tensor] = None,
                 gate_mode: str = "none", out: Optional[torch.Tensor] = None,
                 slot_mode: str = "clamp", err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Varlen extend over a radix-cached prefix (qwen3_8/full_attention.py:179-213, 244-283):
    query i of request b attends to positions <= seq_len_b - extend_len_b + i.  q is packed
    [T, Hq, D] in request order.  Returns out [T, Hq, D]."""
    return _C.paged_extend(q, k_buffer, v_buffer, req_to_token, req_pool_indices, seq_lens,
                           extend_lens, float(scale), int(max_seq_len), int(max_extend_len), gate,
                           GATE_MODES[gate_mode], out, SLOT_MODES[slot_mode], err)

# ---------------------------------------------------------------------------------------------
# a5-a9. Gated DeltaNet
# ---------------------------------------------------------------------------------------------
def gdn_decode(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state, req_pool_indices,
               num_k_heads: int, head_k_dim: int, head_v_dim: int, conv_bias=None, z=None,
               norm_weight=None, norm_eps: float = 1e-6, out=None, err=None) -> torch.Tensor:
    """Batched one-token GDN step (qwen3_8/linear_attention.py:244-298) updating conv_state and
    ssm_state in place at the request rows; with z given, the gated RMSNorm of
    qwen3_8/rms_norm_gated.py:26-40 is fused.  Returns out [B, Hv*dv]."""
    return _C.gdn_decode(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state,
                         req_pool_indices, int(num_k_heads), int(head_k_dim), int(head_v_dim),
                         conv_bias, z, norm_weight, float(norm_eps), out, err)

def gdn_extend(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state, req_pool_indices,
               extend_lens, num_k_heads: int, head_k_dim: int, head_v_dim: int,
               max_extend_len: int, conv_bias=None, z=None, norm_weight=None,
               norm_eps: float = 1e-6, out=None, err=None) -> torch.Tensor:
    """Varlen GDN over packed tokens of several requests (extend / mixed batches), replacing the
    per-request loop of qwen3_8/linear_attention.py:329-358.  Returns out [T, Hv*dv]."""
    return _C.gdn_extend(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state,
                         req_pool_indices, extend_lens, int(num_k_heads), int(head_k_dim),
                         int(head_v_dim), int(max_extend_len), conv_bias, z, norm_weight,
                         float(norm_eps), out, err)

def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, head_dim: int,
                  eps: float = 1e-6, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """w * x/rms_head(x) * silu(z) (qwen3_8/rms_norm_gated.py:26-40); x, z [T, H*hd]."""
    return _C.gated_rmsnorm(x, z, weight, int(head_dim), float(eps), out)

# ---------------------------------------------------------------------------------------------
# GDN state-slot snapshots: copies / resets of every linear layer's rows in one launch
# ---------------------------------------------------------------------------------------------
def state_slot_ops_valid(src, dst) -> None:
    """The ops of one state_slots_copy call run concurrently: reject a batch whose result would
    depend on their order (a destination written twice, or read by another op)."""
    if len(src) != len(dst):
        raise ValueError("src and dst lists differ in length")
    dsts = [int(d) for d in dst]
    if len(set(dsts)) != len(dsts):
        raise ValueError(f"a destination slot appears twice: {dsts}")
    for i, s in enumerate(src):
        if s is not None and int(s) != dsts[i] and int(s) in set(dsts):
            raise ValueError(f"slot {int(s)} is both read and written in one batch")


def state_slots_copy(conv_state: Optional[torch.Tensor], ssm_state: Optional[torch.Tensor],
                     src_slots, dst_slots, err: Optional[torch.Tensor] = None) -> None:
    """For each op i: every layer's rows of slot dst_slots[i] in both pools become a copy of slot
    src_slots[i] (ReqToStatePool.capture_snapshot / restore_snapshot,
    req_to_state_pool.py:160-194), or zeros where the source is None / -1 (reset_working_state,
    free_snapshot, req_to_state_pool.py:120-153).  One launch for all ops, layers and both pools.

    conv_state [L, slots, conv_dim, K-1] and ssm_state [L, slots, Hv, dk, dv] as the reference
    allocates them (either may be None).  The slot lists are host sequences (checked for order
    dependence here, then copied to the device) or int64 CUDA tensors (used as they are)."""
    pools = [p for p in (conv_state, ssm_state) if p is not None]
    if not pools:
        return
    dev = _need_cuda(*pools)
    L, S = pools[0].shape[0], pools[0].shape[1]
    for p in pools[1:]:
        if p.shape[0] != L or p.shape[1] != S:
            raise ValueError("conv_state and ssm_state disagree on layers or slots")
    if isinstance(src_slots, torch.Tensor) or isinstance(dst_slots, torch.Tensor):
        src_t = _i64(src_slots, "src_slots")
        dst_t = _i64(dst_slots, "dst_slots")
        _need_cuda(src_t, dst_t)
        if src_t.numel() != dst_t.numel():
            raise ValueError("src_slots and dst_slots differ in length")
    else:
        state_slot_ops_valid(src_slots, dst_slots)
        if not dst_slots:
            return
        host = torch.tensor([[-1 if s is None else int(s) for s in src_slots],
                             [int(d) for d in dst_slots]], dtype=torch.int64).pin_memory()
        both = host.to(dev, non_blocking=True)
        src_t, dst_t = both[0], both[1]
    if dst_t.numel() == 0:
        return
    _C.state_slots_copy(conv_state, ssm_state, src_t, dst_t, err)


# ---------------------------------------------------------------------------------------------
# per-step runtime: req_to_token sync and batched sampling
# ---------------------------------------------------------------------------------------------
def req_to_token_sync(req_to_token: torch.Tensor, segments: torch.Tensor, values: torch.Tensor,
                      err: Optional[torch.Tensor] = None) -> None:
    """req_to_token[row, col:col+len] = values[src:src+len] for every (row, col, len, src) row of
    segments [n, 4] int64 (the incremental sync of ModelRunner._prepare_forward_batch,
    engine/model_runner.py:147-166), one launch."""
    _C.req_to_token_sync(req_to_token, segments, values, err)


def sample_tokens(logits: torch.Tensor, temperature: torch.Tensor,
                  uniform: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Next token of every row of logits [B, V] (ModelRunner._sample_one,
    engine/model_runner.py:574-578): argmax where temperature <= 1e-5 (or uniform is None), else
    the inverse-CDF draw of softmax(logits / T) at uniform[b] in [0, 1).  Returns int64 [B]."""
    return _C.sample_tokens(logits, temperature, uniform, out)


# ---------------------------------------------------------------------------------------------
# block-FP8 linear
# ---------------------------------------------------------------------------------------------
def fp8_quantize(x2d: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(q [M, K] float8_e4m3fn, x_scale [1] float32) of the dynamic per-tensor activation
    quantization of triton_block_fp8_linear (qwen3_8/fp8_triton.py:124-130), bit-exact."""
    return _C.fp8_quantize(x2d)


def fp8_block_gemm(q: torch.Tensor, x_scale: torch.Tensor, weight: torch.Tensor,
                   weight_scale_inv: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                   out_dtype: torch.dtype, block_h: int = 128, block_w: int = 128,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out [M, N] = (q @ weight^T per 128-wide K block * weight_scale_inv[n/bh, k/bw]) * x_scale
    + bias, on the tensor cores (the kernel of qwen3_8/fp8_triton.py:17-98)."""
    if out_dtype not in _DTYPES:
        raise TypeError(f"unsupported output dtype {out_dtype}")
    return _C.fp8_block_gemm(q, x_scale, weight, weight_scale_inv, bias, _DTYPES[out_dtype],
                             int(block_h), int(block_w), out)


def block_fp8_linear(x: torch.Tensor, weight: torch.Tensor,
                     weight_scale_inv: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                     block_h: int = 128, block_w: int = 128) -> torch.Tensor:
    """triton_block_fp8_linear (qwen3_8/fp8_triton.py:109-181) with the same arguments and result:
    dynamic per-tensor e4m3 activations, e4m3 weight [N, K] with block scales
    weight_scale_inv [ceil(N/bh), ceil(K/bw)] (or None), output in x's dtype."""
    N, K = weight.shape
    x2d = x.reshape(-1, K)
    if x2d.stride(1) != 1:
        x2d = x2d.contiguous()
    q, scale = fp8_quantize(x2d)
    out = fp8_block_gemm(q, scale, weight, weight_scale_inv, bias, x.dtype, block_h, block_w)
    return out.reshape(*x.shape[:-1], N)
