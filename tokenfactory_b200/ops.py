"""torch-tensor front end of the C ABI (libtfattn.so).

Each function takes torch CUDA tensors in the reference's layouts, checks shapes, fills the C
argument structure with data pointers and strides, and launches on the current torch stream of the
tensors' device.  Scratch memory comes from a per-(device, stream) workspace that is grown on demand
and reused in stream order.  Nothing here computes on the CPU.
"""

import ctypes
from typing import Dict, Optional, Tuple

import torch

from . import _capi as C

_DTYPES = {torch.float32: C.TF_DTYPE_F32, torch.bfloat16: C.TF_DTYPE_BF16,
           torch.float16: C.TF_DTYPE_F16}
GATE_MODES = {"none": C.TF_GATE_NONE, "silu": C.TF_GATE_SILU, "sigmoid": C.TF_GATE_SIGMOID}
SLOT_MODES = {"clamp": C.TF_SLOT_CLAMP, "wrap": C.TF_SLOT_WRAP}

_workspaces: Dict[Tuple[int, int], torch.Tensor] = {}


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


def workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    """A 256-byte aligned scratch buffer of at least `nbytes` for the current stream of `dev`."""
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), _stream(dev))
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _workspaces[key] = buf
    return buf


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
    dev = _need_cuda(k_buffer, v_buffer, out_cache_loc, k, v)
    if k.dim() != 3 or k.shape != v.shape or k_buffer.shape != v_buffer.shape:
        raise ValueError(f"kv_store shapes: k {tuple(k.shape)} v {tuple(v.shape)} "
                         f"pool {tuple(k_buffer.shape)} / {tuple(v_buffer.shape)}")
    if k_buffer.stride() != v_buffer.stride() or k_buffer.stride(2) != 1 or k.stride(2) != 1 or \
            v.stride(2) != 1:
        raise ValueError("kv_store needs unit stride on head_dim and equal pool strides")
    if k.shape[1:] != k_buffer.shape[1:] or k.dtype != k_buffer.dtype or v.dtype != k.dtype:
        raise ValueError("kv_store: k/v rows must match the pool's [Hkv, D] and dtype")
    loc = _i64(out_cache_loc, "out_cache_loc")
    if loc.numel() != k.shape[0]:
        raise ValueError("out_cache_loc must have one entry per token")
    a = C.KVStoreArgs(
        k_buffer=k_buffer.data_ptr(), v_buffer=v_buffer.data_ptr(),
        buf_stride_slot=k_buffer.stride(0), buf_stride_head=k_buffer.stride(1),
        num_slots=k_buffer.shape[0], k=k.data_ptr(), v=v.data_ptr(),
        k_stride_tok=k.stride(0), k_stride_head=k.stride(1),
        v_stride_tok=v.stride(0), v_stride_head=v.stride(1),
        out_cache_loc=loc.data_ptr(), num_tokens=k.shape[0], num_kv_heads=k.shape[1],
        head_dim=k.shape[2], dtype=_dtype(k), err=_ptr(err))
    with torch.cuda.device(dev):
        C.check("tf_kv_store", C.load().tf_kv_store(ctypes.byref(a), _stream(dev)))


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
    dev = _need_cuda(q, k, v, q_norm_weight, k_norm_weight, positions, inv_freq, k_buffer,
                     v_buffer, out_cache_loc)
    if q.dim() != 3 or k.dim() != 3 or k.shape != v.shape or k_buffer.shape != v_buffer.shape:
        raise ValueError(f"attn_prologue shapes: q {tuple(q.shape)} k {tuple(k.shape)} "
                         f"v {tuple(v.shape)} pool {tuple(k_buffer.shape)}")
    t, hq, d = q.shape
    if k.shape[0] != t or k.shape[2] != d or k.shape[1:] != k_buffer.shape[1:]:
        raise ValueError("attn_prologue: k/v rows must be [T, Hkv, D] matching the pool")
    if q.stride(2) != 1 or k.stride(2) != 1 or v.stride(2) != 1 or k_buffer.stride(2) != 1 or \
            k_buffer.stride() != v_buffer.stride():
        raise ValueError("attn_prologue needs unit stride on head_dim and equal pool strides")
    if len({q.dtype, k.dtype, v.dtype, k_buffer.dtype}) != 1:
        raise TypeError("attn_prologue: q, k, v and the pools share a dtype")
    if q_norm_weight.dtype != k_norm_weight.dtype or q_norm_weight.dtype not in (q.dtype,
                                                                                torch.float32):
        raise TypeError("attn_prologue: norm weights are float32 or of the activation dtype")
    if q_norm_weight.numel() != d or k_norm_weight.numel() != d:
        raise ValueError("norm weights must have head_dim entries")
    if inv_freq.dtype != torch.float32 or inv_freq.dim() != 1 or not inv_freq.is_contiguous():
        raise TypeError("inv_freq must be a contiguous float32 vector")
    pos = _i64(positions, "positions")
    if pos.dim() == 1:
        rows, pstride = 1, 0
        if pos.shape[0] != t:
            raise ValueError("positions must have one entry per token")
    elif pos.dim() == 2 and pos.shape[0] == 3 and pos.shape[1] == t:
        if pos.stride(1) != 1:
            pos = pos.contiguous()
        rows, pstride = 3, pos.stride(0)
    else:
        raise ValueError(f"positions must be [T] or [3, T], got {tuple(pos.shape)}")
    loc = _i64(out_cache_loc, "out_cache_loc")
    if loc.numel() != t:
        raise ValueError("out_cache_loc must have one entry per token")
    if q_out is None:
        q_out = torch.empty((t, hq, d), dtype=q.dtype, device=q.device)
    qw, kw = q_norm_weight.contiguous(), k_norm_weight.contiguous()
    a = C.AttnPrologueArgs(
        q=q.data_ptr(), q_stride_tok=q.stride(0), q_stride_head=q.stride(1),
        k=k.data_ptr(), k_stride_tok=k.stride(0), k_stride_head=k.stride(1),
        v=v.data_ptr(), v_stride_tok=v.stride(0), v_stride_head=v.stride(1),
        q_norm_weight=qw.data_ptr(), k_norm_weight=kw.data_ptr(),
        positions=pos.data_ptr(), pos_stride=pstride, inv_freq=inv_freq.data_ptr(),
        q_out=q_out.data_ptr(), q_out_stride_tok=q_out.stride(0),
        q_out_stride_head=q_out.stride(1),
        k_buffer=k_buffer.data_ptr(), v_buffer=v_buffer.data_ptr(),
        buf_stride_slot=k_buffer.stride(0), buf_stride_head=k_buffer.stride(1),
        num_slots=k_buffer.shape[0], out_cache_loc=loc.data_ptr(), num_tokens=t,
        eps=float(eps), pos_rows=rows, mrope_section=(ctypes.c_int32 * 3)(*mrope_section),
        mrope_interleaved=int(bool(mrope_interleaved)), rotary_dim=2 * inv_freq.numel(),
        num_q_heads=hq, num_kv_heads=k.shape[1], head_dim=d, dtype=_dtype(q),
        norm_weight_dtype=_dtype(qw), err=_ptr(err))
    with torch.cuda.device(dev):
        C.check("tf_attn_prologue", C.load().tf_attn_prologue(ctypes.byref(a), _stream(dev)))
    del pos, loc, qw, kw
    return q_out


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
    dev = _need_cuda(q, k_buffer, v_buffer, req_to_token, req_pool_indices, seq_lens, gate)
    if out is None:
        out = torch.empty_like(q)
    args, keep = _paged_args(q, k_buffer, v_buffer, req_to_token, req_pool_indices, seq_lens,
                             None, scale, gate, gate_mode, out, max_seq_len, 1, slot_mode, err)
    lib = C.load()
    with torch.cuda.device(dev):
        nbytes = lib.tf_paged_decode_workspace_size(ctypes.byref(args))
        ws = workspace(dev, nbytes) if nbytes else None
        C.check("tf_paged_decode_attn",
                lib.tf_paged_decode_attn(ctypes.byref(args), _ptr(ws), nbytes, _stream(dev)))
    del keep
    return out


def paged_extend(q: torch.Tensor, k_buffer: torch.Tensor, v_buffer: torch.Tensor,
                 req_to_token: torch.Tensor, req_pool_indices: torch.Tensor,
                 seq_lens: torch.Tensor, extend_lens: torch.Tensor, scale: float,
                 max_seq_len: int, max_extend_len: int, gate: Optional[torch.Tensor] = None,
                 gate_mode: str = "none", out: Optional[torch.Tensor] = None,
                 slot_mode: str = "clamp", err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Varlen extend over a radix-cached prefix (qwen3_8/full_attention.py:179-213, 244-283):
    query i of request b attends to positions <= seq_len_b - extend_len_b + i.  q is packed
    [T, Hq, D] in request order.  Returns out [T, Hq, D]."""
    dev = _need_cuda(q, k_buffer, v_buffer, req_to_token, req_pool_indices, seq_lens,
                     extend_lens, gate)
    if out is None:
        out = torch.empty_like(q)
    args, keep = _paged_args(q, k_buffer, v_buffer, req_to_token, req_pool_indices, seq_lens,
                             extend_lens, scale, gate, gate_mode, out, max_seq_len,
                             max_extend_len, slot_mode, err)
    lib = C.load()
    with torch.cuda.device(dev):
        nbytes = lib.tf_paged_extend_workspace_size(ctypes.byref(args))
        ws = workspace(dev, nbytes) if nbytes else None
        C.check("tf_paged_extend_attn",
                lib.tf_paged_extend_attn(ctypes.byref(args), _ptr(ws), nbytes, _stream(dev)))
    del keep
    return out


# ---------------------------------------------------------------------------------------------
# a5-a9. Gated DeltaNet
# ---------------------------------------------------------------------------------------------
def _gdn_args(qkv, b, a, conv_weight, conv_bias, A_log, dt_bias, conv_state, ssm_state,
              req_pool_indices, extend_lens, z, norm_weight, norm_eps, out, num_k_heads,
              head_k_dim, head_v_dim, max_extend_len, err):
    t, conv_dim = qkv.shape
    hv = b.shape[1]
    kc = conv_weight.shape[-1]
    if conv_dim != 2 * num_k_heads * head_k_dim + hv * head_v_dim:
        raise ValueError(f"qkv width {conv_dim} != 2*Hk*dk + Hv*dv")
    if conv_state.dim() != 3 or conv_state.shape[1:] != (conv_dim, kc - 1) or \
            conv_state.stride(2) != 1 or conv_state.stride(1) != kc - 1:
        raise ValueError(f"conv_state must be a [slots, {conv_dim}, {kc - 1}] view, channel-major")
    if ssm_state.dim() != 4 or ssm_state.shape[1:] != (hv, head_k_dim, head_v_dim) or \
            ssm_state.dtype != torch.float32 or \
            ssm_state.stride()[1:] != (head_k_dim * head_v_dim, head_v_dim, 1):
        raise ValueError("ssm_state must be a float32 [slots, Hv, dk, dv] view, contiguous per slot")
    if conv_state.shape[0] != ssm_state.shape[0]:
        raise ValueError("conv_state and ssm_state must have the same slots")
    for name, x in (("qkv", qkv), ("b", b), ("a", a), ("out", out)):
        if x.stride(-1) != 1:
            raise ValueError(f"{name} needs unit stride on its last dim")
    if z is not None and z.stride(-1) != 1:
        raise ValueError("z needs unit stride on its last dim")
    cw = conv_weight.reshape(conv_dim, kc)
    if not cw.is_contiguous():
        cw = cw.contiguous()
    dt = qkv.dtype
    for name, x in (("b", b), ("a", a), ("conv_weight", cw), ("A_log", A_log),
                    ("dt_bias", dt_bias), ("conv_state", conv_state), ("out", out)):
        if x.dtype != dt:
            raise TypeError(f"{name} has dtype {x.dtype}, expected {dt} (one model dtype)")
    rpi = _i64(req_pool_indices, "req_pool_indices")
    el = None if extend_lens is None else _i64(extend_lens, "extend_lens")
    A_log_c, dt_bias_c = A_log.contiguous(), dt_bias.contiguous()
    nw = None if norm_weight is None else norm_weight.contiguous()
    bias = None if conv_bias is None else conv_bias.contiguous()
    args = C.GdnArgs(
        qkv=qkv.data_ptr(), qkv_stride_tok=qkv.stride(0), b=b.data_ptr(), b_stride_tok=b.stride(0),
        a=a.data_ptr(), a_stride_tok=a.stride(0), conv_weight=cw.data_ptr(), conv_bias=_ptr(bias),
        A_log=A_log_c.data_ptr(), dt_bias=dt_bias_c.data_ptr(),
        conv_state=conv_state.data_ptr(), conv_stride_slot=conv_state.stride(0),
        ssm_state=ssm_state.data_ptr(), ssm_stride_slot=ssm_state.stride(0),
        num_slots=ssm_state.shape[0], req_pool_indices=rpi.data_ptr(),
        extend_lens=_ptr(el), z=_ptr(z), z_stride_tok=0 if z is None else z.stride(0),
        norm_weight=_ptr(nw), norm_weight_len=0 if nw is None else nw.numel(),
        norm_eps=float(norm_eps), out=out.data_ptr(), out_stride_tok=out.stride(0),
        batch_size=rpi.numel(), num_tokens=t, max_extend_len=int(max_extend_len),
        num_k_heads=num_k_heads, num_v_heads=hv, head_k_dim=head_k_dim, head_v_dim=head_v_dim,
        conv_kernel=kc, dtype=_dtype(qkv), err=_ptr(err))
    return args, (cw, rpi, el, A_log_c, dt_bias_c, nw, bias)


def gdn_decode(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state, req_pool_indices,
               num_k_heads: int, head_k_dim: int, head_v_dim: int, conv_bias=None, z=None,
               norm_weight=None, norm_eps: float = 1e-6, out=None, err=None) -> torch.Tensor:
    """Batched one-token GDN step (qwen3_8/linear_attention.py:244-298) updating conv_state and
    ssm_state in place at the request rows; with z given, the gated RMSNorm of
    qwen3_8/rms_norm_gated.py:26-40 is fused.  Returns out [B, Hv*dv]."""
    dev = _need_cuda(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state,
                     req_pool_indices, z, norm_weight)
    if out is None:
        out = torch.empty((qkv.shape[0], b.shape[1] * head_v_dim), dtype=qkv.dtype, device=dev)
    args, keep = _gdn_args(qkv, b, a, conv_weight, conv_bias, A_log, dt_bias, conv_state,
                           ssm_state, req_pool_indices, None, z, norm_weight, norm_eps, out,
                           num_k_heads, head_k_dim, head_v_dim, 1, err)
    with torch.cuda.device(dev):
        C.check("tf_gdn_decode", C.load().tf_gdn_decode(ctypes.byref(args), _stream(dev)))
    del keep
    return out


def gdn_extend(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state, req_pool_indices,
               extend_lens, num_k_heads: int, head_k_dim: int, head_v_dim: int,
               max_extend_len: int, conv_bias=None, z=None, norm_weight=None,
               norm_eps: float = 1e-6, out=None, err=None) -> torch.Tensor:
    """Varlen GDN over packed tokens of several requests (extend / mixed batches), replacing the
    per-request loop of qwen3_8/linear_attention.py:329-358.  Returns out [T, Hv*dv]."""
    dev = _need_cuda(qkv, b, a, conv_weight, A_log, dt_bias, conv_state, ssm_state,
                     req_pool_indices, extend_lens, z, norm_weight)
    if out is None:
        out = torch.empty((qkv.shape[0], b.shape[1] * head_v_dim), dtype=qkv.dtype, device=dev)
    args, keep = _gdn_args(qkv, b, a, conv_weight, conv_bias, A_log, dt_bias, conv_state,
                           ssm_state, req_pool_indices, extend_lens, z, norm_weight, norm_eps,
                           out, num_k_heads, head_k_dim, head_v_dim, max_extend_len, err)
    lib = C.load()
    with torch.cuda.device(dev):
        nbytes = lib.tf_gdn_extend_workspace_size(ctypes.byref(args))
        ws = workspace(dev, nbytes) if nbytes else None
        C.check("tf_gdn_extend",
                lib.tf_gdn_extend(ctypes.byref(args), _ptr(ws), nbytes, _stream(dev)))
    del keep
    return out


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, head_dim: int,
                  eps: float = 1e-6, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """w * x/rms_head(x) * silu(z) (qwen3_8/rms_norm_gated.py:26-40); x, z [T, H*hd]."""
    dev = _need_cuda(x, z, weight)
    if out is None:
        out = torch.empty_like(x)
    if x.shape != z.shape or x.stride(-1) != 1 or z.stride(-1) != 1 or x.shape[1] % head_dim:
        raise ValueError("gated_rmsnorm: x and z must be [T, H*head_dim] with unit inner stride")
    w = weight.contiguous()
    args = C.GatedRMSNormArgs(
        x=x.data_ptr(), x_stride_tok=x.stride(0), z=z.data_ptr(), z_stride_tok=z.stride(0),
        weight=w.data_ptr(), weight_len=w.numel(), out=out.data_ptr(),
        out_stride_tok=out.stride(0), num_tokens=x.shape[0], num_heads=x.shape[1] // head_dim,
        head_dim=head_dim, eps=float(eps), dtype=_dtype(x))
    with torch.cuda.device(dev):
        C.check("tf_gated_rmsnorm", C.load().tf_gated_rmsnorm(ctypes.byref(args), _stream(dev)))
    return out


# ---------------------------------------------------------------------------------------------
# GDN state-slot snapshots: copies / resets of every linear layer's rows in one launch
# ---------------------------------------------------------------------------------------------
def _slot_rows(pool: Optional[torch.Tensor], name: str):
    """(pointer, layer stride, slot stride, elements per slot, dtype) of a [L, slots, ...] pool."""
    if pool is None:
        return None, 0, 0, 0, C.TF_DTYPE_F32
    if pool.dim() < 2:
        raise ValueError(f"{name} must be [layers, slots, ...], got {tuple(pool.shape)}")
    if pool.numel() and not pool[0, 0].is_contiguous():
        raise ValueError(f"{name}: the rows of one slot in one layer must be contiguous")
    elems = 1
    for d in pool.shape[2:]:
        elems *= d
    return pool.data_ptr(), pool.stride(0), pool.stride(1), elems, _dtype(pool)


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
    n = dst_t.numel()
    if n == 0:
        return
    cp, cl, cs, ce, cd = _slot_rows(conv_state, "conv_state")
    sp, sl, ss, se, sd = _slot_rows(ssm_state, "ssm_state")
    args = C.StateCopyArgs(
        conv_state=cp, conv_stride_layer=cl, conv_stride_slot=cs, conv_slot_elems=ce,
        conv_dtype=cd, ssm_state=sp, ssm_stride_layer=sl, ssm_stride_slot=ss, ssm_slot_elems=se,
        ssm_dtype=sd, num_layers=L, num_slots=S, src_slots=src_t.data_ptr(),
        dst_slots=dst_t.data_ptr(), num_ops=n, err=_ptr(err))
    C.check("tf_state_slots_copy", C.load().tf_state_slots_copy(ctypes.byref(args), _stream(dev)))


# ---------------------------------------------------------------------------------------------
# per-step runtime: req_to_token sync and batched sampling
# ---------------------------------------------------------------------------------------------
def req_to_token_sync(req_to_token: torch.Tensor, segments: torch.Tensor, values: torch.Tensor,
                      err: Optional[torch.Tensor] = None) -> None:
    """req_to_token[row, col:col+len] = values[src:src+len] for every (row, col, len, src) row of
    segments [n, 4] int64 (the incremental sync of ModelRunner._prepare_forward_batch,
    engine/model_runner.py:147-166), one launch."""
    dev = _need_cuda(req_to_token, segments, values)
    if req_to_token.dtype != torch.int64 or req_to_token.dim() != 2 or req_to_token.stride(1) != 1:
        raise ValueError("req_to_token must be a row-major [rows, cols] int64 tensor")
    segments, values = _i64(segments, "segments"), _i64(values, "values")
    if segments.dim() != 2 or segments.shape[1] != 4:
        raise ValueError("segments must be [n, 4] (row, col, len, src)")
    args = C.R2TSyncArgs(
        req_to_token=req_to_token.data_ptr(), r2t_stride=req_to_token.stride(0),
        r2t_rows=req_to_token.shape[0], r2t_cols=req_to_token.shape[1],
        segments=segments.data_ptr(), num_segments=segments.shape[0],
        values=values.data_ptr(), num_values=values.numel(), err=_ptr(err))
    C.check("tf_req_to_token_sync", C.load().tf_req_to_token_sync(ctypes.byref(args), _stream(dev)))


def sample_tokens(logits: torch.Tensor, temperature: torch.Tensor,
                  uniform: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Next token of every row of logits [B, V] (ModelRunner._sample_one,
    engine/model_runner.py:574-578): argmax where temperature <= 1e-5 (or uniform is None), else
    the inverse-CDF draw of softmax(logits / T) at uniform[b] in [0, 1).  Returns int64 [B]."""
    dev = _need_cuda(logits, temperature, uniform, out)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be [B, V] with contiguous rows")
    B, V = logits.shape
    if temperature.dtype != torch.float32 or temperature.numel() != B:
        raise ValueError("temperature must be float32 [B]")
    if uniform is not None and (uniform.dtype != torch.float32 or uniform.numel() != B):
        raise ValueError("uniform must be float32 [B]")
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    args = C.SampleArgs(logits=logits.data_ptr(), logits_stride=logits.stride(0), batch_size=B,
                        vocab_size=V, dtype=_dtype(logits),
                        temperature=temperature.contiguous().data_ptr(), uniform=_ptr(uniform),
                        out=out.data_ptr())
    C.check("tf_sample_tokens", C.load().tf_sample_tokens(ctypes.byref(args), _stream(dev)))
    return out


# ---------------------------------------------------------------------------------------------
# block-FP8 linear
# ---------------------------------------------------------------------------------------------
def fp8_quantize(x2d: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(q [M, K] float8_e4m3fn, x_scale [1] float32) of the dynamic per-tensor activation
    quantization of triton_block_fp8_linear (qwen3_8/fp8_triton.py:124-130), bit-exact."""
    dev = _need_cuda(x2d)
    if x2d.dim() != 2 or x2d.stride(1) != 1:
        raise ValueError("fp8_quantize takes [M, K] with contiguous rows")
    M, K = x2d.shape
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=dev)
    scale = torch.empty(1, dtype=torch.float32, device=dev)
    scratch = torch.empty(4, dtype=torch.int32, device=dev)
    args = C.FP8QuantArgs(x=x2d.data_ptr(), x_stride=x2d.stride(0), M=M, K=K, dtype=_dtype(x2d),
                          q=q.data_ptr(), x_scale=scale.data_ptr(), workspace=scratch.data_ptr())
    with torch.cuda.device(dev):
        C.check("tf_fp8_quantize", C.load().tf_fp8_quantize(ctypes.byref(args), _stream(dev)))
    return q, scale


def fp8_block_gemm(q: torch.Tensor, x_scale: torch.Tensor, weight: torch.Tensor,
                   weight_scale_inv: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                   out_dtype: torch.dtype, block_h: int = 128, block_w: int = 128,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out [M, N] = (q @ weight^T per 128-wide K block * weight_scale_inv[n/bh, k/bw]) * x_scale
    + bias, on the tensor cores (the kernel of qwen3_8/fp8_triton.py:17-98)."""
    dev = _need_cuda(q, x_scale, weight, weight_scale_inv, bias)
    M, K = q.shape
    N = weight.shape[0]
    if weight.shape[1] != K or weight.stride(1) != 1 or q.stride(1) != 1:
        raise ValueError("q [M, K] and weight [N, K] need contiguous rows of the same K")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=dev)
    ws = None
    if weight_scale_inv is not None:
        ws = weight_scale_inv if weight_scale_inv.dtype == torch.float32 else weight_scale_inv.float()
    args = C.FP8GemmArgs(
        q=q.data_ptr(), q_stride=q.stride(0), x_scale=x_scale.data_ptr(),
        w=weight.data_ptr(), w_stride=weight.stride(0),
        w_scale=_ptr(ws), ws_stride_n=ws.stride(0) if ws is not None else 0,
        ws_stride_k=ws.stride(1) if ws is not None else 0, block_h=block_h, block_w=block_w,
        bias=_ptr(bias), bias_dtype=_dtype(bias) if bias is not None else 0,
        out=out.data_ptr(), out_stride=out.stride(0), out_dtype=_dtype(out), M=M, N=N, K=K)
    with torch.cuda.device(dev):
        C.check("tf_fp8_block_gemm", C.load().tf_fp8_block_gemm(ctypes.byref(args), _stream(dev)))
    return out


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
