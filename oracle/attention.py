"""Oracle for the paged GQA full-attention hot path (TEST INFRASTRUCTURE; numpy).

Restates qwen3_8/full_attention.py of yz29528/tokenFactory:
  kv_store             - :147-149   layer_k_buffer[out_cache_loc] = k (same for v)
  slot_based_attention - :163-283   the three branches of _slot_based_attention
  output_gate          - :157-158   attn_output * act(gate)
  attn_prologue        - :142-149   q/k RMSNorm (qwen3_8/rms_norm.py:19-24), partial (M-)RoPE
                                    (qwen3_8/rotary_embedding.py:46-95) and the pool write

Arrays: bf16 tensors are uint16 bit patterns (see oracle.bf16); index tensors are int64.
The attention itself is evaluated in float32 from the stored values (the "fp32 evaluation" the
parity tolerances are stated against); rounding to the output dtype is left to the caller.
"""

from typing import Optional, Sequence

import numpy as np

from . import bf16 as _bf


def kv_store(k_buf: np.ndarray, v_buf: np.ndarray, out_cache_loc: np.ndarray,
             k: np.ndarray, v: np.ndarray) -> None:
    """In-place scatter of new K/V rows into the layer's pool (qwen3_8/full_attention.py:147-149).

    numpy fancy assignment has torch's index semantics here: negative locations wrap, and an
    out-of-range location raises IndexError.  With duplicate locations the last row wins.
    """
    loc = np.asarray(out_cache_loc, dtype=np.int64)
    k_buf[loc] = k
    v_buf[loc] = v


def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    m = np.max(scores, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
    p = np.exp(scores - m)
    return p / np.sum(p, axis=-1, keepdims=True)


def _attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, allowed: np.ndarray,
            scale: float) -> np.ndarray:
    """q [E,Hq,D], k/v [L,Hkv,D] float32, allowed [E,L] bool -> [E,Hq,D] float32.

    GQA: query head h reads kv head h // (Hq/Hkv), i.e. torch.repeat_interleave on the head axis
    (qwen3_8/full_attention.py:191-193, 221-227).
    """
    e, hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    qg = q.reshape(e, hkv, g, d)
    scores = np.einsum("ehgd,lhd->hgel", qg, k, optimize=True) * np.float32(scale)
    scores = np.where(allowed[None, None], scores, np.float32(-np.inf)).astype(np.float32)
    p = _softmax_rows(scores)
    out = np.einsum("hgel,lhd->ehgd", p, v, optimize=True)
    return out.reshape(e, hq, d).astype(np.float32)


def slot_based_attention(q: np.ndarray, k_buf: np.ndarray, v_buf: np.ndarray,
                         req_to_token: np.ndarray, req_pool_indices: Sequence[int],
                         seq_lens: Sequence[int], extend_lens: Sequence[int], scale: float,
                         dtype: str = "bf16", max_seq_len: Optional[int] = None,
                         q_chunk: int = 256) -> np.ndarray:
    """Paged attention through req_to_token (qwen3_8/full_attention.py:163-283).

    q [T,Hq,D] and the pools [S,Hkv,D] are stored as `dtype`; returns float32 [T,Hq,D].

    Branches, as in the reference:
      bsz == 1  (:179-213): slots = req_to_token[req, :max_seq_len] WITHOUT clamping (a negative
                entry wraps like torch indexing); causal mask only when ext_len > 1, with query i at
                absolute position seq_len - ext_len + i.
      decode    (:215-242): slots clamped at 0 (:216-218); keys j < seq_len_b.
      extend    (:244-283): keys j <= P_b + i and j < seq_len_b, P_b = seq_len_b - ext_len_b.
                Padded query rows of the reference attend to column 0 and are dropped (:273-274,283);
                only the T real rows exist here.
    """
    qf = _bf.as_f32(q, dtype)
    kb = k_buf
    vb = v_buf
    bsz = len(seq_lens)
    seq_lens = [int(x) for x in seq_lens]
    extend_lens = [int(x) for x in extend_lens]
    req_pool_indices = [int(x) for x in req_pool_indices]
    if max_seq_len is None:
        max_seq_len = max(seq_lens) if seq_lens else 0
    out = np.zeros(qf.shape, dtype=np.float32)
    num_slots = kb.shape[0]
    t0 = 0
    for b in range(bsz):
        ext = extend_lens[b]
        if bsz == 1:
            seq_len = max_seq_len
            slots = np.asarray(req_to_token[req_pool_indices[b], :seq_len], dtype=np.int64)
            slots = np.where(slots < 0, slots + num_slots, slots)
        else:
            seq_len = seq_lens[b]
            slots = np.asarray(req_to_token[req_pool_indices[b], :seq_len], dtype=np.int64)
            slots = np.maximum(slots, 0)
        k = _bf.as_f32(kb[slots], dtype)
        v = _bf.as_f32(vb[slots], dtype)
        prefix = seq_len - ext
        kpos = np.arange(seq_len)
        for c0 in range(0, ext, q_chunk):
            c1 = min(ext, c0 + q_chunk)
            qpos = prefix + np.arange(c0, c1)
            if bsz == 1 and ext == 1:
                allowed = np.ones((c1 - c0, seq_len), dtype=bool)
            else:
                allowed = kpos[None, :] <= qpos[:, None]
            out[t0 + c0:t0 + c1] = _attend(qf[t0 + c0:t0 + c1], k, v, allowed, scale)
        t0 += ext
    return out


def output_gate(attn: np.ndarray, gate: np.ndarray, mode: str, dtype: str) -> np.ndarray:
    """attn * act(gate) with the reference's rounding (qwen3_8/full_attention.py:157-158).

    attn is the attention output already rounded to `dtype` (float32 values); gate is stored as
    `dtype`.  The reference computes F.silu(gate) as a `dtype` tensor, then the product in `dtype`.
    mode: "silu" (the reference line), "sigmoid" (the gate of the benchmark configurations), "none".
    """
    if mode == "none":
        return attn.astype(np.float32)
    g = _bf.as_f32(gate, dtype).astype(np.float32)
    if mode == "silu":
        act = g / (np.float32(1.0) + np.exp(-g))
    elif mode == "sigmoid":
        act = np.float32(1.0) / (np.float32(1.0) + np.exp(-g))
    else:
        raise ValueError(f"unknown gate mode {mode!r}")
    act = _bf.round_to(act.astype(np.float32), dtype)
    return _bf.round_to((attn.astype(np.float32) * act).astype(np.float32), dtype)


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """Qwen3_8RMSNorm.forward (qwen3_8/rms_norm.py:19-24): fp32 inside, one rounding to `dtype`.
    x, weight float32 values; normalises over the last axis."""
    xf = x.astype(np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    xn = xf * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))
    return _bf.round_to((weight.astype(np.float32) * xn).astype(np.float32), dtype)


def rope_cos_sin(positions: np.ndarray, inv_freq: np.ndarray, dtype: str,
                 mrope_section: Sequence[int] = (11, 11, 10), interleaved: bool = True):
    """PartialRotaryEmbedding._compute_cos_sin (qwen3_8/rotary_embedding.py:46-76): cos and sin
    [T, rotary_dim] of positions [T] or [3, T], cast to `dtype` (returned as float32 values)."""
    inv = inv_freq.astype(np.float32)
    pos = np.asarray(positions)
    if pos.ndim == 1:
        freqs = pos.astype(np.float32)[:, None] * inv[None, :]
    else:
        f3 = pos.astype(np.float32)[:, :, None] * inv[None, None, :]
        if interleaved:
            freqs = f3[0].copy()
            for dim_idx in (1, 2):
                limit = mrope_section[dim_idx] * 3
                freqs[:, dim_idx:limit:3] = f3[dim_idx, :, dim_idx:limit:3]
        else:
            edges = np.cumsum([0] + list(mrope_section))
            freqs = np.concatenate([f3[i, :, edges[i]:edges[i + 1]] for i in range(3)], axis=-1)
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float32)
    return _bf.round_to(np.cos(emb), dtype), _bf.round_to(np.sin(emb), dtype)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """PartialRotaryEmbedding.forward on one tensor (qwen3_8/rotary_embedding.py:78-95):
    x [T, H, D] float32 values of `dtype`, cos/sin [T, rotary_dim]; each torch op rounds."""
    rot = cos.shape[-1]
    half = rot // 2
    xr, xp = x[..., :rot], x[..., rot:]
    rh = np.concatenate([-xr[..., half:], xr[..., :half]], axis=-1)
    a = _bf.round_to((xr * cos[:, None, :]).astype(np.float32), dtype)
    b = _bf.round_to((rh * sin[:, None, :]).astype(np.float32), dtype)
    out = _bf.round_to((a + b).astype(np.float32), dtype)
    return np.concatenate([out, xp], axis=-1)


def attn_prologue(q: np.ndarray, k: np.ndarray, v: np.ndarray, q_norm_weight: np.ndarray,
                  k_norm_weight: np.ndarray, positions: np.ndarray, inv_freq: np.ndarray,
                  k_buf: np.ndarray, v_buf: np.ndarray, out_cache_loc: np.ndarray, dtype: str,
                  eps: float = 1e-6, mrope_section: Sequence[int] = (11, 11, 10),
                  interleaved: bool = True) -> np.ndarray:
    """q/k RMSNorm, partial RoPE and the pool write of Qwen3_8FullAttention.forward
    (qwen3_8/full_attention.py:142-149).  Tensors in storage form of `dtype`; the pools are
    updated in place, the rotated q is returned in storage form."""
    qv, kv = _bf.as_f32(q, dtype), _bf.as_f32(k, dtype)
    qn = rms_norm(qv, _bf.as_f32(q_norm_weight, dtype), eps, dtype)
    kn = rms_norm(kv, _bf.as_f32(k_norm_weight, dtype), eps, dtype)
    cos, sin = rope_cos_sin(positions, inv_freq, dtype, mrope_section, interleaved)
    qo = apply_rope(qn, cos, sin, dtype)
    ko = apply_rope(kn, cos, sin, dtype)
    kv_store(k_buf, v_buf, out_cache_loc, _bf.store(ko, dtype), v)
    return _bf.store(qo, dtype)
