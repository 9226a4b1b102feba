"""Drop-in replacement of tokenFactory's hybrid-attention hot path on the module surface.

The reference has no plugin registry: its hot path is the methods of two nn.Modules
(qwen3_8/full_attention.py:112-283, qwen3_8/linear_attention.py:244-364).  This module provides

* ``FullAttentionHotPath`` / ``LinearAttentionHotPath``: mixins that override those methods with
  the same signatures and return values, running the CUDA kernels of ``ops``.  They use only
  attributes both the reference classes and the mirrors in ``layers.py`` define (the projections,
  norms, rotary embedding, head counts), so ``type(name, (Mixin, ReferenceClass), {})`` is a drop-in
  subclass whose state_dict is the reference's;
* ``install()``: patches the reference package so models built afterwards use the drop-ins
  (``qwen3_8.decoder_layer`` instantiates the classes by these names); ``uninstall()`` undoes it;
* functional cores (``full_attention_core``, ``slot_based_attention``, ``linear_attention_core``)
  for callers that hold tensors rather than modules.

The pool tensors, ForwardBatch fields and all module signatures stay as in the reference, so
model_runner, scheduler and radix_tree run unchanged above this boundary.
"""

import importlib
from typing import Dict, Optional, Tuple

import torch

from . import ops

# ---------------------------------------------------------------------------------------------
# functional cores
# ---------------------------------------------------------------------------------------------


def _attend(q: torch.Tensor, k_buf: torch.Tensor, v_buf: torch.Tensor, batch, scaling: float,
            gate: Optional[torch.Tensor], gate_mode: str) -> torch.Tensor:
    """Dispatch of qwen3_8/full_attention.py:174-283 onto the kernels.

    bsz == 1   -> slots read with torch's wrap-around for negative entries (:188);
    all decode -> tf_paged_decode_attn (:232-242);
    otherwise  -> tf_paged_extend_attn (:244-283, varlen, no padded rows).
    """
    bsz = batch.batch_size
    slot_mode = "wrap" if bsz == 1 else "clamp"
    max_seq = int(batch.max_seq_len) if batch.max_seq_len else int(batch.seq_lens.max().item())
    max_ext = int(batch.max_extend_len) if batch.max_extend_len else max(batch.extend_lens)
    if max_ext == 1:
        return ops.paged_decode(q, k_buf, v_buf, batch.req_to_token, batch.req_pool_indices,
                                batch.seq_lens, scaling, max_seq, gate=gate,
                                gate_mode=gate_mode if gate is not None else "none",
                                slot_mode=slot_mode)
    ext = batch.extend_lens_tensor
    if ext is None:
        ext = torch.tensor(batch.extend_lens, dtype=torch.long, device=q.device)
    return ops.paged_extend(q, k_buf, v_buf, batch.req_to_token, batch.req_pool_indices,
                            batch.seq_lens, ext, scaling, max_seq, max_ext, gate=gate,
                            gate_mode=gate_mode if gate is not None else "none",
                            slot_mode=slot_mode)


def slot_based_attention(q: torch.Tensor, layer_k_buffer: torch.Tensor,
                         layer_v_buffer: torch.Tensor, batch, scaling: float) -> torch.Tensor:
    """Same inputs and output as Qwen3_8FullAttention._slot_based_attention
    (qwen3_8/full_attention.py:163-283): q [T, Hq, D] -> attention output [T, Hq, D]."""
    return _attend(q, layer_k_buffer, layer_v_buffer, batch, scaling, None, "none")


def full_attention_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        gate: Optional[torch.Tensor], layer_k_buffer: torch.Tensor,
                        layer_v_buffer: torch.Tensor, batch, scaling: float,
                        gate_mode: str = "silu") -> torch.Tensor:
    """Pool write + attention + output gate: qwen3_8/full_attention.py:146-158.

    q [T, Hq, D] (normed, rotated), k/v [T, Hkv, D], gate [T, Hq, D] view or None.
    Returns [T, Hq*D] ready for o_proj."""
    ops.kv_store(layer_k_buffer, layer_v_buffer, batch.out_cache_loc, k, v)
    out = _attend(q, layer_k_buffer, layer_v_buffer, batch, scaling, gate, gate_mode)
    return out.reshape(q.shape[0], q.shape[1] * q.shape[2])


def linear_attention_core(qkv: torch.Tensor, z: torch.Tensor, b: torch.Tensor, a: torch.Tensor,
                          conv_weight: torch.Tensor, conv_bias: Optional[torch.Tensor],
                          A_log: torch.Tensor, dt_bias: torch.Tensor,
                          norm_weight: Optional[torch.Tensor], norm_eps: float,
                          layer_conv_state: torch.Tensor, layer_ssm_state: torch.Tensor, batch,
                          num_k_heads: int, head_k_dim: int, head_v_dim: int) -> torch.Tensor:
    """GDN between the projections and out_proj: qwen3_8/linear_attention.py:312-363.

    All-decode batches take the fused decode kernel (the reference's :316-326 fast path); any
    other batch takes the varlen extend launch sequence instead of the per-request loop
    (:329-358).  With norm_weight given, the gated RMSNorm (:363) is fused.  Returns [T, Hv*dv]."""
    kw = dict(num_k_heads=num_k_heads, head_k_dim=head_k_dim, head_v_dim=head_v_dim,
              conv_bias=conv_bias, z=z if norm_weight is not None else None,
              norm_weight=norm_weight, norm_eps=norm_eps)
    if all(int(e) == 1 for e in batch.extend_lens):
        return ops.gdn_decode(qkv, b, a, conv_weight, A_log, dt_bias, layer_conv_state,
                              layer_ssm_state, batch.req_pool_indices, **kw)
    ext = batch.extend_lens_tensor
    if ext is None:
        ext = torch.tensor(batch.extend_lens, dtype=torch.long, device=qkv.device)
    max_ext = int(batch.max_extend_len) if batch.max_extend_len else max(batch.extend_lens)
    return ops.gdn_extend(qkv, b, a, conv_weight, A_log, dt_bias, layer_conv_state,
                          layer_ssm_state, batch.req_pool_indices, ext, max_extend_len=max_ext,
                          **kw)


# ---------------------------------------------------------------------------------------------
# module mixins (method-for-method overrides of the reference classes)
# ---------------------------------------------------------------------------------------------


def _prologue_fusable(layer, q: torch.Tensor, positions: torch.Tensor) -> bool:
    """Whether tf_attn_prologue builds this layer's q/k norm + RoPE: equal q/k eps, head_dim
    64/128/256, rotary_dim/2 a multiple of 32 or a power of two below 32, 1-D positions or M-RoPE
    sections that cover rotary_dim/2, norm weights in fp32 or the activation dtype.  Other layers
    run their own modules (torch on the same device) before the fused attention."""
    rot, qn, kn = layer.rotary_emb, layer.q_norm, layer.k_norm
    if not all(hasattr(rot, x) for x in ("inv_freq", "rotary_dim", "mrope_section",
                                         "mrope_interleaved")):
        return False
    if getattr(qn, "eps", None) != getattr(kn, "eps", None) or qn.eps is None:
        return False
    if layer.head_dim not in (64, 128, 256) or rot.inv_freq.dtype != torch.float32:
        return False
    half = rot.rotary_dim // 2
    if rot.rotary_dim % 2 or rot.rotary_dim > layer.head_dim or half < 1 or \
            not (half % 32 == 0 or (half < 32 and half & (half - 1) == 0)):
        return False
    if positions.dim() == 2 and (positions.shape[0] != 3 or sum(rot.mrope_section) != half):
        return False
    if positions.dim() not in (1, 2):
        return False
    return qn.weight.dtype in (q.dtype, torch.float32) and qn.weight.dtype == kn.weight.dtype


class FullAttentionHotPath:
    """Overrides Qwen3_8FullAttention.forward / _slot_based_attention.

    ``output_gate_mode`` selects the gate activation: "silu" is the reference line
    (qwen3_8/full_attention.py:157-158); "sigmoid" is the gate of the Qwen3-Next checkpoints."""

    output_gate_mode = "silu"

    def _slot_based_attention(self, q, layer_k_buffer, layer_v_buffer, batch):
        return slot_based_attention(q, layer_k_buffer, layer_v_buffer, batch, self.scaling)

    def forward(self, hidden_states, positions, cache_pool, forward_batch):
        num_tokens = hidden_states.shape[0]
        d = self.head_dim
        if self.attn_output_gate:
            qg = self.q_proj(hidden_states).view(num_tokens, self.num_heads, 2 * d)
            q, gate = qg[..., :d], qg[..., d:]  # the gate stays a strided view: no copy
        else:
            q = self.q_proj(hidden_states).view(num_tokens, self.num_heads, d)
            gate = None
        k = self.k_proj(hidden_states).view(num_tokens, self.num_kv_heads, d)
        v = self.v_proj(hidden_states).view(num_tokens, self.num_kv_heads, d)
        layer_k_buffer, layer_v_buffer = cache_pool.get_full_kv_buffers(self.layer_idx)
        if _prologue_fusable(self, q, positions):
            # q/k RMSNorm + partial RoPE + pool write in one pass (:142-149)
            rot = self.rotary_emb
            q = ops.attn_prologue(q, k, v, self.q_norm.weight, self.k_norm.weight, positions,
                                  rot.inv_freq, layer_k_buffer, layer_v_buffer,
                                  forward_batch.out_cache_loc, eps=self.q_norm.eps,
                                  mrope_section=tuple(rot.mrope_section),
                                  mrope_interleaved=rot.mrope_interleaved)
            out = _attend(q, layer_k_buffer, layer_v_buffer, forward_batch, self.scaling, gate,
                          self.output_gate_mode).reshape(num_tokens, self.num_heads * d)
            return self.o_proj(out)
        q = self.q_norm(q)
        k = self.k_norm(k)
        q, k = self.rotary_emb(q, k, positions)
        out = full_attention_core(q.contiguous(), k, v.contiguous(), gate, layer_k_buffer,
                                  layer_v_buffer, forward_batch, self.scaling,
                                  self.output_gate_mode)
        return self.o_proj(out)


class LinearAttentionHotPath:
    """Overrides Qwen3_8LinearAttention.forward / _batched_decode_step."""

    def _batched_decode_step(self, qkv, b, a, layer_conv_state, layer_ssm_state, req_indices):
        return ops.gdn_decode(qkv, b, a, self.conv1d.weight, self.A_log, self.dt_bias,
                              layer_conv_state, layer_ssm_state, req_indices,
                              num_k_heads=self.num_k_heads, head_k_dim=self.head_k_dim,
                              head_v_dim=self.head_v_dim, conv_bias=self.conv1d.bias)

    def forward(self, hidden_states, cache_pool, forward_batch):
        qkv = self.in_proj_qkv(hidden_states)
        z = self.in_proj_z(hidden_states)
        b = self.in_proj_b(hidden_states)
        a = self.in_proj_a(hidden_states)
        layer_conv_state, layer_ssm_state = cache_pool.get_linear_states(self.layer_idx)
        norm_head = getattr(self.norm, "head_dim", None)
        fused = norm_head == self.head_v_dim
        out = linear_attention_core(qkv, z, b, a, self.conv1d.weight, self.conv1d.bias,
                                    self.A_log, self.dt_bias,
                                    self.norm.weight if fused else None, self.norm.eps,
                                    layer_conv_state, layer_ssm_state, forward_batch,
                                    self.num_k_heads, self.head_k_dim, self.head_v_dim)
        if not fused:  # a norm over the whole value dim is not fused: run the module itself
            out = self.norm(out, z)
        return self.out_proj(out)


def drop_in(reference_cls: type, mixin: type) -> type:
    """A subclass of the reference class with the hot-path methods replaced."""
    return type(reference_cls.__name__, (mixin, reference_cls),
                {"__module__": __name__, "__doc__": reference_cls.__doc__})


_saved: Dict[Tuple[str, str], type] = {}


def install(package: str = "qwen3_8") -> Tuple[type, type]:
    """Patch the reference package so models built afterwards run the B200 hot path.

    Replaces Qwen3_8FullAttention / Qwen3_8LinearAttention in qwen3_8.full_attention,
    qwen3_8.linear_attention, qwen3_8.decoder_layer (where Qwen3_8DecoderLayer instantiates them)
    and the package namespace.  Returns the two drop-in classes.  Idempotent."""
    fa_mod = importlib.import_module(f"{package}.full_attention")
    la_mod = importlib.import_module(f"{package}.linear_attention")
    dl_mod = importlib.import_module(f"{package}.decoder_layer")
    pkg = importlib.import_module(package)
    fa_ref = _saved.get((package, "full"), fa_mod.Qwen3_8FullAttention)
    la_ref = _saved.get((package, "linear"), la_mod.Qwen3_8LinearAttention)
    _saved[(package, "full")] = fa_ref
    _saved[(package, "linear")] = la_ref
    fa_new = drop_in(fa_ref, FullAttentionHotPath)
    la_new = drop_in(la_ref, LinearAttentionHotPath)
    for mod in (fa_mod, dl_mod, pkg):
        mod.Qwen3_8FullAttention = fa_new
    for mod in (la_mod, dl_mod, pkg):
        mod.Qwen3_8LinearAttention = la_new
    return fa_new, la_new


def uninstall(package: str = "qwen3_8") -> None:
    """Restore the reference classes patched by install()."""
    if (package, "full") not in _saved:
        return
    fa_mod = importlib.import_module(f"{package}.full_attention")
    la_mod = importlib.import_module(f"{package}.linear_attention")
    dl_mod = importlib.import_module(f"{package}.decoder_layer")
    pkg = importlib.import_module(package)
    for mod in (fa_mod, dl_mod, pkg):
        mod.Qwen3_8FullAttention = _saved[(package, "full")]
    for mod in (la_mod, dl_mod, pkg):
        mod.Qwen3_8LinearAttention = _saved[(package, "linear")]
    del _saved[(package, "full")], _saved[(package, "linear")]
