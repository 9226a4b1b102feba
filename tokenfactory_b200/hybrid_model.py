"""A compact Qwen3.8 hybrid decoder around the drop-in attention layers.

The reference's model (qwen3_8/causal_lm.py:14-151, decoder_layer.py:13-81, mlp.py:9-54,
rms_norm.py:5-24, hybrid_cache_pool.py:14-113) is plain Python that runs above the hot path and
stays unchanged when the drop-ins are installed into it.  Where the reference package is not
available (a GPU box that only has this repository) this module assembles the same model from the
same pieces so that whole decode/extend steps can run through the kernels:

* ``HybridForCausalLM``: embed_tokens -> layers (pre-norm attention block, pre-norm SwiGLU MLP
  block) -> norm -> lm_head on each request's last token, with the reference's state-dict names
  (``model.language_model.layers.{i}.linear_attn.in_proj_qkv.weight`` ...), so a reference
  state_dict loads into it; its attention layers are ``layers.Qwen3_8FullAttention`` /
  ``layers.Qwen3_8LinearAttention`` (the B200 hot path).
* ``HybridCachePool``: the K/V pool and the GDN state pool in the reference's layouts
  (k_buffer [n_full, slots, Hkv, D]; conv_state [n_lin, slots, conv_dim, K-1];
  ssm_state [n_lin, slots, Hv, dk, dv] fp32) with ``get_full_kv_buffers`` /
  ``get_linear_states``.

Tensor parallelism follows the reference's Megatron split: attention heads as in ``layers``,
gate/up projections by output rows, down projection by input columns, one all-reduce after each
row-parallel projection (``set_all_reduce_fn`` or torch.distributed).
"""

from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layers import (AttentionConfig, Qwen3_8FullAttention, Qwen3_8LinearAttention, RMSNorm,
                     RowParallelLinear)


@dataclass
class HybridConfig(AttentionConfig):
    """AttentionConfig plus the model-level fields of qwen3_8/config.py:15-75."""

    vocab_size: int = 248320
    intermediate_size: int = 17408
    num_hidden_layers: int = 64
    layer_types: List[str] = field(default_factory=list)
    tie_word_embeddings: bool = False
    output_gate_mode: str = "silu"  # "silu" is the reference's line; "sigmoid" the Qwen3-Next gate

    def __post_init__(self) -> None:
        if not self.layer_types:  # every 4th layer full attention (qwen3_8/config.py:68-75)
            self.layer_types = ["full_attention" if (i + 1) % 4 == 0 else "linear_attention"
                                for i in range(self.num_hidden_layers)]


class HybridMLP(nn.Module):
    """down_proj(silu(gate_proj(x)) * up_proj(x)) (qwen3_8/mlp.py:53-54), column / row split."""

    def __init__(self, config: HybridConfig):
        super().__init__()
        tp = config.tp_size
        assert config.intermediate_size % tp == 0
        inter = config.intermediate_size // tp
        self.gate_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.down_proj = RowParallelLinear(inter, config.hidden_size, False, tp)

    @torch.no_grad()
    def load_tp_from_full_mlp(self, full: "HybridMLP", rank: int) -> None:
        n = self.gate_proj.weight.shape[0]
        rows = slice(rank * n, (rank + 1) * n)
        self.gate_proj.weight.copy_(full.gate_proj.weight[rows])
        self.up_proj.weight.copy_(full.up_proj.weight[rows])
        self.down_proj.weight.copy_(full.down_proj.weight[:, rows])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class HybridDecoderLayer(nn.Module):
    """Pre-norm attention block then pre-norm MLP block (qwen3_8/decoder_layer.py:57-81)."""

    def __init__(self, config: HybridConfig, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.layer_type = config.layer_types[layer_idx]
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        if self.layer_type == "full_attention":
            self.self_attn = Qwen3_8FullAttention(config, layer_idx)
            self.self_attn.output_gate_mode = config.output_gate_mode
        elif self.layer_type == "linear_attention":
            self.linear_attn = Qwen3_8LinearAttention(config, layer_idx)
        else:
            raise ValueError(f"unknown layer_type {self.layer_type}")
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.mlp = HybridMLP(config)

    def attention(self, normed, positions, cache_pool, forward_batch):
        if self.layer_type == "full_attention":
            return self.self_attn(normed, positions, cache_pool, forward_batch)
        return self.linear_attn(normed, cache_pool, forward_batch)

    def forward(self, hidden_states, positions, cache_pool, forward_batch):
        h = hidden_states + self.attention(self.input_layernorm(hidden_states), positions,
                                           cache_pool, forward_batch)
        return h + self.mlp(self.post_attention_layernorm(h))


class _TextModel(nn.Module):
    def __init__(self, config: HybridConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([HybridDecoderLayer(config, i)
                                     for i in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)


class _ModelWrapper(nn.Module):
    def __init__(self, config: HybridConfig):
        super().__init__()
        self.language_model = _TextModel(config)


class HybridForCausalLM(nn.Module):
    """Qwen3_8ForCausalLM's forward (qwen3_8/causal_lm.py:117-151) on the drop-in layers:
    logits of each request's last token of the step."""

    def __init__(self, config: HybridConfig):
        super().__init__()
        self.config = config
        self.model = _ModelWrapper(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.language_model.embed_tokens.weight

    @property
    def layers(self) -> nn.ModuleList:
        return self.model.language_model.layers

    def set_all_reduce_fn(self, fn: Optional[Callable[[torch.Tensor], torch.Tensor]]) -> None:
        for m in self.modules():
            if isinstance(m, RowParallelLinear):
                m.all_reduce_fn = fn

    @torch.no_grad()
    def load_tp_from_full_model(self, full: "HybridForCausalLM") -> None:
        """This rank's shard of a tp_size=1 model (qwen3_8/causal_lm.py:96-115)."""
        lm = self.model.language_model
        src = full.model.language_model
        lm.embed_tokens.weight.copy_(src.embed_tokens.weight)
        lm.norm.weight.copy_(src.norm.weight)
        self.lm_head.weight.copy_(full.lm_head.weight)
        for mine, theirs in zip(lm.layers, src.layers):
            mine.input_layernorm.weight.copy_(theirs.input_layernorm.weight)
            mine.post_attention_layernorm.weight.copy_(theirs.post_attention_layernorm.weight)
            attn = mine.self_attn if mine.layer_type == "full_attention" else mine.linear_attn
            attn.load_tp_from_full_layer(theirs.self_attn if mine.layer_type == "full_attention"
                                         else theirs.linear_attn)
            mine.mlp.load_tp_from_full_mlp(theirs.mlp, self.config.tp_rank)

    def hidden(self, input_ids, positions, cache_pool, forward_batch,
               attn_timer: Optional[Callable] = None) -> torch.Tensor:
        """Final hidden states of every token (before the top norm).  ``attn_timer(layer, fn)``,
        when given, wraps each layer's attention call (for timing the hot path)."""
        lm = self.model.language_model
        h = lm.embed_tokens(input_ids)
        for layer in lm.layers:
            if attn_timer is None:
                h = layer(h, positions, cache_pool, forward_batch)
                continue
            normed = layer.input_layernorm(h)
            h = h + attn_timer(layer, lambda: layer.attention(normed, positions, cache_pool,
                                                              forward_batch))
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        return h

    @torch.inference_mode()
    def forward(self, input_ids, positions, cache_pool, forward_batch,
                attn_timer: Optional[Callable] = None) -> torch.Tensor:
        h = self.hidden(input_ids, positions, cache_pool, forward_batch, attn_timer)
        ext = forward_batch.extend_lens_tensor
        if ext is None:
            ext = torch.tensor(forward_batch.extend_lens, dtype=torch.long, device=h.device)
        last = torch.cumsum(ext, dim=0) - 1
        return self.lm_head(self.model.language_model.norm(h[last]))


class HybridCachePool:
    """K/V and GDN state pools of one rank in the reference's layouts
    (qwen3_8/hybrid_cache_pool.py:14-113, req_to_state_pool.py:34-108).  GDN state slots
    [0, max_reqs) are the working zone, [max_reqs, max_reqs + max_snapshots) the snapshots."""

    def __init__(self, config: HybridConfig, max_total_tokens: int, max_reqs: int,
                 max_snapshots: int = 0, dtype=torch.bfloat16, device="cuda"):
        types = config.layer_types
        self.full_layers = [i for i, t in enumerate(types) if t == "full_attention"]
        self.linear_layers = [i for i, t in enumerate(types) if t == "linear_attention"]
        self.full_map = {l: j for j, l in enumerate(self.full_layers)}
        self.linear_map = {l: j for j, l in enumerate(self.linear_layers)}
        tp = config.tp_size
        hkv = max(1, config.num_key_value_heads // tp)
        d = config.head_dim
        self.k_buffer = torch.zeros((len(self.full_layers), max_total_tokens, hkv, d), dtype=dtype,
                                    device=device)
        self.v_buffer = torch.zeros_like(self.k_buffer)
        nk = config.linear_num_key_heads // tp
        nv = config.linear_num_value_heads // tp
        dk, dv = config.linear_key_head_dim, config.linear_value_head_dim
        conv_dim = 2 * nk * dk + nv * dv
        slots = max_reqs + max_snapshots
        kc = config.linear_conv_kernel_dim
        self.conv_state = torch.zeros((len(self.linear_layers), slots, conv_dim, kc - 1),
                                      dtype=dtype, device=device)
        self.ssm_state = torch.zeros((len(self.linear_layers), slots, nv, dk, dv),
                                     dtype=torch.float32, device=device)

    def get_full_kv_buffers(self, layer_idx: int):
        j = self.full_map[layer_idx]
        return self.k_buffer[j], self.v_buffer[j]

    def get_linear_states(self, layer_idx: int):
        j = self.linear_map[layer_idx]
        return self.conv_state[j], self.ssm_state[j]
