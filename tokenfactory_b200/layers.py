"""Stand-alone attention layers with the reference's module surface, running the B200 hot path.

``Qwen3_8FullAttention`` and ``Qwen3_8LinearAttention`` here have the constructor
``(config, layer_idx)``, the forward signatures, the sub-module and parameter names and the
tensor-parallel head split of qwen3_8/full_attention.py:25-110 and qwen3_8/linear_attention.py:29-131,
so a reference state_dict loads into them and they plug into the reference's decoder layer.  The
projections are plain linear layers (the FP8 path of the reference is outside the hot path), the
q/k RMSNorm and partial RoPE restate qwen3_8/rms_norm.py and qwen3_8/rotary_embedding.py in torch;
the hot path itself comes from the mixins of ``hybrid_attention``.  Use these where the reference
package is not installed; with it installed, ``hybrid_attention.install()`` patches the reference
classes instead.
"""

from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .hybrid_attention import FullAttentionHotPath, LinearAttentionHotPath
from .tp import gdn_conv_channels, head_shard


@dataclass
class AttentionConfig:
    """The configuration fields the attention layers read, with the reference's names and
    defaults (qwen3_8/config.py:15-66).  The reference's Qwen3_8Config works as well."""

    hidden_size: int = 5120
    rms_norm_eps: float = 1e-6
    num_attention_heads: int = 24
    num_key_value_heads: int = 4
    head_dim: int = 256
    attention_bias: bool = False
    attn_output_gate: bool = True
    partial_rotary_factor: float = 0.25
    rope_theta: float = 10000000.0
    mrope_interleaved: bool = True
    mrope_section: List[int] = field(default_factory=lambda: [11, 11, 10])
    linear_conv_kernel_dim: int = 4
    linear_key_head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 48
    linear_value_head_dim: int = 128
    tp_size: int = 1
    tp_rank: int = 0


class RMSNorm(nn.Module):
    """w * x / rms(x) in fp32, cast back (qwen3_8/rms_norm.py:19-24)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        xn = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return (self.weight.float() * xn).to(x.dtype)


class RMSNormGated(nn.Module):
    """Per-head gated RMSNorm parameters (qwen3_8/rms_norm_gated.py:12-40).  The hot path fuses
    this norm into the GDN kernels; forward() is kept for callers that use it on its own."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, head_dim: Optional[int] = None):
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = eps
        self.head_dim = head_dim
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        from . import ops
        hd = self.head_dim or x.shape[-1]
        return ops.gated_rmsnorm(x, gate, self.weight, hd, self.eps)


class PartialRotaryEmbedding(nn.Module):
    """RoPE on the first head_dim*partial_rotary_factor dims, rotate_half convention, 1-D positions
    or interleaved / sectioned M-RoPE positions [3, T] (qwen3_8/rotary_embedding.py:13-95)."""

    def __init__(self, head_dim: int = 256, partial_rotary_factor: float = 0.25,
                 rope_theta: float = 10000000.0, mrope_section: Optional[List[int]] = None,
                 mrope_interleaved: bool = True):
        super().__init__()
        self.head_dim = head_dim
        self.rotary_dim = int(head_dim * partial_rotary_factor)
        self.mrope_section = mrope_section or [11, 11, 10]
        self.mrope_interleaved = mrope_interleaved
        inv = 1.0 / (rope_theta ** (torch.arange(0, self.rotary_dim, 2, dtype=torch.float32)
                                    / self.rotary_dim))
        self.register_buffer("inv_freq", inv, persistent=False)

    def _cos_sin(self, positions: torch.Tensor, dtype: torch.dtype):
        if positions.ndim == 1:
            freqs = torch.outer(positions.float(), self.inv_freq)
        else:
            f3 = torch.einsum("cn,d->cnd", positions.float(), self.inv_freq)
            if self.mrope_interleaved:
                freqs = f3[0].clone()
                for i in (1, 2):
                    lim = self.mrope_section[i] * 3
                    freqs[:, i:lim:3] = f3[i, :, i:lim:3]
            else:
                freqs = torch.cat([c[i] for i, c in enumerate(f3.split(self.mrope_section, -1))],
                                  dim=-1)
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().unsqueeze(1).to(dtype), emb.sin().unsqueeze(1).to(dtype)

    @staticmethod
    def _rotate_half(x: torch.Tensor) -> torch.Tensor:
        h = x.shape[-1] // 2
        return torch.cat((-x[..., h:], x[..., :h]), dim=-1)

    def forward(self, q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor):
        cos, sin = self._cos_sin(positions, q.dtype)
        r = self.rotary_dim
        qr = q[..., :r] * cos + self._rotate_half(q[..., :r]) * sin
        kr = k[..., :r] * cos + self._rotate_half(k[..., :r]) * sin
        return torch.cat((qr, q[..., r:]), dim=-1), torch.cat((kr, k[..., r:]), dim=-1)


class RowParallelLinear(nn.Linear):
    """y = x W^T summed over tensor-parallel ranks by ``all_reduce_fn`` (or torch.distributed),
    as RowParallelFP8Linear does after the hot path (qwen3_8/fp8_linear.py:434-449)."""

    def __init__(self, in_features: int, out_features: int, bias: bool, tp_size: int):
        super().__init__(in_features, out_features, bias=bias)
        self.tp_size = tp_size
        self.all_reduce_fn: Optional[Callable[[torch.Tensor], torch.Tensor]] = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x, self.weight)
        if self.tp_size > 1:
            if self.all_reduce_fn is not None:
                y = self.all_reduce_fn(y)
            else:
                import torch.distributed as dist
                dist.all_reduce(y)
        return y if self.bias is None else y + self.bias


class _FullAttentionModule(nn.Module):
    """Sub-modules and head split of qwen3_8/full_attention.py:25-100."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.tp_size, self.tp_rank = config.tp_size, config.tp_rank
        assert config.num_attention_heads % self.tp_size == 0
        self.hidden_size = config.hidden_size
        self.head_dim = config.head_dim
        self.scaling = self.head_dim ** -0.5
        self.attn_output_gate = config.attn_output_gate
        self.num_heads = config.num_attention_heads // self.tp_size
        if config.num_key_value_heads >= self.tp_size:
            assert config.num_key_value_heads % self.tp_size == 0
            self.num_kv_heads = config.num_key_value_heads // self.tp_size
        else:
            assert self.tp_size % config.num_key_value_heads == 0
            self.num_kv_heads = 1
        self.num_queries_per_kv = self.num_heads // self.num_kv_heads
        qo = self.num_heads * self.head_dim * (2 if self.attn_output_gate else 1)
        kvo = self.num_kv_heads * self.head_dim
        bias = config.attention_bias
        self.q_proj = nn.Linear(self.hidden_size, qo, bias=bias)
        self.k_proj = nn.Linear(self.hidden_size, kvo, bias=bias)
        self.v_proj = nn.Linear(self.hidden_size, kvo, bias=bias)
        self.q_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.rotary_emb = PartialRotaryEmbedding(self.head_dim, config.partial_rotary_factor,
                                                 config.rope_theta, config.mrope_section,
                                                 config.mrope_interleaved)
        self.o_proj = RowParallelLinear(self.num_heads * self.head_dim, self.hidden_size, bias,
                                        self.tp_size)

    @torch.no_grad()
    def load_tp_from_full_layer(self, full_layer) -> None:
        """Take this rank's heads from a tp_size=1 layer (qwen3_8/full_attention.py:103-110)."""
        c = self.config
        sh = head_shard(c.num_attention_heads, c.num_key_value_heads, self.tp_size, self.tp_size,
                        self.tp_rank, self.tp_size)
        d, qw = self.head_dim, (2 if self.attn_output_gate else 1) * self.head_dim
        self.q_proj.weight.copy_(full_layer.q_proj.weight[sh.q_heads.start * qw:sh.q_heads.stop * qw])
        kv = slice(sh.kv_heads.start * d, sh.kv_heads.stop * d)
        self.k_proj.weight.copy_(full_layer.k_proj.weight[kv])
        self.v_proj.weight.copy_(full_layer.v_proj.weight[kv])
        self.o_proj.weight.copy_(full_layer.o_proj.weight[:, sh.q_heads.start * d:sh.q_heads.stop * d])
        self.q_norm.weight.copy_(full_layer.q_norm.weight)
        self.k_norm.weight.copy_(full_layer.k_norm.weight)


class _LinearAttentionModule(nn.Module):
    """Sub-modules and head split of qwen3_8/linear_attention.py:29-106."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.tp_size, self.tp_rank = config.tp_size, config.tp_rank
        assert config.linear_num_key_heads % self.tp_size == 0
        assert config.linear_num_value_heads % self.tp_size == 0
        self.hidden_size = config.hidden_size
        self.head_k_dim = config.linear_key_head_dim
        self.head_v_dim = config.linear_value_head_dim
        self.num_k_heads = config.linear_num_key_heads // self.tp_size
        self.num_v_heads = config.linear_num_value_heads // self.tp_size
        self.num_v_per_k = self.num_v_heads // self.num_k_heads
        self.key_dim = self.num_k_heads * self.head_k_dim
        self.value_dim = self.num_v_heads * self.head_v_dim
        self.conv_dim = self.key_dim * 2 + self.value_dim
        self.conv_kernel_size = config.linear_conv_kernel_dim
        self.in_proj_qkv = nn.Linear(self.hidden_size, self.conv_dim, bias=False)
        self.in_proj_z = nn.Linear(self.hidden_size, self.value_dim, bias=False)
        self.in_proj_b = nn.Linear(self.hidden_size, self.num_v_heads, bias=False)
        self.in_proj_a = nn.Linear(self.hidden_size, self.num_v_heads, bias=False)
        self.conv1d = nn.Conv1d(self.conv_dim, self.conv_dim, self.conv_kernel_size,
                                groups=self.conv_dim, padding=self.conv_kernel_size - 1,
                                bias=False)
        self.A_log = nn.Parameter(torch.zeros(self.num_v_heads))
        self.dt_bias = nn.Parameter(torch.ones(self.num_v_heads))
        self.norm = RMSNormGated(self.value_dim, eps=config.rms_norm_eps,
                                 head_dim=self.head_v_dim)
        self.out_proj = RowParallelLinear(self.value_dim, self.hidden_size, False, self.tp_size)

    @torch.no_grad()
    def load_tp_from_full_layer(self, full_layer) -> None:
        """Take this rank's heads and conv channels from a tp_size=1 layer
        (qwen3_8/linear_attention.py:109-131)."""
        c = self.config
        sh = head_shard(self.tp_size, self.tp_size, c.linear_num_key_heads,
                        c.linear_num_value_heads, self.tp_rank, self.tp_size)
        ch = torch.tensor(gdn_conv_channels(sh, self.head_k_dim, self.head_v_dim,
                                            c.linear_num_key_heads), dtype=torch.long)
        self.in_proj_qkv.weight.copy_(full_layer.in_proj_qkv.weight[ch])
        self.conv1d.weight.copy_(full_layer.conv1d.weight[ch])
        vh = slice(sh.v_heads.start, sh.v_heads.stop)
        vd = slice(sh.v_heads.start * self.head_v_dim, sh.v_heads.stop * self.head_v_dim)
        self.in_proj_z.weight.copy_(full_layer.in_proj_z.weight[vd])
        self.in_proj_b.weight.copy_(full_layer.in_proj_b.weight[vh])
        self.in_proj_a.weight.copy_(full_layer.in_proj_a.weight[vh])
        self.A_log.copy_(full_layer.A_log[vh])
        self.dt_bias.copy_(full_layer.dt_bias[vh])
        self.norm.weight.copy_(full_layer.norm.weight[vd])
        self.out_proj.weight.copy_(full_layer.out_proj.weight[:, vd])


class Qwen3_8FullAttention(FullAttentionHotPath, _FullAttentionModule):
    """Full-attention layer (qwen3_8/full_attention.py) whose hot path runs on the B200 kernels."""


class Qwen3_8LinearAttention(LinearAttentionHotPath, _LinearAttentionModule):
    """Gated DeltaNet layer (qwen3_8/linear_attention.py) whose hot path runs on the B200
    kernels."""
