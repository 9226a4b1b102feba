"""The drop-in boundary on CPU: the module surface the reference's callers see is unchanged.

* the stand-alone layers (tokenfactory_b200.layers) have the reference classes' state_dict keys and
  shapes, head split, and forward signatures;
* hybrid_attention.install() swaps the classes the reference's decoder layer instantiates, keeps
  their state_dict, and uninstall() restores them;
* the mixins override exactly the reference's hot-path methods.
"""

import inspect

import pytest
import torch

from tests.golden import cases as C


def _cfg(ref_cfg_cls, tp_size=1, tp_rank=0):
    m = C.MODULE_DIMS
    return ref_cfg_cls(hidden_size=m["hidden"], intermediate_size=64, num_hidden_layers=4,
                       layer_types=["linear_attention"] * 3 + ["full_attention"],
                       num_attention_heads=m["hq"], num_key_value_heads=m["hkv"], head_dim=m["d"],
                       linear_num_key_heads=m["nk"], linear_num_value_heads=m["nv"],
                       linear_key_head_dim=m["dk"], linear_value_head_dim=m["dv"],
                       tp_size=tp_size, tp_rank=tp_rank)


def _params(fn):
    """Parameter names, kinds and defaults of a callable (annotations ignored)."""
    return [(n, p.kind, p.default) for n, p in inspect.signature(fn).parameters.items()]


def _shapes(mod):
    return {k: tuple(v.shape) for k, v in mod.state_dict().items()}


@pytest.mark.parametrize("tp", [1, 2])
def test_layers_match_reference_state_dict_and_head_split(reference_root, tp):
    from qwen3_8 import Qwen3_8Config
    from qwen3_8.full_attention import Qwen3_8FullAttention as RefFull
    from qwen3_8.linear_attention import Qwen3_8LinearAttention as RefLin

    from tokenfactory_b200 import layers

    cfg = _cfg(Qwen3_8Config, tp_size=tp, tp_rank=tp - 1)
    for ref_cls, ours_cls in ((RefFull, layers.Qwen3_8FullAttention),
                              (RefLin, layers.Qwen3_8LinearAttention)):
        ref, ours = ref_cls(cfg, 0), ours_cls(cfg, 0)
        assert _shapes(ours) == _shapes(ref), ref_cls.__name__
        assert _params(ours.forward) == _params(ref.forward)
    rf, of = RefFull(cfg, 3), layers.Qwen3_8FullAttention(cfg, 3)
    assert (of.num_heads, of.num_kv_heads, of.num_queries_per_kv) == \
        (rf.num_heads, rf.num_kv_heads, rf.num_queries_per_kv)
    rl, ol = RefLin(cfg, 0), layers.Qwen3_8LinearAttention(cfg, 0)
    assert (ol.num_k_heads, ol.num_v_heads, ol.conv_dim) == (rl.num_k_heads, rl.num_v_heads,
                                                              rl.conv_dim)


def test_install_patches_decoder_layer_and_keeps_state_dict(reference_root):
    import qwen3_8
    from qwen3_8 import Qwen3_8Config, decoder_layer

    from tokenfactory_b200 import hybrid_attention as HA

    ref_full = qwen3_8.full_attention.Qwen3_8FullAttention
    ref_lin = qwen3_8.linear_attention.Qwen3_8LinearAttention
    cfg = _cfg(Qwen3_8Config)
    before = {i: _shapes(decoder_layer.Qwen3_8DecoderLayer(cfg, i)) for i in (0, 3)}
    try:
        full_cls, lin_cls = HA.install()
        again = HA.install()  # idempotent: patches from the saved reference classes
        assert issubclass(again[0], ref_full) and issubclass(again[1], ref_lin)
        full_cls, lin_cls = again
        assert issubclass(full_cls, ref_full) and issubclass(full_cls, HA.FullAttentionHotPath)
        assert issubclass(lin_cls, ref_lin) and issubclass(lin_cls, HA.LinearAttentionHotPath)
        layer3 = decoder_layer.Qwen3_8DecoderLayer(cfg, 3)
        layer0 = decoder_layer.Qwen3_8DecoderLayer(cfg, 0)
        assert isinstance(layer3.self_attn, HA.FullAttentionHotPath)
        assert isinstance(layer0.linear_attn, HA.LinearAttentionHotPath)
        assert _shapes(layer3) == before[3] and _shapes(layer0) == before[0]
        # the overridden methods are the reference's hot-path methods, same signatures
        for meth in ("forward", "_slot_based_attention"):
            assert getattr(full_cls, meth) is getattr(HA.FullAttentionHotPath, meth)
            assert _params(getattr(full_cls, meth)) == _params(getattr(ref_full, meth))
        for meth in ("forward", "_batched_decode_step"):
            assert getattr(lin_cls, meth) is getattr(HA.LinearAttentionHotPath, meth)
            assert _params(getattr(lin_cls, meth)) == _params(getattr(ref_lin, meth))
        # the rest of the reference class (weight loading for TP) is inherited untouched
        assert full_cls.load_tp_from_full_layer is ref_full.load_tp_from_full_layer
    finally:
        HA.uninstall()
    assert qwen3_8.full_attention.Qwen3_8FullAttention is ref_full
    assert decoder_layer.Qwen3_8LinearAttention is ref_lin


def test_hot_path_refuses_cpu_tensors():
    """No CPU fallback: the kernels reject host tensors with a clear error."""
    from tokenfactory_b200 import ops
    q = torch.zeros((1, 8, 64), dtype=torch.bfloat16)
    kb = torch.zeros((4, 1, 64), dtype=torch.bfloat16)
    idx = torch.zeros(1, dtype=torch.int64)
    with pytest.raises(ValueError, match="CUDA"):
        ops.paged_decode(q, kb, kb, torch.zeros((1, 4), dtype=torch.int64), idx, idx + 1, 0.125, 1)
