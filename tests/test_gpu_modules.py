"""Whole-layer parity on the GPU: the stand-alone drop-in layers (same parameter names as the
reference) loaded with the reference's weights, run on a mixed / decode / single-request batch,
against the outputs the reference's own forward produced (tests/golden/make_golden.py):
qwen3_8/full_attention.py:112-161 and qwen3_8/linear_attention.py:300-364, including the
projections, q/k norms, RoPE, pool writes, GDN states and output gates."""

import numpy as np
import pytest

from oracle import bf16 as BF
from tests.golden import cases as C
from tests.golden.load import module_case
from tests.helpers import to_numpy, values

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


class _Pool:
    def __init__(self, k=None, v=None, c=None, s=None):
        self.k, self.v, self.c, self.s = k, v, c, s

    def get_full_kv_buffers(self, layer_idx):
        return self.k, self.v

    def get_linear_states(self, layer_idx):
        return self.c, self.s


def _cfg():
    from tokenfactory_b200.layers import AttentionConfig
    m = C.MODULE_DIMS
    return AttentionConfig(hidden_size=m["hidden"], num_attention_heads=m["hq"],
                           num_key_value_heads=m["hkv"], head_dim=m["d"],
                           linear_num_key_heads=m["nk"], linear_num_value_heads=m["nv"],
                           linear_key_head_dim=m["dk"], linear_value_head_dim=m["dv"],
                           linear_conv_kernel_dim=m["kc"])


def _close(got, ref, dtype, what, tol_f32=2e-4, tol_bf16=(3e-2, 3e-3)):
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    d = np.abs(got - ref)
    scale = max(1.0, np.abs(ref).max())
    if dtype == "f32":
        assert d.max() <= tol_f32 * scale, f"{what}: max {d.max():.3g}"
    else:
        assert d.max() <= tol_bf16[0] * scale, f"{what}: max {d.max():.3g}"
        assert d.mean() <= tol_bf16[1] * scale, f"{what}: mean {d.mean():.3g}"


@pytest.mark.parametrize("name", sorted(C.MODULE_CASES))
def test_layer_forward_matches_reference(name):
    from tokenfactory_b200 import ForwardBatch, layers
    spec, w, inp, gold = module_case(name)
    dt = spec["dtype"]
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    dev = "cuda"
    cls = layers.Qwen3_8FullAttention if spec["kind"] == "full" else layers.Qwen3_8LinearAttention
    mod = cls(_cfg(), 3 if spec["kind"] == "full" else 0)
    missing = mod.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()}, strict=False)
    assert not missing.unexpected_keys
    mod = mod.eval().to(device=dev, dtype=tdt)
    hidden = torch.from_numpy(inp["hidden"]).to(dev, tdt)
    ext = spec["ext"]
    T = int(sum(ext))
    i64 = lambda k: torch.from_numpy(inp[k]).to(dev)  # noqa: E731
    with torch.inference_mode():
        if spec["kind"] == "full":
            kb = torch.from_numpy(inp["k_buf"]).to(dev, tdt)
            vb = torch.from_numpy(inp["v_buf"]).to(dev, tdt)
            fb = ForwardBatch(batch_size=len(ext), req_pool_indices=i64("req_pool_indices"),
                              seq_lens=i64("seq_lens"),
                              prefix_lens=i64("seq_lens") - i64("extend_lens"),
                              extend_lens=list(ext), out_cache_loc=i64("out_cache_loc"),
                              req_to_token=i64("req_to_token"), is_prefill=max(ext) > 1)
            y = mod(hidden, i64("positions"), _Pool(kb, vb), fb)
            loc = i64("out_cache_loc")
            _close(values(kb[loc], dt), BF.as_f32(gold["k_rows"], dt), dt, f"{name} k rows")
            _close(values(vb[loc], dt), BF.as_f32(gold["v_rows"], dt), dt, f"{name} v rows")
        else:
            cs = torch.from_numpy(inp["conv_state"]).to(dev, tdt)
            ss = torch.from_numpy(inp["ssm_state"]).to(dev)
            fb = ForwardBatch(batch_size=len(ext), req_pool_indices=i64("req_pool_indices"),
                              seq_lens=i64("extend_lens") + 5,
                              prefix_lens=torch.full((len(ext),), 5, dtype=torch.long, device=dev),
                              extend_lens=list(ext),
                              out_cache_loc=torch.zeros(T, dtype=torch.long, device=dev),
                              req_to_token=torch.zeros((1, 1), dtype=torch.long, device=dev),
                              is_prefill=max(ext) > 1)
            y = mod(hidden, _Pool(c=cs, s=ss), fb)
            _close(values(cs, dt), BF.as_f32(gold["conv_state"], dt), dt, f"{name} conv state")
            _close(to_numpy(ss), gold["ssm_state"], "f32", f"{name} ssm state", tol_f32=2e-3)
        torch.cuda.synchronize()
    _close(values(y, dt), BF.as_f32(gold["out"], dt), dt, f"{name} output")
