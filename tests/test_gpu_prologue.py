"""Fused attention prologue (q/k RMSNorm + partial (M-)RoPE + KV store) on the GPU against the
golden vectors of the reference's own modules (qwen3_8/rms_norm.py, qwen3_8/rotary_embedding.py,
the pool write of qwen3_8/full_attention.py:147-149) and the CPU oracle.

The v rows are a copy and must match bit for bit.  q and k go through cos/sin and rsqrt, whose
fp32 results on the GPU may differ by an ulp from torch's CPU ones; after the bf16 rounding almost
every element is identical, and the few others differ by one bf16 ulp.
"""

import numpy as np
import pytest

from oracle import attention as OA
from oracle import bf16 as BF
from tests.golden import cases as C
from tests.golden.load import prologue_case
from tests.helpers import to_numpy, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _run(spec, inp, gold, err=None):
    from tokenfactory_b200 import ops
    dt = spec["dtype"]
    d = spec["d"]
    qg = to_torch(inp["qg"], dt)
    q = qg[..., :d] if spec.get("strided") else qg
    kb, vb = to_torch(inp["k_buf"], dt), to_torch(inp["v_buf"], dt)
    sec, inter = spec["mrope"] if spec["mrope"] else ([11, 11, 10], True)
    qo = ops.attn_prologue(q, to_torch(inp["k"], dt), to_torch(inp["v"], dt),
                           to_torch(inp["q_norm_weight"], dt), to_torch(inp["k_norm_weight"], dt),
                           torch.from_numpy(inp["positions"]).cuda(),
                           torch.from_numpy(gold["inv_freq"]).cuda(), kb, vb,
                           torch.from_numpy(inp["out_cache_loc"]).cuda(), eps=C.PROLOGUE_EPS,
                           mrope_section=sec, mrope_interleaved=inter, err=err)
    torch.cuda.synchronize()
    return to_numpy(qo), to_numpy(kb), to_numpy(vb)


def _ulp_close(got, want, dt, what, min_exact=0.99):
    if dt == "bf16":
        g, w = BF.as_f32(got, dt), BF.as_f32(want, dt)
        exact = np.mean(got == want)
        # one bf16 ulp of the larger magnitude
        ulp = np.maximum(np.abs(w), np.abs(g)) * np.float32(2.0 ** -7) + np.float32(1e-30)
        assert np.all(np.abs(g - w) <= ulp), f"{what}: a difference above one bf16 ulp"
        assert exact >= min_exact, f"{what}: only {exact:.4f} of the elements bit-exact"
    else:
        np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-6, err_msg=what)


@pytest.mark.parametrize("name", sorted(C.PROLOGUE_CASES))
def test_prologue_matches_reference_modules(name):
    spec, inp, gold = prologue_case(name)
    qo, kb, vb = _run(spec, inp, gold)
    dt = spec["dtype"]
    np.testing.assert_array_equal(vb, gold["v_buf"])  # the v copy is bit-exact
    _ulp_close(qo, gold["q_out"], dt, f"{name} q_out")
    _ulp_close(kb, gold["k_buf"], dt, f"{name} k rows")
    # and against the oracle restatement (identical to the golden outputs in bf16)
    kb2, vb2 = inp["k_buf"].copy(), inp["v_buf"].copy()
    sec, inter = spec["mrope"] if spec["mrope"] else ([11, 11, 10], True)
    qo2 = OA.attn_prologue(C.prologue_q(inp, spec), inp["k"], inp["v"], inp["q_norm_weight"],
                           inp["k_norm_weight"], inp["positions"], gold["inv_freq"], kb2, vb2,
                           inp["out_cache_loc"], dt, C.PROLOGUE_EPS, sec, inter)
    _ulp_close(qo, qo2, dt, f"{name} q_out vs oracle")


def test_prologue_out_of_range_location_is_recorded_and_skipped():
    spec, inp, gold = prologue_case("pro_bf16_d256")
    inp = dict(inp)
    loc = inp["out_cache_loc"].copy()
    loc[5] = spec["slots"] + 3  # beyond the pool, even after wrapping
    inp["out_cache_loc"] = loc
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _, kb, vb = _run(spec, inp, gold, err=err)
    assert int(err.item()) != 0
    # every other row was written exactly as the reference writes it
    want_v = inp["v_buf"].copy()
    ok = np.arange(spec["t"]) != 5
    want_v[loc[ok]] = inp["v"][ok]
    np.testing.assert_array_equal(vb, want_v)

