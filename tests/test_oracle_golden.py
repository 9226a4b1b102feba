"""Pin the CPU oracle against golden vectors produced by the reference's own functions.

The oracle (oracle/) is the checker of every GPU parity test; here it is checked against
outputs recorded from qwen3_8/full_attention.py and qwen3_8/linear_attention.py themselves
(tests/golden/make_golden.py).  Runs on CPU.
"""

import numpy as np
import pytest

from oracle import attention as OA
from oracle import bf16 as BF
from oracle import gdn as OG
from tests.golden import cases as C
from tests.golden.load import attention_case, gdn_case


def _vals(x, dtype):
    return BF.as_f32(x, dtype)


@pytest.mark.parametrize("name", sorted(C.ATTN_CASES))
def test_attention_oracle_matches_reference(name):
    spec, inp, gold = attention_case(name)
    dt = spec["dtype"]
    out = OA.slot_based_attention(inp["q"], inp["k_buf"], inp["v_buf"], inp["req_to_token"],
                                  inp["req_pool_indices"], inp["seq_lens"], inp["extend_lens"],
                                  spec["d"] ** -0.5, dt)
    ref = _vals(gold["out"], dt)
    if dt == "f32":
        np.testing.assert_allclose(out, ref, rtol=2e-5, atol=2e-6)
    else:
        # the reference runs SDPA on bf16 tensors (bf16 mask and intermediate roundings): the fp32
        # oracle rounded to bf16 stays within a couple of bf16 ulps of it
        diff = np.abs(BF.round_f32(out) - ref)
        assert diff.max() <= 2 ** -6 * max(1.0, np.abs(ref).max()), diff.max()
        assert diff.mean() < 1e-3
    # output gate: reference silu line and the sigmoid variant
    t = out.shape[0]
    attn_r = BF.round_to(out, dt).reshape(t, -1)
    for mode in ("silu", "sigmoid"):
        key = f"out_{mode}"
        if key not in gold:
            continue
        g = OA.output_gate(attn_r, inp["gate"].reshape(t, -1), mode, dt)
        refg = _vals(gold[key], dt)
        if dt == "f32":
            np.testing.assert_allclose(g, refg, rtol=2e-5, atol=2e-6)
        else:
            diff = np.abs(g - refg)
            assert diff.max() <= 2 ** -6 * max(1.0, np.abs(refg).max()), diff.max()


@pytest.mark.parametrize("name", sorted(C.GDN_CASES))
def test_gdn_oracle_matches_reference(name):
    spec, inp, gold = gdn_case(name)
    dt = spec["dtype"]
    conv_state = inp["conv_state"].copy()
    ssm_state = inp["ssm_state"].copy()
    params = dict(conv_weight=inp["conv_weight"], conv_bias=None, A_log=inp["A_log"],
                  dt_bias=inp["dt_bias"], norm_weight=inp["norm_weight"])
    raw = OG.linear_attention_core(inp["qkv"], inp["b"], inp["a"], None, params, conv_state,
                                   ssm_state, spec["req"], spec["ext"], C.gdn_dims(spec), dt)
    req = spec["req"]
    # conv-state roll is a copy: bit-exact
    np.testing.assert_array_equal(conv_state[req], gold["conv_state"])
    np.testing.assert_allclose(ssm_state[req], gold["ssm_state"], rtol=1e-4, atol=2e-6)
    ref = _vals(gold["raw"], dt)
    if dt == "f32":
        np.testing.assert_allclose(raw, ref, rtol=1e-4, atol=2e-6)
    else:
        diff = np.abs(raw - ref)
        assert diff.max() <= 2 ** -7 * max(1.0, np.abs(ref).max()), diff.max()
    normed = OG.rms_norm_gated(raw, _vals(inp["z"], dt), _vals(inp["norm_weight"], dt),
                               spec["dv"], 1e-6, dt)
    refn = _vals(gold["normed"], dt)
    if dt == "f32":
        np.testing.assert_allclose(normed, refn, rtol=1e-4, atol=1e-5)
    else:
        diff = np.abs(normed - refn)
        assert diff.max() <= 2 ** -6 * max(1.0, np.abs(refn).max()), diff.max()


def test_kv_store_oracle_matches_torch_index_put():
    """The reference's pool write is torch advanced-index assignment
    (qwen3_8/full_attention.py:148-149); the oracle must have the same semantics, including
    wrap-around of negative locations and last-write-wins for duplicates."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    kb = rng.standard_normal((50, 2, 8)).astype(np.float32)
    vb = rng.standard_normal((50, 2, 8)).astype(np.float32)
    k = rng.standard_normal((6, 2, 8)).astype(np.float32)
    v = rng.standard_normal((6, 2, 8)).astype(np.float32)
    loc = np.array([3, 17, -1, 49, 0, 8], dtype=np.int64)
    kt, vt = torch.from_numpy(kb.copy()), torch.from_numpy(vb.copy())
    kt[torch.from_numpy(loc)] = torch.from_numpy(k)
    vt[torch.from_numpy(loc)] = torch.from_numpy(v)
    OA.kv_store(kb, vb, loc, k, v)
    np.testing.assert_array_equal(kb, kt.numpy())
    np.testing.assert_array_equal(vb, vt.numpy())
    with pytest.raises(IndexError):
        OA.kv_store(kb, vb, np.array([50]), k[:1], v[:1])


def test_bf16_roundtrip_matches_torch():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(0).standard_normal(4096).astype(np.float32) * 100
    x[:4] = [0.0, -0.0, np.inf, -np.inf]
    ours = BF.from_f32(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, theirs)
    np.testing.assert_array_equal(BF.to_f32(ours), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_every_golden_fixture_matches_its_regenerated_inputs():
    """The committed fixtures were computed from exactly the inputs tests/golden/cases.py
    regenerates (checksummed), so every GPU comparison against them is meaningful."""
    from tests.golden.load import module_case
    for name in C.ATTN_CASES:
        attention_case(name)
    for name in C.GDN_CASES:
        gdn_case(name)
    for name in C.MODULE_CASES:
        module_case(name)
    from tests.golden.load import prologue_case
    for name in C.PROLOGUE_CASES:
        prologue_case(name)


@pytest.mark.parametrize("name", sorted(C.PROLOGUE_CASES))
def test_prologue_oracle_matches_reference(name):
    """q/k RMSNorm + partial (M-)RoPE + pool write: the oracle reproduces the reference's modules
    bit for bit in bf16 (every torch op rounds where the oracle rounds) and to fp32 rounding in
    fp32."""
    from tests.golden.load import prologue_case
    spec, inp, gold = prologue_case(name)
    dt = spec["dtype"]
    kb, vb = inp["k_buf"].copy(), inp["v_buf"].copy()
    sec, inter = spec["mrope"] if spec["mrope"] else ([11, 11, 10], True)
    qo = OA.attn_prologue(C.prologue_q(inp, spec), inp["k"], inp["v"], inp["q_norm_weight"],
                          inp["k_norm_weight"], inp["positions"], gold["inv_freq"], kb, vb,
                          inp["out_cache_loc"], dt, C.PROLOGUE_EPS, sec, inter)
    np.testing.assert_array_equal(vb, gold["v_buf"])
    if dt == "bf16":
        np.testing.assert_array_equal(qo, gold["q_out"])
        np.testing.assert_array_equal(kb, gold["k_buf"])
    else:
        np.testing.assert_allclose(qo, gold["q_out"], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(kb, gold["k_buf"], rtol=1e-6, atol=1e-6)
