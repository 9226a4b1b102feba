"""GPU parity of the Gated DeltaNet hot path (a5-a9) through the C ABI.

Compared against the golden outputs of the reference's own functions and against the oracle.
conv_state rolls are copies and must be bit-exact; the fp32 recurrent state within rtol 1e-4 per
step and within 1e-3 relative after 256 sequential steps; outputs within the bf16 tolerance.
"""

import numpy as np
import pytest

from oracle import bf16 as BF
from oracle import gdn as OG
from tests.golden import cases as C
from tests.golden.load import gdn_case
from tests.helpers import assert_close, to_numpy, to_torch, values

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _tensors(inp, dt):
    return {k: to_torch(v, "f32" if k == "ssm_state" else dt) for k, v in inp.items()}


def _run(spec, t, fused_norm: bool, force_extend=False):
    from tokenfactory_b200 import ops
    ext = spec["ext"]
    kw = dict(num_k_heads=spec["nk"], head_k_dim=spec["dk"], head_v_dim=spec["dv"])
    z = t["z"] if fused_norm else None
    nw = t["norm_weight"] if fused_norm else None
    if all(e == 1 for e in ext) and not force_extend:
        out = ops.gdn_decode(t["qkv"], t["b"], t["a"], t["conv_weight"], t["A_log"], t["dt_bias"],
                             t["conv_state"], t["ssm_state"], t["req_pool_indices"], z=z,
                             norm_weight=nw, **kw)
    else:
        out = ops.gdn_extend(t["qkv"], t["b"], t["a"], t["conv_weight"], t["A_log"],
                             t["dt_bias"], t["conv_state"], t["ssm_state"], t["req_pool_indices"],
                             t["extend_lens"], max_extend_len=max(ext), z=z, norm_weight=nw, **kw)
    torch.cuda.synchronize()
    return out


def _oracle(spec, inp, with_norm):
    cs, ss = inp["conv_state"].copy(), inp["ssm_state"].copy()
    params = dict(conv_weight=inp["conv_weight"], conv_bias=None, A_log=inp["A_log"],
                  dt_bias=inp["dt_bias"], norm_weight=inp["norm_weight"])
    out = OG.linear_attention_core(inp["qkv"], inp["b"], inp["a"],
                                   inp["z"] if with_norm else None, params, cs, ss, spec["req"],
                                   spec["ext"], C.gdn_dims(spec), spec["dtype"])
    return out, cs, ss


@pytest.mark.parametrize("name", sorted(C.GDN_CASES))
@pytest.mark.parametrize("fused_norm", [False, True])
def test_gdn_matches_golden_and_oracle(name, fused_norm):
    spec, inp, gold = gdn_case(name)
    dt = spec["dtype"]
    t = _tensors(inp, dt)
    out = values(_run(spec, t, fused_norm), dt)
    orc, cs, ss = _oracle(spec, inp, fused_norm)
    req = spec["req"]
    np.testing.assert_array_equal(to_numpy(t["conv_state"])[req], gold["conv_state"])
    np.testing.assert_array_equal(to_numpy(t["conv_state"]), cs)
    got_ss = to_numpy(t["ssm_state"])
    np.testing.assert_allclose(got_ss[req], gold["ssm_state"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(got_ss, ss, rtol=1e-4, atol=1e-5)
    ref = BF.as_f32(gold["normed" if fused_norm else "raw"], dt)
    assert_close(out, orc, dt, what=f"{name} vs oracle")
    assert_close(out, ref, dt, what=f"{name} vs golden", f32_rtol=2e-4, f32_atol=2e-5)


@pytest.mark.parametrize("name", ["gdn_decode_bf16", "gdn_decode_bf16_d128", "gdn_decode_f32_d64"])
def test_decode_batch_through_extend_path(name):
    """An all-decode batch through tf_gdn_extend equals tf_gdn_decode (same state updates)."""
    spec, inp, _ = gdn_case(name)
    dt = spec["dtype"]
    t1, t2 = _tensors(inp, dt), _tensors(inp, dt)
    a = values(_run(spec, t1, True), dt)
    b = values(_run(spec, t2, True, force_extend=True), dt)
    assert_close(a, b, dt, what="decode vs extend")
    np.testing.assert_array_equal(to_numpy(t1["conv_state"]), to_numpy(t2["conv_state"]))
    # the extend path may run the state products on the tensor cores as three bf16 products
    # (about 2^-16 relative each): the same bound as the golden extend comparisons
    np.testing.assert_allclose(to_numpy(t1["ssm_state"]), to_numpy(t2["ssm_state"]), rtol=1e-4,
                               atol=1e-5)


def test_state_after_256_decode_steps_within_1e3():
    """the recurrent state after 256 sequential decode steps stays within 1e-3
    relative of the fp32 oracle (27B head shapes, GVA 3:1)."""
    from tokenfactory_b200 import ops
    spec = dict(dtype="bf16", nk=2, nv=6, dk=128, dv=128, kc=4, ext=[1] * 3, req=[4, 0, 2],
                slots=5, seed=77)
    inp = C.gdn_inputs(spec)
    t = _tensors(inp, "bf16")
    cs, ss = inp["conv_state"].copy(), inp["ssm_state"].copy()
    params = dict(conv_weight=inp["conv_weight"], conv_bias=None, A_log=inp["A_log"],
                  dt_bias=inp["dt_bias"], norm_weight=inp["norm_weight"])
    rng = np.random.default_rng(78)
    conv_dim = inp["qkv"].shape[1]
    for step in range(256):
        qkv = BF.from_f32(rng.standard_normal((3, conv_dim)).astype(np.float32))
        b = BF.from_f32(rng.standard_normal((3, 6)).astype(np.float32))
        a = BF.from_f32(rng.standard_normal((3, 6)).astype(np.float32))
        OG.linear_attention_core(qkv, b, a, None, params, cs, ss, spec["req"], [1, 1, 1],
                                 C.gdn_dims(spec), "bf16")
        ops.gdn_decode(to_torch(qkv, "bf16"), to_torch(b, "bf16"), to_torch(a, "bf16"),
                       t["conv_weight"], t["A_log"], t["dt_bias"], t["conv_state"],
                       t["ssm_state"], t["req_pool_indices"], num_k_heads=2, head_k_dim=128,
                       head_v_dim=128)
    torch.cuda.synchronize()
    got = to_numpy(t["ssm_state"])[spec["req"]].astype(np.float64)
    want = ss[spec["req"]].astype(np.float64)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel < 1e-3, rel
    np.testing.assert_array_equal(to_numpy(t["conv_state"]), cs)


def test_decode_many_items_with_a_skipped_request():
    """More (request, k-head) items than the persistent decode grid holds (800 items; 2 CTAs per
    SM), so CTAs walk several items with the next item's state prefetched across the boundary.
    Request 150 (items 300-301, the middle items of their CTAs on a 148-SM part) has an index out
    of range: it is recorded and skipped, and every other request is stepped as the oracle steps
    it."""
    from tokenfactory_b200 import ops
    B, bad = 400, 150
    req = np.random.default_rng(90).permutation(B + 8)[:B].tolist()
    spec = dict(dtype="bf16", nk=2, nv=6, dk=128, dv=128, kc=4, ext=[1] * B, req=req,
                slots=B + 8, seed=91)
    inp = C.gdn_inputs(spec)
    t = _tensors(inp, "bf16")
    t["req_pool_indices"][bad] = B + 8 + 5
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.gdn_decode(t["qkv"], t["b"], t["a"], t["conv_weight"], t["A_log"], t["dt_bias"],
                         t["conv_state"], t["ssm_state"], t["req_pool_indices"], z=t["z"],
                         norm_weight=t["norm_weight"], num_k_heads=2, head_k_dim=128,
                         head_v_dim=128, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 2  # TF_KERR_REQ_RANGE
    keep = [i for i in range(B) if i != bad]
    sub = dict(inp)
    for k in ("qkv", "b", "a", "z"):
        sub[k] = inp[k][keep]
    orc, cs, ss = _oracle(dict(spec, req=[req[i] for i in keep], ext=[1] * len(keep)), sub, True)
    assert_close(values(out, "bf16")[keep], orc, "bf16", what="decode, 800 items")
    np.testing.assert_array_equal(to_numpy(t["conv_state"]), cs)
    np.testing.assert_allclose(to_numpy(t["ssm_state"]), ss, rtol=1e-4, atol=1e-5)


def test_extend_long_request_27b_heads_vs_oracle():
    """A 1000-token request (16 chunks: the tensor-core chunk kernel alternates its two sets of
    chunk buffers and barriers many times) between short ones, against the oracle.  The gated
    outputs are rounded twice by the reference: two bf16 steps allowed (tests/helpers.py); the
    un-normed outputs, rounded once, are held to the plain bound."""
    ext = [3, 1000, 130]
    spec = dict(dtype="bf16", nk=2, nv=6, dk=128, dv=128, kc=4, ext=ext, req=[2, 0, 3],
                slots=5, seed=1133)
    inp = C.gdn_inputs(spec)
    t = _tensors(inp, "bf16")
    out = values(_run(spec, t, True), "bf16")
    orc, cs, ss = _oracle(spec, inp, True)
    assert_close(out, orc, "bf16", what="extend with a 1000-token request", bf16_steps=2)
    np.testing.assert_array_equal(to_numpy(t["conv_state"]), cs)
    np.testing.assert_allclose(to_numpy(t["ssm_state"]), ss, rtol=2e-3, atol=2e-5)
    # the un-normed outputs (one rounding) at the plain bound
    t_raw = _tensors(inp, "bf16")
    raw = values(_run(spec, t_raw, False), "bf16")
    orc_raw, _, _ = _oracle(spec, inp, False)
    assert_close(raw, orc_raw, "bf16", what="extend with a 1000-token request, raw outputs")


def test_extend_more_ctas_than_sms_vs_oracle():
    """30 requests x 6 v-heads = 180 chunk-kernel CTAs (more than the SMs), lengths 1-200 in the
    longest-first order, so SMs run a second CTA after the first released TMEM.  Of 2.3M gated
    outputs, a dozen sit two bf16 steps from the reference (its double rounding), the raw outputs
    within 3e-4."""
    ext = np.random.default_rng(1180).integers(1, 201, 30).tolist()
    req = np.random.default_rng(1181).permutation(34)[:30].tolist()
    spec = dict(dtype="bf16", nk=2, nv=6, dk=128, dv=128, kc=4, ext=ext, req=req, slots=34,
                seed=1182)
    inp = C.gdn_inputs(spec)
    t = _tensors(inp, "bf16")
    out = values(_run(spec, t, True), "bf16")
    orc, cs, ss = _oracle(spec, inp, True)
    assert_close(out, orc, "bf16", what="extend, 180 CTAs", bf16_steps=2)
    np.testing.assert_array_equal(to_numpy(t["conv_state"]), cs)
    np.testing.assert_allclose(to_numpy(t["ssm_state"]), ss, rtol=2e-3, atol=2e-5)


@pytest.mark.parametrize("ext", [[1, 300, 7, 64], [65, 1, 1, 129]])
def test_extend_random_27b_heads_vs_oracle(ext):
    spec = dict(dtype="bf16", nk=2, nv=6, dk=128, dv=128, kc=4, ext=ext,
                req=[3, 0, 5, 1][:len(ext)], slots=6, seed=sum(ext))
    inp = C.gdn_inputs(spec)
    t = _tensors(inp, "bf16")
    out = values(_run(spec, t, True), "bf16")
    orc, cs, ss = _oracle(spec, inp, True)
    assert_close(out, orc, "bf16", what=f"extend {ext}")
    np.testing.assert_array_equal(to_numpy(t["conv_state"]), cs)
    np.testing.assert_allclose(to_numpy(t["ssm_state"]), ss, rtol=2e-3, atol=2e-5)


def test_extend_config4_lengths_from_cached_state():
    """Config 4's longest GDN extend: a 2048-token request and a 1500-token one at the 27B head
    shapes (dk = dv = 128, GVA 3:1) from non-zero cached conv and recurrent states, on the
    tcgen05 chunk kernel.  The raw (un-normed) outputs are held to the plain bf16 bound
    (max-abs 2e-2, mean-abs 2e-3); the gated outputs, which the reference rounds twice, to two
    bf16 steps; the final states to the extend bound."""
    ext = [2048, 1500]
    spec = dict(dtype="bf16", nk=2, nv=6, dk=128, dv=128, kc=4, ext=ext, req=[2, 0], slots=3,
                seed=2048)
    inp = C.gdn_inputs(spec)
    assert np.abs(inp["ssm_state"]).max() > 0 and np.abs(BF.to_f32(inp["conv_state"])).max() > 0
    t_raw, t_gated = _tensors(inp, "bf16"), _tensors(inp, "bf16")
    raw = values(_run(spec, t_raw, False), "bf16")
    gated = values(_run(spec, t_gated, True), "bf16")
    orc_raw, cs, ss = _oracle(spec, inp, False)
    orc_gated, _, _ = _oracle(spec, inp, True)
    assert_close(raw, orc_raw, "bf16", what="extend 2048 + 1500, raw outputs")
    assert_close(gated, orc_gated, "bf16", what="extend 2048 + 1500, gated", bf16_steps=2)
    for t in (t_raw, t_gated):
        np.testing.assert_array_equal(to_numpy(t["conv_state"]), cs)
        np.testing.assert_allclose(to_numpy(t["ssm_state"]), ss, rtol=2e-3, atol=2e-5)


def test_extend_180_ctas_raw_outputs_at_the_plain_bound():
    """The un-normed outputs of the 180-CTA batch (test_extend_more_ctas_than_sms_vs_oracle) at
    the plain bf16 bound, beside the gated ones there."""
    ext = np.random.default_rng(1180).integers(1, 201, 30).tolist()
    req = np.random.default_rng(1181).permutation(34)[:30].tolist()
    spec = dict(dtype="bf16", nk=2, nv=6, dk=128, dv=128, kc=4, ext=ext, req=req, slots=34,
                seed=1182)
    inp = C.gdn_inputs(spec)
    t = _tensors(inp, "bf16")
    out = values(_run(spec, t, False), "bf16")
    orc, cs, ss = _oracle(spec, inp, False)
    assert_close(out, orc, "bf16", what="extend, 180 CTAs, raw outputs")
    np.testing.assert_allclose(to_numpy(t["ssm_state"]), ss, rtol=2e-3, atol=2e-5)


def test_gated_rmsnorm_standalone():
    from tokenfactory_b200 import ops
    rng = np.random.default_rng(3)
    x = BF.from_f32(rng.standard_normal((37, 6 * 128)).astype(np.float32))
    z = BF.from_f32(rng.standard_normal((37, 6 * 128)).astype(np.float32))
    for wlen in (6 * 128, 128):
        w = BF.from_f32((1 + 0.1 * rng.standard_normal(wlen)).astype(np.float32))
        got = values(ops.gated_rmsnorm(to_torch(x, "bf16"), to_torch(z, "bf16"),
                                       to_torch(w, "bf16"), 128), "bf16")
        want = OG.rms_norm_gated(BF.to_f32(x), BF.to_f32(z), BF.to_f32(w), 128, 1e-6, "bf16")
        assert_close(got, want, "bf16", what=f"gated rmsnorm w{wlen}")


def test_bad_request_index_is_recorded():
    from tokenfactory_b200 import ops
    spec, inp, _ = gdn_case("gdn_decode_bf16")
    t = _tensors(inp, "bf16")
    t["req_pool_indices"][1] = 99
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.gdn_decode(t["qkv"], t["b"], t["a"], t["conv_weight"], t["A_log"], t["dt_bias"],
                   t["conv_state"], t["ssm_state"], t["req_pool_indices"], num_k_heads=2,
                   head_k_dim=16, head_v_dim=16, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 2  # TF_KERR_REQ_RANGE
