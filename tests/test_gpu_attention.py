"""GPU parity of the paged full-attention hot path (a1-a4) through the C ABI.

Each case runs the CUDA kernels on seeded inputs and compares with (1) the golden outputs recorded
from the reference's own functions and (2) the CPU oracle.  Tolerances: bf16 outputs within
max-abs 2e-2 / mean-abs 2e-3 of the fp32 evaluation; fp32 within rtol 1e-4; index work
(KV store, slot gathers) bit-exact.
"""

import numpy as np
import pytest

from oracle import attention as OA
from oracle import bf16 as BF
from tests.golden import cases as C
from tests.golden.load import attention_case
from tests.helpers import assert_close, to_numpy, to_torch, values

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _run(inp, spec, gate_mode="none", force_extend=False):
    dt = spec["dtype"]
    from tokenfactory_b200 import ops
    q = to_torch(inp["q"], dt)
    kb, vb = to_torch(inp["k_buf"], dt), to_torch(inp["v_buf"], dt)
    r2t = to_torch(inp["req_to_token"], dt)
    rpi = to_torch(inp["req_pool_indices"], dt)
    sl = to_torch(inp["seq_lens"], dt)
    el = to_torch(inp["extend_lens"], dt)
    gate = to_torch(inp["gate"], dt) if gate_mode != "none" else None
    seq, ext = spec["seq"], spec["ext"]
    bsz = len(seq)
    slot_mode = "wrap" if bsz == 1 else "clamp"
    scale = spec["d"] ** -0.5
    if max(ext) == 1 and not force_extend:
        out = ops.paged_decode(q, kb, vb, r2t, rpi, sl, scale, max(seq), gate=gate,
                               gate_mode=gate_mode, slot_mode=slot_mode)
    else:
        out = ops.paged_extend(q, kb, vb, r2t, rpi, sl, el, scale, max(seq), max(ext), gate=gate,
                               gate_mode=gate_mode, slot_mode=slot_mode)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("name", sorted(C.ATTN_CASES))
def test_attention_matches_golden_and_oracle(name):
    spec, inp, gold = attention_case(name)
    dt = spec["dtype"]
    out = values(_run(inp, spec), dt)
    ref = BF.as_f32(gold["out"], dt)
    orc = OA.slot_based_attention(inp["q"], inp["k_buf"], inp["v_buf"], inp["req_to_token"],
                                  inp["req_pool_indices"], inp["seq_lens"], inp["extend_lens"],
                                  spec["d"] ** -0.5, dt)
    assert_close(out, orc, dt, what=f"{name} vs oracle")
    assert_close(out, ref, dt, what=f"{name} vs reference golden", f32_rtol=2e-4, f32_atol=2e-5)


@pytest.mark.parametrize("name", ["decode_bf16", "decode_d256_bf16", "extend_mixed_bf16",
                                  "bsz1_decode_f32", "decode_f32"])
@pytest.mark.parametrize("mode", ["silu", "sigmoid"])
def test_fused_output_gate(name, mode):
    spec, inp, gold = attention_case(name)
    dt = spec["dtype"]
    out = values(_run(inp, spec, gate_mode=mode), dt).reshape(sum(spec["ext"]), -1)
    orc = OA.slot_based_attention(inp["q"], inp["k_buf"], inp["v_buf"], inp["req_to_token"],
                                  inp["req_pool_indices"], inp["seq_lens"], inp["extend_lens"],
                                  spec["d"] ** -0.5, dt)
    t = orc.shape[0]
    want = OA.output_gate(BF.round_to(orc, dt).reshape(t, -1), inp["gate"].reshape(t, -1), mode, dt)
    assert_close(out, want, dt, what=f"{name} gate {mode}")
    key = f"out_{mode}"
    if key in gold:
        assert_close(out, BF.as_f32(gold[key], dt), dt, what=f"{name} gate {mode} vs golden",
                     f32_rtol=2e-4, f32_atol=2e-5)


def test_decode_through_extend_kernel_agrees():
    """A pure-decode batch sent through the varlen extend entry point gives the same result."""
    spec, inp, _ = attention_case("decode_bf16")
    a = values(_run(inp, spec), "bf16")
    b = values(_run(inp, spec, force_extend=True), "bf16")
    assert_close(a, b, "bf16", what="decode vs extend path")


def _random_decode(seed, B, hq, hkv, d, lmin, lmax, slots, dtype="bf16"):
    spec = dict(dtype=dtype, hq=hq, hkv=hkv, d=d, seq=[], ext=[1] * B, req=[], slots=slots,
                rows=B + 3, cols=lmax + 8, seed=seed)
    rng = np.random.default_rng(seed)
    spec["seq"] = [int(x) for x in rng.integers(lmin, lmax + 1, B)]
    spec["req"] = [int(x) for x in rng.permutation(B + 3)[:B]]
    return spec


@pytest.mark.parametrize("shape", [
    # (B, Hq, Hkv, D, Lmin, Lmax): balanced split across all SMs, GQA 8 / 4 / 1 and head dims
    (16, 32, 4, 256, 64, 3000),
    (3, 8, 1, 256, 5000, 9000),     # few long units cut over many CTAs
    (1, 8, 1, 256, 20000, 20000),   # one unit over every CTA
    (5, 4, 1, 256, 1, 40),          # fewer tiles than SMs
    (12, 16, 2, 128, 1, 2000),
    (8, 8, 8, 64, 100, 700),        # MHA
    (7, 12, 2, 64, 30, 900),        # group 6 (padded to 8)
])
def test_decode_random_shapes_vs_oracle(shape):
    B, hq, hkv, d, lmin, lmax = shape
    total = None
    spec = _random_decode(100 + sum(shape), B, hq, hkv, d, lmin, lmax, slots=1)
    total = sum(spec["seq"])
    spec["slots"] = total + 17
    inp = C.attn_inputs(spec)
    out = values(_run(inp, spec, gate_mode="sigmoid"), "bf16").reshape(B, -1)
    orc = OA.slot_based_attention(inp["q"], inp["k_buf"], inp["v_buf"], inp["req_to_token"],
                                  inp["req_pool_indices"], inp["seq_lens"], inp["extend_lens"],
                                  d ** -0.5, "bf16")
    want = OA.output_gate(BF.round_f32(orc).reshape(B, -1), inp["gate"].reshape(B, -1),
                          "sigmoid", "bf16")
    assert_close(out, want, "bf16", what=f"decode {shape}")


def test_decode_batch_beyond_the_tensor_core_schedule():
    """A decode batch of 60,000 requests is above the tensor-core kernel's schedule bound (its
    combine keeps one int32 per request in shared memory): the workspace size is 0 and the call
    runs the CUDA-core kernel, checked against a vectorised fp32 torch evaluation of the
    reference's batched decode (qwen3_8/full_attention.py:215-242)."""
    from tokenfactory_b200 import _capi, ops
    B, hq, hkv, d, lmax = 60_000, 8, 1, 64, 4
    g = torch.Generator(device="cuda").manual_seed(60)
    lens = torch.randint(1, lmax + 1, (B,), generator=g, device="cuda")
    slots = B * lmax + 1
    r2t = (torch.randperm(slots - 1, generator=g, device="cuda") + 1)[:B * lmax].view(B, lmax)
    r2t = torch.where(torch.arange(lmax, device="cuda")[None] < lens[:, None], r2t, -1)
    kb = torch.randn((slots, hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    vb = torch.randn((slots, hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn((B, hq, d), generator=g, device="cuda").to(torch.bfloat16)
    rpi = torch.arange(B, device="cuda")
    args, keep = ops._paged_args(q, kb, vb, r2t, rpi, lens, None, d ** -0.5, None, "none",
                                 q, lmax, 1, "clamp", None)
    import ctypes
    assert _capi.load().tf_paged_decode_workspace_size(ctypes.byref(args)) == 0
    del keep
    out = ops.paged_decode(q, kb, vb, r2t, rpi, lens, d ** -0.5, lmax)
    idx = r2t.clamp(min=0)
    k = kb[idx][:, :, 0].float()                      # [B, L, D] (one kv head)
    v = vb[idx][:, :, 0].float()
    s = torch.einsum("bhd,bld->bhl", q.float(), k) * d ** -0.5
    s = s.masked_fill(torch.arange(lmax, device="cuda")[None, None] >= lens[:, None, None],
                      float("-inf"))
    want = torch.einsum("bhl,bld->bhd", torch.softmax(s, -1), v)
    torch.cuda.synchronize()
    assert_close(values(out, "bf16"), want.cpu().numpy(), "bf16", what="decode B=60000")


@pytest.mark.parametrize("B,lmax,d,hkv", [(9000, 40, 64, 2), (8192, 300, 128, 1)])
def test_decode_large_batch_schedules(B, lmax, d, hkv):
    """Batches of up to 8192 requests compute their cost-balanced schedule in every decode and
    combine CTA; above that a 1-CTA plan kernel computes equal tile ranges once (9,000 requests,
    lengths up to 40: many requests per CTA range, ranges cut inside requests).  Both against a
    vectorised fp32 torch evaluation of the reference's batched decode
    (qwen3_8/full_attention.py:215-242), with lengths of 0 (NaN rows) among them."""
    from tokenfactory_b200 import ops
    hq = 8 * hkv
    g = torch.Generator(device="cuda").manual_seed(B + lmax)
    lens = torch.randint(1, lmax + 1, (B,), generator=g, device="cuda")
    lens[::997] = 0
    slots = B * lmax + 1
    r2t = (torch.randperm(slots - 1, generator=g, device="cuda") + 1)[:B * lmax].view(B, lmax)
    r2t = torch.where(torch.arange(lmax, device="cuda")[None] < lens[:, None], r2t, -1)
    kb = torch.randn((slots, hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    vb = torch.randn((slots, hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn((B, hq, d), generator=g, device="cuda").to(torch.bfloat16)
    rpi = torch.arange(B, device="cuda")
    out = ops.paged_decode(q, kb, vb, r2t, rpi, lens, d ** -0.5, lmax)
    idx = r2t.clamp(min=0)
    k = kb[idx].float()                               # [B, L, Hkv, D]
    v = vb[idx].float()
    qh = q.float().view(B, hkv, hq // hkv, d)
    s = torch.einsum("bkgd,blkd->bkgl", qh, k) * d ** -0.5
    s = s.masked_fill(torch.arange(lmax, device="cuda")[None, None, None] >= lens[:, None, None, None],
                      float("-inf"))
    want = torch.einsum("bkgl,blkd->bkgd", torch.softmax(s, -1), v).reshape(B, hq, d)
    torch.cuda.synchronize()
    got = values(out, "bf16").reshape(B, hq, d)
    empty = (lens == 0).cpu().numpy()
    assert np.isnan(got[empty]).all()
    assert_close(got[~empty], want.cpu().numpy()[~empty], "bf16", what=f"decode B={B}")


def test_decode_request_without_keys_gives_nan_rows():
    """A request with no keys (seq_len 0) among others: its output rows are NaN, as the
    reference's softmax over an empty row, and the other rows match the batch where it has keys
    (the split points move, so within the bf16 tolerance)."""
    spec = _random_decode(321, 6, 32, 4, 256, 200, 5000, slots=1)
    spec["slots"] = sum(spec["seq"]) + 3
    inp = C.attn_inputs(spec)
    B = len(spec["seq"])
    ref = values(_run(inp, spec, gate_mode="sigmoid"), "bf16").reshape(B, -1)
    sl = inp["seq_lens"].copy()
    sl[2] = 0
    seq = list(spec["seq"])
    seq[2] = 0
    out = values(_run(dict(inp, seq_lens=sl), dict(spec, seq=seq), gate_mode="sigmoid"),
                 "bf16").reshape(B, -1)
    assert np.isnan(out[2]).all()
    keep = [i for i in range(B) if i != 2]
    assert_close(out[keep], ref[keep], "bf16", what="decode beside an empty request")


def test_decode_repeat_is_deterministic():
    spec = _random_decode(7, 9, 32, 4, 256, 10, 4000, slots=1)
    spec["slots"] = sum(spec["seq"]) + 1
    inp = C.attn_inputs(spec)
    a = to_numpy(_run(inp, spec))
    b = to_numpy(_run(inp, spec))
    np.testing.assert_array_equal(a, b)


# ------------------------------------------------------------------------------------------
# a1. KV store: bit-exact, torch index semantics
# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dt,d", [("bf16", 256), ("bf16", 64), ("f32", 32), ("bf16", 30)])
def test_kv_store_bit_exact(dt, d):
    from tokenfactory_b200 import ops
    rng = np.random.default_rng(d)
    S, H, T = 300, 2, 41
    kb = BF.store(rng.standard_normal((S, H, d)).astype(np.float32), dt)
    vb = BF.store(rng.standard_normal((S, H, d)).astype(np.float32), dt)
    k = BF.store(rng.standard_normal((T, H, d)).astype(np.float32), dt)
    v = BF.store(rng.standard_normal((T, H, d)).astype(np.float32), dt)
    loc = rng.permutation(np.arange(1, S))[:T].astype(np.int64)
    loc[3] = -5  # wraps like torch indexing
    kb_t, vb_t = to_torch(kb, dt), to_torch(vb, dt)
    ops.kv_store(kb_t, vb_t, to_torch(loc, dt), to_torch(k, dt), to_torch(v, dt))
    torch.cuda.synchronize()
    OA.kv_store(kb, vb, loc, k, v)
    np.testing.assert_array_equal(to_numpy(kb_t), kb)
    np.testing.assert_array_equal(to_numpy(vb_t), vb)


def test_kv_store_out_of_range_is_recorded_not_written():
    from tokenfactory_b200 import ops
    kb = torch.zeros((10, 1, 64), dtype=torch.bfloat16, device="cuda")
    vb = torch.zeros_like(kb)
    k = torch.ones((2, 1, 64), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.kv_store(kb, vb, torch.tensor([3, 10], device="cuda"), k, k, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1  # TF_KERR_SLOT_RANGE
    assert kb[3].float().sum().item() == 64 and kb.float().sum().item() == 64


def test_out_of_range_slot_is_recorded():
    from tokenfactory_b200 import ops
    spec, inp, _ = attention_case("decode_bf16")
    r2t = inp["req_to_token"].copy()
    r2t[spec["req"][1], 4] = 10 ** 9
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.paged_decode(to_torch(inp["q"], "bf16"), to_torch(inp["k_buf"], "bf16"),
                     to_torch(inp["v_buf"], "bf16"), to_torch(r2t, "bf16"),
                     to_torch(inp["req_pool_indices"], "bf16"), to_torch(inp["seq_lens"], "bf16"),
                     64 ** -0.5, max(spec["seq"]), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1


def test_bad_arguments_raise():
    from tokenfactory_b200 import _capi, ops
    q = torch.zeros((2, 6, 64), dtype=torch.bfloat16, device="cuda")
    kb = torch.zeros((10, 4, 64), dtype=torch.bfloat16, device="cuda")
    r2t = torch.zeros((2, 8), dtype=torch.int64, device="cuda")
    idx = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):  # 6 q heads over 4 kv heads
        ops.paged_decode(q, kb, kb, r2t, idx, idx + 1, 0.125, 1)
    q = torch.zeros((2, 8, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_capi.TFAttnError):  # max_seq_len beyond the table
        ops.paged_decode(q, kb, kb, r2t, idx, idx + 1, 0.125, 9)


def test_empty_batch_is_a_no_op():
    from tokenfactory_b200 import ops
    q = torch.zeros((0, 8, 64), dtype=torch.bfloat16, device="cuda")
    kb = torch.zeros((10, 1, 64), dtype=torch.bfloat16, device="cuda")
    r2t = torch.zeros((2, 8), dtype=torch.int64, device="cuda")
    e = torch.zeros(0, dtype=torch.int64, device="cuda")
    out = ops.paged_decode(q, kb, kb, r2t, e, e, 0.125, 0)
    assert out.shape == (0, 8, 64)


@pytest.mark.parametrize("shape", [
    # (Hq, Hkv, D, [(prefix, extend), ...]): tcgen05 extend path (bf16, D 64/128/256, G 1..16)
    (32, 4, 256, [(0, 300), (700, 129), (13, 1), (64, 64)]),
    (8, 2, 256, [(1000, 77), (0, 17)]),
    (16, 8, 128, [(250, 200), (5, 3)]),
    (8, 8, 64, [(90, 140)]),
    (16, 1, 128, [(40, 33), (0, 8)]),
])
def test_extend_random_shapes_vs_oracle(shape):
    hq, hkv, d, reqs = shape
    seq = [p + e for p, e in reqs]
    ext = [e for _, e in reqs]
    B = len(reqs)
    spec = dict(dtype="bf16", hq=hq, hkv=hkv, d=d, seq=seq, ext=ext,
                req=[int(x) for x in np.random.default_rng(d + hq).permutation(B + 2)[:B]],
                slots=sum(seq) + 11, rows=B + 2, cols=max(seq) + 5, seed=hq * d + sum(seq))
    inp = C.attn_inputs(spec)
    out = values(_run(inp, spec, gate_mode="sigmoid"), "bf16").reshape(sum(ext), -1)
    orc = OA.slot_based_attention(inp["q"], inp["k_buf"], inp["v_buf"], inp["req_to_token"],
                                  inp["req_pool_indices"], inp["seq_lens"], inp["extend_lens"],
                                  d ** -0.5, "bf16")
    t = orc.shape[0]
    want = OA.output_gate(BF.round_f32(orc).reshape(t, -1), inp["gate"].reshape(t, -1),
                          "sigmoid", "bf16")
    assert_close(out, want, "bf16", what=f"extend {shape}")


@pytest.mark.parametrize("growing", [False, True])
def test_extend_at_config4_lengths_vs_oracle(growing):
    """Config 4's longest requests: a prefix of 4096 with an extend of 2048 (up to 6144 keys and
    16 query tiles of 128 rows at G = 8) next to (3000, 1500), on the SM-pair tcgen05 kernel at
    head_dim 256, against the oracle at the plain bf16 bound.  growing=True scales each key row by
    1 + position / 600 so that a query row's running max keeps rising along the 48 key tiles:
    the kernel's lazy O rescale (taken when the row max grows by more than 2^8) then fires many
    times per row.  That case runs without the output gate: its softmax is so peaked that the
    attention output sits near single V values of up to ~4, where the reference's second
    rounding (after the gate) can land an element that crossed 4 before gating two bf16 steps
    away; the ungated output has one rounding and meets the plain bound."""
    hq, hkv, d = 8, 1, 256
    reqs = [(4096, 2048), (3000, 1500)]
    seq = [p + e for p, e in reqs]
    ext = [e for _, e in reqs]
    B = len(reqs)
    spec = dict(dtype="bf16", hq=hq, hkv=hkv, d=d, seq=seq, ext=ext, req=[1, 0],
                slots=sum(seq) + 11, rows=B + 1, cols=max(seq) + 5, seed=4096 + int(growing))
    inp = C.attn_inputs(spec)
    if growing:
        pos = np.zeros(spec["slots"], np.float32)
        for b, r in enumerate(spec["req"]):
            sl = inp["req_to_token"][r, :seq[b]]
            pos[sl[sl >= 0]] = np.arange(seq[b])[sl >= 0]
        kf = BF.as_f32(inp["k_buf"], "bf16") * (1.0 + pos / 600.0)[:, None, None]
        inp["k_buf"] = BF.from_f32(kf.astype(np.float32))
    mode = "none" if growing else "sigmoid"
    out = values(_run(inp, spec, gate_mode=mode), "bf16").reshape(sum(ext), -1)
    orc = OA.slot_based_attention(inp["q"], inp["k_buf"], inp["v_buf"], inp["req_to_token"],
                                  inp["req_pool_indices"], inp["seq_lens"], inp["extend_lens"],
                                  d ** -0.5, "bf16")
    t = orc.shape[0]
    want = orc.reshape(t, -1) if growing else OA.output_gate(
        BF.round_f32(orc).reshape(t, -1), inp["gate"].reshape(t, -1), "sigmoid", "bf16")
    assert_close(out, want, "bf16", what=f"extend config-4 lengths growing={growing}")


@pytest.mark.parametrize("d,hq,hkv", [(128, 16, 8), (256, 8, 1)])
def test_extend_unaligned_gate_rows_vs_oracle(d, hq, hkv):
    """A gate view whose head rows do not start on 16-byte boundaries (rows d + 1 elements apart,
    one element into their buffer) takes the SM-pair kernel's element-by-element epilogue; the
    aligned gate takes the vector one.  Both match the oracle at the bf16 bound."""
    from tokenfactory_b200 import ops
    reqs = [(250, 200), (5, 3)]
    seq = [p + e for p, e in reqs]
    ext = [e for _, e in reqs]
    B = len(reqs)
    spec = dict(dtype="bf16", hq=hq, hkv=hkv, d=d, seq=seq, ext=ext, req=[2, 0],
                slots=sum(seq) + 11, rows=B + 2, cols=max(seq) + 5, seed=d + 5 * hq)
    inp = C.attn_inputs(spec)
    aligned = values(_run(inp, spec, gate_mode="silu"), "bf16").reshape(sum(ext), -1)
    q = to_torch(inp["q"], "bf16")
    kb, vb = to_torch(inp["k_buf"], "bf16"), to_torch(inp["v_buf"], "bf16")
    r2t = to_torch(inp["req_to_token"], "bf16")
    rpi, sl = to_torch(inp["req_pool_indices"], "bf16"), to_torch(inp["seq_lens"], "bf16")
    el = to_torch(inp["extend_lens"], "bf16")
    g = to_torch(inp["gate"], "bf16")
    wide = torch.zeros((g.shape[0], hq, d + 1), dtype=g.dtype, device=g.device)
    wide[:, :, 1:] = g
    g_view = wide[:, :, 1:]
    assert g_view.data_ptr() % 16 != 0 and g_view.stride(1) == d + 1
    out = ops.paged_extend(q, kb, vb, r2t, rpi, sl, el, d ** -0.5, max(seq), max(ext), gate=g_view,
                           gate_mode="silu")
    torch.cuda.synchronize()
    unaligned = values(out, "bf16").reshape(sum(ext), -1)
    orc = OA.slot_based_attention(inp["q"], inp["k_buf"], inp["v_buf"], inp["req_to_token"],
                                  inp["req_pool_indices"], inp["seq_lens"], inp["extend_lens"],
                                  d ** -0.5, "bf16")
    t = orc.shape[0]
    want = OA.output_gate(BF.round_f32(orc).reshape(t, -1), inp["gate"].reshape(t, -1), "silu",
                          "bf16")
    assert_close(aligned, want, "bf16", what=f"extend d={d} aligned gate")
    assert_close(unaligned, want, "bf16", what=f"extend d={d} unaligned gate")
