"""Seeded case definitions shared by the golden-vector generator and the tests.

Inputs are regenerated from these specs with numpy's PCG64 generator (stable across machines and
numpy versions), so the committed fixtures (tests/golden/*.npz) hold only the reference's outputs
plus a checksum of the inputs they were computed from.  Shapes follow the reference's own test
dimensions (heads 4/1, head_dim 32, GDN 2/6 heads with dk=dv=16; tests/test_hybrid_radix_cache.py
:127-146) and slices of the 27B shapes (head_dim 256, GQA 8, dk=dv=128).
"""

import hashlib
from typing import Dict, List

import numpy as np

from oracle import bf16 as _bf

ATTN_CASES: Dict[str, dict] = {
    # batched decode (qwen3_8/full_attention.py:215-242)
    "decode_bf16": dict(dtype="bf16", hq=8, hkv=2, d=64, seq=[1, 17, 64, 100], ext=[1, 1, 1, 1],
                        req=[3, 0, 5, 1], slots=300, rows=6, cols=128, seed=11),
    "decode_f32": dict(dtype="f32", hq=8, hkv=2, d=64, seq=[33, 2, 90], ext=[1, 1, 1],
                       req=[1, 2, 0], slots=200, rows=4, cols=96, seed=12),
    "decode_d256_bf16": dict(dtype="bf16", hq=8, hkv=1, d=256, seq=[5, 300, 129], ext=[1, 1, 1],
                             req=[0, 2, 1], slots=480, rows=3, cols=320, seed=13),
    "decode_d32_mha_bf16": dict(dtype="bf16", hq=4, hkv=4, d=32, seq=[7, 40], ext=[1, 1],
                                req=[1, 0], slots=64, rows=2, cols=48, seed=14),
    # -1 entries inside seq_len read padding slot 0 (clamp, :216-218)
    "decode_negslot_bf16": dict(dtype="bf16", hq=4, hkv=1, d=32, seq=[20, 9], ext=[1, 1],
                                req=[0, 1], slots=64, rows=2, cols=32, seed=15, neg=[(0, 3), (1, 8)]),
    # varlen extend / mixed (qwen3_8/full_attention.py:244-283)
    "extend_mixed_bf16": dict(dtype="bf16", hq=4, hkv=1, d=32, seq=[21, 9, 103], ext=[1, 9, 70],
                              req=[2, 0, 1], slots=256, rows=3, cols=128, seed=21),
    "extend_mixed_f32": dict(dtype="f32", hq=8, hkv=2, d=64, seq=[40, 66, 5], ext=[17, 66, 1],
                             req=[0, 1, 2], slots=160, rows=3, cols=80, seed=22),
    "extend_d256_gqa4_bf16": dict(dtype="bf16", hq=4, hkv=1, d=256, seq=[140, 10], ext=[40, 3],
                                  req=[1, 0], slots=200, rows=2, cols=160, seed=23),
    "extend_d128_bf16": dict(dtype="bf16", hq=4, hkv=2, d=128, seq=[150, 66], ext=[70, 66],
                             req=[0, 1], slots=256, rows=2, cols=160, seed=24),
    # single-request path (qwen3_8/full_attention.py:179-213)
    "bsz1_extend_bf16": dict(dtype="bf16", hq=8, hkv=2, d=128, seq=[53], ext=[13], req=[1],
                             slots=64, rows=2, cols=64, seed=31),
    "bsz1_decode_f32": dict(dtype="f32", hq=8, hkv=2, d=64, seq=[77], ext=[1], req=[0],
                            slots=100, rows=1, cols=80, seed=32),
    # a -1 inside seq_len wraps to the last slot on the single-request path (:188)
    "bsz1_negslot_f32": dict(dtype="f32", hq=4, hkv=2, d=32, seq=[12], ext=[1], req=[0],
                             slots=40, rows=1, cols=16, seed=33, neg=[(0, 5)]),
}

GDN_CASES: Dict[str, dict] = {
    # batched decode (qwen3_8/linear_attention.py:244-298)
    "gdn_decode_bf16": dict(dtype="bf16", nk=2, nv=6, dk=16, dv=16, kc=4, ext=[1, 1, 1],
                            req=[2, 0, 3], slots=5, seed=41),
    "gdn_decode_f32_d64": dict(dtype="f32", nk=2, nv=4, dk=64, dv=64, kc=4, ext=[1, 1],
                               req=[1, 0], slots=3, seed=42),
    "gdn_decode_bf16_d128": dict(dtype="bf16", nk=1, nv=2, dk=128, dv=128, kc=4, ext=[1, 1],
                                 req=[0, 2], slots=3, seed=43),
    # per-request extend loop (qwen3_8/linear_attention.py:329-363)
    "gdn_extend_bf16_mixed": dict(dtype="bf16", nk=2, nv=6, dk=16, dv=16, kc=4,
                                  ext=[1, 5, 70, 64], req=[3, 1, 0, 2], slots=5, seed=51),
    "gdn_extend_f32_mixed": dict(dtype="f32", nk=2, nv=4, dk=64, dv=64, kc=4, ext=[3, 1, 130],
                                 req=[2, 0, 1], slots=4, seed=52),
    "gdn_extend_bf16_d128": dict(dtype="bf16", nk=1, nv=3, dk=128, dv=128, kc=4, ext=[129, 2],
                                 req=[1, 0], slots=2, seed=53),
}


def _normal(rng, shape, scale=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(np.float32)


def attn_inputs(spec: dict) -> dict:
    """Pools, req_to_token, q and gate of an attention case (storage form of spec['dtype'])."""
    rng = np.random.default_rng(spec["seed"])
    dt = spec["dtype"]
    hq, hkv, d = spec["hq"], spec["hkv"], spec["d"]
    s = spec["slots"]
    seq, ext, req = spec["seq"], spec["ext"], spec["req"]
    t = int(sum(ext))
    k_buf = _bf.store(_normal(rng, (s, hkv, d)), dt)
    v_buf = _bf.store(_normal(rng, (s, hkv, d)), dt)
    q = _bf.store(_normal(rng, (t, hq, d)), dt)
    gate = _bf.store(_normal(rng, (t, hq, d)), dt)
    r2t = np.full((spec["rows"], spec["cols"]), -1, dtype=np.int64)
    perm = rng.permutation(np.arange(1, s, dtype=np.int64))
    off = 0
    for b, L in enumerate(seq):
        r2t[req[b], :L] = perm[off:off + L]
        off += L
    for (b, pos) in spec.get("neg", []):
        r2t[req[b], pos] = -1
    out_loc = np.concatenate([r2t[req[b], seq[b] - ext[b]:seq[b]] for b in range(len(seq))])
    return dict(q=q, k_buf=k_buf, v_buf=v_buf, gate=gate, req_to_token=r2t,
                req_pool_indices=np.asarray(req, np.int64), seq_lens=np.asarray(seq, np.int64),
                extend_lens=np.asarray(ext, np.int64), out_cache_loc=out_loc.astype(np.int64))


def gdn_inputs(spec: dict) -> dict:
    """Projected activations, parameters and the state pools of a GDN case."""
    rng = np.random.default_rng(spec["seed"])
    dt = spec["dtype"]
    nk, nv, dk, dv, kc = spec["nk"], spec["nv"], spec["dk"], spec["dv"], spec["kc"]
    conv_dim = 2 * nk * dk + nv * dv
    t = int(sum(spec["ext"]))
    slots = spec["slots"]
    return dict(
        qkv=_bf.store(_normal(rng, (t, conv_dim)), dt),
        b=_bf.store(_normal(rng, (t, nv)), dt),
        a=_bf.store(_normal(rng, (t, nv)), dt),
        z=_bf.store(_normal(rng, (t, nv * dv)), dt),
        conv_weight=_bf.store(_normal(rng, (conv_dim, kc), 0.5), dt),
        A_log=_bf.store(rng.uniform(0.0, 1.5, nv).astype(np.float32), dt),
        dt_bias=_bf.store(_normal(rng, (nv,), 0.5), dt),
        norm_weight=_bf.store((1.0 + _normal(rng, (nv * dv,), 0.1)).astype(np.float32), dt),
        conv_state=_bf.store(_normal(rng, (slots, conv_dim, kc - 1)), dt),
        ssm_state=_normal(rng, (slots, nv, dk, dv), 0.02),
        req_pool_indices=np.asarray(spec["req"], np.int64),
        extend_lens=np.asarray(spec["ext"], np.int64),
    )


def gdn_dims(spec: dict) -> dict:
    return dict(num_k_heads=spec["nk"], num_v_heads=spec["nv"], head_k_dim=spec["dk"],
                head_v_dim=spec["dv"])


def checksum(arrays: dict) -> str:
    """sha256 over the inputs (sorted by name) - detects drift between generator and tests."""
    h = hashlib.sha256()
    for k in sorted(arrays):
        a = np.ascontiguousarray(arrays[k])
        h.update(k.encode())
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------------------------
# module-level cases: a whole Qwen3_8FullAttention / Qwen3_8LinearAttention forward
# ---------------------------------------------------------------------------------------------
MODULE_DIMS = dict(hidden=128, hq=8, hkv=2, d=64, nk=2, nv=4, dk=32, dv=32, kc=4)

MODULE_CASES: Dict[str, dict] = {
    "full_mixed_f32": dict(kind="full", dtype="f32", seq=[10, 6, 16], ext=[1, 6, 11],
                           req=[2, 0, 1], slots=96, rows=4, cols=32, seed=61),
    "full_decode_bf16": dict(kind="full", dtype="bf16", seq=[9, 30, 2, 17], ext=[1, 1, 1, 1],
                             req=[3, 1, 0, 2], slots=96, rows=4, cols=32, seed=62),
    "full_mixed_bf16": dict(kind="full", dtype="bf16", seq=[12, 7], ext=[5, 7], req=[1, 0],
                            slots=64, rows=2, cols=16, seed=63),
    "full_bsz1_bf16": dict(kind="full", dtype="bf16", seq=[20], ext=[20], req=[1],
                           slots=64, rows=2, cols=32, seed=64),
    "linear_mixed_f32": dict(kind="linear", dtype="f32", ext=[1, 9, 70], req=[2, 0, 1],
                             slots=4, seed=65),
    "linear_decode_bf16": dict(kind="linear", dtype="bf16", ext=[1, 1, 1], req=[1, 3, 0],
                               slots=4, seed=66),
    "linear_mixed_bf16": dict(kind="linear", dtype="bf16", ext=[3, 1, 40], req=[0, 2, 1],
                              slots=3, seed=67),
}


def module_weights(spec: dict) -> dict:
    """float32 weights of the case's module, with the reference's parameter names."""
    rng = np.random.default_rng(1000 + spec["seed"])
    m = MODULE_DIMS
    h = m["hidden"]
    if spec["kind"] == "full":
        return {
            "q_proj.weight": _normal(rng, (m["hq"] * m["d"] * 2, h), 0.08),
            "k_proj.weight": _normal(rng, (m["hkv"] * m["d"], h), 0.08),
            "v_proj.weight": _normal(rng, (m["hkv"] * m["d"], h), 0.08),
            "o_proj.weight": _normal(rng, (h, m["hq"] * m["d"]), 0.08),
            "q_norm.weight": (1.0 + _normal(rng, (m["d"],), 0.1)).astype(np.float32),
            "k_norm.weight": (1.0 + _normal(rng, (m["d"],), 0.1)).astype(np.float32),
        }
    conv_dim = 2 * m["nk"] * m["dk"] + m["nv"] * m["dv"]
    return {
        "in_proj_qkv.weight": _normal(rng, (conv_dim, h), 0.08),
        "in_proj_z.weight": _normal(rng, (m["nv"] * m["dv"], h), 0.08),
        "in_proj_b.weight": _normal(rng, (m["nv"], h), 0.08),
        "in_proj_a.weight": _normal(rng, (m["nv"], h), 0.08),
        "conv1d.weight": _normal(rng, (conv_dim, 1, m["kc"]), 0.5),
        "A_log": rng.uniform(0.0, 1.5, m["nv"]).astype(np.float32),
        "dt_bias": _normal(rng, (m["nv"],), 0.5),
        "norm.weight": (1.0 + _normal(rng, (m["nv"] * m["dv"],), 0.1)).astype(np.float32),
        "out_proj.weight": _normal(rng, (h, m["nv"] * m["dv"]), 0.08),
    }


def module_inputs(spec: dict) -> dict:
    """hidden states, positions, batch metadata and the pools (float32 values)."""
    rng = np.random.default_rng(2000 + spec["seed"])
    m = MODULE_DIMS
    t = int(sum(spec["ext"]))
    out = dict(hidden=_normal(rng, (t, m["hidden"])),
               req_pool_indices=np.asarray(spec["req"], np.int64),
               extend_lens=np.asarray(spec["ext"], np.int64))
    if spec["kind"] == "full":
        seq, ext, req = spec["seq"], spec["ext"], spec["req"]
        s = spec["slots"]
        out["k_buf"] = _normal(rng, (s, m["hkv"], m["d"]))
        out["v_buf"] = _normal(rng, (s, m["hkv"], m["d"]))
        r2t = np.full((spec["rows"], spec["cols"]), -1, dtype=np.int64)
        perm = rng.permutation(np.arange(1, s, dtype=np.int64))
        off = 0
        for b, L in enumerate(seq):
            r2t[req[b], :L] = perm[off:off + L]
            off += L
        out["req_to_token"] = r2t
        out["seq_lens"] = np.asarray(seq, np.int64)
        out["out_cache_loc"] = np.concatenate(
            [r2t[req[b], seq[b] - ext[b]:seq[b]] for b in range(len(seq))]).astype(np.int64)
        out["positions"] = np.concatenate(
            [np.arange(seq[b] - ext[b], seq[b]) for b in range(len(seq))]).astype(np.int64)
    else:
        conv_dim = 2 * m["nk"] * m["dk"] + m["nv"] * m["dv"]
        out["conv_state"] = _normal(rng, (spec["slots"], conv_dim, m["kc"] - 1))
        out["ssm_state"] = _normal(rng, (spec["slots"], m["nv"], m["dk"], m["dv"]), 0.05)
    return out


# ---------------------------------------------------------------------------------------------
# fused attention prologue: q/k RMSNorm + partial (M-)RoPE + KV store
# (qwen3_8/full_attention.py:142-149, qwen3_8/rms_norm.py, qwen3_8/rotary_embedding.py)
# ---------------------------------------------------------------------------------------------
PROLOGUE_CASES: Dict[str, dict] = {
    "pro_bf16_d256": dict(dtype="bf16", hq=8, hkv=2, d=256, t=37, slots=64, pos_max=40000,
                          mrope=None, seed=70),
    "pro_bf16_d256_mrope": dict(dtype="bf16", hq=4, hkv=1, d=256, t=21, slots=32, pos_max=5000,
                                mrope=([11, 11, 10], True), seed=71),
    "pro_bf16_d256_mrope_chunked": dict(dtype="bf16", hq=4, hkv=2, d=256, t=9, slots=16,
                                        pos_max=300, mrope=([11, 11, 10], False), seed=72),
    "pro_bf16_d128_gqa_strided": dict(dtype="bf16", hq=16, hkv=1, d=128, t=29, slots=48,
                                      pos_max=200000, mrope=None, strided=True, neg=[3, 10],
                                      seed=73),
    "pro_f32_d64": dict(dtype="f32", hq=4, hkv=4, d=64, t=13, slots=20, pos_max=1000, mrope=None,
                        seed=74),
}
PROLOGUE_THETA = 10000000.0
PROLOGUE_EPS = 1e-6


def prologue_inputs(spec: dict) -> dict:
    """q (inside a [T, Hq, 2D] q_proj output when spec['strided']), k, v, the two norm weights,
    positions ([T] or [3, T]), the pools and out_cache_loc of a prologue case."""
    rng = np.random.default_rng(spec["seed"])
    dt = spec["dtype"]
    hq, hkv, d, t, s = spec["hq"], spec["hkv"], spec["d"], spec["t"], spec["slots"]
    qg = _bf.store(_normal(rng, (t, hq, 2 * d if spec.get("strided") else d)), dt)
    k = _bf.store(_normal(rng, (t, hkv, d)), dt)
    v = _bf.store(_normal(rng, (t, hkv, d)), dt)
    qw = _bf.store((1.0 + 0.1 * _normal(rng, (d,))).astype(np.float32), dt)
    kw = _bf.store((1.0 + 0.1 * _normal(rng, (d,))).astype(np.float32), dt)
    rows = 3 if spec["mrope"] else 1
    pos = rng.integers(0, spec["pos_max"], (rows, t), dtype=np.int64)
    if rows == 1:
        pos = pos[0]
    k_buf = _bf.store(_normal(rng, (s, hkv, d)), dt)
    v_buf = _bf.store(_normal(rng, (s, hkv, d)), dt)
    loc = rng.permutation(np.arange(1, s, dtype=np.int64))[:t]
    for i in spec.get("neg", []):
        loc[i] = loc[i] - s  # the same slot through a negative index
    return dict(qg=qg, k=k, v=v, q_norm_weight=qw, k_norm_weight=kw, positions=pos,
                k_buf=k_buf, v_buf=v_buf, out_cache_loc=loc)


def prologue_q(inp: dict, spec: dict) -> np.ndarray:
    """The q view of the case: the first half of each head's q_proj row when strided."""
    return inp["qg"][..., :spec["d"]] if spec.get("strided") else inp["qg"]


# ---------------------------------------------------------------------------------------------
# GDN state-slot snapshots (ReqToStatePool, req_to_state_pool.py:120-194)
# ---------------------------------------------------------------------------------------------
# A small pool (3 linear layers, 4 working + 3 snapshot slots) filled with seeded values, then a
# script of the pool's calls.  ("alloc",) records the slot alloc_snapshot() returns; the others
# name the method and its arguments as the scheduler and radix tree pass them.
STATE_POOL_SCRIPT: List[tuple] = [
    ("alloc",), ("capture", 0, 4, "node_A"), ("alloc",), ("capture", 1, 5, None),
    ("restore", 4, 2), ("reset", 1), ("alloc",), ("capture", 2, 6, None), ("free", 5),
    ("restore", 6, 3), ("free", 4), ("alloc",), ("capture", 3, 4, "node_B"), ("reset", 0),
    ("restore", 4, 1),
]

STATE_POOL_CASES: Dict[str, dict] = {
    "pool_bf16_conv_f32_ssm": dict(max_reqs=4, max_snapshots=3, layers=3, nk=2, nv=4, dk=16,
                                   dv=16, kc=4, dtype="bf16", seed=80),
}


def state_pool_inputs(spec: dict) -> dict:
    """Initial contents of the pool's two tensors: conv_state [L, slots, conv_dim, K-1] in the
    pool dtype and ssm_state [L, slots, Hv, dk, dv] fp32 (the reference allocates them zeroed;
    the cases fill every slot so that copies and resets are visible)."""
    rng = np.random.default_rng(spec["seed"])
    slots = spec["max_reqs"] + spec["max_snapshots"]
    conv_dim = 2 * spec["nk"] * spec["dk"] + spec["nv"] * spec["dv"]
    return dict(
        conv_state=_bf.store(_normal(rng, (spec["layers"], slots, conv_dim, spec["kc"] - 1)),
                             spec["dtype"]),
        ssm_state=_normal(rng, (spec["layers"], slots, spec["nv"], spec["dk"], spec["dv"]), 0.02),
    )


# ---------------------------------------------------------------------------------------------
# per-step batch construction (ModelRunner._prepare_forward_batch, engine/model_runner.py:108-188)
# ---------------------------------------------------------------------------------------------
# Three steps over a 4-row req_to_token table: prefill chunks (row 2 starts after a 4-token radix
# prefix the scheduler wrote into the host table), then decodes plus a new prefill, then a
# rollback (dirty_from) that forces a stale prefix of row 0 to be re-synced.  Each request is
# (req_pool_idx, cur_start_pos, chunk length, is_prefilled); token ids and slots are seeded.
RUNNER_CASE = dict(max_reqs=4, max_ctx=48, seed=90, steps=[
    dict(reqs=[(0, 0, 5, False), (2, 4, 3, False)], prefix={2: 4}),
    dict(reqs=[(0, 5, 1, True), (2, 7, 1, True), (1, 0, 6, False)]),
    dict(reqs=[(0, 6, 1, True), (1, 6, 1, True), (3, 0, 9, False)], dirty={0: 3},
         rewrite={0: (3, 6)}),
])


def runner_script(case: dict = RUNNER_CASE):
    """The steps as (requests, host req_to_token table before the step, dirty_from or None) with
    the requests as plain dicts; the table evolves the way the scheduler writes it (prefix slots
    before the step, the step's out_cache_loc after it, a rewrite for the rollback)."""
    rng = np.random.default_rng(case["seed"])
    table = [[-1] * case["max_ctx"] for _ in range(case["max_reqs"])]
    steps = []
    for st in case["steps"]:
        for r, n in st.get("prefix", {}).items():
            table[r][:n] = [int(x) for x in rng.integers(1, 10_000, n)]
        for r, (a, b) in st.get("rewrite", {}).items():
            table[r][a:b] = [int(x) for x in rng.integers(1, 10_000, b - a)]
        reqs = []
        for r, start, n, done in st["reqs"]:
            reqs.append(dict(req_pool_idx=r, cur_start_pos=start, cur_seq_len=start + n,
                             cur_chunk_tokens=[int(x) for x in rng.integers(0, 1000, n)],
                             out_cache_loc=[int(x) for x in rng.integers(1, 10_000, n)],
                             is_prefilled=done))
        dirty = None
        if "dirty" in st:
            dirty = [10**9] * case["max_reqs"]
            for r, p in st["dirty"].items():
                dirty[r] = p
        steps.append((reqs, [row[:] for row in table], dirty))
        for q in reqs:
            table[q["req_pool_idx"]][q["cur_start_pos"]:q["cur_seq_len"]] = q["out_cache_loc"]
    return steps


# ---------------------------------------------------------------------------------------------
# block-FP8 linear (triton_block_fp8_linear, qwen3_8/fp8_triton.py:109-181)
# ---------------------------------------------------------------------------------------------
FP8_CASES: Dict[str, dict] = {
    "fp8_bf16_blocks": dict(dtype="bf16", M=5, N=200, K=256, scales=True, bias=False, seed=100),
    "fp8_bf16_bias_tail": dict(dtype="bf16", M=130, N=256, K=272, scales=True, bias=True, seed=101),
    "fp8_f32_per_tensor": dict(dtype="f32", M=3, N=128, K=128, scales=False, bias=False, seed=102),
    "fp8_bf16_m64": dict(dtype="bf16", M=64, N=384, K=512, scales=True, bias=True, seed=103),
}


def fp8_inputs(spec: dict) -> dict:
    """Activations x [M, K] in the case dtype, an e4m3 weight [N, K] (bit patterns), its block
    scales [ceil(N/128), ceil(K/128)] fp32 (when spec['scales']) and a bias [N] of the case dtype."""
    from oracle.fp8 import e4m3_encode

    rng = np.random.default_rng(spec["seed"])
    M, N, K = spec["M"], spec["N"], spec["K"]
    out = dict(x=_bf.store(_normal(rng, (M, K)), spec["dtype"]),
               w=e4m3_encode(np.clip(_normal(rng, (N, K), 0.8), -448, 448)))
    if spec["scales"]:
        out["w_scale"] = rng.uniform(0.5, 1.5, ((N + 127) // 128, (K + 127) // 128)).astype(np.float32)
    if spec["bias"]:
        out["bias"] = _bf.store(_normal(rng, (N,), 0.1), spec["dtype"])
    return out


# ---------------------------------------------------------------------------------------------
# engine-level cases: whole runs of the reference's Scheduler recorded as a trace
# (tests/golden/make_engine_golden.py) and replayed on the GPU through the drop-in layers
# ---------------------------------------------------------------------------------------------
# model dims: fields of Qwen3_8Config / tokenfactory_b200.hybrid_model.HybridConfig
ENGINE_MODELS: Dict[str, dict] = {
    # vocab 1024, hidden 256, [lin, lin, lin, full], Hq 8 / Hkv 2 / D 64,
    # theta 1e7, sigmoid output gate, Hk 4 / Hv 8 / dk = dv = 64, conv 4, MLP 512, fp32
    "config1": dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                    num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                    rope_theta=10000000.0, linear_num_key_heads=4, linear_key_head_dim=64,
                    linear_num_value_heads=8, linear_value_head_dim=64,
                    linear_conv_kernel_dim=4, output_gate_mode="sigmoid"),
    # the mini model of the reference's prefix-reuse test (tests/test_hybrid_radix_cache.py:127-146)
    "prefix": dict(vocab_size=500, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
                   num_attention_heads=4, num_key_value_heads=1, head_dim=32,
                   linear_num_key_heads=2, linear_key_head_dim=16, linear_num_value_heads=6,
                   linear_value_head_dim=16, output_gate_mode="silu"),
    # the model of the reference's TP test (tests/test_tensor_parallel.py:104-126)
    "tp": dict(vocab_size=500, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
               num_attention_heads=4, num_key_value_heads=2, head_dim=32, linear_num_key_heads=4,
               linear_key_head_dim=16, linear_num_value_heads=12, linear_value_head_dim=16,
               output_gate_mode="silu"),
}

ENGINE_WEIGHT_SEED = {"config1": 11, "prefix": 42, "tp": 2026}

# scheduler scenarios: (model, scheduler kwargs, requests); the requests of a phase are queued
# together and the scheduler is stepped until it is idle (or for `steps` steps)
ENGINE_RUNS: Dict[str, dict] = {
    "config1": dict(model="config1",
                    sched=dict(max_reqs=8, max_context_len=128, max_total_tokens=512,
                               max_snapshots=8, chunked_prefill_size=32),
                    phases=[dict(prompts="config1", max_new_tokens=32)]),
    # reference test_hybrid_scheduler_prefix_reuse_exact_equivalence, its cached scheduler ...
    "prefix_cached": dict(model="prefix",
                          sched=dict(max_reqs=4, max_context_len=32, max_total_tokens=64,
                                     max_snapshots=4, chunked_prefill_size=4),
                          phases=[dict(prompts=[[10, 20, 30, 40, 50, 60]], max_new_tokens=2),
                                  dict(prompts=[[10, 20, 30, 40, 50, 60, 70, 80]],
                                       max_new_tokens=1, steps=1)]),
    # ... and its fresh one, which computes the whole prompt in one step
    "prefix_fresh": dict(model="prefix",
                         sched=dict(max_reqs=4, max_context_len=32, max_total_tokens=64,
                                    max_snapshots=4, chunked_prefill_size=16),
                         phases=[dict(prompts=[[10, 20, 30, 40, 50, 60, 70, 80]],
                                      max_new_tokens=1, steps=1)]),
}


def engine_prompts(name) -> List[List[int]]:
    """Config 1's four prompts: lengths 16/32/48/64 of uniform token ids in [0, 1024), seed 0."""
    if name != "config1":
        return name
    rng = np.random.default_rng(0)
    return [[int(x) for x in rng.integers(0, 1024, n)] for n in (16, 32, 48, 64)]


def engine_weights(shapes: Dict[str, tuple], seed: int) -> Dict[str, np.ndarray]:
    """Seeded float32 weights for a model's state_dict, by parameter name (the same for the
    reference model and the drop-in assembly, which share names): norms 1 + 0.1 N, A_log
    U(0, 1.5), dt_bias 0.5 N, conv taps 0.5 N, embeddings N(0, 1), lm_head N(0, 1/64) (logits of
    a few units, so greedy choices have clear margins), other projections N(0, 1/fan_in)."""
    import zlib

    out = {}
    for name in sorted(shapes):
        shp = tuple(shapes[name])
        rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
        if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            w = 1.0 + 0.1 * rng.standard_normal(shp)
        elif name.endswith("A_log"):
            w = rng.uniform(0.0, 1.5, shp)
        elif name.endswith("dt_bias"):
            w = 0.5 * rng.standard_normal(shp)
        elif "conv1d" in name:
            w = 0.5 * rng.standard_normal(shp)
        elif "embed_tokens" in name:
            w = rng.standard_normal(shp)
        elif name == "lm_head.weight":
            w = rng.standard_normal(shp) / 8.0
        else:
            w = rng.standard_normal(shp) / np.sqrt(shp[-1])
        out[name] = w.astype(np.float32)
    return out


# the reference TP test's batches (tests/test_tensor_parallel.py:181-250): a 2-request prefill
# (4 + 3 tokens) then one decode step
TP_PREFILL = dict(positions=[0, 1, 2, 3, 0, 1, 2], req_pool_indices=[0, 1], seq_lens=[4, 3],
                  prefix_lens=[0, 0], extend_lens=[4, 3], out_cache_loc=[1, 2, 3, 4, 5, 6, 7],
                  rows={0: [1, 2, 3, 4], 1: [5, 6, 7]})
TP_DECODE = dict(positions=[4, 3], req_pool_indices=[0, 1], seq_lens=[5, 4], prefix_lens=[4, 3],
                 extend_lens=[1, 1], out_cache_loc=[8, 9], rows={0: [1, 2, 3, 4, 8],
                                                                 1: [5, 6, 7, 9]})
