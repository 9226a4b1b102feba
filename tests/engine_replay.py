"""Replay of recorded reference-engine runs (tests/golden/engine_golden.npz) on the drop-in model.

tests/golden/make_engine_golden.py records what the reference's Scheduler did on the CPU: every
model forward with its batch, and every GDN state-slot copy or reset in between.  ``replay`` runs
the same events on tokenfactory_b200.hybrid_model (the kernels through the drop-in layers) with the
same seeded weights and returns, per forward, the logits at the recorded top-16 ids and the greedy
token, so the tests can hold them to the reference's.
"""

import json
import os

import numpy as np

from tests.golden import cases as C

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "engine_golden.npz")
_Z = {}


def fixture():
    if "z" not in _Z:
        _Z["z"] = np.load(FIXTURE)
    return _Z["z"]


def meta(run: str) -> dict:
    return json.loads(bytes(fixture()[f"{run}/meta"]).decode())


def forwards(run: str):
    z, m = fixture(), meta(run)
    keys = ("input_ids", "positions", "req_pool_indices", "seq_lens", "prefix_lens",
            "extend_lens", "out_cache_loc", "r2t", "top_idx", "top_val", "row_sum", "row_sq",
            "tokens")
    return [{k: z[f"{run}/fwd{i}/{k}"] for k in keys} for i in range(m["num_forwards"])]


def events(run: str) -> np.ndarray:
    return fixture()[f"{run}/events"]


def hybrid_config(model: str, tp_size: int = 1, tp_rank: int = 0):
    from tokenfactory_b200.hybrid_model import HybridConfig
    return HybridConfig(tp_size=tp_size, tp_rank=tp_rank, **C.ENGINE_MODELS[model])


def build_model(model: str, device="cuda", tp_size: int = 1, tp_rank: int = 0, full=None):
    """The drop-in model with the fixture's seeded weights (fp32); with tp_size > 1 this rank's
    shard of `full` (a tp_size=1 model), as the reference's load_tp_from_full_model does."""
    import torch
    from tokenfactory_b200.hybrid_model import HybridForCausalLM

    m = HybridForCausalLM(hybrid_config(model, tp_size, tp_rank)).to(device).eval()
    if full is not None:
        m.load_tp_from_full_model(full)
        return m
    shapes = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    w = C.engine_weights(shapes, C.ENGINE_WEIGHT_SEED[model])
    m.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()})
    return m


def replay(run: str, device="cuda"):
    """Replay one recorded run; returns [(logits at top_idx, greedy tokens, full logits)]."""
    import torch
    from tokenfactory_b200 import ForwardBatch, ops
    from tokenfactory_b200.hybrid_model import HybridCachePool

    m = meta(run)
    sched = m["sched"]
    model = build_model(m["model"], device)
    cfg = model.config
    pool = HybridCachePool(cfg, sched["max_total_tokens"], sched["max_reqs"],
                           sched["max_snapshots"], dtype=torch.float32, device=device)
    assert pool.conv_state.shape[1] == m["state_pool_slots"]
    r2t = torch.full((sched["max_reqs"], sched["max_context_len"]), -1, dtype=torch.long,
                     device=device)
    fwd = forwards(run)
    out = []
    for kind, a, b in events(run).tolist():
        if kind == 1:    # zero a GDN state slot in every linear layer (reset / free)
            ops.state_slots_copy(pool.conv_state, pool.ssm_state, [None], [a])
        elif kind == 2:  # copy slot a into slot b (capture / restore)
            ops.state_slots_copy(pool.conv_state, pool.ssm_state, [a], [b])
        else:
            f = fwd[a]
            for i, r in enumerate(f["req_pool_indices"].tolist()):
                n = int(f["seq_lens"][i])
                r2t[r, :n] = torch.from_numpy(f["r2t"][i, :n]).to(device)
            t = {k: torch.from_numpy(f[k]).to(device) for k in
                 ("input_ids", "positions", "req_pool_indices", "seq_lens", "prefix_lens",
                  "out_cache_loc")}
            ext = [int(x) for x in f["extend_lens"]]
            fb = ForwardBatch(batch_size=len(ext), req_pool_indices=t["req_pool_indices"],
                              seq_lens=t["seq_lens"], prefix_lens=t["prefix_lens"],
                              extend_lens=ext, out_cache_loc=t["out_cache_loc"],
                              req_to_token=r2t, is_prefill=max(ext) > 1,
                              max_seq_len=int(f["seq_lens"].max()), max_extend_len=max(ext))
            logits = model(t["input_ids"], t["positions"], pool, fb)
            idx = torch.from_numpy(f["top_idx"]).to(device)
            out.append((torch.gather(logits, 1, idx).cpu().numpy(),
                        logits.argmax(dim=1).cpu().numpy(), logits.double().cpu().numpy()))
    return out
