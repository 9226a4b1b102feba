"""Record whole runs of the REFERENCE engine as traces the GPU tests replay through the drop-ins.

    python tests/golden/make_engine_golden.py --reference <path to a yz29528/tokenFactory checkout>

The reference engine (Scheduler, ModelRunner, RadixCache, ReqToStatePool and Qwen3_8ForCausalLM,
engine/scheduler.py:34-538, engine/model_runner.py:108-224, radix_tree.py, req_to_state_pool.py,
qwen3_8/causal_lm.py:117-151) runs here on the CPU in fp32 with seeded weights
(tests/golden/cases.py: engine_weights).  Every call of the model's forward is recorded with the
batch it was given (input ids, positions, req_pool_indices, seq_lens, prefix_lens, extend_lens,
out_cache_loc and the request rows of req_to_token), and with the 16 largest logits of each row
(values and ids) plus the row's sum and sum of squares; every GDN state-slot copy or reset the
scheduler and radix tree make through ReqToStatePool (req_to_state_pool.py:120-194) is recorded in
order between them.  The GPU test (tests/test_gpu_engine.py) replays the same events on the
drop-in model and compares logits and greedy tokens: the scheduler's decisions are the recorded
ones, the numbers are the kernels'.

Runs (tests/golden/cases.py: ENGINE_RUNS):
  config1        BASELINE config 1: tiny hybrid model, 4 requests (16/32/48/64 prompt tokens),
                 32 greedy tokens each, chunked prefill mixed with decode; the output gate of
                 qwen3_8/full_attention.py:157-158 swapped to sigmoid (the config's gate)
  prefix_cached  the reference's prefix-reuse test (tests/test_hybrid_radix_cache.py:111-223): a
                 request, then one sharing its first 6 tokens that restores the GDN snapshot and
                 extends over the cached KV prefix
  prefix_fresh   the same second prompt computed from scratch by a fresh scheduler
  tp             the reference's TP test batches (tests/test_tensor_parallel.py:93-271) through
                 the tp_size=1 model: prefill and decode logits and the GDN states after prefill

Writes tests/golden/engine_golden.npz.
"""

import argparse
import contextlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import cases as C  # noqa: E402

TOPK = 16


def _config(ref_root: str, model: str, **over):
    from dataclasses import replace

    from qwen3_8 import Qwen3_8Config

    base = Qwen3_8Config.from_json_file(os.path.join(ref_root, "qwen3.8 27B", "config.json"))
    dims = {k: v for k, v in C.ENGINE_MODELS[model].items() if k != "output_gate_mode"}
    layer_types = ["full_attention" if (i + 1) % 4 == 0 else "linear_attention"
                   for i in range(dims["num_hidden_layers"])]
    return replace(base, layer_types=layer_types, quantization_config=None, **dims, **over)


def _set_weights(model, name: str) -> None:
    sd = model.state_dict()
    w = C.engine_weights({k: tuple(v.shape) for k, v in sd.items()}, C.ENGINE_WEIGHT_SEED[name])
    model.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()})


@contextlib.contextmanager
def _gate(mode: str):
    """The output gate of qwen3_8/full_attention.py:157-158 is `attn * F.silu(gate)`; for the
    sigmoid gate of BASELINE config 1 that one name is pointed at torch.sigmoid (the module's `F`
    is swapped for a namespace that differs from torch.nn.functional only in `silu`)."""
    import qwen3_8.full_attention as FA

    if mode == "silu":
        yield
        return
    real = FA.F
    ns = types.SimpleNamespace(**{k: getattr(real, k) for k in dir(real) if not k.startswith("__")})
    ns.silu = torch.sigmoid
    FA.F = ns
    try:
        yield
    finally:
        FA.F = real


class Recorder:
    """Wraps a scheduler's model forward and its state pool's slot operations."""

    def __init__(self):
        self.events = []    # (kind, a, b): 0 forward #a, 1 zero slot a, 2 copy slot a -> slot b
        self.forwards = []

    def attach(self, scheduler) -> None:
        model = scheduler.model_runner.model
        orig = model.forward

        def forward(input_ids, positions, cache_pool, forward_batch, return_all_logits=False):
            logits = orig(input_ids, positions, cache_pool, forward_batch, return_all_logits)
            self._forward(input_ids, positions, forward_batch, logits)
            return logits

        model.forward = forward
        pool = scheduler.req_to_state_pool
        real = {n: getattr(pool, n) for n in ("reset_working_state", "free_snapshot",
                                              "capture_snapshot", "restore_snapshot")}

        def reset_working_state(req_idx):
            self.events.append((1, int(req_idx), -1))
            return real["reset_working_state"](req_idx)

        def free_snapshot(slot):
            self.events.append((1, int(slot), -1))
            return real["free_snapshot"](slot)

        def capture_snapshot(req_idx, snapshot_slot, debug_tag=None):
            self.events.append((2, int(req_idx), int(snapshot_slot)))
            return real["capture_snapshot"](req_idx, snapshot_slot, debug_tag)

        def restore_snapshot(snapshot_slot, req_idx):
            self.events.append((2, int(snapshot_slot), int(req_idx)))
            return real["restore_snapshot"](snapshot_slot, req_idx)

        pool.reset_working_state = reset_working_state
        pool.free_snapshot = free_snapshot
        pool.capture_snapshot = capture_snapshot
        pool.restore_snapshot = restore_snapshot

    def _forward(self, input_ids, positions, fb, logits) -> None:
        rpi = fb.req_pool_indices.cpu().numpy().astype(np.int64)
        seq = fb.seq_lens.cpu().numpy().astype(np.int64)
        maxl = int(seq.max())
        r2t = fb.req_to_token[torch.as_tensor(rpi), :maxl].cpu().numpy().astype(np.int64)
        lg = logits.detach().double().cpu().numpy()
        order = np.argsort(-lg, axis=1, kind="stable")[:, :TOPK]
        self.events.append((0, len(self.forwards), -1))
        self.forwards.append(dict(
            input_ids=input_ids.cpu().numpy().astype(np.int64),
            positions=positions.cpu().numpy().astype(np.int64),
            req_pool_indices=rpi, seq_lens=seq,
            prefix_lens=fb.prefix_lens.cpu().numpy().astype(np.int64),
            extend_lens=np.asarray(fb.extend_lens, np.int64),
            out_cache_loc=fb.out_cache_loc.cpu().numpy().astype(np.int64), r2t=r2t,
            top_idx=order.astype(np.int64),
            top_val=np.take_along_axis(lg, order, axis=1).astype(np.float32),
            row_sum=lg.sum(axis=1), row_sq=(lg * lg).sum(axis=1),
            tokens=lg.argmax(axis=1).astype(np.int64)))


def run_scheduler(ref_root: str, name: str) -> dict:
    from engine.request import Request
    from engine.scheduler import Scheduler

    spec = C.ENGINE_RUNS[name]
    model = spec["model"]
    cfg = _config(ref_root, model)
    torch.manual_seed(0)
    sched = Scheduler(config=cfg, device="cpu", **spec["sched"])
    _set_weights(sched.model_runner.model, model)
    rec = Recorder()
    rec.attach(sched)
    outputs, cached = [], []
    with _gate(C.ENGINE_MODELS[model]["output_gate_mode"]), torch.inference_mode():
        for p, phase in enumerate(spec["phases"]):
            reqs = [Request(req_id=f"{name}-{p}-{i}", prompt_text="", prompt_ids=ids,
                            max_new_tokens=phase["max_new_tokens"], temperature=0.0)
                    for i, ids in enumerate(C.engine_prompts(phase["prompts"]))]
            sched.waiting_queue.extend(reqs)
            n = 0
            while sched.waiting_queue or sched.inflight_prefill_queue or sched.running_batch:
                out = sched.step()
                n += 1
                if out is not None and getattr(out, "cached_prefix_lens", None):
                    cached.append([int(x) for x in out.cached_prefix_lens])
                if phase.get("steps") and n >= phase["steps"]:
                    break
            outputs.append([list(map(int, r.output_ids)) for r in reqs])
    arrays = {}
    for i, f in enumerate(rec.forwards):
        for k, v in f.items():
            arrays[f"{name}/fwd{i}/{k}"] = v
    arrays[f"{name}/events"] = np.asarray(rec.events, np.int64).reshape(-1, 3)
    margins = [float(f["top_val"][r, 0] - f["top_val"][r, 1]) for f in rec.forwards
               for r in range(f["top_val"].shape[0])]
    meta = dict(model=model, sched=spec["sched"], outputs=outputs, cached_prefix_lens=cached,
                num_forwards=len(rec.forwards), min_top2_margin=min(margins),
                state_dict_keys=sorted(sched.model_runner.model.state_dict().keys()),
                state_pool_slots=int(sched.req_to_state_pool.total_slots))
    arrays[f"{name}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    print(f"{name}: {len(rec.forwards)} forwards, {len(rec.events)} events, outputs {outputs}, "
          f"cached {cached}, min top-2 margin {min(margins):.3g}")
    return arrays


def tp_golden(ref_root: str) -> dict:
    from qwen3_8 import ForwardBatch
    from qwen3_8.causal_lm import Qwen3_8ForCausalLM
    from qwen3_8.hybrid_cache_pool import Qwen3_8HybridCachePool

    cfg = _config(ref_root, "tp", tp_size=1, tp_rank=0)
    model = Qwen3_8ForCausalLM(cfg).eval()
    _set_weights(model, "tp")
    pool = Qwen3_8HybridCachePool(cfg, max_reqs=4, max_total_tokens=32, max_snapshots=4,
                                  dtype=torch.float32)
    ids = np.random.default_rng(2026).integers(0, cfg.vocab_size, 7).astype(np.int64)
    r2t = torch.full((4, 16), -1, dtype=torch.long)

    def batch(b):
        for r, row in b["rows"].items():
            r2t[r, :len(row)] = torch.tensor(row)
        return ForwardBatch(batch_size=2, req_pool_indices=torch.tensor(b["req_pool_indices"]),
                            seq_lens=torch.tensor(b["seq_lens"]),
                            prefix_lens=torch.tensor(b["prefix_lens"]),
                            extend_lens=list(b["extend_lens"]),
                            out_cache_loc=torch.tensor(b["out_cache_loc"]), req_to_token=r2t,
                            is_prefill=max(b["extend_lens"]) > 1)

    with torch.inference_mode():
        pre = model(torch.from_numpy(ids), torch.tensor(C.TP_PREFILL["positions"]), pool,
                    batch(C.TP_PREFILL))
        ssm = pool.ssm_state[:, :2].clone()
        dec_ids = torch.argmax(pre, dim=-1)
        dec = model(dec_ids, torch.tensor(C.TP_DECODE["positions"]), pool, batch(C.TP_DECODE))
    print(f"tp: prefill logits {tuple(pre.shape)}, decode ids {dec_ids.tolist()}")
    return {"tp/input_ids": ids, "tp/prefill_logits": pre.numpy().astype(np.float32),
            "tp/decode_ids": dec_ids.numpy().astype(np.int64),
            "tp/decode_logits": dec.numpy().astype(np.float32),
            "tp/ssm_state_after_prefill": ssm.numpy().astype(np.float32),
            "tp/state_dict_keys": np.frombuffer(json.dumps(sorted(model.state_dict().keys()))
                                                .encode(), dtype=np.uint8)}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True,
                    help="root of a yz29528/tokenFactory checkout")
    args = ap.parse_args()
    root = os.path.abspath(args.reference)
    sys.path.insert(0, root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    arrays = {}
    for name in C.ENGINE_RUNS:
        arrays.update(run_scheduler(root, name))
    arrays.update(tp_golden(root))
    f = os.path.join(HERE, "engine_golden.npz")
    np.savez_compressed(f, **arrays)
    print(os.path.basename(f), os.path.getsize(f), "bytes")


if __name__ == "__main__":
    main()
