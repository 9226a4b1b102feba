"""Benchmark of the B200 hybrid-attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5|6] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU, NCCL)

Default line (the configuration the headline metric is quoted on): paged GQA
decode, bf16, 128 requests, 32 q heads / 4 kv heads, head_dim 256, seq_lens ~ U[512, 8192],
token-granular pages: each request's slots are a random draw from a 1.2M-slot pool (slot 0
reserved), q and K/V ~ N(0,1), sigmoid output gate from N(0,1) logits, scale 1/16.  One step = the
decode step of one full-attention layer: KV store of the new token (a1) + paged decode with fused
gate (a2, a4).  With N GPUs the heads are sharded exactly like the reference's tensor-parallel
split (qwen3_8/full_attention.py:43-52, kv heads replicated once N > 4) and every rank decodes the
whole batch for its heads: total work is fixed, so scaling is "strong"; `value` is the whole job's
tokens/s, `value_per_gpu` beside it.  The rest of the metric rides in the same line, each leg timed
on its own: `gdn_decode` (config 3: Gated DeltaNet recurrent decode, B=256, Hk=16, Hv=48,
dk=dv=128, fp32 state) and `extend` (config 4: 16 requests, prefix U[0,4096], extend U[512,2048]:
causal extend attention in TFLOP/s, the GDN extend of the same tokens, the fused prologue and the
admission-time state snapshots).
--config 3 / 4: those legs alone, with their own headline.
--config 5: the 27B-shape hybrid model end to end (256 requests x (1024 + 256) tokens).
--config 6: the block-FP8 GEMM of the 27B MLP up projection.

Timing: W warm-up steps, then K steps between CUDA events on the launching stream, bracketed by a
barrier and synchronize; the max over ranks is reported.  The K/V read per step (2.3 GB) is far
larger than L2, so no flush is needed.  `e2e` repeats the measurement through the public API with
the step's inputs copied from pinned host memory and its output copied back inside the timed
region, the copies of neighbouring steps overlapping the kernels (runner.PipelinedStep);
`e2e_serial` is the same with the copies in series, `e2e_eager` the step issued call by call.
`cpu_baseline` times the CPU oracle (a restatement of the reference's torch algorithm, pinned to
its outputs) on a bounded sample on this host's cores; `--impl reference` times only that.
"""

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode attn tok/s/GPU + % of 8 TB/s HBM; extend attn TFLOP/s; 1/2/4/8 GPU"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------------------------------------
# environment
# ---------------------------------------------------------------------------------------------
def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    """SM clocks and throttle reasons sampled while the timed region runs: NVML read back to back
    from a thread (two calls a sample, about 0.7 ms; the calls release the GIL, so the thread keeps
    sampling while the main thread waits for the device), with nvidia-smi at 100 ms as the
    fallback when NVML cannot be loaded.  Reads only."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._stop = threading.Event()
        self._thread = None
        self._max_mhz = 0

    def _nvml_sample(self, handle, nv) -> bool:
        try:
            sm = nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(handle)
            self.lines.append(f"{sm}, {self._max_mhz}, 0, {bits:#x}")
            return True
        except Exception:  # noqa: BLE001 - a failed read is just a missing sample
            return False

    def _nvml_loop(self, handle, nv):
        while not self._stop.is_set():
            if not self._nvml_sample(handle, nv):
                time.sleep(0.001)  # a failing read must not spin on the interpreter lock

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            idx = torch.cuda._get_nvml_device_index(self.gpu)
            handle = nv.nvmlDeviceGetHandleByIndex(idx)
            self._max_mhz = nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM)  # fixed
            self._nvml = (handle, nv)
            self._thread = threading.Thread(target=self._nvml_loop, args=(handle, nv), daemon=True)
            self._thread.start()
            return self
        except Exception:  # noqa: BLE001 - no NVML: fall back to nvidia-smi
            self._thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            if not self.lines:  # a region too short for the thread to be scheduled: one read now
                self._nvml_sample(*self._nvml)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 4:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
                bits = int(parts[3], 16)
            except ValueError:
                continue
            for bit, name in _REASONS.items():
                if bits & bit and name != "gpu_idle":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# dram__bytes_read.sum + dram__bytes_write.sum per launch of each leg's dominant kernel, from an
# ncu capture of exactly that leg's default workload on one GPU (the commands and the figures are
# in profiles/).  A run with other sizes or more GPUs reports null: its traffic was not measured.
NCU_TRAFFIC_N1 = {"decode": 2_297_680_000, "gdn_decode": 1_593_400_000, "extend": 1_199_900_000}


# ---------------------------------------------------------------------------------------------
# config 2: paged GQA decode
# ---------------------------------------------------------------------------------------------
C2 = dict(B=128, Hq=32, Hkv=4, D=256, Lmin=512, Lmax=8192, slots=1_200_000)
E2E_WARM = 100  # untimed steps before each e2e leg of config 2 (see bench_decode)


def _tp_heads(hq, hkv, rank, world):
    """Local q heads and kv heads under the reference's TP split (tokenfactory_b200.tp)."""
    from tokenfactory_b200.tp import head_shard
    sh = head_shard(hq, hkv, world, world, rank, world)
    return len(sh.q_heads), len(sh.kv_heads)


def _decode_inputs(seed: int, rank: int, world: int, dev):
    B, Hq, Hkv, D, S = C2["B"], C2["Hq"], C2["Hkv"], C2["D"], C2["slots"]
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(C2["Lmin"], C2["Lmax"] + 1, (B,), generator=gen)
    if int(lens.sum()) > S - 1:
        raise ValueError(f"pool of {S} slots too small for {int(lens.sum())} tokens")
    perm = torch.randperm(S - 1, generator=gen)[: int(lens.sum())] + 1
    r2t = torch.full((B, C2["Lmax"]), -1, dtype=torch.int64)
    off = 0
    for b in range(B):
        n = int(lens[b])
        r2t[b, :n] = perm[off:off + n]
        off += n
    lq, lkv = _tp_heads(Hq, Hkv, rank, world)
    g = torch.Generator(device=dev).manual_seed(seed + 1 + rank)
    kb = torch.randn((S, lkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    vb = torch.randn((S, lkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn((B, lq, D), generator=g, device=dev, dtype=torch.bfloat16)
    gate = torch.randn((B, lq, D), generator=g, device=dev, dtype=torch.bfloat16)
    knew = torch.randn((B, lkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    vnew = torch.randn((B, lkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    out_loc = r2t[torch.arange(B), lens - 1].clone()
    return dict(lens=lens, r2t=r2t, kb=kb, vb=vb, q=q, gate=gate, knew=knew, vnew=vnew,
                out_loc=out_loc, lq=lq, lkv=lkv)


def _decode_bytes(lens, lq, lkv, D):
    """Algorithmic HBM bytes of one decode launch: K+V rows of every visible token, the int64
    req_to_token entries, and q, gate, out."""
    sl = int(lens.sum())
    return sl * lkv * D * 2 * 2 + sl * 8 + 3 * len(lens) * lq * D * 2


def bench_decode(args, rank, world, dev):
    from tokenfactory_b200 import ops

    inp = _decode_inputs(0, rank, args.head_split or world, dev)
    B, D = C2["B"], C2["D"]
    lens_d = inp["lens"].to(dev)
    r2t_d = inp["r2t"].to(dev)
    rpi_d = torch.arange(B, dtype=torch.int64, device=dev)
    loc_d = inp["out_loc"].to(dev)
    scale = D ** -0.5
    maxL = int(inp["lens"].max())
    out = torch.empty_like(inp["q"])
    stream = torch.cuda.current_stream()

    def step():
        ops.kv_store(inp["kb"], inp["vb"], loc_d, inp["knew"], inp["vnew"])
        ops.paged_decode(inp["q"], inp["kb"], inp["vb"], r2t_d, rpi_d, lens_d, scale, maxL,
                         gate=inp["gate"], gate_mode="sigmoid", out=out)

    for _ in range(args.warmup):
        step()
    # device time of the whole step, plus of the decode call alone (roofline)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            e_a, e_b, e_c = ev[i]
            e_a.record(stream)
            ops.kv_store(inp["kb"], inp["vb"], loc_d, inp["knew"], inp["vnew"])
            e_b.record(stream)
            ops.paged_decode(inp["q"], inp["kb"], inp["vb"], r2t_d, rpi_d, lens_d, scale, maxL,
                             gate=inp["gate"], gate_mode="sigmoid", out=out)
            e_c.record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
    _barrier(world)
    elapsed = _max_over_ranks(t0.elapsed_time(t1) / 1e3, world)
    dec_s = sum(e_b.elapsed_time(e_c) for _, e_b, e_c in ev) / 1e3 / args.steps
    dec_s = _max_over_ranks(dec_s, world)

    hbm, peak_kind = _peaks()
    nbytes = _decode_bytes(inp["lens"], inp["lq"], inp["lkv"], D)
    achieved = nbytes / dec_s / 1e9
    if args.no_e2e:
        return dict(value=B * args.steps / elapsed, ms=elapsed / args.steps * 1e3,
                    achieved_gbs=achieved, frac=achieved / hbm)

    # e2e through the public API: per-step inputs from pinned host memory, output back to host
    h_q = inp["q"].cpu().pin_memory()
    h_gate = inp["gate"].cpu().pin_memory()
    h_k, h_v = inp["knew"].cpu().pin_memory(), inp["vnew"].cpu().pin_memory()
    h_loc = inp["out_loc"].pin_memory()
    h_rpi = torch.arange(B, dtype=torch.int64).pin_memory()
    h_lens = inp["lens"].pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d_q, d_gate = torch.empty_like(inp["q"]), torch.empty_like(inp["gate"])
    d_k, d_v = torch.empty_like(inp["knew"]), torch.empty_like(inp["vnew"])
    d_loc, d_rpi, d_lens = torch.empty_like(loc_d), torch.empty_like(rpi_d), torch.empty_like(lens_d)
    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_gate, h_k, h_v, h_loc, h_rpi, h_lens))
    d2h = h_out.numel() * h_out.element_size()

    def e2e_step():
        for d, h in ((d_q, h_q), (d_gate, h_gate), (d_k, h_k), (d_v, h_v), (d_loc, h_loc),
                     (d_rpi, h_rpi), (d_lens, h_lens)):
            d.copy_(h, non_blocking=True)
        ops.kv_store(inp["kb"], inp["vb"], d_loc, d_k, d_v)
        ops.paged_decode(d_q, inp["kb"], inp["vb"], r2t_d, d_rpi, d_lens, scale, maxL,
                         gate=d_gate, gate_mode="sigmoid", out=out)
        h_out.copy_(out, non_blocking=True)

    # each e2e leg starts after host-side set-up (pinned buffers, graph capture) during which the
    # GPU idles and its clocks drop; E2E_WARM steps (about 50 ms of work) bring them back before
    # the timed steps, which a short timed region would otherwise start on
    for _ in range(max(E2E_WARM, args.warmup)):
        e2e_step()
    _barrier(world)
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    e2e_s = _max_over_ranks(s0.elapsed_time(s1) / 1e3, world)

    # the same e2e step captured once as a CUDA graph (runner.CapturedStep): the copies from the
    # pinned host buffers, the KV store, the decode and the copy back replay as one graph
    from tokenfactory_b200.runner import CapturedStep

    def e2e_body():
        e2e_step()
        return None

    cap = CapturedStep(lambda: e2e_body(), {}, warmup=max(3, args.warmup))
    for _ in range(max(E2E_WARM, args.warmup)):
        cap()
    _barrier(world)
    torch.cuda.synchronize()
    s0.record(stream)
    for _ in range(args.steps):
        cap()
    s1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    e2e_graph_s = _max_over_ranks(s0.elapsed_time(s1) / 1e3, world)
    del cap

    # the same step streamed through runner.PipelinedStep: two buffer sets, each a captured graph;
    # step i+1's inputs are copied in and step i-1's output copied out while step i computes
    from tokenfactory_b200.runner import PipelinedStep

    def e2e_fn(q, gate, knew, vnew, loc, rpi, lens):
        ops.kv_store(inp["kb"], inp["vb"], loc, knew, vnew)
        return ops.paged_decode(q, inp["kb"], inp["vb"], r2t_d, rpi, lens, scale, maxL,
                                gate=gate, gate_mode="sigmoid")

    host_in = dict(q=h_q, gate=h_gate, knew=h_k, vnew=h_v, loc=h_loc, rpi=h_rpi, lens=h_lens)
    pipe = PipelinedStep(e2e_fn, host_in, warmup=max(3, args.warmup))
    for _ in range(max(E2E_WARM, args.warmup)):
        pipe.submit(**host_in)
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    s0.record(stream)
    pipe.fence()
    last = None
    for _ in range(args.steps):
        last = pipe.submit(**host_in)
    pipe.join()
    s1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    e2e_pipe_s = _max_over_ranks(s0.elapsed_time(s1) / 1e3, world)
    if not torch.equal(last.wait().to(dev), out):
        raise RuntimeError("pipelined e2e step output differs from the device-timed step's")
    del pipe

    rt = _step_runtime(B, dev, stream)

    default_size = (B, C2["slots"]) == (128, 1_200_000)
    traffic = NCU_TRAFFIC_N1["decode"] if world == 1 and default_size else None
    res = {
        "metric": METRIC, "value": B * args.steps / elapsed, "unit": "tok/s",
        "value_per_gpu": B * args.steps / elapsed / world,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2 paged GQA decode (one full-attention layer step)",
                   "value": "whole-job tokens/s over all GPUs (each rank decodes every request "
                            "for its heads); value_per_gpu = value / n_gpus",
                   "batch": B, "q_heads": C2["Hq"], "kv_heads": C2["Hkv"], "head_dim": D,
                   "seq_len": f"U[{C2['Lmin']},{C2['Lmax']}]", "sum_seq_len": int(inp["lens"].sum()),
                   "pool_slots": C2["slots"], "page_size": 1, "gate": "sigmoid",
                   "parallelism": f"tp{world}", "local_q_heads": inp["lq"],
                   "local_kv_heads": inp["lkv"],
                   "l2": "no flush: each step reads 2.3 GB of K/V, far above the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": peak_kind,
                     "kernel": "tf_paged_decode_attn (plan + decode + combine)",
                     "bytes_per_launch": nbytes,
                     "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS,
                     "traffic": traffic},
        "e2e": {"value": B * args.steps / e2e_pipe_s, "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "how": "per step: 7 copies from pinned host buffers, KV store, paged decode, "
                       "copy of the output to pinned host memory (runner.PipelinedStep: two "
                       "buffer sets each replayed as a CUDA graph, copies on two copy streams, "
                       "so step i+1's inputs and step i-1's output cross PCIe while step i "
                       "computes); every step's copies lie inside the timed region"},
        "e2e_serial": {"value": B * args.steps / e2e_graph_s, "unit": "tok/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "how": "the same step as one CUDA graph per step, copies in series with "
                              "the kernels (runner.CapturedStep)"},
        "e2e_eager": {"value": B * args.steps / e2e_s, "unit": "tok/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "how": "the same step issued call by call from Python"},
        "step_runtime": rt,
        "gpu_launches": 4 * args.steps,
        "clocks": clk.summary(),
    }
    return res


def _step_runtime(B: int, dev, stream, vocab: int = 248320, reps: int = 20) -> dict:
    """Host + device wall time of the per-step runtime at a decode batch of B requests: building
    the ForwardBatch (runner.prepare_forward_batch: one packed copy + one sync launch) and
    sampling B rows of a 27B-vocabulary logits matrix (runner.sample: one launch, one copy back),
    each beside the reference's sequence restated in torch (engine/model_runner.py:108-188: one
    torch.tensor copy per field and one slice assignment per request; :574-581: one argmax and
    one .item() per row).  Wall clock, synchronised on both sides, median of `reps`."""
    import time
    from types import SimpleNamespace

    from tokenfactory_b200 import runner as R

    rng = np.random.default_rng(7)
    max_ctx = 8192
    r2t = torch.full((B, max_ctx), -1, dtype=torch.int64, device=dev)
    lens = rng.integers(512, max_ctx - 1, B)
    reqs = [SimpleNamespace(req_pool_idx=b, cur_start_pos=int(lens[b]), cur_seq_len=int(lens[b]) + 1,
                            cur_chunk_tokens=[int(rng.integers(0, vocab))],
                            out_cache_loc=[int(rng.integers(1, 1 << 20))], is_prefilled=True,
                            temperature=0.0) for b in range(B)]
    table = [[0] * max_ctx for _ in range(B)]

    def ours():
        synced = [int(l) for l in lens]
        R.prepare_forward_batch(reqs, table, r2t, synced)

    def torch_ref():
        ids = torch.tensor([t for r in reqs for t in r.cur_chunk_tokens], dtype=torch.long, device=dev)
        pos = torch.tensor([r.cur_start_pos for r in reqs], dtype=torch.long, device=dev)
        loc = torch.tensor([l for r in reqs for l in r.out_cache_loc], dtype=torch.long, device=dev)
        for i, r in enumerate(reqs):
            r2t[r.req_pool_idx, r.cur_start_pos:r.cur_seq_len] = loc[i:i + 1]
        for f in ("req_pool_idx", "cur_seq_len", "cur_start_pos"):
            torch.tensor([getattr(r, f) for r in reqs], dtype=torch.long, device=dev)
        torch.tensor([1] * B, dtype=torch.long, device=dev)
        return ids, pos

    g = torch.Generator(device=dev).manual_seed(9)
    logits = torch.randn((B, vocab), generator=g, device=dev, dtype=torch.bfloat16)

    def sample_ours():
        R.sample(logits, [0.0] * B)

    def sample_torch():
        return [int(torch.argmax(logits[i], dim=-1).item()) for i in range(B)]

    def wall(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(reps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        return float(np.median(ts)) * 1e3

    return {"batch": B, "vocab": vocab, "prepare_ms": wall(ours), "prepare_torch_ms": wall(torch_ref),
            "sample_ms": wall(sample_ours), "sample_torch_ms": wall(sample_torch),
            "how": "wall clock with a synchronize on both sides, median of 20"}


# ---------------------------------------------------------------------------------------------
# config 3: GDN recurrent decode
# ---------------------------------------------------------------------------------------------
C3 = dict(B=256, Hk=16, Hv=48, dk=128, dv=128, K=4, slots=512)


def bench_gdn_decode(args, rank, world, dev):
    from tokenfactory_b200 import ops

    B, dk, dv, K = C3["B"], C3["dk"], C3["dv"], C3["K"]
    hk, hv = C3["Hk"] // world, C3["Hv"] // world
    conv_dim = 2 * hk * dk + hv * dv
    g = torch.Generator(device=dev).manual_seed(3 + rank)
    bf = torch.bfloat16
    S = C3["slots"]
    ssm = torch.randn((S, hv, dk, dv), generator=g, device=dev) * 0.02
    conv = torch.randn((S, conv_dim, K - 1), generator=g, device=dev, dtype=bf)
    rpi = torch.randperm(S, generator=torch.Generator().manual_seed(4))[:B].to(dev)
    qkv = torch.randn((B, conv_dim), generator=g, device=dev, dtype=bf)
    bb = torch.randn((B, hv), generator=g, device=dev, dtype=bf)
    aa = torch.randn((B, hv), generator=g, device=dev, dtype=bf)
    z = torch.randn((B, hv * dv), generator=g, device=dev, dtype=bf)
    w = torch.randn((conv_dim, 1, K), generator=g, device=dev, dtype=bf) * 0.5
    A_log = (torch.rand((hv,), generator=g, device=dev) * 1.5).to(bf)
    dt_bias = torch.randn((hv,), generator=g, device=dev, dtype=bf) * 0.5
    nw = torch.ones((hv * dv,), device=dev, dtype=bf)
    out = torch.empty((B, hv * dv), device=dev, dtype=bf)

    def step():
        ops.gdn_decode(qkv, bb, aa, w, A_log, dt_bias, conv, ssm, rpi, num_k_heads=hk,
                       head_k_dim=dk, head_v_dim=dv, z=z, norm_weight=nw, out=out)

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.current_stream()
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
    _barrier(world)
    el = _max_over_ranks(t0.elapsed_time(t1) / 1e3, world)
    nbytes = (B * hv * dk * dv * 4 * 2 + B * conv_dim * (K - 1) * 2 * 2 + B * conv_dim * 2 +
              B * hv * dv * 2 * 2 + 2 * B * hv * 2)
    hbm, peak_kind = _peaks()
    achieved = nbytes / (el / args.steps) / 1e9
    return {
        "metric": "GDN recurrent decode tok/s", "value": B * args.steps / el, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config3 GDN recurrent decode", "batch": B, "k_heads": C3["Hk"],
                   "v_heads": C3["Hv"], "dk": dk, "dv": dv, "parallelism": f"tp{world}",
                   "l2": "no flush: each step streams 1.6 GB of fp32 state"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": peak_kind,
                     "kernel": "tf_gdn_decode", "bytes_per_launch": nbytes,
                     "traffic": NCU_TRAFFIC_N1["gdn_decode"] if world == 1 else None},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }


# ---------------------------------------------------------------------------------------------
# config 4: extend / prefill over a radix-cached prefix
# ---------------------------------------------------------------------------------------------
C4 = dict(B=16, Pmax=4096, Emin=512, Emax=2048, Hq=32, Hkv=4, D=256, Hk=16, Hv=48, dk=128,
          dv=128, K=4, slots=1_200_000)


def _peak_tflops(timed_region_s: float = 0.0):
    """bf16 dense peak: the burst figure for a kernel timed in a short region, the sustained one
    (the GPU settles at its power cap within about a second of dense tensor work) when the timed
    region of back-to-back launches lasts longer than that."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peaks = json.load(f)
        if timed_region_s > 1.0 and "bf16_tflops_sustained" in peaks:
            return float(peaks["bf16_tflops_sustained"]), "measured (sustained)"
        return float(peaks["bf16_tflops"]), "measured (burst)"
    return (1400.0, "fallback (sustained)") if timed_region_s > 1.0 else (1590.0, "fallback (burst)")


def bench_extend(args, rank, world, dev):
    from tokenfactory_b200 import ops
    from tokenfactory_b200.tp import head_shard

    B, D = args.requests, C4["D"]
    sh = head_shard(C4["Hq"], C4["Hkv"], C4["Hk"], C4["Hv"], rank, world)
    hq, hkv, hk, hv = len(sh.q_heads), len(sh.kv_heads), len(sh.k_heads), len(sh.v_heads)
    gen = torch.Generator().manual_seed(4)
    P = torch.randint(0, C4["Pmax"] + 1, (max(B, C4["B"]),), generator=gen)[:B]
    E = torch.randint(C4["Emin"], C4["Emax"] + 1, (max(B, C4["B"]),), generator=gen)[:B]
    L = P + E
    T = int(E.sum())
    S = args.ext_pool_slots
    perm = torch.randperm(S - 1, generator=gen)[: int(L.sum())] + 1
    Lmax = int(L.max())
    r2t = torch.full((B, Lmax), -1, dtype=torch.int64)
    off = 0
    for b in range(B):
        r2t[b, :int(L[b])] = perm[off:off + int(L[b])]
        off += int(L[b])
    out_loc = torch.cat([r2t[b, int(P[b]):int(L[b])] for b in range(B)])
    g = torch.Generator(device=dev).manual_seed(40 + rank)
    bf = torch.bfloat16
    kb = torch.randn((S, hkv, D), generator=g, device=dev, dtype=bf)
    vb = torch.randn((S, hkv, D), generator=g, device=dev, dtype=bf)
    q = torch.randn((T, hq, D), generator=g, device=dev, dtype=bf)
    gate = torch.randn((T, hq, D), generator=g, device=dev, dtype=bf)
    knew = torch.randn((T, hkv, D), generator=g, device=dev, dtype=bf)
    vnew = torch.randn((T, hkv, D), generator=g, device=dev, dtype=bf)
    r2t_d, loc_d = r2t.to(dev), out_loc.to(dev)
    rpi = torch.arange(B, dtype=torch.int64, device=dev)
    L_d, E_d = L.to(dev), E.to(dev)
    attn_out = torch.empty_like(q)
    # GDN extend inputs for the same requests (state resident at their pool rows)
    dk, dv, K = C4["dk"], C4["dv"], C4["K"]
    conv_dim = 2 * hk * dk + hv * dv
    ssm = torch.randn((2 * B, hv, dk, dv), generator=g, device=dev) * 0.02
    conv = torch.randn((2 * B, conv_dim, K - 1), generator=g, device=dev, dtype=bf)
    qkv = torch.randn((T, conv_dim), generator=g, device=dev, dtype=bf)
    bb = torch.randn((T, hv), generator=g, device=dev, dtype=bf)
    aa = torch.randn((T, hv), generator=g, device=dev, dtype=bf)
    z = torch.randn((T, hv * dv), generator=g, device=dev, dtype=bf)
    w = torch.randn((conv_dim, 1, K), generator=g, device=dev, dtype=bf) * 0.5
    A_log = (torch.rand((hv,), generator=g, device=dev) * 1.5).to(bf)
    dt_bias = torch.randn((hv,), generator=g, device=dev, dtype=bf) * 0.5
    nw = torch.ones((hv * dv,), device=dev, dtype=bf)
    gdn_out = torch.empty((T, hv * dv), device=dev, dtype=bf)
    scale = D ** -0.5
    stream = torch.cuda.current_stream()

    def attn_step():
        ops.kv_store(kb, vb, loc_d, knew, vnew)
        ops.paged_extend(q, kb, vb, r2t_d, rpi, L_d, E_d, scale, Lmax, int(E.max()), gate=gate,
                         gate_mode="sigmoid", out=attn_out)

    def gdn_step():
        ops.gdn_extend(qkv, bb, aa, w, A_log, dt_bias, conv, ssm, rpi, E_d, num_k_heads=hk,
                       head_k_dim=dk, head_v_dim=dv, max_extend_len=int(E.max()), z=z,
                       norm_weight=nw, out=gdn_out)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        _barrier(world)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize()
        _barrier(world)
        return _max_over_ranks(t0.elapsed_time(t1) / 1e3, world) / steps

    # fused prologue of the same layer (q/k RMSNorm + partial RoPE + KV store), q read as the
    # strided half of a [T, Hq, 2D] q_proj output as in the module
    qg = torch.randn((T, hq, 2 * D), generator=g, device=dev, dtype=bf)
    kp = torch.randn((T, hkv, D), generator=g, device=dev, dtype=bf)
    vp = torch.randn((T, hkv, D), generator=g, device=dev, dtype=bf)
    qnw = (1.0 + 0.1 * torch.randn((D,), generator=g, device=dev)).to(bf)
    knw = (1.0 + 0.1 * torch.randn((D,), generator=g, device=dev)).to(bf)
    rot = D // 4
    inv_freq = 1.0 / (1e7 ** (torch.arange(0, rot, 2, dtype=torch.float32, device=dev) / rot))
    pos_d = torch.cat([torch.arange(int(P[b]), int(L[b])) for b in range(B)]).to(dev)
    q_pro = torch.empty((T, hq, D), dtype=bf, device=dev)

    def pro_step():
        ops.attn_prologue(qg[..., :D], kp, vp, qnw, knw, pos_d, inv_freq, kb, vb, loc_d,
                          q_out=q_pro)

    # GDN state snapshots at admission: every request restores its prefix's snapshot into its
    # working slot, all 48 linear layers of the 27B shape (ReqToStatePool, [L, slots, ...] pools)
    n_lin = 48
    snap_conv = torch.randn((n_lin, 2 * B, conv_dim, K - 1), generator=g, device=dev, dtype=bf)
    snap_ssm = torch.randn((n_lin, 2 * B, hv, dk, dv), generator=g, device=dev)
    snap_src = torch.arange(B, 2 * B, dtype=torch.int64, device=dev)
    snap_dst = torch.arange(0, B, dtype=torch.int64, device=dev)
    snap_bytes = 2 * B * n_lin * (conv_dim * (K - 1) * 2 + hv * dk * dv * 4)

    def snap_step():
        ops.state_slots_copy(snap_conv, snap_ssm, snap_src, snap_dst)

    def snap_step_torch():  # the reference's restore_snapshot: two torch copies per request
        for b in range(B):
            snap_conv[:, b].copy_(snap_conv[:, B + b])
            snap_ssm[:, b].copy_(snap_ssm[:, B + b])

    with ClockSampler(torch.cuda.current_device()) as clk:
        attn_s = timed(attn_step, args.steps)
        gdn_s = timed(gdn_step, max(1, args.steps // 4))
        pro_s = timed(pro_step, args.steps)
        snap_s = timed(snap_step, args.steps)
        snap_torch_s = timed(snap_step_torch, max(1, args.steps // 4))
    pro_bytes = 2 * T * (hq + 2 * hkv) * D * 2 + 2 * T * 8
    # GDN extend algorithmic bytes (this rank's heads): qkv in, z in, out, the recurrent states
    # read and written once, conv states read and written, a and b
    gdn_bytes = (T * conv_dim * 2 + 2 * T * hv * dv * 2 + B * hv * dk * dv * 4 * 2 +
                 B * conv_dim * (K - 1) * 2 * 2 + 2 * T * hv * 2)
    Pf, Ef = P.double(), E.double()
    flops = float((4 * C4["Hq"] * D * (Ef * Pf + Ef * (Ef + 1) / 2)).sum())  # whole job
    gdn_flops_tok = C4["Hv"] * (6 * dk * dv + 3 * 64 * dv) + C4["Hk"] * 4 * 64 * dk
    peak, peak_kind = _peak_tflops(attn_s * args.steps)
    tflops = flops / attn_s / 1e12
    per_gpu = tflops / world
    return {
        "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": attn_s * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "config4 extend over a cached prefix (one full-attention layer: "
                               "KV store + causal extend attention with sigmoid gate)",
                   "requests": B, "prefix": f"U[0,{C4['Pmax']}]",
                   "extend": f"U[{C4['Emin']},{C4['Emax']}]", "new_tokens": T,
                   "q_heads": C4["Hq"], "kv_heads": C4["Hkv"], "head_dim": D,
                   "parallelism": f"tp{world}",
                   "l2": "K/V of the prefixes re-read from L2 by the query tiles; no flush"},
        "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                     "frac": per_gpu / peak, "peak_kind": peak_kind,
                     "kernel": "tf_paged_extend_attn (tcgen05)", "flops_per_launch": flops / world,
                     "traffic": NCU_TRAFFIC_N1["extend"] if world == 1 and B == C4["B"] and
                     S == C4["slots"] else None},
        "gdn_extend": {"tok_per_s": T / gdn_s, "ms_per_step": gdn_s * 1e3,
                       "tflops_min_count": T * gdn_flops_tok / gdn_s / 1e12,
                       "tflops_frac_of_peak": T * gdn_flops_tok / world / gdn_s / 1e12 / peak,
                       "roofline": {"bound": "hbm", "achieved": gdn_bytes / gdn_s / 1e9,
                                    "peak": _peaks()[0], "unit": "GB/s",
                                    "frac": gdn_bytes / gdn_s / 1e9 / _peaks()[0],
                                    "peak_kind": _peaks()[1], "bytes_per_launch": gdn_bytes,
                                    "why": "the minimal FLOP count takes T*6.42 MFLOP / peak, "
                                           "less time than streaming qkv, z, out and the states "
                                           "once; HBM binds"},
                       "kernel": "tf_gdn_extend (varlen conv + chunked WY delta rule, C=64, tcgen05 with bf16x3 split products, fp32 state)"},
        "prologue": {"gb_per_s": pro_bytes / pro_s / 1e9, "ms_per_step": pro_s * 1e3,
                     "frac_of_hbm_peak": pro_bytes / pro_s / 1e9 / _peaks()[0], "peak_kind": _peaks()[1],
                     "bytes_per_launch": pro_bytes,
                     "kernel": "tf_attn_prologue (q/k RMSNorm + partial RoPE + KV store)"},
        "state_snapshot": {"gb_per_s": snap_bytes / snap_s / 1e9, "ms_per_step": snap_s * 1e3,
                           "frac_of_hbm_peak": snap_bytes / snap_s / 1e9 / _peaks()[0],
                           "peak_kind": _peaks()[1], "bytes_per_launch": snap_bytes,
                           "restores": B, "linear_layers": n_lin,
                           "torch_copies_ms": snap_torch_s * 1e3,
                           "kernel": "tf_state_slots_copy (all layers, both pools, one launch)"},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }


# ---------------------------------------------------------------------------------------------
# config 6: block-FP8 linear at a 27B projection shape
# ---------------------------------------------------------------------------------------------
C6 = dict(N=17408, K=5120, M_prefill=8192, M_decode=128)


def bench_fp8(args, rank, world, dev):
    """triton_block_fp8_linear's job (qwen3_8/fp8_triton.py:109-181) on the 27B MLP up projection
    (hidden 5120 -> intermediate 17408, e4m3 weights with 128 x 128 block scales, bf16
    activations): the activation quantization plus the tcgen05 GEMM, timed with CUDA events on
    the launching stream.  Column-parallel under TP: each rank owns N / world output columns."""
    from tokenfactory_b200 import ops

    N, K = C6["N"] // world, C6["K"]
    g = torch.Generator(device=dev).manual_seed(6 + rank)
    w = (torch.randn((N, K), generator=g, device=dev) * 0.5).to(torch.float8_e4m3fn)
    ws = torch.rand(((N + 127) // 128, (K + 127) // 128), generator=g, device=dev) + 0.5
    stream = torch.cuda.current_stream()

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        _barrier(world)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize()
        _barrier(world)
        return _max_over_ranks(t0.elapsed_time(t1) / 1e3, world) / steps

    res = {}
    with ClockSampler(torch.cuda.current_device()) as clk:
        for tag, M in (("prefill", C6["M_prefill"]), ("decode", C6["M_decode"])):
            x = torch.randn((M, K), generator=g, device=dev, dtype=torch.bfloat16)
            q, s = ops.fp8_quantize(x)
            out = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
            full = timed(lambda: ops.block_fp8_linear(x, w, ws, None), args.steps)
            gemm = timed(lambda: ops.fp8_block_gemm(q, s, w, ws, None, torch.bfloat16, out=out),
                         args.steps)

            def scaled_mm_loop():  # the reference's non-Triton path (fp8_linear.py:124-179), restated
                acc = torch.zeros((M, N), dtype=torch.float32, device=dev)
                one = torch.ones((1,), dtype=torch.float32, device=dev)
                for kb, k0 in enumerate(range(0, K, 128)):
                    blk = torch._scaled_mm(q[:, k0:k0 + 128].contiguous(),
                                           w[:, k0:k0 + 128].contiguous().t(), scale_a=s,
                                           scale_b=one, out_dtype=torch.float32)
                    acc += blk * ws[:, kb].repeat_interleave(128)[:N].unsqueeze(0)
                return acc.to(torch.bfloat16)

            ref_s = timed(scaled_mm_loop, max(1, args.steps // 10))
            flops = 2.0 * M * N * K
            res[tag] = {"M": M, "ms_linear": full * 1e3, "ms_gemm": gemm * 1e3,
                        "tflops_gemm": flops / gemm / 1e12, "tflops_linear": flops / full / 1e12,
                        "weight_gb_per_s_gemm": N * K / gemm / 1e9,
                        "torch_scaled_mm_loop_ms": ref_s * 1e3}
    pre = res["prefill"]
    bf16_peak, peak_kind = _peak_tflops(pre["ms_gemm"] / 1e3 * args.steps)
    fp8_peak = 2 * bf16_peak
    return {
        "metric": "block-FP8 linear TFLOP/s (27B MLP up projection 5120 -> 17408, 128x128 block scales)",
        "value": pre["tflops_gemm"] * world, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": pre["ms_gemm"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp8_e4m3",
        "data": "synthetic",
        "config": {"workload": "config6 block-FP8 GEMM (qwen3_8/fp8_triton.py)", "M": pre["M"],
                   "N": C6["N"], "K": K, "parallelism": f"tp{world}",
                   "l2": "weights (89 MB) and activations (84 MB) re-read from L2 across tiles"},
        "roofline": {"bound": "tensor", "achieved": pre["tflops_gemm"], "peak": fp8_peak,
                     "unit": "TFLOP/s", "frac": pre["tflops_gemm"] / fp8_peak,
                     "peak_kind": f"2x {peak_kind} bf16 (the dense e4m3 rate is twice bf16's)",
                     "kernel": "tf_fp8_block_gemm (tcgen05 kind::f8f6f4)"},
        "prefill": pre, "decode": res["decode"],
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }


# ---------------------------------------------------------------------------------------------
# config 5: 27B-shape hybrid decoder end to end
# ---------------------------------------------------------------------------------------------
C5 = dict(requests=256, prompt=1024, gen=256, layers=64, prefill_chunk=16)


class _HotPathTimer:
    """CUDA events around every hot-path call of the drop-in layers (the fused prologue and the
    paged attention of full layers: a1-a4; the GDN conv + recurrence + gated norm of linear
    layers: a5-a9), so that the projections, the MLP and the all-reduce stay outside.  Wraps
    ops.attn_prologue, hybrid_attention._attend and hybrid_attention.linear_attention_core."""

    def __init__(self):
        from tokenfactory_b200 import hybrid_attention as H, ops
        self.H, self.ops = H, ops
        self.pairs = []
        self.saved = (ops.attn_prologue, H._attend, H.linear_attention_core)

    def _wrap(self, fn):
        def timed(*a, **k):
            s = torch.cuda.current_stream()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            r = fn(*a, **k)
            e1.record(s)
            self.pairs.append((e0, e1))
            return r
        return timed

    def __enter__(self):
        self.ops.attn_prologue = self._wrap(self.saved[0])
        self.H._attend = self._wrap(self.saved[1])
        self.H.linear_attention_core = self._wrap(self.saved[2])
        return self

    def __exit__(self, *exc):
        self.ops.attn_prologue, self.H._attend, self.H.linear_attention_core = self.saved

    def take_ms(self) -> float:
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in self.pairs)
        self.pairs = []
        return ms


def bench_e2e(args, rank, world, dev):
    """a random-init bf16 27B-shape hybrid decoder (hidden 5120, 64 layers,
    every 4th full attention with the heads of config 2, GDN layers with those of config 3, MLP
    17408, vocab 248320, MTP off) under head-sharded TP over `world` GPUs, on 256 concurrent
    requests of 1024 uniform-random prompt tokens that each generate 256 greedy tokens: the
    prompts prefill in chunks of 16 requests (16K tokens per forward), then all requests decode
    together for 256 steps, each step's tokens sampled on the device (ops.sample_tokens) and fed
    back without a host sync.  The hot-path calls are bracketed by CUDA events (_HotPathTimer):
    the row-parallel all-reduces (NCCL) and the projections stay outside that figure."""
    from tokenfactory_b200 import ForwardBatch, ops
    from tokenfactory_b200.hybrid_model import HybridCachePool, HybridConfig, HybridForCausalLM

    R, P, G, nl = args.c5_requests, args.c5_prompt, args.c5_gen, args.c5_layers
    chunk = min(C5["prefill_chunk"], R)
    cfg = HybridConfig(hidden_size=5120, intermediate_size=17408, num_hidden_layers=nl,
                       vocab_size=248320, num_attention_heads=C2["Hq"],
                       num_key_value_heads=C2["Hkv"], head_dim=C2["D"],
                       linear_num_key_heads=C3["Hk"], linear_num_value_heads=C3["Hv"],
                       linear_key_head_dim=C3["dk"], linear_value_head_dim=C3["dv"],
                       output_gate_mode="sigmoid", tp_size=world, tp_rank=rank)
    t_init = time.perf_counter()
    torch.manual_seed(5 + rank)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = HybridForCausalLM(cfg).eval()
    finally:
        torch.set_default_dtype(prev)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if n.endswith("norm.weight") or n.endswith("layernorm.weight"):
                p.fill_(1.0)
            elif n.endswith("A_log"):
                p.uniform_(0.0, 1.5)
            elif n.endswith("dt_bias"):
                p.normal_(0.0, 0.5)
            elif "conv1d" in n:
                p.normal_(0.0, 0.5)
            else:
                p.normal_(0.0, 0.02)
    slots = R * (P + G) + 1
    pool = HybridCachePool(cfg, slots, R, 0, dtype=torch.bfloat16, device=dev)
    gen = torch.Generator().manual_seed(55)
    perm = torch.randperm(slots - 1, generator=gen)[: R * (P + G)] + 1
    r2t = perm.view(R, P + G).to(dev)
    prompts = torch.randint(0, cfg.vocab_size, (R, P), generator=gen).to(dev)
    temps = torch.zeros(R, dtype=torch.float32, device=dev)
    weights_gb = sum(p.numel() * p.element_size() for p in model.parameters()) / 1e9
    init_s = time.perf_counter() - t_init

    def prefill(c):
        rows = torch.arange(c * chunk, (c + 1) * chunk, device=dev)
        ext = [P] * chunk
        fb = ForwardBatch(batch_size=chunk, req_pool_indices=rows,
                          seq_lens=torch.full((chunk,), P, device=dev),
                          prefix_lens=torch.zeros(chunk, dtype=torch.long, device=dev),
                          extend_lens=ext, out_cache_loc=r2t[rows, :P].reshape(-1),
                          req_to_token=r2t, is_prefill=True, max_seq_len=P, max_extend_len=P,
                          extend_lens_tensor=torch.full((chunk,), P, device=dev),
                          req_pool_indices_list=list(range(c * chunk, (c + 1) * chunk)))
        pos = torch.arange(P, device=dev).repeat(chunk)
        return model(prompts[c * chunk:(c + 1) * chunk].reshape(-1), pos, pool, fb)

    rows_all = torch.arange(R, device=dev)
    ones = torch.ones(R, dtype=torch.long, device=dev)

    def decode(step, ids):
        L = P + step + 1
        fb = ForwardBatch(batch_size=R, req_pool_indices=rows_all,
                          seq_lens=torch.full((R,), L, device=dev),
                          prefix_lens=torch.full((R,), L - 1, device=dev), extend_lens=[1] * R,
                          out_cache_loc=r2t[:, L - 1], req_to_token=r2t, is_prefill=False,
                          max_seq_len=L, max_extend_len=1, extend_lens_tensor=ones,
                          req_pool_indices_list=list(range(R)))
        return model(ids, torch.full((R,), L - 1, device=dev), pool, fb)

    def run(timer):
        pool.conv_state.zero_()
        pool.ssm_state.zero_()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        stream = torch.cuda.current_stream()
        ev[0].record(stream)
        first = []
        for c in range(R // chunk):
            first.append(ops.sample_tokens(prefill(c), temps[:chunk]))
        ev[1].record(stream)
        pre_attn = timer.take_ms() if timer else 0.0
        ids = torch.cat(first)
        for step in range(G - 1):  # the prefill produced each request's first token
            ids = ops.sample_tokens(decode(step, ids), temps)
        ev[2].record(stream)
        torch.cuda.synchronize()
        dec_attn = timer.take_ms() if timer else 0.0
        return ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), pre_attn, dec_attn

    # warm-up: one prefill chunk and a few decode steps (kernel set-up, cuBLAS heuristics)
    pool.ssm_state.zero_()
    out = prefill(0)
    ids = torch.zeros(R, dtype=torch.long, device=dev)
    for step in range(min(3, G - 1)):
        decode(step, ids)
    torch.cuda.synchronize()
    _barrier(world)
    with ClockSampler(torch.cuda.current_device()) as clk, _HotPathTimer() as timer:
        timer.take_ms()
        pre_ms, dec_ms, pre_attn, dec_attn = run(timer)
    _barrier(world)
    pre_ms = _max_over_ranks(pre_ms, world)
    dec_ms = _max_over_ranks(dec_ms, world)
    pre_attn = _max_over_ranks(pre_attn, world)
    dec_attn = _max_over_ranks(dec_attn, world)
    total_s = (pre_ms + dec_ms) / 1e3
    toks = R * (P + G)
    del out
    return {
        "metric": "27B-shape hybrid end to end: tokens/s and attention hot-path time (config 5)",
        "value": toks / total_s, "unit": "tok/s (prompt + generated, whole job)",
        "n_gpus": world, "steps": 1, "warmup": 1, "ms_per_step": (pre_ms + dec_ms),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights ~N(0, 0.02), uniform-random prompt ids)",
        "config": {"workload": "config5 27B-shape hybrid decoder, continuous batch of "
                               f"{R} requests x ({P} prompt + {G} generated) tokens",
                   "hidden": 5120, "layers": nl, "full_attention_layers": nl // 4,
                   "q_heads": C2["Hq"], "kv_heads": C2["Hkv"], "head_dim": C2["D"],
                   "gdn_heads": f"{C3['Hk']}/{C3['Hv']} dk=dv=128", "mlp": 17408,
                   "vocab": 248320, "parallelism": f"tp{world}", "prefill_chunk_requests": chunk,
                   "weights_gb_per_rank": weights_gb, "init_s": init_s},
        "prefill": {"ms": pre_ms, "tok_per_s": R * P / (pre_ms / 1e3),
                    "attention_hot_path_ms": pre_attn,
                    "attention_share": pre_attn / pre_ms if pre_ms else None},
        "decode": {"ms": dec_ms, "steps": G - 1, "ms_per_step": dec_ms / max(1, G - 1),
                   "tok_per_s": R * (G - 1) / (dec_ms / 1e3), "attention_hot_path_ms": dec_attn,
                   "attention_share": dec_attn / dec_ms if dec_ms else None},
        "attention_hot_path_ms": pre_attn + dec_attn,
        "how": "CUDA events on the launching stream around the whole run and around every "
               "hot-path call (prologue + paged attention of the 16 full layers, GDN conv + "
               "recurrence + gated norm of the 48 linear layers); max over ranks; the "
               "row-parallel all-reduces (NCCL) and projections are outside the hot-path figure",
        "gpu_launches": None,
        "clocks": clk.summary(),
    }


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle (restatement of the reference's torch algorithm) on this host
# ---------------------------------------------------------------------------------------------
def _cpu_decode_sample(n_requests: int, seed: int = 0):
    """A bounded CPU sample of config 2: requests with the config's length distribution and heads
    over a host pool of config 2's own size (1.2M slots, 4.9 GB of bf16 K and V), so the gathers
    walk the same memory footprint as on the GPU.  The pool's rows repeat a random block of 64K
    rows (finite bf16 patterns; the work does not depend on the values)."""
    rng = np.random.default_rng(seed)
    S = C2["slots"]
    D, Hkv, Hq = C2["D"], C2["Hkv"], C2["Hq"]
    lens = rng.integers(C2["Lmin"], C2["Lmax"] + 1, n_requests)
    blk = 1 << 16
    reps = (S + blk - 1) // blk
    kb = np.tile(rng.integers(0x3C00, 0x4000, (blk, Hkv, D), dtype=np.uint16), (reps, 1, 1))[:S]
    vb = np.tile(rng.integers(0x3C00, 0x4000, (blk, Hkv, D), dtype=np.uint16), (reps, 1, 1))[:S]
    r2t = np.full((n_requests, C2["Lmax"]), -1, dtype=np.int64)
    for b in range(n_requests):
        r2t[b, :lens[b]] = rng.integers(1, S, lens[b])
    q = rng.integers(0x3C00, 0x4000, (n_requests, Hq, D), dtype=np.uint16)
    return lens, kb, vb, r2t, q


def cpu_decode_baseline(budget_s: float, threads: int):
    """Time the oracle's slot_based_attention (one decode request per call, `threads` in
    parallel) for about `budget_s` seconds; returns (tok/s, requests timed)."""
    from concurrent.futures import ThreadPoolExecutor

    sys.path.insert(0, ROOT)
    from oracle import attention as OA

    n = 32
    lens, kb, vb, r2t, q = _cpu_decode_sample(n)
    scale = C2["D"] ** -0.5

    def one(b):
        OA.slot_based_attention(q[b:b + 1], kb, vb, r2t, [b], [int(lens[b])], [1], scale,
                                "bf16", max_seq_len=int(lens[b]))
        return 1

    one(0)  # warm
    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        while time.perf_counter() - t0 < budget_s:
            done += sum(ex.map(one, [(done + i) % n for i in range(threads)]))
    el = time.perf_counter() - t0
    return done / el, done


def run_reference(args, rank, world):
    """--impl reference: the reference algorithm (oracle port) on the host CPU, rank 0 only."""
    if rank != 0:
        return None
    from concurrent.futures import ThreadPoolExecutor

    sys.path.insert(0, ROOT)
    from oracle import attention as OA

    threads = os.cpu_count() or 1
    n = 32
    lens, kb, vb, r2t, q = _cpu_decode_sample(n)
    scale = C2["D"] ** -0.5

    def one(b):
        OA.slot_based_attention(q[b:b + 1], kb, vb, r2t, [b], [int(lens[b])], [1], scale,
                                "bf16", max_seq_len=int(lens[b]))

    with ThreadPoolExecutor(max_workers=threads) as ex:
        for w in range(args.warmup):
            list(ex.map(one, [(w * threads + i) % n for i in range(threads)]))
        t0 = time.perf_counter()
        for s in range(args.steps):
            list(ex.map(one, [(s * threads + i) % n for i in range(threads)]))
        el = time.perf_counter() - t0
    v = threads * args.steps / el
    sample = (f"{threads} decode requests per step (one per thread) of config 2's length "
              f"distribution and heads over a host pool of config 2's {C2['slots']} slots")
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "config2 paged GQA decode (one full-attention layer step)",
                   "value": "whole-job tokens/s over all GPUs (each rank decodes every request "
                            "for its heads); value_per_gpu = value / n_gpus",
                   "batch": C2["B"], "q_heads": C2["Hq"], "kv_heads": C2["Hkv"],
                   "head_dim": C2["D"], "seq_len": f"U[{C2['Lmin']},{C2['Lmax']}]",
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample, "same_config": True,
                         "why_port": "the reference's path is Python over torch; its sources "
                                     "cannot travel to the GPU box, so the arm is the oracle's "
                                     "restatement of _slot_based_attention, pinned to the "
                                     "reference's own outputs by committed fixtures"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5, 6])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-baseline-seconds", type=float, default=12.0)
    ap.add_argument("--batch", type=int, default=C2["B"],
                    help="profiling only: decode batch (default: config 2's 128)")
    ap.add_argument("--pool-slots", type=int, default=C2["slots"],
                    help="profiling only: KV pool slots (default: config 2's 1.2M)")
    ap.add_argument("--requests", type=int, default=C4["B"],
                    help="config 4: requests in the extend batch (smaller cases for ncu captures)")
    ap.add_argument("--ext-pool-slots", type=int, default=C4["slots"],
                    help="config 4: KV pool slots")
    ap.add_argument("--no-e2e", action="store_true",
                    help="profiling only: device-timed leg alone, short output")
    ap.add_argument("--c5-requests", type=int, default=C5["requests"],
                    help="config 5: concurrent requests")
    ap.add_argument("--c5-prompt", type=int, default=C5["prompt"], help="config 5: prompt tokens")
    ap.add_argument("--c5-gen", type=int, default=C5["gen"], help="config 5: generated tokens")
    ap.add_argument("--c5-layers", type=int, default=C5["layers"], help="config 5: layers")
    ap.add_argument("--decode-only", action="store_true",
                    help="config 2 without the config 3 / config 4 legs that the default line carries")
    ap.add_argument("--head-split", type=int, default=0,
                    help="profiling only: config 2's decode on the heads rank 0 owns in an N-GPU "
                         "run, timed on this one GPU")
    args = ap.parse_args()
    C2["B"], C2["slots"] = args.batch, args.pool_slots
    args.warmup = max(3, args.warmup)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    rank, world, local = _dist()
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    dev = torch.device("cuda", torch.cuda.current_device())
    res = {2: bench_decode, 3: bench_gdn_decode, 4: bench_extend, 5: bench_e2e,
           6: bench_fp8}[args.config](args, rank, world, dev)
    if args.config == 2 and not args.no_e2e and not args.decode_only:
        # the rest of the metric in the same line: config 3 (GDN decode) and config 4 (extend
        # attention TFLOP/s, GDN extend), each timed on its own with CUDA events and clocks
        torch.cuda.empty_cache()
        g = bench_gdn_decode(args, rank, world, dev)
        res["gdn_decode"] = {k: g[k] for k in ("metric", "value", "unit", "ms_per_step", "config",
                                               "roofline", "clocks")}
        torch.cuda.empty_cache()
        e = bench_extend(args, rank, world, dev)
        res["extend"] = {k: e[k] for k in ("value", "unit", "ms_per_step", "config", "roofline",
                                           "gdn_extend", "prologue", "state_snapshot", "clocks")}
        res["extend"]["metric"] = "extend attn TFLOP/s (config 4, whole job)"
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and args.config == 2 and not args.no_e2e and \
            args.cpu_baseline_seconds > 0:
        threads = os.cpu_count() or 1
        v, n = cpu_decode_baseline(args.cpu_baseline_seconds, threads)
        res["cpu_baseline"] = {
            "value": v, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode requests of config 2's length distribution and heads over "
                      f"a {C2['slots']}-slot host pool ({args.cpu_baseline_seconds:.0f} s budget, "
                      f"{threads} threads)", "same_config": True}
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
