"""Per-step host work around the hot path: ForwardBatch construction, the device req_to_token
sync and sampling, without per-request device calls or host synchronisation.

The reference's ModelRunner builds each step's metadata with eight ``torch.tensor(list)`` copies
plus one slice assignment (and one more copy for a stale prefix) per request
(``_prepare_forward_batch``, engine/model_runner.py:108-188), and samples with one argmax or
softmax + multinomial and one ``.item()`` per request (``_sample``, :574-581).  Here:

* ``prepare_forward_batch``: the same outputs (input_ids, positions, ForwardBatch, the updated
  device req_to_token and synced lengths) from ONE pinned host buffer, ONE host->device copy and
  ONE tf_req_to_token_sync launch; the ForwardBatch carries its host-side maxima and lists, so
  nothing downstream reads a device value back;
* ``sample``: every row in one tf_sample_tokens launch and one device->host copy;
* ``ModelRunnerHotPath``: mixin overriding ``_prepare_forward_batch`` and ``_sample`` with the
  reference's signatures; ``install()`` patches ``engine.model_runner.ModelRunner``.
* ``CapturedStep`` / ``PipelinedStep``: a step replayed as a CUDA graph with new inputs; the
  pipelined form overlaps each step's host<->device copies with its neighbours' kernels.
"""

import importlib
import sys
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import ops
from .forward_batch import ForwardBatch as _OwnForwardBatch

_saved: Dict[str, type] = {}


def _forward_batch_cls(owner) -> type:
    """The ForwardBatch class of the module that defines `owner`'s class (the reference's own
    dataclass when the runner is the reference's), else this package's mirror."""
    for klass in type(owner).__mro__:
        mod = sys.modules.get(klass.__module__)
        fb = getattr(mod, "ForwardBatch", None) if mod is not None else None
        if isinstance(fb, type):
            return fb
    return _OwnForwardBatch


class PackedBatch:
    """One step's metadata as one int64 host array: ids | positions | out_cache_loc |
    req_pool_indices | seq_lens | prefix_lens | extend_lens | stale prefix values | segments
    (row, col, len, src) of the req_to_token sync, src indexing this same array."""

    def __init__(self, host: np.ndarray, B: int, T: int, n_stale: int, n_segs: int,
                 rpi: List[int], seq: List[int], ext: List[int], is_prefill: bool):
        self.host, self.B, self.T = host, B, T
        self.rpi, self.seq, self.ext, self.is_prefill = rpi, seq, ext, is_prefill
        self.o_ids, self.o_pos, self.o_loc, self.o_rpi = 0, T, 2 * T, 3 * T
        self.o_seq, self.o_pre, self.o_ext = 3 * T + B, 3 * T + 2 * B, 3 * T + 3 * B
        self.o_stale = 3 * T + 4 * B
        self.o_seg = self.o_stale + n_stale
        self.n_segs = n_segs

    def segments(self) -> np.ndarray:
        return self.host[self.o_seg:self.o_seg + 4 * self.n_segs].reshape(-1, 4)


def pack_batch(batch_reqs: Sequence, req_to_token_table: Sequence[Sequence[int]],
               synced_lens: List[int], dirty_from: Optional[List[int]] = None,
               pinned: bool = False) -> PackedBatch:
    """The host half of ModelRunner._prepare_forward_batch (engine/model_runner.py:108-188): the
    flattened step tensors and the req_to_token segments to sync, in one int64 array; updates
    synced_lens / dirty_from as the reference does.  Requests need req_pool_idx,
    cur_chunk_tokens, out_cache_loc, cur_start_pos, cur_seq_len and is_prefilled."""
    B = len(batch_reqs)
    ids: List[int] = []
    locs: List[int] = []
    pos_parts: List[np.ndarray] = []
    rpi, seq, pre, ext = [], [], [], []
    for req in batch_reqs:
        assert req.req_pool_idx is not None
        n = len(req.cur_chunk_tokens)
        assert n > 0 and n == len(req.out_cache_loc)
        assert req.cur_seq_len - req.cur_start_pos == n, "chunk length != cur_seq_len - cur_start_pos"
        rpi.append(req.req_pool_idx)
        seq.append(req.cur_seq_len)
        pre.append(req.cur_start_pos)
        ext.append(n)
        ids.extend(req.cur_chunk_tokens)
        locs.extend(req.out_cache_loc)
        pos_parts.append(np.arange(req.cur_start_pos, req.cur_seq_len, dtype=np.int64))
    T = len(ids)
    o_loc, o_stale = 2 * T, 3 * T + 4 * B
    segs: List[Tuple[int, int, int, int]] = []
    stale: List[Sequence[int]] = []
    n_stale = 0
    loc_off = 0
    for req, n in zip(batch_reqs, ext):
        r = req.req_pool_idx
        synced = synced_lens[r]
        if dirty_from is not None and dirty_from[r] < synced:
            synced = dirty_from[r]
        if synced < req.cur_start_pos:
            part = req_to_token_table[r][synced:req.cur_start_pos]
            segs.append((r, synced, len(part), o_stale + n_stale))
            stale.append(part)
            n_stale += len(part)
        segs.append((r, req.cur_start_pos, n, o_loc + loc_off))
        synced_lens[r] = req.cur_seq_len
        if dirty_from is not None:
            dirty_from[r] = req.cur_seq_len
        loc_off += n
    total = o_stale + n_stale + 4 * len(segs)
    host_t = torch.empty(total, dtype=torch.int64, pin_memory=pinned)
    pk = PackedBatch(host_t.numpy(), B, T, n_stale, len(segs), rpi, seq, ext,
                     any(not r.is_prefilled for r in batch_reqs))
    pk.tensor = host_t
    h = pk.host
    h[pk.o_ids:pk.o_ids + T] = ids
    if pos_parts:
        h[pk.o_pos:pk.o_pos + T] = np.concatenate(pos_parts)
    h[pk.o_loc:pk.o_loc + T] = locs
    h[pk.o_rpi:pk.o_rpi + B] = rpi
    h[pk.o_seq:pk.o_seq + B] = seq
    h[pk.o_pre:pk.o_pre + B] = pre
    h[pk.o_ext:pk.o_ext + B] = ext
    if n_stale:
        h[o_stale:o_stale + n_stale] = np.concatenate([np.asarray(p, np.int64) for p in stale])
    if segs:
        h[pk.o_seg:total] = np.asarray(segs, np.int64).reshape(-1)
    return pk


def prepare_forward_batch(batch_reqs: Sequence, req_to_token_table: Sequence[Sequence[int]],
                          req_to_token: torch.Tensor, synced_lens: List[int],
                          dirty_from: Optional[List[int]] = None,
                          forward_batch_cls: type = _OwnForwardBatch
                          ) -> Tuple[torch.Tensor, torch.Tensor, object]:
    """ModelRunner._prepare_forward_batch (engine/model_runner.py:108-188) with one host->device
    copy and one kernel: returns (input_ids, positions, ForwardBatch) and updates req_to_token
    (device) and synced_lens / dirty_from (host) exactly as the reference does."""
    ops._need_cuda(req_to_token)
    pk = pack_batch(batch_reqs, req_to_token_table, synced_lens, dirty_from, pinned=True)
    buf = pk.tensor.to(req_to_token.device, non_blocking=True)
    if pk.n_segs:
        ops.req_to_token_sync(req_to_token, buf[pk.o_seg:pk.o_seg + 4 * pk.n_segs].view(-1, 4),
                              buf[:pk.o_seg])
    B, T = pk.B, pk.T
    fb = forward_batch_cls(
        batch_size=B,
        req_pool_indices=buf[pk.o_rpi:pk.o_rpi + B],
        seq_lens=buf[pk.o_seq:pk.o_seq + B],
        prefix_lens=buf[pk.o_pre:pk.o_pre + B],
        extend_lens=pk.ext,
        out_cache_loc=buf[pk.o_loc:pk.o_loc + T],
        req_to_token=req_to_token,
        is_prefill=pk.is_prefill,
        max_seq_len=max(pk.seq) if pk.seq else 0,
        max_extend_len=max(pk.ext) if pk.ext else 0,
        extend_lens_tensor=buf[pk.o_ext:pk.o_ext + B],
        req_pool_indices_list=pk.rpi,
    )
    return buf[pk.o_ids:pk.o_ids + T], buf[pk.o_pos:pk.o_pos + T], fb


def sample(logits: torch.Tensor, temperatures: Sequence[float],
           generator: Optional[torch.Generator] = None) -> List[int]:
    """ModelRunner._sample (engine/model_runner.py:580-581) for all rows in one launch: greedy
    rows (temperature <= 1e-5) take the argmax, the others a draw from softmax(logits / T) with a
    uniform from torch's CUDA generator.  One device->host copy."""
    B = logits.shape[0]
    temp_h = torch.tensor([float(t) for t in temperatures], dtype=torch.float32).pin_memory()
    temp = temp_h.to(logits.device, non_blocking=True)
    uniform = None
    if any(t > 1e-5 for t in temperatures):
        uniform = torch.rand(B, device=logits.device, dtype=torch.float32, generator=generator)
    rows = logits if logits.stride(-1) == 1 else logits.contiguous()
    return ops.sample_tokens(rows, temp, uniform).tolist()


class ModelRunnerHotPath:
    """Overrides of ModelRunner._prepare_forward_batch and _sample (engine/model_runner.py:
    108-188, 574-581), using the attributes the reference's constructor sets: device,
    req_to_token_tensor, _req_synced_lens."""

    def _prepare_forward_batch(self, batch_reqs, req_to_token_table, dirty_from=None):
        return prepare_forward_batch(batch_reqs, req_to_token_table, self.req_to_token_tensor,
                                     self._req_synced_lens, dirty_from,
                                     forward_batch_cls=_forward_batch_cls(self))

    def _sample(self, logits, batch_reqs):
        return sample(logits, [r.temperature for r in batch_reqs])


def install(module: str = "engine.model_runner") -> type:
    """Patch ModelRunner in the reference's engine (and in already-imported modules that bound it
    by name) with the overrides; returns the patched class."""
    mod = importlib.import_module(module)
    ref = _saved.setdefault(module, mod.ModelRunner)
    cls = type(ref.__name__, (ModelRunnerHotPath, ref), {"__module__": ref.__module__,
                                                         "__doc__": ref.__doc__})
    for m in list(sys.modules.values()):
        if m is not None and getattr(m, "ModelRunner", None) is ref:
            m.ModelRunner = cls
    return cls


def uninstall(module: str = "engine.model_runner") -> None:
    ref = _saved.pop(module, None)
    if ref is None:
        return
    for m in list(sys.modules.values()):
        cur = getattr(m, "ModelRunner", None) if m is not None else None
        if isinstance(cur, type) and issubclass(cur, ModelRunnerHotPath) and ref in cur.__mro__:
            m.ModelRunner = ref


class CapturedStep:
    """A step function captured once as a CUDA graph and replayed with new inputs.

    ``fn(**inputs)`` must be graph-safe: every hot-path op of this package is (no host reads of
    device values; the decode's split plan is computed on the device from seq_lens, so a
    ``max_seq_len`` bound can be fixed at capture).  Inputs are copied into static buffers of the
    captured shapes (host tensors from pinned memory copy asynchronously), the graph is
    replayed, and the static outputs are returned (overwritten by the next call).

    Construction runs ``fn`` eagerly ``warmup`` times on the example inputs before capturing it
    (lazy initialisation must not happen inside the capture).  Those runs update whatever ``fn``
    updates in place - KV-pool rows, recurrent GDN states - exactly like real steps.  List such
    tensors in ``state`` to have them saved before the warm-up and restored after it (one
    temporary copy of each); otherwise the warm-up steps stay applied to them."""

    def __init__(self, fn, example_inputs: Dict[str, torch.Tensor], warmup: int = 2,
                 pool=None, state: Sequence[torch.Tensor] = ()):
        self.static = {k: torch.empty_like(v, device=v.device if v.is_cuda else "cuda")
                       for k, v in example_inputs.items()}
        for k, v in example_inputs.items():
            self.static[k].copy_(v)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            saved = [t.clone() for t in state] if warmup > 0 else []
            for _ in range(warmup):
                fn(**self.static)
            for t, c in zip(state, saved):
                t.copy_(c)
        torch.cuda.current_stream().wait_stream(side)
        del saved
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool):
            self.outputs = fn(**self.static)

    def __call__(self, **inputs):
        for k, v in inputs.items():
            dst = self.static[k]
            if v.shape != dst.shape:
                raise ValueError(f"{k}: shape {tuple(v.shape)} != captured {tuple(dst.shape)}")
            dst.copy_(v, non_blocking=True)
        self.graph.replay()
        return self.outputs


class PipelinedResult:
    """The host outputs of one PipelinedStep.submit: valid once `wait()` returns, until the
    same buffer set is submitted again (`depth` submits later)."""

    def __init__(self, host: Tuple[torch.Tensor, ...], copied_out: torch.cuda.Event,
                 copied_in: torch.cuda.Event):
        self.host = host
        self.copied_out = copied_out
        self.inputs_consumed = copied_in  # the host inputs may be overwritten once this completes

    def wait(self):
        self.copied_out.synchronize()
        return self.host[0] if len(self.host) == 1 else self.host


class _Slot:
    def __init__(self, cap: CapturedStep):
        self.cap = cap
        outs = cap.outputs if isinstance(cap.outputs, tuple) else (cap.outputs,)
        self.outs = outs
        self.host = tuple(torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs)
        self.copied_in = torch.cuda.Event()
        self.computed = torch.cuda.Event()
        self.copied_out = torch.cuda.Event()
        self.used = False


class PipelinedStep:
    """A captured step streamed over `depth` buffer sets so that host<->device copies overlap
    the kernels of the neighbouring steps.

    Each buffer set holds device copies of the inputs, a CUDA graph of ``fn`` captured over them
    (a CapturedStep) and pinned host copies of its outputs.  ``submit(**host_inputs)`` (pinned
    host tensors of the example shapes):

    * copy-in stream: waits until the set's previous step has finished its kernels, then copies
      the inputs in;
    * the caller's current stream: waits for those copies (and for the set's previous outputs to
      have left the device), replays the set's graph;
    * copy-out stream: waits for the graph, copies the outputs to the set's pinned host tensors.

    So step i+1's inputs travel while step i computes, and step i's outputs while step i+1
    computes.  The graphs replay in submission order on one stream, so state that ``fn`` updates
    in place (KV pool, recurrent state) sees the steps in order, as with CapturedStep.
    ``fence()`` orders later copies after work already issued on the current stream; ``join()``
    makes the current stream wait for every copy issued so far.

    Construction runs ``fn`` eagerly ``warmup`` times (for the first buffer set only; the other
    sets are captured without running it), with the same effect on in-place state as
    CapturedStep: pass the tensors ``fn`` updates in place as ``state`` to have them restored."""

    def __init__(self, fn, example_inputs: Dict[str, torch.Tensor], depth: int = 2,
                 warmup: int = 2, state: Sequence[torch.Tensor] = ()):
        if depth < 2:
            raise ValueError("depth must be at least 2")
        self.slots = [_Slot(CapturedStep(fn, example_inputs, warmup=warmup if i == 0 else 0,
                                         state=state)) for i in range(depth)]
        self.copy_in = torch.cuda.Stream()
        self.copy_out = torch.cuda.Stream()
        self.n = 0

    def fence(self):
        cur = torch.cuda.current_stream()
        self.copy_in.wait_stream(cur)
        self.copy_out.wait_stream(cur)

    def join(self):
        cur = torch.cuda.current_stream()
        cur.wait_stream(self.copy_in)
        cur.wait_stream(self.copy_out)

    def submit(self, **host_inputs) -> PipelinedResult:
        slot = self.slots[self.n % len(self.slots)]
        self.n += 1
        compute = torch.cuda.current_stream()
        static = slot.cap.static
        for k, v in host_inputs.items():
            if v.shape != static[k].shape:
                raise ValueError(f"{k}: shape {tuple(v.shape)} != captured {tuple(static[k].shape)}")
        if slot.used:
            self.copy_in.wait_event(slot.computed)  # the previous step read these inputs
        with torch.cuda.stream(self.copy_in):
            for k, v in host_inputs.items():
                static[k].copy_(v, non_blocking=True)
            slot.copied_in.record(self.copy_in)
        compute.wait_event(slot.copied_in)
        if slot.used:
            compute.wait_event(slot.copied_out)  # the previous outputs have left the device
        slot.cap.graph.replay()
        slot.computed.record(compute)
        self.copy_out.wait_event(slot.computed)
        with torch.cuda.stream(self.copy_out):
            for h, d in zip(slot.host, slot.outs):
                h.copy_(d, non_blocking=True)
            slot.copied_out.record(self.copy_out)
        slot.used = True
        return PipelinedResult(slot.host, slot.copied_out, slot.copied_in)
