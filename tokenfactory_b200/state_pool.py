"""Drop-in for the GDN state snapshots of tokenFactory's ReqToStatePool (req_to_state_pool.py).

ReqToStatePool keeps every linear layer's conv_state and ssm_state in one [L, slots, ...] tensor
each: a working zone (slots [0, max_reqs), one per request row) that the GDN kernels update in
place, and a snapshot zone ([max_reqs, max_reqs + max_snapshots)) owned by radix-tree nodes.  A
prefix hit restores a snapshot into the request's working slot, a miss zeroes it
(engine/scheduler.py:227-232), the radix tree captures snapshots and frees them on eviction
(radix_tree.py:275-302, :475-479).  The reference moves a slot with two torch copies (or zero
fills) per call, about 151 MB per slot at the 27B shape (48 layers x 48 x 128 x 128 fp32 plus the
conv rows).  Here:

* ``StatePoolHotPath``: mixin overriding reset_working_state, free_snapshot, free_snapshots,
  capture_snapshot and restore_snapshot (req_to_state_pool.py:120-194) with the same arguments,
  assertions and bookkeeping; the tensors move through tf_state_slots_copy, one launch for all
  layers and both pools.  ``apply_slot_ops`` batches any number of restores, resets and captures
  (the admission of a whole batch of requests) into one launch;
* ``ReqToStatePool``: the pool with the reference's constructor and bookkeeping plus the mixin,
  for use where the reference package is not installed;
* ``install()`` / ``uninstall()``: patch the reference's class in ``req_to_state_pool`` and in the
  modules that already imported it by name.
"""

import importlib
import sys
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import ops

_saved: Dict[str, type] = {}


class StatePoolHotPath:
    """Overrides of ReqToStatePool's copy methods.  Uses the attributes the reference class sets
    in its constructor (req_to_state_pool.py:34-108): max_reqs, total_slots, free_snapshot_slots,
    is_snapshot_occupied, state_debug_tags, conv_state, ssm_state."""

    def _slots_copy(self, src: Sequence[Optional[int]], dst: Sequence[int]) -> None:
        # the reference touches the tensors only when both exist (config given)
        if self.conv_state is None or self.ssm_state is None or not dst:
            return
        ops.state_slots_copy(self.conv_state, self.ssm_state, list(src), list(dst))

    def _check_working(self, req_idx: int) -> None:
        assert 0 <= req_idx < self.max_reqs, f"invalid working slot index: {req_idx}"

    def _check_snapshot(self, slot: int, action: str) -> None:
        assert self.max_reqs <= slot < self.total_slots, (
            f"slot {slot} is outside the snapshot zone [{self.max_reqs}, {self.total_slots})")
        assert self.is_snapshot_occupied[slot], f"snapshot slot {slot} is not allocated ({action})"

    # req_to_state_pool.py:120-127
    def reset_working_state(self, req_idx: int) -> None:
        self._check_working(req_idx)
        self._slots_copy([None], [req_idx])
        self.state_debug_tags[req_idx] = "ZERO_STATE"

    # req_to_state_pool.py:140-153
    def free_snapshot(self, slot: int) -> None:
        self.free_snapshots([slot])

    # req_to_state_pool.py:155-158: the same per-slot checks and bookkeeping in order, the
    # zeroing of all freed slots in one launch (also for the slots freed before a failed check)
    def free_snapshots(self, slots: List[int]) -> None:
        done: List[int] = []
        try:
            for slot in slots:
                assert self.max_reqs <= slot < self.total_slots, (
                    f"slot {slot} is outside the snapshot zone [{self.max_reqs}, {self.total_slots})")
                assert self.is_snapshot_occupied[slot], f"double free of snapshot slot {slot}"
                self.is_snapshot_occupied[slot] = False
                self.state_debug_tags[slot] = None
                self.free_snapshot_slots.append(slot)
                done.append(slot)
        finally:
            self._slots_copy([None] * len(done), done)

    # req_to_state_pool.py:160-176
    def capture_snapshot(self, req_idx: int, snapshot_slot: int,
                         debug_tag: Optional[str] = None) -> None:
        self._check_working(req_idx)
        self._check_snapshot(snapshot_slot, "capture")
        self._slots_copy([req_idx], [snapshot_slot])
        self.state_debug_tags[snapshot_slot] = (
            debug_tag or self.state_debug_tags[req_idx] or f"Snap(from_req_{req_idx})")

    # req_to_state_pool.py:178-194
    def restore_snapshot(self, snapshot_slot: int, req_idx: int) -> None:
        self._check_working(req_idx)
        self._check_snapshot(snapshot_slot, "restore")
        self._slots_copy([snapshot_slot], [req_idx])
        self.state_debug_tags[req_idx] = self.state_debug_tags[snapshot_slot]

    def apply_slot_ops(self, restores: Sequence[Tuple[int, int]] = (),
                       resets: Sequence[int] = (),
                       captures: Sequence[Tuple[int, int, Optional[str]]] = ()) -> None:
        """restore_snapshot(snap, req) for each (snap, req), reset_working_state(req) for each req
        and capture_snapshot(req, snap, tag) for each (req, snap, tag) with one launch.  The calls
        must not depend on one another (no slot written twice, none both read and written); the
        bookkeeping follows the order restores, resets, captures."""
        src: List[Optional[int]] = []
        dst: List[int] = []
        for snap, req in restores:
            self._check_working(req)
            self._check_snapshot(snap, "restore")
            src.append(snap)
            dst.append(req)
        for req in resets:
            self._check_working(req)
            src.append(None)
            dst.append(req)
        for req, snap, _ in captures:
            self._check_working(req)
            self._check_snapshot(snap, "capture")
            src.append(req)
            dst.append(snap)
        ops.state_slot_ops_valid(src, dst)
        self._slots_copy(src, dst)
        for snap, req in restores:
            self.state_debug_tags[req] = self.state_debug_tags[snap]
        for req in resets:
            self.state_debug_tags[req] = "ZERO_STATE"
        for req, snap, tag in captures:
            self.state_debug_tags[snap] = (
                tag or self.state_debug_tags[req] or f"Snap(from_req_{req})")


class _StatePoolBase:
    """ReqToStatePool's constructor and bookkeeping (req_to_state_pool.py:34-158): the dual-zone
    [L, max_reqs + max_snapshots, ...] tensors sized from the config's linear layers and local
    (tensor-parallel) heads, ssm_state in fp32 unless mamba_ssm_dtype says otherwise."""

    def __init__(self, max_reqs: int, max_snapshots: int = 16, config=None, device: str = "cpu",
                 dtype=None):
        self.max_reqs = max_reqs
        self.max_snapshots = max_snapshots
        self.total_slots = max_reqs + max_snapshots
        self.config = config
        self.device = device
        self.dtype = dtype if dtype is not None else torch.bfloat16
        self.free_snapshot_slots: List[int] = list(range(self.total_slots - 1, max_reqs - 1, -1))
        self.is_snapshot_occupied: Dict[int, bool] = {
            s: False for s in range(max_reqs, self.total_slots)}
        self.state_debug_tags: List[Optional[str]] = [None] * self.total_slots
        self.linear_layer_map: Dict[int, int] = {}
        self.conv_state: Optional[torch.Tensor] = None
        self.ssm_state: Optional[torch.Tensor] = None
        if config is None:
            return
        self.linear_layer_map = {l: i for i, l in enumerate(config.linear_attention_layer_indices)}
        n = len(self.linear_layer_map)
        nk = config.linear_num_key_heads // config.tp_size
        nv = config.linear_num_value_heads // config.tp_size
        dk, dv = config.linear_key_head_dim, config.linear_value_head_dim
        conv_dim = 2 * nk * dk + nv * dv
        self.conv_state = torch.zeros((n, self.total_slots, conv_dim,
                                       config.linear_conv_kernel_dim - 1),
                                      device=device, dtype=self.dtype)
        ssm_dtype = torch.float32 if config.mamba_ssm_dtype == "float32" else self.dtype
        self.ssm_state = torch.zeros((n, self.total_slots, nv, dk, dv), device=device,
                                     dtype=ssm_dtype)

    def available_snapshot_size(self) -> int:
        return len(self.free_snapshot_slots)

    def get_layer_states(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        assert self.conv_state is not None and self.ssm_state is not None
        i = self.linear_layer_map[layer_idx]
        return self.conv_state[i], self.ssm_state[i]

    def alloc_snapshot(self) -> Optional[int]:
        if not self.free_snapshot_slots:
            return None
        slot = self.free_snapshot_slots.pop()
        assert not self.is_snapshot_occupied[slot], f"snapshot slot {slot} is already occupied"
        self.is_snapshot_occupied[slot] = True
        return slot


class ReqToStatePool(StatePoolHotPath, _StatePoolBase):
    """ReqToStatePool with the snapshot copies on the GPU, without the reference package."""


def drop_in(reference_cls: type) -> type:
    """A subclass of the reference's ReqToStatePool with the copy methods overridden."""
    return type(reference_cls.__name__, (StatePoolHotPath, reference_cls),
                {"__module__": __name__, "__doc__": reference_cls.__doc__})


def install(module: str = "req_to_state_pool") -> type:
    """Patch ReqToStatePool in the reference module and in every already-imported module that
    bound it by name (qwen3_8.hybrid_cache_pool, engine.model_runner, engine.scheduler import it
    with ``from req_to_state_pool import ReqToStatePool``); modules imported later pick up the
    patched class.  Returns the drop-in class."""
    mod = importlib.import_module(module)
    ref = _saved.setdefault(module, mod.ReqToStatePool)
    cls = drop_in(ref)
    for m in list(sys.modules.values()):
        if m is not None and getattr(m, "ReqToStatePool", None) is ref:
            m.ReqToStatePool = cls
    return cls


def uninstall(module: str = "req_to_state_pool") -> None:
    """Restore the reference class everywhere install() replaced it."""
    ref = _saved.pop(module, None)
    if ref is None:
        return
    for m in list(sys.modules.values()):
        cur = getattr(m, "ReqToStatePool", None) if m is not None else None
        if isinstance(cur, type) and issubclass(cur, StatePoolHotPath) and ref in cur.__mro__:
            m.ReqToStatePool = ref
