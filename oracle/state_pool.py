"""Oracle for the GDN state-slot snapshots (TEST INFRASTRUCTURE; numpy).

Restates the tensor effects and the bookkeeping of ReqToStatePool (req_to_state_pool.py of
yz29528/tokenFactory):
  __init__             - req_to_state_pool.py:34-60     free stack (descending, pop from the end),
                                                         occupancy map, debug tags
  reset_working_state  - req_to_state_pool.py:120-127   zero every layer's rows of a working slot
  alloc_snapshot       - req_to_state_pool.py:129-138
  free_snapshot        - req_to_state_pool.py:140-153   zero the rows, push the slot back
  free_snapshots       - req_to_state_pool.py:155-158
  capture_snapshot     - req_to_state_pool.py:160-176   working slot -> snapshot slot
  restore_snapshot     - req_to_state_pool.py:178-194   snapshot slot -> working slot

conv_state [L, slots, conv_dim, K-1] is stored in its pool dtype (bf16 as uint16 bit patterns) and
ssm_state [L, slots, Hv, dk, dv] as float32; every operation is a whole-slot copy or zeroing
across all layers, so the oracle is exact by construction and comparisons are bit-exact.
"""

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


def slots_copy(conv_state: Optional[np.ndarray], ssm_state: Optional[np.ndarray],
               src: Sequence[Optional[int]], dst: Sequence[int]) -> None:
    """dst rows <- src rows (or zeros for a None / -1 source) in every layer of both pools, op by
    op in order (the reference's loop of copy_ / zero_ calls)."""
    for s, d in zip(src, dst):
        for pool in (conv_state, ssm_state):
            if pool is None:
                continue
            if s is None or s == -1:
                pool[:, d] = 0
            else:
                pool[:, d] = pool[:, s]


class StatePool:
    """The reference's ReqToStatePool on numpy arrays (pools may be None, as with config=None)."""

    def __init__(self, max_reqs: int, max_snapshots: int, conv_state: Optional[np.ndarray] = None,
                 ssm_state: Optional[np.ndarray] = None):
        self.max_reqs = max_reqs
        self.max_snapshots = max_snapshots
        self.total_slots = max_reqs + max_snapshots
        self.free_snapshot_slots: List[int] = list(range(self.total_slots - 1, max_reqs - 1, -1))
        self.is_snapshot_occupied: Dict[int, bool] = {
            s: False for s in range(max_reqs, self.total_slots)}
        self.state_debug_tags: List[Optional[str]] = [None] * self.total_slots
        self.conv_state = conv_state
        self.ssm_state = ssm_state

    def _copy(self, src, dst) -> None:
        if self.conv_state is not None and self.ssm_state is not None:
            slots_copy(self.conv_state, self.ssm_state, [src], [dst])

    def reset_working_state(self, req_idx: int) -> None:
        assert 0 <= req_idx < self.max_reqs
        self._copy(None, req_idx)
        self.state_debug_tags[req_idx] = "ZERO_STATE"

    def alloc_snapshot(self) -> Optional[int]:
        if not self.free_snapshot_slots:
            return None
        slot = self.free_snapshot_slots.pop()
        assert not self.is_snapshot_occupied[slot]
        self.is_snapshot_occupied[slot] = True
        return slot

    def free_snapshot(self, slot: int) -> None:
        assert self.max_reqs <= slot < self.total_slots
        assert self.is_snapshot_occupied[slot]
        self.is_snapshot_occupied[slot] = False
        self._copy(None, slot)
        self.state_debug_tags[slot] = None
        self.free_snapshot_slots.append(slot)

    def free_snapshots(self, slots: Sequence[int]) -> None:  # req_to_state_pool.py:155-158
        for s in slots:
            self.free_snapshot(s)

    def capture_snapshot(self, req_idx: int, snapshot_slot: int,
                         debug_tag: Optional[str] = None) -> None:
        assert 0 <= req_idx < self.max_reqs
        assert self.max_reqs <= snapshot_slot < self.total_slots
        assert self.is_snapshot_occupied[snapshot_slot]
        self._copy(req_idx, snapshot_slot)
        self.state_debug_tags[snapshot_slot] = (
            debug_tag or self.state_debug_tags[req_idx] or f"Snap(from_req_{req_idx})")

    def restore_snapshot(self, snapshot_slot: int, req_idx: int) -> None:
        assert 0 <= req_idx < self.max_reqs
        assert self.max_reqs <= snapshot_slot < self.total_slots
        assert self.is_snapshot_occupied[snapshot_slot]
        self._copy(snapshot_slot, req_idx)
        self.state_debug_tags[req_idx] = self.state_debug_tags[snapshot_slot]


def run_script(pool, script: Sequence[tuple]) -> List[Optional[int]]:
    """Apply a script of pool calls (tests/golden/cases.py STATE_POOL_SCRIPT) to any object with
    the ReqToStatePool methods; returns the slots alloc_snapshot() handed out."""
    allocs: List[Optional[int]] = []
    for op in script:
        name, args = op[0], op[1:]
        if name == "alloc":
            allocs.append(pool.alloc_snapshot())
        elif name == "capture":
            pool.capture_snapshot(args[0], args[1], debug_tag=args[2])
        elif name == "restore":
            pool.restore_snapshot(args[0], args[1])
        elif name == "reset":
            pool.reset_working_state(args[0])
        elif name == "free":
            pool.free_snapshot(args[0])
        else:
            raise ValueError(f"unknown pool call {name}")
    return allocs


def bookkeeping(pool) -> Tuple[List[int], List[bool], List[str]]:
    """(free stack, occupancy in slot order, debug tags with None as "") of a pool."""
    occ = [bool(pool.is_snapshot_occupied[s]) for s in range(pool.max_reqs, pool.total_slots)]
    tags = ["" if t is None else str(t) for t in pool.state_debug_tags]
    return list(pool.free_snapshot_slots), occ, tags
