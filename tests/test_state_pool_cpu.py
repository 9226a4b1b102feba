"""GDN state snapshots (ReqToStatePool, req_to_state_pool.py:34-194) on CPU.

* the oracle replays the golden script and matches the reference's recorded tensors and
  bookkeeping bit for bit;
* the drop-in pool keeps the reference's bookkeeping (free stack, occupancy, tags, assertions) and
  method signatures, installs over the reference class and uninstalls cleanly;
* batches whose result would depend on the order of their copies are rejected;
* with real tensors on the CPU the product path refuses to run (no CPU fallback).
"""

import inspect

import numpy as np
import pytest
import torch

from oracle import state_pool as OS
from tests.golden import cases as C
from tests.golden.load import state_pool_case


def test_oracle_matches_reference_golden_script():
    spec, inp, gold = state_pool_case("pool_bf16_conv_f32_ssm")
    pool = OS.StatePool(spec["max_reqs"], spec["max_snapshots"], inp["conv_state"].copy(),
                        inp["ssm_state"].copy())
    allocs = OS.run_script(pool, C.STATE_POOL_SCRIPT)
    free, occ, tags = OS.bookkeeping(pool)
    assert allocs == gold["allocs"].tolist()
    assert free == gold["free_slots"].tolist()
    assert occ == gold["occupied"].tolist()
    assert tags == gold["tags"].tolist()
    np.testing.assert_array_equal(pool.conv_state, gold["conv_state"])
    np.testing.assert_array_equal(pool.ssm_state, gold["ssm_state"])


def _script_with_frees(pool):
    allocs = OS.run_script(pool, C.STATE_POOL_SCRIPT)
    extra = [pool.alloc_snapshot(), pool.alloc_snapshot()]
    pool.free_snapshots([s for s in extra if s is not None])
    return allocs + extra


def test_mirror_pool_bookkeeping_matches_oracle():
    from tokenfactory_b200.state_pool import ReqToStatePool
    mirror, orc = ReqToStatePool(4, 3), OS.StatePool(4, 3)
    assert _script_with_frees(mirror) == _script_with_frees(orc)
    assert OS.bookkeeping(mirror) == OS.bookkeeping(orc)
    assert mirror.available_snapshot_size() == len(orc.free_snapshot_slots)
    with pytest.raises(AssertionError):
        mirror.free_snapshot(mirror.max_reqs + 1)  # double free (slot 5 is free after the script)
    with pytest.raises(AssertionError):
        mirror.restore_snapshot(mirror.max_reqs + 1, 0)
    with pytest.raises(AssertionError):
        mirror.reset_working_state(mirror.max_reqs)


def test_dropin_over_reference_class(reference_root):
    import req_to_state_pool as ref_mod
    from tokenfactory_b200 import state_pool as SP
    ref_cls = ref_mod.ReqToStatePool
    for name in ("reset_working_state", "free_snapshot", "free_snapshots", "capture_snapshot",
                 "restore_snapshot"):
        ours = inspect.signature(getattr(SP.StatePoolHotPath, name)).parameters
        theirs = inspect.signature(getattr(ref_cls, name)).parameters
        assert [(n, p.default) for n, p in ours.items()] == \
            [(n, p.default) for n, p in theirs.items()], name
    import qwen3_8.hybrid_cache_pool as hcp
    cls = SP.install()
    try:
        assert ref_mod.ReqToStatePool is cls and hcp.ReqToStatePool is cls
        assert issubclass(cls, ref_cls)
        ref_pool, ours = ref_cls(4, 3), cls(4, 3)  # config None: bookkeeping only
        assert _script_with_frees(ours) == _script_with_frees(ref_pool)
        assert OS.bookkeeping(ours) == OS.bookkeeping(ref_pool)
    finally:
        SP.uninstall()
    assert ref_mod.ReqToStatePool is ref_cls and hcp.ReqToStatePool is ref_cls


def test_mirror_pool_allocates_the_reference_shapes(reference_root):
    from qwen3_8 import Qwen3_8Config
    from req_to_state_pool import ReqToStatePool as Ref

    from tokenfactory_b200.state_pool import ReqToStatePool
    for tp in (1, 2):
        cfg = Qwen3_8Config(num_hidden_layers=8, linear_num_key_heads=4, linear_num_value_heads=8,
                            linear_key_head_dim=16, linear_value_head_dim=32, tp_size=tp)
        a, b = Ref(3, 2, config=cfg), ReqToStatePool(3, 2, config=cfg)
        for x, y in ((a.conv_state, b.conv_state), (a.ssm_state, b.ssm_state)):
            assert x.shape == y.shape and x.dtype == y.dtype
        assert a.linear_layer_map == b.linear_layer_map
        assert a.get_layer_states(0)[1].shape == b.get_layer_states(0)[1].shape


def test_order_dependent_batches_are_rejected():
    from tokenfactory_b200 import ops
    ops.state_slot_ops_valid([4, None, 2], [0, 1, 5])  # disjoint: fine
    ops.state_slot_ops_valid([3, 3], [0, 1])            # a shared source: fine
    with pytest.raises(ValueError):
        ops.state_slot_ops_valid([4, 5], [0, 0])        # one slot written twice
    with pytest.raises(ValueError):
        ops.state_slot_ops_valid([4, 0], [0, 5])        # slot 0 read and written
    with pytest.raises(ValueError):
        ops.state_slot_ops_valid([4], [0, 1])


def test_no_cpu_fallback():
    from tokenfactory_b200 import ops
    conv = torch.zeros(2, 5, 8, 3, dtype=torch.bfloat16)
    ssm = torch.zeros(2, 5, 2, 4, 4)
    with pytest.raises(ValueError, match="CUDA"):
        ops.state_slots_copy(conv, ssm, [0], [4])
