"""GPU parity of the GDN state-slot snapshots (tf_state_slots_copy) through the C ABI.

Every operation is a whole-slot copy or zeroing, so results must be bit-exact: against the
reference's own ReqToStatePool (golden script), and against the oracle for batched calls, both
pool layouts (layer-major as the reference allocates, slot-major views), tiles with ragged tails,
the unaligned byte path, out-of-range slots (recorded, op skipped) and src == dst.
"""

import numpy as np
import pytest

from oracle import state_pool as OS
from tests.golden import cases as C
from tests.golden.load import state_pool_case
from tests.helpers import to_numpy, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_golden_script_through_dropin_pool():
    from tokenfactory_b200.state_pool import ReqToStatePool
    spec, inp, gold = state_pool_case("pool_bf16_conv_f32_ssm")
    pool = ReqToStatePool(spec["max_reqs"], spec["max_snapshots"])
    pool.conv_state = to_torch(inp["conv_state"], spec["dtype"])
    pool.ssm_state = to_torch(inp["ssm_state"], "f32")
    allocs = OS.run_script(pool, C.STATE_POOL_SCRIPT)
    torch.cuda.synchronize()
    free, occ, tags = OS.bookkeeping(pool)
    assert allocs == gold["allocs"].tolist()
    assert (free, occ, tags) == (gold["free_slots"].tolist(), gold["occupied"].tolist(),
                                 gold["tags"].tolist())
    np.testing.assert_array_equal(to_numpy(pool.conv_state), gold["conv_state"])
    np.testing.assert_array_equal(to_numpy(pool.ssm_state), gold["ssm_state"])


def _pools(rng, L, S, conv_dim, kc, hv, dk, dv, slot_major=False):
    conv = rng.standard_normal((L, S, conv_dim, kc - 1)).astype(np.float32)
    ssm = rng.standard_normal((L, S, hv, dk, dv)).astype(np.float32)
    ct = torch.from_numpy(conv).to("cuda", torch.bfloat16)
    st = torch.from_numpy(ssm).cuda()
    if slot_major:  # [S, L, ...] storage seen as [L, S, ...]
        ct = ct.transpose(0, 1).contiguous().transpose(0, 1)
        st = st.transpose(0, 1).contiguous().transpose(0, 1)
    return ct, st


def _random_batch(rng, S, n):
    slots = rng.permutation(S)
    src, dst = [], []
    for i in range(n):
        d = int(slots[i])
        r = rng.random()
        src.append(None if r < 0.3 else int(slots[n + i]) if r < 0.9 else d)
        dst.append(d)
    return src, dst


@pytest.mark.parametrize("shape", [
    dict(L=5, S=12, conv_dim=1024, kc=4, hv=8, dk=64, dv=64),      # 128 KB ssm slots, 4 tiles
    dict(L=3, S=9, conv_dim=352, kc=4, hv=6, dk=48, dv=48),        # ragged last tile
    dict(L=2, S=7, conv_dim=37, kc=4, hv=3, dk=5, dv=7),           # rows not 16-byte multiples
])
@pytest.mark.parametrize("slot_major", [False, True])
def test_batches_match_oracle(shape, slot_major):
    from tokenfactory_b200 import ops
    rng = np.random.default_rng(sum(shape.values()) + slot_major)
    ct, st = _pools(rng, **shape, slot_major=slot_major)
    conv_ref, ssm_ref = to_numpy(ct).copy(), to_numpy(st).copy()
    for step in range(4):
        src, dst = _random_batch(rng, shape["S"], n=min(4, shape["S"] // 2))
        ops.state_slots_copy(ct, st, src, dst)
        OS.slots_copy(conv_ref, ssm_ref, src, dst)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_numpy(ct), conv_ref)
    np.testing.assert_array_equal(to_numpy(st), ssm_ref)


def test_apply_slot_ops_batches_admission():
    """restores + resets + captures of several requests in one launch equal the reference's
    one-call-at-a-time sequence (oracle pool)."""
    from tokenfactory_b200.state_pool import ReqToStatePool
    rng = np.random.default_rng(5)
    max_reqs, max_snaps = 6, 6
    ct, st = _pools(rng, 4, max_reqs + max_snaps, 256, 4, 4, 32, 32)
    pool = ReqToStatePool(max_reqs, max_snaps)
    pool.conv_state, pool.ssm_state = ct, st
    orc = OS.StatePool(max_reqs, max_snaps, to_numpy(ct).copy(), to_numpy(st).copy())
    for p in (pool, orc):
        for _ in range(4):
            p.alloc_snapshot()           # slots 6..9
        p.capture_snapshot(0, 6, "a")
        p.capture_snapshot(1, 7, None)
    pool.apply_slot_ops(restores=[(6, 2), (7, 3)], resets=[4], captures=[(5, 8, "c"), (0, 9, None)])
    orc.restore_snapshot(6, 2)
    orc.restore_snapshot(7, 3)
    orc.reset_working_state(4)
    orc.capture_snapshot(5, 8, "c")
    orc.capture_snapshot(0, 9, None)
    pool.free_snapshots([7, 8])
    orc.free_snapshots([7, 8])
    torch.cuda.synchronize()
    assert OS.bookkeeping(pool) == OS.bookkeeping(orc)
    np.testing.assert_array_equal(to_numpy(pool.conv_state), orc.conv_state)
    np.testing.assert_array_equal(to_numpy(pool.ssm_state), orc.ssm_state)
    with pytest.raises(ValueError):  # slot 2 written by a restore and read by a capture
        pool.apply_slot_ops(restores=[(6, 2)], captures=[(2, 9, None)])


def test_out_of_range_slots_are_recorded_and_skipped():
    from tokenfactory_b200 import _capi, ops
    rng = np.random.default_rng(9)
    ct, st = _pools(rng, 2, 6, 64, 4, 2, 16, 16)
    conv_ref, ssm_ref = to_numpy(ct).copy(), to_numpy(st).copy()
    src = torch.tensor([1, 9, -1, 2, -5], dtype=torch.int64, device="cuda")
    dst = torch.tensor([0, 3, 4, 2, 5], dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.state_slots_copy(ct, st, src, dst, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == _capi.TF_KERR_SLOT_RANGE
    OS.slots_copy(conv_ref, ssm_ref, [1, None], [0, 4])  # ops 2 and 5 skipped, op 4 a no-op
    np.testing.assert_array_equal(to_numpy(ct), conv_ref)
    np.testing.assert_array_equal(to_numpy(st), ssm_ref)
