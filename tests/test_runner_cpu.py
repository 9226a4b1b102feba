"""Per-step runtime (ForwardBatch construction, req_to_token sync, sampling) on CPU.

* the oracle restatement reproduces the reference's _prepare_forward_batch fixture;
* the host packing (pack_batch) gives the same flattened tensors, and its sync segments, applied
  to the table, the same req_to_token, synced lengths and dirty_from as the reference;
* the mixin keeps the reference's method signatures and installs over its ModelRunner;
* the product path refuses CPU tensors (no CPU fallback).
"""

import inspect
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import runner as OR
from tests.golden import cases as C
from tests.golden.load import _npz


def _gold(i):
    z = _npz("runner_golden.npz")
    return {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(f"step{i}/")}


def test_oracle_matches_reference_fixture():
    case = C.RUNNER_CASE
    r2t = np.full((case["max_reqs"], case["max_ctx"]), -1, np.int64)
    synced = [0] * case["max_reqs"]
    for i, (reqs, table, dirty) in enumerate(C.runner_script()):
        g = _gold(i)
        d = None if dirty is None else list(dirty)
        res = OR.prepare_forward_batch(reqs, table, r2t, synced, d)
        for k, v in res.items():
            np.testing.assert_array_equal(v, g[k], err_msg=f"step {i} {k}")
        np.testing.assert_array_equal(r2t, g["req_to_token"])
        assert synced == g["synced_lens"].tolist()
        if d is not None:
            assert d == g["dirty_from"].tolist()


def test_pack_batch_segments_reproduce_reference():
    from tokenfactory_b200.runner import pack_batch
    case = C.RUNNER_CASE
    r2t = np.full((case["max_reqs"], case["max_ctx"]), -1, np.int64)
    synced = [0] * case["max_reqs"]
    for i, (reqs, table, dirty) in enumerate(C.runner_script()):
        g = _gold(i)
        d = None if dirty is None else list(dirty)
        pk = pack_batch([SimpleNamespace(**r) for r in reqs], table, synced, d)
        h, B, T = pk.host, pk.B, pk.T
        for name, off, n in (("input_ids", pk.o_ids, T), ("positions", pk.o_pos, T),
                             ("out_cache_loc", pk.o_loc, T), ("req_pool_indices", pk.o_rpi, B),
                             ("seq_lens", pk.o_seq, B), ("prefix_lens", pk.o_pre, B),
                             ("extend_lens", pk.o_ext, B)):
            np.testing.assert_array_equal(h[off:off + n], g[name], err_msg=f"step {i} {name}")
        for row, col, ln, src in pk.segments():  # what tf_req_to_token_sync does
            r2t[row, col:col + ln] = h[src:src + ln]
        np.testing.assert_array_equal(r2t, g["req_to_token"], err_msg=f"step {i}")
        assert synced == g["synced_lens"].tolist()
        assert [pk.B, int(pk.is_prefill), max(pk.seq), max(pk.ext)] == g["meta"].tolist()
        if d is not None:
            assert d == g["dirty_from"].tolist()


def test_sampling_oracle_follows_torch_argmax():
    rng = np.random.default_rng(1)
    for _ in range(20):
        x = rng.standard_normal(50).astype(np.float32)
        x[rng.integers(0, 50, 3)] = x.max()          # ties: the first maximum wins
        assert OR.argmax_first(x) == int(torch.argmax(torch.from_numpy(x)))
    x = np.array([1.0, np.nan, 3.0, np.nan], np.float32)
    assert OR.argmax_first(x) == int(torch.argmax(torch.from_numpy(x))) == 1
    lo, hi, i = OR.inverse_cdf_bracket(np.array([0.0, 0.0, 0.0, 0.0], np.float32), 1.0, 0.6)
    assert i == 2 and lo[i] <= 0.6 < hi[i]


def test_dropin_runner_over_reference(reference_root):
    import engine.model_runner as mr

    from tokenfactory_b200 import runner as R
    ref = mr.ModelRunner
    for name in ("_prepare_forward_batch", "_sample"):
        ours = inspect.signature(getattr(R.ModelRunnerHotPath, name)).parameters
        theirs = inspect.signature(getattr(ref, name)).parameters
        assert [(n, p.default) for n, p in ours.items()] == \
            [(n, p.default) for n, p in theirs.items()], name
    cls = R.install()
    try:
        assert mr.ModelRunner is cls and issubclass(cls, ref)
        from qwen3_8.forward_batch import ForwardBatch as RefFB
        assert R._forward_batch_cls(object.__new__(cls)) is RefFB
    finally:
        R.uninstall()
    assert mr.ModelRunner is ref


def test_no_cpu_fallback():
    from tokenfactory_b200 import ops, runner
    r2t = torch.full((4, 16), -1, dtype=torch.int64)
    req = SimpleNamespace(req_pool_idx=0, cur_start_pos=0, cur_seq_len=2, cur_chunk_tokens=[1, 2],
                          out_cache_loc=[5, 6], is_prefilled=False)
    with pytest.raises(ValueError, match="CUDA"):
        runner.prepare_forward_batch([req], [[-1] * 16] * 4, r2t, [0] * 4)
    with pytest.raises(ValueError, match="CUDA"):
        ops.sample_tokens(torch.zeros(2, 8), torch.zeros(2))


def test_pipelined_step_needs_two_buffer_sets():
    """A single buffer set could not overlap one step's copies with another step's kernels."""
    from tokenfactory_b200.runner import PipelinedStep
    with pytest.raises(ValueError, match="depth"):
        PipelinedStep(lambda **kw: None, {}, depth=1)
