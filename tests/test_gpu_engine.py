"""Engine-level parity on the GPU: whole runs of the reference's own engine replayed on the kernels.

The reference's Scheduler / ModelRunner / RadixCache ran these workloads on the CPU in fp32
(tests/golden/make_engine_golden.py); the same events replay here through the drop-in model
(tokenfactory_b200.hybrid_model: the paged attention, GDN and state-slot kernels), with the same
weights.  Greedy tokens must be identical at every step and the logits within fp32 tolerance
(max-abs 1e-3 on the top-16 logits of every row, values of a few units).

* BASELINE config 1 (4 requests, 16/32/48/64 prompt tokens, 32 greedy tokens each, chunked
  prefill mixed with decode, sigmoid output gate);
* the reference's prefix-reuse pin (tests/test_hybrid_radix_cache.py:111-223): the request that
  restores the radix cache's GDN snapshot and extends over the cached KV prefix gives the token a
  fresh recompute gives;
* the reference's TP pin (tests/test_tensor_parallel.py:93-271): two tensor-parallel ranks (one
  thread each, a barrier all-reduce, both on this GPU) give the tp_size=1 logits within 1e-5,
  with 8 all-reduces per rank and the GDN states of the two ranks concatenating to the full one.
"""

import threading

import numpy as np
import pytest

from tests import engine_replay as R

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LOGIT_ATOL = 1e-3


def _check_run(run: str):
    got = R.replay(run)
    ref = R.forwards(run)
    assert len(got) == len(ref)
    worst = 0.0
    for i, ((vals, toks, full), f) in enumerate(zip(got, ref)):
        d = np.abs(vals.astype(np.float64) - f["top_val"].astype(np.float64))
        worst = max(worst, float(d.max()))
        assert d.max() <= LOGIT_ATOL, f"{run} forward {i}: top-16 logits differ by {d.max():.3g}"
        np.testing.assert_allclose(full.sum(axis=1), f["row_sum"], rtol=1e-4, atol=0.05,
                                   err_msg=f"{run} forward {i}: row sums")
        np.testing.assert_array_equal(toks, f["tokens"], err_msg=f"{run} forward {i}: tokens")
    return got, worst


def test_config1_engine_run_tokens_identical():
    got, worst = _check_run("config1")
    m = R.meta("config1")
    # the tokens each request was handed: the last token of each of its forwards once prefilled
    outs = m["outputs"][0]
    fwd = R.forwards("config1")
    produced = {}
    for (vals, toks, _), f in zip(got, fwd):
        for i, r in enumerate(f["req_pool_indices"].tolist()):
            produced.setdefault(r, []).append(int(toks[i]))
    tails = sorted(tuple(v[-32:]) for v in produced.values())
    assert tails == sorted(tuple(o) for o in outs), "greedy outputs differ from the reference run"
    print(f"config1: {len(got)} forwards, top-16 logits within {worst:.2e}")


def test_prefix_reuse_matches_fresh_recompute():
    cached, _ = _check_run("prefix_cached")
    fresh, _ = _check_run("prefix_fresh")
    assert R.meta("prefix_cached")["cached_prefix_lens"][-1] == [6]
    ev = R.events("prefix_cached").tolist()
    assert any(k == 2 and a >= R.meta("prefix_cached")["sched"]["max_reqs"] for k, a, _ in ev), \
        "the cached run restores a GDN snapshot"
    assert int(cached[-1][1][0]) == int(fresh[-1][1][0]) == R.meta("prefix_fresh")["outputs"][0][0][0]


def test_tp2_equals_tp1_with_fake_all_reduce():
    import tokenfactory_b200  # noqa: F401
    from tokenfactory_b200 import ForwardBatch
    from tokenfactory_b200.hybrid_model import HybridCachePool
    from tests.golden import cases as C

    z = R.fixture()
    full = R.build_model("tp")
    tp = 2
    ranks = [R.build_model("tp", tp_size=tp, tp_rank=r, full=full) for r in range(tp)]
    pools = [HybridCachePool(m.config, 32, 4, 4, dtype=torch.float32) for m in [full] + ranks]
    assert pools[1].k_buffer.shape[2] == pools[0].k_buffer.shape[2] // tp
    assert pools[1].ssm_state.shape[2] == pools[0].ssm_state.shape[2] // tp
    assert pools[1].conv_state.shape[2] == pools[0].conv_state.shape[2] // tp

    barrier = threading.Barrier(tp)
    shared = [None] * tp
    counts = [0] * tp

    def all_reduce_for(rank):
        def _ar(x):
            shared[rank] = x
            counts[rank] += 1
            barrier.wait()
            s = shared[0] + shared[1]
            barrier.wait()
            return s
        return _ar

    for r, m in enumerate(ranks):
        m.set_all_reduce_fn(all_reduce_for(r))
    r2t = torch.full((4, 16), -1, dtype=torch.long, device="cuda")

    def batch(b):
        for r, row in b["rows"].items():
            r2t[r, :len(row)] = torch.tensor(row, device="cuda")
        dev = lambda k: torch.tensor(b[k], device="cuda")  # noqa: E731
        return ForwardBatch(batch_size=2, req_pool_indices=dev("req_pool_indices"),
                            seq_lens=dev("seq_lens"), prefix_lens=dev("prefix_lens"),
                            extend_lens=list(b["extend_lens"]),
                            out_cache_loc=dev("out_cache_loc"), req_to_token=r2t,
                            is_prefill=max(b["extend_lens"]) > 1)

    def run_all(ids, spec):
        fb = batch(spec)
        pos = torch.tensor(spec["positions"], device="cuda")
        ref = full(ids, pos, pools[0], fb)
        outs = [None] * tp

        def go(r):
            outs[r] = ranks[r](ids, pos, pools[1 + r], fb)

        ts = [threading.Thread(target=go, args=(r,)) for r in range(tp)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        torch.cuda.synchronize()
        return ref, outs

    ids = torch.from_numpy(z["tp/input_ids"]).cuda()
    ref, outs = run_all(ids, C.TP_PREFILL)
    assert counts == [8, 8], counts
    for o in outs:
        torch.testing.assert_close(o, ref, atol=1e-5, rtol=0)
    np.testing.assert_allclose(ref.cpu().numpy(), z["tp/prefill_logits"], atol=1e-4, rtol=0)
    ssm = torch.cat([pools[1].ssm_state, pools[2].ssm_state], dim=2)
    torch.testing.assert_close(ssm, pools[0].ssm_state, atol=1e-5, rtol=0)
    np.testing.assert_allclose(pools[0].ssm_state[:, :2].cpu().numpy(),
                               z["tp/ssm_state_after_prefill"], atol=1e-5, rtol=1e-4)

    dec_ids = torch.argmax(ref, dim=-1)
    assert dec_ids.tolist() == z["tp/decode_ids"].tolist()
    ref, outs = run_all(dec_ids, C.TP_DECODE)
    for o in outs:
        torch.testing.assert_close(o, ref, atol=1e-5, rtol=0)
    np.testing.assert_allclose(ref.cpu().numpy(), z["tp/decode_logits"], atol=1e-4, rtol=0)
