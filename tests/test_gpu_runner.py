"""GPU checks of the per-step runtime (tf_req_to_token_sync, tf_sample_tokens, graph capture).

* prepare_forward_batch reproduces the reference's _prepare_forward_batch fixture bit for bit,
  through the ModelRunner mixin, without a host synchronisation;
* greedy sampling equals torch.argmax (ties, NaN rows, fp32 / bf16, vector and scalar paths);
  temperature sampling picks the index whose float64 CDF bracket holds the uniform and follows
  softmax(x / T) in distribution;
* a decode step (KV store + paged decode + GDN decode) captured as a CUDA graph and replayed with
  new inputs gives the eager results bit for bit.
"""

from types import SimpleNamespace

import numpy as np
import pytest

from oracle import runner as OR
from tests.golden import cases as C
from tests.golden.load import _npz

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _gold(i):
    z = _npz("runner_golden.npz")
    return {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(f"step{i}/")}


def test_prepare_forward_batch_matches_reference_fixture():
    from tokenfactory_b200.runner import ModelRunnerHotPath
    case = C.RUNNER_CASE
    runner = SimpleNamespace(device="cuda", _req_synced_lens=[0] * case["max_reqs"],
                             req_to_token_tensor=torch.full((case["max_reqs"], case["max_ctx"]),
                                                            -1, dtype=torch.int64, device="cuda"))
    for i, (reqs, table, dirty) in enumerate(C.runner_script()):
        g = _gold(i)
        d = None if dirty is None else list(dirty)
        torch.cuda.set_sync_debug_mode("error")  # any host synchronisation raises
        try:
            ids, pos, fb = ModelRunnerHotPath._prepare_forward_batch(
                runner, [SimpleNamespace(**r) for r in reqs], table, d)
        finally:
            torch.cuda.set_sync_debug_mode("default")
        torch.cuda.synchronize()
        got = dict(input_ids=ids, positions=pos, out_cache_loc=fb.out_cache_loc,
                   req_pool_indices=fb.req_pool_indices, seq_lens=fb.seq_lens,
                   prefix_lens=fb.prefix_lens, extend_lens=fb.extend_lens_tensor)
        for k, v in got.items():
            np.testing.assert_array_equal(v.cpu().numpy(), g[k], err_msg=f"step {i} {k}")
        assert [fb.batch_size, int(fb.is_prefill), fb.max_seq_len, fb.max_extend_len] == \
            g["meta"].tolist()
        assert fb.req_pool_indices_list == g["req_pool_indices"].tolist()
        np.testing.assert_array_equal(runner.req_to_token_tensor.cpu().numpy(), g["req_to_token"])
        assert runner._req_synced_lens == g["synced_lens"].tolist()
        if d is not None:
            assert d == g["dirty_from"].tolist()


def test_req_to_token_sync_records_bad_segments():
    from tokenfactory_b200 import _capi, ops
    r2t = torch.full((3, 10), -1, dtype=torch.int64, device="cuda")
    vals = torch.arange(100, 120, dtype=torch.int64, device="cuda")
    segs = torch.tensor([[0, 2, 3, 0], [1, 8, 3, 3], [5, 0, 1, 0], [2, 0, 4, 18], [2, 5, 5, 10]],
                        dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.req_to_token_sync(r2t, segs, vals, err=err)
    want = np.full((3, 10), -1, np.int64)
    want[0, 2:5] = [100, 101, 102]
    want[2, 5:10] = np.arange(110, 115)
    np.testing.assert_array_equal(r2t.cpu().numpy(), want)
    assert int(err.item()) == _capi.TF_KERR_REQ_RANGE


@pytest.mark.parametrize("dtype,V", [(torch.bfloat16, 248320), (torch.float32, 151936),
                                     (torch.bfloat16, 1001), (torch.float16, 4099)])
def test_greedy_matches_torch_argmax(dtype, V):
    from tokenfactory_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(V)
    x = torch.randn((40, V), generator=g, device="cuda").to(dtype)
    x[3, 17] = x[3, 900] = x[3].max() + 1      # tie: the first maximum wins
    x[5, :] = 0.0                               # all equal
    x[7, 123] = float("nan")                    # NaN counts as the maximum
    x[8, V - 1] = x[8].max() + 2                # maximum in the last element (ragged tail)
    got = ops.sample_tokens(x, torch.zeros(40, device="cuda"))
    torch.testing.assert_close(got, torch.argmax(x, dim=-1), rtol=0, atol=0)
    rows = torch.tensor([0, 3, 5, 7], device="cuda")  # a uniform only matters where T > 1e-5
    got = ops.sample_tokens(x[rows], torch.zeros(4, device="cuda"),
                            torch.rand(4, device="cuda", generator=g))
    torch.testing.assert_close(got, torch.argmax(x[rows], dim=-1), rtol=0, atol=0)


def test_temperature_draw_lands_in_its_cdf_bracket():
    from tokenfactory_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(3)
    B, V = 96, 5000
    x = (torch.randn((B, V), generator=g, device="cuda") * 3).to(torch.bfloat16)
    temp = torch.rand(B, generator=g, device="cuda") * 1.5 + 0.1
    u = torch.rand(B, generator=g, device="cuda")
    u[0], u[1] = 0.0, 0.999999
    got = ops.sample_tokens(x, temp, u).cpu().numpy()
    xs, ts, us = x.float().cpu().numpy(), temp.cpu().numpy(), u.cpu().numpy()
    for b in range(B):
        lo, hi, want = OR.inverse_cdf_bracket(xs[b], float(ts[b]), float(us[b]))
        i = int(got[b])
        assert lo[i] <= us[b] + 1e-5 and hi[i] >= us[b] - 1e-5, (b, i, want)


def test_temperature_draws_follow_softmax():
    from tokenfactory_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(5)
    logits = torch.tensor([1.0, 0.2, -0.5, 2.0, 0.0, -3.0], device="cuda")
    N, T = 16384, 0.7
    x = logits.expand(N, -1).contiguous()
    got = ops.sample_tokens(x, torch.full((N,), T, device="cuda"),
                            torch.rand(N, generator=g, device="cuda"))
    freq = torch.bincount(got, minlength=6).double().cpu().numpy() / N
    p = torch.softmax(logits.double() / T, 0).cpu().numpy()
    sigma = np.sqrt(p * (1 - p) / N)
    assert np.all(np.abs(freq - p) <= 5 * sigma + 1e-9), (freq, p)


def test_captured_decode_step_matches_eager():
    from tokenfactory_b200 import ops
    from tokenfactory_b200.runner import CapturedStep
    g = torch.Generator(device="cuda").manual_seed(11)
    B, S, Hq, Hkv, D, maxL = 24, 20000, 8, 2, 128, 600
    nk, nv, dk, dv, K = 2, 4, 64, 64, 4
    conv_dim = 2 * nk * dk + nv * dv
    bf = torch.bfloat16
    pools = dict(kb=torch.randn((S, Hkv, D), generator=g, device="cuda", dtype=bf),
                 vb=torch.randn((S, Hkv, D), generator=g, device="cuda", dtype=bf),
                 conv=torch.randn((B + 4, conv_dim, K - 1), generator=g, device="cuda", dtype=bf),
                 ssm=torch.randn((B + 4, nv, dk, dv), generator=g, device="cuda") * 0.02)
    r2t = torch.randint(1, S, (B, maxL), generator=g, device="cuda")
    w = torch.randn((conv_dim, 1, K), generator=g, device="cuda", dtype=bf) * 0.5
    A_log = (torch.rand((nv,), generator=g, device="cuda") * 1.5).to(bf)
    dt_bias = torch.randn((nv,), generator=g, device="cuda", dtype=bf) * 0.5

    def inputs():
        return dict(q=torch.randn((B, Hq, D), generator=g, device="cuda", dtype=bf),
                    gate=torch.randn((B, Hq, D), generator=g, device="cuda", dtype=bf),
                    k=torch.randn((B, Hkv, D), generator=g, device="cuda", dtype=bf),
                    v=torch.randn((B, Hkv, D), generator=g, device="cuda", dtype=bf),
                    loc=torch.randperm(S - 1, generator=g, device="cuda")[:B] + 1,
                    rpi=torch.randperm(B + 4, generator=g, device="cuda")[:B],
                    lens=torch.randint(1, maxL + 1, (B,), generator=g, device="cuda"),
                    qkv=torch.randn((B, conv_dim), generator=g, device="cuda", dtype=bf),
                    b=torch.randn((B, nv), generator=g, device="cuda", dtype=bf),
                    a=torch.randn((B, nv), generator=g, device="cuda", dtype=bf))

    def step(P, q, gate, k, v, loc, rpi, lens, qkv, b, a):
        ops.kv_store(P["kb"], P["vb"], loc, k, v)
        o = ops.paged_decode(q, P["kb"], P["vb"], r2t, rpi, lens, D ** -0.5, maxL, gate=gate,
                             gate_mode="sigmoid")
        y = ops.gdn_decode(qkv, b, a, w, A_log, dt_bias, P["conv"], P["ssm"], rpi,
                           num_k_heads=nk, head_k_dim=dk, head_v_dim=dv)
        return o, y

    graph_pools = {k: v.clone() for k, v in pools.items()}
    cap = CapturedStep(lambda **kw: step(graph_pools, **kw), inputs())
    eager_pools = {k: v.clone() for k, v in graph_pools.items()}  # state after the capture runs
    for _ in range(3):
        inp = inputs()
        go, gy = cap(**inp)
        eo, ey = step(eager_pools, **inp)
        torch.cuda.synchronize()
        assert torch.equal(go, eo) and torch.equal(gy, ey)
        for k in pools:
            assert torch.equal(graph_pools[k], eager_pools[k]), k


def test_pipelined_decode_step_matches_eager():
    """PipelinedStep: every submit's host output equals the eager step on the same inputs, with
    the steps' in-place pool updates applied in submission order."""
    from tokenfactory_b200 import ops
    from tokenfactory_b200.runner import PipelinedStep
    g = torch.Generator(device="cuda").manual_seed(12)
    B, S, Hq, Hkv, D, maxL = 20, 12000, 8, 2, 128, 500
    bf = torch.bfloat16
    pools = dict(kb=torch.randn((S, Hkv, D), generator=g, device="cuda", dtype=bf),
                 vb=torch.randn((S, Hkv, D), generator=g, device="cuda", dtype=bf))
    # distinct slots, as the allocator hands them out: two tokens of one step never share a slot
    r2t = (torch.randperm(S - 1, generator=g, device="cuda")[:B * maxL] + 1).view(B, maxL)

    def inputs():
        d = dict(q=torch.randn((B, Hq, D), generator=g, device="cuda", dtype=bf),
                 gate=torch.randn((B, Hq, D), generator=g, device="cuda", dtype=bf),
                 k=torch.randn((B, Hkv, D), generator=g, device="cuda", dtype=bf),
                 v=torch.randn((B, Hkv, D), generator=g, device="cuda", dtype=bf),
                 # a few slots of each step lie in the windows later steps read
                 loc=r2t[torch.arange(B, device="cuda"), torch.randint(0, 50, (B,), generator=g,
                                                                        device="cuda")],
                 rpi=torch.randperm(B, generator=g, device="cuda"),
                 lens=torch.randint(1, maxL + 1, (B,), generator=g, device="cuda"))
        return {k: v.cpu().pin_memory() for k, v in d.items()}

    def step(P, q, gate, k, v, loc, rpi, lens):
        ops.kv_store(P["kb"], P["vb"], loc, k, v)
        o = ops.paged_decode(q, P["kb"], P["vb"], r2t, rpi, lens, D ** -0.5, maxL, gate=gate,
                             gate_mode="sigmoid")
        return o, o.float().sum(dim=-1)

    pipe_pools = {k: v.clone() for k, v in pools.items()}
    eager_pools = {k: v.clone() for k, v in pipe_pools.items()}
    # the pools are in-place state: construction's warm-up runs must leave them as they were
    pipe = PipelinedStep(lambda **kw: step(pipe_pools, **kw), inputs(),
                         state=list(pipe_pools.values()))
    torch.cuda.synchronize()
    for k in pools:
        assert torch.equal(pipe_pools[k], eager_pools[k]), f"{k} changed by construction"
    steps = [inputs() for _ in range(6)]
    pending = []
    for i, inp in enumerate(steps):
        pending.append((pipe.submit(**inp), step(eager_pools, **{k: v.cuda() for k, v in inp.items()})))
        if len(pending) == 2:  # a buffer set's host outputs are read before it is submitted again
            res, (eo, es) = pending.pop(0)
            po, ps = res.wait()
            assert torch.equal(po, eo.cpu()) and torch.equal(ps, es.cpu())
    res, (eo, es) = pending.pop(0)
    po, ps = res.wait()
    assert torch.equal(po, eo.cpu()) and torch.equal(ps, es.cpu())
    pipe.join()
    torch.cuda.synchronize()
    for k in pools:
        assert torch.equal(pipe_pools[k], eager_pools[k]), k
