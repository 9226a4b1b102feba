"""CPU checks of the recorded reference-engine runs and of the drop-in model's surface.

* the drop-in model (tokenfactory_b200.hybrid_model) has exactly the reference model's state_dict
  names and shapes, so the seeded weights the recorder loaded into the reference load into it;
* each recorded run is a consistent trace: forwards appear in order, a request's decode input is
  the token the previous forward produced for it (so replaying the recorded inputs is the same as
  feeding back greedy tokens), and every output the reference returned is one of those tokens.
"""

import pytest

from tests import engine_replay as R
from tests.golden import cases as C

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("run", ["config1", "prefix_cached", "tp"])
def test_dropin_model_has_the_reference_state_dict(run):
    from tokenfactory_b200.hybrid_model import HybridForCausalLM
    import json
    model = R.meta(run)["model"] if run != "tp" else "tp"
    keys = R.meta(run)["state_dict_keys"] if run != "tp" else json.loads(
        bytes(R.fixture()["tp/state_dict_keys"]).decode())
    m = HybridForCausalLM(R.hybrid_config(model))
    assert sorted(m.state_dict().keys()) == keys
    w = C.engine_weights({k: tuple(v.shape) for k, v in m.state_dict().items()},
                         C.ENGINE_WEIGHT_SEED[model])
    m.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()})


@pytest.mark.parametrize("run", sorted(C.ENGINE_RUNS))
def test_recorded_run_is_a_consistent_greedy_trace(run):
    fwd = R.forwards(run)
    ev = R.events(run)
    assert [a for k, a, _ in ev.tolist() if k == 0] == list(range(len(fwd)))
    last = {}
    for f in fwd:
        off = 0
        for i, r in enumerate(f["req_pool_indices"].tolist()):
            n = int(f["extend_lens"][i])
            if n == 1 and r in last:
                assert int(f["input_ids"][off]) == last[r], "decode input is the previous token"
            assert int(f["seq_lens"][i]) == int(f["prefix_lens"][i]) + n
            assert (f["r2t"][i, int(f["prefix_lens"][i]):int(f["seq_lens"][i])] ==
                    f["out_cache_loc"][off:off + n]).all()
            last[r] = int(f["tokens"][i])
            off += n
        assert off == f["input_ids"].shape[0]
    produced = {int(t) for f in fwd for t in f["tokens"]}
    for phase in R.meta(run)["outputs"]:
        for out in phase:
            assert set(out) <= produced
