"""Head-sharded runs of the kernels reproduce the unsharded result (one GPU, tp 2/4/8 emulated).

Each emulated rank gets exactly what the reference's TP split gives it (tokenfactory_b200.tp):
its query heads, its kv heads of the pool (one replicated head when tp > Hkv), its GDN heads and
conv channels; the concatenated per-rank outputs and states must equal the tp=1 run.
"""

import numpy as np
import pytest

from tests.golden import cases as C
from tests.helpers import assert_close, to_numpy, to_torch, values

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_paged_decode_head_shards(world):
    from tokenfactory_b200 import ops
    from tokenfactory_b200.tp import head_shard
    rng = np.random.default_rng(world)
    B, hq, hkv, d = 6, 32, 4, 256
    seq = [int(x) for x in rng.integers(1, 2000, B)]
    spec = dict(dtype="bf16", hq=hq, hkv=hkv, d=d, seq=seq, ext=[1] * B, req=list(range(B)),
                slots=sum(seq) + 5, rows=B, cols=2000, seed=90 + world)
    t = {k: to_torch(v, "bf16") for k, v in C.attn_inputs(spec).items()}
    args = (t["req_to_token"], t["req_pool_indices"], t["seq_lens"], d ** -0.5, max(seq))
    full = ops.paged_decode(t["q"], t["k_buf"], t["v_buf"], *args, gate=t["gate"],
                            gate_mode="sigmoid")
    parts = []
    for r in range(world):
        sh = head_shard(hq, hkv, world, world, r, world)
        qh = slice(sh.q_heads.start, sh.q_heads.stop)
        kvh = slice(sh.kv_heads.start, sh.kv_heads.stop)
        kb = t["k_buf"][:, kvh].contiguous()  # this rank's pool holds only its kv heads
        vb = t["v_buf"][:, kvh].contiguous()
        parts.append(ops.paged_decode(t["q"][:, qh].contiguous(), kb, vb, *args,
                                      gate=t["gate"][:, qh], gate_mode="sigmoid"))
    torch.cuda.synchronize()
    assert_close(values(torch.cat(parts, dim=1), "bf16"), values(full, "bf16"), "bf16",
                 what=f"tp{world} decode shards")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gdn_decode_head_shards(world):
    from tokenfactory_b200 import ops
    from tokenfactory_b200.tp import gdn_conv_channels, head_shard
    spec = dict(dtype="bf16", nk=8, nv=24, dk=128, dv=128, kc=4, ext=[1] * 3, req=[2, 0, 3],
                slots=4, seed=95 + world)
    inp = C.gdn_inputs(spec)
    T = {k: to_torch(v, "f32" if k == "ssm_state" else "bf16") for k, v in inp.items()}
    full_cs, full_ss = T["conv_state"].clone(), T["ssm_state"].clone()
    full = ops.gdn_decode(T["qkv"], T["b"], T["a"], T["conv_weight"], T["A_log"], T["dt_bias"],
                          full_cs, full_ss, T["req_pool_indices"], num_k_heads=8, head_k_dim=128,
                          head_v_dim=128, z=T["z"], norm_weight=T["norm_weight"])
    outs = []
    for r in range(world):
        sh = head_shard(world, world, 8, 24, r, world)
        ch = torch.tensor(gdn_conv_channels(sh, 128, 128, 8), device="cuda")
        vh = slice(sh.v_heads.start, sh.v_heads.stop)
        vd = slice(sh.v_heads.start * 128, sh.v_heads.stop * 128)
        cs = T["conv_state"][:, ch].contiguous()
        ss = T["ssm_state"][:, vh].contiguous()
        out = ops.gdn_decode(T["qkv"][:, ch].contiguous(), T["b"][:, vh].contiguous(),
                             T["a"][:, vh].contiguous(), T["conv_weight"][ch], T["A_log"][vh],
                             T["dt_bias"][vh], cs, ss, T["req_pool_indices"],
                             num_k_heads=8 // world, head_k_dim=128, head_v_dim=128,
                             z=T["z"][:, vd].contiguous(), norm_weight=T["norm_weight"][vd])
        outs.append(out)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(to_numpy(cs), to_numpy(full_cs[:, ch]))
        np.testing.assert_array_equal(to_numpy(ss), to_numpy(full_ss[:, vh]))
    np.testing.assert_array_equal(to_numpy(torch.cat(outs, dim=1)), to_numpy(full))
