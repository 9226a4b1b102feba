"""Tensor-parallel head split of the hot path, on CPU.

* world_size 2 over gloo (127.0.0.1): every rank derives its shard, the gathered shards partition
  the query / GDN heads, kv heads follow the reference's split, and each rank's TP-sliced layer
  weights reassemble into the full layer's;
* the slicing equals the reference's own load_tp_from_full_layer (qwen3_8/full_attention.py:103-110,
  qwen3_8/linear_attention.py:109-131) for tp 2, 4 and 8, when the reference checkout is present.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.golden import cases as C


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg(cls, tp, rank):
    m = C.MODULE_DIMS
    return cls(hidden_size=m["hidden"], num_attention_heads=m["hq"], num_key_value_heads=m["hkv"],
               head_dim=m["d"], linear_num_key_heads=m["nk"], linear_num_value_heads=m["nv"],
               linear_key_head_dim=m["dk"], linear_value_head_dim=m["dv"], tp_size=tp,
               tp_rank=rank)


def _full_layers():
    from tokenfactory_b200 import layers
    torch.manual_seed(0)
    cfg = _cfg(layers.AttentionConfig, 1, 0)
    fa, la = layers.Qwen3_8FullAttention(cfg, 3), layers.Qwen3_8LinearAttention(cfg, 0)
    for p in list(fa.parameters()) + list(la.parameters()):
        torch.nn.init.normal_(p)
    return fa, la


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from tokenfactory_b200 import layers
        from tokenfactory_b200.tp import head_shard
        sh = head_shard(32, 4, 16, 48, rank, world)
        shards = [None] * world
        dist.all_gather_object(shards, (list(sh.q_heads), list(sh.kv_heads), list(sh.k_heads),
                                        list(sh.v_heads)))
        fa, la = _full_layers()
        cfg = _cfg(layers.AttentionConfig, world, rank)
        tfa, tla = layers.Qwen3_8FullAttention(cfg, 3), layers.Qwen3_8LinearAttention(cfg, 0)
        tfa.load_tp_from_full_layer(fa)
        tla.load_tp_from_full_layer(la)
        parts = {}
        for name, t in (("q", tfa.q_proj.weight), ("o", tfa.o_proj.weight),
                        ("z", tla.in_proj_z.weight), ("norm", tla.norm.weight),
                        ("out", tla.out_proj.weight), ("A", tla.A_log)):
            g = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(g, t.contiguous())
            parts[name] = g
        ok = (torch.equal(torch.cat(parts["q"], 0), fa.q_proj.weight) and
              torch.equal(torch.cat(parts["o"], 1), fa.o_proj.weight) and
              torch.equal(torch.cat(parts["z"], 0), la.in_proj_z.weight) and
              torch.equal(torch.cat(parts["norm"], 0), la.norm.weight) and
              torch.equal(torch.cat(parts["out"], 1), la.out_proj.weight) and
              torch.equal(torch.cat(parts["A"], 0), la.A_log))
        dist.destroy_process_group()
        q.put((rank, shards, ok, None))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, None, False, repr(e)))


def test_head_split_and_weight_slicing_over_gloo_world_2():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, shards, ok, err in res:
        assert err is None, err
        assert ok, f"rank {rank}: sliced weights do not reassemble"
    shards = res[0][1]
    qs = sorted(h for s in shards for h in s[0])
    assert qs == list(range(32))
    assert [s[1] for s in shards] == [[0, 1], [2, 3]]
    assert sorted(h for s in shards for h in s[3]) == list(range(48))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_split_replicates_kv_heads_like_the_reference(world):
    from tokenfactory_b200.tp import head_shard
    shards = [head_shard(32, 4, 16, 48, r, world) for r in range(world)]
    assert sorted(h for s in shards for h in s.q_heads) == list(range(32))
    for s in shards:  # each rank's q heads read only its kv heads
        g = 32 // 4
        assert {h // g for h in s.q_heads} <= set(s.kv_heads)
        assert s.kv_replication == max(1, world // 4)


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_slicing_matches_reference_load_tp(reference_root, tp):
    from qwen3_8 import Qwen3_8Config
    from qwen3_8.full_attention import Qwen3_8FullAttention as RefFull
    from qwen3_8.linear_attention import Qwen3_8LinearAttention as RefLin

    from tokenfactory_b200 import layers

    m = C.MODULE_DIMS
    kw = dict(hidden_size=m["hidden"], intermediate_size=64, num_hidden_layers=4,
              layer_types=["linear_attention"] * 3 + ["full_attention"],
              num_attention_heads=16, num_key_value_heads=4, head_dim=m["d"],
              linear_num_key_heads=8, linear_num_value_heads=16, linear_key_head_dim=m["dk"],
              linear_value_head_dim=m["dv"])
    torch.manual_seed(1)
    full_cfg = Qwen3_8Config(**kw)
    ref_fa, ref_la = RefFull(full_cfg, 3), RefLin(full_cfg, 0)
    for p in list(ref_fa.parameters()) + list(ref_la.parameters()):
        torch.nn.init.normal_(p)
    ours_full_cfg = layers.AttentionConfig(**{k: v for k, v in kw.items()
                                              if k in layers.AttentionConfig.__dataclass_fields__})
    our_fa = layers.Qwen3_8FullAttention(ours_full_cfg, 3)
    our_la = layers.Qwen3_8LinearAttention(ours_full_cfg, 0)
    our_fa.load_state_dict(ref_fa.state_dict(), strict=False)
    our_la.load_state_dict(ref_la.state_dict(), strict=False)
    for rank in range(tp):
        rcfg = Qwen3_8Config(**kw, tp_size=tp, tp_rank=rank)
        ocfg = layers.AttentionConfig(**{**{k: v for k, v in kw.items()
                                            if k in layers.AttentionConfig.__dataclass_fields__},
                                         "tp_size": tp, "tp_rank": rank})
        for RefC, OurC, ref_full, our_full in ((RefFull, layers.Qwen3_8FullAttention, ref_fa, our_fa),
                                               (RefLin, layers.Qwen3_8LinearAttention, ref_la, our_la)):
            r = RefC(rcfg, 3)
            r.load_tp_from_full_layer(ref_full)
            o = OurC(ocfg, 3)
            o.load_tp_from_full_layer(our_full)
            rs, os_ = r.state_dict(), o.state_dict()
            for k, v in os_.items():
                assert torch.equal(v, rs[k]), f"tp{tp} rank{rank} {RefC.__name__}.{k}"
