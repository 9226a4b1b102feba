"""Tensor-parallel head split of the hot path, exactly as the reference shards it.

Full attention (qwen3_8/full_attention.py:43-52, qwen3_8/fp8_linear.py:248-255,320): rank r of t
owns query heads [r*Hq/t, (r+1)*Hq/t); it owns kv heads [r*Hkv/t, (r+1)*Hkv/t) when Hkv >= t,
otherwise the single kv head r // (t/Hkv), replicated on t/Hkv ranks.  The K/V pool of a rank holds
only its kv heads (qwen3_8/hybrid_cache_pool.py:48).

Gated DeltaNet (qwen3_8/linear_attention.py:49-61,109-131; the grouped column split of
in_proj_qkv, qwen3_8/fp8_linear.py:280-318): rank r owns k heads [r*Hk/t, ...) and v heads
[r*Hv/t, ...); its conv channels are the r-th slice of each of the q, k and v channel segments, and
A_log, dt_bias, in_proj_b/a and the gated-norm weight are sliced by v head.

The hot path needs no collective: every rank runs the kernels on its own heads; the row-parallel
out/o projection all-reduce follows outside it.
"""

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    q_heads: range      # full-attention query heads owned by this rank
    kv_heads: range     # full-attention kv heads held by this rank (one replicated head if t > Hkv)
    k_heads: range      # GDN key heads
    v_heads: range      # GDN value heads
    kv_replication: int  # ranks holding the same kv head (1 when kv heads are split)


def head_shard(num_q_heads: int, num_kv_heads: int, num_k_heads: int, num_v_heads: int,
               rank: int, world: int) -> HeadShard:
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    for name, n in (("num_attention_heads", num_q_heads), ("linear_num_key_heads", num_k_heads),
                    ("linear_num_value_heads", num_v_heads)):
        if n % world:
            raise ValueError(f"{name}={n} is not divisible by tp_size={world}")
    lq = num_q_heads // world
    if num_kv_heads >= world:
        if num_kv_heads % world:
            raise ValueError(f"num_key_value_heads={num_kv_heads} not divisible by {world}")
        lkv = num_kv_heads // world
        kv = range(rank * lkv, (rank + 1) * lkv)
    else:
        if world % num_kv_heads:
            raise ValueError(f"tp_size={world} is not a multiple of num_kv_heads={num_kv_heads}")
        h = rank // (world // num_kv_heads)
        kv = range(h, h + 1)
    lk, lv = num_k_heads // world, num_v_heads // world
    return HeadShard(rank, world, range(rank * lq, (rank + 1) * lq), kv,
                     range(rank * lk, (rank + 1) * lk), range(rank * lv, (rank + 1) * lv),
                     max(1, world // num_kv_heads))


def gdn_conv_channels(shard: HeadShard, head_k_dim: int, head_v_dim: int, num_k_heads: int):
    """Global conv / in_proj_qkv channel indices of a rank: its slice of the q, k and v segments."""
    key_dim = num_k_heads * head_k_dim
    q = range(shard.k_heads.start * head_k_dim, shard.k_heads.stop * head_k_dim)
    k = range(key_dim + q.start, key_dim + q.stop)
    v = range(2 * key_dim + shard.v_heads.start * head_v_dim,
              2 * key_dim + shard.v_heads.stop * head_v_dim)
    return list(q) + list(k) + list(v)
