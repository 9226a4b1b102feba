"""Oracle for the per-step runtime around the hot path (TEST INFRASTRUCTURE; numpy).

Restates engine/model_runner.py of yz29528/tokenFactory:
  prepare_forward_batch - model_runner.py:108-188   flattened ids / positions / out_cache_loc, the
                                                     per-request tensors, and the incremental
                                                     req_to_token sync (stale prefix from the host
                                                     table, then the chunk's slots)
  sample_one            - model_runner.py:574-578   greedy argmax (first maximum, NaN wins as in
                                                     torch.argmax); the sampled branch restated as
                                                     an inverse-CDF draw in float64 at a given
                                                     uniform (the reference draws with
                                                     torch.multinomial from softmax(x / T))
"""

from typing import Dict, List, Optional, Sequence

import numpy as np


def prepare_forward_batch(reqs: Sequence[dict], table: Sequence[Sequence[int]],
                          req_to_token: np.ndarray, synced_lens: List[int],
                          dirty_from: Optional[List[int]] = None) -> Dict[str, np.ndarray]:
    out = {k: [] for k in ("input_ids", "positions", "out_cache_loc", "req_pool_indices",
                           "seq_lens", "prefix_lens", "extend_lens")}
    for r in reqs:
        n = len(r["cur_chunk_tokens"])
        assert n > 0 and n == len(r["out_cache_loc"])
        out["req_pool_indices"].append(r["req_pool_idx"])
        out["seq_lens"].append(r["cur_seq_len"])
        out["prefix_lens"].append(r["cur_start_pos"])
        out["extend_lens"].append(n)
        out["input_ids"].extend(r["cur_chunk_tokens"])
        out["positions"].extend(range(r["cur_start_pos"], r["cur_seq_len"]))
        out["out_cache_loc"].extend(r["out_cache_loc"])
    loc = np.asarray(out["out_cache_loc"], np.int64)
    off = 0
    for r in reqs:
        i, n = r["req_pool_idx"], len(r["cur_chunk_tokens"])
        synced = synced_lens[i]
        if dirty_from is not None and dirty_from[i] < synced:
            synced = dirty_from[i]
        if synced < r["cur_start_pos"]:
            req_to_token[i, synced:r["cur_start_pos"]] = table[i][synced:r["cur_start_pos"]]
        req_to_token[i, r["cur_start_pos"]:r["cur_seq_len"]] = loc[off:off + n]
        synced_lens[i] = r["cur_seq_len"]
        if dirty_from is not None:
            dirty_from[i] = r["cur_seq_len"]
        off += n
    res = {k: np.asarray(v, np.int64) for k, v in out.items()}
    res["meta"] = np.asarray([len(reqs), int(any(not r["is_prefilled"] for r in reqs)),
                              max(out["seq_lens"]) if reqs else 0,
                              max(out["extend_lens"]) if reqs else 0], np.int64)
    return res


def argmax_first(x: np.ndarray) -> int:
    """torch.argmax of a row: the first NaN if any, else the first maximum."""
    nan = np.flatnonzero(np.isnan(x))
    if nan.size:
        return int(nan[0])
    return int(np.argmax(x))


def inverse_cdf_bracket(x: np.ndarray, temperature: float, u: float):
    """(cdf just below each index, cdf at each index) of softmax(x / T) in float64, and the
    exact draw for uniform u: the smallest i with cdf_i > u."""
    z = (x.astype(np.float64) - np.max(x.astype(np.float64))) / temperature
    p = np.exp(z)
    c = np.cumsum(p) / p.sum()
    lo = np.concatenate([[0.0], c[:-1]])
    return lo, c, int(np.searchsorted(c, u, side="right"))
