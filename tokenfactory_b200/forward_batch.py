"""ForwardBatch: the hot path's batch metadata, with the reference's fields and defaults
(qwen3_8/forward_batch.py:7-45).  The kernels accept any object with these attributes, so the
reference's own ForwardBatch works unchanged."""

from dataclasses import dataclass
from typing import List, Optional

import torch


@dataclass
class ForwardBatch:
    batch_size: int
    req_pool_indices: torch.Tensor  # [B] int64, rows of req_to_token / req_to_state_pool
    seq_lens: torch.Tensor          # [B] int64, lengths after this step
    prefix_lens: torch.Tensor       # [B] int64, cached prefix lengths
    extend_lens: List[int]          # new tokens per request (all 1 in decode)
    out_cache_loc: torch.Tensor     # [T] int64, KV slots of this step's tokens
    req_to_token: torch.Tensor      # [max_reqs, max_context_len] int64, -1 = empty
    is_prefill: bool = True
    max_seq_len: int = 0
    max_extend_len: int = 0
    extend_lens_tensor: Optional[torch.Tensor] = None
    req_pool_indices_list: Optional[List[int]] = None

    def __post_init__(self) -> None:
        # same host-side completion as the reference (qwen3_8/forward_batch.py:33-45)
        if self.max_extend_len == 0 and self.extend_lens:
            self.max_extend_len = max(self.extend_lens)
        if self.extend_lens_tensor is None and self.extend_lens:
            self.extend_lens_tensor = torch.tensor(self.extend_lens, dtype=torch.long,
                                                   device=self.out_cache_loc.device)
        if self.max_seq_len == 0 and self.seq_lens.numel() > 0:
            self.max_seq_len = int(self.seq_lens.max().item())
        if self.req_pool_indices_list is None and self.req_pool_indices.numel() > 0:
            self.req_pool_indices_list = [int(x) for x in self.req_pool_indices.tolist()]
