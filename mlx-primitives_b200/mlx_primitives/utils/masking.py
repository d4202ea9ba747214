"""create_causal_mask (mlx_primitives/utils/masking.py:14-66), for callers that want the
additive mask itself; the kernels never materialise it."""

from __future__ import annotations

from typing import Optional

import torch

from ..constants import ATTENTION_MASK_VALUE


def create_causal_mask(seq_q: int, seq_kv: int, dtype: torch.dtype = torch.float32,
                       device: Optional[torch.device] = None) -> torch.Tensor:
    """Additive (seq_q, seq_kv) mask: 0 where query i may attend key j, ATTENTION_MASK_VALUE
    above the diagonal, aligned bottom-right (diagonal offset seq_kv - seq_q + 1) so that the
    last query sees every key."""
    full = torch.full((seq_q, seq_kv), ATTENTION_MASK_VALUE, dtype=dtype, device=device)
    return torch.triu(full, diagonal=seq_kv - seq_q + 1)
