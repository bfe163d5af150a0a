"""On-device token sampling with the reference's deterministic semantics.

Restates ``agent/src/inference/runtime.rs:461-601`` (device path): greedy argmax when
temperature <= 0 or top_p <= 0; otherwise softmax(logits / T); with top_p >= 1 the first index
whose running CDF reaches the seed's threshold; else a descending sort, keep-mask
``cumsum - p < top_p``, renormalise, CDF over the sorted order, first crossing, mapped back
through the sort order. Thresholds come from the splitmix finaliser of the seed
(``deterministic_sample_threshold``), computed on the host in float64 as the reference does.
"""
from __future__ import annotations

from typing import List, Sequence

import torch

from ..oracle.tensor_ops import deterministic_sample_threshold


def sample(logits: torch.Tensor, temperature: float, top_p: float, seeds: Sequence[int]) -> torch.Tensor:
    """logits [B, V] (any float dtype) -> int64 token ids [B] on the same device."""
    B = logits.shape[0]
    if len(seeds) != B:
        raise ValueError(f"Device sampling received {B} rows but {len(seeds)} seeds")
    if temperature <= 0.0 or top_p <= 0.0:
        return logits.float().argmax(-1)
    x = logits.float()
    if temperature != 1.0:
        x = x * (1.0 / temperature)
    probs = torch.softmax(x, -1)
    thr = torch.tensor([deterministic_sample_threshold(s) for s in seeds], dtype=torch.float32,
                       device=logits.device)[:, None]
    if top_p >= 1.0:
        cdf = probs.cumsum(-1)
        crossing = (cdf >= thr).to(torch.int32)
        return crossing.argmax(-1)
    sp, si = probs.sort(dim=-1, descending=True, stable=True)
    keep = (sp.cumsum(-1) - sp) < top_p
    f = torch.where(keep, sp, torch.zeros_like(sp))
    f = f * (1.0 / f.sum(-1, keepdim=True))
    cdf = f.cumsum(-1)
    idx = (cdf >= thr).to(torch.int32).argmax(-1)
    return si.gather(1, idx[:, None])[:, 0]
