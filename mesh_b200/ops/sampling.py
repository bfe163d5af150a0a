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


class DeviceSampler:
    """Temperature / top-p sampling with the reference's device semantics on vocabulary-parallel
    fp32 logits, entirely on the GPU: the sm_100a kernels of ``csrc/kernels/sampling.cu`` plus, at
    TP > 1, small collectives (a max and a fixed-point mass gather per row, one 256-bin histogram sum
    per radix pass, a final min). Masses are 2^-40 fixed-point integers, so the chosen tokens are
    bitwise the same run to run and at every TP degree. All buffers are allocated once per batch
    size, so the whole call can be captured in a CUDA graph."""

    def __init__(self, max_batch: int, device, group=None, world: int = 1, rank: int = 0):
        self.B = max_batch
        self.group, self.world, self.rank = group, world, rank
        d = torch.device(device)
        self.gmax = torch.empty(max_batch, dtype=torch.float32, device=d)
        self.mass = torch.empty(max_batch, dtype=torch.int64, device=d)
        self.masses = torch.empty(world * max_batch, dtype=torch.int64, device=d)
        self.st = torch.zeros(6 * max_batch, dtype=torch.int64, device=d)
        self.active = torch.zeros(max_batch, dtype=torch.int32, device=d)
        self.hist = torch.empty(max_batch, 256, dtype=torch.int64, device=d)
        self.cand = torch.empty(max_batch, dtype=torch.int32, device=d)

    def sample(self, logits: torch.Tensor, inv_t: torch.Tensor, top_p: torch.Tensor, thr: torch.Tensor,
               greedy_ids: torch.Tensor, vocab_offset: int, out_ids: torch.Tensor, nucleus: bool = True):
        """logits [B, V_loc] fp32 (this rank's vocabulary slice starting at ``vocab_offset``); per-row
        inv_t (1/T, 0 = greedy), top_p and threshold r (``deterministic_sample_threshold`` of the
        row's seed) as fp32 [B]; greedy_ids int32 [B] (used for greedy rows). Writes out_ids int32
        [B]. ``nucleus=False`` skips the radix passes when no row has 0 < top_p < 1."""
        import torch.distributed as dist
        from . import ext, _count
        B = logits.shape[0]
        if B > self.B:
            raise ValueError(f"batch {B} exceeds the sampler's {self.B} rows")
        E = ext()
        gmax, mass, active = self.gmax[:B], self.mass[:B], self.active[:B]
        st = self.st[:6 * B].view(6, B)
        masses = self.masses[:self.world * B].view(self.world, B)
        hist, cand = self.hist[:B], self.cand[:B]
        E.samp_stats(logits, inv_t, gmax, gmax, 0)
        if self.world > 1:
            dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=self.group)
        E.samp_stats(logits, inv_t, gmax, mass, 1)
        if self.world > 1:
            dist.all_gather_into_tensor(masses, mass.contiguous(), group=self.group)
        else:
            masses[0].copy_(mass)
        stc = st
        E.samp_init(0, self.world, self.rank, inv_t, top_p, thr, masses, stc, active)
        n = 4
        if nucleus:
            for stage in (0, 1):
                if stage == 1:
                    E.samp_init(1, self.world, self.rank, inv_t, top_p, thr, masses, stc, active)
                for shift in (24, 16, 8, 0):
                    E.samp_radix(logits, inv_t, gmax, stc, active, hist, shift, 0)
                    if self.world > 1:
                        dist.all_reduce(hist, group=self.group)
                    E.samp_radix(logits, inv_t, gmax, stc, active, hist, shift, 1)
                    n += 2
        E.samp_find(logits, inv_t, gmax, top_p, thr, stc, active, vocab_offset, cand)
        if self.world > 1:
            dist.all_reduce(cand, op=dist.ReduceOp.MIN, group=self.group)
        E.samp_merge(inv_t, top_p, cand, greedy_ids, out_ids)
        _count(n)
        return out_ids
