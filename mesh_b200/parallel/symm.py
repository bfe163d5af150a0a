"""Symmetric NVLink workspace for the fused tensor-parallel collectives.

One allocation per rank, mapped into every peer of the TP group (CUDA VMM/IPC through
``torch.distributed._symmetric_memory``). Layout (byte offsets, identical on every rank):

    [flags: 2 phases x 256 blocks x 8 ranks x u32] [fused-GEMM flags: 2 phases x 8 source ranks x
    256 source CTAs x u32] [partial slot 0: T_max x H bf16] [partial slot 1]
    [resid: T_max x H bf16] [normed: T_max x H bf16] [push slots, parity 0 and 1: world x T_max x H]

The o_proj / down_proj GEMMs write their partial sums into a partial slot; the ``ar_fused_norm``
kernel reads the peers' slots over NVLink, adds the residual, applies RMSNorm and writes
``resid`` / ``normed`` (locally for one-shot, into every peer for two-shot). For decode-sized steps
``gemm_allreduce_norm`` does all of it in the GEMM's own launch: the epilogue pushes each partial
token row into the push slot of the rank that owns the row, and the same kernel then reduces the
owned rows, adds the residual, applies RMSNorm and writes the normed rows into every rank. Peer
memory is touched by plain P2P loads and stores, or, when the allocation is bound to an NVLink multicast object
(NVSwitch NVLS), by ``multimem`` loads that return the sum over all ranks and ``multimem`` stores
that write every rank at once. No TMA (and no multicast TMA) ever reads a peer address.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


@dataclass
class SymmLayout:
    t_max: int
    hidden: int
    world: int
    off_flags: int
    off_gflags: int
    off_gcount: int
    off_p0: int
    off_p1: int
    off_resid: int
    off_normed: int
    off_push0: int
    off_push1: int
    total: int

    @classmethod
    def make(cls, t_max: int, hidden: int, flags_bytes: int, world: int = 1) -> "SymmLayout":
        row = t_max * hidden * 2
        o = 0
        off_flags = o; o = _align(o + flags_bytes)
        off_gflags = o; o = _align(o + 2 * 8 * 256 * 4)
        off_gcount = o
        off_p0 = o; o = _align(o + row)
        off_p1 = o; o = _align(o + row)
        off_resid = o; o = _align(o + row)
        off_normed = o; o = _align(o + row)
        # fused reduce-scatter targets: per parity, one [t_max, H] slot per source rank
        off_push0 = o; o = _align(o + world * row)
        off_push1 = o; o = _align(o + world * row)
        return cls(t_max, hidden, world, off_flags, off_gflags, off_gcount, off_p0, off_p1, off_resid, off_normed,
                   off_push0, off_push1, o)


class SymmWorkspace:
    """Owns the symmetric buffer of this rank plus the peer address table."""

    def __init__(self, t_max: int, hidden: int, device: torch.device, group=None,
                 multicast: Optional[bool] = None):
        import torch.distributed._symmetric_memory as symm_mem
        self.device = device
        self.group = group or dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.layout = SymmLayout.make(t_max, hidden, ops.ext().ar_flags_bytes(), self.world)
        self.buf = symm_mem.empty(self.layout.total, dtype=torch.uint8, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        gname = self.group.group_name
        self.handle = symm_mem.rendezvous(self.buf, gname)
        ptrs: List[int] = list(self.handle.buffer_ptrs)
        if len(ptrs) != self.world:
            raise RuntimeError(f"symmetric rendezvous returned {len(ptrs)} peers for world {self.world}")
        # peer tables are allocation bases; the workspace must start there for the offsets to hold
        delta = self.buf.data_ptr() - ptrs[self.rank]
        if delta != 0:
            raise RuntimeError(f"symmetric workspace is at offset {delta} inside its allocation")
        self.bases = torch.tensor(ptrs, dtype=torch.int64)
        self._bases = [int(b) for b in ptrs]
        # NVLS multicast address of the same allocation (0: plain peer loads). MESH_NVLS=0 turns it off.
        if multicast is None:
            multicast = os.environ.get("MESH_NVLS", "1") != "0"
        mc = 0
        if multicast and self.world > 1:
            try:
                mc = int(self.handle.multicast_ptr)
            except Exception:
                mc = 0
        # every rank must agree, or some would multicast into an allocation others read unicast
        flag = torch.tensor([1 if mc else 0], dtype=torch.int32, device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        self.mc_base = mc if int(flag.item()) == 1 else 0
        self.epoch = torch.zeros(256, dtype=torch.int32, device=device)
        self.gepoch = torch.zeros(1, dtype=torch.int32, device=device)  # fused GEMM + all-reduce launches
        self._no_trace = torch.empty(0, dtype=torch.int64, device=device)
        dist.barrier(self.group)

    def view(self, off: int, rows: int) -> torch.Tensor:
        L = self.layout
        n = rows * L.hidden
        return self.buf[off: off + n * 2].view(torch.bfloat16).view(rows, L.hidden)

    def partial(self, parity: int, rows: int) -> torch.Tensor:
        return self.view(self.layout.off_p0 if parity % 2 == 0 else self.layout.off_p1, rows)

    def resid(self, rows: int) -> torch.Tensor:
        return self.view(self.layout.off_resid, rows)

    def normed(self, rows: int) -> torch.Tensor:
        return self.view(self.layout.off_normed, rows)

    def fused_allreduce_norm(self, T: int, parity: int, gamma: torch.Tensor, eps: float, two_shot: bool,
                             nblocks: int = 0, timeout_s: float = 5.0, multicast: bool = True,
                             trace: Optional[torch.Tensor] = None):
        """``multicast`` uses NVLS loads/stores when the workspace has them; ``trace`` (CUDA int64,
        >= 4) receives block 0's %globaltimer at start, after the entry barrier, after the rows and
        at the end."""
        L = self.layout
        if T > L.t_max:
            raise ValueError(f"T={T} exceeds symmetric workspace capacity {L.t_max}")
        if nblocks <= 0:
            rows = (T + self.world - 1) // self.world if two_shot else T
            nblocks = max(1, min((rows + 7) // 8, 255))  # 8 warps per block, one row per warp
        s = ops.scratch(self.device)
        ops.ext().ar_fused_norm(self.bases, L.off_flags, L.off_p0, L.off_p1, L.off_resid, L.off_normed,
                                self.rank, self.world, T, L.hidden, parity, gamma, eps, self.epoch, s.err,
                                nblocks, two_shot, timeout_s, self.mc_base if multicast else 0,
                                self._no_trace if trace is None else trace)
        ops._count()

    def push_args(self, T: int, parity: int, two_shot: bool) -> list:
        """GEMM epilogue push table: [mode, my_rank, world, rows, slot_stride, ldo, peer bases...]."""
        L = self.layout
        off = L.off_push0 if parity % 2 == 0 else L.off_push1
        return [1 if two_shot else 2, self.rank, self.world, T, L.t_max * L.hidden, L.hidden] + \
            [int(b) + off for b in self.bases.tolist()]

    def push_reduce_norm(self, T: int, parity: int, gamma: torch.Tensor, eps: float, two_shot: bool,
                         nblocks: int = 0, timeout_s: float = 5.0):
        L = self.layout
        if T > L.t_max:
            raise ValueError(f"T={T} exceeds symmetric workspace capacity {L.t_max}")
        if nblocks <= 0:
            rows = (T + self.world - 1) // self.world if two_shot else T
            nblocks = max(1, min((rows + 7) // 8, 255))
        s = ops.scratch(self.device)
        off = L.off_push0 if parity % 2 == 0 else L.off_push1
        ops.ext().ar_push_reduce_norm(self.bases, L.off_flags, off, L.off_resid, L.off_normed, self.rank,
                                      self.world, T, L.t_max, L.hidden, gamma, eps, self.epoch, s.err, nblocks,
                                      two_shot, timeout_s)
        ops._count()

    def gemm_allreduce_norm(self, x: torch.Tensor, w: torch.Tensor, parity: int, gamma: torch.Tensor, eps: float,
                            timeout_s: float = 5.0, mode: int = 0, multicast: bool = True,
                            trace: Optional[torch.Tensor] = None):
        """One launch: partial = x @ w.T on this rank, summed over the TP group, added to ``resid``
        and RMS-normalised into ``normed`` on every rank. Decode-sized T (swap-AB GEMM). Each rank
        keeps only the ``resid`` rows it owns current (the same rows in every call with this T);
        ``multicast`` writes the normed rows with NVLS stores when the workspace has them."""
        L = self.layout
        T = x.shape[0]
        if T > L.t_max:
            raise ValueError(f"T={T} exceeds symmetric workspace capacity {L.t_max}")
        off = L.off_push0 if parity % 2 == 0 else L.off_push1
        push = [1, self.rank, self.world, T, L.t_max * L.hidden, L.hidden] + [int(b) + off for b in self._bases]
        cfg = [L.t_max, L.off_gflags, L.off_gcount, off, L.off_resid, L.off_normed,
               self.mc_base if multicast else 0, int(timeout_s * 1e9)] + self._bases
        local = self.view(off + self.rank * L.t_max * L.hidden * 2, T)
        ops.gemm_allreduce_norm(w, x, local, push, cfg, gamma, eps, self.gepoch, mode, trace)

    def reset(self):
        """Collective: zero the flags and epoch counters on every rank. Needed after a timed-out
        collective left the ranks' epochs out of step."""
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        self.buf[: self.layout.off_p0].zero_()
        self.epoch.zero_()
        self.gepoch.zero_()
        ops.scratch(self.device).err.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    def barrier(self, timeout_s: float = 5.0):
        s = ops.scratch(self.device)
        ops.ext().ar_barrier(self.bases, self.layout.off_flags, self.rank, self.world, self.epoch, s.err,
                             timeout_s, self.epoch)


class SymmTable:
    """A read-only table sharded by rows over the TP group and mapped into every peer: rank r holds
    rows [start_r, start_r + n_r) (near-equal contiguous ranges, larger first) of a [rows, cols]
    bf16 table; ``bases`` lists every rank's allocation as mapped here, so a kernel can read any row
    from its owner over NVLink. Used for the vocabulary-parallel embedding (each rank keeps 1/TP of
    the table instead of all of it)."""

    def __init__(self, local: torch.Tensor, total_rows: int, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        rows_max = -(-total_rows // self.world)
        cols = local.shape[1]
        # every rank allocates the same size (the largest shard)
        self.buf = symm_mem.empty(rows_max * cols, dtype=torch.bfloat16, device=local.device)
        self.buf[: local.numel()].copy_(local.reshape(-1))
        torch.cuda.synchronize(local.device)
        self.handle = symm_mem.rendezvous(self.buf, self.group.group_name)
        ptrs = list(self.handle.buffer_ptrs)
        if ptrs[self.rank] != self.buf.data_ptr():
            raise RuntimeError("symmetric table is not at the start of its allocation")
        self.bases = torch.tensor(ptrs, dtype=torch.int64)
        self.local = self.buf[: local.numel()].view(local.shape)
        dist.barrier(self.group)

