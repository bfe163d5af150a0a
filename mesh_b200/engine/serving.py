"""The serving engine of one TP rank: sessions, paged KV, prefill chunks and CUDA-graph decode.

Mirrors the reference ``zip`` engine's execution model (``agent/src/inference/coordinator.rs``):
a session is prefilled (possibly in several chunks), then joins the decode queue; each decode step
runs one microbatch of sessions; a session completes after ``max_new_tokens``. The scheduler here
is prefill-first continuous batching: waiting prompts are prefilled in token-budgeted chunks, and
running sessions decode together in fixed batch slots.

B200 specifics:
* KV pages live in one HBM pool per rank (16-token pages); block tables are device tensors, the
  attention kernels read pages in place (no per-step K/V materialisation as in the reference's
  ``build_active_tensors``, forward_pass.rs:633-680).
* Decode steps replay a CUDA graph per batch bucket. Token ids never leave the device between
  steps: the graph reads and overwrites the same ids buffer; a history buffer keeps every
  generated token and is copied to the host once per ``sync_every`` steps (or when asked).
* All ranks of a TP group run the same schedule: rank 0 decides and broadcasts, or (as in the
  benchmark) every rank receives the same request list and makes the same decisions.
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from ..config import EngineConfig, ModelConfig
from ..models.llama import LlamaRunner, StepMeta
from .pages import PageAllocator


@dataclass
class Session:
    sid: int
    prompt: List[int]
    max_new_tokens: int
    temperature: float = 0.0
    top_p: float = 1.0
    seed_base: int = 0
    eos_token: Optional[int] = None
    generated: List[int] = field(default_factory=list)
    pages: List[int] = field(default_factory=list)
    kv_len: int = 0            # tokens whose K/V are in the pool
    prefilled: int = 0         # prompt tokens prefilled so far
    slot: int = -1             # decode batch slot
    n_generated: int = 0       # tokens generated (device-side count, known on host)
    decode_steps_served: int = 0
    status: str = "waiting"    # waiting | prefilling | decoding | finished
    t_submit: float = 0.0
    ttft_event: Optional[torch.cuda.Event] = None

    @property
    def done(self) -> bool:
        return self.n_generated >= self.max_new_tokens


def _on_device(fn):
    """Run an Engine method with the engine's GPU as the current device: its CUDA events, capture
    stream and staging-ring fences then belong to that GPU even when the process's current device
    is another one (several engines in one process)."""
    import functools

    @functools.wraps(fn)
    def wrapped(self, *a, **k):
        if self.device.type != "cuda":
            return fn(self, *a, **k)
        with torch.cuda.device(self.device):
            return fn(self, *a, **k)
    return wrapped


@dataclass
class SessionHandoff:
    """A decoding session lifted out of one engine: its request, the tokens so far and its KV pages
    gathered into one device buffer ``kv`` [2, layers, pages, page_elems] (K then V). Moving it to
    another GPU is one peer copy (``to``); ``Engine.import_session`` continues it there."""
    prompt: List[int]
    generated: List[int]
    max_new_tokens: int
    temperature: float
    top_p: float
    seed_base: int
    eos_token: Optional[int]
    kv_len: int
    page_size: int
    kv: torch.Tensor

    def to(self, device) -> "SessionHandoff":
        import dataclasses
        return dataclasses.replace(self, kv=self.kv.to(device, non_blocking=True))


class DecodeGraphs:
    """Static decode buffers shared by all buckets plus one captured graph per bucket."""

    def __init__(self, runner: LlamaRunner, max_batch: int, max_pages_per_seq: int, use_graphs: bool,
                 buckets):
        dev = runner.device
        self.runner = runner
        self.max_batch = max_batch
        self.ids = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.slot = torch.full((max_batch,), -1, dtype=torch.int64, device=dev)
        self.seq_lens = torch.ones(max_batch, dtype=torch.int32, device=dev)
        self.block_tables = torch.zeros(max_batch, max_pages_per_seq, dtype=torch.int32, device=dev)
        # per-slot sampling parameters (1/T with 0 = greedy, top_p, threshold) of sampled steps
        self.samp = torch.zeros(3, max_batch, dtype=torch.float32, device=dev)
        self.max_pages = max_pages_per_seq
        self.use_graphs = use_graphs
        self.buckets = [b for b in buckets if b <= max_batch] or [max_batch]
        if self.buckets[-1] < max_batch:
            self.buckets.append(max_batch)
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: Dict[int, int] = {}
        self.bufs: Dict[int, dict] = {}
        self.outs: Dict[int, torch.Tensor] = {}
        self.pool = None

    def bucket_for(self, n: int) -> int:
        for b in self.buckets:
            if n <= b:
                return b
        raise ValueError(f"decode batch {n} exceeds max batch {self.max_batch}")

    def meta(self, b: int, mode: int = 0) -> StepMeta:
        """mode 0 greedy, 1 sampled (vocabulary-order CDF rows only), 2 sampled with top-p rows."""
        m = StepMeta(ids=self.ids[:b], pos=self.pos[:b], slot=self.slot[:b], block_tables=self.block_tables[:b],
                     seq_lens=self.seq_lens[:b], max_q_len=self.max_pages * self.runner.kv.page_size,
                     decode=True)
        if mode:
            m.inv_t, m.top_p, m.thr, m.nucleus = self.samp[0, :b], self.samp[1, :b], self.samp[2, :b], mode == 2
        return m

    def _run(self, key):
        b, mode = key if isinstance(key, tuple) else (key, 0)
        out = self.runner.forward(self.meta(b, mode), self.bufs.setdefault(key, {}))
        # next ids overwrite the input ids in place (embedding already consumed them)
        self.ids[:b].copy_(out)
        return out

    def capture(self, key):
        if key in self.graphs or not self.use_graphs:
            return
        b = key[0] if isinstance(key, tuple) else key
        # warm-up outside capture sizes the workspaces and sets kernel attributes
        saved = (self.ids.clone(), self.pos.clone(), self.slot.clone(), self.seq_lens.clone())
        self.slot[:b].fill_(-1)
        self._run(key)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        from .. import ops
        n0 = ops.LAUNCHES[0]
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, pool=self.pool):
                self._run(key)
        self.graph_launches[key] = ops.LAUNCHES[0] - n0
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        if self.pool is None:
            self.pool = g.pool()
        self.graphs[key] = g
        self.ids.copy_(saved[0]); self.pos.copy_(saved[1]); self.slot.copy_(saved[2]); self.seq_lens.copy_(saved[3])

    def step(self, b: int, mode: int = 0):
        key = (b, mode) if mode else b
        if self.use_graphs:
            if key not in self.graphs:
                self.capture(key)
            self.graphs[key].replay()
            from .. import ops
            ops._count(self.graph_launches[key])
        else:
            self._run(key)

    def release(self):
        self.graphs.clear()
        self.bufs.clear()
        self.pool = None


class Engine:
    """One rank's engine. All ranks of a TP group must call the same methods in the same order."""

    def __init__(self, runner: LlamaRunner, ecfg: EngineConfig, max_batch: int = 64, sync_every: int = 0,
                 history_steps: int = 4096):
        self.runner = runner
        self.cfg: ModelConfig = runner.cfg
        self.ecfg = ecfg
        self.device = runner.device
        ps = runner.kv.page_size
        self.page_size = ps
        self.alloc = PageAllocator(runner.kv.num_pages, reserved=1)
        self.max_pages_per_seq = (ecfg.max_seq_len + ps - 1) // ps
        self.dec = DecodeGraphs(runner, max_batch, self.max_pages_per_seq, ecfg.use_cuda_graphs,
                                ecfg.decode_batch_buckets)
        self.sessions: Dict[int, Session] = {}
        self.waiting: deque = deque()
        self.running: List[Optional[Session]] = [None] * max_batch
        self.next_sid = 0
        self.max_batch = max_batch
        self.sync_every = sync_every
        # generated-token history: row = decode step, column = batch slot
        self.history = torch.zeros(history_steps, max_batch, dtype=torch.int32, device=self.device)
        self.hist_rows: List[List[Optional[int]]] = []   # per row: slot -> sid mapping
        self.hist_first: List[tuple] = []                # (sid, device tensor idx) of prefill tokens
        self.prefill_tokens_buf = None
        self.bt_host = np.zeros((max_batch, self.max_pages_per_seq), dtype=np.int32)
        self.bt_dirty = True
        # Pinned host staging for the per-step decode metadata (positions, lengths, KV slots), in a
        # small ring so a step never rewrites a buffer whose copy to the device may still be queued
        # (each slot waits on the event recorded after its last copy). Saves three pinned
        # allocations per decode step, which counts when the host must keep ahead of a ~2.7 ms step.
        self._stage = []
        if self.device.type == "cuda":
            for _ in range(4):
                t = torch.empty(max_batch * 4, dtype=torch.int32).pin_memory()  # pos | seq | slot (int64)
                self._stage.append((t, torch.cuda.Event()))
        self._stage_i = 0
        self._fstage = []
        if self.device.type == "cuda":
            for _ in range(4):
                self._fstage.append((torch.empty(max_batch * 3, dtype=torch.float32).pin_memory(), torch.cuda.Event()))
        self._fstage_i = 0
        self.steps = 0
        self.stats = dict(prefill_tokens=0, decode_tokens=0, decode_steps=0, prefill_chunks=0,
                          peak_batch_size=0)
        # reference inference-stats keys this engine feeds (GpuBackend drains them into the
        # coordinator's InferenceStats): layers, collectives and their NVLink bytes, kernel launches
        self.counters: Dict[str, float] = {}
        from .. import ops
        self._launch_mark = ops.LAUNCHES[0]

    def _account(self, tokens: int) -> None:
        """Count one forward over ``tokens`` rows: two tensor-parallel all-reduces per layer, each
        a device-resident collective that moves (world-1) partial [tokens, H] bf16 rows per rank."""
        from .. import ops
        r = self.runner
        L, w = self.cfg.num_layers, r.world
        c = self.counters
        add = lambda k, v: c.__setitem__(k, c.get(k, 0) + v)
        add("total_layers_processed", L)
        add("kernel_launches", ops.LAUNCHES[0] - self._launch_mark)
        self._launch_mark = ops.LAUNCHES[0]
        if w > 1:
            n = 2 * L
            moved = n * tokens * r.H * 2 * (w - 1)
            add("allreduce_operations", n)
            add("total_collective_operations", n)
            add("total_device_resident_collectives", n)
            add("total_collective_worker_participants", n * w)
            add("fused_allreduce_operations" if r.use_fused_ar else "nccl_allreduce_operations", n)
            add("total_collective_bytes_sent", moved)
            add("total_collective_bytes_received", moved)

    def drain_counters(self) -> Dict[str, float]:
        out, self.counters = self.counters, {}
        return out

    # ----------------------------------------------------------------------------- requests
    def submit(self, prompt: List[int], max_new_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
               seed_base: int = 0, eos_token: Optional[int] = None) -> int:
        if not prompt:
            raise ValueError("Cannot prefill an empty prompt without an explicit BOS policy")
        if len(prompt) + max_new_tokens > self.ecfg.max_seq_len:
            raise ValueError(f"prompt {len(prompt)} + {max_new_tokens} new tokens exceeds max_seq_len "
                             f"{self.ecfg.max_seq_len}")
        sid = self.next_sid
        self.next_sid += 1
        s = Session(sid, list(prompt), max_new_tokens, temperature, top_p, seed_base, eos_token,
                    t_submit=time.perf_counter())
        self.sessions[sid] = s
        self.waiting.append(s)
        return sid

    def has_work(self) -> bool:
        return bool(self.waiting) or any(s is not None for s in self.running)

    # ----------------------------------------------------------------------------- pages
    def _ensure_pages(self, s: Session, upto_tokens: int):
        need = (upto_tokens + self.page_size - 1) // self.page_size
        if need > self.max_pages_per_seq:
            raise RuntimeError(f"session {s.sid} exceeds {self.max_pages_per_seq} pages")
        while len(s.pages) < need:
            p = self.alloc.alloc(1)
            if p is None:
                raise RuntimeError("KV page pool exhausted")
            s.pages.append(p[0])
            if s.slot >= 0:
                self.bt_host[s.slot, len(s.pages) - 1] = p[0]
                self.bt_dirty = True

    def _free_session(self, s: Session):
        self.alloc.free(s.pages)
        s.pages = []
        if s.slot >= 0:
            self.running[s.slot] = None
            self.bt_host[s.slot, :] = 0
            self.bt_dirty = True
            s.slot = -1

    # ----------------------------------------------------------------------------- prefill
    def _free_slots(self) -> List[int]:
        return [i for i, s in enumerate(self.running) if s is None]

    @_on_device
    def prefill_step(self, token_budget: Optional[int] = None) -> List[Session]:
        """Prefill a chunk of waiting prompts (whole prompts or the next piece of a long one)."""
        budget = token_budget or self.ecfg.prefill_chunk_tokens
        free = self._free_slots()
        items = []  # (session, start, end)
        used = 0
        while self.waiting and used < budget:
            s = self.waiting[0]
            if s.slot < 0:
                if not free:
                    break
            take = min(len(s.prompt) - s.prefilled, budget - used)
            if take <= 0:
                break
            if s.slot < 0:
                s.slot = free.pop(0)
                self.running[s.slot] = s
                s.status = "prefilling"
            items.append((s, s.prefilled, s.prefilled + take))
            used += take
            if s.prefilled + take == len(s.prompt):
                self.waiting.popleft()
            else:
                break  # a partially prefilled prompt ends the chunk
        if not items:
            return []
        dev = self.device
        ids, pos, slot, cu, klen, last = [], [], [], [0], [], []
        bt = np.zeros((len(items), self.max_pages_per_seq), dtype=np.int32)
        for i, (s, a, b) in enumerate(items):
            self._ensure_pages(s, b)
            ids.extend(s.prompt[a:b])
            pr = np.arange(a, b)
            pos.extend(pr.tolist())
            pages = np.asarray(s.pages, dtype=np.int64)
            slot.extend((pages[pr // self.page_size] * self.page_size + pr % self.page_size).tolist())
            cu.append(cu[-1] + (b - a))
            klen.append(b)
            last.append(cu[-1] - 1)
            bt[i, :len(s.pages)] = s.pages
            self.bt_host[s.slot, :len(s.pages)] = s.pages
        self.bt_dirty = True
        T = len(ids)
        pin = lambda a, dt: torch.tensor(a, dtype=dt).pin_memory().to(dev, non_blocking=True)
        m = StepMeta(ids=pin(ids, torch.int32), pos=pin(pos, torch.int32), slot=pin(slot, torch.int64),
                     block_tables=torch.from_numpy(bt).pin_memory().to(dev, non_blocking=True),
                     seq_lens=pin(klen, torch.int32), cu_q=pin(cu, torch.int32), last_idx=pin(last, torch.int64),
                     max_q_len=max(b - a for _, a, b in items), decode=False, cu_host=cu)
        sampled = [i for i, (s, a, b) in enumerate(items)
                   if s.temperature > 0.0 and s.top_p > 0.0 and b == len(s.prompt)]
        if sampled:
            # the first token of a sampled session is drawn on the device like the decode steps'
            from ..oracle.tensor_ops import deterministic_sample_threshold
            prm = np.zeros((3, len(items)), dtype=np.float32)
            for i in sampled:
                s_ = items[i][0]
                prm[0, i] = 1.0 / s_.temperature
                prm[1, i] = s_.top_p
                prm[2, i] = deterministic_sample_threshold(s_.seed_base ^ len(s_.prompt))
            pd = torch.from_numpy(prm).pin_memory().to(dev, non_blocking=True)
            m.inv_t, m.top_p, m.thr = pd[0], pd[1], pd[2]
            m.nucleus = bool((prm[1][sampled] < 1.0).any())
        next_ids = self.runner.forward(m)
        finished_prompts = []
        rows, slots = [], []
        for i, (s, a, b) in enumerate(items):
            s.prefilled = b
            s.kv_len = b
            if b == len(s.prompt):
                rows.append(i)
                slots.append(s.slot)
                finished_prompts.append(s)
        if rows:
            ri = torch.tensor(rows, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            si = torch.tensor(slots, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            toks = next_ids.index_select(0, ri)
            self.dec.ids.index_copy_(0, si, toks)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            for s in finished_prompts:
                s.status = "decoding"
                s.n_generated = 1
                s.ttft_event = ev
            self.hist_first.append(([s.sid for s in finished_prompts], toks))
        self.stats["prefill_tokens"] += T
        self.stats["prefill_chunks"] += 1
        self._account(T)
        for s in finished_prompts:
            if s.done:
                self._retire(s)
        return finished_prompts

    # ----------------------------------------------------------------------------- decode
    @_on_device
    def decode_step(self, only=None) -> int:
        """One decode step over the sessions in the decode phase (all of them, or the ``only``
        subset chosen by a microbatch planner); returns the batch size."""
        act = [s for s in self.running if s is not None and s.status == "decoding"
               and (only is None or s.sid in only)]
        if not act:
            return 0
        hi = max(s.slot for s in act) + 1
        b = self.dec.bucket_for(hi)
        mode = self._stage_sampling(act, b)
        staged = None
        if self._stage and b <= self._stage[0][0].shape[0] // 4:
            staged, ev = self._stage[self._stage_i]
            self._stage_i = (self._stage_i + 1) % len(self._stage)
            ev.synchronize()
            buf = staged.numpy()
            pos, seq = buf[:b], buf[b:2 * b]
            slot = buf[2 * b:].view(np.int64)[:b]
            pos[:] = 0
            seq[:] = 1
            slot[:] = -1
        else:
            pos = np.zeros(b, dtype=np.int32)
            seq = np.ones(b, dtype=np.int32)
            slot = np.full(b, -1, dtype=np.int64)
        for s in act:
            p = s.kv_len  # position of the token being fed
            self._ensure_pages(s, p + 1)
            pos[s.slot] = p
            seq[s.slot] = p + 1
            slot[s.slot] = s.pages[p // self.page_size] * self.page_size + p % self.page_size
        d = self.dec
        partial = only is not None and any(
            s is not None and s.status == "decoding" and s.slot < b and s not in act for s in self.running)
        if partial:
            keep_ids = d.ids[:b].clone()
            mask = torch.zeros(b, dtype=torch.bool)
            for s in act:
                mask[s.slot] = True
            mask = mask.pin_memory().to(self.device, non_blocking=True)
        if staged is not None:
            d.pos[:b].copy_(staged[:b], non_blocking=True)
            d.seq_lens[:b].copy_(staged[b:2 * b], non_blocking=True)
            d.slot[:b].copy_(staged[2 * b:4 * b].view(torch.int64)[:b], non_blocking=True)
            ev.record()
        else:
            d.pos[:b].copy_(torch.from_numpy(pos).pin_memory(), non_blocking=True)
            d.seq_lens[:b].copy_(torch.from_numpy(seq).pin_memory(), non_blocking=True)
            d.slot[:b].copy_(torch.from_numpy(slot).pin_memory(), non_blocking=True)
        if self.bt_dirty:
            d.block_tables.copy_(torch.from_numpy(self.bt_host).pin_memory(), non_blocking=True)
            self.bt_dirty = False
        d.step(b, mode)
        if partial:
            d.ids[:b].copy_(torch.where(mask, d.ids[:b], keep_ids))
        row = len(self.hist_rows)
        if row >= self.history.shape[0]:
            self.flush_history()
            row = 0
        self.history[row, :b].copy_(d.ids[:b])
        mapping = [None] * b
        for s in act:
            mapping[s.slot] = s.sid
            s.kv_len += 1
            s.n_generated += 1
            s.decode_steps_served += 1
        self.hist_rows.append(mapping)
        self.stats["decode_tokens"] += len(act)
        self.stats["decode_steps"] += 1
        self._account(b)
        self.stats["peak_batch_size"] = max(self.stats["peak_batch_size"], len(act))
        for s in act:
            if s.done:
                self._retire(s)
        return len(act)

    def _stage_sampling(self, act, b: int) -> int:
        """Per-slot sampling parameters of this decode step (1/T, top_p, threshold of the seed for the
        token's position) copied to the device; returns the graph mode (0 greedy, 1 sampled with
        vocabulary-order rows only, 2 with top-p rows)."""
        samp = [s for s in act if s.temperature > 0.0 and s.top_p > 0.0]
        if not samp:
            return 0
        from ..oracle.tensor_ops import deterministic_sample_threshold
        buf, ev = self._fstage[self._fstage_i]
        self._fstage_i = (self._fstage_i + 1) % len(self._fstage)
        ev.synchronize()
        h = buf.numpy()[:3 * b].reshape(3, b)
        h[:] = 0.0
        nucleus = False
        for s in samp:
            h[0, s.slot] = 1.0 / s.temperature
            h[1, s.slot] = s.top_p
            h[2, s.slot] = deterministic_sample_threshold(s.seed_base ^ (s.kv_len + 1))
            nucleus |= s.top_p < 1.0
        self.dec.samp[:, :b].copy_(buf[:3 * b].view(3, b), non_blocking=True)
        ev.record()
        return 2 if nucleus else 1

    # ----------------------------------------------------------------------------- handoff
    @_on_device
    def export_session(self, sid: int) -> SessionHandoff:
        """Take a decoding session out of this engine (reference: moving a session between decode
        queues with its KV, coordinator.rs:1916-1957). The generated tokens are read back first; the
        session's pages are gathered on the device and then returned to this engine's pool."""
        from .. import ops
        s = self.sessions[sid]
        if s.status != "decoding":
            raise ValueError(f"session {sid} is {s.status}; only decoding sessions can be handed off")
        self.flush_history()
        n = (s.kv_len + self.page_size - 1) // self.page_size
        kv = ops.kv_pages_gather(self.runner.kv.k, self.runner.kv.v, s.pages[:n])
        h = SessionHandoff(list(s.prompt), list(s.generated), s.max_new_tokens, s.temperature, s.top_p,
                           s.seed_base, s.eos_token, s.kv_len, self.page_size, kv)
        # the gather is ordered before any later reuse of these pages by this engine's stream
        self._free_session(s)
        s.status = "handed_off"
        del self.sessions[sid]
        return h

    @_on_device
    def import_session(self, h: SessionHandoff) -> int:
        """Continue a session exported by ``export_session`` (from this or another engine with the
        same model shard geometry); returns its id here."""
        from .. import ops
        if h.page_size != self.page_size:
            raise ValueError(f"handoff pages hold {h.page_size} tokens, this pool {self.page_size}")
        L, _, hkv, ps, D = self.runner.kv.k.shape
        n = (h.kv_len + ps - 1) // ps
        if tuple(h.kv.shape) != (2, L, n, hkv * ps * D):
            raise ValueError(f"handoff KV {tuple(h.kv.shape)} does not fit this pool ({L} layers, {hkv} KV heads)")
        free = self._free_slots()
        if not free:
            raise RuntimeError("no free decode slot for the imported session")
        pages = self.alloc.alloc(n) if n else []
        if pages is None:
            raise RuntimeError("KV page pool exhausted during import")
        sid = self.next_sid
        self.next_sid += 1
        s = Session(sid, list(h.prompt), h.max_new_tokens, h.temperature, h.top_p, h.seed_base, h.eos_token,
                    generated=list(h.generated), pages=list(pages), kv_len=h.kv_len, prefilled=len(h.prompt),
                    n_generated=len(h.generated), status="decoding", t_submit=time.perf_counter())
        ops.kv_pages_scatter(self.runner.kv.k, self.runner.kv.v, s.pages, h.kv.to(self.device))
        s.slot = free[0]
        self.running[s.slot] = s
        self.bt_host[s.slot, :] = 0
        self.bt_host[s.slot, :len(s.pages)] = s.pages
        self.bt_dirty = True
        self.dec.ids[s.slot] = int(h.generated[-1])
        self.sessions[sid] = s
        if s.done:
            self._retire(s)
        return sid

    def _retire(self, s: Session):
        s.status = "finished"
        self._free_session(s)

    # ----------------------------------------------------------------------------- outputs
    def check_device(self):
        """Raise if a kernel of this engine recorded an error (a bounded wait that ran out because a
        peer rank never arrived, a pipeline timeout, a bad argument). The error word is cleared, so
        the engine can be reset (``runner.symm.reset()`` on every rank) and used again."""
        from .. import ops
        ops.scratch(self.device).check("engine step")

    @_on_device
    def flush_history(self):
        """Copy generated tokens to the host (one D2H copy) and append them to sessions, after
        checking that no kernel of the steps being read back recorded an error."""
        if self.device.type == "cuda":
            self.check_device()
        for sids, toks in self.hist_first:
            vals = toks.cpu().tolist()
            for sid, t in zip(sids, vals):
                self.sessions[sid].generated.append(int(t))
        self.hist_first = []
        n = len(self.hist_rows)
        if n:
            h = self.history[:n].cpu().numpy()
            for r, mapping in enumerate(self.hist_rows):
                for slot_i, sid in enumerate(mapping):
                    if sid is not None:
                        self.sessions[sid].generated.append(int(h[r, slot_i]))
        self.hist_rows = []

    def step(self) -> None:
        if self.waiting and self._free_slots():
            self.prefill_step()
        else:
            self.decode_step()

    @_on_device
    def run(self):
        while self.has_work():
            self.step()
        self.flush_history()

    @_on_device
    def generate(self, prompts: List[List[int]], max_new_tokens: int) -> List[List[int]]:
        sids = [self.submit(p, max_new_tokens) for p in prompts]
        self.run()
        return [self.sessions[s].generated[:max_new_tokens] for s in sids]

    @_on_device
    def close(self):
        self.dec.release()
