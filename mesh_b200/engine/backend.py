"""Execution backends of the coordinator.

The reference has one provider-polymorphic backend (cpu / metal / cuda through candle,
``agent/src/inference/backend.rs:30-398``). Here there are exactly two, with no dispatch inside
the hot path:

* ``GpuBackend``: sessions on the sm_100a serving engine (paged KV in HBM, CUDA-graph decode);
* ``CpuReferenceBackend``: the fp32 host oracle, which is also the ``cpu`` provider.

Both implement: ``prefill(h, prompt, temperature, top_p, seed_base) -> token``,
``decode([(h, temperature, top_p, seed_base)]) -> [token]``, ``release(h)``, ``kv_bytes(h)``,
``export_kv(h) -> bytes``, ``import_kv(h, payload, prompt, generated)``. Sampling seeds are
``seed_base ^ position`` with position = tokens processed so far (``coordinator.rs:2236``).
"""
from __future__ import annotations

from typing import Dict, List

import cbor2
import numpy as np

from ..oracle.forward import LocalForwardPass, OracleWeights
from ..oracle.tensor_ops import sample_greedy, sample_token

DECODE_TOKEN_BUCKETS = (2048, 8192, 16384, 32768, 65536)  # fast_path.rs:15-17


def token_ceiling(n: int) -> int:
    for b in DECODE_TOKEN_BUCKETS:
        if n <= b:
            return b
    return -1


class CpuReferenceBackend:
    provider = "cpu"
    class_key = 0

    def __init__(self, weights: OracleWeights, window: int = 4096):
        self.w = weights
        self.window = window
        self.sess: Dict[int, LocalForwardPass] = {}
        self.last: Dict[int, int] = {}

    def token_ceiling(self, n: int) -> int:
        return -1  # no fast-path buckets on the host provider

    @staticmethod
    def _sample(logits, temperature, top_p, seed):
        if temperature <= 0.0:
            return sample_greedy(logits)
        return sample_token(logits, temperature, top_p, seed)

    def prefill(self, h, prompt, temperature, top_p, seed_base):
        f = LocalForwardPass(self.w, max_seq_len=self.window)
        logits = f.prefill(prompt)
        self.sess[h] = f
        tok = self._sample(logits, temperature, top_p, seed_base ^ f.position)
        self.last[h] = tok
        return tok

    def decode(self, items):
        out = []
        for h, temperature, top_p, seed_base in items:
            f = self.sess[h]
            logits = f.decode_step(self.last[h])
            tok = self._sample(logits, temperature, top_p, seed_base ^ f.position)
            self.last[h] = tok
            out.append(tok)
        return out

    def release(self, h):
        self.sess.pop(h, None)
        self.last.pop(h, None)

    def kv_bytes(self, h) -> int:
        f = self.sess.get(h)
        if f is None or f.k_cache[0] is None:
            return 0
        return sum(k.nbytes + v.nbytes for k, v in zip(f.k_cache, f.v_cache))

    def export_kv(self, h) -> bytes:
        f = self.sess[h]
        return cbor2.dumps({
            "encoding": "host_f32_v1", "base_position": f.base_position, "position": f.position,
            "last_token": self.last[h],
            "k": [k.astype(np.float32).tobytes() for k in f.k_cache],
            "v": [v.astype(np.float32).tobytes() for v in f.v_cache],
            "rows": int(f.k_cache[0].shape[0]), "width": int(f.k_cache[0].shape[1]),
        })

    def import_kv(self, h, payload: bytes, prompt: List[int], generated: List[int]):
        d = cbor2.loads(payload)
        if d.get("encoding") != "host_f32_v1":
            raise ValueError("CPU backend imports host_f32_v1 snapshots only")
        f = LocalForwardPass(self.w, max_seq_len=self.window)
        shape = (d["rows"], d["width"])
        f.k_cache = [np.frombuffer(b, dtype=np.float32).reshape(shape).copy() for b in d["k"]]
        f.v_cache = [np.frombuffer(b, dtype=np.float32).reshape(shape).copy() for b in d["v"]]
        f.base_position, f.position = d["base_position"], d["position"]
        self.sess[h] = f
        self.last[h] = generated[-1] if generated else d["last_token"]


class GpuBackend:
    """Coordinator sessions on the sm_100a serving engine (one rank, or rank 0 driving a TP group
    whose other ranks replay the same calls)."""
    provider = "cuda"
    class_key = 1

    def __init__(self, engine):
        self.eng = engine
        self.map: Dict[int, int] = {}  # coordinator handle -> engine session id

    def token_ceiling(self, n: int) -> int:
        return token_ceiling(n)

    def prefill(self, h, prompt, temperature, top_p, seed_base):
        e = self.eng
        max_new = e.ecfg.max_seq_len - len(prompt)
        sid = e.submit(prompt, max_new, temperature=temperature, top_p=top_p, seed_base=seed_base)
        self.map[h] = sid
        s = e.sessions[sid]
        while s.status in ("waiting", "prefilling"):
            e.prefill_step()
        e.flush_history()
        return s.generated[-1]

    def decode(self, items):
        e = self.eng
        sids = [self.map[h] for h, *_ in items]
        e.decode_step(only=set(sids))
        e.flush_history()
        out = []
        for sid in sids:
            g = e.sessions[sid].generated
            out.append(g[-1])
        return out

    def drain_counters(self) -> Dict[str, float]:
        """Engine counters since the last call (layers, collectives, bytes, kernel launches)."""
        return self.eng.drain_counters()

    def release(self, h):
        sid = self.map.pop(h, None)
        if sid is not None:
            s = self.eng.sessions.pop(sid, None)
            if s is not None and s.status != "finished":
                self.eng._free_session(s)
                s.status = "finished"

    def kv_bytes(self, h) -> int:
        sid = self.map.get(h)
        if sid is None or sid not in self.eng.sessions:
            return 0
        s = self.eng.sessions[sid]
        r = self.eng.runner
        from ..models.llama import KVPool
        return len(s.pages) * KVPool.bytes_per_page(r.cfg, r.hkv, r.kv.page_size)

    def export_kv(self, h) -> bytes:
        from .kv_snapshot import KVSequenceState, export_snapshot
        s = self.eng.sessions[self.map[h]]
        kv = self.eng.runner.kv
        snap = export_snapshot(kv.k, kv.v, s.pages, KVSequenceState(0, s.kv_len, s.kv_len), self.eng.cfg.name)
        return snap.to_bytes()

    def import_kv(self, h, payload: bytes, prompt: List[int], generated: List[int]):
        import torch
        from .kv_snapshot import KVCacheSnapshot, import_snapshot
        e = self.eng
        snap = KVCacheSnapshot.from_bytes(payload)
        kv = e.runner.kv
        pages = import_snapshot(kv.k, kv.v, e.alloc, snap)
        sid = e.submit(prompt, e.ecfg.max_seq_len - len(prompt))
        s = e.sessions[sid]
        e.waiting.remove(s)
        free = e._free_slots()
        if not free:
            raise RuntimeError("no free decode slot for the hydrated session")
        s.slot = free[0]
        e.running[s.slot] = s
        s.pages = pages
        e.bt_host[s.slot, :] = 0
        e.bt_host[s.slot, :len(pages)] = pages
        e.bt_dirty = True
        s.prefilled = len(prompt)
        s.kv_len = snap.sequence.seq_len
        s.generated = list(generated)
        s.n_generated = len(generated)
        s.status = "decoding"
        e.dec.ids[s.slot] = int(generated[-1])
        self.map[h] = sid
