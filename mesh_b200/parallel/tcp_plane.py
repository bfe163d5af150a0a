"""TCP tensor plane and host ring all-reduce, for CPU ranks and cross-host transfers.

On one B200 box tensor traffic stays on NVLink (fused peer-memory kernels, NCCL). This plane
serves what cannot use NVLink: the ``cpu`` provider (the reference's TinyLlama TP=2 loopback
configuration) and bulk / checkpoint lanes between hosts. It is wire compatible with the
reference's serving frames: a 49-byte big-endian header (collective id, seq, sender, layer, step,
slot, stream, element count, lane tag; ``agent/src/network/tensor_message.rs:71-218``) followed by
little-endian f32 elements. The receive side demultiplexes frames into a mailbox keyed by the
slot key (``tensor_plane.rs:1647-1791``); messages above the frame cap (10 MiB by default,
``tensor_plane.rs:26``) are rejected.

``WorkerRing.all_reduce`` is the textbook ring: reduce-scatter then all-gather, n-1 steps each,
sending to the right neighbour and receiving from the left concurrently
(``agent/src/executor/ring_allreduce.rs:776-892``, chunk plan ``:1444-1488``).
"""
from __future__ import annotations

import socket
import struct
import threading
import time
import uuid
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

from .. import _runtime

HEADER = 49
LANES = {"reduce_scatter": 0, "all_gather": 1, "control": 2, "bulk_transfer": 3, "checkpoint": 4}
DEFAULT_MAX_MESSAGE_BYTES = 10 * 1024 * 1024


class TensorPlaneError(RuntimeError):
    pass


@dataclass
class PlaneMetrics:
    bytes_sent: int = 0
    bytes_received: int = 0
    send_count: int = 0
    receive_count: int = 0
    receive_timeouts: int = 0
    oversized_rejections: int = 0
    per_lane_sent: Dict[int, int] = field(default_factory=lambda: defaultdict(int))


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("peer closed")
        buf += chunk
    return bytes(buf)


class TensorPlane:
    """One rank's listener plus outbound connections; frames land in a keyed mailbox."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0, max_message_bytes: int = DEFAULT_MAX_MESSAGE_BYTES):
        self.max_message_bytes = max_message_bytes
        self.metrics = PlaneMetrics()
        self._mail: Dict[tuple, List[np.ndarray]] = defaultdict(list)
        self._cv = threading.Condition()
        self._out: Dict[Tuple[str, int], socket.socket] = {}
        self._out_lock = threading.Lock()
        self._srv = socket.create_server((host, port))
        self.addr = self._srv.getsockname()
        self._closing = False
        threading.Thread(target=self._accept_loop, daemon=True, name="tensor-plane-accept").start()

    def _accept_loop(self):
        while not self._closing:
            try:
                conn, _ = self._srv.accept()
            except OSError:
                return
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            threading.Thread(target=self._reader, args=(conn,), daemon=True).start()

    def _reader(self, conn: socket.socket):
        try:
            while True:
                hdr = _recv_exact(conn, HEADER)
                cid, seq, sender, layer, step, slot, stream, count, lane = _runtime.decode_frame_header(hdr)
                nbytes = count * 4
                if nbytes > self.max_message_bytes:
                    self.metrics.oversized_rejections += 1
                    raise TensorPlaneError(f"frame of {nbytes} bytes exceeds the {self.max_message_bytes} cap")
                data = np.frombuffer(_recv_exact(conn, nbytes), dtype="<f4").copy()
                key = (cid, seq, sender, lane, layer, step, slot, stream)
                with self._cv:
                    self._mail[key].append(data)
                    self.metrics.bytes_received += HEADER + nbytes
                    self.metrics.receive_count += 1
                    self._cv.notify_all()
        except (ConnectionError, OSError, TensorPlaneError):
            conn.close()

    def _conn(self, addr: Tuple[str, int]) -> socket.socket:
        with self._out_lock:
            s = self._out.get(addr)
            if s is None:
                s = socket.create_connection(addr, timeout=30)
                s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
                self._out[addr] = s
            return s

    def send(self, addr: Tuple[str, int], data: np.ndarray, *, collective_id: bytes, seq: int, sender: int,
             layer: int = 0, step: int = 0, slot: int = 0, stream: int = 0, lane: str = "reduce_scatter") -> None:
        arr = np.ascontiguousarray(data, dtype="<f4")
        if arr.nbytes > self.max_message_bytes:
            self.metrics.oversized_rejections += 1
            raise TensorPlaneError(f"message of {arr.nbytes} bytes exceeds the {self.max_message_bytes} cap")
        hdr = _runtime.encode_frame_header(collective_id, seq, sender, layer, step, slot, stream, arr.size,
                                           LANES[lane])
        s = self._conn(tuple(addr))
        s.sendall(hdr + arr.tobytes())
        self.metrics.bytes_sent += HEADER + arr.nbytes
        self.metrics.send_count += 1
        self.metrics.per_lane_sent[LANES[lane]] += arr.nbytes

    def recv(self, *, collective_id: bytes, seq: int, sender: int, layer: int = 0, step: int = 0, slot: int = 0,
             stream: int = 0, lane: str = "reduce_scatter", timeout_s: float = 30.0) -> np.ndarray:
        key = (collective_id, seq, sender, LANES[lane], layer, step, slot, stream)
        deadline = time.monotonic() + timeout_s
        with self._cv:
            while not self._mail.get(key):
                left = deadline - time.monotonic()
                if left <= 0:
                    self.metrics.receive_timeouts += 1
                    raise TimeoutError(f"tensor plane receive timed out for slot {key[1:]}")
                self._cv.wait(left)
            q = self._mail[key]
            data = q.pop(0)
            if not q:
                del self._mail[key]
            return data

    def close(self):
        self._closing = True
        try:
            self._srv.close()
        except OSError:
            pass
        with self._out_lock:
            for s in self._out.values():
                try:
                    s.close()
                except OSError:
                    pass
            self._out.clear()


class WorkerRing:
    """Ring all-reduce among ``n`` positions over tensor planes (each rank owns one plane)."""

    def __init__(self, plane: TensorPlane, position: int, addrs: List[Tuple[str, int]], timeout_s: float = 30.0,
                 collective_id: Optional[bytes] = None):
        self.plane = plane
        self.position = position
        self.addrs = addrs
        self.n = len(addrs)
        self.timeout_s = timeout_s
        self.cid = collective_id or uuid.UUID(int=0).bytes
        self.seq = 0
        self.operations = 0
        self.time_ms = 0.0

    @property
    def right(self):
        return self.addrs[(self.position + 1) % self.n]

    def all_reduce(self, x: np.ndarray, layer: int = 0) -> np.ndarray:
        """Sum of ``x`` over all positions (fp32), returned on every position."""
        t0 = time.perf_counter()
        self.seq += 1
        n, p = self.n, self.position
        flat = np.ascontiguousarray(x, dtype=np.float32).reshape(-1).copy()
        if n == 1:
            return flat.reshape(x.shape)
        ranges = _runtime.chunk_ranges(flat.size, n)
        left = (p - 1) % n
        for s in range(n - 1):
            send_i, recv_i = _runtime.ring_chunk_plan(p, n, s, False)
            a, b = ranges[send_i]
            self.plane.send(self.right, flat[a:b], collective_id=self.cid, seq=self.seq, sender=p, layer=layer,
                            step=s, slot=send_i, lane="reduce_scatter")
            got = self.plane.recv(collective_id=self.cid, seq=self.seq, sender=left, layer=layer, step=s, slot=recv_i,
                                  lane="reduce_scatter", timeout_s=self.timeout_s)
            a, b = ranges[recv_i]
            flat[a:b] += got
        for s in range(n - 1):
            send_i, recv_i = _runtime.ring_chunk_plan(p, n, s, True)
            a, b = ranges[send_i]
            self.plane.send(self.right, flat[a:b], collective_id=self.cid, seq=self.seq, sender=p, layer=layer,
                            step=s, slot=send_i, lane="all_gather")
            got = self.plane.recv(collective_id=self.cid, seq=self.seq, sender=left, layer=layer, step=s, slot=recv_i,
                                  lane="all_gather", timeout_s=self.timeout_s)
            a, b = ranges[recv_i]
            flat[a:b] = got
        self.operations += 1
        self.time_ms += (time.perf_counter() - t0) * 1e3
        return flat.reshape(x.shape)

    def barrier(self) -> None:
        """Token passed once around the ring (reference ``ring_allreduce.rs:1146-1177``)."""
        self.all_reduce(np.zeros(self.n, dtype=np.float32), layer=0xFFFF)
