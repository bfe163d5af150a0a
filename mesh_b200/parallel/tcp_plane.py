"""TCP tensor plane and host ring all-reduce, for CPU ranks and cross-host transfers.

On one B200 box tensor traffic stays on NVLink (fused peer-memory kernels, NCCL). This plane
serves what cannot use NVLink: the ``cpu`` provider (the reference's TinyLlama TP=2 loopback
configuration) and bulk / checkpoint lanes between hosts. It is wire compatible with the
reference's serving frames: a 49-byte big-endian header (collective id, seq, sender, layer, step,
slot, stream, element count, lane tag; ``agent/src/network/tensor_message.rs:71-218``) followed by
little-endian f32 elements. The receive side demultiplexes frames into a mailbox keyed by the
slot key (``tensor_plane.rs:1647-1791``); messages above the frame cap (10 MiB by default,
``tensor_plane.rs:26``) are rejected.

Flow control (the behaviour of ``tensor_plane.rs:25-31``, ``:818-870``, ``:1476-1645``,
``:1938-2136``, in a design of this module's own):

* Every lane has a traffic class: ``control`` is latency-critical, ``all_gather`` interactive,
  ``reduce_scatter``, ``bulk_transfer`` and ``checkpoint`` bulk.
* A sender holds bytes of three budgets while a frame is on the wire: the plane's total outbound
  budget, then the class budget (a reserved priority budget for latency-critical and interactive
  frames, so a checkpoint upload can never starve a collective), and for bulk frames also a
  per-peer bulk budget (no single peer can take the whole bulk budget). A send that finds a budget
  full waits (counted as back-pressure) up to the I/O timeout.
* The receiver admits a frame only within its inbound byte and message budgets; the bytes are
  returned when ``recv`` takes the frame out of the mailbox. A reader that finds the budget full
  stops reading its socket for up to the I/O timeout (TCP then pushes back on the sender), and
  drops the frame, counted, if no space appears.
* Each (peer, lane) has a pool of up to ``max_streams_per_peer`` connections; a frame travels on
  stream ``stream % pool size``, so independent streams (e.g. a layer's chunks) do not queue
  behind one another. How many streams a lane gets depends on the profile, provider and runtime
  mode (``lane_stream_count``).
* A send that fails (peer restarted, socket reset or timed out) evicts that lane's pool,
  reconnects once and resends; the metrics count refresh attempts and successes.
* Bulk lanes can be paced to a byte rate (token bucket); ``spawn`` sends a frame from a worker
  thread and returns a future, for background checkpoint and KV uploads.

``WorkerRing.all_reduce`` is the textbook ring: reduce-scatter then all-gather, n-1 steps each,
sending to the right neighbour and receiving from the left concurrently
(``agent/src/executor/ring_allreduce.rs:776-892``, chunk plan ``:1444-1488``).
"""
from __future__ import annotations

import socket
import threading
import time
import uuid
from collections import defaultdict, deque
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import asdict, dataclass, field
from typing import Deque, Dict, List, Optional, Tuple

import numpy as np

from .. import _runtime

HEADER = 49
LANES = {"reduce_scatter": 0, "all_gather": 1, "control": 2, "bulk_transfer": 3, "checkpoint": 4}
LANE_NAMES = {v: k for k, v in LANES.items()}
LATENCY_CRITICAL, INTERACTIVE, BULK = "latency_critical", "interactive", "bulk"
LANE_CLASS = {"control": LATENCY_CRITICAL, "all_gather": INTERACTIVE, "reduce_scatter": BULK,
              "bulk_transfer": BULK, "checkpoint": BULK}
DEFAULT_MAX_MESSAGE_BYTES = 10 * 1024 * 1024
DEFAULT_MAX_INBOUND_MESSAGES = 64
DEFAULT_MAX_INBOUND_QUEUED_BYTES = 64 * 1024 * 1024
DEFAULT_MAX_OUTBOUND_INFLIGHT_BYTES = 64 * 1024 * 1024
DEFAULT_MAX_STREAMS_PER_PEER = 3


class TensorPlaneError(RuntimeError):
    pass


@dataclass
class PlaneConfig:
    """Sizes and policies of one plane. ``profile`` is ``lan`` (a trusted fast network) or
    ``conservative`` (fewer parallel streams); ``provider`` and ``runtime_mode`` select the lane
    stream counts. ``bulk_bytes_per_s`` paces bulk lanes (0: unpaced)."""
    max_message_bytes: int = DEFAULT_MAX_MESSAGE_BYTES
    max_inbound_messages: int = DEFAULT_MAX_INBOUND_MESSAGES
    max_inbound_queued_bytes: int = DEFAULT_MAX_INBOUND_QUEUED_BYTES
    max_outbound_inflight_bytes: int = DEFAULT_MAX_OUTBOUND_INFLIGHT_BYTES
    max_streams_per_peer: int = DEFAULT_MAX_STREAMS_PER_PEER
    profile: str = "lan"
    provider: str = "cpu"
    runtime_mode: str = "throughput_first"
    connect_timeout_s: float = 5.0
    io_timeout_s: float = 30.0
    bulk_bytes_per_s: float = 0.0

    def sanitized(self) -> "PlaneConfig":
        c = PlaneConfig(**asdict(self))
        c.max_message_bytes = max(1024, int(c.max_message_bytes))
        c.max_inbound_messages = max(1, int(c.max_inbound_messages))
        c.max_inbound_queued_bytes = max(c.max_message_bytes + HEADER, int(c.max_inbound_queued_bytes))
        c.max_outbound_inflight_bytes = max(c.max_message_bytes + HEADER, int(c.max_outbound_inflight_bytes))
        c.max_streams_per_peer = max(1, int(c.max_streams_per_peer))
        if c.profile not in ("lan", "conservative"):
            raise ValueError(f"unknown tensor plane profile {c.profile!r}")
        return c

    # budget split -----------------------------------------------------------------------------
    @property
    def priority_budget(self) -> int:
        """Outbound bytes reserved for latency-critical and interactive frames: a quarter of the
        total, at least one full frame, at most the total."""
        frame = self.max_message_bytes + HEADER
        return min(max(self.max_outbound_inflight_bytes // 4, frame), self.max_outbound_inflight_bytes)

    @property
    def bulk_budget(self) -> int:
        return max(self.max_outbound_inflight_bytes - self.priority_budget, self.max_message_bytes + HEADER)

    @property
    def per_peer_bulk_budget(self) -> int:
        """No one peer may hold more than half of the bulk budget (at least one frame)."""
        return max(self.bulk_budget // 2, self.max_message_bytes + HEADER)


def lane_stream_count(lane: str, profile: str, provider: str, runtime_mode: str, max_streams: int) -> int:
    """Parallel connections per peer for ``lane``. Bulk lanes get the most where the link is
    fast and the job is throughput-bound (a GPU provider, throughput-first, on a LAN); latency
    work gets a few so a long frame does not block a short one; the control lane always one; CPU
    ranks and fit-first jobs, whose compute is the bottleneck, one."""
    m = max(1, max_streams)
    if lane == "control" or provider == "cpu" or runtime_mode == "fit_first":
        return 1
    gpu = provider in ("cuda", "metal")
    if runtime_mode == "throughput_first" and gpu:
        bulk = m if profile == "lan" else max(1, m // 2)
    elif runtime_mode == "latency_first" and gpu:
        bulk = min(m, 2)
    else:
        bulk = max(1, m // 2)
    if lane in ("reduce_scatter", "bulk_transfer"):
        return bulk
    if lane == "checkpoint":
        return bulk if runtime_mode == "throughput_first" else 1
    return min(bulk, 2)  # all_gather (interactive)


class ByteBudget:
    """A counting semaphore over bytes. ``acquire`` waits (bounded) until ``n`` bytes are free;
    a request larger than the capacity can never be met and raises at once."""

    def __init__(self, capacity: int, name: str):
        self.capacity = int(capacity)
        self.name = name
        self.used = 0
        self.peak = 0
        self._cv = threading.Condition()

    def try_acquire(self, n: int) -> bool:
        with self._cv:
            if self.used + n > self.capacity:
                return False
            self._take(n)
            return True

    def acquire(self, n: int, timeout_s: float) -> float:
        """Take ``n`` bytes; returns the seconds spent waiting. Raises ``TimeoutError``."""
        if n > self.capacity:
            raise TensorPlaneError(f"{n} bytes can never fit the {self.name} ({self.capacity} bytes)")
        with self._cv:
            if self.used + n <= self.capacity:
                self._take(n)
                return 0.0
            t0 = time.monotonic()
            deadline = t0 + timeout_s
            while self.used + n > self.capacity:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"{self.name} stayed full for {timeout_s:.1f} s")
                self._cv.wait(left)
            self._take(n)
            return time.monotonic() - t0

    def _take(self, n):
        self.used += n
        self.peak = max(self.peak, self.used)

    def release(self, n: int) -> None:
        with self._cv:
            self.used -= n
            self._cv.notify_all()


class TokenBucket:
    """Byte-rate pacing: ``take(n)`` sleeps until ``n`` bytes of credit have accrued at ``rate``
    bytes/s (bursts of up to one second of credit). Returns the seconds slept."""

    def __init__(self, rate: float):
        self.rate = float(rate)
        self.credit = self.rate
        self.t = time.monotonic()
        self._lock = threading.Lock()

    def take(self, n: int) -> float:
        if self.rate <= 0:
            return 0.0
        with self._lock:
            now = time.monotonic()
            self.credit = min(self.rate, self.credit + (now - self.t) * self.rate)
            self.t = now
            self.credit -= n
            wait = -self.credit / self.rate if self.credit < 0 else 0.0
        if wait > 0:
            time.sleep(wait)
        return wait


@dataclass
class PlaneMetrics:
    bytes_sent: int = 0
    bytes_received: int = 0
    send_count: int = 0
    receive_count: int = 0
    send_timeouts: int = 0
    receive_timeouts: int = 0
    oversized_rejections: int = 0
    inbound_byte_budget_rejections: int = 0
    inbound_queue_full_rejections: int = 0
    inbound_backpressure_waits: int = 0
    outbound_backpressure_waits: int = 0
    outbound_backpressure_wait_ms: float = 0.0
    bandwidth_waits: int = 0
    bandwidth_wait_ms: float = 0.0
    receive_queue_wait_ms: float = 0.0
    connection_refresh_attempts: int = 0
    connection_refresh_successes: int = 0
    connection_evictions: int = 0
    current_outbound_connections: int = 0
    per_lane_sent: Dict[int, int] = field(default_factory=lambda: defaultdict(int))
    per_lane_received: Dict[int, int] = field(default_factory=lambda: defaultdict(int))
    per_class_sends: Dict[str, int] = field(default_factory=lambda: defaultdict(int))


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("peer closed")
        buf += chunk
    return bytes(buf)


class _Conn:
    """One outbound connection; its lock keeps frames whole on the wire."""

    def __init__(self, sock: socket.socket):
        self.sock = sock
        self.lock = threading.Lock()

    def close(self):
        try:
            self.sock.close()
        except OSError:
            pass


class TensorPlane:
    """One rank's listener plus pooled outbound connections; frames land in a keyed mailbox.

    ``TensorPlane(host, port, max_message_bytes=…)`` keeps the short form; ``config=PlaneConfig``
    sets every budget and policy."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0, max_message_bytes: Optional[int] = None,
                 config: Optional[PlaneConfig] = None):
        cfg = config or PlaneConfig()
        if max_message_bytes is not None:
            cfg = PlaneConfig(**{**asdict(cfg), "max_message_bytes": max_message_bytes})
        self.config = cfg = cfg.sanitized()
        self.max_message_bytes = cfg.max_message_bytes
        self.metrics = PlaneMetrics()
        self._mlock = threading.Lock()
        # inbound: mailbox of (payload, admitted bytes) per slot key, and its two budgets
        self._mail: Dict[tuple, Deque[Tuple[np.ndarray, int, float]]] = defaultdict(deque)
        self._cv = threading.Condition()
        self._inbound_bytes = ByteBudget(cfg.max_inbound_queued_bytes, "inbound byte budget")
        self._inbound_msgs = ByteBudget(cfg.max_inbound_messages, "inbound message budget")
        # outbound budgets
        self._out_total = ByteBudget(cfg.max_outbound_inflight_bytes, "outbound byte budget")
        self._out_priority = ByteBudget(cfg.priority_budget, "priority outbound byte budget")
        self._out_bulk = ByteBudget(cfg.bulk_budget, "bulk outbound byte budget")
        self._out_peer: Dict[Tuple[str, int], ByteBudget] = {}
        self._pace = TokenBucket(cfg.bulk_bytes_per_s)
        # connection pools per (peer, lane name)
        self._pools: Dict[Tuple[Tuple[str, int], str], List[Optional[_Conn]]] = {}
        self._pool_lock = threading.Lock()
        self._bg: Optional[ThreadPoolExecutor] = None
        self._srv = socket.create_server((host, port))
        self.addr = self._srv.getsockname()
        self._closing = False
        self._readers: List[socket.socket] = []
        threading.Thread(target=self._accept_loop, daemon=True, name="tensor-plane-accept").start()

    # ------------------------------------------------------------------ policy views
    def stream_count(self, lane: str) -> int:
        c = self.config
        return min(c.max_streams_per_peer,
                   lane_stream_count(lane, c.profile, c.provider, c.runtime_mode, c.max_streams_per_peer))

    def capabilities(self) -> dict:
        c = self.config
        return {"profile": c.profile, "max_message_bytes": c.max_message_bytes,
                "inbound_queue_byte_capacity": c.max_inbound_queued_bytes,
                "inbound_queue_message_capacity": c.max_inbound_messages,
                "outbound_inflight_byte_capacity": c.max_outbound_inflight_bytes,
                "reserved_priority_outbound_inflight_bytes": c.priority_budget,
                "bulk_outbound_inflight_byte_capacity": c.bulk_budget,
                "peer_bulk_outbound_byte_capacity": c.per_peer_bulk_budget,
                "bulk_send_bandwidth_bytes_per_sec": c.bulk_bytes_per_s,
                "max_concurrent_outbound_streams_per_peer": c.max_streams_per_peer,
                "lane_streams": {lane: self.stream_count(lane) for lane in LANES},
                "prioritized_traffic_classes": True, "per_peer_bulk_fairness": True,
                "runtime_mode_aware_traffic_policies": True, "concurrent_receive_waiters": True}

    def metrics_snapshot(self) -> dict:
        with self._mlock:
            m = asdict(self.metrics)
        m["per_lane_sent"] = {LANE_NAMES[k]: v for k, v in self.metrics.per_lane_sent.items()}
        m["per_lane_received"] = {LANE_NAMES[k]: v for k, v in self.metrics.per_lane_received.items()}
        m["per_class_sends"] = dict(self.metrics.per_class_sends)
        m.update(current_inbound_queued_bytes=self._inbound_bytes.used, peak_inbound_queued_bytes=self._inbound_bytes.peak,
                 current_outbound_inflight_bytes=self._out_total.used, peak_outbound_inflight_bytes=self._out_total.peak)
        return m

    def _count(self, **kw):
        with self._mlock:
            for k, v in kw.items():
                setattr(self.metrics, k, getattr(self.metrics, k) + v)

    # ------------------------------------------------------------------ inbound
    def _accept_loop(self):
        while not self._closing:
            try:
                conn, _ = self._srv.accept()
            except OSError:
                return
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            self._readers.append(conn)
            threading.Thread(target=self._reader, args=(conn,), daemon=True).start()

    def _admit(self, nbytes: int) -> bool:
        """Reserve inbound budget for one frame; wait up to the I/O timeout (not reading the
        socket meanwhile, which pushes back on the sender), else reject."""
        if self._inbound_msgs.try_acquire(1):
            if self._inbound_bytes.try_acquire(nbytes):
                return True
            self._inbound_msgs.release(1)
        self._count(inbound_backpressure_waits=1)
        t = self.config.io_timeout_s
        try:
            self._inbound_msgs.acquire(1, t)
        except TimeoutError:
            self._count(inbound_queue_full_rejections=1)
            return False
        try:
            self._inbound_bytes.acquire(nbytes, t)
        except (TimeoutError, TensorPlaneError):
            self._inbound_msgs.release(1)
            self._count(inbound_byte_budget_rejections=1)
            return False
        return True

    def _reader(self, conn: socket.socket):
        try:
            while True:
                hdr = _recv_exact(conn, HEADER)
                cid, seq, sender, layer, step, slot, stream, count, lane = _runtime.decode_frame_header(hdr)
                nbytes = count * 4
                if nbytes > self.max_message_bytes:
                    self._count(oversized_rejections=1)
                    raise TensorPlaneError(f"frame of {nbytes} bytes exceeds the {self.max_message_bytes} cap")
                data = np.frombuffer(_recv_exact(conn, nbytes), dtype="<f4").copy()
                size = HEADER + nbytes
                if not self._admit(size):
                    continue
                key = (cid, seq, sender, lane, layer, step, slot, stream)
                with self._cv:
                    self._mail[key].append((data, size, time.monotonic()))
                    self._cv.notify_all()
                with self._mlock:
                    self.metrics.bytes_received += size
                    self.metrics.receive_count += 1
                    self.metrics.per_lane_received[lane] += nbytes
        except (ConnectionError, OSError, TensorPlaneError):
            conn.close()

    def recv(self, *, collective_id: bytes, seq: int, sender: int, layer: int = 0, step: int = 0, slot: int = 0,
             stream: int = 0, lane: str = "reduce_scatter", timeout_s: float = 30.0) -> np.ndarray:
        key = (collective_id, seq, sender, LANES[lane], layer, step, slot, stream)
        deadline = time.monotonic() + timeout_s
        with self._cv:
            while not self._mail.get(key):
                left = deadline - time.monotonic()
                if left <= 0:
                    self._count(receive_timeouts=1)
                    raise TimeoutError(f"tensor plane receive timed out for slot {key[1:]}")
                self._cv.wait(left)
            q = self._mail[key]
            data, size, t_in = q.popleft()
            if not q:
                del self._mail[key]
        self._inbound_bytes.release(size)
        self._inbound_msgs.release(1)
        self._count(receive_queue_wait_ms=(time.monotonic() - t_in) * 1e3)
        return data

    def recv_bytes(self, **kw) -> bytes:
        """A frame sent with ``send_bytes``: its payload with the padding removed (the first
        element holds the unpadded length)."""
        arr = self.recv(**kw)
        n = int(arr[:1].view("<u4")[0])
        return arr[1:].tobytes()[:n]

    # ------------------------------------------------------------------ outbound
    def _connect(self, addr: Tuple[str, int]) -> _Conn:
        try:
            s = socket.create_connection(addr, timeout=self.config.connect_timeout_s)
        except OSError as e:
            raise TensorPlaneError(f"cannot connect to tensor plane peer {addr}: {e}") from e
        s.settimeout(self.config.io_timeout_s)
        s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self._count(current_outbound_connections=1)
        return _Conn(s)

    def _stream(self, addr: Tuple[str, int], lane: str, stream: int) -> _Conn:
        n = self.stream_count(lane)
        idx = 0 if n == 1 else stream % n
        key = (addr, lane)
        with self._pool_lock:
            pool = self._pools.setdefault(key, [None] * n)
            c = pool[idx]
        if c is not None:
            return c
        c = self._connect(addr)
        with self._pool_lock:
            pool = self._pools.setdefault(key, [None] * n)
            if pool[idx] is None:
                pool[idx] = c
                return c
        c.close()  # another thread connected this stream first
        self._count(current_outbound_connections=-1)
        return pool[idx]

    def _evict(self, addr: Tuple[str, int], lane: str) -> None:
        with self._pool_lock:
            pool = self._pools.pop((addr, lane), None)
        if pool:
            live = [c for c in pool if c is not None]
            for c in live:
                c.close()
            self._count(connection_evictions=1, current_outbound_connections=-len(live))

    def reset_peer(self, addr: Tuple[str, int]) -> None:
        """Drop every pooled connection to ``addr`` (all lanes); the next send reconnects."""
        for lane in LANES:
            self._evict(tuple(addr), lane)

    def _budgets(self, addr, cls: str) -> List[ByteBudget]:
        if cls == BULK:
            with self._pool_lock:
                peer = self._out_peer.get(addr)
                if peer is None:
                    peer = self._out_peer[addr] = ByteBudget(self.config.per_peer_bulk_budget,
                                                             f"per-peer bulk outbound byte budget ({addr})")
            return [self._out_total, self._out_bulk, peer]
        return [self._out_total, self._out_priority]

    def _write(self, addr, lane: str, stream: int, frame: bytes) -> None:
        try:
            c = self._stream(addr, lane, stream)
            with c.lock:
                c.sock.sendall(frame)
            return
        except (OSError, TensorPlaneError):
            pass
        # one refresh: drop the lane's pool, reconnect, resend
        self._count(connection_refresh_attempts=1)
        self._evict(addr, lane)
        try:
            c = self._stream(addr, lane, stream)
            with c.lock:
                c.sock.sendall(frame)
        except socket.timeout as e:
            self._count(send_timeouts=1)
            raise TensorPlaneError(f"timed out sending a {lane} frame to {addr}") from e
        except OSError as e:
            raise TensorPlaneError(f"cannot send a {lane} frame to {addr}: {e}") from e
        self._count(connection_refresh_successes=1)

    def send(self, addr: Tuple[str, int], data: np.ndarray, *, collective_id: bytes, seq: int, sender: int,
             layer: int = 0, step: int = 0, slot: int = 0, stream: int = 0, lane: str = "reduce_scatter") -> None:
        arr = np.ascontiguousarray(data, dtype="<f4")
        if arr.nbytes > self.max_message_bytes:
            self._count(oversized_rejections=1)
            raise TensorPlaneError(f"message of {arr.nbytes} bytes exceeds the {self.max_message_bytes} cap")
        addr = tuple(addr)
        cls = LANE_CLASS[lane]
        hdr = _runtime.encode_frame_header(collective_id, seq, sender, layer, step, slot, stream, arr.size,
                                           LANES[lane])
        size = HEADER + arr.nbytes
        held: List[ByteBudget] = []
        waited = 0.0
        try:
            for b in self._budgets(addr, cls):
                try:
                    waited += b.acquire(size, self.config.io_timeout_s)
                except TimeoutError as e:
                    self._count(send_timeouts=1)
                    raise TensorPlaneError(str(e)) from e
                held.append(b)
            if waited > 0:
                self._count(outbound_backpressure_waits=1, outbound_backpressure_wait_ms=waited * 1e3)
            if cls == BULK:
                slept = self._pace.take(size)
                if slept > 0:
                    self._count(bandwidth_waits=1, bandwidth_wait_ms=slept * 1e3)
            self._write(addr, lane, stream, hdr + arr.tobytes())
        finally:
            for b in held:
                b.release(size)
        with self._mlock:
            self.metrics.bytes_sent += size
            self.metrics.send_count += 1
            self.metrics.per_lane_sent[LANES[lane]] += arr.nbytes
            self.metrics.per_class_sends[cls] += 1

    def send_bytes(self, addr, payload: bytes, **kw) -> None:
        """Raw bytes (a checkpoint or a CBOR blob) as one frame: a little-endian u32 length, the
        bytes, zero padding to a whole number of 4-byte elements (the reference's framing of raw
        payloads, ``tensor_plane.rs:2264-2274``)."""
        n = len(payload)
        framed = n.to_bytes(4, "little") + bytes(payload) + b"\0" * ((-(4 + n)) % 4)
        self.send(addr, np.frombuffer(framed, dtype="<f4"), **kw)

    def spawn(self, addr, data, **kw) -> Future:
        """Send from a background thread (bulk and checkpoint uploads); the future holds the
        outcome. Budgets and pacing apply as for ``send``."""
        if self._bg is None:
            with self._pool_lock:
                if self._bg is None:
                    self._bg = ThreadPoolExecutor(max_workers=4, thread_name_prefix="tensor-plane-bg")
        fn = self.send_bytes if isinstance(data, (bytes, bytearray, memoryview)) else self.send
        return self._bg.submit(fn, addr, data, **kw)

    def close(self):
        self._closing = True
        try:  # shutdown wakes the thread blocked in accept(); close alone leaves the port listening
            self._srv.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        try:
            self._srv.close()
        except OSError:
            pass
        if self._bg is not None:
            self._bg.shutdown(wait=False, cancel_futures=True)
        with self._pool_lock:
            pools, self._pools = self._pools, {}
        for pool in pools.values():
            for c in pool:
                if c is not None:
                    c.close()
        for r in self._readers:
            try:
                r.close()
            except OSError:
                pass


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
