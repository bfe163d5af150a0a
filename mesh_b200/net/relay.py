"""Optional TCP relay for nodes without a direct path to each other.

The reference runs a libp2p circuit relay (``relay-server/src/relay.rs:14-127``) so that nodes
behind NAT can reach each other. Here the same role is a small TCP forwarder: a client connects,
registers its node id (32 bytes), and then sends frames ``[dst node id (32)][len u32 LE][payload]``;
the relay forwards each frame to the destination as ``[src node id (32)][len u32 LE][payload]``.
Frames to unknown destinations are dropped and counted. Payloads above ``max_frame`` close the
sender's connection.
"""
from __future__ import annotations

import socket
import struct
import threading
from typing import Dict, Optional, Tuple

ID_LEN = 32
DEFAULT_MAX_FRAME = 16 * 1024 * 1024


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("peer closed")
        buf += chunk
    return bytes(buf)


class RelayServer:
    def __init__(self, host: str = "127.0.0.1", port: int = 0, max_frame: int = DEFAULT_MAX_FRAME):
        self.max_frame = max_frame
        self._srv = socket.create_server((host, port))
        self.addr = self._srv.getsockname()
        self._clients: Dict[bytes, socket.socket] = {}
        self._locks: Dict[bytes, threading.Lock] = {}
        self._mu = threading.Lock()
        self.forwarded = 0
        self.dropped = 0
        self._closing = False
        threading.Thread(target=self._accept, daemon=True, name="relay-accept").start()

    def _accept(self):
        while not self._closing:
            try:
                conn, _ = self._srv.accept()
            except OSError:
                return
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            threading.Thread(target=self._serve, args=(conn,), daemon=True).start()

    def _serve(self, conn: socket.socket):
        node = None
        try:
            node = _recv_exact(conn, ID_LEN)
            with self._mu:
                self._clients[node] = conn
                self._locks[node] = threading.Lock()
            while True:
                dst = _recv_exact(conn, ID_LEN)
                (n,) = struct.unpack("<I", _recv_exact(conn, 4))
                if n > self.max_frame:
                    raise ConnectionError("frame too large")
                payload = _recv_exact(conn, n)
                with self._mu:
                    out, lk = self._clients.get(dst), self._locks.get(dst)
                if out is None:
                    self.dropped += 1
                    continue
                with lk:
                    try:
                        out.sendall(node + struct.pack("<I", n) + payload)
                        self.forwarded += 1
                    except OSError:
                        self.dropped += 1
        except (ConnectionError, OSError):
            pass
        finally:
            if node is not None:
                with self._mu:
                    if self._clients.get(node) is conn:
                        del self._clients[node]
            conn.close()

    def close(self):
        self._closing = True
        self._srv.close()
        with self._mu:
            for c in self._clients.values():
                try:
                    c.close()
                except OSError:
                    pass


class RelayClient:
    def __init__(self, addr: Tuple[str, int], node_id: bytes, timeout_s: float = 10.0):
        assert len(node_id) == ID_LEN
        self.node_id = node_id
        self._sock = socket.create_connection(addr, timeout=timeout_s)
        self._sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self._sock.sendall(node_id)
        self._send_lock = threading.Lock()

    def send(self, dst: bytes, payload: bytes):
        with self._send_lock:
            self._sock.sendall(dst + struct.pack("<I", len(payload)) + payload)

    def recv(self, timeout_s: Optional[float] = None) -> Tuple[bytes, bytes]:
        self._sock.settimeout(timeout_s)
        src = _recv_exact(self._sock, ID_LEN)
        (n,) = struct.unpack("<I", _recv_exact(self._sock, 4))
        return src, _recv_exact(self._sock, n)

    def close(self):
        self._sock.close()
