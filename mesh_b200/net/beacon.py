"""LAN discovery: signed pool beacons over UDP (a LAN group address by default) and a peer cache.

Behaviour follows the reference's discovery service (``agent/src/discovery/beacon.rs``): every
5 s a node announces each pool it belongs to on 239.192.0.1:42424 (``:22-31``); a beacon carries
the pool id, node id, device public key, a QUIC port, the key fingerprint (first 8 bytes), the hash
of the node's membership certificate, a capability bitmap and a timestamp, signed by the device key
over the same byte layout as the reference (``:154-236``); receivers verify the signature and the
node id / fingerprint derivations, ignore their own beacons and keep a per-pool peer cache whose
entries go stale after 30 s. Messages are CBOR maps tagged by kind, as serde encodes the
reference's ``BeaconMessage`` enum.
"""
from __future__ import annotations

import socket
import struct
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Tuple

import cbor2

from .pki import KeyPair, MembershipCert, node_id_from_pubkey, verify_signature

GROUP_ADDR = "239.192.0.1"
BEACON_PORT = 42424
BEACON_INTERVAL_S = 5.0
STALE_PEER_S = 30.0

CAP_CAN_SIGN_CERTS = 0x0001
CAP_ACCEPTING_JOINS = 0x0002
CAP_HAS_RELAY = 0x0004
CAP_HAS_CONTROL_PLANE = 0x0008


@dataclass
class PoolBeacon:
    pool_id: bytes
    node_id: bytes
    device_pubkey: bytes
    quic_port: int
    pubkey_fingerprint: bytes
    membership_cert_hash: bytes
    capabilities: int
    timestamp: int
    signature: bytes = b""
    version: int = 1
    peer_id: Optional[str] = None

    def payload(self) -> bytes:
        return (bytes([self.version]) + self.pool_id + self.node_id + self.device_pubkey +
                struct.pack("<H", self.quic_port) + self.pubkey_fingerprint + self.membership_cert_hash +
                struct.pack("<I", self.capabilities) + struct.pack("<Q", self.timestamp))

    @classmethod
    def create(cls, device: KeyPair, cert: MembershipCert, quic_port: int = 0, capabilities: int = 0,
               peer_id: Optional[str] = None, admin: bool = False) -> "PoolBeacon":
        caps = capabilities | ((CAP_CAN_SIGN_CERTS | CAP_ACCEPTING_JOINS) if admin else 0)
        b = cls(cert.pool_id, device.node_id, device.public, quic_port, device.public[:8], cert.hash(), caps,
                int(time.time()), peer_id=peer_id)
        b.signature = device.sign(b.payload())
        return b

    def verify(self) -> bool:
        if self.node_id != node_id_from_pubkey(self.device_pubkey):
            return False
        if self.pubkey_fingerprint != self.device_pubkey[:8]:
            return False
        return verify_signature(self.device_pubkey, self.payload(), self.signature)

    def to_wire(self) -> bytes:
        return cbor2.dumps({"PoolBeacon": {
            "version": self.version, "pool_id": self.pool_id, "node_id": self.node_id,
            "device_pubkey": self.device_pubkey, "peer_id": self.peer_id, "quic_port": self.quic_port,
            "pubkey_fingerprint": self.pubkey_fingerprint, "membership_cert_hash": self.membership_cert_hash,
            "capabilities_bitmap": self.capabilities, "timestamp": self.timestamp,
            "signature": self.signature.hex()}})

    @classmethod
    def from_wire(cls, data: bytes) -> Optional["PoolBeacon"]:
        try:
            d = cbor2.loads(data)["PoolBeacon"]
            return cls(bytes(d["pool_id"]), bytes(d["node_id"]), bytes(d["device_pubkey"]), int(d["quic_port"]),
                       bytes(d["pubkey_fingerprint"]), bytes(d["membership_cert_hash"]),
                       int(d["capabilities_bitmap"]), int(d["timestamp"]), bytes.fromhex(d["signature"]),
                       int(d["version"]), d.get("peer_id"))
        except (KeyError, TypeError, ValueError, cbor2.CBORDecodeError):
            return None


@dataclass
class DiscoveredPeer:
    node_id: bytes
    device_pubkey: bytes
    addr: Tuple[str, int]
    quic_port: int
    capabilities: int
    last_seen: float
    peer_id: Optional[str] = None


@dataclass
class PeerCache:
    """Peers of one pool seen on the LAN, keyed by node id."""
    pool_id: bytes
    peers: Dict[bytes, DiscoveredPeer] = field(default_factory=dict)

    def update(self, beacon: PoolBeacon, addr: Tuple[str, int], now: Optional[float] = None):
        self.peers[beacon.node_id] = DiscoveredPeer(beacon.node_id, beacon.device_pubkey, addr, beacon.quic_port,
                                                    beacon.capabilities, time.time() if now is None else now,
                                                    beacon.peer_id)

    def live(self, now: Optional[float] = None, stale_s: float = STALE_PEER_S) -> List[DiscoveredPeer]:
        now = time.time() if now is None else now
        return [p for p in self.peers.values() if now - p.last_seen < stale_s]

    def prune(self, now: Optional[float] = None, stale_s: float = STALE_PEER_S) -> int:
        now = time.time() if now is None else now
        dead = [k for k, p in self.peers.items() if now - p.last_seen >= stale_s]
        for k in dead:
            del self.peers[k]
        return len(dead)


class BeaconService:
    """Announces this node's pools and listens for peers' beacons.

    ``targets`` are the destinations of announcements (the LAN group address by default; unicast
    addresses work where group delivery is unavailable, e.g. tests on loopback)."""

    def __init__(self, device: KeyPair, pools: Iterable[MembershipCert], bind: Tuple[str, int] = ("0.0.0.0",
                 BEACON_PORT), targets: Optional[List[Tuple[str, int]]] = None, interval_s: float = BEACON_INTERVAL_S,
                 join_group: bool = True, quic_port: int = 0, admin: bool = False):
        self.device = device
        self.pools = list(pools)
        self.interval_s = interval_s
        self.quic_port = quic_port
        self.admin = admin
        self.caches: Dict[bytes, PeerCache] = {c.pool_id: PeerCache(c.pool_id) for c in self.pools}
        self.rejected = 0
        self._sock = socket.socket(socket.AF_INET, socket.SOCK_DGRAM, socket.IPPROTO_UDP)
        self._sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        if hasattr(socket, "SO_REUSEPORT"):
            try:
                self._sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEPORT, 1)
            except OSError:
                pass
        self._sock.bind(bind)
        self.addr = self._sock.getsockname()
        if join_group:
            mreq = struct.pack("4sl", socket.inet_aton(GROUP_ADDR), socket.INADDR_ANY)
            try:
                self._sock.setsockopt(socket.IPPROTO_IP, socket.IP_ADD_MEMBERSHIP, mreq)
            except OSError:
                pass  # no route for the group address: unicast targets still work
        self.targets = targets if targets is not None else [(GROUP_ADDR, BEACON_PORT)]
        self._stop = threading.Event()
        self._threads: List[threading.Thread] = []
        self._lock = threading.Lock()

    def announce_once(self):
        for cert in self.pools:
            wire = PoolBeacon.create(self.device, cert, self.quic_port, admin=self.admin).to_wire()
            for t in self.targets:
                try:
                    self._sock.sendto(wire, t)
                except OSError:
                    pass

    def handle(self, data: bytes, addr: Tuple[str, int]) -> Optional[PoolBeacon]:
        b = PoolBeacon.from_wire(data)
        if b is None or not b.verify():
            self.rejected += 1
            return None
        if b.node_id == self.device.node_id or b.pool_id not in self.caches:
            return None
        with self._lock:
            self.caches[b.pool_id].update(b, addr)
        return b

    def start(self):
        def announcer():
            while not self._stop.is_set():
                self.announce_once()
                self._stop.wait(self.interval_s)

        def listener():
            self._sock.settimeout(0.2)
            while not self._stop.is_set():
                try:
                    data, addr = self._sock.recvfrom(65536)
                except socket.timeout:
                    continue
                except OSError:
                    return
                self.handle(data, addr)

        for fn in (announcer, listener):
            t = threading.Thread(target=fn, daemon=True, name=f"beacon-{fn.__name__}")
            t.start()
            self._threads.append(t)
        return self

    def peers(self, pool_id: bytes) -> List[DiscoveredPeer]:
        with self._lock:
            return self.caches[pool_id].live()

    def close(self):
        self._stop.set()
        for t in self._threads:
            t.join(timeout=2)
        self._sock.close()
