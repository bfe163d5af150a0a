"""Signed ring-state gossip for LAN pools.

Behaviour follows the reference's ring gossip (``agent/src/network/ring_gossip.rs``): a ring state
is the set of members of one pool (node id, optional peer id / LAN address, last-seen time,
status), ordered by a 64-bit hash of the node id; members split a fixed space of 8192 columns
evenly by ring position, the last one taking the remainder (``:262-276``); merging another state is
last-writer-wins per member on ``last_seen``, drops members silent for 60 s and bumps the version
past both inputs when anything changed (``:279-330``); a gossip message is signed by the sender's
device key over pool id || node id || device pubkey || version (u64 LE) || CBOR(ring state).

Ring order uses the first 8 bytes of sha256(node id) as the member key. (The reference hashes
with Rust's process-independent default hasher; the order is deterministic here as well, but two
implementations gossiping on one LAN would disagree on positions.)
"""
from __future__ import annotations

import hashlib
import struct
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import cbor2

from .pki import KeyPair, node_id_from_pubkey, verify_signature

TOTAL_COLUMNS = 8192
MEMBER_TIMEOUT_S = 60
STATUSES = ("joining", "active", "leaving", "failed")


def member_key(node_id: bytes) -> int:
    return struct.unpack("<Q", hashlib.sha256(node_id).digest()[:8])[0]


@dataclass
class RingMember:
    node_id: bytes
    last_seen: int
    status: str = "joining"
    peer_id: Optional[str] = None
    lan_addr: Optional[str] = None


@dataclass
class RingState:
    pool_id: bytes
    members: Dict[int, RingMember] = field(default_factory=dict)
    version: int = 0

    def add_member(self, m: RingMember):
        self.members[member_key(m.node_id)] = m
        self.version += 1

    def remove_member(self, node_id: bytes):
        self.members.pop(member_key(node_id), None)
        self.version += 1

    def update_status(self, node_id: bytes, status: str, now: Optional[int] = None) -> bool:
        m = self.members.get(member_key(node_id))
        if m is None:
            return False
        assert status in STATUSES
        m.status = status
        m.last_seen = int(time.time() if now is None else now)
        self.version += 1
        return True

    def ordered(self) -> List[RingMember]:
        return [self.members[k] for k in sorted(self.members)]

    def position(self, node_id: bytes) -> Optional[int]:
        keys = sorted(self.members)
        k = member_key(node_id)
        return keys.index(k) if k in self.members else None

    def neighbors(self, node_id: bytes) -> Optional[Tuple[bytes, bytes]]:
        pos = self.position(node_id)
        ms = self.ordered()
        if pos is None or len(ms) < 2:
            return None
        n = len(ms)
        return ms[(pos - 1) % n].node_id, ms[(pos + 1) % n].node_id

    def shard_range(self, node_id: bytes) -> Optional[Tuple[int, int]]:
        pos = self.position(node_id)
        if pos is None:
            return None
        n = len(self.members)
        per = TOTAL_COLUMNS // n
        start = pos * per
        return start, (TOTAL_COLUMNS if pos == n - 1 else start + per)

    def merge(self, other: "RingState", now: Optional[int] = None) -> bool:
        if other.pool_id != self.pool_id:
            return False
        changed = False
        for k, m in other.members.items():
            mine = self.members.get(k)
            if mine is None or mine.last_seen < m.last_seen:
                self.members[k] = RingMember(m.node_id, m.last_seen, m.status, m.peer_id, m.lan_addr)
                changed = True
        now = int(time.time() if now is None else now)
        for k in [k for k, m in self.members.items() if now - m.last_seen >= MEMBER_TIMEOUT_S]:
            del self.members[k]
            changed = True
        if changed:
            self.version = max(self.version, other.version) + 1
        return changed

    def is_stable(self) -> bool:
        return all(m.status == "active" for m in self.members.values())

    def to_obj(self) -> dict:
        return {"pool_id": self.pool_id, "version": self.version,
                "members": [[k, {"node_id": m.node_id, "peer_id": m.peer_id, "lan_addr": m.lan_addr,
                                 "last_seen": m.last_seen, "status": m.status}] for k, m in sorted(self.members.items())]}

    @classmethod
    def from_obj(cls, d: dict) -> "RingState":
        st = cls(bytes(d["pool_id"]), version=int(d["version"]))
        for k, m in d["members"]:
            st.members[int(k)] = RingMember(bytes(m["node_id"]), int(m["last_seen"]), m["status"], m.get("peer_id"),
                                            m.get("lan_addr"))
        return st


@dataclass
class RingGossipMessage:
    pool_id: bytes
    ring_state: RingState
    sender_node_id: bytes
    sender_pubkey: bytes
    version: int
    signature: bytes = b""

    def _payload(self) -> bytes:
        return (self.pool_id + self.sender_node_id + self.sender_pubkey + struct.pack("<Q", self.version) +
                cbor2.dumps(self.ring_state.to_obj(), canonical=True))

    @classmethod
    def create(cls, state: RingState, device: KeyPair) -> "RingGossipMessage":
        m = cls(state.pool_id, state, device.node_id, device.public, state.version)
        m.signature = device.sign(m._payload())
        return m

    def verify(self) -> bool:
        if self.sender_node_id != node_id_from_pubkey(self.sender_pubkey):
            return False
        return verify_signature(self.sender_pubkey, self._payload(), self.signature)

    def to_wire(self) -> bytes:
        return cbor2.dumps({"RingGossip": {"pool_id": self.pool_id, "ring_state": self.ring_state.to_obj(),
                                           "sender_node_id": self.sender_node_id,
                                           "sender_device_pubkey": self.sender_pubkey, "version": self.version,
                                           "signature": self.signature.hex()}})

    @classmethod
    def from_wire(cls, data: bytes) -> Optional["RingGossipMessage"]:
        try:
            d = cbor2.loads(data)["RingGossip"]
            return cls(bytes(d["pool_id"]), RingState.from_obj(d["ring_state"]), bytes(d["sender_node_id"]),
                       bytes(d["sender_device_pubkey"]), int(d["version"]), bytes.fromhex(d["signature"]))
        except (KeyError, TypeError, ValueError, cbor2.CBORDecodeError):
            return None


class RingGossip:
    """One node's view of a pool's ring: applies verified gossip from members of the pool."""

    def __init__(self, device: KeyPair, pool_id: bytes, lan_addr: Optional[str] = None):
        self.device = device
        self.state = RingState(pool_id)
        self.state.add_member(RingMember(device.node_id, int(time.time()), "active", lan_addr=lan_addr))
        self.rejected = 0

    def heartbeat(self, now: Optional[int] = None):
        self.state.update_status(self.device.node_id, "active", now)

    def outgoing(self) -> bytes:
        return RingGossipMessage.create(self.state, self.device).to_wire()

    def receive(self, data: bytes, now: Optional[int] = None) -> bool:
        msg = RingGossipMessage.from_wire(data)
        if msg is None or not msg.verify() or msg.pool_id != self.state.pool_id:
            self.rejected += 1
            return False
        return self.state.merge(msg.ring_state, now)
