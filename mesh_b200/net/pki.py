"""Pool and device identities: ed25519 keys, pool/node ids, pool membership certificates.

Identifiers and signing payloads keep the reference's byte layout so that records signed by one
implementation verify in the other (``agent/src/pki/types.rs:11-68`` ids,
``:230-361`` membership certificate):

* pool id = sha256(b"meshnet-pool-v1" || pool root public key)
* node id = sha256(b"meshnet-node-v1" || device public key)
* certificate payload = device pubkey || pool id || role byte (member 0, admin 1) || expires_at u64 LE
* certificate hash = sha256(payload || signature)
"""
from __future__ import annotations

import hashlib
import struct
import time
from dataclasses import dataclass
from typing import Optional

from cryptography.exceptions import InvalidSignature
from cryptography.hazmat.primitives import serialization
from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PrivateKey, Ed25519PublicKey

ROLE_MEMBER = "member"
ROLE_ADMIN = "admin"
_ROLE_BYTE = {ROLE_MEMBER: 0, ROLE_ADMIN: 1}


def pool_id_from_pubkey(pub: bytes) -> bytes:
    return hashlib.sha256(b"meshnet-pool-v1" + pub).digest()


def node_id_from_pubkey(pub: bytes) -> bytes:
    return hashlib.sha256(b"meshnet-node-v1" + pub).digest()


def verify_signature(pub: bytes, payload: bytes, signature: bytes) -> bool:
    try:
        Ed25519PublicKey.from_public_bytes(bytes(pub)).verify(bytes(signature), bytes(payload))
        return True
    except (InvalidSignature, ValueError):
        return False


class KeyPair:
    """An ed25519 key pair (device key or pool root key)."""

    def __init__(self, private: Optional[Ed25519PrivateKey] = None):
        self._sk = private or Ed25519PrivateKey.generate()
        self.public = self._sk.public_key().public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)

    @classmethod
    def from_seed(cls, seed: bytes) -> "KeyPair":
        return cls(Ed25519PrivateKey.from_private_bytes(bytes(seed)))

    def seed(self) -> bytes:
        return self._sk.private_bytes(serialization.Encoding.Raw, serialization.PrivateFormat.Raw,
                                      serialization.NoEncryption())

    def sign(self, payload: bytes) -> bytes:
        return self._sk.sign(bytes(payload))

    @property
    def node_id(self) -> bytes:
        return node_id_from_pubkey(self.public)

    @property
    def pool_id(self) -> bytes:
        return pool_id_from_pubkey(self.public)


@dataclass
class MembershipCert:
    device_pubkey: bytes
    pool_id: bytes
    role: str
    expires_at: int
    signature: bytes

    @staticmethod
    def _payload(device_pubkey: bytes, pool_id: bytes, role: str, expires_at: int) -> bytes:
        return bytes(device_pubkey) + bytes(pool_id) + bytes([_ROLE_BYTE[role]]) + struct.pack("<Q", expires_at)

    @classmethod
    def issue(cls, device_pubkey: bytes, pool_root: KeyPair, role: str = ROLE_MEMBER,
              expires_at: Optional[int] = None) -> "MembershipCert":
        expires_at = int(expires_at if expires_at is not None else time.time() + 365 * 86400)
        pid = pool_root.pool_id
        sig = pool_root.sign(cls._payload(device_pubkey, pid, role, expires_at))
        return cls(bytes(device_pubkey), pid, role, expires_at, sig)

    def verify(self, pool_root_pubkey: bytes, now: Optional[int] = None) -> bool:
        now = int(time.time() if now is None else now)
        if now >= self.expires_at or self.pool_id != pool_id_from_pubkey(pool_root_pubkey):
            return False
        return verify_signature(pool_root_pubkey,
                                self._payload(self.device_pubkey, self.pool_id, self.role, self.expires_at),
                                self.signature)

    def hash(self) -> bytes:
        return hashlib.sha256(self._payload(self.device_pubkey, self.pool_id, self.role, self.expires_at) +
                              self.signature).digest()

    @property
    def node_id(self) -> bytes:
        return node_id_from_pubkey(self.device_pubkey)

    def to_dict(self) -> dict:
        return {"device_pubkey": self.device_pubkey.hex(), "pool_id": self.pool_id.hex(), "role": self.role,
                "expires_at": self.expires_at, "signature": self.signature.hex()}

    @classmethod
    def from_dict(cls, d: dict) -> "MembershipCert":
        return cls(bytes.fromhex(d["device_pubkey"]), bytes.fromhex(d["pool_id"]), d["role"], int(d["expires_at"]),
                   bytes.fromhex(d["signature"]))
