"""Device certificates issued by the control plane (``control-plane/src/services/certificate.rs:18-200``).

At registration the control plane signs a certificate binding the device id, its network and its
ed25519 public key, valid for 30 days. The blob is CBOR ``{"certificate": <CBOR of the fields>,
"signature": <64-byte ed25519 signature over those bytes>}``, the reference's layout, so either
side can check the other's certificates. The signing key is kept in a file (hex of the 32-byte
seed, created on first use) or, without a path, lives only as long as the process.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import cbor2
from cryptography.exceptions import InvalidSignature
from cryptography.hazmat.primitives import serialization
from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PrivateKey, Ed25519PublicKey

VALIDITY_DAYS = 30


class CertificateError(ValueError):
    pass


@dataclass
class DeviceCertificate:
    device_id: str
    network_id: str
    public_key: bytes
    issued_at: str
    expires_at: str

    def expired(self, now: Optional[datetime.datetime] = None) -> bool:
        now = now or datetime.datetime.now(datetime.timezone.utc)
        return now >= datetime.datetime.fromisoformat(self.expires_at.replace("Z", "+00:00"))


def _rfc3339(t: datetime.datetime) -> str:
    return t.astimezone(datetime.timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ")


class ControlPlaneKeypair:
    def __init__(self, key: Ed25519PrivateKey):
        self.key = key

    @classmethod
    def generate(cls) -> "ControlPlaneKeypair":
        return cls(Ed25519PrivateKey.generate())

    @classmethod
    def load_or_generate(cls, path) -> "ControlPlaneKeypair":
        """The key stored at ``path`` (hex of its 32-byte seed); a new one is written there (mode
        0600) when the file does not exist."""
        p = Path(path)
        if p.exists():
            try:
                seed = bytes.fromhex(p.read_text().strip())
                return cls(Ed25519PrivateKey.from_private_bytes(seed))
            except ValueError as e:
                raise CertificateError(f"invalid control-plane key file {p}: {e}") from e
        kp = cls.generate()
        p.parent.mkdir(parents=True, exist_ok=True)
        seed = kp.key.private_bytes(serialization.Encoding.Raw, serialization.PrivateFormat.Raw,
                                    serialization.NoEncryption())
        fd = os.open(str(p), os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o600)
        with os.fdopen(fd, "w") as f:
            f.write(seed.hex())
        return kp

    def public_key(self) -> bytes:
        return self.key.public_key().public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)

    def generate_certificate(self, device_id: str, network_id: str, public_key: bytes,
                             now: Optional[datetime.datetime] = None) -> bytes:
        if len(public_key) != 32:
            raise CertificateError("public key must be 32 bytes (ed25519)")
        now = now or datetime.datetime.now(datetime.timezone.utc)
        fields = {"device_id": device_id, "network_id": network_id, "public_key": bytes(public_key),
                  "issued_at": _rfc3339(now), "expires_at": _rfc3339(now + datetime.timedelta(days=VALIDITY_DAYS))}
        body = cbor2.dumps(fields)
        return cbor2.dumps({"certificate": body, "signature": self.key.sign(body)})

    def verify_certificate(self, blob: bytes) -> DeviceCertificate:
        return verify_certificate(blob, self.public_key())


def verify_certificate(blob: bytes, control_plane_public_key: bytes) -> DeviceCertificate:
    """Check the signature with the control plane's public key; returns the certificate's fields."""
    try:
        outer = cbor2.loads(blob)
        body, sig = outer["certificate"], outer["signature"]
    except Exception as e:
        raise CertificateError(f"malformed certificate: {e}") from e
    if len(sig) != 64:
        raise CertificateError("invalid signature length")
    try:
        Ed25519PublicKey.from_public_bytes(bytes(control_plane_public_key)).verify(bytes(sig), bytes(body))
    except InvalidSignature as e:
        raise CertificateError("invalid certificate signature") from e
    f = cbor2.loads(body)
    return DeviceCertificate(f["device_id"], f["network_id"], bytes(f["public_key"]), f["issued_at"], f["expires_at"])
