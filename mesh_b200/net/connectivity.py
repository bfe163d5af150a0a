"""Connectivity records: how a device is reached, and which direct addresses to dial first.

Types and ranking follow the reference (``agent/src/connectivity.rs:10-105``, ``:297-520``):
a device's state is a path (direct or relayed), an optional active endpoint and a status; direct
candidates are multiaddrs classified by transport (QUIC before TCP) and address scope (public 0,
DNS 10, private 20, loopback 30; priority = scope rank + transport rank); circuit-relay addresses
and unsupported scopes (unspecified, group-address, broadcast, documentation ranges) are never direct
candidates; candidates observed from outside expire after 5 minutes, locally listened ones do
not; ranking is priority, then observed-before-local, then most recently updated, then endpoint
text, with duplicates removed. State and observed addresses persist as JSON under the mesh home.
"""
from __future__ import annotations

import ipaddress
import json
import os
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import List, Optional

OBSERVED_MAX_AGE_MS = 5 * 60 * 1000

SCOPE_RANK = {"public": 0, "dns": 10, "private": 20, "loopback": 30}
TRANSPORT_RANK = {"quic": 0, "tcp": 1}
SOURCE_RANK = {"observed_external": 0, "local_listen": 1}


def now_ms() -> int:
    return int(time.time() * 1000)


@dataclass
class ConnectivityAttachment:
    kind: str          # "libp2p_relay" in the reference; here any relay kind ("tcp_relay")
    endpoint: str
    priority: int = 0


@dataclass
class NetworkConnectivity:
    preferred_path: str = "direct"    # "direct" | "relayed"
    attachments: List[ConnectivityAttachment] = field(default_factory=list)

    def preferred_attachment(self) -> Optional[ConnectivityAttachment]:
        return min(self.attachments, key=lambda a: a.priority) if self.attachments else None

    def configured_state(self) -> "DeviceConnectivityState":
        a = self.preferred_attachment()
        return DeviceConnectivityState(self.preferred_path, a.endpoint if a else None, "connected")


@dataclass
class DeviceConnectivityState:
    active_path: str = "direct"
    active_endpoint: Optional[str] = None
    status: str = "unknown"          # unknown | connected | degraded | disconnected


@dataclass
class DirectCandidate:
    endpoint: str
    transport: str
    scope: str
    source: str = "local_listen"
    priority: int = 0
    last_updated_ms: int = 0


@dataclass
class CandidateSeed:
    endpoint: str
    source: str = "local_listen"
    last_updated_ms: int = 0


def _parts(addr: str) -> List[str]:
    return [p for p in addr.split("/") if p]


def _ip_scope(ip: str) -> Optional[str]:
    try:
        a = ipaddress.ip_address(ip)
    except ValueError:
        return None
    if a.is_loopback:
        return "loopback"
    doc4 = [ipaddress.ip_network(n) for n in ("192.0.2.0/24", "198.51.100.0/24", "203.0.113.0/24")]
    group = ipaddress.ip_network("224.0.0.0/4" if a.version == 4 else "ff00::/8")  # one-to-many ranges
    if a.is_unspecified or a in group or (a.version == 4 and (str(a) == "255.255.255.255" or
                                                              any(a in n for n in doc4))):
        return None
    if a.version == 6 and a in ipaddress.ip_network("2001:db8::/32"):
        return None
    if a.is_private or a.is_link_local:
        return "private"
    return "public"


def classify(addr: str) -> Optional[DirectCandidate]:
    """Direct-dial candidate for a multiaddr string, or None if it cannot be dialled directly."""
    parts = _parts(addr)
    if "p2p-circuit" in parts:
        return None
    scope, transport = "dns", None
    i = 0
    while i < len(parts):
        p = parts[i]
        if p in ("ip4", "ip6") and i + 1 < len(parts):
            scope = _ip_scope(parts[i + 1])
            if scope is None:
                return None
            i += 2
            continue
        if p in ("dns", "dns4", "dns6", "dnsaddr"):
            scope = "dns"
        elif p in ("quic", "quic-v1"):
            transport = "quic"
        elif p == "tcp" and transport is None:
            transport = "tcp"
        i += 1
    if transport is None:
        return None
    return DirectCandidate(addr, transport, scope, "local_listen", SCOPE_RANK[scope] + TRANSPORT_RANK[transport],
                           now_ms())


def _canonical(addr: str, peer_id: Optional[str]) -> str:
    if peer_id is None or "p2p" in _parts(addr):
        return addr
    return addr.rstrip("/") + f"/p2p/{peer_id}"


def build_candidates(seeds: List[CandidateSeed], peer_id: Optional[str] = None,
                     now: Optional[int] = None) -> List[DirectCandidate]:
    now = now_ms() if now is None else now
    out = []
    for s in seeds:
        if s.source == "observed_external" and now - s.last_updated_ms > OBSERVED_MAX_AGE_MS:
            continue
        c = classify(s.endpoint)
        if c is None or c.scope == "loopback":
            continue
        c.endpoint = _canonical(s.endpoint, peer_id)
        c.source = s.source
        c.last_updated_ms = s.last_updated_ms
        out.append(c)
    out.sort(key=lambda c: (c.priority, SOURCE_RANK[c.source], -c.last_updated_ms, c.endpoint))
    seen, uniq = set(), []
    for c in out:
        if c.endpoint not in seen:
            seen.add(c.endpoint)
            uniq.append(c)
    return uniq


def select_dial_addrs(addrs: List[str], peer_id: Optional[str] = None) -> List[str]:
    ranked = []
    for a in addrs:
        c = classify(a)
        if c is not None:
            ranked.append((c.priority, _canonical(a, peer_id)))
    ranked.sort()
    seen, out = set(), []
    for _, a in ranked:
        if a not in seen:
            seen.add(a)
            out.append(a)
    return out


def advertisable(addrs: List[str]) -> List[str]:
    """Addresses worth advertising to peers: dataplane URLs, and direct candidates except loopback."""
    seen, out = set(), []
    for a in addrs:
        ok = a.startswith("dataplane://")
        if not ok:
            c = classify(a)
            ok = c is not None and c.scope != "loopback"
        if ok and a not in seen:
            seen.add(a)
            out.append(a)
    return out


def _home() -> Path:
    return Path(os.environ.get("MESHNET_HOME", os.path.expanduser("~/.meshnet")))


def persist_state(state: DeviceConnectivityState, home: Optional[Path] = None) -> Path:
    p = (home or _home()) / "runtime" / "connectivity_state.json"
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(json.dumps(asdict(state)))
    return p


def load_state(home: Optional[Path] = None) -> Optional[DeviceConnectivityState]:
    p = (home or _home()) / "runtime" / "connectivity_state.json"
    try:
        return DeviceConnectivityState(**json.loads(p.read_text()))
    except (OSError, ValueError, TypeError):
        return None


def record_observed(addr: str, home: Optional[Path] = None, now: Optional[int] = None) -> List[CandidateSeed]:
    """Remember an externally observed address (fresh records only, newest timestamp per endpoint)."""
    now = now_ms() if now is None else now
    p = (home or _home()) / "runtime" / "observed_reachability.json"
    p.parent.mkdir(parents=True, exist_ok=True)
    try:
        recs = [CandidateSeed(**r) for r in json.loads(p.read_text())]
    except (OSError, ValueError, TypeError):
        recs = []
    recs = [r for r in recs if r.endpoint != addr and now - r.last_updated_ms <= OBSERVED_MAX_AGE_MS]
    recs.append(CandidateSeed(addr, "observed_external", now))
    p.write_text(json.dumps([asdict(r) for r in recs]))
    return recs
