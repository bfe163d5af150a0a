"""LAN discovery, ring gossip, relay and connectivity ranking (CPU, loopback sockets)."""
import time

from mesh_b200.net import beacon, connectivity as cn, gossip, pki, relay


def _member(pool_root, role=pki.ROLE_MEMBER):
    dev = pki.KeyPair()
    return dev, pki.MembershipCert.issue(dev.public, pool_root, role)


def test_ids_and_membership_cert():
    root = pki.KeyPair()
    dev, cert = _member(root)
    assert len(root.pool_id) == 32 and root.pool_id != dev.node_id
    assert cert.verify(root.public)
    assert not cert.verify(pki.KeyPair().public)                       # other pool
    assert not cert.verify(root.public, now=cert.expires_at)           # expired
    bad = pki.MembershipCert(cert.device_pubkey, cert.pool_id, pki.ROLE_ADMIN, cert.expires_at, cert.signature)
    assert not bad.verify(root.public)                                 # role is signed
    assert pki.MembershipCert.from_dict(cert.to_dict()) == cert
    assert cert.hash() != bad.hash()


def test_beacon_sign_verify_and_tamper():
    root = pki.KeyPair()
    dev, cert = _member(root)
    b = beacon.PoolBeacon.create(dev, cert, quic_port=4433, admin=True)
    assert b.verify() and b.capabilities & beacon.CAP_CAN_SIGN_CERTS
    w = beacon.PoolBeacon.from_wire(b.to_wire())
    assert w is not None and w.verify() and w.node_id == dev.node_id
    w.quic_port = 1
    assert not w.verify()
    assert beacon.PoolBeacon.from_wire(b"garbage") is None


def test_beacon_service_discovers_peers_on_loopback():
    root = pki.KeyPair()
    (d1, c1), (d2, c2) = _member(root), _member(root)
    s1 = beacon.BeaconService(d1, [c1], bind=("127.0.0.1", 0), targets=[], join_group=False, interval_s=0.05)
    s2 = beacon.BeaconService(d2, [c2], bind=("127.0.0.1", 0), targets=[s1.addr], join_group=False, interval_s=0.05)
    s1.targets = [s2.addr]
    s1.start(), s2.start()
    try:
        deadline = time.time() + 5
        while time.time() < deadline and not (s1.peers(root.pool_id) and s2.peers(root.pool_id)):
            time.sleep(0.05)
        assert [p.node_id for p in s1.peers(root.pool_id)] == [d2.node_id]
        assert [p.node_id for p in s2.peers(root.pool_id)] == [d1.node_id]
        before = s1.rejected
        s1.handle(b"not a beacon", ("127.0.0.1", 1))
        assert s1.rejected == before + 1
    finally:
        s1.close(), s2.close()
    cache = beacon.PeerCache(root.pool_id)
    cache.update(beacon.PoolBeacon.create(d2, c2), ("10.0.0.2", 1), now=100.0)
    assert cache.live(now=120.0) and not cache.live(now=131.0)
    assert cache.prune(now=131.0) == 1


def test_ring_state_shards_neighbors_and_merge():
    root = pki.KeyPair()
    devs = [pki.KeyPair() for _ in range(3)]
    now = int(time.time())
    st = gossip.RingState(root.pool_id)
    for d in devs:
        st.add_member(gossip.RingMember(d.node_id, now, "active"))
    ranges = sorted(st.shard_range(d.node_id) for d in devs)
    assert ranges == [(0, 2730), (2730, 5460), (5460, 8192)]
    left, right = st.neighbors(devs[0].node_id)
    assert {left, right} <= {d.node_id for d in devs[1:]}
    other = gossip.RingState(root.pool_id, version=10)
    for k, m in st.members.items():
        other.members[k] = gossip.RingMember(m.node_id, m.last_seen + 5, "leaving")
    assert st.merge(other, now=now + 5)
    assert st.version == 11 and all(m.status == "leaving" for m in st.members.values())
    assert st.merge(gossip.RingState(root.pool_id), now=now + 100)      # everyone silent for 60 s
    assert not st.members


def test_ring_gossip_signed_exchange():
    root = pki.KeyPair()
    a, b = gossip.RingGossip(pki.KeyPair(), root.pool_id), gossip.RingGossip(pki.KeyPair(), root.pool_id)
    assert b.receive(a.outgoing()) and a.receive(b.outgoing())
    assert len(a.state.members) == len(b.state.members) == 2
    msg = gossip.RingGossipMessage.from_wire(a.outgoing())
    msg.version += 1                                                     # tampered
    assert not b.receive(msg.to_wire())
    foreign = gossip.RingGossip(pki.KeyPair(), pki.KeyPair().pool_id)
    assert not a.receive(foreign.outgoing())


def test_relay_forwards_between_registered_nodes():
    srv = relay.RelayServer()
    n1, n2 = pki.KeyPair().node_id, pki.KeyPair().node_id
    c1, c2 = relay.RelayClient(srv.addr, n1), relay.RelayClient(srv.addr, n2)
    try:
        time.sleep(0.1)
        c1.send(n2, b"hello")
        src, data = c2.recv(timeout_s=5)
        assert src == n1 and data == b"hello"
        c2.send(n1, b"x" * 100000)
        src, data = c1.recv(timeout_s=5)
        assert src == n2 and len(data) == 100000
    finally:
        c1.close(), c2.close(), srv.close()


def test_connectivity_ranking_and_persistence(tmp_path):
    addrs = ["/ip4/192.168.1.4/tcp/4001", "/ip4/8.8.8.8/udp/4001/quic-v1", "/ip4/127.0.0.1/tcp/1",
             "/ip4/8.8.8.8/tcp/4001", "/dns4/node.example/tcp/4001", "/ip4/1.2.3.4/tcp/1/p2p-circuit",
             "/ip4/0.0.0.0/tcp/1", "/ip4/192.0.2.5/tcp/1"]
    ranked = cn.select_dial_addrs(addrs, peer_id="12D3Koo")
    assert ranked[0].startswith("/ip4/8.8.8.8/udp/4001/quic-v1") and ranked[0].endswith("/p2p/12D3Koo")
    assert [a.split("/p2p")[0] for a in ranked] == ["/ip4/8.8.8.8/udp/4001/quic-v1", "/ip4/8.8.8.8/tcp/4001",
                                                    "/dns4/node.example/tcp/4001", "/ip4/192.168.1.4/tcp/4001",
                                                    "/ip4/127.0.0.1/tcp/1"]
    now = cn.now_ms()
    seeds = [cn.CandidateSeed("/ip4/9.9.9.9/tcp/1", "observed_external", now - cn.OBSERVED_MAX_AGE_MS - 1),
             cn.CandidateSeed("/ip4/192.168.1.44/tcp/4001", "local_listen", now),
             cn.CandidateSeed("/ip4/9.9.9.8/tcp/1", "observed_external", now)]
    cands = cn.build_candidates(seeds, now=now)
    assert [c.endpoint for c in cands] == ["/ip4/9.9.9.8/tcp/1", "/ip4/192.168.1.44/tcp/4001"]
    assert cn.advertisable(["dataplane://x", "/ip4/127.0.0.1/tcp/1", "/ip4/10.0.0.1/tcp/2"]) == \
        ["dataplane://x", "/ip4/10.0.0.1/tcp/2"]
    st = cn.NetworkConnectivity("relayed", [cn.ConnectivityAttachment("tcp_relay", "10.0.0.9:9", 1)]).configured_state()
    cn.persist_state(st, home=tmp_path)
    assert cn.load_state(home=tmp_path) == st
    recs = cn.record_observed("/ip4/9.9.9.9/tcp/1", home=tmp_path)
    recs = cn.record_observed("/ip4/9.9.9.9/tcp/1", home=tmp_path)
    assert len(recs) == 1
