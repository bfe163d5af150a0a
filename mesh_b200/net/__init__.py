"""LAN and wide-area plumbing outside the GPU hot path: device/pool identities (``pki``), signed
UDP pool beacons and peer caches (``beacon``), signed ring-state gossip (``gossip``), an optional
TCP relay (``relay``) and connectivity records with direct-dial ranking (``connectivity``)."""
