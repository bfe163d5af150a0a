"""The zip-equivalent serving engine: sessions, decode queue and microbatching, paged KV,
KV snapshots and checkpoints, statistics."""
