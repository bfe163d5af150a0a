"""Control plane: device registry, ring topology and shard assignment, inference job dispatch
(submit / claim / lease / progress / result), decode queue, KV transfer and checkpoint stores,
failover and presence, credits and ledger. FastAPI + SQLite with the reference's routes and JSON.
"""
