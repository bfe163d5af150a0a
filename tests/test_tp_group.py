"""TP worker group: the leader's backend calls replayed by the followers.

CPU: two gloo ranks with a recording fake backend check that followers make exactly the leader's
calls in order (prefill, decode, release), that KV export gathers one part per rank and import
scatters them back, and that a stop message ends the follower loop.
GPU (2 GPUs): a model written to disk in the reference shard format, served by a 2-GPU group
driven through the coordinator from rank 0, gives the same tokens as both ranks running the same
program themselves.
"""
import os
import socket
import tempfile
import uuid

import pytest
import torch


class _Recorder:
    provider = "cuda"
    class_key = 1

    def __init__(self, rank):
        self.rank = rank
        self.log = []
        self.imported = {}

    def token_ceiling(self, n):
        return n

    def prefill(self, h, prompt, temperature, top_p, seed_base):
        self.log.append(("prefill", h, tuple(prompt)))
        return 100 + h

    def decode(self, items):
        self.log.append(("decode", tuple(h for h, *_ in items)))
        return [200 + h for h, *_ in items]

    def release(self, h):
        self.log.append(("release", h))

    def kv_bytes(self, h):
        return 10

    def export_kv(self, h):
        self.log.append(("export", h))
        return f"kv-{h}-rank{self.rank}".encode()

    def import_kv(self, h, payload, prompt, generated):
        self.log.append(("import", h))
        self.imported[h] = payload


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_rank(rank, world, port, d):
    import torch.distributed as dist
    from mesh_b200.runtime.tp_group import TPGroupBackend, follow
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    b = _Recorder(rank)
    if rank == 0:
        tb = TPGroupBackend(b, dist.group.WORLD, world)
        assert tb.prefill(1, [5, 6], 0.0, 1.0, 0) == 101
        assert tb.decode([(1, 7)]) == [201]
        blob = tb.export_kv(1)
        tb.import_kv(2, blob, [5, 6], [7])
        tb.release(1)
        assert tb.kv_bytes(1) == 10 * world
        tb.stop()
    else:
        n = follow(b, dist.group.WORLD)
        assert n == 5
    with open(os.path.join(d, f"log{rank}"), "w") as f:
        f.write(repr((b.log, b.imported)))
    dist.destroy_process_group()


def test_followers_replay_leader_calls_cpu():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_cpu_rank, args=(2, _free_port(), d), nprocs=2, join=True)
        logs = [eval(open(os.path.join(d, f"log{r}")).read()) for r in range(2)]
    want = [("prefill", 1, (5, 6)), ("decode", (1,)), ("export", 1), ("import", 2), ("release", 1)]
    for r, (log, imported) in enumerate(logs):
        assert log == want, (r, log)
        # every rank got back its own part of the group checkpoint
        assert imported == {2: f"kv-1-rank{r}".encode()}


def test_import_rejects_other_tp_degree():
    from mesh_b200.runtime.tp_group import TPGroupBackend
    import cbor2
    tb = TPGroupBackend(_Recorder(0), None, 2)
    with pytest.raises(ValueError):
        tb.import_kv(1, cbor2.dumps({"encoding": "tp_parts_v1", "world": 4, "parts": [b""] * 4}), [1], [2])
    with pytest.raises(ValueError):
        tb.import_kv(1, b"not a group checkpoint", [1], [2])


# ------------------------------------------------------------------------------------------ GPU
def _leader_generate(tb, cfg, ecfg):
    """Rank 0 of the group: serve three prompts through the coordinator, greedy."""
    from mesh_b200.engine.coordinator import InferenceCoordinator
    from mesh_b200.engine.types import ExecutionPhase, GenerationConfig, InferenceRequest
    coord = InferenceCoordinator(tb, ecfg, model_id=cfg.name)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 30, 17)]
    out = {}
    for i, p in enumerate(prompts):
        req = InferenceRequest(network_id="n", model_id=cfg.name, prompt_tokens=p, executor_id="gpu",
                               job_id=str(uuid.UUID(int=i + 1)), session_id=f"s{i}", phase=ExecutionPhase.PREFILL,
                               config=GenerationConfig(max_tokens=6, temperature=0.0, top_p=1.0))
        coord.process_segment(req)
    while len(out) < len(prompts):
        for res in coord.step():
            out[res.job_id] = list(res.generated_tokens)
    return {"prompts": prompts, "tokens": [out[str(uuid.UUID(int=i + 1))] for i in range(len(prompts))]}


@pytest.mark.gpu
def test_tp2_group_from_disk_replays_leader():
    """A 2-GPU group loading its shards from disk and driven by rank 0 alone gives exactly the
    tokens of the same program run by both ranks themselves (same kernels, same collectives)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from mesh_b200.config import get_preset
    from mesh_b200.models.artifacts import write_model
    from mesh_b200.models.weights import synthetic_reference_weights
    from mesh_b200.runtime.tp_group import GroupSpec, run_group
    cfg = get_preset("small").replace(name="small-disk")
    w = synthetic_reference_weights(cfg, seed=11)
    with tempfile.TemporaryDirectory() as d:
        write_model(os.path.join(d, "tp2"), cfg.name, w, 2)
        spec = GroupSpec(world=2, model_dir=os.path.join(d, "tp2", cfg.name), max_seq_len=256, num_pages=256,
                         max_batch=8, max_tokens=512, timeout_s=60.0)
        res = {}
        for spmd in (False, True):
            wd = os.path.join(d, f"run{int(spmd)}")
            os.makedirs(wd)
            res[spmd] = run_group(spec, _leader_generate, wd, spmd=spmd)
    assert res[False]["prompts"] == res[True]["prompts"]
    assert all(len(t) == 6 for t in res[False]["tokens"])
    assert res[False]["tokens"] == res[True]["tokens"]
