"""Session handoff between two serving engines (two decode queues), on one GPU and across two.

The sessions of engine A decode a few tokens, are exported (each one's KV pages gathered into one
device buffer by the page-copy kernel), moved to engine B (a peer copy when B is on the other GPU),
imported into freshly allocated pages there and finished. B decodes the same batch A would have,
so the tokens must equal, bit for bit, those of the same sessions run start to finish in one
engine.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _engine(dev, seed=7):
    from mesh_b200.config import EngineConfig, get_preset
    from mesh_b200.engine.serving import Engine
    from mesh_b200.models.llama import KVPool, LlamaRunner
    from mesh_b200.models.weights import synthetic_device_weights
    cfg = get_preset("small")
    ecfg = EngineConfig(max_seq_len=256, use_cuda_graphs=True)
    w = synthetic_device_weights(cfg, 0, 1, seed=seed, device=dev)
    kv = KVPool(cfg, w.layout.local_kv_heads, 96, 16, dev)
    return Engine(LlamaRunner(w, ecfg, kv, dev, max_tokens=512), ecfg, max_batch=4), cfg


def _prompts(cfg):
    g = torch.Generator().manual_seed(21)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (23, 41, 9)]


def _handoff_case(dev_a, dev_b):
    from mesh_b200 import ops
    ref_eng, cfg = _engine(dev_a)
    prompts = _prompts(cfg)
    want = ref_eng.generate(prompts, 10)
    ref_eng.close()

    a, _ = _engine(dev_a)
    b, _ = _engine(dev_b)
    sids = [a.submit(p, 10) for p in prompts]
    while a.waiting:
        a.prefill_step()
    for _ in range(4):
        a.decode_step()
    # the whole decode queue moves, so B decodes the same batch A would have: bitwise the same tokens
    handoffs = [a.export_session(sid) for sid in sids]
    assert all(len(h.generated) == 5 and h.kv.device == torch.device(dev_a) for h in handoffs)
    assert a.alloc.num_used == 0 and not a.has_work()
    sids_b = [b.import_session(h.to(dev_b)) for h in handoffs]
    b.run()
    torch.cuda.synchronize(dev_a)
    torch.cuda.synchronize(dev_b)
    ops.scratch(dev_a).check("engine A")
    ops.scratch(dev_b).check("engine B")
    assert [b.sessions[s].generated for s in sids_b] == want
    assert b.alloc.num_used == 0  # every page returned
    a.close()
    b.close()


def test_handoff_between_engines_one_gpu():
    _handoff_case("cuda:0", "cuda:0")


def test_handoff_between_engines_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _handoff_case("cuda:0", "cuda:1")


def test_kv_pages_gather_scatter_roundtrip():
    from mesh_b200 import ops
    dev = "cuda:0"
    L, P, hkv, ps, D = 3, 20, 2, 16, 128
    k = torch.randn(L, P, hkv, ps, D, device=dev).to(torch.bfloat16)
    v = torch.randn(L, P, hkv, ps, D, device=dev).to(torch.bfloat16)
    pages = [7, 2, 13]
    buf = ops.kv_pages_gather(k, v, pages)
    assert torch.equal(buf[0], k[:, pages].reshape(L, 3, -1))
    assert torch.equal(buf[1], v[:, pages].reshape(L, 3, -1))
    k2, v2 = torch.zeros_like(k), torch.zeros_like(v)
    ops.kv_pages_scatter(k2, v2, [1, 5, 9], buf)
    assert torch.equal(k2[:, [1, 5, 9]], k[:, pages]) and torch.equal(v2[:, [1, 5, 9]], v[:, pages])
    assert k2[:, 0].abs().sum() == 0
    with pytest.raises(ValueError):
        ops.kv_pages_gather(k, v, [P])
