"""The TP=1 decoder built from the sm_100a kernels against the fp32 host oracle."""
import numpy as np
import pytest
import torch

from mesh_b200.config import EngineConfig, get_preset
from mesh_b200.engine.serving import Engine
from mesh_b200.models.llama import KVPool, LlamaRunner, StepMeta
from mesh_b200.models.weights import device_weights_from_reference, synthetic_reference_weights
from mesh_b200.oracle import LocalForwardPass

pytestmark = pytest.mark.gpu


def _setup(name="tiny-gqa", seed=3, graphs=False):
    cfg = get_preset(name)
    wref = synthetic_reference_weights(cfg, seed=seed)
    dev = torch.device("cuda", 0)
    w = device_weights_from_reference(wref, 0, 1, device=dev)
    ecfg = EngineConfig(max_seq_len=256, prefill_chunk_tokens=256, use_cuda_graphs=graphs)
    kv = KVPool(cfg, w.layout.local_kv_heads, 64, 16, dev)
    runner = LlamaRunner(w, ecfg, kv, dev, max_tokens=512)
    return cfg, wref, runner, dev


def _rel(a, b):
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-9))


def test_prefill_and_decode_logits_match_oracle():
    cfg, wref, runner, dev = _setup()
    runner.keep_logits = True
    prompt = [5, 77, 3, 900, 12, 1, 64, 255, 31, 8, 600, 2, 9, 14, 15, 16, 17, 300]
    T = len(prompt)
    pages = [3, 9]
    slot = [pages[i // 16] * 16 + i % 16 for i in range(T)]
    bt = torch.zeros(1, 4, dtype=torch.int32, device=dev)
    bt[0, :2] = torch.tensor(pages)
    m = StepMeta(ids=torch.tensor(prompt, dtype=torch.int32, device=dev),
                 pos=torch.arange(T, dtype=torch.int32, device=dev),
                 slot=torch.tensor(slot, dtype=torch.int64, device=dev), block_tables=bt,
                 seq_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                 cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev),
                 last_idx=torch.tensor([T - 1], dtype=torch.int64, device=dev), max_q_len=T, decode=False)
    nxt = runner.forward(m)
    torch.cuda.synchronize()
    got = runner.last_logits[0].cpu().numpy()
    orc = LocalForwardPass(wref)
    want = orc.prefill(prompt)
    assert _rel(got, want) < 3e-2
    tok = int(np.argmax(want))
    # decode three steps feeding the oracle's greedy token to both
    for step in range(3):
        p = T + step
        m = StepMeta(ids=torch.tensor([tok], dtype=torch.int32, device=dev),
                     pos=torch.tensor([p], dtype=torch.int32, device=dev),
                     slot=torch.tensor([pages[p // 16] * 16 + p % 16], dtype=torch.int64, device=dev),
                     block_tables=bt, seq_lens=torch.tensor([p + 1], dtype=torch.int32, device=dev),
                     max_q_len=64, decode=True)
        runner.forward(m)
        torch.cuda.synchronize()
        got = runner.last_logits[0].cpu().numpy()
        want = orc.decode_step(tok)
        assert _rel(got, want) < 3e-2, step
        tok = int(np.argmax(want))


@pytest.mark.parametrize("graphs", [False, True])
def test_engine_generate_batch_consistency(graphs):
    """Sessions decoded together in one batch give the same tokens as each decoded alone."""
    cfg, wref, runner, dev = _setup(graphs=graphs)
    eng = Engine(runner, runner.ecfg, max_batch=8)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 40, 17)]
    together = eng.generate(prompts, 6)
    alone = [eng.generate([p], 6)[0] for p in prompts]
    eng.close()
    assert together == alone
    assert all(len(o) == 6 for o in together)
    assert eng.alloc.num_used == 0  # all pages returned


def test_fused_argmax_head_matches_logits_path():
    cfg, wref, runner, dev = _setup()
    x = torch.randn(37, cfg.hidden_dim, device=dev).to(torch.bfloat16)
    from mesh_b200 import ops
    w = runner.w
    tiles = torch.empty((w.vocab_local + 127) // 128, 37, 2, device=dev)
    cand = torch.empty(37, 2, device=dev)
    ops.lm_head_argmax(x, w.lm_head, 0, tiles, cand)
    logits = ops.linear(x, w.lm_head, epi=ops.EPI_STORE_F32)
    torch.cuda.synchronize()
    idx = cand[:, 1].contiguous().view(torch.int32)
    assert idx.tolist() == logits.argmax(-1).tolist()
    assert torch.allclose(cand[:, 0], logits.max(-1).values)


def test_engine_matches_oracle_greedy_first_token():
    cfg, wref, runner, dev = _setup()
    eng = Engine(runner, runner.ecfg, max_batch=4)
    prompt = list(range(3, 40))
    out = eng.generate([prompt], 1)[0]
    want = int(np.argmax(LocalForwardPass(wref).prefill(prompt)))
    assert out[0] == want


def test_poisoned_scratch_gives_same_tokens(monkeypatch):
    """With every activation scratch buffer filled with NaN before each step, generation is
    unchanged: each kernel writes all of the output it is responsible for."""
    from mesh_b200.models import llama
    cfg, wref, runner, dev = _setup()
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 33)]
    eng = Engine(runner, runner.ecfg, max_batch=8)
    clean = eng.generate(prompts, 5)
    monkeypatch.setattr(llama, "_POISON", True)
    poisoned = eng.generate(prompts, 5)
    eng.close()
    assert poisoned == clean
