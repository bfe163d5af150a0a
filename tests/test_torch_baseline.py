"""The plain-PyTorch comparison arm (``baselines.torch_tp.TorchTPRunner``) against the fp32 oracle.

Runs on the CPU (bf16 weights, fp32 oracle): prefill of a whole prompt, a prompt prefilled in two
chunks (the second chunk attends to a cached prefix), and batched decode steps whose padded slot
writes to the scratch page. The same runner drives the GPU baseline arm of the benchmark.
"""
import numpy as np
import torch

from mesh_b200.baselines.torch_tp import TorchTPRunner
from mesh_b200.config import EngineConfig, get_preset
from mesh_b200.models.llama import KVPool, StepMeta
from mesh_b200.models.weights import device_weights_from_reference, synthetic_reference_weights
from mesh_b200.oracle import LocalForwardPass


def _rel(a, b):
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-9))


def _runner(name="tiny-gqa", seed=5):
    cfg = get_preset(name)
    wref = synthetic_reference_weights(cfg, seed=seed)
    w = device_weights_from_reference(wref, 0, 1, device="cpu")
    ecfg = EngineConfig(max_seq_len=256)
    kv = KVPool(cfg, w.layout.local_kv_heads, 32, 16, "cpu")
    r = TorchTPRunner(w, ecfg, kv, "cpu", max_tokens=512)
    r.keep_logits = True
    return cfg, wref, r


def _prefill_meta(tokens, start, pages, kl, maxp=4):
    T = len(tokens)
    pos = list(range(start, start + T))
    slot = [pages[p // 16] * 16 + p % 16 for p in pos]
    bt = torch.zeros(1, maxp, dtype=torch.int32)
    bt[0, :len(pages)] = torch.tensor(pages)
    return StepMeta(ids=torch.tensor(tokens, dtype=torch.int32), pos=torch.tensor(pos, dtype=torch.int32),
                    slot=torch.tensor(slot, dtype=torch.int64), block_tables=bt,
                    seq_lens=torch.tensor([kl], dtype=torch.int32), cu_q=torch.tensor([0, T], dtype=torch.int32),
                    last_idx=torch.tensor([T - 1], dtype=torch.int64), max_q_len=T, decode=False)


def test_torch_baseline_prefill_chunks_and_decode_match_oracle():
    cfg, wref, r = _runner()
    prompt = [5, 77, 3, 900, 12, 1, 64, 255, 31, 8, 600, 2, 9, 14, 15, 16, 17, 300, 41, 42]
    pages = [3, 9]
    orc = LocalForwardPass(wref)
    want = orc.prefill(prompt)
    # chunk 1: 11 tokens; chunk 2: 9 tokens attending to the 11 cached ones
    r.forward(_prefill_meta(prompt[:11], 0, pages, 11))
    nxt = r.forward(_prefill_meta(prompt[11:], 11, pages, len(prompt)))
    assert _rel(r.last_logits[0].numpy(), want) < 3e-2
    assert int(nxt[0]) == int(np.argmax(r.last_logits[0].numpy()))
    tok = int(np.argmax(want))
    T = len(prompt)
    for step in range(3):
        p = T + step
        # batch of 2 slots: slot 0 is the session, slot 1 is padding (KV slot -1)
        bt = torch.zeros(2, 4, dtype=torch.int32)
        bt[0, :2] = torch.tensor(pages)
        m = StepMeta(ids=torch.tensor([tok, 0], dtype=torch.int32), pos=torch.tensor([p, 0], dtype=torch.int32),
                     slot=torch.tensor([pages[p // 16] * 16 + p % 16, -1], dtype=torch.int64), block_tables=bt,
                     seq_lens=torch.tensor([p + 1, 1], dtype=torch.int32), max_q_len=64, decode=True)
        r.forward(m)
        want = orc.decode_step(tok)
        assert _rel(r.last_logits[0].numpy(), want) < 3e-2, step
        tok = int(np.argmax(want))
