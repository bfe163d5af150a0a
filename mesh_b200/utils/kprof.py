"""Profiling driver: runs eager decode steps (no CUDA graphs) of a model so that a profiler sees
one launch per kernel.

    python -m mesh_b200.utils.kprof --model llama3-8b --batch 64 --ctx 576 --steps 2 [--layers L]
"""
from __future__ import annotations

import argparse

import torch

from ..config import EngineConfig, get_preset
from ..models.llama import KVPool, LlamaRunner, StepMeta
from ..models.weights import synthetic_device_weights


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=576)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--prefill", type=int, default=0, help="run a prefill of this many tokens per step instead")
    a = ap.parse_args()
    cfg = get_preset(a.model)
    if a.layers:
        cfg = cfg.replace(num_layers=a.layers)
    dev = torch.device("cuda", 0)
    w = synthetic_device_weights(cfg, 0, 1, device=dev)
    B, ps = a.batch, 16
    ppseq = (a.ctx + ps) // ps + 1
    kv = KVPool(cfg, w.layout.local_kv_heads, B * ppseq + 1, ps, dev)
    ecfg = EngineConfig(max_seq_len=ppseq * ps)
    T = a.prefill or B
    runner = LlamaRunner(w, ecfg, kv, dev, max_tokens=max(T, B))
    bt = (torch.arange(B * ppseq, device=dev, dtype=torch.int32) + 1).view(B, ppseq)
    if a.prefill:
        P = 512
        S = T // P
        m = StepMeta(ids=torch.randint(0, cfg.vocab_size, (T,), device=dev, dtype=torch.int32),
                     pos=torch.arange(P, device=dev, dtype=torch.int32).repeat(S),
                     slot=(bt[:S, :P // ps].long().repeat_interleave(ps, 1) * ps +
                           torch.arange(P, device=dev) % ps).reshape(-1),
                     block_tables=bt[:S], seq_lens=torch.full((S,), P, device=dev, dtype=torch.int32),
                     cu_q=torch.arange(S + 1, device=dev, dtype=torch.int32) * P,
                     last_idx=torch.arange(S, device=dev) * P + P - 1, max_q_len=P, decode=False)
    else:
        m = StepMeta(ids=torch.randint(0, cfg.vocab_size, (B,), device=dev, dtype=torch.int32),
                     pos=torch.full((B,), a.ctx - 1, device=dev, dtype=torch.int32),
                     slot=(bt[:, (a.ctx - 1) // ps].long() * ps + (a.ctx - 1) % ps),
                     block_tables=bt, seq_lens=torch.full((B,), a.ctx, device=dev, dtype=torch.int32),
                     max_q_len=ppseq * ps, decode=True)
    for _ in range(a.steps):
        runner.forward(m)
    torch.cuda.synchronize()
    print("kprof done")


if __name__ == "__main__":
    main()
