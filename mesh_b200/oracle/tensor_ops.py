"""Host fp32 math with the reference's exact semantics (numpy).

Each function restates one routine of ``agent/src/inference/tensor_ops.rs``:
matmul ``:219``, gelu ``:248``, silu ``:268``, rms_norm ``:285``, layer_norm ``:309``,
softmax ``:350``, the splitmix-style sampling threshold ``:372-385``, sample_token ``:394-458``,
sample_greedy ``:461``, embed_tokens ``:482``, apply_rope (half-split rotation) ``:509-560``.
``sample_tokens_device_semantics`` restates the batched device sampler of ``runtime.rs:534-601``
(cdf crossing with ``>=``; top-p keep-mask ``cumsum - p < top_p``).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
_MASK64 = (1 << 64) - 1


def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"Matmul shape mismatch: {a.shape[0]}x{a.shape[1]} @ {b.shape[0]}x{b.shape[1]}")
    return (a.astype(F32) @ b.astype(F32)).astype(F32)


def gelu(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32)
    c = F32(np.sqrt(2.0 / np.pi))
    return (F32(0.5) * x * (F32(1.0) + np.tanh(c * (x + F32(0.044715) * x * x * x)))).astype(F32)


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def rms_norm(x: np.ndarray, gamma: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(F32)
    if x.shape[-1] != gamma.shape[0]:
        raise ValueError(f"RMS norm dimension mismatch: tensor cols {x.shape[-1]} vs gamma {gamma.shape[0]}")
    ms = (x * x).sum(-1, keepdims=True, dtype=F32) / F32(x.shape[-1])
    inv = F32(1.0) / np.sqrt(ms + F32(eps))
    return (x * inv * gamma.astype(F32)).astype(F32)


def layer_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(F32)
    mean = x.mean(-1, keepdims=True, dtype=F32)
    var = ((x - mean) ** 2).mean(-1, keepdims=True, dtype=F32)
    return (((x - mean) / np.sqrt(var + F32(eps))) * gamma + beta).astype(F32)


def softmax(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32)
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(-1, keepdims=True, dtype=F32)).astype(F32)


def deterministic_sample_threshold(seed: int) -> float:
    """64-bit splitmix finaliser of ``seed``; the top 24 bits become a uniform in [0, 1)."""
    x = (seed + 0x9E3779B97F4A7C15) & _MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _MASK64
    x ^= x >> 31
    upper = x >> 40
    t = upper / float(1 << 24)
    t = min(max(t, 0.0), 1.0 - np.finfo(np.float64).eps)
    return float(F32(t))


def sample_greedy(logits: np.ndarray) -> int:
    # first index of the maximum (strict '>' scan)
    return int(np.argmax(logits.astype(F32)))


def sample_token(logits: np.ndarray, temperature: float, top_p: float, rng_seed: int) -> int:
    """Host sampler: temperature, softmax, descending sort, nucleus cut, threshold walk."""
    x = logits.astype(F32)
    if temperature != 1.0 and temperature > 0.0:
        x = (x / F32(temperature)).astype(F32)
    m = x.max()
    e = np.exp(x - m).astype(F32)
    s = F32(0.0)
    for v in e:  # sequential f32 sum as the reference does
        s = F32(s + v)
    probs = (e / s).astype(F32)
    order = np.argsort(-probs, kind="stable")
    cutoff = len(order)
    c = F32(0.0)
    for i, idx in enumerate(order):
        c = F32(c + probs[idx])
        if c >= F32(top_p):
            cutoff = i + 1
            break
    r = F32(deterministic_sample_threshold(rng_seed))
    if top_p >= 1.0:
        c = F32(0.0)
        for idx, p in enumerate(probs):
            c = F32(c + p)
            if r < c:
                return idx
        return int(order[0])
    sel = order[:cutoff]
    ssum = F32(0.0)
    for idx in sel:
        ssum = F32(ssum + probs[idx])
    c = F32(0.0)
    for idx in sel:
        c = F32(c + F32(probs[idx] / ssum))
        if r < c:
            return int(idx)
    return int(order[0])


def sample_tokens_device_semantics(logits: np.ndarray, temperature: float, top_p: float, seeds) -> list:
    """Batched sampler with the device path's rules (greedy when temperature<=0 or top_p<=0)."""
    logits = np.atleast_2d(logits).astype(F32)
    if len(seeds) != logits.shape[0]:
        raise ValueError(f"Device sampling received {logits.shape[0]} rows but {len(seeds)} seeds")
    if temperature <= 0.0 or top_p <= 0.0:
        return [int(np.argmax(r)) for r in logits]
    out = []
    for row, seed in zip(logits, seeds):
        x = row if temperature == 1.0 else (row * F32(1.0 / temperature)).astype(F32)
        p = softmax(x[None])[0]
        thr = F32(deterministic_sample_threshold(seed))
        if top_p >= 1.0:
            cdf = np.cumsum(p, dtype=F32)
            hit = np.nonzero(cdf >= thr)[0]
            out.append(int(hit[0]) if len(hit) else 0)
            continue
        order = np.argsort(-p, kind="stable")
        sp = p[order]
        keep = (np.cumsum(sp, dtype=F32) - sp) < F32(top_p)
        f = np.where(keep, sp, F32(0.0)).astype(F32)
        f = (f * (F32(1.0) / f.sum(dtype=F32))).astype(F32)
        cdf = np.cumsum(f, dtype=F32)
        hit = np.nonzero(cdf >= thr)[0]
        out.append(int(order[hit[0] if len(hit) else 0]))
    return out


def embed_tokens(table: np.ndarray, tokens) -> np.ndarray:
    tokens = np.asarray(tokens, dtype=np.int64)
    if tokens.size and (tokens.max() >= table.shape[0] or tokens.min() < 0):
        bad = int(tokens[(tokens >= table.shape[0]) | (tokens < 0)][0])
        raise ValueError(f"Token {bad} out of vocabulary bounds {table.shape[0]}")
    return table[tokens].astype(F32)


def rope_inv_freq(head_dim: int, base: float) -> np.ndarray:
    half = head_dim // 2
    return np.array([1.0 / (F32(base) ** (F32(i) * F32(2.0) / F32(head_dim))) for i in range(half)], dtype=F32)


def apply_rope(x: np.ndarray, positions, head_dim: int, base: float) -> np.ndarray:
    """Half-split rotation: pairs (d, d + head_dim/2) of each head rotate by position*inv_freq[d]."""
    x = x.astype(F32)
    positions = np.asarray(positions)
    if x.shape[0] != len(positions):
        raise ValueError(f"RoPE position count {len(positions)} doesn't match sequence length {x.shape[0]}")
    if head_dim % 2:
        raise ValueError(f"RoPE requires even head_dim, got {head_dim}")
    if x.shape[1] % head_dim:
        raise ValueError(f"RoPE head_dim {head_dim} does not divide tensor width {x.shape[1]}")
    half = head_dim // 2
    inv = rope_inv_freq(head_dim, base)
    theta = positions.astype(F32)[:, None] * inv[None, :]
    cos, sin = np.cos(theta).astype(F32), np.sin(theta).astype(F32)
    h = x.reshape(x.shape[0], -1, head_dim)
    left, right = h[..., :half], h[..., half:]
    out = np.concatenate([left * cos[:, None] - right * sin[:, None], left * sin[:, None] + right * cos[:, None]], -1)
    return out.reshape(x.shape).astype(F32)
