"""Plain fp32 PyTorch versions of the kernels, used by tests as the numerical oracle."""
from __future__ import annotations

import math

import torch


def rmsnorm(x, gamma, eps):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()


def rope(x, pos, head_dim, base):
    """Half-split rotation on [T, heads*D]."""
    T = x.shape[0]
    half = head_dim // 2
    inv = 1.0 / (torch.tensor(base, dtype=torch.float64) ** (torch.arange(half, dtype=torch.float64) * 2.0 / head_dim))
    th = pos.double()[:, None].cpu() * inv[None, :]
    c, s = torch.cos(th).float().to(x.device), torch.sin(th).float().to(x.device)
    h = x.float().reshape(T, -1, head_dim)
    l, r = h[..., :half], h[..., half:]
    return torch.cat([l * c[:, None] - r * s[:, None], l * s[:, None] + r * c[:, None]], -1).reshape(T, -1)


def attention(q, k, v, q_pos, k_pos, scale, window=0):
    """q [Tq, Hq, D], k/v [Tk, Hkv, D], causal on absolute positions, GQA by head // group."""
    Hq, Hkv = q.shape[1], k.shape[1]
    g = Hq // Hkv
    kk = k.float().repeat_interleave(g, 1)
    vv = v.float().repeat_interleave(g, 1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk) * scale
    mask = k_pos[None, :] <= q_pos[:, None]
    if window > 0:
        mask &= k_pos[None, :] > (q_pos[:, None] - window)
    s = s.masked_fill(~mask[None], float("-inf"))
    p = torch.softmax(s, -1)
    p = torch.nan_to_num(p)
    return torch.einsum("hqk,khd->qhd", p, vv)


def silu_mul_interleaved(y, block=64):
    """y [T, 2*I] with gate/up interleaved in blocks of `block` -> silu(g)*u [T, I]."""
    T, two_i = y.shape
    x = y.float().reshape(T, two_i // (2 * block), 2, block)
    g, u = x[:, :, 0], x[:, :, 1]
    return (torch.nn.functional.silu(g) * u).reshape(T, -1)
