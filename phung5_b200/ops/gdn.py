"""Gated DeltaNet ops (csrc/gdn.cu) with their plain-torch definitions for CPU tensors.

Token batches are ragged: request r owns tokens [tok_start[r], tok_start[r+1]) and recurrent/conv state
slot slot[r]. See csrc/gdn.cu for the recurrence and the verify / fold split.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import ext, status_tensor  # noqa: F401


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """a, b [T, HV] -> g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b) (fp32)."""
    if a.is_cuda:
        g = torch.empty(a.shape, dtype=torch.float32, device=a.device)
        beta = torch.empty_like(g)
        ext().gdn_gates(a.contiguous(), b.contiguous(), A_log.float().contiguous(), dt_bias.float().contiguous(), g, beta)
        return g, beta
    x = a.float() + dt_bias.float()
    sp = torch.where(x > 20, x, torch.log1p(torch.exp(x)))
    return -torch.exp(A_log.float()) * sp, torch.sigmoid(b.float())


def gdn_recurrent(q, k, v, g, beta, state, tok_start, slot, scale: float, write_state: bool, stash: bool = True):
    """q, k [T, HK, 128]; v [T, HV, 128]; g, beta [T, HV]; state [slots, HV, 128, 128] fp32 (modified only
    when write_state). Returns (out [T, HV, 128], stash (k_hat, v', g) or None)."""
    t, hv = v.shape[0], v.shape[1]
    st = None
    if q.is_cuda:
        out = torch.empty(t, hv, 128, dtype=torch.bfloat16, device=q.device)
        if stash:
            st = (torch.empty(t, hv, 128, dtype=torch.float32, device=q.device),
                  torch.empty(t, hv, 128, dtype=torch.float32, device=q.device),
                  torch.empty(t, hv, dtype=torch.float32, device=q.device))
        ext().gdn_recurrent(q.contiguous(), k.contiguous(), v.contiguous(), g.contiguous(), beta.contiguous(), state,
                            tok_start, slot, scale, out, write_state, *(st if st else (None, None, None)))
        return out, st
    hk = q.shape[1]
    rep = hv // hk
    out = torch.empty(t, hv, 128, dtype=v.dtype)
    if stash:
        st = (torch.zeros(t, hv, 128), torch.zeros(t, hv, 128), torch.zeros(t, hv))
    ts = tok_start.tolist()
    for r in range(len(ts) - 1):
        S = state[int(slot[r])].clone()
        for i in range(ts[r], ts[r + 1]):
            qq = q[i].float().repeat_interleave(rep, 0)
            kk = k[i].float().repeat_interleave(rep, 0)
            qq = qq / torch.sqrt((qq * qq).sum(-1, keepdim=True) + 1e-6) * scale
            kk = kk / torch.sqrt((kk * kk).sum(-1, keepdim=True) + 1e-6)
            S = S * torch.exp(g[i].float())[:, None, None]
            vp = (v[i].float() - torch.einsum("hij,hi->hj", S, kk)) * beta[i].float()[:, None]
            S = S + kk[:, :, None] * vp[:, None, :]
            out[i] = torch.einsum("hij,hi->hj", S, qq).to(out.dtype)
            if stash:
                st[0][i], st[1][i], st[2][i] = kk, vp, g[i].float()
        if write_state:
            state[int(slot[r])] = S
    return out, st


def gdn_fold(state, tok_start, slot, n_accept, st) -> None:
    """Commit the first n_accept[r] stashed tokens of request r into its state."""
    if state.is_cuda:
        ext().gdn_fold(state, tok_start, slot, n_accept.to(torch.int32), *st)
        return
    ts = tok_start.tolist()
    for r in range(len(ts) - 1):
        S = state[int(slot[r])]
        for i in range(ts[r], ts[r] + int(n_accept[r])):
            S.mul_(torch.exp(st[2][i])[:, None, None]).add_(st[0][i][:, :, None] * st[1][i][:, None, :])


def causal_conv1d(x, window, w, bias, tok_start, slot, n_commit=None):
    """x [T, C]; window [slots, W-1, C] (updated with the first n_commit tokens of each request, all when
    None); w [C, W]. Returns silu(causal conv) [T, C]."""
    if x.is_cuda:
        y = torch.empty_like(x)
        ext().causal_conv1d(x.contiguous(), window, w.contiguous(), bias,
                            tok_start, slot, None if n_commit is None else n_commit.to(torch.int32), y)
        return y
    W = w.shape[1]
    y = torch.empty_like(x)
    ts = tok_start.tolist()
    for r in range(len(ts) - 1):
        a, b = ts[r], ts[r + 1]
        s = int(slot[r])
        seq = torch.cat([window[s].float(), x[a:b].float()], 0)          # [W-1 + n, C]
        for i in range(b - a):
            acc = (seq[i:i + W] * w.float().t()).sum(0)
            if bias is not None:
                acc = acc + bias.float()
            y[a + i] = F.silu(acc).to(y.dtype)
        n = (b - a) if n_commit is None else int(n_commit[r])
        window[s] = seq[n:n + W - 1].to(window.dtype)
    return y


def gated_rmsnorm(o, z, w, eps: float):
    """o, z [..., D] -> rmsnorm(o) * w * silu(z) over the last dim."""
    if o.is_cuda:
        y = torch.empty_like(o)
        ext().gated_rmsnorm(o.contiguous(), z.contiguous(), w.contiguous(), eps, y)
        return y
    of = o.float()
    return (of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * w.float() * F.silu(z.float())).to(o.dtype)
