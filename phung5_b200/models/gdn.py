"""Gated DeltaNet layer of hybrid models (Qwen3-Next-style linear attention), on csrc/gdn.cu.

    x -> in_proj -> [q | k | v | z],  [b | a]
    [q | k | v] -> causal depthwise conv (W taps) + SiLU          (window per request slot)
    g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
    o = gated delta rule over the request's tokens               (state [HV, 128, 128] per slot)
    y = out_proj(rmsnorm(o) * w * silu(z))

Speculative verification (the reference's DFlash verify on its GDN layers) runs the
draft window from the committed state without modifying it (`mode="verify"`), keeping a stash; after
acceptance `commit(n_accept)` folds the accepted prefix into the state and advances the conv window —
the reference's braw verify + fold (docker/opt/kern/braw/kernels.py) and its conv-window commit.
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field
from typing import Optional

import torch

from ..ops import gdn as G
from .llama import Linear


@dataclass
class GDNLayer:
    w_in: Linear          # [2*HK*128 + 2*HV*128, H]  (q, k, v, z)
    w_ba: torch.Tensor    # [2*HV, H]                 (b, a)
    conv_w: torch.Tensor  # [C, W], C = 2*HK*128 + HV*128
    A_log: torch.Tensor   # [HV] fp32
    dt_bias: torch.Tensor  # [HV] fp32
    norm_w: torch.Tensor  # [128]
    w_out: Linear         # [H, HV*128]
    hk: int
    hv: int
    eps: float = 1e-6
    _stash: Optional[tuple] = field(default=None, repr=False)

    @property
    def conv_channels(self) -> int:
        return (2 * self.hk + self.hv) * 128

    def forward(self, x, tok_start: torch.Tensor, slot: torch.Tensor, window: torch.Tensor, state: torch.Tensor,
                mode: str = "prefill") -> torch.Tensor:
        """x [T, H] (bf16 / fp32 on CPU). mode "prefill" advances state and window over all tokens;
        mode "verify" leaves them unchanged and keeps what `commit` needs."""
        t = x.shape[0]
        C = self.conv_channels
        proj = x.float() @ self.w_in.w.float().t() if not x.is_cuda else self.w_in(x)
        ba = x.float() @ self.w_ba.float().t() if not x.is_cuda else (x @ self.w_ba.t())
        qkv, z = proj[:, :C].contiguous(), proj[:, C:].contiguous()
        b, a = ba[:, : self.hv].contiguous(), ba[:, self.hv:].contiguous()
        verify = mode == "verify"
        n_commit = torch.zeros(slot.shape[0], dtype=torch.int32, device=x.device) if verify else None
        conv = G.causal_conv1d(qkv.to(x.dtype), window, self.conv_w, None, tok_start, slot, n_commit)
        q = conv[:, : self.hk * 128].reshape(t, self.hk, 128)
        k = conv[:, self.hk * 128: 2 * self.hk * 128].reshape(t, self.hk, 128)
        v = conv[:, 2 * self.hk * 128:].reshape(t, self.hv, 128)
        g, beta = G.gdn_gates(a.to(x.dtype), b.to(x.dtype), self.A_log, self.dt_bias)
        o, st = G.gdn_recurrent(q, k, v, g, beta, state, tok_start, slot, 1.0 / math.sqrt(128),
                                write_state=not verify, stash=verify)
        if verify:
            self._stash = (st, qkv.to(x.dtype), tok_start, slot)
        y = G.gated_rmsnorm(o, z.reshape(t, self.hv, 128).to(o.dtype), self.norm_w, self.eps).reshape(t, -1)
        return y.float() @ self.w_out.w.float().t() if not x.is_cuda else self.w_out(y)

    def commit(self, n_accept: torch.Tensor, window: torch.Tensor, state: torch.Tensor) -> None:
        """Fold the first n_accept[r] verified tokens of every request into its state and conv window."""
        st, qkv, tok_start, slot = self._stash
        G.gdn_fold(state, tok_start, slot, n_accept, st)
        G.causal_conv1d(qkv, window, self.conv_w, None, tok_start, slot, n_accept.to(torch.int32))
        self._stash = None


def random_gdn_layer(hidden: int, hk: int, hv: int, device, seed: int = 0, conv_w: int = 4, std: float = 0.02,
                     dtype=torch.bfloat16) -> GDNLayer:
    g = torch.Generator().manual_seed(zlib.crc32(repr(("gdn", seed)).encode()))
    C = (2 * hk + hv) * 128

    def r(*shape, s=std):
        return (torch.randn(*shape, generator=g) * s).to(device=device, dtype=dtype)

    return GDNLayer(w_in=Linear(r(C + hv * 128, hidden)), w_ba=r(2 * hv, hidden),
                    conv_w=r(C, conv_w, s=0.3), A_log=torch.log(torch.rand(hv, generator=g) * 15 + 1).to(device),
                    dt_bias=(torch.rand(hv, generator=g) * 0.5).to(device), norm_w=torch.ones(128, device=device, dtype=dtype),
                    w_out=Linear(r(hidden, hv * 128)), hk=hk, hv=hv)
