"""Block-scaled FP8 (e4m3) quantization, the checkpoint format of block-scaled FP8 Llama-3-70B.

Weights: one fp32 scale per 128x128 block, stored HF-style as ``<name>_scale_inv`` [ceil(N/128),
ceil(K/128)] so that ``w_fp32 ~= w_fp8 * scale_inv`` (the DeepSeek/Qwen FP8 checkpoint layout).
Activations: one fp32 scale per token per 128 channels, computed at run time by the fused norm /
SwiGLU kernels; this module holds the torch definition those kernels are tested against.

The scale is the smallest power of two >= amax / 448 (448 = largest finite e4m3 value). The reference's
per-token quant uses amax / 448 itself (docker/opt/v5/fusedq/silu_quant.cuh:28-79); rounding it up to a
power of two makes every scale exactly representable as UE8M0, the scale format the Blackwell tensor core
applies in hardware (tcgen05 kind::mxf8f6f4 block scaling), so the GEMM needs no scale arithmetic of its
own. The e4m3 relative precision is unchanged (only the top binade of the range may go unused). A zero
block gets scale 1 so that it quantizes to exact zeros. Checkpoints whose scales are not powers of two are
requantized once at load (`ensure_pow2`).
"""
from __future__ import annotations

from typing import Tuple

import torch

FP8_MAX = 448.0
FP8_DTYPE = torch.float8_e4m3fn
BLOCK = 128


def pow2_scale(amax: torch.Tensor) -> torch.Tensor:
    """Smallest power of two >= amax / 448 (1 where amax == 0), fp32; exact (frexp / ldexp)."""
    f = amax.float() / FP8_MAX
    mant, exp = torch.frexp(f)                      # f = mant * 2^exp, mant in [0.5, 1)
    exp = exp - (mant == 0.5).to(exp.dtype)         # an exact power of two keeps its exponent
    s = torch.ldexp(torch.ones_like(f), exp)
    return torch.where(amax > 0, s, torch.ones_like(f))


def is_pow2(s: torch.Tensor) -> bool:
    """True when every scale is a positive normal power of two (UE8M0-representable)."""
    mant, _ = torch.frexp(s.float())
    return bool(((mant == 0.5) & (s > 0)).all())


def quant_weight_block(w: torch.Tensor, block: int = BLOCK) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32/bf16 [N, K] -> (fp8 [N, K], fp32 scale_inv [ceil(N/b), ceil(K/b)])."""
    n, k = w.shape
    nb, kb = (n + block - 1) // block, (k + block - 1) // block
    wp = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    wp[:n, :k] = w.float()
    blocks = wp.view(nb, block, kb, block)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = pow2_scale(amax)
    q = (blocks / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(FP8_DTYPE)
    return q.view(nb * block, kb * block)[:n, :k].contiguous(), scale


def ensure_pow2(wq: torch.Tensor, ws: torch.Tensor, block: int = BLOCK) -> Tuple[torch.Tensor, torch.Tensor]:
    """(fp8 [N, K], scale_inv) with arbitrary fp32 block scales -> the same weight with power-of-two scales
    (dequantize, requantize; one extra e4m3 rounding). Unchanged when the scales already are powers of two."""
    if is_pow2(ws):
        return wq, ws.float()
    n, k = wq.shape
    s = ws.float().repeat_interleave(block, 0)[:n].repeat_interleave(block, 1)[:, :k]
    return quant_weight_block(wq.float() * s, block)


def quant_act_block(x: torch.Tensor, block: int = BLOCK) -> Tuple[torch.Tensor, torch.Tensor]:
    """[M, K] -> (fp8 [M, K], fp32 scales [K/128, M]) — the scale tensor is stored k-block major
    (M contiguous) so that a GEMM tile reads one contiguous run of M scales per K block."""
    m, k = x.shape
    assert k % block == 0, "activation width must be a multiple of 128"
    xb = x.float().view(m, k // block, block)
    amax = xb.abs().amax(-1)
    scale = pow2_scale(amax)
    q = (xb / scale[..., None]).clamp(-FP8_MAX, FP8_MAX).to(FP8_DTYPE).view(m, k)
    return q, scale.t().contiguous()


def dequant_act_block(q: torch.Tensor, s: torch.Tensor, block: int = BLOCK) -> torch.Tensor:
    m, k = q.shape
    return (q.float().view(m, k // block, block) * s.t()[..., None]).view(m, k)


def gemm_fp8_block_ref(xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                       block: int = BLOCK) -> torch.Tensor:
    """fp32 oracle of the block-scaled GEMM: out[m, n] = sum_kb xs[kb, m] * ws[n/128, kb] *
    sum_{k in kb} xq[m, k] * wq[n, k]. Returns fp32 [M, N]."""
    m, k = xq.shape
    n = wq.shape[0]
    kb = k // block
    out = torch.zeros(m, n, dtype=torch.float32, device=xq.device)
    xf, wf = xq.float(), wq.float()
    wsn = ws.float().repeat_interleave(block, 0)[:n]  # [N, KB]
    for b in range(kb):
        sl = slice(b * block, (b + 1) * block)
        part = xf[:, sl] @ wf[:, sl].t()
        out += part * xs[b].float()[:, None] * wsn[:, b][None, :]
    return out
