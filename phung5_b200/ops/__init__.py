"""Python entry points of the sm_100a kernels.

Every op runs its native kernel when given CUDA tensors; if the extension is missing on a CUDA
tensor the op raises (there is no silent eager fallback on the GPU). CPU tensors run the plain-torch
definition of the op, which is also the oracle the GPU tests compare against and what the CPU test
suite exercises (engine logic, multi-rank gloo runs).

Kernel status: kernels with bounded waits write a nonzero code into a per-device int32 status word
instead of hanging; `check_status()` raises if any kernel reported a timeout.
"""
from __future__ import annotations

import math
import os
from typing import Optional, Tuple

import torch

from ..weights.quant import FP8_DTYPE, dequant_act_block, gemm_fp8_block_ref, quant_act_block
from . import check as _check

try:  # the in-tree extension (python setup.py build_ext --inplace)
    from .. import _C  # type: ignore
    _C_ERR: Optional[BaseException] = None
except ImportError as e:  # pragma: no cover - depends on the build
    _C = None
    _C_ERR = e

_STATUS = {}

STATUS_CODES = {1: "timeout in TMA producer", 2: "timeout in MMA issuer", 3: "timeout in epilogue",
                4: "timeout waiting for a peer rank", 5: "bad arguments",
                6: "fp8 block scale is not a power of two (hardware-scaled GEMM)",
                7: "timeout in a split-K GEMM part waiting for the other parts of its tile"}


_LAUNCHES = [0]


def launches() -> int:
    """Number of native kernel launches issued through this module so far (all devices)."""
    return _LAUNCHES[0]


def ext():
    _LAUNCHES[0] += 1
    if _C is None:
        raise RuntimeError(f"phung5_b200._C is not built (python setup.py build_ext --inplace): {_C_ERR}")
    return _TIMED if OP_TIMING else _C


# ------------------------------------------------------------------------------------------------
# Per-kernel-class device timing (PHX_OP_TIMING=1, eager steps only: a graph replay issues no ext() call).
# Every native launch is bracketed by two CUDA events on the launching stream and filed under
# (phase, binding name); `set_phase` marks engine phase boundaries with an event as well, so a phase's
# device time minus its native kernels' time is the time of torch glue kernels and idle gaps.
# ------------------------------------------------------------------------------------------------

OP_TIMING = os.environ.get("PHX_OP_TIMING", "0") == "1"
_TIMING_LOG: list = []          # (phase, name, start event, end event)
_PHASE_LOG: list = []           # (phase, event at its start)
_PHASE = ["-"]


class _TimedExt:
    def __getattr__(self, name):
        fn = getattr(_C, name)

        def call(*args, **kw):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            r = fn(*args, **kw)
            b.record()
            _TIMING_LOG.append((_PHASE[0], name, a, b))
            return r
        return call


_TIMED = _TimedExt()


def set_phase(name: str) -> None:
    if not OP_TIMING or not torch.cuda.is_available():
        return
    _PHASE[0] = name
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    _PHASE_LOG.append((name, e))


def timing_reset() -> None:
    _TIMING_LOG.clear()
    _PHASE_LOG.clear()


def timing_report() -> dict:
    """{"kernels": {"phase/name": [ms, launches]}, "phases": {phase: ms}} since the last reset (synchronizes)."""
    torch.cuda.synchronize()
    kern: dict = {}
    for ph, name, a, b in _TIMING_LOG:
        k = f"{ph}/{name}"
        ms, n = kern.get(k, (0.0, 0))
        kern[k] = (ms + a.elapsed_time(b), n + 1)
    phases: dict = {}
    for (ph, a), (_, b) in zip(_PHASE_LOG, _PHASE_LOG[1:]):
        phases[ph] = phases.get(ph, 0.0) + a.elapsed_time(b)
    return {"kernels": {k: [round(v[0], 4), v[1]] for k, v in kern.items()},
            "phases": {k: round(v, 4) for k, v in phases.items()}}


def native_available() -> bool:
    return _C is not None


def status_tensor(device) -> torch.Tensor:
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=f"cuda:{idx}")
        _STATUS[idx] = t
    return t


def check_status(device=None) -> None:
    """Raise if a kernel on `device` recorded an error; clears the status word."""
    if not torch.cuda.is_available():
        return
    devs = [torch.device(device)] if device is not None else [torch.device("cuda", i) for i in _STATUS]
    for d in devs:
        t = status_tensor(d)
        v = int(t[0].item())
        if v:
            t.zero_()
            raise RuntimeError(f"kernel status on {d}: {STATUS_CODES.get(v, v)}")


# ------------------------------------------------------------------------------------------------
# GEMMs
# ------------------------------------------------------------------------------------------------

# The tensor core applies the block scales itself (tcgen05 kind::mxf8f6f4, UE8M0 scales): every scale the
# framework produces is a power of two. PHX_FP8_PROMOTE=1 selects the software per-K-block promotion instead
# (any fp32 scales).
FP8_HW_SCALE = os.environ.get("PHX_FP8_PROMOTE", "0") != "1"
# The gate/up projection runs SwiGLU + FP8 quant in its GEMM epilogue (PHX_SWIGLU_FUSED=0: GEMM, then
# silu_mul_quant). Measured 1.877 -> 1.630 ms at 4096 x 57344 x 8192, 0.314 -> 0.280 ms at the TP8 shape.
SWIGLU_FUSED = os.environ.get("PHX_SWIGLU_FUSED", "1") != "0"
# PHX_GEMM_PAIR=1: hardware-scaled 256-wide tiles run as 256 x 256 tiles on CTA pairs (tcgen05 cta_group::2,
# clusters of two). Off by default: measured no faster than the single-CTA tile under the power cap.
GEMM_PAIR = os.environ.get("PHX_GEMM_PAIR", "0") == "1"
# Plain GEMMs whose last wave of tiles leaves most SMs idle split those tiles over K (csrc/gemm_sm100.cu,
# SplitArgs); PHX_GEMM_SPLIT=0 keeps every tile whole unless a caller asks for a split.
GEMM_SPLIT = os.environ.get("PHX_GEMM_SPLIT", "1") != "0"
# The scatter epilogue (row-parallel projections under tensor parallelism) hands each staged output row to the
# TMA engine as one bulk copy into its owner's receive slot; PHX_SCATTER_BULK=0 stores the rows with
# row-contiguous 16-byte lane stores instead.
SCATTER_BULK = os.environ.get("PHX_SCATTER_BULK", "1") != "0"


def _table_choice(kind: str, n: int, k: int, m: int, bn: int, hw_scale, pair, use_table: bool, split=None):
    """The measured per-shape configuration (ops/gemm_table.json) unless the caller chose one. Returns
    (bn, hws, pair, split); split 0 = the kernel's automatic split-K tail, 1 = off."""
    auto = 0 if GEMM_SPLIT else 1
    if not use_table or bn or hw_scale is not None or pair is not None or split is not None:
        return bn, hw_scale, pair, (auto if split is None else split)
    from . import gemm_table
    e = gemm_table.lookup(kind, n, k, m)
    if e is None:
        return bn, hw_scale, pair, auto
    hws = e.get("hws")
    if hws is not None and not FP8_HW_SCALE:
        hws = False            # arbitrary-scale mode: never hand scales to the hardware path
    return int(e["bn"]), hws, e.get("pair"), int(e.get("split", auto))


def gemm_fp8_block(xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                   out: Optional[torch.Tensor] = None, bn: int = 0, max_ctas: int = 0,
                   hw_scale: Optional[bool] = None, pair: Optional[bool] = None, use_table: bool = True,
                   split: Optional[int] = None) -> torch.Tensor:
    """Block-scaled FP8 linear: xq [M,K] e4m3, xs [K/128, M] fp32, wq [N,K] e4m3, ws [N/128, K/128]
    fp32 -> bf16 [M, N]. hw_scale (default FP8_HW_SCALE) needs power-of-two scales. Unless bn / hw_scale / pair
    / split are given, the measured per-shape table (ops/gemm_table.py) picks them. split: parts of the split-K
    tail of grids whose last wave is mostly idle (0 automatic, 1 off, >= 2 that many)."""
    m, n = xq.shape[0], wq.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=xq.device)
    if xq.is_cuda:
        bn, hw_scale, pair, split = _table_choice("fp8", n, xq.shape[1], m, bn, hw_scale, pair, use_table, split)
        hws = FP8_HW_SCALE if hw_scale is None else hw_scale
        if _check.active():
            _check.gemm_fp8_block(xq, xs, wq, ws, out, hws)
        ext().gemm_fp8_block(xq, xs, wq, ws, out, status_tensor(xq.device), bn, max_ctas, hws,
                             GEMM_PAIR if pair is None else pair, split)
    else:
        if _check.active():
            _check.gemm_fp8_block(xq, xs, wq, ws, out, False)
        out.copy_(gemm_fp8_block_ref(xq, xs, wq, ws).to(out.dtype))
    return out


def gemm_bf16(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None, bn: int = 0,
              max_ctas: int = 0, use_table: bool = True, split: Optional[int] = None) -> torch.Tensor:
    """x [M,K] bf16 @ w [N,K]^T -> bf16 [M,N] (fp32 accumulate); split as for gemm_fp8_block."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=torch.bfloat16 if x.is_cuda else x.dtype, device=x.device)
    if _check.active():
        _check.gemm_bf16(x, w, out)
    if x.is_cuda:
        bn, _, _, split = _table_choice("bf16", w.shape[0], x.shape[1], x.shape[0], bn, None, None, use_table, split)
        ext().gemm_bf16(x, w, out, status_tensor(x.device), bn, max_ctas, split)
    else:
        out.copy_((x.float() @ w.float().t()).to(out.dtype))
    return out


def gemm_grouped(x, w: torch.Tensor, ws: Optional[torch.Tensor], offsets: torch.Tensor, n: int,
                 out: Optional[torch.Tensor] = None, rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Grouped linear for MoE experts. x = (xq, xs) block-scaled fp8 or a bf16 tensor, rows sorted by group;
    group e owns rows [offsets[e], offsets[e+1]) (int32 device tensor, no host sync) and weight rows
    [e*n, (e+1)*n) of w (ws: fp8 block scales [G*ceil(n/128), K/128]). Rows past offsets[-1] are not
    written. rows (int32 [M], fp8 only): GEMM row r is activation row rows[r], so the expert dispatch (the
    token gather) happens inside the GEMM's A loads (TMA gather4) instead of as a separate copy."""
    xq = x[0] if isinstance(x, tuple) else x
    if rows is not None and not (xq.is_cuda and ws is not None and FP8_HW_SCALE):
        x = (x[0][rows.long()], x[1][:, rows.long()].contiguous()) if ws is not None else x[rows.long()]
        xq, rows = (x[0] if isinstance(x, tuple) else x), None
    m = xq.shape[0] if rows is None else rows.shape[0]
    if _check.active():
        _check.gemm_grouped(xq.shape[0], w, n, offsets, rows)
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16 if xq.is_cuda else (torch.float32 if ws is not None else xq.dtype),
                          device=xq.device)
    if xq.is_cuda:
        if ws is not None:
            ext().gemm_fp8_grouped(x[0], x[1], w, ws, offsets, out, status_tensor(xq.device), FP8_HW_SCALE,
                                   None if rows is None else rows.int().contiguous())
        else:
            ext().gemm_bf16_grouped(x, w, offsets, out, status_tensor(xq.device))
        return out
    off = offsets.tolist()
    nb = (n + 127) // 128
    for e in range(len(off) - 1):
        a, b = off[e], off[e + 1]
        if b <= a:
            continue
        if ws is not None:
            out[a:b] = gemm_fp8_block_ref(x[0][a:b], x[1][:, a:b], w[e * n:(e + 1) * n], ws[e * nb:(e + 1) * nb]).to(out.dtype)
        else:
            out[a:b] = (x[a:b].float() @ w[e * n:(e + 1) * n].float().t()).to(out.dtype)
    return out


# ------------------------------------------------------------------------------------------------
# sampling
# ------------------------------------------------------------------------------------------------

def gemm_fp8_swiglu(xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor):
    """Gate/up projection with the SwiGLU + FP8 quant epilogue. wq [2F, K] / ws [2F/128, K/128] hold the gate
    and up weights interleaved in 128-row blocks (models.llama.interleave_gate_up). -> (q [M, F] e4m3,
    scales [F/128, M]), equal to silu_mul_quant of the plain gate/up GEMM's bf16 output."""
    m, f = xq.shape[0], wq.shape[0] // 2
    q = torch.empty(m, f, dtype=FP8_DTYPE, device=xq.device)
    s = torch.empty(f // 128, m, dtype=torch.float32, device=xq.device)
    ext().gemm_fp8_swiglu(xq, xs, wq, ws, q, s, status_tensor(xq.device))
    return q, s


def moe_combine(y: torch.Tensor, pos: torch.Tensor, w: torch.Tensor, local: torch.Tensor,
                out: torch.Tensor) -> torch.Tensor:
    """out[t] = sum_j local[t, j] * w[t, j] * y[pos[t, j]] (bf16, fp32 accumulate): the MoE combine of the
    expert rows (grouped-GEMM order) back to tokens; `out` may be a strided view (a reduction's buffer)."""
    if _check.active():
        _check.moe_combine(y, pos, w, local, out)
    if y.is_cuda:
        ext().moe_combine(y, pos, w, local, out)
        return out
    g = y[torch.where(local.bool(), pos, torch.zeros_like(pos)).clamp(min=0)].float()   # non-local pos unread
    out.copy_(torch.where(local[..., None], g * w[..., None], torch.zeros(())).sum(1).to(out.dtype))
    return out


def topk_logprobs(logits: torch.Tensor, k: int, temperature: float = 1.0, vocab_offset: int = 0,
                  with_lse: bool = True):
    """Fused top-k of log-softmax(logits / T) per row: returns (logprobs [R, k] fp32, indices [R, k] int64
    (+ vocab_offset), logsumexp [R] fp32). On a vocab shard the results are shard-local (the lse of the
    shard), which a tensor-parallel merge combines. with_lse=False (argmax use) skips the normalisation:
    the values are x / T and lse is 0."""
    r = logits.shape[0]
    if _check.active():
        _check.topk_logprobs(logits, k, temperature)
    if logits.is_cuda:
        lp = torch.empty(r, k, dtype=torch.float32, device=logits.device)
        idx = torch.empty(r, k, dtype=torch.int64, device=logits.device)
        if with_lse:
            lse = torch.empty(r, dtype=torch.float32, device=logits.device)
        ext().topk_logprobs(logits.contiguous() if logits.stride(-1) != 1 else logits, k, temperature, lp, idx,
                            lse if with_lse else None, vocab_offset)
        return lp, idx, (lse if with_lse else torch.zeros(r, dtype=torch.float32, device=logits.device))
    x = logits.float() / temperature
    lse = torch.logsumexp(x, -1) if with_lse else torch.zeros(r, dtype=torch.float32)
    v, i = torch.topk(x, k, dim=-1)
    return v - lse[:, None], i + vocab_offset, lse


SAMPLE_MAX_TOPK = 64
# PHX_DEVICE_SAMPLING=0 sends every sampled request to the dense torch definition (engine/sampling.py)
DEVICE_SAMPLING = os.environ.get("PHX_DEVICE_SAMPLING", "1") != "0"


def sample_kc(top_ks, temps) -> int:
    """Candidates per vocab chunk for the device sampling path: 16 if every sampled request keeps at most 16
    tokens, else 64 (greedy rows need 1)."""
    ks = [k for k, t in zip(top_ks, temps) if t > 0]
    return 16 if all(1 <= k <= 16 for k in ks) else 64


def device_sampling_ok(top_ks, temps) -> bool:
    """The device path serves greedy rows and rows with 1 <= top_k <= 64 (no host synchronisation); other rows
    (no top-k cut, or a larger one) take the dense torch definition."""
    return DEVICE_SAMPLING and all(t <= 0 or 1 <= k <= SAMPLE_MAX_TOPK for k, t in zip(top_ks, temps))


def spec_sample_accept(logits: torch.Tensor, tokens: torch.Tensor, parent: torch.Tensor, temp: torch.Tensor,
                       top_k: torch.Tensor, top_p: torch.Tensor, seed: torch.Tensor, committed: torch.Tensor,
                       depth: int, kc: int, vocab_offset: int = 0, gather=None):
    """Seeded target-only tree acceptance on the device (csrc/sample.cu). logits [R*N, V_local] bf16 verify rows
    of this rank's vocab shard (request r's node j at row r*N + j), tokens/parent [R, N] int64, per-request
    temp/top_p fp32, top_k int32, seed/committed int64. `gather(parts)` exchanges the shard candidates across
    tensor-parallel ranks ([W, ...] per part); None on one GPU. Returns (accepted node ids [R, D] int64, -1
    padded; bonus tokens [R] int64) -- the definition of engine.sampling.tree_accept_reference restricted to
    greedy rows and 1 <= top_k <= kc."""
    R, N = tokens.shape
    rows, vl = logits.shape
    if _check.active():
        _check.spec_sample_accept(logits, tokens, parent, top_k, temp, depth, kc, vocab_offset)
    nch = int(ext().sample_chunks(vl))
    cv = torch.empty(rows, nch, kc, dtype=torch.float32, device=logits.device)
    ci = torch.empty(rows, nch, kc, dtype=torch.int32, device=logits.device)
    ext().sample_candidates(logits, kc, temp, N, vocab_offset, cv, ci, None, status_tensor(logits.device))
    ranks = 1
    if gather is not None:
        cv, ci = gather([cv, ci])
        ranks = cv.shape[0]
    acc = torch.empty(R, depth, dtype=torch.int64, device=logits.device)
    bonus = torch.empty(R, dtype=torch.int64, device=logits.device)
    ext().spec_accept(cv, ci, ranks, nch, kc, tokens.contiguous(), parent.contiguous(), temp, top_k, top_p, seed,
                      committed, depth, acc, bonus)
    return acc, bonus


# ------------------------------------------------------------------------------------------------
# norms / activations / quant
# ------------------------------------------------------------------------------------------------

def add_rmsnorm_quant(h: torch.Tensor, delta: Optional[torch.Tensor], w: torch.Tensor, eps: float,
                      quant: bool = True, out_bf16: bool = False):
    """In place h <- bf16(h + delta) (if delta), y = rmsnorm(h) * w. Returns (q, qs, y_bf16) with q/qs the
    block-scaled fp8 of y (or None) and y_bf16 (or None)."""
    m, hd = h.shape
    if _check.active():
        _check.add_rmsnorm_quant(h, delta, w, quant)
    q = qs = y = None
    if quant:
        q = torch.empty(m, hd, dtype=FP8_DTYPE, device=h.device)
        qs = torch.empty(hd // 128, m, dtype=torch.float32, device=h.device)
    if out_bf16:
        y = torch.empty(m, hd, dtype=torch.bfloat16 if h.is_cuda else h.dtype, device=h.device)
    if h.is_cuda:
        ext().add_rmsnorm_quant(h, delta, w, eps, q, qs, y)
        return q, qs, y
    if delta is not None:
        h.copy_((h.float() + delta.float()).to(h.dtype))
    hf = h.float()
    yf = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    if quant:
        q_, s_ = quant_act_block(yf)
        q.copy_(q_)
        qs.copy_(s_)
    if out_bf16:
        y.copy_(yf)
    return q, qs, y


def silu_mul_quant(gu: torch.Tensor, quant: bool = True, out_bf16: bool = False):
    """gu [M, 2F] = [gate | up] -> a = bf16(silu(gate) * up) as block-scaled fp8 (q, qs) and/or bf16."""
    m, f2 = gu.shape
    f = f2 // 2
    if _check.active():
        _check.silu_mul_quant(gu, quant)
    q = qs = y = None
    if quant:
        q = torch.empty(m, f, dtype=FP8_DTYPE, device=gu.device)
        qs = torch.empty(f // 128, m, dtype=torch.float32, device=gu.device)
    if out_bf16:
        y = torch.empty(m, f, dtype=torch.bfloat16 if gu.is_cuda else gu.dtype, device=gu.device)
    if gu.is_cuda:
        ext().silu_mul_quant(gu, q, qs, y)
        return q, qs, y
    g, u = gu[:, :f].float(), gu[:, f:].float()
    a = (torch.nn.functional.silu(g) * u)
    if gu.dtype == torch.bfloat16:
        a = a.to(torch.bfloat16)
    if quant:
        q_, s_ = quant_act_block(a.float())
        q.copy_(q_)
        qs.copy_(s_)
    if out_bf16:
        y.copy_(a)
    return q, qs, y


def act_quant(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    m, k = x.shape
    if x.is_cuda:
        q = torch.empty(m, k, dtype=FP8_DTYPE, device=x.device)
        qs = torch.empty(k // 128, m, dtype=torch.float32, device=x.device)
        ext().act_quant(x, q, qs)
        return q, qs
    return quant_act_block(x.float())


# ------------------------------------------------------------------------------------------------
# RoPE + paged KV
# ------------------------------------------------------------------------------------------------

def rope_table(max_pos: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """[max_pos, head_dim/2, 2] fp32 (cos, sin), computed in float64 (rotate-half convention)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.stack([ang.cos(), ang.sin()], -1).float().to(device)


def rope_kv_write(qkv: torch.Tensor, pos: torch.Tensor, slots: Optional[torch.Tensor], cos_sin: torch.Tensor,
                  k_cache: Optional[torch.Tensor], v_cache: Optional[torch.Tensor], hq: int, hkv: int, d: int,
                  q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """qkv [M, (hq+2hkv)*d] -> roped q [M, hq, d]; roped k and v written at `slots` (page*page_size+off)
    of the paged cache [pages, hkv, page_size, d]."""
    m = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty(m, hq, d, dtype=qkv.dtype, device=qkv.device)
    page_size = k_cache.shape[2] if k_cache is not None else 1
    if _check.active():
        _check.rope_kv_write(qkv, pos, slots, cos_sin, k_cache, hq, hkv, d)
    if qkv.is_cuda:
        ext().rope_kv_write(qkv, pos, slots, cos_sin, q_out, k_cache, v_cache, hq, hkv, d, page_size)
        return q_out
    cs = cos_sin[pos.long()]  # [M, d/2, 2]
    cos, sin = cs[..., 0][:, None, :], cs[..., 1][:, None, :]

    def rot(x, sel=None):
        x = x.float()
        c, s = (cos, sin) if sel is None else (cos[sel], sin[sel])
        x1, x2 = x[..., : d // 2], x[..., d // 2:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    q = qkv[:, : hq * d].view(m, hq, d)
    k = qkv[:, hq * d: (hq + hkv) * d].view(m, hkv, d)
    v = qkv[:, (hq + hkv) * d:].view(m, hkv, d)
    q_out.copy_(rot(q).to(q_out.dtype))
    if k_cache is not None and slots is not None:
        ok = slots >= 0
        sl = slots[ok].long()
        pg, off = sl // page_size, sl % page_size
        k_cache[pg, :, off, :] = rot(k[ok], ok).to(k_cache.dtype)
        v_cache[pg, :, off, :] = v[ok].to(v_cache.dtype)
    return q_out


# ------------------------------------------------------------------------------------------------
# attention
# ------------------------------------------------------------------------------------------------

ATTN_IMPL = {"impl": "tc"}   # "tc" = tcgen05 kernel (256-row tiles), "mma" = mma.sync kernel (64-row tiles)


def attn_rows(impl: Optional[str] = None) -> int:
    """Query rows per work tile for the selected attention kernel."""
    return 256 if (impl or ATTN_IMPL["impl"]) == "tc" else 64


def paged_attention(q, k_cache, v_cache, meta, softmax_scale: float, o_in=None, lse_in=None, o_part=None,
                    lse_part=None, out=None, out_q=None, out_qs=None, items=None, tiles=None, impl=None):
    """Run one attention pass described by `meta` (an AttnMeta from engine/attn_meta.py) and a work list
    (`items`, `tiles` = (tile_item, tile_row0, num_tiles) built with attn_rows(impl) rows per tile); see
    csrc/attention.cu for the semantics. impl: "tc" (tcgen05, default) or "mma" (mma.sync)."""
    if _check.active() and items is not None:
        _check.attention(q, k_cache, meta, items, tiles, q.shape[1] // k_cache.shape[1], attn_rows(impl))
    if q.is_cuda:
        ti, tr, nt = tiles
        impl = impl or ATTN_IMPL["impl"]
        if impl == "tc":
            ext().paged_attention_tc(q, k_cache, v_cache, meta.pages, meta.page_indptr, meta.prefix_len,
                                     meta.q_start, meta.tree, items, ti, tr, nt, meta.causal, softmax_scale, o_in,
                                     lse_in, o_part, lse_part, out, out_q, out_qs, status_tensor(q.device))
        else:
            ext().paged_attention(q, k_cache, v_cache, meta.pages, meta.page_indptr, meta.prefix_len, meta.q_start,
                                  meta.tree, items, ti, tr, nt, meta.causal, softmax_scale, o_in, lse_in, o_part,
                                  lse_part, out, out_q, out_qs)
        return
    from ..engine.attn_meta import attention_reference
    attention_reference(q, k_cache, v_cache, meta, softmax_scale, items, o_in, lse_in, o_part, lse_part, out,
                        out_q, out_qs)
