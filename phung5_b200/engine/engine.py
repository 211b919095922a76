"""The serving engine: continuous batching over a paged KV pool with speculative decoding.

Public API (the call a user makes):
    eng = LLMEngine(EngineConfig(...), device="cuda")
    rid = eng.add_request(prompt_ids, SamplingParams(...))
    outs = eng.step()            # one scheduling step: prefill chunk(s) and/or one speculative step
    tokens = eng.generate(prompts, params)

One speculative step for the R running requests (all on device, one host round trip at the end):
  1. draft catch-up: the drafter consumes every token committed since its last step plus the root
     (pending token) — for EAGLE paired with the target's hidden state at the previous position;
  2. tree expansion: `depth` rounds; each round runs the drafter on the K frontier nodes of every
     request (tree-masked over the draft scratch KV), takes the top-K children of each by draft
     log-probability, and keeps the K best children (cumulative score) as the next frontier;
  3. the N-1 best candidates (ancestor-closed) become the verify tree, node 0 = root;
  4. verify: one target forward over R*N nodes with ancestor masks; cascade attention shares the
     prefix pages common to several requests;
  5. accept: greedy match, seeded target-only tree sampling, or the synthetic geometric length;
  6. commit: accepted nodes' KV rows and hidden states move to their final slots; one D2H copy of
     (accepted count, tokens, bonus) per step feeds the host scheduler.
The reference performs the same step inside SGLang's DFlash worker with chain drafts.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .. import ops
from ..config import EngineConfig, ModelConfig, preset
from ..models.llama import Communicator, ForwardBatch, LlamaModel, ModelWeights, random_packed_weights
from .attn_meta import PageTables, build_items, cascade_groups, make_meta, pack_work, upload
from .kv_pool import KVPool
from .oracle import SamplingParams
from ..utils import nvtx as _nvtx
from .sampling import geometric_accept_len, sample_from, seeded_coins, target_probs, tree_accept_reference


@dataclass
class Request:
    rid: int
    tokens: List[int]
    prompt_len: int
    params: SamplingParams
    pages: List[int] = field(default_factory=list)
    committed: int = 0        # tokens whose target KV is written
    prefilled: int = 0        # prompt tokens processed so far
    root: Optional[int] = None
    dlen: int = 0             # positions with draft KV written
    out: List[int] = field(default_factory=list)
    finished: bool = False
    finish_reason: Optional[str] = None
    steps: int = 0
    accepted: List[int] = field(default_factory=list)
    t_arrive: float = 0.0
    t_first: float = 0.0
    t_done: float = 0.0
    gslot: int = -1           # hybrid models: GDN state slot
    resume_root: Optional[int] = None   # preempted: the pending token to resume with after the recompute
    mm: List[Tuple[int, torch.Tensor]] = field(default_factory=list)   # (prompt position, image features [n, H])


@dataclass
class StepOutput:
    rid: int
    new_tokens: List[int]
    finished: bool
    finish_reason: Optional[str] = None     # "stop" (a stop token), "length" (max tokens or context), "abort"


class _VocabOps:
    """Top-k / log-softmax / argmax over vocab-sharded logits. Single rank: local ops."""

    def __init__(self, comm: Communicator, vocab_start: int):
        self.comm = comm
        self.v0 = vocab_start

    def topk_logprobs(self, logits: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Top-k of log-softmax over the full vocab: the fused kernel on this rank's shard, then (TP) a
        merge of every shard's k candidates and log-sum-exp."""
        lp, i, lse = ops.topk_logprobs(logits, k, vocab_offset=self.v0)
        if self.comm.size == 1:
            return lp, i
        return self.comm.topk_logprobs_merge(lp + lse[:, None], i, lse[:, None], k)

    def argmax(self, logits: torch.Tensor) -> torch.Tensor:
        lp, i, lse = ops.topk_logprobs(logits, 1, vocab_offset=self.v0, with_lse=False)
        if self.comm.size == 1:
            return i[:, 0]
        return self.comm.argmax_merge(lp[:, 0] + lse, i[:, 0])

    def full(self, logits: torch.Tensor) -> torch.Tensor:
        return logits if self.comm.size == 1 else self.comm.all_gather_vocab(logits)


class _EagerMeta:
    """Attention metadata of the speculative step's forwards, built on the host per forward (page tables
    shared by the step, per-forward lengths and work lists uploaded in one copy each)."""

    def __init__(self, eng: "LLMEngine", tables: PageTables, groups, c_h: List[int]):
        self.eng, self.tables, self.groups, self.c_h = eng, tables, groups, c_h

    def draft(self, d: int, bits: torch.Tensor):
        e, R = self.eng, len(self.c_h)
        dmeta = self.tables.meta([ch + 1 for ch in self.c_h], [e.K] * R, bits, False)
        # the draft scratch holds d*K entries after this round; keys [prefix, prefix + d*K)
        dmeta.h_kv_len = [ch + 1 + d * e.K for ch in self.c_h]
        return (dmeta,) + e._work(dmeta, self.groups)

    def verify(self, tbits: torch.Tensor):
        e, R = self.eng, len(self.c_h)
        vmeta = self.tables.meta(self.c_h, [e.N] * R, tbits, False)
        return (vmeta,) + e._work(vmeta, self.groups)


class LLMEngine:
    def __init__(self, cfg: EngineConfig, device="cuda", target: Optional[ModelWeights] = None,
                 drafter=None, comm: Optional[Communicator] = None, num_pages: Optional[int] = None,
                 max_context: int = 16384, dtype: torch.dtype = torch.bfloat16):
        self.cfg = cfg
        self.device = torch.device(device)
        self.comm = comm or Communicator()
        self.dtype = dtype
        mc = cfg.model
        tp = self.comm.size
        self.hybrid = mc.arch == "hybrid_gdn"
        gdn_layers = None
        if self.hybrid:
            if tp > 1:
                raise ValueError("hybrid GDN models run with tensor_parallel_size 1 (replicate them for scale-out)")
            if cfg.spec.enabled and cfg.spec.mode == "tree":
                raise ValueError("hybrid GDN models verify chains only: set spec.mode = 'chain'")
            if target is None:
                from ..models.hybrid import random_hybrid
                target, gdn_layers = random_hybrid(mc, self.device, seed=cfg.seed, dtype=dtype)
            else:
                target, gdn_layers = target
        elif target is None:
            target = random_packed_weights(mc, self.device, seed=cfg.seed, tp_rank=self.comm.rank, tp_size=tp)
        self.tw = target
        self.ps = cfg.cache.page_size
        hkv = mc.num_kv_heads // tp
        spec = cfg.spec
        self.K = spec.topk if spec.mode == "tree" else 1
        self.D = spec.depth if spec.mode == "tree" else spec.num_draft
        self.N = spec.tree_nodes if spec.mode == "tree" else spec.num_draft + 1
        self.spec_on = spec.enabled
        self.eagle = cfg.draft.kind == "eagle"
        draft_layers = 0
        if self.spec_on:
            draft_layers = 1 if self.eagle else (drafter.cfg.num_layers if drafter is not None else cfg.draft.num_layers)
        n_kv_layers = len(target.layers)        # hybrid: only the full-attention layers have a KV cache
        if num_pages is None:
            num_pages = cfg.cache.num_pages or self._pages_from_memory(mc, hkv, draft_layers, n_kv_layers)
        self.pool = KVPool(n_kv_layers, num_pages, hkv, self.ps, mc.head_dim, self.device,
                           draft_layers=draft_layers, hidden=mc.hidden if (self.spec_on and self.eagle) else 0,
                           dtype=dtype)
        self.cos_sin = ops.rope_table(max_context + 2 * self.ps, mc.head_dim, mc.rope_theta, self.device)
        self.max_context = max_context
        if self.hybrid:
            from ..models.hybrid import GdnPool, HybridModel, gdn_heads
            g0 = next(g for g in gdn_layers if g is not None)
            self.gdn_pool = GdnPool(sum(g is not None for g in gdn_layers), cfg.cache.max_seqs, g0.gdn.conv_channels,
                                    g0.gdn.conv_w.shape[1], gdn_heads(mc)[1], self.device, dtype)
            self.target = HybridModel(target, gdn_layers, self.pool.k, self.pool.v, self.cos_sin, self.gdn_pool,
                                      self.comm)
        else:
            self.target = LlamaModel(target, self.pool.k, self.pool.v, self.cos_sin, self.comm)
            self.target.moe_a2a = cfg.parallel.moe_dispatch == "a2a"
        self.drafter = None
        if self.spec_on:
            if self.eagle:
                from ..models.eagle import EagleHead, random_eagle
                ew = drafter if drafter is not None else random_eagle(mc, self.device, seed=cfg.seed + 1,
                                                                      tp_rank=self.comm.rank, tp_size=tp)
                self.drafter = EagleHead(ew, target, self.pool.dk, self.pool.dv, self.cos_sin, self.comm)
            else:
                dw = drafter
                if dw is None:
                    dcfg = preset("tiny-draft") if mc.name == "tiny" else ModelConfig(
                        **{**mc.to_dict(), "num_layers": cfg.draft.num_layers,
                           "arch": "llama" if mc.arch == "hybrid_gdn" else mc.arch})
                    dw = random_packed_weights(dcfg, self.device, seed=cfg.seed + 1, tp_rank=self.comm.rank, tp_size=tp)
                self.drafter = LlamaModel(dw, self.pool.dk, self.pool.dv, self.cos_sin, self.comm)
        self.vocab = _VocabOps(self.comm, target.vocab_start)
        self.dvocab = _VocabOps(self.comm, self.drafter.w.vocab_start if (self.drafter is not None and not self.eagle)
                                else target.vocab_start)
        self.reqs: Dict[int, Request] = {}
        self.waiting: List[Request] = []
        self.running: List[Request] = []
        self._next_rid = 0
        self.stats = {"steps": 0, "spec_steps": 0, "tokens_out": 0, "accepted": 0, "prefill_tokens": 0,
                      "h2d_bytes": 0, "d2h_bytes": 0, "graph_replays": 0, "preempted": 0}
        self.use_cascade = cfg.cache.enable_cascade
        import os as _os
        self._host_timing = _os.environ.get("PHX_HOST_TIMING") == "1"
        # CUDA graphs of the speculative step (one per batch size): on by default on CUDA
        self._graphs = {} if (self.device.type == "cuda" and _os.environ.get("PHX_GRAPHS", "1") != "0") else None
        self._graph_cache = 4
        self._has_moe = any(getattr(lw, "moe", None) is not None for lw in self.tw.layers)
        self._consts: Dict[object, torch.Tensor] = {}
        self.host_times: Dict[str, float] = {}
        self._mark_name, self._mark_t = None, 0.0
        self._nvtx_open = False

    # ------------------------------------------------------------------------------------------
    def _pages_from_memory(self, mc: ModelConfig, hkv: int, draft_layers: int, kv_layers: int) -> int:
        per = KVPool.bytes_per_page(kv_layers, hkv, self.ps, mc.head_dim, draft_layers,
                                    mc.hidden if self.eagle else 0)
        if self.device.type == "cuda":
            free, _ = torch.cuda.mem_get_info(self.device)
            budget = free * self.cfg.cache.mem_fraction - 8 * 1024 ** 3
            return max(64, int(budget // per))
        return 512

    # ------------------------------------------------------------------------------------------
    def add_request(self, prompt: Sequence[int], params: Optional[SamplingParams] = None,
                    mm: Optional[Sequence[Tuple[int, torch.Tensor]]] = None) -> int:
        """mm: image inputs as (position, features [n, hidden]): prompt[position:position + n] are the image's
        placeholder ids (models/vision.py), whose token embeddings prefill replaces by the features."""
        rid = self._next_rid
        self._next_rid += 1
        r = Request(rid=rid, tokens=list(prompt), prompt_len=len(prompt), params=params or SamplingParams(),
                    t_arrive=time.perf_counter())
        if mm:
            if self.hybrid:
                raise ValueError("image inputs are served by the attention-only models")
            for pos, f in mm:
                if pos < 0 or pos + f.shape[0] > len(prompt) or f.shape[-1] != self.cfg.model.hidden:
                    raise ValueError("image features do not fit the prompt's placeholder span")
            r.mm = [(int(pos), f.to(self.device)) for pos, f in mm]
        self.reqs[rid] = r
        self.waiting.append(r)
        return rid

    # ------------------------------------------------------------------------------------------
    # sleep / wake: weights to pinned host memory and back, KV pool released and rebuilt (the
    # reference's burst swap relies on SGLang release/resume_memory_occupation and vLLM /sleep, /wake_up,
    # docker/opt/sgl/lb_proxy.py:13-25)
    # ------------------------------------------------------------------------------------------
    @property
    def sleeping(self) -> bool:
        return getattr(self, "_host_copies", None) is not None

    def _weight_tensors(self):
        seen, out = set(), []

        def walk(o):
            if isinstance(o, torch.Tensor):
                if id(o) not in seen:
                    seen.add(id(o))
                    out.append(o)
            elif isinstance(o, (list, tuple)):
                for x in o:
                    walk(x)
            elif hasattr(o, "__dataclass_fields__"):
                for f in o.__dataclass_fields__:
                    walk(getattr(o, f))
        walk(self.tw)
        if self.drafter is not None:
            walk(self.drafter.ew if self.eagle else self.drafter.w)
        return out

    def sleep(self) -> None:
        """Offload every weight to pinned host memory and drop the KV pool (requests must be finished)."""
        if self.sleeping:
            return
        if self.has_work():
            raise RuntimeError("sleep() with requests in flight")
        copies = []
        for t in self._weight_tensors():
            h = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=self.device.type == "cuda")
            h.copy_(t, non_blocking=True)
            copies.append((t, h))
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        for t, h in copies:
            t.data = torch.empty(0, dtype=t.dtype, device=t.device)
        self._host_copies = copies
        self._pool_shape = (self.pool.k.shape, self.pool.dk.shape if self.pool.dk is not None else None,
                            None if self.pool.hidden is None else self.pool.hidden.shape)
        for name in ("k", "v", "dk", "dv", "hidden"):
            t = getattr(self.pool, name)
            if t is not None:
                t.data = torch.empty(0, dtype=t.dtype, device=t.device)
        self.pool.prefix = type(self.pool.prefix)(self.pool.alloc, self.ps)   # cached pages are gone
        self.pool.alloc = type(self.pool.alloc)(self.pool.num_pages, reserved=1)
        self.pool.prefix.alloc = self.pool.alloc
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def wake_up(self) -> None:
        if not self.sleeping:
            return
        for t, h in self._host_copies:
            t.data = h.to(self.device, non_blocking=True)
        kshape, dshape, hshape = self._pool_shape
        for name, shape in (("k", kshape), ("v", kshape), ("dk", dshape), ("dv", dshape), ("hidden", hshape)):
            t = getattr(self.pool, name)
            if t is not None and shape is not None:
                t.data = torch.zeros(shape, dtype=t.dtype, device=self.device)
        self._host_copies = None
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def has_work(self) -> bool:
        return bool(self.waiting) or any(not r.finished for r in self.running)

    def generate(self, prompts: Sequence[Sequence[int]], params: Optional[SamplingParams] = None) -> List[List[int]]:
        rids = [self.add_request(p, params) for p in prompts]
        while self.has_work():
            self.step()
        return [self.reqs[r].out for r in rids]

    def step(self) -> List[StepOutput]:
        outs: List[StepOutput] = []
        if self.waiting:
            outs += self._prefill()
        live = [r for r in self.running if not r.finished and r.root is not None]
        if live:
            live = self._make_room(live)
            if self.spec_on:
                outs += self._spec_step(live)
            else:
                outs += self._decode_step(live)
        self.running = [r for r in self.running if not r.finished]
        self.stats["steps"] += 1
        return outs

    # ------------------------------------------------------------------------------------------
    # admission and preemption: a request is admitted only while fewer than max_running run and the KV pool
    # can hold its prompt plus every running request's next step; when a step's pages do not fit, the most
    # recently admitted requests are preempted (pages released, their full pages left in the prefix cache) and
    # requeued first in line to recompute their committed tokens, resuming with their pending token
    # ------------------------------------------------------------------------------------------
    def _step_tokens(self) -> int:
        """Positions past `committed` a running request's next step writes (verify tree / draft scratch)."""
        if not self.spec_on:
            return 1
        return max(self.N, 1 + (self.D - 1) * self.K) + 1

    def _step_need(self, r: Request) -> int:
        return max(0, -(-(r.committed + self._step_tokens()) // self.ps) - len(r.pages))

    def _make_room(self, live: List[Request]) -> List[Request]:
        need = sum(self._step_need(r) for r in live)
        while need > self.pool.prefix.obtainable() and len(live) > 1:
            victim = live.pop()
            need -= self._step_need(victim)
            self._preempt(victim)
        return live

    def _preempt(self, r: Request) -> None:
        if self.hybrid and r.gslot >= 0:
            self.gdn_pool.release(r.gslot)
            r.gslot = -1
        n_full = min(r.committed, len(r.tokens)) // self.ps
        self.pool.prefix.insert(self._cache_tokens(r), r.pages, n_full)
        self.pool.prefix.release(r.pages)
        r.pages = []
        r.resume_root, r.root = r.root, None
        r.prompt_len = r.committed            # recompute prompt + accepted output, then continue
        r.prefilled = r.committed = r.dlen = 0
        self.running.remove(r)
        self.waiting.insert(0, r)
        self.stats["preempted"] += 1

    def _new_pages(self, r: Request, local_keys: Dict[int, int]) -> Tuple[int, int]:
        """(pages a new request must allocate for its prompt and first step, cached pages it would take out of
        the evictable set): its leading full pages already in the prefix cache, or being written by a request
        earlier in this prefill pass, are shared, not allocated."""
        total = -(-(r.prompt_len + self._step_tokens()) // self.ps)
        if self.hybrid:
            return total, 0
        pc = self.pool.prefix
        hit = lru_hit = 0
        for k in pc.chain_keys(self._cache_tokens(r), self.ps, (r.prompt_len - 1) // self.ps):
            if k in pc.table:
                lru_hit += k in pc.lru
            elif k not in local_keys:
                break
            hit += 1
        return total - hit, lru_hit

    def _admissible(self, r: Request, n_new: int, reserve: int, local_keys: Dict[int, int]) -> Tuple[bool, int]:
        """(admit?, pages it will allocate)."""
        if len(self.running) + n_new >= self.cfg.max_running:
            return False, 0
        if self.hybrid and not self.gdn_pool.free:
            return False, 0
        need, lru_hit = self._new_pages(r, local_keys)
        ok = need + reserve <= self.pool.prefix.obtainable() - lru_hit or (not self.running and n_new == 0)
        return ok, need

    # ------------------------------------------------------------------------------------------
    def _slot(self, r: Request, pos: int) -> int:
        return r.pages[pos // self.ps] * self.ps + pos % self.ps

    def _ensure_pages(self, r: Request, upto: int) -> None:
        need = (upto + self.ps - 1) // self.ps - len(r.pages)
        if need > 0:
            r.pages += self.pool.prefix.alloc_pages(need)

    def _h2d(self, data, dtype) -> torch.Tensor:
        t = torch.tensor(data, dtype=dtype)
        if self.device.type == "cuda":
            t = t.pin_memory()
            self.stats["h2d_bytes"] += t.numel() * t.element_size()
            return t.to(self.device, non_blocking=True)
        return t

    def _gdn_batch(self, lens: List[int], reqs: List[Request], mode: str):
        from ..models.hybrid import GdnBatch
        ts = [0]
        for n in lens:
            ts.append(ts[-1] + n)
        packed = self._h2d(ts + [r.gslot for r in reqs], torch.int32)
        return GdnBatch(tok_start=packed[:len(ts)], slot=packed[len(ts):], mode=mode)

    @staticmethod
    def _cache_tokens(r: Request) -> List[int]:
        """Prefix-cache key of a request's tokens: image rows enter as negative ids, so a page holding image KV
        never matches text that happens to use the same placeholder ids."""
        if not r.mm:
            return r.tokens
        t = list(r.tokens)
        for pos, f in r.mm:
            for i in range(pos, pos + f.shape[0]):
                t[i] = -1 - t[i]
        return t

    def _finish(self, r: Request) -> None:
        if self.hybrid and r.gslot >= 0:
            self.gdn_pool.release(r.gslot)
            r.gslot = -1
        r.finished = True
        r.t_done = time.perf_counter()
        n_full = min(r.committed, len(r.tokens)) // self.ps
        self.pool.prefix.insert(self._cache_tokens(r), r.pages, n_full)
        self.pool.prefix.release(r.pages)
        r.pages = []

    def _emit(self, r: Request, new: List[int]) -> StepOutput:
        room = r.params.max_new_tokens - len(r.out)
        new = new[:room]
        stop = r.params.stop_token_ids
        hit = False
        if stop:
            for k, t in enumerate(new):
                if t in stop:                  # the stop token ends the output and is not part of it
                    new, hit = new[:k], True
                    break
        r.out += new
        self.stats["tokens_out"] += len(new)
        done = hit or len(r.out) >= r.params.max_new_tokens or r.committed + self.N + 2 * self.ps >= self.max_context
        if done:
            r.finish_reason = "stop" if hit else "length"
            self._finish(r)
        return StepOutput(r.rid, new, done, r.finish_reason)

    def abort(self, rid: int) -> bool:
        """End a request now (client gone, stop string seen): its pages are released (full ones kept in the
        prefix cache). False if it is unknown or already finished."""
        r = self.reqs.get(rid)
        if r is None or r.finished:
            return False
        if any(x is r for x in self.waiting):
            self.waiting = [x for x in self.waiting if x is not r]
            if self.hybrid and r.gslot >= 0:
                self.gdn_pool.release(r.gslot)
                r.gslot = -1
            self.pool.prefix.release(r.pages)
            r.pages = []
            r.finished = True
            r.t_done = time.perf_counter()
        else:
            self._finish(r)
        r.finish_reason = "abort"
        return True

    def _first_token(self, logits: torch.Tensor, reqs: List[Request]) -> List[int]:
        full = self.vocab.full(logits)
        temp = torch.tensor([r.params.temperature for r in reqs])
        if float(temp.max()) <= 0:
            return full.argmax(-1).tolist()
        probs = target_probs(full.float().cpu(), temp, torch.tensor([r.params.top_k for r in reqs]),
                             torch.tensor([r.params.top_p for r in reqs]))
        coins = seeded_coins(torch.tensor([r.params.seed for r in reqs]),
                             torch.tensor([r.prompt_len - 1 for r in reqs]), 1)[:, 0]
        toks = sample_from(probs, coins)
        return [int(t) if r.params.temperature > 0 else int(a) for t, a, r in
                zip(toks, full.argmax(-1).cpu(), reqs)]

    # ------------------------------------------------------------------------------------------
    # prefill
    # ------------------------------------------------------------------------------------------
    def _prefill(self) -> List[StepOutput]:
        budget = self.cfg.max_prefill_tokens
        batch: List[Tuple[Request, int, int]] = []  # (req, start, end)
        local_keys: Dict[int, int] = {}
        reserve = sum(self._step_need(x) for x in self.running if not x.finished)
        n_new = 0
        while self.waiting and budget > 0:
            r = self.waiting[0]
            if r.prefilled == 0 and not r.pages:
                ok, need = self._admissible(r, n_new, reserve, local_keys)
                if not ok:
                    break
                n_new += 1
                reserve += need
            if self.hybrid and r.gslot < 0:
                r.gslot = self.gdn_pool.alloc()
            if r.prefilled == 0 and not r.pages and not self.hybrid:
                # prefix cache (and pages being written by requests earlier in this pass); hybrid models
                # recompute prompts: a cached KV prefix carries no GDN state
                n_match = (r.prompt_len - 1) // self.ps
                ctoks = self._cache_tokens(r)
                keys = self.pool.prefix.chain_keys(ctoks, self.ps, n_match)
                pages = self.pool.prefix.match(ctoks, (r.prompt_len - 1))
                for k in keys[len(pages):]:
                    p = local_keys.get(k)
                    if p is None:
                        break
                    pages.append(p)
                    self.pool.alloc.incref([p])
                r.pages = pages
                r.prefilled = len(pages) * self.ps
                r.committed = r.prefilled
                r.dlen = r.prefilled
            start = r.prefilled
            end = min(r.prompt_len, start + budget)
            self._ensure_pages(r, end)
            for i, k in enumerate(self.pool.prefix.chain_keys(self._cache_tokens(r), self.ps, end // self.ps)):
                local_keys.setdefault(k, r.pages[i])
            batch.append((r, start, end))
            budget -= end - start
            r.prefilled = end
            if end == r.prompt_len:
                self.waiting.pop(0)
            else:
                break
        toks, pos, slots, last_rows = [], [], [], []
        mm_rows, mm_feats = [], []
        for r, s, e in batch:
            base = len(toks)
            for ipos, f in r.mm:                  # image rows of this chunk get the image features
                a, b = max(ipos, s), min(ipos + f.shape[0], e)
                if a < b:
                    mm_rows += list(range(base + a - s, base + b - s))
                    mm_feats.append(f[a - ipos:b - ipos])
            toks += r.tokens[s:e]
            pos += list(range(s, e))
            slots += [self._slot(r, p) for p in range(s, e)]
            last_rows.append(len(toks) - 1)
        meta = make_meta([r.pages for r, _, _ in batch], [s for _, s, _ in batch], [e - s for _, s, e in batch],
                         None, True, self.device)
        g = self.target.hq // self.target.hkv
        _, p2 = build_items(meta, g)
        fb = ForwardBatch(tokens=self._h2d(toks, torch.int64), positions=self._h2d(pos, torch.int32),
                          slots=self._h2d(slots, torch.int64), meta=meta, work2=pack_work(p2, g, self.device),
                          logits_rows=self._h2d(last_rows, torch.int64))
        if mm_rows:
            fb.mm_rows = self._h2d(mm_rows, torch.int64)
            fb.mm_feats = torch.cat(mm_feats)
        if self.hybrid:
            fb.gdn = self._gdn_batch([e - s for _, s, e in batch], [r for r, _, _ in batch], "prefill")
        logits, h = self.target.forward(fb, want_hidden=True)
        if self.pool.hidden is not None:
            self.pool.hidden[fb.slots] = h
        self.stats["prefill_tokens"] += len(toks)
        outs = []
        done = [(i, r) for i, (r, s, e) in enumerate(batch) if e == r.prompt_len]
        for r, s, e in batch:
            r.committed = e
        if not self.hybrid:
            # a finished prompt's full pages join the prefix cache now (later prefill passes share them); its draft
            # KV is written by this step's catch-up, before any later request can match them
            for _, r in done:
                self.pool.prefix.insert(self._cache_tokens(r), r.pages, r.prompt_len // self.ps)
        resumed = [r for _, r in done if r.resume_root is not None]
        for r in resumed:                      # recomputed after a preemption: the pending token is known
            r.root, r.resume_root = r.resume_root, None
            self.running.append(r)
        done = [(i, r) for i, r in done if all(r is not x for x in resumed)]
        if done:
            firsts = self._first_token(logits[[i for i, _ in done]], [r for _, r in done])
            for (i, r), t in zip(done, firsts):
                r.root = t
                r.tokens.append(t)
                r.t_first = time.perf_counter()
                self.running.append(r)
                outs.append(self._emit(r, [t]))
        return outs

    # ------------------------------------------------------------------------------------------
    # plain decode (speculation off)
    # ------------------------------------------------------------------------------------------
    def _decode_step(self, reqs: List[Request]) -> List[StepOutput]:
        for r in reqs:
            self._ensure_pages(r, r.committed + 1)
        meta = make_meta([r.pages for r in reqs], [r.committed for r in reqs], [1] * len(reqs), None, True,
                         self.device)
        g = self.target.hq // self.target.hkv
        _, p2 = build_items(meta, g)
        fb = ForwardBatch(tokens=self._h2d([r.root for r in reqs], torch.int64),
                          positions=self._h2d([r.committed for r in reqs], torch.int32),
                          slots=self._h2d([self._slot(r, r.committed) for r in reqs], torch.int64), meta=meta,
                          work2=pack_work(p2, g, self.device))
        if self.hybrid:
            fb.gdn = self._gdn_batch([1] * len(reqs), reqs, "prefill")
        logits, _ = self.target.forward(fb)
        nxt = self._first_token(logits, reqs) if any(r.params.temperature > 0 for r in reqs) else \
            self.vocab.argmax(logits).tolist()
        outs = []
        for r, t in zip(reqs, nxt):
            r.committed += 1
            r.root = t
            r.tokens.append(t)
            outs.append(self._emit(r, [t]))
        return outs

    # ------------------------------------------------------------------------------------------
    # speculative step
    # ------------------------------------------------------------------------------------------
    def _draft_forward(self, fb: ForwardBatch, hidden_in: Optional[torch.Tensor]):
        if self.eagle:
            return self.drafter.forward(fb, hidden_in)
        logits, _ = self.drafter.forward(fb)
        return logits, None

    def _groups(self, meta):
        if not self.use_cascade:
            return None
        gr = cascade_groups(meta, self.ps)
        return gr or None

    def _clip_groups(self, groups, prefix):
        """Groups whose shared keys do not exceed any member's visible prefix (catch-up prefixes are shorter
        than the committed lengths the groups were computed from)."""
        if not groups:
            return None
        out = []
        for a, b, L in groups:
            m = min(prefix[a:b + 1])
            L2 = min(L, (m // self.ps) * self.ps)
            if L2 > 0:
                out.append((a, b, L2))
        return out or None

    def _work(self, meta, groups):
        g = self.target.hq // self.target.hkv
        p1, p2 = build_items(meta, g, groups)
        return (pack_work(p1, g, self.device) if p1 else None), pack_work(p2, g, self.device)

    def _mark(self, name: str) -> None:
        """Host-side phase timer (PHX_HOST_TIMING=1): accumulates host wall time between marks per phase;
        with the device running asynchronously this is the time the host spends enqueuing each phase
        (the final commit phase includes waiting for the device)."""
        ops.set_phase(name)
        if _nvtx.ON:
            if self._nvtx_open:
                _nvtx.pop()
            self._nvtx_open = name != "host_tail"
            if self._nvtx_open:
                _nvtx.push(name)
        if not self._host_timing:
            return
        now = time.perf_counter()
        if self._mark_name is not None:
            self.host_times[self._mark_name] = self.host_times.get(self._mark_name, 0.0) + now - self._mark_t
        self._mark_name, self._mark_t = name, now

    def _spec_step(self, reqs: List[Request]) -> List[StepOutput]:
        self._mark("setup")
        dev = self.device
        R, K, D, N = len(reqs), self.K, self.D, self.N
        scratch = 1 + (D - 1) * K
        for r in reqs:
            self._ensure_pages(r, r.committed + max(N, scratch) + 1)
        c_h = [r.committed for r in reqs]
        tables = PageTables([r.pages for r in reqs], dev, self.ps)
        groups = (tables.groups(c_h) or None) if self.use_cascade else None

        self._mark("draft_catchup")
        logits, root_feat = self._catchup(reqs, tables, groups)
        mode, ngeo_h = self._accept_mode(reqs)

        graph = self._spec_graph(R, mode, reqs)
        if graph is not None:
            self._mark("graph_replay")
            packed_dev = graph.run(reqs, tables, groups, c_h, logits, root_feat, ngeo_h)
            self.stats["graph_replays"] += 1
        else:
            self._mark("draft_tree")
            pt = tables.padded_device(dev)
            c = upload(c_h, torch.int64, dev)
            roots = upload([r.root for r in reqs], torch.int64, dev)
            ngeo = upload(ngeo_h, torch.int64, dev) if ngeo_h is not None else None
            packed_dev = self._spec_core(_EagerMeta(self, tables, groups, c_h), pt, c, roots, logits, root_feat,
                                         mode, ngeo, reqs)

        self._mark("commit_sync")
        packed = packed_dev.cpu()
        self.stats["d2h_bytes"] += packed.numel() * packed.element_size()
        outs = []
        for i, r in enumerate(reqs):
            n = int(packed[i, 0])
            new = [int(x) for x in packed[i, 1:1 + n]] + [int(packed[i, -1])]
            r.tokens += new
            r.committed += 1 + n
            r.root = new[-1]
            r.steps += 1
            r.accepted.append(n)
            self.stats["accepted"] += n
            outs.append(self._emit(r, new))
        self.stats["spec_steps"] += 1
        self._mark("host_tail")
        self._mark_name = None
        return outs

    def _catchup(self, reqs: List[Request], tables: "PageTables", groups):
        """Draft forward over each request's positions [dlen, committed] (the root at `committed`): the
        drafter's KV catches up with the tokens accepted last step. -> (logits [R, V_local] of the roots,
        root features [R, H] or None)."""
        cu_tok, cu_pos, cu_slot, cu_hslot, last = [], [], [], [], []
        for r in reqs:
            for p in range(r.dlen, r.committed + 1):
                cu_tok.append(r.tokens[p])
                cu_pos.append(p)
                cu_slot.append(self._slot(r, p))
                cu_hslot.append(self._slot(r, p - 1) if p > 0 else 0)
            last.append(len(cu_tok) - 1)
        meta = tables.meta([r.dlen for r in reqs], [r.committed + 1 - r.dlen for r in reqs], None, True)
        w1, w2 = self._work(meta, self._clip_groups(groups, [r.dlen for r in reqs]))
        packed = self._h2d(cu_tok + cu_slot + cu_hslot + last + cu_pos, torch.int64)
        T, R = len(cu_tok), len(reqs)
        fb = ForwardBatch(tokens=packed[:T], positions=packed[3 * T + R:].to(torch.int32), slots=packed[T:2 * T],
                          meta=meta, work1=w1, work2=w2, logits_rows=packed[3 * T:3 * T + R])
        hid_in = self.pool.hidden[packed[2 * T:3 * T]] if self.eagle else None
        logits, feat = self._draft_forward(fb, hid_in)
        for r in reqs:
            r.dlen = r.committed + 1
        return logits, (feat[fb.logits_rows] if feat is not None else None)

    def _accept_mode(self, reqs: List[Request]):
        """("geometric", accept lengths) | ("greedy", None) | ("sample", None)."""
        spec = self.cfg.spec
        if spec.accept == "geometric":
            steps = torch.tensor([r.steps for r in reqs])
            rid = torch.tensor([r.rid for r in reqs])
            return "geometric", geometric_accept_len(spec.accept_seed, steps, rid, spec.accept_p, spec.accept_cap)
        if all(r.params.temperature <= 0 for r in reqs):
            return "greedy", None
        return "sample", None

    def _spec_graph(self, R: int, mode: str, reqs: List[Request]):
        """The CUDA-graph runner for this batch shape and accept mode, or None to run the step eagerly. Seeded
        sampling is captured when the device accept path serves every request."""
        if (self._graphs is None or not self.eagle or self.hybrid
                or (self.comm.size != 1 and not getattr(self.comm, "fused", False))
                or (mode == "sample" and not self._device_sampling(reqs))):
            return None
        kc = ops.sample_kc([r.params.top_k for r in reqs], [r.params.temperature for r in reqs]) \
            if mode == "sample" else 0
        key = (R, mode, kc)
        g = self._graphs.get(key)
        if g is None:
            from .spec_graph import SpecGraph
            if len(self._graphs) >= self._graph_cache:
                self._graphs.pop(next(iter(self._graphs)))
            g = SpecGraph(self, R, mode, kc)
            self._graphs[key] = g
        return g

    def _spec_core(self, mp, pt, c, roots, logits, root_feat, mode, ngeo, reqs=None, sp=None):
        """Tree expansion, selection, verification, acceptance and the KV move of one speculative step, on
        device tensors only (no host synchronisation unless mode == "sample" takes the dense torch definition).
        `sp`: sampling tensors (mode "sample"; None: uploaded from reqs). `mp` supplies the attention
        metadata and work lists of the draft rounds and of verification. Returns packed [R, 2 + D] int64:
        accepted count, accepted tokens (-1 padded), bonus token."""
        dev = self.device
        R, K, D, N = pt.shape[0], self.K, self.D, self.N

        def slots_of(pos):  # pos [R, n] (device) -> slots
            return pt.gather(1, pos // self.ps) * self.ps + pos % self.ps

        synth = mode == "geometric" and K > 1
        # ---- tree expansion ----
        lp, ti = self.dvocab.topk_logprobs(logits, K)          # [R, K]
        pool_tok, pool_score = [ti], [lp]
        pool_par = [torch.full((R, K), -1, dtype=torch.int64, device=dev)]
        pool_depth = [torch.ones(R, K, dtype=torch.int64, device=dev)]
        front_idx = torch.arange(K, device=dev).expand(R, K)        # pool indices of the frontier
        front_tok, front_score = ti, lp
        front_bits_parent = torch.zeros(R, K, dtype=torch.int64, device=dev)
        front_feat = root_feat[:, None, :].expand(R, K, -1) if root_feat is not None else None
        n_pool = K
        for d in range(1, D):
            j = torch.arange(K, device=dev)
            sidx = (d - 1) * K + j                                   # scratch entry of each frontier node
            bits = front_bits_parent | (torch.ones_like(front_bits_parent) << sidx[None, :])
            pos = (c[:, None] + d).expand(R, K)
            sl = slots_of(c[:, None] + 1 + sidx[None, :])
            dmeta, dw1, dw2 = mp.draft(d, bits.reshape(-1))
            fb = ForwardBatch(tokens=front_tok.reshape(-1), positions=pos.reshape(-1).to(torch.int32),
                              slots=sl.reshape(-1), meta=dmeta, work1=dw1, work2=dw2)
            lg, fe = self._draft_forward(fb, front_feat.reshape(R * K, -1) if front_feat is not None else None)
            clp, cti = self.dvocab.topk_logprobs(lg, K)              # [R*K, K]
            cscore = (front_score.reshape(-1, 1) + clp).reshape(R, K * K)
            ctok = cti.reshape(R, K * K)
            cpar = front_idx.reshape(R, K, 1).expand(R, K, K).reshape(R, K * K)
            pool_tok.append(ctok)
            pool_score.append(cscore)
            pool_par.append(cpar)
            pool_depth.append(torch.full((R, K * K), d + 1, dtype=torch.int64, device=dev))
            base = n_pool
            n_pool += K * K
            # next frontier: K best children. Synthetic acceptance keeps the spine (frontier row 0 is the
            # spine node; column 0 is its best child) so the drawn accept length is realizable.
            sel_score = cscore
            if synth:
                sel_score = cscore.clone()
                sel_score[:, 0] = float("inf")
            _, fi = torch.topk(sel_score, K, dim=-1)
            fs = cscore.gather(1, fi)
            front_idx = base + fi
            front_tok = ctok.gather(1, fi)
            front_score = fs
            prow = fi // K                                          # which frontier row produced it
            front_bits_parent = bits.gather(1, prow)
            if fe is not None:
                fe = fe.reshape(R, K, -1)
                front_feat = fe.gather(1, prow[..., None].expand(R, K, fe.shape[-1]))
        P_tok = torch.cat(pool_tok, 1)
        P_score = torch.cat(pool_score, 1)
        P_par = torch.cat(pool_par, 1)
        P_depth = torch.cat(pool_depth, 1)

        self._mark("select")
        # ---- select the verify tree ----
        nsel = N - 1
        adj = P_score - 1e-4 * P_depth.float()
        if synth:
            # spine nodes (best child of the spine at every depth) are pool entries 0, K, K+K*K, ...
            spine = self._spine_index(dev)
            adj = adj.index_fill(1, spine, 0.0) + torch.zeros_like(adj).index_fill(1, spine, 1e6)
        _, sel = torch.topk(adj, nsel, dim=-1)
        key = P_depth.gather(1, sel).float() * 1e4 - adj.gather(1, sel)
        order = torch.argsort(key, dim=-1)
        sel = sel.gather(1, order)                                    # pool idx of nodes 1..N-1
        node_of = torch.zeros(R, n_pool, dtype=torch.int64, device=dev)
        node_of.scatter_(1, sel, torch.arange(1, N, device=dev).expand(R, nsel))
        par_pool = P_par.gather(1, sel)
        parent = torch.cat([torch.full((R, 1), -1, device=dev, dtype=torch.int64),
                            torch.where(par_pool < 0, torch.zeros_like(par_pool),
                                        node_of.gather(1, par_pool.clamp(min=0)))], 1)      # [R, N]
        depth = torch.cat([torch.zeros(R, 1, dtype=torch.int64, device=dev), P_depth.gather(1, sel)], 1)
        tokens = torch.cat([roots[:, None], P_tok.gather(1, sel)], 1)
        nb = torch.ones(R, N, dtype=torch.int64, device=dev) << torch.arange(N, device=dev)[None, :]
        tbits = nb.clone()
        for dd in range(1, D + 1):
            pb = tbits.gather(1, parent.clamp(min=0))
            tbits = torch.where(depth == dd, pb | nb, tbits)

        self._mark("verify")
        # ---- verify ----
        vpos = c[:, None] + depth
        vslot = slots_of(c[:, None] + torch.arange(N, device=dev)[None, :])
        vmeta, vw1, vw2 = mp.verify(tbits.reshape(-1))
        fb = ForwardBatch(tokens=tokens.reshape(-1), positions=vpos.reshape(-1).to(torch.int32),
                          slots=vslot.reshape(-1), meta=vmeta, work1=vw1, work2=vw2)
        if self.hybrid:      # chain: request r's N verify tokens are rows [r*N, (r+1)*N)
            fb.gdn = self._gdn_batch([N] * R, reqs, "verify")
        vlogits, vh = self.target.forward(fb, want_hidden=self.eagle)
        if self.pool.hidden is not None:
            self.pool.hidden[fb.slots] = vh

        self._mark("accept")
        # ---- accept ----
        vl = vlogits.reshape(R, N, -1)
        if mode == "sample":
            acc_nodes, bonus = self._accept_sample(reqs, vl, tokens, parent, c, sp)
        else:
            acc_nodes, bonus = self._accept_static(vl, tokens, parent, ngeo)

        # ---- commit: move the accepted nodes' KV to the committed positions (fixed shape, masked) ----
        valid = acc_nodes >= 0
        if self.hybrid:      # fold the root and the accepted chain into the GDN states
            self.target.commit(valid.sum(1) + 1)
        jj = torch.arange(D, device=dev)[None, :].expand(R, D)
        dst = slots_of(c[:, None] + 1 + jj)
        src = torch.where(valid, slots_of(c[:, None] + acc_nodes.clamp(min=0)), dst)
        self.pool.move_slots(src.reshape(-1), dst.reshape(-1))
        acc_tok = torch.where(valid, tokens.gather(1, acc_nodes.clamp(min=0)), torch.full_like(acc_nodes, -1))
        return torch.cat([valid.sum(1, keepdim=True), acc_tok, bonus[:, None]], 1)

    def _spine_index(self, dev) -> torch.Tensor:
        key = ("spine", str(dev))
        t = self._consts.get(key)
        if t is None:
            K, D = self.K, self.D
            t = upload([0] + [K + (d - 1) * K * K for d in range(1, D)], torch.int64, dev)
            self._consts[key] = t
        return t

    def _accept_static(self, logits, tokens, parent, ngeo):
        """Greedy (target argmax along the tree) or synthetic geometric acceptance; device ops only.
        Returns (accepted node ids [R, D] (-1 = none), bonus tokens [R])."""
        dev = self.device
        R, N, D = tokens.shape[0], self.N, self.D
        cur = torch.zeros(R, dtype=torch.int64, device=dev)
        alive = torch.ones(R, dtype=torch.bool, device=dev)
        acc = torch.full((R, D), -1, dtype=torch.int64, device=dev)
        nidx = torch.arange(N, device=dev)[None, :]
        tgt = self.vocab.argmax(logits.reshape(R * N, -1)).reshape(R, N)
        for d in range(1, D + 1):
            kids = parent == cur[:, None]
            if ngeo is not None:
                match = kids & (d <= ngeo)[:, None]
            else:
                match = kids & (tokens == tgt.gather(1, cur[:, None]))
            match &= alive[:, None]
            has = match.any(1)
            first = torch.where(match, nidx.expand(R, N), torch.full_like(tokens, N)).min(1).values
            acc[:, d - 1] = torch.where(has, first, torch.full_like(first, -1))
            cur = torch.where(has, first, cur)
            alive &= has
        return acc, tgt.gather(1, cur[:, None])[:, 0]

    def sample_tensors(self, reqs: List[Request]):
        """Per-request sampling parameters as device tensors: (temperature fp32, top_k int32, top_p fp32, seed
        int64, candidates per chunk) for the device accept path."""
        dev = self.device
        temps = [r.params.temperature for r in reqs]
        ks = [r.params.top_k for r in reqs]
        return (upload(temps, torch.float32, dev), upload(ks, torch.int32, dev),
                upload([r.params.top_p for r in reqs], torch.float32, dev),
                upload([r.params.seed & 0xFFFFFFFF for r in reqs], torch.int64, dev), ops.sample_kc(ks, temps))

    def _device_sampling(self, reqs: List[Request]) -> bool:
        return self.device.type == "cuda" and ops.device_sampling_ok([r.params.top_k for r in reqs],
                                                                      [r.params.temperature for r in reqs])

    def _accept_sample(self, reqs, logits, tokens, parent, c, sp=None):
        """Seeded target-only tree sampling (per-request temperature / top-k / top-p). On the GPU, for greedy
        rows and 1 <= top_k <= 64, one candidate kernel per vocab shard plus one accept kernel (csrc/sample.cu),
        no host synchronisation (used inside the step's CUDA graph, where `sp` holds static buffers); otherwise
        the dense torch definition (engine/sampling.py). Returns (accepted node ids [R, D] (-1 = none), bonus
        tokens [R])."""
        R, N, D = tokens.shape[0], self.N, self.D
        if sp is None:
            sp = self.sample_tensors(reqs)
        temp, topk, topp, seed, kc = sp
        if reqs is None or self._device_sampling(reqs):
            gather = None if self.comm.size == 1 else self.comm.gather
            return ops.spec_sample_accept(logits.reshape(R * N, -1), tokens, parent, temp, topk, topp, seed, c, D, kc,
                                          self.vocab.v0, gather)
        coins = seeded_coins(seed, c, D + 2)
        rows = torch.arange(R, device=self.device)
        return tree_accept_reference(lambda cur: self.vocab.full(logits[rows, cur]), tokens, parent, temp,
                                     topk.long(), topp, coins, D)
