"""OpenAI-compatible HTTP server over `LLMEngine`.

The engine runs on one background thread (every `step()` is one scheduling step: prefill and/or one
speculative step for all running requests); HTTP handlers submit requests through a queue and await
per-request streams. Endpoints mirror what the reference's clients use of SGLang/vLLM
(pipeline_service/llm/session.py:150-270, docker/opt/sgl/lb_proxy.py:13-25):

  GET  /health                      200 while serving, 503 while asleep or after an engine error
  GET  /v1/models
  POST /v1/completions              prompt: str | [int]; max_tokens, temperature, top_p, top_k, seed, stream, stop
                                    (strings), stop_token_ids, ignore_eos (generation ends at the tokenizer's EOS
                                    otherwise); finish_reason "stop" / "length"; a caller that goes away aborts
  POST /v1/chat/completions         messages (chat template of the tokenizer); same sampling fields; with a vision
                                    tower, `image_url` content parts (data URLs) -- sent once with a `uuid`, later
                                    by `uuid` alone; an unknown uuid answers 400 so the client resends in full
  GET  /get_load                    {"num_running", "num_waiting"}
  GET  /metrics                     Prometheus text (tokens, accept length, step latency, TPOT)
  POST /sleep, /wake_up             weights to host memory and back (vLLM names)
  POST /release_memory_occupation, /resume_memory_occupation   (SGLang names, same actions)

    python -m phung5_b200.serve.server --model llama3-8b --port 8001 [--spec tree] [--device cuda]
    torchrun --nproc-per-node 8 -m phung5_b200.serve.server --model llama3-70b-fp8   (tensor parallel; rank 0 serves)
"""
from __future__ import annotations

import argparse
import asyncio
import json
import queue
import threading
import time
import traceback
import uuid
from dataclasses import dataclass, field
from typing import AsyncIterator, Dict, List, Optional

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..engine.oracle import SamplingParams
from .metrics import EngineMetrics


@dataclass
class _Pending:
    prompt: List[int]
    params: SamplingParams
    out: "asyncio.Queue"
    loop: asyncio.AbstractEventLoop
    rid: int = -1
    mm: Optional[list] = None          # image inputs: [(position, features [n, H])]
    cancelled: bool = False            # the caller went away before the engine took the request


class AsyncEngine:
    """Drives an LLMEngine from a background thread; thread-safe submission, asyncio streams out.

    Tensor parallel serving: with `group` (a gloo process group over the TP ranks) this thread runs on
    rank 0 and, every loop iteration, broadcasts what it is about to apply (control ops, new requests and
    its step count) to the other ranks, which run `tp_worker_loop`; every rank then applies the same
    commands and takes the same engine step, so the replicated scheduler state never diverges. When idle,
    the broadcast is a heartbeat every 50 ms."""

    def __init__(self, engine, metrics: Optional[EngineMetrics] = None, group=None):
        self.engine = engine
        self.group = group
        self.steps = 0
        self.metrics = metrics or EngineMetrics()
        self._submit: "queue.Queue[_Pending]" = queue.Queue()
        self._control: "queue.Queue" = queue.Queue()
        self._streams: Dict[int, _Pending] = {}
        self._wake = threading.Event()
        self._stop = False
        self.error: Optional[str] = None
        self._thread = threading.Thread(target=self._run, name="phx-engine", daemon=True)
        self._thread.start()

    # -- engine thread --------------------------------------------------------------------------
    def _run(self):
        eng = self.engine
        while not self._stop:
            try:
                ops, subs = [], []
                while True:
                    try:
                        ops.append(self._control.get_nowait())
                    except queue.Empty:
                        break
                while True:
                    try:
                        subs.append(self._submit.get_nowait())
                    except queue.Empty:
                        break
                subs = [p for p in subs if not p.cancelled]
                # aborts name engine request ids, so every rank drops the same request
                ops = [(op, (a.rid,) if op == "abort" else a, fut, loop) for op, a, fut, loop in ops
                       if not (op == "abort" and a.rid < 0)]
                if self.group is not None:
                    _broadcast_cmds({"ops": [(o[0], o[1]) for o in ops],
                                     "reqs": [(p.prompt, p.params, _mm_to_host(p.mm)) for p in subs],
                                     "steps": self.steps, "stop": False}, self.group)
                for op, args, fut, loop in ops:
                    try:
                        getattr(eng, op)(*args)
                        if op == "abort":
                            self._streams.pop(args[0], None)
                        if fut is not None:
                            loop.call_soon_threadsafe(fut.set_result, True)
                    except Exception as e:  # pragma: no cover - surfaced to the caller
                        if fut is not None:
                            loop.call_soon_threadsafe(fut.set_exception, e)
                for p in subs:
                    p.rid = eng.add_request(p.prompt, p.params, mm=p.mm)
                    self._streams[p.rid] = p
                if not eng.has_work():
                    self._wake.wait(0.05)
                    self._wake.clear()
                    continue
                t0 = time.perf_counter()
                outs = eng.step()
                self.steps += 1
                dt = time.perf_counter() - t0
                self.metrics.observe_step(dt, outs, eng)
                for o in outs:
                    p = self._streams.get(o.rid)
                    if p is None:
                        continue
                    if p.cancelled or not _deliver(p, o):
                        # the caller is gone (its abort may still be queued): drop the request now; every
                        # tensor-parallel rank learns of it through the abort op that the caller queued
                        del self._streams[o.rid]
                        if self.group is None and not o.finished:
                            eng.abort(o.rid)
                        continue
                    if o.finished:
                        del self._streams[o.rid]
            except Exception:  # keep serving health; report the error
                self.error = traceback.format_exc()
                for p in list(self._streams.values()):
                    _deliver(p, None)
                self._streams.clear()
                time.sleep(0.1)

    # -- asyncio side ---------------------------------------------------------------------------
    async def generate(self, prompt: List[int], params: SamplingParams, mm: Optional[list] = None) -> AsyncIterator:
        """Stream a request's StepOutputs; a caller that stops early (client gone, stop string) aborts it."""
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        p = _Pending(prompt, params, q, loop, mm=mm)
        self._submit.put(p)
        self._wake.set()
        done = False
        try:
            while True:
                o = await q.get()
                if o is None:
                    raise RuntimeError(self.error or "engine error")
                done = o.finished
                yield o
                if o.finished:
                    return
        finally:
            if not done:
                self.abort(p)

    def abort(self, p: _Pending) -> None:
        p.cancelled = True
        self._control.put(("abort", p, None, None))
        self._wake.set()

    async def control(self, op: str):
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self._control.put((op, (), fut, loop))
        self._wake.set()
        return await fut

    def load(self) -> Dict[str, int]:
        return {"num_running": len(self.engine.running), "num_waiting": len(self.engine.waiting) + self._submit.qsize()}

    def shutdown(self):
        self._stop = True
        self._wake.set()
        self._thread.join(timeout=5)
        if self.group is not None:
            _broadcast_cmds({"ops": [], "reqs": [], "steps": self.steps, "stop": True}, self.group)


def _deliver(p: _Pending, item) -> bool:
    """Hand a step's output to the caller's event loop; False if that loop is gone."""
    try:
        p.loop.call_soon_threadsafe(p.out.put_nowait, item)
        return True
    except RuntimeError:            # the loop was closed
        p.cancelled = True
        return False


def _mm_to_host(mm):
    """Image features travel to the other tensor-parallel ranks with the request (host copies)."""
    return None if not mm else [(pos, f.detach().to("cpu")) for pos, f in mm]


def _broadcast_cmds(cmds: Optional[dict], group) -> dict:
    import torch.distributed as dist
    box = [cmds]
    dist.broadcast_object_list(box, src=0, group=group)
    return box[0]


def tp_worker_loop(engine, group) -> None:
    """Ranks 1..TP-1 of a tensor-parallel server: apply rank 0's commands, take the same steps."""
    steps = 0
    while True:
        cmds = _broadcast_cmds(None, group)
        if cmds["stop"]:
            return
        if cmds["steps"] != steps:
            raise RuntimeError(f"TP ranks diverged: rank 0 took {cmds['steps']} steps, this rank {steps}")
        for op, args in cmds["ops"]:
            getattr(engine, op)(*args)
        for prompt, params, mm in cmds["reqs"]:
            engine.add_request(prompt, params, mm=mm)
        if engine.has_work():
            engine.step()
            steps += 1


def _sampling(body: dict, default_max: int = 256, eos_ids=()) -> SamplingParams:
    """Request fields -> SamplingParams; generation stops at the tokenizer's end-of-sequence / end-of-turn ids
    (unless `ignore_eos`) and at any of `stop_token_ids`."""
    stop = [int(t) for t in (body.get("stop_token_ids") or [])]
    if not body.get("ignore_eos"):
        stop += [int(t) for t in eos_ids if t is not None]
    return SamplingParams(temperature=float(body.get("temperature", 0.0) or 0.0),
                          top_k=int(body.get("top_k", 0) or 0), top_p=float(body.get("top_p", 1.0) or 1.0),
                          seed=int(body.get("seed", 42) if body.get("seed") is not None else 42),
                          max_new_tokens=int(body.get("max_tokens", body.get("max_completion_tokens", default_max))
                                             or default_max),
                          stop_token_ids=tuple(stop))


def _stop_strings(body: dict) -> List[str]:
    s = body.get("stop")
    if not s:
        return []
    return [s] if isinstance(s, str) else [x for x in s if isinstance(x, str) and x]


def _cut_at_stop(text: str, stops: List[str]) -> Optional[int]:
    """Index where the earliest stop string starts in `text`, or None."""
    hits = [i for i in (text.find(x) for x in stops) if i >= 0]
    return min(hits) if hits else None


class UnknownImage(Exception):
    """A content part referenced an image uuid the encoder cache does not hold (evicted or never sent)."""


def encode_chat(tokenizer, messages: List[dict], vision=None, vocab: int = 0):
    """Chat messages -> (token ids, image inputs [(position, features)]). Without image parts this is the
    tokenizer's chat template. With them (and a vision encoder) each message is laid out as the role header, its
    text parts, and for each image part the image's placeholder ids (models/vision.py), whose rows prefill
    feeds with the image features. An image part is {"type": "image_url", "image_url": {"url": "data:..."}}
    with an optional "uuid" (the client's key), or {"type": "image_url", "uuid": ...} alone for an image sent
    before."""
    has_image = any(isinstance(m.get("content"), list) and any(isinstance(p, dict) and p.get("type") == "image_url"
                                                                for p in m["content"]) for m in messages)
    if not has_image or vision is None:
        return tokenizer.encode(tokenizer.apply_chat_template(messages)), []
    from ..models.vision import image_placeholders
    ids: List[int] = []
    mm = []
    for m in messages:
        ids += tokenizer.encode(f"<|{m.get('role', 'user')}|>\n")
        c = m.get("content", "")
        parts = c if isinstance(c, list) else [{"type": "text", "text": c}]
        for p in parts:
            if not isinstance(p, dict):
                continue
            if p.get("type") == "image_url":
                url = (p.get("image_url") or {}).get("url")
                key = p.get("uuid")
                if url:
                    digest, feats = vision.encode(url, digest=key)
                else:
                    feats = vision.lookup(key) if key else None
                    digest = key
                    if feats is None:
                        raise UnknownImage(key)
                mm.append((len(ids), feats))
                ids += image_placeholders(digest, feats.shape[0], vocab)
            elif p.get("type") == "text":
                ids += tokenizer.encode(p.get("text", ""))
        ids += tokenizer.encode("\n")
    ids += tokenizer.encode("<|assistant|>\n")
    return ids, mm


def build_app(aeng: AsyncEngine, tokenizer, model_name: str = "phung5_b200", vision=None):
    app = FastAPI(title="phung5_b200")

    @app.get("/health")
    async def health():
        if aeng.error or aeng.engine.sleeping:
            return JSONResponse({"status": "unavailable", "error": aeng.error, "sleeping": aeng.engine.sleeping},
                                status_code=503)
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "phung5_b200"}]}

    @app.get("/get_load")
    async def get_load():
        return aeng.load()

    @app.get("/metrics")
    async def metrics():
        return PlainTextResponse(aeng.metrics.render(), media_type="text/plain; version=0.0.4")

    async def _control(op):
        await aeng.control(op)
        return {"ok": True, "sleeping": aeng.engine.sleeping}

    @app.post("/sleep")
    async def sleep():
        return await _control("sleep")

    @app.post("/wake_up")
    async def wake_up():
        return await _control("wake_up")

    @app.post("/release_memory_occupation")
    async def release():
        return await _control("sleep")

    @app.post("/resume_memory_occupation")
    async def resume():
        return await _control("wake_up")

    async def _complete(ids: List[int], body: dict, chat: bool, mm: Optional[list] = None):
        sp = _sampling(body, eos_ids=getattr(tokenizer, "stop_ids", None) or [getattr(tokenizer, "eos_id", None)])
        stops = _stop_strings(body)
        rid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex[:16]}"
        created = int(time.time())

        async def pieces():
            """(text delta, token ids, finish reason or None); a stop string ends the text before it and the
            request (leaving the generator aborts it in the engine)."""
            toks: List[int] = []
            sent = 0
            gen = aeng.generate(ids, sp, mm)
            try:
                async for o in gen:
                    toks += o.new_tokens
                    text = tokenizer.decode(toks)
                    cut = _cut_at_stop(text, stops) if stops else None
                    if cut is not None:
                        yield text[sent:cut], o.new_tokens, "stop"
                        return
                    # hold back a tail that could still grow into a stop string
                    hold = max((len(x) - 1 for x in stops), default=0)
                    upto = len(text) if o.finished else max(sent, len(text) - hold)
                    yield text[sent:upto], o.new_tokens, (o.finish_reason or "length") if o.finished else None
                    sent = upto
                    if o.finished:
                        return
            finally:
                await gen.aclose()

        if body.get("stream"):
            async def events():
                async for text, new, fin in pieces():
                    if chat:
                        chunk = {"id": rid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                                 "choices": [{"index": 0, "delta": {"content": text}, "finish_reason": fin}]}
                    else:
                        chunk = {"id": rid, "object": "text_completion", "created": created, "model": model_name,
                                 "choices": [{"index": 0, "text": text, "token_ids": new, "finish_reason": fin}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(events(), media_type="text/event-stream")
        parts, toks, fin = [], [], "length"
        async for text, new, f in pieces():
            parts.append(text)
            toks += new
            fin = f or fin
        text = "".join(parts)
        usage = {"prompt_tokens": len(ids), "completion_tokens": len(toks), "total_tokens": len(ids) + len(toks)}
        if chat:
            return {"id": rid, "object": "chat.completion", "created": created, "model": model_name,
                    "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                                 "finish_reason": fin}], "usage": usage}
        return {"id": rid, "object": "text_completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "text": text, "token_ids": toks, "finish_reason": fin}], "usage": usage}

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        prompt = body.get("prompt", "")
        ids = list(prompt) if isinstance(prompt, list) else tokenizer.encode(prompt)
        if not ids:
            return JSONResponse({"error": "empty prompt"}, status_code=400)
        return await _complete(ids, body, chat=False)

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        try:
            ids, mm = encode_chat(tokenizer, body.get("messages", []), vision, aeng.engine.cfg.model.vocab)
        except UnknownImage as e:
            return JSONResponse({"error": f"unknown image uuid {e.args[0]!r}: send the image in full"},
                                status_code=400)
        return await _complete(ids, body, chat=True, mm=mm)

    return app


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="small-bf16")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8001)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--spec", default="tree", choices=["off", "chain", "tree"])
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--model-path", default=None,
                    help="HF checkpoint directory (config.json + safetensors); overrides --model's random weights")
    ap.add_argument("--draft-path", default=None, help="EAGLE head checkpoint directory (else a random head)")
    ap.add_argument("--vision", action="store_true", help="serve image inputs with a (seeded random) vision tower")
    ap.add_argument("--num-pages", type=int, default=0)
    ap.add_argument("--max-num-seqs", type=int, default=256,
                    help="requests decoded at once; more wait (admission also waits for KV pages)")
    ap.add_argument("--comm", default="fused", choices=["nccl", "fused"],
                    help="tensor-parallel collectives when launched with torchrun over several GPUs")
    args = ap.parse_args(argv)
    import os

    import uvicorn
    from ..config import CacheConfig, DraftConfig, EngineConfig, ParallelConfig, SpecConfig, preset
    from ..engine.engine import LLMEngine
    world = int(os.environ.get("WORLD_SIZE", "1"))
    comm, group, device = None, None, args.device
    if world > 1:
        import torch.distributed as dist
        from ..parallel.comm import NcclCommunicator, init_distributed
        rank, world, local = init_distributed()
        device = f"cuda:{local}"
        comm = NcclCommunicator()
        if args.comm == "fused":
            from ..parallel.fused import FusedCommunicator
            comm = FusedCommunicator()
        group = dist.new_group(backend="gloo")
    spec = SpecConfig(enabled=args.spec != "off", mode=args.spec if args.spec != "off" else "chain")
    target = drafter = None
    model_cfg = preset(args.model) if args.model_path is None else None
    if args.model_path is not None:
        from ..weights.loader import load_eagle, load_model
        rank_ = comm.rank if comm is not None else 0
        model_cfg, target = load_model(args.model_path, device, rank_, world)
        if args.draft_path is not None:
            drafter = load_eagle(args.draft_path, model_cfg, device, rank_, world)
    cfg = EngineConfig(model=model_cfg, spec=spec, draft=DraftConfig(kind="eagle"),
                       cache=CacheConfig(num_pages=args.num_pages), parallel=ParallelConfig(tp=world, comm=args.comm),
                       max_running=args.max_num_seqs)
    eng = LLMEngine(cfg, device=device, comm=comm, target=target, drafter=drafter)
    if group is not None and comm.rank != 0:
        tp_worker_loop(eng, group)
        return
    aeng = AsyncEngine(eng, group=group)
    vision = None
    if args.vision:
        import torch
        from ..models.vision import VisionConfig, VisionEncoder
        vision = VisionEncoder(VisionConfig(out_hidden=model_cfg.hidden), device=device,
                               dtype=torch.bfloat16 if str(device).startswith("cuda") else torch.float32)
    from .tokenizer import has_tokenizer, load_tokenizer
    tok_path = args.tokenizer or (args.model_path if has_tokenizer(args.model_path) else None)
    uvicorn.run(build_app(aeng, load_tokenizer(tok_path), model_cfg.name if args.model_path else args.model,
                          vision=vision), host=args.host, port=args.port, log_level="warning")
    aeng.shutdown()


if __name__ == "__main__":
    main()
