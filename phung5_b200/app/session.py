"""LLM session layer: chat loop with tool calls and schema-validated replies over any OpenAI-compatible backend.

Reference: `SessionAgent` (pipeline_service/llm/session.py:45-316), `SessionStore` (llm/session_store.py:8-65),
`Tool` (llm/tools.py:24-62), `async_retry` (utils/retry.py:11-39) and the image re-send rewriter
(llm/mm_resend.py:81-170).

Backends implement one coroutine, `chat(body: dict) -> dict` (an OpenAI chat-completions response):
`HTTPBackend` posts to one server, `phung5_b200.serve.router.LoadBalancedClient` spreads calls over replicas
with per-task affinity, and tests pass a stub. Every call is timed and its token usage recorded in the
backend-independent `CallLog`, which batch statistics read.

Behaviour kept from the reference:
- tool calls loop until the model answers without one (bounded turns);
- a reply that fails the pydantic schema is answered with the validation error and retried (bounded);
- a context-overflow 400 lowers `max_tokens` to what the prompt leaves and retries once;
- transport errors retry with exponential backoff, except timeouts (a slow server is not helped by more load).
"""
from __future__ import annotations

import asyncio
import contextvars
import hashlib
import json
import re
import time
import uuid
from dataclasses import dataclass, field
from typing import Any, Awaitable, Callable, Dict, List, Optional, Type

import httpx

try:
    from pydantic import BaseModel, ValidationError
except ImportError:  # pragma: no cover - pydantic ships with fastapi
    BaseModel = object
    ValidationError = Exception


class BackendError(Exception):
    def __init__(self, status: int, body: str):
        super().__init__(f"HTTP {status}: {body[:300]}")
        self.status = status
        self.body = body


# --------------------------------------------------------------------------------------------------- retry


async def async_retry(fn: Callable[[], Awaitable], attempts: int = 3, base_delay: float = 0.5,
                      no_retry: tuple = (asyncio.TimeoutError, httpx.TimeoutException), on_retry=None):
    """Await fn() up to `attempts` times with exponential backoff; exceptions in `no_retry` propagate at once."""
    for k in range(attempts):
        try:
            return await fn()
        except no_retry:
            raise
        except asyncio.CancelledError:
            raise
        except Exception as e:  # noqa: BLE001 - retried, then re-raised
            if isinstance(e, BackendError) and 400 <= e.status < 500 and e.status not in (408, 429):
                raise
            if k == attempts - 1:
                raise
            if on_retry is not None:
                on_retry(k, e)
            await asyncio.sleep(base_delay * (2 ** k))


# ------------------------------------------------------------------------------------------------ backends


@dataclass
class CallRecord:
    client: str
    seconds: float
    prompt_tokens: int
    completion_tokens: int
    ok: bool
    purpose: str = ""


class CallLog:
    """Append-only record of LLM calls (read by batch statistics)."""

    def __init__(self):
        self.records: List[CallRecord] = []

    def add(self, rec: CallRecord):
        self.records.append(rec)

    def since(self, idx: int) -> List[CallRecord]:
        return self.records[idx:]

    def summary(self, records: Optional[List[CallRecord]] = None) -> Dict[str, Dict[str, float]]:
        out: Dict[str, Dict[str, float]] = {}
        for r in (self.records if records is None else records):
            s = out.setdefault(r.client, {"calls": 0, "errors": 0, "seconds": 0.0, "prompt_tokens": 0,
                                          "completion_tokens": 0})
            s["calls"] += 1
            s["errors"] += 0 if r.ok else 1
            s["seconds"] += r.seconds
            s["prompt_tokens"] += r.prompt_tokens
            s["completion_tokens"] += r.completion_tokens
        return out


CALL_LOG = CallLog()
purpose_var: contextvars.ContextVar[str] = contextvars.ContextVar("llm_purpose", default="")


class HTTPBackend:
    """One OpenAI-compatible server."""

    def __init__(self, base_url: str, timeout: float = 600.0, client: Optional[httpx.AsyncClient] = None,
                 api_key: Optional[str] = None):
        self.url = base_url.rstrip("/")
        self.http = client or httpx.AsyncClient(timeout=httpx.Timeout(timeout, connect=10.0))
        self.headers = {"Authorization": f"Bearer {api_key}"} if api_key else {}

    async def chat(self, body: dict) -> dict:
        r = await self.http.post(self.url + "/v1/chat/completions", json=body, headers=self.headers)
        if r.status_code >= 400:
            raise BackendError(r.status_code, r.text)
        return r.json()


class InstrumentedBackend:
    """Wraps a backend: times each call and logs usage under `name`."""

    def __init__(self, inner, name: str, log: CallLog = CALL_LOG):
        self.inner, self.name, self.log = inner, name, log

    async def chat(self, body: dict) -> dict:
        t0 = time.monotonic()
        ok, usage = False, {}
        try:
            out = await self.inner.chat(body)
            usage = out.get("usage") or {}
            ok = True
            return out
        finally:
            self.log.add(CallRecord(self.name, time.monotonic() - t0, int(usage.get("prompt_tokens", 0)),
                                    int(usage.get("completion_tokens", 0)), ok, purpose_var.get()))


class ImageResendBackend:
    """Sends each image once, then by reference.

    The first request carrying a data-URL image sends it in full with a `uuid` (the sha1 of the data); later
    requests replace the URL by that uuid so the server's multimodal processor cache serves it without the
    payload. A 400 answer (the server has evicted it) resends the request in full and forgets the uuids.
    """

    def __init__(self, inner):
        self.inner = inner
        self.sent: set = set()
        self.resends = 0

    @staticmethod
    def _key(url: str) -> str:
        return hashlib.sha1(url.encode()).hexdigest()

    def _rewrite(self, body: dict, compact: bool) -> tuple:
        keys = []
        msgs = []
        for m in body.get("messages", []):
            c = m.get("content")
            if not isinstance(c, list):
                msgs.append(m)
                continue
            parts = []
            for p in c:
                if p.get("type") == "image_url":
                    url = (p.get("image_url") or {}).get("url", "")
                    if url.startswith("data:"):
                        k = self._key(url)
                        keys.append(k)
                        if compact and k in self.sent:
                            parts.append({"type": "image_url", "uuid": k, "image_url": None})
                            continue
                        parts.append({"type": "image_url", "uuid": k, "image_url": {"url": url}})
                        continue
                parts.append(p)
            msgs.append({**m, "content": parts})
        return {**body, "messages": msgs}, keys

    async def chat(self, body: dict) -> dict:
        compact, keys = self._rewrite(body, compact=True)
        try:
            out = await self.inner.chat(compact)
        except BackendError as e:
            if e.status != 400 or not any(k in self.sent for k in keys):
                raise
            self.resends += 1
            self.sent.difference_update(keys)
            full, _ = self._rewrite(body, compact=False)
            out = await self.inner.chat(full)
        self.sent.update(keys)
        return out


# ----------------------------------------------------------------------------------------------------- tools


@dataclass
class Tool:
    name: str
    description: str
    parameters: Dict[str, Any]
    fn: Callable[..., Any]

    def spec(self) -> dict:
        return {"type": "function", "function": {"name": self.name, "description": self.description,
                                                 "parameters": self.parameters}}

    async def call(self, arguments: str) -> str:
        try:
            args = json.loads(arguments or "{}")
        except json.JSONDecodeError as e:
            return json.dumps({"error": f"arguments are not JSON: {e}"})
        try:
            r = self.fn(**args)
            if asyncio.iscoroutine(r):
                r = await r
        except Exception as e:  # noqa: BLE001 - reported to the model
            return json.dumps({"error": f"{type(e).__name__}: {e}"})
        return r if isinstance(r, str) else json.dumps(r)


# --------------------------------------------------------------------------------------------------- sessions


_JSON_FENCE = re.compile(r"```(?:json)?\s*\n(.*?)```", re.S)


def extract_json(text: str):
    """The JSON object of a reply: a fenced block, else the outermost {...} span."""
    m = _JSON_FENCE.search(text or "")
    if m:
        return json.loads(m.group(1))
    s = (text or "").strip()
    if s.startswith("{") or s.startswith("["):
        return json.loads(s)
    i, j = s.find("{"), s.rfind("}")
    if i >= 0 and j > i:
        return json.loads(s[i:j + 1])
    raise json.JSONDecodeError("no JSON object in reply", s, 0)


_CTX_LIMIT = re.compile(r"maximum context length is (\d+)", re.I)
_CTX_USED = re.compile(r"(\d+) in the messages|(\d+) (?:input|prompt) tokens|prompt contains (\d+)", re.I)


def context_overflow(body: str):
    """(context limit, prompt tokens) from an OpenAI-style context-length error, or None."""
    m, u = _CTX_LIMIT.search(body or ""), _CTX_USED.search(body or "")
    if not m or not u:
        return None
    return int(m.group(1)), int(next(g for g in u.groups() if g))


class SessionStore:
    """Conversation histories by session id (critic/refine loops continue a coder's conversation)."""

    def __init__(self, max_sessions: int = 4096):
        self.data: Dict[str, List[dict]] = {}
        self.max = max_sessions

    def get(self, sid: str) -> List[dict]:
        return list(self.data.get(sid, []))

    def put(self, sid: str, messages: List[dict]) -> None:
        if sid not in self.data and len(self.data) >= self.max:
            self.data.pop(next(iter(self.data)))
        self.data[sid] = list(messages)

    def drop(self, sid: str) -> None:
        self.data.pop(sid, None)

    def new_id(self) -> str:
        return uuid.uuid4().hex


@dataclass
class SessionResult:
    content: str
    parsed: Any = None
    messages: List[dict] = field(default_factory=list)
    turns: int = 0
    usage: Dict[str, int] = field(default_factory=dict)


class SessionAgent:
    """One model role (coder, judge, critic, planner) with its system prompt, tools and reply schema."""

    def __init__(self, backend, model: str, system: str = "", tools: Optional[List[Tool]] = None,
                 schema: Optional[Type] = None, max_tokens: int = 4096, temperature: float = 0.7,
                 top_p: float = 1.0, max_turns: int = 8, validation_retries: int = 2, transport_retries: int = 3,
                 timeout: float = 600.0, extra_body: Optional[dict] = None):
        self.backend, self.model, self.system = backend, model, system
        self.tools = {t.name: t for t in (tools or [])}
        self.schema = schema
        self.max_tokens, self.temperature, self.top_p = max_tokens, temperature, top_p
        self.max_turns, self.validation_retries, self.transport_retries = max_turns, validation_retries, transport_retries
        self.timeout = timeout
        self.extra_body = extra_body or {}

    def _body(self, messages, max_tokens, seed) -> dict:
        body = {"model": self.model, "messages": messages, "max_tokens": max_tokens, "temperature": self.temperature,
                "top_p": self.top_p, **self.extra_body}
        if seed is not None:
            body["seed"] = int(seed)
        if self.tools:
            body["tools"] = [t.spec() for t in self.tools.values()]
        return body

    async def _call(self, messages, seed) -> dict:
        max_tokens = self.max_tokens
        for _ in range(2):
            try:
                return await async_retry(lambda: asyncio.wait_for(self.backend.chat(self._body(messages, max_tokens, seed)),
                                                                  self.timeout), attempts=self.transport_retries)
            except BackendError as e:
                ov = context_overflow(e.body)
                if e.status == 400 and ov:
                    limit, used = ov
                    room = limit - used - 16
                    if room <= 64 or room >= max_tokens:
                        raise
                    max_tokens = room
                    continue
                raise
        raise RuntimeError("unreachable")

    async def run(self, user: Any, history: Optional[List[dict]] = None, seed: Optional[int] = None) -> SessionResult:
        messages: List[dict] = list(history or [])
        if self.system and not (messages and messages[0].get("role") == "system"):
            messages.insert(0, {"role": "system", "content": self.system})
        messages.append({"role": "user", "content": user})
        usage = {"prompt_tokens": 0, "completion_tokens": 0}
        bad_replies = 0
        for turn in range(1, self.max_turns + 1):
            out = await self._call(messages, None if seed is None else seed + turn - 1)
            u = out.get("usage") or {}
            usage["prompt_tokens"] += int(u.get("prompt_tokens", 0))
            usage["completion_tokens"] += int(u.get("completion_tokens", 0))
            msg = (out.get("choices") or [{}])[0].get("message") or {}
            calls = msg.get("tool_calls") or []
            content = msg.get("content") or ""
            if calls and self.tools:
                messages.append({"role": "assistant", "content": content, "tool_calls": calls})
                for c in calls:
                    fn = c.get("function", {})
                    tool = self.tools.get(fn.get("name"))
                    res = await tool.call(fn.get("arguments", "{}")) if tool else json.dumps(
                        {"error": f"unknown tool {fn.get('name')}"})
                    messages.append({"role": "tool", "tool_call_id": c.get("id", ""), "content": res})
                continue
            messages.append({"role": "assistant", "content": content})
            if self.schema is None:
                return SessionResult(content, None, messages, turn, usage)
            try:
                parsed = self.schema.model_validate(extract_json(content))
                return SessionResult(content, parsed, messages, turn, usage)
            except (json.JSONDecodeError, ValidationError, ValueError) as e:
                bad_replies += 1
                if bad_replies > self.validation_retries:
                    raise ValueError(f"reply failed the {self.schema.__name__} schema {bad_replies} times: {e}") from e
                messages.append({"role": "user", "content": f"Your reply did not match the required JSON schema: "
                                                            f"{str(e)[:600]}. Reply again with only the JSON object."})
        raise RuntimeError(f"no final answer within {self.max_turns} turns")
