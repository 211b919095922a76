"""Image inputs on CPU: the vision tower's features replace the placeholder rows' embeddings in prefill, so the
engine's speculative output equals the fp32 oracle's greedy decode with the same rows injected; the encoder
cache serves repeated images; the HTTP chat endpoint takes image parts in full or by uuid, answers 400 for an
unknown uuid, and the client's send-once-then-by-uuid backend recovers by resending in full."""
import base64
import io

import numpy as np
import pytest
import torch
from starlette.testclient import TestClient

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import SamplingParams, greedy_generate
from phung5_b200.models.llama import pack_weights
from phung5_b200.models.reference import RefModel
from phung5_b200.models.vision import VisionConfig, VisionEncoder, image_placeholders
from phung5_b200.weights.init import random_weights


def _png(seed, size=48):
    from PIL import Image
    g = np.random.default_rng(seed)
    arr = (g.random((size, size, 3)) * 255).astype(np.uint8)
    buf = io.BytesIO()
    Image.fromarray(arr).save(buf, format="PNG")
    return "data:image/png;base64," + base64.b64encode(buf.getvalue()).decode()


def _engine():
    tcfg, dcfg = preset("tiny"), preset("tiny-draft")
    tw, dw = random_weights(tcfg, seed=0, std=0.05), random_weights(dcfg, seed=1, std=0.05)
    cfg = EngineConfig(model=tcfg, spec=SpecConfig(mode="chain", num_draft=3), draft=DraftConfig(kind="model"),
                       cache=CacheConfig(page_size=16, num_pages=256))
    eng = LLMEngine(cfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", dtype=torch.float32),
                    drafter=pack_weights(dcfg, dw, "cpu", dtype=torch.float32), dtype=torch.float32,
                    max_context=1024)
    vis = VisionEncoder(VisionConfig(image_size=56, patch=14, merge=2, out_hidden=tcfg.hidden))
    return eng, vis, RefModel(tcfg, tw)


def test_image_rows_feed_prefill_and_match_the_oracle():
    eng, vis, ref = _engine()
    outs = {}
    for name, url in (("a", _png(1)), ("b", _png(2))):
        digest, feats = vis.encode(url)
        assert feats.shape == (4, 256)
        ph = image_placeholders(digest, feats.shape[0], eng.cfg.model.vocab)
        prompt = list(range(20, 40)) + ph + list(range(50, 60))
        out = eng.generate([prompt], SamplingParams(max_new_tokens=10))
        rid = eng.add_request(prompt, SamplingParams(max_new_tokens=10), mm=[(20, feats)])
        while eng.has_work():
            eng.step()
        with_img = eng.reqs[rid].out
        want = greedy_generate(ref, prompt, 10, embeds=(torch.arange(20, 24), feats))
        assert with_img == want                        # speculative output = target greedy with the image rows
        assert with_img != out[0]                      # the features, not the placeholder embeddings, were used
        outs[name] = with_img
    assert outs["a"] != outs["b"]
    _, again = vis.encode(_png(1))
    assert vis.stats["encoded"] == 2 and vis.stats["hits"] == 1


def test_chat_with_image_parts_and_uuid_resend():
    from phung5_b200.app.session import ImageResendBackend
    from phung5_b200.serve.server import AsyncEngine, build_app
    from phung5_b200.serve.tokenizer import ByteTokenizer
    eng, vis, _ = _engine()
    aeng = AsyncEngine(eng)
    app = build_app(aeng, ByteTokenizer(), "tiny", vision=vis)
    url = _png(3)
    msg = lambda part: {"messages": [{"role": "user", "content": [{"type": "text", "text": "what is this?"}, part]}],
                        "max_tokens": 6, "temperature": 0}
    try:
        with TestClient(app) as c:
            full = c.post("/v1/chat/completions", json=msg({"type": "image_url", "uuid": "k1",
                                                            "image_url": {"url": url}}))
            assert full.status_code == 200, full.text
            by_ref = c.post("/v1/chat/completions", json=msg({"type": "image_url", "uuid": "k1", "image_url": None}))
            assert by_ref.status_code == 200
            assert by_ref.json()["choices"][0]["message"] == full.json()["choices"][0]["message"]
            assert vis.stats["encoded"] == 1 and vis.stats["hits"] >= 1
            missing = c.post("/v1/chat/completions", json=msg({"type": "image_url", "uuid": "nope", "image_url": None}))
            assert missing.status_code == 400

            class Inner:       # the client backend over this app: a 400 raises BackendError
                async def chat(self, body):
                    from phung5_b200.app.session import BackendError
                    r = c.post("/v1/chat/completions", json=body)
                    if r.status_code != 200:
                        raise BackendError(r.status_code, r.text)
                    return r.json()
            import asyncio
            be = ImageResendBackend(Inner())
            body = msg({"type": "image_url", "image_url": {"url": _png(4)}})
            asyncio.run(be.chat(body))
            vis.cache.clear()                             # the server evicts the image
            out = asyncio.run(be.chat(body))              # compact send -> 400 -> full resend
            assert be.resends == 1 and out["choices"][0]["message"]["content"] is not None
    finally:
        aeng.shutdown()
