"""Serving a checkpoint over HTTP on the GPU: a small block-scaled FP8 Llama-shaped checkpoint and its EAGLE
head are written as HF safetensors directories, `python -m phung5_b200.serve.server --model-path ...
--draft-path ...` serves them, and a greedy completion returns exactly the tokens of an in-process engine
built from the same weights in memory."""
import os
import socket
import subprocess
import sys
import time

import httpx
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_server_serves_a_safetensors_checkpoint(tmp_path):
    from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
    from phung5_b200.engine.engine import LLMEngine
    from phung5_b200.engine.oracle import SamplingParams
    from phung5_b200.models.eagle import pack_eagle
    from phung5_b200.models.llama import pack_weights
    from phung5_b200.weights.init import random_eagle_weights, random_weights
    from phung5_b200.weights.loader import save_checkpoint
    cfg = preset("small-fp8")
    hf = random_weights(cfg, seed=0, std=0.05)
    ew = random_eagle_weights(cfg, seed=1, std=0.05)
    save_checkpoint(hf, cfg, str(tmp_path / "model"), shards=2)
    save_checkpoint({k[len("eagle."):]: v for k, v in ew.items()}, cfg, str(tmp_path / "eagle"))
    prompt = torch.randint(0, cfg.vocab, (90,), generator=torch.Generator().manual_seed(9)).tolist()

    ecfg = EngineConfig(model=cfg, spec=SpecConfig(mode="tree"), draft=DraftConfig(kind="eagle"),
                        cache=CacheConfig(num_pages=256))
    eng = LLMEngine(ecfg, device="cuda", target=pack_weights(cfg, hf, "cuda"), drafter=pack_eagle(cfg, ew, "cuda"))
    want = eng.generate([prompt], SamplingParams(max_new_tokens=16))[0]
    del eng
    torch.cuda.empty_cache()

    port = _port()
    proc = subprocess.Popen([sys.executable, "-m", "phung5_b200.serve.server", "--model-path", str(tmp_path / "model"),
                             "--draft-path", str(tmp_path / "eagle"), "--port", str(port), "--num-pages", "256",
                             "--spec", "tree"], cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    try:
        t0 = time.time()
        while True:
            assert proc.poll() is None, proc.stdout.read().decode()[-2000:]
            try:
                if httpx.get(f"http://127.0.0.1:{port}/health", timeout=2).status_code == 200:
                    break
            except httpx.HTTPError:
                pass
            assert time.time() - t0 < 240, "server did not come up"
            time.sleep(1)
        r = httpx.post(f"http://127.0.0.1:{port}/v1/completions",
                       json={"prompt": prompt, "max_tokens": 16, "temperature": 0, "ignore_eos": True}, timeout=120)
        assert r.status_code == 200, r.text
        assert r.json()["choices"][0]["token_ids"] == want
    finally:
        proc.terminate()
        try:
            proc.wait(timeout=30)
        except subprocess.TimeoutExpired:
            proc.kill()
