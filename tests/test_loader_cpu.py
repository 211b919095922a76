"""HF safetensors checkpoints (weights/loader.py) on CPU: config.json -> ModelConfig, a sharded checkpoint
read lazily packs exactly the tensors of the in-memory path (bf16/fp32 and fp8 block-scaled), per-channel fp8
is requantized within one e4m3 step, the EAGLE head loads from its own directory, and two gloo ranks each
reading only their shard produce the single-rank engine's greedy output."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.models.llama import pack_weights
from phung5_b200.weights.init import random_eagle_weights, random_weights
from phung5_b200.weights.loader import Checkpoint, load_config, load_eagle, open_checkpoint, save_checkpoint


def _packed_equal(a, b):
    assert torch.equal(a.embed, b.embed) and torch.equal(a.lm_head, b.lm_head)
    assert torch.equal(a.final_norm, b.final_norm)
    for la, lb in zip(a.layers, b.layers):
        for name in ("qkv", "o", "gu", "down"):
            x, y = getattr(la, name), getattr(lb, name)
            assert torch.equal(x.w.float(), y.w.float()), name
            assert (x.ws is None) == (y.ws is None) and (x.ws is None or torch.equal(x.ws, y.ws))
        assert torch.equal(la.in_norm, lb.in_norm) and torch.equal(la.post_norm, lb.post_norm)


@pytest.mark.parametrize("name,shards", [("tiny", 1), ("tiny", 3), ("small-fp8", 2)])
def test_checkpoint_round_trip_packs_identically(tmp_path, name, shards):
    cfg = preset(name)
    hf = random_weights(cfg, seed=0, std=0.05)
    if cfg.quant != "fp8_block":
        hf = {k: v.bfloat16() for k, v in hf.items()}
    save_checkpoint(hf, cfg, str(tmp_path), shards=shards)
    assert (shards > 1) == os.path.exists(tmp_path / "model.safetensors.index.json")
    mc = load_config(str(tmp_path))
    for f in ("num_layers", "hidden", "num_heads", "num_kv_heads", "head_dim", "ffn", "vocab", "quant",
              "rope_theta", "rms_eps"):
        assert getattr(mc, f) == getattr(cfg, f), f
    mc, ck = open_checkpoint(str(tmp_path))
    assert set(ck) == set(hf)
    for rank, world in ((0, 1), (0, 2), (1, 2)):
        _packed_equal(pack_weights(cfg, ck, "cpu", rank, world), pack_weights(cfg, hf, "cpu", rank, world))


def test_lazy_slices_read_only_the_shard(tmp_path):
    cfg = preset("tiny")
    hf = random_weights(cfg, seed=1)
    save_checkpoint(hf, cfg, str(tmp_path), shards=2)
    ck = Checkpoint(str(tmp_path))
    t = ck["model.layers.0.mlp.down_proj.weight"]
    assert t.shape == hf["model.layers.0.mlp.down_proj.weight"].shape
    assert torch.equal(t[:, 100:200], hf["model.layers.0.mlp.down_proj.weight"][:, 100:200])
    assert torch.equal(t[3:9], hf["model.layers.0.mlp.down_proj.weight"][3:9])


def test_per_channel_fp8_is_requantized_to_block_scales(tmp_path):
    from safetensors.torch import save_file
    from phung5_b200.models.reference import dequant_block_fp8 as dequant_weight_block
    from phung5_b200.weights.quant import FP8_DTYPE
    cfg = preset("small-fp8")
    hf = random_weights(cfg, seed=2, std=0.05, fp8=False)
    out, ref = {}, {}
    for k, v in hf.items():
        if k.endswith("proj.weight"):
            s = v.abs().amax(1, keepdim=True) / 448.0           # per output channel
            q = (v / s).to(FP8_DTYPE)
            out[k], out[k[:-len("weight")] + "weight_scale"] = q, s.float()
            ref[k] = q.float() * s
        else:
            out[k] = v.bfloat16()
    save_checkpoint({}, cfg, str(tmp_path))
    os.remove(tmp_path / "model.safetensors")
    save_file(out, str(tmp_path / "model.safetensors"))
    ck = Checkpoint(str(tmp_path))
    assert not any(k.endswith("weight_scale") for k in ck)
    w = pack_weights(cfg, ck, "cpu")
    lin = w.layers[0].o
    got = dequant_weight_block(lin.w, lin.ws)
    want = ref["model.layers.0.self_attn.o_proj.weight"]
    rel = ((got - want).abs() / want.abs().clamp(min=1e-3)).max().item()
    assert rel <= 1 / 8 + 1e-6, rel            # one extra e4m3 rounding at most


def test_eagle_head_loads_from_its_directory(tmp_path):
    from phung5_b200.models.eagle import pack_eagle
    cfg = preset("tiny")
    ew = random_eagle_weights(cfg, seed=3, std=0.05)
    plain = {k[len("eagle."):]: v.bfloat16() for k, v in ew.items()}       # EAGLE checkpoint names
    save_checkpoint(plain, cfg, str(tmp_path), shards=1)
    got = load_eagle(str(tmp_path), cfg, "cpu")
    want = pack_eagle(cfg, {k: v.bfloat16() for k, v in ew.items()}, "cpu")
    assert torch.equal(got.fc.w, want.fc.w) and torch.equal(got.norm, want.norm)
    assert torch.equal(got.layer.qkv.w, want.layer.qkv.w)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, path, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phung5_b200.engine.engine import LLMEngine
        from phung5_b200.engine.oracle import SamplingParams
        from phung5_b200.parallel.comm import NcclCommunicator
        from phung5_b200.weights.loader import load_model
        comm = NcclCommunicator() if world > 1 else None
        mc, tw = load_model(path, "cpu", rank, world)
        dw = pack_weights(preset("tiny-draft"), random_weights(preset("tiny-draft"), seed=1, std=0.05), "cpu", rank,
                          world, dtype=torch.float32)
        tw32 = pack_weights(mc, {k: v for k, v in Checkpoint(path).items()}, "cpu", rank, world, dtype=torch.float32)
        ecfg = EngineConfig(model=mc, spec=SpecConfig(mode="chain", num_draft=3), draft=DraftConfig(kind="model"),
                            cache=CacheConfig(page_size=16, num_pages=200))
        eng = LLMEngine(ecfg, device="cpu", target=tw32, drafter=dw, comm=comm, dtype=torch.float32,
                        max_context=1024)
        g = torch.Generator().manual_seed(3)
        prompts = [torch.randint(0, mc.vocab, (40,), generator=g).tolist() for _ in range(2)]
        q.put((rank, eng.generate(prompts, SamplingParams(max_new_tokens=12)), tw.layers[0].qkv.w.shape))
    finally:
        if world > 1:
            dist.destroy_process_group()


def test_tp2_gloo_ranks_load_their_shards_and_match_tp1(tmp_path):
    cfg = preset("tiny")
    save_checkpoint(random_weights(cfg, seed=0, std=0.05), cfg, str(tmp_path), shards=2)
    ctx = mp.get_context("spawn")
    res = {}
    for world in (1, 2):
        q = ctx.Queue()
        port = _port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), q)) for r in range(world)]
        for p in procs:
            p.start()
        got = sorted(q.get(timeout=240) for _ in range(world))
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
        res[world] = got
    assert res[2][0][1] == res[2][1][1] == res[1][0][1]           # same greedy tokens on every rank and at TP1
    assert res[2][0][2][0] * 2 == res[1][0][2][0]                  # each rank packed half of the qkv rows
