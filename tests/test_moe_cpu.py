"""Mixtral-style MoE on CPU: the engine's grouped-expert block (device-side sort by expert, grouped
GEMMs, select-based combine) against the per-expert fp32 oracle, single rank and 2-rank expert
parallelism (gloo)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
from phung5_b200.engine.engine import LLMEngine
from phung5_b200.engine.oracle import SamplingParams, greedy_generate
from phung5_b200.models.llama import pack_weights
from phung5_b200.models.reference import RefModel, moe_mlp
from phung5_b200.weights.init import random_weights

F32 = torch.float32


def test_moe_block_matches_oracle():
    cfg = preset("tiny-moe")
    w = random_weights(cfg, seed=0, std=0.05)
    mw = pack_weights(cfg, w, "cpu", dtype=F32)
    x = torch.randn(37, cfg.hidden)
    got = mw.layers[0].moe(x, x)
    ref = moe_mlp(x, w, "model.layers.0.", cfg)
    assert (got - ref).abs().max() < 1e-4


def test_moe_engine_greedy_matches_oracle():
    cfg = preset("tiny-moe")
    w = random_weights(cfg, seed=0, std=0.05)
    ecfg = EngineConfig(model=cfg, spec=SpecConfig(mode="chain", num_draft=3), draft=DraftConfig(kind="model"),
                        cache=CacheConfig(page_size=16, num_pages=200))
    dcfg = preset("tiny-draft")
    dw = random_weights(dcfg, seed=1, std=0.05)
    eng = LLMEngine(ecfg, device="cpu", target=pack_weights(cfg, w, "cpu", dtype=F32),
                    drafter=pack_weights(dcfg, dw, "cpu", dtype=F32), dtype=F32, max_context=1024)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 4096, (30,), generator=g).tolist() for _ in range(2)]
    outs = eng.generate(prompts, SamplingParams(max_new_tokens=12))
    ref = RefModel(cfg, w)
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 12)


def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phung5_b200.parallel.comm import NcclCommunicator
        cfg = preset("tiny-moe")
        w = random_weights(cfg, seed=0, std=0.05)
        ecfg = EngineConfig(model=cfg, spec=SpecConfig(enabled=False), cache=CacheConfig(page_size=16, num_pages=200))
        eng = LLMEngine(ecfg, device="cpu", target=pack_weights(cfg, w, "cpu", rank, world, dtype=F32),
                        comm=NcclCommunicator(), dtype=F32, max_context=1024)
        assert eng.tw.layers[0].moe.e_local == 2
        g = torch.Generator().manual_seed(4)
        prompts = [torch.randint(0, 4096, (25,), generator=g).tolist() for _ in range(2)]
        q.put((rank, eng.generate(prompts, SamplingParams(max_new_tokens=10)), prompts))
    finally:
        dist.destroy_process_group()


def test_moe_expert_parallel_2_ranks():
    from tests.test_tp_cpu import _free_port
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in procs])
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    outs, prompts = res[0][1], res[0][2]
    assert res[1][1] == outs
    ref = RefModel(preset("tiny-moe"), random_weights(preset("tiny-moe"), seed=0, std=0.05))
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 10)


def _a2a_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phung5_b200.config import ParallelConfig
        from phung5_b200.parallel.comm import NcclCommunicator
        cfg = preset("tiny-moe")
        w = random_weights(cfg, seed=0, std=0.05)
        comm = NcclCommunicator()
        # the block alone: this rank's share of 37 rows through all-to-all dispatch equals the oracle's rows
        tw = pack_weights(cfg, w, "cpu", rank, world, dtype=F32)
        x = torch.randn(37, cfg.hidden, generator=torch.Generator().manual_seed(9))
        per = (37 + world - 1) // world
        lo, hi = min(37, rank * per), min(37, (rank + 1) * per)
        got = tw.layers[0].moe.forward_a2a(x[lo:hi].contiguous(), comm)
        ref = moe_mlp(x, w, "model.layers.0.", cfg)[lo:hi]
        block_err = float((got - ref).abs().max()) if hi > lo else 0.0
        # the engine with all-to-all dispatch on the collective path
        ecfg = EngineConfig(model=cfg, spec=SpecConfig(mode="chain", num_draft=3), draft=DraftConfig(kind="model"),
                            parallel=ParallelConfig(tp=world, comm="nccl", moe_dispatch="a2a"),
                            cache=CacheConfig(page_size=16, num_pages=200))
        dcfg = preset("tiny-draft")
        dw = random_weights(dcfg, seed=1, std=0.05)
        eng = LLMEngine(ecfg, device="cpu", target=pack_weights(cfg, w, "cpu", rank, world, dtype=F32),
                        drafter=pack_weights(dcfg, dw, "cpu", rank, world, dtype=F32), comm=comm, dtype=F32,
                        max_context=1024)
        assert eng.target.moe_a2a
        g = torch.Generator().manual_seed(4)
        prompts = [torch.randint(0, 4096, (25,), generator=g).tolist() for _ in range(3)]
        q.put((rank, eng.generate(prompts, SamplingParams(max_new_tokens=10)), prompts, block_err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_moe_all_to_all_dispatch_matches_oracle(world):
    """Expert parallelism by all-to-all (each rank routes its own tokens, rows travel to the experts' ranks and
    back) over 2 and 4 gloo ranks: the block equals the per-expert oracle on every rank's share, and chain
    speculative decoding emits the oracle's greedy tokens on every rank."""
    from tests.test_tp_cpu import _free_port
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_a2a_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    assert all(r[3] < 1e-4 for r in res), [r[3] for r in res]
    outs, prompts = res[0][1], res[0][2]
    assert all(r[1] == outs for r in res)
    ref = RefModel(preset("tiny-moe"), random_weights(preset("tiny-moe"), seed=0, std=0.05))
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 10)
