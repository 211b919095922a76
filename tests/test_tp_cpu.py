"""Tensor parallelism on CPU ranks (gloo, world size 2): sharded weights, all-reduce after o/down,
vocab-sharded top-k and argmax merges. The TP engine must reproduce the single-rank oracle's greedy
output (fp32)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q, num_pages=200, n_req=2, new_tokens=16):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phung5_b200.engine.engine import LLMEngine
        from phung5_b200.engine.oracle import SamplingParams
        from phung5_b200.models.llama import pack_weights
        from phung5_b200.parallel.comm import NcclCommunicator
        from phung5_b200.weights.init import random_weights
        tcfg, dcfg = preset("tiny"), preset("tiny-draft")
        tw = random_weights(tcfg, seed=0, std=0.05)
        dw = random_weights(dcfg, seed=1, std=0.05)
        comm = NcclCommunicator()
        spec = SpecConfig(mode=mode, num_draft=3, tree_nodes=10, topk=3, depth=3)
        ecfg = EngineConfig(model=tcfg, spec=spec, draft=DraftConfig(kind="model"),
                            cache=CacheConfig(page_size=16, num_pages=num_pages))
        eng = LLMEngine(ecfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", rank, world, dtype=torch.float32),
                        drafter=pack_weights(dcfg, dw, "cpu", rank, world, dtype=torch.float32), comm=comm,
                        dtype=torch.float32, max_context=1024)
        g = torch.Generator().manual_seed(3)
        prompts = [torch.randint(0, 4096, (40,), generator=g).tolist() for _ in range(n_req)]
        outs = eng.generate(prompts, SamplingParams(max_new_tokens=new_tokens))
        q.put((rank, outs, prompts, eng.stats["preempted"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["chain", "tree"])
def test_tp2_engine_matches_oracle(mode):
    from phung5_b200.engine.oracle import greedy_generate
    from phung5_b200.models.reference import RefModel
    from phung5_b200.weights.init import random_weights
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    res.sort()
    outs0, prompts = res[0][1], res[0][2]
    assert res[1][1] == outs0   # every rank takes the same decisions
    ref = RefModel(preset("tiny"), random_weights(preset("tiny"), seed=0, std=0.05))
    for p, o in zip(prompts, outs0):
        assert o == greedy_generate(ref, p, 16)


def _fused_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phung5_b200.engine.engine import LLMEngine
        from phung5_b200.engine.oracle import SamplingParams
        from phung5_b200.models.llama import pack_weights
        from phung5_b200.parallel.fused import FusedEmulator
        from phung5_b200.weights.init import random_weights
        tcfg, dcfg = preset("tiny"), preset("tiny-draft")
        tw, dw = random_weights(tcfg, seed=0, std=0.05), random_weights(dcfg, seed=1, std=0.05)
        comm = FusedEmulator(max_tokens=512, hidden=tcfg.hidden)
        ecfg = EngineConfig(model=tcfg, spec=SpecConfig(mode="tree", tree_nodes=10, topk=3, depth=3),
                            draft=DraftConfig(kind="model"), cache=CacheConfig(page_size=16, num_pages=200))
        eng = LLMEngine(ecfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", rank, world, dtype=torch.float32),
                        drafter=pack_weights(dcfg, dw, "cpu", rank, world, dtype=torch.float32), comm=comm,
                        dtype=torch.float32, max_context=1024)
        g = torch.Generator().manual_seed(3)
        prompts = [torch.randint(0, 4096, (40,), generator=g).tolist() for _ in range(2)]
        q.put((rank, eng.generate(prompts, SamplingParams(max_new_tokens=12)), prompts))
    finally:
        dist.destroy_process_group()


def test_tp2_fused_forward_plumbing_matches_oracle():
    from phung5_b200.engine.oracle import greedy_generate
    from phung5_b200.models.reference import RefModel
    from phung5_b200.weights.init import random_weights
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in procs])
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    outs, prompts = res[0][1], res[0][2]
    ref = RefModel(preset("tiny"), random_weights(preset("tiny"), seed=0, std=0.05))
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 12)


def _serve_worker(rank, world, port, q):
    """Rank 0 drives AsyncEngine (the HTTP server's engine thread) with two concurrent requests; rank 1 runs
    the TP worker loop. Both must take identical steps and rank 0's streams must equal the oracle."""
    import asyncio
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phung5_b200.engine.engine import LLMEngine
        from phung5_b200.engine.oracle import SamplingParams
        from phung5_b200.models.llama import pack_weights
        from phung5_b200.parallel.comm import NcclCommunicator
        from phung5_b200.serve.server import AsyncEngine, tp_worker_loop
        from phung5_b200.weights.init import random_weights
        tcfg, dcfg = preset("tiny"), preset("tiny-draft")
        tw = random_weights(tcfg, seed=0, std=0.05)
        dw = random_weights(dcfg, seed=1, std=0.05)
        comm = NcclCommunicator()
        group = dist.new_group(backend="gloo")
        ecfg = EngineConfig(model=tcfg, spec=SpecConfig(mode="tree", tree_nodes=10, topk=3, depth=3),
                            draft=DraftConfig(kind="model"), cache=CacheConfig(page_size=16, num_pages=200))
        eng = LLMEngine(ecfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", rank, world, dtype=torch.float32),
                        drafter=pack_weights(dcfg, dw, "cpu", rank, world, dtype=torch.float32), comm=comm,
                        dtype=torch.float32, max_context=1024)
        if rank != 0:
            tp_worker_loop(eng, group)
            q.put((rank, None, None))
            return
        g = torch.Generator().manual_seed(5)
        prompts = [torch.randint(0, 4096, (30,), generator=g).tolist() for _ in range(2)]
        aeng = AsyncEngine(eng, group=group)

        async def one(p):
            toks = []
            async for o in aeng.generate(p, SamplingParams(max_new_tokens=12)):
                toks += o.new_tokens
            return toks

        async def both():
            return await asyncio.gather(*(one(p) for p in prompts))
        outs = asyncio.run(both())
        aeng.shutdown()
        q.put((rank, outs, prompts))
    finally:
        dist.destroy_process_group()


def test_tp2_server_loop_matches_oracle():
    from phung5_b200.engine.oracle import greedy_generate
    from phung5_b200.models.reference import RefModel
    from phung5_b200.weights.init import random_weights
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_serve_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    outs, prompts = res[0][1], res[0][2]
    ref = RefModel(preset("tiny"), random_weights(preset("tiny"), seed=0, std=0.05))
    for p, o in zip(prompts, outs):
        assert o == greedy_generate(ref, p, 12)


def _eagle_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from phung5_b200.engine.engine import LLMEngine
        from phung5_b200.engine.oracle import SamplingParams
        from phung5_b200.models.llama import pack_weights
        from phung5_b200.parallel.comm import NcclCommunicator
        from phung5_b200.parallel.fused import FusedEmulator
        from phung5_b200.weights.init import random_weights
        tcfg = preset("tiny")
        tw = random_weights(tcfg, seed=0, std=0.05)
        g = torch.Generator().manual_seed(9)
        prompts = [torch.randint(0, 4096, (40,), generator=g).tolist() for _ in range(3)]
        outs = []
        for comm in (NcclCommunicator(), FusedEmulator(max_tokens=512, hidden=tcfg.hidden)):
            ecfg = EngineConfig(model=tcfg, spec=SpecConfig(mode="tree", tree_nodes=10, topk=3, depth=3),
                                draft=DraftConfig(kind="eagle"), cache=CacheConfig(page_size=16, num_pages=200))
            eng = LLMEngine(ecfg, device="cpu", target=pack_weights(tcfg, tw, "cpu", rank, world, dtype=torch.float32),
                            comm=comm, dtype=torch.float32, max_context=1024)
            outs.append(eng.generate(prompts, SamplingParams(max_new_tokens=12)))
        q.put((rank, outs, prompts))
    finally:
        dist.destroy_process_group()


def test_tp2_eagle_head_fused_path_matches_nccl_path():
    """The EAGLE head's layer on the fused communicator (workspace residual, ar_norm reductions) drafts the
    same trees as on the NCCL path; both emit the target's greedy tokens."""
    from phung5_b200.engine.oracle import greedy_generate
    from phung5_b200.models.reference import RefModel
    from phung5_b200.weights.init import random_weights
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_eagle_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    (nccl_out, fused_out), prompts = res[0][1], res[0][2]
    assert nccl_out == fused_out and res[1][1][1] == fused_out
    ref = RefModel(preset("tiny"), random_weights(preset("tiny"), seed=0, std=0.05))
    for p, o in zip(prompts, fused_out):
        assert o == greedy_generate(ref, p, 12)


def test_tp2_preemption_stays_in_step_across_ranks():
    """A KV pool too small for every request: both ranks admit, preempt and resume the same requests (the
    scheduler is replicated), and the output still equals the oracle's."""
    from phung5_b200.engine.oracle import greedy_generate
    from phung5_b200.models.reference import RefModel
    from phung5_b200.weights.init import random_weights
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, "chain", q, 16, 4, 40)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    assert res[0][1] == res[1][1] and res[0][3] == res[1][3] > 0
    ref = RefModel(preset("tiny"), random_weights(preset("tiny"), seed=0, std=0.05))
    for p, o in zip(res[0][2], res[0][1]):
        assert o == greedy_generate(ref, p, 40)
