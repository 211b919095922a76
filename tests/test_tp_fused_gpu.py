"""The fused NVLink all-reduce + RMSNorm + FP8 quant kernel (csrc/tp_fused.cu) and the GEMM scatter epilogue on
2, 4 and 8 GPUs (as many as the box has): the fused forward equals the NCCL forward, the reduction's residual
is bitwise the bf16 definition and its fp8 rows within one e4m3 step, and a peer that never arrives makes the
bounded wait report kErrTimeoutPeer through the status word instead of hanging; a collective reset then
restores a working communicator. These runs keep NVLS off (NCCL_NVLS_ENABLE=0, no multicast objects in the
symmetric workspace): a rank that leaves while its memory is bound to a multicast object can fault its peers."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


WORLDS = [2, 4, 8]
NO_NVLS = dict(NCCL_NVLS_ENABLE="0", TORCH_SYMM_MEM_DISABLE_MULTICAST="1", PHX_NVLS="0")


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), **NO_NVLS)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from phung5_b200 import ops
        from phung5_b200.config import preset
        from phung5_b200.engine.attn_meta import build_items, make_meta, pack_work
        from phung5_b200.models.llama import ForwardBatch, LlamaModel, random_packed_weights
        from phung5_b200.parallel.comm import NcclCommunicator
        from phung5_b200.parallel.fused import FusedCommunicator
        cfg = preset("small-fp8-kv8")
        dev = torch.device("cuda", rank)
        w = random_packed_weights(cfg, dev, seed=0, tp_rank=rank, tp_size=world)
        hkv = cfg.num_kv_heads // world
        cs = ops.rope_table(2048, cfg.head_dim, cfg.rope_theta, dev)
        fused = FusedCommunicator(max_tokens=1024, hidden=cfg.hidden)
        # kernel-level check: seeded partials of every rank -> ar_norm vs a local torch reference
        m, hd = 77, cfg.hidden
        parts = [torch.randn(m, hd, generator=torch.Generator().manual_seed(100 + r)).bfloat16() for r in range(world)]
        h0 = torch.randn(m, hd, generator=torch.Generator().manual_seed(7)).bfloat16()
        wn = (1 + 0.1 * torch.randn(hd, generator=torch.Generator().manual_seed(8))).bfloat16()
        tot = sum(p.float() for p in parts).bfloat16()
        h_ref = (h0.float() + tot.float()).bfloat16()
        # without push_h only the rows this rank owns get the new residual
        fused.partial(m).copy_(parts[rank])
        fused.h(m).copy_(h0)
        torch.cuda.synchronize()
        fused.ar_norm(m, wn.to(dev), cfg.rms_eps)
        torch.cuda.synchronize()
        per = (m + world - 1) // world
        own = torch.zeros(m, dtype=torch.bool)
        own[rank * per:(rank + 1) * per] = True
        hl = fused.h(m).cpu()
        h_local_ok = torch.equal(hl[own], h_ref[own]) and torch.equal(hl[~own], h0[~own])
        # with push_h every rank holds every new residual row
        fused.partial(m).copy_(parts[rank])
        fused.h(m).copy_(h0)
        torch.cuda.synchronize()
        qf, sf = fused.ar_norm(m, wn.to(dev), cfg.rms_eps, push_h=True)
        torch.cuda.synchronize()
        # small all-gather of mixed dtypes in one exchange
        ga, gb = fused.gather([torch.full((3, 5), float(rank), device=dev),
                               torch.arange(7, device=dev, dtype=torch.int64) + 100 * rank])
        gather_ok = (torch.equal(ga.cpu(), torch.stack([torch.full((3, 5), float(r)) for r in range(world)]))
                     and torch.equal(gb.cpu(), torch.stack([torch.arange(7) + 100 * r for r in range(world)])))
        hf = h_ref.float()
        y_ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * wn.float()
        deq = qf.float().cpu().view(m, hd // 128, 128) * sf.cpu().t()[..., None]
        h_exact = torch.equal(fused.h(m).cpu(), h_ref)
        y_err = ((deq.view(m, hd) - y_ref).abs().view(m, hd // 128, 128).amax(-1)
                 / y_ref.abs().view(m, hd // 128, 128).amax(-1)).max().item()
        res = {}
        for name, comm in (("nccl", NcclCommunicator()), ("fused", fused)):
            kk = torch.zeros(cfg.num_layers, 16, hkv, 64, 128, device=dev, dtype=torch.bfloat16)
            vv = torch.zeros_like(kk)
            model = LlamaModel(w, kk, vv, cs, comm)
            n = 300
            g = torch.Generator().manual_seed(5)
            toks = torch.randint(0, cfg.vocab, (n,), generator=g).to(dev)
            pages = list(range(1, 6))
            meta = make_meta([pages], [0], [n], None, True, dev)
            gg = model.hq // model.hkv
            _, p2 = build_items(meta, gg)
            slots = torch.tensor([pages[i // 64] * 64 + i % 64 for i in range(n)], device=dev)
            fb = ForwardBatch(tokens=toks, positions=torch.arange(n, device=dev, dtype=torch.int32), slots=slots,
                              meta=meta, work2=pack_work(p2, gg, dev))
            for _ in range(2):      # twice: epochs advance, barriers reused
                logits, h = model.forward(fb, want_hidden=True)
            torch.cuda.synchronize()
            ops.check_status(dev)
            res[name] = (logits.float().cpu(), h.float().cpu().clone())
        rel = ((res["fused"][0] - res["nccl"][0]).norm() / res["nccl"][0].norm()).item()
        relh = ((res["fused"][1] - res["nccl"][1]).norm() / res["nccl"][1].norm()).item()
        # timeout: only rank 0 launches the kernel; rank 1's flag never arrives
        dist.barrier()
        status = None
        if rank == 0:
            fused.ar_norm(8 * world, w.layers[0].post_norm, cfg.rms_eps)
            torch.cuda.synchronize()
            status = int(ops.status_tensor(dev)[0].item())
            ops.status_tensor(dev).zero_()
        dist.barrier()
        # recovery: the communicator is reset collectively and the next reduction is complete and correct
        fused.reset()
        fused.partial(m).copy_(parts[rank])
        fused.h(m).copy_(h0)
        torch.cuda.synchronize()
        fused.ar_norm(m, wn.to(dev), cfg.rms_eps, push_h=True)
        torch.cuda.synchronize()
        recovered = int(ops.status_tensor(dev)[0].item()) == 0 and torch.equal(fused.h(m).cpu(), h_ref)
        q.put((rank, rel, relh, status, h_exact and h_local_ok and gather_ok and recovered, y_err))
    finally:
        import torch.distributed as dist2
        dist2.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_fused_tp_equals_nccl_and_times_out_cleanly(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue as _queue
    import time as _time
    res, t0 = [], _time.time()
    while len(res) < world:               # fail fast if a worker dies instead of waiting on the queue
        try:
            res.append(q.get(timeout=5))
        except _queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead and _time.time() - t0 < 240, f"worker failed: {dead}"
    res.sort()
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for rank, rel, relh, status, h_exact, y_err in res:
        assert h_exact          # reduce + residual add is the bf16 definition exactly; own rows; gather
        assert y_err <= 1.0 / 15, y_err         # fp8 rows within one e4m3 step of the definition
        # whole 2-layer fp8 model: every activation is re-quantized, so tiny order differences compound
        assert rel < 5e-2, rel
        assert relh < 5e-2, relh
    assert res[0][3] == 4     # kErrTimeoutPeer


def _engine_worker(rank, world, port, q):
    """TP2 engine on the fused communicator (EAGLE head on the fused path, fused vocab merges): the
    CUDA-graph speculative step must emit the eager step's tokens on every rank."""
    import datetime
    import torch.distributed as dist
    # no failure injection here: the fused kernels may use NVLS (closed collectively below)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from phung5_b200 import ops
        from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
        from phung5_b200.engine.engine import LLMEngine
        from phung5_b200.engine.oracle import SamplingParams
        from phung5_b200.parallel.fused import FusedCommunicator
        cfg = preset("small-fp8-kv8")
        g = torch.Generator().manual_seed(6)
        shared = torch.randint(0, cfg.vocab, (128,), generator=g).tolist()
        prompts = [shared + torch.randint(0, cfg.vocab, (64,), generator=g).tolist() for _ in range(8)]
        outs, replays = {}, 0
        for graphs in ("1", "0"):
            os.environ["PHX_GRAPHS"] = graphs
            comm = FusedCommunicator(max_tokens=1024, hidden=cfg.hidden)
            spec = SpecConfig(mode="tree", tree_nodes=64, topk=8, depth=6, accept="geometric")
            eng = LLMEngine(EngineConfig(model=cfg, spec=spec, draft=DraftConfig(kind="eagle"),
                                         cache=CacheConfig(num_pages=256)), device=f"cuda:{rank}", comm=comm,
                            max_context=2048)
            outs[graphs] = eng.generate(prompts, SamplingParams(max_new_tokens=40))
            ops.check_status()
            if graphs == "1":
                replays = eng.stats["graph_replays"]
            del eng
            torch.cuda.synchronize()
            comm.close()
        q.put((rank, outs["1"] == outs["0"], replays, outs["1"][0][:8]))
    finally:
        import torch.distributed as dist2
        dist2.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_fused_tp_graph_step_equals_eager(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_engine_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue as _queue
    import time as _time
    res, t0 = [], _time.time()
    while len(res) < world:
        try:
            res.append(q.get(timeout=5))
        except _queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead and _time.time() - t0 < 300, f"worker failed: {dead}"
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    res.sort()
    assert all(ok for _, ok, _, _ in res), res
    assert all(n >= 5 for _, _, n, _ in res), res
    assert all(r[3] == res[0][3] for r in res)   # every rank emits the same tokens


def _nvls_worker(rank, world, port, q):
    """NVLS variant of the fused reduction (multimem.ld_reduce reduce-scatter, multimem.st all-gather) against
    the same torch definition; all ranks agree to skip when any lacks a multicast address. The communicator is
    torn down collectively before the process group, so no rank leaves while bound to the multicast object."""
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", PHX_NVLS="1")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    fused = None
    try:
        from phung5_b200 import ops
        from phung5_b200.parallel.fused import FusedCommunicator
        dev = torch.device("cuda", rank)
        hd = 1024
        fused = FusedCommunicator(max_tokens=1024, hidden=hd)
        have = torch.tensor([1 if fused.mc else 0], device=dev)
        dist.all_reduce(have, op=dist.ReduceOp.MIN)
        if not int(have.item()):
            q.put((rank, "skip", 0.0, 0.0, True))
            return
        m = 133
        parts = [torch.randn(m, hd, generator=torch.Generator().manual_seed(100 + r)).bfloat16() for r in range(world)]
        h0 = torch.randn(m, hd, generator=torch.Generator().manual_seed(7)).bfloat16()
        wn = (1 + 0.1 * torch.randn(hd, generator=torch.Generator().manual_seed(8))).bfloat16()
        h_ref = (h0.float() + sum(p.float() for p in parts)).bfloat16()
        errs = []
        for _ in range(2):                          # twice: the barrier epochs advance
            fused.partial(m).copy_(parts[rank])
            fused.h(m).copy_(h0)
            torch.cuda.synchronize()
            qf, sf = fused.ar_norm(m, wn.to(dev), 1e-5, push_h=True)
            torch.cuda.synchronize()
            ops.check_status(dev)
            hg = fused.h(m).cpu().float()
            # in units of the bf16 step of the partial sum's magnitude: the switch adds in fp32 (in its own
            # order) and rounds once, then the residual is added and rounded; a wrong sum is many steps off
            mag = (h0.float().abs() + sum(p.float().abs() for p in parts)).clamp(min=1e-3)
            step = torch.exp2(torch.floor(torch.log2(mag)) - 7)
            errs.append(((hg - h_ref.float()).abs() / step).max().item())
        hf = fused.h(m).cpu().float()
        y_ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * wn.float()
        deq = qf.float().cpu().view(m, hd // 128, 128) * sf.cpu().t()[..., None]
        y_err = ((deq.view(m, hd) - y_ref).abs().view(m, hd // 128, 128).amax(-1)
                 / y_ref.abs().view(m, hd // 128, 128).amax(-1)).max().item()
        ga, = fused.gather([torch.full((5, 7), float(rank), device=dev)])
        gather_ok = torch.equal(ga.cpu(), torch.stack([torch.full((5, 7), float(r)) for r in range(world)]))
        q.put((rank, "ran", max(errs), y_err, gather_ok))
    finally:
        if fused is not None:
            fused.close()
        import torch.distributed as dist2
        dist2.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_fused_tp_nvls_reduction_matches_definition(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_nvls_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue as _queue
    import time as _time
    res, t0 = [], _time.time()
    while len(res) < world:
        try:
            res.append(q.get(timeout=5))
        except _queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead and _time.time() - t0 < 240, f"worker failed: {dead}"
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    if res[0][1] == "skip":
        pytest.skip("no NVLink multicast on this box")
    for rank, _, h_err, y_err, gather_ok in res:
        # within two bf16 steps (of the summed magnitudes) of the fp32-sum definition
        assert h_err <= 2.0, h_err
        assert y_err <= 1.0 / 15 + 3e-2, y_err
        assert gather_ok
