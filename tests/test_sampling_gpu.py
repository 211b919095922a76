"""Device-side speculative sampling (csrc/sample.cu) against its torch definition (engine/sampling.py):
candidate selection per vocab chunk (exact top-KC of x / T, ties toward the lower index), the seeded tree
accept walk and the bonus draw, on one vocab and on a vocab split into tensor-parallel shards; and the engine's
seeded-sampling steps (device path, eager and CUDA graph) emitting exactly the torch definition's tokens."""
import pytest
import torch

from phung5_b200 import ops
from phung5_b200.engine.sampling import seeded_coins, tree_accept_reference

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _logits(rows, V, seed, ties=True):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(rows, V, device=DEV, generator=g) * 2.0
    if ties:       # coarse values: many exact ties, also at the top-k boundary
        x = (x * 4).round() / 4
    return x.bfloat16()


def _tree(R, N, logits, seed):
    """Random trees (parent[j] < j); each child's token is one of the parent's five best tokens or a random one,
    so some children are accepted and some rejected."""
    g = torch.Generator().manual_seed(seed)
    V = logits.shape[-1]
    lg = logits.float().view(R, N, V).cpu()
    parent = torch.full((R, N), -1, dtype=torch.int64)
    tokens = torch.zeros(R, N, dtype=torch.int64)
    for r in range(R):
        tokens[r, 0] = int(torch.randint(0, V, (1,), generator=g))
        for j in range(1, N):
            p = int(torch.randint(0, j, (1,), generator=g))
            parent[r, j] = p
            top = torch.topk(lg[r, p], 5).indices
            tokens[r, j] = int(top[int(torch.randint(0, 5, (1,), generator=g))]) if torch.rand(1, generator=g) < 0.8 \
                else int(torch.randint(0, V, (1,), generator=g))
    return tokens.to(DEV), parent.to(DEV)


def _params(R):
    temps = torch.tensor([0.0, 0.7, 1.0, 1.3, 1.0, 0.5, 2.0, 1.0][:R], device=DEV)
    top_k = torch.tensor([1, 8, 16, 50, 64, 5, 3, 12][:R], device=DEV, dtype=torch.int32)
    top_p = torch.tensor([1.0, 0.9, 0.95, 0.9, 0.5, 1.0, 0.8, 0.3][:R], device=DEV)
    seed = torch.tensor([11, 12, 13, 14, 15, 16, 17, 2 ** 31 + 5][:R], device=DEV, dtype=torch.int64)
    committed = torch.tensor([100, 2 ** 33 + 7, 5, 4000, 77, 1, 999, 123456][:R], device=DEV, dtype=torch.int64)
    return temps, top_k, top_p, seed, committed


def _reference(logits, tokens, parent, temps, top_k, top_p, seed, committed, D):
    R, N = tokens.shape
    coins = seeded_coins(seed.cpu(), committed.cpu(), D + 2).to(DEV)
    return tree_accept_reference(logits.view(R, N, -1), tokens, parent, temps, top_k.long(), top_p, coins, D)


@pytest.mark.parametrize("V,kc", [(40000, 64), (40000, 16), (16032, 64), (128256, 64)])
def test_candidates_are_exact_topk(V, kc):
    rows = 12
    x = _logits(rows, V, seed=V + kc)
    temp = torch.linspace(0.5, 1.5, rows // 3, device=DEV)
    nch = int(ops.ext().sample_chunks(V))
    cv = torch.empty(rows, nch, kc, device=DEV)
    ci = torch.empty(rows, nch, kc, device=DEV, dtype=torch.int32)
    ops.ext().sample_candidates(x, kc, temp, 3, 1000, cv, ci, None, ops.status_tensor(x.device))
    torch.cuda.synchronize()
    xf = x.float() / temp.repeat_interleave(3)[:, None]
    for c in range(nch):
        a, b = c * 16384, min(V, (c + 1) * 16384)
        sv, si = torch.sort(xf[:, a:b], dim=-1, descending=True, stable=True)
        want_i = (si[:, :kc] + a + 1000).int()
        got_v, order = torch.sort(cv[:, c], dim=-1, descending=True, stable=True)
        got_i = ci[:, c].gather(1, order)
        # equal values may come in either order inside the kernel's list: compare as (value, index) pairs
        key_got = sorted(zip(got_v.flatten().tolist(), got_i.flatten().tolist()))
        key_want = sorted(zip(sv[:, :kc].flatten().tolist(), want_i.flatten().tolist()))
        assert key_got == key_want, c


def test_candidates_with_massive_ties_take_the_exact_path():
    """A flat row (every logit equal) overflows the fast path's candidate buffer; the exact radix kernel then
    returns the lowest indices."""
    x = torch.zeros(3, 40000, device=DEV, dtype=torch.bfloat16)
    x[1, 777] = 1.0                                    # one clear winner, the rest tied
    cv = torch.empty(3, 3, 16, device=DEV)
    ci = torch.empty(3, 3, 16, device=DEV, dtype=torch.int32)
    cms = torch.empty(3, 3, 2, device=DEV)
    ops.ext().sample_candidates(x, 16, None, 1, 0, cv, ci, cms, ops.status_tensor(x.device))
    torch.cuda.synchronize()
    assert torch.equal(ci[0, 0].sort().values.cpu(), torch.arange(16, dtype=torch.int32))
    assert torch.equal(ci[0, 2].sort().values.cpu(), torch.arange(32768, 32768 + 16, dtype=torch.int32))
    got = ci[1, 0].sort().values.cpu().tolist()
    assert 777 in got and got == sorted([777] + list(range(15)))
    assert torch.allclose(cms[0, :, 1].cpu(), torch.tensor([16384.0, 16384.0, 40000 - 32768.0]))


@pytest.mark.parametrize("V,ranks", [(40000, 1), (128256, 1), (128256, 8), (64128, 2)])
def test_accept_walk_matches_torch_definition(V, ranks):
    R, N, D = 8, 24, 6
    x = _logits(R * N, V, seed=3 + V + ranks)
    tokens, parent = _tree(R, N, x, seed=ranks)
    temps, top_k, top_p, seed, committed = _params(R)
    acc_ref, bonus_ref = _reference(x, tokens, parent, temps, top_k, top_p, seed, committed, D)
    if ranks == 1:
        acc, bonus = ops.spec_sample_accept(x, tokens, parent, temps, top_k, top_p, seed, committed, D, 64)
    else:       # vocab shards on one GPU: candidates per shard, stacked as if gathered from every rank
        vs = V // ranks
        nch = int(ops.ext().sample_chunks(vs))
        cv = torch.empty(ranks, R * N, nch, 64, device=DEV)
        ci = torch.empty(ranks, R * N, nch, 64, device=DEV, dtype=torch.int32)
        for w in range(ranks):
            ops.ext().sample_candidates(x[:, w * vs:(w + 1) * vs].contiguous(), 64, temps, N, w * vs, cv[w], ci[w],
                                        None, ops.status_tensor(x.device))
        acc = torch.empty(R, D, dtype=torch.int64, device=DEV)
        bonus = torch.empty(R, dtype=torch.int64, device=DEV)
        ops.ext().spec_accept(cv, ci, ranks, nch, 64, tokens, parent, temps, top_k, top_p, seed, committed, D, acc,
                              bonus)
    torch.cuda.synchronize()
    assert torch.equal(acc.cpu(), acc_ref.cpu()), (acc, acc_ref)
    assert torch.equal(bonus.cpu(), bonus_ref.cpu()), (bonus, bonus_ref)
    assert (acc_ref >= 0).any() and (acc_ref < 0).any()        # the case exercises accepts and rejections


def test_engine_seeded_sampling_device_path_equals_torch_definition(monkeypatch):
    from phung5_b200.config import CacheConfig, DraftConfig, EngineConfig, SpecConfig, preset
    from phung5_b200.engine.engine import LLMEngine
    from phung5_b200.engine.oracle import SamplingParams
    from phung5_b200.models.llama import pack_weights
    from phung5_b200.weights.init import random_weights
    cfg = preset("small-bf16")
    hf = random_weights(cfg, seed=0, std=0.05)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab, (150,), generator=g).tolist() for _ in range(4)]
    sps = [SamplingParams(temperature=t, top_k=k, top_p=p, seed=s, max_new_tokens=24)
           for t, k, p, s in ((0.8, 20, 0.9, 1), (1.0, 8, 1.0, 2), (0.0, 0, 1.0, 3), (1.2, 50, 0.7, 4))]
    outs = {}
    for name, dev_sampling, graphs in (("torch", False, "0"), ("device_eager", True, "0"), ("device_graph", True, "1")):
        monkeypatch.setattr(ops, "DEVICE_SAMPLING", dev_sampling)
        monkeypatch.setenv("PHX_GRAPHS", graphs)
        spec = SpecConfig(mode="tree", tree_nodes=32, topk=4, depth=4)
        eng = LLMEngine(EngineConfig(model=cfg, spec=spec, draft=DraftConfig(kind="eagle"),
                                     cache=CacheConfig(num_pages=256)),
                        device=DEV, target=pack_weights(cfg, hf, DEV), max_context=2048)
        rids = [eng.add_request(p, sp) for p, sp in zip(prompts, sps)]
        while eng.has_work():
            eng.step()
        ops.check_status()
        outs[name] = [eng.reqs[r].out for r in rids]
        if name == "device_graph":
            assert eng.stats["graph_replays"] > 0
    assert outs["device_eager"] == outs["torch"]
    assert outs["device_graph"] == outs["torch"]
