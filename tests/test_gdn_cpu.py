"""Gated DeltaNet on CPU: verify (state untouched) + commit of the accepted prefix equals running the
accepted tokens in prefill mode; the chunked ragged batch equals per-request processing."""
import torch

from phung5_b200.models.gdn import random_gdn_layer

H, HK, HV = 256, 1, 2


def _setup(slots=4):
    layer = random_gdn_layer(H, HK, HV, "cpu", seed=1, dtype=torch.float32)
    window = torch.randn(slots, 3, layer.conv_channels) * 0.1
    state = torch.randn(slots, HV, 128, 128) * 0.01
    return layer, window, state


def _ts(lens):
    return torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)


def test_verify_commit_equals_prefill_of_accepted():
    layer, win, st = _setup()
    win2, st2 = win.clone(), st.clone()
    x = torch.randn(3 + 5, H)
    slot = torch.tensor([1, 3], dtype=torch.int32)
    ts = _ts([3, 5])
    y_v = layer.forward(x, ts, slot, win, st, mode="verify")
    assert torch.equal(win, win2) and torch.equal(st, st2)          # verify leaves state alone
    n_acc = torch.tensor([2, 4], dtype=torch.int32)
    layer.commit(n_acc, win, st)
    # prefill only the accepted tokens from the original state
    xa = torch.cat([x[0:2], x[3:7]])
    y_p = layer.forward(xa, _ts([2, 4]), slot, win2, st2, mode="prefill")
    assert torch.allclose(st, st2, atol=1e-5) and torch.allclose(win, win2, atol=1e-6)
    assert torch.allclose(y_v[0:2], y_p[0:2], atol=1e-5) and torch.allclose(y_v[3:7], y_p[2:6], atol=1e-5)


def test_ragged_batch_equals_single_requests():
    layer, win, st = _setup()
    x = torch.randn(10, H)
    slot = torch.tensor([0, 2], dtype=torch.int32)
    w1, s1 = win.clone(), st.clone()
    y = layer.forward(x, _ts([4, 6]), slot, win, st)
    ya = layer.forward(x[:4], _ts([4]), slot[:1], w1, s1)
    yb = layer.forward(x[4:], _ts([6]), slot[1:], w1, s1)
    assert torch.allclose(y, torch.cat([ya, yb]), atol=1e-5)
    assert torch.allclose(st, s1, atol=1e-6)
