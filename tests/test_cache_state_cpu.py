"""Checkpoint / resume of the device-resident decode state (the reference copies its per-layer
state with clone_states, oracle/v4_fast.py:150-159, and copy.deepcopy, oracle/decode_engine.py:167):
state_dict -> torch.save -> torch.load -> load_state_dict restores every buffer, clone is
independent. The cache is plain tensors, so this runs on the CPU."""
import importlib
import io

import pytest
import torch

D = importlib.import_module("deepseek-v4-flash-mlx_b200.decode")


def _filled(max_comp, seed, page_order=None):
    g = torch.Generator().manual_seed(seed)
    c = D.SparseMLACache(2, max_comp, device="cpu", page_order=page_order)
    for name, t in c.state_dict().items():
        if name == "meta":
            continue
        if t.dtype == torch.uint8:
            t.copy_(torch.randint(0, 256, t.shape, generator=g, dtype=torch.uint8))
        elif t.is_floating_point():
            t.copy_(torch.randn(t.shape, generator=g).to(t.dtype))
    return c


@pytest.mark.parametrize("max_comp", [0, 100])
def test_state_dict_round_trip(max_comp):
    perm = torch.randperm(2 * ((max_comp + 63) // 64), generator=torch.Generator().manual_seed(1))
    c = _filled(max_comp, 2, page_order=perm)
    c.image_stale = True
    buf = io.BytesIO()
    torch.save(c.state_dict(), buf)
    buf.seek(0)
    fresh = D.SparseMLACache(2, max_comp, device="cpu")
    fresh.load_state_dict(torch.load(buf))
    a, b = c.state_dict(), fresh.state_dict()
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert fresh.image_stale


def test_clone_is_independent_and_layout_is_checked():
    c = _filled(100, 3)
    cl = c.clone()
    before = c.kv_pool.clone()
    cl.kv_pool.add_(1)
    cl.key_image[0].zero_()
    assert torch.equal(c.kv_pool, before)
    assert not torch.equal(c.key_image[0], cl.key_image[0])
    with pytest.raises(ValueError):
        D.SparseMLACache(2, 64, device="cpu").load_state_dict(c.state_dict())
