"""compressor_decode_pair (the main and indexer compressors' decode steps in one launch) against the
same two steps as separate compressor_decode_step launches: rings, emitted rows and the key image
bit for bit, over positions that emit and positions that do not."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

PKG = "deepseek-v4-flash-mlx_b200"
DEV = "cuda"


def _fill(c, g):
    for t in (c.ring_kv, c.ring_score, c.ring_k_idx, c.ring_s_idx):
        t.copy_(torch.randn(t.shape, generator=g))


@pytest.mark.parametrize("b,act_quant,hd", [(1, 0, 512), (5, 0, 512), (32, 1, 512), (4, 0, 1024)])
def test_pair_matches_two_steps(b, act_quant, hd):
    """hd 1024: rows wider than the one-launch kernel takes, so the pair runs as two launches."""
    dsv4 = importlib.import_module(PKG)
    D = importlib.import_module(PKG + ".decode")
    layer = importlib.import_module(PKG + ".layer")
    g = torch.Generator().manual_seed(b * 7 + act_quant)
    caches = [D.SparseMLACache(b, 256, head_dim=hd, device=DEV) for _ in range(2)]
    st = torch.Generator().manual_seed(11)
    for c in caches:
        _fill(c, st)
        st.manual_seed(11)
    idd = 128
    ape_c, ape_i = torch.randn(4, 2 * hd, generator=g) * 0.1, torch.randn(4, 2 * idd, generator=g) * 0.1
    nw_c, nw_i = torch.rand(hd, generator=g) + 0.5, torch.rand(idd, generator=g) + 0.5
    ape_c, ape_i, nw_c, nw_i = (t.to(DEV) for t in (ape_c, ape_i, nw_c, nw_i))
    freqs = layer.layer_rope_freqs(layer.DIMS, DEV)
    pos0 = torch.tensor([200 + 5 * i for i in range(b)], dtype=torch.int32)
    for step in range(8):
        pos = (pos0 + step).to(DEV)
        c_kv, c_sc = (torch.randn(b, 2 * hd, generator=g).to(DEV) for _ in range(2))
        i_kv, i_sc = (torch.randn(b, 2 * idd, generator=g).to(DEV) for _ in range(2))
        for k, c in enumerate(caches):
            _, comp_rows, key_rows = D.decode_rows(c, pos)
            if k == 0:
                dsv4.compressor_decode_step(c_kv, None, None, ape_c, nw_c, c.ring_kv, c.ring_score, pos, c.kv_pool,
                                            comp_rows, head_dim=hd, freqs=freqs, proj=(c_kv, c_sc),
                                            act_quant=act_quant)
                dsv4.compressor_decode_step(i_kv, None, None, ape_i, nw_i, c.ring_k_idx, c.ring_s_idx, pos,
                                            c.k_idx.view(-1, idd), key_rows, head_dim=idd, freqs=freqs,
                                            proj=(i_kv, i_sc), key_image=(*c.key_image, c.max_comp))
            else:
                dsv4.compressor_decode_pair(
                    dsv4.CompressorStep((c_kv, c_sc), ape_c, nw_c, c.ring_kv, c.ring_score, c.kv_pool, comp_rows, hd,
                                        act_quant=act_quant),
                    dsv4.CompressorStep((i_kv, i_sc), ape_i, nw_i, c.ring_k_idx, c.ring_s_idx,
                                        c.k_idx.view(-1, idd), key_rows, idd, key_image=(*c.key_image, c.max_comp)),
                    pos, freqs=freqs)
    torch.cuda.synchronize()
    a, p = caches
    for name in ("ring_kv", "ring_score", "ring_k_idx", "ring_s_idx", "kv_pool", "k_idx"):
        assert torch.equal(getattr(a, name), getattr(p, name)), name
    for i, (ta, tp) in enumerate(zip(a.key_image, p.key_image)):
        assert torch.equal(ta, tp), f"key_image.{i}"
    assert a.kv_pool.abs().sum().item() > 0   # rows were emitted


def test_pair_rejects_a_key_image_on_the_first_step():
    dsv4 = importlib.import_module(PKG)
    e = torch.empty(0)
    s = dsv4.CompressorStep((e, e), e, None, e, e, e, e, 128, key_image=(e, e, e, 1))
    with pytest.raises(ValueError):
        dsv4.compressor_decode_pair(s, s, e)
