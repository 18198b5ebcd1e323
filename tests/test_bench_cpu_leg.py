"""bench.py's CPU leg (the reference arm and the cpu_baseline entry) on a tiny time budget: the
workload is set up once, repeated until the budget of timed work is spent, and the block configs'
weights are dequantised once, to the same fp32 values the oracle uses."""
import importlib

import torch

import bench
from oracle.layer_ref import _w


def test_cpu_reference_repeats_to_budget():
    v, cores, desc = bench.cpu_reference("c2", 1, threads=2, min_seconds=0.05)
    assert v > 0 and cores == 2
    assert "repetitions" in desc and "timed CPU work" in desc


def test_dequantized_weights_equal_the_oracles():
    Lm = importlib.import_module("deepseek-v4-flash-mlx_b200.layer")
    C = importlib.import_module("deepseek-v4-flash-mlx_b200.configs")
    W = Lm.make_attention_weights(0, dims=C.LayerDims(dim=256, q_lora=128), quant=True)
    Wd = bench._dequantized(W)
    for name in Lm.MATRICES:
        got = getattr(Wd, name)
        assert got.dtype == torch.float32 and torch.equal(got, _w(getattr(W, name))), name
    assert torch.equal(Wd.sinks, W.sinks)
