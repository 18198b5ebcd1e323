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


def test_reference_arm_prints_the_gpu_arms_config():
    """The reference arm's line carries the GPU arm's config dict at the same N (config 2 at N=2: two
    replica sequences), and exactly K timed steps."""
    line = bench.reference_line("c2", steps=2, warmup=1, world=2, per_step_seconds=0.01)
    assert line["config"] == bench.config_dict("c2", 2)
    assert line["config"]["global_batch"] == 2 and line["steps"] == 2 and line["impl"] == "reference"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
    for name in ("c3", "c4", "c5"):
        assert bench.config_dict(name, 8)["global_batch"] == (1 if name == "c4" else bench.CONFIGS[name]["batch"])
