"""Argument checks of the host-buffer entry points, on the CPU: they refuse what they cannot copy
asynchronously before any device work is queued."""
import importlib

import pytest
import torch

PKG = "deepseek-v4-flash-mlx_b200"


def test_host_prefill_rejects_unpinned_buffers():
    P = importlib.import_module(PKG + ".prefill")
    q = torch.empty(4, 64, 512, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="pinned"):
        P.attend_queries_host(q, torch.empty(4, 64, 128), torch.empty(4, 64), None, None, None, None, 0, 4,
                              torch.empty(4, 64, 512, dtype=torch.bfloat16))
