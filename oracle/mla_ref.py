"""Oracle: MLA projections (restating v4mlx/mla.py:16-56 in torch fp32). Test-only."""
import torch

N_HEADS, HEAD_DIM, N_GROUPS, O_LORA = 64, 512, 8, 1024


def linear(x, W):
    """v4mlx/mla.py:16-18: y = x @ W.T, W [out, in]."""
    return x.float() @ W.float().T


def q_up(qln, wq_b, heads=N_HEADS, head_dim=HEAD_DIM):
    """v4mlx/mla.py:31-34."""
    q = linear(qln, wq_b)
    return q.reshape(*q.shape[:-1], heads, head_dim)


def o_grouped(o, wo_a, wo_b, groups=N_GROUPS):
    """v4mlx/mla.py:42-56: per-group [.., in/groups] x wo_a[g]^T, concatenated, then x wo_b^T."""
    lead = o.shape[:-1]
    og = o.float().reshape(*lead, groups, -1)
    wa = wo_a.float().reshape(groups, -1, og.shape[-1])
    mid = torch.einsum("...gd,grd->...gr", og, wa).reshape(*lead, -1)
    return linear(mid, wo_b)


def dequant_int8_g64(q, scale):
    """Symmetric 8-bit weights with one scale per (row, 64 inputs): w = q * scale (exact in fp32)."""
    return q.float() * scale.float().repeat_interleave(64, dim=-1)
