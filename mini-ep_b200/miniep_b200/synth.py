"""Seeded synthetic inputs for the MoE layer, shared by the tests, the bench and
the CPU checker so that every side sees bit-identical tensors.

Draw order (one ``torch.Generator`` per layer, seeded ``seed``): router (E,H),
w_in (E,2I,H), w_out (E,H,I), then the tokens x (N,H). Weights are drawn as
N(0,1)*0.02 in fp32 and cast afterwards; tokens are N(0,1). The reference loads
these tensors from a checkpoint (miniep/weights.py:37-61); the checkpoint is not
available here, so seeded random weights of the same shapes stand in for it.

The skewed-routing workloads add a per-layer router bias before top-k:
``b_l = scale * log(p)[perm_l]`` with ``p_r ∝ r^-s`` (Zipf over experts,
r = 1..E) and ``perm_l`` an independent random permutation per layer, drawn
layer by layer from a generator seeded ``bias_seed``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

# Layer shapes used by the workloads: (a) is the GraniteMoE layer, (b) the larger one.
SHAPES = {
    "a": dict(hidden=1024, experts=32, topk=8, inter=512),
    "b": dict(hidden=4096, experts=64, topk=6, inter=1408),
}

# GraniteMoE's residual_multiplier (the scale applied to the MoE output before
# the residual add, miniep/modeling.py:197).
GRANITE_RESIDUAL_MULTIPLIER = 0.22


@dataclass
class LayerTensors:
    router: torch.Tensor  # (E, H)
    w_in: torch.Tensor    # (E, 2I, H) fused gate+up, gate = rows [0, I)
    w_out: torch.Tensor   # (E, H, I)
    x: torch.Tensor       # (N, H)


def make_layer(hidden: int, experts: int, inter: int, n_tokens: int, seed: int = 0,
               dtype: torch.dtype = torch.float32, device: str | torch.device = "cpu"
               ) -> LayerTensors:
    """Seeded weights and tokens for one MoE layer.

    On the CPU the values are identical on every machine with the same torch;
    ``device="cuda"`` draws from the CUDA generator instead (same distribution,
    different values), which the bench uses to build large inputs quickly.
    """
    g = torch.Generator(device=device).manual_seed(seed)
    router = torch.randn(experts, hidden, generator=g, device=device) * 0.02
    w_in = torch.randn(experts, 2 * inter, hidden, generator=g, device=device) * 0.02
    w_out = torch.randn(experts, hidden, inter, generator=g, device=device) * 0.02
    x = torch.randn(n_tokens, hidden, generator=g, device=device)
    return LayerTensors(router.to(dtype), w_in.to(dtype), w_out.to(dtype), x.to(dtype))


def make_tokens(n_tokens: int, hidden: int, seed: int, dtype: torch.dtype = torch.float32,
                device: str | torch.device = "cpu") -> torch.Tensor:
    """Extra N(0,1) token batches (e.g. residual stream h) from their own seed."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(n_tokens, hidden, generator=g, device=device).to(dtype)


def zipf_router_bias(num_layers: int, experts: int, s: float = 1.2, scale: float = 2.0,
                     seed: int = 1) -> torch.Tensor:
    """(L, E) float32 router bias giving Zipf(s)-skewed expert popularity per layer."""
    g = torch.Generator().manual_seed(seed)
    r = torch.arange(1, experts + 1, dtype=torch.float64)
    p = r.pow(-s)
    p = p / p.sum()
    logp = scale * torch.log(p)
    rows = []
    for _ in range(num_layers):
        perm = torch.randperm(experts, generator=g)
        rows.append(logp[perm].to(torch.float32))
    return torch.stack(rows)


def split_tokens(n_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous even split of a global token batch: [start, stop) of ``rank``."""
    per = n_tokens // world
    rem = n_tokens % world
    start = rank * per + min(rank, rem)
    return start, start + per + (1 if rank < rem else 0)
