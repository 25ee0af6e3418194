"""CPU checker for the expert-parallel MoE layer (TEST INFRASTRUCTURE ONLY).

This module restates, on the CPU with torch/numpy, the arithmetic of the
reference's MoE-layer hot path (kanwarpal-brar/mini-ep, ``miniep/``), so that the
CUDA path can be checked against it on machines where the reference itself is
absent. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import it, and only as the checker / the timed CPU baseline;
the product path never calls into it.

Parity of this restatement is pinned by ``tests/test_oracle_golden.py`` against
fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py`` produced by
importing and running the reference's own code (``LocalMoEBackend``,
``EPMoEBackend`` over gloo ranks, ``Placement.dest_ranks``, ``plan_balanced``).

Every function cites the reference lines it restates.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F


# --------------------------------------------------------------------------
# router  (miniep/modeling.py:193-195)
# --------------------------------------------------------------------------
def router_logits(x: torch.Tensor, router_w: torch.Tensor,
                  bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x_flat @ router.T`` in the model dtype (modeling.py:193), plus the
    optional skew bias (cast to the model dtype) added before top-k."""
    logits = x @ router_w.T
    if bias is not None:
        logits = logits + bias.to(logits.dtype)
    return logits


def router_topk(x: torch.Tensor, router_w: torch.Tensor, k: int,
                bias: torch.Tensor | None = None):
    """Top-k of the logits, softmax over the k selected logits in fp32, cast back
    to the model dtype (modeling.py:193-195). Returns (idx int64, gate, logits)."""
    logits = router_logits(x, router_w, bias)
    topk_logits, topk_idx = logits.topk(k, dim=-1)
    topk_gate = torch.softmax(topk_logits.float(), dim=-1).to(x.dtype)
    return topk_idx, topk_gate, logits


def topk_lowest_index(logits: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k with a deterministic tie rule (larger value first, then lower expert
    index): the rule the CUDA router applies. torch's CPU ``topk`` breaks exact
    ties in no fixed order, so parity on selection is only defined where the
    top-(k+1) logits hold no exact tie (see ``boundary_ties``)."""
    v = logits.float().numpy()
    idx = np.broadcast_to(np.arange(v.shape[-1]), v.shape)
    order = np.lexsort((idx, -v), axis=-1)
    return torch.from_numpy(order[:, :k].astype(np.int64))


def boundary_ties(logits: torch.Tensor, k: int) -> torch.Tensor:
    """(N,) bool: token has an exact tie among its sorted top-(k+1) logits."""
    srt = logits.float().sort(dim=-1, descending=True).values[:, : k + 1]
    return (srt[:, 1:] == srt[:, :-1]).any(dim=-1)


def softmax_topk(topk_logits: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """softmax over the selected logits in fp32, cast to the model dtype (modeling.py:195)."""
    return torch.softmax(topk_logits.float(), dim=-1).to(dtype)


# --------------------------------------------------------------------------
# entry flattening / expert compute / combine  (miniep/modeling.py:83-145)
# --------------------------------------------------------------------------
def flatten_topk(n: int, k: int, valid_mask: torch.Tensor | None = None):
    """(token_ids, slot_ids, keep_e) of the kept entries in flat token-major,
    slot-minor order (modeling.py:107-117)."""
    keep = torch.ones(n, dtype=torch.bool) if valid_mask is None else valid_mask.bool()
    keep_e = keep.repeat_interleave(k)
    token_ids = torch.arange(n).repeat_interleave(k)[keep_e]
    slot_ids = torch.arange(k).repeat(n)[keep_e]
    return token_ids, slot_ids, keep_e


def run_experts(x: torch.Tensor, expert_ids: torch.Tensor, w_in: torch.Tensor,
                w_out: torch.Tensor) -> torch.Tensor:
    """Rows grouped by expert (stable), ``h = x_e @ w_in[e].T``, gate = first I
    columns, ``(silu(gate) * up) @ w_out[e].T``, scattered back to input order
    (modeling.py:83-104)."""
    out = torch.zeros(x.shape[0], w_out.shape[1], dtype=x.dtype)
    if x.shape[0] == 0:
        return out
    order = torch.argsort(expert_ids, stable=True)
    sorted_ids = expert_ids[order]
    uniq, counts = torch.unique_consecutive(sorted_ids, return_counts=True)
    start = 0
    for e, n in zip(uniq.tolist(), counts.tolist()):
        rows = order[start:start + n]
        start += n
        h = x[rows] @ w_in[e].T
        gate, up = h.chunk(2, dim=-1)
        out[rows] = (F.silu(gate) * up) @ w_out[e].T
    return out


def scatter_combine(gated, token_ids, slot_ids, n, k, hidden):
    """Each (token, slot) cell written once, then summed over the k slots
    (modeling.py:120-128)."""
    buf = torch.zeros(n, k, hidden, dtype=gated.dtype)
    buf[token_ids, slot_ids] = gated
    return buf.sum(dim=1)


def local_moe(x, topk_idx, topk_gate, w_in, w_out, valid_mask=None):
    """Single-process MoE backend (modeling.py:131-145)."""
    n, k = topk_idx.shape
    token_ids, slot_ids, keep_e = flatten_topk(n, k, valid_mask)
    expert_ids = topk_idx.reshape(-1)[keep_e]
    outs = run_experts(x[token_ids], expert_ids, w_in, w_out)
    gated = outs * topk_gate.reshape(-1)[keep_e].unsqueeze(1)
    return scatter_combine(gated, token_ids, slot_ids, n, k, x.shape[1])


def residual_add(h, moe_out, residual_multiplier):
    """``h + moe_out * residual_multiplier`` (modeling.py:197)."""
    return h + moe_out * residual_multiplier


def rms_norm(x, weight, eps):
    """``weight * (x * rsqrt(mean(x^2) + eps))`` in the activation dtype
    (modeling.py:51-52)."""
    return weight * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def moe_block_from_h(h, norm_w, eps, router_w, w_in, w_out, k, residual_multiplier, bias=None,
                     valid_mask=None):
    """The MoE half of ``Block.forward`` from the residual stream
    (modeling.py:192-197): post-attention RMSNorm, router, MoE, residual."""
    x = rms_norm(h, norm_w, eps)
    out, idx, gate = moe_block(h, x, router_w, w_in, w_out, k, residual_multiplier, bias,
                               valid_mask)
    return out, idx, gate, x


def moe_block(h, x, router_w, w_in, w_out, k, residual_multiplier,
              bias=None, valid_mask=None):
    """Router + MoE + residual for one layer (modeling.py:192-197), local experts."""
    idx, gate, _ = router_topk(x, router_w, k, bias)
    out = local_moe(x, idx, gate, w_in, w_out, valid_mask)
    return residual_add(h, out, residual_multiplier), idx, gate


# --------------------------------------------------------------------------
# placement / replica round-robin  (miniep/ep.py:20-96)
# --------------------------------------------------------------------------
def naive_owners(num_layers: int, num_experts: int, world: int):
    """Contiguous placement: expert e on rank e // (E/world) (ep.py:47-52)."""
    assert num_experts % world == 0
    per = num_experts // world
    return [[[e // per] for e in range(num_experts)] for _ in range(num_layers)]


def owners_from_plan(plan: dict):
    """Owner lists from the plan JSON, each sorted (ep.py:54-60)."""
    return [
        [sorted(lo[str(e)]) for e in range(len(lo))]
        for lo in (plan["owners"][str(l)] for l in range(len(plan["owners"])))
    ]


def build_table(owners_l):
    """table[e, j] = rank of e's j-th replica, n_rep[e] (ep.py:35-45)."""
    n_exp = len(owners_l)
    rmax = max(len(o) for o in owners_l)
    table = np.zeros((n_exp, rmax), dtype=np.int64)
    n_rep = np.zeros(n_exp, dtype=np.int64)
    for e, o in enumerate(owners_l):
        table[e, :len(o)] = o
        n_rep[e] = len(o)
    return table, n_rep


def dest_ranks(table: np.ndarray, n_rep: np.ndarray, rr: np.ndarray,
               expert_ids: np.ndarray) -> np.ndarray:
    """Destination rank per entry; the i-th occurrence (flat order) of expert e
    goes to replica (rr[e] + i) % n_rep[e]; afterwards rr[e] += count[e]
    (ep.py:76-96). ``rr`` is updated in place; with no replicated expert in
    the layer it is left untouched (ep.py:84-85)."""
    expert_ids = np.asarray(expert_ids, dtype=np.int64)
    if (n_rep == 1).all():
        return table[expert_ids, 0].copy()
    m = expert_ids.size
    counts = np.bincount(expert_ids, minlength=table.shape[0])
    order = np.argsort(expert_ids, kind="stable")
    srt = expert_ids[order]
    starts = np.cumsum(counts) - counts
    within = np.empty(m, dtype=np.int64)
    within[order] = np.arange(m, dtype=np.int64) - starts[srt]
    slot = (rr[expert_ids] + within) % n_rep[expert_ids]
    rr += counts
    return table[expert_ids, slot]


def experts_of_rank(owners_l, rank: int):
    """Sorted experts resident on ``rank`` for one layer (ep.py:67-71)."""
    return sorted(e for e in range(len(owners_l)) if rank in owners_l[e])


# --------------------------------------------------------------------------
# expert-parallel forward, all ranks simulated in one process
# (miniep/ep.py:210-249 with Comm.exchange_counts/all_to_all, ep.py:120-136)
# --------------------------------------------------------------------------
@dataclass
class EPResult:
    outputs: list                 # per rank (N_r, H)
    route_counts: np.ndarray      # (W, E) source-side histograms
    recv_tokens: np.ndarray       # (W,) entries computed per rank
    send_counts: np.ndarray       # (W, W) [src, dst]
    dest: list = field(default_factory=list)  # per rank (M_r,) destinations


def ep_forward(xs, idxs, gates, w_in, w_out, owners_l, rr=None, valids=None):
    """One layer step of ``EPMoEBackend.__call__`` on every rank.

    xs/idxs/gates/valids: per-rank token shards. ``w_in``/``w_out`` hold ALL
    experts (global ids); each rank computes with the slice of its resident
    experts in sorted order, as the reference's local row order does. ``rr``
    is the (E,) round-robin state per source rank (list of arrays), zero by
    default, updated in place.
    """
    world = len(xs)
    num_experts = len(owners_l)
    table, n_rep = build_table(owners_l)
    if rr is None:
        rr = [np.zeros(num_experts, dtype=np.int64) for _ in range(world)]
    valids = valids or [None] * world
    send = []
    route_counts = np.zeros((world, num_experts), dtype=np.int64)
    send_counts = np.zeros((world, world), dtype=np.int64)
    dests = []
    for r in range(world):
        n, k = idxs[r].shape
        token_ids, slot_ids, keep_e = flatten_topk(n, k, valids[r])
        flat_expert = idxs[r].reshape(-1)[keep_e]
        flat_gate = gates[r].reshape(-1)[keep_e]
        route_counts[r] = np.bincount(flat_expert.numpy(), minlength=num_experts)
        dest = dest_ranks(table, n_rep, rr[r], flat_expert.numpy())
        order = np.argsort(dest, kind="stable")
        send_counts[r] = np.bincount(dest, minlength=world)
        send.append((token_ids, slot_ids, flat_expert, flat_gate, order, n, k))
        dests.append(dest)
    # each destination concatenates its received rows in source-rank order
    results = {}
    recv_tokens = np.zeros(world, dtype=np.int64)
    for d in range(world):
        local = experts_of_rank(owners_l, d)
        g2l = {e: i for i, e in enumerate(local)}
        rows, ids, origin = [], [], []
        for s in range(world):
            token_ids, _, flat_expert, _, order, _, _ = send[s]
            o = torch.from_numpy(order)
            sel = o[torch.from_numpy(dests[s])[o] == d]
            rows.append(xs[s][token_ids[sel]])
            ids.append(flat_expert[sel])
            origin.append((s, sel))
        rx = torch.cat(rows)
        rid = torch.cat(ids)
        assert all(int(e) in g2l for e in rid), "entry routed to a non-resident expert"
        local_ids = torch.tensor([g2l[int(e)] for e in rid], dtype=torch.long)
        out = run_experts(rx, local_ids, w_in[local], w_out[local])
        recv_tokens[d] = rx.shape[0]
        pos = 0
        for s, sel in origin:
            results[(s, d)] = (sel, out[pos:pos + sel.numel()])
            pos += sel.numel()
    outputs = []
    for s in range(world):
        token_ids, slot_ids, flat_expert, flat_gate, order, n, k = send[s]
        back = torch.zeros(flat_expert.numel(), w_out.shape[1], dtype=xs[s].dtype)
        for d in range(world):
            sel, out = results[(s, d)]
            back[sel] = out
        gated = back * flat_gate.unsqueeze(1)
        outputs.append(scatter_combine(gated, token_ids, slot_ids, n, k, xs[s].shape[1]))
    return EPResult(outputs, route_counts, recv_tokens, send_counts, dests)
