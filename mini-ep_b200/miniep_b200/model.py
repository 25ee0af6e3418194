"""GraniteMoE decoder and lockstep engine with device-resident state.

The reference's model (miniep/modeling.py:24-262) and engine
(miniep/worker.py:38-138) are CPU-bound: positions, masks and the RoPE tables
are built on the host and the KV cache grows by concatenation. Here the same
computation runs on the device:

  * every tensor of a step lives on the model's device; positions, masks and
    the RoPE tables are built there;
  * the KV cache is allocated once per shard (prompt length + decode budget)
    and written in place, in the reference's layout: prompt keys in columns
    [0, T) (right-padded rows), decode step t in column T + t for every row,
    RoPE at each row's own position;
  * the MoE half of each block (router + experts + residual,
    modeling.py:192-197) is one call into the expert-parallel layer
    (``EPMoEBackend.moe_block``: router, routing, dispatch, tcgen05 experts,
    combine and residual on the GPU).

Attention uses torch's fused scaled-dot-product attention (GQA without
repeating K/V; the memory-efficient, flash or math kernels). In bf16 the RoPE tables are cast to the model dtype before
use, as HF GraniteMoe does; the reference multiplies bf16 activations by fp32
tables, which turns q and k into fp32 and leaves its bf16 attention without a
common dtype. In fp32 both are the same arithmetic.
"""
from __future__ import annotations

import json
import time
from dataclasses import dataclass, fields
from pathlib import Path

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

# torch's cuDNN attention backend queries the device properties on every call
# (tens of ms of host time per call on this image), so attention is kept on
# the fused memory-efficient / flash kernels, or math on the host
_SDPA = [SDPBackend.EFFICIENT_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.MATH]


@dataclass
class ModelConfig:
    """Same fields as the reference's ModelConfig (modeling.py:24-49)."""
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    num_local_experts: int
    num_experts_per_tok: int
    vocab_size: int
    rms_norm_eps: float
    rope_theta: float
    embedding_multiplier: float
    attention_multiplier: float
    residual_multiplier: float
    logits_scaling: float
    max_position_embeddings: int
    eos_token_id: int = 0
    pad_token_id: int = 0

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @staticmethod
    def from_dict(raw: dict) -> "ModelConfig":
        return ModelConfig(**{f.name: raw[f.name] for f in fields(ModelConfig) if f.name in raw})

    @staticmethod
    def from_json(path) -> "ModelConfig":
        return ModelConfig.from_dict(json.loads(Path(path).read_text()))


# the Granite-3.0-1B-A400M shape (24 layers, hidden 1024,
# 16 query / 8 KV heads of 64, 32 experts of 512, top-8, vocab 49155, RoPE
# theta 10000) with that model's multipliers. Weights are synthetic.
GRANITE_1B_A400M = dict(
    hidden_size=1024, intermediate_size=512, num_hidden_layers=24, num_attention_heads=16,
    num_key_value_heads=8, num_local_experts=32, num_experts_per_tok=8, vocab_size=49155,
    rms_norm_eps=1e-6, rope_theta=10000.0, embedding_multiplier=12.0,
    attention_multiplier=0.015625, residual_multiplier=0.22, logits_scaling=6.0,
    max_position_embeddings=4096)


def weight_keys(cfg: ModelConfig) -> list[tuple[str, tuple]]:
    """(name, shape) of every weight, in the reference checkpoint's key names
    (modeling.py:150-160, :233-235) and in the draw order of random_weights."""
    H, I, E, V = cfg.hidden_size, cfg.intermediate_size, cfg.num_local_experts, cfg.vocab_size
    d, hq, hk = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    out = [("model.embed_tokens.weight", (V, H))]
    for l in range(cfg.num_hidden_layers):
        p = f"model.layers.{l}."
        out += [(p + "input_layernorm.weight", (H,)),
                (p + "self_attn.q_proj.weight", (hq * d, H)),
                (p + "self_attn.k_proj.weight", (hk * d, H)),
                (p + "self_attn.v_proj.weight", (hk * d, H)),
                (p + "self_attn.o_proj.weight", (H, hq * d)),
                (p + "post_attention_layernorm.weight", (H,)),
                (p + "block_sparse_moe.router.layer.weight", (E, H)),
                (p + "block_sparse_moe.input_linear.weight", (E, 2 * I, H)),
                (p + "block_sparse_moe.output_linear.weight", (E, H, I))]
    out.append(("model.norm.weight", (H,)))
    return out


def random_weights(cfg: ModelConfig, seed: int = 0, dtype=torch.float32) -> dict:
    """Synthetic weights on the host: matrices N(0, 1) * 0.02, norm weights
    1 + N(0, 1) * 0.02, drawn in weight_keys order from one generator, in fp32,
    then cast."""
    g = torch.Generator().manual_seed(seed)
    w = {}
    for name, shape in weight_keys(cfg):
        t = torch.randn(shape, generator=g, dtype=torch.float32) * 0.02
        if name.endswith("norm.weight"):
            t = t + 1.0
        w[name] = t.to(dtype)
    return w


def expert_weight_keys(layer: int) -> tuple[str, str]:
    """(input_linear, output_linear) keys of one layer (weights.py:22-26)."""
    p = f"model.layers.{layer}.block_sparse_moe."
    return p + "input_linear.weight", p + "output_linear.weight"


def rms_norm(x, weight, eps):
    """modeling.py:51-52, in the activation dtype."""
    return weight * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def _rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


class Rope:
    """modeling.py:60-80 with the tables on the device."""

    def __init__(self, cfg: ModelConfig, device, dtype):
        d = cfg.head_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        t = torch.arange(cfg.max_position_embeddings, dtype=torch.float32)
        emb = torch.cat((torch.outer(t, inv),) * 2, dim=-1)
        self.cos = emb.cos().to(device=device, dtype=dtype)
        self.sin = emb.sin().to(device=device, dtype=dtype)

    def apply(self, q, k, positions):
        cos = self.cos[positions].unsqueeze(1)
        sin = self.sin[positions].unsqueeze(1)
        return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


class Shard:
    """One rank's right-padded slice of the batch (worker.py:38-75) with its KV
    cache preallocated on the device for `max_new` decode steps."""

    def __init__(self, prompts: list[list[int]], cfg: ModelConfig, max_new: int, device,
                 dtype):
        if not prompts:
            raise ValueError("a shard needs at least one prompt (use a dummy prompt to idle)")
        self.B = len(prompts)
        self.lengths = torch.tensor([len(p) for p in prompts], device=device)
        self.T = max(len(p) for p in prompts)
        self.cap = self.T + max_new
        self.input = torch.full((self.B, self.T), cfg.pad_token_id, dtype=torch.long)
        for i, p in enumerate(prompts):
            self.input[i, :len(p)] = torch.tensor(p)
        self.input = self.input.to(device)
        shape = (cfg.num_hidden_layers, self.B, cfg.num_key_value_heads, self.cap, cfg.head_dim)
        # zeroed: columns not yet written are masked out of attention, and a
        # masked zero contributes exactly nothing (a masked NaN would not)
        self.k = torch.zeros(shape, device=device, dtype=dtype)
        self.v = torch.zeros(shape, device=device, dtype=dtype)
        self.used = 0  # cache columns written
        self.decoded = 0
        self.generated = [[] for _ in range(self.B)]
        self.last_tokens = None
        self.last_prefill_logits = None
        self.last_logits = None
        cols = torch.arange(self.cap, device=device)
        # key columns a query may see: prompt columns inside the row's length,
        # every decode column (worker.py:60-74)
        self.key_valid = (cols[None, :] < self.lengths[:, None]) | (cols[None, :] >= self.T)

    def prefill_masks(self):
        """(B,1,T,T) keep-mask causal & key valid, and the MoE valid mask (B,T)."""
        t = torch.arange(self.T, device=self.input.device)
        causal = t[None, :] <= t[:, None]
        valid = self.key_valid[:, :self.T]
        return (causal[None] & valid[:, None, :])[:, None], valid

    def decode_mask(self):
        """(B,1,1,T+t+1) keep-mask of decode step t."""
        return self.key_valid[:, None, None, :self.used + 1]

    def decode_positions(self):
        return (self.lengths + self.decoded).unsqueeze(1)


class DeviceModel:
    """GraniteMoeModel (modeling.py:148-262) on the device. `moe_blocks[l]`
    computes the MoE half of block l: (h_flat, x_flat, router_w, rm, valid)
    -> h_flat + moe(x_flat) * rm."""

    def __init__(self, cfg: ModelConfig, weights: dict, moe_blocks: list, device=None):
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else \
            weights["model.embed_tokens.weight"].device
        dt = weights["model.embed_tokens.weight"].dtype
        self.dtype = dt
        w = {k: v.to(self.device) for k, v in weights.items()
             if not k.endswith(("input_linear.weight", "output_linear.weight"))}
        self.w = w
        self.moe_blocks = moe_blocks
        self.rope = Rope(cfg, self.device, dt)

    def _attention(self, l, x, positions, shard: Shard, col0, mask):
        """col0: first cache column of these T positions: an int (keys are the
        columns [0, col0 + T)), or a one-element device tensor for a one-token
        step (keys are all cache columns; `mask` hides the unwritten ones)."""
        cfg, p = self.cfg, f"model.layers.{l}.self_attn."
        B, T, H = x.shape
        d = cfg.head_dim
        q = (x @ self.w[p + "q_proj.weight"].T).view(B, T, cfg.num_attention_heads, d).transpose(1, 2)
        k = (x @ self.w[p + "k_proj.weight"].T).view(B, T, cfg.num_key_value_heads, d).transpose(1, 2)
        v = (x @ self.w[p + "v_proj.weight"].T).view(B, T, cfg.num_key_value_heads, d).transpose(1, 2)
        q, k = self.rope.apply(q, k, positions)
        if isinstance(col0, torch.Tensor):
            shard.k[l].index_copy_(2, col0, k)
            shard.v[l].index_copy_(2, col0, v)
            keys, vals = shard.k[l], shard.v[l]
        else:
            shard.k[l, :, :, col0:col0 + T] = k
            shard.v[l, :, :, col0:col0 + T] = v
            keys = shard.k[l, :, :, :col0 + T]
            vals = shard.v[l, :, :, :col0 + T]
        o = self._sdpa(q, keys, vals, mask)
        return o.transpose(1, 2).reshape(B, T, H) @ self.w[p + "o_proj.weight"].T

    def _sdpa(self, q, k, v, mask):
        """Attention of q (B, Hq, T, D) over k, v (B, Hk, S, D), query head h
        on KV head h // (Hq / Hk).

        mask None (prefill, keys = the T prompt columns): causal. For every
        query inside its row's prompt the causal keys are exactly the valid
        ones (padding sits after the prompt), so this equals the reference's
        causal-and-valid mask there; padded positions are never read (their
        expert entries are masked and decode masks their cache columns).
        mask (B, 1, 1, S) (decode: depends on the key only): the query heads of
        one KV head are folded into that head's query rows, plain attention
        with a broadcast mask, no GQA support needed from the kernel."""
        cfg = self.cfg
        if mask is None:
            with sdpa_kernel(_SDPA):
                return F.scaled_dot_product_attention(q, k, v, is_causal=True,
                                                      scale=cfg.attention_multiplier,
                                                      enable_gqa=True)
        B, Hq, T, D = q.shape
        Hk = k.shape[1]
        qg = q.reshape(B, Hk, (Hq // Hk) * T, D)
        with sdpa_kernel(_SDPA):
            o = F.scaled_dot_product_attention(qg, k, v, attn_mask=mask,
                                               scale=cfg.attention_multiplier)
        return o.reshape(B, Hq, T, D)

    def forward(self, ids, positions, shard: Shard, col0: int, mask, moe_valid, logits_at=None):
        cfg = self.cfg
        B, T = ids.shape
        h = self.w["model.embed_tokens.weight"][ids] * cfg.embedding_multiplier
        valid = None if moe_valid is None else moe_valid.reshape(-1)
        for l in range(cfg.num_hidden_layers):
            p = f"model.layers.{l}."
            x = rms_norm(h, self.w[p + "input_layernorm.weight"], cfg.rms_norm_eps)
            h = h + self._attention(l, x, positions, shard, col0, mask) * cfg.residual_multiplier
            x = rms_norm(h, self.w[p + "post_attention_layernorm.weight"], cfg.rms_norm_eps)
            h = self.moe_blocks[l](h.reshape(B * T, -1), x.reshape(B * T, -1),
                                   self.w[p + "block_sparse_moe.router.layer.weight"],
                                   cfg.residual_multiplier, valid).reshape(B, T, -1)
        if logits_at is not None:
            h = h[torch.arange(B, device=h.device), logits_at].unsqueeze(1)
        h = rms_norm(h, self.w["model.norm.weight"], cfg.rms_norm_eps)
        emb = self.w["model.embed_tokens.weight"]
        return (h @ emb.T) / cfg.logits_scaling


class Engine:
    """Lockstep prefill / greedy decode over one rank's shard
    (worker.py:100-138). Every rank runs the same number of forwards; a rank
    without prompts runs dummy forwards that add no expert load."""

    def __init__(self, model: DeviceModel, reset_rr=None):
        self.model = model
        self.reset_rr = reset_rr or (lambda: None)
        self.steps = 0

    @torch.no_grad()
    def prefill(self, shard: Shard, dummy: bool = False):
        self.reset_rr()
        _, valid = shard.prefill_masks()
        if dummy:
            valid = torch.zeros_like(valid)
        pos = torch.arange(shard.T, device=shard.input.device).unsqueeze(0).expand(shard.B, -1)
        logits = self.model.forward(shard.input, pos, shard, 0, None, valid,
                                    logits_at=shard.lengths - 1)
        shard.used = shard.T
        self.steps += 1
        shard.last_prefill_logits = logits[:, 0]
        shard.last_tokens = logits[:, 0].argmax(dim=-1)
        return shard.last_tokens

    @torch.no_grad()
    def decode_step(self, shard: Shard, active=None):
        self.reset_rr()
        toks = shard.last_tokens.tolist()
        act = None if active is None else active.tolist()
        for i in range(shard.B):
            if act is None or act[i]:
                shard.generated[i].append(int(toks[i]))
        mask = shard.decode_mask()
        moe_valid = None if active is None else active.unsqueeze(1)
        logits = self.model.forward(shard.last_tokens.unsqueeze(1), shard.decode_positions(),
                                    shard, shard.used, mask, moe_valid)
        shard.used += 1
        shard.decoded += 1
        self.steps += 1
        shard.last_logits = logits[:, -1]
        shard.last_tokens = shard.last_logits.argmax(dim=-1)
        return shard.last_tokens

    @torch.no_grad()
    def decode_graphed(self, shard: Shard, steps: int, idle: bool = False):
        """`steps` greedy decode steps of every row (all active), each one
        CUDA-graph replay: attention runs over every cache column with the
        unwritten ones masked on the device, and the cache column, the
        positions and the fed-back tokens are device tensors the graph
        advances. The first step runs eagerly (it also warms the kernels up),
        the second is captured and replayed for the rest. Same results as
        `decode_step` in fp32 up to the attention kernel's summation order.
        Every rank calls it at the same point with the same `steps`; an idle
        rank (dummy shard) passes idle=True and adds no expert load."""
        if steps < 1:
            return shard.last_tokens
        m, dev = self.model, shard.input.device
        cols = torch.arange(shard.cap, device=dev)
        col = torch.full((1,), shard.used, dtype=torch.long, device=dev)
        pos = (shard.lengths + shard.decoded).unsqueeze(1).clone()
        tok = shard.last_tokens.clone()
        gen = torch.zeros(shard.B, steps, dtype=torch.long, device=dev)
        j = torch.zeros(1, dtype=torch.long, device=dev)
        last = torch.empty(shard.B, m.cfg.vocab_size, dtype=m.dtype, device=dev)
        moe_valid = torch.zeros(shard.B, 1, dtype=torch.bool, device=dev) if idle else None

        def step():
            self.reset_rr()
            gen.index_copy_(1, j, tok.unsqueeze(1))
            mask = (shard.key_valid & (cols[None, :] <= col))[:, None, None, :]
            logits = m.forward(tok.unsqueeze(1), pos, shard, col, mask, moe_valid)
            last.copy_(logits[:, -1])
            tok.copy_(last.argmax(dim=-1))
            col.add_(1)
            pos.add_(1)
            j.add_(1)

        step()
        if steps > 1:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step()
            for _ in range(steps - 1):
                g.replay()
        gl = gen.tolist()
        for i in range(shard.B):
            shard.generated[i].extend(gl[i])
        shard.used += steps
        shard.decoded += steps
        self.steps += steps
        shard.last_logits = last
        shard.last_tokens = tok
        return tok

    def generate(self, shard: Shard, max_new: int, dummy: bool = False):
        """Prefill then `max_new` decode steps; returns (generated ids per row,
        positions processed, seconds). Positions follow worker.py:214-217:
        valid prompt positions plus one per row per decode step."""
        t0 = time.perf_counter()
        self.prefill(shard, dummy=dummy)
        for _ in range(max_new):
            self.decode_step(shard)
        if self.model.device.type == "cuda":
            torch.cuda.synchronize(self.model.device)
        dt = time.perf_counter() - t0
        positions = 0 if dummy else int(shard.lengths.sum()) + shard.B * max_new
        return shard.generated, positions, dt


def ep_moe_blocks(backends) -> list:
    """Per-layer MoE-block callables over expert-parallel backends
    (EPMoEBackend.moe_block: router, expert-parallel layer and residual in one
    call into the library)."""
    def make(be):
        def run(h, x, router_w, rm, valid):
            return be.moe_block(h, x, router_w, rm, valid_mask=valid)[0]
        return run
    return [make(be) for be in backends]
