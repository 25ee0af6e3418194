"""The device-resident GraniteMoE model and engine on a B200 with the CUDA
expert layer in every block:

* fp32, the reference's two-layer model driven like its engine
  (tests/golden/model_tiny.npz): prefill and every decode step's logits within
  1e-4 of max|ref|, greedy tokens identical;
* bf16, the Granite-3.0-1B-A400M layer shape (two layers), through the tcgen05
  experts: a prefill + decode run repeats bit for bit, and a dummy prefill on
  the same context leaves the next real step's result unchanged.
"""
import json

import numpy as np
import pytest
import torch

from gpu_util import require_gpu
from miniep_b200 import Comm, EPMoEBackend, EPStats, Placement
from miniep_b200.model import (GRANITE_1B_A400M, DeviceModel, Engine, ModelConfig, Shard,
                               ep_moe_blocks, expert_weight_keys, random_weights)

pytestmark = pytest.mark.gpu


def _build(cfg, w, max_tokens, dtype):
    L, E = cfg.num_hidden_layers, cfg.num_local_experts
    comm = Comm(num_layers=L, num_experts=E, topk=cfg.num_experts_per_tok, hidden=cfg.hidden_size,
                inter=cfg.intermediate_size, max_tokens=max_tokens, dtype=dtype,
                single_process=True)
    placement = Placement.naive(L, E, 1)
    comm.install(placement)
    stats = EPStats(L, E)
    backends = []
    for l in range(L):
        a, b = expert_weight_keys(l)
        backends.append(EPMoEBackend(l, comm, placement, list(range(E)), w[a].cuda(), w[b].cuda(),
                                     stats))
    dense = {k: v for k, v in w.items() if "block_sparse_moe.input_linear" not in k
             and "block_sparse_moe.output_linear" not in k}
    model = DeviceModel(cfg, {k: v.cuda() for k, v in dense.items()}, ep_moe_blocks(backends))
    return comm, placement, stats, model


def test_model_fp32_matches_reference_engine(golden):
    require_gpu()
    g = np.load(golden / "model_tiny.npz")
    cfg = ModelConfig.from_dict(json.loads(str(g["config"])))
    w = random_weights(cfg, seed=5, dtype=torch.float32)
    lens = g["prompt_lens"].tolist()
    flat, prompts, i = g["prompts"].tolist(), [], 0
    for n in lens:
        prompts.append(flat[i:i + n])
        i += n
    steps = g["decode_logits"].shape[0]
    comm, placement, stats, model = _build(cfg, w, len(prompts) * max(lens), torch.float32)
    shard = Shard(prompts, cfg, steps, "cuda", torch.float32)
    eng = Engine(model, reset_rr=placement.reset_rr)
    eng.prefill(shard)
    ref = torch.from_numpy(g["prefill_logits"])
    assert (shard.last_prefill_logits.cpu() - ref).abs().max() <= 1e-4 * ref.abs().max()
    for t in range(steps):
        eng.decode_step(shard)
        want = torch.from_numpy(g["decode_logits"][t])
        assert (shard.last_logits.cpu() - want).abs().max() <= 1e-4 * want.abs().max()
    assert shard.generated == g["generated"].tolist()
    comm.check()
    # the same decode as graph replays (attention over the whole masked cache)
    shard2 = Shard(prompts, cfg, steps, "cuda", torch.float32)
    eng.prefill(shard2)
    eng.decode_graphed(shard2, steps)
    assert shard2.generated == g["generated"].tolist()
    want = torch.from_numpy(g["decode_logits"][steps - 1])
    assert (shard2.last_logits.cpu() - want).abs().max() <= 1e-4 * want.abs().max()
    # every valid prompt position and every decode row went through the experts
    snap = stats.snapshot()
    assert snap["recv_tokens_per_layer"] == [2 * (sum(lens) + len(lens) * steps) * cfg.num_experts_per_tok] * 2
    comm.close()


def test_model_bf16_granite_layers_repeat_exactly():
    require_gpu()
    cfg = ModelConfig.from_dict(dict(GRANITE_1B_A400M, num_hidden_layers=2, vocab_size=4096))
    w = random_weights(cfg, seed=3, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(4)
    prompts = [torch.randint(1, cfg.vocab_size, (n,), generator=gen).tolist() for n in (96, 128, 40)]
    comm, placement, stats, model = _build(cfg, w, 3 * 128, torch.bfloat16)
    eng = Engine(model, reset_rr=placement.reset_rr)
    runs = []
    for dummy_first in (False, True):
        shard = Shard(prompts, cfg, 8, "cuda", torch.bfloat16)
        if dummy_first:  # an idle rank's prefill on a scratch shard, then the real run
            eng.prefill(Shard([[1, 2, 3, 4]], cfg, 1, "cuda", torch.bfloat16), dummy=True)
        gen_ids, positions, _ = eng.generate(shard, 8)
        runs.append((gen_ids, shard.last_logits.float().cpu()))
        assert positions == sum(len(p) for p in prompts) + 3 * 8
    assert runs[0][0] == runs[1][0]
    assert torch.equal(runs[0][1], runs[1][1])
    assert torch.isfinite(runs[0][1]).all()
    # graph-replayed decode steps give the eager steps' tokens and logits
    shard = Shard(prompts, cfg, 8, "cuda", torch.bfloat16)
    eng.prefill(shard)
    eng.decode_graphed(shard, 8)
    assert shard.generated == runs[0][0]
    assert torch.equal(shard.last_logits.float().cpu(), runs[0][1])
    comm.check()
    comm.close()
