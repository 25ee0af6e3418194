"""The device-resident model and engine (miniep_b200.model) against the
reference's GraniteMoeModel driven like its engine (tests/golden/model_tiny.npz:
prefill of a right-padded three-prompt shard, six greedy decode steps, fp32).
Here the model code runs on the host with the checker's MoE block in each
layer, which isolates the non-expert half (RoPE, masks, the preallocated KV
cache, GQA attention, logits at each row's last position) from the kernels;
the GPU test runs the same fixture through the CUDA expert layer."""
import json

import numpy as np
import torch

from miniep_b200.model import DeviceModel, Engine, ModelConfig, Shard, expert_weight_keys, random_weights
from oracle import moe_oracle as O


def _prompts(g):
    lens = g["prompt_lens"].tolist()
    flat = g["prompts"].tolist()
    out, i = [], 0
    for n in lens:
        out.append(flat[i:i + n])
        i += n
    return out


def test_model_and_engine_match_reference_on_host(golden):
    g = np.load(golden / "model_tiny.npz")
    raw = json.loads(str(g["config"]))
    cfg = ModelConfig.from_dict(raw)
    w = random_weights(cfg, seed=5, dtype=torch.float32)

    def moe(l):
        a, b = expert_weight_keys(l)

        def run(h, x, router_w, rm, valid):
            return O.moe_block(h, x, router_w, w[a], w[b], cfg.num_experts_per_tok, rm,
                               valid_mask=valid)[0]
        return run

    model = DeviceModel(cfg, w, [moe(l) for l in range(cfg.num_hidden_layers)], device="cpu")
    steps = g["decode_logits"].shape[0]
    shard = Shard(_prompts(g), cfg, steps, "cpu", torch.float32)
    eng = Engine(model)
    eng.prefill(shard)
    ref = torch.from_numpy(g["prefill_logits"])
    assert (shard.last_prefill_logits - ref).abs().max() <= 1e-5 * ref.abs().max()
    for t in range(steps):
        eng.decode_step(shard)
        want = torch.from_numpy(g["decode_logits"][t])
        assert (shard.last_logits - want).abs().max() <= 1e-5 * want.abs().max()
        assert shard.last_tokens.tolist() == want.argmax(-1).tolist()
    assert shard.generated == g["generated"].tolist()
    assert eng.steps == 1 + steps


def test_dummy_prefill_adds_no_expert_rows(golden):
    g = np.load(golden / "model_tiny.npz")
    cfg = ModelConfig.from_dict(json.loads(str(g["config"])))
    w = random_weights(cfg, seed=5, dtype=torch.float32)
    seen = []

    def moe(h, x, router_w, rm, valid):
        seen.append(int(valid.sum()) if valid is not None else x.shape[0])
        return h

    model = DeviceModel(cfg, w, [moe] * cfg.num_hidden_layers, device="cpu")
    shard = Shard([[1, 2, 3]], cfg, 2, "cpu", torch.float32)
    Engine(model).prefill(shard, dummy=True)
    assert seen == [0] * cfg.num_hidden_layers
