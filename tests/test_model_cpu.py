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


def test_shard_masks_follow_the_reference_engine():
    """worker.py:55-75: prefill keeps causal keys inside each row's length and
    expert entries inside it; decode step t sees the row's prompt keys and
    every decode column written so far; positions continue each row's own."""
    cfg = ModelConfig(hidden_size=64, intermediate_size=32, num_hidden_layers=1,
                      num_attention_heads=2, num_key_value_heads=1, num_local_experts=4,
                      num_experts_per_tok=2, vocab_size=16, rms_norm_eps=1e-6, rope_theta=1e4,
                      embedding_multiplier=1.0, attention_multiplier=0.125,
                      residual_multiplier=1.0, logits_scaling=1.0, max_position_embeddings=32)
    sh = Shard([[1, 2, 3], [4], [5, 6]], cfg, 2, "cpu", torch.float32)
    assert (sh.T, sh.cap) == (3, 5)
    assert sh.input.tolist() == [[1, 2, 3], [4, 0, 0], [5, 6, 0]]
    mask, valid = sh.prefill_masks()
    assert valid.tolist() == [[True] * 3, [True, False, False], [True, True, False]]
    # row 1, query 2 (padding): only its valid key 0
    assert mask[1, 0, 2].tolist() == [True, False, False]
    assert mask[0, 0].tolist() == [[True, False, False], [True, True, False], [True, True, True]]
    sh.used = sh.T
    assert sh.decode_mask()[:, 0, 0].tolist() == [[True, True, True, True],
                                                   [True, False, False, True],
                                                   [True, True, False, True]]
    assert sh.decode_positions().view(-1).tolist() == [3, 1, 2]
    sh.used, sh.decoded = sh.T + 1, 1
    assert sh.decode_mask()[1, 0, 0].tolist() == [True, False, False, True, True]
    assert sh.decode_positions().view(-1).tolist() == [4, 2, 3]
