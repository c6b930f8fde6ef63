"""Model geometry, seeded weights and request stream of the runner fixture
(runner_steps.npz).

make_golden.py runs the reference's TinyQwen2ForCausalLM, build_model_batch
and execute_model_batch (runtime/model_runner.py:37-272) on them; the runner
tests replay the recorded steps through this package.  Weights come from a
seeded CPU generator on both sides, so the fixture holds only the request
stream and the reference's outputs.  head_dim 64 and block_size 16 put the
BF16 run on the tensor-core prefill and the balanced decode.
"""

from __future__ import annotations

import torch

CONFIG = dict(vocab_size=64, hidden_size=128, intermediate_size=128, num_hidden_layers=2, num_attention_heads=2,
              num_key_value_heads=1, max_position_embeddings=128, rope_theta=1_000_000.0, rms_norm_eps=1e-6)
BLOCK_SIZE = 16
NUM_BLOCKS = 24
PROMPT_LENS = {"A": 37, "B": 5, "C": 16, "D": 23}
BLOCKS_PER_REQUEST = {"A": 3, "B": 1, "C": 2, "D": 2}
# Step 1: whole prompts A, B, C.  Step 2: prompt D with decodes of A, B, C.
# Step 3: decodes of A, B, C, D.
STEPS = [(["A", "B", "C"], []), (["D"], ["A", "B", "C"]), ([], ["A", "B", "C", "D"])]


def weights(seed: int = 7) -> dict[str, torch.Tensor]:
    """FP32 state dict under the reference's parameter names."""
    g = torch.Generator().manual_seed(seed)
    h, inter, vocab = CONFIG["hidden_size"], CONFIG["intermediate_size"], CONFIG["vocab_size"]
    d = h // CONFIG["num_attention_heads"]
    hq, hkv = CONFIG["num_attention_heads"] * d, CONFIG["num_key_value_heads"] * d

    def lin(out_f, in_f):
        return (torch.rand(out_f, in_f, generator=g) * 2 - 1) / in_f ** 0.5

    def vec(n, lo, hi):
        return torch.rand(n, generator=g) * (hi - lo) + lo

    sd = {"model.embed_tokens.weight": torch.randn(vocab, h, generator=g)}
    for i in range(CONFIG["num_hidden_layers"]):
        p = f"model.layers.{i}."
        sd[p + "self_attn.qkv_proj.q_proj.weight"] = lin(hq, h)
        sd[p + "self_attn.qkv_proj.q_proj.bias"] = vec(hq, -0.5, 0.5)
        sd[p + "self_attn.qkv_proj.v_proj.weight"] = lin(hkv, h)
        sd[p + "self_attn.qkv_proj.v_proj.bias"] = vec(hkv, -0.5, 0.5)
        sd[p + "self_attn.qkv_proj.k_proj.weight"] = lin(hkv, h)
        sd[p + "self_attn.qkv_proj.k_proj.bias"] = vec(hkv, -0.5, 0.5)
        sd[p + "self_attn.o_proj.weight"] = lin(h, h)
        sd[p + "mlp.gate_proj.weight"] = lin(inter, h)
        sd[p + "mlp.up_proj.weight"] = lin(inter, h)
        sd[p + "mlp.down_proj.weight"] = lin(h, inter)
        sd[p + "input_layernorm.weight"] = vec(h, 0.5, 1.5)
        sd[p + "post_attention_layernorm.weight"] = vec(h, 0.5, 1.5)
    sd["model.norm.weight"] = vec(h, 0.5, 1.5)
    sd["lm_head.weight"] = lin(vocab, h)
    return sd


def prompts(seed: int = 3) -> dict[str, list[int]]:
    g = torch.Generator().manual_seed(seed)
    return {rid: torch.randint(0, CONFIG["vocab_size"], (n,), generator=g).tolist() for rid, n in PROMPT_LENS.items()}


def block_tables(seed: int = 5) -> dict[str, list[int]]:
    perm = torch.randperm(NUM_BLOCKS, generator=torch.Generator().manual_seed(seed)).tolist()
    out, cur = {}, 0
    for rid, n in BLOCKS_PER_REQUEST.items():
        out[rid] = perm[cur:cur + n]
        cur += n
    return out
