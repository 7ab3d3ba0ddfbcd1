"""Seeded random-init models and calibration tokens of the benchmark shapes.

There are no checkpoints or datasets on the machines this runs on, so the
end-to-end GPTQ runs use Llama-architecture models with random weights and
uniformly random token ids:

* ``c1``: 2 decoder layers, hidden 1024, intermediate 2816, 16 heads (8 KV
  heads), head_dim 64, vocab 32000, RMSNorm eps 1e-5, RoPE theta 500000;
  32 sequences x 512 tokens.
* ``llama3_8b``: the Llama-3-8B shape (32 layers, hidden 4096, intermediate
  14336, 32 heads / 8 KV heads, vocab 128256); 512 sequences x 2048 tokens.
* ``qwen3_30b_a3b``: the Qwen3-30B-A3B MoE shape (48 layers, hidden 2048,
  128 experts top-8, expert intermediate 768, 32 heads / 4 KV heads,
  head_dim 128, vocab 151936); 256 sequences x 2048 tokens.
* ``c3tiny``: a 2-layer Qwen3-MoE of that architecture at reduced width
  (hidden 256, 8 experts top-2, expert intermediate 128, 4 heads / 2 KV
  heads, head_dim 64, vocab 1000); 16 sequences x 256 tokens.

Every 2-D and 3-D parameter (Linear, embedding, router and fused expert
weights) is drawn ~N(0, 0.02) in float32 from one seeded generator, walking
the parameters in name order, and rounded to bf16; RMSNorm weights are ones.  Tokens are
``torch.randint(0, vocab, (n, L))`` from a generator seeded with 1.  The same
function builds the model for the fixture generator (the reference run on
CPU), the GPU tests and the benchmark, so all of them quantize identical
weights.
"""
from __future__ import annotations

import torch

CONFIGS = {
    "c1": dict(num_hidden_layers=2, hidden_size=1024, intermediate_size=2816, num_attention_heads=16,
               num_key_value_heads=8, head_dim=64, vocab_size=32000),
    "llama3_8b": dict(num_hidden_layers=32, hidden_size=4096, intermediate_size=14336, num_attention_heads=32,
                      num_key_value_heads=8, head_dim=128, vocab_size=128256),
}
MOE_CONFIGS = {
    "qwen3_30b_a3b": dict(num_hidden_layers=48, hidden_size=2048, moe_intermediate_size=768, num_experts=128,
                          num_experts_per_tok=8, num_attention_heads=32, num_key_value_heads=4, head_dim=128,
                          vocab_size=151936, intermediate_size=6144),
    "c3tiny": dict(num_hidden_layers=2, hidden_size=256, moe_intermediate_size=128, num_experts=8,
                   num_experts_per_tok=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                   vocab_size=1000, intermediate_size=512),
}
CALIBRATION = {"c1": (32, 512), "llama3_8b": (512, 2048), "qwen3_30b_a3b": (256, 2048), "c3tiny": (16, 256)}


def qwen3_moe_config(name: str, **overrides):
    from transformers import Qwen3MoeConfig

    kw = dict(MOE_CONFIGS[name])
    kw.update(rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=False, max_position_embeddings=8192,
              norm_topk_prob=True, decoder_sparse_step=1, mlp_only_layers=[])
    kw.update(overrides)
    cfg = Qwen3MoeConfig(**kw)
    cfg._attn_implementation = "sdpa"
    return cfg


def llama_config(name: str, **overrides):
    from transformers import LlamaConfig

    kw = dict(CONFIGS[name])
    kw.update(rms_norm_eps=1e-5, rope_theta=5e5, tie_word_embeddings=False, max_position_embeddings=8192)
    kw.update(overrides)
    cfg = LlamaConfig(**kw)
    cfg._attn_implementation = "sdpa"
    return cfg


@torch.no_grad()
def random_llama(name: str = "c1", seed: int = 0, device: str | torch.device = "cpu", init_device=None, **overrides):
    """``LlamaForCausalLM`` of config ``name`` in bf16 with seeded ~N(0, 0.02)
    weights.  ``init_device``: where the random numbers are drawn ("cpu" by
    default: the same values on every machine; "cuda" draws on the GPU, much
    faster for large models but with other values)."""
    from transformers import LlamaForCausalLM

    return _random(LlamaForCausalLM, llama_config(name, **overrides), seed, device, init_device)


@torch.no_grad()
def random_qwen3_moe(name: str = "c3tiny", seed: int = 0, device: str | torch.device = "cpu", init_device=None,
                     **overrides):
    """``Qwen3MoeForCausalLM`` of config ``name`` (fused experts, as
    transformers builds it) in bf16 with seeded ~N(0, 0.02) weights."""
    from transformers import Qwen3MoeForCausalLM

    return _random(Qwen3MoeForCausalLM, qwen3_moe_config(name, **overrides), seed, device, init_device)


def _random(model_cls, cfg, seed, device, init_device):
    init_device = torch.device(init_device or "cpu")
    with torch.device("meta"):
        model = model_cls(cfg)
    model = model.to_empty(device=device).to(torch.bfloat16)
    g = torch.Generator(device=init_device).manual_seed(seed)
    for _, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
        if p.ndim >= 2:
            p.copy_((0.02 * torch.randn(p.shape, generator=g, device=init_device)).to(torch.bfloat16))
        else:
            p.fill_(1.0)  # RMSNorm weights
    # buffers (rotary frequencies) were never materialised: rebuild the modules that own them
    for mod in model.modules():
        if "inv_freq" in getattr(mod, "_buffers", {}):
            fresh = type(mod)(mod.config, device=torch.device(device))
            for bname, buf in fresh.named_buffers(recurse=False):
                mod._buffers[bname] = buf  # float32, as a checkpoint-loaded model keeps them
            mod.attention_scaling = fresh.attention_scaling
    model.eval()
    return model


def calibration_tokens(name: str = "c1", n: int | None = None, seq_len: int | None = None, seed: int = 1,
                       vocab: int | None = None) -> torch.Tensor:
    """(n, seq_len) int64 token ids, uniform over the vocabulary."""
    n0, l0 = CALIBRATION[name]
    n = n or n0
    seq_len = seq_len or l0
    vocab = vocab or (CONFIGS.get(name) or MOE_CONFIGS[name])["vocab_size"]
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, seq_len), generator=g)
