"""Host side of the fused decoder-layer forward (``layer_forward``), on CPU.

* The HF forwards that the fused ones restate have the same source text in
  every model family the fused forwards are installed on (a transformers
  upgrade that changes one of them fails here).
* ``fused_layer_ops`` installs instance forwards on the norms, MLPs and
  decoder layers and the rotary function of the attention's module, and
  removes all of them on exit -- also when the block raises.
* On CPU float32 tensors the fused forwards take the HF path: a layer's
  output is bit-identical with and without them (the structure of the
  restated decoder forward; the kernels themselves are checked on the GPU).
"""
import importlib
import inspect
import textwrap

import pytest
import torch

from llmcompressor_b200 import layer_forward as LF
from llmcompressor_b200 import synthetic

FAMILIES = {"llama": "Llama", "mistral": "Mistral", "qwen2": "Qwen2", "qwen3": "Qwen3", "qwen3_moe": "Qwen3Moe"}


def _src(obj) -> str:
    return textwrap.dedent(inspect.getsource(obj))


@pytest.mark.parametrize("family", sorted(FAMILIES))
def test_restated_forwards_have_one_source(family):
    base = importlib.import_module("transformers.models.llama.modeling_llama")
    mod = importlib.import_module(f"transformers.models.{family}.modeling_{family}")
    p = FAMILIES[family]
    for suffix, names in (("RMSNorm", LF.RMSNORM_CLASSES), ("MLP", LF.MLP_CLASSES),
                          ("DecoderLayer", LF.LAYER_CLASSES)):
        assert p + suffix in names
        assert _src(getattr(mod, p + suffix).forward) == _src(getattr(base, "Llama" + suffix).forward), (family, suffix)
    for fn in ("apply_rotary_pos_emb", "rotate_half"):
        assert _src(getattr(mod, fn)) == _src(getattr(base, fn)), (family, fn)


def _tiny_llama():
    cfg = synthetic.llama_config("c1")
    cfg.num_hidden_layers = 1
    cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads, cfg.num_key_value_heads = 64, 128, 4, 2
    cfg.head_dim = 16
    from transformers import LlamaForCausalLM

    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).float().eval()


def test_install_and_remove():
    import transformers.models.llama.modeling_llama as ML

    model = _tiny_llama()
    layer = model.model.layers[0]
    orig_rope = ML.apply_rotary_pos_emb
    with LF.fused_layer_ops(layer):
        assert "forward" in layer.__dict__
        assert "forward" in layer.input_layernorm.__dict__ and "forward" in layer.mlp.__dict__
        assert ML.apply_rotary_pos_emb is not orig_rope and ML.apply_rotary_pos_emb.llmc_fused_from is orig_rope
        with LF.fused_layer_ops(layer):  # nested: the outer forwards stay, nothing is wrapped twice
            assert ML.apply_rotary_pos_emb.llmc_fused_from is orig_rope
        assert "forward" in layer.__dict__
    assert all("forward" not in m.__dict__ for m in layer.modules())
    assert ML.apply_rotary_pos_emb is orig_rope
    with pytest.raises(RuntimeError, match="boom"):
        with LF.fused_layer_ops(layer):
            raise RuntimeError("boom")
    assert all("forward" not in m.__dict__ for m in layer.modules())
    assert ML.apply_rotary_pos_emb is orig_rope
    with LF.fused_layer_ops(layer, enabled=False):
        assert "forward" not in layer.__dict__


def test_cpu_float_path_is_the_hf_forward():
    model = _tiny_llama()
    ids = torch.randint(0, 1000, (2, 24))
    captured = {}

    def pre(mod, args, kwargs):
        captured["args"], captured["kwargs"] = args, kwargs

    layer = model.model.layers[0]
    h = layer.register_forward_pre_hook(pre, with_kwargs=True)
    with torch.no_grad():
        model(ids)
    h.remove()
    seen = {}
    hooks = [m.register_forward_pre_hook(lambda mod, a, n=n: seen.setdefault(n, []).append(a[0].clone()))
             for n, m in layer.named_modules() if isinstance(m, torch.nn.Linear)]
    with torch.no_grad():
        ref = layer(*captured["args"], **captured["kwargs"])
        ref_seen = {k: list(v) for k, v in seen.items()}
        seen.clear()
        with LF.fused_layer_ops(layer):
            out = layer(*captured["args"], **captured["kwargs"])
    for hk in hooks:
        hk.remove()
    ref = ref[0] if isinstance(ref, tuple) else ref
    out = out[0] if isinstance(out, tuple) else out
    assert torch.equal(out, ref)
    assert set(seen) == set(ref_seen) and len(seen) == 7
    for k in seen:  # every Linear still called as a module, on the same inputs
        assert all(torch.equal(a, b) for a, b in zip(seen[k], ref_seen[k])), k
