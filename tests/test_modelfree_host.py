"""Host logic of the model-free shard driver (CPU only): fused-set grouping,
MoE expert splitting, tensor selection and file assignment."""
import torch
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

from llmcompressor_b200 import modelfree


def test_fused_groups_follow_reference_families():
    names = [
        "model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.k_proj.weight",
        "model.layers.0.self_attn.v_proj.weight", "model.layers.0.self_attn.o_proj.weight",
        "model.layers.0.mlp.gate_proj.weight", "model.layers.0.mlp.up_proj.weight",
        "model.layers.0.mlp.down_proj.weight", "model.layers.1.self_attn.q_proj.weight",
        "model.layers.3.self_attn.wq_a.weight", "model.layers.3.self_attn.wkv_a_with_mqa.weight",
        "model.layers.4.block_sparse_moe.experts.7.w1.weight", "model.layers.4.block_sparse_moe.experts.7.w3.weight",
        "model.layers.4.block_sparse_moe.experts.7.w2.weight",
    ]
    groups = sorted(modelfree.fused_groups(names))
    assert ["model.layers.0.mlp.gate_proj.weight", "model.layers.0.mlp.up_proj.weight"] in groups
    assert ["model.layers.0.self_attn.k_proj.weight", "model.layers.0.self_attn.q_proj.weight",
            "model.layers.0.self_attn.v_proj.weight"] in groups
    assert ["model.layers.1.self_attn.q_proj.weight"] in groups  # a partial set stays a set
    assert ["model.layers.3.self_attn.wkv_a_with_mqa.weight", "model.layers.3.self_attn.wq_a.weight"] in groups
    assert ["model.layers.4.block_sparse_moe.experts.7.w1.weight",
            "model.layers.4.block_sparse_moe.experts.7.w3.weight"] in groups
    flat = {n for g in groups for n in g}
    assert "model.layers.0.self_attn.o_proj.weight" not in flat
    assert "model.layers.0.mlp.down_proj.weight" not in flat


def test_split_fused_moe_experts_like_reference():
    gu = torch.arange(2 * 6 * 4, dtype=torch.float32).reshape(2, 6, 4)
    dn = torch.arange(2 * 4 * 3, dtype=torch.float32).reshape(2, 4, 3)
    out = modelfree.split_fused_moe_experts({"m.experts.gate_up_proj": gu, "m.experts.down_proj": dn,
                                             "m.norm.weight": torch.ones(4)})
    assert set(out) == {"m.experts.0.gate_proj.weight", "m.experts.0.up_proj.weight", "m.experts.1.gate_proj.weight",
                        "m.experts.1.up_proj.weight", "m.experts.0.down_proj.weight", "m.experts.1.down_proj.weight",
                        "m.norm.weight"}
    assert torch.equal(out["m.experts.1.up_proj.weight"], gu[1, 3:])
    assert torch.equal(out["m.experts.0.down_proj.weight"], dn[0])


def test_quantizable_skips_norms_ignored_and_non_weights():
    t = {"a.q_proj.weight": torch.zeros(2, 2), "a.input_layernorm.weight": torch.zeros(2),
         "lm_head.weight": torch.zeros(2, 2), "a.q_proj.bias": torch.zeros(2)}
    scheme = preset_name_to_scheme("W4A16", ["Linear"])
    got = modelfree.quantizable(t, ["lm_head"], scheme.targets)
    assert got == [("a.q_proj", "a.q_proj.weight")]
    assert modelfree.is_microscale_scheme(preset_name_to_scheme("NVFP4A16", ["Linear"]))
    assert not modelfree.is_microscale_scheme(preset_name_to_scheme("MXFP4A16", ["Linear"]))


def test_assign_files_balances_bytes():
    sizes = {"a": 10, "b": 9, "c": 5, "d": 4, "e": 1}
    own = modelfree.assign_files(sizes, 2)
    load = [sum(s for f, s in sizes.items() if own[f] == r) for r in range(2)]
    assert sorted(load) == [14, 15]
    assert modelfree.assign_files(sizes, 1) == {f: 0 for f in sizes}
