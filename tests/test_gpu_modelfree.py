"""GPU model-free shard driver (S/entrypoints/model_free/process.py) end to end:
a synthetic safetensors shard in, the compressed shard out, every quantized
tensor bit-exact against the CPU oracle (NVFP4 with the fused-set global
scales of q/k/v and gate/up)."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme
from safetensors.torch import load_file, save_file

from gpu_util import bits, np_f32, rand_bf16
from llmcompressor_b200 import modelfree
from oracle import casts as ocasts
from oracle import numerics as onum

pytestmark = pytest.mark.gpu


def _shard(seed=0):
    H, I, E = 256, 384, 2
    t = {
        "model.layers.0.self_attn.q_proj.weight": rand_bf16(256, H, seed + 1),
        "model.layers.0.self_attn.k_proj.weight": rand_bf16(128, H, seed + 2),
        "model.layers.0.self_attn.v_proj.weight": rand_bf16(128, H, seed + 3),
        "model.layers.0.self_attn.o_proj.weight": rand_bf16(H, 256, seed + 4),
        "model.layers.0.mlp.gate_proj.weight": rand_bf16(I, H, seed + 5, kind="student_t"),
        "model.layers.0.mlp.up_proj.weight": rand_bf16(I, H, seed + 6),
        "model.layers.0.mlp.down_proj.weight": rand_bf16(H, I, seed + 7),
        "model.layers.0.input_layernorm.weight": torch.ones(H, dtype=torch.bfloat16),
        "lm_head.weight": rand_bf16(64, H, seed + 8),
        "model.layers.1.mlp.experts.gate_up_proj": torch.stack([rand_bf16(2 * 128, H, seed + 9 + e) for e in range(E)]),
        "model.layers.1.mlp.experts.down_proj": torch.stack([rand_bf16(H, 128, seed + 20 + e) for e in range(E)]),
    }
    return t


@pytest.mark.parametrize("scheme_name", ["W4A16", "NVFP4A16", "FP8_BLOCK", "MXFP4A16"])
def test_process_file_bit_exact(tmp_path, scheme_name):
    src = _shard()
    path = tmp_path / "model-00001-of-00001.safetensors"
    save_file(src, str(path))
    scheme = preset_name_to_scheme(scheme_name, ["Linear"])
    out_path = tmp_path / "out" / path.name
    total, wmap = modelfree.process_file(path, out_path, scheme, ignore=["lm_head"])
    got = load_file(str(out_path))
    assert total == sum(v.nbytes for v in got.values())
    assert set(wmap) == set(got)
    # untouched tensors pass through
    assert torch.equal(got["lm_head.weight"], src["lm_head.weight"])
    assert torch.equal(got["model.layers.0.input_layernorm.weight"], src["model.layers.0.input_layernorm.weight"])
    split = modelfree.split_fused_moe_experts(src)
    names = [n for _, n in modelfree.quantizable(split, ["lm_head"], scheme.targets)]
    assert "model.layers.1.mlp.experts.1.up_proj.weight" in names
    gs = {}
    if modelfree.is_microscale_scheme(scheme):
        for grp in modelfree.fused_groups(names):
            g = ocasts.nvfp4_global_scale([np_f32(split[n]) for n in grp])
            gs.update({n: g for n in grp})
    for n in names:
        ref = ocasts.modelfree_tensor(np_f32(split[n].contiguous()), scheme_name, global_scale=gs.get(n))
        mod = n[: -len(".weight")]
        if "weight" not in ref:  # packed formats replace the weight
            assert f"{mod}.weight" not in got
        for k, v in ref.items():
            key = f"{mod}.{k}"
            assert key in got, key
            g = bits(got[key])
            if v.dtype == np.float32 and k == "weight_scale":
                v = onum.f32_to_bf16_bits(v)
            np.testing.assert_array_equal(g.reshape(v.shape), v, err_msg=key)
