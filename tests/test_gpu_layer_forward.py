"""The fused decoder-layer kernels (``csrc/layer_ops.cu``) against the HF
eager ops they replace, on the GPU.

* rotary (``apply_rotary_pos_emb``) and SiLU * up: bit-identical, on the
  transposed projection views the attention passes, batch-shared and
  per-batch cos / sin.
* RMSNorm: the float32 sum of squares runs in another order than torch's
  reduction, so bf16(x * rsqrt(...)) may move by one bf16 unit, which the
  weight product can turn into two units of the output when it crosses a
  power of two: with unit weights at most one unit, with random weights at
  most two; >= 99.5% of values bit-identical either way.  The residual
  output of the fused add + norm is bit-identical to ``residual + x``.
* A whole Llama-3-8B-shaped decoder layer (one layer, 2 x 2048 tokens) and a
  Qwen3-MoE-shaped one: the fused forward's output within 1% relative
  Frobenius error of the eager one; the calibration hooks see the same
  q/k/v inputs (RMSNorm output) to one bf16 unit and the same MLP inputs
  within 1%.
"""
import pytest
import torch

from llmcompressor_b200 import layer_forward as LF
from llmcompressor_b200 import synthetic

pytestmark = pytest.mark.gpu


def _bf16_units(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in bf16 units (ordered integer representation)."""
    def ordered(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -32768 - i, i)

    return (ordered(a) - ordered(b)).abs()


def test_rotary_bit_identical():
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    g = torch.Generator(device="cuda").manual_seed(0)
    for B, S, H, Hk, D, shared in ((2, 300, 8, 2, 128, True), (3, 64, 4, 4, 64, False), (1, 17, 2, 1, 16, True)):
        q = torch.randn(B, S, H * D, device="cuda", generator=g).to(torch.bfloat16).view(B, S, H, D).transpose(1, 2)
        k = torch.randn(B, S, Hk * D, device="cuda", generator=g).to(torch.bfloat16).view(B, S, Hk, D).transpose(1, 2)
        nb = 1 if shared else B
        ang = torch.rand(nb, S, D // 2, device="cuda", generator=g) * 100
        emb = torch.cat([ang, ang], dim=-1)
        cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
        rq, rk = apply_rotary_pos_emb(q, k, cos, sin)
        assert LF._rotary_ok(q, cos, sin) and LF._rotary_ok(k, cos, sin)
        fq, fk = LF.rotary(q, cos, sin), LF.rotary(k, cos, sin)
        assert fq.shape == rq.shape and fk.shape == rk.shape
        assert torch.equal(fq, rq) and torch.equal(fk, rk), (B, S, H, D)


def _same_bits_or_nan(ours, ref):
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(ours), nan)
    assert torch.equal(ours[~nan].view(torch.int16), ref[~nan].view(torch.int16))


def test_silu_mul_every_bf16_gate():
    """Every bf16 bit pattern as the gate (zeros, subnormals, infinities,
    NaNs), times 1 and times random up values: the same bits as torch's
    SiLU and product (NaN as NaN)."""
    g = torch.arange(-32768, 32768, dtype=torch.int32, device="cuda").to(torch.int16).view(torch.bfloat16)
    one = torch.ones_like(g)
    _same_bits_or_nan(LF.silu_mul(g, one), torch.nn.functional.silu(g) * one)
    gen = torch.Generator(device="cuda").manual_seed(5)
    u = (torch.randn(g.numel(), device="cuda", generator=gen) * 3).to(torch.bfloat16)
    _same_bits_or_nan(LF.silu_mul(g, u), torch.nn.functional.silu(g) * u)
    # the stacked-expert kernel (act output) on the same values
    act, _ = LF.silu_mul_scaled(g.view(256, 256), u.view(256, 256), 64, None, act=True, scaled=False)
    _same_bits_or_nan(act.reshape(-1), torch.nn.functional.silu(g) * u)


def test_silu_mul_bit_identical():
    g = torch.Generator(device="cuda").manual_seed(1)
    for n in (8, 4096 * 37, 14336 * 300):
        a = (torch.randn(n, device="cuda", generator=g) * 4).to(torch.bfloat16)
        b = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
        assert torch.equal(LF.silu_mul(a, b), torch.nn.functional.silu(a) * b), n


@pytest.mark.parametrize("unit_weight", [True, False])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1000, 128), (37, 2048), (5, 8)])
def test_rmsnorm_within_units(rows, cols, unit_weight):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    norm = LlamaRMSNorm(cols, eps=1e-5).cuda().to(torch.bfloat16)
    if not unit_weight:
        norm.weight.data.copy_((1 + 0.1 * torch.randn(cols, device="cuda", generator=g)).to(torch.bfloat16))
    bound = 1 if unit_weight else 2
    x = (torch.randn(rows, cols, device="cuda", generator=g) * 3).to(torch.bfloat16)
    r = torch.randn(rows, cols, device="cuda", generator=g).to(torch.bfloat16)
    with torch.no_grad():
        ref = norm(x)
        ours = LF.rmsnorm(x, norm.weight, norm.variance_epsilon)
        d = _bf16_units(ours, ref)
        assert int(d.max()) <= bound and float((d == 0).float().mean()) >= 0.995
        h_ref = r + x
        h, out = LF.rmsnorm(x, norm.weight, norm.variance_epsilon, residual=r)
        assert torch.equal(h, h_ref)
        d = _bf16_units(out, norm(h_ref))
        assert int(d.max()) <= bound and float((d == 0).float().mean()) >= 0.995


class _Stop(Exception):
    pass


def _layer_inputs(model, ids):
    got = {}

    def pre(mod, args, kwargs):
        got["args"], got["kwargs"] = args, kwargs
        raise _Stop

    layer = model.model.layers[0]
    h = layer.register_forward_pre_hook(pre, with_kwargs=True)
    try:
        with torch.no_grad():
            model.model(ids)
    except _Stop:
        pass
    h.remove()
    return got["args"], got["kwargs"]


def _compare_layer(model, ids):
    layer = model.model.layers[0]
    args, kwargs = _layer_inputs(model, ids)
    seen = {}
    names = [n for n, m in layer.named_modules() if n.endswith(("q_proj", "gate_proj")) and
             isinstance(m, torch.nn.Linear)][:2]
    hooks = [layer.get_submodule(n).register_forward_pre_hook(
        lambda mod, a, n=n: seen.setdefault(n, []).append(a[0].clone())) for n in names]
    with torch.no_grad():
        ref = layer(*args, **kwargs)
        ref_seen = dict(seen)
        seen.clear()
        with LF.fused_layer_ops(layer):
            out = layer(*args, **kwargs)
    for hk in hooks:
        hk.remove()
    ref = ref[0] if isinstance(ref, tuple) else ref
    out = out[0] if isinstance(out, tuple) else out
    rel = float(torch.linalg.norm((out.float() - ref.float())) / torch.linalg.norm(ref.float()))
    assert rel < 0.01, rel
    for n in names:
        a, b = seen[n][0].float(), ref_seen[n][0].float()
        if n.endswith("q_proj"):  # input_layernorm's output: one bf16 unit at most
            assert int(_bf16_units(seen[n][0], ref_seen[n][0]).max()) <= 1, n
        else:  # after attention: the norm's unit differences have gone through it
            assert float(torch.linalg.norm(a - b) / torch.linalg.norm(b)) < 0.01, n
    return rel


def test_llama3_8b_layer():
    model = synthetic.random_llama("llama3_8b", device="cuda", init_device="cuda", num_hidden_layers=1)
    ids = torch.randint(0, model.config.vocab_size, (2, 2048), device="cuda")
    _compare_layer(model, ids)


def test_qwen3_moe_layer():
    from llmcompressor_b200 import moe

    model = synthetic.random_qwen3_moe("c3tiny").cuda()
    moe.linearize_experts(model)
    ids = synthetic.calibration_tokens("c3tiny")[:4].cuda()
    with moe.calibrate_all_experts(True):
        _compare_layer(model, ids)


def test_deferred_down_projection_is_the_same_output():
    """The propagation pass may stop a layer before its down projection
    (``defer_down``) and finish it later (``finish_deferred``): the same
    bits as the whole fused forward."""
    model = synthetic.random_llama("c1", device="cuda")
    layer = model.model.layers[1]
    ids = synthetic.calibration_tokens("c1")[:4].cuda()
    args, kwargs = _layer_inputs(model, ids)
    assert LF.deferrable_down(layer) is layer.mlp.down_proj
    with torch.no_grad(), LF.fused_layer_ops(layer):
        whole = layer(*args, **kwargs)
        store = []
        with LF.defer_down(store):
            assert layer(*args, **kwargs) is None
        late = LF.finish_deferred(store[0])
    whole = whole[0] if isinstance(whole, tuple) else whole
    assert torch.equal(late, whole)
