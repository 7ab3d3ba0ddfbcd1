"""Fused elementwise forward of Llama-family decoder layers for the
sequential calibration pipeline.

The reference's sequential pipeline (S/pipelines/sequential/pipeline.py:70-118)
runs each decoder layer's HF forward eagerly, once to calibrate and once to
propagate.  Its elementwise ops -- RMSNorm's float32 detour (LlamaRMSNorm),
rotary's ``cat``/``neg``/mul/add (``apply_rotary_pos_emb``), SiLU and the
gate*up product (LlamaMLP), the residual adds (LlamaDecoderLayer) -- each make
full passes over the activations and cost about as much as the layer's GEMMs.

``fused_layer_ops(layer)`` installs, for the duration of a ``with`` block,
instance-level forwards that run each of those as one kernel of
``csrc/layer_ops.cu``, while every Linear is still called as a module (so the
calibration hooks see the same inputs):

* RMSNorm modules of the Llama family -> ``llmc_rmsnorm_bf16``;
* the decoder layer's post-attention ``residual + h`` and its
  ``post_attention_layernorm`` -> one ``llmc_rmsnorm_bf16`` with residual;
* MLPs with SiLU (dense and the per-expert MLPs of linearized MoE blocks) ->
  gate / up / down as module calls, SiLU * up fused;
* ``apply_rotary_pos_emb`` of the attention's module -> ``llmc_rotary_bf16``.

The roundings are those of the eager ops: rotary, SiLU * up and the residual
add give the same bits; RMSNorm sums its float32 squares in another order.
Modules with hooks of their own, dtypes other than bf16 and layouts the
kernels do not take keep the HF forward: these are the reference's own ops on
the GPU, not a CPU path.
"""
from __future__ import annotations

import contextlib
import ctypes
import sys
import types

import torch

from . import _lib

_P, _I64, _F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
_lib.extend_signatures({
    "llmc_rmsnorm_bf16": [_P, _P, _I64, _I64, _P, _F, _P, _P, _P],
    "llmc_rotary_bf16": [_P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _P, _P],
    "llmc_silu_mul_bf16": [_P, _P, _I64, _P, _P],
    "llmc_silu_mul_scaled_bf16": [_P, _P, _I64, _I64, _I64, _P, _I64, _P, _P, _P],
    "llmc_scale_groups_bf16": [_P, _I64, _I64, _I64, _P, _I64, _P, _P],
    "llmc_moe_combine_bf16": [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _P],
})

# HF classes whose forwards the fused ones restate (the same source text in
# every one of them; tests/test_layer_forward.py checks it).
RMSNORM_CLASSES = ("LlamaRMSNorm", "MistralRMSNorm", "Qwen2RMSNorm", "Qwen3RMSNorm", "Qwen3MoeRMSNorm")
MLP_CLASSES = ("LlamaMLP", "MistralMLP", "Qwen2MLP", "Qwen3MLP", "Qwen3MoeMLP", "ExpertMLP")
LAYER_CLASSES = ("LlamaDecoderLayer", "MistralDecoderLayer", "Qwen2DecoderLayer", "Qwen3DecoderLayer",
                 "Qwen3MoeDecoderLayer")


def _aligned(*ts: torch.Tensor) -> bool:
    return all(t.data_ptr() % 16 == 0 for t in ts)


def _hooked(m: torch.nn.Module) -> bool:
    return bool(m._forward_hooks or m._forward_pre_hooks or getattr(m, "_forward_hooks_with_kwargs", None))


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """``weight * bf16(x * rsqrt(mean(x^2) + eps))`` over the last dim; with
    ``residual``, x is first replaced by ``residual + x`` and the pair
    ``(residual + x, normed)`` is returned."""
    cols = x.shape[-1]
    out = torch.empty_like(x)
    res_out = torch.empty_like(x) if residual is not None else None
    _lib.check(_lib.lib().llmc_rmsnorm_bf16(
        x.data_ptr(), _lib.ptr(residual), x.numel() // cols, cols, weight.data_ptr(), float(eps), out.data_ptr(),
        _lib.ptr(res_out), _lib.stream_ptr(x.device)), "rmsnorm")
    return (res_out, out) if residual is not None else out


def _norm_ok(x: torch.Tensor, weight: torch.Tensor, *others: torch.Tensor) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and x.is_contiguous()
            and weight.is_contiguous() and weight.dim() == 1 and weight.numel() == x.shape[-1]
            and x.shape[-1] % 8 == 0 and _aligned(x, weight, *others)
            and all(o.shape == x.shape and o.dtype == x.dtype and o.is_contiguous() for o in others))


def rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x * cos + rotate_half(x) * sin`` for x (batch, heads, seq, head_dim)
    and cos / sin (batch or 1, seq, head_dim); the result is laid out
    (batch, seq, heads, head_dim) in memory, as the eager ops lay it out for
    the transposed projection views, and returned as (batch, heads, seq,
    head_dim)."""
    B, H, S, D = x.shape
    out = torch.empty((B, S, H, D), dtype=x.dtype, device=x.device)
    cb = cos.stride(0) if cos.shape[0] > 1 else 0
    _lib.check(_lib.lib().llmc_rotary_bf16(
        x.data_ptr(), B, H, S, D, x.stride(0), x.stride(1), x.stride(2), cos.data_ptr(), sin.data_ptr(), cb,
        out.data_ptr(), _lib.stream_ptr(x.device)), "rotary")
    return out.transpose(1, 2)


def _rotary_ok(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> bool:
    if not (x.dim() == 4 and cos.dim() == 3 and x.dtype == cos.dtype == sin.dtype == torch.bfloat16 and x.is_cuda):
        return False
    B, H, S, D = x.shape
    if cos.shape != sin.shape or cos.shape[1:] != (S, D) or cos.shape[0] not in (1, B) or cos.stride() != sin.stride():
        return False
    if x.stride(3) != 1 or cos.stride(2) != 1 or cos.stride(1) != D or D % 16:
        return False
    if any(s % 8 for s in (x.stride(0), x.stride(1), x.stride(2), cos.stride(0))):
        return False
    return _aligned(x, cos, sin)


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(g)
    _lib.check(_lib.lib().llmc_silu_mul_bf16(g.data_ptr(), u.data_ptr(), g.numel(), out.data_ptr(),
                                             _lib.stream_ptr(g.device)), "silu_mul")
    return out


def silu_mul_scaled(g: torch.Tensor, u: torch.Tensor, group: int, weights: torch.Tensor | None,
                    act: bool = True, scaled: bool = True):
    """For stacked expert projections g, u (rows, E * group): ``act`` =
    bf16(silu(g)) * u and ``scaled`` = bf16(act * weights[row, e]) (float32
    dense routing weights (rows, E), zero where not routed -> exact zero).
    Returns (act or None, scaled or None)."""
    rows, cols = g.shape
    a = torch.empty_like(g) if act else None
    sc = torch.empty_like(g) if scaled else None
    _lib.check(_lib.lib().llmc_silu_mul_scaled_bf16(
        g.data_ptr(), u.data_ptr(), rows, cols, group, _lib.ptr(weights) if scaled else None,
        weights.stride(0) if scaled else 0, _lib.ptr(a), _lib.ptr(sc), _lib.stream_ptr(g.device)), "silu_mul_scaled")
    return a, sc


def scale_groups(x: torch.Tensor, group: int, weights: torch.Tensor) -> torch.Tensor:
    """bf16(x * weights[row, column // group]) (zero weight -> exact zero)."""
    rows, cols = x.shape
    out = torch.empty_like(x)
    _lib.check(_lib.lib().llmc_scale_groups_bf16(x.data_ptr(), rows, cols, group, weights.data_ptr(),
                                                 weights.stride(0), out.data_ptr(), _lib.stream_ptr(x.device)),
               "scale_groups")
    return out


def moe_combine(y: torch.Tensor, pos: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """out[t] = sum over k of bf16(y[pos[t, k]] * weights[t, k]), added in k
    order with a bf16 rounding per add (the per-expert ``index_add_``)."""
    T, K = pos.shape
    out = torch.empty(T, y.shape[1], dtype=y.dtype, device=y.device)
    pos = pos.to(torch.int32).contiguous()
    weights = weights.to(torch.float32).contiguous()
    _lib.check(_lib.lib().llmc_moe_combine_bf16(y.data_ptr(), y.shape[0], pos.data_ptr(), weights.data_ptr(), T, K,
                                                y.shape[1], out.data_ptr(), _lib.stream_ptr(y.device)), "moe_combine")
    return out


def _silu(act) -> bool:
    from transformers.activations import SiLUActivation

    return isinstance(act, (torch.nn.SiLU, SiLUActivation))


# ------------------------------------------------------------ forwards
def _norm_forward(self, hidden_states):
    w = self.weight
    if _norm_ok(hidden_states, w):
        return rmsnorm(hidden_states, w, self.variance_epsilon)
    return type(self).forward(self, hidden_states)


def _mlp_forward(self, x):
    g = self.gate_proj(x)
    u = self.up_proj(x)
    if (g.dtype == u.dtype == torch.bfloat16 and g.shape == u.shape and g.is_contiguous() and u.is_contiguous()
            and g.numel() % 8 == 0 and _aligned(g, u)):
        return self.down_proj(silu_mul(g, u))
    return self.down_proj(self.act_fn(g) * u)


# While a list is set here, decoder layers whose MLP can defer stop before
# the down projection: they append (mlp, act, residual) and return None, and
# the caller finishes them later with ``finish_deferred`` (the propagation
# pass runs the layer's other GEMMs while the down projection is still being
# quantized).
_DEFER: list | None = None


@contextlib.contextmanager
def defer_down(store: list):
    """Within the block, layers with fused forwards whose MLP can defer
    (``deferrable_down``) put their down projection's input into ``store``
    instead of finishing."""
    global _DEFER
    prev, _DEFER = _DEFER, store
    try:
        yield
    finally:
        _DEFER = prev


def deferrable_down(layer: torch.nn.Module) -> torch.nn.Module | None:
    """The down projection a decoder layer can defer (a Llama-family layer
    and SiLU MLP the fused forwards take, no hooks on the MLP or the down
    projection), else None."""
    mlp = getattr(layer, "mlp", None)
    if (mlp is None or not _module_classes(layer, LAYER_CLASSES) or not _module_classes(mlp, MLP_CLASSES)
            or not _silu(getattr(mlp, "act_fn", None))):
        return None
    down = getattr(mlp, "down_proj", None)
    if down is None or _hooked(mlp) or _hooked(down):
        return None
    return down


def finish_deferred(item) -> torch.Tensor:
    """The layer output of a deferred (mlp, act, residual): residual +
    down_proj(act), as the decoder layer adds it."""
    mlp, act, residual = item
    return residual + mlp.down_proj(act)


def _layer_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                   use_cache=False, position_embeddings=None, **kwargs):
    """LlamaDecoderLayer.forward with the post-attention residual add fused
    into post_attention_layernorm."""
    residual = hidden_states
    h = self.input_layernorm(hidden_states)
    h, _ = self.self_attn(hidden_states=h, attention_mask=attention_mask, position_ids=position_ids,
                          past_key_values=past_key_values, use_cache=use_cache,
                          position_embeddings=position_embeddings, **kwargs)
    norm = self.post_attention_layernorm
    if not _hooked(norm) and _norm_ok(h, norm.weight, residual):
        residual, h = rmsnorm(h, norm.weight, norm.variance_epsilon, residual=residual)
    else:
        residual = residual + h
        h = norm(residual)
    mlp = self.mlp
    if _DEFER is not None and mlp.__dict__.get("forward") is not None and deferrable_down(self) is not None:
        g = mlp.gate_proj(h)
        u = mlp.up_proj(h)
        if (g.dtype == u.dtype == torch.bfloat16 and g.shape == u.shape and g.is_contiguous()
                and u.is_contiguous() and g.numel() % 8 == 0 and _aligned(g, u)):
            act = silu_mul(g, u)
        else:
            act = mlp.act_fn(g) * u
        _DEFER.append((mlp, act, residual))
        return None
    h = mlp(h)
    return residual + h


def _make_rotary(orig):
    def apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=1):
        if unsqueeze_dim == 1 and _rotary_ok(q, cos, sin) and _rotary_ok(k, cos, sin):
            return rotary(q, cos, sin), rotary(k, cos, sin)
        return orig(q, k, cos, sin, unsqueeze_dim)

    apply_rotary_pos_emb.llmc_fused_from = orig
    return apply_rotary_pos_emb


def _module_classes(m: torch.nn.Module, names) -> bool:
    t = type(m)
    return t.__name__ in names and (t.__module__.startswith("transformers.models.")
                                    or t.__module__ == "llmcompressor_b200.moe")


@contextlib.contextmanager
def fused_layer_ops(*layers: torch.nn.Module, enabled: bool = True):
    """Run the given decoder layers with the fused elementwise forwards for
    the duration of the block (no-op when ``enabled`` is false)."""
    if not enabled:
        yield
        return
    _lib.lib()  # the kernels are the product path: fail loudly without them
    installed: list[torch.nn.Module] = []
    patched: list[tuple[types.ModuleType, object]] = []
    try:
        for layer in layers:
            for m in layer.modules():
                if "forward" in m.__dict__:
                    continue
                if _module_classes(m, RMSNORM_CLASSES) and hasattr(m, "variance_epsilon"):
                    m.forward = types.MethodType(_norm_forward, m)
                elif _module_classes(m, MLP_CLASSES) and _silu(getattr(m, "act_fn", None)):
                    m.forward = types.MethodType(_mlp_forward, m)
                elif _module_classes(m, LAYER_CLASSES):
                    m.forward = types.MethodType(_layer_forward, m)
                else:
                    continue
                installed.append(m)
                attn = getattr(m, "self_attn", None)
                if attn is not None:
                    mod = sys.modules.get(type(attn).__module__)
                    orig = getattr(mod, "apply_rotary_pos_emb", None)
                    if orig is not None and not hasattr(orig, "llmc_fused_from"):
                        patched.append((mod, orig))
                        mod.apply_rotary_pos_emb = _make_rotary(orig)
        yield
    finally:
        for m in installed:
            m.__dict__.pop("forward", None)
        for mod, orig in patched:
            mod.apply_rotary_pos_emb = orig
