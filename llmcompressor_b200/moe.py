"""Mixture-of-experts layers for GPTQ calibration.

The reference calibrates MoE models with every expert seeing every token
(``moe_calibrate_all_experts=True``, S/entrypoints/oneshot.py:236-256): fused
expert weights (3-D ``gate_up_proj`` (E, 2I, H) and ``down_proj`` (E, H, I))
are first split into per-expert Linear modules (``linearize_moe``,
S/modeling/moe/linearize.py:96-137, ``LinearExperts2D``,
S/modeling/moe/linear_experts.py), whose forward runs each expert on all
tokens and keeps the routed tokens' outputs (:244-277).  Every expert's
gate/up projection then reads the same input (one Hessian serves all of
them) and every expert's down projection its own.

``linearize_experts`` does the split here; the module names
(``experts.{e}.gate_proj`` / ``up_proj`` / ``down_proj``) are the reference's,
so checkpoints and ignore patterns carry over.

All-expert mode (the whole oneshot, calibration and propagation passes, as
in the reference) has two forms:

* per expert (``stacked=False``, or experts the stacked form does not take):
  each expert's output over all tokens is weighted by its dense routing
  column (zero for tokens not routed to it) and added in expert order -- the
  same bf16 products added in the same order as the reference's gather /
  ``index_add_``, bit for bit, without a host sync per expert;
* stacked (the default for bf16 SiLU experts on the GPU): the experts'
  gate, up and down weights are concatenated once per pass, so the layer
  runs three GEMMs for all experts instead of three per expert: gate and up
  as (tokens, E*I) products, SiLU * up and the routing weight in one kernel
  (``llmc_silu_mul_scaled_bf16``), and the down projection with the
  weighted combine folded into one GEMM over K = E*I (float32 accumulation
  across experts instead of bf16 adds per expert: the same sum, rounded
  once).  A calibration sink (``calib_sink``, set by the GPTQ calibration)
  receives the shared gate/up input and the concatenated down inputs, whose
  per-expert Hessians one grouped launch accumulates.

Outside all-expert mode each expert runs on its routed tokens only, grouped
with one host sync per call.
"""
from __future__ import annotations

import contextlib

import torch
import torch.nn.functional as F

__all__ = ["ExpertMLP", "LinearExperts", "linearize_experts", "calibrate_all_experts", "all_experts_enabled",
           "release_stacked"]

_ALL_EXPERTS = False


@contextlib.contextmanager
def calibrate_all_experts(enabled: bool = True):
    """Within the context every ``LinearExperts`` runs all experts on all
    tokens (the reference's ``moe_calibration_context``)."""
    global _ALL_EXPERTS
    prev, _ALL_EXPERTS = _ALL_EXPERTS, enabled
    try:
        yield
    finally:
        _ALL_EXPERTS = prev


def all_experts_enabled() -> bool:
    return _ALL_EXPERTS


class ExpertMLP(torch.nn.Module):
    """One expert: down(act(gate(x)) * up(x))."""

    def __init__(self, hidden: int, inter: int, act_fn, dtype, device=None):
        super().__init__()
        kw = dict(bias=False, dtype=dtype, device=device)
        self.gate_proj = torch.nn.Linear(hidden, inter, **kw)
        self.up_proj = torch.nn.Linear(hidden, inter, **kw)
        self.down_proj = torch.nn.Linear(inter, hidden, **kw)
        self.act_fn = act_fn

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))


# the stacked weights of one experts module at a time: (owner id, key, (Wg, Wu, Wd))
_STACK: dict = {}
STACKED_CALLS = 0  # forwards that took the stacked all-expert form (tests read it)


def release_stacked() -> None:
    """Drop the cached stacked expert weights (the pipeline calls it when a
    layer is done)."""
    _STACK.clear()


def _hooked(m: torch.nn.Module) -> bool:
    return bool(m._forward_hooks or m._forward_pre_hooks)


class LinearExperts(torch.nn.ModuleList):
    """Per-expert Linear modules in place of a fused experts module; same
    call signature ``(hidden_states, top_k_index, top_k_weights)``."""

    def __init__(self, num_experts: int, hidden: int, inter: int, act_fn, dtype, device=None):
        super().__init__([ExpertMLP(hidden, inter, act_fn, dtype, device) for _ in range(num_experts)])
        self.num_experts = num_experts
        self.stacked = True
        # calibration: sink(module, x, act) receives the input shared by every
        # expert's gate/up and the experts' concatenated down inputs (tokens,
        # E * I); it may raise to end the pass there
        self.calib_sink = None

    def stacked_ready(self) -> bool:
        """Whether the stacked all-expert form takes these experts: bf16
        weights on the GPU, no biases, SiLU, sizes multiples of 8, and no
        hooks on the expert modules (the stacked form does not call them)."""
        from .layer_forward import _silu

        if not self.stacked or self.num_experts == 0:
            return False
        e0 = self[0]
        if not _silu(e0.act_fn):
            return False
        inter, hidden = e0.gate_proj.out_features, e0.gate_proj.in_features
        if inter % 8 or hidden % 8:
            return False
        for ex in self:
            for lin in (ex.gate_proj, ex.up_proj, ex.down_proj):
                w = lin.weight
                if lin.bias is not None or w.dtype != torch.bfloat16 or not w.is_cuda or _hooked(lin):
                    return False
            if _hooked(ex):
                return False
        return True

    def _stacked_weights(self, form: str = "all"):
        """Concatenated expert weights: gate and up as (E*I, hidden); down as
        (hidden, E*I) for the all-expert form (``form="all"``) or (E, hidden,
        I) for the routed one.  Cached for one experts module at a time and
        rebuilt when any expert weight changed."""
        ws = [(ex.gate_proj.weight, ex.up_proj.weight, ex.down_proj.weight) for ex in self]
        key = tuple((w.data_ptr(), w._version) for t in ws for w in t)
        if _STACK.get("owner") != id(self) or _STACK.get("key") != key:
            _STACK.clear()  # one module's copies at a time
            _STACK.update(owner=id(self), key=key, gate=torch.cat([t[0] for t in ws], 0),
                          up=torch.cat([t[1] for t in ws], 0))
        if form not in _STACK:
            _STACK[form] = (torch.cat([t[2] for t in ws], 1) if form == "all"
                            else torch.stack([t[2] for t in ws], 0))
        return _STACK["gate"], _STACK["up"], _STACK[form]

    def _forward_stacked(self, x, top_k_index, top_k_weights):
        from . import layer_forward as LF

        global STACKED_CALLS
        STACKED_CALLS += 1
        if not (x.dim() == 2 and x.is_contiguous() and x.dtype == torch.bfloat16 and x.data_ptr() % 16 == 0):
            raise ValueError("stacked experts take contiguous bf16 (tokens, hidden) inputs")
        inter = self[0].gate_proj.out_features
        Wg, Wu, Wd = self._stacked_weights("all")
        g = F.linear(x, Wg)
        u = F.linear(x, Wu)
        dense = torch.zeros(x.shape[0], self.num_experts, dtype=torch.float32, device=x.device)
        dense.scatter_(1, top_k_index, top_k_weights.to(torch.float32))
        sink = self.calib_sink
        if sink is not None:
            act, _ = LF.silu_mul_scaled(g, u, inter, None, act=True, scaled=False)
            del g, u
            sink(self, x, act)  # may end the pass here
            scaled = LF.scale_groups(act, inter, dense)
            del act
        else:
            _, scaled = LF.silu_mul_scaled(g, u, inter, dense, act=False, scaled=True)
            del g, u
        return F.linear(scaled, Wd)

    @classmethod
    @torch.no_grad()
    def from_fused(cls, experts: torch.nn.Module) -> "LinearExperts":
        gu, dn = experts.gate_up_proj, experts.down_proj
        E, two_i, H = gu.shape
        inter = two_i // 2
        self = cls(E, H, inter, experts.act_fn, gu.dtype, device="meta")
        for e, ex in enumerate(self):
            ex.gate_proj.weight = torch.nn.Parameter(gu[e, :inter].contiguous(), requires_grad=False)
            ex.up_proj.weight = torch.nn.Parameter(gu[e, inter:].contiguous(), requires_grad=False)
            ex.down_proj.weight = torch.nn.Parameter(dn[e].contiguous(), requires_grad=False)
        return self

    def _forward_routed_stacked(self, x, top_k_index, top_k_weights):
        """Routed tokens only, without a host sync: the (token, expert) pairs
        sorted by expert, gate / up / down as grouped GEMMs over the experts'
        row segments (``torch._grouped_mm``; per segment the same products as
        one GEMM per expert), SiLU * up in one kernel, and the weighted
        outputs added per token in increasing expert order with a bf16
        rounding per add (``llmc_moe_combine_bf16``) -- the reference's
        per-expert ``index_add_``."""
        from . import layer_forward as LF

        global STACKED_CALLS
        STACKED_CALLS += 1
        if not (x.dim() == 2 and x.dtype == torch.bfloat16):
            raise ValueError("stacked experts take bf16 (tokens, hidden) inputs")
        E = self.num_experts
        inter = self[0].gate_proj.out_features
        T, K = top_k_index.shape
        hidden = x.shape[1]
        Wg, Wu, Wd3 = self._stacked_weights("routed")
        idx, kperm = torch.sort(top_k_index, dim=1)  # each token's experts in increasing order
        w = torch.gather(top_k_weights, 1, kperm)
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)  # pairs grouped by expert
        offs = torch.cumsum(torch.bincount(flat, minlength=E), 0).to(torch.int32)
        xs = x[torch.div(order, K, rounding_mode="floor")]
        g = torch._grouped_mm(xs, Wg.view(E, inter, hidden).transpose(1, 2), offs=offs)
        u = torch._grouped_mm(xs, Wu.view(E, inter, hidden).transpose(1, 2), offs=offs)
        del xs
        act = LF.silu_mul(g, u)
        del g, u
        y = torch._grouped_mm(act, Wd3.transpose(1, 2), offs=offs)  # (T*K, hidden), expert-sorted rows
        pos = torch.empty_like(order)
        pos[order] = torch.arange(order.numel(), device=x.device)
        return LF.moe_combine(y, pos.view(T, K), w)

    def forward(self, hidden_states, top_k_index, top_k_weights):
        if _ALL_EXPERTS and (self.calib_sink is not None or self.stacked_ready()):
            return self._forward_stacked(hidden_states, top_k_index, top_k_weights)
        if not _ALL_EXPERTS and self.stacked_ready():
            return self._forward_routed_stacked(hidden_states, top_k_index, top_k_weights)
        final = torch.zeros_like(hidden_states)
        if _ALL_EXPERTS:
            # dense routing weights (T, E), zero where a token is not routed
            dense = torch.zeros(hidden_states.shape[0], self.num_experts, dtype=top_k_weights.dtype,
                                device=hidden_states.device)
            dense.scatter_(1, top_k_index, top_k_weights)
            for e, expert in enumerate(self):
                out = expert(hidden_states)
                final += (out * dense[:, e:e + 1]).to(final.dtype)
            return final
        # routed tokens only: group them by expert with one host sync
        T, K = top_k_index.shape
        flat = top_k_index.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=self.num_experts).tolist()
        tok = (order // K)
        pos = order % K
        start = 0
        for e, expert in enumerate(self):
            c = counts[e]
            if c == 0:
                continue
            ti, pi = tok[start:start + c], pos[start:start + c]
            start += c
            out = expert(hidden_states[ti]) * top_k_weights[ti, pi, None]
            final.index_add_(0, ti, out.to(final.dtype))
        return final


def _is_fused_experts(mod: torch.nn.Module) -> bool:
    gu = getattr(mod, "gate_up_proj", None)
    dn = getattr(mod, "down_proj", None)
    return (isinstance(gu, torch.nn.Parameter) and isinstance(dn, torch.nn.Parameter) and gu.ndim == 3
            and dn.ndim == 3 and hasattr(mod, "act_fn"))


def linearize_experts(model: torch.nn.Module) -> int:
    """Replace every fused experts module of ``model`` (``linearize_moe``);
    returns how many were replaced."""
    targets = [(n, m) for n, m in model.named_modules() if _is_fused_experts(m)]
    for name, mod in targets:
        model.set_submodule(name, LinearExperts.from_fused(mod))
    return len(targets)
