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
so checkpoints and ignore patterns carry over.  The combine differs in form,
not in result: in all-expert mode (the whole oneshot, calibration and
propagation passes, as in the reference) each expert's output over all
tokens is weighted by its dense routing column (zero for tokens not routed
to it) and added in expert order, which adds the same bf16 products in the
same order as the reference's gather / ``index_add_`` without a host sync per
expert; outside that mode each expert runs on its routed tokens only,
grouped with one host sync per call.
"""
from __future__ import annotations

import contextlib

import torch

__all__ = ["ExpertMLP", "LinearExperts", "linearize_experts", "calibrate_all_experts", "all_experts_enabled"]

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


class LinearExperts(torch.nn.ModuleList):
    """Per-expert Linear modules in place of a fused experts module; same
    call signature ``(hidden_states, top_k_index, top_k_weights)``."""

    def __init__(self, num_experts: int, hidden: int, inter: int, act_fn, dtype, device=None):
        super().__init__([ExpertMLP(hidden, inter, act_fn, dtype, device) for _ in range(num_experts)])
        self.num_experts = num_experts

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

    def forward(self, hidden_states, top_k_index, top_k_weights):
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
