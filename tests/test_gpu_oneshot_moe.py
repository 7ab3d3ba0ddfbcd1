"""``oneshot`` GPTQ W4A16 with all-expert calibration on a 2-layer Qwen3-MoE at
reduced width (``synthetic`` "c3tiny": 8 experts top-2) against the
reference's own oneshot run (``tests/golden/oneshot_c3tiny.npz``, made on CPU
by ``tests/golden/make_golden.py oneshot_c3tiny``).

Every expert's gate/up projection reads the same tokens (one shared Hessian
for all of them) and every expert's down projection its own; the bars are
those of the dense C1 test: layer 0's q/k/v codes >= 99% identical (same
inputs up to RMSNorm rounding), and per module ||(W - Q) X||^2 / ||W X||^2
over this run's calibration inputs within 1% of the reference's Q on the
same X, plus the final hidden-state error within 5% of the reference's.

The run above hooks every Linear (to record the calibration inputs), which
keeps the experts on the per-expert form.  A second run with no hooks on the
expert modules takes the stacked all-expert form (three GEMMs for all
experts, down Hessians from one grouped launch): the same bars, with that
run's own calibration inputs as X."""
import numpy as np
import pytest
import torch

from golden_io import load
from llmcompressor_b200 import moe
from llmcompressor_b200 import oneshot as O
from llmcompressor_b200 import synthetic
from test_gpu_oneshot import bf16_of, unpack_int4

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c3_run():
    ref = load("oneshot_c3tiny")
    model = synthetic.random_qwen3_moe("c3tiny")
    assert moe.linearize_experts(model) == 2
    model = model.cuda()
    ids = synthetic.calibration_tokens("c3tiny")
    w0 = {n: m.weight.detach().clone() for n, m in model.named_modules()
          if isinstance(m, torch.nn.Linear) and n != "lm_head"}
    grams, calls = {}, {}

    def hook(name):
        def f(mod, args, out):
            if calls.get(name, 0) == 0:  # the calibration pass
                x = args[0].reshape(-1, args[0].shape[-1]).double()
                grams[name] = x.T @ x
            calls[name] = calls.get(name, 0) + 1
        return f

    hs = [m.register_forward_hook(hook(n)) for n, m in model.named_modules() if n in w0]
    O.oneshot(model, ids, recipe=O.GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head", "re:.*mlp.gate$"],
                                                 actorder=None), num_calibration_samples=len(ids))
    for h in hs:
        h.remove()
    torch.cuda.synchronize()
    return model, ref, w0, grams, ids


def test_c3tiny_modules(c3_run):
    model, ref, w0, grams, ids = c3_run
    names = sorted(str(n) for n in ref["modules"])
    ours = sorted(n for n, m in model.named_modules() if hasattr(m, "weight_scale"))
    assert ours == names
    assert len([n for n in ours if ".experts." in n]) == 2 * 8 * 3
    stats = O.LAST_STATS
    assert all(np.isfinite(v) and v > 0 for v in stats.losses.values())


def test_c3tiny_layer0_attention_codes(c3_run):
    model, ref, w0, grams, ids = c3_run
    for n in ("model.layers.0.self_attn.q_proj", "model.layers.0.self_attn.k_proj",
              "model.layers.0.self_attn.v_proj"):
        m = model.get_submodule(n)
        theirs = unpack_int4(ref[f"{n}.weight_packed"], m.weight.shape[1])
        s = m.weight_scale.detach().float().repeat_interleave(128, dim=1)
        mine = torch.round(m.weight.detach().float() / s).clamp(-8, 7).cpu().numpy().astype(np.int32)
        assert float(np.mean(mine == theirs)) >= 0.99, n


def test_c3tiny_output_error_within_1pct_of_reference(c3_run):
    model, ref, w0, grams, ids = c3_run
    for n in [str(x) for x in ref["modules"]]:
        m = model.get_submodule(n)
        codes = torch.from_numpy(unpack_int4(ref[f"{n}.weight_packed"], m.weight.shape[1])).float()
        scale = bf16_of(ref[f"{n}.weight_scale"]).float().repeat_interleave(128, dim=1)
        q_ref = (codes * scale).to(torch.bfloat16).cuda().double()
        W, H, q_our = w0[n].double(), grams[n], m.weight.detach().double()

        def err(Q):
            D = W - Q
            return float(torch.einsum("ij,jk,ik->", D, H, D) / torch.einsum("ij,jk,ik->", W, H, W))

        e_our, e_ref = err(q_our), err(q_ref)
        assert e_our <= 1.01 * e_ref, (n, e_our, e_ref)
        assert e_our >= 0.90 * e_ref, (n, e_our, e_ref)


def test_c3tiny_final_hidden_state_error(c3_run):
    model, ref, w0, grams, ids = c3_run
    fp = synthetic.random_qwen3_moe("c3tiny").cuda()
    with torch.no_grad():
        hq = model.model(ids[:4].cuda()).last_hidden_state.float()
        hf = fp.model(ids[:4].cuda()).last_hidden_state.float()
    rel = (torch.linalg.norm((hq - hf).reshape(4, -1), dim=1) / torch.linalg.norm(hf.reshape(4, -1), dim=1)).cpu()
    theirs = torch.from_numpy(ref["hidden_rel_err"])
    assert torch.all((rel - theirs).abs() <= 0.05 * theirs), (rel, theirs)


@pytest.fixture(scope="module")
def c3_stacked():
    """The stacked run, recording its own calibration inputs: hooks on the
    attention projections, and on each experts module's input (a hook on
    the experts module itself keeps the stacked form); the down inputs are
    recomputed from that input and the unquantized expert weights."""
    model = synthetic.random_qwen3_moe("c3tiny")
    moe.linearize_experts(model)
    model = model.cuda()
    ids = synthetic.calibration_tokens("c3tiny")
    w0 = {n: m.weight.detach().clone() for n, m in model.named_modules()
          if isinstance(m, torch.nn.Linear) and n != "lm_head"}
    grams, seen = {}, set()

    def lin_hook(name):
        def f(mod, args, out):
            if name not in seen:
                seen.add(name)
                x = args[0].reshape(-1, args[0].shape[-1]).double()
                grams[name] = x.T @ x
        return f

    def experts_hook(name, le):
        def f(mod, args):
            if name in seen:
                return
            seen.add(name)
            x = args[0].reshape(-1, args[0].shape[-1])
            xd = x.double()
            for e in range(le.num_experts):
                p = f"{name}.{e}"
                grams[f"{p}.gate_proj"] = grams[f"{p}.up_proj"] = xd.T @ xd
                g = x.float() @ w0[f"{p}.gate_proj"].float().T
                u = x.float() @ w0[f"{p}.up_proj"].float().T
                a = (torch.nn.functional.silu(g) * u).double()
                grams[f"{p}.down_proj"] = a.T @ a
        return f

    hs = []
    for n, m in model.named_modules():
        if isinstance(m, moe.LinearExperts):
            hs.append(m.register_forward_pre_hook(experts_hook(n, m)))
        elif n in w0 and ".experts." not in n:
            hs.append(m.register_forward_hook(lin_hook(n)))
    before = moe.STACKED_CALLS
    O.oneshot(model, ids, recipe=O.GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head", "re:.*mlp.gate$"],
                                                 actorder=None), num_calibration_samples=len(ids))
    for h in hs:
        h.remove()
    torch.cuda.synchronize()
    return model, moe.STACKED_CALLS - before, w0, grams


def test_c3tiny_stacked_output_error_within_1pct_of_reference(c3_run, c3_stacked):
    ref = c3_run[1]
    model, calls, w0, grams = c3_stacked
    assert calls > 0  # the stacked form ran
    for n in [str(x) for x in ref["modules"]]:
        m = model.get_submodule(n)
        codes = torch.from_numpy(unpack_int4(ref[f"{n}.weight_packed"], m.weight.shape[1])).float()
        scale = bf16_of(ref[f"{n}.weight_scale"]).float().repeat_interleave(128, dim=1)
        q_ref = (codes * scale).to(torch.bfloat16).cuda().double()
        W, H, q_our = w0[n].double(), grams[n], m.weight.detach().double()

        def err(Q):
            D = W - Q
            return float(torch.einsum("ij,jk,ik->", D, H, D) / torch.einsum("ij,jk,ik->", W, H, W))

        e_our, e_ref = err(q_our), err(q_ref)
        assert e_our <= 1.01 * e_ref, (n, e_our, e_ref)
        assert e_our >= 0.90 * e_ref, (n, e_our, e_ref)


def test_c3tiny_stacked_final_hidden_state_error(c3_run, c3_stacked):
    _, ref, _, _, ids = c3_run
    model = c3_stacked[0]
    fp = synthetic.random_qwen3_moe("c3tiny").cuda()
    with torch.no_grad():
        hq = model.model(ids[:4].cuda()).last_hidden_state.float()
        hf = fp.model(ids[:4].cuda()).last_hidden_state.float()
    rel = (torch.linalg.norm((hq - hf).reshape(4, -1), dim=1) / torch.linalg.norm(hf.reshape(4, -1), dim=1)).cpu()
    theirs = torch.from_numpy(ref["hidden_rel_err"])
    assert torch.all((rel - theirs).abs() <= 0.05 * theirs), (rel, theirs)


def test_stacked_forward_matches_per_expert():
    """The stacked all-expert forward against the per-expert one on the
    same inputs: within bf16 rounding of the per-expert sum."""
    model = synthetic.random_qwen3_moe("c3tiny")
    moe.linearize_experts(model)
    model = model.cuda()
    le = model.model.layers[0].mlp.experts
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(3000, 256, device="cuda", generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(8, device="cuda", generator=g)[:2] for _ in range(3000)])
    w = torch.softmax(torch.randn(3000, 2, device="cuda", generator=g), dim=-1)
    with torch.no_grad(), moe.calibrate_all_experts(True):
        assert le.stacked_ready()
        ours = le(x, idx, w)
        le.stacked = False
        theirs = le(x, idx, w)
        le.stacked = True
    rel = float(torch.linalg.norm(ours.float() - theirs.float()) / torch.linalg.norm(theirs.float()))
    assert rel < 5e-3, rel


def test_routed_stacked_forward_matches_per_expert():
    """The routed forward as grouped GEMMs over the experts' row segments
    (the same products as one GEMM per expert) with the weighted outputs
    added per token in increasing expert order, bf16 rounding per add (the
    per-expert ``index_add_``): bit-identical to the per-expert routed loop."""
    model = synthetic.random_qwen3_moe("c3tiny")
    moe.linearize_experts(model)
    model = model.cuda()
    le = model.model.layers[1].mlp.experts
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(2500, 256, device="cuda", generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(8, device="cuda", generator=g)[:2] for _ in range(2500)])
    w = torch.softmax(torch.randn(2500, 2, device="cuda", generator=g), dim=-1)
    before = moe.STACKED_CALLS
    with torch.no_grad():
        ours = le(x, idx, w)
        assert moe.STACKED_CALLS == before + 1
        le.stacked = False
        theirs = le(x, idx, w)
        le.stacked = True
    assert torch.equal(ours, theirs)
