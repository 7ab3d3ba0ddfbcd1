"""``oneshot`` GPTQ W4A16 end to end on the 2-layer Llama (config C1) against
the reference's own ``oneshot`` run (``tests/golden/oneshot_c1.npz``, made on
CPU by ``tests/golden/make_golden.py oneshot_c1`` from the same seeded model
and tokens).

What can be held equal, and the bars:

* Layer 0's q/k/v read RMSNorm(embedding) -- the same values on both sides up
  to the norm's float32 rounding -- so their GPTQ codes must be >= 99%
  identical.
* Every other module's inputs come from decoder forward passes, which no GPU
  reproduces bit for bit from a CPU run (the reference agrees with itself on
  only 84-96% of the downstream codes when just its attention kernel changes
  from sdpa to eager).  For those the bar is the quantization quality on the
  same inputs: per module, ||(W - Q) X||^2 / ||W X||^2 over this run's
  calibration inputs X must be within 1% of the same ratio for the
  reference's Q (measured: the reference's own sdpa and eager runs differ by
  at most 0.6% here, 3.7% on one module whose error is 10x smaller than the
  rest).  GPTQ rows are independent given X, so the fixture's first 128 rows
  of every module are a fair sample.
"""
import numpy as np
import pytest
import torch

from golden_io import load
from llmcompressor_b200 import oneshot as O
from llmcompressor_b200 import synthetic

pytestmark = pytest.mark.gpu


def unpack_int4(packed: np.ndarray, cols: int) -> np.ndarray:
    """compressed-tensors pack_to_int32 inverse: 8 codes per int32, code j at bits 4j, offset +8."""
    p = packed.astype(np.int64) & 0xFFFFFFFF
    codes = np.stack([(p >> (4 * j)) & 0xF for j in range(8)], axis=-1).reshape(p.shape[0], -1)[:, :cols]
    return codes.astype(np.int32) - 8


def bf16_of(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


@pytest.fixture(scope="module")
def c1_run():
    ref = load("oneshot_c1")
    rows = int(ref["rows"])
    model = synthetic.random_llama("c1").cuda()
    ids = synthetic.calibration_tokens("c1")
    w0 = {n: m.weight.detach()[:rows].clone() for n, m in model.named_modules()
          if isinstance(m, torch.nn.Linear) and n != "lm_head"}
    grams, calls = {}, {}

    def hook(name):
        def f(mod, args, out):
            if calls.get(name, 0) == 0:  # the calibration pass (the propagation pass follows the solve)
                x = args[0].reshape(-1, args[0].shape[-1]).double()
                grams[name] = x.T @ x
            calls[name] = calls.get(name, 0) + 1
        return f

    hs = [m.register_forward_hook(hook(n)) for n, m in model.named_modules() if n in w0]
    data = [{"input_ids": ids[i:i + 1], "attention_mask": torch.ones_like(ids[i:i + 1])} for i in range(len(ids))]
    O.oneshot(model, data, recipe=O.GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head"],
                                                  actorder=None, block_size=128, dampening_frac=0.01),
              num_calibration_samples=len(ids))
    for h in hs:
        h.remove()
    torch.cuda.synchronize()
    return model, ref, rows, w0, grams, ids


def test_c1_modules_and_stats(c1_run):
    model, ref, rows, w0, grams, ids = c1_run
    names = [str(n) for n in ref["modules"]]
    ours = sorted(n for n, m in model.named_modules() if hasattr(m, "weight_scale"))
    assert ours == sorted(names)
    stats = O.LAST_STATS
    assert stats.samples == 32 and stats.tokens == 32 * 512
    assert all(np.isfinite(v) and v > 0 for v in stats.losses.values())
    for n in names:
        m = model.get_submodule(n)
        assert m.weight_scale.dtype == torch.bfloat16 and m.weight_scale.shape == (m.weight.shape[0],
                                                                                    m.weight.shape[1] // 128)


def test_c1_layer0_qkv_codes_match_reference(c1_run):
    model, ref, rows, w0, grams, ids = c1_run
    for n in ("model.layers.0.self_attn.q_proj", "model.layers.0.self_attn.k_proj",
              "model.layers.0.self_attn.v_proj"):
        m = model.get_submodule(n)
        cols = m.weight.shape[1]
        theirs = unpack_int4(ref[f"{n}.weight_packed"], cols)
        s = m.weight_scale.detach()[:rows].float().repeat_interleave(128, dim=1)
        mine = torch.round(m.weight.detach()[:rows].float() / s).clamp(-8, 7).cpu().numpy().astype(np.int32)
        agree = float(np.mean(mine == theirs))
        assert agree >= 0.99, (n, agree)
        sc_ref = bf16_of(ref[f"{n}.weight_scale"]).float()
        assert torch.equal(m.weight_scale.detach()[:rows].float().cpu(), sc_ref), n  # scales: the unmodified weight's


def test_c1_output_error_within_1pct_of_reference(c1_run):
    model, ref, rows, w0, grams, ids = c1_run
    for n in [str(x) for x in ref["modules"]]:
        m = model.get_submodule(n)
        cols = m.weight.shape[1]
        codes = torch.from_numpy(unpack_int4(ref[f"{n}.weight_packed"], cols)).float()
        scale = bf16_of(ref[f"{n}.weight_scale"]).float().repeat_interleave(128, dim=1)
        q_ref = (codes * scale).to(torch.bfloat16).cuda().double()
        W = w0[n].double()
        H = grams[n]
        q_our = m.weight.detach()[:rows].double()

        def err(Q):
            D = W - Q
            return float(torch.einsum("ij,jk,ik->", D, H, D) / torch.einsum("ij,jk,ik->", W, H, W))

        e_our, e_ref = err(q_our), err(q_ref)
        assert e_our <= 1.01 * e_ref, (n, e_our, e_ref)
        assert e_our >= 0.90 * e_ref, (n, e_our, e_ref)  # not a different algorithm


def test_c1_final_hidden_state_error_matches_reference(c1_run):
    model, ref, rows, w0, grams, ids = c1_run
    fp = synthetic.random_llama("c1").cuda()
    with torch.no_grad():
        hq = model.model(ids[:4].cuda()).last_hidden_state.float()
        hf = fp.model(ids[:4].cuda()).last_hidden_state.float()
    rel = (torch.linalg.norm((hq - hf).reshape(4, -1), dim=1) / torch.linalg.norm(hf.reshape(4, -1), dim=1)).cpu()
    theirs = torch.from_numpy(ref["hidden_rel_err"])
    assert torch.all((rel - theirs).abs() <= 0.05 * theirs), (rel, theirs)
