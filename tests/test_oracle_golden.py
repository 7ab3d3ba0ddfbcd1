"""Pin the CPU oracle to the reference: every oracle function against the
golden fixtures made by running the reference itself (tests/golden/make_golden.py),
plus the reference's own known-answer tests.  CPU only."""
import numpy as np
import pytest

from oracle import casts, gptq, numerics, observers
from oracle.observers import QArgs
from golden_io import bf16, load

OBS_CASES = {
    "int4_sym_group128": QArgs(4, "int", True, "group", 128),
    "int4_asym_group128": QArgs(4, "int", False, "group", 128),
    "int8_sym_channel": QArgs(8, "int", True, "channel", None),
    "int4_sym_tensor": QArgs(4, "int", True, "tensor", None),
    "fp8_block_128": QArgs(8, "float", True, "block", None, (128, 128), zp_dtype="fp8"),
    "int8_asym_channel": QArgs(8, "int", False, "channel", None),
}


@pytest.mark.parametrize("case", sorted(OBS_CASES))
def test_observer_qparams_bit_exact(case):
    g = load(f"observer_{case}")
    args = OBS_CASES[case]
    w = bf16(g["weight"])
    mn, mx = observers.minmax(w, args)
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(mn), g["min_vals"].reshape(mn.shape))
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(mx), g["max_vals"].reshape(mx.shape))
    scale, zp = observers.calculate_qparams(mn, mx, args)
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(scale), g["scale"].reshape(scale.shape))
    if args.zp_dtype == "int8":
        np.testing.assert_array_equal(zp, g["zero_point"].reshape(zp.shape))


@pytest.mark.parametrize("scheme", ["W4A16", "W4A16_ASYM", "W8A16", "FP8_DYNAMIC", "FP8", "FP8_BLOCK", "MXFP4A16", "NVFP4A16"])
def test_modelfree_bit_exact(scheme):
    g = load(f"modelfree_{scheme}")
    w = bf16(g["weight"])
    out = casts.modelfree_tensor(w, scheme)
    for k, v in out.items():
        ref = g["out_" + k]
        if k == "weight_scale" and v.dtype == np.float32:
            v = numerics.f32_to_bf16_bits(v)
        np.testing.assert_array_equal(np.asarray(v).reshape(ref.shape), ref, err_msg=f"{scheme}:{k}")
    assert set("out_" + k for k in out) <= set(g)


def test_nvfp4_fused_global_scale_bit_exact():
    g = load("modelfree_NVFP4A16_fused_qkv")
    names = ("q_proj", "k_proj", "v_proj")
    ws = [bf16(g[f"{n}_weight"]) for n in names]
    gs = casts.nvfp4_global_scale(ws)
    for n, w in zip(names, ws):
        out = casts.modelfree_tensor(w, "NVFP4A16", global_scale=gs)
        for k, v in out.items():
            np.testing.assert_array_equal(np.asarray(v).reshape(g[f"{n}_out_{k}"].shape), g[f"{n}_out_{k}"], err_msg=f"{n}:{k}")


def test_hessian_matches_reference():
    g = load("hessian")
    d = g["H"].shape[0]
    H = np.zeros((d, d), np.float32)
    n = 0
    for i in range(3):
        H, n = gptq.accumulate_hessian(bf16(g[f"x{i}"]), H, n)
    assert n == float(g["num_samples"])
    rel = np.linalg.norm(H - g["H"]) / np.linalg.norm(g["H"])
    assert rel <= 1e-5, rel


# case -> (args, actorder); block size from the fixture
GPTQ_CASES = {
    "int4_group128": (QArgs(4, "int", True, "group", 128), None),
    "int4_channel_dead": (QArgs(4, "int", True, "channel", None), None),
    "int8_group64_asym": (QArgs(8, "int", False, "group", 64), None),
    "int4_group128_actweight": (QArgs(4, "int", True, "group", 128), "weight"),
    "int4_group32_actgroup": (QArgs(4, "int", True, "group", 32), "group"),
    "int4_channel_actstatic": (QArgs(4, "int", True, "channel", None), "static"),
    "int8_block32x64_bs64": (QArgs(8, "int", True, "block", None, (32, 64)), None),
    "int8_block48x96_actweight": (QArgs(8, "int", True, "block", None, (48, 96)), "weight"),
    "fp8_channel": (QArgs(8, "float", True, "channel", None, zp_dtype="fp8"), None),
    "nvfp4_actweight": (QArgs(4, "float", True, "tensor_group", 16, scale_dtype="fp8", zp_dtype="fp8"), "weight"),
    "mxfp4": (QArgs(4, "float", True, "group", 32, scale_dtype="uint8", zp_dtype="uint8"), None),
}


@pytest.mark.parametrize("case", sorted(GPTQ_CASES))
def test_gptq_oracle_matches_reference(case):
    g = load(f"gptq_{case}")
    args, order = GPTQ_CASES[case]
    w = bf16(g["weight"])
    bs = int(g["blocksize"]) if "blocksize" in g else 128
    res = gptq.quantize_weight(w, g["hessian"], args, blocksize=bs, actorder=order)
    loss, wq, scale, zp, ok = res[:5]
    extra = res[5] if len(res) > 5 else {}
    assert ok
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(scale), g["out_scale"].reshape(scale.shape))
    g_idx = extra.get("g_idx")
    if "out_g_idx" in g:
        np.testing.assert_array_equal(g_idx, g["out_g_idx"])
    gs = extra.get("global_scale")
    if "out_global_scale" in g:
        np.testing.assert_array_equal(numerics.f32_to_bf16_bits(np.float32(gs)).reshape(-1), g["out_global_scale"].reshape(-1))
    ref_wq = bf16(g["out_weight"])
    codes = gptq.codes_from_weight(wq, scale, zp, args, g_idx, gs)
    ref_codes = gptq.codes_from_weight(ref_wq, scale, zp, args, g_idx, gs)
    agree = float(np.mean(codes == ref_codes))
    assert agree >= 0.99, agree
    assert abs(loss - float(g["loss"])) <= 0.01 * abs(float(g["loss"]))
    x = bf16(g["x"])
    e_ref = gptq.layer_output_error(w, ref_wq, x)
    e_new = gptq.layer_output_error(w, wq, x)
    assert abs(e_new - e_ref) <= 0.01 * e_ref, (e_new, e_ref)


# --- known-answer tests of the reference's own suite -------------------------
# T/llmcompressor/modifiers/calibration/test_lifecycle.py:16-121: weight = arange(24) as 4x6 bf16
LIFECYCLE = [
    (QArgs(4, "int", True, "tensor", None), [0.0], [23.0],
     [[0.0, 0.0, 3.0625, 3.0625, 3.0625, 6.125], [6.125, 6.125, 9.1875, 9.1875, 9.1875, 12.25],
      [12.25, 12.25, 15.3125, 15.3125, 15.3125, 18.375], [18.375, 18.375, 21.5, 21.5, 21.5, 21.5]]),
    (QArgs(4, "int", True, "channel", None), [[0], [6], [12], [18]], [[5], [11], [17], [23]],
     [[0.0, 1.3359, 2.0, 2.6719, 4.0, 4.6875], [5.875, 7.3438, 7.3438, 8.8125, 10.25, 10.25],
      [11.3125, 13.625, 13.625, 15.875, 15.875, 15.875], [18.375, 18.375, 21.5, 21.5, 21.5, 21.5]]),
    (QArgs(4, "int", True, "group", 3), [[0, 3], [6, 9], [12, 15], [18, 21]], [[2, 5], [8, 11], [14, 17], [20, 23]],
     [[0.0, 1.0703, 1.875, 2.6719, 4.0, 4.6875], [6.4375, 7.5, 7.5, 8.8125, 10.25, 10.25],
      [11.1875, 13.0625, 13.0625, 15.875, 15.875, 15.875], [18.75, 18.75, 18.75, 21.5, 21.5, 21.5]]),
    (QArgs(4, "float", True, "tensor_group", 3, scale_dtype="fp8", zp_dtype="fp8"),
     [[0, 3], [6, 9], [12, 15], [18, 21]], [[2, 5], [8, 11], [14, 17], [20, 23]],
     [[0.0, 1.0234, 2.0469, 3.2812, 3.2812, 4.9375], [5.4688, 8.1875, 8.1875, 10.6875, 10.6875, 10.6875],
      [9.875, 14.75, 14.75, 16.375, 16.375, 16.375], [19.75, 19.75, 19.75, 23.0, 23.0, 23.0]]),
    (QArgs(4, "int", True, "block", None, (2, 3)), [[0, 3], [12, 15]], [[8, 11], [20, 23]],
     [[0.0, 1.0703, 2.1406, 2.9375, 4.4062, 4.4062], [6.4375, 7.5, 7.5, 8.8125, 10.25, 10.25],
      [10.6875, 13.375, 13.375, 15.3125, 15.3125, 18.375], [18.75, 18.75, 18.75, 21.5, 21.5, 21.5]]),
]


def _fake_quant_weight(w, args):
    """Weight fake-quant of a bf16 weight (forward_quantize on the weight)."""
    mn, mx = observers.minmax(w, args)
    gsc = None
    if args.strategy == "tensor_group":
        gsc = observers.generate_gparam(observers.fused_absmax([(mn, mx)]))
    scale, zp = observers.calculate_qparams(mn, mx, args, global_scale=gsc)
    s = casts.expand_scale(scale, args, w.shape)
    lo, hi = observers.calculate_range(args)
    if args.type == "float":
        eff = (s / np.float32(gsc)).astype(np.float32)
        q = numerics.cast_to_fp4(np.clip((w / eff).astype(np.float32), lo, hi))
        return mn, mx, numerics.rb((q * eff).astype(np.float32))
    q = np.rint(np.clip(numerics.rb(w / s), lo, hi)).astype(np.float32)
    return mn, mx, numerics.rb(q * s)


@pytest.mark.parametrize("idx", range(len(LIFECYCLE)))
def test_reference_lifecycle_known_answers(idx):
    args, exp_min, exp_max, exp_q = LIFECYCLE[idx]
    w = np.arange(24, dtype=np.float32).reshape(4, 6)
    mn, mx, fq = _fake_quant_weight(w, args)
    np.testing.assert_array_equal(mn.reshape(-1), np.asarray(exp_min, np.float32).reshape(-1))
    np.testing.assert_array_equal(mx.reshape(-1), np.asarray(exp_max, np.float32).reshape(-1))
    # the reference compares with torch.allclose (rtol 1e-5, atol 1e-8) against 4-5 digit values
    np.testing.assert_allclose(fq, np.asarray(exp_q, np.float32), rtol=1e-3, atol=1e-3)


def test_reference_min_max_known_answers():
    """T/llmcompressor/observers/test_min_max.py:8-29: int8 on [1,1,1,1,1]."""
    x = np.ones((1, 5), np.float32)
    for sym, exp_s, exp_zp in ((True, 0.0078, 0), (False, 0.0039, -128)):
        args = QArgs(8, "int", sym, "tensor", None)
        mn, mx = observers.minmax(x, args)
        s, zp = observers.calculate_qparams(mn, mx, args, dtype="f32")
        assert round(float(s[0]), 4) == exp_s and int(zp[0]) == exp_zp


def test_fp8_rounding_exhaustive_against_torch():
    """The fp8 restatement against torch's own float -> e4m3fn cast for every bf16 value."""
    import torch

    u = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = bf16(u)
    x = x[np.isfinite(x)]
    x = np.clip(x, -448, 448)
    ours = numerics.fp8_e4m3_bits(numerics.round_fp8_e4m3(x))
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, ref)


def test_bf16_rounding_against_torch():
    import torch

    rng = np.random.default_rng(0)
    x = (rng.standard_normal(200000) * np.exp(rng.uniform(-30, 30, 200000))).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.uint16).numpy()
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(x), ref)


MSE_CASES = {
    "int4_sym_group128": QArgs(4, "int", True, "group", 128),
    "int4_asym_group128": QArgs(4, "int", False, "group", 128),
    "int8_sym_channel": QArgs(8, "int", True, "channel", None),
    "int8_asym_channel": QArgs(8, "int", False, "channel", None),
    "int4_sym_tensor": QArgs(4, "int", True, "tensor", None),
    "fp8_block_128": QArgs(8, "float", True, "block", None, (128, 128), zp_dtype="fp8"),
    "int4_sym_group32": QArgs(4, "int", True, "group", 32),
}


@pytest.mark.parametrize("case", sorted(MSE_CASES))
def test_mse_observer_bit_exact(case):
    """``memoryless_mse`` grid search (S/observers/mse_quant.py) on bf16 weights."""
    g = load(f"mse_{case}")
    args = MSE_CASES[case]
    mn, mx = observers.mse_minmax(bf16(g["weight"]), args)
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(mn), g["min_vals"].reshape(mn.shape))
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(mx), g["max_vals"].reshape(mx.shape))
    scale, zp = observers.calculate_qparams(mn, mx, args)
    np.testing.assert_array_equal(numerics.f32_to_bf16_bits(scale), g["scale"].reshape(scale.shape))


# T/llmcompressor/observers/test_mse.py:9-44: float32 arange(24)/24 as 6x4, 8 bits
MSE_KNOWN = [
    ("tensor", True, 4.8103e-06), ("tensor", False, 1.1258e-06),
    ("channel", True, 2.5675e-06), ("channel", False, 2.3696e-07),
    ("group", True, 3.1282e-06), ("group", False, 1.3794e-07),
    ("block", True, 2.8968e-06), ("block", False, 5.6068e-07),
]


@pytest.mark.parametrize("strategy,symmetric,exp_loss", MSE_KNOWN)
def test_reference_mse_known_answers(strategy, symmetric, exp_loss):
    t = (np.arange(24, dtype=np.float32) / np.float32(24)).reshape(6, 4)
    args = QArgs(8, "int", symmetric, strategy, 2 if strategy == "group" else None,
                 (3, 2) if strategy == "block" else None)
    mn, mx = observers.mse_minmax(t, args, dtype="f32")
    scale, zp = observers.calculate_qparams(mn, mx, args, dtype="f32")
    f = observers.flatten_weight(t, args)
    q = observers.fake_quant_groups(f, scale.reshape(f.shape[:-1]), np.asarray(zp, np.float32).reshape(f.shape[:-1]),
                                    args, dtype="f32")
    loss = float(np.sum(np.abs(f - q) ** 2) / t.size)
    assert loss == pytest.approx(exp_loss, abs=1e-10)


def test_repack_int4_int8_bit_exact():
    """S/utils/pack_int4_to_int8.py:13-28 on int4 codes and on arbitrary int8 values."""
    g = load("repack_int4_int8")
    np.testing.assert_array_equal(casts.pack_int4_to_int8(g["codes"]), g["codes_packed"])
    np.testing.assert_array_equal(casts.pack_int4_to_int8(g["wild"]), g["wild_packed"])


# --- activation observers of static activation schemes ------------------------
# case -> (observer, QArgs, averaging constant)
ACT_OBS_CASES = {
    "minmax_int8_tensor": ("minmax", QArgs(8, "int", True, "tensor", None), 0.01),
    "static_int8_asym_tensor": ("static_minmax", QArgs(8, "int", False, "tensor", None), 0.01),
    "minmax_nvfp4_tensor_group": ("minmax", QArgs(4, "float", True, "tensor_group", 16, scale_dtype="fp8",
                                                  zp_dtype="fp8"), 0.01),
    "memoryless_int8_group128": ("memoryless_minmax", QArgs(8, "int", False, "group", 128), 0.01),
    "static_fp8_kv_tensor": ("static_minmax", QArgs(8, "float", True, "tensor", None, zp_dtype="fp8"), 0.01),
    "minmax_c05_fp8_tensor": ("minmax", QArgs(8, "float", True, "tensor", None, zp_dtype="fp8"), 0.5),
}


@pytest.mark.parametrize("case", sorted(ACT_OBS_CASES))
def test_activation_observers_oracle_matches_reference(case):
    from oracle.observers import (activation_minmax, calculate_qparams, fused_absmax, generate_gparam,
                                  update_activation_minmax)

    g = load(f"actobs_{case}")
    obs, args, c = ACT_OBS_CASES[case]
    mn = mx = None
    for b in range(4):
        nmn, nmx = activation_minmax(bf16(g[f"x{b}"]), args)
        mn, mx = update_activation_minmax(mn, mx, nmn, nmx, obs, c)
        np.testing.assert_array_equal(numerics.f32_to_bf16_bits(mn), g[f"min{b}"], err_msg=f"min after batch {b}")
        np.testing.assert_array_equal(numerics.f32_to_bf16_bits(mx), g[f"max{b}"], err_msg=f"max after batch {b}")
    gs = generate_gparam(fused_absmax([(mn, mx)])) if args.strategy == "tensor_group" else None
    scale, zp = calculate_qparams(mn, mx, args, global_scale=gs)
    if gs is not None:
        np.testing.assert_array_equal(np.float32(gs).reshape(-1), g["global_scale"].reshape(-1))
        np.testing.assert_array_equal(scale.astype(np.float32).reshape(-1), g["scale"].reshape(-1))
    else:
        np.testing.assert_array_equal(numerics.f32_to_bf16_bits(scale).reshape(-1), g["scale"].reshape(-1))
    if args.type == "int":
        np.testing.assert_array_equal(np.asarray(zp).astype(np.int64).reshape(-1),
                                      g["zero_point"].astype(np.int64).reshape(-1))
    else:
        assert not np.any(g["zero_point"])


def test_activation_minmax_observer_known_answers():
    """T/llmcompressor/observers/test_min_max.py:48-86 (minmax on a tensor
    input, moving average with the default constant 0.01), float32 stats."""
    from oracle.observers import activation_minmax, update_activation_minmax

    args = QArgs(8, "int", True, "tensor", None)
    base = [1, 1, 1, 1, 1]
    seq = [base, base, [127, 1, 1, 1, 1], base, [-128, 1, 1, 1, 1]]
    mn = mx = None
    cur_min, cur_max = 1.0, 1.0
    for i, row in enumerate(seq):
        nmn, nmx = activation_minmax(np.array([row], np.float32), args)
        mn, mx = update_activation_minmax(mn, mx, nmn, nmx, "minmax", 0.01, dtype="f32")
        cur_max, cur_min = max(float(mx[0]), cur_max), min(float(mn[0]), cur_min)
        if i < 2:
            assert cur_max == 1 and cur_min == 1
        elif i < 4:
            assert abs(cur_max - 2.26) < 1e-6 and cur_min == 1
        else:
            assert abs(cur_max - 2.26) < 1e-6 and abs(cur_min - (-0.29)) < 1e-6
