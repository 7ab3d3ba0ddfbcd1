"""GPU parity of the observer / qparams / cast kernels (called through the C ABI).

Bar: bit-exact against the golden fixtures produced by the reference itself
and against the CPU oracle on larger seeded inputs."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

from golden_io import bf16, load
from gpu_util import bits, np_f32, rand_bf16, to_dev_bf16
from llmcompressor_b200 import _lib, ops
from oracle import casts as ocasts
from oracle import numerics as onum
from oracle import observers as oobs

pytestmark = pytest.mark.gpu

SCHEMES = ["W4A16", "W4A16_ASYM", "W8A16", "FP8_DYNAMIC", "FP8", "FP8_BLOCK", "MXFP4A16", "NVFP4A16"]


def _weights_args(name):
    return preset_name_to_scheme(name, ["Linear"]).weights


def _cmp_state(out: dict, ref: dict, prefix: str, tag: str):
    for k, v in out.items():
        key = prefix + k
        assert key in ref, f"{tag}: unexpected key {k}"
        r = ref[key]
        got = bits(v).reshape(r.shape)
        np.testing.assert_array_equal(got, r, err_msg=f"{tag}:{k}")
    produced = {prefix + k for k in out}
    expected = {k for k in ref if k.startswith(prefix) and not k.endswith("input_scale")}
    assert expected <= produced, f"{tag}: missing {expected - produced}"


@pytest.mark.parametrize("scheme", SCHEMES)
def test_modelfree_golden_bit_exact(scheme):
    g = load(f"modelfree_{scheme}")
    w = to_dev_bf16(g["weight"])
    out = ops.modelfree_quantize(w, _weights_args(scheme))
    torch.cuda.synchronize()
    _cmp_state(out, {k: v for k, v in g.items() if k != "weight"}, "out_", scheme)


def test_nvfp4_fused_qkv_golden_bit_exact():
    g = load("modelfree_NVFP4A16_fused_qkv")
    names = ("q_proj", "k_proj", "v_proj")
    ws = [to_dev_bf16(g[f"{n}_weight"]) for n in names]
    gs = ops.fused_global_scale(ws)
    args = _weights_args("NVFP4A16")
    for n, w in zip(names, ws):
        out = ops.modelfree_quantize(w, args, global_scale=gs)
        _cmp_state(out, g, f"{n}_out_", n)


OBS = {
    "int4_sym_group128": QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128),
    "int4_asym_group128": QuantizationArgs(num_bits=4, type="int", symmetric=False, strategy="group", group_size=128),
    "int8_sym_channel": QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="channel"),
    "int4_sym_tensor": QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="tensor"),
    "fp8_block_128": QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="block", block_structure=[128, 128]),
    "int8_asym_channel": QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="channel"),
}


@pytest.mark.parametrize("case", sorted(OBS))
def test_observer_and_qparams_golden_bit_exact(case):
    g = load(f"observer_{case}")
    args = OBS[case]
    w = to_dev_bf16(g["weight"])
    mn, mx = ops.observe_minmax(w, args)
    np.testing.assert_array_equal(bits(mn).reshape(g["min_vals"].shape), g["min_vals"])
    np.testing.assert_array_equal(bits(mx).reshape(g["max_vals"].shape), g["max_vals"])
    scale, zp = ops.calculate_qparams(mn, mx, args)
    np.testing.assert_array_equal(bits(scale).reshape(g["scale"].shape), g["scale"])
    np.testing.assert_array_equal(bits(zp).reshape(g["zero_point"].shape), g["zero_point"])


LARGE = [
    ("W4A16", 1024, 4096, "normal"),
    ("W4A16_ASYM", 512, 2048, "normal"),
    ("W8A16", 384, 3072, "normal"),
    ("FP8_DYNAMIC", 256, 7168, "student_t"),
    ("FP8_BLOCK", 576, 7168, "student_t"),  # 576 rows: padded last block row
    ("FP8_BLOCK", 300, 1000, "student_t"),  # ragged in both dims, cols % 8 != 0
    ("MXFP4A16", 1024, 2048, "student_t"),
    ("NVFP4A16", 1024, 4096, "normal"),
    ("FP8", 128, 4096, "normal"),
    # shapes that select each kernel: channel rows held in 1/2/4/8 registers
    # pieces or too long for them, per-tensor with a ragged tail, group-16
    # spans with numel % 32 != 0
    ("FP8_DYNAMIC", 64, 28672, "student_t"),
    ("FP8_DYNAMIC", 16, 40000, "normal"),
    ("W8A16", 96, 14336, "normal"),
    ("FP8", 33, 1000, "student_t"),
    ("FP8", 256, 4100, "normal"),
    ("NVFP4A16", 33, 1040, "normal"),
    ("MXFP4A16", 7, 4096, "student_t"),
]


@pytest.mark.parametrize("scheme,rows,cols,kind", LARGE)
def test_modelfree_vs_oracle_bit_exact(scheme, rows, cols, kind):
    wt = rand_bf16(rows, cols, seed=rows * 7 + cols, kind=kind)
    w = wt.cuda()
    out = ops.modelfree_quantize(w, _weights_args(scheme))
    ref = ocasts.modelfree_tensor(np_f32(wt), scheme)
    for k, v in ref.items():
        got = bits(out[k])
        if v.dtype == np.float32 and k == "weight_scale":
            v = onum.f32_to_bf16_bits(v)
        np.testing.assert_array_equal(got.reshape(v.shape), v, err_msg=f"{scheme}:{k}")


@pytest.mark.parametrize("scheme", ["W4A16", "W8A16", "FP8_DYNAMIC", "FP8_BLOCK", "MXFP4A16", "NVFP4A16", "W4A16_ASYM"])
def test_quantize_pack_given_qparams_matches_fused(scheme):
    """The compressor path (observer -> qparams -> quantize_pack) equals the fused pass."""
    args = _weights_args(scheme)
    w = rand_bf16(256, 1024, seed=5).cuda()
    fused = ops.modelfree_quantize(w, args)
    mn, mx = ops.observe_minmax(w, args)
    gs = ops.fused_global_scale([w]) if scheme == "NVFP4A16" else None
    scale, zp = ops.calculate_qparams(mn, mx, args, global_scale=gs)
    packed = ops.quantize_pack(w, args, scale, zp, global_scale=gs)
    key = "weight" if scheme.startswith("FP8") else "weight_packed"
    np.testing.assert_array_equal(bits(packed), bits(fused[key]))


def test_fp8_cast_every_bf16_value_matches_torch():
    """All finite bf16 values through the FP8 cast with scale 1 vs torch's own cast."""
    u = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = bf16(u)
    x = np.where(np.isfinite(x), x, 0).astype(np.float32)
    wt = torch.from_numpy(x).to(torch.bfloat16).reshape(256, 256)
    args = QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="tensor")
    out = ops.quantize_pack(wt.cuda(), args, torch.ones(1, dtype=torch.bfloat16, device="cuda"))
    ref = torch.clamp(wt.float(), -448, 448).to(torch.float8_e4m3fn)
    np.testing.assert_array_equal(bits(out), bits(ref))


def test_int8_quotient_rounding_random_scales():
    """bf16 quotient + round at 8-bit resolution with random per-group scales vs the oracle:
    exercises the reciprocal fast path and its exact fallback."""
    rows, cols, gsz = 512, 4096, 64
    g = torch.Generator().manual_seed(3)
    wt = (torch.randn(rows, cols, generator=g) * 3).to(torch.bfloat16)
    st = (torch.rand(rows, cols // gsz, generator=g) * 0.05 + 1e-3).to(torch.bfloat16)
    args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="group", group_size=gsz)
    out = ops.quantize_pack(wt.cuda(), args, st.cuda(), fmt=_lib.FMT_INT8)
    qa = oobs.QArgs(8, "int", True, "group", gsz)
    ref = ocasts.quantize_int(np_f32(wt), np_f32(st), None, qa)
    np.testing.assert_array_equal(bits(out), ref)


def test_known_answer_lifecycle_stats_on_gpu():
    """T/llmcompressor/modifiers/calibration/test_lifecycle.py:16-121 statistics
    (arange(24) as 4x6 bf16) through the kernels, for every strategy there."""
    w = torch.arange(24, dtype=torch.bfloat16).reshape(4, 6).cuda()
    cases = [
        (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="tensor"), [0.0], [23.0]),
        (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="channel"), [0, 6, 12, 18], [5, 11, 17, 23]),
        (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=3),
         [0, 3, 6, 9, 12, 15, 18, 21], [2, 5, 8, 11, 14, 17, 20, 23]),
        (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="block", block_structure=[2, 3]),
         [0, 3, 12, 15], [8, 11, 20, 23]),
    ]
    for args, emn, emx in cases:
        mn, mx = ops.observe_minmax(w, args)
        assert mn.float().cpu().reshape(-1).tolist() == [float(v) for v in emn]
        assert mx.float().cpu().reshape(-1).tolist() == [float(v) for v in emx]
        scale, _ = ops.calculate_qparams(mn, mx, args)
        qa = oobs.QArgs(4, "int", True, getattr(args.strategy, "value", args.strategy), args.group_size,
                        tuple(args.block_structure) if args.block_structure else None)
        omn, omx = oobs.minmax(np.arange(24, dtype=np.float32).reshape(4, 6), qa)
        osc, _ = oobs.calculate_qparams(omn, omx, qa)
        np.testing.assert_array_equal(bits(scale).reshape(-1), onum.f32_to_bf16_bits(osc).reshape(-1))


def test_edge_cases_and_errors():
    args = QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128)
    empty = torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")
    out = ops.modelfree_quantize(empty, args)
    assert out["weight_packed"].shape == (0, 32)
    with pytest.raises(ValueError):
        ops.modelfree_quantize(torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda"), args)
    g3 = QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=3)
    with pytest.raises(NotImplementedError):
        ops.modelfree_quantize(torch.zeros(4, 6, dtype=torch.bfloat16, device="cuda"), g3)
    with pytest.raises(NotImplementedError):
        ops.modelfree_quantize(torch.zeros(4, 256, dtype=torch.float16, device="cuda"), args)
    with pytest.raises(ValueError):
        ops.modelfree_quantize(torch.zeros(4, 4, 256, dtype=torch.bfloat16, device="cuda"), args)
    # all-zero weight: eps scales, zero codes
    z = ops.modelfree_quantize(torch.zeros(8, 256, dtype=torch.bfloat16, device="cuda"), args)
    assert torch.all(z["weight_scale"].float() == 2.0**-7)
    assert torch.all(z["weight_packed"] == 0x88888888 - 2**32)


@pytest.mark.parametrize("scheme", ["W4A16", "W4A16_ASYM", "W8A16", "FP8_DYNAMIC", "FP8", "FP8_BLOCK", "MXFP4A16",
                                    "NVFP4A16"])
def test_unaligned_views_match_aligned(scheme):
    """A weight view 16 bytes past an aligned address (not 32-byte aligned) takes
    the general kernels; its results equal the aligned copy's bit for bit."""
    rows, cols = 256, 2048
    args = _weights_args(scheme)
    base = rand_bf16(rows * cols + 8, 1, seed=11).reshape(-1).cuda()
    view = base[8:].view(rows, cols)
    assert view.data_ptr() % 32 == 16
    dense = view.clone()
    gs = ops.fused_global_scale([dense]) if scheme == "NVFP4A16" else None
    a = ops.modelfree_quantize(view, args, gs)
    b = ops.modelfree_quantize(dense, args, gs)
    for k in b:
        np.testing.assert_array_equal(bits(a[k]), bits(b[k]), err_msg=f"{scheme}:{k}")


def test_float32_scales_quotient_matches_torch():
    """Stored float32 scales: float32 quotient, round half-even, clamp, as torch
    evaluates x.float() / s -- many random scales through the paired fast path."""
    rows, cols, gsz = 512, 4096, 128
    g = torch.Generator().manual_seed(9)
    wt = (torch.randn(rows, cols, generator=g) * 2).to(torch.bfloat16)
    st = torch.rand(rows, cols // gsz, generator=g) * 0.03 + 1e-4
    args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="group", group_size=gsz)
    out = ops.quantize_pack(wt.cuda(), args, st.cuda(), fmt=_lib.FMT_INT8)
    q = wt.float() / st.repeat_interleave(gsz, dim=1)
    ref = torch.clamp(torch.round(q), -128, 127).to(torch.int8)
    np.testing.assert_array_equal(bits(out), bits(ref))


def test_overflowing_and_tiny_scales_match_torch():
    """Quotients that overflow float32 (huge weights, tiny stored scales) and
    scales whose reciprocal is not a normal float take the exact division."""
    rows, cols, gsz = 64, 256, 32
    g = torch.Generator().manual_seed(4)
    wt = torch.randn(rows, cols, generator=g)
    wt[:, :64] *= 1e30
    wt = wt.to(torch.bfloat16)
    st = torch.full((rows, cols // gsz), 0.5)
    st[:, 0] = 1e-12      # x / s overflows for the 1e30 columns
    st[:, 1] = 1e-38      # reciprocal above the normal range
    st[:, 2] = 3e38       # reciprocal below it
    st = st.to(torch.bfloat16)
    args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="group", group_size=gsz)
    out = ops.quantize_pack(wt.cuda(), args, st.cuda(), fmt=_lib.FMT_INT8)
    q = (wt.float() / st.float().repeat_interleave(gsz, dim=1)).to(torch.bfloat16).float()
    ref = torch.clamp(torch.round(q), -128, 127).to(torch.int8)
    np.testing.assert_array_equal(bits(out), bits(ref))


@pytest.mark.parametrize("scheme", ["W4A16", "W4A16_ASYM", "W8A16", "FP8_DYNAMIC", "FP8_BLOCK", "MXFP4A16",
                                    "NVFP4A16", "FP8"])
def test_modelfree_batch_matches_single(scheme):
    """The batched launch equals one launch per tensor, bit for bit, across
    shapes the batched kernels take and shapes they hand back (unaligned view,
    ragged columns), and across more tensors than one batch holds."""
    args = _weights_args(scheme)
    shapes = [(64, 1024), (128, 2048), (32, 4096), (256, 512)] * 13  # 52 tensors: two batches
    ws = [rand_bf16(r, c, seed=i, kind="student_t" if i % 3 == 0 else "normal").cuda() for i, (r, c) in enumerate(shapes)]
    base = rand_bf16(64 * 1024 + 8, 1, seed=99).reshape(-1).cuda()
    ws.append(base[8:].view(64, 1024))  # 16 bytes past alignment
    if scheme in ("FP8_DYNAMIC", "W8A16"):
        ws.append(rand_bf16(48, 1000, seed=77).cuda())  # cols % 16 != 0
    gss = [ops.fused_global_scale([w]) for w in ws] if scheme == "NVFP4A16" else None
    got = ops.modelfree_quantize_batch(ws, args, gss)
    for i, w in enumerate(ws):
        ref = ops.modelfree_quantize(w, args, gss[i] if gss else None)
        assert set(got[i]) == set(ref)
        for k in ref:
            np.testing.assert_array_equal(bits(got[i][k]), bits(ref[k]), err_msg=f"{scheme}[{i}]:{k}")


def test_repack_int4_int8_golden_and_large():
    g = load("repack_int4_int8")
    for k in ("codes", "wild"):
        got = ops.pack_int4_to_int8(torch.from_numpy(g[k]).cuda())
        np.testing.assert_array_equal(got.cpu().numpy(), g[f"{k}_packed"])
    gen = torch.Generator().manual_seed(5)
    for rows, cols in ((4096, 14336), (33, 1000)):  # vector path, then the bytewise path
        t = torch.randint(-128, 128, (rows, cols), generator=gen, dtype=torch.int8)
        got = ops.pack_int4_to_int8(t.cuda())
        np.testing.assert_array_equal(got.cpu().numpy(), ocasts.pack_int4_to_int8(t.numpy()))
    with pytest.raises(ValueError):
        ops.pack_int4_to_int8(torch.zeros(4, 3, dtype=torch.int8, device="cuda"))


@pytest.mark.gpu
@pytest.mark.parametrize("scheme", ["NVFP4A16", "MXFP4A16"])
def test_fp4_groups_with_nonfinite_values_agree_across_kernels(scheme):
    """FP4 groups whose values are all finite skip the explicit clamp to
    [-6, 6] (the saturating E2M1 conversion clamps them); groups holding NaN
    or +-inf keep it and take the IEEE quotient for the infinite values.  The
    single-tensor kernel, the batched kernel and the general kernel (taken
    for a weight that is not 32-byte aligned) must give the same bytes for
    both kinds of group.  (For a group holding NaN or inf the reference's own
    statistics are not finite; there is no reference value to hold the
    kernels to, only their agreement.)"""
    qa = preset_name_to_scheme(scheme, ["Linear"]).weights
    rows, cols = 256, 1024
    group = qa.group_size
    g = torch.Generator().manual_seed(5)
    w = 0.02 * torch.randn(rows, cols, generator=g)
    w[0, 3] = 7.0  # one large value: its group's scale clamps the others
    idx = torch.randperm(rows * cols, generator=g)[:48]
    w.view(-1)[idx] = torch.tensor([float("nan"), float("inf"), -float("inf")]).repeat(16)
    finite_groups = torch.isfinite(w).view(rows, cols // group, group).all(dim=-1)
    w = w.to(torch.bfloat16).cuda()
    store = torch.empty(rows * cols + 8, dtype=torch.bfloat16, device="cuda")
    unaligned = store[8:].view(rows, cols)
    unaligned.copy_(w)
    finite = torch.nan_to_num(w, nan=0.0, posinf=0.0, neginf=0.0)
    gs = ops.fused_global_scale([finite]) if scheme == "NVFP4A16" else None
    single = ops.modelfree_quantize(w, qa, gs)
    general = ops.modelfree_quantize(unaligned, qa, gs)
    batched = ops.ModelfreeBatch([w, w], qa, [gs, gs]).run().results
    for key in ("weight_packed", "weight_scale"):
        ref = bits(single[key])
        for r in batched:
            np.testing.assert_array_equal(bits(r[key]), ref, err_msg=key)
        np.testing.assert_array_equal(bits(general[key]), ref, err_msg=key)
    assert not bool(finite_groups.all())  # both kinds of group were exercised
