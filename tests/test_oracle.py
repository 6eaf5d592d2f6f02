"""The CPU oracle, pinned against the reference before anything is compared
with it: golden fixtures from the reference's own kernels, torch's e4m3 cast,
and the known-answer cases of the reference's stress tests."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8gq_oracle as O

GOLDEN = sorted(p for p in (Path(__file__).parent / "golden").glob("*.npz") if not p.stem.startswith("writer_"))
WRITER_GOLDEN = sorted((Path(__file__).parent / "golden").glob("writer_*.npz"))


def test_golden_fixtures_present():
    names = {p.stem for p in GOLDEN}
    for want in ("grid_row_m1", "grid_tm_m16", "grid_swiglu_m1", "rand_row_m1", "rand_tm_m3",
                 "rand_swiglu_m1", "ident_row_m1", "ident_tm_m4"):
        assert want in names


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_oracle_matches_reference_kernels_bit_exact(path):
    """The reference's Triton kernels (run in Triton's CPU interpreter) and the
    oracle produce the same bf16 bits on every golden case."""
    d = np.load(path)
    x = O.bf16_from_bits(d["x_bf16"])
    fn = O.fused_gemv_quant if str(d["kind"]) == "gemv" else O.fused_swiglu_q_gemm
    out, exact, xq, sx = fn(x, d["wq"], d["ws"])
    ref = O.bf16_from_bits(d["out_bf16"])
    assert np.array_equal(out, ref), f"{path.stem}: {np.mean(out != ref) * 100:.2f}% of outputs differ"


@pytest.mark.parametrize("name", ["ident_row_m1", "ident_tm_m4"])
def test_identity_probe_pins_quant_bytes(name):
    """With an identity weight the reference output is bf16(xq * sx) per
    element, a fingerprint of the reference kernel's quantised activation."""
    d = np.load(Path(__file__).parent / "golden" / f"{name}.npz")
    x = O.bf16_from_bits(d["x_bf16"])
    xq, sx = O.group_quant(x)
    fingerprint = O.bf16_round((O.E4M3_TABLE[xq] * np.repeat(sx, 128, axis=1)).astype(np.float32))
    assert np.array_equal(fingerprint, O.bf16_from_bits(d["out_bf16"]))
    # the all-zero first group: eps floor, every code +0
    assert sx[0, 0] == np.float32(1e-10) / np.float32(448.0)
    assert np.all(xq[0, :128] == 0)


def test_e4m3_encoder_matches_torch_cast():
    rng = np.random.default_rng(0)
    y = np.concatenate([rng.standard_normal(400_000).astype(np.float32) * np.float32(60),
                        rng.standard_normal(100_000).astype(np.float32) * np.float32(0.02),
                        rng.standard_normal(100_000).astype(np.float32) * np.float32(1e-4)])
    y = np.clip(y, -448, 448).astype(np.float32)
    ours = O.e4m3_encode_rne(y)
    theirs = torch.from_numpy(y).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)


def test_e4m3_encoder_ties_and_neighbours():
    vals = O.E4M3_TABLE[:0x7F].astype(np.float64)
    mids = ((vals[:-1] + vals[1:]) / 2).astype(np.float32)
    cand = np.concatenate([mids, np.nextafter(mids, np.float32(0)), np.nextafter(mids, np.float32(1e3)),
                           vals.astype(np.float32)])
    cand = np.clip(np.concatenate([cand, -cand]), -448, 448).astype(np.float32)
    theirs = torch.from_numpy(cand).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_encode_rne(cand), theirs)


def test_e4m3_decode_table():
    codes = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    ours = O.e4m3_decode(codes)
    finite = ~np.isnan(ref)
    assert np.array_equal(ours[finite], ref[finite]) and np.all(np.isnan(ours[~finite]))


def test_exp_accuracy_within_one_ulp():
    xs = np.linspace(-88, 88, 400_001).astype(np.float32)
    e = O.exp_f32(xs).astype(np.float64)
    ex = np.exp(xs.astype(np.float64))
    ulp = np.spacing(ex.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(e - ex) / ulp) <= 1.0
    assert O.exp_f32(np.float32([100.0]))[0] == np.inf
    assert O.exp_f32(np.float32([-100.0]))[0] == 0.0


def test_silu_close_to_float64():
    g = np.linspace(-30, 30, 100_001).astype(np.float32)
    u = np.ones_like(g)
    ours = O.silu_mul(g, u).astype(np.float64)
    gd = g.astype(np.float64)
    ref = gd / (1 + np.exp(-gd))
    assert np.max(np.abs(ours - ref) / np.maximum(np.abs(ref), 1e-30)) < 4e-7


def test_known_answer_zero_group():
    """All-zero group: amax floors at 1e-10, every code is +0
    (benchmarks/stress_tests.py:159-165 checks the same for its formula)."""
    xq, sx = O.group_quant(np.zeros((2, 256), np.float32))
    assert np.all(xq == 0)
    assert np.all(sx == np.float32(1e-10) / np.float32(448.0))


def test_known_answer_saturation():
    """The group maximum lands exactly on +-448 (code 0x7E / 0xFE)
    (benchmarks/stress_tests.py:167-176)."""
    x = np.full((1, 128), 3.0, np.float32)
    x[0, 7] = -400.0
    xq, sx = O.group_quant(x)
    assert xq[0, 7] == 0xFE
    assert sx[0, 0] == np.float32(400.0) / np.float32(448.0)
    assert np.all(np.abs(O.E4M3_TABLE[xq]) <= 448.0)


def test_known_answer_negative_gate_finite():
    """silu(-50) * u stays finite and near zero (benchmarks/stress_tests.py:178-185)."""
    g = np.full(256, -50.0, np.float32)
    u = np.linspace(-3, 3, 256).astype(np.float32)
    act = O.silu_mul(g, u)
    assert np.all(np.isfinite(act)) and np.max(np.abs(act)) < 1e-18


def test_determinism():
    x = O.make_activation(3, 512, seed=5)
    a = O.group_quant(x)
    b = O.group_quant(x.copy())
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


# ------------------------------------------ stand-alone SwiGLU writers --

def test_writer_fixtures_present():
    assert {p.stem for p in WRITER_GOLDEN} == {"writer_grid", "writer_rand", "writer_extreme", "writer_zero",
                                                "writer_sat"}


@pytest.mark.parametrize("path", WRITER_GOLDEN, ids=[p.stem for p in WRITER_GOLDEN])
def test_writer_oracle_matches_reference_kernels(path):
    """kernels/fused_swiglu_fp8.py's fused_swiglu and fused_swiglu_quant (run in
    Triton's CPU interpreter) against the oracle: every e4m3 code and every
    bf16 output equal; scales equal, or within one fp32 ulp where the
    reference's exp and the oracle's differ in the last bit (its own test
    allows rtol 1e-5, kernels/fused_swiglu_fp8.py:99-100)."""
    d = np.load(path)
    g, u = O.bf16_from_bits(d["g_bf16"]), O.bf16_from_bits(d["u_bf16"])
    q, scale, _ = O.swiglu_quant_writer(g, u)
    assert np.array_equal(q, d["q"])
    assert np.array_equal(O.bf16_bits(O.swiglu_writer(g, u)), d["y_bf16"])
    assert np.allclose(scale, d["scale"], rtol=2.0 ** -22, atol=0.0)
    if path.stem in ("writer_grid", "writer_zero", "writer_sat"):
        assert np.array_equal(scale, d["scale"])      # exact inputs: exact scales


def test_writer_known_answers():
    """benchmarks/stress_tests.py:159-176: all-zero input gives q = 0 and the
    1e-30 scale floor; gate = up = 20 reaches exactly |q| = 448."""
    z = np.zeros((2, 256), np.float32)
    q, s, _ = O.swiglu_quant_writer(z, z)
    assert np.all(q == 0) and np.all(s == np.float32(1e-30))
    t = np.full((2, 256), 20.0, np.float32)
    q, s, _ = O.swiglu_quant_writer(t, t)
    assert np.max(np.abs(O.E4M3_TABLE[q])) == 448.0


def test_writer_formula_differs_from_gemv_prologue():
    """The writer divides by the scale (kernels/fused_swiglu_fp8.py:42); the
    GEMV prologue multiplies by its rounded reciprocal
    (kernels/fused_gemv_quant.py:42) and floors amax at 1e-10 where the writer
    floors the scale at 1e-30.  Both differences change codes, which is why
    the two quantisers are kept apart."""
    f = np.float32
    y, sc = f(57.31668472290039), f(2.729365825653076)
    div = f(y / sc)                          # 21.0 exactly: a tie, RNE -> 20
    rcp = f(y * f(f(1.0) / sc))              # 21.000002 -> 22
    assert div == f(21.0) and rcp > div
    assert O.e4m3_encode_rne(np.array([div]))[0] != O.e4m3_encode_rne(np.array([rcp]))[0]
    tiny = np.full((1, 128), 1e-12, np.float32)     # amax below the prologue's 1e-10 floor
    qw, sw, _ = O.swiglu_quant_writer(np.full((1, 128), 30.0, np.float32), tiny)
    qg, sg = O.group_quant(O.silu_mul(np.full((1, 128), 30.0, np.float32), tiny))
    assert sw[0, 0] != sg[0, 0] and qw[0, 0] != qg[0, 0]


# ---------------------------------------------------- add + RMSNorm prologue --

def test_add_rmsnorm_close_to_torch():
    """The fixed-order fp32 evaluation agrees with torch's rms_norm of the
    same sum within one bf16 rounding (kernels/fused_rmsnorm.py:74-75 asks
    rtol 1e-4 of its fp32 outputs; ours are bf16)."""
    rng = np.random.default_rng(1)
    x = O.bf16_round(rng.standard_normal((4, 2560)).astype(np.float32))
    r = O.bf16_round(rng.standard_normal((4, 2560)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal(2560) * 0.1).astype(np.float32))
    h, res, rstd = O.add_rmsnorm(x, r, w)
    s = torch.from_numpy(x) + torch.from_numpy(r)
    ref = torch.nn.functional.rms_norm(s, (2560,), torch.from_numpy(w), 1e-6).numpy()
    assert np.all(np.abs(h - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-6)
    assert np.array_equal(res, O.bf16_round(s.numpy()))


def test_add_rmsnorm_known_answers():
    """benchmarks/stress_tests.py:122-146: zero rows give zero outputs (rstd =
    1/sqrt(eps)); weight 1 gives the plain normalisation; 1e6-scale inputs
    stay finite."""
    z = np.zeros((2, 256), np.float32)
    h, res, rstd = O.add_rmsnorm(z, z, np.ones(256, np.float32))
    assert np.all(h == 0) and np.all(res == 0)
    assert rstd[0] == np.float32(1.0) / np.sqrt(np.float32(1e-6))
    rng = np.random.default_rng(2)
    x = O.bf16_round(rng.standard_normal((3, 512)).astype(np.float32) * 1e6)
    h, _, _ = O.add_rmsnorm(x, np.zeros_like(x), np.ones(512, np.float32))
    assert np.all(np.isfinite(h))
    ms = np.mean(h.astype(np.float64) ** 2, axis=1)
    assert np.allclose(ms, 1.0, rtol=2e-2)


def test_torch_reference_path_agrees_with_oracle():
    """The timed CPU baseline (torch quantise / dequantise / matmul) computes
    the same function as the numpy oracle, to bf16 tolerance."""
    from tests._util import bf16_tensor, f32_tensor, fp8_tensor
    x = O.make_activation(2, 512, seed=11)
    wq, ws = O.make_weight(256, 512, seed=12)
    got = O.torch_reference_path(bf16_tensor(x), fp8_tensor(wq), f32_tensor(ws)).float().numpy()
    _, exact, _, _ = O.fused_gemv_quant(x, wq, ws)
    assert O.rms_tolerance_ok(got, exact)
    assert np.max(np.abs(got - exact)) <= O.ref_atol(exact, 2.0)
    xq, _ = O.group_quant(x)
    # its quant is the same formula: the bytes agree
    xt = bf16_tensor(x).float().view(2, 4, 128)
    sxt = xt.abs().amax(-1, keepdim=True).clamp_min(1e-10) / 448.0
    q = (xt * (1.0 / sxt)).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).view(2, 512).numpy()
    assert np.array_equal(q, xq)


def test_make_weight_block_quant():
    wq, ws = O.make_weight(256, 384, seed=3)
    assert wq.shape == (256, 384) and ws.shape == (2, 3)
    deq = O.dequant_weight(wq, ws)
    # every block's max |w| maps to the top code 0x7E / 0xFE
    blk = np.abs(O.E4M3_TABLE[wq]).reshape(2, 128, 3, 128).max(axis=(1, 3))
    assert np.all(blk == 448.0)
    assert np.all(np.isfinite(deq))


def test_reduce_add_rmsnorm_one_partial_is_add_rmsnorm():
    rng = np.random.default_rng(3)
    x = O.bf16_round(rng.standard_normal((2, 512)).astype(np.float32))
    r = O.bf16_round(rng.standard_normal((2, 512)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal(512) * 0.1 + 1).astype(np.float32))
    for a, b in zip(O.add_rmsnorm(x, r, w), O.reduce_add_rmsnorm([x], r, w)):
        assert np.array_equal(a, b)


def test_reduce_add_rmsnorm_adds_in_rank_order():
    """((p0 + p1) + p2) + r, left to right: with p0 = 2^26, p1 = -2^26, p2 = 1
    the sum is 1 (right to left it would round to 0)."""
    K = 128
    p0 = np.full((1, K), 2.0 ** 26, np.float32)
    p1 = -p0
    p2 = np.ones((1, K), np.float32)
    r = np.full((1, K), 0.5, np.float32)
    w = np.ones(K, np.float32)
    _, res, _ = O.reduce_add_rmsnorm([p0, p1, p2], r, w)
    assert np.all(res == np.float32(1.5))
    assert np.float32(p0[0, 0] + np.float32(p1[0, 0] + p2[0, 0])) + np.float32(0.5) == np.float32(0.5)


def test_k_sharded_partials_sum_to_the_full_gemv():
    """A K-sharded linear's partials (each rank quantises its own 128-groups,
    which are the full activation's groups) add up to the unsharded GEMV
    within the GEMV tolerance."""
    M, K, N, world = 2, 1024, 512, 4
    x = O.make_activation(M, K, seed=11)
    wq, ws = O.make_weight(N, K, seed=12)
    _, full, _, _ = O.fused_gemv_quant(x, wq, ws)
    kr = K // world
    parts = []
    for r in range(world):
        out, _, _, _ = O.fused_gemv_quant(x[:, r * kr:(r + 1) * kr], wq[:, r * kr:(r + 1) * kr],
                                          ws[:, r * kr // 128:(r + 1) * kr // 128])
        parts.append(out)
    acc = parts[0]
    for p in parts[1:]:
        acc = (acc + p).astype(np.float32)
    assert O.rms_tolerance_ok(acc, full)
