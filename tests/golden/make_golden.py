"""Generate the golden fixtures in this directory by running the reference's
own Triton kernels (wafik/sglang-triton-fusion, ``kernels/``) in Triton's CPU
interpreter (``TRITON_INTERPRET=1``).

Run from the repository root with the path of a reference checkout (or set
SGLANG_TRITON_FUSION_ROOT to it):

    python tests/golden/make_golden.py /path/to/reference

The fixtures (``*.npz``) are committed; tests never read the reference.

What is run, unmodified:
  * ``kernels/fused_gemv_quant_tm.py``: ``fused_gemv_quant`` (routes M==1 to
    ``gemv_quant_row_kernel`` and M>1 to ``gemv_quant_tm_kernel``);
  * ``kernels/fused_gemv_quant.py``: ``fused_gemv_quant`` (row-parallel twin);
  * ``kernels/fused_swiglu_quant_gemv.py``: ``fused_swiglu_q_gemm``.

Those modules import sglang at top level for their ``__main__`` self-tests
only (``fused_gemv_quant_tm.py:16-19`` and its twins); sglang is absent, so
stub modules are registered under those names.  The kernels never call them.

Triton 3.6's interpreter gets two down-conversions wrong (both asserted
below, so the reason stays on record):

* fp32 -> bf16 (the kernels' final ``acc.to(out_ptr.dtype.element_ty)``)
  truncates, where Triton on a GPU rounds to nearest even;
* fp32 -> e4m3 (``.to(tl.float8e4nv)``) rounds ties up, drops the carry out
  of the 3-bit significand at a binade edge (125.2 -> 64) and truncates
  subnormals, where the GPU's ``cvt.rn.satfinite.e4m3x2.f32`` rounds to
  nearest even.

The fp32 -> bf16 store is replaced by torch's RNE cast in every case.
Two families of cases:

``grid_*``  -- "exact-grid" inputs: every 128-group holds +-448 * 2^e and
    otherwise e4m3 values times 2^e, so amax/448, its reciprocal and
    x * (1/sx) are exact and the fp32 -> e4m3 cast needs no rounding; the
    interpreter's own e4m3 encoder is used.

``rand_*``  -- seeded random inputs with the reference benchmarks' value
    distributions; the fp32 -> e4m3 conversion is also replaced by torch's
    round-to-nearest-even cast (the values are already clamped to +-448, so
    saturation plays no part).
    The ``ident_*`` cases among them use an identity weight (1.0 on the
    diagonal, unit block scales), so the reference output is
    bf16(xq[m, n] * sx[m, n/128]) -- a per-element fingerprint of the
    reference kernel's quantised activation.
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import fp8gq_oracle as O  # noqa: E402


def _stub_sglang():
    names = ["sglang", "sglang.kernels", "sglang.kernels.ops", "sglang.kernels.ops.gemm",
             "sglang.kernels.ops.gemm.fp8_blockwise_gemm", "sglang.srt", "sglang.srt.layers",
             "sglang.srt.layers.quantization", "sglang.srt.layers.quantization.fp8_utils"]
    for n in names:
        sys.modules.setdefault(n, types.ModuleType(n))
    sys.modules["sglang.kernels.ops.gemm.fp8_blockwise_gemm"].fp8_blockwise_scaled_mm = None
    sys.modules["sglang.srt.layers.quantization.fp8_utils"].sglang_per_token_group_quant_fp8_row_padded = None


def _interp_builder():
    import triton.runtime.interpreter as interp
    return interp, interp.InterpreterBuilder


class _RneRounding:
    """Context manager: route the interpreter's fp32 -> bf16 conversion and,
    with ``e4m3=True``, its fp32 -> fp8e4nv conversion to torch's RNE casts;
    every other conversion is untouched."""

    def __init__(self, e4m3: bool):
        self.e4m3 = e4m3

    def __enter__(self):
        import triton.language as tl
        interp, B = _interp_builder()
        self._orig_fp = B.create_fp_to_fp
        self._orig_cast = B.cast_impl
        orig_fp, orig_cast, e4m3 = self._orig_fp, self._orig_cast, self.e4m3

        def create_fp_to_fp(builder, src, dst_type, rounding_mode):
            if e4m3 and src.dtype.scalar == tl.float32 and dst_type.scalar == tl.float8e4nv:
                t = torch.from_numpy(np.ascontiguousarray(src.data, dtype=np.float32))
                codes = t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
                return interp.TensorHandle(codes, dst_type.scalar)
            return orig_fp(builder, src, dst_type, rounding_mode)

        def cast_impl(builder, src, dst_type):
            if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
                t = torch.from_numpy(np.ascontiguousarray(src.data, dtype=np.float32))
                bits = t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
                return interp.TensorHandle(bits, dst_type.scalar)
            return orig_cast(builder, src, dst_type)

        B.create_fp_to_fp = create_fp_to_fp
        B.cast_impl = cast_impl
        return self

    def __exit__(self, *exc):
        _, B = _interp_builder()
        B.create_fp_to_fp = self._orig_fp
        B.cast_impl = self._orig_cast


def _check_interpreter_rounding_bugs():
    """Record why the replacement conversions are needed."""
    import triton
    import triton.language as tl

    @triton.jit
    def enc(x_ptr, o_ptr, BLOCK: tl.constexpr):
        offs = tl.arange(0, BLOCK)
        x = tl.load(x_ptr + offs).to(tl.float32)
        tl.store(o_ptr + offs, x.to(tl.float8e4nv).to(tl.float32))

    @triton.jit
    def to_bf16(x_ptr, o_ptr, BLOCK: tl.constexpr):
        offs = tl.arange(0, BLOCK)
        tl.store(o_ptr + offs, tl.load(x_ptr + offs).to(tl.bfloat16))

    x = torch.tensor([125.1636, 100.0, 17.0, 0.015], dtype=torch.float32)
    out = torch.empty_like(x)
    enc[(1,)](x, out, BLOCK=4)
    want = x.to(torch.float8_e4m3fn).float()
    bad = (out != want).sum().item()
    print(f"interpreter e4m3 encoder: {bad}/4 known cases differ from RNE "
          f"(got {out.tolist()}, RNE {want.tolist()})")
    assert bad > 0
    y = torch.tensor([1.00390625 + 2.0 ** -9, -3.0 - 2.0 ** -6], dtype=torch.float32)  # round up in RNE
    ob = torch.empty(2, dtype=torch.bfloat16)
    to_bf16[(1,)](y, ob, BLOCK=2)
    print(f"interpreter bf16 store: got {ob.float().tolist()}, RNE {y.bfloat16().float().tolist()}")
    assert not torch.equal(ob, y.bfloat16())
    with _RneRounding(e4m3=True):
        enc[(1,)](x, out, BLOCK=4)
        to_bf16[(1,)](y, ob, BLOCK=2)
    assert torch.equal(out, want) and torch.equal(ob, y.bfloat16())


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(O.bf16_bits(a).view(np.int16).copy()).view(torch.bfloat16)


def _fp8(codes: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(codes, dtype=np.uint8)).view(torch.float8_e4m3fn)


def _grid_activation(rng, M, K, with_gate=False):
    """Exact-grid activation: per group one +-448 element, the rest random
    finite e4m3 codes; everything times 2^e (e per group)."""
    codes = rng.integers(0, 0x7F, size=(M, K)).astype(np.uint8)   # 0..0x7E, finite
    codes |= (rng.integers(0, 2, size=(M, K)) << 7).astype(np.uint8)
    g = codes.reshape(M, K // 128, 128)
    pos = rng.integers(0, 128, size=(M, K // 128))
    for m in range(M):
        for b in range(K // 128):
            g[m, b, pos[m, b]] = 0x7E | (0x80 if rng.integers(0, 2) else 0)
    e = rng.integers(-8, 5, size=(M, K // 128)).astype(np.float32)
    vals = O.E4M3_TABLE[codes].reshape(M, K // 128, 128) * np.exp2(e)[..., None]
    return vals.reshape(M, K).astype(np.float32)


def _grid_weight(rng, N, K):
    codes = rng.integers(0, 0x7F, size=(N, K)).astype(np.uint8)
    codes |= (rng.integers(0, 2, size=(N, K)) << 7).astype(np.uint8)
    ws = np.exp2(rng.integers(-12, -4, size=(N // 128, K // 128))).astype(np.float32)
    return codes, ws


def main(ref_root: str):
    _stub_sglang()
    sys.path.insert(0, str(Path(ref_root) / "kernels"))
    import fused_gemv_quant as ref_twin          # kernels/fused_gemv_quant.py
    import fused_gemv_quant_tm as ref_tm         # kernels/fused_gemv_quant_tm.py
    import fused_swiglu_quant_gemv as ref_swi    # kernels/fused_swiglu_quant_gemv.py

    _check_interpreter_rounding_bugs()
    rng = np.random.default_rng(20261201)
    cases = {}

    def run_gemv(fn, x, wq, ws, patched):
        with _RneRounding(e4m3=patched):
            out = fn(_bf16(x), _fp8(wq), torch.from_numpy(ws))
        return out.view(torch.int16).numpy().view(np.uint16)

    # ---- exact-grid cases (interpreter's own e4m3 encoder) ----
    for name, fn, M, K, N in [
        ("grid_row_m1", ref_tm.fused_gemv_quant, 1, 384, 256),
        ("grid_tm_m2", ref_tm.fused_gemv_quant, 2, 256, 256),
        ("grid_tm_m5", ref_tm.fused_gemv_quant, 5, 256, 384),
        ("grid_tm_m16", ref_tm.fused_gemv_quant, 16, 256, 256),
        ("grid_tm_m20", ref_tm.fused_gemv_quant, 20, 256, 128),
        ("grid_twin_m3", ref_twin.fused_gemv_quant, 3, 256, 256),
    ]:
        x = _grid_activation(rng, M, K)
        wq, ws = _grid_weight(rng, N, K)
        out = run_gemv(fn, x, wq, ws, patched=False)
        cases[name] = dict(kind="gemv", x=O.bf16_bits(x), wq=wq, ws=ws, out=out)

    # SwiGLU exact-grid: gate = +32 (sigmoid == 1 in fp32) on "on" lanes and
    # -32 elsewhere (silu ~ -4e-13, quantises to a signed zero); up carries
    # the grid values / 32 so act = 32 * up is exact.
    for name, M, I, N in [("grid_swiglu_m1", 1, 256, 256), ("grid_swiglu_m2", 2, 256, 128)]:
        act = _grid_activation(rng, M, I)
        on = rng.random((M, I)) < 0.75
        on |= np.abs(act) == np.abs(act).reshape(M, I // 128, 128).max(-1).repeat(128, -1)
        gate = np.where(on, np.float32(32.0), np.float32(-32.0)).astype(np.float32)
        up = (act / np.float32(32.0)).astype(np.float32)
        gu = np.concatenate([gate, up], axis=1)
        wq, ws = _grid_weight(rng, N, I)
        out = run_gemv(ref_swi.fused_swiglu_q_gemm, gu, wq, ws, patched=False)
        cases[name] = dict(kind="swiglu", x=O.bf16_bits(gu), wq=wq, ws=ws, out=out)

    # ---- random cases (RNE e4m3 encoder) ----
    for name, fn, M, K, N in [
        ("rand_row_m1", ref_tm.fused_gemv_quant, 1, 512, 256),
        ("rand_tm_m3", ref_tm.fused_gemv_quant, 3, 256, 256),
        ("rand_tm_m16", ref_tm.fused_gemv_quant, 16, 256, 128),
        ("rand_twin_m1", ref_twin.fused_gemv_quant, 1, 256, 384),
    ]:
        x = O.make_activation(M, K, seed=int(rng.integers(1 << 30)))
        wq, ws = O.make_weight(N, K, seed=int(rng.integers(1 << 30)))
        out = run_gemv(fn, x, wq, ws, patched=True)
        cases[name] = dict(kind="gemv", x=O.bf16_bits(x), wq=wq, ws=ws, out=out)

    for name, M, I, N in [("rand_swiglu_m1", 1, 384, 256), ("rand_swiglu_m2", 2, 256, 128)]:
        gu = O.make_activation(M, 2 * I, seed=int(rng.integers(1 << 30)), std=1.5, outlier_frac=0.0)
        wq, ws = O.make_weight(N, I, seed=int(rng.integers(1 << 30)))
        out = run_gemv(ref_swi.fused_swiglu_q_gemm, gu, wq, ws, patched=True)
        cases[name] = dict(kind="swiglu", x=O.bf16_bits(gu), wq=wq, ws=ws, out=out)

    # identity-weight probes: out = bf16(xq * sx) elementwise
    for name, fn, M, K in [("ident_row_m1", ref_tm.fused_gemv_quant, 1, 512),
                           ("ident_tm_m4", ref_tm.fused_gemv_quant, 4, 256)]:
        x = O.make_activation(M, K, seed=int(rng.integers(1 << 30)))
        x[0, :128] = 0.0                       # an all-zero group: eps floor, q = 0
        wq = np.where(np.eye(K, dtype=bool), np.uint8(0x38), np.uint8(0)).astype(np.uint8)
        ws = np.ones((K // 128, K // 128), np.float32)
        out = run_gemv(fn, x, wq, ws, patched=True)
        cases[name] = dict(kind="gemv", x=O.bf16_bits(x), wq=wq, ws=ws, out=out)

    for name, c in cases.items():
        np.savez_compressed(HERE / f"{name}.npz", kind=np.array(c["kind"]), x_bf16=c["x"],
                            wq=c["wq"], ws=c["ws"], out_bf16=c["out"])
        print(f"wrote {name}.npz  x{c['x'].shape} w{c['wq'].shape}")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SGLANG_TRITON_FUSION_ROOT")
    if not root:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference  (or set SGLANG_TRITON_FUSION_ROOT)")
    main(root)
