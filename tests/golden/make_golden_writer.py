"""Generate the golden fixtures of the stand-alone SwiGLU writers by running
the reference's own Triton kernels (wafik/sglang-triton-fusion,
``kernels/fused_swiglu_fp8.py``: ``fused_swiglu`` and ``fused_swiglu_quant``)
in Triton's CPU interpreter (``TRITON_INTERPRET=1``).

Run from the repository root with the path of a reference checkout (or set
SGLANG_TRITON_FUSION_ROOT to it):

    python tests/golden/make_golden_writer.py /path/to/reference

The fixtures (``writer_*.npz``) are committed; tests never read the reference.
The module imports only torch and triton, so it runs unmodified.  The
interpreter's fp32 -> bf16 and fp32 -> e4m3 conversions are replaced by
torch's round-to-nearest-even casts, exactly as in make_golden.py (which
documents and asserts the two interpreter bugs).

Cases (each stores gate and up as bf16 bits, the bf16 SwiGLU output, the e4m3
codes and the fp32 scales):

``writer_grid``     gate = +-32 (sigmoid(32) == 1 in fp32; silu(-32) ~ -4e-13),
                    up = exact-grid values / 32, so y = 32 * up is exact on the
                    "on" lanes and every group's scale is a power of two: the
                    codes and scales are exact, any correct evaluation of the
                    formula reproduces them bit for bit.
``writer_rand``     gate, up ~ N(0, 1) (the module's __main__ inputs).
``writer_extreme``  gate, up ~ N(0, 10) (benchmarks/stress_tests.py:186-191).
``writer_zero``     gate = up = 0: q = 0, scale = 1e-30 (stress_tests.py:159-165).
``writer_sat``      gate = up = 20: max |q| = 448 (stress_tests.py:167-176).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

from oracle import fp8gq_oracle as O  # noqa: E402
from make_golden import _RneRounding, _check_interpreter_rounding_bugs, _grid_activation  # noqa: E402


def main(ref_root: str):
    sys.path.insert(0, str(Path(ref_root) / "kernels"))
    import fused_swiglu_fp8 as ref_w            # kernels/fused_swiglu_fp8.py

    _check_interpreter_rounding_bugs()
    rng = np.random.default_rng(20261202)

    def bf16(a):
        return torch.from_numpy(O.bf16_bits(np.asarray(a, np.float32)).view(np.int16).copy()).view(torch.bfloat16)

    def run(gate, up):
        gate, up = O.bf16_round(gate), O.bf16_round(up)     # the bf16 inputs, stored as given
        g, u = bf16(gate), bf16(up)
        with _RneRounding(e4m3=True):
            y = ref_w.fused_swiglu(g, u)
            q, s = ref_w.fused_swiglu_quant(g, u)
        return dict(g_bf16=O.bf16_bits(gate), u_bf16=O.bf16_bits(up),
                    y_bf16=y.view(torch.int16).numpy().view(np.uint16),
                    q=q.view(torch.uint8).numpy().copy(), scale=s.numpy().copy())

    cases = {}
    M, I = 3, 512
    act = _grid_activation(rng, M, I)
    on = rng.random((M, I)) < 0.75
    on |= np.abs(act) == np.abs(act).reshape(M, I // 128, 128).max(-1).repeat(128, -1)
    gate = np.where(on, np.float32(32.0), np.float32(-32.0)).astype(np.float32)
    cases["writer_grid"] = run(gate, (act / np.float32(32.0)).astype(np.float32))

    cases["writer_rand"] = run(rng.standard_normal((4, 1024)).astype(np.float32),
                               rng.standard_normal((4, 1024)).astype(np.float32))
    cases["writer_extreme"] = run((rng.standard_normal((4, 1024)) * 10).astype(np.float32),
                                  (rng.standard_normal((4, 1024)) * 10).astype(np.float32))
    z = np.zeros((4, 768), np.float32)
    cases["writer_zero"] = run(z, z)
    t = np.full((2, 768), 20.0, np.float32)
    cases["writer_sat"] = run(t, t)

    for name, c in cases.items():
        np.savez_compressed(HERE / f"{name}.npz", kind=np.array("writer"), **c)
        print(f"wrote {name}.npz  gate{c['g_bf16'].shape}")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SGLANG_TRITON_FUSION_ROOT")
    if not root:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference  (or set SGLANG_TRITON_FUSION_ROOT)")
    main(root)
