"""Helpers shared by the tests: numpy oracle arrays <-> torch tensors."""
import numpy as np
import torch

from oracle import fp8gq_oracle as O


def bf16_tensor(a: np.ndarray, device="cpu") -> torch.Tensor:
    """float32 array holding bf16 values -> torch bf16 tensor."""
    bits = O.bf16_bits(np.asarray(a, np.float32)).view(np.int16).copy()
    return torch.from_numpy(bits).view(torch.bfloat16).to(device)


def bf16_bits_tensor(bits: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.asarray(bits, np.uint16).view(np.int16).copy()).view(torch.bfloat16).to(device)


def fp8_tensor(codes: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(codes, np.uint8)).view(torch.float8_e4m3fn).to(device)


def f32_tensor(a: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def to_u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.uint8).numpy() if t.dtype != torch.uint8 else t.detach().cpu().numpy()


def ulp_report(got: np.ndarray, ref: np.ndarray) -> str:
    d = np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))
    ulp = O.bf16_ulp_at(float(np.abs(ref).max()))
    return f"maxabs {d.max():.4g} ({d.max() / ulp:.2f} ulp of max |ref| {np.abs(ref).max():.4g})"


def assert_close(got, ref_exact, ulps: float):
    """Both tolerances: the relative one (rtol 1e-2, atol 1e-2 * RMS) and the
    reference self-test's (atol = ulps * ulp_bf16(max|ref|) + 1e-3, rtol 0)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref_exact, np.float64)
    assert O.rms_tolerance_ok(got, ref), "rtol 1e-2 / atol 1e-2*RMS tolerance: " + ulp_report(got, ref)
    atol = O.ref_atol(ref, ulps)
    assert np.all(np.abs(got - ref) <= atol), f"reference tolerance {ulps} ulp: " + ulp_report(got, ref)
