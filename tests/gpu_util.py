"""Helpers shared by the GPU parity tests."""

import numpy as np
import torch

from oracle import ltx_block_oracle as O


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def codes(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy()


def from_bits(bits: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def within_ulps(got: np.ndarray, ref: np.ndarray, ulps: float = 1.0, atol: float = 0.0) -> tuple[bool, float]:
    """|got - ref| <= atol + ulps * bf16-ulp(ref) elementwise; returns (ok, worst ratio)."""
    ref = np.asarray(ref, np.float32)
    mag = np.maximum(np.abs(ref), np.float32(2.0 ** -126))
    ulp = np.exp2(np.floor(np.log2(mag)) - 7.0)
    bound = atol + ulps * ulp
    d = np.abs(np.asarray(got, np.float32) - ref)
    return bool((d <= bound).all()), float((d / bound).max())


def block_tolerance(got: np.ndarray, ref: np.ndarray, *, atol: float = 2e-2, mean_rel: float = 1e-2) -> dict:
    """The north-star tolerance: max-abs <= 2e-2 (plus one bf16 ulp of |ref|, the rounding of a
    bf16 output alone) and sum|d| / sum|ref| <= 1e-2.  Returns the measured figures."""
    d = np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))
    excess = d - (atol + np.abs(ref) * 2.0 ** -7)
    ref_formula = float((d / np.maximum(np.abs(ref), 1e-6)).mean())  # the reference's own mean_rel
    return {
        "max_abs": float(d.max()),
        "max_excess": float(excess.max()),
        "mean_rel": float(d.sum() / max(np.abs(ref).sum(), 1e-30)),
        "ref_mean_rel": ref_formula,
        "ok": bool(excess.max() <= 0 and d.sum() / max(np.abs(ref).sum(), 1e-30) <= mean_rel),
    }


def status_clean():
    from opengenie_b200 import _lib

    torch.cuda.synchronize()
    return _lib.device_status(clear=True) == 0


__all__ = ["O", "to_np", "bf16_bits", "codes", "from_bits", "within_ulps", "block_tolerance", "status_clean"]
