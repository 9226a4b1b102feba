"""Conversions between the oracle's numpy storage and torch tensors, and parity checks."""

import numpy as np

from oracle import bf16 as BF

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


def to_torch(x: np.ndarray, dtype: str, device="cuda"):
    """numpy storage (uint16 bits for bf16, float32, int64) -> torch tensor on `device`."""
    if x.dtype == np.int64:
        return torch.from_numpy(np.ascontiguousarray(x)).to(device)
    if dtype == "bf16":
        t = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16)
        return t.to(device)
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device)


def to_numpy(t) -> np.ndarray:
    """torch tensor -> numpy storage (bf16 -> uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def values(t, dtype: str) -> np.ndarray:
    """float32 values of a torch tensor of the case dtype."""
    return BF.as_f32(to_numpy(t), dtype)


def bf16_step(x: np.ndarray) -> np.ndarray:
    """Distance between adjacent bf16 values at |x| (2^(e-7) for |x| in [2^e, 2^(e+1)))."""
    e = np.floor(np.log2(np.maximum(np.abs(x.astype(np.float64)), 2.0 ** -126)))
    return np.exp2(e - 7)


def assert_close_bf16(got: np.ndarray, ref: np.ndarray, max_abs=2e-2, mean_abs=2e-3, what="",
                      steps=1):
    """The hot path's bf16 tolerance: max-abs 2e-2, mean-abs 2e-3.

    For |ref| >= 4 one bf16 step (2^-5 and up) is itself above 2e-2, so an element there passes
    when it is within one step of the reference value; everywhere else the absolute bound holds.
    steps=2 is for outputs the reference rounds twice to bf16 (the gated RMSNorm of an output
    that was itself rounded, rms_norm_gated.py after linear_attention.py:298): an fp32-level
    difference that flips the first rounding moves the normalised value by one step of its own
    before the second rounding, so such an element may sit two steps from the reference.
    """
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    r = ref.astype(np.float64)
    d = np.abs(got.astype(np.float64) - r)
    bound = np.maximum(max_abs, steps * bf16_step(r))
    worst = int(np.argmax(d - bound))
    assert (d <= bound).all(), (f"{what}: |diff| {d.ravel()[worst]:.3g} > {bound.ravel()[worst]:.3g}"
                                f" at ref {r.ravel()[worst]:.4g} (max-abs {d.max():.3g})")
    assert d.mean() <= mean_abs, f"{what}: mean-abs {d.mean():.3g} > {mean_abs}"


def assert_close(got, ref, dtype: str, what="", f32_rtol=1e-4, f32_atol=1e-5, bf16_steps=1):
    if dtype == "f32":
        np.testing.assert_allclose(got, ref, rtol=f32_rtol, atol=f32_atol, err_msg=what)
    else:
        assert_close_bf16(got, ref, what=what, steps=bf16_steps)
