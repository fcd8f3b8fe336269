"""Test helpers: tolerances, seeded inputs, comparisons, CUDA tensor glue."""
import numpy as np

# Tolerances from the north star: f16/bf16 inputs with f32 accumulation, and
# the reference's own f32 bar (test_flash_attention_tiled.rs:123-130).
TOL_16BIT_MAXABS = 2e-3
TOL_16BIT_COS = 0.9999
TOL_F32_MAXABS = 1e-5


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def randn(seed: int, n: int) -> np.ndarray:
    """Seeded N(0,1) f32 samples (numpy PCG64)."""
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


def torch_dtype(dt: int):
    import torch
    return {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[dt]


def rounded(x: np.ndarray, dt: int):
    """(CUDA tensor of dtype dt, f32 numpy of the rounded values the kernel sees)."""
    import torch
    t = torch.from_numpy(x).to(torch_dtype(dt))
    return t.cuda(), t.float().numpy().ravel()


def half_ulp(x: np.ndarray, dt: int) -> np.ndarray:
    """Half a unit in the last place of |x| in output type dt (0 for f32)."""
    if dt == 0:
        return np.zeros_like(x)
    mant = 10 if dt == 1 else 7  # f16 / bf16 explicit mantissa bits
    e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -14)))
    return 0.5 * 2.0 ** (e - mant)


def check_16bit(out, ref, what="", out_dt=0):
    """North-star bar for 16-bit inputs with f32 accumulation: max-abs <= 2e-3
    and cosine > 0.9999 against the f32 oracle on the same rounded inputs.
    When the kernel stores a 16-bit output, the storage rounding (half an
    output ulp) is added to the max-abs bound."""
    out = np.asarray(out, np.float32).ravel()
    ref = np.asarray(ref, np.float32).ravel()
    err = float((np.abs(out - ref) - half_ulp(ref, out_dt)).max())
    cos = cosine(out, ref)
    assert np.all(np.isfinite(out)), f"{what}: non-finite output"
    assert err <= TOL_16BIT_MAXABS and cos > TOL_16BIT_COS, f"{what}: max-abs {err:.3g} cos {cos:.8f}"
    return err, cos


def check_f32(out, ref, what="", tol=TOL_F32_MAXABS):
    out = np.asarray(out, np.float32).ravel()
    ref = np.asarray(ref, np.float32).ravel()
    err = float(np.abs(out - ref).max())
    assert np.all(np.isfinite(out)), f"{what}: non-finite output"
    assert err <= tol, f"{what}: max-abs {err:.3g} > {tol}"
    return err
