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


def check_16bit(out, ref, what=""):
    out = np.asarray(out, np.float32).ravel()
    ref = np.asarray(ref, np.float32).ravel()
    err = float(np.abs(out - ref).max())
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
