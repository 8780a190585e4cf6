"""Shared test helpers (tolerances are written here, once)."""
import numpy as np

# per-output relative error <= 1e-3 for matvec,
# graded as |y - y64| / max(|y64|, 1e-3 * rms(y64)).
MATVEC_REL = 1e-3
# crates/soso-llm-api/tests/cuda_matvec.rs:85-92 (`cerca`): max |a-b| / (1+|b|) < 2e-4.
CERCA = 2e-4


def matvec_rel_err(y: np.ndarray, y64: np.ndarray) -> float:
    y64 = np.asarray(y64, dtype=np.float64)
    rms = float(np.sqrt(np.mean(y64 ** 2))) if y64.size else 0.0
    den = np.maximum(np.abs(y64), 1e-3 * rms)
    den = np.where(den == 0, 1.0, den)
    return float(np.max(np.abs(np.asarray(y, dtype=np.float64) - y64) / den)) if y64.size else 0.0


def assert_matvec_close(y, y64, what=""):
    e = matvec_rel_err(y, y64)
    assert e <= MATVEC_REL, f"{what}: max rel err {e:.3e} > {MATVEC_REL}"


def cerca(a, b, what=""):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    peor = float(np.max(np.abs(a - b) / (1.0 + np.abs(b)))) if a.size else 0.0
    assert peor < CERCA, f"{what}: error relativo maximo {peor}"
