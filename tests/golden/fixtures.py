"""Loader for the committed golden fixtures (made by make_golden.py)."""

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load(name: str) -> dict:
    with np.load(HERE / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
