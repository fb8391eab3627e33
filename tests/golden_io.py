"""Loading of the golden fixtures in tests/golden/ (written by make_golden.py)."""

from pathlib import Path

import numpy as np
import torch

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def names(prefix=""):
    return sorted(p.stem for p in GOLDEN_DIR.glob(f"{prefix}*.npz"))


def load(name):
    with np.load(GOLDEN_DIR / f"{name}.npz") as data:
        return {key: data[key] for key in data.files}


def tensor(array, device="cpu"):
    return torch.from_numpy(np.ascontiguousarray(array)).to(device)
