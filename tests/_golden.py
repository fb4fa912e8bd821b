"""Readers for the golden fixtures under tests/golden (made by tests/golden/make_golden.py)."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def tensor(array: np.ndarray, dtype: str = "float32") -> torch.Tensor:
    if array.dtype == np.uint16:  # bf16 stored as its bit pattern
        return torch.from_numpy(array.astype(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(array))


def load(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as data:
        return {key: data[key] for key in data.files}


def ulysses_cases() -> list[str]:
    return sorted(p.name for p in GOLDEN.glob("ulysses_*.npz"))


def rope_cases() -> list[str]:
    return sorted(p.name for p in GOLDEN.glob("rope_*.npz"))


def narrow_cases() -> list[str]:
    return sorted(p.name for p in GOLDEN.glob("narrow_*.npz"))
