"""Helpers to read the committed golden fixtures."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def from_bits16(a: np.ndarray) -> torch.Tensor:
    """bf16 bit patterns (stored as int16) -> fp32 tensor."""
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).float()
