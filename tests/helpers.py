"""Conversions between numpy golden arrays and torch device tensors for the tests."""

from __future__ import annotations

import numpy as np
import torch


def bf16_from_bits(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def bits_from_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def e4m3_from_bits(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits)).view(torch.float8_e4m3fn).to(device)


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))
