"""Helpers shared by the tests: conversions between torch tensors and the oracle's numpy arrays."""
import os

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def f32(t):
    """Any float tensor -> float32 numpy (exact widening for bf16/fp16)."""
    return t.detach().float().cpu().numpy()


def bits16(t):
    """bf16 tensor -> uint16 numpy bit patterns."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def u8(t):
    """int8 / float8 tensor -> uint8 numpy bytes."""
    return t.detach().contiguous().cpu().view(torch.uint8).numpy()


def bf16_from_bits(b, device=None):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).to(device)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_randn(*shape, scale=1.0, gen=None, device="cpu"):
    return (torch.randn(*shape, generator=gen) * scale).to(torch.bfloat16).to(device)
