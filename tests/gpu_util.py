"""Helpers shared by the GPU parity tests (bf16 bit patterns <-> tensors)."""
import numpy as np
import torch


def to_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> numpy uint16 bit patterns."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b: np.ndarray, device="cuda") -> torch.Tensor:
    """numpy uint16 bit patterns -> bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint16).view(np.int16)).view(
        torch.bfloat16).to(device)


def seeded_bf16(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def seeded_f32(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * std
