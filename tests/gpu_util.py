"""Helpers shared by the GPU tests: numpy <-> torch, bf16 bits."""
import numpy as np
import torch


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bf16_bits_of(values: np.ndarray) -> np.ndarray:
    """The bf16 bit pattern of float32 values that bf16 holds exactly."""
    return (np.ascontiguousarray(values, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
