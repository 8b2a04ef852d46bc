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


def same_up_to_sum_order(got, want, rounded: bool) -> bool:
    """Equal up to the order of the fp32 sums. Stream-K cuts a tile's k range
    by the launch's tile count, so a weight launched alone or in a group, or
    a call cut into row chunks, may round its last bits differently: fp32
    outputs within 1e-5 of the largest value, bf16-rounded outputs within one
    bf16 step of each value."""
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    if rounded:
        return bool(np.all(np.abs(g - w) <= np.abs(w) * 2.0 ** -7))
    return bool(np.max(np.abs(g - w)) <= 1e-5 * max(np.max(np.abs(w)), 1e-30))
