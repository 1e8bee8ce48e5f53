"""Helpers shared by the GPU tests (device transfer of bf16/u32 numpy arrays, metrics)."""
import numpy as np

from hyperion_b200.synth import bf16_bits_to_f32


def dev(a: np.ndarray):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    if a.dtype == np.float32:
        return torch.from_numpy(a).cuda()
    raise TypeError(a.dtype)


def host(t) -> np.ndarray:
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


def rel_l2(got_bits: np.ndarray, want_bits: np.ndarray) -> float:
    g = bf16_bits_to_f32(got_bits).astype(np.float64)
    w = bf16_bits_to_f32(want_bits).astype(np.float64)
    return float(np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30))


def max_ulp(got_bits: np.ndarray, want_bits: np.ndarray) -> int:
    """Largest distance in bf16 units in the last place (same-sign values)."""
    g = got_bits.astype(np.int32)
    w = want_bits.astype(np.int32)
    # map sign-magnitude to a monotone integer line
    g = np.where(g & 0x8000, -(g & 0x7FFF), g)
    w = np.where(w & 0x8000, -(w & 0x7FFF), w)
    return int(np.abs(g - w).max()) if g.size else 0


def within_one_ulp(got_bits: np.ndarray, want_bits: np.ndarray) -> float:
    """Fraction of elements within one bf16 ulp of the reference."""
    g = got_bits.astype(np.int32)
    w = want_bits.astype(np.int32)
    g = np.where(g & 0x8000, -(g & 0x7FFF), g)
    w = np.where(w & 0x8000, -(w & 0x7FFF), w)
    return float((np.abs(g - w) <= 1).mean())
