"""Shared helpers for the GPU parity tests (numpy <-> CUDA tensors)."""
import numpy as np
import torch


def dev(a: np.ndarray) -> torch.Tensor:
    """numpy array -> CUDA tensor with the same bytes."""
    a = np.ascontiguousarray(a)
    view = {1: np.uint8, 2: np.int16, 4: np.int32, 8: np.int64}[a.dtype.itemsize]
    if a.dtype.kind == "f" and a.dtype.itemsize == 4:
        return torch.from_numpy(a).cuda()
    return torch.from_numpy(a.view(view) if a.dtype.itemsize > 1 else a.view(np.uint8)).cuda()


def host(t: torch.Tensor, dtype) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy().view(dtype).copy()


def h16(signs=None) -> np.ndarray:
    from oracle import oracle
    i = np.arange(16)
    par = np.array([[bin(a & b).count("1") & 1 for b in i] for a in i])
    h = np.where(par == 0, 0.25, -0.25).astype(np.float32)
    if signs is not None:
        h = h * np.asarray(signs, np.float32)[None, :]
    return oracle.f32_to_bf16(h)


def activations(rng, k: int, outlier_frac: float = 0.001, outlier_scale: float = 50.0):
    """N(0,1) with a fraction of entries scaled by `outlier_scale`, as bf16 bits
    (the BASELINE configs' value distribution)."""
    from oracle import oracle
    x = rng.standard_normal(k).astype(np.float32)
    if outlier_frac > 0:
        idx = rng.random(k) < outlier_frac
        x[idx] *= outlier_scale
    return oracle.f32_to_bf16(x)


def fp4_step_diff(orc, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Per-element |decode(a) - decode(b)| in units of the larger code's grid step."""
    da = orc.e2m1_decode(orc.unpack_nibbles(a)).astype(np.float64)
    db = orc.e2m1_decode(orc.unpack_nibbles(b)).astype(np.float64)
    return np.abs(da - db)
