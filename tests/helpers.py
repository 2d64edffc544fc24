"""Test helpers: host<->device copies of the bit-pattern arrays and the
error metrics the parity tests use."""
import numpy as np

TORCH_DT = {"f32": "float32", "f16": "float16", "bf16": "bfloat16", "i8": "int8", "i32": "int32"}
CUDA_T = {"f32": 0, "f16": 2, "i8": 3, "i32": 10, "bf16": 14}


def to_dev(a: np.ndarray, kind: str, pad: int = 0, fill: int = 0):
    """Copies host array (bit patterns for 16-bit kinds) to a flat device
    tensor of the given kind, with `pad` extra trailing canary elements."""
    import torch
    a = np.ascontiguousarray(a).reshape(-1)
    if kind in ("f16", "bf16"):
        t = torch.from_numpy(a.view(np.int16).copy())
    else:
        t = torch.from_numpy(a.copy())
    if pad:
        extra = torch.full((pad,), fill, dtype=t.dtype)
        t = torch.cat([t, extra])
    t = t.cuda()
    if kind in ("f16", "bf16"):
        t = t.view(getattr(torch, TORCH_DT[kind]))
    return t


def from_dev(t, kind: str) -> np.ndarray:
    import torch
    t = t.detach().cpu()
    if kind in ("f16", "bf16"):
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def as_float(a: np.ndarray, kind: str) -> np.ndarray:
    from zlift_b200 import inputs
    if kind in ("f16", "bf16"):
        return inputs.bits_to_float(a, kind).astype(np.float64)
    return a.astype(np.float64)


def normwise(x: np.ndarray, ref: np.ndarray) -> float:
    """max |x - ref| / max |ref| over the whole tensor."""
    den = float(np.max(np.abs(ref))) if ref.size else 0.0
    num = float(np.max(np.abs(x - ref))) if ref.size else 0.0
    return num / den if den > 0 else num
