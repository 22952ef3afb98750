"""Small helpers shared by the tests (bit-pattern conversion, error metrics)."""
import numpy as np
import torch


def bf16_tensor(bits: np.ndarray, device=None) -> torch.Tensor:
    """uint16 bf16 bit patterns -> torch bf16 tensor."""
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t if device is None else t.to(device)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a, b) -> float:
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())
