"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

import oracle as O
from deepseek_v32_gtx1650_b200 import _lib

DEV = "cuda"


def cuda(x: np.ndarray, dtype=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def bf16_from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(DEV)


def npy(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def f32_of(t: torch.Tensor) -> np.ndarray:
    """Exact fp32 image of an fp32/fp16/bf16 tensor (what the reference's x.float() gives)."""
    return t.detach().cpu().float().numpy()


def assert_no_device_error():
    code = _lib.device_status(torch.cuda.current_device())
    assert code == 0, f"kernel reported an internal wait timeout: {code:#x}"


def sample_rows(M: int, n: int = 48, seed: int = 0) -> np.ndarray:
    """A seeded sample of query / row indices that always includes the first and last rows."""
    rng = np.random.default_rng(seed)
    mid = rng.choice(np.arange(1, max(M - 1, 1)), size=min(n, max(M - 2, 0)), replace=False) if M > 2 else []
    return np.unique(np.concatenate([[0, M - 1], np.asarray(mid, dtype=np.int64)])).astype(np.int64)


rel_err = O.rel_err
