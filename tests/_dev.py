"""Device-buffer helpers for the GPU tests (torch is only the allocator)."""
import numpy as np
import torch

_NP2T = {np.int8: torch.int8, np.uint8: torch.uint8, np.int32: torch.int32,
         np.float32: torch.float32, np.uint16: torch.int16, np.int64: torch.int64,
         np.float16: torch.float16}


def to_dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


def empty(shape, dtype) -> torch.Tensor:
    return torch.empty(shape, dtype=_NP2T[np.dtype(dtype).type], device="cuda")


def zeros(shape, dtype) -> torch.Tensor:
    return torch.zeros(shape, dtype=_NP2T[np.dtype(dtype).type], device="cuda")


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()
