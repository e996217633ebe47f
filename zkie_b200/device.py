"""Device-memory plumbing: torch owns the HBM buffers and streams, the
kernels come from libzkie_b200.so.  Field elements are torch.uint64 tensors.
"""
import numpy as np
import torch

P = 0xFFFFFFFF00000001


def device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("zkie_b200 needs a CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def to_dev(a) -> torch.Tensor:
    """numpy / sequence / tensor of u64 -> contiguous torch.uint64 on the current GPU."""
    if isinstance(a, torch.Tensor):
        t = a if a.dtype == torch.uint64 else a.to(torch.uint64)
        return t.to(device()).contiguous()
    arr = np.ascontiguousarray(np.asarray(a, dtype=np.uint64))
    return torch.from_numpy(arr).to(device())


def empty(n, *shape) -> torch.Tensor:
    shape = (n,) + shape if shape else (n,)
    return torch.empty(shape, dtype=torch.uint64, device=device())


def zeros(n) -> torch.Tensor:
    return torch.zeros(n, dtype=torch.uint64, device=device())


def ptr(t: torch.Tensor) -> int:
    assert t.is_cuda and t.is_contiguous() and t.dtype == torch.uint64
    return t.data_ptr()


def stream_handle(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def to_host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()
