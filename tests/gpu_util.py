"""Helpers for the GPU parity tests: device buffers via torch (plumbing only)
and tolerance reporting."""
import numpy as np

_VIEW = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32, np.dtype(np.uint8): np.uint8,
         np.dtype(np.int32): np.int32, np.dtype(np.float32): np.float32, np.dtype(np.int16): np.int16}


def dev(a: np.ndarray):
    import torch
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(_VIEW[a.dtype])).cuda()


def empty(shape, dtype):
    import torch
    tdt = {np.uint16: torch.int16, np.float32: torch.float32, np.int32: torch.int32, np.uint8: torch.uint8}[dtype]
    return torch.empty(shape, dtype=tdt, device="cuda")


def host(t, dtype):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy().view(dtype)


def ptr(t):
    return t.data_ptr()


def stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def f16(bits):
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float64)


def ulp_diff(a_bits, e_bits):
    a, e = f16(a_bits), f16(e_bits)
    mag = np.maximum(np.abs(e), 2.0 ** -14)
    return np.abs(a - e) / 2.0 ** (np.floor(np.log2(mag)) - 10)
