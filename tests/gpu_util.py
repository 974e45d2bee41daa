"""Helpers for the GPU parity tests: device buffers via torch (plumbing only)
and tolerance reporting."""
import ctypes

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


def rand_w4(r, E, N, K, zp_random=True, scale_range=(1e-3, 1e-2)):
    """Random MatMulNBits weights [E, N, K]: uint4 pairs, fp16 scales per
    32-block, zero points (random or the constant 8), fp16 bias."""
    int4 = r.integers(0, 256, size=(E, N, K // 2), dtype=np.uint8)
    sc = r.uniform(*scale_range, size=(E, N, K // 32)).astype(np.float16).view(np.uint16)
    zb = (K // 32 + 1) // 2
    zp = r.integers(0, 256, size=(E, N, zb), dtype=np.uint8) if zp_random else np.full((E, N, zb), 0x88, np.uint8)
    bias = r.normal(0, 0.05, size=(E, N)).astype(np.float16).view(np.uint16)
    return int4, sc, zp, bias


def w4_handle(L, int4, sc, zp, bias):
    """A ts_cuda_w4 weight handle on device 0 (caller destroys it)."""
    E, N, K2 = int4.shape
    err = ctypes.create_string_buffer(512)
    h = L.ts_cuda_w4_create(0, int4.ctypes.data, sc.ctypes.data, zp.ctypes.data if zp is not None else None,
                            bias.ctypes.data, E, N, K2 * 2, err, 512)
    assert h, err.value
    return h
