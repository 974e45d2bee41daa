"""ctypes binding of libtextsift_cuda.so (include/textsift_cuda.h).

The library is loaded from this package directory; if it is missing the
import fails loudly -- there is no CPU fallback for the forward pass.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtextsift_cuda.so")

TS_OK = 0
TS_ERR_ARG = -1
TS_ERR_STATE = -2
TS_ERR_CUDA = -3
TS_ERR_UNSUPPORTED = -4
TS_ERR_DEVICE = -5

TS_DTYPE_U8, TS_DTYPE_F16, TS_DTYPE_F32, TS_DTYPE_I32 = 0, 1, 2, 3
TS_MODE_FAST, TS_MODE_EXACT = 0, 1
PHASES = ("expert_gate_up", "expert_down", "qkv", "attention", "o_proj", "router", "other")

P = ctypes.c_void_p
U32 = ctypes.c_uint32
I32 = ctypes.c_int32


class Cfg(ctypes.Structure):
    """Mirror of ts_cuda_cfg."""
    _fields_ = [("device", I32),
                ("vocab", U32), ("d_model", U32), ("n_layers", U32), ("n_heads", U32),
                ("n_kv_heads", U32), ("head_dim", U32), ("window", U32),
                ("d_ff", U32), ("n_experts", U32), ("top_k", U32), ("n_classes", U32),
                ("eps", ctypes.c_float),
                ("rope_theta", ctypes.c_double), ("rope_factor", ctypes.c_double),
                ("rope_original_max_pos", ctypes.c_double), ("rope_beta_fast", ctypes.c_double),
                ("rope_beta_slow", ctypes.c_double),
                ("max_tokens", U32), ("max_seq_len", U32), ("mode", I32)]


class TextsiftCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"textsift_cuda error {code}: {msg}")
        self.code = code


_lib = None

# (name, restype, argtypes) for every function of include/textsift_cuda.h
SIGNATURES = [
    ("ts_cuda_abi_version", ctypes.c_int, []),
    ("ts_cuda_default_cfg", None, [ctypes.POINTER(Cfg)]),
    ("ts_cuda_create", P, [ctypes.POINTER(Cfg), ctypes.c_char_p, ctypes.c_size_t]),
    ("ts_cuda_load_tensor", ctypes.c_int, [P, ctypes.c_char_p, I32, ctypes.POINTER(ctypes.c_int64), I32, P,
                                           ctypes.c_size_t]),
    ("ts_cuda_load_onnx", ctypes.c_int, [P, P, ctypes.c_size_t, P, ctypes.c_size_t, P, ctypes.c_size_t]),
    ("ts_cuda_onnx_tensor_info", ctypes.c_int, [P, ctypes.c_size_t, ctypes.c_char_p, P, P, P, P, P, P]),
    ("ts_cuda_finalize", ctypes.c_int, [P]),
    ("ts_cuda_set_mode", ctypes.c_int, [P, I32]),
    ("ts_cuda_forward", ctypes.c_int, [P, P, P, U32, P]),
    ("ts_cuda_forward_packed", ctypes.c_int, [P, P, P, P, U32, P]),
    ("ts_cuda_forward_packed_begin", ctypes.c_int, [P, P, P, P, U32, U32]),
    ("ts_cuda_forward_packed_end", ctypes.c_int, [P, U32, P]),
    ("ts_cuda_forward_packed_device", ctypes.c_int, [P, P, P, P, U32, P, P]),
    ("ts_cuda_forward_packed_tags", ctypes.c_int, [P, P, P, P, U32, P, P]),
    ("ts_cuda_forward_trace", ctypes.c_int, [P, P, P, P, U32, P, P]),
    ("ts_cuda_check", ctypes.c_int, [P, P]),
    ("ts_cuda_device_name", ctypes.c_char_p, [P]),
    ("ts_cuda_profile", ctypes.c_int, [P, I32]),
    ("ts_cuda_profile_read", ctypes.c_int, [P, P, P, P, P]),
    ("ts_cuda_last_error", ctypes.c_char_p, []),
    ("ts_cuda_destroy", None, [P]),
    ("ts_cuda_op_gather_bq", ctypes.c_int, [P, P, P, P, P, U32, U32, U32, P]),
    ("ts_cuda_op_rmsnorm", ctypes.c_int, [P, P, P, P, P, U32, U32, ctypes.c_float, P]),
    ("ts_cuda_w4_create", P, [I32, P, P, P, P, U32, U32, U32, ctypes.c_char_p, ctypes.c_size_t]),
    ("ts_cuda_w4_destroy", None, [P]),
    ("ts_cuda_op_dequant", ctypes.c_int, [P, U32, P, P]),
    ("ts_cuda_op_matmul_nbits", ctypes.c_int, [P, U32, P, I32, P, I32, U32, I32, P]),
    ("ts_cuda_op_router_topk", ctypes.c_int, [P, U32, P, P, P, U32, P]),
    ("ts_cuda_op_moe", ctypes.c_int, [P, U32, P, P, P, P, U32, P]),
    ("ts_cuda_op_banded_attention", ctypes.c_int, [P, P, P, P, P, P, U32, U32, U32, U32, U32, P, U32, I32, P]),
    ("ts_cuda_op_viterbi", ctypes.c_int, [P, P, U32, P, P, P]),
    ("ts_cuda_op_banded_attention_noalloc", ctypes.c_int, [P, P, P, P, P, P, U32, U32, U32, U32, U32, P, U32, I32,
                                                           P]),
    ("ts_cuda_rope_tables", ctypes.c_int, [P, U32, P, P]),
    ("ts_cuda_op_attention", ctypes.c_int, [P, P, P, P, P, P, P, P, U32, P]),
    ("ts_cuda_op_rope", ctypes.c_int, [P, P, P, P, P, U32, U32, U32, P]),
    ("ts_cuda_op_qkv_rope", ctypes.c_int, [P, U32, P, P, U32, P, P, P, P]),
    ("ts_cuda_op_router_addnorm", ctypes.c_int, [P, U32, P, P, P, P, P, U32, P]),
    ("ts_cuda_ep_unique_id", ctypes.c_size_t, [P, ctypes.c_size_t]),
    ("ts_cuda_ep_init", ctypes.c_int, [P, I32, I32, P, ctypes.c_size_t]),
    ("ts_cuda_ep_plan", ctypes.c_int, [P, P, I32, I32, I32, P, P, P, U32, P]),
    ("ts_cuda_selftest_wait_timeout", ctypes.c_int, [P, U32, P, P]),
    # host tokenizer
    ("ts_tok_create", P, [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]),
    ("ts_tok_destroy", None, [P]),
    ("ts_tok_vocab_size", U32, [P]),
    ("ts_tok_encode", ctypes.c_int, [P, ctypes.c_char_p, ctypes.c_size_t, P, P, P, ctypes.c_size_t, P]),
    ("ts_tok_encode_batch", ctypes.c_int, [P, P, P, U32, U32, P, P, P, ctypes.c_size_t, P]),
    ("ts_tok_decode", ctypes.c_int, [P, P, ctypes.c_size_t, P, ctypes.c_size_t, P]),
]


def lib():
    """Load libtextsift_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m textsift_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().ts_cuda_last_error() or b"").decode(errors="replace")


def check(rc: int) -> None:
    if rc != TS_OK:
        raise TextsiftCudaError(rc, last_error())


def default_cfg() -> Cfg:
    c = Cfg()
    lib().ts_cuda_default_cfg(ctypes.byref(c))
    return c
