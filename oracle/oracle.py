"""ctypes binding of the CPU oracle (oracle/_build/libts_oracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA backend and the
timed CPU baseline of bench.py.  Only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference legs import this module.  The
product path (textsift_b200) never imports it.

The C sources restate packages/textsift/src/zig/wasm_exports.zig,
zig/math.zig and browser/inference/*.ts of teamchong/textsift; see the
citations in ts_oracle_kernels.c and ts_oracle_model.c.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libts_oracle.so")
_lib = None

P = ctypes.c_void_p
U32 = ctypes.c_uint32
I32 = ctypes.c_int
F32 = ctypes.c_float


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class _RopeCfg(ctypes.Structure):
    _fields_ = [("head_dim", ctypes.c_uint32), ("theta", ctypes.c_double),
                ("factor", ctypes.c_double), ("original_max_pos", ctypes.c_double),
                ("beta_fast", ctypes.c_double), ("beta_slow", ctypes.c_double),
                ("truncate", ctypes.c_int)]


class _Cfg(ctypes.Structure):
    _fields_ = [("vocab", U32), ("d_model", U32), ("n_layers", U32), ("n_heads", U32),
                ("n_kv_heads", U32), ("head_dim", U32), ("window", U32), ("d_ff", U32),
                ("n_experts", U32), ("top_k", U32), ("n_classes", U32), ("eps", F32),
                ("rope", _RopeCfg)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.tso_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.tso_f16_to_f32.restype = F32
        L.tso_f32_to_f16.argtypes = [F32]
        L.tso_f32_to_f16.restype = ctypes.c_uint16
        L.tso_f32_to_bf16.argtypes = [F32]
        L.tso_f32_to_bf16.restype = ctypes.c_uint16
        L.tso_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.tso_bf16_to_f32.restype = F32
        L.tso_exp_approx.argtypes = [F32]
        L.tso_exp_approx.restype = F32
        L.tso_rms_norm.argtypes = [P, P, P, U32, U32, F32]
        L.tso_rms_norm_fp16_to_f32.argtypes = [P, P, P, U32, U32, F32]
        L.tso_add_rmsnorm_fp16_to_f32.argtypes = [P, P, P, P, P, U32, U32, F32]
        L.tso_topk_partial_f32.argtypes = [P, P, P, U32, U32, U32]
        L.tso_matmul_int4.argtypes = [I32, I32, P, P, P, P, P, P, U32, U32, U32]
        L.tso_matmul_int4_scalar.argtypes = [I32, I32, P, P, P, P, P, P, U32, U32, U32]
        L.tso_swiglu_clamp_f32.argtypes = [P, P, U32, U32]
        L.tso_softmax_f32.argtypes = [P, P, U32, U32]
        L.tso_add_fp16.argtypes = [P, P, P, U32]
        L.tso_gather_f32.argtypes = [P, P, P, U32, U32]
        L.tso_scatter_add_weighted_f32.argtypes = [P, P, P, P, U32, U32]
        L.tso_convert_fp16_to_f32.argtypes = [P, P, U32]
        L.tso_cast_f32_to_fp16_scaled.argtypes = [P, P, U32, F32]
        L.tso_banded_attention.argtypes = [P, P, P, P, P, P, U32, U32, U32, U32, U32, U32, U32]
        L.tso_rope_apply.argtypes = [P, P, P, U32, U32, U32]
        L.tso_embed_lookup_int4.argtypes = [P, P, P, P, P, U32, U32, U32]
        L.tso_dequant_int4.argtypes = [P, P, P, P, U32, U32]
        L.tso_build_rope_tables.argtypes = [ctypes.POINTER(_RopeCfg), U32, P, P]
        L.tso_model_create.argtypes = [ctypes.POINTER(_Cfg)]
        L.tso_model_create.restype = P
        L.tso_model_destroy.argtypes = [P]
        L.tso_model_set.argtypes = [P, ctypes.c_char_p, P, ctypes.c_size_t]
        L.tso_model_set.restype = I32
        L.tso_model_forward.argtypes = [P, P, P, U32, P, I32, P, P, P]
        L.tso_model_forward.restype = I32
        L.tso_model_forward_forced.argtypes = [P, P, P, U32, P, I32, P, P, P, P]
        L.tso_model_forward_forced.restype = I32
        L.tso_moe_forward.argtypes = [P, U32, P, U32, P, P, P, I32]
        L.tso_moe_forward.restype = I32
        L.tso_viterbi_tables.argtypes = [P, P, P]
        L.tso_viterbi.argtypes = [P, U32, P, P, P, P]
        L.tso_bioes_spans.argtypes = [P, U32, P, U32]
        L.tso_bioes_spans.restype = U32
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- scalar helpers
def f16_to_f32(bits: int) -> float:
    return lib().tso_f16_to_f32(int(bits))


def f32_to_f16(x: float) -> int:
    return lib().tso_f32_to_f16(float(x))


def f32_to_bf16(x: float) -> int:
    return lib().tso_f32_to_bf16(float(x))


def bf16_to_f32(b: int) -> float:
    return lib().tso_bf16_to_f32(int(b))


def f16_to_f32_array(bits: np.ndarray) -> np.ndarray:
    """Vector form of math.zig fp16ToF32 (the reference's activation decode)."""
    u = bits.astype(np.uint32)
    sign = (u & 0x8000) << 16
    rest = u & 0x7FFF
    biased = np.where(rest == 0, 0, (rest << 13) + (112 << 23)).astype(np.uint32)
    return (sign | biased).astype(np.uint32).view(np.float32)


# ---------------------------------------------------------------- kernels
def rms_norm(x16, gamma16, eps):
    x16 = _c(x16, np.uint16); T, D = x16.shape
    out = np.empty_like(x16)
    lib().tso_rms_norm(_p(x16), _p(_c(gamma16, np.uint16)), _p(out), T, D, eps)
    return out


def rms_norm_fp16_to_f32(x16, gamma16, eps):
    x16 = _c(x16, np.uint16); T, D = x16.shape
    out = np.empty((T, D), np.float32)
    lib().tso_rms_norm_fp16_to_f32(_p(x16), _p(_c(gamma16, np.uint16)), _p(out), T, D, eps)
    return out


def add_rmsnorm_fp16_to_f32(a16, b16, gamma16, eps):
    a16 = _c(a16, np.uint16); b16 = _c(b16, np.uint16); T, D = a16.shape
    s = np.empty_like(a16); n = np.empty((T, D), np.float32)
    lib().tso_add_rmsnorm_fp16_to_f32(_p(a16), _p(b16), _p(_c(gamma16, np.uint16)), _p(s), _p(n), T, D, eps)
    return s, n


def topk(x, k):
    x = _c(x, np.float32); R, C = x.shape
    idx = np.empty((R, k), np.int32); val = np.empty((R, k), np.float32)
    lib().tso_topk_partial_f32(_p(x), _p(idx), _p(val), R, C, k)
    return idx, val


def softmax(x):
    x = _c(x, np.float32); R, C = x.shape
    out = np.empty_like(x)
    lib().tso_softmax_f32(_p(x), _p(out), R, C)
    return out


def matmul_int4(x, w_int4, w_scales, w_zp, bias, out_f32: bool, scalar: bool = False):
    """y = x @ dequant(W).T + bias.  x: float32 (f32 path) or uint16 (fp16 bits)."""
    x_f32 = x.dtype == np.float32
    x = _c(x, np.float32 if x_f32 else np.uint16)
    T, D = x.shape
    N = w_int4.shape[0]
    out = np.empty((T, N), np.float32 if out_f32 else np.uint16)
    zp = None if w_zp is None else _c(w_zp, np.uint8)
    fn = lib().tso_matmul_int4_scalar if scalar else lib().tso_matmul_int4
    fn(int(x_f32), int(out_f32), _p(x), _p(_c(w_int4, np.uint8)),
                          _p(_c(w_scales, np.uint16)), _p(zp), _p(_c(bias, np.uint16)), _p(out), T, N, D)
    return out


def dequant_int4(w_int4, w_scales, w_zp, N, D):
    out = np.empty((N, D), np.uint16)
    zp = None if w_zp is None else _c(w_zp, np.uint8)
    lib().tso_dequant_int4(_p(_c(w_int4, np.uint8)), _p(_c(w_scales, np.uint16)), _p(zp), _p(out), N, D)
    return out


def swiglu_clamp(gate_up):
    gate_up = _c(gate_up, np.float32); T, D2 = gate_up.shape
    out = np.empty((T, D2 // 2), np.float32)
    lib().tso_swiglu_clamp_f32(_p(gate_up), _p(out), T, D2 // 2)
    return out


def add_fp16(a, b):
    a = _c(a, np.uint16); b = _c(b, np.uint16)
    out = np.empty_like(a)
    lib().tso_add_fp16(_p(a), _p(b), _p(out), a.size)
    return out


def convert_fp16_to_f32(src):
    src = _c(src, np.uint16); out = np.empty(src.shape, np.float32)
    lib().tso_convert_fp16_to_f32(_p(src), _p(out), src.size)
    return out


def cast_f32_to_fp16_scaled(src, scale):
    src = _c(src, np.float32); out = np.empty(src.shape, np.uint16)
    lib().tso_cast_f32_to_fp16_scaled(_p(src), _p(out), src.size, scale)
    return out


def banded_attention(q, k, v, sinks, mask, T, Hq, Hkv, hd, window, h0=0, h1=None):
    q = _c(q, np.uint16); k = _c(k, np.uint16); v = _c(v, np.uint16)
    out = np.zeros((T, Hq * hd), np.uint16)
    m = None if mask is None else _c(mask, np.uint8)
    lib().tso_banded_attention(_p(q), _p(k), _p(v), _p(_c(sinks, np.float32)), _p(m), _p(out),
                               T, Hq, Hkv, hd, window, h0, Hq if h1 is None else h1)
    return out


def rope_apply(qk, cos16, sin16, T, H, hd):
    qk = np.array(qk, dtype=np.uint16, copy=True, order="C")
    lib().tso_rope_apply(_p(qk), _p(_c(cos16, np.uint16)), _p(_c(sin16, np.uint16)), T, H, hd)
    return qk


def embed_lookup_int4(embed_int4, embed_scales, embed_zp, ids, V, D):
    ids = _c(ids, np.int32); T = ids.size
    out = np.empty((T, D), np.uint16)
    lib().tso_embed_lookup_int4(_p(_c(embed_int4, np.uint8)), _p(_c(embed_scales, np.uint16)),
                                _p(_c(embed_zp, np.uint8)), _p(ids), _p(out), T, V, D)
    return out


def exp_approx(x: float) -> float:
    return lib().tso_exp_approx(float(x))


ZERO_CALIBRATION = (0.0, 0.0, 0.0, 0.0, 0.0, 0.0)


def viterbi_tables(cal=ZERO_CALIBRATION):
    """browser/inference/viterbi.ts:155-225: (trans [to, from] f32[33,33], start f32[33])."""
    trans = np.zeros((33, 33), np.float32)
    start = np.zeros(33, np.float32)
    lib().tso_viterbi_tables(_p(np.asarray(cal, np.float32)), _p(trans), _p(start))
    return trans, start


def viterbi(logits, cal=ZERO_CALIBRATION):
    """browser/inference/viterbi.ts:75-145: BIOES tags u8[T] of logits f32[T,33]."""
    lg = _c(logits, np.float32).reshape(-1, 33)
    T = lg.shape[0]
    tags = np.zeros(T, np.uint8)
    alpha = np.zeros(max(T, 1) * 33, np.float32)
    back = np.zeros(max(T, 1) * 33, np.uint8)
    lib().tso_viterbi(_p(lg), T, _p(np.asarray(cal, np.float32)), _p(tags), _p(alpha), _p(back))
    return tags


def bioes_spans(tags):
    """browser/inference/spans.ts:29-104 at token level: [(first, last, label)]."""
    tg = _c(tags, np.uint8)
    cap = max(int(tg.size), 1)
    out = np.zeros((cap, 3), np.int32)
    n = lib().tso_bioes_spans(_p(tg), tg.size, _p(out), cap)
    return [tuple(int(v) for v in out[i]) for i in range(n)]


def rope_cfg(head_dim=64, theta=150000.0, factor=32.0, orig=4096.0, beta_fast=32.0,
             beta_slow=1.0, truncate=0):
    return _RopeCfg(head_dim, theta, factor, orig, beta_fast, beta_slow, truncate)


def rope_tables(T, cfg=None):
    cfg = cfg or rope_cfg()
    half = cfg.head_dim // 2
    c = np.empty((T, half), np.uint16); s = np.empty((T, half), np.uint16)
    lib().tso_build_rope_tables(ctypes.byref(cfg), T, _p(c), _p(s))
    return c, s


# ---------------------------------------------------------------- model
class OracleModel:
    """The reference forward (modelForward) over a dict of named tensors in
    the layout loadOnnxWeights produces (browser/backends/wasm.ts:328-453)."""

    def __init__(self, cfg: dict, tensors: dict):
        r = cfg.get("rope", {})
        c = _Cfg(cfg["vocab"], cfg["d_model"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
                 cfg["head_dim"], cfg["window"], cfg["d_ff"], cfg["n_experts"], cfg["top_k"],
                 cfg["n_classes"], cfg["eps"],
                 rope_cfg(cfg["head_dim"], r.get("theta", 150000.0), r.get("factor", 32.0),
                          r.get("orig", 4096.0), r.get("beta_fast", 32.0), r.get("beta_slow", 1.0), 0))
        self.cfg = cfg
        self._h = lib().tso_model_create(ctypes.byref(c))
        if not self._h:
            raise RuntimeError("tso_model_create failed")
        self._keep = {}
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr)
            self._keep[name] = a
            if lib().tso_model_set(self._h, name.encode(), _p(a), a.nbytes) != 0:
                raise KeyError(f"oracle: unknown tensor name {name!r}")

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.tso_model_destroy(h)
            self._h = None

    def forward(self, ids, mask=None, n_threads=1, trace=False, forced_topk=None):
        """Logits f32 [T, n_classes].  trace=True also returns per-layer
        residual streams, top-k experts and router inputs; forced_topk
        (i32 [n_layers, T, top_k]) imposes the expert choice of every layer."""
        ids = _c(ids, np.int32); T = ids.size
        c = self.cfg
        logits = np.empty((T, c["n_classes"]), np.float32)
        m = None if mask is None else _c(mask, np.uint8)
        ht = tk = nt = None
        if trace:
            ht = np.empty((c["n_layers"] + 1, T, c["d_model"]), np.uint16)
            tk = np.empty((c["n_layers"], T, c["top_k"]), np.int32)
            nt = np.empty((c["n_layers"], T, c["d_model"]), np.float32)
        fk = None if forced_topk is None else _c(forced_topk, np.int32)
        if fk is not None and fk.shape != (c["n_layers"], T, c["top_k"]):
            raise ValueError("forced_topk must be [n_layers, T, top_k]")
        rc = lib().tso_model_forward_forced(self._h, _p(ids), _p(m), T, _p(logits), n_threads,
                                            _p(ht), _p(tk), _p(nt), _p(fk))
        if rc != 0:
            raise RuntimeError(f"tso_model_forward failed: {rc}")
        if trace:
            return logits, {"hidden": ht, "topk": tk, "normed": nt}
        return logits

    def moe(self, layer, normed, n_threads=1):
        normed = _c(normed, np.float32); T = normed.shape[0]
        c = self.cfg
        out = np.empty((T, c["d_model"]), np.uint16)
        idx = np.empty((T, c["top_k"]), np.int32)
        w = np.empty((T, c["top_k"]), np.float32)
        rc = lib().tso_moe_forward(self._h, layer, _p(normed), T, _p(out), _p(idx), _p(w), n_threads)
        if rc != 0:
            raise RuntimeError("tso_moe_forward failed")
        return out, idx, w
