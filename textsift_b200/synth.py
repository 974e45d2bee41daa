"""Seeded synthetic q4f16 weights for the privacy-filter architecture.

The real openai/privacy-filter weights are not available offline, so every
benchmark and parity case uses weights drawn from a seed with the shapes and
distributions the benchmark configuration names: uint4 nibbles uniform in
0..15, block 32 along K, fp16 scales uniform in [1e-3, 1e-2], zero point 8
(0x88 bytes), norm weights 1.0, biases and sinks 0 unless asked otherwise.
Tensor names and layouts are those loadOnnxWeights produces
(packages/textsift/src/browser/backends/wasm.ts:358-446).
"""
from __future__ import annotations

import numpy as np

PF_CONFIG = dict(vocab=200064, d_model=640, n_layers=8, n_heads=14, n_kv_heads=2, head_dim=64,
                 window=128, d_ff=640, n_experts=128, top_k=4, n_classes=33, eps=1e-5,
                 rope=dict(theta=150000.0, factor=32.0, orig=4096.0, beta_fast=32.0, beta_slow=1.0))


def small_config(**over) -> dict:
    """A reduced model for fast parity tests (real hidden sizes, fewer layers,
    a small vocabulary)."""
    c = dict(PF_CONFIG)
    c.update(vocab=4096, n_layers=2)
    c.update(over)
    return c


def _fp16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x.astype(np.float16)).view(np.uint16)


def _i4(rng, E, N, K, scale_lo, scale_hi, zp_mode, bias_std):
    shape = (N,) if E is None else (E, N)
    e = 1 if E is None else E
    int4 = rng.integers(0, 256, size=(e * N * K // 2,), dtype=np.uint8).reshape(*shape, K // 2)
    sc = _fp16_bits(rng.uniform(scale_lo, scale_hi, size=(e * N * (K // 32),)).astype(np.float32))
    sc = sc.reshape(*shape, K // 32)
    zb = (K // 32 + 1) // 2
    if zp_mode == "const8":
        zp = np.full((*shape, zb), 0x88, dtype=np.uint8)
    else:
        zp = rng.integers(0, 256, size=(e * N * zb,), dtype=np.uint8).reshape(*shape, zb)
    if bias_std > 0:
        bias = _fp16_bits(rng.normal(0.0, bias_std, size=(e * N,)).astype(np.float32)).reshape(shape)
    else:
        bias = np.zeros(shape, dtype=np.uint16)
    return int4, sc, zp, bias


def make_weights(cfg: dict, seed: int = 0, bias_std: float = 0.0, sink_range: float = 0.0,
                 zp_mode: str = "const8", scale_range=(1e-3, 1e-2), router_bias=None) -> dict:
    """Name -> numpy array (uint8 / fp16 bits as uint16 / float32)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    D, V, C, E, F = cfg["d_model"], cfg["vocab"], cfg["n_classes"], cfg["n_experts"], cfg["d_ff"]
    Hq, Hkv, hd = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    lo, hi = scale_range
    w: dict[str, np.ndarray] = {}
    i4, sc, zp, _ = _i4(rng, None, V, D, lo, hi, zp_mode, 0.0)
    w["embed.int4"], w["embed.scales"], w["embed.zp"] = i4, sc, zp
    w["final_norm"] = np.full((D,), 0x3C00, dtype=np.uint16)
    i4, sc, zp, _ = _i4(rng, None, C, D, lo, hi, zp_mode, 0.0)
    # wasm.ts:377: the classifier has no bias in the ONNX; the loader adds zeros
    w["score.int4"], w["score.scales"], w["score.zp"] = i4, sc, zp
    w["score.bias"] = np.zeros((C,), dtype=np.uint16)
    for L in range(cfg["n_layers"]):
        p = f"layers.{L}."
        w[p + "input_layernorm"] = np.full((D,), 0x3C00, dtype=np.uint16)
        w[p + "post_attention_layernorm"] = np.full((D,), 0x3C00, dtype=np.uint16)
        for name, N, K in (("q_proj", Hq * hd, D), ("k_proj", Hkv * hd, D), ("v_proj", Hkv * hd, D),
                           ("o_proj", D, Hq * hd)):
            i4, sc, zp, b = _i4(rng, None, N, K, lo, hi, zp_mode, bias_std)
            for f, a in zip(("int4", "scales", "zp", "bias"), (i4, sc, zp, b)):
                w[f"{p}attn.{name}.{f}"] = a
        if sink_range > 0:
            w[p + "attn.sinks"] = rng.uniform(-sink_range, sink_range, size=(Hq,)).astype(np.float32)
        else:
            w[p + "attn.sinks"] = np.zeros((Hq,), dtype=np.float32)
        i4, sc, zp, b = _i4(rng, None, E, D, lo, hi, zp_mode, bias_std)
        if router_bias is not None:
            b = _fp16_bits(np.asarray(router_bias, dtype=np.float32))
        for f, a in zip(("int4", "scales", "zp", "bias"), (i4, sc, zp, b)):
            w[f"{p}router.{f}"] = a
        for name, N, K in (("gate_up", 2 * F, D), ("down", D, F)):
            i4, sc, zp, b = _i4(rng, E, N, K, lo, hi, zp_mode, bias_std)
            for f, a in zip(("int4", "scales", "zp", "bias"), (i4, sc, zp, b)):
                w[f"{p}experts.{name}.{f}"] = a
    return w


def quantize_int4(wf: np.ndarray):
    """Asymmetric block-32 uint4 quantisation of an f32 [N, K] matrix into
    (int4 [N, K/2], fp16 scales [N, K/32], zp [N, ceil(K/64)]) -- used to turn
    the benchmark's 'router weights fp16 N(0, 0.02)' into the int4 router the
    reference model actually has."""
    N, K = wf.shape
    nb = K // 32
    blk = wf.reshape(N, nb, 32).astype(np.float32)
    mn, mx = blk.min(axis=2), blk.max(axis=2)
    scale = np.maximum((mx - mn) / 15.0, 1e-8).astype(np.float16).astype(np.float32)
    zpv = np.clip(np.rint(-mn / scale), 0, 15).astype(np.int32)
    q = np.clip(np.rint(blk / scale[:, :, None]) + zpv[:, :, None], 0, 15).astype(np.uint8).reshape(N, K)
    int4 = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    zb = (nb + 1) // 2
    zpad = np.zeros((N, zb * 2), dtype=np.uint8)
    zpad[:, :nb] = zpv
    zp = (zpad[:, 0::2] | (zpad[:, 1::2] << 4)).astype(np.uint8)
    return int4, _fp16_bits(scale), zp


def zipf_router_bias(n_experts: int, s: float, seed: int) -> np.ndarray:
    """bias_e = -s * ln(rank_e) over a seeded permutation of ranks 1..E."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ranks = rng.permutation(n_experts) + 1
    return (-s * np.log(ranks)).astype(np.float32)


def tensor_dtype(arr: np.ndarray) -> int:
    from .abi import TS_DTYPE_F16, TS_DTYPE_F32, TS_DTYPE_I32, TS_DTYPE_U8
    return {np.dtype(np.uint8): TS_DTYPE_U8, np.dtype(np.uint16): TS_DTYPE_F16,
            np.dtype(np.float32): TS_DTYPE_F32, np.dtype(np.int32): TS_DTYPE_I32}[arr.dtype]
