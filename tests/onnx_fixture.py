"""A synthetic onnx/model_q4f16.onnx (+ model_q4f16.onnx_data) holding
textsift_b200.make_weights tensors under the initializer names and storage
types textsift's loader reads (packages/textsift/src/browser/backends/
wasm.ts:328-453): router scales and bias as f32, sinks as f32 [1, Hq, 1, 1],
no expert zero points and no classifier bias (the loader synthesises both).
Tensors of ext_threshold bytes or more go to the external-data file.

A minimal protobuf writer; ONNX field numbers from onnx.proto (ModelProto:
ir_version 1, graph 7; GraphProto: name 2, initializer 5; TensorProto: dims 1,
data_type 2, name 8, raw_data 9, external_data 13, data_location 14;
StringStringEntryProto: key 1, value 2).
"""
import numpy as np

ONNX_FLOAT, ONNX_UINT8, ONNX_FLOAT16 = 1, 2, 10


def _varint(v: int) -> bytes:
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _ld(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _vi(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v)


def tensor_proto(name, data: bytes, dtype, dims, external=None, packed_dims=True) -> bytes:
    out = _ld(8, name.encode()) + _vi(2, dtype)
    if packed_dims:
        out += _ld(1, b"".join(_varint(int(d)) for d in dims))
    else:
        out += b"".join(_vi(1, int(d)) for d in dims)
    if external is None:
        out += _ld(9, data)
    else:
        off, ln = external
        for k, v in (("location", "model_q4f16.onnx_data"), ("offset", str(off)), ("length", str(ln))):
            out += _ld(13, _ld(1, k.encode()) + _ld(2, v.encode()))
        out += _vi(14, 1)
    return out


def _widen(bits) -> np.ndarray:
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


def initializers(w: dict, cfg: dict):
    """(onnx name, array, onnx data type, dims) in the model's naming."""
    nL = cfg["n_layers"]
    out = [("model_embed_tokens_weight_quant", w["embed.int4"], ONNX_UINT8),
           ("model_embed_tokens_weight_scales", w["embed.scales"], ONNX_FLOAT16),
           ("model_embed_tokens_weight_zp", w["embed.zp"], ONNX_UINT8),
           (f"model.layers.{nL}.final_norm_layernorm.weight", w["final_norm"], ONNX_FLOAT16),
           ("model_score_MatMul_weight_quant", w["score.int4"], ONNX_UINT8),
           ("model_score_MatMul_weight_scales", w["score.scales"], ONNX_FLOAT16),
           ("model_score_MatMul_weight_zp", w["score.zp"], ONNX_UINT8)]
    assert not np.any(w["score.bias"]), "the ONNX graph has no classifier bias"
    for L in range(nL):
        p = f"layers.{L}."
        for n in ("input_layernorm", "post_attention_layernorm"):
            out.append((f"model.layers.{L}.{n}.weight", w[p + n], ONNX_FLOAT16))
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            qb = f"model_layers_{L}_attn_{proj}_MatMul"
            out += [(qb + "_weight_quant", w[f"{p}attn.{proj}.int4"], ONNX_UINT8),
                    (qb + "_weight_scales", w[f"{p}attn.{proj}.scales"], ONNX_FLOAT16),
                    (qb + "_weight_zp", w[f"{p}attn.{proj}.zp"], ONNX_UINT8),
                    (f"model.layers.{L}.attn.{proj}.Add.bias", w[f"{p}attn.{proj}.bias"], ONNX_FLOAT16)]
        sinks = np.asarray(w[p + "attn.sinks"], np.float32)
        out.append((f"model.layers.{L}.attn.sinks", sinks.reshape(1, -1, 1, 1), ONNX_FLOAT))
        rb = f"/model/layers_{L}/moe/router/MatMul"
        out += [(rb + "_weight_fp32_quant", w[p + "router.int4"], ONNX_UINT8),
                (rb + "_weight_fp32_scales", _widen(w[p + "router.scales"]).reshape(w[p + "router.scales"].shape),
                 ONNX_FLOAT),
                (rb + "_weight_fp32_zp", w[p + "router.zp"], ONNX_UINT8),
                (f"/model/layers.{L}/moe/router/Add.bias_fp32", _widen(w[p + "router.bias"]), ONNX_FLOAT)]
        for proj, ours in (("gate_up_proj", "gate_up"), ("down_proj", "down")):
            eb = f"model_layers_{L}_moe_experts_{proj}"
            assert np.all(w[f"{p}experts.{ours}.zp"] == 0x88), "the ONNX graph has no expert zero points"
            out += [(eb + "_weight_quant", w[f"{p}experts.{ours}.int4"], ONNX_UINT8),
                    (eb + "_weight_scales", w[f"{p}experts.{ours}.scales"], ONNX_FLOAT16),
                    (f"model.layers.{L}.moe.experts.{proj}.bias", w[f"{p}experts.{ours}.bias"], ONNX_FLOAT16)]
    return [(n, np.ascontiguousarray(a), t, np.asarray(a).shape) for n, a, t in out]


def write_model(w: dict, cfg: dict, ext_threshold: int = 4096, packed_dims: bool = True, drop: str | None = None):
    """(graph bytes, external-data bytes, {name: (external, offset, nbytes)})."""
    graph = b""
    ext = bytearray()
    where = {}
    for name, arr, dt, dims in initializers(w, cfg):
        if name == drop:
            continue
        data = arr.tobytes()
        if len(data) >= ext_threshold:
            off = len(ext)
            ext += data
            ext += b"\0" * ((-len(ext)) % 64)  # the real file aligns tensors too
            graph += _ld(5, tensor_proto(name, data, dt, dims, (off, len(data)), packed_dims))
            where[name] = (True, off, len(data))
        else:
            graph += _ld(5, tensor_proto(name, data, dt, dims, None, packed_dims))
            where[name] = (False, None, len(data))
    model = _vi(1, 8) + _ld(7, _ld(2, b"textsift_b200 synthetic") + graph)
    return bytes(model), bytes(ext), where
