"""Weight upload from the model's ONNX files (ts_cuda_load_onnx), the addon's
counterpart of loadOnnxWeights (packages/textsift/src/browser/backends/
wasm.ts:328-453), on a synthetic model written in the real model's naming
(tests/onnx_fixture.py).

CPU: the protobuf reader (ts_cuda_onnx_tensor_info) finds every initializer
with its type, dims and bytes, inline or external, packed or unpacked dims.
GPU: a backend loaded from the ONNX files computes bit-identical logits to one
loaded tensor by tensor; missing or out-of-range tensors fail with a message.
"""
import ctypes

import numpy as np
import pytest

from onnx_fixture import initializers, write_model


@pytest.fixture(scope="module")
def model():
    from textsift_b200 import make_weights, small_config
    cfg = small_config(n_layers=2, vocab=512, n_experts=16)
    w = make_weights(cfg, seed=41, bias_std=0.03, sink_range=1.0)
    return cfg, w


def _info(L, graph, name):
    dt, nd, ext = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    off, nb = ctypes.c_uint64(), ctypes.c_uint64()
    dims = (ctypes.c_int64 * 8)()
    g = np.frombuffer(graph, np.uint8)
    rc = L.ts_cuda_onnx_tensor_info(g.ctypes.data, g.size, name.encode(), ctypes.byref(dt), dims, ctypes.byref(nd),
                                    ctypes.byref(ext), ctypes.byref(off), ctypes.byref(nb))
    return rc, dt.value, tuple(dims[i] for i in range(nd.value)), bool(ext.value), off.value, nb.value


@pytest.mark.parametrize("packed", [True, False])
def test_reader_finds_every_initializer(cuda_lib, model, packed):
    cfg, w = model
    graph, ext, where = write_model(w, cfg, packed_dims=packed)
    for name, arr, dtype, dims in initializers(w, cfg):
        rc, dt, got_dims, is_ext, off, nb = _info(cuda_lib, graph, name)
        assert rc == 0 and dt == dtype and got_dims == tuple(dims), name
        assert is_ext == where[name][0] and nb == arr.nbytes
        blob = ext[off:off + nb] if is_ext else graph[off:off + nb]
        assert blob == arr.tobytes(), name
    assert _info(cuda_lib, graph, "no.such.tensor")[0] == -1
    assert _info(cuda_lib, b"\xff\xff\xff", "x")[0] == -1      # truncated varint
    assert _info(cuda_lib, graph[:len(graph) // 2], "model_embed_tokens_weight_quant")[0] == -1


@pytest.mark.gpu
def test_onnx_backend_matches_tensor_backend(cuda_lib, model):
    from textsift_b200 import CudaBackend
    cfg, w = model
    graph, ext, _ = write_model(w, cfg)
    ref = CudaBackend(w, cfg, max_tokens=2048, max_seq_len=2048)
    onx = CudaBackend.from_onnx(graph, ext, cfg, max_tokens=2048, max_seq_len=2048)
    try:
        ref.warmup()
        onx.warmup()
        r = np.random.Generator(np.random.PCG64(42))
        chunks = [r.integers(0, cfg["vocab"], size=n).astype(np.int32) for n in (200, 31, 600)]
        for mode in (0, 1):
            ref.set_mode(mode)
            onx.set_mode(mode)
            for a, b in zip(ref.forward_packed(chunks), onx.forward_packed(chunks)):
                assert np.array_equal(a.data.view(np.uint32), b.data.view(np.uint32))
    finally:
        ref.dispose()
        onx.dispose()


@pytest.mark.gpu
def test_onnx_load_errors(cuda_lib, model):
    from textsift_b200 import CudaBackend, TextsiftCudaError
    cfg, w = model
    graph, ext, _ = write_model(w, cfg, drop="model.layers.1.attn.sinks")
    b = CudaBackend.from_onnx(graph, ext, cfg, max_tokens=1024, max_seq_len=1024)
    with pytest.raises(TextsiftCudaError, match="model.layers.1.attn.sinks"):
        b.warmup()
    b.dispose()
    graph, ext, _ = write_model(w, cfg)
    b = CudaBackend.from_onnx(graph, ext[: len(ext) // 2], cfg, max_tokens=1024, max_seq_len=1024)
    with pytest.raises(TextsiftCudaError, match="external range"):
        b.warmup()
    b.dispose()
