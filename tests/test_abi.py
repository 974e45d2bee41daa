"""CPU checks of the C-ABI boundary: the library builds for sm_100a, loads
without a GPU, and exports exactly what include/textsift_cuda.h declares."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "textsift_cuda.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ts_(?:cuda|tok)_\w+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("ts_cuda_create", "ts_cuda_load_tensor", "ts_cuda_finalize", "ts_cuda_forward",
                     "ts_cuda_forward_packed", "ts_cuda_device_name", "ts_cuda_last_error", "ts_cuda_destroy",
                     "ts_cuda_op_gather_bq", "ts_cuda_op_matmul_nbits", "ts_cuda_op_router_topk", "ts_cuda_op_moe",
                     "ts_cuda_op_banded_attention", "ts_cuda_op_rmsnorm", "ts_cuda_op_dequant"):
        assert required in names


def test_library_exports_every_declared_symbol(cuda_lib):
    missing = [n for n in declared_functions() if not hasattr(cuda_lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from textsift_b200 import abi
    bound = {n for n, _, _ in abi.SIGNATURES}
    assert bound == set(declared_functions())


def test_abi_version_and_defaults(cuda_lib):
    from textsift_b200 import abi
    assert cuda_lib.ts_cuda_abi_version() == 1
    c = abi.default_cfg()
    # browser/backends/wasm.ts:464-483
    assert (c.d_model, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.window, c.d_ff, c.n_experts, c.top_k,
            c.n_classes) == (640, 8, 14, 2, 64, 128, 640, 128, 4, 33)
    assert c.vocab == 200064 and abs(c.eps - 1e-5) < 1e-12 and c.rope_theta == 150000.0 and c.rope_factor == 32.0


def test_create_without_gpu_fails_cleanly(cuda_lib):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from textsift_b200 import abi
    c = abi.default_cfg()
    err = ctypes.create_string_buffer(256)
    assert not cuda_lib.ts_cuda_create(ctypes.byref(c), err, 256)
    assert b"device" in err.value.lower()


def test_backend_contract_errors():
    """forward before warmup raises, like WasmBackend.forward (wasm.ts:733-735)."""
    from textsift_b200 import CudaBackend, small_config
    b = CudaBackend({}, small_config())
    with pytest.raises(RuntimeError):
        b.forward([1, 2, 3], [1, 1, 1])
    b.dispose()
    b.dispose()  # idempotent (abstract.ts:55)


def test_loader_names_match_reference_loader():
    """make_weights produces exactly the names loadOnnxWeights builds
    (browser/backends/wasm.ts:358-446) for a 1-layer model."""
    from textsift_b200 import make_weights, small_config
    w = make_weights(small_config(n_layers=1, vocab=64, n_experts=4), seed=1)
    names = set(w)
    expect = {"embed.int4", "embed.scales", "embed.zp", "final_norm", "score.int4", "score.scales", "score.zp",
              "score.bias", "layers.0.input_layernorm", "layers.0.post_attention_layernorm", "layers.0.attn.sinks"}
    for pr in ("attn.q_proj", "attn.k_proj", "attn.v_proj", "attn.o_proj", "router", "experts.gate_up",
               "experts.down"):
        for f in ("int4", "scales", "zp", "bias"):
            expect.add(f"layers.0.{pr}.{f}")
    assert names == expect
