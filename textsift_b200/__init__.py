"""textsift_b200 -- a B200 (sm_100a) backend for textsift's privacy-filter
forward pass.

The compute lives in libtextsift_cuda.so (C ABI: include/textsift_cuda.h);
this package is the host-side mirror of textsift's InferenceBackend contract
(CudaBackend) plus the synthetic-weight generator used by the benchmarks.
"""
from .abi import (TS_MODE_EXACT, TS_MODE_FAST, TextsiftCudaError, lib)  # noqa: F401
from .backend import CudaBackend, Logits, make_cfg  # noqa: F401
from .synth import PF_CONFIG, make_weights, small_config  # noqa: F401
