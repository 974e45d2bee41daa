"""CudaBackend: textsift's InferenceBackend contract over libtextsift_cuda.

Mirrors packages/textsift/src/browser/backends/abstract.ts:36-56:
    name, warmup(), forward(token_ids, attention_mask) -> Logits, dispose()
with Logits {data: float32[T * 33] row-major, sequence_length, num_classes}
(abstract.ts:29-34).  Errors follow the reference's behaviour: forward before
warmup raises, a mask whose length differs from the ids raises
(browser/backends/wasm.ts:740-750), dispose() is idempotent.

forward_packed() is the batched entry the B200 build adds: many chunks in
one launch, each computed exactly as its own forward.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Iterable, Iterator, Mapping, Sequence

import numpy as np

from . import abi
from .synth import PF_CONFIG, tensor_dtype


@dataclass
class Logits:
    data: np.ndarray          # float32 [sequence_length * num_classes]
    sequence_length: int
    num_classes: int

    def as_2d(self) -> np.ndarray:
        return self.data.reshape(self.sequence_length, self.num_classes)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def make_cfg(cfg: Mapping | None = None, *, device: int = 0, max_tokens: int = 65536,
             max_seq_len: int = 8192, mode: int = abi.TS_MODE_FAST) -> abi.Cfg:
    c = abi.default_cfg()
    m = dict(PF_CONFIG)
    if cfg:
        m.update(cfg)
    r = m.get("rope", {})
    c.device = device
    for k in ("vocab", "d_model", "n_layers", "n_heads", "n_kv_heads", "head_dim", "window", "d_ff",
              "n_experts", "top_k", "n_classes"):
        setattr(c, k, int(m[k]))
    c.eps = float(m["eps"])
    c.rope_theta = float(r.get("theta", 150000.0))
    c.rope_factor = float(r.get("factor", 32.0))
    c.rope_original_max_pos = float(r.get("orig", 4096.0))
    c.rope_beta_fast = float(r.get("beta_fast", 32.0))
    c.rope_beta_slow = float(r.get("beta_slow", 1.0))
    c.max_tokens = int(max_tokens)
    c.max_seq_len = int(max_seq_len)
    c.mode = int(mode)
    return c


class CudaBackend:
    """InferenceBackend implemented by the B200 kernels."""

    name = "cuda"

    def __init__(self, tensors: Mapping[str, np.ndarray], cfg: Mapping | None = None, *, device: int = 0,
                 max_tokens: int = 65536, max_seq_len: int = 8192, mode: int = abi.TS_MODE_FAST):
        self._tensors = tensors
        self._onnx = None  # (graph bytes, external-data bytes) for from_onnx
        self._cfg = make_cfg(cfg, device=device, max_tokens=max_tokens, max_seq_len=max_seq_len, mode=mode)
        self.num_classes = int(self._cfg.n_classes)
        self._h = None
        self._ready = False

    @classmethod
    def from_onnx(cls, graph: bytes | str, ext_data: bytes | str | None = None, cfg: Mapping | None = None,
                  **kw) -> "CudaBackend":
        """Weights from the model's ONNX files (onnx/model_q4f16.onnx and
        onnx/model_q4f16.onnx_data; bytes or paths), mapped and converted by
        the addon the way loadOnnxWeights does (browser/backends/wasm.ts)."""
        def _bytes(x):
            if x is None or isinstance(x, (bytes, bytearray)):
                return x
            with open(x, "rb") as f:
                return f.read()
        b = cls({}, cfg, **kw)
        b._onnx = (_bytes(graph), _bytes(ext_data))
        return b

    # -- lifecycle -------------------------------------------------------
    def _create(self) -> None:
        L = abi.lib()
        if self._h is None:
            err = ctypes.create_string_buffer(1024)
            h = L.ts_cuda_create(ctypes.byref(self._cfg), err, 1024)
            if not h:
                raise abi.TextsiftCudaError(abi.TS_ERR_CUDA, err.value.decode(errors="replace"))
            self._h = h

    def ep_init(self, rank: int, world: int, nccl_id: bytes) -> None:
        """Expert parallelism over `world` ranks (call on every rank before
        warmup, with the same id from ep_unique_id() on rank 0): this
        backend keeps experts [rank E / world, (rank + 1) E / world)."""
        self._create()
        ident = np.frombuffer(nccl_id, dtype=np.uint8)
        abi.check(abi.lib().ts_cuda_ep_init(self._h, rank, world, _ptr(ident), ident.size))

    @staticmethod
    def ep_unique_id() -> bytes:
        L = abi.lib()
        n = L.ts_cuda_ep_unique_id(None, 0)
        buf = (ctypes.c_uint8 * n)()
        if L.ts_cuda_ep_unique_id(buf, n) != n:
            raise abi.TextsiftCudaError(abi.TS_ERR_CUDA, abi.last_error())
        return bytes(buf)

    def warmup(self) -> None:
        """Create the device context, upload and repack weights (idempotent)."""
        if self._ready:
            return
        L = abi.lib()
        self._create()
        if self._onnx is not None:
            graph, ext = self._onnx
            g = np.frombuffer(graph, dtype=np.uint8)
            e = np.frombuffer(ext, dtype=np.uint8) if ext else None
            err = ctypes.create_string_buffer(1024)
            rc = L.ts_cuda_load_onnx(self._h, _ptr(g), g.size, _ptr(e), 0 if e is None else e.size, err, 1024)
            if rc != 0:
                raise abi.TextsiftCudaError(rc, err.value.decode(errors="replace"))
            self._onnx = None
        for name, arr in self._tensors.items():
            a = np.ascontiguousarray(arr)
            shape = (ctypes.c_int64 * a.ndim)(*a.shape)
            abi.check(L.ts_cuda_load_tensor(self._h, name.encode(), tensor_dtype(a), shape, a.ndim,
                                            _ptr(a), a.nbytes))
        abi.check(L.ts_cuda_finalize(self._h))
        self._tensors = {}  # the library holds its own copy now
        self._ready = True

    def dispose(self) -> None:
        if self._h is not None:
            abi.lib().ts_cuda_destroy(self._h)
            self._h = None
        self._ready = False

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def device_name(self) -> str:
        return abi.lib().ts_cuda_device_name(self._h).decode() if self._h else ""

    def set_mode(self, mode: int) -> None:
        abi.check(abi.lib().ts_cuda_set_mode(self._h, int(mode)))

    # -- inference -------------------------------------------------------
    def forward(self, token_ids: Sequence[int] | np.ndarray, attention_mask: Sequence[int] | np.ndarray) -> Logits:
        if not self._ready:
            raise RuntimeError("CudaBackend: call warmup() before forward()")
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int32))
        mask = np.ascontiguousarray(np.asarray(attention_mask, dtype=np.uint8))
        T = ids.size
        if mask.size != T:
            raise ValueError(f"CudaBackend.forward: attentionMask length {mask.size} does not match "
                             f"tokenIds length {T}")
        out = np.empty((T * self.num_classes,), dtype=np.float32)
        if T:
            abi.check(abi.lib().ts_cuda_forward(self._h, _ptr(ids), _ptr(mask), T, _ptr(out)))
        return Logits(out, T, self.num_classes)

    def forward_trace(self, token_ids, attention_mask=None):
        """One sequence; returns (Logits, top-k experts i32 [n_layers, T, top_k])."""
        if not self._ready:
            raise RuntimeError("CudaBackend: call warmup() before forward_trace()")
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int32))
        T = ids.size
        mask = None if attention_mask is None else np.ascontiguousarray(np.asarray(attention_mask, dtype=np.uint8))
        offs = np.array([0, T], np.uint32)
        out = np.empty((T * self.num_classes,), dtype=np.float32)
        topk = np.empty((int(self._cfg.n_layers), T, int(self._cfg.top_k)), dtype=np.int32)
        abi.check(abi.lib().ts_cuda_forward_trace(self._h, _ptr(ids), _ptr(mask), _ptr(offs), 1, _ptr(out),
                                                  _ptr(topk)))
        return Logits(out, T, self.num_classes), topk

    def forward_packed(self, chunks: Sequence[np.ndarray], masks: Sequence[np.ndarray] | None = None) -> list[Logits]:
        """Forward many chunks in one launch; returns one Logits per chunk."""
        if not self._ready:
            raise RuntimeError("CudaBackend: call warmup() before forward_packed()")
        lens = [int(np.asarray(c).size) for c in chunks]
        offs = np.zeros(len(lens) + 1, dtype=np.uint32)
        offs[1:] = np.cumsum(lens)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(c, dtype=np.int32) for c in chunks]))
        mask = None
        if masks is not None:
            mask = np.ascontiguousarray(np.concatenate([np.asarray(m, dtype=np.uint8) for m in masks]))
            if mask.size != ids.size:
                raise ValueError("forward_packed: masks and chunks differ in length")
        out = np.empty((ids.size * self.num_classes,), dtype=np.float32)
        abi.check(abi.lib().ts_cuda_forward_packed(self._h, _ptr(ids), _ptr(mask), _ptr(offs), len(lens),
                                                   _ptr(out)))
        res = []
        for s, n in enumerate(lens):
            o = int(offs[s]) * self.num_classes
            res.append(Logits(out[o:o + n * self.num_classes].copy(), n, self.num_classes))
        return res

    def forward_packed_stream(self, batches: Iterable[Sequence[np.ndarray]]) -> Iterator[list[Logits]]:
        """forward_packed over a stream of batches (each a list of chunks),
        yielding each batch's Logits in order while the next batch runs: batch
        i + 1 is begun in the other pinned slot before batch i is collected
        (ts_cuda_forward_packed_begin/_end).  Results equal forward_packed's."""
        if not self._ready:
            raise RuntimeError("CudaBackend: call warmup() before forward_packed_stream()")
        L = abi.lib()
        pending = None  # (slot, lens, offsets) of the batch in flight
        slot = 0
        try:
            for chunks in batches:
                lens = [int(np.asarray(c).size) for c in chunks]
                offs = np.zeros(len(lens) + 1, dtype=np.uint32)
                offs[1:] = np.cumsum(lens)
                ids = np.ascontiguousarray(np.concatenate([np.asarray(c, dtype=np.int32) for c in chunks]))
                abi.check(L.ts_cuda_forward_packed_begin(self._h, _ptr(ids), None, _ptr(offs), len(lens), slot))
                done, pending = pending, (slot, lens, offs)
                slot ^= 1
                if done is not None:
                    yield self._collect(*done)
            if pending is not None:
                done, pending = pending, None
                yield self._collect(*done)
        finally:
            if pending is not None:  # the caller stopped early: free the slot
                self._collect(*pending)

    def _collect(self, slot: int, lens: list[int], offs: np.ndarray) -> list[Logits]:
        out = np.empty((int(offs[-1]) * self.num_classes,), dtype=np.float32)
        abi.check(abi.lib().ts_cuda_forward_packed_end(self._h, slot, _ptr(out)))
        return [Logits(out[int(offs[s]) * self.num_classes:(int(offs[s]) + n) * self.num_classes].copy(), n,
                       self.num_classes) for s, n in enumerate(lens)]

    def forward_packed_tags(self, chunks: Sequence[np.ndarray], calibration: Sequence[float],
                            masks: Sequence[np.ndarray] | None = None) -> list[np.ndarray]:
        """Forward many chunks and decode each on the GPU with the BIOES
        Viterbi decoder (ViterbiDecoder.decode, browser/inference/viterbi.ts):
        one u8 tag array per chunk.  calibration: the six transition biases of
        ViterbiCalibration (browser/model/calibration.ts:29-36) in field order."""
        if not self._ready:
            raise RuntimeError("CudaBackend: call warmup() before forward_packed_tags()")
        cal = np.ascontiguousarray(np.asarray(calibration, dtype=np.float32))
        if cal.size != 6:
            raise ValueError("forward_packed_tags: calibration needs 6 values")
        lens = [int(np.asarray(c).size) for c in chunks]
        offs = np.zeros(len(lens) + 1, dtype=np.uint32)
        offs[1:] = np.cumsum(lens)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(c, dtype=np.int32) for c in chunks]))
        mask = None
        if masks is not None:
            mask = np.ascontiguousarray(np.concatenate([np.asarray(m, dtype=np.uint8) for m in masks]))
            if mask.size != ids.size:
                raise ValueError("forward_packed_tags: masks and chunks differ in length")
        tags = np.empty(ids.size, dtype=np.uint8)
        abi.check(abi.lib().ts_cuda_forward_packed_tags(self._h, _ptr(ids), _ptr(mask), _ptr(offs), len(lens),
                                                        _ptr(cal), _ptr(tags)))
        return [tags[int(offs[s]):int(offs[s + 1])].copy() for s in range(len(lens))]
