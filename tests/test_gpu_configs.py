"""BASELINE.json configs [1]-[3] at their full sizes on the GPU, through the
C ABI, against the oracle.  The launch always covers the whole configuration;
the oracle checks sampled rows (its cost grows with the sample, not with the
launch), with the same tolerances as the per-op tests.

  [1] MatMulNBits, A fp16 N(0,1) [M=16384, K=640], N in {640, 1280}
  [2] one MoE layer on 16384 tokens, router N(0, 0.02) quantised to int4,
      uniform and Zipf(s=1.2)-skewed expert popularity (top-k bit-exact in
      both modes)
  [3] banded attention, batch 64 x 8192, 14/2 heads, head_dim 64, window
      +-128, RoPE (theta 150000, the reference's YaRN tables) applied to q/k,
      keys masked on the last 10% of every sequence
"""
import numpy as np
import pytest

from gpu_util import dev, empty, f16, host, ptr, rand_w4, stream, ulp_diff, w4_handle

pytestmark = pytest.mark.gpu

F16 = np.uint16


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


@pytest.fixture(scope="module")
def L(cuda_lib):
    import torch
    assert torch.cuda.is_available()
    return cuda_lib


# ------------------------------------------------------------------ config[1]
@pytest.mark.parametrize("N", [640, 1280])
def test_config1_matmul_16384(L, oracle, N):
    M, K = 16384, 640
    r = rng(100 + N)
    int4, sc, zp, bias = rand_w4(r, 1, N, K, zp_random=False)
    x = r.normal(0, 1, size=(M, K)).astype(np.float16).view(F16)
    h = w4_handle(L, int4, sc, zp, bias)
    try:
        out = empty((M, N), np.float32)
        assert L.ts_cuda_op_matmul_nbits(h, 0, ptr(dev(x)), 1, ptr(out), 2, M, 0, stream()) == 0
        got = host(out, np.float32)
    finally:
        L.ts_cuda_w4_destroy(h)
    rows = np.unique(np.concatenate([[0, 1, M - 1], r.integers(0, M, size=509)]))
    ref = oracle.matmul_int4(x[rows], int4[0], sc[0], zp[0], bias[0], True)
    err = np.abs(got[rows] - ref)
    assert err.max() <= 2e-3 * np.abs(ref).max() + 1e-3, err.max()
    assert np.sqrt((err ** 2).mean() / (ref ** 2).mean()) < 1e-3


# ------------------------------------------------------------------ config[2]
@pytest.fixture(scope="module", params=["uniform", "zipf"])
def moe_case(request, oracle, cuda_lib):
    from textsift_b200 import CudaBackend, make_weights, small_config
    from textsift_b200.synth import quantize_int4, zipf_router_bias
    cfg = small_config(n_layers=1, vocab=256)
    bias = zipf_router_bias(cfg["n_experts"], 1.2, seed=5) if request.param == "zipf" else None
    w = make_weights(cfg, seed=21, bias_std=0.02, router_bias=bias)
    # the benchmark's router: fp16 N(0, 0.02) weights, stored the way the model
    # stores them (int4 MatMulNBits with fp16 scales and zero points)
    i4, sc, zp = quantize_int4(rng(22).normal(0, 0.02, size=(cfg["n_experts"], cfg["d_model"])).astype(np.float32))
    w["layers.0.router.int4"], w["layers.0.router.scales"], w["layers.0.router.zp"] = i4, sc, zp
    b = CudaBackend(w, cfg, max_tokens=16384, max_seq_len=2048)
    b.warmup()
    x = rng(23).normal(0, 1, size=(16384, 640)).astype(np.float32)
    # canonical single-thread order (the bit-exact reference), the same for both GPU modes
    ref, ridx, _ = oracle.OracleModel(cfg, w).moe(0, x, n_threads=1)
    yield request.param, b, x, ref, ridx
    b.dispose()


@pytest.mark.parametrize("mode", [1, 0])
def test_config2_moe_layer_16384(moe_case, cuda_lib, mode):
    from textsift_b200 import abi
    regime, b, x, ref, ridx = moe_case
    T = x.shape[0]
    b.set_mode(mode)
    try:
        out = empty((T, 640), np.uint16)
        idx = empty((T, 4), np.int32)
        assert cuda_lib.ts_cuda_op_moe(b.handle, 0, ptr(dev(x)), ptr(out), ptr(idx), None, T, stream()) == 0, \
            abi.last_error()
        got, gidx = host(out, np.uint16), host(idx, np.int32)
    finally:
        b.set_mode(0)
    hist = np.bincount(ridx.reshape(-1), minlength=128)
    print(f"{regime}: busiest expert {hist.max()} routes, idlest {hist.min()}, "
          f"top-8 share {np.sort(hist)[-8:].sum() / hist.sum():.3f}")
    if regime == "zipf":
        assert np.sort(hist)[-8:].sum() / hist.sum() > 0.2  # the skew is real
    # the router is the reference's on the same f32 input in both modes
    assert np.array_equal(gidx, ridx)
    if mode == abi.TS_MODE_EXACT:
        assert ulp_diff(got, ref).max() <= 1 and (got == ref).mean() > 0.99
    else:
        e = np.abs(f16(got) - f16(ref))
        assert e.max() <= 1e-2 * np.abs(f16(ref)).max(), e.max()
        assert np.sqrt((e ** 2).mean() / (f16(ref) ** 2).mean()) < 3e-3


# ------------------------------------------------------------------ config[3]
def _rope_torch(x, cos_t, sin_t, H):
    """The reference's RoPE (rope_apply, wasm_exports.zig:1460-1502) on fp16
    [T, H*64] with tables [T, 32]: three fp16 roundings per output."""
    import torch
    T = x.shape[0]
    v = x.view(T, H, 32, 2)
    a, b = v[..., 0].float(), v[..., 1].float()
    c = cos_t.view(T, 1, 32).float()
    s = sin_t.view(T, 1, 32).float()
    ac, bs = (a * c).half().float(), (b * s).half().float()
    bc, as_ = (b * c).half().float(), (a * s).half().float()
    out = torch.stack([(ac - bs).half(), (bc + as_).half()], dim=-1)
    return out.reshape(T, H * 64)


@pytest.fixture(scope="module")
def attn_case(L, oracle):
    import torch
    B, S, Hq, Hkv, hd = 64, 8192, 14, 2, 64
    T = B * S
    g = torch.Generator(device="cuda").manual_seed(33)
    q = torch.randn((T, Hq * hd), generator=g, device="cuda").half()
    k = torch.randn((T, Hkv * hd), generator=g, device="cuda").half()
    v = torch.randn((T, Hkv * hd), generator=g, device="cuda").half()
    cos16, sin16 = oracle.rope_tables(S)
    cos_t = torch.from_numpy(np.tile(cos16.view(np.float16), (B, 1))).cuda()
    sin_t = torch.from_numpy(np.tile(sin16.view(np.float16), (B, 1))).cuda()
    q = _rope_torch(q, cos_t, sin_t, Hq)
    k = _rope_torch(k, cos_t, sin_t, Hkv)
    mask = np.ones(T, np.uint8)
    for bi in range(B):
        mask[bi * S + int(S * 0.9):(bi + 1) * S] = 0
    sinks = np.zeros(Hq, np.float32)
    offs = (np.arange(B + 1) * S).astype(np.uint32)
    return dict(q=q, k=k, v=v, mask=mask, sinks=sinks, offs=offs, T=T, S=S, B=B, Hq=Hq, Hkv=Hkv)


@pytest.mark.parametrize("mode", [0, 1])
def test_config3_attention_64x8192(L, oracle, attn_case, mode):
    import torch
    c = attn_case
    T, S, Hq, Hkv, W = c["T"], c["S"], c["Hq"], c["Hkv"], 128
    out = empty((T, Hq * 64), np.uint16)
    assert L.ts_cuda_op_banded_attention(c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(),
                                         ptr(dev(c["sinks"])), ptr(dev(c["mask"])), ptr(out), T, Hq, Hkv, 64, W,
                                         c["offs"].ctypes.data, c["B"], mode, stream()) == 0, L.ts_cuda_last_error()
    torch.cuda.synchronize()
    # blocks of 128 consecutive queries: sequence starts, the mask boundary,
    # the last tokens, and random interior positions of several sequences
    r = rng(34 + mode)
    blocks = [(0, 0), (3, S - 128), (5, int(S * 0.9) - 64), (11, int(S * 0.9)), (63, S - 128)]
    blocks += [(int(r.integers(0, c["B"])), int(r.integers(0, S - 128))) for _ in range(7)]
    errs, ulps = [], []
    for seq, t0 in blocks:
        base = seq * S
        a, b = max(0, t0 - W), min(S, t0 + 128 + W)
        rows = slice(base + a, base + b)
        qs = c["q"][rows].cpu().numpy().view(F16)
        ks = c["k"][rows].cpu().numpy().view(F16)
        vs = c["v"][rows].cpu().numpy().view(F16)
        ref = oracle.banded_attention(qs, ks, vs, c["sinks"], c["mask"][rows], b - a, Hq, Hkv, 64, W)
        got = out[base + t0: base + t0 + 128].cpu().numpy().view(F16)
        want = ref[t0 - a: t0 - a + 128]
        errs.append(np.abs(f16(got) - f16(want)))
        ulps.append(ulp_diff(got, want))
    e = np.concatenate(errs)
    if mode == 1:
        u = np.concatenate(ulps)
        assert u.max() <= 1 and (u == 0).mean() > 0.99
    else:
        assert e.max() <= 4e-3 and e.mean() < 3e-4, (e.max(), e.mean())
