// k_router.cu — the fast-mode router, exact on identical inputs.
//
// The router logits of the tensor-core GEMM (fp16 operands, f32
// accumulation) pick, per token, the experts that may belong to the exact top
// 4 (the kEpiRouterCert epilogue of k_gemm_tc.cu, with a proven bound on the
// difference to the reference's f32 logits).  router_cert_kernel evaluates
// exactly those candidates in the reference's order -- matmulInt4BlockImpl's
// tile or tail path (zig/wasm_exports.zig:560-708) on the f32 router input --
// and selects the top k from their exact logits with the reference's tie rule
// (wasm_exports.zig:367-426), then the softmax over k with the exact
// exponential and x 1/k (wasm_exports.zig:919-958, browser/inference/
// block.ts:98-102).  Indices and weights are therefore those of the
// reference on the same f32 input, bit for bit.
//
// One warp per token.  The f32 router input is either given (the per-op
// entry) or rebuilt exactly as the fast add+RMSNorm computed it
// (rmsnorm_fast_kernel<true>): its stored fp16 sum times its stored 1 / rms
// times the norm weight, the same products.  The lanes then split the
// candidates' 32-blocks between them, and each candidate's blocks are added
// in the reference's order.
#include "ts_common.cuh"
#include "ts_kernels.h"
#include "ts_simt.h"

#include <cmath>
#include <cstring>

namespace ts {

namespace {

constexpr uint32_t kCertThreads = 256;  // 8 warps, one token at a time each
constexpr uint32_t kCertTokens = 32;    // tokens per block, inside one permutation chunk
constexpr int kPairBatch = 2;           // (candidate, block) pairs per lane whose loads go out together
static_assert(kPermChunk % kCertTokens == 0, "a block's tokens share one permutation chunk");

// The reference's value of one 32-block of int4 weights (16 bytes pk, low
// nibble = even element) against 32 f32 inputs xb (16-byte aligned, in
// shared memory): the tile path's four lane chains of eight fused
// multiply-adds (zig/wasm_exports.zig:615-646) or the tail path's even / odd
// chunk accumulators (689-697), exactly as matmul_w4_exact_kernel.  Two
// chains at a time run as one packed f32x2 instruction (each half an IEEE
// fused multiply-add or add, so the same bits as the scalar chains); the
// weight values are nibble - zp, exact (nzz = -(2^23 + zp) twice).
__device__ __forceinline__ float block_dot_ref(const float* xb, uint4 pk, uint64_t nzz, bool tile_path) {
  const uint32_t wd[4] = {pk.x, pk.y, pk.z, pk.w};
  if (tile_path) {
    uint64_t v01 = 0u, v23 = 0u;  // (v0, v1), (v2, v3)
#pragma unroll
    for (int c = 0; c < 8; c++) {
      // elements 4c .. 4c + 3: bytes 2 (c & 1) and 2 (c & 1) + 1 of word c / 2
      const float4 x = *reinterpret_cast<const float4*>(xb + 4 * c);
      const uint32_t w = wd[c >> 1], lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
      const uint32_t j0 = 2u * (uint32_t)(c & 1);
      const uint64_t q01 = add_f32x2(f2pack(nib_raw(lo, j0), nib_raw(hi, j0)), nzz);
      const uint64_t q23 = add_f32x2(f2pack(nib_raw(lo, j0 + 1u), nib_raw(hi, j0 + 1u)), nzz);
      v01 = fma_f32x2(f2pack(x.x, x.y), q01, v01);
      v23 = fma_f32x2(f2pack(x.z, x.w), q23, v23);
    }
    float v0, v1, v2, v3;
    f2unpack(v01, v0, v1);
    f2unpack(v23, v2, v3);
    return __fadd_rn(__fadd_rn(v0, v1), __fadd_rn(v2, v3));
  }
  uint64_t a01 = 0u, a23 = 0u, b01 = 0u, b23 = 0u;  // (a0[0], a0[1]), (a0[2], a0[3]), the same of a1
#pragma unroll
  for (int k = 0; k < 4; k++) {
    // elements 8k .. 8k + 7: word k (byte j holds 8k + 2j and 8k + 2j + 1)
    const float4 x0 = *reinterpret_cast<const float4*>(xb + 8 * k);
    const float4 x1 = *reinterpret_cast<const float4*>(xb + 8 * k + 4);
    const uint32_t lo = wd[k] & 0x0F0F0F0Fu, hi = (wd[k] >> 4) & 0x0F0F0F0Fu;
    a01 = fma_f32x2(f2pack(x0.x, x0.y), add_f32x2(f2pack(nib_raw(lo, 0), nib_raw(hi, 0)), nzz), a01);
    a23 = fma_f32x2(f2pack(x0.z, x0.w), add_f32x2(f2pack(nib_raw(lo, 1), nib_raw(hi, 1)), nzz), a23);
    b01 = fma_f32x2(f2pack(x1.x, x1.y), add_f32x2(f2pack(nib_raw(lo, 2), nib_raw(hi, 2)), nzz), b01);
    b23 = fma_f32x2(f2pack(x1.z, x1.w), add_f32x2(f2pack(nib_raw(lo, 3), nib_raw(hi, 3)), nzz), b23);
  }
  // c_j = a0[j] + a1[j], then (c0 + c1) + (c2 + c3)
  float c0, c1, c2, c3;
  f2unpack(add_f32x2(a01, b01), c0, c1);
  f2unpack(add_f32x2(a23, b23), c2, c3);
  return __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));
}

// A candidate as one 64-bit key whose unsigned maximum is the reference's
// first choice (value descending, then expert id ascending): the float's
// bits made monotonic in the high word, the complemented id in the low word.
__device__ __forceinline__ uint64_t cand_key(float v, uint32_t e) {
  uint32_t u = __float_as_uint(v + 0.0f);  // -0 as +0: equal values tie on the id
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((uint64_t)u << 32) | (uint64_t)(~e);
}
__device__ __forceinline__ float key_value(uint64_t k) {
  const uint32_t u = (uint32_t)(k >> 32);
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

}  // namespace

// Shared memory of one warp: the token's f32 router input (each 32-block
// padded to 36 floats so that lanes reading different blocks hit different
// banks), the per-(candidate, block) products of one batch of 32 candidates
// (rows padded to nb + 1), and every candidate's exact logit and expert id.
__host__ __device__ constexpr uint32_t cert_x_floats(uint32_t D) { return D / 32 * 36; }
__host__ __device__ constexpr uint32_t cert_warp_floats(uint32_t D) {
  return cert_x_floats(D) + 32 * (D / 32 + 1) + 2 * kMaxRouterExperts;
}

template <int SRC>
__global__ void __launch_bounds__(kCertThreads, 4) router_cert_kernel(const RouterCertArgs a) {
  extern __shared__ __align__(16) float cert_smem[];
  __shared__ int h[kMaxRouterExperts];
  pdl_trigger();
  for (uint32_t i = threadIdx.x; i < a.E; i += blockDim.x) h[i] = 0;
  __syncthreads();
  pdl_wait();
  const uint32_t D = a.D, nb = D / 32, K = a.K, E = a.E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* xs = cert_smem + (size_t)warp * cert_warp_floats(D);
  float* pb = xs + cert_x_floats(D);     // [32][nb + 1]
  float* cv = pb + 32 * (nb + 1);        // [kMaxRouterExperts] exact logits
  int* ci = reinterpret_cast<int*>(cv + kMaxRouterExperts);  // their expert ids
  const uint32_t t_begin = blockIdx.x * kCertTokens;
  for (uint32_t tl = (uint32_t)warp; tl < kCertTokens; tl += kCertThreads / 32) {
    const uint32_t t = t_begin + tl;
    if (t >= a.T) break;
    // the candidate record: byte 0 = count, byte k + 1 = expert id k
    const uint32_t cnt = a.cand[(size_t)t * 32];
    const uint32_t rec_id = lane < 31 ? a.cand[(size_t)t * 32 + 1 + lane] : 0u;  // candidate `lane`
    const bool all = cnt > 31u;
    const uint32_t n_c = all ? E : cnt;
    uint32_t loc, len;
    if (a.rloc) { loc = (uint32_t)a.rloc[t]; len = (uint32_t)a.rlen[t]; }
    else { loc = t; len = a.T; }
    const bool tile_path = loc < (len & ~7u);

    // ---- the f32 router input into xs ----
    const size_t base = (size_t)t * D;
    if constexpr (SRC == kRouterSrcAddNorm) {
      // rmsnorm_fast_kernel<true>'s product (x * inv_rms) * gamma on the fp16
      // sum it stored and the 1 / rms it stored: the same f32 bits (two
      // products per lane of an f32x2 multiply are two IEEE products)
      const float inv = a.inv[t];
      const uint64_t inv2 = f2pack(inv, inv);
      for (uint32_t c = (uint32_t)lane; c < D / 8u; c += 32u) {
        const uint4 xv = *reinterpret_cast<const uint4*>(a.a + base + 8 * c);
        const uint4 gv = *reinterpret_cast<const uint4*>(a.gamma + 8 * c);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
        float o8[8];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&xw[j]));
          const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&gw[j]));
          f2unpack(mul_f32x2(mul_f32x2(f2pack(x.x, x.y), inv2), f2pack(g.x, g.y)), o8[2 * j], o8[2 * j + 1]);
        }
        float* dst = xs + (c >> 2) * 36u + (c & 3u) * 8u;
        *reinterpret_cast<float4*>(dst) = make_float4(o8[0], o8[1], o8[2], o8[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(o8[4], o8[5], o8[6], o8[7]);
      }
    } else {
      for (uint32_t i = (uint32_t)lane * 4u; i < D; i += 128u) {
        const float4 v = *reinterpret_cast<const float4*>(a.x32 + base + i);
        *reinterpret_cast<float4*>(xs + (i >> 5) * 36u + (i & 31u)) = v;
      }
    }
    __syncwarp();

    // ---- exact logits of up to 32 candidates (candidate c = cb + lane has
    // id myid): lanes take (candidate, block) pairs, then lane c adds
    // candidate c's blocks in order and the bias ----
    auto batch_logits = [&](uint32_t cb, uint32_t nbt, uint32_t myid) -> float {
      const uint32_t npairs = nbt * nb;
      // pair p = c * nb + b; this lane's pairs are lane, lane + 32, ..., their
      // (c, b) stepped by (32 / nb, 32 % nb) and at most one carry instead of
      // a division per pair
      uint32_t c_n = (uint32_t)lane / nb, b_n = (uint32_t)lane - c_n * nb;
      const uint32_t step_c = 32u / nb, step_b = 32u - step_c * nb;
      for (uint32_t p0 = 0; p0 < npairs; p0 += 32u * kPairBatch) {
        // every load of this lane's (up to) kPairBatch pairs first, then the arithmetic
        uint4 wv[kPairBatch];
        float2 sz[kPairBatch];
        uint32_t cc[kPairBatch], bb[kPairBatch];
#pragma unroll
        for (int u = 0; u < kPairBatch; u++) {
          const bool ok = p0 + (uint32_t)lane + 32u * u < npairs;
          const uint32_t c = ok ? c_n : 0u, b = ok ? b_n : 0u;
          const uint32_t e = __shfl_sync(0xffffffffu, myid, c);
          cc[u] = c;
          bb[u] = b;
          wv[u] = make_uint4(0u, 0u, 0u, 0u);
          sz[u] = make_float2(0.0f, 0.0f);
          if (ok) {
            wv[u] = *reinterpret_cast<const uint4*>(a.w_int4 + (size_t)e * (D / 2) + 16 * b);
            sz[u] = *reinterpret_cast<const float2*>(a.w_sz + 2 * ((size_t)e * nb + b));
          }
          b_n += step_b;
          c_n += step_c;
          if (b_n >= nb) { b_n -= nb; c_n++; }
        }
#pragma unroll
        for (int u = 0; u < kPairBatch; u++) {
          if (p0 + (uint32_t)lane + 32u * u >= npairs) break;
          pb[cc[u] * (nb + 1) + bb[u]] =
              __fmul_rn(block_dot_ref(xs + bb[u] * 36u, wv[u], f2pack(sz[u].y, sz[u].y), tile_path), sz[u].x);
        }
      }
      __syncwarp();
      float v = 0.0f;
      if ((uint32_t)lane < nbt) {
        float sum = 0.0f;
        for (uint32_t b = 0; b < nb; b++) sum = __fadd_rn(sum, pb[lane * (nb + 1) + b]);
        v = __fadd_rn(sum, f16_ref_to_f32(a.bias[myid]));
      }
      __syncwarp();
      return v;
    };

    // ---- the top K, (value descending, then expert id ascending: the order of
    // router_topk_kernel and the reference's insertion); lane r < K ends up
    // holding choice r in sel_v / sel_e ----
    float sel_v = 0.0f;
    uint32_t sel_e = 0u;
    if (!all) {
      // one candidate per lane: its rank is the number of better candidates
      const float v = batch_logits(0u, n_c, rec_id);
      const bool valid = (uint32_t)lane < n_c;
      const uint64_t key = valid ? cand_key(v, rec_id) : 0u;
      uint32_t rank = 0;
      for (uint32_t j = 0; j < n_c; j++) rank += __shfl_sync(0xffffffffu, key, j) > key ? 1u : 0u;
      uint32_t src = 0;
#pragma unroll
      for (uint32_t r = 0; r < 8; r++) {
        const uint32_t bal = __ballot_sync(0xffffffffu, valid && rank == r);
        if ((uint32_t)lane == r && bal) src = (uint32_t)(__ffs(bal) - 1);
      }
      sel_v = __shfl_sync(0xffffffffu, v, src);
      sel_e = __shfl_sync(0xffffffffu, rec_id, src);
    } else {
      // every expert: batches of 32 into shared memory, then K rounds of a
      // warp-wide maximum of the keys
      for (uint32_t cb = 0; cb < E; cb += 32u) {
        const uint32_t nbt = min(32u, E - cb);
        const float v = batch_logits(cb, nbt, cb + (uint32_t)lane);
        if ((uint32_t)lane < nbt) {
          cv[cb + lane] = v;
          ci[cb + lane] = (int)(cb + lane);
        }
      }
      __syncwarp();
      uint64_t kr[4];  // this lane's entries lane + 32 j (0 = none or taken)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const uint32_t k = (uint32_t)lane + 32u * j;
        kr[j] = k < E ? cand_key(cv[k], (uint32_t)ci[k]) : 0u;
      }
#pragma unroll
      for (uint32_t r = 0; r < 8; r++) {
        if (r >= K) break;
        uint64_t best = kr[0];
#pragma unroll
        for (int j = 1; j < 4; j++) best = kr[j] > best ? kr[j] : best;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
          best = other > best ? other : best;
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
          if (kr[j] == best) kr[j] = 0u;
        if ((uint32_t)lane == r) {
          sel_v = key_value(best);
          sel_e = ~(uint32_t)best;
        }
      }
    }
    // softmax over the K values in order (wasm_exports.zig:919-958), x 1/K in
    // double; the first choice holds the maximum
    const float m = __shfl_sync(0xffffffffu, sel_v, 0);
    const float ex = (uint32_t)lane < K ? expf_ref(__fsub_rn(sel_v, m)) : 0.0f;
    float ssum = 0.0f;
#pragma unroll
    for (uint32_t r = 0; r < 8; r++) {
      const float er = __shfl_sync(0xffffffffu, ex, r);
      if (r < K) ssum = __fadd_rn(ssum, er);
    }
    const float inv = ssum > 0.0f ? __fdiv_rn(1.0f, ssum) : __fdiv_rn(1.0f, (float)K);
    if ((uint32_t)lane < K) {
      a.idx[(size_t)t * K + lane] = (int32_t)sel_e;
      a.w[(size_t)t * K + lane] = (float)((double)__fmul_rn(ex, inv) * (1.0 / (double)K));
      atomicAdd(&h[sel_e], 1);
    }
    __syncwarp();
  }
  __syncthreads();
  if (a.hist) {
    int* row = a.hist + (size_t)(blockIdx.x * kCertTokens / kPermChunk) * E;
    for (uint32_t i = threadIdx.x; i < E; i += blockDim.x)
      if (h[i]) atomicAdd(row + i, h[i]);
  }
}

// One warp per row: fp16 round-to-nearest copy of an f32 row and the sum of
// its absolute values (the bound's S for the router candidates).
__global__ void __launch_bounds__(256) f32_to_f16_absum_kernel(const float* __restrict__ x, uint16_t* __restrict__ y,
                                                               float* __restrict__ absum, uint32_t T, uint32_t D) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  float s = 0.0f;
  for (uint32_t i = (uint32_t)lane * 2; i < D; i += 64) {
    const float2 v = *reinterpret_cast<const float2*>(x + (size_t)row * D + i);
    s += fabsf(v.x) + fabsf(v.y);
    *reinterpret_cast<uint32_t*>(y + (size_t)row * D + i) = f32x2_to_h2(v.x, v.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) absum[row] = s;
}

cudaError_t launch_router_cert(const RouterCertArgs& a, int src, cudaStream_t st) {
  if (a.T == 0) return cudaSuccess;
  if (a.E > kMaxRouterExperts || a.K == 0 || a.K > 8 || a.K > a.E || a.D % 32 || a.D > 1024)
    return cudaErrorInvalidValue;
  const dim3 grid((a.T + kCertTokens - 1) / kCertTokens);
  const size_t smem = (size_t)(kCertThreads / 32) * cert_warp_floats(a.D) * sizeof(float);
  constexpr int kMaxSmem = (int)((kCertThreads / 32) * cert_warp_floats(1024) * sizeof(float));
  static std::atomic<uint64_t> done_f32{0}, done_add{0};
  if (src == kRouterSrcAddNorm) {
    if (cudaError_t e = smem_attr_per_device(router_cert_kernel<kRouterSrcAddNorm>, kMaxSmem, done_add); e != cudaSuccess)
      return e;
    return launch_pdl(router_cert_kernel<kRouterSrcAddNorm>, grid, dim3(kCertThreads), smem, st, a);
  }
  if (cudaError_t e = smem_attr_per_device(router_cert_kernel<kRouterSrcF32>, kMaxSmem, done_f32); e != cudaSuccess)
    return e;
  return launch_pdl(router_cert_kernel<kRouterSrcF32>, grid, dim3(kCertThreads), smem, st, a);
}

cudaError_t launch_f32_to_f16_absum(const float* x, uint16_t* y, float* absum, uint32_t T, uint32_t D,
                                    cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (D % 2) return cudaErrorInvalidValue;
  return launch_pdl(f32_to_f16_absum_kernel, dim3((T + 7) / 8), dim3(256), 0, st, x, y, absum, T, D);
}

// Host: the tables of a router weight in reference layout (int4 [E][D/2],
// fp16 scales [E][D/32], zero points [E][ceil(D/64)] or none):
//   bound[e] = max_i |w_ei|, bound[kMaxRouterExperts + e] = sum_i |w_ei| *
//   2^-24 + 1e-6, with |w_ei| = |q - zp| * |scale| and the scale decoded both
//   ways (IEEE and the reference's subnormal quirk), taking the larger; then
//   the largest of each (bound[2 kMaxRouterExperts], [.. + 1]);
//   sz[2 (e nb + b)] = the block's scale as the reference decodes it,
//   sz[2 (e nb + b) + 1] = -(2^23 + zp) (router_cert_kernel's nibble offset).
void router_bound_table(const uint8_t* int4, const uint16_t* scales, const uint8_t* zp, uint32_t E, uint32_t D,
                        float* bound, float* sz) {
  const uint32_t nb = D / 32, zs = (nb + 1) / 2;
  for (uint32_t i = 0; i < 2 * kMaxRouterExperts + 2; i++) bound[i] = 0.0f;
  for (uint32_t e = 0; e < E && e < kMaxRouterExperts; e++) {
    double wmax = 0.0, wsum = 0.0;
    for (uint32_t b = 0; b < nb; b++) {
      const uint16_t s16 = scales[(size_t)e * nb + b];
      const uint32_t mant = s16 & 0x3ffu, ex = (s16 >> 10) & 0x1fu;
      double ieee = ex == 0 ? std::ldexp((double)mant, -24) : std::ldexp(1.0 + mant / 1024.0, (int)ex - 15);
      if (ex == 31) ieee = INFINITY;
      // the reference's decode (math.zig:45-52): a subnormal is read as if normal
      const double quirk = ex == 0 && mant ? std::ldexp(1.0 + mant / 1024.0, -15) : ieee;
      const double sc = std::fmax(ieee, quirk);  // both decodes are bounded
      int z = 0;
      if (zp) {
        const uint8_t zb = zp[(size_t)e * zs + (b >> 1)];
        z = (b & 1) ? (zb >> 4) & 15 : zb & 15;
      }
      // the scale exactly as f16_ref_to_f32 reads it on the device
      const uint32_t rest = s16 & 0x7fffu;
      const uint32_t bits = ((uint32_t)(s16 & 0x8000u) << 16) | (rest ? (rest << 13) + (112u << 23) : 0u);
      float ref;
      std::memcpy(&ref, &bits, 4);
      sz[2 * ((size_t)e * nb + b)] = ref;
      sz[2 * ((size_t)e * nb + b) + 1] = -(8388608.0f + (float)z);
      for (uint32_t i = 0; i < 32; i++) {
        const uint8_t byte = int4[(size_t)e * (D / 2) + 16 * b + i / 2];
        const int qv = (i & 1) ? (byte >> 4) & 15 : byte & 15;
        const double w = std::fabs((double)(qv - z)) * sc;
        wmax = std::fmax(wmax, w);
        wsum += w;
      }
    }
    bound[e] = (float)(wmax * (1.0 + 1e-6));
    bound[kMaxRouterExperts + e] = (float)(wsum * std::ldexp(1.0, -24) + 1e-6);
    bound[2 * kMaxRouterExperts] = std::fmax(bound[2 * kMaxRouterExperts], bound[e]);
    bound[2 * kMaxRouterExperts + 1] = std::fmax(bound[2 * kMaxRouterExperts + 1], bound[kMaxRouterExperts + e]);
  }
}

}  // namespace ts
