// k_simt.cu — CUDA-core kernels of the privacy-filter forward.
//
// These are the memory-bound and order-sensitive steps.  Each one restates
// the reference kernel's arithmetic in the reference's own order
// (packages/textsift/src/zig/wasm_exports.zig), so for identical inputs the
// output is bit-identical to textsift's WASM path:
//   embed_gather      wasm_exports.zig:1523-1573  GatherBlockQuantized
//   rmsnorm           wasm_exports.zig:229-277
//   add_rmsnorm       wasm_exports.zig:288-350
//   matmul_w4_exact   wasm_exports.zig:560-708    f32 int4 GEMM, tile/tail order
//   router_topk       wasm_exports.zig:367-426 + 919-958, block.ts:201-206
//   moe permute       expert.ts:127-145 (ascending token order per expert)
//   moe combine       wasm_exports.zig:1027-1055 + 1153-1164 + 969-990
//   swiglu_exact      wasm_exports.zig:855-903
//   split_rope        wasm_exports.zig:1460-1502
#include "ts_common.cuh"
#include "ts_kernels.h"
#include "ts_simt.h"

namespace ts {

// ---------------------------------------------------------------------------
// Per-token sequence bookkeeping for packed multi-sequence launches.
// ---------------------------------------------------------------------------
__global__ void seq_info_kernel(const uint32_t* __restrict__ offs, uint32_t n_seqs, uint32_t T, int* __restrict__ pos,
                                int* __restrict__ sstart, int* __restrict__ slen) {
  uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  uint32_t lo = 0, hi = n_seqs;  // find s with offs[s] <= t < offs[s+1]
  while (hi - lo > 1) {
    uint32_t mid = (lo + hi) >> 1;
    if (offs[mid] <= t) lo = mid; else hi = mid;
  }
  pos[t] = (int)(t - offs[lo]);
  sstart[t] = (int)offs[lo];
  slen[t] = (int)(offs[lo + 1] - offs[lo]);
}

// ---------------------------------------------------------------------------
// GatherBlockQuantized embedding: out[t, d] = f16((u4 - zp) * f32(scale)).
// One thread per (token, 32-block); out-of-range ids give zero rows.
// ---------------------------------------------------------------------------
__global__ void embed_gather_kernel(const uint8_t* __restrict__ w, const uint16_t* __restrict__ sc,
                                    const uint8_t* __restrict__ zp, const int32_t* __restrict__ ids,
                                    uint16_t* __restrict__ out, uint32_t T, uint32_t V, uint32_t D) {
  const uint32_t nb = D / 32, zs = (nb + 1) / 2;
  uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= T * nb) return;
  uint32_t t = gid / nb, b = gid % nb;
  int32_t id = ids[t];
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)t * D + b * 32);
  if (id < 0 || (uint32_t)id >= V) {
    for (int i = 0; i < 4; i++) o[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4 pk = *reinterpret_cast<const uint4*>(w + (size_t)id * (D / 2) + b * 16);
  const float s = f16_ref_to_f32(sc[(size_t)id * nb + b]);
  const uint8_t zb = zp[(size_t)id * zs + (b >> 1)];
  const int z = (b & 1) ? (zb >> 4) & 15 : zb & 15;
  const uint32_t wd[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {  // byte j of word q holds elements 8q+2j (lo) and 8q+2j+1 (hi)
      uint32_t byte = (wd[q] >> (8 * j)) & 0xffu;
      float lo = __fmul_rn((float)((int)(byte & 15u) - z), s);
      float hi = __fmul_rn((float)((int)(byte >> 4) - z), s);
      r[j] = (uint32_t)f32_to_f16_ref(lo) | ((uint32_t)f32_to_f16_ref(hi) << 16);
    }
    o[q] = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm fp16 -> f32 (and/or the fp16 tensor-core operand), one warp per row.
// Lanes 0..3 accumulate the four 4-lane partial sums of squares in order.
// ---------------------------------------------------------------------------
template <bool ADD>
__global__ void rmsnorm_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                               const uint16_t* __restrict__ gamma, uint16_t* __restrict__ sum_out,
                               float* __restrict__ out32, uint16_t* __restrict__ out16, uint32_t T, uint32_t D,
                               float eps) {
  extern __shared__ float rs_smem[];  // [warps][D] f32 (sum before rounding) + [warps][D] f32 (value read back)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= T) return;
  float* xs = rs_smem + (size_t)warp * 2 * D;  // squares source
  float* xr = xs + D;                          // value used by pass 2
  const uint16_t* ar = a + (size_t)row * D;
  for (uint32_t d = lane; d < D; d += 32) {
    float v = f16_ref_to_f32(ar[d]);
    if constexpr (ADD) {
      float sv = __fadd_rn(v, f16_ref_to_f32(b[(size_t)row * D + d]));
      uint16_t s16 = f32_to_f16_ref(sv);
      sum_out[(size_t)row * D + d] = s16;
      xs[d] = sv;
      xr[d] = f16_ref_to_f32(s16);
    } else {
      xs[d] = v;
      xr[d] = v;
    }
  }
  __syncwarp();
  const uint32_t D4 = D & ~3u;  // the 4-lane body covers [0, D4), the scalar tail [D4, D)
  float part = 0.0f;
  if (lane < 4)
    for (uint32_t d = lane; d < D4; d += 4) part = __fadd_rn(part, __fmul_rn(xs[d], xs[d]));
  float s0 = __shfl_sync(0xffffffffu, part, 0), s1 = __shfl_sync(0xffffffffu, part, 1);
  float s2 = __shfl_sync(0xffffffffu, part, 2), s3 = __shfl_sync(0xffffffffu, part, 3);
  float sumsq = __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
  for (uint32_t d = D4; d < D; d++) sumsq = __fadd_rn(sumsq, __fmul_rn(xs[d], xs[d]));
  const float d_inv = __fdiv_rn(1.0f, (float)D);
  const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(sumsq, d_inv), eps)));
  for (uint32_t d = lane; d < D; d += 32) {
    float y = __fmul_rn(__fmul_rn(xr[d], inv_rms), f16_ref_to_f32(gamma[d]));
    if (out32) out32[(size_t)row * D + d] = y;
    if (out16) out16[(size_t)row * D + d] = __half_as_ushort(__float2half_rn(y));
  }
}

// ---------------------------------------------------------------------------
// Exact-order int4 matmul on CUDA cores (wasm_exports.zig:560-708).
// Block = 128 output columns; each block walks a 128-row tile in groups of 8
// rows staged in shared memory.  Row r uses the tile-path order when its
// index inside its sequence is < 8*floor(len/8), the tail-path order
// otherwise, exactly as the single-thread reference partitions rows.
// ---------------------------------------------------------------------------
template <bool X_F32, int OUT>
__global__ void __launch_bounds__(256) matmul_w4_exact_kernel(const ExactArgs a) {
  extern __shared__ __align__(16) float xs[];  // [2 groups][8 rows][K]
  const uint32_t K = a.K, nb = K / 32, zs = (nb + 1) / 2;
  uint32_t expert = 0, row0, row_end, seg_start = 0, seg_len = 0;
  const bool grouped = a.tiles != nullptr;
  if (grouped) {
    if ((int)blockIdx.y >= *a.n_tiles) return;
    int4 t = a.tiles[blockIdx.y];
    expert = (uint32_t)t.x; row0 = (uint32_t)t.y; row_end = (uint32_t)t.z; seg_start = (uint32_t)t.w;
    seg_len = (uint32_t)a.seg_end[expert] - seg_start;
  } else {
    row0 = blockIdx.y * 128u;
    row_end = min(a.M, row0 + 128u);
  }
  const uint32_t half = threadIdx.x >> 7;  // which 8-row group of a pair this thread works on
  const uint32_t n = blockIdx.x * 128u + (threadIdx.x & 127u);
  const bool n_ok = n < a.N;
  const uint8_t* wr = a.w_int4 + (size_t)expert * a.w_int4_estride + (size_t)(n_ok ? n : 0) * (K / 2);
  const uint16_t* sr = a.w_scales + (size_t)expert * a.w_scales_estride + (size_t)(n_ok ? n : 0) * nb;
  const uint8_t* zr = a.w_zp ? a.w_zp + (size_t)expert * a.w_zp_estride + (size_t)(n_ok ? n : 0) * zs : nullptr;
  const float bias = n_ok ? f16_ref_to_f32(a.bias[(size_t)expert * a.bias_estride + n]) : 0.0f;
  float* myx = xs + (size_t)half * 8 * K;

  for (uint32_t gp = row0; gp < row_end; gp += 16) {
    __syncthreads();
    const uint32_t rows_pair = min(16u, row_end - gp);
    for (uint32_t i = threadIdx.x; i < rows_pair * K; i += blockDim.x) {
      const uint32_t r = i / K, k = i % K;
      const size_t src = (size_t)(gp + r) * a.ldx + k;
      xs[r * K + k] = X_F32 ? reinterpret_cast<const float*>(a.x)[src]
                            : f16_ref_to_f32(reinterpret_cast<const uint16_t*>(a.x)[src]);
    }
    __syncthreads();
    const uint32_t g0 = gp + half * 8;
    if (!n_ok || g0 >= row_end) continue;
    const uint32_t gr = min(8u, row_end - g0);
    bool tile_path[8];
#pragma unroll
    for (int r = 0; r < 8; r++) {
      uint32_t loc, len;
      const uint32_t row = g0 + r;
      if (grouped) { loc = row - seg_start; len = seg_len; }
      else if (a.rloc) { loc = row < a.M ? (uint32_t)a.rloc[row] : 0; len = row < a.M ? (uint32_t)a.rlen[row] : 1; }
      else { loc = row; len = a.M; }
      tile_path[r] = loc < (len & ~7u);
    }
    float sum[8];
#pragma unroll
    for (int r = 0; r < 8; r++) sum[r] = 0.0f;
    for (uint32_t b = 0; b < nb; b++) {
      const float scale = f16_ref_to_f32(sr[b]);
      int zp = 0;
      if (zr) { uint8_t zb = zr[b >> 1]; zp = (b & 1) ? (zb >> 4) & 15 : zb & 15; }
      const uint4 pk = *reinterpret_cast<const uint4*>(wr + b * 16);
      const uint32_t wd[4] = {pk.x, pk.y, pk.z, pk.w};
      float q[32];
#pragma unroll
      for (int i = 0; i < 16; i++) {
        uint32_t byte = (wd[i >> 2] >> (8 * (i & 3))) & 0xffu;
        q[2 * i] = (float)((int)(byte & 15u) - zp);
        q[2 * i + 1] = (float)((int)(byte >> 4) - zp);
      }
#pragma unroll
      for (int r = 0; r < 8; r++) {
        if ((uint32_t)r >= gr) break;
        const float4* x4 = reinterpret_cast<const float4*>(myx + r * K + b * 32);
        float bs;
        if (tile_path[r]) {
          float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const float4 xv = x4[c];
            v0 = __fmaf_rn(xv.x, q[4 * c + 0], v0);
            v1 = __fmaf_rn(xv.y, q[4 * c + 1], v1);
            v2 = __fmaf_rn(xv.z, q[4 * c + 2], v2);
            v3 = __fmaf_rn(xv.w, q[4 * c + 3], v3);
          }
          bs = __fadd_rn(__fadd_rn(v0, v1), __fadd_rn(v2, v3));
        } else {
          float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const float4 x0 = x4[2 * k], x1 = x4[2 * k + 1];
            a0[0] = __fmaf_rn(x0.x, q[8 * k + 0], a0[0]);
            a0[1] = __fmaf_rn(x0.y, q[8 * k + 1], a0[1]);
            a0[2] = __fmaf_rn(x0.z, q[8 * k + 2], a0[2]);
            a0[3] = __fmaf_rn(x0.w, q[8 * k + 3], a0[3]);
            a1[0] = __fmaf_rn(x1.x, q[8 * k + 4], a1[0]);
            a1[1] = __fmaf_rn(x1.y, q[8 * k + 5], a1[1]);
            a1[2] = __fmaf_rn(x1.z, q[8 * k + 6], a1[2]);
            a1[3] = __fmaf_rn(x1.w, q[8 * k + 7], a1[3]);
          }
          float c0 = __fadd_rn(a0[0], a1[0]), c1 = __fadd_rn(a0[1], a1[1]);
          float c2 = __fadd_rn(a0[2], a1[2]), c3 = __fadd_rn(a0[3], a1[3]);
          bs = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));
        }
        sum[r] = __fadd_rn(sum[r], __fmul_rn(bs, scale));
      }
    }
#pragma unroll
    for (int r = 0; r < 8; r++) {
      if ((uint32_t)r >= gr) break;
      const float v = __fadd_rn(sum[r], bias);
      const size_t o = (size_t)(g0 + r) * a.ldo + n;
      if constexpr (OUT == kOutF16) reinterpret_cast<uint16_t*>(a.out)[o] = f32_to_f16_ref(v);
      else if constexpr (OUT == kOutF32) reinterpret_cast<float*>(a.out)[o] = v;
      else reinterpret_cast<float*>(a.out)[o] = f16_ieee_to_f32(f32_to_f16_ref(v));
    }
  }
}

// ---------------------------------------------------------------------------
// Router top-k: insertion top-k (strict '>', ties keep the lower index,
// output descending), softmax over k with expf, then x (1/k) as the JS
// caller does in doubles (exact for k a power of two).
// ---------------------------------------------------------------------------
__global__ void router_topk_kernel(const float* __restrict__ logits, int32_t* __restrict__ idx,
                                   float* __restrict__ w, uint32_t T, uint32_t E, uint32_t K, double inv_k) {
  uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float* row = logits + (size_t)t * E;
  float ov[8];
  int oi[8];
  for (uint32_t i = 0; i < K; i++) { oi[i] = (int)i; ov[i] = row[i]; }
  for (uint32_t s = 1; s < K; s++)
    for (uint32_t j = s; j > 0 && ov[j] > ov[j - 1]; j--) {
      float tv = ov[j]; ov[j] = ov[j - 1]; ov[j - 1] = tv;
      int ti = oi[j]; oi[j] = oi[j - 1]; oi[j - 1] = ti;
    }
  for (uint32_t c = K; c < E; c++) {
    float v = row[c];
    if (v > ov[K - 1]) {
      ov[K - 1] = v; oi[K - 1] = (int)c;
      for (uint32_t j = K - 1; j > 0 && ov[j] > ov[j - 1]; j--) {
        float tv = ov[j]; ov[j] = ov[j - 1]; ov[j - 1] = tv;
        int ti = oi[j]; oi[j] = oi[j - 1]; oi[j - 1] = ti;
      }
    }
  }
  float m = ov[0];
  for (uint32_t c = 1; c < K; c++) if (ov[c] > m) m = ov[c];
  float e[8], sum = 0.0f;
  for (uint32_t c = 0; c < K; c++) { e[c] = expf_ref(__fsub_rn(ov[c], m)); sum = __fadd_rn(sum, e[c]); }
  const float inv = sum > 0.0f ? __fdiv_rn(1.0f, sum) : __fdiv_rn(1.0f, (float)K);
  for (uint32_t c = 0; c < K; c++) {
    idx[(size_t)t * K + c] = oi[c];
    w[(size_t)t * K + c] = (float)((double)__fmul_rn(e[c], inv) * inv_k);
  }
}

// ---------------------------------------------------------------------------
// MoE permutation.  count: one block per expert counts its routes.  scatter:
// one block per expert computes its segment offset and tile offset from the
// counts, writes its 128-row tiles, and compacts its (token, slot) routes in
// ascending route order (= ascending token, since a token selects an expert
// at most once), the order expert.ts:137-145 builds.
// ---------------------------------------------------------------------------
__global__ void moe_count_kernel(const int32_t* __restrict__ idx, uint32_t n_routes, int* __restrict__ counts) {
  const int e = blockIdx.x;
  int c = 0;
  for (uint32_t i = threadIdx.x; i < n_routes; i += blockDim.x) c += idx[i] == e;
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  __shared__ int ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (uint32_t i = 0; i < blockDim.x / 32; i++) s += ws[i];
    counts[e] = s;
  }
}

__global__ void moe_scatter_kernel(const int32_t* __restrict__ idx, uint32_t n_routes, uint32_t K,
                                   const int* __restrict__ counts, uint32_t E, int* __restrict__ perm_tok,
                                   int* __restrict__ route_pos, int4* __restrict__ tiles, int* __restrict__ n_tiles,
                                   int* __restrict__ seg_end) {
  const int e = blockIdx.x;
  __shared__ int s_off, s_tile_off, s_base;
  __shared__ int wsum[32];
  if (threadIdx.x == 0) {
    int off = 0, toff = 0, tot_t = 0;
    for (int i = 0; i < (int)E; i++) {
      int c = counts[i];
      int nt = (c + 127) / 128;
      if (i < e) { off += c; toff += nt; }
      tot_t += nt;
    }
    s_off = off; s_tile_off = toff; s_base = 0;
    if (e == 0) *n_tiles = tot_t;
    seg_end[e] = off + counts[e];
  }
  __syncthreads();
  const int cnt = counts[e];
  for (int tt = threadIdx.x; tt * 128 < cnt; tt += blockDim.x)
    tiles[s_tile_off + tt] = make_int4(e, s_off + tt * 128, s_off + min(cnt, tt * 128 + 128), s_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (uint32_t base = 0; base < n_routes; base += blockDim.x) {
    const uint32_t i = base + threadIdx.x;
    const bool hit = i < n_routes && idx[i] == e;
    const uint32_t bal = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < nw; w++) { int c = wsum[w]; if (w < warp) before += c; total += c; }
    if (hit) {
      const int p = s_off + s_base + before + __popc(bal & ((1u << lane) - 1u));
      perm_tok[p] = (int)(i / K);
      route_pos[i] = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_base += total;
    __syncthreads();
  }
}

// dst[p, :] = src[perm_tok[p], :] (row bytes a multiple of 16)
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                   const int* __restrict__ perm_tok, const int* __restrict__ n_rows_dev,
                                   uint32_t n_rows, uint32_t row_bytes) {
  const uint32_t rows = n_rows_dev ? (uint32_t)*n_rows_dev : n_rows;
  const uint32_t per_row = row_bytes / 16;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < rows * per_row; i += gridDim.x * blockDim.x) {
    const uint32_t p = i / per_row, c = i % per_row;
    reinterpret_cast<uint4*>(dst + (size_t)p * row_bytes)[c] =
        reinterpret_cast<const uint4*>(src + (size_t)perm_tok[p] * row_bytes)[c];
  }
}

// Deterministic MoE combine per token: acc = 0; for its experts in ascending
// id: acc = fma(w, v, acc); moe = f16(acc * K); out = f16(res + moe) (or moe).
__global__ void moe_combine_kernel(const float* __restrict__ down, const int32_t* __restrict__ idx,
                                   const float* __restrict__ w, const int* __restrict__ route_pos,
                                   const uint16_t* __restrict__ res, uint16_t* __restrict__ out, uint32_t T,
                                   uint32_t D, uint32_t K, uint32_t E) {
  const uint32_t t = blockIdx.x;
  if (t >= T) return;
  int ek[8], pk[8];
  float wk[8];
  uint32_t n = 0;
  for (uint32_t k = 0; k < K; k++) {
    int e = idx[(size_t)t * K + k];
    if (e < 0 || (uint32_t)e >= E) continue;
    uint32_t j = n++;
    ek[j] = e; wk[j] = w[(size_t)t * K + k]; pk[j] = route_pos[(size_t)t * K + k];
    while (j > 0 && ek[j] < ek[j - 1]) {
      int te = ek[j]; ek[j] = ek[j - 1]; ek[j - 1] = te;
      float tw = wk[j]; wk[j] = wk[j - 1]; wk[j - 1] = tw;
      int tp = pk[j]; pk[j] = pk[j - 1]; pk[j - 1] = tp;
      j--;
    }
  }
  const float kf = (float)K;
  for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.0f;
    for (uint32_t j = 0; j < n; j++) acc = __fmaf_rn(wk[j], down[(size_t)pk[j] * D + d], acc);
    const uint16_t m16 = f32_to_f16_ref(__fmul_rn(acc, kf));
    const size_t o = (size_t)t * D + d;
    out[o] = res ? f32_to_f16_ref(__fadd_rn(f16_ref_to_f32(res[o]), f16_ref_to_f32(m16))) : m16;
  }
}

// SwiGLU-clamp on f32 (gate even, up odd), 4-lane polynomial body.
__global__ void swiglu_exact_kernel(const float* __restrict__ gu, float* __restrict__ out,
                                    const int* __restrict__ n_rows_dev, uint32_t n_rows, uint32_t D) {
  const uint32_t rows = n_rows_dev ? (uint32_t)*n_rows_dev : n_rows;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)rows * D; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / D, d = i % D;
    out[i] = swiglu_ref(gu[r * 2 * D + 2 * d], gu[r * 2 * D + 2 * d + 1]);
  }
}

// Split a fused [T, q+k+v] fp16 projection and apply the reference RoPE
// (three fp16 roundings) to the q and k heads.
__global__ void split_rope_kernel(const uint16_t* __restrict__ qkv, uint16_t* __restrict__ q,
                                  uint16_t* __restrict__ k, uint16_t* __restrict__ v, const int* __restrict__ pos,
                                  const uint16_t* __restrict__ cos_t, const uint16_t* __restrict__ sin_t,
                                  uint32_t T, uint32_t qc, uint32_t kc, uint32_t vc, uint32_t hd) {
  const uint32_t W = qc + kc + vc, half = hd / 2;
  const uint32_t pairs = W / 2;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)T * pairs; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t t = (uint32_t)(i / pairs), c = (uint32_t)(i % pairs) * 2;
    uint16_t a16 = qkv[(size_t)t * W + c], b16 = qkv[(size_t)t * W + c + 1];
    if (c < qc + kc) {
      const uint32_t p = (c % hd) / 2;
      const uint16_t c16 = cos_t[(size_t)pos[t] * half + p], s16 = sin_t[(size_t)pos[t] * half + p];
      float cf = f16_ref_to_f32(c16), sf = f16_ref_to_f32(s16);
      float af = f16_ref_to_f32(a16), bf = f16_ref_to_f32(b16);
      float ac = f16_ref_to_f32(f32_to_f16_ref(__fmul_rn(af, cf)));
      float bs = f16_ref_to_f32(f32_to_f16_ref(__fmul_rn(bf, sf)));
      float bc = f16_ref_to_f32(f32_to_f16_ref(__fmul_rn(bf, cf)));
      float as = f16_ref_to_f32(f32_to_f16_ref(__fmul_rn(af, sf)));
      a16 = f32_to_f16_ref(__fsub_rn(ac, bs));
      b16 = f32_to_f16_ref(__fadd_rn(bc, as));
    }
    uint16_t* dst;
    uint32_t col, ld;
    if (c < qc) { dst = q; col = c; ld = qc; }
    else if (c < qc + kc) { dst = k; col = c - qc; ld = kc; }
    else { dst = v; col = c - qc - kc; ld = vc; }
    dst[(size_t)t * ld + col] = a16;
    dst[(size_t)t * ld + col + 1] = b16;
  }
}

// fp16 -> f32 widen with the reference decode (wasm_exports.zig:1106-1116).
__global__ void f16_to_f32_ref_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = f16_ref_to_f32(src[i]);
}

// f32 -> fp16 round-to-nearest (tensor-core operand of an f32 activation).
__global__ void f32_to_f16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __half_as_ushort(__float2half_rn(src[i]));
}

// The dequantised operand exactly as the tensor-core GEMM forms it in shared
// memory, written row-major [N, K] to global (parity probe for the tile).
__global__ void dequant_tiles_kernel(const uint8_t* __restrict__ blobs, uint32_t N, uint32_t K, uint32_t BN,
                                     uint32_t n_kc, uint16_t* __restrict__ out) {
  const uint32_t n = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t kc = blockIdx.y;
  if (n >= N) return;
  const uint32_t nt = n / BN, r = n % BN;
  const uint8_t* raw = blobs + ((size_t)nt * n_kc + kc) * w4_blob_bytes(BN);
  const uint4 h0 = *reinterpret_cast<const uint4*>(raw + r * 16);
  const uint4 h1 = *reinterpret_cast<const uint4*>(raw + BN * 16 + r * 16);
  const uint32_t sc = *reinterpret_cast<const uint32_t*>(raw + BN * 32 + r * 4);
  const uint32_t z = raw[BN * 36 + r];
  const uint32_t s0 = (sc & 0xffffu) * 0x00010001u, s1 = (sc >> 16) * 0x00010001u;
  const uint32_t z0 = (0x6400u | (z & 15u)) * 0x00010001u, z1 = (0x6400u | (z >> 4)) * 0x00010001u;
  const uint32_t wds[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  for (int c = 0; c < 8; c++) {
    const uint32_t sz = c < 4 ? s0 : s1, zz = c < 4 ? z0 : z1;
    for (int j = 0; j < 4; j++) {
      const uint32_t k = kc * 64 + 8 * c + 2 * j;
      const uint32_t bits = ((wds[c] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
      __half2 qh = __hsub2(*reinterpret_cast<const __half2*>(&bits), *reinterpret_cast<const __half2*>(&zz));
      __half2 d = __hmul2(qh, *reinterpret_cast<const __half2*>(&sz));
      if (k < K) out[(size_t)n * K + k] = __half_as_ushort(__low2half(d));
      if (k + 1 < K) out[(size_t)n * K + k + 1] = __half_as_ushort(__high2half(d));
    }
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
static inline unsigned nblk(size_t n, unsigned b) { return (unsigned)((n + b - 1) / b); }
static inline unsigned gs_blocks(size_t n, unsigned b) {
  size_t g = (n + b - 1) / b;
  return (unsigned)(g > 148u * 16u ? 148u * 16u : (g == 0 ? 1 : g));
}

cudaError_t launch_seq_info(const uint32_t* offs, uint32_t n_seqs, uint32_t T, int* pos, int* sstart, int* slen,
                            cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  seq_info_kernel<<<nblk(T, 256), 256, 0, st>>>(offs, n_seqs, T, pos, sstart, slen);
  return cudaGetLastError();
}

cudaError_t launch_embed(const uint8_t* w, const uint16_t* sc, const uint8_t* zp, const int32_t* ids, uint16_t* out,
                         uint32_t T, uint32_t V, uint32_t D, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  embed_gather_kernel<<<nblk((size_t)T * (D / 32), 128), 128, 0, st>>>(w, sc, zp, ids, out, T, V, D);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* gamma, float* out32, uint16_t* out16, uint32_t T,
                           uint32_t D, float eps, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const unsigned warps = 4;
  rmsnorm_kernel<false><<<nblk(T, warps), warps * 32, warps * 2 * D * sizeof(float), st>>>(
      x, nullptr, gamma, nullptr, out32, out16, T, D, eps);
  return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, uint16_t* sum_out,
                               float* out32, uint16_t* out16, uint32_t T, uint32_t D, float eps, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const unsigned warps = 4;
  rmsnorm_kernel<true><<<nblk(T, warps), warps * 32, warps * 2 * D * sizeof(float), st>>>(a, b, gamma, sum_out, out32,
                                                                                         out16, T, D, eps);
  return cudaGetLastError();
}

cudaError_t launch_matmul_exact(const ExactArgs& a, bool x_f32, int out_mode, uint32_t grid_m, cudaStream_t st) {
  if (grid_m == 0) return cudaSuccess;
  if (a.K % 32 || a.K > 2048) return cudaErrorInvalidValue;
  dim3 grid(nblk(a.N, 128), grid_m);
  const size_t sm = (size_t)16 * a.K * sizeof(float);
  static bool attr = false;
  if (!attr) {
    const int mx = 16 * 2048 * 4;
    cudaFuncSetAttribute(matmul_w4_exact_kernel<true, kOutF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(matmul_w4_exact_kernel<true, kOutF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(matmul_w4_exact_kernel<true, kOutF16Widen>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(matmul_w4_exact_kernel<false, kOutF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    cudaFuncSetAttribute(matmul_w4_exact_kernel<false, kOutF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    attr = true;
  }
  if (x_f32) {
    if (out_mode == kOutF16) matmul_w4_exact_kernel<true, kOutF16><<<grid, 256, sm, st>>>(a);
    else if (out_mode == kOutF32) matmul_w4_exact_kernel<true, kOutF32><<<grid, 256, sm, st>>>(a);
    else matmul_w4_exact_kernel<true, kOutF16Widen><<<grid, 256, sm, st>>>(a);
  } else {
    if (out_mode == kOutF16) matmul_w4_exact_kernel<false, kOutF16><<<grid, 256, sm, st>>>(a);
    else if (out_mode == kOutF32) matmul_w4_exact_kernel<false, kOutF32><<<grid, 256, sm, st>>>(a);
    else return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_router_topk(const float* logits, int32_t* idx, float* w, uint32_t T, uint32_t E, uint32_t K,
                               cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (K > 8 || K > E) return cudaErrorInvalidValue;
  router_topk_kernel<<<nblk(T, 128), 128, 0, st>>>(logits, idx, w, T, E, K, 1.0 / (double)K);
  return cudaGetLastError();
}

cudaError_t launch_moe_permute(const int32_t* idx, uint32_t T, uint32_t K, uint32_t E, int* counts, int* perm_tok,
                               int* route_pos, int4* tiles, int* n_tiles, int* seg_end, cudaStream_t st) {
  const uint32_t n_routes = T * K;
  moe_count_kernel<<<E, 256, 0, st>>>(idx, n_routes, counts);
  moe_scatter_kernel<<<E, 256, 0, st>>>(idx, n_routes, K, counts, E, perm_tok, route_pos, tiles, n_tiles, seg_end);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const void* src, void* dst, const int* perm_tok, const int* n_rows_dev,
                               uint32_t max_rows, uint32_t row_bytes, cudaStream_t st) {
  if (max_rows == 0) return cudaSuccess;
  gather_rows_kernel<<<gs_blocks((size_t)max_rows * row_bytes / 16, 256), 256, 0, st>>>(
      (const uint8_t*)src, (uint8_t*)dst, perm_tok, n_rows_dev, max_rows, row_bytes);
  return cudaGetLastError();
}

cudaError_t launch_moe_combine(const float* down, const int32_t* idx, const float* w, const int* route_pos,
                               const uint16_t* res, uint16_t* out, uint32_t T, uint32_t D, uint32_t K, uint32_t E,
                               cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  moe_combine_kernel<<<T, 160, 0, st>>>(down, idx, w, route_pos, res, out, T, D, K, E);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_exact(const float* gu, float* out, const int* n_rows_dev, uint32_t max_rows, uint32_t D,
                                cudaStream_t st) {
  if (max_rows == 0) return cudaSuccess;
  swiglu_exact_kernel<<<gs_blocks((size_t)max_rows * D, 256), 256, 0, st>>>(gu, out, n_rows_dev, max_rows, D);
  return cudaGetLastError();
}

cudaError_t launch_split_rope(const uint16_t* qkv, uint16_t* q, uint16_t* k, uint16_t* v, const int* pos,
                              const uint16_t* cos_t, const uint16_t* sin_t, uint32_t T, uint32_t qc, uint32_t kc,
                              uint32_t vc, uint32_t hd, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  split_rope_kernel<<<gs_blocks((size_t)T * (qc + kc + vc) / 2, 256), 256, 0, st>>>(qkv, q, k, v, pos, cos_t, sin_t, T,
                                                                                   qc, kc, vc, hd);
  return cudaGetLastError();
}

cudaError_t launch_f16_to_f32_ref(const uint16_t* src, float* dst, size_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  f16_to_f32_ref_kernel<<<gs_blocks(n, 256), 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_f16(const float* src, uint16_t* dst, size_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  f32_to_f16_kernel<<<gs_blocks(n, 256), 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_dequant_tiles(const uint8_t* blobs, uint32_t N, uint32_t K, uint32_t BN, uint32_t n_kc,
                                 uint16_t* out, cudaStream_t st) {
  dim3 grid(nblk(N, 128), n_kc);
  dequant_tiles_kernel<<<grid, 128, 0, st>>>(blobs, N, K, BN, n_kc, out);
  return cudaGetLastError();
}

}  // namespace ts
