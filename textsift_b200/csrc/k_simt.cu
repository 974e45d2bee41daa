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
//   router_topk       wasm_exports.zig:367-426 + 919-958, block.ts:98-102
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
  pdl_trigger();
  pdl_wait();
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
// One 32-block of an int4 embedding row (16 bytes pk, low nibble = even
// element) dequantised as the reference does (zig/wasm_exports.zig:1523-1570):
// f32 (q - zp) * scale, then its f32 -> fp16 encode.  Hardware round-to-
// nearest-even equals that encode for zero and normal fp16 results, so a
// pair takes one packed conversion and only pairs with a subnormal or
// overflowing value go through the reference routine.  q - zp is formed
// exactly as 2^23 + q (byte permute) minus 2^23 + zp.
__device__ __forceinline__ void embed_block_ref(uint4 pk, float s, int z, uint4* dst) {
  const uint32_t wd[4] = {pk.x, pk.y, pk.z, pk.w};
  const float off = 8388608.0f + (float)z;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const uint32_t lo4 = wd[q] & 0x0F0F0F0Fu, hi4 = (wd[q] >> 4) & 0x0F0F0F0Fu;
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {  // byte j of word q holds elements 8q+2j (lo) and 8q+2j+1 (hi)
      const float lo = __fmul_rn(__fsub_rn(__uint_as_float(__byte_perm(lo4, 0x4B000000u, 0x7650u | (uint32_t)j)), off), s);
      const float hi = __fmul_rn(__fsub_rn(__uint_as_float(__byte_perm(hi4, 0x4B000000u, 0x7650u | (uint32_t)j)), off), s);
      const float alo = fabsf(lo), ahi = fabsf(hi);
      const bool fast = (alo >= 6.103515625e-05f || alo == 0.0f) && alo < 65520.0f &&
                        (ahi >= 6.103515625e-05f || ahi == 0.0f) && ahi < 65520.0f;
      r[j] = fast ? f32x2_to_h2(lo, hi) : ((uint32_t)f32_to_f16_ref(lo) | ((uint32_t)f32_to_f16_ref(hi) << 16));
    }
    dst[q] = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

__global__ void embed_gather_kernel(const uint8_t* __restrict__ w, const uint16_t* __restrict__ sc,
                                    const uint8_t* __restrict__ zp, const int32_t* __restrict__ ids,
                                    uint16_t* __restrict__ out, uint32_t T, uint32_t V, uint32_t D) {
  pdl_trigger();
  pdl_wait();
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
  embed_block_ref(pk, s, z, o);
}

__global__ void embed_rows_kernel(const uint8_t* __restrict__ rows, uint32_t row_bytes, const int32_t* __restrict__ ids,
                                  uint16_t* __restrict__ out, uint32_t T, uint32_t V, uint32_t D) {
  pdl_trigger();
  pdl_wait();
  const uint32_t nb = D / 32;
  uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= T * nb) return;
  uint32_t t = gid / nb, b = gid % nb;
  int32_t id = ids[t];
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)t * D + b * 32);
  if (id < 0 || (uint32_t)id >= V) {
    for (int i = 0; i < 4; i++) o[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint8_t* row = rows + (size_t)id * row_bytes;
  const uint4 pk = *reinterpret_cast<const uint4*>(row + b * 16);
  const float s = f16_ref_to_f32(*reinterpret_cast<const uint16_t*>(row + D / 2 + 2 * b));
  const uint8_t zb = row[D / 2 + 2 * nb + (b >> 1)];
  const int z = (b & 1) ? (zb >> 4) & 15 : zb & 15;
  embed_block_ref(pk, s, z, o);
}

// Builds the packed table: one thread per (row, byte) of the packed row.
__global__ void embed_pack_kernel(const uint8_t* __restrict__ w, const uint16_t* __restrict__ sc,
                                  const uint8_t* __restrict__ zp, uint8_t* __restrict__ rows, uint32_t row_bytes,
                                  uint32_t V, uint32_t D) {
  const uint32_t nb = D / 32, zs = (nb + 1) / 2;
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)V * row_bytes) return;
  const uint32_t r = (uint32_t)(i / row_bytes), c = (uint32_t)(i % row_bytes);
  uint8_t v = 0;
  if (c < D / 2) v = w[(size_t)r * (D / 2) + c];
  else if (c < D / 2 + 2 * nb) v = reinterpret_cast<const uint8_t*>(sc + (size_t)r * nb)[c - D / 2];
  else if (c < D / 2 + 2 * nb + zs) v = zp[(size_t)r * zs + (c - D / 2 - 2 * nb)];
  rows[i] = v;
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
  extern __shared__ float rs_smem[];  // per warp: [D] f32 squared-sum source, [D] f32 value read back
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= T) return;
  float* xs = rs_smem + (size_t)warp * 2 * D;
  float* xr = xs + D;
  const size_t base = (size_t)row * D;
  // D is a multiple of 8: 16-byte accesses
  for (uint32_t c = lane; c < D / 8; c += 32) {
    const uint4 av = *reinterpret_cast<const uint4*>(a + base + 8 * c);
    const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
    uint32_t bw[4] = {0, 0, 0, 0}, sw[4];
    if constexpr (ADD) {
      const uint4 bv = *reinterpret_cast<const uint4*>(b + base + 8 * c);
      bw[0] = bv.x; bw[1] = bv.y; bw[2] = bv.z; bw[3] = bv.w;
    }
    float vs[8], vr[8];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      uint16_t s16[2] = {0, 0};
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        const float v = f16_ref_to_f32((uint16_t)(aw[j] >> (16 * hh)));
        if constexpr (ADD) {
          const float sv = __fadd_rn(v, f16_ref_to_f32((uint16_t)(bw[j] >> (16 * hh))));
          s16[hh] = f32_to_f16_fast(sv);
          vs[2 * j + hh] = sv;
          vr[2 * j + hh] = f16_ref_to_f32(s16[hh]);
        } else {
          vs[2 * j + hh] = v;
          vr[2 * j + hh] = v;
        }
      }
      sw[j] = (uint32_t)s16[0] | ((uint32_t)s16[1] << 16);
    }
    float4* xs4 = reinterpret_cast<float4*>(xs + 8 * c);
    float4* xr4 = reinterpret_cast<float4*>(xr + 8 * c);
    xs4[0] = make_float4(vs[0], vs[1], vs[2], vs[3]);
    xs4[1] = make_float4(vs[4], vs[5], vs[6], vs[7]);
    xr4[0] = make_float4(vr[0], vr[1], vr[2], vr[3]);
    xr4[1] = make_float4(vr[4], vr[5], vr[6], vr[7]);
    if constexpr (ADD) *reinterpret_cast<uint4*>(sum_out + base + 8 * c) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
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
  for (uint32_t c = lane; c < D / 4; c += 32) {
    const uint2 gv = *reinterpret_cast<const uint2*>(gamma + 4 * c);
    const uint16_t g[4] = {(uint16_t)(gv.x & 0xffffu), (uint16_t)(gv.x >> 16), (uint16_t)(gv.y & 0xffffu),
                           (uint16_t)(gv.y >> 16)};
    const float4 x4 = *reinterpret_cast<const float4*>(xr + 4 * c);
    const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; j++) y[j] = __fmul_rn(__fmul_rn(xv[j], inv_rms), f16_ref_to_f32(g[j]));
    if (out32) *reinterpret_cast<float4*>(out32 + base + 4 * c) = make_float4(y[0], y[1], y[2], y[3]);
    if (out16) {
      __half2 lo = __floats2half2_rn(y[0], y[1]), hi = __floats2half2_rn(y[2], y[3]);
      *reinterpret_cast<uint2*>(out16 + base + 4 * c) =
          make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    }
  }
}

// Shared-memory layout of the exact kernel: the 128-column weight tile
// (packed nibbles, rows padded so that eight consecutive rows hit distinct
// 16-byte bank groups), its scales and zero points, then two groups of 8
// activation rows in f32.
__host__ __device__ inline uint32_t exact_wstride(uint32_t K) { return (K / 2 + 31u) / 32u * 32u + 16u; }
__host__ __device__ inline size_t exact_smem_bytes(uint32_t K) {
  const size_t w = 128u * exact_wstride(K), sc = 128u * (K / 32) * 2u, zp = 128u * ((K / 32 + 1) / 2);
  return ((w + sc + zp + 15u) & ~size_t(15)) + 16u * K * sizeof(float);
}

template <bool X_F32, int OUT>
__global__ void __launch_bounds__(256) matmul_w4_exact_kernel(const ExactArgs a) {
  extern __shared__ __align__(16) uint8_t ex_smem[];
  const uint32_t K = a.K, nb = K / 32, zs = (nb + 1) / 2, wst = exact_wstride(K);
  uint8_t* sw = ex_smem;
  uint16_t* ssc = reinterpret_cast<uint16_t*>(ex_smem + 128u * wst);
  uint8_t* szp = ex_smem + 128u * wst + 128u * nb * 2u;
  float* xs = reinterpret_cast<float*>(ex_smem + ((128u * wst + 128u * nb * 2u + 128u * zs + 15u) & ~15u));
  uint32_t expert = 0, row0, row_end, seg_start = 0, seg_len = 0;
  const bool grouped = a.tiles != nullptr;
  if (grouped) {
    if ((int)blockIdx.y >= *a.n_tiles) return;
    int4 t = a.tiles[blockIdx.y];
    expert = (uint32_t)t.x; row0 = (uint32_t)t.y; row_end = (uint32_t)t.z; seg_start = (uint32_t)t.w;
    seg_len = (uint32_t)a.seg_end[expert] - seg_start;
  } else {
    row0 = blockIdx.y * a.rows_per_block;
    row_end = min(a.M, row0 + a.rows_per_block);
  }
  // ---- stage the weight tile of columns [n_base, n_base + 128) ----
  const uint32_t n_base = blockIdx.x * 128u;
  const uint32_t ncols = min(128u, a.N - n_base);
  {
    // every load of a thread's share is issued before its stores
    const uint8_t* w0 = a.w_int4 + (size_t)expert * a.w_int4_estride + (size_t)n_base * (K / 2);
    const uint32_t rowb = K / 2;  // a multiple of 16
    const uint32_t n16 = ncols * (rowb / 16);
#pragma unroll 1
    for (uint32_t i0 = threadIdx.x; i0 < n16; i0 += 4u * blockDim.x) {
      uint4 v[4];
#pragma unroll
      for (uint32_t u = 0; u < 4; u++) {
        const uint32_t i = i0 + u * blockDim.x, r = i / (rowb / 16), c = i % (rowb / 16);
        if (i < n16) v[u] = *reinterpret_cast<const uint4*>(w0 + (size_t)r * rowb + c * 16);
      }
#pragma unroll
      for (uint32_t u = 0; u < 4; u++) {
        const uint32_t i = i0 + u * blockDim.x, r = i / (rowb / 16), c = i % (rowb / 16);
        if (i < n16) *reinterpret_cast<uint4*>(sw + r * wst + c * 16) = v[u];
      }
    }
    // the tile's scales and zero points are contiguous in global memory
    const uint16_t* s0 = a.w_scales + (size_t)expert * a.w_scales_estride + (size_t)n_base * nb;
    const uint8_t* z0 = a.w_zp ? a.w_zp + (size_t)expert * a.w_zp_estride + (size_t)n_base * zs : nullptr;
    const uint32_t sbytes = ncols * nb * 2u, zbytes = z0 ? ncols * zs : 0u;
    if ((reinterpret_cast<uintptr_t>(s0) & 15u) == 0 && sbytes % 16u == 0) {
      for (uint32_t i = threadIdx.x; i < sbytes / 16u; i += blockDim.x)
        reinterpret_cast<uint4*>(ssc)[i] = reinterpret_cast<const uint4*>(s0)[i];
    } else {
      for (uint32_t i = threadIdx.x; i < ncols * nb; i += blockDim.x) ssc[i] = s0[i];
    }
    if (z0) {
      if ((reinterpret_cast<uintptr_t>(z0) & 15u) == 0 && zbytes % 16u == 0 &&
          (reinterpret_cast<uintptr_t>(szp) & 15u) == 0) {
        for (uint32_t i = threadIdx.x; i < zbytes / 16u; i += blockDim.x)
          reinterpret_cast<uint4*>(szp)[i] = reinterpret_cast<const uint4*>(z0)[i];
      } else {
        for (uint32_t i = threadIdx.x; i < zbytes; i += blockDim.x) szp[i] = z0[i];
      }
    }
  }
  const uint32_t half = threadIdx.x >> 7;  // which 8-row group of a pair this thread works on
  const uint32_t nl = threadIdx.x & 127u;
  const uint32_t n = n_base + nl;
  const bool n_ok = nl < ncols;
  const uint8_t* wr = sw + (size_t)(n_ok ? nl : 0) * wst;
  const uint16_t* sr = ssc + (size_t)(n_ok ? nl : 0) * nb;
  const uint8_t* zr = szp + (size_t)(n_ok ? nl : 0) * zs;
  const bool has_zp = a.w_zp != nullptr;
  const float bias = n_ok ? f16_ref_to_f32(a.bias[(size_t)expert * a.bias_estride + n]) : 0.0f;
  float* myx = xs + (size_t)half * 8 * K;
  // rows of x start on 16-byte boundaries: stage them 16 bytes at a time
  const bool vec_x = (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 && (a.ldx * (X_F32 ? 4u : 2u)) % 16u == 0;

  for (uint32_t gp = row0; gp < row_end; gp += 16) {
    __syncthreads();
    const uint32_t rows_pair = min(16u, row_end - gp);
    if (vec_x) {
      // 8-element pieces, 64 bytes per thread in flight before any is stored
      constexpr uint32_t kDepth = X_F32 ? 2u : 4u;
      const uint32_t ppr = K / 8u, n_pieces = rows_pair * ppr;
#pragma unroll 1
      for (uint32_t i0 = threadIdx.x; i0 < n_pieces; i0 += kDepth * blockDim.x) {
        uint4 raw[kDepth][X_F32 ? 2 : 1];
#pragma unroll
        for (uint32_t u = 0; u < kDepth; u++) {
          const uint32_t i = i0 + u * blockDim.x;
          if (i < n_pieces) {
            const uint32_t r = i / ppr, k = (i - r * ppr) * 8u;
            const size_t src = (size_t)(gp + r) * a.ldx + k;
            if constexpr (X_F32) {
              raw[u][0] = *reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(a.x) + src);
              raw[u][1] = *reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(a.x) + src + 4);
            } else {
              raw[u][0] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.x) + src);
            }
          }
        }
#pragma unroll
        for (uint32_t u = 0; u < kDepth; u++) {
          const uint32_t i = i0 + u * blockDim.x;
          if (i < n_pieces) {
            const uint32_t r = i / ppr, k = (i - r * ppr) * 8u;
            float4* dst = reinterpret_cast<float4*>(xs + r * K + k);
            if constexpr (X_F32) {
              dst[0] = *reinterpret_cast<const float4*>(&raw[u][0]);
              dst[1] = *reinterpret_cast<const float4*>(&raw[u][1]);
            } else {
              const uint32_t w[4] = {raw[u][0].x, raw[u][0].y, raw[u][0].z, raw[u][0].w};
              dst[0] = make_float4(f16_ref_to_f32((uint16_t)(w[0] & 0xffffu)), f16_ref_to_f32((uint16_t)(w[0] >> 16)),
                                   f16_ref_to_f32((uint16_t)(w[1] & 0xffffu)), f16_ref_to_f32((uint16_t)(w[1] >> 16)));
              dst[1] = make_float4(f16_ref_to_f32((uint16_t)(w[2] & 0xffffu)), f16_ref_to_f32((uint16_t)(w[2] >> 16)),
                                   f16_ref_to_f32((uint16_t)(w[3] & 0xffffu)), f16_ref_to_f32((uint16_t)(w[3] >> 16)));
            }
          }
        }
      }
    } else {
      for (uint32_t i = threadIdx.x; i < rows_pair * K; i += blockDim.x) {
        const uint32_t r = i / K, k = i % K;
        const size_t src = (size_t)(gp + r) * a.ldx + k;
        xs[r * K + k] = X_F32 ? reinterpret_cast<const float*>(a.x)[src]
                              : f16_ref_to_f32(reinterpret_cast<const uint16_t*>(a.x)[src]);
      }
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
      if (has_zp) { uint8_t zb = zr[b >> 1]; zp = (b & 1) ? (zb >> 4) & 15 : zb & 15; }
      const uint4 pk = *reinterpret_cast<const uint4*>(wr + b * 16);
      const uint32_t wd[4] = {pk.x, pk.y, pk.z, pk.w};
      // byte i holds elements 2i (low nibble) and 2i + 1: one f32 pair each,
      // q - zp exactly as (2^23 + q) - (2^23 + zp) in one packed add.
      // The chains below run two at a time as packed f32x2 fused multiply-adds
      // and adds (each half an IEEE operation: the same bits as scalar chains).
      const float nz = -(8388608.0f + (float)zp);
      const uint64_t nzz = f2pack(nz, nz);
      uint64_t q2[16];
#pragma unroll
      for (int w = 0; w < 4; w++) {
        const uint32_t lo = wd[w] & 0x0F0F0F0Fu, hi = (wd[w] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (uint32_t j = 0; j < 4; j++) q2[4 * w + j] = add_f32x2(f2pack(nib_raw(lo, j), nib_raw(hi, j)), nzz);
      }
#pragma unroll
      for (int r = 0; r < 8; r++) {
        if ((uint32_t)r >= gr) break;
        const ulonglong2* x4 = reinterpret_cast<const ulonglong2*>(myx + r * K + b * 32);
        float bs;
        if (tile_path[r]) {
          // v0..v3 over elements 4c + l: (v0, v1) and (v2, v3) as pairs
          uint64_t v01 = 0u, v23 = 0u;
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const ulonglong2 xv = x4[c];
            v01 = fma_f32x2(xv.x, q2[2 * c], v01);
            v23 = fma_f32x2(xv.y, q2[2 * c + 1], v23);
          }
          float v0, v1, v2, v3;
          f2unpack(v01, v0, v1);
          f2unpack(v23, v2, v3);
          bs = __fadd_rn(__fadd_rn(v0, v1), __fadd_rn(v2, v3));
        } else {
          // a0[l] over elements 8k + l, a1[l] over 8k + 4 + l, as pairs
          uint64_t a001 = 0u, a023 = 0u, a101 = 0u, a123 = 0u;
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const ulonglong2 x0 = x4[2 * k], x1 = x4[2 * k + 1];
            a001 = fma_f32x2(x0.x, q2[4 * k], a001);
            a023 = fma_f32x2(x0.y, q2[4 * k + 1], a023);
            a101 = fma_f32x2(x1.x, q2[4 * k + 2], a101);
            a123 = fma_f32x2(x1.y, q2[4 * k + 3], a123);
          }
          float c0, c1, c2, c3;
          f2unpack(add_f32x2(a001, a101), c0, c1);
          f2unpack(add_f32x2(a023, a123), c2, c3);
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
// Router top-k (wasm_exports.zig:367-426 + 919-958, block.ts:98-102): the
// k largest logits by (value descending, index ascending) -- exactly the set
// and order the reference's strict-'>' insertion sort produces -- then softmax
// over the k values in that order and x (1/k) in double like the JS caller.
// One warp per token (lane l holds logits l, l+32, ...), 128 tokens per block;
// each block also adds its routes per expert into the permutation chunk's
// row hist[token / kPermChunk][e].
// ---------------------------------------------------------------------------
constexpr uint32_t kRouteChunk = 128;  // tokens per top-k block
static_assert(kPermChunk % kRouteChunk == 0 && kPermChunk == 1024, "permutation chunk = 32 words of 32 tokens");
constexpr uint32_t kMaxExperts = 256;

// One warp per token: K rounds of a warp arg-max (value desc, index asc: the
// reference's insertion order, wasm_exports.zig:367-426) over SLOTS logits
// per lane, then the softmax over the K values in order
// (wasm_exports.zig:919-958) with the K exact exponentials computed at once
// on lanes 0..K-1.  hist: per-chunk expert counts for the permutation.
template <int SLOTS>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int32_t* __restrict__ idx,
                                                          float* __restrict__ w, int* __restrict__ hist, uint32_t T,
                                                          uint32_t E, uint32_t K, double inv_k) {
  __shared__ int h[kMaxExperts];
  for (uint32_t i = threadIdx.x; i < E; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t t0 = blockIdx.x * kRouteChunk;
  for (uint32_t tl = (uint32_t)warp; tl < kRouteChunk; tl += blockDim.x >> 5) {
    const uint32_t t = t0 + tl;
    if (t >= T) break;
    const float* row = logits + (size_t)t * E;
    float v[SLOTS];
    bool avail[SLOTS];
#pragma unroll
    for (int j = 0; j < SLOTS; j++) {
      const uint32_t c = lane + 32 * j;
      avail[j] = c < E;
      v[j] = avail[j] ? row[c] : 0.0f;
    }
    float ov[8];
    int oi[8];
#pragma unroll
    for (uint32_t k = 0; k < 8; k++) {
      ov[k] = 0.0f;
      oi[k] = 0;
      if (k >= K) continue;
      float bv = 0.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < SLOTS; j++) {
        const int c = lane + 32 * j;
        if (avail[j] && (bi == 0x7fffffff || v[j] > bv || (v[j] == bv && c < bi))) { bv = v[j]; bi = c; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ovv = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oii = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oii != 0x7fffffff && (bi == 0x7fffffff || ovv > bv || (ovv == bv && oii < bi))) { bv = ovv; bi = oii; }
      }
      ov[k] = bv;
      oi[k] = bi;
#pragma unroll
      for (int j = 0; j < SLOTS; j++)
        if (lane + 32 * j == bi) avail[j] = false;
    }
    float m = ov[0];
    for (uint32_t c = 1; c < K; c++) if (ov[c] > m) m = ov[c];
    // lane c < K: exp of entry c (one exact exponential per lane, no divergence)
    float mine = ov[0];
#pragma unroll
    for (int c = 1; c < 8; c++)
      if (lane == c) mine = ov[c];
    const float my_e = expf_ref(__fsub_rn(mine, m));
    float e[8];
#pragma unroll
    for (uint32_t c = 0; c < 8; c++) e[c] = __shfl_sync(0xffffffffu, my_e, c);
    if (lane == 0) {
      float sum = 0.0f;
      for (uint32_t c = 0; c < K; c++) sum = __fadd_rn(sum, e[c]);
      const float inv = sum > 0.0f ? __fdiv_rn(1.0f, sum) : __fdiv_rn(1.0f, (float)K);
      for (uint32_t c = 0; c < K; c++) {
        idx[(size_t)t * K + c] = oi[c];
        w[(size_t)t * K + c] = (float)((double)__fmul_rn(e[c], inv) * inv_k);
        atomicAdd(&h[oi[c]], 1);
      }
    }
  }
  __syncthreads();
  if (hist) {
    int* row = hist + (size_t)(blockIdx.x / (kPermChunk / kRouteChunk)) * E;
    for (uint32_t i = threadIdx.x; i < E; i += blockDim.x)
      if (h[i]) atomicAdd(row + i, h[i]);
  }
}

// ---------------------------------------------------------------------------
// MoE permutation, stable (ascending token within each expert, the order
// expert.ts:137-145 builds), over chunks of kPermChunk tokens whose expert
// counts the router's top-k left in hist[chunk][e].  scan: one block turns
// hist into each (chunk, expert)'s base position inside the expert's segment,
// then the expert segments, their GEMM tiles and the tile counts.  place: one
// block per chunk; a route's rank inside its chunk is the number of earlier
// tokens of the chunk that chose the same expert (a 1024-bit token mask per
// expert with per-word prefix counts).
// ---------------------------------------------------------------------------
// Exclusive prefix sum of one int per thread over the block (warp shuffles,
// then the warp totals in warp_tot[blockDim.x / 32]).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int base = 0;
  for (int i = 0; i < warp; i++) base += warp_tot[i];
  __syncthreads();  // warp_tot may be reused by the caller
  return base + incl - v;
}

// One block of 1024 threads: G = 1024 / E threads per expert each sum a run
// of chunks, then rewrite hist[c][e] as the exclusive prefix over chunks; the
// expert totals (counts) give the segments, the 128-row GEMM tiles (exact
// path), the rows_tc-row tiles (tensor-core path) and both tile counts.
__global__ void __launch_bounds__(1024) moe_scan_segments_kernel(int* __restrict__ hist, uint32_t n_chunks, uint32_t E,
                                                                 int* __restrict__ counts, int4* __restrict__ tiles,
                                                                 int* __restrict__ n_tiles, int4* __restrict__ tiles_tc,
                                                                 int* __restrict__ n_tiles_tc, int rows_tc,
                                                                 int* __restrict__ seg_start,
                                                                 int* __restrict__ seg_end) {
  pdl_trigger();
  pdl_wait();
  __shared__ int part[1024];
  __shared__ int wt[32];
  const uint32_t G = 1024u / E, tid = threadIdx.x;
  const uint32_t e = tid % E, g = tid / E;
  const bool act = g < G;
  const uint32_t L = (n_chunks + G - 1) / G;
  const uint32_t c0 = min(n_chunks, g * L), c1 = min(n_chunks, c0 + L);
  // the chunk counts eight at a time: loads in flight together, then summed
  int s = 0;
  if (act)
    for (uint32_t c = c0; c < c1; c += 8) {
      int v[8];
#pragma unroll
      for (uint32_t u = 0; u < 8; u++) v[u] = c + u < c1 ? hist[(size_t)(c + u) * E + e] : 0;
#pragma unroll
      for (uint32_t u = 0; u < 8; u++) s += v[u];
    }
  part[tid] = s;
  __syncthreads();
  int run = 0, total = 0;
  if (act) {
    for (uint32_t gg = 0; gg < G; gg++) {
      const int v = part[gg * E + e];
      if (gg < g) run += v;
      total += v;
    }
    for (uint32_t c = c0; c < c1; c += 8) {
      int v[8];
#pragma unroll
      for (uint32_t u = 0; u < 8; u++) v[u] = c + u < c1 ? hist[(size_t)(c + u) * E + e] : 0;
#pragma unroll
      for (uint32_t u = 0; u < 8; u++) {
        if (c + u < c1) hist[(size_t)(c + u) * E + e] = run;
        run += v[u];
      }
    }
  }
  // expert e's total sits with thread e (g == 0)
  const int cnt = tid < E ? total : 0;
  if (tid < E) counts[e] = cnt;
  const int t1 = (cnt + 127) / 128, t2 = (cnt + rows_tc - 1) / rows_tc;
  const int base = block_exclusive_scan(cnt, wt);
  const int tb1 = block_exclusive_scan(t1, wt);
  const int tb2 = block_exclusive_scan(t2, wt);
  if (tid < E) {
    seg_start[e] = base;
    seg_end[e] = base + cnt;
    for (int tt = 0; tt < t1; tt++)
      tiles[tb1 + tt] = make_int4((int)e, base + tt * 128, base + min(cnt, tt * 128 + 128), base);
    if (tiles_tc)
      for (int tt = 0; tt < t2; tt++)
        tiles_tc[tb2 + tt] = make_int4((int)e, base + tt * rows_tc, base + min(cnt, (tt + 1) * rows_tc), base);
  }
  if (tid == E - 1) {
    *n_tiles = tb1 + t1;
    if (n_tiles_tc) *n_tiles_tc = tb2 + t2;
  }
}

__global__ void __launch_bounds__(kPermChunk) moe_place_kernel(const int32_t* __restrict__ idx,
                                                               int* __restrict__ hist,
                                                               const int* __restrict__ seg_start, uint32_t T,
                                                               uint32_t K, uint32_t E, int* __restrict__ perm_tok,
                                                               int* __restrict__ route_pos) {
  constexpr uint32_t kWords = kPermChunk / 32;
  __shared__ uint32_t mask[kMaxExperts][kWords];  // bit b of word w: token 32 w + b chose the expert
  __shared__ uint16_t pref[kMaxExperts][kWords];  // the expert's tokens in words < w
  pdl_trigger();
  pdl_wait();
  const uint32_t tl = threadIdx.x, t = blockIdx.x * kPermChunk + tl;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (uint32_t i = threadIdx.x; i < E * kWords; i += blockDim.x) mask[i / kWords][i % kWords] = 0;
  __syncthreads();
  int ek[8];
  const bool ok = t < T;
  for (uint32_t k = 0; k < K; k++) {
    ek[k] = ok ? idx[(size_t)t * K + k] : -1;
    if (ek[k] >= 0 && (uint32_t)ek[k] < E) atomicOr(&mask[ek[k]][tl >> 5], 1u << (tl & 31));
  }
  __syncthreads();
  // per expert, one warp scans the popcounts of its 32 words (lane = word)
  for (uint32_t x = (uint32_t)warp; x < E; x += blockDim.x >> 5) {
    const int c = __popc(mask[x][lane]);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    pref[x][lane] = (uint16_t)(incl - c);
  }
  __syncthreads();
  for (uint32_t k = 0; k < K && ok; k++) {
    const int e = ek[k];
    if (e < 0 || (uint32_t)e >= E) { route_pos[(size_t)t * K + k] = -1; continue; }
    const int rank = (int)pref[e][tl >> 5] + __popc(mask[e][tl >> 5] & ((1u << (tl & 31)) - 1u));
    const int p = seg_start[e] + hist[(size_t)blockIdx.x * E + e] + rank;
    perm_tok[p] = (int)t;
    route_pos[(size_t)t * K + k] = p;
  }
  // this chunk's row is consumed: leave it zero for the next top-k, which
  // accumulates expert counts into it
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < E; i += blockDim.x) hist[(size_t)blockIdx.x * E + i] = 0;
}

// dst[p, :] = src[perm_tok[p], :] (row bytes a multiple of 16)
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                   const int* __restrict__ perm_tok, const int* __restrict__ n_rows_dev,
                                   uint32_t n_rows, uint32_t row_bytes) {
  pdl_trigger();
  pdl_wait();
  const uint32_t rows = n_rows_dev ? (uint32_t)*n_rows_dev : n_rows;
  const uint32_t per_row = row_bytes / 16, total = rows * per_row;
  const uint32_t stride = gridDim.x * blockDim.x;
  // four independent 16-byte pieces per thread and pass: every load out
  // before the first store; the stores stream past L2 (evict-first) so the
  // source rows, read once per route, stay resident
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += 4u * stride) {
    uint4 v[4];
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
      const uint32_t j = i + k * stride;
      if (j < total) {
        const uint32_t p = j / per_row, c = j - p * per_row;
        v[k] = __ldg(reinterpret_cast<const uint4*>(src + (size_t)perm_tok[p] * row_bytes) + c);
      }
    }
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
      const uint32_t j = i + k * stride;
      if (j < total) {
        const uint32_t p = j / per_row, c = j - p * per_row;
        __stcs(reinterpret_cast<uint4*>(dst + (size_t)p * row_bytes) + c, v[k]);
      }
    }
  }
}

// The same gather for rows of 80 or 160 16-byte pieces (1280 / 2560 bytes:
// the forward's fp16 and f32 expert operands): a warp moves 160 pieces per
// pass -- two rows of 80 or one of 160 -- lane l the pieces l, l + 32, ...,
// with the rows' source indices loaded once and all five loads of a lane
// issued before its stores (no per-piece division or index load).
template <uint32_t P>
__global__ void gather_rows_warp_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                        const int* __restrict__ perm_tok, const int* __restrict__ n_rows_dev,
                                        uint32_t n_rows) {
  static_assert(P == 80 || P == 160, "two rows of 80 pieces or one of 160 per warp pass");
  constexpr uint32_t RW = 160 / P;
  pdl_trigger();
  pdl_wait();
  const uint32_t rows = n_rows_dev ? (uint32_t)*n_rows_dev : n_rows;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t r0 = gw * RW; r0 < rows; r0 += nw * RW) {
    const int s0 = perm_tok[r0];
    const int s1 = RW > 1 && r0 + 1 < rows ? perm_tok[r0 + 1] : 0;
    uint4 v[5];
#pragma unroll
    for (uint32_t u = 0; u < 5; u++) {
      const uint32_t q = lane + 32u * u, k = q / P, c = q - k * P;
      if (r0 + k < rows)
        v[u] = __ldg(reinterpret_cast<const uint4*>(src + (size_t)(k ? s1 : s0) * (P * 16u)) + c);
    }
#pragma unroll
    for (uint32_t u = 0; u < 5; u++) {
      const uint32_t q = lane + 32u * u, k = q / P, c = q - k * P;
      if (r0 + k < rows) __stcs(reinterpret_cast<uint4*>(dst + (size_t)(r0 + k) * (P * 16u)) + c, v[u]);
    }
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
  for (uint32_t c = threadIdx.x; c < D / 4; c += blockDim.x) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t j = 0; j < n; j++) {
      const float4 v = *reinterpret_cast<const float4*>(down + (size_t)pk[j] * D + 4 * c);
      acc[0] = __fmaf_rn(wk[j], v.x, acc[0]);
      acc[1] = __fmaf_rn(wk[j], v.y, acc[1]);
      acc[2] = __fmaf_rn(wk[j], v.z, acc[2]);
      acc[3] = __fmaf_rn(wk[j], v.w, acc[3]);
    }
    const size_t o = (size_t)t * D + 4 * c;
    uint16_t r16[4];
    if (res) {
      const uint2 rv = *reinterpret_cast<const uint2*>(res + o);
      r16[0] = (uint16_t)(rv.x & 0xffffu); r16[1] = (uint16_t)(rv.x >> 16);
      r16[2] = (uint16_t)(rv.y & 0xffffu); r16[3] = (uint16_t)(rv.y >> 16);
    }
    uint16_t o16[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint16_t m16 = f32_to_f16_fast(__fmul_rn(acc[j], kf));
      o16[j] = res ? f32_to_f16_fast(__fadd_rn(f16_ref_to_f32(r16[j]), f16_ref_to_f32(m16))) : m16;
    }
    *reinterpret_cast<uint2*>(out + o) =
        make_uint2((uint32_t)o16[0] | ((uint32_t)o16[1] << 16), (uint32_t)o16[2] | ((uint32_t)o16[3] << 16));
  }
}

// ---------------------------------------------------------------------------
// Fast-mode (tensor-core path) norms and combine: any summation order,
// hardware round-to-nearest-even conversions, everything held in registers.
// ---------------------------------------------------------------------------

// One warp per row, D <= 1024 and a multiple of 8.  With ADD: sum_out =
// fp16(a + b); the squares are taken of the f32 sum and the normalised value
// is the fp16-rounded sum (as in the reference-order kernel above).
template <bool ADD>
__global__ void __launch_bounds__(256) rmsnorm_fast_kernel(const uint16_t* __restrict__ a,
                                                           const uint16_t* __restrict__ b,
                                                           const uint16_t* __restrict__ gamma,
                                                           uint16_t* __restrict__ sum_out,
                                                           uint16_t* __restrict__ out16, uint32_t T, uint32_t D,
                                                           float eps, float* __restrict__ absum,
                                                           float* __restrict__ inv_out, float* __restrict__ out32) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= T) return;
  const uint32_t nc = D / 8;
  const size_t base = (size_t)row * D;
  uint4 xr[4];  // the value to normalise (fp16x2 words), chunks lane, lane+32, ...
  float ss = 0.0f;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const uint32_t c = (uint32_t)lane + 32u * r;
    if (c >= nc) break;
    uint4 av = *reinterpret_cast<const uint4*>(a + base + 8 * c);
    if constexpr (ADD) {
      const uint4 bv = *reinterpret_cast<const uint4*>(b + base + 8 * c);
      uint32_t aw[4] = {av.x, av.y, av.z, av.w};
      const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&aw[j]));
        const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&bw[j]));
        const float s0 = fa.x + fb.x, s1 = fa.y + fb.y;
        ss = fmaf(s0, s0, ss);
        ss = fmaf(s1, s1, ss);
        aw[j] = f32x2_to_h2(s0, s1);
      }
      av = make_uint4(aw[0], aw[1], aw[2], aw[3]);
      *reinterpret_cast<uint4*>(sum_out + base + 8 * c) = av;
    } else {
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&aw[j]));
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
    xr[r] = av;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv_rms = rsqrtf(ss / (float)D + eps);
  if (inv_out && lane == 0) inv_out[row] = inv_rms;  // the router's exact pass rebuilds its input from it
  float as = 0.0f;  // sum of |normalised value| (the router's error bound, k_router.cu)
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const uint32_t c = (uint32_t)lane + 32u * r;
    if (c >= nc) break;
    const uint4 gv = *reinterpret_cast<const uint4*>(gamma + 8 * c);
    const uint32_t xw[4] = {xr[r].x, xr[r].y, xr[r].z, xr[r].w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t ow[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&xw[j]));
      const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&gw[j]));
      const float n0 = x.x * inv_rms * g.x, n1 = x.y * inv_rms * g.y;
      as += fabsf(n0) + fabsf(n1);
      ow[j] = f32x2_to_h2(n0, n1);
      if (out32) *reinterpret_cast<float2*>(out32 + base + 8 * c + 2 * j) = make_float2(n0, n1);
    }
    *reinterpret_cast<uint4*>(out16 + base + 8 * c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
  if (absum) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) as += __shfl_xor_sync(0xffffffffu, as, o);
    if (lane == 0) absum[row] = as;
  }
}

// MoE combine from fp16 expert outputs, one warp per token: lanes 0..K-1
// read the token's routes and order them by expert id (ties by slot), the
// warp then streams the rows in 8-column chunks: acc = sum over the experts
// in ascending id of w * v (fma, from 0); out = fp16(res + fp16(acc * K))
// (or fp16(acc * K) without a residual).
template <int KMAX>
__global__ void __launch_bounds__(256, 4) moe_combine_fast_kernel(const uint16_t* __restrict__ down,
                                                               const int32_t* __restrict__ idx,
                                                               const float* __restrict__ w,
                                                               const int* __restrict__ route_pos,
                                                               const uint16_t* __restrict__ res,
                                                               uint16_t* __restrict__ out, uint32_t T, uint32_t D,
                                                               uint32_t K, uint32_t E,
                                                               const uint16_t* __restrict__ norm_gamma,
                                                               uint16_t* __restrict__ norm_out, float eps) {
  pdl_trigger();
  pdl_wait();
  const uint32_t t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  int my_e = 0x7fffffff, my_p = 0;
  float my_w = 0.0f;
  if ((uint32_t)lane < K) {
    const int e = idx[(size_t)t * K + lane];
    if (e >= 0 && (uint32_t)e < E) {
      my_e = e;
      my_w = w[(size_t)t * K + lane];
      my_p = route_pos[(size_t)t * K + lane];
    }
  }
  // rank of this lane's route among the valid ones: (expert id, slot) order
  int rank = 0, n = 0;
#pragma unroll
  for (int j = 0; j < KMAX; j++) {
    const int ej = __shfl_sync(0xffffffffu, my_e, j);
    if ((uint32_t)j < K && ej != 0x7fffffff) {
      n++;
      rank += (ej < my_e || (ej == my_e && j < lane)) ? 1 : 0;
    }
  }
  int pk[KMAX];
  float wk[KMAX];
#pragma unroll
  for (int r = 0; r < KMAX; r++) {
    // the lane whose route has rank r
    const unsigned sel = __ballot_sync(0xffffffffu, (uint32_t)lane < K && my_e != 0x7fffffff && rank == r);
    const int src = sel ? __ffs(sel) - 1 : 0;
    pk[r] = __shfl_sync(0xffffffffu, my_p, src);
    wk[r] = __shfl_sync(0xffffffffu, my_w, src);
  }
  const float kf = (float)K;
  const uint32_t nc = D / 8;
  float ss = 0.0f;  // sum of squares of this lane's outputs, in rmsnorm_fast_kernel's order
#pragma unroll 1
  for (uint32_t c = (uint32_t)lane; c < nc; c += 32) {
    // every route's 16 bytes (and the residual's) in flight before the math
    const size_t o = (size_t)t * D + 8 * c;
    uint4 vv[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; j++)
      vv[j] = j < n ? __ldg(reinterpret_cast<const uint4*>(down + (size_t)pk[j] * D + 8 * c)) : make_uint4(0, 0, 0, 0);
    const uint4 rv = res ? __ldg(reinterpret_cast<const uint4*>(res + o)) : make_uint4(0, 0, 0, 0);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
      if (j >= n) break;
      const uint32_t vw[4] = {vv[j].x, vv[j].y, vv[j].z, vv[j].w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&vw[q]));
        acc[2 * q] = fmaf(wk[j], f.x, acc[2 * q]);
        acc[2 * q + 1] = fmaf(wk[j], f.y, acc[2 * q + 1]);
      }
    }
    uint32_t ow[4];
    if (res) {
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint32_t m = f32x2_to_h2(acc[2 * q] * kf, acc[2 * q + 1] * kf);
        const float2 mf = __half22float2(*reinterpret_cast<const __half2*>(&m));
        const float2 rf = __half22float2(*reinterpret_cast<const __half2*>(&rw[q]));
        ow[q] = f32x2_to_h2(rf.x + mf.x, rf.y + mf.y);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; q++) ow[q] = f32x2_to_h2(acc[2 * q] * kf, acc[2 * q + 1] * kf);
    }
    *reinterpret_cast<uint4*>(out + o) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    if (norm_gamma) {
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ow[q]));
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  }
  if (!norm_gamma) return;
  // the next RMSNorm of this token's new residual, exactly as rmsnorm_fast_kernel<false>
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv_rms = rsqrtf(ss / (float)D + eps);
  // each lane reads back the chunks it wrote above (L2-resident): cheaper than
  // holding them in registers across the loop, which halves the occupancy
#pragma unroll 1
  for (uint32_t c = (uint32_t)lane; c < nc; c += 32) {
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(norm_gamma + 8 * c));
    const uint4 xv = *reinterpret_cast<const uint4*>(out + (size_t)t * D + 8 * c);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t nw[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&xw[j]));
      const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&gw[j]));
      nw[j] = f32x2_to_h2(x.x * inv_rms * g.x, x.y * inv_rms * g.y);
    }
    *reinterpret_cast<uint4*>(norm_out + (size_t)t * D + 8 * c) = make_uint4(nw[0], nw[1], nw[2], nw[3]);
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
    const uint32_t ab = *reinterpret_cast<const uint32_t*>(qkv + (size_t)t * W + c);
    uint16_t a16 = (uint16_t)(ab & 0xffffu), b16 = (uint16_t)(ab >> 16);
    if (c < qc + kc) {
      const uint32_t p = (c % hd) / 2;
      rope_pair_ref(a16, b16, cos_t[(size_t)pos[t] * half + p], sin_t[(size_t)pos[t] * half + p]);
    }
    uint16_t* dst;
    uint32_t col, ld;
    if (c < qc) { dst = q; col = c; ld = qc; }
    else if (c < qc + kc) { dst = k; col = c - qc; ld = kc; }
    else { dst = v; col = c - qc - kc; ld = vc; }
    if (dst) *reinterpret_cast<uint32_t*>(dst + (size_t)t * ld + col) = (uint32_t)a16 | ((uint32_t)b16 << 16);
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
  return launch_pdl(seq_info_kernel, dim3(nblk(T, 256)), dim3(256), 0, st, offs, n_seqs, T, pos, sstart, slen);
}

uint32_t embed_row_bytes(uint32_t D) { return (D / 2 + 2 * (D / 32) + (D / 32 + 1) / 2 + 127) & ~127u; }

cudaError_t launch_embed_pack(const uint8_t* w, const uint16_t* sc, const uint8_t* zp, uint8_t* rows, uint32_t V,
                              uint32_t D, cudaStream_t st) {
  const size_t n = (size_t)V * embed_row_bytes(D);
  if (n == 0) return cudaSuccess;
  embed_pack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, sc, zp, rows, embed_row_bytes(D), V, D);
  return cudaGetLastError();
}

cudaError_t launch_embed_rows(const uint8_t* rows, const int32_t* ids, uint16_t* out, uint32_t T, uint32_t V,
                              uint32_t D, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  return launch_pdl(embed_rows_kernel, dim3(nblk((size_t)T * (D / 32), 128)), dim3(128), 0, st, rows,
                    embed_row_bytes(D), ids, out, T, V, D);
}

cudaError_t launch_embed(const uint8_t* w, const uint16_t* sc, const uint8_t* zp, const int32_t* ids, uint16_t* out,
                         uint32_t T, uint32_t V, uint32_t D, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  return launch_pdl(embed_gather_kernel, dim3(nblk((size_t)T * (D / 32), 128)), dim3(128), 0, st, w, sc, zp, ids, out, T,
                    V, D);
}

cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* gamma, float* out32, uint16_t* out16, uint32_t T,
                           uint32_t D, float eps, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  const unsigned warps = 4;
  rmsnorm_kernel<false><<<nblk(T, warps), warps * 32, warps * 2 * D * sizeof(float), st>>>(
      x, nullptr, gamma, nullptr, out32, out16, T, D, eps);
  return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, uint16_t* sum_out,
                               float* out32, uint16_t* out16, uint32_t T, uint32_t D, float eps, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  const unsigned warps = 4;
  rmsnorm_kernel<true><<<nblk(T, warps), warps * 32, warps * 2 * D * sizeof(float), st>>>(a, b, gamma, sum_out, out32,
                                                                                         out16, T, D, eps);
  return cudaGetLastError();
}

cudaError_t launch_matmul_exact(const ExactArgs& a_in, bool x_f32, int out_mode, uint32_t grid_m, cudaStream_t st) {
  if (grid_m == 0) return cudaSuccess;
  if (a_in.K % 32 || a_in.K > 1024) return cudaErrorInvalidValue;
  ExactArgs a = a_in;
  if (a.rows_per_block == 0) a.rows_per_block = 128;
  if (!a.tiles) grid_m = (a.M + a.rows_per_block - 1) / a.rows_per_block;
  dim3 grid(nblk(a.N, 128), grid_m);
  const size_t sm = exact_smem_bytes(a.K);
  if (sm > 227 * 1024) return cudaErrorInvalidValue;
  // the largest limit set so far on each device (function attributes belong
  // to a device's context); devices past 63 set it on every call
  static std::atomic<size_t> attr_bytes[64];
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
  if (sm > 48 * 1024 && (dev < 0 || dev >= 64 || sm > attr_bytes[dev].load(std::memory_order_relaxed))) {
    const int v = (int)sm;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(matmul_w4_exact_kernel<true, kOutF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, v)) ||
        (e = cudaFuncSetAttribute(matmul_w4_exact_kernel<true, kOutF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, v)) ||
        (e = cudaFuncSetAttribute(matmul_w4_exact_kernel<true, kOutF16Widen>, cudaFuncAttributeMaxDynamicSharedMemorySize, v)) ||
        (e = cudaFuncSetAttribute(matmul_w4_exact_kernel<false, kOutF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, v)) ||
        (e = cudaFuncSetAttribute(matmul_w4_exact_kernel<false, kOutF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, v)))
      return e;
    if (dev >= 0 && dev < 64) attr_bytes[dev].store(sm, std::memory_order_relaxed);
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

uint32_t route_chunks(uint32_t T) { return (T + kPermChunk - 1) / kPermChunk; }

cudaError_t launch_router_topk(const float* logits, int32_t* idx, float* w, int* hist, uint32_t T, uint32_t E,
                               uint32_t K, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (K > 8 || K > E || E > kMaxExperts) return cudaErrorInvalidValue;
  const uint32_t blocks = (T + kRouteChunk - 1) / kRouteChunk;
  if (E <= 128)
    router_topk_kernel<4><<<blocks, 256, 0, st>>>(logits, idx, w, hist, T, E, K, 1.0 / (double)K);
  else
    router_topk_kernel<kMaxExperts / 32><<<blocks, 256, 0, st>>>(logits, idx, w, hist, T, E, K, 1.0 / (double)K);
  return cudaGetLastError();
}

cudaError_t launch_moe_permute(const int32_t* idx, int* hist, uint32_t T, uint32_t K, uint32_t E, int* counts,
                               int* perm_tok, int* route_pos, int4* tiles, int* n_tiles, int4* tiles_tc,
                               int* n_tiles_tc, uint32_t rows_tc, int* seg_start, int* seg_end, cudaStream_t st) {
  if (E > kMaxExperts || K > 8 || (tiles_tc && rows_tc == 0)) return cudaErrorInvalidValue;
  if (T == 0 || E == 0) return cudaSuccess;
  const uint32_t nc = route_chunks(T);
  cudaError_t e = launch_pdl(moe_scan_segments_kernel, dim3(1), dim3(1024), 0, st, hist, nc, E, counts, tiles, n_tiles,
                             tiles_tc, n_tiles_tc, (int)rows_tc, seg_start, seg_end);
  if (e != cudaSuccess) return e;
  return launch_pdl(moe_place_kernel, dim3(nc), dim3(kPermChunk), 0, st, idx, hist, seg_start, T, K, E, perm_tok,
                    route_pos);
}

cudaError_t launch_gather_rows(const void* src, void* dst, const int* perm_tok, const int* n_rows_dev,
                               uint32_t max_rows, uint32_t row_bytes, cudaStream_t st) {
  if (max_rows == 0) return cudaSuccess;
  if (row_bytes == 1280u || row_bytes == 2560u) {
    const uint32_t rw = row_bytes == 1280u ? 2u : 1u;  // rows per warp pass
    const unsigned blocks = gs_blocks(((size_t)max_rows + rw - 1) / rw * 32u, 256);
    if (row_bytes == 1280u)
      return launch_pdl(gather_rows_warp_kernel<80>, dim3(blocks), dim3(256), 0, st, (const uint8_t*)src,
                        (uint8_t*)dst, perm_tok, n_rows_dev, max_rows);
    return launch_pdl(gather_rows_warp_kernel<160>, dim3(blocks), dim3(256), 0, st, (const uint8_t*)src,
                      (uint8_t*)dst, perm_tok, n_rows_dev, max_rows);
  }
  return launch_pdl(gather_rows_kernel, dim3(gs_blocks((size_t)max_rows * row_bytes / 16, 256)), dim3(256), 0, st,
                    (const uint8_t*)src, (uint8_t*)dst, perm_tok, n_rows_dev, max_rows, row_bytes);
}

cudaError_t launch_moe_combine(const float* down, const int32_t* idx, const float* w, const int* route_pos,
                               const uint16_t* res, uint16_t* out, uint32_t T, uint32_t D, uint32_t K, uint32_t E,
                               cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (D % 4) return cudaErrorInvalidValue;
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

cudaError_t launch_rmsnorm_fast(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, uint16_t* sum_out,
                                uint16_t* out16, uint32_t T, uint32_t D, float eps, cudaStream_t st, float* absum,
                                float* inv_out, float* out32) {
  if (T == 0) return cudaSuccess;
  if (D % 8 || D > 1024 || !out16 || (b && !sum_out)) return cudaErrorInvalidValue;
  const uint32_t blocks = (T + 7) / 8;
  if (b)
    return launch_pdl(rmsnorm_fast_kernel<true>, dim3(blocks), dim3(256), 0, st, a, b, gamma, sum_out, out16, T, D, eps,
                      absum, inv_out, out32);
  return launch_pdl(rmsnorm_fast_kernel<false>, dim3(blocks), dim3(256), 0, st, a, (const uint16_t*)nullptr, gamma,
                    (uint16_t*)nullptr, out16, T, D, eps, absum, inv_out, out32);
}

cudaError_t launch_moe_combine_fast(const uint16_t* down, const int32_t* idx, const float* w, const int* route_pos,
                                    const uint16_t* res, uint16_t* out, uint32_t T, uint32_t D, uint32_t K,
                                    uint32_t E, const uint16_t* norm_gamma, uint16_t* norm_out, float eps,
                                    cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (D % 8 || K > 8 || D > 8 * 32 * 4 || (norm_gamma && !norm_out)) return cudaErrorInvalidValue;
  if (K <= 4)
    return launch_pdl(moe_combine_fast_kernel<4>, dim3((T + 7) / 8), dim3(256), 0, st, down, idx, w, route_pos, res, out,
                      T, D, K, E, norm_gamma, norm_out, eps);
  return launch_pdl(moe_combine_fast_kernel<8>, dim3((T + 7) / 8), dim3(256), 0, st, down, idx, w, route_pos, res, out, T,
                    D, K, E, norm_gamma, norm_out, eps);
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
