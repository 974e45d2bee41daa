// k_attn.cu — banded bidirectional GQA attention with sinks.
//
// Reference: packages/textsift/src/zig/wasm_exports.zig:1286-1379
// (bandedAttentionBody).  For query t of a sequence of length L and head h:
//   keys ws..we-1 with ws = max(0, t-W), we = min(L, t+W+1)  (n_keys = we-ws)
//   score = q . k (no 1/sqrt(d) scale), padding keys -> -inf
//   softmax over [scores..., sink_h]; entries 0..4*floor((n_keys+1)/4)-1 use
//   the reference's polynomial exp, the remaining 0-3 entries (the sink may
//   be one of them) use exp; out = sum_j p_j v_j (sink excluded), fp16 RNE.
//
// attn_exact_kernel   CUDA cores, the reference's exact summation order
//                     (bit-identical for identical inputs up to expf ulps).
// attn_tc_kernel      mma.sync m16n8k16 (fp16 in, f32 accumulate): one CTA
//                     per (16 queries, KV head) with one warp per query head
//                     of the GQA group sharing the K/V band staged in smem.
//                     Two passes over the band: row max, then
//                     exp/sum/P.V with the same per-index exp choice.
#include "ts_common.cuh"
#include "ts_simt.h"

#include <climits>
#include <cmath>

namespace ts {

// wasm_exports.zig:1232-1267
__device__ __forceinline__ float dot_ref(const uint16_t* a, const uint16_t* b, uint32_t n) {
  float acc[4][4];
#pragma unroll
  for (int u = 0; u < 4; u++)
#pragma unroll
    for (int l = 0; l < 4; l++) acc[u][l] = 0.0f;
  uint32_t i = 0;
  for (; i + 16 <= n; i += 16)
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int l = 0; l < 4; l++)
        acc[u][l] = __fmaf_rn(f16_ref_to_f32(a[i + 4 * u + l]), f16_ref_to_f32(b[i + 4 * u + l]), acc[u][l]);
  for (; i + 4 <= n; i += 4)
#pragma unroll
    for (int l = 0; l < 4; l++) acc[0][l] = __fmaf_rn(f16_ref_to_f32(a[i + l]), f16_ref_to_f32(b[i + l]), acc[0][l]);
  float c[4];
#pragma unroll
  for (int l = 0; l < 4; l++) c[l] = __fadd_rn(__fadd_rn(acc[0][l], acc[1][l]), __fadd_rn(acc[2][l], acc[3][l]));
  float s = __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[1]), c[2]), c[3]);
  for (; i < n; i++) s = __fadd_rn(s, __fmul_rn(f16_ref_to_f32(a[i]), f16_ref_to_f32(b[i])));
  return s;
}

__global__ void attn_exact_kernel(const AttnArgs a) {
  extern __shared__ float sc[];  // [n_keys + 1] scores / exps, then [1] inv
  const uint32_t t = blockIdx.x, h = blockIdx.y;
  const uint32_t hd = a.hd, W = a.window, group = a.Hq / a.Hkv, hk = h / group;
  const uint32_t s0 = a.sstart ? (uint32_t)a.sstart[t] : 0u;
  const uint32_t L = a.slen ? (uint32_t)a.slen[t] : a.T;
  const uint32_t tl = t - s0;
  const uint32_t ws = tl > W ? tl - W : 0u;
  const uint32_t we = (tl + W + 1 < L) ? tl + W + 1 : L;
  const uint32_t nk = we - ws;
  const uint16_t* qr = a.q + (size_t)t * a.Hq * hd + (size_t)h * hd;
  const size_t kstr = (size_t)a.Hkv * hd;
  for (uint32_t j = threadIdx.x; j < nk; j += blockDim.x) {
    const uint32_t key = s0 + ws + j;
    const bool valid = a.mask ? a.mask[key] != 0 : true;
    sc[j] = valid ? dot_ref(qr, a.k + key * kstr + (size_t)hk * hd, hd) : -INFINITY;
  }
  __syncthreads();
  float* inv_slot = sc + nk + 1;
  if (threadIdx.x == 0) {
    const float sink = a.sinks[h];
    float mx = sink;
    for (uint32_t j = 0; j < nk; j++)
      if (sc[j] > mx) mx = sc[j];
    sc[nk] = sink;
    const uint32_t total = nk + 1;
    float sv[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t i = 0;
    for (; i + 4 <= total; i += 4)
      for (int l = 0; l < 4; l++) {
        float e = exp_approx_ref(__fsub_rn(sc[i + l], mx));
        sc[i + l] = e;
        sv[l] = __fadd_rn(sv[l], e);
      }
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(sv[0], sv[1]), sv[2]), sv[3]);
    for (; i < total; i++) {
      float e = expf_ref(__fsub_rn(sc[i], mx));
      sc[i] = e;
      sum = __fadd_rn(sum, e);
    }
    *inv_slot = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
  }
  __syncthreads();
  const float inv = *inv_slot;
  for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (uint32_t j = 0; j < nk; j++) {
      const float p = __fmul_rn(sc[j], inv);
      acc = __fmaf_rn(p, f16_ref_to_f32(a.v[(s0 + ws + j) * kstr + (size_t)hk * hd + d]), acc);
    }
    a.out[(size_t)t * a.Hq * hd + (size_t)h * hd + d] = f32_to_f16_ref(acc);
  }
}

// dot_ref on operands already decoded with f16_ref_to_f32: the same products,
// chains and additions, so the same bits.
__device__ __forceinline__ float dot_ref_f32(const float* a, const float* b, uint32_t n) {
  float acc[4][4];
#pragma unroll
  for (int u = 0; u < 4; u++)
#pragma unroll
    for (int l = 0; l < 4; l++) acc[u][l] = 0.0f;
  uint32_t i = 0;
  for (; i + 16 <= n; i += 16)
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int l = 0; l < 4; l++) acc[u][l] = __fmaf_rn(a[i + 4 * u + l], b[i + 4 * u + l], acc[u][l]);
  for (; i + 4 <= n; i += 4)
#pragma unroll
    for (int l = 0; l < 4; l++) acc[0][l] = __fmaf_rn(a[i + l], b[i + l], acc[0][l]);
  float c[4];
#pragma unroll
  for (int l = 0; l < 4; l++) c[l] = __fadd_rn(__fadd_rn(acc[0][l], acc[1][l]), __fadd_rn(acc[2][l], acc[3][l]));
  float s = __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[1]), c[2]), c[3]);
  for (; i < n; i++) s = __fadd_rn(s, __fmul_rn(a[i], b[i]));
  return s;
}

// attn_exact_kernel's result (the reference's order, bit for bit) for a tile
// of the tensor-core path's list: one block per (16-query tile, KV head)
// stages the keys and values any query of the tile can see, decoded once
// with the reference's fp16 decode, and its 32 warps take the tile's (query,
// head of the group) pairs one at a time.  Per pair: scores with dot_ref's
// chains (lanes over keys), the maximum, every exponential with the
// reference's choice of routine per index (lanes over indices), the sum in
// the reference's four lane chains and tail, then each output column's
// P.V chain over the keys in order (lanes over columns).
constexpr uint32_t kExQ = 16;          // queries per tile of the list
constexpr uint32_t kExMaxRows = 272;   // staged key rows: 16 + 2 W at W = 128
constexpr uint32_t kExHd = 64;         // head_dim handled
constexpr uint32_t kExKStride = 65;    // floats per staged K row: lanes reading one column of
                                       // different rows hit different banks
constexpr uint32_t kExThreads = 1024;
constexpr size_t kExSmem = ((size_t)kExMaxRows * kExKStride + (size_t)kExMaxRows * kExHd + 32 * kExHd +
                            32 * (kExMaxRows + 1)) * sizeof(float);
static_assert(kExSmem <= 227u * 1024u, "shared memory budget");

__global__ void __launch_bounds__(kExThreads, 1) attn_exact_tile_kernel(const AttnArgs a) {
  extern __shared__ float ex_smem[];
  float* sK = ex_smem;                        // [rows][kExKStride]
  float* sV = sK + kExMaxRows * kExKStride;   // [rows][kExHd]
  float* sQ = sV + kExMaxRows * kExHd;        // [warp][kExHd]
  float* sE = sQ + 32 * kExHd;                // [warp][kExMaxRows + 1] scores, then exponentials
  const int2 tile = a.tiles[blockIdx.x];
  const uint32_t hk = blockIdx.y, hd = a.hd, W = a.window, group = a.Hq / a.Hkv;
  const uint32_t q0 = (uint32_t)tile.x, nq = min(kExQ, (uint32_t)tile.y - q0);
  const uint32_t s0 = a.sstart ? (uint32_t)a.sstart[q0] : 0u;
  const uint32_t L = a.slen ? (uint32_t)a.slen[q0] : a.T;
  // keys [kb, ke) of the sequence that some query of the tile attends
  const uint32_t tl0 = q0 - s0, tl1 = tl0 + nq - 1u;
  const uint32_t kb = s0 + (tl0 > W ? tl0 - W : 0u);
  const uint32_t ke = s0 + min(tl1 + W + 1u, L);
  const size_t kstr = (size_t)a.Hkv * hd;
  for (uint32_t idx = threadIdx.x; idx < (ke - kb) * hd; idx += blockDim.x) {
    const uint32_t r = idx / hd, c = idx % hd;
    const size_t g = (size_t)(kb + r) * kstr + (size_t)hk * hd + c;
    sK[r * kExKStride + c] = f16_ref_to_f32(a.k[g]);
    sV[r * kExHd + c] = f16_ref_to_f32(a.v[g]);
  }
  __syncthreads();
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* qw = sQ + warp * kExHd;
  float* ew = sE + warp * (kExMaxRows + 1);
  for (uint32_t p = warp; p < nq * group; p += kExThreads / 32) {
    const uint32_t t = q0 + p % nq, h = hk * group + p / nq;
    const uint32_t tl = t - s0;
    const uint32_t ws = tl > W ? tl - W : 0u, we = min(tl + W + 1u, L), nk = we - ws;
    const uint16_t* qr = a.q + (size_t)t * a.Hq * hd + (size_t)h * hd;
    for (uint32_t i = lane; i < hd; i += 32) qw[i] = f16_ref_to_f32(qr[i]);
    __syncwarp();
    const float sink = a.sinks[h];
    // scores, and the maximum over them and the sink (attn_exact_kernel's
    // running maximum: a value replaces it only when larger)
    float mx = sink;
    for (uint32_t j = lane; j < nk; j += 32) {
      const uint32_t key = s0 + ws + j;
      const bool valid = a.mask ? a.mask[key] != 0 : true;
      const float sc = valid ? dot_ref_f32(qw, sK + (key - kb) * kExKStride, hd) : -INFINITY;
      ew[j] = sc;
      if (sc > mx) mx = sc;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, mx, o);
      if (other > mx) mx = other;
    }
    __syncwarp();
    // exponentials: the polynomial for the first 4 floor(total / 4) entries,
    // exp for the rest (the sink is entry nk)
    const uint32_t total = nk + 1u, nfull = total & ~3u;
    for (uint32_t i = lane; i < total; i += 32) {
      const float x = __fsub_rn(i < nk ? ew[i] : sink, mx);
      ew[i] = i < nfull ? exp_approx_ref(x) : expf_ref(x);
    }
    __syncwarp();
    float part = 0.0f;
    if (lane < 4)
      for (uint32_t i = lane; i < nfull; i += 4) part = __fadd_rn(part, ew[i]);
    const float p0 = __shfl_sync(0xffffffffu, part, 0), p1 = __shfl_sync(0xffffffffu, part, 1);
    const float p2 = __shfl_sync(0xffffffffu, part, 2), p3 = __shfl_sync(0xffffffffu, part, 3);
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(p0, p1), p2), p3);
    for (uint32_t i = nfull; i < total; i++) sum = __fadd_rn(sum, ew[i]);
    const float inv = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
    // P.V: output column d's chain over the keys in order
    const float* vrow = sV + (s0 + ws - kb) * kExHd;
    for (uint32_t d = lane; d < hd; d += 64) {
      const bool two = d + 32u < hd;
      float acc0 = 0.0f, acc1 = 0.0f;
      for (uint32_t j = 0; j < nk; j++) {
        const float pj = __fmul_rn(ew[j], inv);
        acc0 = __fmaf_rn(pj, vrow[j * kExHd + d], acc0);
        if (two) acc1 = __fmaf_rn(pj, vrow[j * kExHd + d + 32u], acc1);
      }
      uint16_t* o = a.out + (size_t)t * a.Hq * hd + (size_t)h * hd + d;
      o[0] = f32_to_f16_ref(acc0);
      if (two) o[32] = f32_to_f16_ref(acc1);
    }
    __syncwarp();  // before the next pair overwrites qw and ew
  }
}

// ---------------------------------------------------------------------------
// Tensor-core path (mma.sync.m16n8k16, fp16 x fp16 -> f32)
// ---------------------------------------------------------------------------
constexpr int kAttnRows = 16;  // query rows per CTA
constexpr int kHD = 64;        // head_dim handled by the tensor-core kernel

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Swizzled offset of (row, 16-byte chunk) in a [rows][64 fp16] smem tile.
__device__ __forceinline__ uint32_t kv_off(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__global__ void __launch_bounds__(7 * 32) attn_tc_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t W = a.window, band = (kAttnRows + 2 * W + 15) & ~15u;
  uint8_t* sK = smem;
  uint8_t* sV = smem + (size_t)band * 128;
  uint8_t* sM = smem + (size_t)band * 256;  // per-key validity of the mask (1 = usable)
  const int2 tile = a.tiles[blockIdx.x];
  const uint32_t q0 = (uint32_t)tile.x, q_end = (uint32_t)tile.y, hk = blockIdx.y;
  const uint32_t group = a.Hq / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t h = hk * group + (uint32_t)warp;
  const int kb0 = (int)q0 - (int)W;  // global key index of smem row 0
  const size_t kld = a.k_ld ? a.k_ld : (size_t)a.Hkv * kHD;
  const size_t vld = a.v_ld ? a.v_ld : (size_t)a.Hkv * kHD;
  const size_t qld = a.q_ld ? a.q_ld : (size_t)a.Hq * kHD;

  // ---- stage the K/V band (zero outside [0, T)) ----
  const uint32_t sK_u = smem_u32(sK), sV_u = smem_u32(sV);
  for (uint32_t i = threadIdx.x; i < band * 8; i += blockDim.x) {
    const uint32_t r = i >> 3, c = i & 7u;
    const int key = kb0 + (int)r;
    const bool in = key >= 0 && key < (int)a.T;
    const size_t kr = (size_t)(in ? key : 0);
    cp_async16(sK_u + kv_off(r, c), a.k + kr * kld + (size_t)hk * kHD + c * 8, in ? 16u : 0u);
    cp_async16(sV_u + kv_off(r, c), a.v + kr * vld + (size_t)hk * kHD + c * 8, in ? 16u : 0u);
  }
  for (uint32_t r = threadIdx.x; r < band; r += blockDim.x) {
    const int key = kb0 + (int)r;
    sM[r] = (key >= 0 && key < (int)a.T && (a.mask == nullptr || a.mask[key] != 0)) ? 1 : 0;
  }
  cp_async_wait_all();
  __syncthreads();
  if (warp >= (int)group) return;

  // ---- per-thread rows: g and g+8 of this CTA's 16 queries ----
  const int g = lane >> 2, tq = lane & 3;
  int r_ws[2], r_we[2], r_p4[2], r_nk[2];
  bool r_ok[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const uint32_t t = q0 + g + 8 * i;
    r_ok[i] = t < q_end;
    if (r_ok[i]) {
      const uint32_t s0 = a.sstart ? (uint32_t)a.sstart[t] : 0u;
      const uint32_t L = a.slen ? (uint32_t)a.slen[t] : a.T;
      const uint32_t tl = t - s0;
      const uint32_t ws = tl > W ? tl - W : 0u;
      const uint32_t we = (tl + W + 1 < L) ? tl + W + 1 : L;
      r_ws[i] = (int)(s0 + ws);
      r_we[i] = (int)(s0 + we);
      r_nk[i] = (int)(we - ws);
      r_p4[i] = 4 * ((r_nk[i] + 1) / 4);
    } else {
      r_ws[i] = r_we[i] = 0;
      r_nk[i] = 0;
      r_p4[i] = 0;
    }
  }
  // Chunk range that any row of this warp touches.
  int lo = min(r_ok[0] ? r_ws[0] : INT_MAX, r_ok[1] ? r_ws[1] : INT_MAX);
  int hi = max(r_ok[0] ? r_we[0] : INT_MIN, r_ok[1] ? r_we[1] : INT_MIN);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, 1));
  lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, 2));
  hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, 1));
  hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, 2));
  if (hi <= lo) {
    // no valid row in this warp
    return;
  }
  const int c_begin = max(0, (lo - kb0) >> 4);
  const int c_end = min((int)(band >> 4), (hi - kb0 + 15) >> 4);

  // ---- Q fragments (A operand), straight from global ----
  uint32_t qa[4][4];
  {
    const uint16_t* qg[2] = {a.q + (size_t)(q0 + g) * qld + (size_t)h * kHD,
                             a.q + (size_t)(q0 + g + 8) * qld + (size_t)h * kHD};
#pragma unroll
    for (int kk = 0; kk < 4; kk++)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        // fragment register j: row g + 8*(j&1), columns c, c+1 (one RoPE pair)
        const int ri = j & 1;
        const int c = kk * 16 + 2 * tq + 8 * (j >> 1);
        uint32_t ab = r_ok[ri] ? *reinterpret_cast<const uint32_t*>(qg[ri] + c) : 0u;
        if (a.q_pos && r_ok[ri]) {
          const size_t trow = (size_t)a.q_pos[q0 + g + 8 * ri] * (kHD / 2) + (c >> 1);
          uint16_t lo = (uint16_t)(ab & 0xffffu), hi = (uint16_t)(ab >> 16);
          rope_pair_ref(lo, hi, a.rope_cos[trow], a.rope_sin[trow]);
          ab = (uint32_t)lo | ((uint32_t)hi << 16);
        }
        qa[kk][j] = ab;
      }
  }
  const float sink = a.sinks[h];

  // S for one 16-key chunk: s[nt][4] for key tiles nt = 0,1.
  auto qk_chunk = [&](int ch, float (&s)[2][4]) {
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) s[nt][i] = 0.0f;
    const uint32_t rbase = (uint32_t)ch * 16u;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      // matrices: (keys 0-7, dims lo8), (keys 0-7, dims hi8), (keys 8-15, lo8), (keys 8-15, hi8)
      const int mi = lane >> 3, rr = lane & 7;
      const uint32_t row = rbase + (uint32_t)((mi >> 1) * 8 + rr);
      const uint32_t chunk = (uint32_t)(kk * 2 + (mi & 1));
      uint32_t b0, b1, b2, b3;
      ldsm_x4(sK_u + kv_off(row, chunk), b0, b1, b2, b3);
      mma16816(s[0], qa[kk], b0, b1);
      mma16816(s[1], qa[kk], b2, b3);
    }
  };

  // ---- pass 1: row max (sink included, padding keys excluded) ----
  float mx[2] = {sink, sink};
  for (int ch = c_begin; ch < c_end; ch++) {
    float s[2][4];
    qk_chunk(ch, s);
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int ri = i >> 1;
        const int key = kb0 + ch * 16 + nt * 8 + 2 * tq + (i & 1);
        const bool inb = key >= r_ws[ri] && key < r_we[ri];
        if (inb && sM[key - kb0] && s[nt][i] > mx[ri]) mx[ri] = s[nt][i];
      }
  }
#pragma unroll
  for (int ri = 0; ri < 2; ri++) {
    mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
    mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
  }

  // ---- pass 2: exp, row sums, O += P V ----
  float o[8][4];
#pragma unroll
  for (int dt = 0; dt < 8; dt++)
#pragma unroll
    for (int i = 0; i < 4; i++) o[dt][i] = 0.0f;
  float lsum[2] = {0.0f, 0.0f};
  for (int ch = c_begin; ch < c_end; ch++) {
    float s[2][4];
    qk_chunk(ch, s);
    float e[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int ri = i >> 1;
        const int key = kb0 + ch * 16 + nt * 8 + 2 * tq + (i & 1);
        float ev = 0.0f;
        if (key >= r_ws[ri] && key < r_we[ri] && sM[key - kb0]) {
          const float x = __fsub_rn(s[nt][i], mx[ri]);
          ev = (key - r_ws[ri]) < r_p4[ri] ? exp_approx_ref(x) : expf_ref(x);
        }
        e[nt][i] = ev;
        lsum[ri] += ev;
      }
    uint32_t pa[4];
    pa[0] = pack_f16x2(e[0][0], e[0][1]);
    pa[1] = pack_f16x2(e[0][2], e[0][3]);
    pa[2] = pack_f16x2(e[1][0], e[1][1]);
    pa[3] = pack_f16x2(e[1][2], e[1][3]);
    const uint32_t rbase = (uint32_t)ch * 16u;
#pragma unroll
    for (int dp = 0; dp < 4; dp++) {
      // matrices: (keys 0-7, dims 16dp..+7), (keys 8-15, same), (keys 0-7, 16dp+8..), (keys 8-15, 16dp+8..)
      const int mi = lane >> 3, rr = lane & 7;
      const uint32_t row = rbase + (uint32_t)((mi & 1) * 8 + rr);
      const uint32_t chunk = (uint32_t)(dp * 2 + (mi >> 1));
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sV_u + kv_off(row, chunk), b0, b1, b2, b3);
      mma16816(o[2 * dp], pa, b0, b1);
      mma16816(o[2 * dp + 1], pa, b2, b3);
    }
  }
  float inv[2];
#pragma unroll
  for (int ri = 0; ri < 2; ri++) {
    float l = lsum[ri];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float xs = __fsub_rn(sink, mx[ri]);
    l += r_nk[ri] < r_p4[ri] ? exp_approx_ref(xs) : expf_ref(xs);  // the sink is entry n_keys
    inv[ri] = l > 0.0f ? __fdiv_rn(1.0f, l) : 0.0f;
  }
#pragma unroll
  for (int ri = 0; ri < 2; ri++) {
    if (!r_ok[ri]) continue;
    uint16_t* orow = a.out + (size_t)(q0 + g + 8 * ri) * a.Hq * kHD + (size_t)h * kHD;
#pragma unroll
    for (int dt = 0; dt < 8; dt++) {
      const uint16_t lo16 = f32_to_f16_fast(__fmul_rn(o[dt][2 * ri], inv[ri]));
      const uint16_t hi16 = f32_to_f16_fast(__fmul_rn(o[dt][2 * ri + 1], inv[ri]));
      *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * tq) = (uint32_t)lo16 | ((uint32_t)hi16 << 16);
    }
  }
}

cudaError_t launch_attention_exact(const AttnArgs& a, cudaStream_t st) {
  if (a.T == 0) return cudaSuccess;
  if (a.tiles && a.n_tiles && a.hd <= kExHd && a.window <= (kExMaxRows - kExQ) / 2 && a.Hkv &&
      a.Hq % a.Hkv == 0) {
    static std::atomic<uint64_t> attr_done{0};
    if (cudaError_t e = smem_attr_per_device(attn_exact_tile_kernel, (int)kExSmem, attr_done); e != cudaSuccess)
      return e;
    attn_exact_tile_kernel<<<dim3(a.n_tiles, a.Hkv), kExThreads, kExSmem, st>>>(a);
    return cudaGetLastError();
  }
  dim3 grid(a.T, a.Hq);
  const size_t sm = (size_t)(2 * a.window + 4) * sizeof(float);
  attn_exact_kernel<<<grid, 64, sm, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_attention_tc(const AttnArgs& a, cudaStream_t st) {
  if (a.T == 0) return cudaSuccess;
  if (attention_umma_supported(a)) return launch_attention_umma(a, st);
  if (a.hd != kHD || a.Hq % a.Hkv != 0 || a.Hq / a.Hkv > 7) return cudaErrorInvalidValue;
  const uint32_t band = (kAttnRows + 2 * a.window + 15) & ~15u;
  const size_t sm = (size_t)band * 256 + band + 16;
  static std::atomic<uint64_t> attr_done{0};
  if (cudaError_t e = smem_attr_per_device(attn_tc_kernel, 200 * 1024, attr_done); e != cudaSuccess) return e;
  if (sm > 200 * 1024) return cudaErrorInvalidValue;
  if (a.n_tiles == 0) return cudaSuccess;
  dim3 grid(a.n_tiles, a.Hkv);
  attn_tc_kernel<<<grid, 7 * 32, sm, st>>>(a);
  return cudaGetLastError();
}

uint32_t attention_max_tiles(uint32_t T, uint32_t n_seqs) { return T / kAttnRows + n_seqs + 1; }

uint32_t attention_tile_rows() { return kAttnRows; }

void attention_tiles(const uint32_t* offs, uint32_t n_seqs, int2* out, uint32_t* n_out) {
  uint32_t n = 0;
  for (uint32_t s = 0; s < n_seqs; s++)
    for (uint32_t q = offs[s]; q < offs[s + 1]; q += kAttnRows) out[n++] = make_int2((int)q, (int)offs[s + 1]);
  *n_out = n;
}

}  // namespace ts
