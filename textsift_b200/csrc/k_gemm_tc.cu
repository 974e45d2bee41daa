// k_gemm_tc.cu — MatMulNBits (uint4, block 32, fp16 scale, uint4 zero point)
// as a tcgen05 tensor-core GEMM for sm_100a.
//
// Reference semantics: packages/textsift/src/zig/wasm_exports.zig:560-766
// (matmulInt4BlockImpl) computes y = x . dequant(W)^T + bias with
// dequant(W)[n,k] = (q - zp) * scale.  Here the dequantised value is formed
// exactly as fp16((q - zp) * s) (bit-identical to the reference helper
// fp16(float(q - zp) * float(s)) for every normal scale) inside shared
// memory, and the product runs on the 5th-generation tensor core with f32
// accumulation in TMEM.  Activations enter as fp16.
//
// Persistent, warp-specialized kernel: one CTA per SM walks output tiles of
// BM = 256 rows x BN = 128 columns (dense: row tiles of A; grouped: the
// 256-row tiles of each expert's segment), 20 warps:
//   warp 0       producer: two TMA boxes of A (2 x 128 rows x 64 fp16, 128B
//                swizzle) and one bulk copy of the packed weight blob per
//                64-wide K chunk, into an S-stage ring that runs across tiles
//   warp 1       MMA issuer: per K=16 step two tcgen05.mma (M=128 each, the
//                two row halves) sharing the dequantised B tile, into one of
//                two TMEM tile buffers; commits free the stage / publish a tile
//   warp 2       TMEM allocator (2 buffers x 2 accumulators x 128 columns)
//   warps 4..11  dequantise each stage's int4 blob into the swizzled fp16 B
//                tile (one 32-K half row per thread)
//   warps 12..19 epilogue of the previous tile while the next one accumulates:
//                tcgen05.ld -> bias -> fused op -> global stores; warp 12+i
//                owns TMEM lanes 32(i%4).. of row half i/4
// Sharing each dequantised B tile between two 128-row accumulators halves the
// dequantisation work per flop, which bounds this kernel's tensor-core rate.
// All waits are bounded (ts_common.cuh) and set the device error flag.
#include "ts_common.cuh"
#include "ts_kernels.h"

#include <algorithm>
#include <cstring>
#include <mutex>

namespace ts {

template <int BN, int BM>
struct GemmCfg {
  static_assert(BM == 128 || BM == 256, "row tile");
  static_assert(BM == 128 || BN == 128, "two 128-row accumulators of BN columns per tile buffer");
  static constexpr int STAGES = (BN == 256 || BM == 256) ? (BM == 256 ? 4 : 3) : 4;
  static constexpr uint32_t A_BYTES = BM * 128;             // BM rows x 64 fp16
  static constexpr uint32_t B_BYTES = BN * 128;             // BN rows x 64 fp16
  static constexpr uint32_t RAW_BYTES = BN * 37;            // packed blob
  static constexpr uint32_t RAW_STRIDE = (RAW_BYTES + 1023) & ~1023u;
  static constexpr uint32_t OFF_B = STAGES * A_BYTES;
  static constexpr uint32_t OFF_RAW = OFF_B + STAGES * B_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_RAW + STAGES * RAW_STRIDE;
  static constexpr uint32_t NUM_BARS = 3 * STAGES + 6;
  // f32 [2][BN], decoded bias of the tile; read as float4, so 16-byte aligned
  static constexpr uint32_t OFF_BIAS = (OFF_BAR + NUM_BARS * 8 + 127u) & ~127u;
  static constexpr uint32_t OFF_MISC = OFF_BIAS + 2 * BN * 4;
  // f32 [2][kMaxRouterExperts]: the router bound table (kEpiRouterCert)
  static constexpr uint32_t OFF_RB = OFF_MISC + 16;
  static constexpr uint32_t SMEM_BYTES = OFF_RB + (2 * kMaxRouterExperts + 4) * 4 + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = 512;                    // two accumulators
  static constexpr uint32_t ACC_STRIDE = 256;                   // column offset of tile buffer 1
  static constexpr uint32_t ACC_ROWS = BM / 128;                // 128-row accumulators per tile buffer
  static constexpr int THREADS = 640;  // TMA, MMA, TMEM alloc, idle, 8 dequant warps, 8 epilogue warps
  static_assert(OFF_BIAS % 16 == 0 && OFF_MISC % 16 == 0, "smem regions read with 16-byte accesses");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};


template <int EPI>
__device__ __forceinline__ void gemm_epilogue_chunk(const GemmArgs& a, uint32_t grow, uint32_t ncol0,
                                                    const float* sbias, const uint32_t (&v)[32]) {
  // sbias: the decoded bias of columns ncol0..ncol0+31 (zero past N), in smem
  float acc[32];
#pragma unroll
  for (int q = 0; q < 8; q++) {
    const float4 b4 = reinterpret_cast<const float4*>(sbias)[q];
    acc[4 * q + 0] = __fadd_rn(__uint_as_float(v[4 * q + 0]), b4.x);
    acc[4 * q + 1] = __fadd_rn(__uint_as_float(v[4 * q + 1]), b4.y);
    acc[4 * q + 2] = __fadd_rn(__uint_as_float(v[4 * q + 2]), b4.z);
    acc[4 * q + 3] = __fadd_rn(__uint_as_float(v[4 * q + 3]), b4.w);
  }
  const bool full = ncol0 + 32 <= a.N;
  if constexpr (EPI == kEpiF16) {
    uint16_t* o = reinterpret_cast<uint16_t*>(a.out0) + (size_t)grow * a.ld0 + ncol0;
    if (full) {
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; j++) w[j] = f32x2_to_h2(acc[2 * j], acc[2 * j + 1]);
      uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
      for (int q = 0; q < 4; q++) o4[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    } else {
      for (int j = 0; j < 32; j++)
        if (ncol0 + j < a.N) o[j] = __half_as_ushort(__float2half_rn(acc[j]));
    }
  } else if constexpr (EPI == kEpiF32) {
    float* o = reinterpret_cast<float*>(a.out0) + (size_t)grow * a.ld0 + ncol0;
    if (full) {
      float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
      for (int q = 0; q < 8; q++) o4[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
    } else {
      for (int j = 0; j < 32; j++)
        if (ncol0 + j < a.N) o[j] = acc[j];
    }
  } else if constexpr (EPI == kEpiF16Widen) {
    float* o = reinterpret_cast<float*>(a.out0) + (size_t)grow * a.ld0 + ncol0;
    for (int j = 0; j < 32; j++)
      if (ncol0 + j < a.N) o[j] = __half2float(__float2half_rn(acc[j]));
  } else if constexpr (EPI == kEpiQkvRope) {
    // Columns [0,q_cols) are Q, [q_cols, q_cols+k_cols) K, the rest V.  Every
    // 32-column chunk lies inside one 64-wide head of one region.
    uint32_t h[16];
#pragma unroll
    for (int j = 0; j < 16; j++) h[j] = f32x2_to_h2(acc[2 * j], acc[2 * j + 1]);
    uint16_t* o;
    if (ncol0 < a.q_cols + a.k_cols) {
      const int p0 = (int)(ncol0 & 63u) >> 1;
      const size_t trow = (size_t)a.pos[grow] * 32;
      const uint4* cr = reinterpret_cast<const uint4*>(a.rope_cos + trow + p0);
      const uint4* sr = reinterpret_cast<const uint4*>(a.rope_sin + trow + p0);
#pragma unroll
      for (int q = 0; q < 2; q++) {
        const uint4 c4 = cr[q], s4 = sr[q];
        const uint32_t cw[4] = {c4.x, c4.y, c4.z, c4.w}, sw[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int p = 8 * q + e;
          h[p] = rope_h2(h[p], (uint16_t)(cw[e >> 1] >> (16 * (e & 1))), (uint16_t)(sw[e >> 1] >> (16 * (e & 1))));
        }
      }
      if (ncol0 < a.q_cols)
        o = reinterpret_cast<uint16_t*>(a.out0) + (size_t)grow * a.ld0 + ncol0;
      else
        o = reinterpret_cast<uint16_t*>(a.out1) + (size_t)grow * a.ld1 + (ncol0 - a.q_cols);
    } else {
      o = reinterpret_cast<uint16_t*>(a.out2) + (size_t)grow * a.ld2 + (ncol0 - a.q_cols - a.k_cols);
    }
    uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
    for (int q = 0; q < 4; q++) o4[q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
  } else if constexpr (EPI == kEpiSwiglu) {
    // gate = even column, up = odd column (wasm_exports.zig:855-903).
    uint16_t* o = reinterpret_cast<uint16_t*>(a.out0) + (size_t)grow * a.ld0 + (ncol0 >> 1);
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const __half2 hv = __floats2half2_rn(swiglu_fast(acc[4 * j], acc[4 * j + 1]), swiglu_fast(acc[4 * j + 2], acc[4 * j + 3]));
      w[j] = *reinterpret_cast<const uint32_t*>(&hv);
    }
    if (full) {
      uint4* o4 = reinterpret_cast<uint4*>(o);
      o4[0] = make_uint4(w[0], w[1], w[2], w[3]);
      o4[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
      for (int j = 0; j < 8; j++) {
        if (ncol0 + 4 * j + 1 < a.N) o[2 * j] = (uint16_t)(w[j] & 0xffff);
        if (ncol0 + 4 * j + 3 < a.N) o[2 * j + 1] = (uint16_t)(w[j] >> 16);
      }
    }
  }
}

// Router candidates on the accumulator row of one token (BM = 256: the thread
// owns all BN = 128 expert columns of its row).  The tensor-core logits
// v_e = acc + bias come from fp16(x) and fp16((q - zp) * s); the reference
// computes the same dot from f32 x and exact int4 values in its own f32
// order.  Their difference is at most
//   B_e = kRouterCertRel * wmax_e * S + add_e + S * 2^-24 + |v_e| * 2^-22,
// with S = sum |x| of the token (a.absum), wmax_e = max_i |w_ei| and add_e
// covering the subnormal and bias-decode terms (the per-expert table
// a.rbound = [wmax_0..wmax_127, add_0..add_127, max wmax, max add], built
// with the weights).
// kRouterCertRel = 1.5e-3 bounds 2 * 2^-11 (the two fp16 roundings) plus
// 2e-4 for the tensor core's f32 accumulation and 2e-6 for the reference's.
// With tau = min over the approximate top 4 of (v_a - B_a), the exact 4th
// largest logit is >= tau, so every expert of the exact top 4 satisfies
// v_e + B_e >= tau: those experts are the candidates written to a.out0 (a
// 32-byte record per token).  router_cert_kernel then evaluates the
// candidates in the reference's order and selects exactly.
constexpr float kRouterCertRel = 1.5e-3f;

__device__ __forceinline__ float router_bound(float cS, float addS, const float* srb, uint32_t e, float v) {
  return fmaf(cS, srb[e], srb[kMaxRouterExperts + e] + addS + 2.384185791015625e-7f * fabsf(v));
}

__device__ __forceinline__ void router_cert_epilogue(const GemmArgs& a, uint32_t acc, uint32_t grow, bool row_ok,
                                                     const float* sbias, const float* srb, uint64_t* acc_empty) {
  const float S = row_ok ? a.absum[grow] : 0.0f;
  const float cS = kRouterCertRel * S, addS = 5.9604644775390625e-8f * S;
  float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f, t3 = 0.0f;
  int i0 = -1, i1 = -1, i2 = -1, i3 = -1;
  bool finite = isfinite(S);
  // pass 1: the approximate top 4 (value descending, ties to the lower expert)
#pragma unroll 1
  for (uint32_t c0 = 0; c0 < 128; c0 += 32) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(acc + c0, v);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const int c = (int)c0 + j;
      if ((uint32_t)c >= a.N) break;
      const float x = __fadd_rn(__uint_as_float(v[j]), sbias[c]);
      finite = finite && isfinite(x);
      if (i3 < 0 || x > t3) {
        if (i2 < 0 || x > t2) {
          t3 = t2; i3 = i2;
          if (i1 < 0 || x > t1) {
            t2 = t1; i2 = i1;
            if (i0 < 0 || x > t0) { t1 = t0; i1 = i0; t0 = x; i0 = c; }
            else { t1 = x; i1 = c; }
          } else { t2 = x; i2 = c; }
        } else { t3 = x; i3 = c; }
      }
    }
  }
  float tau = t0 - router_bound(cS, addS, srb, (uint32_t)i0, t0);
  tau = fminf(tau, t1 - router_bound(cS, addS, srb, (uint32_t)i1, t1));
  tau = fminf(tau, t2 - router_bound(cS, addS, srb, (uint32_t)i2, t2));
  tau = fminf(tau, t3 - router_bound(cS, addS, srb, (uint32_t)i3, t3));
  // pass 2: every expert whose logit may reach tau, as a 32-byte record:
  // byte 0 = the count, bytes 1..31 = expert ids (count 0xFF: more than 31,
  // or a value that is not finite -- every expert is then a candidate).  A
  // column below tau by more than the largest bound of the table is no
  // candidate without its own bound.
  const float reach = tau - 1.0001f * fmaf(cS, srb[2 * kMaxRouterExperts], srb[2 * kMaxRouterExperts + 1] + addS);
  uint8_t* rec = reinterpret_cast<uint8_t*>(a.out0) + 32 * (size_t)grow;
  uint32_t n = 0;
#pragma unroll 1
  for (uint32_t c0 = 0; c0 < 128; c0 += 32) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(acc + c0, v);
    tmem_ld_wait();
    if (c0 == 96) {
      // every TMEM read of this buffer by this thread is complete: release it
      tc_fence_before();
      mbar_arrive(acc_empty);
    }
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const uint32_t c = c0 + (uint32_t)j;
      if (c >= a.N) break;
      const float x = __fadd_rn(__uint_as_float(v[j]), sbias[c]);
      if (x + 2.384185791015625e-7f * fabsf(x) >= reach && x + router_bound(cS, addS, srb, c, x) >= tau) {
        n++;
        if (row_ok && n < 32) rec[n] = (uint8_t)c;
      }
    }
  }
  if (!row_ok) return;
  rec[0] = (uint8_t)((!finite || n > 31) ? 0xFFu : n);
}

struct TileInfo {
  uint32_t expert, row0, row_end, n_tile;
};

template <int BM>
__device__ __forceinline__ TileInfo tile_info(const GemmArgs& a, uint32_t tile, uint32_t n_ntiles) {
  TileInfo ti;
  const uint32_t m = tile / n_ntiles;
  ti.n_tile = tile % n_ntiles;
  if (a.tiles) {
    const int4 t = a.tiles[m];
    ti.expert = (uint32_t)t.x;
    ti.row0 = (uint32_t)t.y;
    ti.row_end = (uint32_t)t.z;
  } else {
    ti.expert = a.dense_expert;
    ti.row0 = m * (uint32_t)BM;
    ti.row_end = min(a.M, ti.row0 + (uint32_t)BM);
  }
  return ti;
}

template <int BN, int BM, int EPI>
__global__ void __launch_bounds__(640, 1)
    gemm_w4_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const GemmArgs args, uint32_t n_ntiles) {
  using C = GemmCfg<BN, BM>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_dyn[];
  // inputs come from the previous kernel of the stream (programmatic launch)
  pdl_trigger();
  pdl_wait();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sR = smem + C::OFF_RAW;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* bready = bars + 2 * S;
  uint64_t* acc_full = bars + 3 * S;       // [2]
  uint64_t* acc_empty = bars + 3 * S + 2;  // [2]
  uint64_t* bias_full = bars + 3 * S + 4;  // [2] the tile's bias is staged
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const uint32_t m_tiles = args.tiles ? (uint32_t)*args.n_tiles : (args.M + (uint32_t)BM - 1u) / (uint32_t)BM;
  const uint32_t total = m_tiles * n_ntiles;
  if (blockIdx.x >= total) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&bready[s], 256);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 256);
      mbar_init(&bias_full[b], 256);
    }
    *abort_flag = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t n_kc = args.n_kc;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileInfo ti = tile_info<BM>(args, tile, n_ntiles);
        const uint8_t* wb = args.wblob + (size_t)ti.expert * args.expert_stride + (size_t)ti.n_tile * n_kc * C::RAW_BYTES;
        for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!wait_or_abort(&empty[s], ph ^ 1u, args.err, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::RAW_BYTES);
#pragma unroll
          for (uint32_t h = 0; h < C::ACC_ROWS; h++)
            tma_load_2d(sA + s * C::A_BYTES + h * 16384u, &tmap_a, (int32_t)(kc * kChunkK), (int32_t)(ti.row0 + 128u * h),
                        &full[s]);
          bulk_g2s(sR + s * C::RAW_STRIDE, wb + (size_t)kc * C::RAW_BYTES, C::RAW_BYTES, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // The whole warp runs the loop in lockstep (cheap issue beside the busy
    // warps of this scheduler); one elected lane issues the MMAs.
    constexpr uint32_t idesc = umma_idesc_f16_f32(128, BN);
    const uint64_t adesc0 = umma_desc_sw128(smem_u32(sA)), bdesc0 = umma_desc_sw128(smem_u32(sB));
    uint32_t it = 0, lt = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x, lt++) {
      const uint32_t b = lt & 1u, bph = (lt >> 1) & 1u;
      ok = __all_sync(0xffffffffu, wait_or_abort(&acc_empty[b], bph ^ 1u, args.err, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * C::ACC_STRIDE;
      for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1u;
        ok = __all_sync(0xffffffffu, wait_or_abort(&full[s], ph, args.err, abort_flag) &&
                                         wait_or_abort(&bready[s], ph, args.err, abort_flag));
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          // descriptor address fields step by bytes / 16
          const uint64_t ad = adesc0 + (uint64_t)((uint32_t)s * (C::A_BYTES >> 4));
          const uint64_t bd = bdesc0 + (uint64_t)((uint32_t)s * (C::B_BYTES >> 4));
#pragma unroll
          for (int k = 0; k < 4; k++)
#pragma unroll
            for (uint32_t h = 0; h < C::ACC_ROWS; h++)
              tc_mma_f16(d_tmem + h * BN, ad + h * 1024u + 2u * k, bd + 2u * k, idesc, (kc | (uint32_t)k) != 0u);
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok && elect_one()) tc_commit(&acc_full[b]);
      __syncwarp();
    }
  } else if (warp >= 4 && warp < 12) {
    // ---- dequantise: half rows (32 K values, one scale and zero point) ----
    const int t = threadIdx.x - 128;  // 0..255
    uint32_t it = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1u;
        if (!wait_or_abort(&full[s], ph, args.err, abort_flag)) { ok = false; break; }
        const uint8_t* raw = sR + s * C::RAW_STRIDE;
        uint8_t* bdst = sB + s * C::B_BYTES;
#pragma unroll
        for (int uu = 0; uu < BN / 128; uu++) {
          // unit u: row u % BN, K half u / BN (a warp takes 32 consecutive rows)
          const int u = t + uu * 256;
          const int r = u % BN, hf = u / BN;
          const uint4 hw = *reinterpret_cast<const uint4*>(raw + hf * BN * 16 + r * 16);
          const uint32_t sc = *reinterpret_cast<const uint16_t*>(raw + BN * 32 + r * 4 + hf * 2);
          const uint32_t z = (raw[BN * 36 + r] >> (4 * hf)) & 15u;
          const uint32_t sz = sc * 0x00010001u, zz = (0x6400u | z) * 0x00010001u;
          const uint32_t wds[4] = {hw.x, hw.y, hw.z, hw.w};
#pragma unroll
          for (int cc = 0; cc < 4; cc++) {
            const uint32_t w = wds[cc];
            const int c = 4 * hf + cc;
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const uint32_t bits = ((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
              __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&bits), *reinterpret_cast<const __half2*>(&zz));
              __half2 d = __hmul2(q, *reinterpret_cast<const __half2*>(&sz));
              o[j] = *reinterpret_cast<uint32_t*>(&d);
            }
            *reinterpret_cast<uint4*>(bdst + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&bready[s]);
      }
    }
  } else if (warp >= 12) {
    // ---- epilogue: 8 warps, lane quarter (warp % 4); warp group g = (warp - 12) / 4
    // takes the column half g (BM = 128) or the 128-row accumulator g (BM = 256) ----
    const uint32_t quarter = (uint32_t)(warp & 3), g = (uint32_t)(warp - 12) >> 2;
    const uint32_t rh = BM == 256 ? g : 0u, chalf = BM == 256 ? 0u : g;
    constexpr uint32_t kCols = BM == 256 ? BN : BN / 2;
    const uint32_t r = rh * 128u + quarter * 32u + (uint32_t)lane;
    const uint32_t et = threadIdx.x - 384;  // 0..255 across the 8 epilogue warps
    float* sbias_all = reinterpret_cast<float*>(smem + C::OFF_BIAS);
    float* srb = reinterpret_cast<float*>(smem + C::OFF_RB);
    // the router bound table, visible to all epilogue warps once the first
    // tile's bias barrier below has completed
    if constexpr (EPI == kEpiRouterCert) {
      srb[et] = args.rbound[et];
      if (et < 2) srb[2 * kMaxRouterExperts + et] = args.rbound[2 * kMaxRouterExperts + et];
    }
    uint32_t lt = 0;
    for (uint32_t tile = blockIdx.x; tile < total; tile += gridDim.x, lt++) {
      const uint32_t b = lt & 1u, bph = (lt >> 1) & 1u;
      const TileInfo ti = tile_info<BM>(args, tile, n_ntiles);
      const uint32_t n0 = ti.n_tile * BN;
      // stage this tile's decoded bias (two buffers: a tile's buffer is only
      // rewritten after every epilogue warp has passed the next tile's barrier)
      float* sbias = sbias_all + b * BN;
      if (et < BN) {
        const uint32_t n = n0 + et;
        sbias[et] = n < args.N ? f16_ref_to_f32(args.bias[(size_t)ti.expert * args.N + n]) : 0.0f;
      }
      mbar_arrive(&bias_full[b]);
      if (!wait_or_abort(&bias_full[b], bph, args.err, abort_flag)) break;
      if (!wait_or_abort(&acc_full[b], bph, args.err, abort_flag)) break;
      tc_fence_after();
      const uint32_t grow = ti.row0 + r;
      const bool row_ok = grow < ti.row_end;
      const uint32_t col_lo = chalf * (BN / 2);
      const uint32_t acc = tmem_base + b * C::ACC_STRIDE + rh * BN + ((quarter * 32u) << 16);
      if constexpr (EPI == kEpiRouterCert) {
        router_cert_epilogue(args, acc, grow, row_ok, sbias, srb, &acc_empty[b]);
      } else {
#pragma unroll 1
        for (uint32_t c0 = col_lo; c0 < col_lo + kCols; c0 += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(acc + c0, v);
          tmem_ld_wait();
          if (c0 + 32 >= col_lo + kCols) {
            // every TMEM read of this buffer by this thread is complete: release it
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
          }
          if (row_ok && n0 + c0 < args.N) gemm_epilogue_chunk<EPI>(args, grow, n0 + c0, sbias + c0, v);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// The router's logits with the candidate epilogue (kEpiRouterCert).  The
// router weight is one small matrix (n_experts <= 128 rows x K <= 640), the
// same for every token tile, so each CTA dequantises it once into shared
// memory, where it stays resident as the MMA's B operand (BN = 128 rows x
// 64 K per chunk, the 128-byte swizzle of gemm_w4_tc_kernel's B tiles); only
// the activations stream, one TMA box of 128 token rows x 64 K per chunk.
// Persistent, 20 warps:
//   warp 0       producer of the activation boxes (SA-stage ring across tiles)
//   warp 1       MMA issuer: 4 x tcgen05.mma (M = 128 tokens, N = 128) per
//                chunk into one of four TMEM accumulators
//   warp 2       TMEM allocator (4 x 128 columns)
//   warps 4..11  dequantise the weight once, chunk by chunk, from global
//                memory into the resident tiles (warps 12..19 stage the bias
//                and the bound table meanwhile)
//   warps 4..19  then four epilogue groups of four warps (one per TMEM lane
//                quarter); group g takes the CTA's tiles g, g + 4, ... from
//                accumulator g, one token row per thread: router_cert_epilogue
//                (the epilogue is latency-bound per thread, so four tiles'
//                epilogues run side by side)
// ---------------------------------------------------------------------------
namespace rg {
constexpr uint32_t BM = 128, BN = 128;
constexpr uint32_t KC_MAX = 10;                // K <= 640
constexpr uint32_t SA = 3;                     // activation stages
constexpr uint32_t A_BYTES = BM * 128;         // 128 rows x 64 fp16
constexpr uint32_t B_BYTES = BN * 128;         // one resident chunk of the weight
constexpr uint32_t RAW_BYTES = BN * 37;        // packed blob of a chunk (w4_blob_bytes(128))
constexpr uint32_t OFF_B = SA * A_BYTES;
constexpr uint32_t OFF_BAR = OFF_B + KC_MAX * B_BYTES;
constexpr uint32_t NACC = 4;                    // TMEM accumulators = epilogue groups
constexpr uint32_t NUM_BARS = 2 * SA + 1 + 2 * NACC + 1;  // full/empty per stage, weight ready, acc full/empty, drain
constexpr uint32_t OFF_BIAS = (OFF_BAR + NUM_BARS * 8 + 15u) & ~15u;  // f32 [BN]
constexpr uint32_t OFF_RB = OFF_BIAS + BN * 4;                          // f32 [2 kMaxRouterExperts + 2]
constexpr uint32_t OFF_MISC = (OFF_RB + (2 * kMaxRouterExperts + 2) * 4 + 15u) & ~15u;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
constexpr uint32_t TMEM_COLS = NACC * BN;
static_assert(OFF_B % 1024 == 0 && B_BYTES % 1024 == 0, "SW128 tiles");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
}  // namespace rg

__global__ void __launch_bounds__(640, 1)
    router_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const GemmArgs args) {
  using namespace rg;
  extern __shared__ uint8_t smem_dyn[];
  pdl_trigger();
  pdl_wait();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + OFF_B;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* full = bars;                   // [SA] activation box landed
  uint64_t* empty = bars + SA;             // [SA] its MMAs completed
  uint64_t* w_ready = bars + 2 * SA;       // the resident weight is in place
  uint64_t* acc_full = bars + 2 * SA + 1;         // [NACC]
  uint64_t* acc_empty = bars + 2 * SA + 1 + NACC; // [NACC]
  uint64_t* drain = bars + 2 * SA + 1 + 2 * NACC; // every MMA issued has completed (teardown)
  float* sbias = reinterpret_cast<float*>(smem + OFF_BIAS);
  float* srb = reinterpret_cast<float*>(smem + OFF_RB);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const uint32_t m_tiles = (args.M + BM - 1u) / BM;
  if (blockIdx.x >= m_tiles) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n_kc = args.n_kc;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < SA; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(w_ready, 256);
    for (uint32_t b = 0; b < NACC; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t m = blockIdx.x; m < m_tiles && ok; m += gridDim.x) {
        for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
          const uint32_t s = it % SA, u = it / SA;
          if (!wait_or_abort(&empty[s], (u & 1u) ^ 1u, args.err, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], A_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmap_a, (int32_t)(kc * kChunkK), (int32_t)(m * BM), &full[s]);
        }
      }
      if (!ok)
        for (uint32_t j = it > SA ? it - SA : 0u; j < it; j++) mbar_wait(&full[j % SA], (j / SA) & 1u, args.err);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = umma_idesc_f16_f32(BM, BN);
    const uint64_t adesc0 = umma_desc_sw128(smem_u32(sA)), bdesc0 = umma_desc_sw128(smem_u32(sB));
    bool ok = __all_sync(0xffffffffu, wait_or_abort(w_ready, 0, args.err, abort_flag));
    uint32_t it = 0, lt = 0;
    for (uint32_t m = blockIdx.x; m < m_tiles && ok; m += gridDim.x, lt++) {
      const uint32_t b = lt % NACC, bph = (lt / NACC) & 1u;
      ok = __all_sync(0xffffffffu, wait_or_abort(&acc_empty[b], bph ^ 1u, args.err, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * BN;
      for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
        const uint32_t s = it % SA;
        ok = __all_sync(0xffffffffu, wait_or_abort(&full[s], (it / SA) & 1u, args.err, abort_flag));
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          // descriptor address fields step by bytes / 16
          const uint64_t ad = adesc0 + (uint64_t)(s * (A_BYTES >> 4));
          const uint64_t bd = bdesc0 + (uint64_t)(kc * (B_BYTES >> 4));
#pragma unroll
          for (uint32_t k = 0; k < 4; k++) tc_mma_f16(d_tmem, ad + 2u * k, bd + 2u * k, idesc, (kc | k) != 0u);
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok && elect_one()) tc_commit(&acc_full[b]);
      __syncwarp();
    }
    // every MMA issued above has completed before TMEM is freed
    if (elect_one()) tc_commit(drain);
    __syncwarp();
    if (lane == 0) mbar_wait(drain, 0, args.err);
  } else if (warp >= 4) {
    if (warp < 12) {
      // ---- the resident weight: unit t = (row t % 128, K half t / 128) of
      // every chunk, read from the packed blobs in global memory ----
      const uint32_t t = threadIdx.x - 128u;  // 0..255
      const uint32_t r = t % BN, hf = t / BN;
      // five chunks' loads in flight at a time, then their arithmetic
      constexpr uint32_t kBatch = 5;
      for (uint32_t kc0 = 0; kc0 < n_kc; kc0 += kBatch) {
        uint4 hwb[kBatch];
        uint32_t scb[kBatch], zbb[kBatch];
#pragma unroll
        for (uint32_t u = 0; u < kBatch; u++) {
          if (kc0 + u < n_kc) {
            const uint8_t* raw = args.wblob + (size_t)(kc0 + u) * RAW_BYTES;
            hwb[u] = *reinterpret_cast<const uint4*>(raw + hf * BN * 16 + r * 16);
            scb[u] = *reinterpret_cast<const uint16_t*>(raw + BN * 32 + r * 4 + hf * 2);
            zbb[u] = raw[BN * 36 + r];
          }
        }
#pragma unroll
        for (uint32_t u = 0; u < kBatch; u++) {
        const uint32_t kc = kc0 + u;
        if (kc >= n_kc) break;
        const uint4 hw = hwb[u];
        const uint32_t sc = scb[u];
        const uint32_t z = (zbb[u] >> (4 * hf)) & 15u;
        const uint32_t sz = sc * 0x00010001u, zz = (0x6400u | z) * 0x00010001u;
        const uint32_t wds[4] = {hw.x, hw.y, hw.z, hw.w};
        uint8_t* bdst = sB + kc * B_BYTES;
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
          const uint32_t w = wds[cc];
          const uint32_t c = 4u * hf + (uint32_t)cc;
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const uint32_t bits = ((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
            __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&bits), *reinterpret_cast<const __half2*>(&zz));
            __half2 d = __hmul2(q, *reinterpret_cast<const __half2*>(&sz));
            o[j] = *reinterpret_cast<uint32_t*>(&d);
          }
          *reinterpret_cast<uint4*>(bdst + r * 128 + ((c ^ (r & 7u)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(w_ready);
    } else {
      // the decoded bias and the router bound table, once for every tile
      const uint32_t et = threadIdx.x - 384u;  // 0..255
      if (et < BN) sbias[et] = et < args.N ? f16_ref_to_f32(args.bias[et]) : 0.0f;
      srb[et] = args.rbound[et];
      if (et < 2) srb[2 * kMaxRouterExperts + et] = args.rbound[2 * kMaxRouterExperts + et];
    }
    asm volatile("bar.sync 1, 512;" ::: "memory");  // warps 4..19: the tables are staged
    // ---- epilogue: NACC groups of four warps (one per TMEM lane quarter);
    // group g takes the CTA's tiles g, g + NACC, ... from accumulator g ----
    const uint32_t quarter = (uint32_t)(warp & 3), g = (uint32_t)(warp - 4) >> 2;
    uint32_t lt = 0;
    for (uint32_t m = blockIdx.x; m < m_tiles; m += gridDim.x, lt++) {
      if (lt % NACC != g) continue;
      const uint32_t b = g, bph = (lt / NACC) & 1u;
      if (!wait_or_abort(&acc_full[b], bph, args.err, abort_flag)) break;
      tc_fence_after();
      const uint32_t grow = m * BM + quarter * 32u + (uint32_t)lane;
      const uint32_t acc = tmem_base + b * BN + ((quarter * 32u) << 16);
      router_cert_epilogue(args, acc, grow, grow < args.M, sbias, srb, &acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// One thread per tile row: gathers the row's 64 K elements of one chunk from
// the reference layout and writes them in blob layout (see ts_kernels.h).
__global__ void w4_repack_kernel(const uint8_t* __restrict__ int4, const uint16_t* __restrict__ scales,
                                 const uint8_t* __restrict__ zp, uint32_t N, uint32_t K, uint32_t BN,
                                 uint32_t n_tiles, uint32_t n_kc, uint8_t* __restrict__ dst) {
  const uint32_t r = threadIdx.x + blockIdx.x * blockDim.x;
  const uint32_t kc = blockIdx.y, nt = blockIdx.z % n_tiles, e = blockIdx.z / n_tiles;
  if (r >= BN) return;
  const uint32_t nb = K / 32, zs = (nb + 1) / 2;
  const uint32_t n = nt * BN + r;
  const size_t erow = (size_t)e * N;  // first row of this expert
  uint8_t* b = dst + (((size_t)e * n_tiles + nt) * n_kc + kc) * w4_blob_bytes(BN);
  uint32_t words[8];
  for (int w = 0; w < 8; w++) {
    uint32_t word = 0;
    for (int j = 0; j < 8; j++) {
      const uint32_t k = kc * kChunkK + 8 * w + j;
      uint32_t q = 8;  // padding: (8 - 8) * 0 = 0
      if (n < N && k < K) {
        const uint8_t byte = int4[(erow + n) * (K / 2) + k / 2];
        q = (k & 1) ? (byte >> 4) & 15u : byte & 15u;
      }
      word |= q << ((j & 1) ? 16 + 4 * (j >> 1) : 4 * (j >> 1));
    }
    words[w] = word;
  }
  uint16_t sc[2] = {0, 0};
  uint32_t zb = 0x88;
  for (int hh = 0; hh < 2; hh++) {
    const uint32_t blk = 2 * kc + hh;
    if (n < N && blk < nb) {
      sc[hh] = scales[(erow + n) * nb + blk];
      uint32_t zv = 0;  // a missing zero-point tensor means zp = 0 (wasm_exports.zig:580)
      if (zp) {
        const uint8_t byte = zp[(erow + n) * zs + (blk >> 1)];
        zv = (blk & 1) ? (byte >> 4) & 15u : byte & 15u;
      }
      zb = hh ? ((zb & 0x0Fu) | (zv << 4)) : ((zb & 0xF0u) | zv);
    }
  }
  uint32_t* w0 = reinterpret_cast<uint32_t*>(b + r * 16);
  uint32_t* w1 = reinterpret_cast<uint32_t*>(b + BN * 16 + r * 16);
  for (int i = 0; i < 4; i++) { w0[i] = words[i]; w1[i] = words[4 + i]; }
  *reinterpret_cast<uint32_t*>(b + BN * 32 + r * 4) = (uint32_t)sc[0] | ((uint32_t)sc[1] << 16);
  b[BN * 36 + r] = (uint8_t)zb;
}

// Counts fp16 scales that are neither zero nor a finite normal number.  The
// tensor-core dequantisation is bit-exact with the reference for all others.
__global__ void count_bad_scales_kernel(const uint16_t* __restrict__ s, size_t n, int* __restrict__ bad) {
  int c = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t e = (s[i] >> 10) & 31u, m = s[i] & 0x3ffu;
    c += (e == 31u) || (e == 0u && m != 0u);
  }
  if (c) atomicAdd(bad, c);
}

cudaError_t launch_w4_repack(const uint8_t* int4, const uint16_t* scales, const uint8_t* zp, uint32_t E, uint32_t N,
                             uint32_t K, uint32_t BN, uint8_t* dst, cudaStream_t st) {
  const uint32_t n_tiles = (N + BN - 1) / BN, n_kc = (K + kChunkK - 1) / kChunkK;
  dim3 grid((BN + 127) / 128, n_kc, E * n_tiles);
  w4_repack_kernel<<<grid, 128, 0, st>>>(int4, scales, zp, N, K, BN, n_tiles, n_kc, dst);
  return cudaGetLastError();
}

cudaError_t launch_count_bad_scales(const uint16_t* s, size_t n, int* bad, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  size_t g = (n + 255) / 256;
  count_bad_scales_kernel<<<(unsigned)(g > 2048 ? 2048 : g), 256, 0, st>>>(s, n, bad);
  return cudaGetLastError();
}

typedef CUresult (*PFN_tmapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                        const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                        CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                        CUtensorMapFloatOOBfill);

static PFN_tmapEncodeTiled get_encode_fn() {
  static PFN_tmapEncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_tmapEncodeTiled>(p);
  });
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                  uint32_t box_rows) {
  PFN_tmapEncodeTiled enc = get_encode_fn();
  if (!enc || rows == 0 || cols == 0 || (reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 2) & 15u) || ld < cols)
    return false;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_act_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t K) {
  PFN_tmapEncodeTiled enc = get_encode_fn();
  if (!enc || rows == 0 || (reinterpret_cast<uintptr_t>(base) & 15u) || ((K * 2) & 15u)) return false;
  cuuint64_t gdim[2] = {K, rows};
  cuuint64_t gstride[1] = {K * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// SM count of the current device (persistent grid size), cached per device
// ordinal; devices past the cache are queried on every call.
int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  const bool cached = dev >= 0 && dev < 64;
  if (cached) {
    const int n = cache[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
  }
  int n = 0;
  if (dev < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (cached) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

template <int BN, int BM, int EPI>
static cudaError_t launch_one(const CUtensorMap& tmap, const GemmArgs& args, uint32_t n_tiles, uint32_t grid_m,
                              cudaStream_t st) {
  using C = GemmCfg<BN, BM>;
  static std::atomic<uint64_t> attr_done{0};
  if (cudaError_t e = smem_attr_per_device(gemm_w4_tc_kernel<BN, BM, EPI>, (int)C::SMEM_BYTES, attr_done);
      e != cudaSuccess)
    return e;
  // persistent: at most one CTA per SM, never more CTAs than tiles can exist
  const uint64_t max_tiles = (uint64_t)grid_m * n_tiles;
  const uint32_t grid = (uint32_t)std::min<uint64_t>(max_tiles, (uint64_t)num_sms());
  return launch_pdl(gemm_w4_tc_kernel<BN, BM, EPI>, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, st, tmap, args,
                    n_tiles);
}

cudaError_t launch_gemm_w4_tc(const W4Tiles& w, const CUtensorMap& tmap_a, GemmArgs args, int epi, uint32_t grid_m,
                              cudaStream_t st) {
  if (grid_m == 0) return cudaSuccess;
  args.wblob = w.blobs;
  args.expert_stride = w.expert_stride;
  args.bias = w.bias;
  args.N = w.N;
  args.n_kc = w.n_kc;
  // 256-row tiles: two 128-row accumulators share each dequantised weight tile
  if (w.BN == 128) {
    switch (epi) {
      case kEpiF16: return launch_one<128, 256, kEpiF16>(tmap_a, args, w.n_tiles, grid_m, st);
      case kEpiF32: return launch_one<128, 256, kEpiF32>(tmap_a, args, w.n_tiles, grid_m, st);
      case kEpiQkvRope: return launch_one<128, 256, kEpiQkvRope>(tmap_a, args, w.n_tiles, grid_m, st);
      case kEpiSwiglu: return launch_one<128, 256, kEpiSwiglu>(tmap_a, args, w.n_tiles, grid_m, st);
      case kEpiF16Widen: return launch_one<128, 256, kEpiF16Widen>(tmap_a, args, w.n_tiles, grid_m, st);
      case kEpiRouterCert:
        if (w.N > kMaxRouterExperts || w.n_tiles != 1 || !args.absum || !args.rbound) return cudaErrorInvalidValue;
        if (!args.tiles && w.n_kc <= rg::KC_MAX) {
          // the whole router weight resident in shared memory
          static std::atomic<uint64_t> attr_done{0};
          if (cudaError_t e = smem_attr_per_device(router_gemm_kernel, (int)rg::SMEM_BYTES, attr_done); e != cudaSuccess)
            return e;
          const uint32_t m_tiles = (args.M + rg::BM - 1u) / rg::BM;
          if (m_tiles == 0) return cudaSuccess;
          const uint32_t grid = std::min<uint32_t>(m_tiles, (uint32_t)num_sms());
          return launch_pdl(router_gemm_kernel, dim3(grid), dim3(640), rg::SMEM_BYTES, st, tmap_a, args);
        }
        return launch_one<128, 256, kEpiRouterCert>(tmap_a, args, w.n_tiles, grid_m, st);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace ts
