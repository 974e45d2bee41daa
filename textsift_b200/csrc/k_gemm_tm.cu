// k_gemm_tm.cu — MatMulNBits (uint4, block 32, fp16 scale, uint4 zero point)
// as a tcgen05 GEMM whose dequantised weight operand lives in tensor memory.
//
// Reference semantics: packages/textsift/src/zig/wasm_exports.zig:560-766
// (matmulInt4BlockImpl), y = x . dequant(W)^T + bias, dequant(W)[n,k] =
// fp16((q - zp) * scale) (bit-identical to the reference helper for every
// normal scale), f32 accumulation.
//
// The product is computed transposed, D^T[n, m] = W[n, :] . x[m, :]: the
// weight tile (128 output rows x 64 K per chunk) is the MMA's A operand and
// is written by the dequantising warps straight into TMEM with tcgen05.st
// (lane = output row, two fp16 of consecutive k per 32-bit column); the
// activations (192 token rows x 64 K, 128B swizzle, one TMA box per chunk)
// are the B operand in shared memory.  Per chunk the shared-memory traffic
// is the activation tile (written by TMA, read once by one M=128 x N=192
// MMA per K=16 step) and the 4.6 KB packed blob; the dequantised weights
// never touch shared memory.
//
// Persistent, warp-specialized: one CTA per SM walks (token tile, 128-wide
// output tile) pairs, 24 warps, over three rings with their own barriers
// (activation tiles and weight blobs in smem, dequantised chunks in TMEM),
// so a TMEM slot is handed back by its MMAs' commit, not by the next copy:
//   warp 0       producer of the x tiles (TMA box per chunk)
//   warp 3       producer of the packed weight blobs (bulk copy per chunk)
//   warp 1       MMA issuer: 4 x tcgen05.mma (A from TMEM) per chunk, from
//                one elected lane of a warp that runs the loop in lockstep
//   warp 2       TMEM allocator: 2 accumulators x 192 columns + 4 A slots
//                x 32 columns = 512
//   warps 4..11  dequantise: warp w owns TMEM lanes 32(w%4).. (output rows);
//                warps 4..7 take the even chunks, 8..11 the odd ones; each
//                reads its blob into registers and releases it at once
//   warps 12..23 epilogue of the previous tile: warp w reads lanes 32(w%4)..
//                (one output column per thread) for tokens 64((w-12)/4)..;
//                lane pairs exchange values so each store is 32 bits
// All waits are bounded (ts_common.cuh) and set the device error flag.
#include "ts_common.cuh"
#include "ts_kernels.h"

#include <algorithm>

namespace ts {

namespace tm {
// Three rings, each with its own full/empty barriers, so that the latency of
// one (a copy from L2, a wake-up) is covered by the depth of the others:
constexpr uint32_t SX = 4;                // activation tiles in smem (TMA)
constexpr uint32_t SR = 4;                // packed weight blobs in smem (bulk copy)
constexpr uint32_t SA = 4;                // dequantised weight chunks in TMEM (MMA A operand)
constexpr uint32_t TOK = 192;             // tokens per tile = MMA N
constexpr uint32_t X_BYTES = TOK * 128;   // 192 rows x 64 fp16
constexpr uint32_t RAW_BYTES = 128 * 37;  // packed blob of a 128-row x 64-K chunk (w4_blob_bytes(128))
constexpr uint32_t RAW_STRIDE = 5120;
constexpr uint32_t OFF_RAW = SX * X_BYTES;
constexpr uint32_t OFF_BAR = OFF_RAW + SR * RAW_STRIDE;
constexpr uint32_t NUM_BARS = 2 * SX + 2 * SR + 2 * SA + 4 + 1;
constexpr uint32_t OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_A = 2 * TOK;  // first A stage column, after the two accumulators
// Role warps per epilogue kind: dequantising and epilogue warps (multiples
// of 4, one per TMEM lane quarter); 4 more warps run the producers, the MMA
// issue and the TMEM allocation.  Every kind has 12 epilogue warps (three
// per scheduler: 64 tokens each) and 8 dequantising warps in two groups
// that take alternate chunks: 24 warps, at most 80 registers a thread.
__host__ __device__ constexpr uint32_t dq_warps(int) { return 8u; }
__host__ __device__ constexpr uint32_t epi_warps(int) { return 12u; }
__host__ __device__ constexpr uint32_t threads(int epi) { return 32u * (4u + dq_warps(epi) + epi_warps(epi)); }
static_assert(X_BYTES % 1024 == 0, "swizzle atoms");
static_assert(COL_A + SA * 32 <= TMEM_COLS, "TMEM budget");
static_assert(SA % 2 == 0, "the two dequantising groups own alternate A slots");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
}  // namespace tm

struct TmTile {
  uint32_t expert, row0, row_end, n_tile;
};

__device__ __forceinline__ TmTile tm_tile(const GemmArgs& a, uint32_t tile, uint32_t n_ntiles) {
  TmTile ti;
  const uint32_t m = tile / n_ntiles;
  ti.n_tile = tile % n_ntiles;
  if (a.tiles) {
    const int4 t = a.tiles[m];
    ti.expert = (uint32_t)t.x;
    ti.row0 = (uint32_t)t.y;
    ti.row_end = (uint32_t)t.z;
  } else {
    ti.expert = a.dense_expert;
    ti.row0 = m * tm::TOK;
    ti.row_end = min(a.M, ti.row0 + tm::TOK);
  }
  return ti;
}

// One 32-token slice of the accumulator column of output n: v[j] is token
// m0 + j.  Lanes 2i and 2i+1 hold outputs n and n+1; one exchange gives the
// even lane both outputs of token m0+2jj and the odd lane those of m0+2jj+1.
template <int EPI>
__device__ __forceinline__ void tm_epilogue_slice(const GemmArgs& a, const TmTile& ti, uint32_t m0, uint32_t n,
                                                  float bv, const uint32_t (&v)[32], int lane, int mypos) {
  const uint32_t odd = (uint32_t)lane & 1u;
  const uint32_t ncol = n & ~1u;
  const bool col_ok = ncol < a.N;
  // bias on tokens 2jj, 2jj+1 with one packed add (fp16 and SwiGLU epilogues)
  auto biased = [&](int jj, float& x0, float& x1) {
    f2unpack(add_f32x2(f2pack(__uint_as_float(v[2 * jj]), __uint_as_float(v[2 * jj + 1])), f2pack(bv, bv)), x0, x1);
  };
  if constexpr (EPI == kEpiF16) {
    uint16_t* o = reinterpret_cast<uint16_t*>(a.out0) + ncol;
#pragma unroll
    for (int jj = 0; jj < 16; jj++) {
      float x0, x1;
      biased(jj, x0, x1);
      const float r = __shfl_xor_sync(0xffffffffu, odd ? x0 : x1, 1);
      const uint32_t m = m0 + 2u * jj + odd;
      if (col_ok && m < ti.row_end)
        *reinterpret_cast<uint32_t*>(o + (size_t)m * a.ld0) = odd ? f32x2_to_h2(r, x1) : f32x2_to_h2(x0, r);
    }
  } else if constexpr (EPI == kEpiSwiglu) {
    // gate = even output column, up = odd (wasm_exports.zig:855-903); output i = n / 2
    const uint32_t bit1 = ((uint32_t)lane >> 1) & 1u;
    const uint32_t icol = (n >> 1) & ~1u;
    uint16_t* o = reinterpret_cast<uint16_t*>(a.out0) + icol;
    const bool ok = icol < (a.N >> 1);
#pragma unroll
    for (int jq = 0; jq < 8; jq++) {
      float gg[2], uu[2], y[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float g0, g1;
        biased(2 * jq + h, g0, g1);
        const float r = __shfl_xor_sync(0xffffffffu, odd ? g0 : g1, 1);
        gg[h] = odd ? r : g0;  // token 4jq + 2h + odd
        uu[h] = odd ? g1 : r;
      }
      swiglu_fast2(gg[0], uu[0], gg[1], uu[1], y[0], y[1]);
      // lanes 4a+{0,1} hold output i (even), 4a+{2,3} output i+1
      const float r2 = __shfl_xor_sync(0xffffffffu, bit1 ? y[0] : y[1], 2);
      const uint32_t m = m0 + 4u * jq + 2u * bit1 + odd;
      if (ok && m < ti.row_end)
        *reinterpret_cast<uint32_t*>(o + (size_t)m * a.ld0) = bit1 ? f32x2_to_h2(r2, y[1]) : f32x2_to_h2(y[0], r2);
    }
  } else if constexpr (EPI == kEpiQkvRope) {
    // the whole 128-column tile lies in one of Q, K, V (launcher checks)
    const uint32_t n0 = ti.n_tile * 128u;
    const bool rope = n0 < a.q_cols + a.k_cols;
    uint16_t* o;
    uint32_t ld;
    if (n0 < a.q_cols) { o = reinterpret_cast<uint16_t*>(a.out0) + ncol; ld = a.ld0; }
    else if (rope) { o = reinterpret_cast<uint16_t*>(a.out1) + (ncol - a.q_cols); ld = a.ld1; }
    else { o = reinterpret_cast<uint16_t*>(a.out2) + (ncol - a.q_cols - a.k_cols); ld = a.ld2; }
    uint32_t csn[16];  // cos | sin << 16
    if (rope) {
      // position of token m0 + lane, then each lane's (cos, sin) of pair (n % 64) / 2
      // mypos: the position of token m0 + lane, loaded before the accumulator wait
      const uint32_t p = (n & 63u) >> 1;
#pragma unroll
      for (int jj = 0; jj < 16; jj++) {
        const int ps = __shfl_sync(0xffffffffu, mypos, 2 * jj + (int)odd);
        csn[jj] = a.rope_cs[(size_t)ps * 32 + p];
      }
    }
#pragma unroll
    for (int jj = 0; jj < 16; jj++) {
      const float x0 = __fadd_rn(__uint_as_float(v[2 * jj]), bv);
      const float x1 = __fadd_rn(__uint_as_float(v[2 * jj + 1]), bv);
      const float r = __shfl_xor_sync(0xffffffffu, odd ? x0 : x1, 1);
      const uint32_t m = m0 + 2u * jj + odd;
      uint32_t h2 = odd ? f32x2_to_h2(r, x1) : f32x2_to_h2(x0, r);
      if (rope) h2 = rope_h2(h2, (uint16_t)(csn[jj] & 0xffffu), (uint16_t)(csn[jj] >> 16));
      if (col_ok && m < ti.row_end) *reinterpret_cast<uint32_t*>(o + (size_t)m * ld) = h2;
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(tm::threads(EPI), 1)
    gemm_w4_tm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmArgs args, uint32_t n_ntiles) {
  using namespace tm;
  constexpr uint32_t kDqWarps = dq_warps(EPI);
  constexpr uint32_t kEpiWarps = epi_warps(EPI);
  constexpr uint32_t kPartTok = TOK / (kEpiWarps / 4);  // tokens per epilogue warp
  static_assert(kPartTok % 32 == 0, "32-token slices");
  extern __shared__ uint8_t smem_dyn[];
  // inputs come from the previous kernel of the stream (programmatic launch)
  pdl_trigger();
  pdl_wait();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;
  uint8_t* sR = smem + OFF_RAW;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* x_full = bars;                 // [SX] activation tile landed
  uint64_t* x_empty = x_full + SX;         // [SX] its MMAs completed
  uint64_t* r_full = x_empty + SX;         // [SR] weight blob landed
  uint64_t* r_empty = r_full + SR;         // [SR] the dequantising group has read it
  uint64_t* a_ready = r_empty + SR;        // [SA] dequantised chunk stored in TMEM
  uint64_t* a_free = a_ready + SA;         // [SA] its MMAs completed
  uint64_t* acc_full = a_free + SA;        // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* drain = acc_empty + 2;         // every MMA issued has completed (teardown)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const uint32_t m_tiles = args.tiles ? (uint32_t)*args.n_tiles : (args.M + TOK - 1u) / TOK;
  const uint32_t total = m_tiles * n_ntiles;
  if (blockIdx.x >= total) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < SX; i++) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (uint32_t i = 0; i < SR; i++) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 128);
    }
    for (uint32_t i = 0; i < SA; i++) {
      mbar_init(&a_ready[i], 128);
      mbar_init(&a_free[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 32u * kEpiWarps);
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
  const uint32_t n_kc = args.n_kc;

  if (warp == 0 || warp == 3) {
    // ---- producers, one lane each: warp 0 the activation tiles (TMA box),
    // warp 3 the weight blobs (bulk copy); each runs as far ahead as its ring
    // allows.  After an abort each waits (bounded) for its copies in flight.
    if (lane == 0) {
      const bool is_x = warp == 0;
      const uint32_t R = is_x ? SX : SR;
      uint64_t* fullb = is_x ? x_full : r_full;
      uint64_t* emptyb = is_x ? x_empty : r_empty;
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TmTile ti = tm_tile(args, tile, n_ntiles);
        const uint8_t* wb = args.wblob + (size_t)ti.expert * args.expert_stride + (size_t)ti.n_tile * n_kc * RAW_BYTES;
        for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
          const uint32_t s = it % R, u = it / R;
          if (!wait_or_abort(&emptyb[s], (u & 1u) ^ 1u, args.err, abort_flag)) { ok = false; break; }
          if (is_x) {
            mbar_arrive_expect_tx(&fullb[s], X_BYTES);
            tma_load_2d(sX + s * X_BYTES, &tmap_x, (int32_t)(kc * kChunkK), (int32_t)ti.row0, &fullb[s]);
          } else {
            mbar_arrive_expect_tx(&fullb[s], RAW_BYTES);
            bulk_g2s(sR + s * RAW_STRIDE, wb + (size_t)kc * RAW_BYTES, RAW_BYTES, &fullb[s]);
          }
        }
      }
      if (!ok)
        for (uint32_t j = it > R ? it - R : 0u; j < it; j++) mbar_wait(&fullb[j % R], (j / R) & 1u, args.err);
    }
  } else if (warp == 1) {
    // The whole warp runs the loop (warp-uniform state, cheap to issue next to
    // the busy dequantising/epilogue warps of this scheduler); one elected
    // lane issues the MMAs and commits.  Descriptors: x slot s starts
    // s * X_BYTES / 16 descriptor units after slot 0's, K step k 2 units.
    constexpr uint32_t idesc = umma_idesc_f16_f32(128, TOK);
    const uint64_t xdesc0 = umma_desc_sw128(smem_u32(sX));
    uint32_t it = 0, lt = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x, lt++) {
      const uint32_t b = lt & 1u, bph = (lt >> 1) & 1u;
      ok = __all_sync(0xffffffffu, wait_or_abort(&acc_empty[b], bph ^ 1u, args.err, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * TOK;
      for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
        const uint32_t sx = it % SX, sa = it % SA;
        ok = __all_sync(0xffffffffu, wait_or_abort(&x_full[sx], (it / SX) & 1u, args.err, abort_flag) &&
                                         wait_or_abort(&a_ready[sa], (it / SA) & 1u, args.err, abort_flag));
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t xd = xdesc0 + (uint64_t)(sx * (X_BYTES >> 4));
          const uint32_t a_tmem = tmem_base + COL_A + sa * 32u;
#pragma unroll
          for (int k = 0; k < 4; k++)
            tc_mma_f16_ts(d_tmem, a_tmem + 8u * k, xd + 2u * k, idesc, (kc | (uint32_t)k) != 0u);
          tc_commit(&x_empty[sx]);
          tc_commit(&a_free[sa]);
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
  } else if (warp >= 4 && warp < 4 + kDqWarps) {
    // ---- dequantise; thread = one output row, both K halves.  With 8 warps,
    // 4..7 take the even chunks and 8..11 the odd ones (two chunks in flight;
    // each group owns alternate A slots); with 4 warps each takes every chunk.
    // The blob is read into registers and released before the A slot's wait. ----
    const uint32_t q = (uint32_t)(warp & 3), grp = (uint32_t)(warp - 4) >> 2;
    const uint32_t r = q * 32u + (uint32_t)lane;
    const uint32_t tcol = tmem_base + ((q * 32u) << 16) + COL_A;
    uint32_t it = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      for (uint32_t kc = 0; kc < n_kc; kc++, it++) {
        if (kDqWarps == 8 && (it & 1u) != grp) continue;
        const uint32_t sr = it % SR, sa = it % SA;
        if (!wait_or_abort(&r_full[sr], (it / SR) & 1u, args.err, abort_flag)) { ok = false; break; }
        const uint8_t* raw = sR + sr * RAW_STRIDE;
        const uint4 h0 = *reinterpret_cast<const uint4*>(raw + r * 16u);
        const uint4 h1 = *reinterpret_cast<const uint4*>(raw + 128u * 16u + r * 16u);
        const uint32_t sc2 = *reinterpret_cast<const uint32_t*>(raw + 128u * 32u + r * 4u);
        const uint32_t zb = raw[128u * 36u + r];
        mbar_arrive(&r_empty[sr]);  // release: the loads above are ordered before it
        uint32_t o[32];
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          const uint32_t sz = ((sc2 >> (16 * hf)) & 0xffffu) * 0x00010001u;
          const uint32_t zz = (0x6400u | ((zb >> (4 * hf)) & 15u)) * 0x00010001u;
          const uint4 hw = hf ? h1 : h0;
          const uint32_t wds[4] = {hw.x, hw.y, hw.z, hw.w};
#pragma unroll
          for (int cc = 0; cc < 4; cc++) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
              // word cc holds k = 8cc..8cc+7 of this half: (k, k+1) = low/high nibble lanes
              const uint32_t bits = ((wds[cc] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
              __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&bits), *reinterpret_cast<const __half2*>(&zz));
              __half2 d = __hmul2(qv, *reinterpret_cast<const __half2*>(&sz));
              o[16 * hf + 4 * cc + j] = *reinterpret_cast<uint32_t*>(&d);
            }
          }
        }
        // the A slot's previous chunk has been consumed by its MMAs
        if (!wait_or_abort(&a_free[sa], ((it / SA) & 1u) ^ 1u, args.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        tmem_st_32x32b_x32(tcol + sa * 32u, o);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&a_ready[sa]);
      }
    }
  } else if (warp >= 4 + kDqWarps) {
    // ---- epilogue: lanes 32(warp%4).. = output columns, token part g of kParts ----
    const uint32_t q = (uint32_t)(warp & 3), g = (uint32_t)(warp - 4 - kDqWarps) >> 2;
    const uint32_t nl = q * 32u + (uint32_t)lane;
    uint32_t lt = 0;
    for (uint32_t tile = blockIdx.x; tile < total; tile += gridDim.x, lt++) {
      const uint32_t b = lt & 1u, bph = (lt >> 1) & 1u;
      const TmTile ti = tm_tile(args, tile, n_ntiles);
      const uint32_t n = ti.n_tile * 128u + nl;
      const float bv = n < args.N ? f16_ref_to_f32(args.bias[(size_t)ti.expert * args.N + n]) : 0.0f;
      // RoPE: each lane's token position for both slices, in flight during the wait
      int pos_s[kPartTok / 32];
#pragma unroll
      for (uint32_t j = 0; j < kPartTok / 32; j++) {
        const uint32_t ml = ti.row0 + g * kPartTok + 32u * j + (uint32_t)lane;
        pos_s[j] = EPI == kEpiQkvRope && ml < ti.row_end ? args.pos[ml] : 0;
      }
      if (!wait_or_abort(&acc_full[b], bph, args.err, abort_flag)) break;
      tc_fence_after();
      const uint32_t acc = tmem_base + ((q * 32u) << 16) + b * TOK + g * kPartTok;
#pragma unroll
      for (uint32_t j = 0; j < kPartTok / 32; j++) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(acc + 32u * j, v);
        tmem_ld_wait();
        if (j + 1 == kPartTok / 32) {
          // every TMEM read of this buffer by this thread is complete: release it
          tc_fence_before();
          mbar_arrive(&acc_empty[b]);
        }
        tm_epilogue_slice<EPI>(args, ti, ti.row0 + g * kPartTok + 32u * j, n, bv, v, lane, pos_s[j]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int EPI>
static cudaError_t launch_tm(const CUtensorMap& tmap, const GemmArgs& args, uint32_t n_tiles, uint32_t grid_m,
                             cudaStream_t st) {
  static std::atomic<uint64_t> attr_done{0};
  if (cudaError_t e = smem_attr_per_device(gemm_w4_tm_kernel<EPI>, (int)tm::SMEM_BYTES, attr_done); e != cudaSuccess)
    return e;
  const uint64_t max_tiles = (uint64_t)grid_m * n_tiles;
  const uint32_t grid = (uint32_t)std::min<uint64_t>(max_tiles, (uint64_t)num_sms());
  return launch_pdl(gemm_w4_tm_kernel<EPI>, dim3(grid), dim3(tm::threads(EPI)), tm::SMEM_BYTES, st, tmap, args, n_tiles);
}

uint32_t gemm_tm_rows() { return tm::TOK; }

cudaError_t launch_gemm_w4_tm(const W4Tiles& w, const void* x, uint64_t x_rows, GemmArgs args, int epi,
                              uint32_t grid_m, cudaStream_t st) {
  if (grid_m == 0 || x_rows == 0) return cudaSuccess;
  if (w.BN != 128 || (w.N & 1u)) return cudaErrorInvalidValue;
  if (epi == kEpiQkvRope && (((args.q_cols | args.k_cols) & 127u) || !args.rope_cs || !args.pos))
    return cudaErrorInvalidValue;
  args.wblob = w.blobs;
  args.expert_stride = w.expert_stride;
  args.bias = w.bias;
  args.N = w.N;
  args.n_kc = w.n_kc;
  CUtensorMap tmap;
  if (!make_tmap_2d(&tmap, x, w.K, x_rows, w.K, 64, tm::TOK)) return cudaErrorInvalidValue;
  switch (epi) {
    case kEpiF16: return launch_tm<kEpiF16>(tmap, args, w.n_tiles, grid_m, st);
    case kEpiSwiglu: return launch_tm<kEpiSwiglu>(tmap, args, w.n_tiles, grid_m, st);
    case kEpiQkvRope: return launch_tm<kEpiQkvRope>(tmap, args, w.n_tiles, grid_m, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ts
