// k_attn_umma.cu — banded bidirectional GQA attention with sinks on the
// 5th-generation tensor cores (tcgen05 + TMEM), fast mode.
//
// Same result definition as the reference's attention
// (packages/textsift/src/zig/wasm_exports.zig:1286-1379, bandedAttentionBody):
// for query t of a sequence, keys in [t - W, t + W] clipped to the sequence
// and not padded, scores q . k unscaled, plus one sink logit per head that
// joins the softmax denominator only.  The exponential here is the SFU's
// 2^x (the reference's polynomial/exp split is kept by the exact kernel), P
// enters P.V as fp16 and the output is rounded to fp16 by the hardware.
//
// Work item = (16-query tile of one sequence, one KV head).  The GQA group's
// query heads are stacked into the 128 rows of one M=128 MMA
// (row = head_in_group * 16 + query), so every K/V band is read once per
// group.  Per item:
//   * the producer warp (warp 0) writes the item's metadata (sequence bounds,
//     usable-key bit words) to smem and has TMA stage Q [128 x 64] and the
//     K/V band [16 + 2W rows x 64] with the 128-byte swizzle, double buffered;
//   * the MMA warp (warp 1) computes S = Q K^T into TMEM (columns kColS..)
//     and, behind the next item's S, O = P V with P read from TMEM and V
//     from smem (an MN-major operand);
//   * sixteen softmax warps, four per TMEM lane quarter (one thread per row,
//     each warp a quarter of the band's columns), find the row max over the
//     usable keys (the four partial maxima meet in smem) and write
//     P = 2^((s - max) log2 e) into TMEM (kColP..), two exponentials per
//     fp16x2 SFU instruction; one item later each reads 16 columns of O and
//     the row sum, divides by (row sum + sink term) and stores fp16;
//   * the row sums come from the tensor core: beside each K step of P.V the
//     MMA warp issues P times a 16-column block of ones (kColL..), so the
//     normaliser is the sum of exactly the fp16 P that entered P.V.
// Every wait is bounded; on a timeout the kernel records kDevErrWaitTimeout,
// drains its copies and MMAs in flight and frees TMEM.
#include "ts_common.cuh"
#include "ts_kernels.h"
#include "ts_simt.h"

#include <algorithm>

namespace ts {
namespace {

constexpr uint32_t kQRows = 16;                     // queries per tile and head
constexpr uint32_t kMaxBand = 272;                  // key rows per tile at W = 128
constexpr uint32_t kQBytes = 128u * 128u;           // 128 rows x 64 fp16
constexpr uint32_t kKVBytes = kMaxBand * 128u;      // one K or V band
constexpr uint32_t kStageBytes = kQBytes + 2u * kKVBytes;
constexpr uint32_t kStages = 2;
constexpr uint32_t kOffOnes = kStages * kStageBytes;  // 16 rows x 64 fp16 ones: the row-sum MMA's B operand
constexpr uint32_t kOffBar = kOffOnes + 2048u;
constexpr uint32_t kOffMeta = kOffBar + 128u;             // ItemMeta[kStages]
constexpr uint32_t kOffRed = kOffMeta + 128u;             // float red_max[4][128]
constexpr uint32_t kSmemBytes = kOffRed + 4u * 128u * 4u + 1024u;  // + alignment slack
constexpr uint32_t kTmemCols = 512;
// S: band columns; P: band / 2 (fp16 pairs); O: 64; row sums: 16 (equal) columns
constexpr uint32_t kColS = 0, kColP = 272, kColO = 416, kColL = 480;
constexpr int kThreads = 640;  // producer, MMA, TMEM allocator, idle, 16 softmax warps
static_assert(kColP >= kColS + kMaxBand && kColO >= kColP + kMaxBand / 2 && kColL >= kColO + 64 &&
                  kColL + 16 <= kTmemCols, "TMEM map");
static_assert(kOffOnes % 1024u == 0, "SW128 alignment");
static_assert(kSmemBytes <= 227u * 1024u, "shared memory budget");
static_assert(kStageBytes % 1024u == 0 && kQBytes % 1024u == 0 && kKVBytes % 1024u == 0, "SW128 alignment");

// What the softmax warps need to know about a stage's item, written by the
// producer warp before it issues the stage's copies.
struct ItemMeta {
  int q0, q_end, s0, len;  // first query, end of its sequence, sequence start and length
  uint32_t kw[10];         // bit b of kw[j]: key q0 - W + 32 j + b is inside [0, T) and not padding
  uint32_t pad[2];
};
static_assert(sizeof(ItemMeta) * kStages <= 128u, "metadata region");

// Bits [lo, hi) of a 32-bit word (clipped to [0, 32)).
__device__ __forceinline__ uint32_t range_bits(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 32);
  if (hi <= lo) return 0u;
  const uint32_t below_hi = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
  return below_hi & ~((1u << lo) - 1u);
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Row max over 32 columns whose usable keys are the set bits of rm.
__device__ __forceinline__ void max32(const uint32_t (&v)[32], uint32_t rm, float& m0, float& m1, float& m2,
                                      float& m3) {
  if (rm == 0u) return;
  if (rm == 0xffffffffu) {
#pragma unroll
    for (int b = 0; b < 32; b += 8) {
      m0 = fmax3(m0, __uint_as_float(v[b]), __uint_as_float(v[b + 1]));
      m1 = fmax3(m1, __uint_as_float(v[b + 2]), __uint_as_float(v[b + 3]));
      m2 = fmax3(m2, __uint_as_float(v[b + 4]), __uint_as_float(v[b + 5]));
      m3 = fmax3(m3, __uint_as_float(v[b + 6]), __uint_as_float(v[b + 7]));
    }
  } else {
#pragma unroll
    for (int b = 0; b < 32; b += 2) {
      m0 = fmaxf(m0, ((rm >> b) & 1u) ? __uint_as_float(v[b]) : -INFINITY);
      m1 = fmaxf(m1, ((rm >> (b + 1)) & 1u) ? __uint_as_float(v[b + 1]) : -INFINITY);
    }
  }
}

// 2^x0, 2^x1 as an fp16x2 word without the special-function unit: x = n + f
// with n = round(x) (the 1.5 * 2^23 addition), 2^f on [-1/2, 1/2] by a cubic
// fitted by least squares on the relative error at Chebyshev nodes (max
// relative error 7.7e-5, under half an fp16 ulp), 2^n added to the f32
// exponent field, then the same rounding conversion as the other path.
// x is clamped at -125 so the exponent stays normal; results below fp16's
// range round to 0.
__device__ __forceinline__ uint32_t exp2_fma_h2(float x0, float x1) {
  const uint64_t xx = f2pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t = add_f32x2(xx, f2pack(12582912.0f, 12582912.0f));       // 1.5 * 2^23 + round(x)
  const uint64_t n = add_f32x2(t, f2pack(-12582912.0f, -12582912.0f));      // round(x)
  const uint64_t f = fma_f32x2(n, f2pack(-1.0f, -1.0f), xx);                // x - round(x)
  uint64_t p = fma_f32x2(f, f2pack(0.05508868396282196f, 0.05508868396282196f),
                         f2pack(0.24260404706001282f, 0.24260404706001282f));
  p = fma_f32x2(p, f, f2pack(0.6932762265205383f, 0.6932762265205383f));
  p = fma_f32x2(p, f, f2pack(0.9999289512634277f, 0.9999289512634277f));
  float p0, p1, t0, t1;
  f2unpack(p, p0, p1);
  f2unpack(t, t0, t1);
  // the low bits of t's pattern hold round(x); shifted by 23 they are 2^n's exponent step
  const float y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  const float y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
  return f32x2_to_h2(y0, y1);
}

// P = 2^(s log2 e - m log2 e) for N columns as fp16 pairs, 0 where rm has no
// bit: one packed FMA, one conversion and one fp16x2 SFU exponential per pair.
// nmb2 holds -m log2 e twice.
template <int N>
__device__ __forceinline__ void exp_pack(const uint32_t (&v)[N], uint32_t rm, uint64_t nmb2, uint32_t (&pk)[N / 2]) {
  const uint64_t l2e2 = f2pack(1.4426950408889634f, 1.4426950408889634f);
  const uint32_t full = N == 32 ? 0xffffffffu : ((1u << N) - 1u);
  if (rm == 0u) {
#pragma unroll
    for (int b = 0; b < N / 2; b++) pk[b] = 0u;
    return;
  }
#pragma unroll
  for (int b = 0; b < N; b += 2) {
    float x0, x1;
    f2unpack(fma_f32x2(f2pack(__uint_as_float(v[b]), __uint_as_float(v[b + 1])), l2e2, nmb2), x0, x1);
    // every third pair on the FMA pipe, the rest on the special-function unit
    pk[b >> 1] = (b >> 1) % 3 == 2 ? exp2_fma_h2(x0, x1) : ex2_h2(f32x2_to_h2(x0, x1));
  }
  if (rm != full) {
#pragma unroll
    for (int b = 0; b < N; b += 2)
      pk[b >> 1] &= (((rm >> b) & 1u) ? 0x0000ffffu : 0u) | (((rm >> (b + 1)) & 1u) ? 0xffff0000u : 0u);
  }
}

// A quarter output row: 16 f32 of O times 1/l, as fp16 (round to nearest even).
__device__ __forceinline__ void store_quarter_row(uint16_t* dst, const uint32_t (&o)[16], float inv) {
#pragma unroll
  for (int c = 0; c < 16; c += 8) {
    uint4 w;
    w.x = pack_half2(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv);
    w.y = pack_half2(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
    w.z = pack_half2(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
    w.w = pack_half2(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
    *reinterpret_cast<uint4*>(dst + c) = w;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_umma_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv, const AttnArgs a, uint32_t band) {
  extern __shared__ uint8_t smem_raw[];
  // inputs come from the previous kernel of the stream (programmatic launch)
  pdl_trigger();
  pdl_wait();
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;       // [2] Q/K/V of a stage landed
  uint64_t* empty = bars + 2;  // [2] the stage's last MMA finished
  uint64_t* s_full = bars + 4;  // S of the item is in TMEM
  uint64_t* s_free = bars + 5;  // the softmax has read S and written P
  uint64_t* o_full = bars + 6;  // P.V (and the row sums) of the item completed
  uint64_t* drain = bars + 7;
  uint64_t* pair_bar = bars + 8;  // [4] the four softmax warps of a lane quarter exchanged row maxima
  uint64_t* o_read = bars + 12;   // the softmax has read O and the row sums of the item
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 13) + 1;
  float* red_max = reinterpret_cast<float*>(smem + kOffRed);
  ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + kOffMeta);

  const uint32_t group = a.Hq / a.Hkv;
  const uint32_t items = a.n_tiles * a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 512);
    mbar_init(o_read, 512);
    for (int q = 0; q < 4; q++) mbar_init(&pair_bar[q], 128);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  // Q rows past group * 16 are never loaded: keep them zero.
  for (uint32_t i = threadIdx.x; i < kStages * (kQBytes / 16u); i += blockDim.x) {
    const uint32_t s = i / (kQBytes / 16u), o = i % (kQBytes / 16u);
    *reinterpret_cast<uint4*>(smem + s * kStageBytes + o * 16u) = make_uint4(0u, 0u, 0u, 0u);
  }
  // fp16 1.0 everywhere: any layout reads the block as ones
  for (uint32_t i = threadIdx.x; i < 2048u / 16u; i += blockDim.x)
    *reinterpret_cast<uint4*>(smem + kOffOnes + i * 16u) = make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
  fence_proxy_async_smem();
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer: item metadata + TMA ----------------
    const uint32_t half = band / 2u;
    const uint32_t tx = group * kQRows * 128u + 2u * band * 128u;
    uint32_t lt = 0;
    for (uint32_t item = blockIdx.x; item < items; item += gridDim.x, lt++) {
      const uint32_t s = lt & 1u;
      // The item's metadata comes from global memory: issue every load before
      // waiting for the stage, so their latency overlaps the wait.
      const int2 tile = a.tiles[item / a.Hkv];
      const uint32_t hk = item % a.Hkv;
      const int q0 = tile.x, kb0 = q0 - (int)a.window;
      uint8_t mk[9];
#pragma unroll
      for (int j = 0; j < 9; j++) {
        const int key = kb0 + 32 * j + lane;
        mk[j] = (32u * j < band && key >= 0 && key < (int)a.T) ? (a.mask ? a.mask[key] : (uint8_t)1) : (uint8_t)0;
      }
      const int s0 = lane == 0 ? (a.sstart ? a.sstart[q0] : 0) : 0;
      const int len = lane == 0 ? (a.slen ? a.slen[q0] : (int)a.T) : 0;
      uint32_t kw_mine = 0u;
#pragma unroll
      for (int j = 0; j < 9; j++) {
        const uint32_t w = __ballot_sync(0xffffffffu, mk[j] != 0);
        if (lane == j) kw_mine = w;
      }
      // lane 0 waits (bounded) and tells the warp, so every lane leaves together
      int go = lane == 0 ? (wait_or_abort(&empty[s], ((lt >> 1) & 1u) ^ 1u, a.err, abort_flag) ? 1 : 0) : 0;
      go = __shfl_sync(0xffffffffu, go, 0);
      if (!go) break;
      ItemMeta& md = meta[s];
      if (lane < 10) md.kw[lane] = kw_mine;  // kw[9] stays 0: the last word's successor
      if (lane == 0) {
        md.q0 = q0;
        md.q_end = tile.y;
        md.s0 = s0;
        md.len = len;
      }
      __syncwarp();
      if (lane == 0) {
        // this arrive releases the metadata stores above to the softmax warps
        mbar_arrive_expect_tx(&full[s], tx);
        uint8_t* st = smem + s * kStageBytes;
        for (uint32_t h = 0; h < group; h++)
          tma_load_2d(st + h * (kQRows * 128u), &tmq, (int32_t)((hk * group + h) * 64u), q0, &full[s]);
        uint8_t* sk = st + kQBytes;
        uint8_t* sv = sk + kKVBytes;
        tma_load_2d(sk, &tmk, (int32_t)(hk * 64u), kb0, &full[s]);
        tma_load_2d(sk + half * 128u, &tmk, (int32_t)(hk * 64u), kb0 + (int)half, &full[s]);
        tma_load_2d(sv, &tmv, (int32_t)(hk * 64u), kb0, &full[s]);
        tma_load_2d(sv + half * 128u, &tmv, (int32_t)(hk * 64u), kb0 + (int)half, &full[s]);
      }
      __syncwarp();
    }
    // copies of the last (up to two) items may still be in flight after an abort
    if (lane == 0)
      for (uint32_t j = lt > 2u ? lt - 2u : 0u; j < lt; j++) mbar_wait(&full[j & 1u], (j >> 1) & 1u, a.err);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop in lockstep (warp-uniform state keeps the
    // issue cheap beside the softmax warps of this scheduler); one elected
    // lane issues.  Descriptor address fields step by bytes / 16.
    const uint32_t n1 = band > 256u ? 128u : band, n2 = band - n1;
    const uint32_t idesc1 = umma_idesc_f16_f32(128, n1);
    const uint32_t idesc2 = umma_idesc_f16_f32(128, n2 > 0u ? n2 : 16u);
    const uint32_t idesc_pv = umma_idesc_f16_f32(128, 64) | (1u << 16);  // B (V) is MN-major
    const uint32_t idesc_l = umma_idesc_f16_f32(128, 16);                 // P x ones: row sums
    const uint64_t ones_d = umma_desc_sw128(smem_u32(smem + kOffOnes));
    const uint32_t nks = band / 16u;
    const uint64_t qd0 = umma_desc_sw128(smem_u32(smem));
    const uint64_t kd0 = umma_desc_sw128(smem_u32(smem + kQBytes));
    const uint64_t vd0 = umma_desc_sw128_mn(smem_u32(smem + kQBytes + kKVBytes));
    constexpr uint32_t kStageUnits = kStageBytes >> 4;
    auto issue_pv = [&](uint32_t s) {
      const uint64_t vd = vd0 + (uint64_t)(s * kStageUnits);
      for (uint32_t j = 0; j < nks; j++) {
        tc_mma_f16_ts(tmem + kColO, tmem + kColP + 8u * j, vd + 128u * j, idesc_pv, j > 0u);
        tc_mma_f16_ts(tmem + kColL, tmem + kColP + 8u * j, ones_d, idesc_l, j > 0u);
      }
    };
    // P.V of item j overwrites O: it waits until the softmax has read O of
    // item j - 1 (o_read phase j - 1), which it does after releasing S.
    auto pv_of = [&](uint32_t j, uint32_t sj) -> bool {
      if (j >= 1u && !__all_sync(0xffffffffu, wait_or_abort(o_read, (j - 1u) & 1u, a.err, abort_flag))) return false;
      tc_fence_after();
      if (elect_one()) {
        issue_pv(sj);
        tc_commit(o_full);
        tc_commit(&empty[sj]);
      }
      __syncwarp();
      return true;
    };
    uint32_t lt = 0, prev_s = 0;
    bool ok = true;
    for (uint32_t item = blockIdx.x; item < items; item += gridDim.x, lt++) {
      const uint32_t s = lt & 1u;
      // the stage has landed, and the softmax of the previous item is done
      // with S (and has written P)
      ok = __all_sync(0xffffffffu, wait_or_abort(&full[s], (lt >> 1) & 1u, a.err, abort_flag) &&
                                       (lt == 0 || wait_or_abort(s_free, (lt - 1u) & 1u, a.err, abort_flag)));
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        // S of this item first: its softmax starts while the softmax warps
        // finish the previous item's output and P.V runs behind it
        const uint64_t qd = qd0 + (uint64_t)(s * kStageUnits), kd = kd0 + (uint64_t)(s * kStageUnits);
#pragma unroll
        for (uint32_t k = 0; k < 4; k++) tc_mma_f16(tmem + kColS, qd + 2u * k, kd + 2u * k, idesc1, k > 0u);
        if (n2 > 0u) {
#pragma unroll
          for (uint32_t k = 0; k < 4; k++)
            tc_mma_f16(tmem + kColS + n1, qd + 2u * k, kd + n1 * 8u + 2u * k, idesc2, k > 0u);
        }
        tc_commit(s_full);
      }
      __syncwarp();
      if (lt > 0 && !(ok = pv_of(lt - 1u, prev_s))) break;
      prev_s = s;
    }
    if (ok && lt > 0 && __all_sync(0xffffffffu, wait_or_abort(s_free, (lt - 1u) & 1u, a.err, abort_flag)))
      pv_of(lt - 1u, prev_s);
    // every MMA issued above has completed before TMEM is freed
    if (elect_one()) tc_commit(drain);
    __syncwarp();
    if (lane == 0) mbar_wait(drain, 0, a.err);
  } else if (warp >= 4) {
    // ---------------- softmax + epilogue ----------------
    // Four warps per TMEM lane quarter: warp (4 + quad + 4 * cq) owns rows
    // quad * 32 .. +31, column part cq of the band (its 16-column groups split
    // in four) and columns 16 cq .. +15 of O.
    const uint32_t quad = (uint32_t)warp & 3u, cq = ((uint32_t)warp - 4u) >> 2;
    const uint32_t r = quad * 32u + (uint32_t)lane;
    const uint32_t hl = r >> 4, i = r & 15u;
    const uint32_t trow = tmem + ((quad * 32u) << 16);
    const int W = (int)a.window;
    constexpr float kL2E = 1.4426950408889634f;
    const size_t out_ld = (size_t)a.Hq * 64u;
    const uint32_t ng = band / 16u;  // 16-column groups of the band
    const uint32_t col_begin = (ng * cq / 4u) * 16u;
    const uint32_t col_end = (ng * (cq + 1u) / 4u) * 16u;
    const uint32_t n32 = (col_end - col_begin) / 32u;
    const bool tail = ((col_end - col_begin) & 31u) != 0u;
    const uint32_t c_tail = col_begin + 32u * n32;
    uint32_t lt = 0;
    bool ok = true;
    bool prev_ok = false;
    float prev_sink_term = 0.0f;
    uint16_t* prev_out = nullptr;
    for (uint32_t item = blockIdx.x; item < items; item += gridDim.x, lt++) {
      const uint32_t s = lt & 1u;
      const uint32_t hk = item % a.Hkv;
      const float sink_g = hl < group ? a.sinks[hk * group + hl] : 0.0f;
      if (!wait_or_abort(s_full, lt & 1u, a.err, abort_flag)) { ok = false; break; }
      // the stage's copies (and the metadata written before them) are complete
      if (!wait_or_abort(&full[s], (lt >> 1) & 1u, a.err, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const ItemMeta& md = meta[s];
      const int q0 = md.q0, kb0 = q0 - W;
      const int t = q0 + (int)i;
      const bool row_ok = hl < group && t < md.q_end;
      const int c_lo = max((int)i, md.s0 - kb0);
      const int c_hi = min((int)i + 2 * W + 1, md.s0 + md.len - kb0);
      const float sink = row_ok ? sink_g : 0.0f;
      // usable-key bits of this row for the 32 columns starting at c
      auto row_mask = [&](uint32_t c) -> uint32_t {
        if (!row_ok) return 0u;
        const uint32_t w = __funnelshift_r(md.kw[c >> 5], md.kw[(c >> 5) + 1u], c & 31u);
        return w & range_bits(c_lo - (int)c, c_hi - (int)c);
      };

      // ---- pass 1: max over this half's usable keys, then over the pair ----
      float m0 = sink, m1 = sink, m2 = sink, m3 = sink;
#pragma unroll 1
      for (uint32_t j = 0; j < n32; j++) {
        const uint32_t c = col_begin + 32u * j;
        uint32_t v[32];
        tmem_ld_32x32b_x32(trow + kColS + c, v);
        const uint32_t rm = row_mask(c);
        tmem_ld_wait();
        max32(v, rm, m0, m1, m2, m3);
      }
      if (tail) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(trow + kColS + c_tail, v);
        const uint32_t rm = row_mask(c_tail) & 0xffffu;
        tmem_ld_wait();
#pragma unroll
        for (int b = 0; b < 16; b++) m0 = fmaxf(m0, ((rm >> b) & 1u) ? __uint_as_float(v[b]) : -INFINITY);
      }
      const float mh = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
      red_max[cq * 128u + r] = mh;
      mbar_arrive(&pair_bar[quad]);
      if (!wait_or_abort(&pair_bar[quad], lt & 1u, a.err, abort_flag)) { ok = false; break; }
      const float m = fmaxf(fmaxf(red_max[r], red_max[128u + r]), fmaxf(red_max[256u + r], red_max[384u + r]));
      const float mb = m * kL2E;
      const uint64_t nmb2 = f2pack(-mb, -mb);

      // ---- pass 2: P = exp(s - max) as fp16 into TMEM ----
      // (P of the previous item must have been consumed by its P.V first; that
      // also completes the previous item's O and row sums)
      if (lt > 0) {
        if (!wait_or_abort(o_full, (lt - 1u) & 1u, a.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
      }
#pragma unroll 1
      for (uint32_t j = 0; j < n32; j++) {
        const uint32_t c = col_begin + 32u * j;
        uint32_t v[32];
        tmem_ld_32x32b_x32(trow + kColS + c, v);
        const uint32_t rm = row_mask(c);
        tmem_ld_wait();
        uint32_t pk[16];
        exp_pack<32>(v, rm, nmb2, pk);
        tmem_st_32x32b_x16(trow + kColP + c / 2u, pk);
      }
      if (tail) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(trow + kColS + c_tail, v);
        const uint32_t rm = row_mask(c_tail) & 0xffffu;
        tmem_ld_wait();
        uint32_t pk[8];
        exp_pack<16>(v, rm, nmb2, pk);
        tmem_st_32x32b_x8(trow + kColP + c_tail / 2u, pk);
      }
      tmem_st_wait();
      // S is read and P written: the next item's S may go ahead
      tc_fence_before();
      mbar_arrive(s_free);

      // ---- the previous item's O (this warp's 16 columns) and row sum ----
      if (lt > 0) {
        uint32_t o[16], lsum;
        tmem_ld_32x32b_x16(trow + kColO + 16u * cq, o);
        tmem_ld_32x32b_x1(trow + kColL, lsum);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(o_read);
        if (prev_ok) store_quarter_row(prev_out, o, __fdiv_rn(1.0f, __uint_as_float(lsum) + prev_sink_term));
      }
      prev_ok = row_ok;
      prev_sink_term = ex2_approx(fmaf(sink, kL2E, -mb));
      prev_out = a.out + (size_t)(row_ok ? t : 0) * out_ld + (size_t)(hk * group + (row_ok ? hl : 0u)) * 64u +
                 16u * cq;
    }
    if (ok && lt > 0 && wait_or_abort(o_full, (lt - 1u) & 1u, a.err, abort_flag)) {
      tc_fence_after();
      uint32_t o[16], lsum;
      tmem_ld_32x32b_x16(trow + kColO + 16u * cq, o);
      tmem_ld_32x32b_x1(trow + kColL, lsum);
      tmem_ld_wait();
      const float inv = __fdiv_rn(1.0f, __uint_as_float(lsum) + prev_sink_term);
      if (prev_ok) store_quarter_row(prev_out, o, inv);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool attention_umma_supported(const AttnArgs& a) {
  if (a.hd != 64 || a.Hkv == 0 || a.Hq % a.Hkv != 0 || a.Hq / a.Hkv > 8) return false;
  if (a.q_pos != nullptr || a.tiles == nullptr) return false;
  const uint32_t band = (kQRows + 2u * a.window + 15u) & ~15u;
  if (band > kMaxBand) return false;
  const size_t qld = a.q_ld ? a.q_ld : (size_t)a.Hq * 64u;
  const size_t kld = a.k_ld ? a.k_ld : (size_t)a.Hkv * 64u;
  const size_t vld = a.v_ld ? a.v_ld : (size_t)a.Hkv * 64u;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return al(a.q) && al(a.k) && al(a.v) && al(a.out) && (qld * 2) % 16 == 0 && (kld * 2) % 16 == 0 &&
         (vld * 2) % 16 == 0;
}

cudaError_t launch_attention_umma(const AttnArgs& a, cudaStream_t st) {
  if (a.T == 0 || a.n_tiles == 0) return cudaSuccess;
  if (!attention_umma_supported(a)) return cudaErrorInvalidValue;
  const uint32_t band = (kQRows + 2u * a.window + 15u) & ~15u;
  const size_t qld = a.q_ld ? a.q_ld : (size_t)a.Hq * 64u;
  const size_t kld = a.k_ld ? a.k_ld : (size_t)a.Hkv * 64u;
  const size_t vld = a.v_ld ? a.v_ld : (size_t)a.Hkv * 64u;
  CUtensorMap tq, tk, tv;
  if (!make_tmap_2d(&tq, a.q, (uint64_t)a.Hq * 64u, a.T, qld, 64, kQRows) ||
      !make_tmap_2d(&tk, a.k, (uint64_t)a.Hkv * 64u, a.T, kld, 64, band / 2u) ||
      !make_tmap_2d(&tv, a.v, (uint64_t)a.Hkv * 64u, a.T, vld, 64, band / 2u))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  if (cudaError_t e = smem_attr_per_device(attn_umma_kernel, (int)kSmemBytes, attr_done); e != cudaSuccess) return e;
  const uint64_t items = (uint64_t)a.n_tiles * a.Hkv;
  const uint32_t grid = (uint32_t)std::min<uint64_t>(items, (uint64_t)num_sms());
  return launch_pdl(attn_umma_kernel, dim3(grid), dim3(kThreads), kSmemBytes, st, tq, tk, tv, a, band);
}

}  // namespace ts
