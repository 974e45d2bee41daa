// k_viterbi.cu — BIOES Viterbi decoding of the classifier logits on the GPU,
// one warp per sequence, bit-identical to the reference decoder.
//
// Reference: packages/textsift/src/browser/inference/viterbi.ts:75-145
// (decode), 155-213 (transition matrix), 215-225 (start scores).  Scores are
// stored as f32, candidate sums alpha[i] + trans are doubles, comparisons are
// a strict '>' from -1e30 (the lowest index wins a tie), alpha = f32(best +
// emission).
//
// The reference's transition matrix has a fixed sparsity that the kernel
// uses instead of scanning all 33 x 33 pairs:
//   O     <- O (background_stay), E_l / S_l (end_to_background)
//   B_l, S_l <- O (background_to_start), E_l' / S_l' (end_to_start)  [same
//            candidates and scores for all 16 targets]
//   I_l, E_l <- B_l, I_l (inside_to_continue / inside_to_end)
// Every other transition is -1e30.  For finite emissions and calibration
// (|value| < 1e20, which fp16-derived logits always are) such a candidate
// sums to below -9e29 and a legal candidate with a finite score exists for
// every state, so the illegal ones never win and the restricted scan gives
// the same maximum and the same (lowest) argmax as the full one.
//
// Lanes: lane k <= 16 holds the state P[k] of {O, E_0, S_0, ..., E_7, S_7}
// (ascending ids 0, 3, 4, 7, 8, ...), lane 17 + l holds B_l and I_l.  Per step
// the warp reduces (score, id) pairs over P for the O target and for the
// shared B/S target; lanes 17..24 do the two-way I_l / E_l choices.  Back
// pointers go to shared memory (33 bytes per step); lane 0 walks them back.
#include "ts_common.cuh"
#include "ts_simt.h"

#include <cmath>

namespace ts {
namespace {

constexpr int kTags = 33;
constexpr double kNeg = -1e30;

__device__ __forceinline__ int p_state(int k) {  // P[k] for k = 0..16
  return k == 0 ? 0 : ((k & 1) ? 3 + 4 * ((k - 1) >> 1) : 4 + 4 * ((k - 2) >> 1));
}

// Warp-wide maximum of (v, id) with the lowest id on ties; NaN never wins.
__device__ __forceinline__ void warp_argmax(double& v, int& id) {
  if (v != v) v = -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (ov > v || (ov == v && oi < id)) {
      v = ov;
      id = oi;
    }
  }
}

// The reference's sequential scan result from the reduced maximum: the scan
// starts at (-1e30, 0) and only a strictly larger candidate replaces it.
__device__ __forceinline__ void scan_result(double& v, int& id) {
  if (!(v > kNeg)) {
    v = kNeg;
    id = 0;
  }
}

__global__ void __launch_bounds__(32) viterbi_kernel(const float* __restrict__ logits,
                                                     const int* __restrict__ offs, float c_stay, float c_start,
                                                     float c_cont, float c_end, float c_end_bg, float c_end_start,
                                                     uint8_t* __restrict__ tags) {
  extern __shared__ uint8_t back[];  // [len][33]
  const int lane = threadIdx.x;
  const int s0 = offs[blockIdx.x], len = offs[blockIdx.x + 1] - s0;
  if (len <= 0) return;
  const float* lg = logits + (size_t)s0 * kTags;
  const bool pl = lane <= 16;                 // holds P[lane]
  const bool bl = lane >= 17 && lane <= 24;   // holds B_l, I_l
  const int l = lane - 17;
  const int ps = pl ? p_state(lane) : 0;
  const int sb = 1 + 4 * l, si = 2 + 4 * l, se = 3 + 4 * l;

  // t = 0: start scores (0 for O, B, S; -1e30 for I, E) plus emissions
  const float negf = (float)kNeg;
  float ap = 0.0f, aB = 0.0f, aI = 0.0f;
  if (pl) ap = (float)(0.0 + (double)lg[ps]);
  if (bl) {
    aB = (float)(0.0 + (double)lg[sb]);
    aI = (float)((double)negf + (double)lg[si]);
  }
  // E_l's start is -1e30 too: lanes 2l+1 hold it
  if (pl && lane > 0 && (lane & 1)) ap = (float)((double)negf + (double)lg[ps]);

  // emissions of the next step, loaded one step ahead
  float eP = 0.0f, eB = 0.0f, eI = 0.0f, eE = 0.0f;
  if (len > 1) {
    if (pl) eP = lg[kTags + ps];
    if (bl) { eB = lg[kTags + sb]; eI = lg[kTags + si]; eE = lg[kTags + se]; }
  }
  for (int t = 1; t < len; t++) {
    const float cP = eP, cB = eB, cI = eI, cE = eE;
    if (t + 1 < len) {
      const float* nx = lg + (size_t)(t + 1) * kTags;
      if (pl) eP = nx[ps];
      if (bl) { eB = nx[sb]; eI = nx[si]; eE = nx[se]; }
    }
    // O target and the shared B/S target over P
    double vo = -INFINITY, vs = -INFINITY;
    int io = 255, is = 255;
    if (pl) {
      vo = (double)ap + (double)(lane == 0 ? c_stay : c_end_bg);
      vs = (double)ap + (double)(lane == 0 ? c_start : c_end_start);
      io = is = ps;
    }
    warp_argmax(vo, io);
    warp_argmax(vs, is);
    scan_result(vo, io);
    scan_result(vs, is);
    // I_l and E_l from B_l, I_l (ascending: B first)
    double vi = kNeg, ve = kNeg;
    int ii = 0, ie = 0;
    if (bl) {
      const double fb = (double)aB, fi = (double)aI;
      double s = fb + (double)c_cont;
      if (s > vi) { vi = s; ii = sb; }
      s = fi + (double)c_cont;
      if (s > vi) { vi = s; ii = si; }
      s = fb + (double)c_end;
      if (s > ve) { ve = s; ie = sb; }
      s = fi + (double)c_end;
      if (s > ve) { ve = s; ie = si; }
    }
    uint8_t* bk = back + (size_t)t * kTags;
    // new alphas (E_l computed on lane 17+l, moved to lane 2l+1)
    float aE = 0.0f;
    if (bl) {
      aE = (float)(ve + (double)cE);
      aB = (float)(vs + (double)cB);
      aI = (float)(vi + (double)cI);
      bk[sb] = (uint8_t)is;
      bk[si] = (uint8_t)ii;
      bk[se] = (uint8_t)ie;
    }
    const int from = 17 + ((lane - 1) >> 1);
    const float aE_in = __shfl_sync(0xffffffffu, aE, (pl && lane > 0) ? from : lane);
    if (pl) {
      if (lane == 0) {
        ap = (float)(vo + (double)cP);
        bk[0] = (uint8_t)io;
      } else if (lane & 1) {
        ap = aE_in;  // E_l: back pointer written by lane 17+l
      } else {
        ap = (float)(vs + (double)cP);  // S_l
        bk[ps] = (uint8_t)is;
      }
    }
  }
  // final argmax over all 33 alphas (ascending ids: B_l before I_l in a lane)
  double vf = -INFINITY;
  int idf = 255;
  if (pl) { vf = (double)ap; idf = ps; }
  if (bl) {
    vf = (double)aB; idf = sb;
    if ((double)aI > vf || (vf != vf && (double)aI == (double)aI)) { vf = (double)aI; idf = si; }
  }
  warp_argmax(vf, idf);
  scan_result(vf, idf);
  __syncwarp();
  if (lane == 0) {
    uint8_t* out = tags + s0;
    int tg = idf;
    out[len - 1] = (uint8_t)tg;
    for (int t = len - 1; t > 0; t--) {
      tg = back[(size_t)t * kTags + tg];
      out[t - 1] = (uint8_t)tg;
    }
  }
}

}  // namespace

uint32_t viterbi_max_len() { return (227u * 1024u) / kTags; }

cudaError_t launch_viterbi(const float* logits, const int* offs_dev, uint32_t n_seqs, uint32_t max_len,
                           const float cal[6], uint8_t* tags, cudaStream_t st) {
  if (n_seqs == 0 || max_len == 0) return cudaSuccess;
  if (max_len > viterbi_max_len()) return cudaErrorInvalidValue;
  const size_t sm = (size_t)max_len * kTags;
  static std::atomic<uint64_t> attr_done{0};
  if (cudaError_t e = smem_attr_per_device(viterbi_kernel, 227 * 1024, attr_done); e != cudaSuccess) return e;
  viterbi_kernel<<<n_seqs, 32, sm, st>>>(logits, offs_dev, cal[0], cal[1], cal[2], cal[3], cal[4], cal[5], tags);
  return cudaGetLastError();
}

}  // namespace ts
