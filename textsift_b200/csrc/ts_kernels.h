// ts_kernels.h — host-side launchers of libtextsift_cuda's kernels.
// Internal to the library (the public C ABI is include/textsift_cuda.h).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace ts {

// ----------------------------------------------------------------------------
// Repacked int4 weight tiles for the tensor-core GEMM.
//
// A MatMulNBits weight [N, K] (uint4 two per byte along K, block 32, fp16
// scale per block, uint4 zero point per block; packages/textsift/src/zig/
// wasm_exports.zig:512-548) is re-laid out at upload into tiles of BN rows x
// 64 K ("chunks"), stored [expert][n_tile][k_chunk], each tile one contiguous
// blob that a single bulk copy brings into shared memory:
//   [0, BN*16)        nibble words of K elements 0..31 of the chunk, row r at r*16
//   [BN*16, BN*32)    nibble words of K elements 32..63, row r at BN*16 + r*16
//   [BN*32, BN*36)    fp16 scales (block 2c, block 2c+1), row r at BN*32 + 4r
//   [BN*36, BN*37)    zero points (low nibble block 2c, high block 2c+1)
// Within a 32-bit nibble word holding elements 8w..8w+7, bits [4j,4j+4) hold
// element 8w+2j and bits [16+4j,16+4j+4) hold element 8w+2j+1, so one
// (word >> 4j) & 0x000F000F yields an fp16x2 pair after OR-ing 0x6400.
// Padding rows/columns carry nibble 8, zero point 8 and scale 0.
// ----------------------------------------------------------------------------
constexpr uint32_t kChunkK = 64;
// Tokens per MoE permutation chunk: the router's top-k adds each token's
// expert counts into hist[token / kPermChunk][expert].
constexpr uint32_t kPermChunk = 1024;
__host__ __device__ constexpr uint32_t w4_blob_bytes(uint32_t bn) { return bn * 37u; }

struct W4Tiles {
  const uint8_t* blobs = nullptr;   // device
  uint64_t expert_stride = 0;       // bytes per expert
  uint32_t N = 0, K = 0, BN = 0;    // logical shape, tile height
  uint32_t n_tiles = 0, n_kc = 0;   // tiles along N, chunks along K
  const uint16_t* bias = nullptr;   // device fp16 bits [E][N] (always present; zeros if absent)
};

// Repack E experts of a reference-layout [E][N][K] weight (device pointers)
// into blob tiles at dst (E * n_tiles * n_kc * w4_blob_bytes(BN) bytes).
cudaError_t launch_w4_repack(const uint8_t* int4, const uint16_t* scales, const uint8_t* zp, uint32_t E, uint32_t N,
                             uint32_t K, uint32_t BN, uint8_t* dst, cudaStream_t st);
// Adds to *bad the number of fp16 scales that are subnormal, inf or NaN.
cudaError_t launch_count_bad_scales(const uint16_t* s, size_t n, int* bad, cudaStream_t st);

// Epilogues of the tensor-core GEMM.
enum GemmEpi : int {
  kEpiF16 = 0,     // out0 fp16 [row][ld0] = f16(acc + bias)
  kEpiF32 = 1,     // out0 f32  [row][ld0] = acc + bias
  kEpiQkvRope = 2, // q/k with the reference's 3-rounding RoPE, v plain (fp16)
  kEpiSwiglu = 3,  // out0 fp16 [row][N/2] = f16(swiglu(gate, up))
  kEpiF16Widen = 4,  // out0 f32 [row][ld0] = f32(f16(acc + bias)) (logits, wasm.ts:776-797)
  kEpiRouterCert = 5,  // router logits -> candidate experts of the exact top 4: out0 32 bytes per row
                       // {count, 31 ids} (count 0xFF: all experts); needs absum, rbound
};

// Largest expert count of the certified router path (one 128-column tile).
constexpr uint32_t kMaxRouterExperts = 128;

struct GemmArgs {
  const uint8_t* wblob = nullptr;
  uint64_t expert_stride = 0;
  const uint16_t* bias = nullptr;   // [E][N]
  uint32_t N = 0, n_kc = 0, M = 0;
  uint32_t dense_expert = 0;        // dense mode: which expert's weights
  const int4* tiles = nullptr;      // grouped: {expert, row0, row_end, seg_start}
  const int* n_tiles = nullptr;     // grouped: device tile count
  void* out0 = nullptr;
  void* out1 = nullptr;
  void* out2 = nullptr;
  uint32_t ld0 = 0, ld1 = 0, ld2 = 0;
  uint32_t q_cols = 0, k_cols = 0;  // kEpiQkvRope column split
  const int* pos = nullptr;         // kEpiQkvRope: position of each row in its sequence
  const uint16_t* rope_cos = nullptr;
  const uint16_t* rope_sin = nullptr;
  const uint32_t* rope_cs = nullptr;  // kEpiQkvRope (launch_gemm_w4_tm): cos | sin << 16, [pos][32]
  const float* absum = nullptr;      // kEpiRouterCert: sum |x| of each row's f32 input
  const float* rbound = nullptr;     // kEpiRouterCert: f32 wmax_e [128], add_e [128], their maxima [2]
  int* err = nullptr;
};

// Build a 2-D TMA descriptor for an fp16 row-major [rows, K] activation
// matrix, box 128 rows x 64 K, 128-byte swizzle.
bool make_act_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t K);
// 2-D fp16 tensor map with the 128-byte swizzle: `rows` rows of `cols`
// elements, `ld` elements apart, copied in boxes of box_cols x box_rows.
bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                  uint32_t box_rows);
// Streaming multiprocessors of the current device.
int num_sms();

// Tensor-core int4 GEMM: y = A(fp16 [M,K]) x dequant(W)^T.  grid_m = number
// of 128-row tiles (dense) or an upper bound on the grouped tile count.
cudaError_t launch_gemm_w4_tc(const W4Tiles& w, const CUtensorMap& tmap_a, GemmArgs args, int epi,
                              uint32_t grid_m, cudaStream_t st);

// Tensor-core int4 GEMM with the dequantised weights in TMEM (epilogues
// kEpiF16, kEpiSwiglu, kEpiQkvRope; BN = 128 blobs).  Token tiles of
// gemm_tm_rows() rows; x is fp16 [x_rows, K]; grid_m = number of token tiles
// (dense) or an upper bound on the grouped tile count (args.tiles).
uint32_t gemm_tm_rows();
cudaError_t launch_gemm_w4_tm(const W4Tiles& w, const void* x, uint64_t x_rows, GemmArgs args, int epi,
                              uint32_t grid_m, cudaStream_t st);

// Bounded-wait self-test (k_selftest.cu): one CTA whose wait runs out after
// limit_ns; result (device, 2 ints, may be null) = {1 if the timed wait
// completed, 1 if the aborted one did}.
cudaError_t launch_wait_selftest(int* err, unsigned long long limit_ns, int* result, cudaStream_t st);

}  // namespace ts
