// ts_simt.h — launchers of the CUDA-core kernels (internal to the library).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ts {

enum ExactOut : int { kOutF16 = 0, kOutF32 = 1, kOutF16Widen = 2 };

// Arguments of the exact-order int4 matmul.  Weight pointers are the
// reference layout ([E][N][K/2] nibbles, [E][N][K/32] scales, [E][N][ceil(K/64)]
// zero points, [E][N] bias), with per-expert strides in elements.
struct ExactArgs {
  const void* x = nullptr;
  uint32_t ldx = 0;
  const uint8_t* w_int4 = nullptr;
  const uint16_t* w_scales = nullptr;
  const uint8_t* w_zp = nullptr;
  const uint16_t* bias = nullptr;
  uint64_t w_int4_estride = 0, w_scales_estride = 0, w_zp_estride = 0, bias_estride = 0;
  uint32_t N = 0, K = 0, M = 0;
  const int* rloc = nullptr;  // dense: index of each row inside its sequence (null: one sequence of M rows)
  const int* rlen = nullptr;  // dense: length of each row's sequence
  const int4* tiles = nullptr;    // grouped: {expert, row0, row_end, seg_start}
  const int* n_tiles = nullptr;   // grouped: device tile count
  const int* seg_end = nullptr;   // grouped: end row of each expert segment
  void* out = nullptr;
  uint32_t ldo = 0;
  uint32_t rows_per_block = 128;  // dense mode
};

cudaError_t launch_seq_info(const uint32_t* offs, uint32_t n_seqs, uint32_t T, int* pos, int* sstart, int* slen,
                            cudaStream_t st);
// The forward's packed embedding table: per vocabulary row its nibbles,
// scales and zero points in one row of embed_row_bytes(D) bytes.
uint32_t embed_row_bytes(uint32_t D);
cudaError_t launch_embed_pack(const uint8_t* w, const uint16_t* sc, const uint8_t* zp, uint8_t* rows, uint32_t V,
                              uint32_t D, cudaStream_t st);
cudaError_t launch_embed_rows(const uint8_t* rows, const int32_t* ids, uint16_t* out, uint32_t T, uint32_t V,
                              uint32_t D, cudaStream_t st);
cudaError_t launch_embed(const uint8_t* w, const uint16_t* sc, const uint8_t* zp, const int32_t* ids, uint16_t* out,
                         uint32_t T, uint32_t V, uint32_t D, cudaStream_t st);
cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* gamma, float* out32, uint16_t* out16, uint32_t T,
                           uint32_t D, float eps, cudaStream_t st);
cudaError_t launch_add_rmsnorm(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, uint16_t* sum_out,
                               float* out32, uint16_t* out16, uint32_t T, uint32_t D, float eps, cudaStream_t st);
cudaError_t launch_matmul_exact(const ExactArgs& a, bool x_f32, int out_mode, uint32_t grid_m, cudaStream_t st);
// Top-k of each token's router logits; hist (may be null) receives the
// per-chunk expert counts that launch_moe_permute consumes.
uint32_t route_chunks(uint32_t T);
cudaError_t launch_router_topk(const float* logits, int32_t* idx, float* w, int* hist, uint32_t T, uint32_t E,
                               uint32_t K, cudaStream_t st);
// Stable expert permutation from idx and the top-k kernel's hist
// (overwritten), the 128-row and (when tiles_tc is set) rows_tc-row
// grouped-GEMM tile lists and their device tile counts.
cudaError_t launch_moe_permute(const int32_t* idx, int* hist, uint32_t T, uint32_t K, uint32_t E, int* counts,
                               int* perm_tok, int* route_pos, int4* tiles, int* n_tiles, int4* tiles_tc,
                               int* n_tiles_tc, uint32_t rows_tc, int* seg_start, int* seg_end, cudaStream_t st);
cudaError_t launch_gather_rows(const void* src, void* dst, const int* perm_tok, const int* n_rows_dev,
                               uint32_t max_rows, uint32_t row_bytes, cudaStream_t st);
cudaError_t launch_moe_combine(const float* down, const int32_t* idx, const float* w, const int* route_pos,
                               const uint16_t* res, uint16_t* out, uint32_t T, uint32_t D, uint32_t K, uint32_t E,
                               cudaStream_t st);
cudaError_t launch_swiglu_exact(const float* gu, float* out, const int* n_rows_dev, uint32_t max_rows, uint32_t D,
                                cudaStream_t st);
cudaError_t launch_split_rope(const uint16_t* qkv, uint16_t* q, uint16_t* k, uint16_t* v, const int* pos,
                              const uint16_t* cos_t, const uint16_t* sin_t, uint32_t T, uint32_t qc, uint32_t kc,
                              uint32_t vc, uint32_t hd, cudaStream_t st);
// BIOES Viterbi decoding (k_viterbi.cu): one warp per sequence of logits
// f32 [len][33] starting at offs_dev[s]; max_len <= viterbi_max_len().
uint32_t viterbi_max_len();
cudaError_t launch_viterbi(const float* logits, const int* offs_dev, uint32_t n_seqs, uint32_t max_len,
                           const float cal[6], uint8_t* tags, cudaStream_t st);
// Fast mode: RMSNorm (b != nullptr: of a + b, the sum written to sum_out)
// to fp16, any summation order; MoE combine from fp16 expert outputs.
cudaError_t launch_rmsnorm_fast(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, uint16_t* sum_out,
                                uint16_t* out16, uint32_t T, uint32_t D, float eps, cudaStream_t st,
                                float* absum = nullptr, float* inv_out = nullptr, float* out32 = nullptr);
// With norm_gamma set it also writes norm_out = RMSNorm(out) * norm_gamma, the
// same bits as launch_rmsnorm_fast on out (D <= 1024).
cudaError_t launch_moe_combine_fast(const uint16_t* down, const int32_t* idx, const float* w, const int* route_pos,
                                    const uint16_t* res, uint16_t* out, uint32_t T, uint32_t D, uint32_t K,
                                    uint32_t E, const uint16_t* norm_gamma, uint16_t* norm_out, float eps,
                                    cudaStream_t st);
cudaError_t launch_f16_to_f32_ref(const uint16_t* src, float* dst, size_t n, cudaStream_t st);
cudaError_t launch_f32_to_f16(const float* src, uint16_t* dst, size_t n, cudaStream_t st);
cudaError_t launch_dequant_tiles(const uint8_t* blobs, uint32_t N, uint32_t K, uint32_t BN, uint32_t n_kc,
                                 uint16_t* out, cudaStream_t st);

// Banded GQA attention with sinks (k_attn.cu).  Sequences are packed along
// T; sstart/slen give each token's sequence (null: one sequence of T tokens).
struct AttnArgs {
  const uint16_t* q = nullptr;   // [T, Hq*hd], row stride q_ld
  const uint16_t* k = nullptr;   // [T, Hkv*hd], row stride k_ld
  const uint16_t* v = nullptr;   // [T, Hkv*hd], row stride v_ld
  uint32_t q_ld = 0, k_ld = 0, v_ld = 0;  // 0 = dense (Hq*hd, Hkv*hd)
  // tensor-core path: when set, the reference RoPE is applied to q as it is
  // loaded (q is then the projection before rotation)
  const int* q_pos = nullptr;
  const uint16_t* rope_cos = nullptr;
  const uint16_t* rope_sin = nullptr;
  const float* sinks = nullptr;  // [Hq]
  const uint8_t* mask = nullptr; // [T] or null
  uint16_t* out = nullptr;       // [T, Hq*hd]
  const int* sstart = nullptr;
  const int* slen = nullptr;
  // tensor-core path: 16-query tiles {first query, end of its sequence}, each
  // tile inside one sequence and aligned to the sequence start, so the key
  // chunking (and every rounding) is the same however sequences are packed
  const int2* tiles = nullptr;
  uint32_t n_tiles = 0;
  uint32_t T = 0, Hq = 0, Hkv = 0, hd = 0, window = 0;
  int* err = nullptr;
};
// tcgen05 attention (k_attn_umma.cu): head_dim 64, group <= 8, window <= 128,
// no fused q rotation, 16-byte aligned operands.
bool attention_umma_supported(const AttnArgs& a);
cudaError_t launch_attention_umma(const AttnArgs& a, cudaStream_t st);
// Host: the tensor-core tile list for packed sequences (offs has n_seqs + 1 entries).
void attention_tiles(const uint32_t* offs, uint32_t n_seqs, int2* out, uint32_t* n_out);
uint32_t attention_max_tiles(uint32_t T, uint32_t n_seqs);
// Queries per tile of that list (a tile never crosses a sequence end).
uint32_t attention_tile_rows();
cudaError_t launch_attention_tc(const AttnArgs& a, cudaStream_t st);     // mma.sync tensor-core path
cudaError_t launch_attention_exact(const AttnArgs& a, cudaStream_t st);  // reference-order CUDA-core path

// The certified fast-mode router (k_router.cu): exact top-k over the
// candidates the kEpiRouterCert GEMM epilogue leaves.
enum RouterSrc : int {
  kRouterSrcF32 = 0,      // the f32 router input is given (x32)
  kRouterSrcAddNorm = 1,  // rebuilt as rmsnorm_fast_kernel<true>(a + b) * gamma computes it
};
struct RouterCertArgs {
  const uint8_t* cand = nullptr;   // uint4 per token from the kEpiRouterCert epilogue
  const float* x32 = nullptr;      // kRouterSrcF32: [T, D]
  const uint16_t* a = nullptr;     // kRouterSrcAddNorm: residual + attention output as fp16 [T, D]
  const float* inv = nullptr;      //   the add+norm's 1 / rms of each token [T]
  const uint16_t* gamma = nullptr; //   norm weight fp16 [D]
  float eps = 0.0f;
  // the router weight: int4 [E][D/2] in reference layout, the table of
  // router_bound_table (scale, -(2^23 + zp) per block), fp16 bias [E]
  const uint8_t* w_int4 = nullptr;
  const float* w_sz = nullptr;  // per (expert, block): scale (reference decode), -(2^23 + zp)
  const uint16_t* bias = nullptr;
  const int* rloc = nullptr;  // token position / sequence length (tile or tail path); null: row t of T
  const int* rlen = nullptr;
  int32_t* idx = nullptr;     // [T, K]
  float* w = nullptr;         // [T, K]
  int* hist = nullptr;        // per-permutation-chunk expert counts (or null)
  uint32_t T = 0, D = 0, E = 0, K = 0;
};
cudaError_t launch_router_cert(const RouterCertArgs& a, int src, cudaStream_t st);
// fp16 copy of f32 rows and each row's sum of |x| (the router bound's S).
cudaError_t launch_f32_to_f16_absum(const float* x, uint16_t* y, float* absum, uint32_t T, uint32_t D, cudaStream_t st);
// Host: the router's bound table, f32 [2 kMaxRouterExperts + 2] (max |w| per
// expert, the additive term per expert, the largest of each), and the per-block scale /
// zero-point table, f32 [E][D/32][2].
void router_bound_table(const uint8_t* int4, const uint16_t* scales, const uint8_t* zp, uint32_t E, uint32_t D,
                        float* bound, float* sz);

// Sets the calling thread's message returned by ts_cuda_last_error().
void set_last_error(const char* msg);

}  // namespace ts
