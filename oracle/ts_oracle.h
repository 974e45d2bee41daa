/*
 * ts_oracle.h — CPU restatement of textsift's WASM/Zig forward path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA backend and the timed CPU baseline in bench.py.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * legs load it.  The product (libtextsift_cuda.so) never links or calls it.
 *
 * Every function restates the arithmetic of one reference kernel with the
 * same rounding points and summation order (cited per function in the .c
 * files, paths relative to packages/textsift/src/ in teamchong/textsift):
 *   zig/wasm_exports.zig   the kernels
 *   zig/math.zig           fp16 <-> f32 bit conversions
 *   c/fma.c                relaxed_madd: fixed here as a fused FMA (fmaf)
 *   browser/inference/{model,block,attention,expert,rope}.ts  composition
 *   browser/backends/wasm.ts                                    loader rules
 *
 * Build: oracle/Makefile (gcc, -ffp-contract=off so that no mul+add pair is
 * contracted into an FMA that the reference does not perform).
 */
#ifndef TS_ORACLE_H
#define TS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numeric helpers (math.zig) ---- */
float    tso_f16_to_f32(uint16_t bits);   /* math.zig:45-52 (subnormals decode "wrongly", on purpose) */
uint16_t tso_f32_to_f16(float f);         /* math.zig:54-82 (RNE normals, half-up subnormals) */
uint16_t tso_f32_to_bf16(float f);        /* math.zig:19-28 */
float    tso_bf16_to_f32(uint16_t b);     /* math.zig:13-16 */
uint16_t tso_js_f32_to_f16(double f);     /* browser/backends/wasm.ts:264-291 (+0 for ±0, double->f32 first) */
float    tso_js_f16_to_f32(uint16_t h);   /* browser/backends/wasm.ts:776-797 (exact widen incl. subnormals) */
float    tso_exp_approx(float x);         /* wasm_exports.zig:812-838 one lane */

/* ---- kernels (wasm_exports.zig) ---- */
void tso_rms_norm(const uint16_t* x, const uint16_t* gamma, uint16_t* out,
                  uint32_t T, uint32_t D, float eps);
void tso_rms_norm_fp16_to_f32(const uint16_t* x, const uint16_t* gamma, float* out,
                              uint32_t T, uint32_t D, float eps);
void tso_add_rmsnorm_fp16_to_f32(const uint16_t* a, const uint16_t* b, const uint16_t* gamma,
                                 uint16_t* sum_out, float* norm_out,
                                 uint32_t T, uint32_t D, float eps);
void tso_topk_partial_f32(const float* x, int32_t* out_idx, float* out_val,
                          uint32_t rows, uint32_t cols, uint32_t k);
/* x_is_f32: 0 -> x is fp16 bits; out_is_f32: 0 -> out is fp16 bits. zp may be NULL. */
void tso_matmul_int4(int x_is_f32, int out_is_f32, const void* x,
                     const uint8_t* w_int4, const uint16_t* w_scales, const uint8_t* w_zp,
                     const uint16_t* bias, void* out, uint32_t T, uint32_t N, uint32_t D);
/* The same computation written lane by lane in scalar C (cross-check of the
 * SIMD form above). */
void tso_matmul_int4_scalar(int x_is_f32, int out_is_f32, const void* x,
                            const uint8_t* w_int4, const uint16_t* w_scales, const uint8_t* w_zp,
                            const uint16_t* bias, void* out, uint32_t T, uint32_t N, uint32_t D);
void tso_swiglu_clamp_f32(const float* gate_up, float* out, uint32_t T, uint32_t D);
void tso_softmax_f32(const float* x, float* out, uint32_t rows, uint32_t cols);
void tso_add_fp16(const uint16_t* a, const uint16_t* b, uint16_t* out, uint32_t n);
void tso_gather_f32(const float* src, const int32_t* idx, float* dst, uint32_t m, uint32_t D);
void tso_scatter_add_weighted_f32(float* target, const float* values, const int32_t* idx,
                                  const float* w, uint32_t m, uint32_t D);
void tso_convert_fp16_to_f32(const uint16_t* src, float* dst, uint32_t n);
void tso_cast_f32_to_fp16_scaled(const float* src, uint16_t* dst, uint32_t n, float scale);
void tso_banded_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          const float* sinks, const uint8_t* mask /* NULL = all valid */,
                          uint16_t* out, uint32_t T, uint32_t Hq, uint32_t Hkv,
                          uint32_t head_dim, uint32_t window,
                          uint32_t h_q_start, uint32_t h_q_end);
void tso_rope_apply(uint16_t* qk, const uint16_t* cos_tab, const uint16_t* sin_tab,
                    uint32_t T, uint32_t H, uint32_t head_dim);
void tso_embed_lookup_int4(const uint8_t* embed_int4, const uint16_t* embed_scales,
                           const uint8_t* embed_zp, const int32_t* ids, uint16_t* out,
                           uint32_t T, uint32_t V, uint32_t D);
/* fp16((q - zp) * s) per element: the value a tensor-core kernel places in
 * its operand tile (row-major [N, D] fp16 bits out). */
void tso_dequant_int4(const uint8_t* w_int4, const uint16_t* w_scales, const uint8_t* w_zp,
                      uint16_t* out, uint32_t N, uint32_t D);

/* ---- rope tables (browser/inference/rope.ts) ---- */
typedef struct {
  uint32_t head_dim;
  double theta, factor;
  double original_max_pos, beta_fast, beta_slow;
  int truncate;
} tso_rope_cfg;
/* Span decoding (ts_oracle_decode.c): browser/inference/viterbi.ts and
 * spans.ts.  cal = {background_stay, background_to_start,
 * inside_to_continue, inside_to_end, end_to_background, end_to_start}. */
void tso_viterbi_tables(const float cal[6], float* trans /* [33*33], [to*33+from] */, float* start /* [33] */);
void tso_viterbi(const float* logits, uint32_t T, const float cal[6], uint8_t* tags, float* alpha_scratch,
                 uint8_t* back_scratch);
uint32_t tso_bioes_spans(const uint8_t* tags, uint32_t T, int32_t* out /* [cap][3] */, uint32_t cap);

void tso_build_rope_tables(const tso_rope_cfg* cfg, uint32_t T, uint16_t* cos_out, uint16_t* sin_out);

/* ---- model composition (model.ts / block.ts / attention.ts / expert.ts) ---- */
typedef struct tso_model tso_model;

typedef struct {
  uint32_t vocab, d_model, n_layers, n_heads, n_kv_heads, head_dim, window;
  uint32_t d_ff, n_experts, top_k, n_classes;
  float eps;
  tso_rope_cfg rope;
} tso_config;

tso_model* tso_model_create(const tso_config* cfg);
void       tso_model_destroy(tso_model* m);
/* Register a tensor under the reference loader's canonical name
 * (browser/backends/wasm.ts:358-446, e.g. "layers.3.attn.q_proj.int4").
 * The bytes are NOT copied: the caller keeps them alive.  Returns 0 on
 * success, -1 for an unknown name. */
int        tso_model_set(tso_model* m, const char* name, const void* data, size_t nbytes);
/* Full forward of one sequence.  mask may be NULL (= all ones); an all-ones
 * mask is treated as NULL like wasm.ts:755-764.  logits_out: f32 [T, n_classes].
 * n_threads <= 1: canonical single-thread order (the bit-exact reference).
 * n_threads > 1: the reference's MtPool partitioning (block.ts:63-95,
 * attention.ts:84-185, mt-expert.ts:63-191).
 * Optional traces (may be NULL): hidden_trace fp16 [n_layers+1, T, d_model]
 * (residual stream after embed and after each block), topk_trace i32
 * [n_layers, T, top_k], normed_trace f32 [n_layers, T, d_model] (router input). */
int        tso_model_forward(const tso_model* m, const int32_t* ids, const uint8_t* mask,
                             uint32_t T, float* logits_out, int n_threads,
                             uint16_t* hidden_trace, int32_t* topk_trace, float* normed_trace);

/* As tso_model_forward, with each layer's expert choice forced to
 * forced_topk i32 [n_layers, T, top_k] (in that order; the routing weights are
 * the softmax of this forward's own router logits at those experts).  Parity
 * tooling: it separates arithmetic differences from top-k flips at near-ties. */
int        tso_model_forward_forced(const tso_model* m, const int32_t* ids, const uint8_t* mask, uint32_t T,
                                    float* logits_out, int n_threads, uint16_t* hidden_trace, int32_t* topk_trace,
                                    float* normed_trace, const int32_t* forced_topk);

/* One MoE block half (router + experts), as blockForward runs it after the
 * post-attention norm: normed f32 [T, D] -> moe_out fp16 [T, D] (= fp16(acc*K)),
 * plus the routing (idx i32 [T, K], weights f32 [T, K]).  Weights of `layer`. */
int        tso_moe_forward(const tso_model* m, uint32_t layer, const float* normed,
                           uint32_t T, uint16_t* moe_out, int32_t* idx_out, float* w_out,
                           int n_threads);

#ifdef __cplusplus
}
#endif
#endif
