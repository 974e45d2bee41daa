/*
 * textsift_cuda.h — C ABI of libtextsift_cuda.so, a B200 (sm_100a) backend for
 * textsift's privacy-filter forward pass.
 *
 * The library replaces, for this one path, what textsift's Node backend binds
 * through N-API (packages/textsift/src/native/backend.ts:34-60 `NativeApi`,
 * exported by packages/textsift/src/native/napi.zig:42-47) and what the WASM
 * backend computes in packages/textsift/src/browser/backends/wasm.ts:728-805
 * (`WasmBackend.forward`).  Weight upload and every device buffer live inside
 * the library; the host passes named tensors once and token ids per forward.
 *
 * Conventions (after packages/textsift/src/native/vulkan/bridge.h:5-8):
 *   - every function returning int returns TS_OK (0) or a negative TS_ERR_*;
 *     ts_cuda_last_error() gives a message for the calling thread;
 *   - constructors return NULL on failure and write a message to err (if any);
 *   - pointers documented "host" are plain host memory, "device" are CUDA
 *     device pointers of the handle's device; `stream` is a cudaStream_t
 *     (NULL = the handle's own stream).
 * Handles are not thread-safe: one caller at a time per handle, as the
 * reference serializes forwards (browser/privacy-filter.ts:522-526).
 */
#ifndef TEXTSIFT_CUDA_H
#define TEXTSIFT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TS_CUDA_ABI_VERSION 1

enum {
  TS_OK = 0,
  TS_ERR_ARG = -1,          /* bad argument (null pointer, size, unknown name) */
  TS_ERR_STATE = -2,        /* handle not ready (weights missing / not finalized) */
  TS_ERR_CUDA = -3,         /* CUDA runtime error */
  TS_ERR_UNSUPPORTED = -4,  /* shape or value the kernels do not handle */
  TS_ERR_DEVICE = -5        /* a kernel reported an error through its device flag */
};

enum { TS_DTYPE_U8 = 0, TS_DTYPE_F16 = 1, TS_DTYPE_F32 = 2, TS_DTYPE_I32 = 3 };

/* TS_MODE_FAST: tensor-core GEMMs (fp16 operands, f32 accumulation) and
 * tensor-core attention.  TS_MODE_EXACT: every GEMM and the attention in the
 * reference's own f32 summation order on CUDA cores. */
enum { TS_MODE_FAST = 0, TS_MODE_EXACT = 1 };

typedef struct ts_cuda ts_cuda_t;
typedef struct ts_cuda_w4 ts_cuda_w4_t;

/* Architecture constants; defaults are packages/textsift/src/browser/
 * backends/wasm.ts:464-483 (PF_CONFIG) with vocab 200064. */
typedef struct ts_cuda_cfg {
  int32_t device;
  uint32_t vocab, d_model, n_layers, n_heads, n_kv_heads, head_dim, window;
  uint32_t d_ff, n_experts, top_k, n_classes;
  float eps;
  double rope_theta, rope_factor, rope_original_max_pos, rope_beta_fast, rope_beta_slow;
  uint32_t max_tokens;  /* largest packed forward (sum of sequence lengths) */
  uint32_t max_seq_len; /* longest single sequence (RoPE table rows) */
  int32_t mode;         /* TS_MODE_FAST or TS_MODE_EXACT */
} ts_cuda_cfg;

int ts_cuda_abi_version(void);
void ts_cuda_default_cfg(ts_cuda_cfg* cfg);

/* Create a backend on cfg->device.  Replaces NativeApi.createBackend
 * (native/backend.ts:36; napi.zig:547 vulkanCreateBackend). */
ts_cuda_t* ts_cuda_create(const ts_cuda_cfg* cfg, char* err, size_t err_cap);

/* Upload one tensor under the name loadOnnxWeights gives it
 * (browser/backends/wasm.ts:358-446), e.g. "embed.int4",
 * "layers.0.attn.q_proj.scales", "layers.3.experts.gate_up.zp", "score.bias".
 * Bytes are copied; shape is checked against cfg.  Replaces
 * NativeApi.createBuffer per weight (native/backend.ts:140-236). */
int ts_cuda_load_tensor(ts_cuda_t* h, const char* name, int32_t dtype, const int64_t* shape, int32_t ndim,
                        const void* host_data, size_t nbytes);

/* Upload every weight from the model's ONNX files: graph = the bytes of
 * onnx/model_q4f16.onnx, ext_data = the bytes of onnx/model_q4f16.onnx_data
 * (may be NULL when no initializer is stored externally).  Replaces
 * loadOnnxWeights (browser/backends/wasm.ts:328-453): the same initializer
 * names, layer-count probe and conversions (router scales and bias f32 ->
 * fp16, expert zero points 0x88, zero classifier bias, sinks flattened to
 * [Hq]), each tensor then loaded as by ts_cuda_load_tensor.  On failure
 * returns TS_ERR_ARG (or the load error) with a message in err. */
int ts_cuda_load_onnx(ts_cuda_t* h, const uint8_t* graph, size_t graph_len, const uint8_t* ext_data, size_t ext_len,
                      char* err, size_t err_cap);

/* Host-only (no device): one initializer of an ONNX graph as the loader sees
 * it -- ONNX data type, dims (up to 8 written, *ndim = their count), whether
 * it is external, and its byte offset (in ext_data, or in graph for inline
 * data) and length.  TS_ERR_ARG if the graph does not parse or has no such
 * tensor.  Parser check for the loader (onnx-reader.ts:158-240). */
int ts_cuda_onnx_tensor_info(const uint8_t* graph, size_t graph_len, const char* name, int32_t* onnx_dtype,
                             int64_t* dims, int32_t* ndim, int32_t* external, uint64_t* offset, uint64_t* nbytes);

/* Check that every tensor is present, repack the int4 GEMM weights into
 * tensor-core tiles and build the YaRN RoPE tables.  Idempotent, like
 * InferenceBackend.warmup (browser/backends/abstract.ts:44). */
int ts_cuda_finalize(ts_cuda_t* h);

int ts_cuda_set_mode(ts_cuda_t* h, int32_t mode);

/* One sequence: ids (host) [T], mask (host, 1 = token, 0 = padding, may be
 * NULL) [T] -> logits (host) f32 [T, n_classes].  Replaces
 * InferenceBackend.forward (browser/backends/abstract.ts:46-55). */
int ts_cuda_forward(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, uint32_t T, float* logits);

/* Many independent sequences packed back to back: sequence s covers tokens
 * [seq_offsets[s], seq_offsets[s+1]) (host, n_seqs+1 entries, offsets[0] = 0).
 * Each sequence is computed exactly as its own forward would be. */
int ts_cuda_forward_packed(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                           uint32_t n_seqs, float* logits);

/* ts_cuda_forward_packed in two halves, for a host loop that keeps the GPU
 * busy: _begin copies ids/mask into pinned slot `slot` (0 or 1), enqueues
 * their upload, the forward and the logits' download into that slot on the
 * handle's stream (the download on a second stream, from the slot's own
 * device buffer), and returns without waiting; _end waits for the slot,
 * reports a device error flag raised by that forward (or by one begun after
 * it) as TS_ERR_DEVICE and copies the logits (f32 [T, n_classes]) to
 * `logits`.  Calling _begin(batch i + 1) before _end(batch i) overlaps batch
 * i's download and host copy with batch i + 1's forward; results are those
 * of ts_cuda_forward_packed.
 * A slot takes one _begin, then one _end (TS_ERR_STATE otherwise).  No
 * counterpart in the reference, whose forward() is one blocking call per
 * chunk (browser/backends/abstract.ts:29-56). */
int ts_cuda_forward_packed_begin(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                                 uint32_t n_seqs, uint32_t slot);
int ts_cuda_forward_packed_end(ts_cuda_t* h, uint32_t slot, float* logits);

/* As ts_cuda_forward_packed with ids/mask/logits in device memory, enqueued on
 * `stream` without synchronizing (seq_offsets stays a host array). */
int ts_cuda_forward_packed_device(ts_cuda_t* h, const int32_t* d_ids, const uint8_t* d_mask,
                                  const uint32_t* seq_offsets, uint32_t n_seqs, float* d_logits, void* stream);

/* As ts_cuda_forward_packed, also copying each layer's top-k expert indices
 * to topk_trace (host, i32 [n_layers][T][top_k], descending router logit).
 * Parity tooling (no counterpart in the reference): it lets a caller
 * compare routing decisions layer by layer. */
int ts_cuda_forward_trace(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                          uint32_t n_seqs, float* logits, int32_t* topk_trace);

/* As ts_cuda_forward_packed, but each sequence's logits are decoded on the
 * GPU into BIOES tags (host, u8 [T], class ids 0..32) and only the tags are
 * copied back.  Replaces the per-chunk pair backend.forward +
 * ViterbiDecoder.decode of runDetection (browser/privacy-filter.ts:497-500;
 * browser/inference/viterbi.ts:75-145), bit-identical to the decoder.
 * calibration (host, 6 values, calibration.ts:29-36): background_stay,
 * background_to_start, inside_to_continue, inside_to_end,
 * end_to_background, end_to_start; each finite with |value| < 1e20.
 * Needs the 33-class head; sequences of at most 7044 tokens. */
int ts_cuda_forward_packed_tags(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                                uint32_t n_seqs, const float* calibration, uint8_t* tags);

/* Synchronize the handle's work on `stream` and report a device-side error
 * flag (bounded waits that timed out, bad indices) as TS_ERR_DEVICE. */
int ts_cuda_check(ts_cuda_t* h, void* stream);

const char* ts_cuda_device_name(ts_cuda_t* h);  /* NativeApi.deviceName (native/backend.ts:38) */

/* Phases timed by ts_cuda_profile.  The reference only measures whole
 * forwards with performance.now() (tests/native/forward-vulkan.js:499-555);
 * these per-phase CUDA-event timings have no counterpart there. */
enum {
  TS_PHASE_EXPERT_GATE_UP = 0, /* grouped gate_up GEMM + SwiGLU epilogue (all experts in exact mode) */
  TS_PHASE_EXPERT_DOWN = 1,    /* grouped down GEMM */
  TS_PHASE_QKV = 2,            /* fused Q/K/V GEMM + RoPE epilogue */
  TS_PHASE_ATTENTION = 3,      /* banded attention */
  TS_PHASE_O = 4,              /* O projection */
  TS_PHASE_ROUTER = 5,         /* router logits + top-k + expert permutation */
  TS_PHASE_OTHER = 6,          /* norms, embedding, gathers, combine, classifier */
  TS_PHASE_COUNT = 7
};

/* enable != 0: bracket every phase of later forwards / MoE ops with CUDA
 * events on the stream they run on; always resets the accumulators and the
 * kernel-launch counter. */
int ts_cuda_profile(ts_cuda_t* h, int32_t enable);

/* Accumulated per-phase device milliseconds, phase executions and algorithmic
 * flops since the last ts_cuda_profile (arrays of TS_PHASE_COUNT, any may be
 * NULL), plus the number of kernels launched (counted with or without
 * profiling).  Waits for the recorded events. */
int ts_cuda_profile_read(ts_cuda_t* h, double* ms, uint64_t* launches, uint64_t* flops, uint64_t* total_launches);
const char* ts_cuda_last_error(void);
void ts_cuda_destroy(ts_cuda_t* h);             /* NativeApi.destroyBackend (native/backend.ts:37) */

/* ---- per-op entry points: the analogue of the reference's
 * vulkanDispatchOneShot conformance path (native/vulkan_backend.zig:239-270,
 * tests/native/vulkan/conformance-all.js).  All device pointers. ---- */

/* GatherBlockQuantized embedding (zig/wasm_exports.zig:1523-1573). */
int ts_cuda_op_gather_bq(const uint8_t* d_int4, const uint16_t* d_scales, const uint8_t* d_zp,
                         const int32_t* d_ids, uint16_t* d_out, uint32_t T, uint32_t V, uint32_t D, void* stream);

/* RMSNorm fp16 -> f32 (zig/wasm_exports.zig:229-277); d_b non-NULL selects
 * the fused add+RMSNorm (288-350), which also writes d_sum (fp16). */
int ts_cuda_op_rmsnorm(const uint16_t* d_a, const uint16_t* d_b, const uint16_t* d_gamma, uint16_t* d_sum,
                       float* d_out, uint32_t T, uint32_t D, float eps, void* stream);

/* A MatMulNBits weight (uint4 [E][N][K/2], fp16 scales [E][N][K/32], uint4
 * zero points [E][N][ceil(K/64)] or NULL, fp16 bias [E][N] or NULL; host
 * memory), uploaded and repacked for the tensor-core kernel. */
ts_cuda_w4_t* ts_cuda_w4_create(int32_t device, const uint8_t* int4, const uint16_t* scales, const uint8_t* zp,
                                const uint16_t* bias, uint32_t E, uint32_t N, uint32_t K, char* err,
                                size_t err_cap);
void ts_cuda_w4_destroy(ts_cuda_w4_t* w);

/* The dequantised fp16 operand fp16((q - zp) * scale) of expert e, exactly as
 * the tensor-core GEMM places it in shared memory, row-major [N, K]. */
int ts_cuda_op_dequant(const ts_cuda_w4_t* w, uint32_t expert, uint16_t* d_out, void* stream);

/* MatMulNBits y = x . dequant(W)^T + b for expert e (zig/wasm_exports.zig:
 * 560-766).  x: [M, K], x_dtype TS_DTYPE_F16 (fast/exact) or TS_DTYPE_F32
 * (exact only); out: [M, N], out_dtype TS_DTYPE_F16 or TS_DTYPE_F32. */
int ts_cuda_op_matmul_nbits(const ts_cuda_w4_t* w, uint32_t expert, const void* d_x, int32_t x_dtype, void* d_out,
                            int32_t out_dtype, uint32_t M, int32_t mode, void* stream);

/* Router of layer `layer`: logits, top-k with the reference tie rule,
 * softmax over k, x 1/k (browser/inference/block.ts:49-103).  Exact mode:
 * f32 logits in the reference order.  Fast mode (the forward's fast path):
 * logits on the tensor cores from fp16(x), top-k in the GEMM epilogue.
 * d_x: f32 [T, d_model]; d_idx: i32 [T, k]; d_w: f32 [T, k]. */
int ts_cuda_op_router_topk(ts_cuda_t* h, uint32_t layer, const float* d_x, int32_t* d_idx, float* d_w, uint32_t T,
                           void* stream);

/* The fast forward's router step of block `layer` from the block's residual
 * and attention output (fp16 [T, d_model] each, device): the add + RMSNorm
 * (ln2, browser/inference/block.ts:145-176), tensor-core logits naming the
 * candidates, and the exact candidate pass, which rebuilds its f32 input from
 * the norm's stored fp16 sum and 1 / rms.  d_x32 (f32 [T, d_model], may be
 * NULL) receives the norm's f32 output: the router input that d_idx / d_w
 * are the reference's top-k and weights of (block.ts:49-103).  Fast mode
 * only (top_k 4, at most 128 experts). */
int ts_cuda_op_router_addnorm(ts_cuda_t* h, uint32_t layer, const uint16_t* d_res, const uint16_t* d_attn,
                              float* d_x32, int32_t* d_idx, float* d_w, uint32_t T, void* stream);

/* MoE half of block `layer` (router + experts, browser/inference/block.ts:
 * 286-299 + expert.ts:104-212): d_x f32 [T, d_model] -> d_out fp16
 * [T, d_model] = fp16(K * sum_k w_k expert_k(x)); routing written to
 * d_idx/d_w when non-NULL.  Uses the handle's mode. */
int ts_cuda_op_moe(ts_cuda_t* h, uint32_t layer, const float* d_x, uint16_t* d_out, int32_t* d_idx, float* d_w,
                   uint32_t T, void* stream);

/* Banded GQA attention with sinks (zig/wasm_exports.zig:1286-1432) over
 * packed sequences (seq_offsets host, NULL = one sequence of T tokens).
 * q fp16 [T, Hq*hd], k/v fp16 [T, Hkv*hd], sinks f32 [Hq], mask u8 [T] or
 * NULL, out fp16 [T, Hq*hd]. */
int ts_cuda_op_banded_attention(const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v, const float* d_sinks,
                                const uint8_t* d_mask, uint16_t* d_out, uint32_t T, uint32_t Hq, uint32_t Hkv,
                                uint32_t head_dim, uint32_t window, const uint32_t* seq_offsets, uint32_t n_seqs,
                                int32_t mode, void* stream);

/* BIOES Viterbi decoding alone (ViterbiDecoder.decode,
 * browser/inference/viterbi.ts:75-145): d_logits f32 [T, 33] (device) with
 * sequences at seq_offsets (host, n_seqs + 1) -> d_tags u8 [T] (device).
 * Calibration as for ts_cuda_forward_packed_tags.  Synchronizes `stream`. */
int ts_cuda_op_viterbi(const float* d_logits, const uint32_t* seq_offsets, uint32_t n_seqs, const float* calibration,
                       uint8_t* d_tags, void* stream);

/* The banded attention above with no device allocation.  No counterpart in
 * the reference: ts_cuda_op_banded_attention allocates its scratch (sequence
 * offsets, per-token sequence info, tile list) with cudaMalloc on every call,
 * which callers that own all device memory under a fixed budget (an embedding
 * runtime, a serving loop) or that cannot afford cudaMalloc/cudaFree's
 * implicit device-wide synchronisation between their kernels cannot allow.
 * This variant keeps that scratch in one static device array of ~221 KB per
 * GPU (held until the process exits) and calls no allocator; the sequence
 * offsets reach the GPU as a kernel parameter and the tile list is built
 * there, so no host memory is copied either.
 * Limits: T <= 16384 tokens, n_seqs <= 1024 sequences per call, otherwise
 * TS_ERR_UNSUPPORTED.  Every call on a GPU shares the array: calls that
 * overlap on the GPU (e.g. on two streams at once) race and must be
 * serialized by the caller.  Every call looks up the array's address for the
 * current device (cudaGetSymbolAddress, which allocates nothing); the first
 * call on a device may load the library's device code there, so make that
 * first call before any stream capture.  Same arguments and results as
 * ts_cuda_op_banded_attention, except that it returns once the work is
 * queued on `stream` (no synchronize): synchronize the stream before reading
 * d_out. */
int ts_cuda_op_banded_attention_noalloc(const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v,
                                        const float* d_sinks, const uint8_t* d_mask, uint16_t* d_out, uint32_t T,
                                        uint32_t Hq, uint32_t Hkv, uint32_t head_dim, uint32_t window,
                                        const uint32_t* seq_offsets, uint32_t n_seqs, int32_t mode, void* stream);

/* The banded attention of the forward on the handle (its Hq, Hkv, head_dim,
 * window and mode; zig/wasm_exports.zig:1286-1432 as in
 * ts_cuda_op_banded_attention) over packed sequences (seq_offsets host,
 * n_seqs + 1 entries, at most max_tokens tokens): d_q fp16 [T, Hq*hd],
 * d_k/d_v fp16 [T, Hkv*hd], d_sinks f32 [Hq], d_mask u8 [T] or NULL ->
 * d_out fp16 [T, Hq*hd].  Scratch comes from the handle's workspace, so it
 * allocates nothing and returns once the work is queued on `stream`. */
int ts_cuda_op_attention(ts_cuda_t* h, const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v,
                         const float* d_sinks, const uint8_t* d_mask, uint16_t* d_out, const uint32_t* seq_offsets,
                         uint32_t n_seqs, void* stream);

/* RoPE alone, the reference routine rope_apply (zig/wasm_exports.zig:
 * 1460-1502; three fp16 roundings per output, its fp16 decode): d_x fp16
 * [T, H * head_dim] (interleaved pairs per head) -> d_out (may equal d_x);
 * token t uses row d_pos[t] (device i32 [T]) of the fp16 tables d_cos/d_sin
 * [rows, head_dim / 2] -- the reference indexes them by t, i.e. d_pos = 0..T-1.
 * The kernel of the exact-mode forward. */
int ts_cuda_op_rope(const uint16_t* d_x, uint16_t* d_out, const uint16_t* d_cos, const uint16_t* d_sin,
                    const int32_t* d_pos, uint32_t T, uint32_t H, uint32_t head_dim, void* stream);

/* The fast-mode Q/K/V projection of block `layer` with RoPE fused into its
 * epilogue, exactly as the forward runs it (the three matmuls and two
 * rope_apply calls of browser/inference/attention.ts:124-145): d_x fp16
 * [T, d_model] (the normed input) over packed sequences (seq_offsets host,
 * n_seqs + 1 entries; positions restart at each sequence) -> d_q fp16
 * [T, Hq*hd], d_k / d_v fp16 [T, Hkv*hd], q and k rotated with the
 * handle's YaRN tables. */
int ts_cuda_op_qkv_rope(ts_cuda_t* h, uint32_t layer, const uint16_t* d_x, const uint32_t* seq_offsets,
                        uint32_t n_seqs, uint16_t* d_q, uint16_t* d_k, uint16_t* d_v, void* stream);

/* ---- expert parallelism (BASELINE config[4]'s expert-parallel variant; the
 * reference runs one process on one device and has no counterpart) ----
 * With R ranks, each GPU holds n_experts / R consecutive experts of every
 * layer and every rank forwards its own sequences; per layer the routed rows
 * go to the ranks that hold their experts and the outputs come back (NCCL
 * grouped send/recv on the forward's stream; libnccl.so.2 is opened at run
 * time), and each token's combine is the single-GPU one (ascending expert
 * id, the reference's order).  Fast mode only; ts_cuda_op_moe is refused on
 * such a handle.  Every rank must run its forwards in the same order, each
 * layer exchanging with every other rank; each layer waits once on the host
 * for the route counts (so ts_cuda_forward_packed_device synchronizes its
 * stream per layer on such a handle). */

/* The NCCL unique id (rank 0 makes it and hands the bytes to every rank):
 * writes it to out when out is non-NULL and cap is large enough; returns its
 * size in bytes, 0 on failure. */
size_t ts_cuda_ep_unique_id(uint8_t* out, size_t cap);

/* Before ts_cuda_finalize: join the ranks' NCCL communicator (blocks until
 * all `world` ranks have called it) and keep only experts
 * [rank * n_experts / world, (rank + 1) * n_experts / world) at finalize. */
int ts_cuda_ep_init(ts_cuda_t* h, int32_t rank, int32_t world, const uint8_t* nccl_id, size_t id_len);

/* Host-only: the exchange plan of one layer on one rank.  counts: this rank's
 * routes per global expert [world * e_local]; recv_counts: routes each source
 * sends to each local expert [world][e_local].  Writes rows to send to /
 * receive from each peer (send_n, recv_n [world], may be NULL) and the local
 * grouped-GEMM tiles {local expert, first row, end row, segment start} over
 * the received rows (source-major, then expert-major; tiles [tiles_cap][4],
 * may be NULL), *n_tiles = their number. */
int ts_cuda_ep_plan(const int32_t* counts, const int32_t* recv_counts, int32_t world, int32_t e_local,
                    int32_t tile_rows, uint64_t* send_n, uint64_t* recv_n, int32_t* tiles, uint32_t tiles_cap,
                    uint32_t* n_tiles);

/* Self-test of the bounded device waits (no counterpart in the reference,
 * whose GPU work is waited for by a host fence, native/vulkan/bridge.h:95-97).
 * Enqueues on `stream` one CTA that holds TMEM while one warp waits on an
 * mbarrier nothing arrives at, with a limit of limit_us microseconds
 * (1..1000000; the kernels' own waits use 4 s), and another warp waits on a
 * second such barrier until the first one's abort releases it; the timeout
 * is recorded in the handle's device error flag and the TMEM is freed before
 * the CTA exits.  The next ts_cuda_check on `stream` then returns
 * TS_ERR_DEVICE ("bounded wait timed out") and clears the flag; the handle
 * stays usable.  d_result (device, 2 x i32, may be NULL) receives 1 for each
 * of the two waits that completed normally, 0 for each that gave up. */
int ts_cuda_selftest_wait_timeout(ts_cuda_t* h, uint32_t limit_us, int32_t* d_result, void* stream);

/* YaRN RoPE tables of the handle (browser/inference/rope.ts:117-135), fp16
 * [rows, head_dim/2] each, copied to host. */
int ts_cuda_rope_tables(ts_cuda_t* h, uint32_t rows, uint16_t* cos_out, uint16_t* sin_out);

/* ---------------------------------------------------------------------
 * Tokenizer (host CPU): the native counterpart of textsift's o200k-style
 * byte-level BPE Tokenizer (src/browser/model/tokenizer.ts), so tokenizing
 * keeps up with the GPU forward.  Same token ids and tokenToCharOffset
 * (UTF-16 code units) as Tokenizer.encode; input is UTF-8.  Calls on one
 * handle must not overlap (ts_tok_encode_batch spreads one batch over its
 * own threads).
 * ------------------------------------------------------------------- */
typedef struct ts_tok ts_tok_t;

/* Tokenizer.fromBundle (tokenizer.ts:134-221): parses tokenizer.json
 * (model.type "BPE", model.vocab, model.merges as [a, b] pairs,
 * added_tokens).  NULL on error, message in err (and ts_cuda_last_error). */
ts_tok_t* ts_tok_create(const char* tokenizer_json, size_t len, char* err, size_t err_cap);
void ts_tok_destroy(ts_tok_t* t);
/* Largest token id + 1 (Tokenizer.vocabSize, tokenizer.ts:233-236). */
uint32_t ts_tok_vocab_size(const ts_tok_t* t);

/* Tokenizer.encode (tokenizer.ts:238-291) of one UTF-8 text.  *n_tokens =
 * the token count; ids [n], char_offsets [n + 1] (UTF-16 start of each token
 * and the end of the last: tokenToCharOffset) and byte_offsets [n + 1] (the
 * same in UTF-8 bytes) are written when non-NULL, if n <= cap (else
 * TS_ERR_ARG).  All three NULL: size query.  Invalid UTF-8 -> TS_ERR_ARG. */
int ts_tok_encode(ts_tok_t* t, const char* utf8, size_t len, int32_t* ids, uint32_t* char_offsets,
                  uint32_t* byte_offsets, size_t cap, size_t* n_tokens);

/* Many texts on up to n_threads threads (0: one per hardware thread).
 * token_begin [n_texts + 1]: text i's tokens are [token_begin[i],
 * token_begin[i + 1]) of ids, starts and ends (UTF-16 start and end of
 * each token within its text), written when non-NULL if the total <= cap.
 * All three NULL: size query.  Every token covers at least one input byte,
 * so cap = the texts' total byte length always suffices and tokenizes each
 * text once (a size query followed by a filling call tokenizes twice). */
int ts_tok_encode_batch(ts_tok_t* t, const char* const* texts, const size_t* lens, uint32_t n_texts,
                        uint32_t n_threads, int32_t* ids, uint32_t* starts, uint32_t* ends, size_t cap,
                        uint64_t* token_begin);

/* Tokenizer.decode (tokenizer.ts:294-334) to UTF-8: *out_len = bytes;
 * written to out when non-NULL and *out_len <= cap.  Unknown ids are
 * skipped. */
int ts_tok_decode(const ts_tok_t* t, const int32_t* ids, size_t n, char* out, size_t cap, size_t* out_len);

#ifdef __cplusplus
}
#endif
#endif /* TEXTSIFT_CUDA_H */
