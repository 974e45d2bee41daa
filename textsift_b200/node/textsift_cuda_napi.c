/*
 * textsift_cuda_napi.c -- the N-API addon that puts libtextsift_cuda.so
 * behind textsift's Node entry point (cuda-backend.ts beside this file).
 *
 * It follows the conventions of the reference's own addon
 * (packages/textsift/src/native/napi.zig): handles travel to JavaScript as
 * BigInt (napi.zig:197-202), typed arrays are read in place through
 * napi_get_typedarray_info (napi.zig:113-126), and a failed call throws a JS
 * Error carrying the library's message (napiThrow, napi.zig:64-67).  Unlike
 * the reference's buffer/dispatch surface (native/backend.ts:34-60), the
 * weights, scratch and dispatch sequence live inside the library: the host
 * passes the ONNX files once and token ids per forward.
 *
 * Build (needs node's headers, e.g. /usr/include/node or
 * ~/.cache/node-gyp/<version>/include/node): make -C textsift_b200/node
 * NODE_INCLUDE=<dir with node_api.h>.  Node is not installed on the build
 * box of this repository, so the addon is not built or run there; its
 * declarations are checked against include/textsift_cuda.h by
 * tests/test_node_binding.py.
 */
#define NAPI_VERSION 8
#include <node_api.h>
#include <stdint.h>
#include <string.h>

#include "textsift_cuda.h"

#define CHECK_NAPI(call)                                                   \
  do {                                                                     \
    if ((call) != napi_ok) {                                               \
      napi_throw_error(env, NULL, "textsift_cuda: N-API call failed");     \
      return NULL;                                                         \
    }                                                                      \
  } while (0)

static napi_value throw_msg(napi_env env, const char* msg) {
  napi_throw_error(env, NULL, msg && msg[0] ? msg : "textsift_cuda: error");
  return NULL;
}

static napi_value throw_last(napi_env env) { return throw_msg(env, ts_cuda_last_error()); }

static napi_value undefined_value(napi_env env) {
  napi_value u;
  napi_get_undefined(env, &u);
  return u;
}

/* Arguments: up to 8, missing ones read as undefined. */
static int get_args(napi_env env, napi_callback_info info, size_t want, napi_value* argv) {
  size_t argc = want;
  if (napi_get_cb_info(env, info, &argc, argv, NULL, NULL) != napi_ok) return 0;
  for (size_t i = argc; i < want; i++) argv[i] = undefined_value(env);
  return 1;
}

static int is_nullish(napi_env env, napi_value v) {
  napi_valuetype t;
  if (napi_typeof(env, v, &t) != napi_ok) return 1;
  return t == napi_undefined || t == napi_null;
}

static void* get_handle(napi_env env, napi_value v) {
  uint64_t h = 0;
  bool lossless = false;
  if (napi_get_value_bigint_uint64(env, v, &h, &lossless) != napi_ok || h == 0) return NULL;
  return (void*)(uintptr_t)h;
}

static napi_value make_handle(napi_env env, const void* p) {
  napi_value out;
  if (napi_create_bigint_uint64(env, (uint64_t)(uintptr_t)p, &out) != napi_ok) return NULL;
  return out;
}

/* A typed array's data pointer and element count, checked against the
 * expected element type (NULL data for null / undefined when allowed). */
static int get_typed(napi_env env, napi_value v, napi_typedarray_type want, int allow_null, void** data,
                     size_t* len) {
  *data = NULL;
  *len = 0;
  if (allow_null && is_nullish(env, v)) return 1;
  bool is_ta = false;
  if (napi_is_typedarray(env, v, &is_ta) != napi_ok || !is_ta) return 0;
  napi_typedarray_type t;
  napi_value ab;
  size_t off;
  if (napi_get_typedarray_info(env, v, &t, len, data, &ab, &off) != napi_ok) return 0;
  return t == want;
}

static int get_u32(napi_env env, napi_value v, uint32_t dflt, uint32_t* out) {
  if (is_nullish(env, v)) {
    *out = dflt;
    return 1;
  }
  return napi_get_value_uint32(env, v, out) == napi_ok;
}

/* cudaCreateBackend(device?: number, maxTokens?: number, maxSeqLen?: number): bigint */
static napi_value CreateBackend(napi_env env, napi_callback_info info) {
  napi_value a[3];
  if (!get_args(env, info, 3, a)) return throw_msg(env, "cudaCreateBackend: bad arguments");
  ts_cuda_cfg cfg;
  ts_cuda_default_cfg(&cfg);
  uint32_t dev = 0;
  if (!get_u32(env, a[0], 0, &dev) || !get_u32(env, a[1], cfg.max_tokens, &cfg.max_tokens) ||
      !get_u32(env, a[2], cfg.max_seq_len, &cfg.max_seq_len))
    return throw_msg(env, "cudaCreateBackend: device, maxTokens and maxSeqLen must be numbers");
  cfg.device = (int32_t)dev;
  char err[1024];
  ts_cuda_t* h = ts_cuda_create(&cfg, err, sizeof err);
  if (!h) return throw_msg(env, err);
  return make_handle(env, h);
}

/* cudaDestroyBackend(h: bigint): void */
static napi_value DestroyBackend(napi_env env, napi_callback_info info) {
  napi_value a[1];
  if (get_args(env, info, 1, a)) ts_cuda_destroy((ts_cuda_t*)get_handle(env, a[0]));
  return undefined_value(env);
}

/* cudaDeviceName(h: bigint): string */
static napi_value DeviceName(napi_env env, napi_callback_info info) {
  napi_value a[1], out;
  if (!get_args(env, info, 1, a)) return throw_msg(env, "cudaDeviceName: bad arguments");
  const char* name = ts_cuda_device_name((ts_cuda_t*)get_handle(env, a[0]));
  CHECK_NAPI(napi_create_string_utf8(env, name, NAPI_AUTO_LENGTH, &out));
  return out;
}

/* cudaLoadOnnx(h, graph: Uint8Array, extData: Uint8Array | null): void --
 * the reference's loadOnnxWeights (browser/backends/wasm.ts:328-453), run
 * inside the library on the model's two files. */
static napi_value LoadOnnx(napi_env env, napi_callback_info info) {
  napi_value a[3];
  void *g, *x;
  size_t gl, xl;
  if (!get_args(env, info, 3, a) || !get_typed(env, a[1], napi_uint8_array, 0, &g, &gl) ||
      !get_typed(env, a[2], napi_uint8_array, 1, &x, &xl))
    return throw_msg(env, "cudaLoadOnnx(h, graph: Uint8Array, extData: Uint8Array | null)");
  char err[1024];
  if (ts_cuda_load_onnx((ts_cuda_t*)get_handle(env, a[0]), (const uint8_t*)g, gl, (const uint8_t*)x, xl, err,
                        sizeof err) != TS_OK)
    return throw_msg(env, err);
  return undefined_value(env);
}

/* cudaLoadTensor(h, name: string, dtype: number, bytes: Uint8Array): void */
static napi_value LoadTensor(napi_env env, napi_callback_info info) {
  napi_value a[4];
  char name[256];
  size_t nl = 0;
  int32_t dtype = 0;
  void* data;
  size_t len;
  if (!get_args(env, info, 4, a) ||
      napi_get_value_string_utf8(env, a[1], name, sizeof name, &nl) != napi_ok ||
      napi_get_value_int32(env, a[2], &dtype) != napi_ok || !get_typed(env, a[3], napi_uint8_array, 0, &data, &len))
    return throw_msg(env, "cudaLoadTensor(h, name: string, dtype: number, bytes: Uint8Array)");
  if (ts_cuda_load_tensor((ts_cuda_t*)get_handle(env, a[0]), name, dtype, NULL, 0, data, len) != TS_OK)
    return throw_last(env);
  return undefined_value(env);
}

/* cudaFinalize(h): void -- InferenceBackend.warmup's upload step (idempotent) */
static napi_value Finalize(napi_env env, napi_callback_info info) {
  napi_value a[1];
  if (!get_args(env, info, 1, a)) return throw_msg(env, "cudaFinalize: bad arguments");
  if (ts_cuda_finalize((ts_cuda_t*)get_handle(env, a[0])) != TS_OK) return throw_last(env);
  return undefined_value(env);
}

static napi_value new_typed(napi_env env, napi_typedarray_type t, size_t n, size_t esz, void** data) {
  napi_value ab, out;
  if (napi_create_arraybuffer(env, n * esz > 0 ? n * esz : 1, data, &ab) != napi_ok) return NULL;
  if (napi_create_typedarray(env, t, n, ab, 0, &out) != napi_ok) return NULL;
  return out;
}

/* cudaForwardPacked(h, ids: Int32Array, mask: Uint8Array | null,
 *                   offsets: Uint32Array): Float32Array [T * 33] --
 * InferenceBackend.forward (browser/backends/abstract.ts:46-55) for many
 * chunks in one launch; one chunk = offsets [0, T]. */
static napi_value ForwardPacked(napi_env env, napi_callback_info info) {
  napi_value a[4];
  void *ids, *mask, *offs;
  size_t T, ml, no;
  if (!get_args(env, info, 4, a) || !get_typed(env, a[1], napi_int32_array, 0, &ids, &T) ||
      !get_typed(env, a[2], napi_uint8_array, 1, &mask, &ml) || !get_typed(env, a[3], napi_uint32_array, 0, &offs, &no))
    return throw_msg(env, "cudaForwardPacked(h, ids: Int32Array, mask: Uint8Array | null, offsets: Uint32Array)");
  if (no < 2 || ((const uint32_t*)offs)[no - 1] != T || (mask && ml != T))
    return throw_msg(env, "cudaForwardPacked: offsets must run from 0 to ids.length, mask as long as ids");
  void* out_data;
  napi_value out = new_typed(env, napi_float32_array, T * 33, sizeof(float), &out_data);
  if (!out) return throw_msg(env, "cudaForwardPacked: allocation failed");
  if (T > 0 && ts_cuda_forward_packed((ts_cuda_t*)get_handle(env, a[0]), (const int32_t*)ids, (const uint8_t*)mask,
                                      (const uint32_t*)offs, (uint32_t)(no - 1), (float*)out_data) != TS_OK)
    return throw_last(env);
  return out;
}

/* cudaForwardPackedTags(h, ids, mask | null, offsets, calibration:
 * Float32Array [6]): Uint8Array [T] -- the per-chunk pair backend.forward +
 * ViterbiDecoder.decode of runDetection (browser/privacy-filter.ts:497-500),
 * decoded on the GPU; only the BIOES tags come back. */
static napi_value ForwardPackedTags(napi_env env, napi_callback_info info) {
  napi_value a[5];
  void *ids, *mask, *offs, *cal;
  size_t T, ml, no, nc;
  if (!get_args(env, info, 5, a) || !get_typed(env, a[1], napi_int32_array, 0, &ids, &T) ||
      !get_typed(env, a[2], napi_uint8_array, 1, &mask, &ml) ||
      !get_typed(env, a[3], napi_uint32_array, 0, &offs, &no) || !get_typed(env, a[4], napi_float32_array, 0, &cal, &nc))
    return throw_msg(env, "cudaForwardPackedTags(h, ids, mask | null, offsets: Uint32Array, calibration: Float32Array)");
  if (no < 2 || ((const uint32_t*)offs)[no - 1] != T || (mask && ml != T) || nc != 6)
    return throw_msg(env, "cudaForwardPackedTags: offsets from 0 to ids.length, mask as long as ids, 6 calibration values");
  void* out_data;
  napi_value out = new_typed(env, napi_uint8_array, T, 1, &out_data);
  if (!out) return throw_msg(env, "cudaForwardPackedTags: allocation failed");
  if (T > 0 && ts_cuda_forward_packed_tags((ts_cuda_t*)get_handle(env, a[0]), (const int32_t*)ids, (const uint8_t*)mask,
                                           (const uint32_t*)offs, (uint32_t)(no - 1), (const float*)cal,
                                           (uint8_t*)out_data) != TS_OK)
    return throw_last(env);
  return out;
}

/* tokCreate(tokenizerJson: Uint8Array): bigint -- Tokenizer.fromBundle
 * (browser/model/tokenizer.ts:134-221) in the library */
static napi_value TokCreate(napi_env env, napi_callback_info info) {
  napi_value a[1];
  void* j;
  size_t jl;
  if (!get_args(env, info, 1, a) || !get_typed(env, a[0], napi_uint8_array, 0, &j, &jl))
    return throw_msg(env, "tokCreate(tokenizerJson: Uint8Array)");
  char err[1024];
  ts_tok_t* t = ts_tok_create((const char*)j, jl, err, sizeof err);
  if (!t) return throw_msg(env, err);
  return make_handle(env, t);
}

/* tokDestroy(t: bigint): void */
static napi_value TokDestroy(napi_env env, napi_callback_info info) {
  napi_value a[1];
  if (get_args(env, info, 1, a)) ts_tok_destroy((ts_tok_t*)get_handle(env, a[0]));
  return undefined_value(env);
}

/* tokEncode(t, utf8: Uint8Array): { ids: Int32Array, charOffsets: Uint32Array }
 * -- Tokenizer.encode (tokenizer.ts:238-291): ids and tokenToCharOffset
 * (UTF-16 code units, one more entry than ids). */
static napi_value TokEncode(napi_env env, napi_callback_info info) {
  napi_value a[2];
  void* s;
  size_t sl;
  if (!get_args(env, info, 2, a) || !get_typed(env, a[1], napi_uint8_array, 0, &s, &sl))
    return throw_msg(env, "tokEncode(t, utf8: Uint8Array)");
  ts_tok_t* t = (ts_tok_t*)get_handle(env, a[0]);
  /* every token covers at least one input byte: sl + 1 entries suffice */
  void *ids_d, *off_d;
  napi_value ids = new_typed(env, napi_int32_array, sl, 4, &ids_d);
  napi_value offs = new_typed(env, napi_uint32_array, sl + 1, 4, &off_d);
  if (!ids || !offs) return throw_msg(env, "tokEncode: allocation failed");
  size_t n = 0;
  if (ts_tok_encode(t, (const char*)s, sl, (int32_t*)ids_d, (uint32_t*)off_d, NULL, sl, &n) != TS_OK)
    return throw_last(env);
  napi_value ids_ab, off_ab, ids_n, off_n, out;
  size_t dummy_len, dummy_off;
  napi_typedarray_type tt;
  void* dummy;
  CHECK_NAPI(napi_get_typedarray_info(env, ids, &tt, &dummy_len, &dummy, &ids_ab, &dummy_off));
  CHECK_NAPI(napi_get_typedarray_info(env, offs, &tt, &dummy_len, &dummy, &off_ab, &dummy_off));
  CHECK_NAPI(napi_create_typedarray(env, napi_int32_array, n, ids_ab, 0, &ids_n));
  CHECK_NAPI(napi_create_typedarray(env, napi_uint32_array, n + 1, off_ab, 0, &off_n));
  CHECK_NAPI(napi_create_object(env, &out));
  CHECK_NAPI(napi_set_named_property(env, out, "ids", ids_n));
  CHECK_NAPI(napi_set_named_property(env, out, "charOffsets", off_n));
  return out;
}

static napi_value Init(napi_env env, napi_value exports) {
  const napi_property_descriptor fns[] = {
      {"cudaCreateBackend", NULL, CreateBackend, NULL, NULL, NULL, napi_default, NULL},
      {"cudaDestroyBackend", NULL, DestroyBackend, NULL, NULL, NULL, napi_default, NULL},
      {"cudaDeviceName", NULL, DeviceName, NULL, NULL, NULL, napi_default, NULL},
      {"cudaLoadOnnx", NULL, LoadOnnx, NULL, NULL, NULL, napi_default, NULL},
      {"cudaLoadTensor", NULL, LoadTensor, NULL, NULL, NULL, napi_default, NULL},
      {"cudaFinalize", NULL, Finalize, NULL, NULL, NULL, napi_default, NULL},
      {"cudaForwardPacked", NULL, ForwardPacked, NULL, NULL, NULL, napi_default, NULL},
      {"cudaForwardPackedTags", NULL, ForwardPackedTags, NULL, NULL, NULL, napi_default, NULL},
      {"tokCreate", NULL, TokCreate, NULL, NULL, NULL, napi_default, NULL},
      {"tokDestroy", NULL, TokDestroy, NULL, NULL, NULL, napi_default, NULL},
      {"tokEncode", NULL, TokEncode, NULL, NULL, NULL, napi_default, NULL},
  };
  if (napi_define_properties(env, exports, sizeof fns / sizeof fns[0], fns) != napi_ok) return NULL;
  return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, Init)
