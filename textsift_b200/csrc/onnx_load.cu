// onnx_load.cu — weight upload straight from the model's ONNX files.
//
// textsift's loader (packages/textsift/src/browser/backends/wasm.ts:328-453,
// loadOnnxWeights) reads onnx/model_q4f16.onnx (graph + small initializers)
// and onnx/model_q4f16.onnx_data (external tensor bytes), maps the ONNX
// initializer names to the kernel tensor names and applies a few conversions.
// This file does the same inside the addon: a protobuf wire-format reader for
// the subset of ONNX it needs (ModelProto.graph -> GraphProto.initializer ->
// TensorProto name / data_type / dims / raw_data / float_data /
// external_data / data_location, as browser/model/onnx-reader.ts reads it),
// then the reference's mapping rules, then ts_cuda_load_tensor per tensor.
//
// Conversions, as the reference loader makes them:
//   router scales and bias   f32 -> fp16 with f32ToFp16Bits (wasm.ts:264-291:
//                            RNE for normals, half-up for subnormals, +0 for
//                            both zeros)
//   expert zero points       synthesised: every byte 0x88 (wasm.ts:428-444)
//   classifier bias          synthesised zeros fp16 [n_classes] (wasm.ts:377)
//   attention sinks          f32 [1, Hq, 1, 1] flattened to [Hq] (406-410)
//   layer count              highest L with model.layers.L.input_layernorm
//                            .weight, plus one (381-385)
#include "textsift_cuda.h"

#include <algorithm>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace {

// ONNX field numbers (onnx.proto): ModelProto.graph = 7; GraphProto.initializer
// = 5; TensorProto: dims 1, data_type 2, float_data 4, name 8, raw_data 9,
// external_data 13 (StringStringEntryProto key 1, value 2), data_location 14.
enum : uint32_t {
  kModelGraph = 7,
  kGraphInitializer = 5,
  kTensorDims = 1,
  kTensorDataType = 2,
  kTensorFloatData = 4,
  kTensorName = 8,
  kTensorRawData = 9,
  kTensorExternalData = 13,
  kTensorDataLocation = 14,
};
// TensorProto.DataType values used by the model
enum : int32_t { kOnnxFloat = 1, kOnnxUint8 = 2, kOnnxFloat16 = 10 };

struct Tensor {
  std::string name;
  int32_t dtype = 0;
  std::vector<int64_t> dims;
  const uint8_t* data = nullptr;  // raw_data / float_data bytes inside the graph buffer
  size_t len = 0;
  bool external = false;
  uint64_t ext_offset = 0, ext_length = 0;
  bool has_length = false;
};

struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;

  bool done() const { return !ok || p >= end; }
  uint64_t varint() {
    uint64_t v = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p >= end) { ok = false; return 0; }
      const uint8_t b = *p++;
      v |= (uint64_t)(b & 0x7f) << shift;
      if (!(b & 0x80)) return v;
    }
    ok = false;
    return 0;
  }
  // length-delimited payload: [q, q + n)
  bool bytes(const uint8_t** q, size_t* n) {
    const uint64_t len = varint();
    if (!ok || len > (uint64_t)(end - p)) { ok = false; return false; }
    *q = p;
    *n = (size_t)len;
    p += len;
    return true;
  }
  void skip(uint32_t wire) {
    switch (wire) {
      case 0: varint(); return;
      case 1: if (end - p < 8) ok = false; else p += 8; return;
      case 2: { const uint8_t* q; size_t n; bytes(&q, &n); return; }
      case 5: if (end - p < 4) ok = false; else p += 4; return;
      default: ok = false;
    }
  }
};

std::string str_of(const uint8_t* q, size_t n) { return std::string(reinterpret_cast<const char*>(q), n); }

bool read_tensor(const uint8_t* q, size_t n, Tensor* t) {
  Reader r{q, q + n};
  while (!r.done()) {
    const uint64_t tag = r.varint();
    const uint32_t field = (uint32_t)(tag >> 3), wire = (uint32_t)(tag & 7);
    if (field == kTensorName && wire == 2) {
      const uint8_t* s; size_t sl;
      if (r.bytes(&s, &sl)) t->name = str_of(s, sl);
    } else if (field == kTensorDataType && wire == 0) {
      t->dtype = (int32_t)r.varint();
    } else if (field == kTensorDims && wire == 0) {
      t->dims.push_back((int64_t)r.varint());
    } else if (field == kTensorDims && wire == 2) {  // packed
      const uint8_t* s; size_t sl;
      if (r.bytes(&s, &sl)) {
        Reader pr{s, s + sl};
        while (!pr.done()) t->dims.push_back((int64_t)pr.varint());
        if (!pr.ok) return false;
      }
    } else if ((field == kTensorRawData || field == kTensorFloatData) && wire == 2) {
      const uint8_t* s; size_t sl;
      if (r.bytes(&s, &sl)) { t->data = s; t->len = sl; }
    } else if (field == kTensorExternalData && wire == 2) {
      const uint8_t* s; size_t sl;
      if (!r.bytes(&s, &sl)) break;
      Reader er{s, s + sl};
      std::string key, value;
      while (!er.done()) {
        const uint64_t et = er.varint();
        const uint32_t ef = (uint32_t)(et >> 3), ew = (uint32_t)(et & 7);
        const uint8_t* v; size_t vl;
        if ((ef == 1 || ef == 2) && ew == 2 && er.bytes(&v, &vl)) (ef == 1 ? key : value) = str_of(v, vl);
        else er.skip(ew);
      }
      if (!er.ok) return false;
      if (key == "offset") t->ext_offset = std::strtoull(value.c_str(), nullptr, 10);
      else if (key == "length") { t->ext_length = std::strtoull(value.c_str(), nullptr, 10); t->has_length = true; }
    } else if (field == kTensorDataLocation && wire == 0) {
      t->external = r.varint() == 1;  // 1 = EXTERNAL
    } else {
      r.skip(wire);
    }
  }
  return r.ok;
}

bool parse_model(const uint8_t* buf, size_t len, std::map<std::string, Tensor>* out) {
  Reader r{buf, buf + len};
  while (!r.done()) {
    const uint64_t tag = r.varint();
    const uint32_t field = (uint32_t)(tag >> 3), wire = (uint32_t)(tag & 7);
    if (field == kModelGraph && wire == 2) {
      const uint8_t* g; size_t gl;
      if (!r.bytes(&g, &gl)) break;
      Reader gr{g, g + gl};
      while (!gr.done()) {
        const uint64_t gt = gr.varint();
        const uint32_t gf = (uint32_t)(gt >> 3), gw = (uint32_t)(gt & 7);
        if (gf == kGraphInitializer && gw == 2) {
          const uint8_t* s; size_t sl;
          if (!gr.bytes(&s, &sl)) break;
          Tensor t;
          if (!read_tensor(s, sl, &t)) return false;
          if (!t.name.empty()) (*out)[t.name] = t;
        } else {
          gr.skip(gw);
        }
      }
      if (!gr.ok) return false;
    } else {
      r.skip(wire);
    }
  }
  return r.ok;
}

// f32ToFp16Bits (browser/backends/wasm.ts:264-291), applied to the f32 value
uint16_t loader_f32_to_f16(float f) {
  if (f == 0.0f) return 0;  // both zeros -> +0
  uint32_t u;
  std::memcpy(&u, &f, 4);
  const uint32_t sign = (u >> 16) & 0x8000u, exp32 = (u >> 23) & 0xffu, mant23 = u & 0x7fffffu;
  if (exp32 == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant23 ? 0x200u : 0u));
  int exp16 = (int)exp32 - 127 + 15;
  if (exp16 >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (exp16 <= 0) {
    if (exp16 < -10) return (uint16_t)sign;
    const uint32_t shift = (uint32_t)(14 - exp16), mant24 = mant23 | 0x800000u;
    return (uint16_t)(sign | ((mant24 + (1u << (shift - 1))) >> shift));
  }
  const uint32_t lsb = (mant23 >> 13) & 1u;
  uint32_t m10 = (mant23 + 0xfffu + lsb) >> 13;
  if (m10 >= 0x400u) {
    m10 = 0;
    exp16 += 1;
    if (exp16 >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  }
  return (uint16_t)(sign | ((uint32_t)exp16 << 10) | m10);
}

struct Loader {
  ts_cuda_t* h;
  const std::map<std::string, Tensor>& g;
  const uint8_t* ext;
  size_t ext_len;
  char* err;
  size_t err_cap;

  int fail(const char* fmt, ...) {
    if (err && err_cap) {
      va_list ap;
      va_start(ap, fmt);
      std::vsnprintf(err, err_cap, fmt, ap);
      va_end(ap);
    }
    return TS_ERR_ARG;
  }
  const Tensor* find(const std::string& n) {
    auto it = g.find(n);
    return it == g.end() ? nullptr : &it->second;
  }
  // The tensor's bytes (inline or a slice of the external data).
  int bytes(const Tensor* t, const uint8_t** p, size_t* n) {
    if (t->external) {
      if (!ext) return fail("tensor \"%s\" is external but no external data was given", t->name.c_str());
      if (!t->has_length || t->ext_offset > ext_len || t->ext_length > ext_len - t->ext_offset)
        return fail("tensor \"%s\": external range outside the data file", t->name.c_str());
      *p = ext + t->ext_offset;
      *n = (size_t)t->ext_length;
    } else {
      if (!t->data) return fail("tensor \"%s\" has no data", t->name.c_str());
      *p = t->data;
      *n = t->len;
    }
    return TS_OK;
  }
  int put(const std::string& key, int32_t dtype, const std::vector<int64_t>& shape, const void* data, size_t n) {
    const int rc = ts_cuda_load_tensor(h, key.c_str(), dtype, shape.data(), (int32_t)shape.size(), data, n);
    if (rc != TS_OK) fail("%s: %s", key.c_str(), ts_cuda_last_error());
    return rc;
  }
  // pass-through of an ONNX initializer of the given ONNX type
  int pass(const std::string& key, const std::string& onnx, int32_t onnx_type, int32_t dtype) {
    const Tensor* t = find(onnx);
    if (!t) return fail("missing ONNX tensor \"%s\"", onnx.c_str());
    if (t->dtype != onnx_type) return fail("ONNX tensor \"%s\" has data type %d, expected %d", onnx.c_str(), t->dtype, onnx_type);
    const uint8_t* p; size_t n;
    int rc = bytes(t, &p, &n);
    return rc ? rc : put(key, dtype, t->dims, p, n);
  }
  // f32 initializer stored as fp16 (router scales and bias)
  int to_fp16(const std::string& key, const std::string& onnx) {
    const Tensor* t = find(onnx);
    if (!t) return fail("missing ONNX tensor \"%s\"", onnx.c_str());
    if (t->dtype != kOnnxFloat) return fail("ONNX tensor \"%s\" is not f32", onnx.c_str());
    const uint8_t* p; size_t n;
    int rc = bytes(t, &p, &n);
    if (rc) return rc;
    std::vector<uint16_t> h16(n / 4);
    for (size_t i = 0; i < h16.size(); i++) {
      float f;
      std::memcpy(&f, p + 4 * i, 4);
      h16[i] = loader_f32_to_f16(f);
    }
    return put(key, TS_DTYPE_F16, t->dims, h16.data(), h16.size() * 2);
  }
};

}  // namespace

extern "C" int ts_cuda_onnx_tensor_info(const uint8_t* graph, size_t graph_len, const char* name,
                                        int32_t* onnx_dtype, int64_t* dims, int32_t* ndim, int32_t* external,
                                        uint64_t* offset, uint64_t* nbytes) {
  if (!graph || !name || !onnx_dtype || !dims || !ndim || !external || !offset || !nbytes) return TS_ERR_ARG;
  std::map<std::string, Tensor> g;
  if (!parse_model(graph, graph_len, &g)) return TS_ERR_ARG;
  auto it = g.find(name);
  if (it == g.end()) return TS_ERR_ARG;
  const Tensor& t = it->second;
  *onnx_dtype = t.dtype;
  const int nd = (int)std::min<size_t>(t.dims.size(), 8);
  for (int i = 0; i < nd; i++) dims[i] = t.dims[i];
  *ndim = (int32_t)t.dims.size();
  *external = t.external ? 1 : 0;
  *offset = t.external ? t.ext_offset : (uint64_t)(t.data ? t.data - graph : 0);
  *nbytes = t.external ? t.ext_length : t.len;
  return TS_OK;
}

extern "C" int ts_cuda_load_onnx(ts_cuda_t* h, const uint8_t* graph, size_t graph_len, const uint8_t* ext_data,
                                 size_t ext_len, char* err, size_t err_cap) {
  if (err && err_cap) err[0] = 0;
  if (!h || !graph || graph_len == 0) return TS_ERR_ARG;
  std::map<std::string, Tensor> g;
  if (!parse_model(graph, graph_len, &g)) {
    if (err && err_cap) std::snprintf(err, err_cap, "not a readable ONNX model");
    return TS_ERR_ARG;
  }
  Loader ld{h, g, ext_data, ext_len, err, err_cap};
  int rc;
  // embedding, final norm, classifier (wasm.ts:356-378)
  if ((rc = ld.pass("embed.int4", "model_embed_tokens_weight_quant", kOnnxUint8, TS_DTYPE_U8)) ||
      (rc = ld.pass("embed.scales", "model_embed_tokens_weight_scales", kOnnxFloat16, TS_DTYPE_F16)) ||
      (rc = ld.pass("embed.zp", "model_embed_tokens_weight_zp", kOnnxUint8, TS_DTYPE_U8)))
    return rc;
  // count the layers first: the final norm is named after the layer past the last
  int n_layers = 0;
  for (int L = 0; L < 64; L++)
    if (ld.find("model.layers." + std::to_string(L) + ".input_layernorm.weight")) n_layers = L + 1;
  if (n_layers == 0) return ld.fail("no transformer layers found");
  if ((rc = ld.pass("final_norm", "model.layers." + std::to_string(n_layers) + ".final_norm_layernorm.weight",
                    kOnnxFloat16, TS_DTYPE_F16)))
    return rc;
  if ((rc = ld.pass("score.int4", "model_score_MatMul_weight_quant", kOnnxUint8, TS_DTYPE_U8)) ||
      (rc = ld.pass("score.scales", "model_score_MatMul_weight_scales", kOnnxFloat16, TS_DTYPE_F16)) ||
      (rc = ld.pass("score.zp", "model_score_MatMul_weight_zp", kOnnxUint8, TS_DTYPE_U8)))
    return rc;
  {
    const Tensor* q = ld.find("model_score_MatMul_weight_quant");
    const int64_t C = q->dims.empty() ? 0 : q->dims[0];
    std::vector<uint16_t> zeros((size_t)C, 0);
    if ((rc = ld.put("score.bias", TS_DTYPE_F16, {C}, zeros.data(), zeros.size() * 2))) return rc;
  }
  for (int L = 0; L < n_layers; L++) {
    const std::string l = std::to_string(L), key = "layers." + l + ".";
    for (const char* n : {"input_layernorm", "post_attention_layernorm"})
      if ((rc = ld.pass(key + n, "model.layers." + l + "." + n + ".weight", kOnnxFloat16, TS_DTYPE_F16))) return rc;
    for (const char* proj : {"q_proj", "k_proj", "v_proj", "o_proj"}) {
      const std::string qb = "model_layers_" + l + "_attn_" + proj + "_MatMul", k = key + "attn." + proj;
      if ((rc = ld.pass(k + ".int4", qb + "_weight_quant", kOnnxUint8, TS_DTYPE_U8)) ||
          (rc = ld.pass(k + ".scales", qb + "_weight_scales", kOnnxFloat16, TS_DTYPE_F16)) ||
          (rc = ld.pass(k + ".zp", qb + "_weight_zp", kOnnxUint8, TS_DTYPE_U8)) ||
          (rc = ld.pass(k + ".bias", "model.layers." + l + ".attn." + proj + ".Add.bias", kOnnxFloat16, TS_DTYPE_F16)))
        return rc;
    }
    {  // sinks: f32 [1, Hq, 1, 1] -> [Hq]
      const std::string sn = "model.layers." + l + ".attn.sinks";
      const Tensor* t = ld.find(sn);
      if (!t) return ld.fail("missing ONNX tensor \"%s\"", sn.c_str());
      if (t->dtype != kOnnxFloat) return ld.fail("ONNX tensor \"%s\" is not f32", sn.c_str());
      int64_t flat = 1;
      for (int64_t d : t->dims) flat *= d;
      const uint8_t* p; size_t n;
      if ((rc = ld.bytes(t, &p, &n)) || (rc = ld.put(key + "attn.sinks", TS_DTYPE_F32, {flat}, p, n))) return rc;
    }
    {  // router: scales and bias f32 -> fp16
      const std::string rb = "/model/layers_" + l + "/moe/router/MatMul", k = key + "router";
      if ((rc = ld.pass(k + ".int4", rb + "_weight_fp32_quant", kOnnxUint8, TS_DTYPE_U8)) ||
          (rc = ld.to_fp16(k + ".scales", rb + "_weight_fp32_scales")) ||
          (rc = ld.pass(k + ".zp", rb + "_weight_fp32_zp", kOnnxUint8, TS_DTYPE_U8)) ||
          (rc = ld.to_fp16(k + ".bias", "/model/layers." + l + "/moe/router/Add.bias_fp32")))
        return rc;
    }
    for (const auto& pr : {std::make_pair("gate_up_proj", "gate_up"), std::make_pair("down_proj", "down")}) {
      const std::string eb = std::string("model_layers_") + l + "_moe_experts_" + pr.first,
                        k = key + "experts." + pr.second;
      const Tensor* q = ld.find(eb + "_weight_quant");
      const Tensor* sc = ld.find(eb + "_weight_scales");
      if (!q || !sc || q->dims.size() != 3 || sc->dims.size() != 3)
        return ld.fail("missing or malformed expert tensors \"%s_weight_*\"", eb.c_str());
      if ((rc = ld.pass(k + ".int4", eb + "_weight_quant", kOnnxUint8, TS_DTYPE_U8)) ||
          (rc = ld.pass(k + ".scales", eb + "_weight_scales", kOnnxFloat16, TS_DTYPE_F16)))
        return rc;
      // no zero-point tensor ships: every nibble is 8 (the weights are centered on 8)
      const int64_t E = q->dims[0], N = q->dims[1], zpr = (sc->dims[2] + 1) / 2;
      std::vector<uint8_t> zp((size_t)(E * N * zpr), 0x88);
      if ((rc = ld.put(k + ".zp", TS_DTYPE_U8, {E, N, zpr}, zp.data(), zp.size())) ||
          (rc = ld.pass(k + ".bias", std::string("model.layers.") + l + ".moe.experts." + pr.first + ".bias",
                        kOnnxFloat16, TS_DTYPE_F16)))
        return rc;
    }
  }
  return TS_OK;
}
