// runtime.cu — libtextsift_cuda: model handle, weight upload, forward pass and
// the extern "C" ABI declared in include/textsift_cuda.h.
//
// Forward composition follows packages/textsift/src/browser/inference/
// model.ts:50-105, block.ts:108-197, attention.ts:45-215 and
// expert.ts:104-212; tensor names follow loadOnnxWeights
// (browser/backends/wasm.ts:358-446).  All weights and activations stay in
// HBM; a forward over many packed sequences is one pass of ~15 launches per
// layer with no host round trip.
#include "textsift_cuda.h"
#include "ts_common.cuh"
#include "ts_kernels.h"
#include "ts_simt.h"
#include "ts_ep.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define TS_CUDA_TRY(expr)                                                                    \
  do {                                                                                       \
    cudaError_t e_ = (expr);                                                                 \
    if (e_ != cudaSuccess) return fail(TS_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// math.zig:54-82 on the host (RoPE tables are built once per handle).
uint16_t host_f32_to_f16_ref(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  uint32_t sign = (u >> 16) & 0x8000u, exp32 = (u >> 23) & 0xffu, mant = u & 0x7fffffu;
  if (exp32 == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
  int e16 = (int)exp32 - 112;
  if (e16 >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (e16 <= 0) {
    if (e16 < -10) return (uint16_t)sign;
    uint32_t shift = (uint32_t)(14 - e16);
    return (uint16_t)(sign | (((mant | 0x800000u) + (1u << (shift - 1))) >> shift));
  }
  uint32_t m10 = (mant + 0xfffu + ((mant >> 13) & 1u)) >> 13;
  uint32_t ue = (uint32_t)e16;
  if (m10 >= 0x400u) {
    m10 = 0;
    if (++ue >= 0x1fu) return (uint16_t)(sign | 0x7c00u);
  }
  return (uint16_t)(sign | (ue << 10) | m10);
}

// YaRN cos/sin tables (browser/inference/rope.ts:27-144): the reference's
// published method in double precision, stored through f32 into fp16 with
// +0 for zero (rope.ts:78-104).
void build_rope_tables(const ts_cuda_cfg& c, uint32_t rows, std::vector<uint16_t>& cs, std::vector<uint16_t>& sn) {
  const uint32_t hd = c.head_dim, half = hd / 2;
  std::vector<float> extrap(half), interp(half), inv(half);
  for (uint32_t i = 0; i < half; i++) {
    double pf = std::pow(c.rope_theta, (double)(2 * i) / (double)hd);
    extrap[i] = (float)(1.0 / pf);
    interp[i] = (float)(1.0 / (c.rope_factor * pf));
  }
  const double two_pi = 2.0 * 3.141592653589793;
  auto corr = [&](double rot) {
    return ((double)hd * std::log(c.rope_original_max_pos / (rot * two_pi))) / (2.0 * std::log(c.rope_theta));
  };
  double lo = corr(c.rope_beta_fast), hi = corr(c.rope_beta_slow);
  if (lo < 0) lo = 0;
  if (hi > (double)(hd - 1)) hi = (double)(hd - 1);
  const double rmax = hi == lo ? lo + 0.001 : hi;
  for (uint32_t i = 0; i < half; i++) {
    double lin = ((double)i - lo) / (rmax - lo);
    double ramp = lin < 0 ? 0 : (lin > 1 ? 1 : lin);
    double ef = 1.0 - ramp;
    double a = (double)interp[i] * (1.0 - ef);
    double b = (double)extrap[i] * ef;
    inv[i] = (float)(a + b);
  }
  const double att = c.rope_factor <= 1.0 ? 1.0 : 0.1 * std::log(c.rope_factor) + 1.0;
  cs.resize((size_t)rows * half);
  sn.resize((size_t)rows * half);
  for (uint32_t t = 0; t < rows; t++)
    for (uint32_t i = 0; i < half; i++) {
      double ang = (double)t * (double)inv[i];
      double cv = std::cos(ang) * att, sv = std::sin(ang) * att;
      cs[(size_t)t * half + i] = cv == 0.0 ? 0 : host_f32_to_f16_ref((float)cv);
      sn[(size_t)t * half + i] = sv == 0.0 ? 0 : host_f32_to_f16_ref((float)sv);
    }
}

template <typename T>
struct DevArr {
  T* p = nullptr;
  size_t n = 0;
  DevArr() = default;
  DevArr(const DevArr&) = delete;
  DevArr& operator=(const DevArr&) = delete;
  ~DevArr() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  cudaError_t alloc(size_t count) {
    if (count <= n && p) return cudaSuccess;
    release();
    n = count;
    return cudaMalloc(&p, count * sizeof(T) + 16);
  }
};

// One MatMulNBits weight (E experts of [N, K]) in reference layout plus its
// tensor-core tiles.
struct W4Dev {
  uint32_t E = 1, N = 0, K = 0, BN = 128;
  DevArr<uint8_t> int4, zp, blobs;
  DevArr<uint16_t> scales, bias;
  bool has_zp = true;
  ts::W4Tiles tiles() const {
    ts::W4Tiles t;
    t.blobs = blobs.p;
    t.N = N;
    t.K = K;
    t.BN = BN;
    t.n_tiles = (N + BN - 1) / BN;
    t.n_kc = (K + ts::kChunkK - 1) / ts::kChunkK;
    t.expert_stride = (uint64_t)t.n_tiles * t.n_kc * ts::w4_blob_bytes(BN);
    t.bias = bias.p;
    return t;
  }
  ts::ExactArgs exact() const {
    ts::ExactArgs a;
    a.w_int4 = int4.p;
    a.w_scales = scales.p;
    a.w_zp = has_zp ? zp.p : nullptr;
    a.bias = bias.p;
    a.w_int4_estride = (uint64_t)N * (K / 2);
    a.w_scales_estride = (uint64_t)N * (K / 32);
    a.w_zp_estride = (uint64_t)N * ((K / 32 + 1) / 2);
    a.bias_estride = N;
    a.N = N;
    a.K = K;
    return a;
  }
};

// Upload host arrays (reference layout) into a W4Dev and build its tiles.
int w4_upload(W4Dev& w, const uint8_t* int4, const uint16_t* scales, const uint8_t* zp, const uint16_t* bias,
              uint32_t E, uint32_t N, uint32_t K, uint32_t BN, bool tc, int* d_bad, cudaStream_t st) {
  if (K % 32 != 0 || N == 0 || K == 0 || E == 0) return fail(TS_ERR_UNSUPPORTED, "int4 weight: K=%u must be a multiple of 32", K);
  w.E = E; w.N = N; w.K = K; w.BN = BN;
  const size_t n4 = (size_t)E * N * (K / 2), ns = (size_t)E * N * (K / 32), nz = (size_t)E * N * ((K / 32 + 1) / 2);
  TS_CUDA_TRY(w.int4.alloc(n4));
  TS_CUDA_TRY(w.scales.alloc(ns));
  TS_CUDA_TRY(w.bias.alloc((size_t)E * N));
  TS_CUDA_TRY(cudaMemcpyAsync(w.int4.p, int4, n4, cudaMemcpyHostToDevice, st));
  TS_CUDA_TRY(cudaMemcpyAsync(w.scales.p, scales, ns * 2, cudaMemcpyHostToDevice, st));
  if (bias) TS_CUDA_TRY(cudaMemcpyAsync(w.bias.p, bias, (size_t)E * N * 2, cudaMemcpyHostToDevice, st));
  else TS_CUDA_TRY(cudaMemsetAsync(w.bias.p, 0, (size_t)E * N * 2, st));
  w.has_zp = zp != nullptr;
  if (zp) {
    TS_CUDA_TRY(w.zp.alloc(nz));
    TS_CUDA_TRY(cudaMemcpyAsync(w.zp.p, zp, nz, cudaMemcpyHostToDevice, st));
  }
  if (tc) {
    ts::W4Tiles t = w.tiles();
    TS_CUDA_TRY(w.blobs.alloc((size_t)E * t.expert_stride));
    TS_CUDA_TRY(ts::launch_w4_repack(w.int4.p, w.scales.p, w.has_zp ? w.zp.p : nullptr, E, N, K, BN, w.blobs.p, st));
    if (d_bad) TS_CUDA_TRY(ts::launch_count_bad_scales(w.scales.p, ns, d_bad, st));
  }
  return TS_OK;
}

struct HostTensor {
  std::vector<uint8_t> bytes;
  int32_t dtype = 0;
};

struct LayerDev {
  DevArr<uint16_t> ln1, ln2;
  DevArr<float> sinks;
  W4Dev qkv, o, router, gate_up, down;
  DevArr<float> rbound;  // the router's bound table (ts::router_bound_table), E <= kMaxRouterExperts
  DevArr<float> rsz;     // the router's per-block scale and zero-point table
};

struct Workspace {
  uint32_t cap = 0;  // tokens
  DevArr<int32_t> ids;
  DevArr<uint8_t> mask, tags;
  DevArr<uint32_t> offs;
  DevArr<int> pos, sstart, slen;
  DevArr<uint16_t> x0, x1, xn16, q, k, v, attn, o16, res2, qkv16, down16;
  DevArr<float> n32, hf32, rlogits, rw;
  DevArr<int32_t> ridx;
  DevArr<int> counts, seg_start, seg_end, perm_tok, route_pos, n_tiles, n_tiles_tc, hist;
  DevArr<int4> tiles, tiles_tc;  // 128-row tiles (exact path), gemm_tm_rows()-row tiles (tensor cores)
  DevArr<int4> rcand;            // router candidates, 32 bytes per token (kEpiRouterCert)
  DevArr<float> absum;           // sum |x| of each token's router input
  DevArr<float> rinv;            // the add+norm's 1 / rms of each token (fast mode)
  DevArr<int2> atiles;
  DevArr<uint16_t> aperm16, glu16;
  DevArr<float> aperm32, gu32, glu32, down32;
  DevArr<float> logits;
  bool exact_ready = false;
};

}  // namespace

struct ts_cuda {
  ts_cuda_cfg cfg{};
  cudaStream_t stream = nullptr;
  std::string name;
  std::map<std::string, HostTensor> staged;
  bool finalized = false;
  // device weights
  DevArr<uint8_t> embed_int4, embed_zp;
  DevArr<uint8_t> embed_rows;  // the packed table the forward gathers from (ts::embed_row_bytes per row)
  DevArr<uint16_t> embed_scales, final_norm;
  W4Dev score;
  std::vector<std::unique_ptr<LayerDev>> layers;
  DevArr<uint16_t> rope_cos, rope_sin;
  DevArr<uint32_t> rope_cs;  // cos | sin << 16 per (position, pair): one load in the QKV epilogue
  DevArr<int> err;
  Workspace ws;
  // pinned staging for the host-pointer forward
  uint8_t* pin = nullptr;
  size_t pin_bytes = 0;
  // pinned ring for each forward's small host -> device copies (sequence
  // offsets, attention tile list): a slot is reused only after the copies
  // queued from it have executed, so the host can run forwards ahead
  struct Stage { uint8_t* p = nullptr; size_t cap = 0; cudaEvent_t done = nullptr; };
  Stage stage[4];
  uint32_t stage_next = 0;
  // ts_cuda_forward_packed_begin/_end: two slots, each with its own device
  // logits and a pinned block (logits, ids, the device error flag, mask); a
  // slot's logits come down on copy_st (after the event `fwd` that ends its
  // forward), so the download overlaps the next forward on `stream`
  struct Slot {
    uint8_t* p = nullptr;
    DevArr<float> dlog;
    cudaEvent_t fwd = nullptr, done = nullptr;
    uint32_t T = 0;
    bool busy = false;
  };
  Slot slot[2];
  cudaStream_t copy_st = nullptr;
  // when set, each layer's top-k experts are copied here ([n_layers][T][top_k])
  int32_t* trace_topk = nullptr;
  // expert parallelism (ts_cuda_ep_init): this rank holds experts
  // [e_first, e_first + e_local) of every layer; ep_world = 0 when off
  int ep_world = 0, ep_rank = 0;
  uint32_t e_first = 0, e_local = 0;
  void* ep_comm = nullptr;
  int* ep_hcounts = nullptr;  // pinned: E route counts of this rank, then [world][e_local] received
  uint64_t ep_cap = 0;        // rows the receive buffers hold
  DevArr<int> ep_rc;          // [world][e_local] route counts received
  DevArr<uint16_t> ep_recv, ep_glu, ep_out;  // received rows, their SwiGLU, their expert outputs
  DevArr<int4> ep_tiles;
  DevArr<int> ep_ntiles;
  // kernel launches issued by forwards / MoE ops (ts_cuda_profile_read)
  uint64_t n_launch = 0;
  // optional per-phase CUDA-event timing (ts_cuda_profile)
  bool prof = false;
  struct Mark { int phase; cudaEvent_t a, b; uint64_t flops; };
  std::vector<Mark> marks;
  std::vector<cudaEvent_t> ev_pool;
  double ph_ms[TS_PHASE_COUNT] = {0};
  uint64_t ph_launch[TS_PHASE_COUNT] = {0}, ph_flops[TS_PHASE_COUNT] = {0};
};

struct ts_cuda_w4 {
  int device = 0;
  cudaStream_t stream = nullptr;
  W4Dev w;
  DevArr<int> err;
};

namespace {

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Expected byte size and dtype of each named tensor (loader layout).
bool expected_tensor(const ts_cuda_cfg& c, const std::string& name, size_t& bytes, int32_t& dtype) {
  const size_t D = c.d_model, V = c.vocab, C = c.n_classes, E = c.n_experts, F = c.d_ff;
  const size_t Hq = c.n_heads, Hkv = c.n_kv_heads, hd = c.head_dim;
  auto i4 = [&](const std::string& f, size_t Ex, size_t N, size_t K) {
    if (f == "int4") { bytes = Ex * N * K / 2; dtype = TS_DTYPE_U8; return true; }
    if (f == "scales") { bytes = Ex * N * (K / 32) * 2; dtype = TS_DTYPE_F16; return true; }
    if (f == "zp") { bytes = Ex * N * ((K / 32 + 1) / 2); dtype = TS_DTYPE_U8; return true; }
    if (f == "bias") { bytes = Ex * N * 2; dtype = TS_DTYPE_F16; return true; }
    return false;
  };
  if (name == "embed.int4") { bytes = V * D / 2; dtype = TS_DTYPE_U8; return true; }
  if (name == "embed.scales") { bytes = V * (D / 32) * 2; dtype = TS_DTYPE_F16; return true; }
  if (name == "embed.zp") { bytes = V * ((D / 32 + 1) / 2); dtype = TS_DTYPE_U8; return true; }
  if (name == "final_norm") { bytes = D * 2; dtype = TS_DTYPE_F16; return true; }
  if (name.rfind("score.", 0) == 0) return i4(name.substr(6), 1, C, D);
  unsigned L = 0;
  int n = 0;
  if (sscanf(name.c_str(), "layers.%u.%n", &L, &n) == 1 && n > 0 && L < c.n_layers) {
    std::string r = name.substr((size_t)n);
    if (r == "input_layernorm" || r == "post_attention_layernorm") { bytes = D * 2; dtype = TS_DTYPE_F16; return true; }
    if (r == "attn.sinks") { bytes = Hq * 4; dtype = TS_DTYPE_F32; return true; }
    if (r.rfind("attn.q_proj.", 0) == 0) return i4(r.substr(12), 1, Hq * hd, D);
    if (r.rfind("attn.k_proj.", 0) == 0) return i4(r.substr(12), 1, Hkv * hd, D);
    if (r.rfind("attn.v_proj.", 0) == 0) return i4(r.substr(12), 1, Hkv * hd, D);
    if (r.rfind("attn.o_proj.", 0) == 0) return i4(r.substr(12), 1, D, Hq * hd);
    if (r.rfind("router.", 0) == 0) return i4(r.substr(7), 1, E, D);
    if (r.rfind("experts.gate_up.", 0) == 0) return i4(r.substr(16), E, 2 * F, D);
    if (r.rfind("experts.down.", 0) == 0) return i4(r.substr(13), E, D, F);
  }
  return false;
}

std::vector<std::string> required_names(const ts_cuda_cfg& c) {
  std::vector<std::string> v = {"embed.int4", "embed.scales", "embed.zp", "final_norm",
                                "score.int4", "score.scales", "score.zp"};
  const char* i4f[] = {"int4", "scales", "zp", "bias"};
  for (uint32_t L = 0; L < c.n_layers; L++) {
    std::string p = "layers." + std::to_string(L) + ".";
    v.push_back(p + "input_layernorm");
    v.push_back(p + "post_attention_layernorm");
    v.push_back(p + "attn.sinks");
    for (const char* pr : {"attn.q_proj.", "attn.k_proj.", "attn.v_proj.", "attn.o_proj.", "router.",
                           "experts.gate_up.", "experts.down."})
      for (const char* f : i4f) v.push_back(p + pr + f);
  }
  return v;
}

const uint8_t* staged_ptr(ts_cuda* h, const std::string& n) {
  auto it = h->staged.find(n);
  return it == h->staged.end() ? nullptr : it->second.bytes.data();
}

int ensure_workspace(ts_cuda* h, bool exact) {
  Workspace& w = h->ws;
  const ts_cuda_cfg& c = h->cfg;
  const size_t T = c.max_tokens, D = c.d_model, K = c.top_k, E = c.n_experts, F = c.d_ff;
  const size_t Q = (size_t)c.n_heads * c.head_dim, KV = (size_t)c.n_kv_heads * c.head_dim;
  const size_t R = T * K;
  if (w.cap == 0) {
    TS_CUDA_TRY(w.ids.alloc(T));
    TS_CUDA_TRY(w.mask.alloc(T));
    TS_CUDA_TRY(w.offs.alloc(T + 1));
    TS_CUDA_TRY(w.tags.alloc(T));
    TS_CUDA_TRY(w.pos.alloc(T));
    TS_CUDA_TRY(w.sstart.alloc(T));
    TS_CUDA_TRY(w.slen.alloc(T));
    TS_CUDA_TRY(w.x0.alloc(T * D));
    TS_CUDA_TRY(w.x1.alloc(T * D));
    TS_CUDA_TRY(w.xn16.alloc(T * D));
    TS_CUDA_TRY(w.q.alloc(T * Q));
    TS_CUDA_TRY(w.k.alloc(T * KV));
    TS_CUDA_TRY(w.v.alloc(T * KV));
    TS_CUDA_TRY(w.attn.alloc(T * Q));
    TS_CUDA_TRY(w.o16.alloc(T * D));
    TS_CUDA_TRY(w.res2.alloc(T * D));
    TS_CUDA_TRY(w.n32.alloc(T * D));
    TS_CUDA_TRY(w.rlogits.alloc(T * E));
    TS_CUDA_TRY(w.ridx.alloc(R));
    TS_CUDA_TRY(w.rcand.alloc(2 * T));
    TS_CUDA_TRY(w.absum.alloc(T));
    TS_CUDA_TRY(w.rinv.alloc(T));
    TS_CUDA_TRY(w.rw.alloc(R));
    TS_CUDA_TRY(w.counts.alloc(E));
    TS_CUDA_TRY(w.hist.alloc((size_t)ts::route_chunks((uint32_t)T) * E));
    TS_CUDA_TRY(w.seg_end.alloc(E));
    TS_CUDA_TRY(w.seg_start.alloc(E));
    TS_CUDA_TRY(w.perm_tok.alloc(R));
    TS_CUDA_TRY(w.route_pos.alloc(R));
    TS_CUDA_TRY(w.n_tiles.alloc(1));
    TS_CUDA_TRY(w.tiles.alloc(R / 128 + E + 1));
    TS_CUDA_TRY(w.n_tiles_tc.alloc(1));
    TS_CUDA_TRY(w.tiles_tc.alloc(R / ts::gemm_tm_rows() + E + 1));
    TS_CUDA_TRY(w.aperm16.alloc(R * D));
    TS_CUDA_TRY(w.glu16.alloc(R * F));
    TS_CUDA_TRY(w.down32.alloc(R * D));
    TS_CUDA_TRY(w.down16.alloc(R * D));
    TS_CUDA_TRY(w.logits.alloc(T * c.n_classes));
    TS_CUDA_TRY(w.qkv16.alloc(T * (Q + 2 * KV)));
    TS_CUDA_TRY(w.atiles.alloc(ts::attention_max_tiles((uint32_t)T, (uint32_t)T)));
    w.cap = (uint32_t)T;
  }
  if (exact && !w.exact_ready) {
    TS_CUDA_TRY(w.hf32.alloc(T * D));
    TS_CUDA_TRY(w.aperm32.alloc(R * D));
    TS_CUDA_TRY(w.gu32.alloc(R * 2 * F));
    TS_CUDA_TRY(w.glu32.alloc(R * F));
    w.exact_ready = true;
  }
  return TS_OK;
}

#define TS_K(expr)                                                                                   \
  do {                                                                                               \
    cudaError_t e_ = (expr);                                                                         \
    if (e_ != cudaSuccess) return fail(TS_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_));        \
  } while (0)

cudaEvent_t pool_event(ts_cuda* h) {
  if (!h->ev_pool.empty()) {
    cudaEvent_t e = h->ev_pool.back();
    h->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Brackets the launches of one phase with CUDA events when profiling is on
// and counts kernel launches always.
struct Phase {
  ts_cuda* h;
  cudaStream_t st;
  int phase;
  uint64_t flops;
  cudaEvent_t a = nullptr;
  Phase(ts_cuda* h_, cudaStream_t st_, int ph, uint64_t fl, int launches) : h(h_), st(st_), phase(ph), flops(fl) {
    h->n_launch += (uint64_t)launches;
    if (h->prof) {
      a = pool_event(h);
      cudaEventRecord(a, st);
    }
  }
  ~Phase() {
    if (a) {
      cudaEvent_t b = pool_event(h);
      cudaEventRecord(b, st);
      h->marks.push_back({phase, a, b, flops});
    }
  }
};

// The MoE half of a block: routing from n32 (f32, exact mode) or xn16 (fp16,
// fast mode), experts, deterministic
// combine.  res == nullptr writes the bare MoE output fp16(K * sum w e(x)).
// next_gamma (fast mode) fuses the next RMSNorm into the combine: xn16 then
// holds RMSNorm(out) * next_gamma on return.
// Where the fast router's exact candidate pass reads its f32 input: given
// (x32) or rebuilt from the add+norm's fp16 sum a (residual + attention
// output), its 1 / rms per token inv and the norm weight gamma; absum = each
// token's sum |x| from the kernel that made xn16.
struct RouterIn {
  int src = ts::kRouterSrcF32;
  const float* x32 = nullptr;
  const uint16_t *a = nullptr, *gamma = nullptr;
  const float* inv = nullptr;
  const float* absum = nullptr;
};

int next_stage(ts_cuda* h, size_t bytes, ts_cuda::Stage** out);

// Expert parallelism: the experts of one layer for the routes in
// w.aperm16 (this rank's permuted operand, expert-major = destination-major),
// with their outputs left in w.down16 at the same positions, as the
// single-GPU grouped GEMMs leave them (ep.cu describes the exchange).
int ep_experts(ts_cuda* h, LayerDev& L, cudaStream_t st) {
  Workspace& w = h->ws;
  const ts_cuda_cfg& c = h->cfg;
  const int world = h->ep_world;
  const uint32_t D = c.d_model, F = c.d_ff, E = c.n_experts, El = h->e_local;
  std::string err;
  std::vector<uint64_t> co(world), cn(world, El);
  for (int p = 0; p < world; p++) co[p] = (uint64_t)p * El;
  {
    Phase p(h, st, TS_PHASE_OTHER, 0, 0);
    // routes per expert: this rank's to each peer's experts, each source's to ours
    if (!ts::ep_exchange(h->ep_comm, world, w.counts.p, co.data(), cn.data(), h->ep_rc.p, co.data(), cn.data(), 4, st,
                         &err))
      return fail(TS_ERR_CUDA, "%s", err.c_str());
    TS_K(cudaMemcpyAsync(h->ep_hcounts, w.counts.p, (size_t)E * 4, cudaMemcpyDeviceToHost, st));
    TS_K(cudaMemcpyAsync(h->ep_hcounts + E, h->ep_rc.p, (size_t)world * El * 4, cudaMemcpyDeviceToHost, st));
    TS_K(cudaStreamSynchronize(st));
  }
  ts::EpPlan plan;
  ts::ep_plan(h->ep_hcounts, h->ep_hcounts + E, world, h->ep_rank, (int)El, (int)ts::gemm_tm_rows(), &plan);
  if (plan.recv_total > h->ep_cap)
    return fail(TS_ERR_UNSUPPORTED, "expert parallelism: %llu routed rows for this rank > capacity %llu",
                (unsigned long long)plan.recv_total, (unsigned long long)h->ep_cap);
  const uint32_t nt = (uint32_t)plan.tiles.size();
  ts_cuda::Stage* sg = nullptr;
  int rc = next_stage(h, 16 + (size_t)nt * sizeof(int4), &sg);
  if (rc) return rc;
  std::memcpy(sg->p, &nt, 4);
  if (nt) std::memcpy(sg->p + 16, plan.tiles.data(), (size_t)nt * sizeof(int4));
  TS_K(cudaMemcpyAsync(h->ep_ntiles.p, sg->p, 4, cudaMemcpyHostToDevice, st));
  if (nt) TS_K(cudaMemcpyAsync(h->ep_tiles.p, sg->p + 16, (size_t)nt * sizeof(int4), cudaMemcpyHostToDevice, st));
  TS_K(cudaEventRecord(sg->done, st));
  {
    Phase p(h, st, TS_PHASE_OTHER, 0, 0);
    if (!ts::ep_exchange(h->ep_comm, world, w.aperm16.p, plan.send_off.data(), plan.send_n.data(), h->ep_recv.p,
                         plan.recv_off.data(), plan.recv_n.data(), (size_t)D * 2, st, &err))
      return fail(TS_ERR_CUDA, "%s", err.c_str());
  }
  const uint64_t rows = plan.recv_total;
  if (nt) {
    ts::GemmArgs g;
    g.tiles = h->ep_tiles.p; g.n_tiles = h->ep_ntiles.p; g.err = h->err.p; g.out0 = h->ep_glu.p; g.ld0 = F;
    {
      Phase p(h, st, TS_PHASE_EXPERT_GATE_UP, 2ull * rows * (2ull * F) * D, 1);
      TS_K(ts::launch_gemm_w4_tm(L.gate_up.tiles(), h->ep_recv.p, rows, g, ts::kEpiSwiglu, nt, st));
    }
    ts::GemmArgs g2;
    g2.tiles = h->ep_tiles.p; g2.n_tiles = h->ep_ntiles.p; g2.err = h->err.p; g2.out0 = h->ep_out.p; g2.ld0 = D;
    {
      Phase p(h, st, TS_PHASE_EXPERT_DOWN, 2ull * rows * D * F, 1);
      TS_K(ts::launch_gemm_w4_tm(L.down.tiles(), h->ep_glu.p, rows, g2, ts::kEpiF16, nt, st));
    }
  }
  Phase p(h, st, TS_PHASE_OTHER, 0, 0);
  // the outputs back to the positions their rows had at their source
  if (!ts::ep_exchange(h->ep_comm, world, h->ep_out.p, plan.recv_off.data(), plan.recv_n.data(), w.down16.p,
                       plan.send_off.data(), plan.send_n.data(), (size_t)D * 2, st, &err))
    return fail(TS_ERR_CUDA, "%s", err.c_str());
  return TS_OK;
}

ts::RouterCertArgs router_cert_args(ts_cuda* h, const LayerDev& L, const RouterIn& rin, const int* rloc,
                                    const int* rlen, int32_t* idx, float* wt, int* hist, uint32_t T) {
  const ts_cuda_cfg& c = h->cfg;
  ts::RouterCertArgs a;
  a.cand = reinterpret_cast<const uint8_t*>(h->ws.rcand.p);
  a.x32 = rin.x32; a.a = rin.a; a.inv = rin.inv; a.gamma = rin.gamma; a.eps = c.eps;
  a.w_int4 = L.router.int4.p; a.w_sz = L.rsz.p;
  a.bias = L.router.bias.p;
  a.rloc = rloc; a.rlen = rlen; a.idx = idx; a.w = wt; a.hist = hist;
  a.T = T; a.D = c.d_model; a.E = c.n_experts; a.K = c.top_k;
  return a;
}

int moe_half(ts_cuda* h, LayerDev& L, const float* n32, const uint16_t* xn16, const uint16_t* res, uint16_t* out,
             uint32_t T, const int* rloc, const int* rlen, bool exact, cudaStream_t st, int layer, const RouterIn& rin,
             const uint16_t* next_gamma = nullptr) {
  Workspace& w = h->ws;
  const ts_cuda_cfg& c = h->cfg;
  const uint32_t D = c.d_model, K = c.top_k, E = c.n_experts, F = c.d_ff;
  const uint32_t R = T * K;
  const uint32_t grid_tiles = R / 128 + E + 1;
  // router logits in the reference order, then top-k
  ts::ExactArgs ra = L.router.exact();
  ra.x = n32; ra.ldx = D; ra.M = T; ra.rloc = rloc; ra.rlen = rlen; ra.out = w.rlogits.p; ra.ldo = E;
  {
    // kernels: logits GEMM, top-k (or the exact candidate pass), 2 permutation kernels
    Phase p(h, st, TS_PHASE_ROUTER, 2ull * T * E * D, 4);
    if (exact) {
      TS_K(ts::launch_matmul_exact(ra, true, ts::kOutF32, (T + 127) / 128, st));
    } else {
      // fast mode: router logits on the tensor cores from the fp16 operand
      CUtensorMap tx;
      if (!ts::make_act_tmap(&tx, xn16, T, D)) return fail(TS_ERR_CUDA, "cuTensorMapEncodeTiled failed (router)");
      ts::GemmArgs gr;
      gr.M = T; gr.err = h->err.p;
      if (K == 4 && E <= ts::kMaxRouterExperts && rin.absum) {
        // candidates of the exact top 4 from the tensor-core logits, then the
        // candidates in the reference's order: the reference's top-k and
        // weights on the same f32 input.  The permutation's expert counts
        // start from zero (the forward or the op zeroes them once, and
        // moe_place zeroes each chunk's row after consuming it)
        gr.out0 = w.rcand.p; gr.absum = rin.absum; gr.rbound = L.rbound.p;
        TS_K(ts::launch_gemm_w4_tc(L.router.tiles(), tx, gr, ts::kEpiRouterCert, (T + 127) / 128, st));
        TS_K(ts::launch_router_cert(router_cert_args(h, L, rin, rloc, rlen, w.ridx.p, w.rw.p, w.hist.p, T), rin.src,
                                    st));
      } else {
        gr.out0 = w.rlogits.p; gr.ld0 = E;
        TS_K(ts::launch_gemm_w4_tc(L.router.tiles(), tx, gr, ts::kEpiF32, (T + 127) / 128, st));
        TS_K(ts::launch_router_topk(w.rlogits.p, w.ridx.p, w.rw.p, w.hist.p, T, E, K, st));
      }
    }
    if (exact) TS_K(ts::launch_router_topk(w.rlogits.p, w.ridx.p, w.rw.p, w.hist.p, T, E, K, st));
    TS_K(ts::launch_moe_permute(w.ridx.p, w.hist.p, T, K, E, w.counts.p, w.perm_tok.p, w.route_pos.p, w.tiles.p,
                                w.n_tiles.p, w.tiles_tc.p, w.n_tiles_tc.p, ts::gemm_tm_rows(), w.seg_start.p,
                                w.seg_end.p, st));
  }
  if (h->trace_topk && layer >= 0)
    TS_K(cudaMemcpyAsync(h->trace_topk + (size_t)layer * T * K, w.ridx.p, (size_t)T * K * 4, cudaMemcpyDeviceToHost, st));
  const uint64_t fl_gu = 2ull * R * (2ull * F) * D, fl_dn = 2ull * R * D * F;
  if (!exact) {
    {
      Phase p(h, st, TS_PHASE_OTHER, 0, 1);
      TS_K(ts::launch_gather_rows(xn16, w.aperm16.p, w.perm_tok.p, nullptr, R, D * 2, st));
    }
    if (h->ep_world > 0) {
      const int rc = ep_experts(h, L, st);
      if (rc) return rc;
    } else {
    const uint32_t grid_tc = R / ts::gemm_tm_rows() + E + 1;
    ts::GemmArgs g;
    g.tiles = w.tiles_tc.p; g.n_tiles = w.n_tiles_tc.p; g.err = h->err.p;
    g.out0 = w.glu16.p; g.ld0 = F;
    {
      Phase p(h, st, TS_PHASE_EXPERT_GATE_UP, fl_gu, 1);
      TS_K(ts::launch_gemm_w4_tm(L.gate_up.tiles(), w.aperm16.p, R, g, ts::kEpiSwiglu, grid_tc, st));
    }
    ts::GemmArgs g2;
    g2.tiles = w.tiles_tc.p; g2.n_tiles = w.n_tiles_tc.p; g2.err = h->err.p;
    g2.out0 = w.down16.p; g2.ld0 = D;
    {
      Phase p(h, st, TS_PHASE_EXPERT_DOWN, fl_dn, 1);
      TS_K(ts::launch_gemm_w4_tm(L.down.tiles(), w.glu16.p, R, g2, ts::kEpiF16, grid_tc, st));
    }
    }
  } else {
    Phase p(h, st, TS_PHASE_EXPERT_GATE_UP, fl_gu + fl_dn, 4);
    TS_K(ts::launch_gather_rows(n32, w.aperm32.p, w.perm_tok.p, nullptr, R, D * 4, st));
    ts::ExactArgs ga = L.gate_up.exact();
    ga.x = w.aperm32.p; ga.ldx = D; ga.tiles = w.tiles.p; ga.n_tiles = w.n_tiles.p; ga.seg_end = w.seg_end.p;
    ga.out = w.gu32.p; ga.ldo = 2 * F;
    TS_K(ts::launch_matmul_exact(ga, true, ts::kOutF32, grid_tiles, st));
    TS_K(ts::launch_swiglu_exact(w.gu32.p, w.glu32.p, nullptr, R, F, st));
    ts::ExactArgs da = L.down.exact();
    da.x = w.glu32.p; da.ldx = F; da.tiles = w.tiles.p; da.n_tiles = w.n_tiles.p; da.seg_end = w.seg_end.p;
    da.out = w.down32.p; da.ldo = D;
    TS_K(ts::launch_matmul_exact(da, true, ts::kOutF32, grid_tiles, st));
  }
  {
    Phase p(h, st, TS_PHASE_OTHER, 0, 1);
    if (exact) TS_K(ts::launch_moe_combine(w.down32.p, w.ridx.p, w.rw.p, w.route_pos.p, res, out, T, D, K, E, st));
    else
      TS_K(ts::launch_moe_combine_fast(w.down16.p, w.ridx.p, w.rw.p, w.route_pos.p, res, out, T, D, K, E,
                                       next_gamma, w.xn16.p, c.eps, st));
  }
  return TS_OK;
}

// Next slot of the pinned staging ring with room for `bytes`, once the copies
// queued from it by an earlier forward have executed.
int next_stage(ts_cuda* h, size_t bytes, ts_cuda::Stage** out) {
  ts_cuda::Stage& sg = h->stage[h->stage_next++ % 4];
  if (sg.done) TS_CUDA_TRY(cudaEventSynchronize(sg.done));
  else TS_CUDA_TRY(cudaEventCreateWithFlags(&sg.done, cudaEventDisableTiming));
  if (sg.cap < bytes) {
    if (sg.p) cudaFreeHost(sg.p);
    sg.p = nullptr;
    sg.cap = 0;
    TS_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&sg.p), bytes, cudaHostAllocDefault));
    sg.cap = bytes;
  }
  *out = &sg;
  return TS_OK;
}

int forward_device(ts_cuda* h, const int32_t* d_ids, const uint8_t* d_mask, const uint32_t* offs, uint32_t n_seqs,
                   float* d_logits, cudaStream_t st) {
  if (!h->finalized) return fail(TS_ERR_STATE, "ts_cuda_finalize has not succeeded");
  const ts_cuda_cfg& c = h->cfg;
  if (!offs || n_seqs == 0) return fail(TS_ERR_ARG, "seq_offsets must hold n_seqs + 1 >= 2 entries");
  if (offs[0] != 0) return fail(TS_ERR_ARG, "seq_offsets[0] must be 0");
  for (uint32_t s = 0; s < n_seqs; s++) {
    if (offs[s + 1] <= offs[s]) return fail(TS_ERR_ARG, "sequence %u is empty or offsets decrease", s);
    if (offs[s + 1] - offs[s] > c.max_seq_len)
      return fail(TS_ERR_UNSUPPORTED, "sequence %u has %u tokens > max_seq_len %u", s, offs[s + 1] - offs[s], c.max_seq_len);
  }
  const uint32_t T = offs[n_seqs];
  if (T > c.max_tokens) return fail(TS_ERR_UNSUPPORTED, "%u tokens > max_tokens %u", T, c.max_tokens);
  const bool exact = c.mode == TS_MODE_EXACT;
  if (exact && h->ep_world > 0) return fail(TS_ERR_UNSUPPORTED, "expert parallelism runs the fast mode only");
  int rc = ensure_workspace(h, exact);
  if (rc) return rc;
  Workspace& w = h->ws;
  const uint32_t D = c.d_model, Q = c.n_heads * c.head_dim, KV = c.n_kv_heads * c.head_dim;

  // small host -> device copies through the pinned ring (offsets, then the
  // attention tile list at a 16-byte aligned offset)
  const size_t offs_bytes = ((size_t)(n_seqs + 1) * 4 + 15) & ~size_t(15);
  ts_cuda::Stage* sg = nullptr;
  int rc0 = next_stage(h, offs_bytes + (size_t)ts::attention_max_tiles(T, n_seqs) * sizeof(int2), &sg);
  if (rc0) return rc0;
  memcpy(sg->p, offs, (size_t)(n_seqs + 1) * 4);
  TS_K(cudaMemcpyAsync(w.offs.p, sg->p, (size_t)(n_seqs + 1) * 4, cudaMemcpyHostToDevice, st));
  TS_K(cudaMemsetAsync(w.hist.p, 0, (size_t)ts::route_chunks(T) * c.n_experts * sizeof(int), st));
  {
    Phase p(h, st, TS_PHASE_OTHER, 0, 2);
    TS_K(ts::launch_seq_info(w.offs.p, n_seqs, T, w.pos.p, w.sstart.p, w.slen.p, st));
    TS_K(ts::launch_embed_rows(h->embed_rows.p, d_ids, w.x0.p, T, c.vocab, D, st));
  }
  uint64_t band_pairs = 0;  // sum over tokens of the keys each query attends (attention flops)
  for (uint32_t s = 0; s < n_seqs; s++) {
    const uint64_t n = offs[s + 1] - offs[s], W = c.window;
    for (uint64_t t = 0; t < n; t++) band_pairs += std::min<uint64_t>(n, t + W + 1) - (t > W ? t - W : 0);
  }
  const uint64_t fl_qkv = 2ull * T * (Q + 2 * KV) * D, fl_o = 2ull * T * D * Q;
  const uint64_t fl_attn = 4ull * c.n_heads * c.head_dim * band_pairs;

  CUtensorMap t_xn;  // the classifier's operand (the other GEMMs build their own maps)
  if (!exact) {
    if (!ts::make_act_tmap(&t_xn, w.xn16.p, T, D))
      return fail(TS_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activation operands");
  }
  ts::AttnArgs aa;
  aa.q = w.q.p; aa.k = w.k.p; aa.v = w.v.p; aa.mask = d_mask; aa.out = w.attn.p;
  aa.sstart = w.sstart.p; aa.slen = w.slen.p; aa.T = T; aa.Hq = c.n_heads; aa.Hkv = c.n_kv_heads;
  aa.hd = c.head_dim; aa.window = c.window; aa.err = h->err.p;
  {
    // 16-query tiles (both modes: the exact kernel works on them too)
    uint32_t nt = 0;
    int2* th = reinterpret_cast<int2*>(sg->p + offs_bytes);
    ts::attention_tiles(offs, n_seqs, th, &nt);
    TS_K(cudaMemcpyAsync(w.atiles.p, th, (size_t)nt * sizeof(int2), cudaMemcpyHostToDevice, st));
    aa.tiles = w.atiles.p;
    aa.n_tiles = nt;
  }
  TS_K(cudaEventRecord(sg->done, st));  // the staging slot is free once this passes

  uint16_t* src = w.x0.p;
  uint16_t* dst = w.x1.p;
  const uint32_t mt = (T + 127) / 128;
  const uint32_t mt_tc = (T + ts::gemm_tm_rows() - 1) / ts::gemm_tm_rows();
  for (uint32_t li = 0; li < c.n_layers; li++) {
    LayerDev& L = *h->layers[li];
    aa.sinks = L.sinks.p;
    if (!exact) {
      if (li == 0) {  // later layers' ln1 comes fused with the previous combine
        Phase p(h, st, TS_PHASE_OTHER, 0, 1);
        TS_K(ts::launch_rmsnorm_fast(src, nullptr, L.ln1.p, nullptr, w.xn16.p, T, D, c.eps, st));
      }
      ts::GemmArgs g;
      g.M = T; g.err = h->err.p;
      {
        // RoPE in the GEMM epilogue: q, k (rotated) and v to their own buffers
        g.out0 = w.q.p; g.ld0 = Q; g.out1 = w.k.p; g.ld1 = KV; g.out2 = w.v.p; g.ld2 = KV;
        g.q_cols = Q; g.k_cols = KV; g.pos = w.pos.p; g.rope_cos = h->rope_cos.p; g.rope_sin = h->rope_sin.p;
        g.rope_cs = h->rope_cs.p;
        Phase p(h, st, TS_PHASE_QKV, fl_qkv, 1);
        TS_K(ts::launch_gemm_w4_tm(L.qkv.tiles(), w.xn16.p, T, g, ts::kEpiQkvRope, mt_tc, st));
      }
      {
        Phase p(h, st, TS_PHASE_ATTENTION, fl_attn, 1);
        TS_K(ts::launch_attention_tc(aa, st));
      }
      ts::GemmArgs go;
      go.M = T; go.err = h->err.p; go.out0 = w.o16.p; go.ld0 = D;
      {
        Phase p(h, st, TS_PHASE_O, fl_o, 1);
        TS_K(ts::launch_gemm_w4_tm(L.o.tiles(), w.attn.p, T, go, ts::kEpiF16, mt_tc, st));
      }
      {
        Phase p(h, st, TS_PHASE_OTHER, 0, 1);
        TS_K(ts::launch_rmsnorm_fast(src, w.o16.p, L.ln2.p, w.res2.p, w.xn16.p, T, D, c.eps, st, w.absum.p, w.rinv.p));
      }
    } else {
      Phase p(h, st, TS_PHASE_OTHER, fl_qkv + fl_o + fl_attn, 6);
      TS_K(ts::launch_rmsnorm(src, L.ln1.p, w.hf32.p, nullptr, T, D, c.eps, st));
      ts::ExactArgs qa = L.qkv.exact();
      qa.x = w.hf32.p; qa.ldx = D; qa.M = T; qa.rloc = w.pos.p; qa.rlen = w.slen.p; qa.out = w.qkv16.p;
      qa.ldo = Q + 2 * KV;
      TS_K(ts::launch_matmul_exact(qa, true, ts::kOutF16, mt, st));
      TS_K(ts::launch_split_rope(w.qkv16.p, w.q.p, w.k.p, w.v.p, w.pos.p, h->rope_cos.p, h->rope_sin.p, T, Q, KV, KV,
                                 c.head_dim, st));
      TS_K(ts::launch_attention_exact(aa, st));
      ts::ExactArgs oa = L.o.exact();
      oa.x = w.attn.p; oa.ldx = Q; oa.M = T; oa.rloc = w.pos.p; oa.rlen = w.slen.p; oa.out = w.o16.p; oa.ldo = D;
      TS_K(ts::launch_matmul_exact(oa, false, ts::kOutF16, mt, st));
      TS_K(ts::launch_add_rmsnorm(src, w.o16.p, L.ln2.p, w.res2.p, w.n32.p, nullptr, T, D, c.eps, st));
    }
    const uint16_t* next_gamma = exact ? nullptr : li + 1 < c.n_layers ? h->layers[li + 1]->ln1.p : h->final_norm.p;
    RouterIn rin;  // fast mode: the router input rebuilt from the block's add + RMSNorm
    rin.src = ts::kRouterSrcAddNorm; rin.a = w.res2.p; rin.inv = w.rinv.p; rin.gamma = L.ln2.p; rin.absum = w.absum.p;
    rc = moe_half(h, L, w.n32.p, w.xn16.p, w.res2.p, dst, T, w.pos.p, w.slen.p, exact, st, (int)li, rin, next_gamma);
    if (rc) return rc;
    std::swap(src, dst);
  }
  Phase p(h, st, TS_PHASE_OTHER, 2ull * T * c.n_classes * D, (!exact && c.n_layers > 0) ? 1 : 2);
  if (!exact) {
    // the final norm comes fused with the last layer's combine
    if (c.n_layers == 0) TS_K(ts::launch_rmsnorm_fast(src, nullptr, h->final_norm.p, nullptr, w.xn16.p, T, D, c.eps, st));
    ts::GemmArgs gs;
    gs.M = T; gs.err = h->err.p; gs.out0 = d_logits; gs.ld0 = c.n_classes;
    TS_K(ts::launch_gemm_w4_tc(h->score.tiles(), t_xn, gs, ts::kEpiF16Widen, mt, st));
    return TS_OK;
  }
  TS_K(ts::launch_rmsnorm(src, h->final_norm.p, w.n32.p, nullptr, T, D, c.eps, st));
  ts::ExactArgs sa = h->score.exact();
  sa.x = w.n32.p; sa.ldx = D; sa.M = T; sa.rloc = w.pos.p; sa.rlen = w.slen.p; sa.out = d_logits; sa.ldo = c.n_classes;
  TS_K(ts::launch_matmul_exact(sa, true, ts::kOutF16Widen, mt, st));
  return TS_OK;
}

int check_dev_err(int* d_err, cudaStream_t st) {
  int herr = 0;
  TS_CUDA_TRY(cudaMemcpyAsync(&herr, d_err, 4, cudaMemcpyDeviceToHost, st));
  TS_CUDA_TRY(cudaStreamSynchronize(st));
  if (herr != 0) {
    cudaMemsetAsync(d_err, 0, 4, st);
    cudaStreamSynchronize(st);
    return fail(TS_ERR_DEVICE, "device error flag %d (%s)", herr,
                herr == ts::kDevErrWaitTimeout ? "bounded wait timed out" : "bad index");
  }
  return TS_OK;
}

}  // namespace

namespace ts {
void set_last_error(const char* msg) { g_err = msg ? msg : ""; }
}  // namespace ts

// =============================================================================
// extern "C" ABI
// =============================================================================
extern "C" {

int ts_cuda_abi_version(void) { return TS_CUDA_ABI_VERSION; }

const char* ts_cuda_last_error(void) { return g_err.c_str(); }

void ts_cuda_default_cfg(ts_cuda_cfg* c) {
  if (!c) return;
  memset(c, 0, sizeof *c);
  c->device = 0;
  c->vocab = 200064;
  c->d_model = 640;
  c->n_layers = 8;
  c->n_heads = 14;
  c->n_kv_heads = 2;
  c->head_dim = 64;
  c->window = 128;
  c->d_ff = 640;
  c->n_experts = 128;
  c->top_k = 4;
  c->n_classes = 33;
  c->eps = 1e-5f;
  c->rope_theta = 150000.0;
  c->rope_factor = 32.0;
  c->rope_original_max_pos = 4096.0;
  c->rope_beta_fast = 32.0;
  c->rope_beta_slow = 1.0;
  c->max_tokens = 65536;
  c->max_seq_len = 8192;
  c->mode = TS_MODE_FAST;
}

ts_cuda_t* ts_cuda_create(const ts_cuda_cfg* cfg, char* err, size_t err_cap) {
  auto bad = [&](const char* msg) -> ts_cuda_t* {
    g_err = msg;
    if (err && err_cap) snprintf(err, err_cap, "%s", msg);
    return nullptr;
  };
  if (!cfg) return bad("ts_cuda_create: cfg is NULL");
  const ts_cuda_cfg& c = *cfg;
  if (c.d_model % 64 || c.d_ff % 64 || (c.n_heads * c.head_dim) % 64 || c.head_dim != 64 || c.n_kv_heads == 0 ||
      c.n_heads % c.n_kv_heads || c.n_heads / c.n_kv_heads > 7 || c.top_k == 0 || c.top_k > 8 ||
      c.top_k > c.n_experts || c.n_experts > 256 || c.d_model > 1024 || c.d_ff > 1024 ||
      c.n_heads * c.head_dim > 1024 || c.n_classes == 0 || c.max_tokens == 0 || c.max_seq_len == 0 || c.n_layers == 0)
    return bad("ts_cuda_create: unsupported configuration (head_dim must be 64, d_model/d_ff multiples of 64, "
               "GQA group <= 7, top_k <= 8)");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || c.device < 0 || c.device >= ndev)
    return bad("ts_cuda_create: no such CUDA device");
  DevGuard g(c.device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, c.device) != cudaSuccess) return bad("ts_cuda_create: cudaGetDeviceProperties failed");
  if (prop.major != 10) return bad("ts_cuda_create: this library is built for sm_100a (B200); device is not compute capability 10.x");
  auto* h = new ts_cuda();
  h->cfg = c;
  h->name = prop.name;
  if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess || h->err.alloc(1) != cudaSuccess ||
      cudaMemset(h->err.p, 0, 4) != cudaSuccess) {
    delete h;
    return bad("ts_cuda_create: CUDA initialisation failed");
  }
  return h;
}

int ts_cuda_load_tensor(ts_cuda_t* h, const char* name, int32_t dtype, const int64_t* shape, int32_t ndim,
                        const void* data, size_t nbytes) {
  if (!h || !name || !data) return fail(TS_ERR_ARG, "ts_cuda_load_tensor: null argument");
  size_t want = 0;
  int32_t wdt = 0;
  if (!expected_tensor(h->cfg, name, want, wdt)) return fail(TS_ERR_ARG, "unknown tensor name \"%s\"", name);
  if (dtype != wdt) return fail(TS_ERR_ARG, "tensor \"%s\": dtype %d, expected %d", name, dtype, wdt);
  if (nbytes != want) return fail(TS_ERR_ARG, "tensor \"%s\": %zu bytes, expected %zu", name, nbytes, want);
  if (shape && ndim > 0) {
    int64_t prod = 1;
    for (int i = 0; i < ndim; i++) prod *= shape[i];
    const int64_t esz = dtype == TS_DTYPE_U8 ? 1 : (dtype == TS_DTYPE_F16 ? 2 : 4);
    if (prod * esz != (int64_t)nbytes && !(dtype == TS_DTYPE_U8 && prod / 2 == (int64_t)nbytes))
      return fail(TS_ERR_ARG, "tensor \"%s\": shape does not match %zu bytes", name, nbytes);
  }
  HostTensor& t = h->staged[name];
  t.bytes.assign((const uint8_t*)data, (const uint8_t*)data + nbytes);
  t.dtype = dtype;
  h->finalized = false;
  return TS_OK;
}

int ts_cuda_finalize(ts_cuda_t* h) {
  if (!h) return fail(TS_ERR_ARG, "ts_cuda_finalize: null handle");
  if (h->finalized) return TS_OK;
  const ts_cuda_cfg& c = h->cfg;
  for (const std::string& n : required_names(c))
    if (!h->staged.count(n)) return fail(TS_ERR_STATE, "tensor \"%s\" has not been loaded", n.c_str());
  DevGuard g(c.device);
  cudaStream_t st = h->stream;
  const uint32_t D = c.d_model, E = c.n_experts, F = c.d_ff, Q = c.n_heads * c.head_dim, KV = c.n_kv_heads * c.head_dim;
  auto up = [&](auto& arr, const std::string& n) -> int {
    const HostTensor& t = h->staged[n];
    using Tp = typename std::remove_reference<decltype(*arr.p)>::type;
    TS_CUDA_TRY(arr.alloc(t.bytes.size() / sizeof(Tp)));
    TS_CUDA_TRY(cudaMemcpyAsync(arr.p, t.bytes.data(), t.bytes.size(), cudaMemcpyHostToDevice, st));
    return TS_OK;
  };
  int rc;
  if ((rc = up(h->embed_int4, "embed.int4")) || (rc = up(h->embed_scales, "embed.scales")) ||
      (rc = up(h->embed_zp, "embed.zp")) || (rc = up(h->final_norm, "final_norm")))
    return rc;
  TS_CUDA_TRY(h->embed_rows.alloc((size_t)c.vocab * ts::embed_row_bytes(D)));
  TS_CUDA_TRY(ts::launch_embed_pack(h->embed_int4.p, h->embed_scales.p, h->embed_zp.p, h->embed_rows.p, c.vocab, D, st));
  auto p8 = [&](const std::string& n) { return staged_ptr(h, n); };
  auto p16 = [&](const std::string& n) { return reinterpret_cast<const uint16_t*>(staged_ptr(h, n)); };
  DevArr<int> bad;
  TS_CUDA_TRY(bad.alloc(1));
  TS_CUDA_TRY(cudaMemsetAsync(bad.p, 0, 4, st));
  // the experts this handle holds: all, or [e_first, e_first + e_local) under
  // expert parallelism (consecutive in the loader layout [E][N][...])
  const uint32_t e0 = h->ep_world > 0 ? h->e_first : 0u, ne = h->ep_world > 0 ? h->e_local : E;
  auto upload_experts = [&](W4Dev& wd, const std::string& pre, uint32_t N, uint32_t K) -> int {
    const size_t nb = K / 32, zs = (nb + 1) / 2;
    // a missing tensor stays a null pointer (no zero points: the constant 8)
    auto at = [&](const auto* base, size_t per_expert) { return base ? base + (size_t)e0 * per_expert : base; };
    return w4_upload(wd, at(p8(pre + "int4"), (size_t)N * (K / 2)), at(p16(pre + "scales"), (size_t)N * nb),
                     at(p8(pre + "zp"), (size_t)N * zs), at(p16(pre + "bias"), (size_t)N), ne, N, K, 128, true, bad.p,
                     st);
  };
  rc = w4_upload(h->score, p8("score.int4"), p16("score.scales"), p8("score.zp"),
                 h->staged.count("score.bias") ? p16("score.bias") : nullptr, 1, c.n_classes, D, 128, true, bad.p, st);
  if (rc) return rc;
  h->layers.clear();
  for (uint32_t li = 0; li < c.n_layers; li++) {
    auto L = std::make_unique<LayerDev>();
    const std::string p = "layers." + std::to_string(li) + ".";
    if ((rc = up(L->ln1, p + "input_layernorm")) || (rc = up(L->ln2, p + "post_attention_layernorm")) ||
        (rc = up(L->sinks, p + "attn.sinks")))
      return rc;
    // Q, K and V fused along N into one [Q + 2 KV, D] weight.
    std::vector<uint8_t> i4, zp;
    std::vector<uint16_t> sc, bs;
    for (const char* pr : {"attn.q_proj.", "attn.k_proj.", "attn.v_proj."}) {
      const HostTensor& a = h->staged[p + pr + "int4"];
      const HostTensor& s = h->staged[p + pr + "scales"];
      const HostTensor& z = h->staged[p + pr + "zp"];
      const HostTensor& b = h->staged[p + pr + "bias"];
      i4.insert(i4.end(), a.bytes.begin(), a.bytes.end());
      zp.insert(zp.end(), z.bytes.begin(), z.bytes.end());
      const uint16_t* sp = reinterpret_cast<const uint16_t*>(s.bytes.data());
      sc.insert(sc.end(), sp, sp + s.bytes.size() / 2);
      const uint16_t* bp = reinterpret_cast<const uint16_t*>(b.bytes.data());
      bs.insert(bs.end(), bp, bp + b.bytes.size() / 2);
    }
    if ((rc = w4_upload(L->qkv, i4.data(), sc.data(), zp.data(), bs.data(), 1, Q + 2 * KV, D, 128, true, bad.p, st)))
      return rc;
    TS_CUDA_TRY(cudaStreamSynchronize(st));  // host vectors above are released at scope end
    if ((rc = w4_upload(L->o, p8(p + "attn.o_proj.int4"), p16(p + "attn.o_proj.scales"), p8(p + "attn.o_proj.zp"),
                        p16(p + "attn.o_proj.bias"), 1, D, Q, 128, true, bad.p, st)) ||
        (rc = w4_upload(L->router, p8(p + "router.int4"), p16(p + "router.scales"), p8(p + "router.zp"),
                        p16(p + "router.bias"), 1, E, D, 128, true, bad.p, st)) ||
        (rc = upload_experts(L->gate_up, p + "experts.gate_up.", 2 * F, D)) ||
        (rc = upload_experts(L->down, p + "experts.down.", D, F)))
      return rc;
    if (E <= ts::kMaxRouterExperts) {
      std::vector<float> tb(2 * ts::kMaxRouterExperts + 2), tsz(2 * (size_t)E * (D / 32));
      ts::router_bound_table(p8(p + "router.int4"), p16(p + "router.scales"), p8(p + "router.zp"), E, D, tb.data(),
                             tsz.data());
      TS_CUDA_TRY(L->rbound.alloc(tb.size()));
      TS_CUDA_TRY(cudaMemcpy(L->rbound.p, tb.data(), tb.size() * 4, cudaMemcpyHostToDevice));
      TS_CUDA_TRY(L->rsz.alloc(tsz.size()));
      TS_CUDA_TRY(cudaMemcpy(L->rsz.p, tsz.data(), tsz.size() * 4, cudaMemcpyHostToDevice));
    }
    h->layers.push_back(std::move(L));
  }
  std::vector<uint16_t> cs, sn;
  build_rope_tables(c, c.max_seq_len, cs, sn);
  TS_CUDA_TRY(h->rope_cos.alloc(cs.size()));
  TS_CUDA_TRY(h->rope_sin.alloc(sn.size()));
  TS_CUDA_TRY(cudaMemcpyAsync(h->rope_cos.p, cs.data(), cs.size() * 2, cudaMemcpyHostToDevice, st));
  TS_CUDA_TRY(cudaMemcpyAsync(h->rope_sin.p, sn.data(), sn.size() * 2, cudaMemcpyHostToDevice, st));
  std::vector<uint32_t> csn(cs.size());
  for (size_t i = 0; i < cs.size(); i++) csn[i] = (uint32_t)cs[i] | ((uint32_t)sn[i] << 16);
  TS_CUDA_TRY(h->rope_cs.alloc(csn.size()));
  TS_CUDA_TRY(cudaMemcpyAsync(h->rope_cs.p, csn.data(), csn.size() * 4, cudaMemcpyHostToDevice, st));
  int nbad = 0;
  TS_CUDA_TRY(cudaMemcpyAsync(&nbad, bad.p, 4, cudaMemcpyDeviceToHost, st));
  TS_CUDA_TRY(cudaStreamSynchronize(st));
  // the forward gathers from the packed table only
  h->embed_int4.release();
  h->embed_scales.release();
  h->embed_zp.release();
  if (nbad)
    return fail(TS_ERR_UNSUPPORTED,
                "%d fp16 weight scales are subnormal, inf or NaN; the tensor-core path reproduces the reference "
                "dequantisation only for zero or normal scales",
                nbad);
  if ((rc = ensure_workspace(h, c.mode == TS_MODE_EXACT))) return rc;
  if (h->ep_world > 0 && !h->ep_hcounts) {
    // every rank may route all of its routes to this one: world * max_tokens * k rows
    h->ep_cap = (uint64_t)h->ep_world * c.max_tokens * c.top_k;
    TS_CUDA_TRY(h->ep_rc.alloc((size_t)h->ep_world * h->e_local));
    TS_CUDA_TRY(h->ep_recv.alloc(h->ep_cap * D));
    TS_CUDA_TRY(h->ep_glu.alloc(h->ep_cap * F));
    TS_CUDA_TRY(h->ep_out.alloc(h->ep_cap * D));
    TS_CUDA_TRY(h->ep_tiles.alloc(h->ep_cap / ts::gemm_tm_rows() + (size_t)h->ep_world * h->e_local + 1));
    TS_CUDA_TRY(h->ep_ntiles.alloc(1));
    TS_CUDA_TRY(cudaMallocHost(&h->ep_hcounts, ((size_t)E + (size_t)h->ep_world * h->e_local) * sizeof(int)));
  }
  const size_t pin_need = (size_t)c.max_tokens * (4 + 1 + 4 * c.n_classes) + 64;
  if (!h->pin) {
    TS_CUDA_TRY(cudaMallocHost(&h->pin, pin_need));
    h->pin_bytes = pin_need;
  }
  h->staged.clear();
  h->finalized = true;
  return TS_OK;
}

int ts_cuda_set_mode(ts_cuda_t* h, int32_t mode) {
  if (!h || (mode != TS_MODE_FAST && mode != TS_MODE_EXACT)) return fail(TS_ERR_ARG, "ts_cuda_set_mode: bad mode");
  h->cfg.mode = mode;
  return TS_OK;
}

int ts_cuda_forward_packed_device(ts_cuda_t* h, const int32_t* d_ids, const uint8_t* d_mask,
                                  const uint32_t* seq_offsets, uint32_t n_seqs, float* d_logits, void* stream) {
  if (!h || !d_ids || !d_logits) return fail(TS_ERR_ARG, "ts_cuda_forward_packed_device: null argument");
  DevGuard g(h->cfg.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  return forward_device(h, d_ids, d_mask, seq_offsets, n_seqs, d_logits, st);
}

int ts_cuda_forward_packed(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                           uint32_t n_seqs, float* logits) {
  if (!h || !ids || !logits || !seq_offsets || n_seqs == 0) return fail(TS_ERR_ARG, "ts_cuda_forward_packed: null argument");
  if (!h->finalized) return fail(TS_ERR_STATE, "ts_cuda_finalize has not succeeded");
  const uint32_t T = seq_offsets[n_seqs];
  if (T > h->cfg.max_tokens) return fail(TS_ERR_UNSUPPORTED, "%u tokens > max_tokens %u", T, h->cfg.max_tokens);
  DevGuard g(h->cfg.device);
  cudaStream_t st = h->stream;
  Workspace& w = h->ws;
  const size_t C = h->cfg.n_classes;
  // host -> pinned -> device (the pinned block is only reused after the sync below)
  uint8_t* pin_ids = h->pin;
  uint8_t* pin_mask = h->pin + (size_t)h->cfg.max_tokens * 4;
  uint8_t* pin_log = pin_mask + h->cfg.max_tokens + 16 - ((uintptr_t)(pin_mask + h->cfg.max_tokens) & 15u);
  memcpy(pin_ids, ids, (size_t)T * 4);
  TS_CUDA_TRY(cudaMemcpyAsync(w.ids.p, pin_ids, (size_t)T * 4, cudaMemcpyHostToDevice, st));
  const uint8_t* dmask = nullptr;
  if (mask) {
    memcpy(pin_mask, mask, T);
    TS_CUDA_TRY(cudaMemcpyAsync(w.mask.p, pin_mask, T, cudaMemcpyHostToDevice, st));
    dmask = w.mask.p;
  }
  int rc = forward_device(h, w.ids.p, dmask, seq_offsets, n_seqs, w.logits.p, st);
  if (rc) {
    cudaStreamSynchronize(st);
    return rc;
  }
  TS_CUDA_TRY(cudaMemcpyAsync(pin_log, w.logits.p, (size_t)T * C * 4, cudaMemcpyDeviceToHost, st));
  rc = check_dev_err(h->err.p, st);
  if (rc) return rc;
  memcpy(logits, pin_log, (size_t)T * C * 4);
  return TS_OK;
}

int ts_cuda_forward_packed_begin(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                                 uint32_t n_seqs, uint32_t slot) {
  if (!h || !ids || !seq_offsets || n_seqs == 0) return fail(TS_ERR_ARG, "ts_cuda_forward_packed_begin: null argument");
  if (slot > 1) return fail(TS_ERR_ARG, "slot must be 0 or 1");
  if (!h->finalized) return fail(TS_ERR_STATE, "ts_cuda_finalize has not succeeded");
  ts_cuda::Slot& sl = h->slot[slot];
  if (sl.busy) return fail(TS_ERR_STATE, "slot %u holds a forward that ts_cuda_forward_packed_end has not collected", slot);
  const uint32_t T = seq_offsets[n_seqs];
  if (T > h->cfg.max_tokens) return fail(TS_ERR_UNSUPPORTED, "%u tokens > max_tokens %u", T, h->cfg.max_tokens);
  DevGuard g(h->cfg.device);
  cudaStream_t st = h->stream;
  Workspace& w = h->ws;
  const size_t C = h->cfg.n_classes, mt = h->cfg.max_tokens;
  // slot layout: logits [mt][C] f32, ids [mt] i32, flag, mask [mt]
  if (!sl.p) {
    if (!h->copy_st) TS_CUDA_TRY(cudaStreamCreateWithFlags(&h->copy_st, cudaStreamNonBlocking));
    if (!sl.fwd) TS_CUDA_TRY(cudaEventCreateWithFlags(&sl.fwd, cudaEventDisableTiming));
    if (!sl.done) TS_CUDA_TRY(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
    TS_CUDA_TRY(sl.dlog.alloc(mt * C));
    TS_CUDA_TRY(cudaMallocHost(&sl.p, mt * (4 * C + 4 + 1) + 16));
  }
  float* pin_log = reinterpret_cast<float*>(sl.p);
  int32_t* pin_ids = reinterpret_cast<int32_t*>(sl.p + mt * C * 4);
  int* pin_flag = reinterpret_cast<int*>(sl.p + mt * (C + 1) * 4);
  uint8_t* pin_mask = sl.p + mt * (C + 1) * 4 + 16;
  // the slot's previous forward was collected by _end, so its copies have run
  memcpy(pin_ids, ids, (size_t)T * 4);
  TS_CUDA_TRY(cudaMemcpyAsync(w.ids.p, pin_ids, (size_t)T * 4, cudaMemcpyHostToDevice, st));
  const uint8_t* dmask = nullptr;
  if (mask) {
    memcpy(pin_mask, mask, T);
    TS_CUDA_TRY(cudaMemcpyAsync(w.mask.p, pin_mask, T, cudaMemcpyHostToDevice, st));
    dmask = w.mask.p;
  }
  int rc = forward_device(h, w.ids.p, dmask, seq_offsets, n_seqs, sl.dlog.p, st);
  if (rc) {
    cudaStreamSynchronize(st);
    return rc;
  }
  TS_CUDA_TRY(cudaEventRecord(sl.fwd, st));
  TS_CUDA_TRY(cudaStreamWaitEvent(h->copy_st, sl.fwd, 0));
  TS_CUDA_TRY(cudaMemcpyAsync(pin_log, sl.dlog.p, (size_t)T * C * 4, cudaMemcpyDeviceToHost, h->copy_st));
  TS_CUDA_TRY(cudaMemcpyAsync(pin_flag, h->err.p, 4, cudaMemcpyDeviceToHost, h->copy_st));
  TS_CUDA_TRY(cudaEventRecord(sl.done, h->copy_st));
  sl.T = T;
  sl.busy = true;
  return TS_OK;
}

int ts_cuda_forward_packed_end(ts_cuda_t* h, uint32_t slot, float* logits) {
  if (!h || !logits) return fail(TS_ERR_ARG, "ts_cuda_forward_packed_end: null argument");
  if (slot > 1) return fail(TS_ERR_ARG, "slot must be 0 or 1");
  ts_cuda::Slot& sl = h->slot[slot];
  if (!sl.busy) return fail(TS_ERR_STATE, "slot %u holds no forward (ts_cuda_forward_packed_begin first)", slot);
  DevGuard g(h->cfg.device);
  sl.busy = false;
  TS_CUDA_TRY(cudaEventSynchronize(sl.done));
  const size_t C = h->cfg.n_classes, mt = h->cfg.max_tokens;
  const int flag = *reinterpret_cast<const int*>(sl.p + mt * (C + 1) * 4);
  if (flag != 0) {
    // everything queued so far completes before the flag is cleared; a later
    // slot whose download already ran reports the same flag
    cudaStreamSynchronize(h->stream);
    cudaStreamSynchronize(h->copy_st);
    cudaMemsetAsync(h->err.p, 0, 4, h->stream);
    cudaStreamSynchronize(h->stream);
    return fail(TS_ERR_DEVICE, "device error flag %d (%s)", flag,
                flag == ts::kDevErrWaitTimeout ? "bounded wait timed out" : "bad index");
  }
  memcpy(logits, sl.p, (size_t)sl.T * C * 4);
  return TS_OK;
}

// Viterbi arguments: calibration values finite and below 1e20 in magnitude
// (the range in which the kernel's restricted candidate scan equals the
// reference's full one), sequences non-empty and short enough for the
// per-warp back-pointer table in shared memory.
static int check_viterbi_args(const uint32_t* offs, uint32_t n_seqs, const float* cal, uint32_t* max_len) {
  if (!cal) return fail(TS_ERR_ARG, "calibration must hold 6 values");
  for (int i = 0; i < 6; i++)
    if (!(std::fabs(cal[i]) < 1e20f)) return fail(TS_ERR_ARG, "calibration[%d] is not a finite value below 1e20", i);
  if (offs[0] != 0) return fail(TS_ERR_ARG, "seq_offsets[0] must be 0");
  uint32_t m = 0;
  for (uint32_t s = 0; s < n_seqs; s++) {
    if (offs[s + 1] <= offs[s]) return fail(TS_ERR_ARG, "sequence %u is empty", s);
    m = std::max(m, offs[s + 1] - offs[s]);
  }
  if (m > ts::viterbi_max_len())
    return fail(TS_ERR_UNSUPPORTED, "sequence of %u tokens > %u for Viterbi decoding", m, ts::viterbi_max_len());
  *max_len = m;
  return TS_OK;
}

int ts_cuda_forward_packed_tags(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                                uint32_t n_seqs, const float* calibration, uint8_t* tags) {
  if (!h || !ids || !tags || !seq_offsets || n_seqs == 0)
    return fail(TS_ERR_ARG, "ts_cuda_forward_packed_tags: null argument");
  if (!h->finalized) return fail(TS_ERR_STATE, "ts_cuda_finalize has not succeeded");
  uint32_t max_len = 0;
  int rc = check_viterbi_args(seq_offsets, n_seqs, calibration, &max_len);
  if (rc) return rc;
  const uint32_t T = seq_offsets[n_seqs];
  if (T > h->cfg.max_tokens) return fail(TS_ERR_UNSUPPORTED, "%u tokens > max_tokens %u", T, h->cfg.max_tokens);
  if (h->cfg.n_classes != 33) return fail(TS_ERR_UNSUPPORTED, "Viterbi decoding needs the 33-class BIOES head");
  DevGuard g(h->cfg.device);
  cudaStream_t st = h->stream;
  Workspace& w = h->ws;
  uint8_t* pin_ids = h->pin;
  uint8_t* pin_mask = h->pin + (size_t)h->cfg.max_tokens * 4;
  uint8_t* pin_tags = pin_mask + h->cfg.max_tokens + 16 - ((uintptr_t)(pin_mask + h->cfg.max_tokens) & 15u);
  memcpy(pin_ids, ids, (size_t)T * 4);
  TS_CUDA_TRY(cudaMemcpyAsync(w.ids.p, pin_ids, (size_t)T * 4, cudaMemcpyHostToDevice, st));
  const uint8_t* dmask = nullptr;
  if (mask) {
    memcpy(pin_mask, mask, T);
    TS_CUDA_TRY(cudaMemcpyAsync(w.mask.p, pin_mask, T, cudaMemcpyHostToDevice, st));
    dmask = w.mask.p;
  }
  rc = forward_device(h, w.ids.p, dmask, seq_offsets, n_seqs, w.logits.p, st);
  if (rc) {
    cudaStreamSynchronize(st);
    return rc;
  }
  // forward_device left the sequence offsets in w.offs
  TS_CUDA_TRY(ts::launch_viterbi(w.logits.p, reinterpret_cast<const int*>(w.offs.p), n_seqs, max_len, calibration,
                                 w.tags.p, st));
  TS_CUDA_TRY(cudaMemcpyAsync(pin_tags, w.tags.p, T, cudaMemcpyDeviceToHost, st));
  rc = check_dev_err(h->err.p, st);
  if (rc) return rc;
  memcpy(tags, pin_tags, T);
  return TS_OK;
}

int ts_cuda_forward_trace(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, const uint32_t* seq_offsets,
                          uint32_t n_seqs, float* logits, int32_t* topk_trace) {
  if (!h || !topk_trace) return fail(TS_ERR_ARG, "ts_cuda_forward_trace: null argument");
  h->trace_topk = topk_trace;
  int rc = ts_cuda_forward_packed(h, ids, mask, seq_offsets, n_seqs, logits);
  h->trace_topk = nullptr;
  return rc;
}

int ts_cuda_forward(ts_cuda_t* h, const int32_t* ids, const uint8_t* mask, uint32_t T, float* logits) {
  if (T == 0) return TS_OK;
  const uint32_t offs[2] = {0, T};
  return ts_cuda_forward_packed(h, ids, mask, offs, 1, logits);
}

int ts_cuda_check(ts_cuda_t* h, void* stream) {
  if (!h) return fail(TS_ERR_ARG, "ts_cuda_check: null handle");
  DevGuard g(h->cfg.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(TS_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
  return check_dev_err(h->err.p, st);
}

const char* ts_cuda_device_name(ts_cuda_t* h) { return h ? h->name.c_str() : ""; }

int ts_cuda_profile(ts_cuda_t* h, int32_t enable) {
  if (!h) return fail(TS_ERR_ARG, "ts_cuda_profile: null handle");
  DevGuard g(h->cfg.device);
  cudaStreamSynchronize(h->stream);
  for (auto& m : h->marks) {
    h->ev_pool.push_back(m.a);
    h->ev_pool.push_back(m.b);
  }
  h->marks.clear();
  for (int i = 0; i < TS_PHASE_COUNT; i++) { h->ph_ms[i] = 0; h->ph_launch[i] = 0; h->ph_flops[i] = 0; }
  h->prof = enable != 0;
  h->n_launch = 0;
  return TS_OK;
}

int ts_cuda_profile_read(ts_cuda_t* h, double* ms, uint64_t* launches, uint64_t* flops, uint64_t* total_launches) {
  if (!h) return fail(TS_ERR_ARG, "ts_cuda_profile_read: null handle");
  DevGuard g(h->cfg.device);
  for (auto& m : h->marks) {
    float t = 0.0f;
    cudaError_t e = cudaEventSynchronize(m.b);
    if (e != cudaSuccess) return fail(TS_ERR_CUDA, "profile event: %s", cudaGetErrorString(e));
    cudaEventElapsedTime(&t, m.a, m.b);
    h->ph_ms[m.phase] += t;
    h->ph_launch[m.phase] += 1;
    h->ph_flops[m.phase] += m.flops;
    h->ev_pool.push_back(m.a);
    h->ev_pool.push_back(m.b);
  }
  h->marks.clear();
  for (int i = 0; i < TS_PHASE_COUNT; i++) {
    if (ms) ms[i] = h->ph_ms[i];
    if (launches) launches[i] = h->ph_launch[i];
    if (flops) flops[i] = h->ph_flops[i];
  }
  if (total_launches) *total_launches = h->n_launch;
  return TS_OK;
}

void ts_cuda_destroy(ts_cuda_t* h) {
  if (!h) return;
  {
    DevGuard g(h->cfg.device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    if (h->pin) cudaFreeHost(h->pin);
    for (auto& sg : h->stage) {
      if (sg.p) cudaFreeHost(sg.p);
      if (sg.done) cudaEventDestroy(sg.done);
    }
    if (h->copy_st) cudaStreamSynchronize(h->copy_st);
    for (auto& sl : h->slot) {
      if (sl.p) cudaFreeHost(sl.p);
      if (sl.fwd) cudaEventDestroy(sl.fwd);
      if (sl.done) cudaEventDestroy(sl.done);
      sl.dlog.release();
    }
    if (h->copy_st) cudaStreamDestroy(h->copy_st);
    h->copy_st = nullptr;
    for (auto& m : h->marks) { cudaEventDestroy(m.a); cudaEventDestroy(m.b); }
    for (auto e : h->ev_pool) cudaEventDestroy(e);
    if (h->ep_hcounts) cudaFreeHost(h->ep_hcounts);
    ts::ep_comm_destroy(h->ep_comm, false);
    h->ep_comm = nullptr;
    h->layers.clear();
    if (h->stream) cudaStreamDestroy(h->stream);
    h->stream = nullptr;
  }
  DevGuard g(h->cfg.device);
  delete h;
}

// ---------------------------------------------------------------------------
// per-op entry points
// ---------------------------------------------------------------------------
int ts_cuda_op_gather_bq(const uint8_t* d_int4, const uint16_t* d_scales, const uint8_t* d_zp, const int32_t* d_ids,
                         uint16_t* d_out, uint32_t T, uint32_t V, uint32_t D, void* stream) {
  if (!d_int4 || !d_scales || !d_zp || !d_ids || !d_out) return fail(TS_ERR_ARG, "ts_cuda_op_gather_bq: null pointer");
  if (D % 32) return fail(TS_ERR_UNSUPPORTED, "D=%u must be a multiple of 32", D);
  TS_CUDA_TRY(ts::launch_embed(d_int4, d_scales, d_zp, d_ids, d_out, T, V, D, (cudaStream_t)stream));
  return TS_OK;
}

int ts_cuda_op_rmsnorm(const uint16_t* d_a, const uint16_t* d_b, const uint16_t* d_gamma, uint16_t* d_sum, float* d_out,
                       uint32_t T, uint32_t D, float eps, void* stream) {
  if (!d_a || !d_gamma || !d_out || (d_b && !d_sum)) return fail(TS_ERR_ARG, "ts_cuda_op_rmsnorm: null pointer");
  if (D > 8192 || D % 8) return fail(TS_ERR_UNSUPPORTED, "D=%u must be a multiple of 8, at most 8192", D);
  cudaStream_t st = (cudaStream_t)stream;
  if (d_b) TS_CUDA_TRY(ts::launch_add_rmsnorm(d_a, d_b, d_gamma, d_sum, d_out, nullptr, T, D, eps, st));
  else TS_CUDA_TRY(ts::launch_rmsnorm(d_a, d_gamma, d_out, nullptr, T, D, eps, st));
  return TS_OK;
}

ts_cuda_w4_t* ts_cuda_w4_create(int32_t device, const uint8_t* int4, const uint16_t* scales, const uint8_t* zp,
                                const uint16_t* bias, uint32_t E, uint32_t N, uint32_t K, char* err, size_t err_cap) {
  auto bad = [&](const char* msg) -> ts_cuda_w4_t* {
    g_err = msg;
    if (err && err_cap) snprintf(err, err_cap, "%s", msg);
    return nullptr;
  };
  if (!int4 || !scales || E == 0 || N == 0 || K == 0) return bad("ts_cuda_w4_create: bad argument");
  DevGuard g(device);
  auto* w = new ts_cuda_w4_t();
  w->device = device;
  if (cudaStreamCreateWithFlags(&w->stream, cudaStreamNonBlocking) != cudaSuccess || w->err.alloc(1) != cudaSuccess ||
      cudaMemset(w->err.p, 0, 4) != cudaSuccess) {
    delete w;
    return bad("ts_cuda_w4_create: CUDA initialisation failed");
  }
  DevArr<int> nb;
  const uint32_t BN = 128;
  int rc = nb.alloc(1) == cudaSuccess && cudaMemsetAsync(nb.p, 0, 4, w->stream) == cudaSuccess
               ? w4_upload(w->w, int4, scales, zp, bias, E, N, K, BN, true, nb.p, w->stream)
               : TS_ERR_CUDA;
  int nbad = 0;
  if (rc == TS_OK && (cudaMemcpyAsync(&nbad, nb.p, 4, cudaMemcpyDeviceToHost, w->stream) != cudaSuccess ||
                      cudaStreamSynchronize(w->stream) != cudaSuccess))
    rc = TS_ERR_CUDA;
  if (rc != TS_OK || nbad) {
    std::string m = rc != TS_OK ? g_err : "weight scales must be zero or normal fp16 numbers";
    if (w->stream) cudaStreamDestroy(w->stream);
    delete w;
    return bad(m.c_str());
  }
  return w;
}

void ts_cuda_w4_destroy(ts_cuda_w4_t* w) {
  if (!w) return;
  DevGuard g(w->device);
  if (w->stream) {
    cudaStreamSynchronize(w->stream);
    cudaStreamDestroy(w->stream);
  }
  delete w;
}

int ts_cuda_op_dequant(const ts_cuda_w4_t* w, uint32_t expert, uint16_t* d_out, void* stream) {
  if (!w || !d_out || expert >= w->w.E) return fail(TS_ERR_ARG, "ts_cuda_op_dequant: bad argument");
  ts::W4Tiles t = w->w.tiles();
  TS_CUDA_TRY(ts::launch_dequant_tiles(t.blobs + (size_t)expert * t.expert_stride, w->w.N, w->w.K, w->w.BN, t.n_kc,
                                       d_out, (cudaStream_t)stream));
  return TS_OK;
}

int ts_cuda_op_matmul_nbits(const ts_cuda_w4_t* w, uint32_t expert, const void* d_x, int32_t x_dtype, void* d_out,
                            int32_t out_dtype, uint32_t M, int32_t mode, void* stream) {
  if (!w || !d_x || !d_out || expert >= w->w.E) return fail(TS_ERR_ARG, "ts_cuda_op_matmul_nbits: bad argument");
  if (M == 0) return TS_OK;
  if (out_dtype != TS_DTYPE_F16 && out_dtype != TS_DTYPE_F32) return fail(TS_ERR_ARG, "out_dtype must be F16 or F32");
  cudaStream_t st = (cudaStream_t)stream;
  if (mode == TS_MODE_FAST) {
    if (x_dtype != TS_DTYPE_F16) return fail(TS_ERR_UNSUPPORTED, "the tensor-core path takes fp16 activations");
    if ((reinterpret_cast<uintptr_t>(d_x) & 15u) || ((w->w.K * 2) & 15u))
      return fail(TS_ERR_UNSUPPORTED, "activation tensor map (16-byte alignment)");
    ts::GemmArgs g;
    g.M = M; g.dense_expert = expert; g.err = w->err.p; g.out0 = d_out; g.ld0 = w->w.N;
    if (out_dtype == TS_DTYPE_F16 && !(w->w.N & 1u) && !(reinterpret_cast<uintptr_t>(d_out) & 3u)) {
      // fp16 output: the GEMM with the weights in TMEM, as the forward runs it
      const uint32_t rows = ts::gemm_tm_rows();
      TS_CUDA_TRY(ts::launch_gemm_w4_tm(w->w.tiles(), d_x, M, g, ts::kEpiF16, (M + rows - 1) / rows, st));
      return TS_OK;
    }
    CUtensorMap tm;
    if (!ts::make_act_tmap(&tm, d_x, M, w->w.K)) return fail(TS_ERR_UNSUPPORTED, "activation tensor map (16-byte alignment)");
    TS_CUDA_TRY(ts::launch_gemm_w4_tc(w->w.tiles(), tm, g, out_dtype == TS_DTYPE_F16 ? ts::kEpiF16 : ts::kEpiF32,
                                      (M + 127) / 128, st));
    return TS_OK;
  }
  if (x_dtype != TS_DTYPE_F16 && x_dtype != TS_DTYPE_F32) return fail(TS_ERR_ARG, "x_dtype must be F16 or F32");
  ts::ExactArgs a = w->w.exact();
  a.w_int4 += (size_t)expert * a.w_int4_estride;
  a.w_scales += (size_t)expert * a.w_scales_estride;
  if (a.w_zp) a.w_zp += (size_t)expert * a.w_zp_estride;
  a.bias += (size_t)expert * a.bias_estride;
  a.x = d_x; a.ldx = w->w.K; a.M = M; a.out = d_out; a.ldo = w->w.N;
  TS_CUDA_TRY(ts::launch_matmul_exact(a, x_dtype == TS_DTYPE_F32, out_dtype == TS_DTYPE_F16 ? ts::kOutF16 : ts::kOutF32,
                                      (M + 127) / 128, st));
  return TS_OK;
}

int ts_cuda_op_router_topk(ts_cuda_t* h, uint32_t layer, const float* d_x, int32_t* d_idx, float* d_w, uint32_t T,
                           void* stream) {
  if (!h || !d_x || !d_idx || !d_w) return fail(TS_ERR_ARG, "ts_cuda_op_router_topk: null argument");
  if (!h->finalized || layer >= h->cfg.n_layers) return fail(TS_ERR_STATE, "handle not finalized or bad layer");
  if (T > h->cfg.max_tokens) return fail(TS_ERR_UNSUPPORTED, "T > max_tokens");
  DevGuard g(h->cfg.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  int rc = ensure_workspace(h, false);
  if (rc) return rc;
  const ts_cuda_cfg& c = h->cfg;
  if (T == 0) return TS_OK;
  if (c.mode != TS_MODE_EXACT && c.top_k == 4 && c.n_experts <= ts::kMaxRouterExperts) {
    // fast mode, as the forward runs it: tensor-core logits from fp16(x)
    // name the candidates, which are then evaluated in the reference's order
    Workspace& w = h->ws;
    TS_CUDA_TRY(ts::launch_f32_to_f16_absum(d_x, w.xn16.p, w.absum.p, T, c.d_model, st));
    CUtensorMap tx;
    if (!ts::make_act_tmap(&tx, w.xn16.p, T, c.d_model)) return fail(TS_ERR_CUDA, "cuTensorMapEncodeTiled failed (router)");
    const LayerDev& L = *h->layers[layer];
    ts::GemmArgs gr;
    gr.M = T; gr.err = h->err.p; gr.out0 = w.rcand.p; gr.absum = w.absum.p; gr.rbound = L.rbound.p;
    TS_CUDA_TRY(ts::launch_gemm_w4_tc(L.router.tiles(), tx, gr, ts::kEpiRouterCert, (T + 127) / 128, st));
    RouterIn rin;
    rin.x32 = d_x; rin.absum = w.absum.p;
    TS_CUDA_TRY(ts::launch_router_cert(router_cert_args(h, L, rin, nullptr, nullptr, d_idx, d_w, nullptr, T),
                                       ts::kRouterSrcF32, st));
    return TS_OK;
  }
  ts::ExactArgs ra = h->layers[layer]->router.exact();
  ra.x = d_x; ra.ldx = c.d_model; ra.M = T; ra.out = h->ws.rlogits.p; ra.ldo = c.n_experts;
  TS_CUDA_TRY(ts::launch_matmul_exact(ra, true, ts::kOutF32, (T + 127) / 128, st));
  TS_CUDA_TRY(ts::launch_router_topk(h->ws.rlogits.p, d_idx, d_w, nullptr, T, c.n_experts, c.top_k, st));
  return TS_OK;
}

int ts_cuda_op_router_addnorm(ts_cuda_t* h, uint32_t layer, const uint16_t* d_res, const uint16_t* d_attn,
                              float* d_x32, int32_t* d_idx, float* d_w, uint32_t T, void* stream) {
  if (!h || !d_res || !d_attn || !d_idx || !d_w) return fail(TS_ERR_ARG, "ts_cuda_op_router_addnorm: null argument");
  if (!h->finalized || layer >= h->cfg.n_layers) return fail(TS_ERR_STATE, "handle not finalized or bad layer");
  const ts_cuda_cfg& c = h->cfg;
  if (c.mode == TS_MODE_EXACT || c.top_k != 4 || c.n_experts > ts::kMaxRouterExperts)
    return fail(TS_ERR_UNSUPPORTED, "ts_cuda_op_router_addnorm: the fast mode's router (top_k 4, <= 128 experts)");
  if (T > c.max_tokens) return fail(TS_ERR_UNSUPPORTED, "T > max_tokens");
  if (T == 0) return TS_OK;
  DevGuard g(c.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  int rc = ensure_workspace(h, false);
  if (rc) return rc;
  Workspace& w = h->ws;
  const LayerDev& L = *h->layers[layer];
  // the forward's steps: add + RMSNorm (sum, 1 / rms, sum |x| and fp16 x
  // kept), candidates from the tensor-core logits, the exact candidate pass
  // on the f32 input rebuilt from the stored sum and 1 / rms
  TS_CUDA_TRY(ts::launch_rmsnorm_fast(d_res, d_attn, L.ln2.p, w.res2.p, w.xn16.p, T, c.d_model, c.eps, st, w.absum.p,
                                      w.rinv.p, d_x32));
  CUtensorMap tx;
  if (!ts::make_act_tmap(&tx, w.xn16.p, T, c.d_model)) return fail(TS_ERR_CUDA, "cuTensorMapEncodeTiled failed (router)");
  ts::GemmArgs gr;
  gr.M = T; gr.err = h->err.p; gr.out0 = w.rcand.p; gr.absum = w.absum.p; gr.rbound = L.rbound.p;
  TS_CUDA_TRY(ts::launch_gemm_w4_tc(L.router.tiles(), tx, gr, ts::kEpiRouterCert, (T + 127) / 128, st));
  RouterIn rin;
  rin.src = ts::kRouterSrcAddNorm; rin.a = w.res2.p; rin.inv = w.rinv.p; rin.gamma = L.ln2.p; rin.absum = w.absum.p;
  TS_CUDA_TRY(ts::launch_router_cert(router_cert_args(h, L, rin, nullptr, nullptr, d_idx, d_w, nullptr, T),
                                     ts::kRouterSrcAddNorm, st));
  h->n_launch += 3;
  return TS_OK;
}

int ts_cuda_op_moe(ts_cuda_t* h, uint32_t layer, const float* d_x, uint16_t* d_out, int32_t* d_idx, float* d_w,
                   uint32_t T, void* stream) {
  if (!h || !d_x || !d_out) return fail(TS_ERR_ARG, "ts_cuda_op_moe: null argument");
  if (h->ep_world > 0) return fail(TS_ERR_UNSUPPORTED, "ts_cuda_op_moe: the handle holds a slice of the experts");
  if (!h->finalized || layer >= h->cfg.n_layers) return fail(TS_ERR_STATE, "handle not finalized or bad layer");
  if (T > h->cfg.max_tokens) return fail(TS_ERR_UNSUPPORTED, "T > max_tokens");
  if (T == 0) return TS_OK;
  DevGuard g(h->cfg.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  const bool exact = h->cfg.mode == TS_MODE_EXACT;
  int rc = ensure_workspace(h, exact);
  if (rc) return rc;
  const ts_cuda_cfg& c = h->cfg;
  if (!exact) TS_CUDA_TRY(ts::launch_f32_to_f16_absum(d_x, h->ws.xn16.p, h->ws.absum.p, T, c.d_model, st));
  // both top-k paths add expert counts into zeroed permutation rows
  TS_CUDA_TRY(cudaMemsetAsync(h->ws.hist.p, 0, (size_t)ts::route_chunks(T) * c.n_experts * sizeof(int), st));
  RouterIn rin;  // the router input is the given f32 x
  rin.x32 = d_x; rin.absum = h->ws.absum.p;
  rc = moe_half(h, *h->layers[layer], d_x, h->ws.xn16.p, nullptr, d_out, T, nullptr, nullptr, exact, st, -1, rin);
  if (rc) return rc;
  if (d_idx) TS_CUDA_TRY(cudaMemcpyAsync(d_idx, h->ws.ridx.p, (size_t)T * c.top_k * 4, cudaMemcpyDeviceToDevice, st));
  if (d_w) TS_CUDA_TRY(cudaMemcpyAsync(d_w, h->ws.rw.p, (size_t)T * c.top_k * 4, cudaMemcpyDeviceToDevice, st));
  return TS_OK;
}

int ts_cuda_op_banded_attention(const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v, const float* d_sinks,
                                const uint8_t* d_mask, uint16_t* d_out, uint32_t T, uint32_t Hq, uint32_t Hkv,
                                uint32_t head_dim, uint32_t window, const uint32_t* seq_offsets, uint32_t n_seqs,
                                int32_t mode, void* stream) {
  if (!d_q || !d_k || !d_v || !d_sinks || !d_out) return fail(TS_ERR_ARG, "ts_cuda_op_banded_attention: null pointer");
  if (T == 0) return TS_OK;
  if (Hkv == 0 || Hq % Hkv) return fail(TS_ERR_ARG, "Hq must be a multiple of Hkv");
  if (window > 1024) return fail(TS_ERR_UNSUPPORTED, "window %u > 1024", window);
  cudaStream_t st = (cudaStream_t)stream;
  // per-token sequence info (a scratch allocation per call: this is a test/benchmark entry point)
  DevArr<uint32_t> offs;
  DevArr<int> pos, ss, sl;
  std::vector<uint32_t> one = {0, T};
  const uint32_t* ho = seq_offsets ? seq_offsets : one.data();
  const uint32_t ns = seq_offsets ? n_seqs : 1;
  if (ns == 0 || ho[0] != 0 || ho[ns] != T) return fail(TS_ERR_ARG, "seq_offsets must run from 0 to T");
  for (uint32_t s = 0; s < ns; s++)
    if (ho[s + 1] <= ho[s]) return fail(TS_ERR_ARG, "empty sequence %u", s);
  TS_CUDA_TRY(offs.alloc(ns + 1));
  TS_CUDA_TRY(pos.alloc(T));
  TS_CUDA_TRY(ss.alloc(T));
  TS_CUDA_TRY(sl.alloc(T));
  TS_CUDA_TRY(cudaMemcpyAsync(offs.p, ho, (size_t)(ns + 1) * 4, cudaMemcpyHostToDevice, st));
  TS_CUDA_TRY(ts::launch_seq_info(offs.p, ns, T, pos.p, ss.p, sl.p, st));
  ts::AttnArgs a;
  a.q = d_q; a.k = d_k; a.v = d_v; a.sinks = d_sinks; a.mask = d_mask; a.out = d_out;
  a.sstart = ss.p; a.slen = sl.p; a.T = T; a.Hq = Hq; a.Hkv = Hkv; a.hd = head_dim; a.window = window;
  if (mode == TS_MODE_FAST && (head_dim != 64 || Hq / Hkv > 7))
    return fail(TS_ERR_UNSUPPORTED, "tensor-core attention needs head_dim 64, group <= 7");
  // 16-query tiles (both modes: the exact kernel works on them too)
  std::vector<int2> th(ts::attention_max_tiles(T, ns));
  uint32_t ntl = 0;
  ts::attention_tiles(ho, ns, th.data(), &ntl);
  DevArr<int2> td;
  TS_CUDA_TRY(td.alloc(ntl));
  TS_CUDA_TRY(cudaMemcpyAsync(td.p, th.data(), (size_t)ntl * sizeof(int2), cudaMemcpyHostToDevice, st));
  a.tiles = td.p;
  a.n_tiles = ntl;
  if (mode == TS_MODE_FAST) TS_CUDA_TRY(ts::launch_attention_tc(a, st));
  else TS_CUDA_TRY(ts::launch_attention_exact(a, st));
  TS_CUDA_TRY(cudaStreamSynchronize(st));  // scratch above is freed on return
  return TS_OK;
}

int ts_cuda_op_viterbi(const float* d_logits, const uint32_t* seq_offsets, uint32_t n_seqs, const float* calibration,
                       uint8_t* d_tags, void* stream) {
  if (!d_logits || !d_tags || !seq_offsets || n_seqs == 0) return fail(TS_ERR_ARG, "ts_cuda_op_viterbi: null argument");
  uint32_t max_len = 0;
  int rc = check_viterbi_args(seq_offsets, n_seqs, calibration, &max_len);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  DevArr<uint32_t> offs;  // a scratch allocation per call: this is a test/benchmark entry point
  TS_CUDA_TRY(offs.alloc(n_seqs + 1));
  TS_CUDA_TRY(cudaMemcpyAsync(offs.p, seq_offsets, (size_t)(n_seqs + 1) * 4, cudaMemcpyHostToDevice, st));
  TS_CUDA_TRY(ts::launch_viterbi(d_logits, reinterpret_cast<const int*>(offs.p), n_seqs, max_len, calibration, d_tags,
                                 st));
  TS_CUDA_TRY(cudaStreamSynchronize(st));  // scratch above is freed on return
  return TS_OK;
}

int ts_cuda_op_rope(const uint16_t* d_x, uint16_t* d_out, const uint16_t* d_cos, const uint16_t* d_sin,
                    const int32_t* d_pos, uint32_t T, uint32_t H, uint32_t head_dim, void* stream) {
  if (!d_x || !d_out || !d_cos || !d_sin || !d_pos) return fail(TS_ERR_ARG, "ts_cuda_op_rope: null pointer");
  if (head_dim == 0 || head_dim % 2 || H == 0) return fail(TS_ERR_ARG, "head_dim must be even and H > 0");
  if (T == 0) return TS_OK;
  // the exact-mode RoPE: the rotation half of split_rope_kernel over one
  // [T, H * head_dim] block (no K or V part)
  TS_CUDA_TRY(ts::launch_split_rope(d_x, d_out, nullptr, nullptr, d_pos, d_cos, d_sin, T, H * head_dim, 0, 0, head_dim,
                                    (cudaStream_t)stream));
  return TS_OK;
}

int ts_cuda_op_qkv_rope(ts_cuda_t* h, uint32_t layer, const uint16_t* d_x, const uint32_t* seq_offsets,
                        uint32_t n_seqs, uint16_t* d_q, uint16_t* d_k, uint16_t* d_v, void* stream) {
  if (!h || !d_x || !d_q || !d_k || !d_v || !seq_offsets || n_seqs == 0)
    return fail(TS_ERR_ARG, "ts_cuda_op_qkv_rope: null argument");
  if (!h->finalized || layer >= h->cfg.n_layers) return fail(TS_ERR_STATE, "handle not finalized or bad layer");
  const ts_cuda_cfg& c = h->cfg;
  if (seq_offsets[0] != 0) return fail(TS_ERR_ARG, "seq_offsets[0] must be 0");
  for (uint32_t s = 0; s < n_seqs; s++) {
    if (seq_offsets[s + 1] <= seq_offsets[s]) return fail(TS_ERR_ARG, "sequence %u is empty", s);
    if (seq_offsets[s + 1] - seq_offsets[s] > c.max_seq_len) return fail(TS_ERR_UNSUPPORTED, "sequence > max_seq_len");
  }
  const uint32_t T = seq_offsets[n_seqs];
  if (T > c.max_tokens) return fail(TS_ERR_UNSUPPORTED, "%u tokens > max_tokens %u", T, c.max_tokens);
  DevGuard g(c.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  int rc = ensure_workspace(h, false);
  if (rc) return rc;
  Workspace& w = h->ws;
  ts_cuda::Stage* sg = nullptr;
  if ((rc = next_stage(h, (size_t)(n_seqs + 1) * 4, &sg))) return rc;
  memcpy(sg->p, seq_offsets, (size_t)(n_seqs + 1) * 4);
  TS_CUDA_TRY(cudaMemcpyAsync(w.offs.p, sg->p, (size_t)(n_seqs + 1) * 4, cudaMemcpyHostToDevice, st));
  TS_CUDA_TRY(cudaEventRecord(sg->done, st));
  TS_CUDA_TRY(ts::launch_seq_info(w.offs.p, n_seqs, T, w.pos.p, w.sstart.p, w.slen.p, st));
  const uint32_t Q = c.n_heads * c.head_dim, KV = c.n_kv_heads * c.head_dim;
  ts::GemmArgs ga;
  ga.M = T; ga.err = h->err.p;
  ga.out0 = d_q; ga.ld0 = Q; ga.out1 = d_k; ga.ld1 = KV; ga.out2 = d_v; ga.ld2 = KV;
  ga.q_cols = Q; ga.k_cols = KV; ga.pos = w.pos.p; ga.rope_cos = h->rope_cos.p; ga.rope_sin = h->rope_sin.p;
  ga.rope_cs = h->rope_cs.p;
  const uint32_t mt_tc = (T + ts::gemm_tm_rows() - 1) / ts::gemm_tm_rows();
  TS_CUDA_TRY(ts::launch_gemm_w4_tm(h->layers[layer]->qkv.tiles(), d_x, T, ga, ts::kEpiQkvRope, mt_tc, st));
  return TS_OK;
}

int ts_cuda_op_attention(ts_cuda_t* h, const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v,
                         const float* d_sinks, const uint8_t* d_mask, uint16_t* d_out, const uint32_t* seq_offsets,
                         uint32_t n_seqs, void* stream) {
  if (!h || !d_q || !d_k || !d_v || !d_sinks || !d_out || !seq_offsets || n_seqs == 0)
    return fail(TS_ERR_ARG, "ts_cuda_op_attention: null argument");
  if (!h->finalized) return fail(TS_ERR_STATE, "ts_cuda_finalize has not succeeded");
  const ts_cuda_cfg& c = h->cfg;
  if (seq_offsets[0] != 0) return fail(TS_ERR_ARG, "seq_offsets[0] must be 0");
  for (uint32_t s = 0; s < n_seqs; s++)
    if (seq_offsets[s + 1] <= seq_offsets[s]) return fail(TS_ERR_ARG, "sequence %u is empty", s);
  const uint32_t T = seq_offsets[n_seqs];
  if (T > c.max_tokens) return fail(TS_ERR_UNSUPPORTED, "%u tokens > max_tokens %u", T, c.max_tokens);
  DevGuard g(c.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  const bool exact = c.mode == TS_MODE_EXACT;
  int rc = ensure_workspace(h, false);
  if (rc) return rc;
  Workspace& w = h->ws;
  // offsets and the tile list through the pinned ring, as in the forward
  const size_t offs_bytes = ((size_t)(n_seqs + 1) * 4 + 15) & ~size_t(15);
  ts_cuda::Stage* sg = nullptr;
  if ((rc = next_stage(h, offs_bytes + (size_t)ts::attention_max_tiles(T, n_seqs) * sizeof(int2), &sg))) return rc;
  memcpy(sg->p, seq_offsets, (size_t)(n_seqs + 1) * 4);
  TS_CUDA_TRY(cudaMemcpyAsync(w.offs.p, sg->p, (size_t)(n_seqs + 1) * 4, cudaMemcpyHostToDevice, st));
  ts::AttnArgs aa;
  aa.q = d_q; aa.k = d_k; aa.v = d_v; aa.sinks = d_sinks; aa.mask = d_mask; aa.out = d_out;
  aa.sstart = w.sstart.p; aa.slen = w.slen.p; aa.T = T; aa.Hq = c.n_heads; aa.Hkv = c.n_kv_heads;
  aa.hd = c.head_dim; aa.window = c.window; aa.err = h->err.p;
  {
    uint32_t nt = 0;
    int2* th = reinterpret_cast<int2*>(sg->p + offs_bytes);
    ts::attention_tiles(seq_offsets, n_seqs, th, &nt);
    TS_CUDA_TRY(cudaMemcpyAsync(w.atiles.p, th, (size_t)nt * sizeof(int2), cudaMemcpyHostToDevice, st));
    aa.tiles = w.atiles.p;
    aa.n_tiles = nt;
  }
  TS_CUDA_TRY(cudaEventRecord(sg->done, st));
  TS_CUDA_TRY(ts::launch_seq_info(w.offs.p, n_seqs, T, w.pos.p, w.sstart.p, w.slen.p, st));
  h->n_launch += 2;
  if (exact) TS_CUDA_TRY(ts::launch_attention_exact(aa, st));
  else TS_CUDA_TRY(ts::launch_attention_tc(aa, st));
  return TS_OK;
}

size_t ts_cuda_ep_unique_id(uint8_t* out, size_t cap) {
  if (!out) return ts::ep_unique_id_bytes();
  std::string err;
  if (!ts::ep_unique_id(out, cap, &err)) {
    fail(TS_ERR_CUDA, "%s", err.c_str());
    return 0;
  }
  return ts::ep_unique_id_bytes();
}

int ts_cuda_ep_init(ts_cuda_t* h, int32_t rank, int32_t world, const uint8_t* nccl_id, size_t id_len) {
  if (!h || !nccl_id || world < 1 || rank < 0 || rank >= world) return fail(TS_ERR_ARG, "ts_cuda_ep_init: bad argument");
  if (h->finalized || h->ep_world > 0) return fail(TS_ERR_STATE, "ts_cuda_ep_init: call it once, before ts_cuda_finalize");
  const ts_cuda_cfg& c = h->cfg;
  if (c.n_experts % (uint32_t)world) return fail(TS_ERR_UNSUPPORTED, "%u experts do not split over %d ranks", c.n_experts, world);
  if (c.top_k != 4 || c.n_experts > ts::kMaxRouterExperts)
    return fail(TS_ERR_UNSUPPORTED, "expert parallelism needs the fast router (top_k 4, at most 128 experts)");
  DevGuard g(c.device);
  std::string err;
  void* comm = nullptr;
  if (!ts::ep_comm_init(&comm, world, nccl_id, id_len, rank, &err)) return fail(TS_ERR_CUDA, "%s", err.c_str());
  h->ep_comm = comm;
  h->ep_world = world;
  h->ep_rank = rank;
  h->e_local = c.n_experts / (uint32_t)world;
  h->e_first = (uint32_t)rank * h->e_local;
  return TS_OK;
}

int ts_cuda_ep_plan(const int32_t* counts, const int32_t* recv_counts, int32_t world, int32_t e_local,
                    int32_t tile_rows, uint64_t* send_n, uint64_t* recv_n, int32_t* tiles, uint32_t tiles_cap,
                    uint32_t* n_tiles) {
  if (!counts || !recv_counts || world < 1 || e_local < 1 || tile_rows < 1 || !n_tiles)
    return fail(TS_ERR_ARG, "ts_cuda_ep_plan: bad argument");
  ts::EpPlan plan;
  ts::ep_plan(counts, recv_counts, world, 0, e_local, tile_rows, &plan);
  for (int p = 0; p < world; p++) {
    if (send_n) send_n[p] = plan.send_n[p];
    if (recv_n) recv_n[p] = plan.recv_n[p];
  }
  *n_tiles = (uint32_t)plan.tiles.size();
  if (tiles) {
    if (plan.tiles.size() > tiles_cap) return fail(TS_ERR_ARG, "ts_cuda_ep_plan: %zu tiles > capacity", plan.tiles.size());
    for (size_t i = 0; i < plan.tiles.size(); i++) {
      tiles[4 * i] = plan.tiles[i].x;
      tiles[4 * i + 1] = plan.tiles[i].y;
      tiles[4 * i + 2] = plan.tiles[i].z;
      tiles[4 * i + 3] = plan.tiles[i].w;
    }
  }
  return TS_OK;
}

int ts_cuda_selftest_wait_timeout(ts_cuda_t* h, uint32_t limit_us, int32_t* d_result, void* stream) {
  if (!h) return fail(TS_ERR_ARG, "ts_cuda_selftest_wait_timeout: null handle");
  if (limit_us == 0 || limit_us > 1000000u) return fail(TS_ERR_ARG, "limit_us must be in [1, 1000000]");
  DevGuard g(h->cfg.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
  TS_CUDA_TRY(ts::launch_wait_selftest(h->err.p, 1000ull * limit_us, d_result, st));
  return TS_OK;
}

int ts_cuda_rope_tables(ts_cuda_t* h, uint32_t rows, uint16_t* cos_out, uint16_t* sin_out) {
  if (!h || !cos_out || !sin_out) return fail(TS_ERR_ARG, "ts_cuda_rope_tables: null argument");
  if (!h->finalized) return fail(TS_ERR_STATE, "handle not finalized");
  if (rows > h->cfg.max_seq_len) return fail(TS_ERR_ARG, "rows > max_seq_len");
  DevGuard g(h->cfg.device);
  const size_t n = (size_t)rows * (h->cfg.head_dim / 2) * 2;
  TS_CUDA_TRY(cudaMemcpy(cos_out, h->rope_cos.p, n, cudaMemcpyDeviceToHost));
  TS_CUDA_TRY(cudaMemcpy(sin_out, h->rope_sin.p, n, cudaMemcpyDeviceToHost));
  return TS_OK;
}

}  // extern "C"
