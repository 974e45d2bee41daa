// noalloc.cu — the allocation-free variant of the banded-attention entry point.
//
// ts_cuda_op_banded_attention (runtime.cu) allocates its scratch (the
// sequence offsets, per-token sequence info and the tensor-core tile list)
// with cudaMalloc on every call.  Some callers cannot allow that: an
// embedding runtime or serving loop that owns every device allocation under a
// fixed budget, or a latency-sensitive loop that cannot afford the implicit
// device-wide synchronisation cudaMalloc/cudaFree may perform between its
// kernels.  This variant runs the same kernels with its scratch in one
// file-scope device array instead, so it allocates nothing.
//
// Limits: at most kNoAllocMaxTokens tokens and kNoAllocMaxSeqs sequences per
// call (larger calls are rejected with TS_ERR_UNSUPPORTED).  The array lives
// on every GPU that loads the library until the process exits, and every
// call on that GPU shares it: calls that overlap on the GPU (e.g. issued on
// two streams at once) race on it and must be serialized by the caller.
// Each call writes every scratch entry it reads before reading it, so nothing
// carries over from the previous call.
#include "textsift_cuda.h"
#include "ts_common.cuh"
#include "ts_simt.h"

#include <mutex>

namespace {

constexpr uint32_t kNoAllocMaxTokens = 16384;
constexpr uint32_t kNoAllocMaxSeqs = 1024;
constexpr uint32_t kNoAllocMaxTiles = kNoAllocMaxTokens / 16 + kNoAllocMaxSeqs + 1;

// Byte offsets inside the scratch array (each region 256-byte aligned).
constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
constexpr size_t kOffOffs = 0;                                                  // uint32 [max_seqs + 1]
constexpr size_t kOffPos = align256(kOffOffs + 4 * (kNoAllocMaxSeqs + 1));     // int [max_tokens]
constexpr size_t kOffStart = align256(kOffPos + 4 * kNoAllocMaxTokens);        // int [max_tokens]
constexpr size_t kOffLen = align256(kOffStart + 4 * kNoAllocMaxTokens);        // int [max_tokens]
constexpr size_t kOffTiles = align256(kOffLen + 4 * kNoAllocMaxTokens);        // int2 [max_tiles]
constexpr size_t kScratchBytes = align256(kOffTiles + 8 * kNoAllocMaxTiles);   // ~221 KB

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

// Device address of g_attn_scratch, looked up once per device.  In host code
// the symbol's name only stands in for the device array; the address a kernel
// can use comes from cudaGetSymbolAddress with that device current.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_scratch_dev[kMaxDevices] = {nullptr};

// Errors go to the library's per-thread message (ts_cuda_last_error).
int noalloc_fail(int code, const char* msg) {
  ts::set_last_error(msg);
  return code;
}

}  // namespace

extern "C" int ts_cuda_op_banded_attention_noalloc(const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v,
                                                   const float* d_sinks, const uint8_t* d_mask, uint16_t* d_out,
                                                   uint32_t T, uint32_t Hq, uint32_t Hkv, uint32_t head_dim,
                                                   uint32_t window, const uint32_t* seq_offsets, uint32_t n_seqs,
                                                   int32_t mode, void* stream) {
  if (!d_q || !d_k || !d_v || !d_sinks || !d_out)
    return noalloc_fail(TS_ERR_ARG, "ts_cuda_op_banded_attention_noalloc: null pointer");
  if (T == 0) return TS_OK;
  if (Hkv == 0 || Hq % Hkv) return noalloc_fail(TS_ERR_ARG, "Hq must be a multiple of Hkv");
  if (window > 1024) return noalloc_fail(TS_ERR_UNSUPPORTED, "window > 1024");
  const uint32_t one[2] = {0, T};
  const uint32_t* ho = seq_offsets ? seq_offsets : one;
  const uint32_t ns = seq_offsets ? n_seqs : 1;
  if (T > kNoAllocMaxTokens || ns > kNoAllocMaxSeqs)
    return noalloc_fail(TS_ERR_UNSUPPORTED,
                        "ts_cuda_op_banded_attention_noalloc: at most 16384 tokens and 1024 sequences per call");
  if (ns == 0 || ho[0] != 0 || ho[ns] != T) return noalloc_fail(TS_ERR_ARG, "seq_offsets must run from 0 to T");
  for (uint32_t s = 0; s < ns; s++)
    if (ho[s + 1] <= ho[s]) return noalloc_fail(TS_ERR_ARG, "empty sequence");
  if (ts::attention_max_tiles(T, ns) > kNoAllocMaxTiles)
    return noalloc_fail(TS_ERR_UNSUPPORTED, "ts_cuda_op_banded_attention_noalloc: tile list exceeds scratch");
  if (mode == TS_MODE_FAST && (head_dim != 64 || Hq / Hkv > 7))
    return noalloc_fail(TS_ERR_UNSUPPORTED, "tensor-core attention needs head_dim 64, group <= 7");

  // once per device: the scratch array's device address
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return noalloc_fail(TS_ERR_CUDA, "cudaGetDevice failed");
  unsigned char* scratch;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_dev[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
      if (e != cudaSuccess || !p) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
      g_scratch_dev[dev] = static_cast<unsigned char*>(p);
    }
    scratch = g_scratch_dev[dev];
  }
  uint32_t* d_offs = reinterpret_cast<uint32_t*>(scratch + kOffOffs);
  int* d_pos = reinterpret_cast<int*>(scratch + kOffPos);
  int* d_start = reinterpret_cast<int*>(scratch + kOffStart);
  int* d_len = reinterpret_cast<int*>(scratch + kOffLen);
  int2* d_tiles = reinterpret_cast<int2*>(scratch + kOffTiles);

  cudaStream_t st = (cudaStream_t)stream;
  // A copy from pageable host memory is staged before cudaMemcpyAsync returns,
  // so the host arrays below may go out of scope afterwards.
  cudaError_t e = cudaMemcpyAsync(d_offs, ho, (size_t)(ns + 1) * 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = ts::launch_seq_info(d_offs, ns, T, d_pos, d_start, d_len, st);
  if (e != cudaSuccess) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
  ts::AttnArgs a;
  a.q = d_q; a.k = d_k; a.v = d_v; a.sinks = d_sinks; a.mask = d_mask; a.out = d_out;
  a.sstart = d_start; a.slen = d_len; a.T = T; a.Hq = Hq; a.Hkv = Hkv; a.hd = head_dim; a.window = window;
  if (mode == TS_MODE_FAST) {
    int2 th[kNoAllocMaxTiles];
    uint32_t ntl = 0;
    ts::attention_tiles(ho, ns, th, &ntl);
    e = cudaMemcpyAsync(d_tiles, th, (size_t)ntl * sizeof(int2), cudaMemcpyHostToDevice, st);
    a.tiles = d_tiles;
    a.n_tiles = ntl;
    if (e == cudaSuccess) e = ts::launch_attention_tc(a, st);
  } else {
    e = ts::launch_attention_exact(a, st);
  }
  if (e != cudaSuccess) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
  return TS_OK;
}
