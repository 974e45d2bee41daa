// noalloc.cu — the allocation-free variant of the banded-attention entry point.
//
// ts_cuda_op_banded_attention (runtime.cu) allocates its scratch (the
// sequence offsets, per-token sequence info and the tensor-core tile list)
// with cudaMalloc on every call.  Some callers cannot allow that: an
// embedding runtime or serving loop that owns every device allocation under a
// fixed budget, or a latency-sensitive loop that cannot afford the implicit
// device-wide synchronisation cudaMalloc/cudaFree may perform between its
// kernels.  This variant runs the same kernels with its scratch in one
// file-scope device array instead, so it allocates nothing, and it copies
// nothing from host memory either: the sequence offsets travel to the GPU as
// a kernel parameter, and the tile list is built on the GPU from them, so a
// call only enqueues kernels and returns.
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

// The sequence offsets by value: 4,100 bytes of kernel parameters (the
// parameter space of sm_70 and later holds up to 32,764 bytes).
struct SeqOffsets {
  uint32_t v[kNoAllocMaxSeqs + 1];
};

// One block of 1024 threads: copies the offsets into the scratch array and
// writes the tile list that attention_tiles() builds on the host for the
// allocating entry point (both attention kernels work on it) -- sequence s contributes
// ceil(len_s / rows) tiles {first query, sequence end} in order, placed after
// the tiles of sequences 0..s-1 (an exclusive scan over one count per thread).
__global__ void __launch_bounds__(1024) noalloc_prep_kernel(const SeqOffsets offs, uint32_t ns, uint32_t rows,
                                                            uint32_t* __restrict__ d_offs, int2* __restrict__ d_tiles) {
  __shared__ uint32_t warp_total[32];
  const uint32_t s = threadIdx.x, lane = s & 31u, warp = s >> 5;
  for (uint32_t i = s; i <= ns; i += blockDim.x) d_offs[i] = offs.v[i];
  const uint32_t lo = s < ns ? offs.v[s] : 0u, hi = s < ns ? offs.v[s + 1] : 0u;
  const uint32_t cnt = (hi - lo + rows - 1) / rows;
  uint32_t incl = cnt;  // inclusive scan within the warp
  for (uint32_t d = 1; d < 32; d <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) warp_total[warp] = incl;
  __syncthreads();
  uint32_t base = incl - cnt;
  for (uint32_t w = 0; w < warp; w++) base += warp_total[w];
  for (uint32_t j = 0; j < cnt; j++) d_tiles[base + j] = make_int2((int)(lo + j * rows), (int)hi);
}

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
  const uint32_t rows = ts::attention_tile_rows();
  uint32_t ntl = 0;
  for (uint32_t s = 0; s < ns; s++) ntl += (ho[s + 1] - ho[s] + rows - 1) / rows;
  if (ntl > kNoAllocMaxTiles)
    return noalloc_fail(TS_ERR_UNSUPPORTED, "ts_cuda_op_banded_attention_noalloc: tile list exceeds scratch");
  if (mode == TS_MODE_FAST && (head_dim != 64 || Hq / Hkv > 7))
    return noalloc_fail(TS_ERR_UNSUPPORTED, "tensor-core attention needs head_dim 64, group <= 7");

  // The scratch array's device address for the current device and context,
  // looked up on every call (no allocation, a table lookup once the module is
  // loaded): a cached address would go stale after cudaDeviceReset or under a
  // different context made current by the caller.
  void* sym = nullptr;
  const cudaError_t se = cudaGetSymbolAddress(&sym, g_attn_scratch);
  if (se != cudaSuccess || !sym) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(se));
  unsigned char* scratch = static_cast<unsigned char*>(sym);
  uint32_t* d_offs = reinterpret_cast<uint32_t*>(scratch + kOffOffs);
  int* d_pos = reinterpret_cast<int*>(scratch + kOffPos);
  int* d_start = reinterpret_cast<int*>(scratch + kOffStart);
  int* d_len = reinterpret_cast<int*>(scratch + kOffLen);
  int2* d_tiles = reinterpret_cast<int2*>(scratch + kOffTiles);

  cudaStream_t st = (cudaStream_t)stream;
  SeqOffsets po;
  for (uint32_t s = 0; s <= ns; s++) po.v[s] = ho[s];
  const bool fast = mode == TS_MODE_FAST;
  noalloc_prep_kernel<<<1, 1024, 0, st>>>(po, ns, rows, d_offs, d_tiles);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = ts::launch_seq_info(d_offs, ns, T, d_pos, d_start, d_len, st);
  if (e != cudaSuccess) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
  ts::AttnArgs a;
  a.q = d_q; a.k = d_k; a.v = d_v; a.sinks = d_sinks; a.mask = d_mask; a.out = d_out;
  a.sstart = d_start; a.slen = d_len; a.T = T; a.Hq = Hq; a.Hkv = Hkv; a.hd = head_dim; a.window = window;
  a.tiles = d_tiles;  // both kernels work on the tile list
  a.n_tiles = ntl;
  e = fast ? ts::launch_attention_tc(a, st) : ts::launch_attention_exact(a, st);
  if (e != cudaSuccess) return noalloc_fail(TS_ERR_CUDA, cudaGetErrorString(e));
  return TS_OK;
}
