// ts_common.cuh — shared device helpers for libtextsift_cuda.
//
// * fp16 <-> f32 conversions that follow textsift's WASM numerics bit for bit
//   (packages/textsift/src/zig/math.zig:45-82).  They are used wherever the
//   reference reads or writes an fp16 activation, bias, scale or table, so
//   that the CUDA kernels round at exactly the same points.
// * PTX wrappers for mbarriers, bulk/tensor copies and tcgen05 (sm_100a).
//   Every wait is bounded: after kWaitLimitNs of %globaltimer the waiting
//   thread records an error code in a device flag and gives up, so a
//   programming error can never hang the GPU.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ts {

// ---------------------------------------------------------------------------
// Reference fp16 conversions (math.zig)
// ---------------------------------------------------------------------------

// math.zig:45-52: sign<<16 | (rest ? (rest<<13) + (112<<23) : 0).  Subnormal
// and inf/NaN fp16 inputs decode to the same (non-IEEE) values as the WASM.
__device__ __forceinline__ float f16_ref_to_f32(uint16_t bits) {
  uint32_t u = bits;
  uint32_t sign = (u & 0x8000u) << 16;
  uint32_t rest = u & 0x7fffu;
  uint32_t biased = rest == 0 ? 0u : (rest << 13) + (112u << 23);
  return __uint_as_float(sign | biased);
}

// math.zig:54-82: RNE for normals, half-up for subnormals, NaN -> 0x7e00|s.
__device__ __forceinline__ uint16_t f32_to_f16_ref(float f) {
  uint32_t u = __float_as_uint(f);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t exp32 = (u >> 23) & 0xffu;
  uint32_t mant = u & 0x7fffffu;
  if (exp32 == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
  int e16 = (int)exp32 - 112;
  if (e16 >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (e16 <= 0) {
    if (e16 < -10) return (uint16_t)sign;
    uint32_t shift = (uint32_t)(14 - e16);
    uint32_t mant24 = mant | 0x800000u;
    return (uint16_t)(sign | ((mant24 + (1u << (shift - 1))) >> shift));
  }
  uint32_t lsb = (mant >> 13) & 1u;
  uint32_t m10 = (mant + 0xfffu + lsb) >> 13;
  uint32_t ue = (uint32_t)e16;
  if (m10 >= 0x400u) {
    m10 = 0;
    ue += 1;
    if (ue >= 0x1fu) return (uint16_t)(sign | 0x7c00u);
  }
  return (uint16_t)(sign | (ue << 10) | m10);
}

// Same result as f32_to_f16_ref for every input: hardware round-to-nearest-
// even is the reference's rounding for normal results, zero and overflow; the
// reference routine itself handles subnormal results (half-up) and NaN.
__device__ __forceinline__ uint16_t f32_to_f16_fast(float f) {
  const float a = fabsf(f);
  if (a >= 6.103515625e-05f && a < 65520.0f) return __half_as_ushort(__float2half_rn(f));
  return f32_to_f16_ref(f);
}

// The reference's RoPE on one interleaved (a, b) fp16 pair with its cos/sin
// table entries: three fp16 roundings per output (wasm_exports.zig:1488-1498).
__device__ __forceinline__ void rope_pair_ref(uint16_t& a16, uint16_t& b16, uint16_t c16, uint16_t s16) {
  const float c = f16_ref_to_f32(c16), s = f16_ref_to_f32(s16);
  const float a = f16_ref_to_f32(a16), b = f16_ref_to_f32(b16);
  const float ac = f16_ref_to_f32(f32_to_f16_fast(__fmul_rn(a, c)));
  const float bs = f16_ref_to_f32(f32_to_f16_fast(__fmul_rn(b, s)));
  const float bc = f16_ref_to_f32(f32_to_f16_fast(__fmul_rn(b, c)));
  const float as = f16_ref_to_f32(f32_to_f16_fast(__fmul_rn(a, s)));
  a16 = f32_to_f16_fast(__fsub_rn(ac, bs));
  b16 = f32_to_f16_fast(__fadd_rn(bc, as));
}

// The same RoPE on an fp16x2 word (a in the low half, b in the high half):
// (a c - b s, b c + a s) with every product and the sum rounded to fp16 by
// the half-precision unit (no contraction into fma).  Products of two fp16
// values and sums of two fp16 values are exact in f32 (or, for sums, too far
// from an fp16 tie to matter), so this equals rope_pair_ref bit for bit
// whenever no input, product or result is an fp16 subnormal; it differs from
// it only there (the reference decodes subnormals as if normal and rounds
// subnormal results half-up).
__device__ __forceinline__ uint32_t rope_h2(uint32_t ab, uint16_t c16, uint16_t s16) {
  const uint32_t cc = (uint32_t)c16 * 0x00010001u, ss = (uint32_t)s16 * 0x00010001u;
  const uint32_t ba = __byte_perm(ab, 0u, 0x1032);
  const __half2 x = __hmul2_rn(*reinterpret_cast<const __half2*>(&ab), *reinterpret_cast<const __half2*>(&cc));
  const __half2 y0 = __hmul2_rn(*reinterpret_cast<const __half2*>(&ba), *reinterpret_cast<const __half2*>(&ss));
  const uint32_t yn = *reinterpret_cast<const uint32_t*>(&y0) ^ 0x00008000u;  // (-b s, a s)
  const __half2 r = __hadd2_rn(x, *reinterpret_cast<const __half2*>(&yn));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Two f32 values as an fp16x2 word, hardware round-to-nearest-even (the
// tensor-core path's output conversion).
__device__ __forceinline__ uint32_t f32x2_to_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Exact fp16 -> f32 (IEEE, subnormals included): packages/textsift/src/
// browser/backends/wasm.ts:776-797 widens the final logits this way.
__device__ __forceinline__ float f16_ieee_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// The reference's exact exponential (Zig @exp on f32, a correctly rounded in
// practice expf) for the few entries that use it: the router softmax over k
// (wasm_exports.zig:919-958) and the 0-3 tail entries of each attention row
// (1354-1358).  Computed in double and rounded once to f32, which gives the
// correctly rounded result.
__device__ __forceinline__ float expf_ref(float x) { return (float)exp((double)x); }

// wasm_exports.zig:812-838, one lane: exp(x) for x <= 0 via 2^(x*log2 e),
// floor split, 5th-degree Horner polynomial (fused steps), exponent twiddle.
// This is the reference's own published approximation, restated.
__device__ __forceinline__ float exp_approx_ref(float x) {
  const float LOG2_E = 1.44269504088896340736f;
  float cl = x > -88.0f ? x : -88.0f;
  float y = __fmul_rn(cl, LOG2_E);
  // floor(y) and its integer without the conversion unit: adding 1.5 * 2^23
  // rounds y to the nearest integer in the low mantissa bits (|y| < 2^22),
  // one step down where that rounded up.  Same result as floorf and the int
  // conversions for every x < 60, NaN included (checked over all such
  // floats); callers pass x <= 0.
  const float t = __fadd_rn(y, 12582912.0f);
  float fl = __fsub_rn(t, 12582912.0f);
  int iv = __float_as_int(t) - 0x4B400000;
  if (fl > y) {
    fl = __fsub_rn(fl, 1.0f);
    iv -= 1;
  }
  float frac = __fsub_rn(y, fl);
  float p = __fmaf_rn(0.001333355f, frac, 0.009679494f);
  p = __fmaf_rn(p, frac, 0.055053319f);
  p = __fmaf_rn(p, frac, 0.240226522f);
  p = __fmaf_rn(p, frac, 0.693154774f);
  p = __fmaf_rn(p, frac, 1.000000012f);
  float scale = __uint_as_float((uint32_t)(iv + 127) << 23);
  return __fmul_rn(p, scale);
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// wasm_exports.zig:844-853
__device__ __forceinline__ float sigmoid_approx_ref(float x) {
  float mn = x < 0.0f ? x : 0.0f;
  float mx = x > 0.0f ? x : 0.0f;
  float e = exp_approx_ref(__fsub_rn(mn, mx));
  float sig_neg = __fdiv_rn(e, __fadd_rn(1.0f, e));
  return x >= 0.0f ? __fsub_rn(1.0f, sig_neg) : sig_neg;
}

// wasm_exports.zig:878-888 (one lane of the 4-lane body): gate<=7, up in
// [-7,7], (up+1) * gate * sigmoid(1.702*gate), every op rounded separately.
__device__ __forceinline__ float swiglu_ref(float g, float u) {
  float gate = g < 7.0f ? g : 7.0f;
  float up = u < 7.0f ? u : 7.0f;
  up = up > -7.0f ? up : -7.0f;
  float sig = sigmoid_approx_ref(__fmul_rn(gate, 1.702f));
  float glu = __fmul_rn(gate, sig);
  return __fmul_rn(__fadd_rn(up, 1.0f), glu);
}

// The same gate for the tensor-core path, whose output is rounded to fp16:
// the sigmoid is 1 / (1 + 2^(-1.702 log2(e) gate)) with the special-function
// unit's 2^x and reciprocal (a few ulp of f32, against the reference
// polynomial's 2.8e-4 relative error) — two SFU operations and a handful of
// FMA-pipe ones per output.
__device__ __forceinline__ float swiglu_fast(float g, float u) {
  const float gate = fminf(g, 7.0f);
  const float up = fmaxf(fminf(u, 7.0f), -7.0f);
  const float e = ex2_approx(gate * -2.45546696f);  // -1.702 * log2(e)
  const float sig = __fdividef(1.0f, 1.0f + e);
  return (up + 1.0f) * (gate * sig);
}

// Packed f32x2 arithmetic (sm_100): one instruction for two round-to-nearest
// f32 adds or multiplies, same results as two scalar ones.
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// Nibble j (0..3 = byte j) of lohi (lo = w & 0x0F0F0F0F or hi = (w >> 4) &
// 0x0F0F0F0F) placed in the mantissa of 2^23: the float 2^23 + nibble.  A
// packed add of -(2^23 + zp) then gives two weights q - zp exactly.
__device__ __forceinline__ float nib_raw(uint32_t lohi, uint32_t j) {
  return __uint_as_float(__byte_perm(lohi, 0x4B000000u, 0x7650u | j));
}
// max(a, b, c) in one instruction (sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// 2^x of both halves of an fp16x2 word on the special-function unit
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Two swiglu_fast evaluations with the adds and multiplies packed: results
// identical to swiglu_fast(g0, u0) and swiglu_fast(g1, u1).
__device__ __forceinline__ void swiglu_fast2(float g0, float u0, float g1, float u1, float& y0, float& y1) {
  const uint64_t gate = f2pack(fminf(g0, 7.0f), fminf(g1, 7.0f));
  const uint64_t up = f2pack(fmaxf(fminf(u0, 7.0f), -7.0f), fmaxf(fminf(u1, 7.0f), -7.0f));
  const uint64_t one = f2pack(1.0f, 1.0f);
  float t0, t1;
  f2unpack(mul_f32x2(gate, f2pack(-2.45546696f, -2.45546696f)), t0, t1);  // -1.702 * log2(e)
  float d0, d1;
  f2unpack(add_f32x2(f2pack(ex2_approx(t0), ex2_approx(t1)), one), d0, d1);
  const uint64_t gs = mul_f32x2(gate, f2pack(__fdividef(1.0f, d0), __fdividef(1.0f, d1)));
  f2unpack(mul_f32x2(add_f32x2(up, one), gs), y0, y1);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Kernels of the forward are launched with
// programmatic stream serialisation: the next grid may be scheduled once every
// block of the running one has called pdl_trigger(), and its blocks run their
// set-up until pdl_wait(), which returns when the previous grid has completed
// and its memory is visible.  Every such kernel calls pdl_trigger() and then
// pdl_wait() before its first access to global memory; launched without the
// attribute both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Raise a kernel's dynamic shared-memory limit once per device: function
// attributes belong to a device's context, so a process that drives several
// GPUs sets them on each.  Bit d of `done` records device d (devices past 63
// set the attribute on every call).
template <typename... KArgs>
inline cudaError_t smem_attr_per_device(void (*kernel)(KArgs...), int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
  if (bit && (done.load(std::memory_order_relaxed) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_relaxed);
  return e;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// Error flag shared by every kernel (bounded waits, bad indices)
// ---------------------------------------------------------------------------
enum DevErr : int {
  kDevErrNone = 0,
  kDevErrWaitTimeout = 1,
  kDevErrBadIndex = 2,
};

constexpr unsigned long long kWaitLimitNs = 4000000000ull;  // 4 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void set_dev_err(int* flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

// ---------------------------------------------------------------------------
// Shared-memory address / mbarrier helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a waiting thread sleeps (issuing nothing)
// until the phase completes or about kSuspendHintNs pass, so warps parked on a
// barrier leave the scheduler's issue slots to the warps sharing it.
#ifndef TS_SUSPEND_HINT_NS
#define TS_SUSPEND_HINT_NS 20000
#endif
constexpr uint32_t kSuspendHintNs = TS_SUSPEND_HINT_NS;

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (and records kDevErrWaitTimeout) if the phase
// did not complete within limit_ns (kWaitLimitNs in every kernel; a shorter
// limit only in the wait self-test, k_selftest.cu).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((++it & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      set_dev_err(err, kDevErrWaitTimeout);
      return false;
    }
  }
}

// Bounded wait that also gives up as soon as another role aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag,
                                              unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((++it & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        set_dev_err(err, kDevErrWaitTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared, completing on an mbarrier (tx bytes).
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled tensor copy global -> shared of this CTA.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int32_t c0, int32_t c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-gen tensor core, TMEM accumulators)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 x fp16 -> f32), 1 CTA.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// row (lane base + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 lanes x 1 column.
__device__ __forceinline__ void tmem_ld_32x32b_x1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Thread i of the warp writes row (lane base + i), columns [col, col+16) / [col, col+8).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem], kind::f16: A (M x 16 per instruction) is
// read from TMEM, row m in lane m, two fp16 of consecutive k per 32-bit column.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}


// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 128 B (64 fp16), 8-row atoms 1024 B apart.
// Fields (sm_100 UMMA descriptor): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version=1 [46,48), base offset [49,52), layout [61,64)
// with 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(16u >> 4) << 16;    // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;  // SBO: 8 rows x 128 B
  d |= (uint64_t)1 << 46;             // version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// Descriptor for an MN-major operand with the 128-byte swizzle whose MN
// extent is one 64-element atom: K rows of 128 B, 8-row groups 1024 B apart
// (SBO); LBO (the stride between MN atoms) is not used at this width.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(16u >> 4) << 16;    // LBO
  d |= (uint64_t)(1024u >> 4) << 32;  // SBO: 8 K-rows x 128 B
  d |= (uint64_t)1 << 46;             // version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D f32, A/B fp16, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(uint32_t M, uint32_t N) {
  return (1u << 4)            // D format: f32
         | (0u << 7)          // A format: f16
         | (0u << 10)         // B format: f16
         | ((N >> 3) << 17)   // N >> 3
         | ((M >> 4) << 24);  // M >> 4
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace ts
