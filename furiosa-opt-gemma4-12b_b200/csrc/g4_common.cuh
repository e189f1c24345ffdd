// Common device helpers for the g4b200 kernels (sm_100a only).
//
// Conversions, bf16 rounding, PTX wrappers for mbarriers / 1-D bulk copies / legacy
// warp MMA, and the bounded-wait helpers every spin in this library goes through.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "g4b200 is built for sm_100a only"
#endif

namespace g4 {

// ---------------------------------------------------------------- model constants
constexpr int H = 3840, L = 15360, W = 262144;
constexpr int NS = 8, GS = 2, DS = 256, QS = 4096, PS = 2048, TS = 1024;
constexpr int GF = 16, DF = 512, QF = 8192, PF = 512, TF = 512, E = 32768;
constexpr float EPS = 1e-6f;
constexpr float LOGIT_SOFTCAP = 30.0f;
constexpr float EMBED_SCALE = 61.967734f;

// Error flags a kernel can raise in the context's device status word.
enum : uint32_t {
  DEV_ERR_TIMEOUT_MBAR = 1u,      // an mbarrier wait ran out of budget
  DEV_ERR_TIMEOUT_GRID = 2u,      // a cross-CTA wait ran out of budget
  DEV_ERR_TIMEOUT_PEER = 4u,      // a cross-GPU wait ran out of budget
  DEV_ERR_BAD_OFFSET = 8u,        // a device-resident offset was out of range
};

// ---------------------------------------------------------------- bf16 / f16
__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
// Round-to-nearest-even f32 -> bf16 (same rounding as torch's .to(torch.bfloat16)).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
// bf16(f) as a float.
__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// x * 2^e as f16 bits: exact for every bf16 value whose scaled magnitude lies in
// the f16 normal range; the caller picks e from the vector's max magnitude.
__device__ __forceinline__ uint16_t f32_to_f16(float f) { return __half_as_ushort(__float2half_rn(f)); }

__device__ __forceinline__ uint32_t pack_u16x2(uint16_t lo, uint16_t hi) {
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// Power-of-two exponent e such that amax * 2^e lies in [2^14, 2^15): f16 operands of
// the MMA then keep every bf16 digit of every element within 2^28 of the maximum.
__device__ __forceinline__ int f16_scale_exponent(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 0;
  int ex;
  frexpf(amax, &ex);  // amax = m * 2^ex, m in [0.5, 1)
  int e = 15 - ex;
  return max(-100, min(100, e));
}

// ---------------------------------------------------------------- FP4 / FP8 decode
// Two E2M1 codes (one byte, low nibble = even element) -> f16x2 (low half = even).
__device__ __forceinline__ uint32_t cvt_e2m1x2(uint32_t byte_in_low8) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1;\n\t"
      "mov.b16 {b0, b1}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
      : "=r"(out)
      : "h"(static_cast<uint16_t>(byte_in_low8)));
  return out;
}
// Four E2M1 pairs of a 32-bit word -> four f16x2 (byte i -> out[i]).
__device__ __forceinline__ void cvt_e2m1x8(uint32_t w, uint32_t& o0, uint32_t& o1, uint32_t& o2,
                                           uint32_t& o3) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o0), "=r"(o1), "=r"(o2), "=r"(o3)
      : "r"(w));
}
// Two E4M3 bytes (low byte = first element) -> f16x2 (exact: E4M3 is a subset of f16).
__device__ __forceinline__ uint32_t cvt_e4m3x2(uint16_t two) {
  uint32_t out;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(two));
  return out;
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// (lo,hi) f16x2 -> (lo,lo) and (hi,hi).
__device__ __forceinline__ uint32_t dup_lo(uint32_t v) { return __byte_perm(v, 0, 0x1010); }
__device__ __forceinline__ uint32_t dup_hi(uint32_t v) { return __byte_perm(v, 0, 0x3232); }

// E2M1 magnitude table (scripts/generate_references.py:87), used by host-visible checks.
__device__ __forceinline__ float e2m1_value(uint32_t code) {
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  float v = mag[code & 7u];
  return (code & 8u) ? -v : v;
}
__device__ __forceinline__ float e4m3_value(uint32_t byte) {
  uint32_t h = cvt_e4m3x2(static_cast<uint16_t>(byte & 0xFFu));
  return __half2float(__ushort_as_half(static_cast<uint16_t>(h & 0xFFFFu)));
}

// ---------------------------------------------------------------- warp MMA (legacy)
// D(16x8,f32) += A(16x16,f16 row) * B(16x8,f16 col)
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- ldmatrix / cp.async
// Four 8x8 b16 matrices from shared memory (lanes 8i..8i+7 address the rows of matrix i).
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// 16-byte global -> shared copy; `src_bytes` 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most N of this thread's committed cp.async groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Two f32 -> packed bf16x2 (low half = a), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  return pack_u16x2(f32_to_bf16(a), f32_to_bf16(b));
}

// ---------------------------------------------------------------- shared memory I/O
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// ---------------------------------------------------------------- time / bounded waits
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Arrive only where `pred` holds, as a predicated instruction (no divergent branch).
__device__ __forceinline__ void mbar_arrive_if(uint64_t* bar, bool pred) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "@p mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n\t}" ::"r"(smem_u32(bar)),
      "r"(static_cast<uint32_t>(pred))
      : "memory");
}
// Shared-memory f32 store only where `pred` holds, as a predicated instruction.
__device__ __forceinline__ void sts_f32_if(uint32_t addr, float v, bool pred) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p st.shared.f32 [%0], %1;\n\t}" ::"r"(addr),
               "f"(v), "r"(static_cast<uint32_t>(pred))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for `parity` to complete; returns false (and leaves) once `deadline_ns` passes.
// Polls with the non-blocking test_wait and a short sleep, so a completed phase is seen
// within tens of nanoseconds instead of after a suspended thread's wake-up interval.
// Hardware-suspending wait (mbarrier.try_wait): frees the scheduler for other warps;
// used where a slightly later wake-up does not matter (the producer).
__device__ __forceinline__ bool mbar_wait_suspend(uint64_t* bar, uint32_t parity, uint64_t deadline_ns) {
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 63u) == 0u && global_ns() > deadline_ns) return false;
  }
  return true;
}
// `eager` waiters never sleep (a lone latency-critical warp).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline_ns,
                                          bool eager = false) {
  uint32_t spins = 0;
  while (!mbar_test_wait(bar, parity)) {
    ++spins;
    if (!eager && spins > 64) __nanosleep(20);
    if ((spins & 255u) == 0u && global_ns() > deadline_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------- 1-D bulk copy (TMA)
// L2 policy for streamed-once weights: evict first, keep activations / KV resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Global -> shared bulk copy completing on `bar` (src, dst 16-byte aligned; bytes % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------- named barriers
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// Let the next kernel on the stream start (its CTAs take SMs as ours exit).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Wait until the previous kernel on the stream has completed and its writes are visible
// (returns at once when the launch was not programmatic).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- global sync helpers
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Peer-exchange words: 16-byte accesses to memory that other GPUs read or write over
// NVLink, each 8-byte element single-copy atomic, coherent at system scope.
__device__ __forceinline__ void st_relaxed_sys_v2u64(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_v2u64(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Self-validating words exchanged between CTAs of one GPU: each carries its own tag, so
// a single-copy-atomic relaxed access needs no fence or flag (the reader re-reads a word
// until its tag is current).
__device__ __forceinline__ void st_relaxed_gpu_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_gpu_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_relaxed_gpu_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_relaxed_gpu_v4u32(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Release-ordered add whose result is not needed: no round trip to wait for.
__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Pull one 128-byte line into L2 and keep it there ahead of streamed (evict-first) data.
__device__ __forceinline__ void prefetch_l2_keep(const void* p) {
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}
__device__ __forceinline__ uint32_t atom_add_release_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

// ---------------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Oracle RMSNorm factor: torch.pow(mean(x^2) + eps, -0.5) == 1 / sqrt(.) with both
// steps correctly rounded (the CPU rsqrt kernel is div(1, sqrt(x))).
__device__ __forceinline__ float rms_factor(float sum_sq, int n) {
  float ms = __fdiv_rn(sum_sq, static_cast<float>(n));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, EPS)));
}

// gelu_pytorch_tanh in f32 (torch's CPU formula): 0.5*x*(1+tanh(sqrt(2/pi)*(x+0.044715 x^3))).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2/pi)
  const float kKappa = 0.044715f;
  float x3 = __fmul_rn(__fmul_rn(x, x), x);
  float inner = __fmul_rn(kBeta, __fadd_rn(x, __fmul_rn(kKappa, x3)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

}  // namespace g4
