// FP8 attention projections of one decode token on the tensor cores:
//   project_qkv        (src/ops.rs:44-124): input RMSNorm -> Q/K/V rows -> per-head
//                      RMSNorm, RoPE, q_out and the K/V cache rows (the head epilogue of
//                      the reference's sliding/full rmsnorm + rope, src/device/*/).
//   attention_output   (src/ops.rs:138-211): [x / running_sum] -> o-proj rows -> RMSNorm
//                      -> + residual, in place.
// Each output row is bf16(dot(x, e4m3 codes) * row scale), as the reference's
// scaled_projection (scripts/generate_references.py:312-321).
//
// Weight stream.  Items are 16-row tiles (attention_output of a full layer: 16 rows x
// half of K), which the checkpoint stores contiguously: the producer warp moves each with
// ONE bulk copy (cp.async.bulk, L2 evict-first; 16 row copies for the half-K tiles) into a
// 3-stage shared-memory ring, starting before the kernel waits for the previous one
// (weights are never written by a kernel).  Large copies keep the copy engine's per-copy
// cost out of the way and about 190 KB per SM in flight.  Four consumer warps share an
// item, one K quarter each; the CTA's two warp groups take alternate items.
//
// Activation pieces.  x (bf16 after the norm) is scaled by 2^e so that max|x| lands in
// [128, 256) and written as three E4M3 pieces p1 = e4m3(xs), p2 = e4m3(xs - p1),
// p3 = e4m3(xs - p1 - p2) (each residual exact in f32): together 12+ significant bits, so
// every bf16 element within 2^-6 of the maximum is represented exactly and smaller ones
// to within 2^-18 of the maximum.  The pieces are the MMA's B columns 0..2
// (mma.sync m16n8k32 e4m3 x e4m3 -> f32; E4M3 x E4M3 products are exact) and the E4M3
// weight codes the A operand: one 16-byte shared-memory load per lane covers 16 k of a
// row, and the k order inside each 64-k block is permuted the same way for A and B so
// every fragment register comes from one load.  The three columns are added and scaled
// by 2^-e.
//
// Each item leaves its 16 partial row sums in global memory; project_qkv then runs one
// small kernel over the heads (norm, RoPE, stores).  attention_output adds an item's four
// K-quarter sums inside the CTA and stores one value per (row, K part); CTA 0 runs the
// norm/residual tail once every other CTA has counted itself done.  Every sum has a fixed
// order, so results are deterministic.
#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {
namespace fp8 {

constexpr int kThreads = 256;            // consumer threads (8 warps)
constexpr int kWarps = kThreads / 32;
constexpr int kAllThreads = kThreads + 32;  // + the producer warp
constexpr int kMaxMats = 3;
constexpr int kMaxStages = 8;
constexpr int kQuarters = 4;              // consumer warps per item (K quarters)
constexpr uint32_t kBarConsumers = 1;     // named barrier of the consumer warps
constexpr uint32_t kBarGroup0 = 2;        // named barriers 2, 3: the two consumer groups

struct Mat {
  const uint8_t* w;        // [rows, K] e4m3 codes
  const uint16_t* scale;   // [rows] bf16
  int rows;
};

struct Args {
  const uint16_t* x;
  int K;
  const uint16_t* in_w;    // project_qkv: input RMSNorm weight (nullptr: x used as is)
  const float* rsum;       // full attention_output: x / rsum[k / dh] first
  int dh;
  Mat m[kMaxMats];
  int nmat, R, P;          // matrices, total rows, K parts per tile (items per tile)
  float* part;             // [R][P * kQuarters] partial row sums (a row's parts contiguous)
  Scratch* scr;
  int qkv;                 // 1: project_qkv head epilogues, 0: attention_output tail
  int D, nq, nk, nv;
  const uint16_t *qn_w, *kn_w;
  const int32_t *kv_off, *rope_off;
  const uint16_t *cosT, *sinT;
  long long table_elems;
  uint16_t *kc, *vc;
  long long cache_elems;
  uint16_t* q_out;
  const uint16_t* post_w;
  uint16_t* residual;
  int kc_bytes;            // K bytes of one item per row
  int stages;
  uint64_t budget_ns;
};

__device__ __forceinline__ void mma_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// f32 -> E4M3 code (round to nearest even, saturating), one byte.
__device__ __forceinline__ uint32_t e4m3_code(float v) {
  uint16_t p;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(p) : "f"(0.0f), "f"(v));
  return (p & 0xFFu) | (p >> 8);  // one byte is the code of +0 (0x00), the other v's
}
// Streamed-once weights: no L1 allocation, evict-first in L2 (keeps activations and KV).
__device__ __forceinline__ uint4 ld_stream(const uint8_t* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ const uint8_t* row_ptr(const Args& a, int r, int& mi) {
  int base = 0;
#pragma unroll
  for (int i = 0; i < kMaxMats; ++i) {
    if (i < a.nmat && r < base + a.m[i].rows) {
      mi = i;
      return a.m[i].w + static_cast<size_t>(r - base) * a.K;
    }
    base += (i < a.nmat) ? a.m[i].rows : 0;
  }
  mi = 0;
  return a.m[0].w;
}
__device__ __forceinline__ float row_scale(const Args& a, int r) {
  int base = 0;
#pragma unroll
  for (int i = 0; i < kMaxMats; ++i) {
    if (i < a.nmat && r < base + a.m[i].rows) return bf16_to_f32(a.m[i].scale[r - base]);
    base += (i < a.nmat) ? a.m[i].rows : 0;
  }
  return 0.f;
}

__device__ __forceinline__ void consumer_sync() { named_bar_sync(kBarConsumers, kThreads); }
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  consumer_sync();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  consumer_sync();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += red[w];
  return s;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  consumer_sync();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  consumer_sync();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s = fmaxf(s, red[w]);
  return s;
}

// x -> (norm | division) -> bf16 -> three E4M3 pieces of x * 2^e in shared memory
// (row stride kp bytes); returns e.  K <= 8192: at most 4 groups of 8 per thread.
// The input norm's weights for stage_pieces, read before griddepcontrol.wait: no kernel
// writes them, and a load issued after the wait queues behind the weight stream this
// kernel's producer already started (2.5 us per launch, measured).
struct NormW {
  uint4 w[4];
};
__device__ __forceinline__ NormW load_norm_w(const Args& a) {
  NormW n;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gi = threadIdx.x + j * kThreads;
    n.w[j] = (a.in_w != nullptr && gi < a.K / 8) ? __ldg(reinterpret_cast<const uint4*>(a.in_w + gi * 8))
                                                 : make_uint4(0u, 0u, 0u, 0u);
  }
  return n;
}
// E4M3 code -> f32 with integer operations (the conversion pipe is the staging's
// bottleneck otherwise): normal codes assemble the f32 bits directly, subnormals
// ((m / 8) * 2^-6) as (1 + m / 8) * 2^-6 - 2^-6, exact.
__device__ __forceinline__ float e4m3_value_alu(uint32_t c) {
  const uint32_t sgn = (c & 0x80u) << 24, ex = (c >> 3) & 0xFu, m = c & 7u;
  if (ex != 0u) return __uint_as_float(sgn | ((ex + 120u) << 23) | (m << 20));
  const float f = __uint_as_float((121u << 23) | (m << 20)) - 0.015625f;
  return __uint_as_float(__float_as_uint(f) | sgn);
}

__device__ int stage_pieces(const Args& a, uint8_t* pieces, int kp, float* red, const NormW& nwr) {
  const int tid = threadIdx.x;
  const int ng = a.K / 8;
  float v[4][8];
  float ss = 0.f, amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gi = tid + j * kThreads;
    if (gi < ng) {
      const uint4 w = *reinterpret_cast<const uint4*>(a.x + gi * 8);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
      const float rs = (a.rsum != nullptr) ? a.rsum[gi * 8 / a.dh] : 1.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float f = bf16_to_f32(static_cast<uint16_t>((i & 1) ? ww[i >> 1] >> 16 : ww[i >> 1] & 0xFFFFu));
        if (a.rsum != nullptr) f = round_bf16(__fdiv_rn(f, rs));
        v[j][i] = f;
        ss = __fadd_rn(ss, __fmul_rn(f, f));
      }
    }
  }
  float r = 1.0f;
  if (a.in_w != nullptr) r = rms_factor(block_sum(ss, red), a.K);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gi = tid + j * kThreads;
    if (gi < ng) {
      const uint4 w = nwr.w[j];
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (a.in_w != nullptr) {
          const float nw = bf16_to_f32(static_cast<uint16_t>((i & 1) ? ww[i >> 1] >> 16 : ww[i >> 1] & 0xFFFFu));
          v[j][i] = round_bf16(__fmul_rn(__fmul_rn(v[j][i], r), nw));
        }
        amax = fmaxf(amax, fabsf(v[j][i]));
      }
    }
  }
  amax = block_max(amax, red);
  int ex = 0;
  if (amax > 0.f && isfinite(amax)) frexpf(amax, &ex);
  const int e = max(-100, min(100, 8 - ex));
  const float scale = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);  // 2^e, exact
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gi = tid + j * kThreads;
    if (gi < ng) {
      uint32_t p[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float rem = __fmul_rn(v[j][i], scale);  // v * 2^e: exact (no overflow, |v| <= max)
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const uint32_t c = e4m3_code(rem);
          rem = __fsub_rn(rem, e4m3_value_alu(c));
          p[k][i >> 2] |= c << (8 * (i & 3));
        }
      }
#pragma unroll
      for (int k = 0; k < 3; ++k)
        *reinterpret_cast<uint2*>(pieces + k * kp + gi * 8) = make_uint2(p[k][0], p[k][1]);
    }
  }
  consumer_sync();
  return e;
}

// project_qkv head epilogue, one CTA per head (thread i owns elements i and i + 256 of a
// 512-wide head): the row's K parts added in order, bf16(sum * row scale), the head's
// RMSNorm (q/k weighted, v unweighted; a full layer's V is the unweighted norm of the raw
// K head), RoPE with the partner element from shared memory, then q_out or the cache row
// at the device byte offset.  Launched right after the projection kernel (programmatic
// dependent launch); everything it reads from that kernel comes after the wait.
__global__ void __launch_bounds__(256) qkv_head_kernel(const __grid_constant__ Args a) {
  __shared__ float nsm[DF];
  __shared__ float red[kWarps];
  const int head = blockIdx.x, tid = threadIdx.x;
  // The attention kernel may start copying the cache rows this kernel does not write (it
  // waits for the one it does): in the decode step that overlap is worth more than the
  // head loads' extra queueing behind its copies (+0.9 % tokens/s measured).
  pdl_launch_dependents();
  const int E2 = a.D / 256;  // elements per thread (1 or 2)
  const bool is_q = head < a.nq;
  const bool is_k = !is_q && head < a.nq + a.nk;
  const uint16_t* nw = is_q ? a.qn_w : a.kn_w;
  const int row0 = head * a.D;
  // independent of the projection kernel: row scales, norm weights
  float rsc[2], nwf[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    rsc[e] = nwf[e] = 0.f;
    if (e < E2) {
      const int i = tid + 256 * e;
      rsc[e] = row_scale(a, row0 + i);
      if (is_q || is_k) nwf[e] = bf16_to_f32(nw[i]);
    }
  }
  pdl_wait();
  const int roff = a.rope_off[0] / 2;
  const int koff = a.kv_off[0] / 2;
  float4 pv[2];
  float cs[2] = {0.f, 0.f}, sn[2] = {0.f, 0.f};
  const bool ok = !(roff < 0 || static_cast<long long>(roff) + a.D > a.table_elems || koff < 0 ||
                    static_cast<long long>(koff) + static_cast<long long>(a.nv > 0 ? a.nk : 1) * a.D > a.cache_elems);
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    if (e < E2) {
      const int i = tid + 256 * e;
      pv[e] = __ldcg(reinterpret_cast<const float4*>(a.part) + row0 + i);
      if (ok && (is_q || is_k)) {
        cs[e] = bf16_to_f32(a.cosT[roff + i]);
        sn[e] = bf16_to_f32(a.sinT[roff + i]);
      }
    }
  }
  float raw[2], ss = 0.f;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    raw[e] = 0.f;
    if (e < E2) {
      raw[e] = round_bf16((((pv[e].x + pv[e].y) + pv[e].z) + pv[e].w) * rsc[e]);
      ss = __fadd_rn(ss, __fmul_rn(raw[e], raw[e]));
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) tot += red[w];
  const float r = rms_factor(tot, a.D);
  if (!ok) {
    if (tid == 0) atomicOr(&a.scr->status, DEV_ERR_BAD_OFFSET);
    return;
  }
  if (!is_q && !is_k) {  // sliding V head: unweighted norm, no RoPE
    const int vh = head - a.nq - a.nk;
#pragma unroll
    for (int e = 0; e < 2; ++e)
      if (e < E2) a.vc[koff + vh * a.D + tid + 256 * e] = f32_to_bf16(__fmul_rn(raw[e], r));
    return;
  }
  if (is_k && a.nv == 0) {  // full (MQA) layer: V is the unweighted norm of the raw K head
#pragma unroll
    for (int e = 0; e < 2; ++e)
      if (e < E2) a.vc[koff + tid + 256 * e] = f32_to_bf16(__fmul_rn(raw[e], r));
  }
  float n[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    n[e] = 0.f;
    if (e < E2) {
      n[e] = round_bf16(__fmul_rn(__fmul_rn(raw[e], r), nwf[e]));
      nsm[tid + 256 * e] = n[e];
    }
  }
  __syncthreads();
  const int half = a.D / 2;
  uint16_t* dst = is_q ? a.q_out + head * a.D : a.kc + koff + (head - a.nq) * a.D;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    if (e < E2) {
      const int i = tid + 256 * e;
      const float partner = nsm[i < half ? i + half : i - half];
      const float o = round_bf16(__fadd_rn(round_bf16(__fmul_rn(n[e], cs[e])), round_bf16(__fmul_rn(partner, sn[e]))));
      dst[i] = f32_to_bf16(o);
    }
  }
}

__device__ __forceinline__ uint4 lds128_at(uint32_t addr) { return lds128(addr); }

template <int BPP>
__global__ void __launch_bounds__(kAllThreads, 1) fp8_gemv_kernel(const __grid_constant__ Args a) {
  extern __shared__ __align__(128) uint8_t fp8_smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ float red[kWarps];
  __shared__ float qsum[kWarps / kQuarters][2][kQuarters][16];  // attention_output: quarter sums per item
  __shared__ int tail_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int kp = a.K + 16;                    // piece row stride: the three rows start in different banks
  uint8_t* pieces = fp8_smem;
  uint8_t* ring = fp8_smem + (3 * kp + 127) / 128 * 128;
  const uint32_t stage_bytes = 16u * static_cast<uint32_t>(a.kc_bytes);
  const int S = a.stages;
  const int N = (a.R / 16) * a.P;
  const int i0 = static_cast<int>(static_cast<long long>(blockIdx.x) * N / gridDim.x);
  const int i1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * N / gridDim.x);
  const int n_items = i1 - i0;
  const uint64_t deadline = global_ns() + a.budget_ns;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kQuarters);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // attention_output: the next kernel may take SMs as this grid's CTAs leave (before its
  // griddepcontrol.wait it only reads weights, which no kernel writes); project_qkv's head
  // kernel is launched as the items finish.
  if (!a.qkv) pdl_launch_dependents();

  if (warp == kWarps) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_items; ++j) {
        const int st = j % S;
        if (j >= S && !mbar_wait(&empty[st], ((j / S) - 1) & 1, deadline)) {
          atomicOr(&a.scr->status, DEV_ERR_TIMEOUT_MBAR);
          ok = false;
          break;
        }
        const int it = i0 + j, tile = it / a.P, p = it % a.P;
        uint8_t* dst = ring + st * stage_bytes;
        int mi;
        const uint8_t* src = row_ptr(a, tile * 16, mi) + static_cast<size_t>(p) * a.kc_bytes;
        mbar_arrive_expect_tx(&full[st], stage_bytes);
        if (a.P == 1) {  // 16 whole rows: one contiguous range
          bulk_g2s(dst, src, stage_bytes, &full[st], pol);
        } else {
          for (int r = 0; r < 16; ++r)
            bulk_g2s(dst + r * a.kc_bytes, src + static_cast<size_t>(r) * a.K, static_cast<uint32_t>(a.kc_bytes),
                     &full[st], pol);
        }
        issued = j + 1;
      }
      // every copy lands before the CTA may exit (the consumers wait for all in a normal run)
      if (!ok) {
        for (int j = (issued > S ? issued - S : 0); j < issued; ++j)
          if (!mbar_wait(&full[j % S], (j / S) & 1, deadline + a.budget_ns)) break;
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const NormW nwr = load_norm_w(a);
  pdl_wait();
  const int e = stage_pieces(a, pieces, kp, red, nwr);
  const float unscale = ldexpf(1.0f, -e);
  const int grp = warp / kQuarters, q = warp % kQuarters;
  const int qbytes = a.kc_bytes / kQuarters;  // = BPP * 64
  const int nparts = a.P * kQuarters;
  const uint32_t ring_s = smem_u32(ring);
  // A warp whose wait gave up keeps walking its items without touching the ring, so the
  // four warps of its group meet at every per-item barrier.
  bool ok = true;
  int jl = 0;  // the group's item count (parity selects the quarter-sum buffer)
  for (int j = grp; j < n_items; j += kWarps / kQuarters, ++jl) {
    const int st = j % S;
    if (ok && !mbar_wait(&full[st], (j / S) & 1, deadline)) {
      atomicOr(&a.scr->status, DEV_ERR_TIMEOUT_MBAR);
      ok = false;
    }
    const int it = i0 + j, tile = it / a.P, p = it % a.P;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      const uint32_t ra = ring_s + st * stage_bytes + g * a.kc_bytes + q * qbytes + 16 * t;
      const uint32_t rb = ra + 8 * a.kc_bytes;
      const uint8_t* pc = pieces + g * kp + p * a.kc_bytes + q * qbytes + 16 * t;
#pragma unroll
      for (int b = 0; b < BPP; ++b) {
        const uint4 wa = lds128(ra + 64 * b), wb = lds128(rb + 64 * b);
        uint2 bv0 = make_uint2(0u, 0u), bv1 = bv0;
        if (g < 3) {
          bv0 = *reinterpret_cast<const uint2*>(pc + 64 * b);
          bv1 = *reinterpret_cast<const uint2*>(pc + 64 * b + 8);
        }
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma_e4m3(d, wa.x, wb.x, wa.y, wb.y, bv0.x, bv0.y);
        mma_e4m3(d, wa.z, wb.z, wa.w, wb.w, bv1.x, bv1.y);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] += d[i];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // columns 0..2 are the pieces: the quad's lanes 0 (cols 0,1) and 1 (col 2)
    float lo = (t == 0) ? acc[0] + acc[1] : (t == 1 ? acc[0] : 0.f);
    float hi = (t == 0) ? acc[2] + acc[3] : (t == 1 ? acc[2] : 0.f);
    lo += __shfl_xor_sync(0xffffffffu, lo, 1);
    hi += __shfl_xor_sync(0xffffffffu, hi, 1);
    if (a.qkv) {
      // the head kernel adds a row's four quarter sums (one float4)
      if (t == 0) {
        float* dst = a.part + static_cast<size_t>(tile * 16 + g) * nparts + p * kQuarters + q;
        dst[0] = lo * unscale;
        dst[8 * nparts] = hi * unscale;
      }
    } else {
      // attention_output: the group adds its four quarter sums per row here, in quarter
      // order, and stores one value per (row, K part)
      float* qs = &qsum[grp][jl & 1][0][0];
      if (t == 0) {
        qs[q * 16 + g] = lo * unscale;
        qs[q * 16 + g + 8] = hi * unscale;
      }
      named_bar_sync(kBarGroup0 + grp, kQuarters * 32);
      if (q == 0 && lane < 16)
        a.part[static_cast<size_t>(tile * 16 + lane) * a.P + p] =
            ((qs[lane] + qs[16 + lane]) + qs[32 + lane]) + qs[48 + lane];
    }
  }
  if (a.qkv) {
    pdl_launch_dependents();
    return;
  }

  // attention_output tail in CTA 0, once every other CTA has published its row sums:
  // y = bf16(sum of the row's K parts * row scale), RMSNorm over the 3840 rows, residual
  // added in place.  Thread c < 240 owns rows [16c, 16c + 16).
  consumer_sync();
  if (blockIdx.x != 0) {
    if (tid == 0) {
      __threadfence();
      red_add_release_gpu(&a.scr->proj_done, 1u);
    }
    return;
  }
  constexpr int kTailRows = 16;
  const bool mine = tid < H / kTailRows;
  uint4 sv[2], wv[2], rv[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    sv[i] = wv[i] = rv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (mine) {  // not written by this grid: in flight while the other CTAs finish
      sv[i] = __ldg(reinterpret_cast<const uint4*>(a.m[0].scale) + 2 * tid + i);
      wv[i] = __ldg(reinterpret_cast<const uint4*>(a.post_w) + 2 * tid + i);
      rv[i] = *reinterpret_cast<const uint4*>(a.residual + kTailRows * tid + 8 * i);
    }
  }
  if (tid == 0) {
    uint32_t spins = 0;
    int fail = 0;
    while (ld_acquire_gpu(&a.scr->proj_done) < gridDim.x - 1u) {
      if ((++spins & 63u) == 0u && global_ns() > deadline) {
        fail = 1;
        atomicOr(&a.scr->status, DEV_ERR_TIMEOUT_GRID);
        break;
      }
    }
    tail_fail = fail;
  }
  consumer_sync();
  float y[kTailRows], ss = 0.f;
  if (mine) {
    // the thread's 16 rows x P parts are contiguous: every load in flight at once
    float ps[kTailRows * 4];
    const float4* pr = reinterpret_cast<const float4*>(a.part + static_cast<size_t>(tid) * kTailRows * a.P);
    if (a.P == 4) {
#pragma unroll
      for (int i = 0; i < kTailRows; ++i) {
        const float4 f = __ldcg(pr + i);
        ps[4 * i] = f.x, ps[4 * i + 1] = f.y, ps[4 * i + 2] = f.z, ps[4 * i + 3] = f.w;
      }
    } else {  // P == 2
#pragma unroll
      for (int i = 0; i < kTailRows / 2; ++i) {
        const float4 f = __ldcg(pr + i);
        ps[8 * i] = f.x, ps[8 * i + 1] = f.y, ps[8 * i + 4] = f.z, ps[8 * i + 5] = f.w;
      }
    }
    const uint32_t sw[8] = {sv[0].x, sv[0].y, sv[0].z, sv[0].w, sv[1].x, sv[1].y, sv[1].z, sv[1].w};
#pragma unroll
    for (int i = 0; i < kTailRows; ++i) {
      float acc = 0.f;  // the row's K parts in order
      acc += ps[4 * i];
      acc += ps[4 * i + 1];
      if (a.P == 4) {
        acc += ps[4 * i + 2];
        acc += ps[4 * i + 3];
      }
      const float sc = bf16_to_f32(static_cast<uint16_t>((i & 1) ? sw[i >> 1] >> 16 : sw[i >> 1] & 0xFFFFu));
      y[i] = round_bf16(acc * sc);
      ss = __fadd_rn(ss, __fmul_rn(y[i], y[i]));
    }
  }
  const float r = rms_factor(block_sum(ss, red), H);
  if (mine && !tail_fail) {
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const uint32_t rw[4] = {rv[h2].x, rv[h2].y, rv[h2].z, rv[h2].w};
      const uint32_t ww[4] = {wv[h2].x, wv[h2].y, wv[h2].z, wv[h2].w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint16_t hb[2];
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const float res = bf16_to_f32(static_cast<uint16_t>(jj ? rw[i] >> 16 : rw[i] & 0xFFFFu));
          const float pw = bf16_to_f32(static_cast<uint16_t>(jj ? ww[i] >> 16 : ww[i] & 0xFFFFu));
          const float nb = round_bf16(__fmul_rn(__fmul_rn(y[8 * h2 + 2 * i + jj], r), pw));
          hb[jj] = f32_to_bf16(__fadd_rn(res, nb));
        }
        o[i] = pack_u16x2(hb[0], hb[1]);
      }
      *reinterpret_cast<uint4*>(a.residual + kTailRows * tid + 8 * h2) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  consumer_sync();
  if (tid == 0) a.scr->proj_done = 0u;  // visible to the next launch at kernel end
}

}  // namespace fp8

static g4_status launch_fp8(g4_ctx* ctx, fp8::Args& a) {
  a.scr = ctx->buf.scratch;
  a.part = ctx->buf.part;
  a.budget_ns = ctx->wait_budget_ns;
  if (static_cast<size_t>(a.P) * fp8::kQuarters * a.R > kPartFloats)
    return fail(ctx, G4_ERR_UNSUPPORTED, "fp8 projection: partial sums exceed the scratch");
  a.kc_bytes = a.K / a.P;
  const int bpp = a.kc_bytes / fp8::kQuarters / 64;  // 64-k blocks per consumer warp and item
  const size_t pieces = (3 * static_cast<size_t>(a.K + 16) + 127) / 128 * 128;
  const size_t stage = 16 * static_cast<size_t>(a.kc_bytes);
  const size_t ring_budget = 200 * 1024 - pieces;
  a.stages = static_cast<int>(ring_budget / stage);
  if (a.stages > fp8::kMaxStages) a.stages = fp8::kMaxStages;
  if (a.stages < 2) return fail(ctx, G4_ERR_UNSUPPORTED, "fp8 projection: shared-memory ring too small");
  const size_t smem = pieces + stage * a.stages;
  const void* fn = bpp == 15 ? (const void*)fp8::fp8_gemv_kernel<15>
                 : bpp == 8  ? (const void*)fp8::fp8_gemv_kernel<8>
                             : nullptr;
  if (fn == nullptr || bpp * 64 * fp8::kQuarters != a.kc_bytes)
    return fail(ctx, G4_ERR_UNSUPPORTED, "fp8 projection: unsupported K split");
  g4_status st = allow_max_dynamic_smem(ctx, fn, smem, "fp8 projection");
  if (st != G4_OK) return st;
  void* args[] = {(void*)&a};
  st = launch_kernel(ctx, fn, dim3(ctx->sm_count), dim3(fp8::kAllThreads), smem, args, false, "fp8 projection");
  if (st != G4_OK) return st;
  if (a.qkv)
    return launch_kernel(ctx, (const void*)fp8::qkv_head_kernel, dim3(a.nq + a.nk + a.nv), dim3(256), 0, args, false,
                         "qkv heads");
  return G4_OK;  // attention_output: the tail ran in CTA 0
}

// project_qkv with FP8 weights on one GPU (the caller routes other cases elsewhere).
g4_status launch_qkv_fp8(g4_ctx* ctx, bool full, const uint16_t* x, const uint8_t* const w[3],
                         const uint16_t* const rs[3], const uint16_t* in_w, const uint16_t* qn_w,
                         const uint16_t* kn_w, const int32_t* kv_off, const int32_t* rope_off, const uint16_t* cosT,
                         const uint16_t* sinT, uint16_t* kcache, uint16_t* vcache, uint16_t* q_out,
                         long long cache_elems) {
  fp8::Args a = {};
  a.x = x;
  a.K = H;
  a.in_w = in_w;
  a.D = full ? DF : DS;
  const int tp = ctx->tp_world;  // tensor parallel: this rank's heads (the full layers' K head is replicated)
  a.nq = (full ? GF : NS * GS) / tp;
  a.nk = full ? 1 : NS / tp;
  a.nv = full ? 0 : NS / tp;
  a.nmat = full ? 2 : 3;
  const int rows[3] = {a.nq * a.D, a.nk * a.D, a.nv * a.D};
  for (int i = 0; i < a.nmat; ++i) a.m[i] = fp8::Mat{w[i], rs[i], rows[i]};
  a.R = rows[0] + rows[1] + rows[2];
  a.P = 1;  // whole 16-row tiles; 4 K quarters of 960 = 15 blocks (the head kernel reads a row's 4 parts as one float4)
  a.qkv = 1;
  a.qn_w = qn_w;
  a.kn_w = kn_w;
  a.kv_off = kv_off;
  a.rope_off = rope_off;
  a.cosT = cosT;
  a.sinT = sinT;
  a.table_elems = static_cast<long long>(E) * a.D;
  a.kc = kcache;
  a.vc = vcache;
  a.cache_elems = cache_elems > 0 ? cache_elems
                                  : (full ? static_cast<long long>(TF) * DF : static_cast<long long>(TS) * a.nk * DS);
  a.q_out = q_out;
  return launch_fp8(ctx, a);
}

// attention_output with FP8 weights on one GPU.
g4_status launch_oproj_fp8(g4_ctx* ctx, bool full, const uint16_t* x, const float* rsum, const uint16_t* post_w,
                           const uint8_t* w, const uint16_t* row_scale, uint16_t* residual) {
  fp8::Args a = {};
  a.x = x;
  a.K = full ? QF : QS;
  a.rsum = full ? rsum : nullptr;
  a.dh = DF;
  a.nmat = 1;
  a.m[0] = fp8::Mat{w, row_scale, H};
  a.R = H;
  a.P = a.K / 2048;  // items of 16 half rows (sliding) or quarter rows (full): quarters of 512 = 8 blocks
  a.qkv = 0;
  a.post_w = post_w;
  a.residual = residual;
  return launch_fp8(ctx, a);
}

}  // namespace g4
