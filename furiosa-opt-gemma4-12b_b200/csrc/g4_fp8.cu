// FP8 attention projections of one decode token on the tensor cores, weights straight
// from HBM into MMA fragments (no conversion, no shared-memory staging):
//   project_qkv        (src/ops.rs:44-124): input RMSNorm -> Q/K/V rows -> per-head
//                      RMSNorm, RoPE, q_out and the K/V cache rows (the head epilogue of
//                      the reference's sliding/full rmsnorm + rope, src/device/*/).
//   attention_output   (src/ops.rs:138-211): [x / running_sum] -> o-proj rows -> RMSNorm
//                      -> + residual, in place.
// Each output row is bf16(dot(x, e4m3 codes) * row scale), as the reference's
// scaled_projection (scripts/generate_references.py:312-321).
//
// Activation pieces.  x (bf16 after the norm) is scaled by 2^e so that max|x| lands in
// [128, 256) and written as three E4M3 pieces p1 = e4m3(xs), p2 = e4m3(xs - p1),
// p3 = e4m3(xs - p1 - p2) (each residual exact in f32): together 12+ significant bits, so
// every bf16 element within 2^-6 of the maximum is represented exactly and smaller ones
// to within 2^-18 of the maximum.  The pieces are the MMA's B columns 0..2
// (mma.sync m16n8k32 e4m3 x e4m3 -> f32; E4M3 x E4M3 products are exact), the E4M3
// weight codes the A operand as loaded: one 16-byte load per lane covers 16 k of a row,
// and the k order inside each 64-k block is permuted the same way for A and B so every
// fragment register comes from one load.  The three columns are added and scaled by 2^-e.
//
// Work split.  Items are (16-row tile, K part); CTAs (one per SM) take contiguous item
// ranges, their 8 warps items in turn; a warp loads all of an item's weights before any
// arithmetic (the first item before waiting for the previous kernel).  Each item writes
// its 16 partial row sums; the warp completing a head's last item runs that head's
// epilogue (project_qkv), the last CTA the norm/residual tail (attention_output).  The
// order of every sum is fixed, so results are deterministic.
#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {
namespace fp8 {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxMats = 3;

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
  int nmat, R, P;          // matrices, total rows, K parts per tile
  float* part;             // [P][R] partial row sums
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

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += red[w];
  return s;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s = fmaxf(s, red[w]);
  return s;
}

// x -> (norm | division) -> bf16 -> three E4M3 pieces of x * 2^e in shared memory
// (row stride kp bytes); returns e.  K <= 8192: at most 4 groups of 8 per thread.
__device__ int stage_pieces(const Args& a, uint8_t* pieces, int kp, float* red) {
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
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (a.in_w != nullptr) w = *reinterpret_cast<const uint4*>(a.in_w + gi * 8);
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
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gi = tid + j * kThreads;
    if (gi < ng) {
      uint32_t p[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float rem = ldexpf(v[j][i], e);
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const uint32_t c = e4m3_code(rem);
          rem = __fsub_rn(rem, e4m3_value(c));
          p[k][i >> 2] |= c << (8 * (i & 3));
        }
      }
#pragma unroll
      for (int k = 0; k < 3; ++k)
        *reinterpret_cast<uint2*>(pieces + k * kp + gi * 8) = make_uint2(p[k][0], p[k][1]);
    }
  }
  __syncthreads();
  return e;
}

// Norm + RoPE + store of one head (lane l owns elements l + 32j).
__device__ void head_epilogue(const Args& a, int head, int lane) {
  constexpr int kMaxJ = 16;
  const int J = a.D / 32;
  float raw[kMaxJ];
  const int row0 = head * a.D;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxJ; ++j) {
    if (j < J) {
      const int row = row0 + lane + 32 * j;
      float acc = 0.f;
      for (int p = 0; p < a.P; ++p) acc += __ldcg(a.part + static_cast<size_t>(p) * a.R + row);
      raw[j] = round_bf16(acc * row_scale(a, row));
      ss = __fadd_rn(ss, __fmul_rn(raw[j], raw[j]));
    }
  }
  const float r = rms_factor(warp_sum(ss), a.D);
  const bool is_q = head < a.nq;
  const bool is_k = !is_q && head < a.nq + a.nk;
  const int roff = __ldg(a.rope_off) / 2;
  const int koff = __ldg(a.kv_off) / 2;
  if (roff < 0 || static_cast<long long>(roff) + a.D > a.table_elems || koff < 0 ||
      static_cast<long long>(koff) + static_cast<long long>(a.nv > 0 ? a.nk : 1) * a.D > a.cache_elems) {
    if (lane == 0) atomicOr(&a.scr->status, DEV_ERR_BAD_OFFSET);
    return;
  }
  if (is_k && a.nv == 0) {  // full (MQA) layer: V is the unweighted norm of the raw K head
    for (int j = 0; j < J; ++j) a.vc[koff + lane + 32 * j] = f32_to_bf16(__fmul_rn(raw[j], r));
  }
  if (!is_q && !is_k) {     // sliding V head: unweighted norm, no RoPE
    const int vh = head - a.nq - a.nk;
    for (int j = 0; j < J; ++j) a.vc[koff + vh * a.D + lane + 32 * j] = f32_to_bf16(__fmul_rn(raw[j], r));
    return;
  }
  const uint16_t* nw = is_q ? a.qn_w : a.kn_w;
  float n[kMaxJ];
#pragma unroll
  for (int j = 0; j < kMaxJ; ++j)
    if (j < J) n[j] = round_bf16(__fmul_rn(__fmul_rn(raw[j], r), bf16_to_f32(nw[lane + 32 * j])));
  const int half = J / 2;
#pragma unroll
  for (int j = 0; j < kMaxJ; ++j) {
    if (j < J) {
      const int i = lane + 32 * j;
      const int pj = (j < half) ? j + half : j - half;
      float partner = 0.f;
#pragma unroll
      for (int q = 0; q < kMaxJ; ++q)
        if (q == pj) partner = n[q];
      const float c = bf16_to_f32(a.cosT[roff + i]);
      const float s = bf16_to_f32(a.sinT[roff + i]);
      const float o = round_bf16(__fadd_rn(round_bf16(__fmul_rn(n[j], c)), round_bf16(__fmul_rn(partner, s))));
      if (is_q)
        a.q_out[head * a.D + i] = f32_to_bf16(o);
      else
        a.kc[koff + (head - a.nq) * a.D + i] = f32_to_bf16(o);
    }
  }
}

// attention_output tail (one CTA): y = bf16(sum * row scale), RMSNorm, residual add.
__device__ void oproj_tail(const Args& a, float* red) {
  constexpr int kPer = (H + kThreads - 1) / kThreads;
  float y[kPer];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int row = threadIdx.x + j * kThreads;
    y[j] = 0.f;
    if (row < H) {
      float acc = 0.f;
      for (int p = 0; p < a.P; ++p) acc += __ldcg(a.part + static_cast<size_t>(p) * a.R + row);
      y[j] = round_bf16(acc * bf16_to_f32(a.m[0].scale[row]));
      ss = __fadd_rn(ss, __fmul_rn(y[j], y[j]));
    }
  }
  const float r = rms_factor(block_sum(ss, red), H);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int row = threadIdx.x + j * kThreads;
    if (row < H) {
      const float nb = round_bf16(__fmul_rn(__fmul_rn(y[j], r), bf16_to_f32(a.post_w[row])));
      a.residual[row] = f32_to_bf16(__fadd_rn(bf16_to_f32(a.residual[row]), nb));
    }
  }
}

template <int BPP>
__global__ void __launch_bounds__(kThreads, 1) fp8_gemv_kernel(const Args a) {
  extern __shared__ __align__(16) uint8_t fp8_pieces[];
  __shared__ float red[kWarps];
  __shared__ int s_done, s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int kp = a.K + 16;  // piece row stride: the three rows start in different banks
  const int N = (a.R / 16) * a.P;
  const int i0 = static_cast<int>(static_cast<long long>(blockIdx.x) * N / gridDim.x);
  const int i1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * N / gridDim.x);
  if (tid == 0) s_done = 0;
  uint4 wa[BPP], wb[BPP];
  const uint64_t pol = l2_evict_first_policy();
  auto load_item = [&](int it) {
    const int tile = it / a.P, p = it % a.P;
    int mi;
    const uint8_t* ra = row_ptr(a, tile * 16 + g, mi) + p * BPP * 64 + 16 * t;
    const uint8_t* rb = row_ptr(a, tile * 16 + g + 8, mi) + p * BPP * 64 + 16 * t;
#pragma unroll
    for (int b = 0; b < BPP; ++b) {
      wa[b] = ld_stream(ra + 64 * b, pol);
      wb[b] = ld_stream(rb + 64 * b, pol);
    }
  };
  int item = i0 + warp;
  if (item < i1) load_item(item);  // weights are never written by an earlier kernel
  pdl_wait();
  const int e = stage_pieces(a, fp8_pieces, kp, red);
  const float unscale = ldexpf(1.0f, -e);
  while (item < i1) {
    const int tile = item / a.P, p = item % a.P;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint8_t* pc = fp8_pieces + g * kp + p * BPP * 64 + 16 * t;
#pragma unroll
    for (int b = 0; b < BPP; ++b) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        uint2 bv = make_uint2(0u, 0u);
        if (g < 3) bv = *reinterpret_cast<const uint2*>(pc + 64 * b + 8 * m);
        if (m == 0)
          mma_e4m3(d, wa[b].x, wb[b].x, wa[b].y, wb[b].y, bv.x, bv.y);
        else
          mma_e4m3(d, wa[b].z, wb[b].z, wa[b].w, wb[b].w, bv.x, bv.y);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += d[i];
    }
    // columns 0..2 are the pieces: the quad's lanes 0 (cols 0,1) and 1 (col 2)
    float lo = (t == 0) ? acc[0] + acc[1] : (t == 1 ? acc[0] : 0.f);
    float hi = (t == 0) ? acc[2] + acc[3] : (t == 1 ? acc[2] : 0.f);
    lo += __shfl_xor_sync(0xffffffffu, lo, 1);
    hi += __shfl_xor_sync(0xffffffffu, hi, 1);
    if (t == 0) {
      float* dst = a.part + static_cast<size_t>(p) * a.R + tile * 16 + g;
      dst[0] = lo * unscale;
      dst[8] = hi * unscale;
    }
    const int next = item + kWarps;
    if (next < i1) load_item(next);
    else pdl_launch_dependents();
    if (a.qkv) {
      __syncwarp();
      const int head = tile * 16 / a.D;
      uint32_t old = 0;
      if (lane == 0) {
        __threadfence();
        old = atom_add_acq_rel_gpu(&a.scr->head_count[head], 1u);
      }
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old + 1 == static_cast<uint32_t>(a.D / 16 * a.P)) {
        __threadfence();
        head_epilogue(a, head, lane);
        if (lane == 0) a.scr->head_count[head] = 0u;
      }
    }
    item = next;
  }
  if (a.qkv) return;
  // attention_output: the last CTA to finish runs the tail
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atom_add_acq_rel_gpu(&a.scr->proj_done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  oproj_tail(a, red);
  if (tid == 0) a.scr->proj_done = 0u;
}

}  // namespace fp8

static g4_status launch_fp8(g4_ctx* ctx, fp8::Args& a, int bpp) {
  a.scr = ctx->buf.scratch;
  a.part = ctx->buf.part;
  if (static_cast<size_t>(a.P) * a.R > kPartFloats)
    return fail(ctx, G4_ERR_UNSUPPORTED, "fp8 projection: partial sums exceed the scratch");
  const size_t smem = 3 * static_cast<size_t>(a.K + 16);
  const void* fn = bpp == 15 ? (const void*)fp8::fp8_gemv_kernel<15> : (const void*)fp8::fp8_gemv_kernel<16>;
  void* args[] = {(void*)&a};
  return launch_kernel(ctx, fn, dim3(ctx->sm_count), dim3(fp8::kThreads), smem, args, false, "fp8 projection");
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
  a.nq = full ? GF : NS * GS;
  a.nk = full ? 1 : NS;
  a.nv = full ? 0 : NS;
  a.nmat = full ? 2 : 3;
  const int rows[3] = {a.nq * a.D, a.nk * a.D, a.nv * a.D};
  for (int i = 0; i < a.nmat; ++i) a.m[i] = fp8::Mat{w[i], rs[i], rows[i]};
  a.R = rows[0] + rows[1] + rows[2];
  a.P = 4;  // 4 parts of 960 k = 15 blocks
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
                                  : (full ? static_cast<long long>(TF) * DF : static_cast<long long>(TS) * NS * DS);
  a.q_out = q_out;
  return launch_fp8(ctx, a, 15);
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
  a.P = a.K / 1024;  // parts of 16 blocks
  a.qkv = 0;
  a.post_w = post_w;
  a.residual = residual;
  return launch_fp8(ctx, a, 16);
}

}  // namespace g4
