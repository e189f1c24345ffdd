// Decode attention (one query token), split-KV ("flash decoding") on the CUDA cores in
// f32: scores, exp and the weighted value sum match the reference's f32 softmax
// (scripts/generate_references.py:324-330, 436-455, 532-556).
//
//  sliding_attention            (src/ops.rs:126-136): GQA 2 q heads per kv head over the
//      1024-slot ring; one CTA per (kv head, 64-slot chunk); slots whose mask is 0 are
//      skipped (no K/V bytes read); the last chunk of a head merges the partials.
//  full_attention_first_page /  (src/ops.rs:160-186, src/device/full/attention.rs:200-334):
//  full_attention_page           one 512-row page per call, 8 chunks, the last chunk
//      merges them with the running max/sum/out state (unnormalised out, bf16).
//  full_attention_paged         every page of a layer in one cooperative launch: CTAs
//      take chunks, a bounded grid wait, then every CTA merges a slice of the 16x512
//      outputs (deterministic order), writing the normalised output.
#include <math_constants.h>

#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {

constexpr int kAttnThreads = 256;
constexpr int kChunk = 64;

// Row source of one chunk.
struct RowSrc {
  const uint16_t* k;   // row r: k + r * stride
  const uint16_t* v;
  long long stride;    // elements between rows
  const float* mask;   // row r valid iff mask[r] > 0 (nullptr: all rows valid up to nvalid)
  int nvalid;          // rows [0, nvalid) exist
};

// CTA-level: partial softmax statistics of NQ heads over up to kChunk rows.
// qs: [NQ][D] f32 in shared memory.  Writes m[NQ], l[NQ], o[NQ][D] to `out`.
template <int D, int NQ>
__device__ void attend_chunk(const float* __restrict__ qs, const RowSrc& src, float* __restrict__ out) {
  __shared__ float s[NQ][kChunk];
  __shared__ float mh[NQ], lh[NQ];
  __shared__ int valid[kChunk];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int EPL = D / 32;  // k elements per lane

  for (int r = tid; r < kChunk; r += kAttnThreads)
    valid[r] = (r < src.nvalid) && (src.mask == nullptr || src.mask[r] > 0.0f);
  __syncthreads();

  for (int r = warp; r < kChunk; r += kAttnThreads / 32) {
    if (!valid[r]) {
      if (lane < NQ) s[lane][r] = -CUDART_INF_F;
      continue;
    }
    const uint16_t* kr = src.k + r * src.stride + lane * EPL;
    float kv[EPL];
#pragma unroll
    for (int c = 0; c < EPL; c += 8) {
      const uint4 w = *reinterpret_cast<const uint4*>(kr + c);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kv[c + 2 * i] = bf16_to_f32(static_cast<uint16_t>(ww[i] & 0xFFFFu));
        kv[c + 2 * i + 1] = bf16_to_f32(static_cast<uint16_t>(ww[i] >> 16));
      }
    }
#pragma unroll
    for (int h = 0; h < NQ; ++h) {
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) d = fmaf(qs[h * D + lane * EPL + i], kv[i], d);
      d = warp_sum(d);
      if (lane == 0) s[h][r] = d;
    }
  }
  __syncthreads();
  for (int h = warp; h < NQ; h += kAttnThreads / 32) {
    float m = -CUDART_INF_F;
    for (int r = lane; r < kChunk; r += 32) m = fmaxf(m, s[h][r]);
    m = warp_max(m);
    float l = 0.f;
    for (int r = lane; r < kChunk; r += 32) {
      const float e = valid[r] ? expf(s[h][r] - m) : 0.f;
      s[h][r] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      mh[h] = m;
      lh[h] = l;
    }
  }
  __syncthreads();
  constexpr int DPT = D / kAttnThreads;  // value dims per thread
  float acc[NQ][DPT];
#pragma unroll
  for (int h = 0; h < NQ; ++h)
#pragma unroll
    for (int i = 0; i < DPT; ++i) acc[h][i] = 0.f;
  for (int r = 0; r < kChunk; ++r) {
    if (!valid[r]) continue;
    const uint16_t* vr = src.v + r * src.stride + tid * DPT;
    float vv[DPT];
    if constexpr (DPT == 2) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(vr);
      vv[0] = bf16_to_f32(static_cast<uint16_t>(w & 0xFFFFu));
      vv[1] = bf16_to_f32(static_cast<uint16_t>(w >> 16));
    } else {
#pragma unroll
      for (int i = 0; i < DPT; ++i) vv[i] = bf16_to_f32(vr[i]);
    }
#pragma unroll
    for (int h = 0; h < NQ; ++h) {
      const float e = s[h][r];
#pragma unroll
      for (int i = 0; i < DPT; ++i) acc[h][i] = fmaf(e, vv[i], acc[h][i]);
    }
  }
  // partial layout: [NQ] m, [NQ] l, [NQ][D] o
  if (tid < NQ) {
    out[tid] = mh[tid];
    out[NQ + tid] = lh[tid];
  }
#pragma unroll
  for (int h = 0; h < NQ; ++h)
#pragma unroll
    for (int i = 0; i < DPT; ++i) out[2 * NQ + h * D + tid * DPT + i] = acc[h][i];
}

// Merge of `nc` chunk partials for output (h, d) of a partial block array.
template <int D, int NQ>
__device__ __forceinline__ void merge_stats(const float* part, int nc, int h, float& M, float& Lsum) {
  constexpr int P = 2 * NQ + NQ * D;
  M = -CUDART_INF_F;
  for (int c = 0; c < nc; ++c) M = fmaxf(M, __ldcg(part + c * P + h));
  Lsum = 0.f;
  if (M == -CUDART_INF_F) return;
  for (int c = 0; c < nc; ++c) {
    const float m = __ldcg(part + c * P + h);
    if (m != -CUDART_INF_F) Lsum += __ldcg(part + c * P + NQ + h) * expf(m - M);
  }
}
template <int D, int NQ>
__device__ __forceinline__ float merge_out(const float* part, int nc, int h, int d, float M) {
  constexpr int P = 2 * NQ + NQ * D;
  float o = 0.f;
  if (M == -CUDART_INF_F) return 0.f;
  for (int c = 0; c < nc; ++c) {
    const float m = __ldcg(part + c * P + h);
    if (m != -CUDART_INF_F) o += __ldcg(part + c * P + 2 * NQ + h * D + d) * expf(m - M);
  }
  return o;
}

template <int D, int NQ>
__device__ __forceinline__ void load_q(const uint16_t* q, float* qs) {
  for (int i = threadIdx.x; i < NQ * D; i += kAttnThreads) qs[i] = bf16_to_f32(q[i]);
  __syncthreads();
}

// ---------------------------------------------------------------------------- sliding
__global__ void __launch_bounds__(kAttnThreads) sliding_attention_kernel(const uint16_t* __restrict__ q,
                                                                         const uint16_t* __restrict__ k,
                                                                         const uint16_t* __restrict__ v,
                                                                         const float* __restrict__ mask, int nkv,
                                                                         uint16_t* __restrict__ out, float* part,
                                                                         Scratch* scr) {
  constexpr int D = DS, NQ = GS, P = 2 * NQ + NQ * D;
  constexpr int S = TS / kChunk;
  __shared__ float qs[NQ * D];
  __shared__ int last;
  const int h = blockIdx.x / S, c = blockIdx.x % S;
  load_q<D, NQ>(q + h * NQ * D, qs);
  RowSrc src;
  src.k = k + (static_cast<long long>(c) * kChunk * nkv + h) * D;
  src.v = v + (static_cast<long long>(c) * kChunk * nkv + h) * D;
  src.stride = static_cast<long long>(nkv) * D;
  src.mask = mask + c * kChunk;
  src.nvalid = kChunk;
  float* mine = part + (h * S + c) * P;
  attend_chunk<D, NQ>(qs, src, mine);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = (atom_add_acq_rel_gpu(&scr->attn_count[h], 1u) == S - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* ph = part + h * S * P;
  for (int o = threadIdx.x; o < NQ * D; o += kAttnThreads) {
    const int hh = o / D, d = o % D;
    float M, Ls;
    merge_stats<D, NQ>(ph, S, hh, M, Ls);
    const float val = merge_out<D, NQ>(ph, S, hh, d, M);
    out[h * NQ * D + o] = f32_to_bf16(Ls > 0.f ? val / Ls : 0.f);
  }
  if (threadIdx.x == 0) scr->attn_count[h] = 0u;
}

// ---------------------------------------------------------------------------- per page
__global__ void __launch_bounds__(kAttnThreads) full_page_kernel(const uint16_t* __restrict__ q,
                                                                 const uint16_t* __restrict__ k,
                                                                 const uint16_t* __restrict__ v,
                                                                 const float* __restrict__ mask, int nq, int first,
                                                                 float* running_max, float* running_sum,
                                                                 uint16_t* out, float* part, Scratch* scr) {
  constexpr int D = DF, NQ = GF, P = 2 * NQ + NQ * D;
  constexpr int S = TF / kChunk;
  __shared__ float qs[NQ * D];
  __shared__ int last;
  const int c = blockIdx.x;
  for (int i = threadIdx.x; i < NQ * D; i += kAttnThreads) qs[i] = (i < nq * D) ? bf16_to_f32(q[i]) : 0.f;
  __syncthreads();
  RowSrc src;
  src.k = k + static_cast<long long>(c) * kChunk * D;
  src.v = v + static_cast<long long>(c) * kChunk * D;
  src.stride = D;
  src.mask = mask + c * kChunk;
  src.nvalid = kChunk;
  attend_chunk<D, NQ>(qs, src, part + c * P);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = (atom_add_acq_rel_gpu(&scr->attn_count[63], 1u) == S - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  __shared__ float Ln[NQ], resc[NQ];
  if (threadIdx.x < nq) {
    const int h = threadIdx.x;
    float M, Ls;
    merge_stats<D, NQ>(part, S, h, M, Ls);
    float Mo = first ? -CUDART_INF_F : running_max[h];
    const float Lo = first ? 0.f : running_sum[h];
    const float Mnew = fmaxf(M, Mo);
    const float ro = (Mo == -CUDART_INF_F) ? 0.f : expf(Mo - Mnew);
    const float rn = (M == -CUDART_INF_F) ? 0.f : expf(M - Mnew);
    resc[h] = ro;
    Ln[h] = rn;  // scale of this page's merged partials
    running_max[h] = Mnew;
    running_sum[h] = Lo * ro + Ls * rn;
  }
  __syncthreads();
  for (int o = threadIdx.x; o < nq * D; o += kAttnThreads) {
    const int h = o / D, d = o % D;
    float M, Ls;
    merge_stats<D, NQ>(part, S, h, M, Ls);
    const float val = merge_out<D, NQ>(part, S, h, d, M) * Ln[h];
    const float old = first ? 0.f : bf16_to_f32(out[o]) * resc[h];
    out[o] = f32_to_bf16(old + val);
  }
  if (threadIdx.x == 0) scr->attn_count[63] = 0u;
}

// ---------------------------------------------------------------------------- all pages
__global__ void __launch_bounds__(kAttnThreads) full_paged_kernel(const uint16_t* __restrict__ q,
                                                                  const uint16_t* const* __restrict__ k_pages,
                                                                  const uint16_t* const* __restrict__ v_pages,
                                                                  int n_pages, int last_row, int nq,
                                                                  float* running_sum, uint16_t* out, float* part,
                                                                  Scratch* scr, uint64_t budget_ns) {
  constexpr int D = DF, NQ = GF, P = 2 * NQ + NQ * D;
  constexpr int CPP = TF / kChunk;  // chunks per page
  __shared__ float qs[NQ * D];
  __shared__ int fail;
  const uint64_t deadline = global_ns() + budget_ns;
  for (int i = threadIdx.x; i < NQ * D; i += kAttnThreads) qs[i] = (i < nq * D) ? bf16_to_f32(q[i]) : 0.f;
  __syncthreads();
  const int nchunks = (n_pages - 1) * CPP + (last_row / kChunk) + 1;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int p = c / CPP, r0 = (c % CPP) * kChunk;
    RowSrc src;
    src.k = k_pages[p] + static_cast<long long>(r0) * D;
    src.v = v_pages[p] + static_cast<long long>(r0) * D;
    src.stride = D;
    src.mask = nullptr;
    src.nvalid = (p == n_pages - 1) ? min(kChunk, last_row + 1 - r0) : kChunk;
    attend_chunk<D, NQ>(qs, src, part + c * P);
    __syncthreads();
  }
  // bounded grid-wide wait
  if (threadIdx.x == 0) {
    __threadfence();
    atom_add_release_gpu(&scr->attn_done, 1u);
    uint32_t spins = 0;
    fail = 0;
    while (ld_acquire_gpu(&scr->attn_done) < gridDim.x) {
      if ((++spins & 63u) == 0u && global_ns() > deadline) {
        fail = 1;
        atomicOr(&scr->status, DEV_ERR_TIMEOUT_GRID);
        break;
      }
    }
  }
  __syncthreads();
  if (!fail) {
    __threadfence();
    for (int o = blockIdx.x * kAttnThreads + threadIdx.x; o < nq * D; o += gridDim.x * kAttnThreads) {
      const int h = o / D, d = o % D;
      float M, Ls;
      merge_stats<D, NQ>(part, nchunks, h, M, Ls);
      const float val = merge_out<D, NQ>(part, nchunks, h, d, M);
      out[o] = f32_to_bf16(Ls > 0.f ? val / Ls : 0.f);
      if (d == 0) running_sum[h] = 1.0f;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // the last CTA to leave resets both counters (every CTA has passed the wait)
    if (atom_add_acq_rel_gpu(&scr->attn_count[62], 1u) == gridDim.x - 1) {
      scr->attn_done = 0u;
      scr->attn_count[62] = 0u;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------- launchers
g4_status launch_sliding_attention(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                   const float* mask, uint16_t* out) {
  const int nkv = NS / ctx->tp_world;
  sliding_attention_kernel<<<nkv * (TS / kChunk), kAttnThreads, 0, ctx->stream>>>(q, k, v, mask, nkv, out,
                                                                                  ctx->buf.attn, ctx->buf.scratch);
  return check_cuda(ctx, cudaGetLastError(), "sliding_attention");
}

g4_status launch_full_page(g4_ctx* ctx, bool first, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                           const float* mask, float* rmax, float* rsum, uint16_t* out) {
  const int nq = GF / ctx->tp_world;
  full_page_kernel<<<TF / kChunk, kAttnThreads, 0, ctx->stream>>>(q, k, v, mask, nq, first ? 1 : 0, rmax, rsum, out,
                                                                  ctx->buf.attn, ctx->buf.scratch);
  return check_cuda(ctx, cudaGetLastError(), "full_attention_page");
}

g4_status launch_full_paged(g4_ctx* ctx, const uint16_t* q, const uint16_t* const* kp, const uint16_t* const* vp,
                            int n_pages, int last_row, float* rsum, uint16_t* out) {
  const int nq = GF / ctx->tp_world;
  const int nchunks = (n_pages - 1) * (TF / kChunk) + last_row / kChunk + 1;
  int grid = nchunks < ctx->sm_count ? nchunks : ctx->sm_count;
  uint64_t budget = ctx->wait_budget_ns;
  float* part = ctx->buf.attn;
  Scratch* scr = ctx->buf.scratch;
  void* args[] = {(void*)&q, (void*)&kp, (void*)&vp, (void*)&n_pages, (void*)&last_row, (void*)&nq,
                  (void*)&rsum, (void*)&out, (void*)&part, (void*)&scr, (void*)&budget};
  return check_cuda(ctx,
                    cudaLaunchCooperativeKernel((const void*)full_paged_kernel, dim3(grid), dim3(kAttnThreads), args,
                                                0, ctx->stream),
                    "full_attention_paged");
}

}  // namespace g4
