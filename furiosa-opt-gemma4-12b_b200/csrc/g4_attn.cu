// Decode attention (one query token), split-KV ("flash decoding"), f32 softmax: scores,
// exp and the weighted value sum follow the reference's f32 softmax
// (scripts/generate_references.py:324-330, 436-455, 532-556).
//
//  sliding_attention            (src/ops.rs:126-136): GQA, 2 q heads per kv head over the
//      1024-slot ring, on the CUDA cores; one CTA per (kv head, 64-slot chunk), 16-byte
//      loads of every valid slot's K and V issued up front; slots whose mask is 0 are not
//      read; the last chunk of a head merges the partials.
//  full_attention_first_page /  (src/ops.rs:160-186, src/device/full/attention.rs:200-334):
//  full_attention_page           the reference's one-page-per-call API: 8 chunks per page,
//      the last chunk merges them into the running max/sum/out state (out unnormalised, bf16).
//  full_attention_paged / the decode workspace's full layers: every row of a layer in one
//      split-KV pass on the tensor cores (mma.sync, 16 q heads = the MMA's 16 rows), then a
//      merge kernel; the row count may live in device memory so CUDA-graph replays follow
//      the position.
#include <cuda.h>
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

// ---------------------------------------------------------------------------- sliding
// One CTA per (kv head, 64-slot chunk): warp w owns slots w*8..w*8+7 of the chunk, lane
// l dims 8l..8l+7.  Every K and V row of a valid slot is loaded with one 16-byte load per
// lane, all issued before any arithmetic; slots whose mask is 0 are not read.  Scores in
// f32 (products of bf16 values are exact), softmax with the chunk's max, then the last
// chunk of a head merges the 16 partials in chunk order.
constexpr int kSaThreads = 256;
constexpr int kSaRows = 64;
constexpr int kSaPart = 2 * GS + GS * DS;  // m[GS], l[GS], o[GS][DS]
constexpr int kMaxSaChunks = E / kSaRows;   // 512 chunks: a 32768-row cache

__device__ __forceinline__ void bf16x8_to_f32(const uint4 w, float (&f)[8]) {
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16_to_f32(static_cast<uint16_t>(ww[i] & 0xFFFFu));
    f[2 * i + 1] = bf16_to_f32(static_cast<uint16_t>(ww[i] >> 16));
  }
}

__global__ void __launch_bounds__(kSaThreads) sliding_attn_kernel(const uint16_t* q, const uint16_t* k,
                                                                  const uint16_t* v, const float* mask, int nkv,
                                                                  int nchunks, uint16_t* out, float* part,
                                                                  Scratch* scr) {
  __shared__ float s[GS][kSaRows];
  __shared__ __align__(16) float red[kSaThreads / 32][GS][DS];
  __shared__ float mh[GS], lh[GS];
  __shared__ int last;
  const int h = blockIdx.x / nchunks, c = blockIdx.x % nchunks;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();  // q, the caches and the mask come from earlier kernels
  const int rbase = c * kSaRows + warp * 8;
  // every row is loaded together with the mask (one round trip, not two); rows the mask
  // excludes are never used
  const float mv = lane < 8 ? mask[rbase + lane] : 0.f;
  const uint16_t* qh = q + static_cast<size_t>(h) * GS * DS + lane * 8;
  const uint4 q0 = *reinterpret_cast<const uint4*>(qh);
  const uint4 q1 = *reinterpret_cast<const uint4*>(qh + DS);
  uint4 kk[8], vv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const size_t off = (static_cast<size_t>(rbase + j) * nkv + h) * DS + lane * 8;
    kk[j] = *reinterpret_cast<const uint4*>(k + off);
    vv[j] = *reinterpret_cast<const uint4*>(v + off);
  }
  const uint32_t valid = __ballot_sync(0xffffffffu, mv > 0.f) & 0xFFu;
  pdl_launch_dependents();
  float qa[8], qb[8];
  bf16x8_to_f32(q0, qa);
  bf16x8_to_f32(q1, qb);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float kf[8];
    bf16x8_to_f32(kk[j], kf);
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      d0 = fmaf(qa[i], kf[i], d0);
      d1 = fmaf(qb[i], kf[i], d1);
    }
    d0 = warp_sum(d0);
    d1 = warp_sum(d1);
    if (lane == 0) {
      const bool ok = (valid >> j) & 1u;
      s[0][warp * 8 + j] = ok ? d0 : -CUDART_INF_F;
      s[1][warp * 8 + j] = ok ? d1 : -CUDART_INF_F;
    }
  }
  __syncthreads();
  if (warp < GS) {
    const float a = s[warp][lane], b = s[warp][lane + 32];
    const float m = warp_max(fmaxf(a, b));
    const float ea = (a == -CUDART_INF_F) ? 0.f : expf(a - m);
    const float eb = (b == -CUDART_INF_F) ? 0.f : expf(b - m);
    const float l = warp_sum(ea + eb);
    s[warp][lane] = ea;
    s[warp][lane + 32] = eb;
    if (lane == 0) {
      mh[warp] = m;
      lh[warp] = l;
    }
  }
  __syncthreads();
  float o0[8], o1[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o0[i] = o1[i] = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if ((valid >> j) & 1u) {
      float vf[8];
      bf16x8_to_f32(vv[j], vf);
      const float p0 = s[0][warp * 8 + j], p1 = s[1][warp * 8 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o0[i] = fmaf(p0, vf[i], o0[i]);
        o1[i] = fmaf(p1, vf[i], o1[i]);
      }
    }
  }
  float4* r0 = reinterpret_cast<float4*>(&red[warp][0][lane * 8]);
  float4* r1 = reinterpret_cast<float4*>(&red[warp][1][lane * 8]);
  r0[0] = make_float4(o0[0], o0[1], o0[2], o0[3]);
  r0[1] = make_float4(o0[4], o0[5], o0[6], o0[7]);
  r1[0] = make_float4(o1[0], o1[1], o1[2], o1[3]);
  r1[1] = make_float4(o1[4], o1[5], o1[6], o1[7]);
  __syncthreads();
  float* mine = part + static_cast<size_t>(h * nchunks + c) * kSaPart;
  for (int o = tid; o < GS * DS; o += kSaThreads) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kSaThreads / 32; ++w) acc += red[w][o / DS][o % DS];
    mine[2 * GS + o] = acc;
  }
  if (tid < GS) {
    mine[tid] = mh[tid];
    mine[GS + tid] = lh[tid];
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = (atom_add_acq_rel_gpu(&scr->attn_count[h], 1u) == static_cast<uint32_t>(nchunks) - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge: every chunk's (m, l) in one parallel load, the weights once per q head, then
  // each output's chunk values with independent loads
  __shared__ float wsm[GS][kMaxSaChunks];
  __shared__ float lsum[GS];
  const float* ph = part + static_cast<size_t>(h) * nchunks * kSaPart;
  for (int i = tid; i < GS * nchunks; i += kSaThreads) {
    const int cc = i / GS, hh = i % GS;
    wsm[hh][cc] = __ldcg(ph + cc * kSaPart + hh);
  }
  __syncthreads();
  if (warp < GS) {
    float M = -CUDART_INF_F;
    for (int cc = lane; cc < nchunks; cc += 32) M = fmaxf(M, wsm[warp][cc]);
    M = warp_max(M);
    float Ls = 0.f;
    for (int cc = lane; cc < nchunks; cc += 32) {
      const float m = wsm[warp][cc];
      const float w = (m == -CUDART_INF_F) ? 0.f : expf(m - M);
      Ls += w * __ldcg(ph + cc * kSaPart + GS + warp);
      wsm[warp][cc] = w;
    }
    Ls = warp_sum(Ls);
    if (lane == 0) lsum[warp] = Ls;
  }
  __syncthreads();
  for (int o = tid; o < GS * DS; o += kSaThreads) {
    const int hh = o / DS;
    float acc = 0.f;
#pragma unroll 8
    for (int cc = 0; cc < nchunks; ++cc) acc += wsm[hh][cc] * __ldcg(ph + cc * kSaPart + 2 * GS + o);
    const float Ls = lsum[hh];
    out[static_cast<size_t>(h) * GS * DS + o] = f32_to_bf16(Ls > 0.f ? acc / Ls : 0.f);
  }
  if (tid == 0) scr->attn_count[h] = 0u;
}

// ---------------------------------------------------------------------------- full (MQA)
// Split-KV over rows [0, n) of the single K/V head: the rows are cut into one contiguous
// range per CTA (a multiple of 8 rows), each range runs in tiles of 32 rows staged in
// shared memory with cp.async (16-byte chunks XOR-swizzled by row, so ldmatrix reads are
// conflict-free), S = Q K^T and O += P V on the tensor cores (mma.sync m16n8k16, bf16
// operands, f32 accumulators; the 16 q heads are the M = 16 rows), online softmax across
// the CTA's tiles.  P enters the MMA as bf16 hi + lo parts, so the weights keep ~16
// mantissa bits.  A second kernel (programmatic dependent launch: it waits for the first
// to complete) merges the per-CTA partials in CTA order and writes the normalised output.
constexpr int kFaThreads = 128;
constexpr int kFaTile = 32;
constexpr int kFaQStride = DF * 2 + 16;          // padded Q row in shared memory (bytes)
constexpr int kFaPart = 2 * GF + GF * DF;        // m[16], l[16], o[16][512]
constexpr int kFaMaxCtas = 512;

struct FaSmem {
  uint8_t k[2][kFaTile * DF * 2];  // two tiles: the next one loads while this one computes
  uint8_t v[2][kFaTile * DF * 2];
  uint8_t q[GF * kFaQStride];
  float s[GF][kFaTile + 1];
  float m[GF], l[GF], alpha[GF];
};

// Where the K/V rows live: a page table of [TF, DF] pages (the reference's page cache)
// or one contiguous [rows, DF] array (the decode workspace); the row count from the host
// or from a device int32 (graph replays), clamped to `max_rows` either way.
struct FaSrc {
  const uint16_t* const* k_pages;
  const uint16_t* const* v_pages;
  const uint16_t* k;
  const uint16_t* v;
  const int32_t* n_dev;
  int n_host;
  int max_rows;
};

__device__ __forceinline__ const uint16_t* fa_row(const FaSrc& s, bool is_v, int r) {
  if (s.k_pages != nullptr)
    return (is_v ? s.v_pages : s.k_pages)[r / TF] + static_cast<size_t>(r % TF) * DF;
  return (is_v ? s.v : s.k) + static_cast<size_t>(r) * DF;
}

// Rows, rows per CTA and active CTAs: the same on both kernels.
__device__ __forceinline__ void fa_split(const FaSrc& s, int grid, int& n, int& rpc, int& nact) {
  n = s.n_dev != nullptr ? *s.n_dev : s.n_host;
  n = max(0, min(n, s.max_rows));
  // at least two 32-row tiles per CTA: a partial (33 KB) costs about as much to write and
  // merge as 16 rows of K and V cost to read
  rpc = (n + grid - 1) / grid;
  rpc = max(64, (rpc + 31) & ~31);
  nact = (n + rpc - 1) / rpc;
}

__global__ void __launch_bounds__(kFaThreads) fa_partial_kernel(const uint16_t* q, int nq, FaSrc src,
                                                                float* part) {
  extern __shared__ __align__(128) uint8_t fa_raw[];
  FaSmem& sm = *reinterpret_cast<FaSmem*>(fa_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  // tile loads: rows [tr, tr + 32) below `lim` into buffer b, one cp.async group per tile
  auto load_tile_lim = [&](int tr, int b, int lim) {
    const uint32_t kbb = smem_u32(sm.k[b]), vbb = smem_u32(sm.v[b]);
    for (int i = tid; i < kFaTile * (DF / 8); i += kFaThreads) {
      const int rr = i / (DF / 8), c = i % (DF / 8);
      const int r = tr + rr;
      const bool ok = r < lim;
      const uint32_t off = rr * (DF * 2) + ((c ^ (rr & 7)) * 16);
      cp_async16(kbb + off, ok ? fa_row(src, false, r) + c * 8 : q, ok ? 16u : 0u);
      cp_async16(vbb + off, ok ? fa_row(src, true, r) + c * 8 : q, ok ? 16u : 0u);
    }
    cp_async_commit();
  };
  // When the grid covers max_rows in 64-row ranges (the launchers size it so), every row
  // count gives this CTA rows [64 c, 64 c + 64): both tiles are copied before the wait.
  // Rows below max_rows exist; all but the newest were written by kernels that completed
  // before this launch could start, and the newest (row n - 1, the projection's) is copied
  // again after the wait.
  const bool early = static_cast<long long>(gridDim.x) * 2 * kFaTile >= src.max_rows;
  if (early) {
    load_tile_lim(blockIdx.x * 2 * kFaTile, 0, src.max_rows);
    load_tile_lim(blockIdx.x * 2 * kFaTile + kFaTile, 1, src.max_rows);
  }
  pdl_wait();  // q and the newest K/V row come from the projection kernel
  int n, rpc, nact;
  fa_split(src, gridDim.x, n, rpc, nact);
  const int r0 = blockIdx.x * rpc, r1 = min(n, r0 + rpc);
  if (r0 >= r1) {
    cp_async_wait_all();  // no copy may still be landing in shared memory at exit
    pdl_launch_dependents();
    return;
  }
  const uint32_t qb = smem_u32(sm.q);
  for (int i = tid; i < GF * (DF / 8); i += kFaThreads) {
    const int hh = i / (DF / 8), c = i % (DF / 8);
    const bool ok = hh < nq;
    cp_async16(qb + hh * kFaQStride + c * 16, ok ? q + hh * DF + c * 8 : q, ok ? 16u : 0u);
  }
  auto load_tile = [&](int tr, int b) { load_tile_lim(tr, b, r1); };
  if (!early) {
    load_tile(r0, 0);
    if (r0 + kFaTile < r1) load_tile(r0 + kFaTile, 1);
  } else {
    cp_async_commit();  // q
    cp_async_wait_all();
    __syncthreads();  // every early copy landed: the rows below can be rewritten
    const int nr = n - 1 - r0;  // the newest row, when this CTA holds it
    const uint32_t zero_from = static_cast<uint32_t>(r1 - r0);  // rows >= n: V to zero (may be stale)
    for (int i = tid; i < 2 * kFaTile * (DF / 8); i += kFaThreads) {
      const int rr = i / (DF / 8), c = i % (DF / 8);
      const uint32_t off = (rr % kFaTile) * (DF * 2) + ((c ^ (rr & 7)) * 16);
      const int b = rr / kFaTile;
      if (rr == nr) {
        cp_async16(smem_u32(sm.k[b]) + off, fa_row(src, false, r0 + rr) + c * 8, 16u);
        cp_async16(smem_u32(sm.v[b]) + off, fa_row(src, true, r0 + rr) + c * 8, 16u);
      } else if (static_cast<uint32_t>(rr) >= zero_from) {
        *reinterpret_cast<uint4*>(sm.v[b] + off) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    cp_async_commit();
    cp_async_wait_all();
  }
  if (tid < GF) {
    sm.m[tid] = -CUDART_INF_F;
    sm.l[tid] = 0.f;
  }
  float acc[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

  pdl_launch_dependents();
  for (int tr = r0, ti = 0; tr < r1; tr += kFaTile, ++ti) {
    const uint32_t kb = smem_u32(sm.k[ti & 1]), vb = smem_u32(sm.v[ti & 1]);
    if (tr + kFaTile < r1)
      cp_async_wait_group<1>();  // this tile (and q) landed; the next may still fly
    else
      cp_async_wait_group<0>();
    __syncthreads();
    // S[16 heads][8 rows of this warp] = Q K^T over the 512 dims
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int j = 0; j < DF / 16; j += 2) {
      uint32_t b0, b1, b2, b3;
      {
        const int row = 8 * warp + (lane & 7), chunk = 2 * j + (lane >> 3);
        ldsm_x4(kb + row * (DF * 2) + ((chunk ^ (row & 7)) * 16), b0, b1, b2, b3);
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        uint32_t a0, a1, a2, a3;
        const int qrow = (lane & 7) + 8 * ((lane >> 3) & 1), qcol = (j + jj) * 16 + 8 * (lane >> 4);
        ldsm_x4(qb + qrow * kFaQStride + qcol * 2, a0, a1, a2, a3);
        mma_bf16(sc, a0, a1, a2, a3, jj ? b2 : b0, jj ? b3 : b1);
      }
    }
    {
      const int rr = 8 * warp + 2 * t;
      const bool v0 = tr + rr < r1, v1 = tr + rr + 1 < r1;
      sm.s[g][rr] = v0 ? sc[0] : -CUDART_INF_F;
      sm.s[g][rr + 1] = v1 ? sc[1] : -CUDART_INF_F;
      sm.s[g + 8][rr] = v0 ? sc[2] : -CUDART_INF_F;
      sm.s[g + 8][rr + 1] = v1 ? sc[3] : -CUDART_INF_F;
    }
    __syncthreads();
    // online softmax: warp w updates heads 4w..4w+3, lane = tile row
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
      const int h = 4 * warp + hh;
      const float sv = sm.s[h][lane];
      const float mold = sm.m[h];
      const float mnew = fmaxf(mold, warp_max(sv));
      const float p = (sv == -CUDART_INF_F) ? 0.f : expf(sv - mnew);
      const float ls = warp_sum(p);
      sm.s[h][lane] = p;
      if (lane == 0) {
        const float a = (mold == -CUDART_INF_F) ? 0.f : expf(mold - mnew);
        sm.alpha[h] = a;
        sm.l[h] = sm.l[h] * a + ls;
        sm.m[h] = mnew;
      }
    }
    __syncthreads();
    // O[16 heads][128 dims of this warp] = O * alpha + P V
    const float al = sm.alpha[g], ah = sm.alpha[g + 8];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      acc[nt][0] *= al;
      acc[nt][1] *= al;
      acc[nt][2] *= ah;
      acc[nt][3] *= ah;
    }
#pragma unroll
    for (int j = 0; j < kFaTile / 16; ++j) {
      const int c0 = 16 * j + 2 * t;
      const float p[8] = {sm.s[g][c0], sm.s[g][c0 + 1], sm.s[g + 8][c0], sm.s[g + 8][c0 + 1],
                          sm.s[g][c0 + 8], sm.s[g][c0 + 9], sm.s[g + 8][c0 + 8], sm.s[g + 8][c0 + 9]};
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x0 = round_bf16(p[2 * i]), x1 = round_bf16(p[2 * i + 1]);
        hi[i] = pack_bf16x2(x0, x1);
        lo[i] = pack_bf16x2(p[2 * i] - x0, p[2 * i + 1] - x1);
      }
#pragma unroll
      for (int nt = 0; nt < 16; nt += 2) {
        uint32_t b0, b1, b2, b3;
        const int vrow = 16 * j + (lane & 7) + 8 * ((lane >> 3) & 1), chunk = 16 * warp + nt + (lane >> 4);
        ldsm_x4_trans(vb + vrow * (DF * 2) + ((chunk ^ (vrow & 7)) * 16), b0, b1, b2, b3);
        mma_bf16(acc[nt], hi[0], hi[1], hi[2], hi[3], b0, b1);
        mma_bf16(acc[nt], lo[0], lo[1], lo[2], lo[3], b0, b1);
        mma_bf16(acc[nt + 1], hi[0], hi[1], hi[2], hi[3], b2, b3);
        mma_bf16(acc[nt + 1], lo[0], lo[1], lo[2], lo[3], b2, b3);
      }
    }
    __syncthreads();  // buffer ti & 1 and S are free again
    if (tr + 2 * kFaTile < r1) load_tile(tr + 2 * kFaTile, ti & 1);
  }
  float* mine = part + static_cast<size_t>(blockIdx.x) * kFaPart;
  if (tid < GF) {
    mine[tid] = sm.m[tid];
    mine[GF + tid] = sm.l[tid];
  }
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = 128 * warp + 8 * nt + 2 * t;
    *reinterpret_cast<float2*>(mine + 2 * GF + g * DF + d) = make_float2(acc[nt][0], acc[nt][1]);
    *reinterpret_cast<float2*>(mine + 2 * GF + (g + 8) * DF + d) = make_float2(acc[nt][2], acc[nt][3]);
  }
}

// Four CTAs per head, 128 dims each: the active partials' (m, l) in one parallel load,
// their weights once; then four thread groups each add a quarter of the partials of every
// output (independent loads, eight in flight per thread) and the groups' sums are added in
// group order.
constexpr int kFaMergeThreads = 512;
constexpr int kFaMergeGroups = kFaMergeThreads / 128;
__global__ void __launch_bounds__(kFaMergeThreads) fa_merge_kernel(const float* part, FaSrc src, int grid,
                                                                   float* running_sum, uint16_t* out) {
  __shared__ float w[kFaMaxCtas];
  __shared__ float red[kFaMergeThreads / 32];
  __shared__ float osum[kFaMergeGroups][128];
  __shared__ float Mall, Lall;
  const int h = blockIdx.x >> 2, quarter = blockIdx.x & 3, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();  // the attention output projection may start streaming its weights
  pdl_wait();  // every partial of the previous kernel is written
  int n, rpc, nact;
  fa_split(src, grid, n, rpc, nact);
  float m = -CUDART_INF_F;
  for (int p = tid; p < nact; p += kFaMergeThreads) {
    const float mp = __ldcg(part + static_cast<size_t>(p) * kFaPart + h);
    w[p] = mp;
    m = fmaxf(m, mp);
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (tid == 0) {
    float x = red[0];
    for (int i = 1; i < kFaMergeThreads / 32; ++i) x = fmaxf(x, red[i]);
    Mall = x;
  }
  __syncthreads();
  const float M = Mall;
  float l = 0.f;
  for (int p = tid; p < nact; p += kFaMergeThreads) {
    const float mp = w[p];
    const float wp = (mp == -CUDART_INF_F || M == -CUDART_INF_F) ? 0.f : expf(mp - M);
    w[p] = wp;
    l += wp * __ldcg(part + static_cast<size_t>(p) * kFaPart + GF + h);
  }
  l = warp_sum(l);
  __syncthreads();
  if (lane == 0) red[warp] = l;
  __syncthreads();
  if (tid == 0) {
    float x = 0.f;
    for (int i = 0; i < kFaMergeThreads / 32; ++i) x += red[i];
    Lall = x;
  }
  __syncthreads();
  const int dl = tid & 127, grp = tid >> 7;
  const int d = quarter * 128 + dl;
  const float* src_o = part + 2 * GF + h * DF + d;
  float o = 0.f;
#pragma unroll 8
  for (int p = grp; p < nact; p += kFaMergeGroups) o += w[p] * __ldcg(src_o + static_cast<size_t>(p) * kFaPart);
  osum[grp][dl] = o;
  __syncthreads();
  if (grp == 0) {
    float t = 0.f;
#pragma unroll
    for (int gi = 0; gi < kFaMergeGroups; ++gi) t += osum[gi][dl];
    out[h * DF + d] = f32_to_bf16(Lall > 0.f ? t / Lall : 0.f);
    if (quarter == 0 && tid == 0) running_sum[h] = 1.0f;
  }
}

// ---------------------------------------------------------------------------- sliding, clustered
// The 1024-slot ring of one KV head in ONE cluster of 8 CTAs.  CTA r copies slots
// [128 r, 128 r + 128) of K and V into shared memory with TMA (the cache viewed as
// [slot][kv head][256]; box 64 dims x 1 head x 128 slots with the 128-byte swizzle, so each
// tensor lands as 4 dim blocks [128 slots][64 dims] in the layout the tensor cores read),
// and both contractions run on the 5th-generation tensor cores (tcgen05.mma .kind::f16,
// bf16 x bf16 -> f32 in tensor memory, issued by one thread):
//   scores  S^T[128 slots][16] = K[128 slots][256] . Q^T, A = the K blocks (K-major),
//           B = the 2 q heads in rows 0-1 of a 16-row tile (the rest zero);
//   values  O^T[128 dims][16] = V^T[128 dims][128 slots] . P^T (twice: dims 0-127 and
//           128-255), A = the V blocks read dims-contiguous (MN-major: 64-dim rows of 8
//           slots per 1 KB atom, the next 8 slots 1 KB on, the next 64 dims 16 KB on),
//           B = P in rows 0-1 (bf16) and its remainders P - bf16(P) in rows 2-3 (bf16), so
//           O = column h + column 2 + h carries about 16 significant bits of P.
// Softmax in f32 as the reference (scripts/generate_references.py:324-330), masked slots
// at -inf; V rows of masked slots are zeroed first (unused ring slots may hold anything,
// and 0 * NaN is NaN).  The cluster merges the 8 partials through distributed shared
// memory: CTA r stores dims [32 c, 32 c + 32) of its partial into CTA c's shared memory,
// one cluster barrier, and CTA c adds the 8 partials of its dims in CTA order.
// The copies start before griddepcontrol.wait.  A ring slot is rewritten only by the
// attention projection of the same layer: when the launch knows that projection's device
// offset (`fresh`, its kv_off), the CTA holding that slot copies its K and V rows again
// after the wait; every other slot was written by kernels that completed before this
// launch could start.
constexpr int kScRows = 128;
constexpr int kScCtas = TS / kScRows;  // 8: the cluster
constexpr int kScThreads = 256;
constexpr int kScBox = kScRows;        // slots per TMA box: a whole dim block in one copy
constexpr int kScDimBlk = 64;          // dims per TMA box (128 bytes: the swizzle span)
constexpr uint32_t kScCols = 64;       // tensor memory: S [0,16), O dims 0-127 [16,32), 128-255 [32,48)
static_assert(GS == 2, "two q heads per KV head");
// kind::f16: D f32, A and B bf16, N = 16, M = 128; A K-major (scores) or MN-major (values)
constexpr uint32_t kScIdescK = (1u << 4) | (1u << 7) | (1u << 10) | (2u << 17) | (8u << 24);
constexpr uint32_t kScIdescMN = kScIdescK | (1u << 15);

struct __align__(1024) ScSmem {  // 128-byte-swizzled operands: 1024-byte aligned
  uint16_t k[DS / kScDimBlk][kScRows][kScDimBlk];  // 64 KB
  uint16_t v[DS / kScDimBlk][kScRows][kScDimBlk];  // 64 KB
  uint16_t qb[DS / kScDimBlk][16][kScDimBlk];      // B of the scores: [dim block][16 rows][64]
  uint16_t pb[kScRows / 64][16][64];               // B of the values: [slot block][16 rows][64]
  float mo[kScCtas][GS][32];  // partial weighted sums of this CTA's 32 dims, from CTA c
  float mm[kScCtas][GS], ml[kScCtas][GS];  // and CTA c's softmax max / sum
  float s[GS][kScRows];
  float valid[kScRows];
  float m[GS], l[GS];
  uint64_t full, sdone, odone;
  uint32_t tmem;
};
// Byte offset of 8-element chunk c (elements 8c .. 8c + 7) of row `row` in a 128-byte
// swizzled block of 128-byte rows.
__device__ __forceinline__ uint32_t sw128_off(int row, int c) {
  return static_cast<uint32_t>(row * 128 + (((c & 7) ^ (row & 7)) << 4));
}
// Shared-memory matrix descriptor, 128-byte swizzle: leading / stride byte offsets in bytes.
__device__ __forceinline__ uint64_t sc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1u) << 46) |
         (static_cast<uint64_t>(2u) << 61);
}
__device__ __forceinline__ void sc_mma(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void sc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void sc_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void sc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void sc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store to the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ void st_cluster_f32(float* local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ void tma_3d_load(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__global__ void __launch_bounds__(kScThreads) sliding_attn_cluster_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                          const __grid_constant__ CUtensorMap vmap,
                                                                          const uint16_t* q, const float* mask,
                                                                          uint16_t* out, Scratch* scr,
                                                                          uint64_t budget_ns, const uint16_t* kc,
                                                                          const uint16_t* vc, const int32_t* fresh) {
  extern __shared__ uint8_t sc_raw[];
  ScSmem& sm = *reinterpret_cast<ScSmem*>((reinterpret_cast<uintptr_t>(sc_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t r = cluster_ctarank();
  const int h = blockIdx.x / kScCtas;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = static_cast<int>(r) * kScRows;
  if (tid == 0) {
    mbar_init(&sm.full, 1);
    mbar_init(&sm.sdone, 1);
    mbar_init(&sm.odone, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem)),
                 "r"(kScCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  // B tiles: every row but the ones written below is zero (q rows 0-1; P rows 0-3)
  for (int i = tid; i < (DS / kScDimBlk) * 16 * 8; i += kScThreads) {
    const int row = (i >> 3) & 15;
    if (row >= GS) reinterpret_cast<uint4*>(&sm.qb[0][0][0])[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  for (int i = tid; i < (kScRows / 64) * 16 * 8; i += kScThreads) {
    const int row = (i >> 3) & 15;
    if (row >= 2 * GS) reinterpret_cast<uint4*>(&sm.pb[0][0][0])[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  sc_fence_before();
  __syncthreads();
  sc_fence_after();
  const uint32_t tbase = sm.tmem;
  cluster_arrive_relaxed();  // waited for before the first store into another CTA
  if (warp == 0) {
    // one 16 KB box per dim block and tensor: lanes 0-3 K, 4-7 V
    const uint64_t pol = l2_evict_first_policy();  // 335 MB of rings per token: streamed
    if (lane == 0) mbar_arrive_expect_tx(&sm.full, 2u * kScRows * DS * 2u);
    __syncwarp();
    if (lane < 2 * (DS / kScDimBlk)) {
      const int b = lane % (DS / kScDimBlk);
      const bool is_k = lane < DS / kScDimBlk;
      tma_3d_load(is_k ? &sm.k[b][0][0] : &sm.v[b][0][0], is_k ? &kmap : &vmap, kScDimBlk * b, h, row0, &sm.full,
                  pol);
    }
  }
  pdl_wait();  // q, the mask and the newest cache row come from earlier kernels
  const uint64_t deadline = global_ns() + budget_ns;
  uint8_t* kbase = reinterpret_cast<uint8_t*>(&sm.k[0][0][0]);
  uint8_t* vbase = reinterpret_cast<uint8_t*>(&sm.v[0][0][0]);
  if (tid < GS * DS / 8) {  // q: head tid / 32, dims 8 (tid % 32) .. +7 into rows 0-1 of its dim block
    const int hh = tid >> 5, c = tid & 31;
    const uint4 w = reinterpret_cast<const uint4*>(q + static_cast<size_t>(h) * GS * DS)[tid];
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(&sm.qb[c >> 3][0][0]) + sw128_off(hh, c)) = w;
  }
  if (tid < kScRows) sm.valid[tid] = mask[row0 + tid];
  const int nkv = static_cast<int>(gridDim.x) / kScCtas;
  int fslot = -1;  // the slot the projection just wrote, when this CTA holds it
  if (fresh != nullptr) {
    const long long off = static_cast<long long>(*fresh) / 2;  // element offset of the slot's row
    const long long slot = off / (static_cast<long long>(nkv) * DS);
    if (off >= 0 && slot >= row0 && slot < row0 + kScRows) fslot = static_cast<int>(slot);
  }
  if (!mbar_wait(&sm.full, 0u, deadline)) atomicOr(&scr->status, DEV_ERR_TIMEOUT_MBAR);
  if (fslot >= 0 && tid < 64) {  // after the boxes landed: these stores come last
    const int c = tid & 31, row = fslot - row0;
    const size_t src = (static_cast<size_t>(fslot) * nkv + h) * DS + 8 * c;
    const uint4 w = *reinterpret_cast<const uint4*>((tid < 32 ? kc : vc) + src);
    uint8_t* blk = (tid < 32 ? kbase : vbase) + (c >> 3) * (kScRows * 128);
    *reinterpret_cast<uint4*>(blk + sw128_off(row, c)) = w;
  }
  fence_proxy_async();  // the generic-proxy writes above (q, the new row) are read by the tensor cores
  // the mask is in; masked slots' V rows go to zero (P is 0 there, and 0 * whatever an
  // unused slot holds must be 0) -- only a ring that is not yet full has any
  if (__syncthreads_or(tid < kScRows && !(sm.valid[tid] > 0.f))) {
    for (int i = tid; i < kScRows * (DS / 8); i += kScThreads) {
      const int slot = i >> 5, c = i & 31;
      if (!(sm.valid[slot] > 0.f))
        *reinterpret_cast<uint4*>(vbase + (c >> 3) * (kScRows * 128) + sw128_off(slot, c)) =
            make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async();
    __syncthreads();
  }
  pdl_launch_dependents();
  // ---- scores: 16 MMAs of K = 16 dims (4 per 64-dim block: +32 bytes in the swizzled row)
  if (tid == 0) {
    sc_fence_after();
    const uint32_t kb = smem_u32(kbase), qb = smem_u32(&sm.qb[0][0][0]);
#pragma unroll
    for (int b = 0; b < DS / kScDimBlk; ++b)
#pragma unroll
      for (int st = 0; st < 4; ++st)
        sc_mma(tbase, sc_desc(kb + b * (kScRows * 128) + 32 * st, 16, 1024),
               sc_desc(qb + b * (16 * 128) + 32 * st, 16, 1024), kScIdescK, (b | st) ? 1u : 0u);
    sc_commit(&sm.sdone);
  }
  // ---- softmax in warps 0-3 straight from tensor memory (warp w: slots 32 w + lane), then
  // P and its remainder into the values' B tile
  if (warp < 4) {
    const bool ok = mbar_wait(&sm.sdone, 0u, deadline, true);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      sc_fence_after();
      sc_ld4(tbase + (static_cast<uint32_t>(32 * warp) << 16), d);
    } else if (lane == 0) {
      atomicOr(&scr->status, DEV_ERR_TIMEOUT_MBAR);
    }
    const int slot = 32 * warp + lane;
    const bool v = sm.valid[slot] > 0.f;
    float sv[GS], mx[GS], e[GS], l[GS];
#pragma unroll
    for (int hh = 0; hh < GS; ++hh) {
      sv[hh] = v ? d[hh] : -CUDART_INF_F;
      const float wm = warp_max(sv[hh]);
      if (lane == 0) sm.s[hh][warp] = wm;  // s[][0..3]: per-warp maxima, then sums
    }
    named_bar_sync(1, 128);
#pragma unroll
    for (int hh = 0; hh < GS; ++hh) {
      mx[hh] = fmaxf(fmaxf(sm.s[hh][0], sm.s[hh][1]), fmaxf(sm.s[hh][2], sm.s[hh][3]));
      e[hh] = (sv[hh] == -CUDART_INF_F) ? 0.f : expf(sv[hh] - mx[hh]);
      l[hh] = warp_sum(e[hh]);
    }
    if (lane == 0) {  // (sums go to s[][4..7], beside the maxima)
      sm.s[0][4 + warp] = l[0];
      sm.s[1][4 + warp] = l[1];
    }
    // P: rows 0-1 bf16, rows 2-3 the remainders; slot `slot` is element slot % 64 of block slot / 64
    uint8_t* blk = reinterpret_cast<uint8_t*>(&sm.pb[slot >> 6][0][0]);
    const int c = (slot & 63) >> 3, eb = (slot & 7) * 2;
#pragma unroll
    for (int hh = 0; hh < GS; ++hh) {
      const float x = round_bf16(e[hh]);
      *reinterpret_cast<uint16_t*>(blk + sw128_off(hh, c) + eb) = f32_to_bf16(x);
      *reinterpret_cast<uint16_t*>(blk + sw128_off(GS + hh, c) + eb) = f32_to_bf16(e[hh] - x);
    }
    named_bar_sync(1, 128);
    if (tid < GS) {
      sm.m[tid] = mx[tid];
      sm.l[tid] = ((sm.s[tid][4] + sm.s[tid][5]) + sm.s[tid][6]) + sm.s[tid][7];
    }
  }
  fence_proxy_async();
  __syncthreads();
  // ---- values: per dim half, 8 MMAs of K = 16 slots (the 8-slot atoms are 1 KB apart)
  if (tid == 0) {
    sc_fence_after();
    const uint32_t vb = smem_u32(vbase), pb = smem_u32(&sm.pb[0][0][0]);
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int j = 0; j < kScRows / 16; ++j)
        sc_mma(tbase + 16u + 16u * half,
               sc_desc(vb + half * 2 * (kScRows * 128) + j * 2048, kScRows * 128, 1024),
               sc_desc(pb + (j >> 2) * (16 * 128) + 32 * (j & 3), 16, 1024), kScIdescMN, j ? 1u : 0u);
    sc_commit(&sm.odone);
  }
  cluster_wait();  // every CTA of the cluster is running: its shared memory may be written
  if (warp < 4) {  // TMEM lane quarter `warp`: dims 128 half + 32 warp + lane
    const bool ok = mbar_wait(&sm.odone, 0u, deadline, true);
    if (!ok && lane == 0) atomicOr(&scr->status, DEV_ERR_TIMEOUT_MBAR);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok) {
        sc_fence_after();
        sc_ld4(tbase + 16u + 16u * half + (static_cast<uint32_t>(32 * warp) << 16), d);
      }
      const int dim = 128 * half + 32 * warp + lane;
      const uint32_t dst = static_cast<uint32_t>(dim >> 5);
      st_cluster_f32(&sm.mo[r][0][dim & 31], dst, d[0] + d[2]);
      st_cluster_f32(&sm.mo[r][1][dim & 31], dst, d[1] + d[3]);
    }
  }
  if (tid < GS * kScCtas) {
    const int gh = tid / kScCtas, c = tid % kScCtas;
    st_cluster_f32(&sm.mm[r][gh], static_cast<uint32_t>(c), sm.m[gh]);
    st_cluster_f32(&sm.ml[r][gh], static_cast<uint32_t>(c), sm.l[gh]);
  }
  // Every CTA's partials are in place; after this barrier a CTA reads only its own shared
  // memory, so it may exit as soon as it is done.
  sc_fence_before();
  cluster_arrive_release();
  cluster_wait_acquire();
  if (tid < GS * 32) {
    const int hh = tid >> 5, dl = tid & 31, d = 32 * static_cast<int>(r) + dl;
    float mc[kScCtas], lc[kScCtas], oc[kScCtas], mx = -CUDART_INF_F;
#pragma unroll
    for (int c = 0; c < kScCtas; ++c) {
      mc[c] = sm.mm[c][hh];
      lc[c] = sm.ml[c][hh];
      oc[c] = sm.mo[c][hh][dl];
      mx = fmaxf(mx, mc[c]);
    }
    float ls = 0.f, acc = 0.f;
#pragma unroll
    for (int c = 0; c < kScCtas; ++c) {
      const float w = (mc[c] == -CUDART_INF_F) ? 0.f : expf(mc[c] - mx);
      ls += w * lc[c];
      acc += w * oc[c];
    }
    out[(static_cast<size_t>(h) * GS + hh) * DS + d] = f32_to_bf16(ls > 0.f ? acc / ls : 0.f);
  }
  if (warp == 2) {  // every tensor-memory read of this CTA completed before the cluster barrier
    sc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kScCols));
  }
}

// ---------------------------------------------------------------------------- full (MQA), tcgen05
// fa_partial_kernel's work on the 5th-generation tensor cores, for launches whose grid
// covers max_rows in 64-row ranges (then CTA c holds rows [64 c, 64 c + 64) for every row
// count).  The rows are copied before griddepcontrol.wait (16-byte cp.async chunks into
// 128-byte-swizzled blocks [8 dim blocks][64 rows][64 dims]); after it the newest row is
// copied again and V rows past the count are zeroed.  Then, with one issuing thread:
//   scores S^T[rows][16 heads] = K . Q^T  (kind::f16, M = 128: rows 64-127 of each
//          descriptor read the next block and are ignored; N = 16, 32 MMAs of 16 dims);
//   softmax over the CTA's 64 rows in f32 (4 warps, 4 heads each);
//   values O^T[128 dims][32] = V^T . [P; P - bf16(P)]^T for each quarter of the 512 dims
//          (A = V read MN-major, B = 16 rows of P and 16 of its remainders, N = 32).
// The CTA's (m, l, o[16][512]) partial goes to the same slot fa_merge_kernel reads.
constexpr int kFtThreads = 128;
constexpr int kFtRows = 64;
constexpr uint32_t kFtCols = 256;  // S [0,16), O quarter j at [16 + 32 j, 48 + 32 j)
constexpr uint32_t kFtIdescS = (1u << 4) | (1u << 7) | (1u << 10) | (2u << 17) | (8u << 24);
constexpr uint32_t kFtIdescO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (4u << 17) | (8u << 24);

struct __align__(1024) FtSmem {
  uint16_t k[DF / 64][kFtRows][64];  // 64 KB
  uint16_t v[DF / 64][kFtRows][64];  // 64 KB (K's M = 128 descriptors read into here: ignored rows)
  uint16_t qb[DF / 64][GF][64];      // 16 KB
  uint16_t pb[2 * GF][kFtRows];      // 4 KB: P rows 0-15, remainders 16-31
  float s[GF][kFtRows];
  float m[GF], l[GF];
  uint64_t sdone, odone;
  uint32_t tmem;
};

__device__ __forceinline__ void ft_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void ft_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kFtThreads) fa_tc_kernel(const uint16_t* q, int nq, FaSrc src, float* part,
                                                           Scratch* scr, uint64_t budget_ns) {
  extern __shared__ uint8_t ft_raw[];
  FtSmem& sm = *reinterpret_cast<FtSmem*>((reinterpret_cast<uintptr_t>(ft_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * kFtRows;
  uint8_t* kbase = reinterpret_cast<uint8_t*>(&sm.k[0][0][0]);
  uint8_t* vbase = reinterpret_cast<uint8_t*>(&sm.v[0][0][0]);
  // chunk c (dims 8c .. 8c + 7) of row rr in a [8][64][64] swizzled operand
  auto off = [](int rr, int c) -> uint32_t {
    return static_cast<uint32_t>((c >> 3) * (kFtRows * 128) + rr * 128 + (((c & 7) ^ (rr & 7)) << 4));
  };
  if (tid == 0) {
    mbar_init(&sm.sdone, 1);
    mbar_init(&sm.odone, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem)),
                 "r"(kFtCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  for (int i = tid; i < kFtRows * (DF / 8); i += kFtThreads) {  // rows below max_rows, before the wait
    const int rr = i / (DF / 8), c = i % (DF / 8), r = r0 + rr;
    const bool ok = r < src.max_rows;
    cp_async16(smem_u32(kbase) + off(rr, c), ok ? fa_row(src, false, r) + c * 8 : q, ok ? 16u : 0u);
    cp_async16(smem_u32(vbase) + off(rr, c), ok ? fa_row(src, true, r) + c * 8 : q, ok ? 16u : 0u);
  }
  cp_async_commit();
  sc_fence_before();
  __syncthreads();
  sc_fence_after();
  const uint32_t tbase = sm.tmem;
  pdl_wait();  // q and the newest K/V row come from the projection kernel
  const uint64_t deadline = global_ns() + budget_ns;
  int n, rpc, nact;
  fa_split(src, gridDim.x, n, rpc, nact);
  const int r1 = min(n, r0 + kFtRows);
  if (r0 < r1) {
    for (int i = tid; i < GF * (DF / 8); i += kFtThreads) {  // Q rows (heads past nq zero)
      const int hh = i / (DF / 8), c = i % (DF / 8);
      const bool ok = hh < nq;
      cp_async16(smem_u32(&sm.qb[0][0][0]) + static_cast<uint32_t>((c >> 3) * (GF * 128) + hh * 128 +
                                                                  (((c & 7) ^ (hh & 7)) << 4)),
                 ok ? q + hh * DF + c * 8 : q, ok ? 16u : 0u);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();  // every early copy landed: the newest row and the rows past n may be rewritten
    const int nr = n - 1 - r0;
    for (int i = tid; i < kFtRows * (DF / 8); i += kFtThreads) {
      const int rr = i / (DF / 8), c = i % (DF / 8);
      if (rr == nr) {
        cp_async16(smem_u32(kbase) + off(rr, c), fa_row(src, false, r0 + rr) + c * 8, 16u);
        cp_async16(smem_u32(vbase) + off(rr, c), fa_row(src, true, r0 + rr) + c * 8, 16u);
      } else if (rr >= r1 - r0) {
        *reinterpret_cast<uint4*>(vbase + off(rr, c)) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    cp_async_commit();
    cp_async_wait_all();
  } else {
    cp_async_wait_all();
  }
  fence_proxy_async();  // the copies and stores above are read by the tensor cores
  __syncthreads();
  pdl_launch_dependents();
  if (r0 < r1) {
    // ---- scores
    if (tid == 0) {
      sc_fence_after();
      const uint32_t kb = smem_u32(kbase), qb = smem_u32(&sm.qb[0][0][0]);
#pragma unroll
      for (int b = 0; b < DF / 64; ++b)
#pragma unroll
        for (int st = 0; st < 4; ++st)
          sc_mma(tbase, sc_desc(kb + b * (kFtRows * 128) + 32 * st, 16, 1024),
                 sc_desc(qb + b * (GF * 128) + 32 * st, 16, 1024), kFtIdescS, (b | st) ? 1u : 0u);
      sc_commit(&sm.sdone);
    }
    if (warp < 2) {  // rows 32 warp + lane (TMEM lanes 0-63)
      const bool ok = mbar_wait(&sm.sdone, 0u, deadline, true);
      float d[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) d[i] = 0.f;
      if (ok) {
        sc_fence_after();
        ft_ld16(tbase + (static_cast<uint32_t>(32 * warp) << 16), d);
      } else if (lane == 0) {
        atomicOr(&scr->status, DEV_ERR_TIMEOUT_MBAR);
      }
      const int rr = 32 * warp + lane;
      const bool v = r0 + rr < r1;
#pragma unroll
      for (int hh = 0; hh < GF; ++hh) sm.s[hh][rr] = v ? d[hh] : -CUDART_INF_F;
    }
    __syncthreads();
    // ---- softmax: warp w heads 4w .. 4w + 3, lane rows lane and lane + 32
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int hh = 4 * warp + j;
      const float a = sm.s[hh][lane], b = sm.s[hh][lane + 32];
      const float mx = warp_max(fmaxf(a, b));
      const float pa = (a == -CUDART_INF_F) ? 0.f : expf(a - mx);
      const float pb = (b == -CUDART_INF_F) ? 0.f : expf(b - mx);
      const float l = warp_sum(pa + pb);
      if (lane == 0) {
        sm.m[hh] = mx;
        sm.l[hh] = l;
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int rr = lane + 32 * e;
        const float p = e ? pb : pa, x = round_bf16(p);
        uint8_t* row_hi = reinterpret_cast<uint8_t*>(&sm.pb[hh][0]);
        uint8_t* row_lo = reinterpret_cast<uint8_t*>(&sm.pb[GF + hh][0]);
        const uint32_t o_hi = (((rr >> 3) ^ (hh & 7)) << 4) + (rr & 7) * 2;
        const uint32_t o_lo = (((rr >> 3) ^ ((GF + hh) & 7)) << 4) + (rr & 7) * 2;
        *reinterpret_cast<uint16_t*>(row_hi + o_hi) = f32_to_bf16(x);
        *reinterpret_cast<uint16_t*>(row_lo + o_lo) = f32_to_bf16(p - x);
      }
    }
    fence_proxy_async();
    __syncthreads();
    // ---- values: dims quarter j (dim blocks 2j, 2j + 1), 4 MMAs of 16 rows each
    if (tid == 0) {
      sc_fence_after();
      const uint32_t vb = smem_u32(vbase), pbb = smem_u32(&sm.pb[0][0]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int ks = 0; ks < kFtRows / 16; ++ks)
          sc_mma(tbase + 16u + 32u * j, sc_desc(vb + 2 * j * (kFtRows * 128) + ks * 2048, kFtRows * 128, 1024),
                 sc_desc(pbb + 32 * ks, 16, 1024), kFtIdescO, ks ? 1u : 0u);
      sc_commit(&sm.odone);
    }
    float* mine = part + static_cast<size_t>(blockIdx.x) * kFaPart;
    {
      const bool ok = mbar_wait(&sm.odone, 0u, deadline, true);
      if (!ok && lane == 0) atomicOr(&scr->status, DEV_ERR_TIMEOUT_MBAR);
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {  // warp w: dims 128 j + 32 w + lane
        float d[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) d[i] = 0.f;
        if (ok) {
          sc_fence_after();
          ft_ld32(tbase + 16u + 32u * j + (static_cast<uint32_t>(32 * warp) << 16), d);
        }
        const int dim = 128 * j + 32 * warp + lane;
#pragma unroll
        for (int hh = 0; hh < GF; ++hh) mine[2 * GF + hh * DF + dim] = d[hh] + d[GF + hh];
      }
    }
    if (tid < GF) {
      mine[tid] = sm.m[tid];
      mine[GF + tid] = sm.l[tid];
    }
  }
  sc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kFtCols));
  }
}

// ---------------------------------------------------------------------------- launchers
g4_status launch_full_page(g4_ctx* ctx, bool first, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                           const float* mask, float* rmax, float* rsum, uint16_t* out) {
  const int nq = GF / ctx->tp_world;
  full_page_kernel<<<TF / kChunk, kAttnThreads, 0, ctx->stream>>>(q, k, v, mask, nq, first ? 1 : 0, rmax, rsum, out,
                                                                  ctx->buf.attn, ctx->buf.scratch);
  return check_cuda(ctx, cudaGetLastError(), "full_attention_page");
}

}  // namespace g4

namespace g4 {

// GQA attention over `rows` cache rows of the sliding layout [rows, Ns/N, Ds] (rows a
// multiple of 64): the reference's sliding_attention at rows = Ts, and the same geometry
// over a longer cache (BASELINE config 3's 8 KV heads of 256 at 8192 positions).
g4_status launch_gqa_attention(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                               const float* mask, int rows, uint16_t* out) {
  static_assert(static_cast<size_t>(NS) * (E / kSaRows) * kSaPart <= kAttnFloats, "partials fit");
  int nkv = NS / ctx->tp_world, nchunks = rows / kSaRows;
  float* part = ctx->buf.attn;
  Scratch* scr = ctx->buf.scratch;
  void* args[] = {(void*)&q, (void*)&k, (void*)&v, (void*)&mask, (void*)&nkv, (void*)&nchunks, (void*)&out,
                  (void*)&part, (void*)&scr};
  return launch_kernel(ctx, (const void*)sliding_attn_kernel, dim3(nkv * nchunks), dim3(kSaThreads), 0, args,
                       false, "gqa attention");
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
// The sliding cache [Ts][nkv][Ds] bf16 as a 3-D tensor (dims: Ds, nkv, Ts), box
// 64 x 1 x 128 (64 dims of a CTA's 128 slots of one head: 128-byte rows, 16 KB) with the
// 128-byte swizzle.
static bool cache_map(CUtensorMap* m, const void* base, int nkv) {
  static EncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
               ? reinterpret_cast<EncodeFn>(p)
               : nullptr;
  }();
  if (fn == nullptr || !aligned16(base)) return false;
  const cuuint64_t dims[3] = {DS, static_cast<cuuint64_t>(nkv), TS};
  const cuuint64_t strides[2] = {DS * 2, static_cast<cuuint64_t>(nkv) * DS * 2};
  const cuuint32_t box[3] = {kScDimBlk, 1, kScBox};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The 1024-slot ring: one cluster of 8 CTAs per KV head (sliding_attn_cluster_kernel);
// where the runtime refuses the cluster launch, the split-KV kernel with a global merge.
g4_status launch_sliding_attention(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                   const float* mask, uint16_t* out) {
  // the newest row of this cache, when the last projection on this context wrote it
  const int32_t* fresh = (ctx->qkv_kc == k) ? ctx->qkv_kv_off : nullptr;
  CUtensorMap km, vm;
  const int nkv = NS / ctx->tp_world;
  if (ctx->cluster_ok && cache_map(&km, k, nkv) && cache_map(&vm, v, nkv)) {
    const void* fn = reinterpret_cast<const void*>(&sliding_attn_cluster_kernel);
    const size_t smem = sizeof(ScSmem) + 1024;
    g4_status st = allow_max_dynamic_smem(ctx, fn, smem, "sliding attention");
    if (st != G4_OK) return st;
    Scratch* scr = ctx->buf.scratch;
    uint64_t budget = ctx->wait_budget_ns;
    void* args[] = {(void*)&km,  (void*)&vm,     (void*)&q, (void*)&mask, (void*)&out,
                    (void*)&scr, (void*)&budget, (void*)&k, (void*)&v,    (void*)&fresh};
    if (launch_kernel(ctx, fn, dim3(nkv * kScCtas), dim3(kScThreads), smem, args, false, "sliding attention",
                      kScCtas) == G4_OK)
      return G4_OK;
    ctx->cluster_ok = false;  // not on this device / runtime: the split-KV kernel from now on
  }
  return launch_gqa_attention(ctx, q, k, v, mask, TS, out);
}

// Full (MQA) attention over rows [0, n) of `src`; grid sized for src.max_rows.
static g4_status launch_full_attention(g4_ctx* ctx, const uint16_t* q, const FaSrc& src, float* rsum,
                                       uint16_t* out) {
  static_assert(static_cast<size_t>(kFaMaxCtas) * kFaPart <= kAttnFloats, "partials fit the attention scratch");
  int nq = GF / ctx->tp_world;
  const int want = (src.max_rows + 63) / 64;
  int grid = 2 * ctx->sm_count;
  if (grid > kFaMaxCtas) grid = kFaMaxCtas;
  if (want < grid) grid = want < 1 ? 1 : want;
  float* part = ctx->buf.attn;
  FaSrc s = src;
  g4_status st;
  if (static_cast<long long>(grid) * kFtRows >= src.max_rows) {  // 64 rows per CTA: the tensor-core kernel
    const size_t smem = sizeof(FtSmem) + 1024;
    st = allow_max_dynamic_smem(ctx, (const void*)fa_tc_kernel, smem, "full attention");
    if (st != G4_OK) return st;
    Scratch* scr = ctx->buf.scratch;
    uint64_t budget = ctx->wait_budget_ns;
    void* a1[] = {(void*)&q, (void*)&nq, (void*)&s, (void*)&part, (void*)&scr, (void*)&budget};
    st = launch_kernel(ctx, (const void*)fa_tc_kernel, dim3(grid), dim3(kFtThreads), smem, a1, false,
                       "full attention partials");
  } else {
    st = allow_max_dynamic_smem(ctx, (const void*)fa_partial_kernel, sizeof(FaSmem), "full attention");
    if (st != G4_OK) return st;
    void* a1[] = {(void*)&q, (void*)&nq, (void*)&s, (void*)&part};
    st = launch_kernel(ctx, (const void*)fa_partial_kernel, dim3(grid), dim3(kFaThreads), sizeof(FaSmem), a1, false,
                       "full attention partials");
  }
  if (st != G4_OK) return st;
  void* a2[] = {(void*)&part, (void*)&s, (void*)&grid, (void*)&rsum, (void*)&out};
  return launch_kernel(ctx, (const void*)fa_merge_kernel, dim3(4 * nq), dim3(kFaMergeThreads), 0, a2, false,
                       "full attention merge");
}

g4_status launch_full_paged(g4_ctx* ctx, const uint16_t* q, const uint16_t* const* kp, const uint16_t* const* vp,
                            int n_pages, int last_row, float* rsum, uint16_t* out) {
  FaSrc s = {};
  s.k_pages = kp;
  s.v_pages = vp;
  s.n_host = (n_pages - 1) * TF + last_row + 1;
  s.max_rows = s.n_host;
  return launch_full_attention(ctx, q, s, rsum, out);
}

g4_status launch_full_rows(g4_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                           const int32_t* n_rows, int max_rows, float* rsum, uint16_t* out) {
  FaSrc s = {};
  s.k = k;
  s.v = v;
  s.n_dev = n_rows;
  s.max_rows = max_rows;
  return launch_full_attention(ctx, q, s, rsum, out);
}

}  // namespace g4
