// Attention projections and the lm_head on the streaming engine.
//
//  QkvOp   : {sliding,full}_project_qkv (src/ops.rs:44-124).  Stage RMSNorm(x); items
//            cover 8 rows of the concatenated [Q;K;V] row space (FP8: both K halves in
//            one item; NVFP4: two row tiles); each item stores raw row sums and bumps its
//            head's counter; the warp completing a head runs the head epilogue: row scale
//            -> bf16, per-head RMSNorm (q/k weighted, v unweighted; full layers derive V
//            from the raw K head, src/device/full/rmsnorm.rs:189-196), RoPE with the
//            kernel-convention tables (sin low half pre-negated, src/host/runtime.rs:
//            271-299), then q_out or the KV-cache row at the device byte offset.
//  OprojOp : {sliding,full}_attention_output (src/ops.rs:138-211).  Stage x (full: x/sum
//            per head first, src/device/full/attention.rs:336-358); items = 8 output rows
//            x two K chunks; last CTA: y -> bf16(y*row_scale) -> RMSNorm(post) -> +residual.
//  LmHeadOp: final_norm_and_logits (src/ops.rs:255-312, src/device/shared/lm_head.rs):
//            stage RMSNorm(x) as bf16; items = 8 vocab rows x both K halves; epilogue
//            bf16 logit -> bf16(tanh(l/30)*30).
#include <cstdlib>
#include <cstring>

#include "g4_internal.h"
#include "g4_stream.cuh"

namespace g4 {

// ============================================================================ QKV
struct QkvOp {
  static constexpr int kPhases = 1;
  // geometry
  int D;            // head dim (256 sliding, 512 full)
  int nq, nk, nv;   // local q / k / v heads (nv = 0: V derived from raw K)
  int nvfp4;        // 1: NVFP4 weights (two row tiles per item), 0: FP8 (two K halves)
  // inputs
  const uint16_t* x;
  const uint16_t* in_w;
  const uint8_t* w[3];       // codes of Q, K, V
  const uint8_t* bs[3];      // NVFP4 block scales
  const uint16_t* rs[3];     // FP8 per-row bf16 scales
  const float* gs[3];        // NVFP4 reciprocal global scales
  const uint16_t* qn_w;
  const uint16_t* kn_w;
  const int32_t* kv_off;
  const int32_t* rope_off;
  const uint16_t* cosT;
  const uint16_t* sinT;
  long long table_elems;     // E * D
  uint16_t* kc;
  uint16_t* vc;
  long long cache_elems;
  uint16_t* q_out;
  Scratch* scr;
  float* rows;               // raw row sums of the concatenated row space
  UnitGeom g;

  __device__ int total_rows() const { return (nq + nk + nv) * D; }
  __device__ int items() const { return nvfp4 ? total_rows() / 16 : total_rows() / 8; }
  __device__ int items(int) const { return items(); }
  __device__ UnitGeom geom(int) const { return g; }
  // matrix index and local row of a concatenated row
  __device__ void locate(int row, int& m, int& r) const {
    if (row < nq * D) {
      m = 0;
      r = row;
    } else if (row < (nq + nk) * D) {
      m = 1;
      r = row - nq * D;
    } else {
      m = 2;
      r = row - (nq + nk) * D;
    }
  }
  // FP8: a unit is 4 rows x both K halves (2 pseudo-rows per row), an item 8 rows;
  // NVFP4: a unit is 8 rows x full K, an item 16 rows.
  __device__ int unit_rows() const { return nvfp4 ? 8 : 4; }
  __device__ UnitDesc unit(int, int it, int half) const {
    UnitDesc u;
    const int row0 = (it * 2 + half) * unit_rows();
    int m, r;
    locate(row0, m, r);
    const uint32_t rowbytes = nvfp4 ? H / 2 : H;
    u.codes = w[m] + static_cast<size_t>(r) * rowbytes;
    u.scales = nvfp4 ? bs[m] + static_cast<size_t>(r) * (H / 16) : nullptr;
    u.code_stride = rowbytes;
    u.scale_stride = H / 16;
    return u;
  }
  __device__ uint32_t* status() const { return &scr->status; }
  __device__ uint32_t* done_counter() const { return &scr->proj_done; }
  __device__ bool has_final() const { return false; }
  __device__ bool between_phases(StreamSmem&, int, uint64_t) const { return true; }
  __device__ void final_epilogue(StreamSmem&, uint8_t*, int) const {}
  // CTA c pulls line c of the input norm weight (read by every CTA's staging) into L2.
  __device__ void prefetch_l2(int cta, int lane) const {
    constexpr int kBytes = H * 2, kLines = kBytes / 128 + 1;
    if (lane == 0 && cta < kLines) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(in_w) + min(cta * 128, kBytes - 1));
  }
  __device__ void stage(StreamSmem& sm, uint8_t* xbuf, int, int tid, const XLayout& xl) const {
    const int e = stage_rmsnorm(x, in_w, H, reinterpret_cast<uint16_t*>(xbuf), true, sm.scratch, xl);
    if (tid == 0) sm.xexp = e;
  }

  // Projection value of one row before the per-head norm: FP8 bf16(acc*scale_row),
  // NVFP4 bf16(bf16(acc)*global).
  __device__ float row_value(int row, float acc) const {
    int m, r;
    locate(row, m, r);
    if (nvfp4) return round_bf16(round_bf16(acc) * __ldg(gs[m]));
    return round_bf16(acc * bf16_to_f32(rs[m][r]));
  }

  __device__ void item_epilogue(StreamSmem& sm, int, int it, int lane, float v) const {
    const float unscale = ldexpf(1.0f, -sm.xexp);
    const int nrows = 2 * unit_rows();
    const int row0 = it * nrows;
    const float rv = sum_pseudo_rows(v, lane, nvfp4 ? 1 : 2);
    if (lane < nrows) rows[row0 + lane] = rv * unscale;
    __syncwarp();
    const int head = row0 / D;
    uint32_t old = 0;
    if (lane == 0) {
      __threadfence();
      old = atom_add_acq_rel_gpu(&scr->head_count[head], 1u);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + 1 == static_cast<uint32_t>(D / nrows)) {
      __threadfence();
      head_epilogue(head, lane);
      if (lane == 0) scr->head_count[head] = 0u;
    }
  }

  // Warp-level: norm + RoPE + store of one head.  Lane l owns elements l + 32j.
  __device__ void head_epilogue(int head, int lane) const {
    constexpr int kMaxJ = 16;
    const int J = D / 32;
    float raw[kMaxJ];
    const int row0 = head * D;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
      if (j < J) {
        raw[j] = row_value(row0 + lane + 32 * j, __ldcg(rows + row0 + lane + 32 * j));
        ss = __fadd_rn(ss, __fmul_rn(raw[j], raw[j]));
      }
    }
    const float r = rms_factor(warp_sum(ss), D);
    const bool is_q = head < nq;
    const bool is_k = !is_q && head < nq + nk;
    const int roff = __ldg(rope_off) / 2;
    const int koff = __ldg(kv_off) / 2;
    if (roff < 0 || static_cast<long long>(roff) + D > table_elems || koff < 0 ||
        static_cast<long long>(koff) + static_cast<long long>(nk > 0 ? (nv > 0 ? nk : 1) : 1) * D > cache_elems) {
      if (lane == 0) atomicOr(&scr->status, DEV_ERR_BAD_OFFSET);
      return;
    }
    // V of a full (MQA) layer: unweighted norm of the raw K head.
    if (is_k && nv == 0) {
      for (int j = 0; j < J; ++j) {
        const int i = lane + 32 * j;
        vc[koff + i] = f32_to_bf16(__fmul_rn(raw[j], r));
      }
    }
    if (!is_q && !is_k) {  // sliding V head: unweighted norm, no RoPE
      const int vh = head - nq - nk;
      for (int j = 0; j < J; ++j) {
        const int i = lane + 32 * j;
        vc[koff + vh * D + i] = f32_to_bf16(__fmul_rn(raw[j], r));
      }
      return;
    }
    const uint16_t* nw = is_q ? qn_w : kn_w;
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
        const float c = bf16_to_f32(cosT[roff + i]);
        const float s = bf16_to_f32(sinT[roff + i]);
        const float o = round_bf16(__fadd_rn(round_bf16(__fmul_rn(n[j], c)), round_bf16(__fmul_rn(partner, s))));
        if (is_q) {
          q_out[head * D + i] = f32_to_bf16(o);
        } else {
          const int kh = head - nq;
          kc[koff + kh * D + i] = f32_to_bf16(o);
        }
      }
    }
  }
};

// ============================================================================ o-proj
struct OprojOp {
  static constexpr int kPhases = 1;
  int K;            // local input width
  int q;            // K segments per row (pseudo-rows per real row)
  int nvfp4;
  int Dh;           // head dim for the running-sum division (0: none)
  const uint16_t* x;
  const float* rsum;
  const uint16_t* post_w;
  const uint8_t* w;
  const uint8_t* bs;
  const uint16_t* row_scale;
  const float* gsc;
  uint16_t* residual;
  Scratch* scr;
  float* part;
  float* ybuf;      // TP over NCCL: partial y (already unscaled) for the all-reduce
  PeerXch xch;      // TP over peer memory (world <= 1: not in use)
  UnitGeom g;

  // a unit is 8/q whole output rows; an item two units (A, B)
  __device__ int unit_rows() const { return 8 / q; }
  __device__ int items(int) const { return H / (2 * unit_rows()); }
  __device__ UnitGeom geom(int) const { return g; }
  __device__ UnitDesc unit(int, int it, int half) const {
    UnitDesc u;
    const int row0 = (it * 2 + half) * unit_rows();
    const uint32_t rowbytes = nvfp4 ? K / 2 : K;
    u.codes = w + static_cast<size_t>(row0) * rowbytes;
    u.scales = nvfp4 ? bs + static_cast<size_t>(row0) * (K / 16) : nullptr;
    u.code_stride = rowbytes;
    u.scale_stride = K / 16;
    return u;
  }
  __device__ uint32_t* status() const { return &scr->status; }
  __device__ uint32_t* done_counter() const { return &scr->proj_done; }
  // The fused tail (CTA 0) reads residual, post_w and the row scales: CTA c pulls line
  // c of each into L2 at kernel start.
  __device__ void prefetch_l2(int cta, int lane) const {
    if (ybuf != nullptr) return;  // TP: the tail runs in its own kernel after the all-reduce
    constexpr int kBytes = H * 2, kLines = kBytes / 128 + 1;
    if (cta >= kLines) return;
    const int off = min(cta * 128, kBytes - 1);
    if (lane == 0) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(post_w) + off);
    if (lane == 1) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(residual) + off);
    if (lane == 2 && !nvfp4) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(row_scale) + off);
    if (lane == 3 && nvfp4 && cta == 0) prefetch_l2_keep(gsc);
  }
  __device__ bool has_final() const { return true; }
  __device__ bool between_phases(StreamSmem&, int, uint64_t) const { return true; }

  // 8 inputs per 16-byte load, all loads issued first (K <= kG * 8 * kConsumerThreads).
  __device__ void stage(StreamSmem& sm, uint8_t* xbuf, int, int tid, const XLayout& xl) const {
    uint16_t* xs = reinterpret_cast<uint16_t*>(xbuf);
    constexpr int kG = 3;
    static_assert(kG * 8 * kConsumerThreads >= 8192, "o-proj staging must cover K = Qf");
    uint4 xv[kG];
    float rs[kG];
#pragma unroll
    for (int k = 0; k < kG; ++k) {
      const int gi = tid + k * kConsumerThreads;
      if (gi * 8 < K) {
        xv[k] = __ldg(reinterpret_cast<const uint4*>(x) + gi);
        rs[k] = (Dh > 0) ? __ldg(rsum + gi * 8 / Dh) : 1.0f;  // 8 | Dh: one head per group
      }
    }
    float v[kG][8];
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < kG; ++k) {
      const int gi = tid + k * kConsumerThreads;
      if (gi * 8 < K) {
        const uint32_t w[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float f = bf16_to_f32(static_cast<uint16_t>((i & 1) ? w[i >> 1] >> 16 : w[i >> 1] & 0xFFFFu));
          if (Dh > 0) f = round_bf16(__fdiv_rn(f, rs[k]));
          v[k][i] = f;
          amax = fmaxf(amax, fabsf(f));
        }
      }
    }
    const int e = f16_scale_exponent(consumer_max(amax, sm.scratch + 32));
    const float sc = ldexpf(1.0f, e);
#pragma unroll
    for (int k = 0; k < kG; ++k) {
      const int gi = tid + k * kConsumerThreads;
      if (gi * 8 < K) {
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = pack_u16x2(f32_to_f16(v[k][2 * i] * sc), f32_to_f16(v[k][2 * i + 1] * sc));
        *reinterpret_cast<uint4*>(xs + x_pos(static_cast<uint32_t>(gi) * 8u, xl)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (tid == 0) sm.xexp = e;
  }

  __device__ void item_epilogue(StreamSmem& sm, int, int it, int lane, float v) const {
    const float rv = sum_pseudo_rows(v, lane, q);
    if (lane < 2 * unit_rows()) part[it * 2 * unit_rows() + lane] = rv * ldexpf(1.0f, -sm.xexp);
  }

  // Thread tid < H/8 owns outputs [8*tid, 8*tid + 8) and issues all of its loads first.
  __device__ void final_epilogue(StreamSmem& sm, uint8_t*, int tid) const {
    const bool mine = tid < H / 8;
    float y[8];
    uint4 rv = make_uint4(0u, 0u, 0u, 0u), wv = rv, sv = rv;
    if (mine) {
      const float4 p0 = __ldcg(reinterpret_cast<const float4*>(part) + 2 * tid);
      const float4 p1 = __ldcg(reinterpret_cast<const float4*>(part) + 2 * tid + 1);
      y[0] = p0.x, y[1] = p0.y, y[2] = p0.z, y[3] = p0.w, y[4] = p1.x, y[5] = p1.y, y[6] = p1.z, y[7] = p1.w;
      if (ybuf == nullptr) {
        rv = *reinterpret_cast<const uint4*>(residual + 8 * tid);
        wv = __ldg(reinterpret_cast<const uint4*>(post_w) + tid);
        if (!nvfp4) sv = __ldg(reinterpret_cast<const uint4*>(row_scale) + tid);
      }
    }
    if (ybuf != nullptr) {
      if (mine) {
        reinterpret_cast<float4*>(ybuf)[2 * tid] = make_float4(y[0], y[1], y[2], y[3]);
        reinterpret_cast<float4*>(ybuf)[2 * tid + 1] = make_float4(y[4], y[5], y[6], y[7]);
      }
      return;
    }
    if (xch.world > 1 && !peer_allreduce(xch, &scr->xch_epoch, y, tid, &scr->status, sm)) return;
    const float gs = nvfp4 ? __ldg(gsc) : 0.f;
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
    float ss = 0.f;
    if (mine) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float rsc = bf16_to_f32(static_cast<uint16_t>((i & 1) ? sw[i >> 1] >> 16 : sw[i >> 1] & 0xFFFFu));
        const float pv = nvfp4 ? round_bf16(round_bf16(y[i]) * gs) : round_bf16(y[i] * rsc);
        y[i] = pv;
        ss = __fadd_rn(ss, __fmul_rn(pv, pv));
      }
    }
    const float r = rms_factor(consumer_sum(ss, sm.scratch), H);
    if (mine) {
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint16_t h2[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float res = bf16_to_f32(static_cast<uint16_t>(j ? rw[i] >> 16 : rw[i] & 0xFFFFu));
          const float pw = bf16_to_f32(static_cast<uint16_t>(j ? ww[i] >> 16 : ww[i] & 0xFFFFu));
          const float nb = round_bf16(__fmul_rn(__fmul_rn(y[2 * i + j], r), pw));
          h2[j] = f32_to_bf16(__fadd_rn(res, nb));
        }
        o[i] = pack_u16x2(h2[0], h2[1]);
      }
      *reinterpret_cast<uint4*>(residual + 8 * tid) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
};

// TP tail of the o-proj after the all-reduce of y.
__global__ void __launch_bounds__(1024) oproj_tp_epilogue_kernel(const float* __restrict__ y, int nvfp4,
                                                                 const uint16_t* __restrict__ row_scale,
                                                                 const float* gsc, const uint16_t* __restrict__ post_w,
                                                                 uint16_t* __restrict__ residual) {
  __shared__ float red[32];
  __shared__ float yb[H];
  float ss = 0.f;
  for (int n = threadIdx.x; n < H; n += blockDim.x) {
    const float pv = nvfp4 ? round_bf16(round_bf16(y[n]) * __ldg(gsc)) : round_bf16(y[n] * bf16_to_f32(row_scale[n]));
    yb[n] = pv;
    ss = __fadd_rn(ss, __fmul_rn(pv, pv));
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) tot += red[w];
  const float r = rms_factor(tot, H);
  for (int n = threadIdx.x; n < H; n += blockDim.x) {
    const float nb = round_bf16(__fmul_rn(__fmul_rn(yb[n], r), bf16_to_f32(post_w[n])));
    residual[n] = f32_to_bf16(__fadd_rn(bf16_to_f32(residual[n]), nb));
  }
}

// ============================================================================ lm_head
struct LmHeadOp {
  static constexpr Fmt kFmt = Fmt::BF16;
  static constexpr int kPhases = 1;
  int rows;               // local vocab rows
  const uint16_t* x;
  const uint16_t* w_norm;
  const uint16_t* wt;     // [rows, H] bf16
  uint16_t* out;
  Scratch* scr;
  UnitGeom g;

  // a unit is 2 vocab rows x 4 K quarters (pseudo-rows), an item 4 rows
  __device__ int items(int) const { return rows / 4; }
  __device__ UnitGeom geom(int) const { return g; }
  __device__ UnitDesc unit(int, int it, int half) const {
    UnitDesc u;
    u.codes = reinterpret_cast<const uint8_t*>(wt + static_cast<size_t>(it * 2 + half) * 2 * H);
    u.scales = nullptr;
    u.code_stride = H * 2;
    u.scale_stride = 0;
    return u;
  }
  __device__ uint32_t* status() const { return &scr->status; }
  __device__ uint32_t* done_counter() const { return &scr->lm_done; }
  __device__ bool has_final() const { return false; }
  __device__ bool between_phases(StreamSmem&, int, uint64_t) const { return true; }
  __device__ void final_epilogue(StreamSmem&, uint8_t*, int) const {}
  // CTA c pulls line c of the final norm weight (read by every CTA's staging) into L2.
  __device__ void prefetch_l2(int cta, int lane) const {
    constexpr int kBytes = H * 2, kLines = kBytes / 128 + 1;
    if (lane == 0 && cta < kLines) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(w_norm) + min(cta * 128, kBytes - 1));
  }
  __device__ void stage(StreamSmem& sm, uint8_t* xbuf, int, int tid, const XLayout& xl) const {
    stage_rmsnorm(x, w_norm, H, reinterpret_cast<uint16_t*>(xbuf), false, sm.scratch, xl);
    if (tid == 0) sm.xexp = 0;
  }
  __device__ void item_epilogue(StreamSmem&, int, int it, int lane, float v) const {
    const float dot = sum_pseudo_rows(v, lane, 4);
    if (lane < 4) {
      const float logit = round_bf16(dot);
      const float capped = __fmul_rn(tanhf(__fdiv_rn(logit, LOGIT_SOFTCAP)), LOGIT_SOFTCAP);
      out[it * 4 + lane] = f32_to_bf16(capped);
    }
  }
};

template <Fmt F>
struct QkvOpF : QkvOp {
  static constexpr Fmt kFmt = F;
};
template <Fmt F>
struct OprojOpF : OprojOp {
  static constexpr Fmt kFmt = F;
};

template <class Op>
__global__ void __launch_bounds__(kThreads, 1)
    stream_kernel(const Op op, const StreamLayout lay, uint32_t slot_bytes, uint64_t budget_ns) {
  stream_body(op, lay, slot_bytes, budget_ns);
}

template <class Op>
static g4_status launch_stream(g4_ctx* ctx, const Op& op, uint32_t slot_bytes, uint32_t nslots, uint32_t x_bytes,
                               int n_items, const char* name) {
  const StreamLayout lay = make_layout(slot_bytes, nslots, x_bytes);
  g4_status st = allow_max_dynamic_smem(ctx, (const void*)stream_kernel<Op>, lay.total, name);
  if (st != G4_OK) return st;
  const int grid = n_items < ctx->sm_count ? n_items : ctx->sm_count;
  uint64_t budget = ctx->wait_budget_ns;
  void* args[] = {(void*)&op, (void*)&lay, (void*)&slot_bytes, (void*)&budget};
  return launch_kernel(ctx, (const void*)stream_kernel<Op>, dim3(grid), dim3(kThreads), lay.total, args, false, name);
}

// ---------------------------------------------------------------------------- launchers
g4_status launch_qkv_fp8(g4_ctx*, bool, const uint16_t*, const uint8_t* const[3], const uint16_t* const[3],
                         const uint16_t*, const uint16_t*, const uint16_t*, const int32_t*, const int32_t*,
                         const uint16_t*, const uint16_t*, uint16_t*, uint16_t*, uint16_t*, long long);
g4_status launch_oproj_fp8(g4_ctx*, bool, const uint16_t*, const float*, const uint16_t*, const uint8_t*,
                           const uint16_t*, uint16_t*);

// FP8 projections: project_qkv runs on the tensor-core GEMV of g4_fp8.cu (any tensor-
// parallel size: a rank's heads need no exchange), the attention output on the streaming
// engine (9.1 / 11.7 us per sliding / full call against 10.1 / 16.5 us there: its work per
// CTA is small and the GEMV's fixed costs weigh more; under tensor parallelism the
// streaming engine's in-kernel all-reduce is needed).
// G4B200_PROJ_KERNEL=stream or =tensor puts both on one kernel (on one GPU).  NVFP4
// weights always use the streaming engine.
static int proj_kernel_env() {
  static const int kind = [] {
    const char* e = std::getenv("G4B200_PROJ_KERNEL");
    if (e != nullptr && std::strcmp(e, "stream") == 0) return 1;
    if (e != nullptr && std::strcmp(e, "tensor") == 0) return 2;
    return 0;
  }();
  return kind;
}
static bool fp8_tensor_path(const g4_ctx* ctx, bool oproj) {
  const int kind = proj_kernel_env();
  if (oproj) return ctx->tp_world == 1 && kind == 2;
  return kind != 1;
}

g4_status launch_qkv(g4_ctx* ctx, bool full, bool nvfp4, const uint16_t* x, const uint8_t* const w[3],
                     const uint8_t* const bs[3], const uint16_t* const rs[3], const float* const gs[3],
                     const uint16_t* in_w, const uint16_t* qn_w, const uint16_t* kn_w, const int32_t* kv_off,
                     const int32_t* rope_off, const uint16_t* cosT, const uint16_t* sinT, uint16_t* kcache,
                     uint16_t* vcache, uint16_t* q_out, long long cache_elems) {
  ctx->qkv_kc = kcache;
  ctx->qkv_kv_off = kv_off;
  if (!nvfp4 && fp8_tensor_path(ctx, false))
    return launch_qkv_fp8(ctx, full, x, w, rs, in_w, qn_w, kn_w, kv_off, rope_off, cosT, sinT, kcache, vcache, q_out,
                          cache_elems);
  QkvOp op;
  const int tp = ctx->tp_world;
  op.D = full ? DF : DS;
  op.nq = (full ? GF : NS * GS) / tp;
  op.nk = full ? 1 : NS / tp;
  op.nv = full ? 0 : NS / tp;
  op.nvfp4 = nvfp4 ? 1 : 0;
  op.x = x;
  op.in_w = in_w;
  for (int i = 0; i < 3; ++i) {
    op.w[i] = w[i];
    op.bs[i] = bs[i];
    op.rs[i] = rs[i];
    op.gs[i] = gs[i];
  }
  op.qn_w = qn_w;
  op.kn_w = kn_w;
  op.kv_off = kv_off;
  op.rope_off = rope_off;
  op.cosT = cosT;
  op.sinT = sinT;
  op.table_elems = static_cast<long long>(E) * op.D;
  op.kc = kcache;
  op.vc = vcache;
  // the reference's cache tensors (one page of a full layer, the whole sliding ring)
  // unless the caller passes a larger contiguous cache (the decode workspace)
  op.cache_elems = cache_elems > 0 ? cache_elems
                                   : (full ? static_cast<long long>(TF) * DF : static_cast<long long>(TS) * op.nk * DS);
  op.q_out = q_out;
  op.scr = ctx->buf.scratch;
  op.rows = ctx->buf.rows;
  op.g = nvfp4 ? make_geom(Fmt::NVFP4, H / 2, 1) : make_geom(Fmt::FP8, H / 2, 2);
  if (!geom_ok(op.g, nvfp4 ? H / 2 : H, H / 16)) return fail(ctx, G4_ERR_UNSUPPORTED, "qkv geometry");
  const int n_items = nvfp4 ? (op.nq + op.nk + op.nv) * op.D / 16 : (op.nq + op.nk + op.nv) * op.D / 8;
  if (nvfp4) {
    QkvOpF<Fmt::NVFP4> o;
    static_cast<QkvOp&>(o) = op;
    return launch_stream(ctx, o, op.g.slot_bytes, 8, H * 2, n_items, "qkv_nvfp4");
  }
  QkvOpF<Fmt::FP8> o;
  static_cast<QkvOp&>(o) = op;
  return launch_stream(ctx, o, op.g.slot_bytes, 8, H * 2, n_items, "qkv_fp8");
}

g4_status launch_oproj(g4_ctx* ctx, bool full, bool nvfp4, const uint16_t* x, const float* rsum, const uint16_t* post_w,
                       const uint8_t* w, const uint8_t* bs, const uint16_t* row_scale, const float* gsc,
                       uint16_t* residual) {
  if (!nvfp4 && fp8_tensor_path(ctx, true)) return launch_oproj_fp8(ctx, full, x, rsum, post_w, w, row_scale, residual);
  OprojOp op;
  const int tp = ctx->tp_world;
  op.K = (full ? QF : QS) / tp;
  op.q = op.K >= 4096 ? 4 : (op.K >= 2048 ? 2 : 1);
  op.nvfp4 = nvfp4 ? 1 : 0;
  op.Dh = full ? DF : 0;
  op.x = x;
  op.rsum = rsum;
  op.post_w = post_w;
  op.w = w;
  op.bs = bs;
  op.row_scale = row_scale;
  op.gsc = gsc;
  op.residual = residual;
  op.scr = ctx->buf.scratch;
  op.part = ctx->buf.part;
  const bool tp_nccl = tp > 1 && ctx->peers.world <= 1;
  op.ybuf = tp_nccl ? ctx->buf.ybuf : nullptr;
  op.xch = ctx->peers;
  const uint32_t rowbytes = nvfp4 ? op.K / 2 : op.K;
  op.g = make_geom(nvfp4 ? Fmt::NVFP4 : Fmt::FP8, rowbytes / op.q, op.q);
  if (!geom_ok(op.g, rowbytes, op.K / 16)) return fail(ctx, G4_ERR_UNSUPPORTED, "o-proj geometry");
  const uint32_t xb = static_cast<uint32_t>(op.K * 2 > H * 4 ? op.K * 2 : H * 4);
  const int n_items = H / (2 * (8 / op.q));
  g4_status st;
  if (nvfp4) {
    OprojOpF<Fmt::NVFP4> o;
    static_cast<OprojOp&>(o) = op;
    st = launch_stream(ctx, o, op.g.slot_bytes, 8, xb, n_items, "oproj_nvfp4");
  } else {
    OprojOpF<Fmt::FP8> o;
    static_cast<OprojOp&>(o) = op;
    st = launch_stream(ctx, o, op.g.slot_bytes, 8, xb, n_items, "oproj_fp8");
  }
  if (st != G4_OK || !tp_nccl) return st;
  st = allreduce_f32(ctx, ctx->buf.ybuf, H);
  if (st != G4_OK) return st;
  oproj_tp_epilogue_kernel<<<1, 1024, 0, ctx->stream>>>(ctx->buf.ybuf, op.nvfp4, row_scale, gsc, post_w, residual);
  return check_cuda(ctx, cudaGetLastError(), "oproj_tp_epilogue");
}

g4_status launch_lm_head(g4_ctx* ctx, const uint16_t* x, const uint16_t* w_norm, const uint16_t* wt, uint16_t* out) {
  LmHeadOp op;
  op.rows = W / ctx->tp_world;
  op.x = x;
  op.w_norm = w_norm;
  op.wt = wt;
  op.out = out;
  op.scr = ctx->buf.scratch;
  op.g = make_geom(Fmt::BF16, H * 2 / 4, 4);  // pseudo-row = 960 bf16 = 1920 bytes
  if (!geom_ok(op.g, H * 2, 0)) return fail(ctx, G4_ERR_UNSUPPORTED, "lm_head geometry");
  return launch_stream(ctx, op, op.g.slot_bytes, 8, H * 2, op.rows / 4, "lm_head");
}

}  // namespace g4
