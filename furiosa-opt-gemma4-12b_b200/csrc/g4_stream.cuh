// Weight-streaming GEMV engine for decode (batch 1): the shared machinery of every
// projection of the hot path (NVFP4 MLP, FP8/NVFP4 attention projections, bf16 lm_head).
//
// Work decomposition.  A weight matrix is cut into UNITS of 8 rows x KC columns.  An
// ITEM is one or two units (A, B) contracted together by one warp-level
// m16n8k16 MMA stream: MMA rows 0-7 are unit A's rows, rows 8-15 unit B's, and the
// activation enters as MMA column 0 (for A) and column 1 (for B), so A and B may use
// different slices of x.  Per lane-quad, one 16-byte shared-memory load covers 64 bytes
// of a row; the physical K order inside those 64 bytes is permuted so that every MMA
// B-fragment is four CONSECUTIVE activation values (one 8-byte load) and every A
// fragment comes straight from the loaded register (no shuffles).
//
// Pipeline.  One producer warp streams units into a ring of shared-memory SLOTS with
// 1-D bulk copies (`cp.async.bulk`, L2 evict-first), completing on per-slot "full"
// mbarriers; NW consumer warps split each item's K range, decode weights in registers
// (E2M1 -> f16 with `cvt.rn.f16x2.e2m1x2`, times the E4M3 block scale, exact in f16;
// E4M3 -> f16 exact; bf16 as is), accumulate in f32 on the tensor cores, release the
// slot on its "empty" mbarrier, and reduce their partial dot products through shared
// memory.  One consumer warp per item then runs the op's epilogue.  CTAs are
// persistent (one per SM), taking items round robin.
//
// Activations are staged in shared memory as f16 scaled by 2^e (e from the vector's max
// magnitude), so f16 x f16 products are exact in f32 and the scale is undone exactly in
// the epilogue; bf16 weights (lm_head) use bf16 activations unscaled.
#pragma once

#include "g4_common.cuh"

namespace g4 {

enum class Fmt : int { NVFP4 = 0, FP8 = 1, BF16 = 2 };

struct UnitDesc {
  const uint8_t* codes;   // row 0 of the unit, first code byte of its K range (nullptr: absent)
  const uint8_t* scales;  // NVFP4 block scales of row 0 (else unused)
  uint32_t code_stride;   // global bytes between consecutive rows
  uint32_t scale_stride;
  uint32_t xoff;          // activation element offset of the unit's K range
};

// Geometry shared by every unit of one launch.
struct UnitGeom {
  uint32_t rb;          // code bytes per row per unit (multiple of 64)
  uint32_t sb;          // block-scale bytes per row per unit (NVFP4: rb/8, else 0)
  uint32_t pitch;       // shared-memory bytes between code rows (pitch % 128 == 64)
  uint32_t spitch;      // shared-memory bytes between scale rows
  uint32_t scale_block; // 1: scales of the 8 rows are one contiguous copy of 8*sb bytes
  uint32_t slot_bytes;  // bytes of one slot (multiple of 128)
};

__host__ __device__ inline UnitGeom make_geom(uint32_t rb, uint32_t sb, bool scale_rows_contiguous) {
  UnitGeom g;
  g.rb = rb;
  g.sb = sb;
  g.pitch = rb + ((64u + 128u - (rb % 128u)) % 128u);
  g.scale_block = (sb % 16u != 0u && scale_rows_contiguous) ? 1u : 0u;
  g.spitch = g.scale_block ? sb : ((sb + 15u) / 16u) * 16u;
  uint32_t bytes = 8u * g.pitch + 8u * g.spitch;
  g.slot_bytes = (bytes + 127u) / 128u * 128u;
  return g;
}

constexpr int kConsumerWarps = 10;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr uint32_t kBarConsumers = 1;  // named barrier id among consumer warps

// Shared-memory header of a streaming kernel (slots and the x buffer follow).
struct StreamSmem {
  uint64_t full[16];
  uint64_t empty[16];
  float red[2][kConsumerWarps][16];
  float scratch[64];        // op-defined (norm reductions, flags)
  int xexp;                 // activation scale exponent: x16 = x * 2^xexp
  int is_last;              // this CTA completed the launch (runs the final epilogue)
  int failed;               // a bounded wait gave up
  int pad_;
};

struct StreamLayout {
  uint32_t nslots;
  uint32_t x_bytes;  // bytes reserved for the activation buffer
  uint32_t slot_off; // offset of slot 0 from the dynamic smem base
  uint32_t total;    // dynamic shared memory bytes
};

__host__ __device__ inline StreamLayout make_layout(uint32_t slot_bytes, uint32_t nslots, uint32_t x_bytes) {
  StreamLayout l;
  l.nslots = nslots;
  l.x_bytes = (x_bytes + 127u) / 128u * 128u;
  uint32_t hdr = (static_cast<uint32_t>(sizeof(StreamSmem)) + 127u) / 128u * 128u;
  l.slot_off = hdr + l.x_bytes;
  l.total = l.slot_off + nslots * slot_bytes;
  return l;
}

// ------------------------------------------------------------------------ producer
// Issues the copies of one unit into `slot` and arms its full barrier.
__device__ __forceinline__ void issue_unit(const UnitDesc& u, const UnitGeom& g, uint8_t* slot,
                                           uint64_t* full, uint64_t policy, Fmt fmt) {
  uint32_t bytes = 8u * g.rb + ((fmt == Fmt::NVFP4) ? 8u * g.sb : 0u);
  mbar_arrive_expect_tx(full, bytes);
#pragma unroll 1
  for (int r = 0; r < 8; ++r)
    bulk_g2s(slot + r * g.pitch, u.codes + static_cast<size_t>(r) * u.code_stride, g.rb, full, policy);
  if (fmt == Fmt::NVFP4) {
    uint8_t* sdst = slot + 8u * g.pitch;
    if (g.scale_block) {
      bulk_g2s(sdst, u.scales, 8u * g.sb, full, policy);
    } else {
#pragma unroll 1
      for (int r = 0; r < 8; ++r)
        bulk_g2s(sdst + r * g.spitch, u.scales + static_cast<size_t>(r) * u.scale_stride, g.sb, full,
                 policy);
    }
  }
}

// ------------------------------------------------------------------------ consumer math
// Contract chunk `c` (64 code bytes per row) of the item's slots into acc.
// xa/xb: shared addresses of the activation slices of units A and B (f16 or bf16).
template <Fmt F>
__device__ __forceinline__ void chunk_mma(float (&acc)[4], uint32_t sa, uint32_t sbs, bool has_b,
                                          const UnitGeom& g, int c, int lane, uint32_t xaddr) {
  const int grp = lane >> 2, t = lane & 3;
  const bool xlane = grp < 2;
  const uint32_t roff = grp * g.pitch + c * 64 + t * 16;
  const uint4 qa = lds128(sa + roff);
  uint4 qb = make_uint4(0, 0, 0, 0);
  if (has_b) qb = lds128(sbs + roff);
  if constexpr (F == Fmt::NVFP4) {
    // lane t holds physical k [128c+32t, +32): byte i -> k 128c+32t+2i+{0,1}
    const uint32_t soff = 8u * g.pitch + grp * g.spitch + c * 8 + t * 2;
    const uint32_t sca = cvt_e4m3x2(lds16(sa + soff));
    const uint32_t scb = has_b ? cvt_e4m3x2(lds16(sbs + soff)) : 0u;
    uint32_t fa[16], fb[16];
    cvt_e2m1x8(qa.x, fa[0], fa[1], fa[2], fa[3]);
    cvt_e2m1x8(qa.y, fa[4], fa[5], fa[6], fa[7]);
    cvt_e2m1x8(qa.z, fa[8], fa[9], fa[10], fa[11]);
    cvt_e2m1x8(qa.w, fa[12], fa[13], fa[14], fa[15]);
    cvt_e2m1x8(qb.x, fb[0], fb[1], fb[2], fb[3]);
    cvt_e2m1x8(qb.y, fb[4], fb[5], fb[6], fb[7]);
    cvt_e2m1x8(qb.z, fb[8], fb[9], fb[10], fb[11]);
    cvt_e2m1x8(qb.w, fb[12], fb[13], fb[14], fb[15]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t s_a = (j < 4) ? dup_lo(sca) : dup_hi(sca);
      const uint32_t s_b = (j < 4) ? dup_lo(scb) : dup_hi(scb);
      const uint32_t a0 = hmul2_u32(fa[2 * j], s_a);
      const uint32_t a2 = hmul2_u32(fa[2 * j + 1], s_a);
      const uint32_t a1 = hmul2_u32(fb[2 * j], s_b);
      const uint32_t a3 = hmul2_u32(fb[2 * j + 1], s_b);
      uint2 b = make_uint2(0, 0);
      if (xlane) b = lds64(xaddr + (c * 128 + t * 32 + 4 * j) * 2);
      mma_f16(acc, a0, a1, a2, a3, b.x, b.y);
    }
  } else if constexpr (F == Fmt::FP8) {
    // lane t holds physical k [64c+16t, +16): bytes 4j..4j+3 -> k 64c+16t+4j+{0..3}
    const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
    const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a0 = cvt_e4m3x2(static_cast<uint16_t>(wa[j] & 0xFFFFu));
      const uint32_t a2 = cvt_e4m3x2(static_cast<uint16_t>(wa[j] >> 16));
      const uint32_t a1 = cvt_e4m3x2(static_cast<uint16_t>(wb[j] & 0xFFFFu));
      const uint32_t a3 = cvt_e4m3x2(static_cast<uint16_t>(wb[j] >> 16));
      uint2 b = make_uint2(0, 0);
      if (xlane) b = lds64(xaddr + (c * 64 + t * 16 + 4 * j) * 2);
      mma_f16(acc, a0, a1, a2, a3, b.x, b.y);
    }
  } else {
    // bf16: lane t holds physical k [32c+8t, +8): word i -> k 32c+8t+2i+{0,1}
    const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
    const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint2 b = make_uint2(0, 0);
      if (xlane) b = lds64(xaddr + (c * 32 + t * 8 + 4 * j) * 2);
      mma_bf16(acc, wa[2 * j], wb[2 * j], wa[2 * j + 1], wb[2 * j + 1], b.x, b.y);
    }
  }
}

// ------------------------------------------------------------------------ kernel body
// Op interface (all __device__ const members):
//   static constexpr Fmt kFmt; static constexpr int kPhases;
//   int items(int phase); UnitGeom geom(int phase); UnitDesc unit(int phase, int item, int half);
//   void stage(StreamSmem&, uint8_t* xbuf, int phase, int tid)      [consumer threads]
//   void item_epilogue(StreamSmem&, int phase, int item, int lane, float v)  [one warp]
//   bool has_final(); void final_epilogue(StreamSmem&, uint8_t* xbuf, int tid) [last CTA]
//   uint32_t* done_counter(); uint32_t* status();
//   bool between_phases(StreamSmem&, int phase, uint64_t deadline)  [consumer threads]
template <class Op>
__device__ __forceinline__ void stream_body(const Op& op, const StreamLayout& lay, uint32_t slot_bytes,
                                            uint64_t budget_ns) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  StreamSmem& sm = *reinterpret_cast<StreamSmem*>(smem_raw);
  uint8_t* xbuf = smem_raw + ((sizeof(StreamSmem) + 127) / 128 * 128);
  uint8_t* slots = smem_raw + lay.slot_off;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const uint32_t S = lay.nslots;
  const uint64_t deadline = global_ns() + budget_ns;

  if (tid == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.is_last = 0;
    sm.failed = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t k = 0;
      bool ok = true;
      for (int ph = 0; ph < Op::kPhases && ok; ++ph) {
        const int n = op.items(ph);
        const UnitGeom g = op.geom(ph);
        for (int it = cta; it < n && ok; it += G) {
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            const UnitDesc u = op.unit(ph, it, half);
            if (u.codes == nullptr) continue;
            const uint32_t s = k % S, use = k / S;
            if (use > 0 && !mbar_wait(&sm.empty[s], (use - 1) & 1u, deadline)) {
              ok = false;
              break;
            }
            issue_unit(u, g, slots + s * slot_bytes, &sm.full[s], pol, Op::kFmt);
            ++k;
          }
        }
      }
      if (!ok) atomicOr(op.status(), DEV_ERR_TIMEOUT_MBAR);
      // drain: no bulk copy may still target this CTA's shared memory when it exits
      const uint32_t first = (k > S) ? k - S : 0u;
      for (uint32_t q = first; q < k; ++q) mbar_wait(&sm.full[q % S], (q / S) & 1u, deadline + budget_ns);
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  uint32_t k = 0, items_done = 0;
  bool ok = true;
  for (int ph = 0; ph < Op::kPhases; ++ph) {
    if (ph > 0) {
      if (!op.between_phases(sm, ph, deadline)) ok = false;
    }
    op.stage(sm, xbuf, ph, tid);
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (sm.failed) ok = false;
    const int n = op.items(ph);
    const UnitGeom g = op.geom(ph);
    for (int it = cta; it < n; it += G) {
      const UnitDesc ua = op.unit(ph, it, 0);
      const UnitDesc ub = op.unit(ph, it, 1);
      const bool has_b = ub.codes != nullptr;
      const uint32_t sa_i = k % S, ua_use = k / S;
      ++k;
      uint32_t sb_i = 0, ub_use = 0;
      if (has_b) {
        sb_i = k % S;
        ub_use = k / S;
        ++k;
      }
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok) {
        ok = mbar_wait(&sm.full[sa_i], ua_use & 1u, deadline);
        if (ok && has_b) ok = mbar_wait(&sm.full[sb_i], ub_use & 1u, deadline);
      }
      if (ok) {
        const uint32_t sa = smem_u32(slots + sa_i * slot_bytes);
        const uint32_t sbb = has_b ? smem_u32(slots + sb_i * slot_bytes) : sa;
        const int grp = lane >> 2;
        const uint32_t xaddr = smem_u32(xbuf) + 2u * ((grp == 0) ? ua.xoff : (has_b ? ub.xoff : ua.xoff));
        const int nch = static_cast<int>(g.rb / 64u);
#pragma unroll 1
        for (int c = warp; c < nch; c += kConsumerWarps) chunk_mma<Op::kFmt>(acc, sa, sbb, has_b, g, c, lane, xaddr);
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.empty[sa_i]);
        if (has_b) mbar_arrive(&sm.empty[sb_i]);
      }
      const int buf = items_done & 1;
      if ((lane & 3) == 0) {
        sm.red[buf][warp][lane >> 2] = acc[0];       // row g of A, column 0
        sm.red[buf][warp][8 + (lane >> 2)] = acc[3]; // row g of B, column 1
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      if (warp == static_cast<int>(items_done % kConsumerWarps)) {
        float v = 0.f;
        if (lane < 16) {
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) v += sm.red[buf][w][lane];
        }
        if (ok) op.item_epilogue(sm, ph, it, lane, v);
      }
      ++items_done;
    }
    if (!ok && tid == 0) atomicOr(op.status(), DEV_ERR_TIMEOUT_MBAR);
  }

  if (op.has_final()) {
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0) {
      __threadfence();
      const uint32_t old = atom_add_acq_rel_gpu(op.done_counter(), 1u);
      sm.is_last = (old == static_cast<uint32_t>(G - 1)) ? 1 : 0;
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (sm.is_last) {
      __threadfence();
      op.final_epilogue(sm, xbuf, tid);
      named_bar_sync(kBarConsumers, kConsumerThreads);
      if (tid == 0) {
        *op.done_counter() = 0u;
        __threadfence();
      }
    }
  }
}

// Grid-wide wait among the consumer threads of every CTA of a cooperative launch:
// arrive on `counter`, then spin (bounded) until `target` arrivals.  Returns false on
// timeout.  Counter targets grow monotonically within a launch; the op resets it.
__device__ __forceinline__ bool grid_wait(uint32_t* counter, uint32_t target, uint64_t deadline,
                                          uint32_t* status, StreamSmem& sm) {
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (threadIdx.x == 0) {
    __threadfence();
    atom_add_release_gpu(counter, 1u);
    uint32_t spins = 0;
    int fail = 0;
    while (ld_acquire_gpu(counter) < target) {
      if ((++spins & 63u) == 0u && global_ns() > deadline) {
        fail = 1;
        atomicOr(status, DEV_ERR_TIMEOUT_GRID);
        break;
      }
    }
    sm.failed = fail;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  return sm.failed == 0;
}

// Block-wide (consumer threads) sum; `slot` is a 64-float scratch region.
__device__ __forceinline__ float consumer_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (lane == 0) scratch[warp] = v;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) s += scratch[w];
  return s;
}
__device__ __forceinline__ float consumer_max(float v, float* scratch) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (lane == 0) scratch[warp] = v;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) s = fmaxf(s, scratch[w]);
  return s;
}

// RMSNorm of a bf16 vector (global) into shared memory as scaled f16 (or bf16) MMA
// operands, by the consumer threads.  Returns the scale exponent (0 for bf16 output).
// out_bf16 (optional): also write the normalised bf16 values to global.
__device__ __forceinline__ int stage_rmsnorm(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                             int n, uint16_t* xs, bool as_f16, float* scratch) {
  const int tid = threadIdx.x;
  float ss = 0.f;
  for (int i = tid; i < n; i += kConsumerThreads) {
    const float v = bf16_to_f32(x[i]);
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  const float r = rms_factor(consumer_sum(ss, scratch), n);
  float amax = 0.f;
  for (int i = tid; i < n; i += kConsumerThreads) {
    const float y = round_bf16(__fmul_rn(__fmul_rn(bf16_to_f32(x[i]), r), bf16_to_f32(w[i])));
    xs[i] = f32_to_bf16(y);
    amax = fmaxf(amax, fabsf(y));
  }
  if (!as_f16) {
    named_bar_sync(kBarConsumers, kConsumerThreads);
    return 0;
  }
  const int e = f16_scale_exponent(consumer_max(amax, scratch + 32));
  const float sc = ldexpf(1.0f, e);
  for (int i = tid; i < n; i += kConsumerThreads) xs[i] = f32_to_f16(bf16_to_f32(xs[i]) * sc);
  named_bar_sync(kBarConsumers, kConsumerThreads);
  return e;
}

}  // namespace g4
