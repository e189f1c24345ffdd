// Weight-streaming GEMV engine for decode (batch 1): the shared machinery of every
// projection of the hot path (NVFP4 MLP, FP8/NVFP4 attention projections, bf16 lm_head).
//
// Work decomposition.  A UNIT is R consecutive weight rows (whole rows, so a unit is ONE
// contiguous range of HBM), each cut into Q equal K segments: 8 = R*Q "pseudo-rows" of
// rb bytes.  An ITEM is one or two units (A, B) contracted together by one warp-level
// m16n8k16 MMA stream: MMA rows 0-7 are A's pseudo-rows, rows 8-15 B's, and the
// activation enters through the 8 MMA columns -- column s (< Q) carries segment s of
// A's x slice, column 4+s segment s of B's -- so each pseudo-row's dot product is one
// (row, column) entry of the MMA result.  Per lane-quad, one 16-byte shared-memory load
// covers 64 bytes of a pseudo-row; the physical K order inside those 64 bytes is
// permuted so every MMA B fragment is four CONSECUTIVE activation values (one 8-byte
// load) and every A fragment comes straight from the loaded register.  Pseudo-rows of
// different columns walk the K chunks in rotated order, so the two rows one 8-lane
// shared-memory phase reads never share banks.
//
// Pipeline.  One producer thread streams units into a ring of shared-memory SLOTS with
// 1-D bulk copies (`cp.async.bulk`, L2 evict-first): one copy for a unit's codes and one
// for its block scales, completing on the slot's "full" mbarrier.  NW consumer warps
// split each item's K chunks, decode weights in registers (E2M1 -> f16 with
// `cvt.rn.f16x2.e2m1x2`, times the E4M3 block scale: exact in f16; E4M3 -> f16 exact;
// bf16 as is), accumulate in f32 on the tensor cores, release the slot on its "empty"
// mbarrier and reduce their partial dot products through shared memory; one consumer
// warp per item runs the op's epilogue.  CTAs are persistent (one per SM), taking items
// round robin.
//
// Activations are staged in shared memory as f16 scaled by 2^e (e from the vector's max
// magnitude), so f16 x f16 products are exact in f32 and the scale is undone exactly in
// the epilogue; bf16 weights (lm_head) use bf16 activations unscaled.
#pragma once

#include "g4_common.cuh"

namespace g4 {

enum class Fmt : int { NVFP4 = 0, FP8 = 1, BF16 = 2 };

struct UnitDesc {
  const uint8_t* codes;   // first code byte of the unit's first row (nullptr: absent)
  const uint8_t* scales;  // NVFP4 block scales of the first row (else unused)
  uint32_t code_stride;   // global bytes between consecutive real rows
  uint32_t scale_stride;
  uint32_t xoff;          // activation element offset of segment 0
};

// Geometry shared by every unit of one phase of a launch.
struct UnitGeom {
  uint32_t rb;         // code bytes per pseudo-row (multiple of 64)
  uint32_t sb;         // block-scale bytes per pseudo-row (NVFP4: rb/8, else 0)
  uint32_t q;          // K segments per real row (1, 2 or 4)
  uint32_t seg;        // activation elements per pseudo-row
  uint32_t slot_bytes; // bytes of one slot (multiple of 128)
};

__host__ __device__ inline UnitGeom make_geom(Fmt f, uint32_t rb, uint32_t q) {
  UnitGeom g;
  g.rb = rb;
  g.q = q;
  g.sb = (f == Fmt::NVFP4) ? rb / 8u : 0u;
  g.seg = (f == Fmt::NVFP4) ? rb * 2u : (f == Fmt::FP8 ? rb : rb / 2u);
  g.slot_bytes = (8u * (g.rb + g.sb) + 127u) / 128u * 128u;
  return g;
}

// Warp roles: kComputeWarps compute warps (0 .. kComputeWarps-1), one epilogue warp
// (kComputeWarps), one producer warp (kComputeWarps+1).  "Consumer" threads = compute +
// epilogue warps: they stage activations and run the final epilogue together.
#ifndef G4_COMPUTE_WARPS
#define G4_COMPUTE_WARPS 15
#endif
constexpr int kComputeWarps = G4_COMPUTE_WARPS;
constexpr int kEpilogueWarp = kComputeWarps;
constexpr int kConsumerWarps = kComputeWarps + 1;
constexpr int kMaxSlots = 8;
constexpr int kProducerLanes = 4;  // slot counts are multiples of this
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr uint32_t kBarConsumers = 1;  // named barrier id among consumer warps

// Shared-memory header of a streaming kernel (the x buffer and the slots follow).
struct StreamSmem {
  uint64_t full[16];
  uint64_t empty[16];
  uint64_t redbar[kMaxSlots];                 // all compute warps wrote the buffer's partials
  uint64_t redfree[kMaxSlots];                // the epilogue warp has read the buffer
  float red[kMaxSlots][kComputeWarps][16];   // per-item partial sums, ring of S buffers
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

// Host-side check of a unit geometry against the strides a launch will use.
__host__ inline bool geom_ok(const UnitGeom& g, uint32_t code_stride, uint32_t scale_stride) {
  const bool contiguous = code_stride == g.q * g.rb && (g.sb == 0 || scale_stride == g.q * g.sb);
  return g.rb % 64u == 0 && (g.q == 1 || g.q == 2 || g.q == 4) && contiguous && (8u * g.sb) % 16u == 0;
}

// ------------------------------------------------------------------------ producer
// One copy for the unit's 8 pseudo-rows of codes, one for their block scales.
__device__ __forceinline__ void issue_unit(const UnitDesc& u, const UnitGeom& g, uint8_t* slot,
                                           uint64_t* full, uint64_t policy) {
  const uint32_t cbytes = 8u * g.rb, sbytes = 8u * g.sb;
  mbar_arrive_expect_tx(full, cbytes + sbytes);
  bulk_g2s(slot, u.codes, cbytes, full, policy);
  if (sbytes) bulk_g2s(slot + cbytes, u.scales, sbytes, full, policy);
}

// ------------------------------------------------------------------------ consumer math
// Shared-memory operands of one chunk (64 code bytes of every pseudo-row) of an item.
struct ChunkRegs {
  uint4 qa, qb;        // this lane's 16 code bytes of its A and B pseudo-rows
  uint32_t sca, scb;   // NVFP4: the two E4M3 block scales of those bytes, as f16x2
  uint32_t xaddr;      // shared byte address of this lane's B-fragment activations
  bool xlane;          // this lane carries a live MMA column
};

// Where lane (grp, t) reads chunk c:  its A/B pseudo-rows are row grp of each slot,
// at column s = grp % q; column j of the MMA carries segment j (A) or j-4 (B); each
// column walks the chunks rotated by its segment.
template <Fmt F>
__device__ __forceinline__ ChunkRegs load_chunk(uint32_t sa, uint32_t sbs, bool has_b, const UnitGeom& g, int c,
                                                int lane, uint32_t xa, uint32_t xb, int nch) {
  ChunkRegs r;
  const int grp = lane >> 2, t = lane & 3;
  const int q = static_cast<int>(g.q);
  const int ch = (c + grp % q) % nch;
  const uint32_t roff = grp * g.rb + ch * 64 + t * 16;
  r.qa = lds128(sa + roff);
  r.qb = has_b ? lds128(sbs + roff) : make_uint4(0, 0, 0, 0);
  if constexpr (F == Fmt::NVFP4) {
    const uint32_t soff = 8u * g.rb + grp * g.sb + ch * 8 + t * 2;
    r.sca = cvt_e4m3x2(lds16(sa + soff));
    r.scb = has_b ? cvt_e4m3x2(lds16(sbs + soff)) : 0u;
  } else {
    r.sca = r.scb = 0u;
  }
  const int xs = (grp < 4) ? grp : grp - 4;
  r.xlane = (grp < q) || (grp >= 4 && xs < q && has_b);
  const uint32_t xbase = (grp < 4 ? xa : xb) + xs * g.seg * 2;
  const int xch = (c + xs) % nch;
  constexpr int kElems = (F == Fmt::NVFP4) ? 128 : (F == Fmt::FP8 ? 64 : 32);  // per chunk
  r.xaddr = xbase + (xch * kElems + t * (kElems / 4)) * 2;
  return r;
}

// Contract one chunk: MMA step j accumulates into acc[j & 1] (two independent chains).
template <Fmt F, bool kHasB>
__device__ __forceinline__ void compute_chunk(float (&acc0)[4], float (&acc1)[4], const ChunkRegs& r) {
  if constexpr (F == Fmt::NVFP4) {
    // lane t holds physical k [128ch+32t, +32): byte i -> k 128ch+32t+2i+{0,1}
    uint32_t fa[16], fb[16];
    cvt_e2m1x8(r.qa.x, fa[0], fa[1], fa[2], fa[3]);
    cvt_e2m1x8(r.qa.y, fa[4], fa[5], fa[6], fa[7]);
    cvt_e2m1x8(r.qa.z, fa[8], fa[9], fa[10], fa[11]);
    cvt_e2m1x8(r.qa.w, fa[12], fa[13], fa[14], fa[15]);
    if constexpr (kHasB) {
      cvt_e2m1x8(r.qb.x, fb[0], fb[1], fb[2], fb[3]);
      cvt_e2m1x8(r.qb.y, fb[4], fb[5], fb[6], fb[7]);
      cvt_e2m1x8(r.qb.z, fb[8], fb[9], fb[10], fb[11]);
      cvt_e2m1x8(r.qb.w, fb[12], fb[13], fb[14], fb[15]);
    }
    const uint32_t sal = dup_lo(r.sca), sah = dup_hi(r.sca);
    const uint32_t sbl = dup_lo(r.scb), sbh = dup_hi(r.scb);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t s_a = (j < 4) ? sal : sah;
      const uint32_t a0 = hmul2_u32(fa[2 * j], s_a);
      const uint32_t a2 = hmul2_u32(fa[2 * j + 1], s_a);
      uint32_t a1 = 0u, a3 = 0u;
      if constexpr (kHasB) {
        const uint32_t s_b = (j < 4) ? sbl : sbh;
        a1 = hmul2_u32(fb[2 * j], s_b);
        a3 = hmul2_u32(fb[2 * j + 1], s_b);
      }
      uint2 b = make_uint2(0, 0);
      if (r.xlane) b = lds64(r.xaddr + 8 * j);
      if (j & 1)
        mma_f16(acc1, a0, a1, a2, a3, b.x, b.y);
      else
        mma_f16(acc0, a0, a1, a2, a3, b.x, b.y);
    }
  } else if constexpr (F == Fmt::FP8) {
    // lane t holds physical k [64ch+16t, +16): bytes 4j..4j+3 -> k 64ch+16t+4j+{0..3}
    const uint32_t wa[4] = {r.qa.x, r.qa.y, r.qa.z, r.qa.w};
    const uint32_t wb[4] = {r.qb.x, r.qb.y, r.qb.z, r.qb.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a0 = cvt_e4m3x2(static_cast<uint16_t>(wa[j] & 0xFFFFu));
      const uint32_t a2 = cvt_e4m3x2(static_cast<uint16_t>(wa[j] >> 16));
      uint32_t a1 = 0u, a3 = 0u;
      if constexpr (kHasB) {
        a1 = cvt_e4m3x2(static_cast<uint16_t>(wb[j] & 0xFFFFu));
        a3 = cvt_e4m3x2(static_cast<uint16_t>(wb[j] >> 16));
      }
      uint2 b = make_uint2(0, 0);
      if (r.xlane) b = lds64(r.xaddr + 8 * j);
      if (j & 1)
        mma_f16(acc1, a0, a1, a2, a3, b.x, b.y);
      else
        mma_f16(acc0, a0, a1, a2, a3, b.x, b.y);
    }
  } else {
    // bf16: lane t holds physical k [32ch+8t, +8): word i -> k 32ch+8t+2i+{0,1}
    const uint32_t wa[4] = {r.qa.x, r.qa.y, r.qa.z, r.qa.w};
    const uint32_t wb[4] = {r.qb.x, r.qb.y, r.qb.z, r.qb.w};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint2 b = make_uint2(0, 0);
      if (r.xlane) b = lds64(r.xaddr + 8 * j);
      if (j & 1)
        mma_bf16(acc1, wa[2 * j], wb[2 * j], wa[2 * j + 1], wb[2 * j + 1], b.x, b.y);
      else
        mma_bf16(acc0, wa[2 * j], wb[2 * j], wa[2 * j + 1], wb[2 * j + 1], b.x, b.y);
    }
  }
}

// This warp's share of an item: chunks warp, warp+NW, ... with the next chunk's shared
// loads issued before the current chunk's math.
template <Fmt F, bool kHasB>
__device__ __forceinline__ void item_mma(float (&acc)[4], uint32_t sa, uint32_t sbs, const UnitGeom& g, int warp,
                                         int lane, uint32_t xa, uint32_t xb) {
  const int nch = static_cast<int>(g.rb / 64u);
  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
  int c = warp;
  if (c < nch) {
    ChunkRegs cur = load_chunk<F>(sa, sbs, kHasB, g, c, lane, xa, xb, nch);
    while (true) {
      const int cn = c + kComputeWarps;
      ChunkRegs nxt;
      if (cn < nch) nxt = load_chunk<F>(sa, sbs, kHasB, g, cn, lane, xa, xb, nch);
      compute_chunk<F, kHasB>(acc0, acc1, cur);
      if (cn >= nch) break;
      cur = nxt;
      c = cn;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = acc0[i] + acc1[i];
}

// ------------------------------------------------------------------------ kernel body
// Op interface (all __device__ const members):
//   static constexpr Fmt kFmt; static constexpr int kPhases;
//   int items(int phase); UnitGeom geom(int phase); UnitDesc unit(int phase, int item, int half);
//   void stage(StreamSmem&, uint8_t* xbuf, int phase, int tid)      [consumer threads]
//   void item_epilogue(StreamSmem&, int phase, int item, int lane, float v)  [one warp]
//       lanes 0-7: pseudo-rows of unit A, lanes 8-15: pseudo-rows of unit B
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
      mbar_init(&sm.empty[s], kComputeWarps);
    }
    for (int s = 0; s < kMaxSlots; ++s) {
      mbar_init(&sm.redbar[s], kComputeWarps);
      mbar_init(&sm.redfree[s], 1);
    }
    sm.is_last = 0;
    sm.failed = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------ producer
    // kProducerLanes lanes issue in parallel (one thread issues a bulk copy only every
    // few hundred ns): lane j owns the units k with k % kProducerLanes == j, i.e. slots
    // j, j + kProducerLanes, ...  Every lane walks the same unit sequence.
    if (lane < kProducerLanes) {
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
            if (k % kProducerLanes == static_cast<uint32_t>(lane)) {
              const uint32_t s = k % S, use = k / S;
              if (use > 0 && !mbar_wait_suspend(&sm.empty[s], (use - 1) & 1u, deadline)) {
                ok = false;
                break;
              }
              issue_unit(u, g, slots + s * slot_bytes, &sm.full[s], pol);
            }
            ++k;
          }
        }
      }
      if (!ok) atomicOr(op.status(), DEV_ERR_TIMEOUT_MBAR);
      // drain: no bulk copy may still target this CTA's shared memory when it exits
      const uint32_t first = (k > S) ? k - S : 0u;
      for (uint32_t q = first; q < k; ++q)
        if (q % kProducerLanes == static_cast<uint32_t>(lane))
          mbar_wait_suspend(&sm.full[q % S], (q / S) & 1u, deadline + budget_ns);
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
    const int grp = lane >> 2, t = lane & 3;
    const int sq = grp % static_cast<int>(g.q);
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
      // Reduction buffer ring: item i uses buffer i % S.  Compute warps write their
      // partial sums and arrive on redbar (release); the epilogue warp waits on it
      // (acquire), sums, marks the buffer free on redfree and runs the item's epilogue.
      // Compute warps release a slot as soon as their own math is done, never wait for
      // one another, and only wait for a buffer to be free before reusing it S items on.
      const int rbuf = static_cast<int>(items_done % S);
      const uint32_t rpar = (items_done / S) & 1u;
      if (warp != kEpilogueWarp) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
          ok = mbar_wait(&sm.full[sa_i], ua_use & 1u, deadline);
          if (ok && has_b) ok = mbar_wait(&sm.full[sb_i], ub_use & 1u, deadline);
        }
        if (ok) {
          const uint32_t sa = smem_u32(slots + sa_i * slot_bytes);
          const uint32_t sbb = has_b ? smem_u32(slots + sb_i * slot_bytes) : sa;
          const uint32_t xa = smem_u32(xbuf) + 2u * ua.xoff;
          const uint32_t xb = smem_u32(xbuf) + 2u * (has_b ? ub.xoff : ua.xoff);
          if (has_b)
            item_mma<Op::kFmt, true>(acc, sa, sbb, g, warp, lane, xa, xb);
          else
            item_mma<Op::kFmt, false>(acc, sa, sbb, g, warp, lane, xa, xb);
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.empty[sa_i]);
          if (has_b) mbar_arrive(&sm.empty[sb_i]);
        }
        if (items_done >= S && ok && !mbar_wait(&sm.redfree[rbuf], rpar ^ 1u, deadline)) ok = false;
        // pseudo-row grp of A sits at (row grp, column sq), of B at (row grp+8, column 4+sq)
        if (t == (sq >> 1)) sm.red[rbuf][warp][grp] = (sq & 1) ? acc[1] : acc[0];
        if (t == 2 + (sq >> 1)) sm.red[rbuf][warp][8 + grp] = (sq & 1) ? acc[3] : acc[2];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.redbar[rbuf]);
      } else {
        if (ok && !mbar_wait(&sm.redbar[rbuf], rpar, deadline, true)) ok = false;
        float v = 0.f;
        if (lane < 16) {
#pragma unroll
          for (int w = 0; w < kComputeWarps; ++w) v += sm.red[rbuf][w][lane];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.redfree[rbuf]);
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

// Sum of the q pseudo-row values of each real row of a unit, in the epilogue warp:
// lane l (< 8/q) receives real row l of unit A, lane 8/q + l real row l of unit B.
// Lanes hold v = pseudo-row values (0-7: A, 8-15: B); the sum order is fixed.
__device__ __forceinline__ float sum_pseudo_rows(float v, int lane, int q) {
  const int rows = 8 / q;
  // source lanes of output lane l: unit (l / rows), real row (l % rows)
  const int unit = lane / rows, r = lane % rows;
  const int src0 = unit * 8 + r * q;
  float s = 0.f;
  for (int i = 0; i < q; ++i) {
    const float x = __shfl_sync(0xffffffffu, v, (src0 + i) & 31);
    s += x;
  }
  return s;
}

// Grid-wide wait among the consumer threads of every CTA of a cooperative launch:
// arrive on `counter`, then spin (bounded) until `target` arrivals.  Returns false on
// timeout.  The op resets the counter once every CTA has passed.
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

// Block-wide (consumer threads) sum / max; `scratch` is a 32-float region.
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
__device__ __forceinline__ int stage_rmsnorm(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                             int n, uint16_t* xs, bool as_f16, float* scratch) {
  // 8 elements (16 bytes) per thread and step; n % 8 == 0, pointers 16-byte aligned
  const int tid = threadIdx.x;
  constexpr int kMaxGroups = 2;  // n <= 2 * 8 * kConsumerThreads
  uint4 xv[kMaxGroups], wv[kMaxGroups];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxGroups; ++k) {
    const int gi = tid + k * kConsumerThreads;
    if (gi * 8 < n) {
      xv[k] = __ldg(reinterpret_cast<const uint4*>(x) + gi);
      wv[k] = __ldg(reinterpret_cast<const uint4*>(w) + gi);
      const uint32_t xw[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = bf16_to_f32(static_cast<uint16_t>(xw[i] & 0xFFFFu));
        const float b = bf16_to_f32(static_cast<uint16_t>(xw[i] >> 16));
        ss = __fadd_rn(ss, __fmul_rn(a, a));
        ss = __fadd_rn(ss, __fmul_rn(b, b));
      }
    }
  }
  const float r = rms_factor(consumer_sum(ss, scratch), n);
  float y[kMaxGroups][8];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxGroups; ++k) {
    const int gi = tid + k * kConsumerThreads;
    if (gi * 8 < n) {
      const uint32_t xw[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
      const uint32_t ww[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint16_t xb = static_cast<uint16_t>((i & 1) ? xw[i >> 1] >> 16 : xw[i >> 1] & 0xFFFFu);
        const uint16_t wb = static_cast<uint16_t>((i & 1) ? ww[i >> 1] >> 16 : ww[i >> 1] & 0xFFFFu);
        y[k][i] = round_bf16(__fmul_rn(__fmul_rn(bf16_to_f32(xb), r), bf16_to_f32(wb)));
        amax = fmaxf(amax, fabsf(y[k][i]));
      }
    }
  }
  int e = 0;
  float sc = 1.0f;
  if (as_f16) {
    e = f16_scale_exponent(consumer_max(amax, scratch + 32));
    sc = ldexpf(1.0f, e);
  }
#pragma unroll
  for (int k = 0; k < kMaxGroups; ++k) {
    const int gi = tid + k * kConsumerThreads;
    if (gi * 8 < n) {
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = as_f16 ? pack_u16x2(f32_to_f16(y[k][2 * i] * sc), f32_to_f16(y[k][2 * i + 1] * sc))
                      : pack_u16x2(f32_to_bf16(y[k][2 * i]), f32_to_bf16(y[k][2 * i + 1]));
      reinterpret_cast<uint4*>(xs)[gi] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  return e;
}

}  // namespace g4
