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
// Pipeline.  A producer warp streams items into a ring of shared-memory item SLOTS with
// 1-D bulk copies (`cp.async.bulk`, L2 evict-first): per unit one copy of its codes and
// one of its block scales, all four of an item completing on the slot's "full" mbarrier.
// The compute warps split each item's K chunks, decode weights in registers (E2M1 -> f16
// with `cvt.rn.f16x2.e2m1x2`, times the E4M3 block scale: exact in f16; E4M3 -> f16
// exact; bf16 as is), accumulate in f32 on the tensor cores, release the slot on its
// "empty" mbarrier and leave their partial dot products in a shared-memory reduction
// buffer; a couple of items later one of them (in rotation) adds the partials up and runs
// the op's epilogue for the item.  CTAs are persistent (one per SM), taking items round
// robin.
//
// Activations are staged in shared memory as f16 scaled by 2^e (e from the vector's max
// magnitude), so f16 x f16 products are exact in f32 and the scale is undone exactly in
// the epilogue; bf16 weights (lm_head) use bf16 activations unscaled.
#pragma once

#include "g4_common.cuh"
#include "g4_internal.h"

namespace g4 {

enum class Fmt : int { NVFP4 = 0, FP8 = 1, BF16 = 2 };

struct UnitDesc {
  const uint8_t* codes;   // first code byte of the unit's first row (nullptr: absent)
  const uint8_t* scales;  // NVFP4 block scales of the first row (else unused)
  uint32_t code_stride;   // global bytes between consecutive real rows
  uint32_t scale_stride;
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

// Warp roles: kComputeWarps compute warps (0 .. kComputeWarps-1) and one producer warp
// (kComputeWarps).  The compute warps ("consumers") also stage activations, run the item
// epilogues (item j by warp j % kComputeWarps, kEpiLag items after contracting it) and
// the final epilogue.  Sixteen warps keep four per scheduler, so a thread may use 128
// registers; the decode/MMA loop needs about 110 to run without stalls.
#ifndef G4_COMPUTE_WARPS
#define G4_COMPUTE_WARPS 15
#endif
constexpr int kComputeWarps = G4_COMPUTE_WARPS;
constexpr int kConsumerWarps = kComputeWarps;
constexpr uint32_t kEpiLag = 2;  // items between contracting an item and running its epilogue
constexpr int kMaxSlots = 8;       // unit slots of a launch's layout (two per item slot)
constexpr int kRedSlots = 8;       // reduction buffers (ring over items)
constexpr int kProducerLanes = 4;  // issuing lanes; item slots = a multiple of this
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr uint32_t kBarConsumers = 1;  // named barrier id among consumer warps
// the vectorised staging and tails give each consumer thread 8 elements of a [3840] vector
static_assert(kConsumerThreads * 8 >= 3840, "too few consumer threads for an [H] vector");

// Shared-memory header of a streaming kernel (the x buffer and the slots follow).
struct StreamSmem {
  uint64_t full[kMaxSlots / 2];               // item slot filled (both units landed)
  uint64_t empty[kMaxSlots / 2];              // every compute warp is done with the item slot
  uint64_t deadline;                          // global_ns() limit of the launch's bounded waits
  float red[kRedSlots][kComputeWarps][16];    // per-item partial sums, ring of buffers
  float scratch[64];        // op-defined (norm reductions, flags)
  int xexp;                 // activation scale exponent: x16 = x * 2^xexp
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

// Chunks (64 code bytes of every pseudo-row) one compute warp handles per item, at most:
// enough for pseudo-rows of up to 45 chunks (2880 bytes).
constexpr int kMaxChunks = (45 + kComputeWarps - 1) / kComputeWarps;

// Host-side check of a unit geometry against the strides a launch will use.
__host__ inline bool geom_ok(const UnitGeom& g, uint32_t code_stride, uint32_t scale_stride) {
  const bool contiguous = code_stride == g.q * g.rb && (g.sb == 0 || scale_stride == g.q * g.sb);
  return g.rb % 64u == 0 && g.rb / 64u <= 45u &&
         (g.q == 1 || g.q == 2 || g.q == 4) && contiguous && (8u * g.sb) % 16u == 0;
}

// ------------------------------------------------------------------ activation layout
// The activation vector sits in shared memory permuted so that each lane's B-fragment
// values of one chunk are 16-byte "pairs" (two MMA steps) it reads with one 16-byte
// load.  Element k of K lies in segment s = k / seg; inside the segment, chunk c holds
// kElems elements: lane t owns elements [t*kElems/4, (t+1)*kElems/4) of the chunk, in
// pairs of 8.  Pair p of lane t is stored at ((p ^ (c & 1)) * 32 + t * 8) elements into
// the chunk (the XOR only when a lane has 2+ pairs), so the two pseudo-rows one 8-lane
// shared-memory phase serves -- always one chunk apart -- read different bank halves.
template <Fmt F>
struct FmtTraits;
template <>
struct FmtTraits<Fmt::NVFP4> {
  static constexpr uint32_t kElems = 128, kSteps = 8, kPairs = 4;
};
template <>
struct FmtTraits<Fmt::FP8> {
  static constexpr uint32_t kElems = 64, kSteps = 4, kPairs = 2;
};
template <>
struct FmtTraits<Fmt::BF16> {
  static constexpr uint32_t kElems = 32, kSteps = 2, kPairs = 1;
};

struct XLayout {
  uint32_t seg;       // activation elements per K segment
  uint32_t log_elems; // log2(elements per chunk)
  uint32_t swz;       // 1: pair index XOR chunk parity
};

__host__ __device__ inline XLayout make_xlayout(Fmt f, const UnitGeom& g) {
  XLayout x;
  x.seg = g.seg;
  x.log_elems = (f == Fmt::NVFP4) ? 7u : (f == Fmt::FP8 ? 6u : 5u);
  x.swz = (f == Fmt::BF16) ? 0u : 1u;
  return x;
}

// Shared-memory element index of activation element k (at most 4 segments).
__device__ __forceinline__ uint32_t x_pos(uint32_t k, const XLayout& xl) {
  uint32_t s = 0, kk = k;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (kk >= xl.seg) {
      kk -= xl.seg;
      ++s;
    }
  }
  const uint32_t c = kk >> xl.log_elems, i = kk & ((1u << xl.log_elems) - 1u);
  const uint32_t lane_elems_log = xl.log_elems - 2u;
  const uint32_t t = i >> lane_elems_log, w = i & ((1u << lane_elems_log) - 1u);
  const uint32_t p = (w >> 3) ^ (xl.swz & c);
  return s * xl.seg + (c << xl.log_elems) + p * 32u + t * 8u + (w & 7u);
}

// ------------------------------------------------------------------------ producer
// One item into one item slot: unit A at the slot start, unit B one unit stride later;
// per unit one copy for its 8 pseudo-rows of codes and one for their block scales, all
// completing on the slot's single "full" barrier.
__device__ __forceinline__ void issue_item(const UnitDesc& a, const UnitDesc& b, const UnitGeom& g, uint8_t* slot,
                                           uint32_t unit_stride, uint64_t* full, uint64_t policy) {
  const uint32_t cbytes = 8u * g.rb, sbytes = 8u * g.sb;
  mbar_arrive_expect_tx(full, 2u * (cbytes + sbytes));
  bulk_g2s(slot, a.codes, cbytes, full, policy);
  if (sbytes) bulk_g2s(slot + cbytes, a.scales, sbytes, full, policy);
  bulk_g2s(slot + unit_stride, b.codes, cbytes, full, policy);
  if (sbytes) bulk_g2s(slot + unit_stride + cbytes, b.scales, sbytes, full, policy);
}

// ------------------------------------------------------------------------ consumer math
// Item-invariant shared-memory offsets of one lane for one phase.  Lane (grp, t) loads
// bytes [ch*64 + t*16, +16) of pseudo-row grp of the A (and B) slot, where the chunk
// ch = c + rot is this warp's chunk c rotated by the row's MMA column, and feeds MMA
// column grp with the matching activation fragment.
//   q >= 2: pseudo-row grp is segment grp % q; column = segment, rotation = segment.
//   q == 1: one segment; even/odd rows take columns 0/1 and rotations 0/1, so the two
//           rows of every 8-lane phase are one chunk (64 bytes) apart.
// B's pseudo-rows use column + 4.  Columns no row uses get an arbitrary (in-bounds)
// activation fragment: MMA columns are independent, so their sums are never read.
struct LanePlan {
  uint32_t roff[kMaxChunks];  // code bytes from the slot base
  uint32_t soff[kMaxChunks];  // block-scale bytes from the slot base (NVFP4)
  uint32_t xe[kMaxChunks];    // activation bytes of even pairs from the x buffer
  uint32_t xo[kMaxChunks];    // ... of odd pairs
  int nc;                     // chunks of this warp
  int col;                    // MMA column of this lane's A pseudo-row (B: col + 4)
};

template <Fmt F>
__device__ __forceinline__ LanePlan make_plan(const UnitGeom& g, int warp, int lane, bool has_b) {
  using T = FmtTraits<F>;
  LanePlan pl;
  const int grp = lane >> 2, t = lane & 3;
  const int q = static_cast<int>(g.q), nch = static_cast<int>(g.rb / 64u);
  const int rot = (q == 1) ? (grp & 1) : (grp & (q - 1));
  pl.col = rot;
  // the activation this lane supplies: column grp (A) or grp - 4 (B)
  const int cg = grp & 3;
  bool live = cg < ((q == 1) ? 2 : q);
  if (grp >= 4 && !has_b) live = false;
  const int xs = (live && q > 1) ? cg : 0;
  const int xr = live ? cg : 0;
  int n = 0;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = warp + i * kComputeWarps;
    pl.roff[i] = pl.soff[i] = pl.xe[i] = pl.xo[i] = 0u;
    if (c < nch) {
      int ch = c + rot;
      if (ch >= nch) ch -= nch;
      int xc = c + xr;
      if (xc >= nch) xc -= nch;
      pl.roff[i] = static_cast<uint32_t>(grp) * g.rb + static_cast<uint32_t>(ch) * 64u + static_cast<uint32_t>(t) * 16u;
      pl.soff[i] = 8u * g.rb + static_cast<uint32_t>(grp) * g.sb + static_cast<uint32_t>(ch) * 8u + static_cast<uint32_t>(t) * 2u;
      const uint32_t sw = (T::kPairs > 1) ? static_cast<uint32_t>(xc & 1) : 0u;
      const uint32_t base = 2u * (static_cast<uint32_t>(xs) * g.seg + static_cast<uint32_t>(xc) * T::kElems +
                                  static_cast<uint32_t>(t) * 8u);
      pl.xe[i] = base + sw * 64u;
      pl.xo[i] = base + (sw ^ 1u) * 64u;
      ++n;
    }
  }
  pl.nc = n;
  return pl;
}

// Code and scale registers of one chunk.
struct ChunkRegs {
  uint4 qa, qb;       // this lane's 16 code bytes of its A and B pseudo-rows
  uint32_t sca, scb;  // NVFP4: their two E4M3 block scales, as f16x2
};

template <Fmt F, bool kHasB>
__device__ __forceinline__ ChunkRegs load_chunk(uint32_t sa, uint32_t sb, uint32_t roff, uint32_t soff) {
  ChunkRegs r;
  r.qa = lds128(sa + roff);
  r.qb = kHasB ? lds128(sb + roff) : make_uint4(0u, 0u, 0u, 0u);
  if constexpr (F == Fmt::NVFP4) {
    r.sca = cvt_e4m3x2(lds16(sa + soff));
    r.scb = kHasB ? cvt_e4m3x2(lds16(sb + soff)) : 0u;
  } else {
    r.sca = r.scb = 0u;
  }
  return r;
}

// Contract one chunk: MMA step j accumulates into acc[j & 1] (two independent chains).
// Step j uses this lane's elements 4j..4j+3 of the chunk: A from the decoded code
// registers, B = activation pair j/2 (one 16-byte load feeds steps 2p and 2p+1).
template <Fmt F, bool kHasB>
__device__ __forceinline__ void compute_chunk(float (&acc0)[4], float (&acc1)[4], const ChunkRegs& r, uint32_t xe,
                                              uint32_t xo) {
  using T = FmtTraits<F>;
  if constexpr (F == Fmt::NVFP4) {
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
    const uint32_t sbl = kHasB ? dup_lo(r.scb) : 0u, sbh = kHasB ? dup_hi(r.scb) : 0u;
#pragma unroll
    for (int p = 0; p < static_cast<int>(T::kPairs); ++p) {
      const uint4 x = lds128(((p & 1) ? xo : xe) + static_cast<uint32_t>(p >> 1) * 128u);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * p + h;
        const uint32_t s_a = (j < 4) ? sal : sah;
        const uint32_t a0 = hmul2_u32(fa[2 * j], s_a);
        const uint32_t a2 = hmul2_u32(fa[2 * j + 1], s_a);
        uint32_t a1 = 0u, a3 = 0u;
        if constexpr (kHasB) {
          const uint32_t s_b = (j < 4) ? sbl : sbh;
          a1 = hmul2_u32(fb[2 * j], s_b);
          a3 = hmul2_u32(fb[2 * j + 1], s_b);
        }
        if (h)
          mma_f16(acc1, a0, a1, a2, a3, x.z, x.w);
        else
          mma_f16(acc0, a0, a1, a2, a3, x.x, x.y);
      }
    }
  } else if constexpr (F == Fmt::FP8) {
    const uint32_t wa[4] = {r.qa.x, r.qa.y, r.qa.z, r.qa.w};
    const uint32_t wb[4] = {r.qb.x, r.qb.y, r.qb.z, r.qb.w};
#pragma unroll
    for (int p = 0; p < static_cast<int>(T::kPairs); ++p) {
      const uint4 x = lds128(((p & 1) ? xo : xe) + static_cast<uint32_t>(p >> 1) * 128u);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * p + h;
        const uint32_t a0 = cvt_e4m3x2(static_cast<uint16_t>(wa[j] & 0xFFFFu));
        const uint32_t a2 = cvt_e4m3x2(static_cast<uint16_t>(wa[j] >> 16));
        uint32_t a1 = 0u, a3 = 0u;
        if constexpr (kHasB) {
          a1 = cvt_e4m3x2(static_cast<uint16_t>(wb[j] & 0xFFFFu));
          a3 = cvt_e4m3x2(static_cast<uint16_t>(wb[j] >> 16));
        }
        if (h)
          mma_f16(acc1, a0, a1, a2, a3, x.z, x.w);
        else
          mma_f16(acc0, a0, a1, a2, a3, x.x, x.y);
      }
    }
  } else {
    const uint4 x = lds128(xe);
    mma_bf16(acc0, r.qa.x, r.qb.x, r.qa.y, r.qb.y, x.x, x.y);
    mma_bf16(acc1, r.qa.z, r.qb.z, r.qa.w, r.qb.w, x.z, x.w);
  }
}

// This warp's share of an item: its pl.nc chunks, each chunk's codes loaded right before
// its math (a one-chunk look-ahead costs more registers than it hides latency).
template <Fmt F, bool kHasB>
__device__ __forceinline__ void item_mma(float (&acc)[4], uint32_t sa, uint32_t sb, uint32_t xbase,
                                         const LanePlan& pl) {
  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    if (i < pl.nc) {
      const ChunkRegs cur = load_chunk<F, kHasB>(sa, sb, pl.roff[i], pl.soff[i]);
      compute_chunk<F, kHasB>(acc0, acc1, cur, xbase + pl.xe[i], xbase + pl.xo[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = acc0[i] + acc1[i];
}

// ------------------------------------------------------------------------ kernel body
// Op interface (all __device__ const members):
//   static constexpr Fmt kFmt; static constexpr int kPhases;
//   int items(int phase); UnitGeom geom(int phase); UnitDesc unit(int phase, int item, int half)
//       (every item is two units, A = half 0 and B = half 1);
//   void stage(StreamSmem&, uint8_t* xbuf, int phase, int tid, const XLayout&)  [consumers]
//   void item_epilogue(StreamSmem&, int phase, int item, int lane, float v)  [one warp]
//       lanes 0-7: pseudo-rows of unit A, lanes 8-15: pseudo-rows of unit B
//   bool has_final(); void final_epilogue(StreamSmem&, uint8_t* xbuf, int tid) [CTA 0, after all]
//   uint32_t* done_counter(); uint32_t* status();
//   bool between_phases(StreamSmem&, int phase, uint64_t deadline)  [consumer threads]
//   void prefetch_l2(int cta, int lane)   [producer warp, at start: L2 prefetches of the
//       staging and final-epilogue operands that no kernel writes]
// `unit_bytes` is the launch's unit slot size (>= every phase's 8 * (rb + sb), a multiple
// of 128); lay.nslots unit slots form lay.nslots / 2 item slots.
template <class Op>
__device__ __forceinline__ void stream_body(const Op& op, const StreamLayout& lay, uint32_t unit_bytes,
                                            uint64_t budget_ns) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  StreamSmem& sm = *reinterpret_cast<StreamSmem*>(smem_raw);
  uint8_t* xbuf = smem_raw + ((sizeof(StreamSmem) + 127) / 128 * 128);
  uint8_t* slots = smem_raw + lay.slot_off;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const uint32_t S = lay.nslots / 2;           // item slots (a multiple of kProducerLanes)
  const uint32_t item_bytes = 2u * unit_bytes;
  const uint64_t deadline = global_ns() + budget_ns;

  if (tid == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kComputeWarps);
    }
    sm.failed = 0;
    sm.deadline = deadline;
    fence_mbar_init();
  }
  __syncthreads();
  // The next launch may start taking SMs as this grid's CTAs exit; before its
  // griddepcontrol.wait it only streams weights and prefetches, which no kernel writes.
  pdl_launch_dependents();

  if (warp == kComputeWarps) {
    // ------------------------------------------------------------------ producer
    // First pull the staging and final-epilogue operands that no kernel writes (norm
    // weights, scales) into L2 (all lanes), so the staging and the tail find them there.
    // kProducerLanes lanes issue in parallel.  Every lane walks the same item sequence
    // k = 0, 1, ...; lane j issues the items k with k % kProducerLanes == j, into item
    // slots j, j + kProducerLanes, ... (k % S), counting its own refills of them.
    op.prefetch_l2(cta, lane);
    if (lane < kProducerLanes) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t k = 0, s = static_cast<uint32_t>(lane), use = 0, mine = 0;
      bool ok = true;
      for (int ph = 0; ph < Op::kPhases && ok; ++ph) {
        const int n = op.items(ph);
        const UnitGeom g = op.geom(ph);
        for (int it = cta; it < n; it += G, ++k) {
          if ((k & (kProducerLanes - 1)) != static_cast<uint32_t>(lane)) continue;
          if (use > 0 && !mbar_wait_suspend(&sm.empty[s], (use - 1) & 1u, deadline)) {
            ok = false;
            break;
          }
          issue_item(op.unit(ph, it, 0), op.unit(ph, it, 1), g, slots + s * item_bytes, unit_bytes, &sm.full[s], pol);
          ++mine;
          s += kProducerLanes;
          if (s >= S) {
            s -= S;
            ++use;
          }
        }
      }
      if (!ok) atomicOr(op.status(), DEV_ERR_TIMEOUT_MBAR);
      // drain: no bulk copy may still target this CTA's shared memory when it exits.
      // This lane's r-th slot (lane + r*kProducerLanes) took fills r, r + S/lanes, ...
      const uint32_t per = S / kProducerLanes;
      for (uint32_t r = 0; r < per; ++r) {
        if (mine <= r) break;
        const uint32_t fills = (mine - r - 1) / per + 1;
        mbar_wait_suspend(&sm.full[lane + r * kProducerLanes], (fills - 1) & 1u, deadline + budget_ns);
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  // The lane plan depends on the geometry alone: work it out while the previous kernel
  // on the stream finishes (and, for later phases, while the grid barrier completes).
  LanePlan pl = make_plan<Op::kFmt>(op.geom(0), warp, lane, true);
  // Everything below may read what the previous kernel on the stream wrote (activations,
  // residual, this context's scratch counters and buffers).
  pdl_wait();
  uint32_t slot = 0, spar = 0;  // next item slot to consume, its fill parity
  uint32_t done = 0;            // items this CTA has contracted, all phases (reduction ring index)
  bool ok = true;
  const int grp = lane >> 2, t = lane & 3;
  const uint32_t xbase = smem_u32(xbuf), slot0 = smem_u32(slots);
  const uint32_t red0 = smem_u32(&sm.red[0][warp][grp]);  // this lane's slot in reduction buffer 0
  constexpr uint32_t kRedStride = sizeof(float) * kComputeWarps * 16;
  // Epilogue of this CTA's item j (global index; m = its index within phase ph).  Item j
  // sits in item slot j % S and leaves its partial sums in reduction buffer j % kRedSlots;
  // every compute warp writes its partials before it arrives on the slot's "empty"
  // barrier (a release), so that barrier's completion for item j (phase j / S) also says
  // "all partials are in".  Add them in fixed warp order and run the op's epilogue.
  // Buffers need no "free" signal: item j + kRedSlots writes buffer j % kRedSlots only
  // after item j + kRedSlots - S was released by every warp, and the warp running item
  // j's epilogue does so before it contracts item j + kEpiLag + 1 <= j + kRedSlots - S.
  static_assert(kRedSlots >= kMaxSlots / 2 + static_cast<int>(kEpiLag) + 1, "reduction ring too short");
  auto epilogue = [&](int ph, uint32_t j, uint32_t m) {
    const uint32_t rb = j % kRedSlots;
    if (ok && !mbar_wait_suspend(&sm.empty[j % S], (j / S) & 1u, deadline)) ok = false;
    float v = 0.f;
    if (lane < 16) {
#pragma unroll
      for (int w = 0; w < kComputeWarps; ++w) v += sm.red[rb][w][lane];
    }
    __syncwarp();
    if (ok) op.item_epilogue(sm, ph, cta + static_cast<int>(m) * G, lane, v);
  };
  for (int ph = 0; ph < Op::kPhases; ++ph) {
    if (ph > 0) {
      pl = make_plan<Op::kFmt>(op.geom(ph), warp, lane, true);
      if (!op.between_phases(sm, ph, deadline)) ok = false;
    }
    const UnitGeom g = op.geom(ph);
    op.stage(sm, xbuf, ph, tid, make_xlayout(Op::kFmt, g));
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (sm.failed) ok = false;
    const int n = op.items(ph);
    const uint32_t count = (cta < n) ? static_cast<uint32_t>((n - cta + G - 1) / G) : 0u;
    const uint32_t first = done;
    // pseudo-row grp of A sits at (row grp, column col), of B at (row grp+8, column 4+col)
    const bool st_a = t == (pl.col >> 1), st_b = t == 2 + (pl.col >> 1), odd = (pl.col & 1) != 0;
    for (uint32_t m = 0; m < count; ++m) {
      // Compute warps write their partial sums, then release the item slot (one arrive
      // per warp), and never wait for one another.
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok && !mbar_wait_suspend(&sm.full[slot], spar, deadline)) ok = false;
      if (ok) {
        const uint32_t sa = slot0 + slot * item_bytes;
        item_mma<Op::kFmt, true>(acc, sa, sa + unit_bytes, xbase, pl);
      }
      const uint32_t ra = red0 + (done % kRedSlots) * kRedStride;
      sts_f32_if(ra, odd ? acc[1] : acc[0], st_a);
      sts_f32_if(ra + 8u * sizeof(float), odd ? acc[3] : acc[2], st_b);
      __syncwarp();
      mbar_arrive_if(&sm.empty[slot], lane == 0);
      if (++slot == S) {
        slot = 0;
        spar ^= 1u;
      }
      ++done;
      if (m >= kEpiLag) {
        const uint32_t j = done - 1u - kEpiLag;
        if (j % kComputeWarps == static_cast<uint32_t>(warp)) epilogue(ph, j, m - kEpiLag);
      }
    }
    // the phase's last kEpiLag epilogues, before anything reads its results
    for (uint32_t m = (count > kEpiLag ? count - kEpiLag : 0u); m < count; ++m) {
      const uint32_t j = first + m;
      if (j % kComputeWarps == static_cast<uint32_t>(warp)) epilogue(ph, j, m);
    }
    if (!ok) atomicOr(op.status(), DEV_ERR_TIMEOUT_MBAR);
  }

  if (op.has_final()) {
    // CTA 0 runs the final epilogue once every other CTA has published its results: they
    // each add 1 to the done counter (release, no round trip) and exit; CTA 0 polls it
    // (acquire) right after its own items, while the others finish.
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (cta != 0) {
      if (tid == 0) red_add_release_gpu(op.done_counter(), 1u);
      return;
    }
    if (tid == 0) {
      uint32_t spins = 0;
      int fail = 0;
      while (ld_acquire_gpu(op.done_counter()) < static_cast<uint32_t>(G - 1)) {
        if ((++spins & 63u) == 0u && global_ns() > deadline) {
          fail = 1;
          atomicOr(op.status(), DEV_ERR_TIMEOUT_GRID);
          break;
        }
      }
      sm.failed = fail;
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (!sm.failed) op.final_epilogue(sm, xbuf, tid);
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0) *op.done_counter() = 0u;  // visible to the next launch at kernel end
  }
}

// Sum of the q pseudo-row values of each real row of a unit, in the warp running the
// item's epilogue:
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
    red_add_release_gpu(counter, 1u);  // release covers this CTA's writes (ordered by the bar.sync)
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

// Tensor parallelism: one-shot all-reduce of an [H] f32 vector over peer memory, run by
// all consumer threads of the CTA doing the final epilogue.  Thread tid < H/8 holds
// elements [8 tid, 8 tid + 8) of this rank's partial in y and receives the sum over all
// ranks, added in rank order so that every rank computes the identical vector.  Each
// value goes to its slot in every rank's exchange buffer as one 64-bit word {value,
// launch number}; the reader polls its own words until all carry this launch's number.
// An 8-byte store is seen whole or not at all, so neither a fence nor a flag is needed.
// The half of the buffer alternates with the launch number: a rank one launch ahead
// never overwrites words a peer still reads, and cannot get two ahead, because it needs
// that peer's words of the launch in between.  Returns false (and sets
// DEV_ERR_TIMEOUT_PEER) if a peer's values do not arrive before the launch's deadline.
__device__ __forceinline__ bool peer_allreduce(const PeerXch& x, uint32_t* launch_ctr, float (&y)[8], int tid,
                                               uint32_t* status, StreamSmem& sm) {
  constexpr int kH = 3840;
  if (tid == 0) {
    sm.scratch[63] = __uint_as_float(*launch_ctr + 1u);
    sm.failed = 0;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint32_t e = __float_as_uint(sm.scratch[63]);
  if (tid < kH / 8) {
    const uint64_t tag = static_cast<uint64_t>(e) << 32;
    const size_t half = static_cast<size_t>(e & 1u) * kMaxTp * kH;
    uint64_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = tag | __float_as_uint(y[i]);
    for (int p = 0; p < x.world; ++p) {
      uint64_t* dst = x.buf[p] + half + static_cast<size_t>(x.rank) * kH + 8 * tid;
#pragma unroll
      for (int j = 0; j < 4; ++j) st_relaxed_sys_v2u64(dst + 2 * j, w[2 * j], w[2 * j + 1]);
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int q = 0; q < x.world && ok; ++q) {
      const uint64_t* src = x.buf[x.rank] + half + static_cast<size_t>(q) * kH + 8 * tid;
      uint64_t v[8];
      uint32_t spins = 0;
      while (true) {
        bool all = true;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ld_relaxed_sys_v2u64(src + 2 * j, v[2 * j], v[2 * j + 1]);
          all = all && static_cast<uint32_t>(v[2 * j] >> 32) == e && static_cast<uint32_t>(v[2 * j + 1] >> 32) == e;
        }
        if (all) break;
        if ((++spins & 255u) == 0u && global_ns() > sm.deadline) {
          ok = false;
          break;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __uint_as_float(static_cast<uint32_t>(v[i]));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = acc[i];
    if (!ok) {
      sm.failed = 1;
      atomicOr(status, DEV_ERR_TIMEOUT_PEER);
    }
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (tid == 0) *launch_ctr = e;
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

// Block-wide (consumer threads) sum of `s` and max of `m` in one barrier round, for the
// first reduction of a launch (nothing reads scratch[0..63] concurrently).
__device__ __forceinline__ float2 consumer_sum_max(float s, float m, float* scratch) {
  s = warp_sum(s);
  m = warp_max(m);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    scratch[warp] = s;
    scratch[32 + warp] = m;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  float ts = 0.f, tm = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    ts += scratch[w];
    tm = fmaxf(tm, scratch[32 + w]);
  }
  return make_float2(ts, tm);
}

// RMSNorm of a bf16 vector (global) into shared memory as scaled f16 (or bf16) MMA
// operands, by the consumer threads.  Returns the scale exponent (0 for bf16 output).
__device__ __forceinline__ int stage_rmsnorm(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                             int n, uint16_t* xs, bool as_f16, float* scratch, const XLayout& xl) {
  // 8 elements (16 bytes) per thread and step; n % 8 == 0, pointers 16-byte aligned
  const int tid = threadIdx.x;
  constexpr int kMaxGroups = 2;  // n <= 2 * 8 * kConsumerThreads
  uint4 xv[kMaxGroups], wv[kMaxGroups];
  float ss = 0.f, pm = 0.f;  // sum of x^2; max |x * w|
#pragma unroll
  for (int k = 0; k < kMaxGroups; ++k) {
    const int gi = tid + k * kConsumerThreads;
    if (gi * 8 < n) {
      xv[k] = __ldg(reinterpret_cast<const uint4*>(x) + gi);
      wv[k] = __ldg(reinterpret_cast<const uint4*>(w) + gi);
      const uint32_t xw[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
      const uint32_t ww[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = bf16_to_f32(static_cast<uint16_t>(xw[i] & 0xFFFFu));
        const float b = bf16_to_f32(static_cast<uint16_t>(xw[i] >> 16));
        ss = __fadd_rn(ss, __fmul_rn(a, a));
        ss = __fadd_rn(ss, __fmul_rn(b, b));
        pm = fmaxf(pm, fabsf(a * bf16_to_f32(static_cast<uint16_t>(ww[i] & 0xFFFFu))));
        pm = fmaxf(pm, fabsf(b * bf16_to_f32(static_cast<uint16_t>(ww[i] >> 16))));
      }
    }
  }
  // One reduction round for both: the f16 scale only needs an upper bound of max |y|,
  // and |y| = |bf16(x * r * w)| <= max|x * w| * r * (1 + 2^-7).
  const float2 red = consumer_sum_max(ss, pm, scratch);
  const float r = rms_factor(red.x, n);
  float y[kMaxGroups][8];
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
      }
    }
  }
  int e = 0;
  float sc = 1.0f;
  if (as_f16) {
    e = f16_scale_exponent(red.y * r * 1.01f);
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
      *reinterpret_cast<uint4*>(xs + x_pos(static_cast<uint32_t>(gi) * 8u, xl)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  return e;
}

}  // namespace g4
