// decoder_feedforward on the 5th-generation tensor cores (single GPU): the NVFP4 GeGLU MLP
// block of one decode token, ONE persistent launch of one CTA per SM (drop-in for
// ops::decoder_feedforward, src/ops.rs:213-253; same math as mlp_kernel in g4_mlp.cu).
//
// Weights never pass through the CUDA cores.  `tcgen05.mma .kind::mxf4nvf4` with 16-element
// E4M3 block scales consumes the checkpoint's E2M1 codes and scales as they are:
//   D[128 rows][16] += (sfa * A[128 rows][64 k]) . (sfb * B[16][64 k])^T      (f32 in TMEM)
// A = 128 weight rows (phase 0: 64 gate + the same 64 up rows; phase 1: 128 down rows),
// streamed by TMA (2-D tiles of 128 rows x 256 k, 128-byte swizzle) through a 10-stage
// shared-memory ring; B = the bf16 activation written as 16 NVFP4 "pieces", two bits of
// a block-aligned fixed-point expansion each (split_block):
//   x = sum_n 2^(gmax - 127 - 2n) * sfb * e2m1_n,   e2m1_n in {0, 0.5, 1, 1.5} * sign,
// exact for every element within 2^24 of its 16-element block's largest.  The epilogue
// adds D's 16 columns with their powers of two.
//
// Work split.  Phase p has T tiles of 128 rows x S stages of 256 k.  The T*S (tile, stage)
// pairs are cut into 148 contiguous ranges (stream-K): CTA c owns pairs
// [c*W/G, (c+1)*W/G).  A CTA's run inside one tile is a segment; its MMAs accumulate in
// one of two TMEM accumulators.  Both phases finish a tile in the CTA holding its first
// k-stages, adding the other parts' partial sums in k order: phase 0 goes on to GeGLU -> h,
// phase 1 stores the tile's 128 sums; the last CTA to finish loads the 3840 sums (not every
// segment's partials) and runs the RMSNorm/residual tail.  Values one CTA hands to another inside a
// launch (gate/up partial sums, h) are words tagged with the launch's number: a reader
// re-reads a word until its tag is current, so neither a flag nor a grid barrier stands
// between the phases, and a value already written costs one round trip.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer, 12-15 write each stage's weight
// scales into tensor memory (tcgen05.st, one lane quarter each: the tensor pipe only runs
// MMAs), 4-7 accumulator epilogue, 2-11 stage the activation pieces (and run the phase
// ends and the tail).
#include <cuda.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {
namespace tc {

constexpr int kStages = 10;       // shared-memory ring of weight stages
constexpr int kMaxCtaSeg = 4;     // segments (tile runs) in one CTA's range, per phase
constexpr uint32_t kWaitGroup = 4; // stages the MMA issuer takes per wait (< kStages)
constexpr int kPieces = 16;       // activation pieces = MMA N
constexpr int kKStage = 256;      // k per stage (128 bytes of codes per row)
constexpr int kMaxLocal = 16;     // k-stages of activation pieces resident per phase
constexpr int kMaxSeg = 8;        // segments per tile (checked on the host)
constexpr int kThreads = 512;
constexpr int kGroupWarp0 = 2;    // warps 2..11: staging group
constexpr int kGroupThreads = 320;
constexpr int kEpiWarp0 = 4;      // warps 4..7: accumulator epilogue (TMEM lane quarters 0..3)
constexpr int kSfWarp0 = 12;      // warps 12..15: weight scales into TMEM (lane quarters 0..3)
constexpr uint32_t kBarGroup = 1, kBarEpi = 2;
// tensor memory columns: D0 [0,16) D1 [16,32); weight scales, 16 per ring slot (4 per
// 64-k step, replicated layout) [32,192); activation scales, 4 per 64-k step [192,448)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSfa = 32, kColSfb = kColSfa + 16 * kStages;
static_assert(kColSfb + 4 * 4 * kMaxLocal <= kTmemCols, "tensor memory columns");
constexpr uint32_t kStageTx = 16384 + 2048;
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kPieces >> 3) << 17) | (8u << 24);

struct __align__(1024) Smem {
  uint8_t a[kStages][16384];          // weight tiles, 128 rows x 128 B, 128-byte swizzle
  uint8_t bpc[kMaxLocal][2048];       // pieces: [k-stage][16 rows][128 B], 128-byte swizzle
  uint8_t sfst[kStages][2048];        // stage scales as loaded: [128 rows][16 B]
  uint8_t sblk[kMaxLocal * 16];       // activation block scales (ue4m3), one per 16-k block
  uint64_t full[kStages], sfready[kStages], empty[kStages];
  uint64_t dfull[2], dempty[2];
  uint64_t pieces;                    // completes once per phase: activation staged
  uint64_t deadline;
  float pw[2][kPieces];               // piece column scales per phase
  float xchg[64];
  float red[16], red2[16];
  int seg_n[2];                       // this CTA's segments per phase, in processing order:
  int seg_tile[2][kMaxCtaSeg];        //   tile, first and end k-stage
  int seg_k0[2][kMaxCtaSeg], seg_k1[2][kMaxCtaSeg];
  uint32_t tmem_base;
  int abort_flag;     // some wait gave up (any warp may set it)
  int grp_abort;      // snapshot of abort_flag taken before a staging-group barrier
  int last_flag;
  uint32_t tag;       // this launch's tag (launches finished + 1) for the words CTAs exchange
  uint32_t xch_tag;   // tensor parallel: this launch's tag in the peer exchange
  int xch_failed;
  float gate_gs, up_gs;
};

struct Args {
  uint16_t* residual;
  const uint16_t* pre_w;
  const uint16_t* post_w;
  const uint16_t* layer_scalar;
  const float* up_gs;
  const float* gate_gs;
  const float* down_gs;
  Scratch* scr;
  float* part;       // [H] down-projection sums
  float* seg;        // [H] the down projection's sums (each down tile's 128, k order)
  uint64_t* ptag;    // [(T0 + T1) * kMaxSeg * 128] segment partials {f32 bits, launch tag}
  uint32_t* htag;    // [L] h {bf16 bits, launch tag in the high half}
  int lrows;         // intermediate rows of this rank's shard
  uint64_t budget_ns;
  PeerXch xch;       // tensor parallel: every rank's exchange buffer (world <= 1: one GPU)
};

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1u) << 16) |
         (static_cast<uint64_t>(1024u >> 4) << 32) | (static_cast<uint64_t>(1u) << 46) |
         (static_cast<uint64_t>(2u) << 61);
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                       uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_commit_at(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t da, uint64_t db, uint32_t sfa, uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(da), "l"(db), "r"(kIdesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
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
// this warp's 32 lanes x 16 columns from registers (tc_wait_st makes them complete)
__device__ __forceinline__ void tc_st16_nowait(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  tc_st16_nowait(taddr, r);
  tc_wait_st();
}
// Activation scales of the phase's resident k-stages into tensor memory, by the four
// epilogue warps (one per lane quarter): 64-k step q at columns kColSfb + 4q .. +3, the
// replicated layout with rows n < 32 (the 16 pieces share one scale per block) in column 0.
__device__ __forceinline__ void write_sfb(const Smem& sm, uint32_t tbase, int nk, int quarter) {
  const uint32_t* words = reinterpret_cast<const uint32_t*>(sm.sblk);  // step q = blocks 4q..4q+3
  for (int q0 = 0; q0 < nk; q0 += 4) {
    uint32_t r[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      r[4 * j] = (q0 + j < nk) ? words[q0 + j] : 0u;
      r[4 * j + 1] = r[4 * j + 2] = r[4 * j + 3] = 0u;
    }
    tc_st16_nowait(tbase + kColSfb + 4u * q0 + (static_cast<uint32_t>(32 * quarter) << 16), r);
  }
  tc_wait_st();
}

// two f32 -> e2m1x2 (lo in the low nibble), saturating
__device__ __forceinline__ uint32_t f32x2_to_e2m1(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\t.reg .b16 h;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tmov.b16 h, {t, 0};\n\t"
      "cvt.u32.u16 %0, h;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t f32_to_e4m3(float v) {
  uint16_t s;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(s) : "f"(v), "f"(v));
  return s & 0xFFu;
}
__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
  const uint32_t h = cvt_e4m3x2(static_cast<uint16_t>(byte & 0xFFu));
  return __half2float(__ushort_as_half(static_cast<uint16_t>(h & 0xFFFFu)));
}
__device__ __forceinline__ float pow2f(int e) { return ldexpf(1.0f, e); }
__device__ __forceinline__ bool aborted(const Smem& sm) { return *reinterpret_cast<const volatile int*>(&sm.abort_flag) != 0; }
// The staging group decides on the abort state together: one thread samples it before
// a group barrier and everyone reads the sample after it.
__device__ __forceinline__ bool group_aborted(Smem& sm, int g);

// ue4m3 code of 2^k, -9 <= k <= 0 (k >= -6 normal, below that subnormal)
__device__ __forceinline__ uint32_t ue4m3_pow2(int k) { return k >= -6 ? static_cast<uint32_t>(k + 7) << 3 : 1u << (k + 9); }

// x >> s with shifts of 32 or more giving 0 (the PTX shift clamps its amount)
__device__ __forceinline__ uint32_t shr_clamped(uint32_t x, uint32_t s) {
  uint32_t r;
  asm("shr.b32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(s));
  return r;
}
// w[b] = byte b of a, b, c, d (in that order, a's in the low byte)
__device__ __forceinline__ void byte_transpose4(uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t (&w)[4]) {
  const uint32_t abl = __byte_perm(a, b, 0x5140), abh = __byte_perm(a, b, 0x7362);
  const uint32_t cdl = __byte_perm(c, d, 0x5140), cdh = __byte_perm(c, d, 0x7362);
  w[0] = __byte_perm(abl, cdl, 0x5410);
  w[1] = __byte_perm(abl, cdl, 0x7632);
  w[2] = __byte_perm(abh, cdh, 0x5410);
  w[3] = __byte_perm(abh, cdh, 0x7632);
}

// Writes one 16-element block of bf16 values (two per word, element 2i in the low half)
// as kPieces NVFP4 pieces at local k-stage kl, block bs of the stage.
//   Every element is aligned to the block's reference exponent eb as a 32-bit fixed-point
//   magnitude T (|x| = T * 2^(eb - 158)); piece n holds bits (31-2n, 30-2n) of T, used as
//   e2m1 codes 0..3 (= 0, 0.5, 1, 1.5) with the element's sign, block scale 2^(eb - gmax)
//   and column scale 2^(gmax - 127 - 2n).  Exact for elements within 2^24 of the block's
//   largest; smaller ones are truncated there (below f32 rounding of the dot product).
//   gmax >= every element's biased exponent; eb >= gmax - 9 keeps the block scale in range.
__device__ __forceinline__ void split_block(const uint32_t (&xw)[8], int gmax, Smem& sm, int kl, int bs) {
  // exponent fields of both halves of each word (a zero exponent -- zero or subnormal --
  // counts as 1, the subnormals' scale); eb = the block's largest, at least gmax - 9
  uint32_t ew[8], emax2 = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ew[i] = (xw[i] >> 7) & 0x00FF00FFu;
    emax2 = __vmaxu2(emax2, ew[i]);
  }
  int eb = max(max(static_cast<int>(emax2 & 0xFFu), static_cast<int>(emax2 >> 16)), 1);
  eb = max(eb, gmax - 9);
  sm.sblk[kl * 16 + bs] = static_cast<uint8_t>(ue4m3_pow2(eb - gmax));  // the same for all pieces
  // T = significand in the top byte, shifted right by eb - e (shifts of 32 or more give 0);
  // the sign of element i goes to bit 4 (i % 8) + 3 of its half's code words
  uint32_t T[16], sgn_lo = 0u, sgn_hi = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t sig = (xw[i] & 0x007F007Fu) | (__vsetne2(ew[i], 0u) << 7);
    const int e0 = max(static_cast<int>(ew[i] & 0xFFu), 1), e1 = max(static_cast<int>(ew[i] >> 16), 1);
    T[2 * i] = shr_clamped(__byte_perm(sig, 0u, 0x0444), static_cast<uint32_t>(eb - e0));
    T[2 * i + 1] = shr_clamped(__byte_perm(sig, 0u, 0x2444), static_cast<uint32_t>(eb - e1));
    const uint32_t sg = ((xw[i] >> 12) & 0x8u) | ((xw[i] >> 24) & 0x80u);
    if (i < 4) sgn_lo |= sg << (8 * i); else sgn_hi |= sg << (8 * (i - 4));
  }
  // Byte transpose: EA[b] = byte b of T of elements 0, 2, 4, 6 and OA[b] of elements
  // 1, 3, 5, 7 (EB, OB: elements 8..15).  Z interleaves them per byte: low nibble from the
  // even element, high nibble from the odd one, so the digit at bits 2p, 2p+1 of byte b of
  // T (piece 15 - 4b - p) of both elements is one shift and mask away; the code word of
  // piece n has element 2j's digit in nibble 2j and element 2j+1's in nibble 2j+1.
  uint32_t EA[4], OA[4], EB[4], OB[4];
  byte_transpose4(T[0], T[2], T[4], T[6], EA);
  byte_transpose4(T[1], T[3], T[5], T[7], OA);
  byte_transpose4(T[8], T[10], T[12], T[14], EB);
  byte_transpose4(T[9], T[11], T[13], T[15], OB);
  uint8_t* codes = sm.bpc[kl];
  const uint32_t half = static_cast<uint32_t>(bs & 1) * 8u, chunk = static_cast<uint32_t>(bs >> 1);
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t zl0 = (EA[b] & 0x0F0F0F0Fu) | ((OA[b] << 4) & 0xF0F0F0F0u);
    const uint32_t zh0 = ((EA[b] >> 4) & 0x0F0F0F0Fu) | (OA[b] & 0xF0F0F0F0u);
    const uint32_t zl1 = (EB[b] & 0x0F0F0F0Fu) | ((OB[b] << 4) & 0xF0F0F0F0u);
    const uint32_t zh1 = ((EB[b] >> 4) & 0x0F0F0F0Fu) | (OB[b] & 0xF0F0F0F0u);
    const uint32_t words[4][2] = {{zl0, zl1}, {zl0 >> 2, zl1 >> 2}, {zh0, zh1}, {zh0 >> 2, zh1 >> 2}};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t n = static_cast<uint32_t>(15 - 4 * b - p);
      const uint32_t off = n * 128u + ((chunk ^ (n & 7u)) << 4) + half;
      *reinterpret_cast<uint2*>(codes + off) =
          make_uint2((words[p][0] & 0x33333333u) | sgn_lo, (words[p][1] & 0x33333333u) | sgn_hi);
    }
  }
}

// Tensor-parallel sum of the down projection over NVLink peer memory, by the last CTA of
// every rank (512 threads; thread t < 480 holds outputs [8t, 8t + 8)): the same one-shot
// protocol as the streaming kernels' exchange.  Each value goes to every rank's buffer as
// one 64-bit word {f32, launch tag} with a relaxed system-scope store; a rank re-reads its
// own buffer until every rank's words carry this launch's tag and adds them in rank
// order, so the ranks' results are bit-identical.  The halves of the buffer alternate
// with the tag, so a rank one launch ahead never overwrites words a peer still reads.
// The wait is bounded (DEV_ERR_TIMEOUT_PEER).
__device__ __forceinline__ bool peer_allreduce_tc(const PeerXch& x, uint32_t* launch_ctr, float (&y)[8], int tid,
                                                  uint32_t* status, Smem& sm) {
  if (tid == 0) {
    sm.xch_tag = *launch_ctr + 1u;
    sm.xch_failed = 0;
  }
  __syncthreads();
  const uint32_t e = sm.xch_tag;
  if (tid < H / 8) {
    const size_t half = static_cast<size_t>(e & 1u) * kMaxTp * H;
    uint64_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = (static_cast<uint64_t>(e) << 32) | __float_as_uint(y[i]);
    for (int p = 0; p < x.world; ++p) {
      uint64_t* dst = x.buf[p] + half + static_cast<size_t>(x.rank) * H + 8 * tid;
#pragma unroll
      for (int j = 0; j < 4; ++j) st_relaxed_sys_v2u64(dst + 2 * j, w[2 * j], w[2 * j + 1]);
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int q = 0; q < x.world && ok; ++q) {
      const uint64_t* src = x.buf[x.rank] + half + static_cast<size_t>(q) * H + 8 * tid;
      uint64_t v[8];
      for (uint32_t spins = 0;; ++spins) {
        bool all = true;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ld_relaxed_sys_v2u64(src + 2 * j, v[2 * j], v[2 * j + 1]);
          all = all && static_cast<uint32_t>(v[2 * j] >> 32) == e && static_cast<uint32_t>(v[2 * j + 1] >> 32) == e;
        }
        if (all) break;
        if ((spins & 255u) == 255u && global_ns() > sm.deadline) {
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
      sm.xch_failed = 1;
      atomicOr(status, DEV_ERR_TIMEOUT_PEER);
    }
  }
  __syncthreads();
  if (tid == 0) *launch_ctr = e;
  return sm.xch_failed == 0;
}

// Stage partition of phase p: W = T*S (tile, k-stage) pairs over G CTAs.
// d = 1 gives the last CTA 1/8 less work than the others: it is the one scheduled on the
// SM held longest by the previous launch (the CTA running its tail), so it starts late.
struct Part {
  int T, S, W, d;
  __host__ __device__ int lo(int c, int G) const {
    return c >= G ? W : static_cast<int>((static_cast<long long>(c) * 8 * W) / (8LL * G - d));
  }
  __host__ __device__ int owner(int i, int G) const {
    const long long c = ((static_cast<long long>(i) + 1) * (8LL * G - d) - 1) / (8LL * W);
    return static_cast<int>(c < G - 1 ? c : G - 1);
  }
};

// Bounded wait on an mbarrier phase.  Only the calling thread polls, and it never sleeps
// (neither a hardware suspend nor __nanosleep: their wake-up latency showed at every phase
// end -- 0.3 us per launch; this kernel's warps are not issue-bound, so spinning costs
// nothing); warps wait through warp_wait, where lane 0 polls for everyone.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Smem& sm, uint32_t* status) {
  const bool ok = mbar_wait(bar, parity, sm.deadline, true);
  if (!ok) {
    sm.abort_flag = 1;
    atomicOr(status, DEV_ERR_TIMEOUT_MBAR);
  }
  return ok;
}
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, Smem& sm, uint32_t* status) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_bar(bar, parity, sm, status) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Group-wide (warps 2..11) sum and max.
__device__ __forceinline__ float2 group_sum_max(float s, float m, Smem& sm, int g) {
  s = warp_sum(s);
  m = warp_max(m);
  const int w = g >> 5, lane = g & 31;
  if (lane == 0) {
    sm.red[w] = s;
    sm.red2[w] = m;
  }
  named_bar_sync(kBarGroup, kGroupThreads);
  float ts = 0.f, tm = 0.f;
#pragma unroll
  for (int i = 0; i < kGroupThreads / 32; ++i) {
    ts += sm.red[i];
    tm = fmaxf(tm, sm.red2[i]);
  }
  named_bar_sync(kBarGroup, kGroupThreads);  // red / red2 free again
  return make_float2(ts, tm);
}

__device__ __forceinline__ bool group_aborted(Smem& sm, int g) {
  if (g == 0) sm.grp_abort = aborted(sm) ? 1 : 0;
  named_bar_sync(kBarGroup, kGroupThreads);
  const bool ab = sm.grp_abort != 0;
  named_bar_sync(kBarGroup, kGroupThreads);
  return ab;
}

__global__ void __launch_bounds__(kThreads, 1)
    mlp_tc_kernel(const __grid_constant__ CUtensorMap tm_gate, const __grid_constant__ CUtensorMap tm_up,
                  const __grid_constant__ CUtensorMap tm_gate_sf, const __grid_constant__ CUtensorMap tm_up_sf,
                  const __grid_constant__ CUtensorMap tm_down, const __grid_constant__ CUtensorMap tm_down_sf,
                  const Args args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  uint32_t* status = &args.scr->status;
  const int L = args.lrows;
  const Part P0{L / 64, H / kKStage, (L / 64) * (H / kKStage), 1};
  const Part P1{H / 128, L / kKStage, (H / 128) * (L / kKStage), 0};
  const Part parts[2] = {P0, P1};

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.sfready[s], 4);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.dfull[b], 1);
      mbar_init(&sm.dempty[b], 4);
    }
    mbar_init(&sm.pieces, 1);
    // Segments: the CTA's stage range cut at tile boundaries.  Phase 0 runs the tail
    // parts of split tiles first (their owners, the CTAs holding the tiles' heads, find
    // them early), then the head parts it owns, then whole tiles, so the phase ends on
    // work that needs no other CTA.  Phase 1 runs in k order.
    for (int ph = 0; ph < 2; ++ph) {
      const Part& P = parts[ph];
      const int lo = P.lo(cta, G), hi = P.lo(cta + 1, G);
      int t[kMaxCtaSeg], a0[kMaxCtaSeg], a1[kMaxCtaSeg], n = 0;
      for (int i = lo; i < hi && n < kMaxCtaSeg;) {
        const int tile = i / P.S, e = min(hi, (tile + 1) * P.S);
        t[n] = tile;
        a0[n] = i - tile * P.S;
        a1[n] = e - tile * P.S;
        ++n;
        i = e;
      }
      int o = 0;
      for (int pass = 0; pass < (ph == 0 ? 3 : 1); ++pass)
        for (int j = 0; j < n; ++j) {
          const int kind = a0[j] > 0 ? 0 : (a1[j] < P.S ? 1 : 2);  // tail, head, whole
          if (ph == 0 && kind != pass) continue;
          sm.seg_tile[ph][o] = t[j];
          sm.seg_k0[ph][o] = a0[j];
          sm.seg_k1[ph][o] = a1[j];
          ++o;
        }
      sm.seg_n[ph] = o;
    }
    sm.deadline = global_ns() + args.budget_ns;
    sm.abort_flag = 0;
    sm.last_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tbase = sm.tmem_base;
  // The tail's operands that no CTA of this launch writes (the residual was written by the
  // previous kernel on the stream).  The last CTA loads them together with the partial
  // sums: one round trip, and no load in flight at the ticket or the teardown barrier.
  uint4 tail_rv = make_uint4(0u, 0u, 0u, 0u), tail_wv = tail_rv;
  float tail_gsd = 0.f, tail_ls = 0.f;
  auto tail_loads = [&]() {
    {
      pdl_wait();
      if (tid < H / 8) {
        tail_rv = __ldcg(reinterpret_cast<const uint4*>(args.residual) + tid);
        tail_wv = __ldg(reinterpret_cast<const uint4*>(args.post_w) + tid);
      }
      tail_gsd = __ldg(args.down_gs);
      tail_ls = bf16_to_f32(__ldg(args.layer_scalar));
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // Lanes 1..3 first pull CTA c's 128-byte line of the norm weights (and CTA 0 the
    // scalars) into L2, where the staging and the tail read them.
    {
      constexpr int kBytes = H * 2, kLines = kBytes / 128;
      if (cta < kLines) {
        if (lane == 1) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(args.pre_w) + cta * 128);
        if (lane == 2) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(args.post_w) + cta * 128);
      }
      if (lane == 3 && cta == 0) {
        prefetch_l2_keep(args.layer_scalar);
        prefetch_l2_keep(args.down_gs);
        prefetch_l2_keep(args.gate_gs);
        prefetch_l2_keep(args.up_gs);
      }
    }
    if (lane == 0) {
      // codes are read once (evict first); a 16-byte scale row is half of a 32-byte sector
      // whose other half the next stage reads, so scales stay in L2
      const uint64_t pol = l2_evict_first_policy();
      uint64_t pol_sf;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_sf));
      uint32_t k = 0;
      bool ok = true;
      for (int ph = 0; ph < 2 && ok; ++ph) {
        for (int si = 0; si < sm.seg_n[ph] && ok; ++si) {
        const int tile = sm.seg_tile[ph][si];
        for (int ks = sm.seg_k0[ph][si]; ks < sm.seg_k1[ph][si]; ++ks, ++k) {
          const uint32_t slot = k % kStages, use = k / kStages;
          if (use > 0 && !wait_bar(&sm.empty[slot], (use - 1) & 1u, sm, status)) {
            ok = false;
            break;
          }
          if (aborted(sm)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[slot], kStageTx);
          const uint32_t a = smem_u32(sm.a[slot]), sf = smem_u32(sm.sfst[slot]);
          if (ph == 0) {
            tma_2d(a, &tm_gate, ks * 128, tile * 64, &sm.full[slot], pol);
            tma_2d(a + 8192u, &tm_up, ks * 128, tile * 64, &sm.full[slot], pol);
            tma_2d(sf, &tm_gate_sf, ks * 16, tile * 64, &sm.full[slot], pol_sf);
            tma_2d(sf + 1024u, &tm_up_sf, ks * 16, tile * 64, &sm.full[slot], pol_sf);
          } else {
            tma_2d(a, &tm_down, ks * 128, tile * 128, &sm.full[slot], pol);
            tma_2d(sf, &tm_down_sf, ks * 16, tile * 128, &sm.full[slot], pol_sf);
          }
        }
        }
      }
      // drain: no copy may still be landing in this CTA's shared memory at exit
      for (uint32_t j = (k > kStages ? k - kStages : 0u); j < k; ++j)
        mbar_wait(&sm.full[j % kStages], (j / kStages) & 1u, sm.deadline + args.budget_ns);
    }
  } else if (warp >= kSfWarp0) {
    // ------------------------------------------------------------------ weight scales
    // Lane l of quarter warp q writes TMEM lane 32q + l: for 64-k step st, columns
    // (16 * slot + 4 * st + j) = the 4 scales of row (l + 32 j) -- the replicated layout
    // the block-scaled MMA reads.  Rows come from the stage's TMA-loaded [128][16 B].
    const uint32_t quarter = static_cast<uint32_t>(warp - kSfWarp0);
    uint32_t k = 0;
    bool ok = true;
    for (int ph = 0; ph < 2 && ok; ++ph) {
      int nst = 0;
      for (int si = 0; si < sm.seg_n[ph]; ++si) nst += sm.seg_k1[ph][si] - sm.seg_k0[ph][si];
      for (int i = 0; i < nst; ++i, ++k) {
        const uint32_t slot = k % kStages, use = k / kStages;
        if (!warp_wait(&sm.full[slot], use & 1u, sm, status)) {
          ok = false;
          break;
        }
        uint4 rows[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) rows[j] = *reinterpret_cast<const uint4*>(sm.sfst[slot] + (lane + 32 * j) * 16);
        const uint32_t r[16] = {rows[0].x, rows[1].x, rows[2].x, rows[3].x, rows[0].y, rows[1].y, rows[2].y, rows[3].y,
                                rows[0].z, rows[1].z, rows[2].z, rows[3].z, rows[0].w, rows[1].w, rows[2].w, rows[3].w};
        tc_st16(tbase + kColSfa + 16u * slot + ((32u * quarter) << 16), r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.sfready[slot]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t k = 0, nseg = 0, slot = 0;  // slot = k % kStages
      bool ok = true;
      // The issuer's per-stage work is a few adds: while it runs, the tensor pipe only has
      // the MMAs already queued.  Descriptors hold address / 16 in their low 14 bits, so a
      // ring slot (16 KB) is +1024 and a 64-k step (32 bytes) +2; a piece stage is +128.
      const uint64_t desc_a0 = desc_sw128(smem_u32(sm.a[0])), desc_b0 = desc_sw128(smem_u32(sm.bpc[0]));
      const uint32_t empty0 = smem_u32(&sm.empty[0]);
      for (int ph = 0; ph < 2 && ok; ++ph) {
        const Part& P = parts[ph];
        const int lo = P.lo(cta, G), hi = P.lo(cta + 1, G);
        // stages of this phase: k .. k_end-1 (the scale warps arrive in this order, so
        // acquiring stage j's barrier also covers every earlier stage: one wait per group
        // of up to kWaitGroup stages -- each acquire here costs as much as a stage's MMAs)
        const uint32_t k_end = k + static_cast<uint32_t>(hi - lo);
        uint32_t ready = k;  // stages below this are known to be staged
        if (!wait_bar(&sm.pieces, static_cast<uint32_t>(ph), sm, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int S = P.S, s_a = lo % S;  // phase 1: first k-stage of the resident window
        for (int si = 0; si < sm.seg_n[ph] && ok; ++si) {
          const int k0 = sm.seg_k0[ph][si], k1 = sm.seg_k1[ph][si];
          const uint32_t buf = nseg & 1u;
          if (nseg >= 2) {
            if (!wait_bar(&sm.dempty[buf], ((nseg >> 1) - 1) & 1u, sm, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const uint32_t d = tbase + buf * 16u;
          // resident k-stage of the activation pieces: ks itself when the whole phase is
          // resident, else the position in this CTA's window (consecutive within a segment)
          uint32_t kl = static_cast<uint32_t>(S <= kMaxLocal ? k0 : (k0 - s_a + S) % S);
          for (int ks = k0; ks < k1; ++ks, ++k) {
            // the scale warps waited for a stage's TMA barrier before arriving, so their
            // barrier covers both the weights and their scales
            if (k >= ready) {
              const uint32_t j = min(k + kWaitGroup - 1u, k_end - 1u);
              if (!wait_bar(&sm.sfready[j % kStages], (j / kStages) & 1u, sm, status)) {
                ok = false;
                break;
              }
              tc_fence_after();
              ready = j + 1u;
            }
            const uint64_t da = desc_a0 + 1024u * slot, db = desc_b0 + 128u * kl;
            const uint32_t t_sfa = tbase + kColSfa + 16u * slot, t_sfb = tbase + kColSfb + 16u * kl;
#pragma unroll
            for (int st = 0; st < 4; ++st)
              tc_mma(d, da + 2u * st, db + 2u * st, t_sfa + 4u * st, t_sfb + 4u * st, (ks == k0 && st == 0) ? 0u : 1u);
            tc_commit_at(empty0 + 8u * slot);
            slot = slot + 1u == static_cast<uint32_t>(kStages) ? 0u : slot + 1u;
            ++kl;
          }
          if (!ok) break;
          tc_commit(&sm.dfull[buf]);
          ++nseg;
        }
      }
      if (!ok) sm.abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------------ staging group
    const int g = tid - kGroupWarp0 * 32;  // 0..287
    const bool epi = warp >= kEpiWarp0 && warp < kEpiWarp0 + 4;
    const int m = (warp - kEpiWarp0) * 32 + lane;  // epilogue: accumulator row
    // ---- phase 0 staging: x = RMSNorm(residual) (bf16-rounded), then pieces
    {
      const int nblk = H / 16;  // 240
      float ss = 0.f, pm = 0.f;
      uint4 xv[2], wv[2];
      if (g < nblk) {  // the norm weight is never written: load it before the wait
        wv[0] = __ldg(reinterpret_cast<const uint4*>(args.pre_w) + 2 * g);
        wv[1] = __ldg(reinterpret_cast<const uint4*>(args.pre_w) + 2 * g + 1);
      }
      // thread 0's scalars: the global scales (never written) before the wait, the launch
      // count (written by the previous launch) after it, beside the residual loads
      float gs_gate = 0.f, gs_up = 0.f;
      uint32_t launches = 0u;
      if (g == 0) {
        gs_gate = __ldg(args.gate_gs);
        gs_up = __ldg(args.up_gs);
      }
      pdl_wait();
      if (g == 0) launches = __ldcg(&args.scr->tc_epoch);
      if (g < nblk) {
        xv[0] = __ldg(reinterpret_cast<const uint4*>(args.residual) + 2 * g);
        xv[1] = __ldg(reinterpret_cast<const uint4*>(args.residual) + 2 * g + 1);
        const uint32_t xw[8] = {xv[0].x, xv[0].y, xv[0].z, xv[0].w, xv[1].x, xv[1].y, xv[1].z, xv[1].w};
        const uint32_t ww[8] = {wv[0].x, wv[0].y, wv[0].z, wv[0].w, wv[1].x, wv[1].y, wv[1].z, wv[1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float a = bf16_to_f32(static_cast<uint16_t>(xw[i] & 0xFFFFu));
          const float b = bf16_to_f32(static_cast<uint16_t>(xw[i] >> 16));
          ss = __fadd_rn(ss, __fmul_rn(a, a));
          ss = __fadd_rn(ss, __fmul_rn(b, b));
          pm = fmaxf(pm, fabsf(a * bf16_to_f32(static_cast<uint16_t>(ww[i] & 0xFFFFu))));
          pm = fmaxf(pm, fabsf(b * bf16_to_f32(static_cast<uint16_t>(ww[i] >> 16))));
        }
      }
      const float2 red = group_sum_max(ss, pm, sm, g);
      const float rf = rms_factor(red.x, H);
      // largest biased exponent of y: from the bound |y| <= max|x w| * r * (1 + 2^-7)
      const int gmax = static_cast<int>((__float_as_uint(red.y * rf * 1.01f) >> 23) & 0xFFu);
      if (g < kPieces) sm.pw[0][g] = pow2f(gmax - 127 - 2 * g);
      if (g == 0) {
        sm.gate_gs = gs_gate;
        sm.up_gs = gs_up;
        sm.tag = launches + 1u;  // the previous launch's count (read after the wait)
      }
      if (g < nblk) {
        const uint32_t xw[8] = {xv[0].x, xv[0].y, xv[0].z, xv[0].w, xv[1].x, xv[1].y, xv[1].z, xv[1].w};
        const uint32_t ww[8] = {wv[0].x, wv[0].y, wv[0].z, wv[0].w, wv[1].x, wv[1].y, wv[1].z, wv[1].w};
        uint32_t yw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint16_t yb[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint16_t xb = static_cast<uint16_t>(j ? xw[i] >> 16 : xw[i] & 0xFFFFu);
            const uint16_t wb = static_cast<uint16_t>(j ? ww[i] >> 16 : ww[i] & 0xFFFFu);
            yb[j] = f32_to_bf16(__fmul_rn(__fmul_rn(bf16_to_f32(xb), rf), bf16_to_f32(wb)));
          }
          yw[i] = pack_u16x2(yb[0], yb[1]);
        }
        split_block(yw, gmax, sm, g >> 4, g & 15);
      }
      fence_proxy_async();
      named_bar_sync(kBarGroup, kGroupThreads);
      if (epi) {
        write_sfb(sm, tbase, (H / kKStage) * 4, warp - kEpiWarp0);
        tc_fence_before();
      }
      named_bar_sync(kBarGroup, kGroupThreads);
      if (g == 0) mbar_arrive(&sm.pieces);
    }

    // ---- accumulator epilogue of one phase (warps 4..7): segments in order, tile ends
    uint32_t nseg = 0;
    auto geglu_store = [&](int tile, float tot) {
      // rows 0..63 of a phase-0 tile are gate rows, 64..127 the same rows of up
      if (m >= 64) sm.xchg[m - 64] = tot;
      named_bar_sync(kBarEpi, 128);
      float hv = 0.f;
      if (m < 64) {
        const float g2 = round_bf16(round_bf16(tot) * sm.gate_gs);
        const float u2 = round_bf16(round_bf16(sm.xchg[m]) * sm.up_gs);
        hv = round_bf16(round_bf16(gelu_tanh(g2)) * u2);
        st_relaxed_gpu_u32(&args.htag[tile * 64 + m], static_cast<uint32_t>(f32_to_bf16(hv)) | (sm.tag << 16));
      }
    };
    // Accumulator epilogue of one phase (warps 4..7), segments in the MMA order.  A whole
    // tile is finished here; a split tile's tail part stores its partial sums as tagged
    // words; the head part's CTA owns the tile: it reads the other parts' words (again
    // until their tags are this launch's: one round trip when they are in), adds the parts
    // in k order and finishes the tile (phase 0: GeGLU -> h; phase 1: the 128 sums).
    auto run_epilogue = [&](int ph) {
      const Part& P = parts[ph];
      const int tbase_idx = (ph == 0) ? 0 : P0.T;
      for (int si = 0; si < sm.seg_n[ph]; ++si) {
        const int tile = sm.seg_tile[ph][si];
        const uint32_t buf = nseg & 1u;
        const int first_owner = P.owner(tile * P.S, G);
        const int nseg_tile = P.owner(tile * P.S + P.S - 1, G) - first_owner + 1;
        const int segi = cta - first_owner;
        const bool ok = warp_wait(&sm.dfull[buf], (nseg >> 1) & 1u, sm, status);
        float v = 0.f;
        if (ok) {
          tc_fence_after();
          float d[16];
          tc_ld16(tbase + buf * 16u + (static_cast<uint32_t>((warp - kEpiWarp0) * 32) << 16), d);
          tc_fence_before();
#pragma unroll
          for (int n = 0; n < kPieces; ++n) v = fmaf(d[n], sm.pw[ph][n], v);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.dempty[buf]);
        ++nseg;
        uint64_t* tagged = args.ptag + static_cast<size_t>(tbase_idx + tile) * kMaxSeg * 128 + m;
        if (segi > 0) {
          st_relaxed_gpu_u64(tagged + segi * 128, (static_cast<uint64_t>(sm.tag) << 32) | __float_as_uint(v));
        } else if (nseg_tile == 1) {
          if (ph == 0) geglu_store(tile, v); else args.seg[tile * 128 + m] = v;
        } else {
          uint64_t w[kMaxSeg];
          for (uint32_t round = 0;; ++round) {  // every part's word re-read each round
            bool all = true;
#pragma unroll
            for (int sgi = 1; sgi < kMaxSeg; ++sgi)
              if (sgi < nseg_tile) {
                w[sgi] = ld_relaxed_gpu_u64(tagged + sgi * 128);
                all = all && static_cast<uint32_t>(w[sgi] >> 32) == sm.tag;
              }
            if (all) break;
            if ((round & 7u) == 7u && global_ns() > sm.deadline) {
              atomicOr(status, DEV_ERR_TIMEOUT_GRID);
              sm.abort_flag = 1;
              break;
            }
          }
          float tot = v;
#pragma unroll
          for (int sgi = 1; sgi < kMaxSeg; ++sgi)  // the parts in k order
            if (sgi < nseg_tile) tot += __uint_as_float(static_cast<uint32_t>(w[sgi]));
          if (ph == 0) geglu_store(tile, tot); else args.seg[tile * 128 + m] = tot;
        }
        named_bar_sync(kBarEpi, 128);
      }
    };

    if (epi) run_epilogue(0);
    named_bar_sync(kBarGroup, kGroupThreads);
    // ---- phase 1 staging: pieces of h over this CTA's window of k-stages
    const bool ab1 = group_aborted(sm, g);
    if (!ab1) {
      // the whole down phase is resident when it fits (tensor-parallel shards), else this
      // CTA's window of k-stages
      const bool whole = P1.S <= kMaxLocal;
      const int lo = P1.lo(cta, G), hi = P1.lo(cta + 1, G);
      const int s_a = whole ? 0 : lo % P1.S;
      const int len = whole ? P1.S : min(hi - lo, P1.S);
      // One 16-element block of h per thread (len * 16 <= 256 < 320), read as tagged
      // words until every tag is this launch's: no grid barrier, and the words of tiles
      // already finished arrive in one round trip.  Rounds follow each other without a
      // sleep (a round is already a memory round trip; a sleep only delays the last one).  The pieces' reference exponent is the
      // largest of this CTA's window (each CTA scales its own partial sums).
      const int kl = g >> 4, bs = g & 15;
      const bool mine = g < len * 16;
      uint32_t hw[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      uint32_t hmax = 0u;
      if (mine) {
        const int kstage = (s_a + kl) % P1.S;
        const uint32_t* src = args.htag + kstage * kKStage + bs * 16;
        const uint32_t tag16 = sm.tag & 0xFFFFu;
        uint32_t t[16];
        for (uint32_t round = 0;; ++round) {  // every word re-read each round: one round trip
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v4 = ld_relaxed_gpu_v4u32(src + 4 * q);
            t[4 * q] = v4.x, t[4 * q + 1] = v4.y, t[4 * q + 2] = v4.z, t[4 * q + 3] = v4.w;
          }
          bool all = true;
#pragma unroll
          for (int i = 0; i < 16; ++i) all = all && (t[i] >> 16) == tag16;
          if (all) break;
          if ((round & 7u) == 7u && global_ns() > sm.deadline) {
            atomicOr(status, DEV_ERR_TIMEOUT_GRID);
            sm.abort_flag = 1;
            break;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          hw[j] = (t[2 * j] & 0xFFFFu) | (t[2 * j + 1] << 16);
          hmax = max(hmax, max(t[2 * j] & 0x7FFFu, t[2 * j + 1] & 0x7FFFu));
        }
      }
      const float2 rm = group_sum_max(0.f, __uint_as_float(hmax << 16), sm, g);
      const int gmax = static_cast<int>((__float_as_uint(rm.y) >> 23) & 0xFFu);
      if (g < kPieces) sm.pw[1][g] = pow2f(gmax - 127 - 2 * g);
      if (mine) split_block(hw, gmax, sm, kl, bs);
    }
    fence_proxy_async();
    named_bar_sync(kBarGroup, kGroupThreads);
    if (epi && !ab1) {
      write_sfb(sm, tbase, (P1.S <= kMaxLocal ? P1.S : min(P1.lo(cta + 1, G) - P1.lo(cta, G), P1.S)) * 4,
                warp - kEpiWarp0);
      tc_fence_before();
    }
    named_bar_sync(kBarGroup, kGroupThreads);
    if (g == 0) mbar_arrive(&sm.pieces);
    if (epi && !ab1) run_epilogue(1);
    named_bar_sync(kBarGroup, kGroupThreads);

    // ---- every CTA reports its partial sums; the last one to report adds the residual
    // branch (its ticket says every other CTA's sums are in: no waiting)
    if (g == 0) sm.last_flag = atom_add_acq_rel_gpu(&args.scr->mlp_done, 1u) == static_cast<uint32_t>(G - 1) ? 1 : 0;
  }

  // ---- teardown: every tensor-core operation has completed (the epilogue consumed the
  // last accumulator, or the launch gave up).  The last CTA then adds the residual branch
  // with all its warps: thread t < 480 owns outputs [8t, 8t + 8), so its partial-sum,
  // residual and norm-weight loads go out in one round.
  tc_fence_before();
  __syncthreads();
  if (sm.last_flag && !aborted(sm)) {
    const int grp = tid;
    float y[8];
    float t[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    tail_loads();
    if (grp < H / 8) {
      // every down tile was finished by the CTA holding its first k-stages (its ticket came
      // after): the 3840 sums, 32 bytes per thread
      const float4* yp = reinterpret_cast<const float4*>(args.seg) + 2 * grp;
      const float4 p0 = __ldcg(yp), p1 = __ldcg(yp + 1);
      t[0] = p0.x, t[1] = p0.y, t[2] = p0.z, t[3] = p0.w, t[4] = p1.x, t[5] = p1.y, t[6] = p1.z, t[7] = p1.w;
    }
    // tensor parallel: every rank's down sums, added in rank order on every rank
    const bool xch_ok = args.xch.world <= 1 || peer_allreduce_tc(args.xch, &args.scr->xch_epoch, t, tid, status, sm);
    float ss = 0.f;
    if (grp < H / 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d2 = round_bf16(round_bf16(t[i]) * tail_gsd);
        y[i] = d2;
        ss = __fadd_rn(ss, __fmul_rn(d2, d2));
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) sm.red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) tot += sm.red[w];
    const float rr = rms_factor(tot, H);
    if (grp < H / 8 && xch_ok) {
      const uint32_t rw[4] = {tail_rv.x, tail_rv.y, tail_rv.z, tail_rv.w};
      const uint32_t ww[4] = {tail_wv.x, tail_wv.y, tail_wv.z, tail_wv.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint16_t h2[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float res = bf16_to_f32(static_cast<uint16_t>(j ? rw[i] >> 16 : rw[i] & 0xFFFFu));
          const float pw = bf16_to_f32(static_cast<uint16_t>(j ? ww[i] >> 16 : ww[i] & 0xFFFFu));
          const float nb = round_bf16(__fmul_rn(__fmul_rn(y[2 * i + j], rr), pw));
          const float r2 = round_bf16(__fadd_rn(res, nb));
          h2[j] = f32_to_bf16(__fmul_rn(r2, tail_ls));
        }
        o[i] = pack_u16x2(h2[0], h2[1]);
      }
      *reinterpret_cast<uint4*>(args.residual + 8 * grp) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (sm.last_flag && tid == 0) {  // every CTA has read this launch's tag and taken a ticket
    args.scr->mlp_done = 0u;
    args.scr->tc_epoch = sm.tag;
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// 2-D byte matrix [rows][cols] (row pitch = cols), box [box_rows][box_cols]
static bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                     uint32_t box_cols, bool swizzle) {
  EncodeFn fn = encoder();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc

// Whether the tensor-core kernel serves this context: the default unless the context asks
// for the streaming kernel (or G4B200_MLP_KERNEL=stream sets the default), on one GPU or
// on a tensor-parallel context of at most kTcMaxTp ranks that exchange over peer memory
// and whose shard the kernel's tiles fit (256-k stages of the down projection, 16-byte
// rows of its scales: TP8's 120-byte rows do not).  The NCCL fallback keeps the
// streaming kernel.
// TP2 and TP4 shards fit the kernel (TP8's 1920-wide down k-slices do not); measured per
// token on B200s: TP2 25.9 us here against 26.8 on the streaming kernel, TP4 28.7 against
// 26.2, so TP4 keeps the streaming kernel.
constexpr int kTcMaxTp = 2;
bool mlp_tc_enabled(const g4_ctx* ctx) {
  static const int env_kind = [] {
    const char* e = std::getenv("G4B200_MLP_KERNEL");
    if (e != nullptr && std::strcmp(e, "stream") == 0) return static_cast<int>(G4_MLP_STREAM);
    return static_cast<int>(G4_MLP_TENSOR);
  }();
  const int kind = ctx->mlp_kernel == G4_MLP_AUTO ? env_kind : ctx->mlp_kernel;
  if (kind != G4_MLP_TENSOR || ctx->buf.tc_seg == nullptr || ctx->buf.tc_ptag == nullptr || ctx->buf.tc_htag == nullptr)
    return false;
  if (ctx->tp_world == 1) return true;
  const int lrows = L / ctx->tp_world;
  return ctx->tp_world <= kTcMaxTp && ctx->peers.world == ctx->tp_world && lrows % tc::kKStage == 0 &&
         (lrows / 16) % 16 == 0 && lrows % 64 == 0;
}

g4_status launch_decoder_feedforward_tc(g4_ctx* ctx, uint16_t* residual, const uint16_t* pre_w, const uint8_t* up_p,
                                        const uint8_t* gate_p, const uint8_t* down_p, const uint8_t* up_s,
                                        const uint8_t* gate_s, const uint8_t* down_s, const float* up_gs,
                                        const float* gate_gs, const float* down_gs, const uint16_t* post_w,
                                        const uint16_t* layer_scalar) {
  using namespace tc;
  const int lrows = L / ctx->tp_world;  // this rank's shard of the intermediate rows
  // host check of the partition: every tile has at most kMaxSeg segments
  const int G = ctx->sm_count;
  for (int ph = 0; ph < 2; ++ph) {
    const int T = ph == 0 ? lrows / 64 : H / 128, S = ph == 0 ? H / kKStage : lrows / kKStage;
    const Part P{T, S, T * S, ph == 0 ? 1 : 0};
    for (int c = 0; c < G; ++c) {
      const int len = P.lo(c + 1, G) - P.lo(c, G);
      if (len < 1 || (S > kMaxLocal && len > kMaxLocal) || len / S + 2 > kMaxCtaSeg)
        return fail(ctx, G4_ERR_UNSUPPORTED, "tensor-core MLP: partition does not fit this kernel");
    }
    for (int t = 0; t < T; ++t)
      if (P.owner(t * S + S - 1, G) - P.owner(t * S, G) + 1 > kMaxSeg)
        return fail(ctx, G4_ERR_UNSUPPORTED, "tensor-core MLP: too many segments per tile");
  }
  CUtensorMap maps[6];
  bool ok = make_map(&maps[0], gate_p, lrows, H / 2, 64, 128, true) &&
            make_map(&maps[1], up_p, lrows, H / 2, 64, 128, true) &&
            make_map(&maps[2], gate_s, lrows, H / 16, 64, 16, false) &&
            make_map(&maps[3], up_s, lrows, H / 16, 64, 16, false) &&
            make_map(&maps[4], down_p, H, lrows / 2, 128, 128, true) &&
            make_map(&maps[5], down_s, H, lrows / 16, 128, 16, false);
  if (!ok) return fail(ctx, G4_ERR_CUDA, "cuTensorMapEncodeTiled failed for the MLP weights");
  Args a;
  a.residual = residual;
  a.pre_w = pre_w;
  a.post_w = post_w;
  a.layer_scalar = layer_scalar;
  a.up_gs = up_gs;
  a.gate_gs = gate_gs;
  a.down_gs = down_gs;
  a.scr = ctx->buf.scratch;
  a.part = ctx->buf.part;
  a.seg = ctx->buf.tc_seg;
  a.ptag = ctx->buf.tc_ptag;
  a.htag = ctx->buf.tc_htag;
  a.lrows = lrows;
  a.budget_ns = ctx->wait_budget_ns;
  a.xch = ctx->tp_world > 1 ? ctx->peers : PeerXch{};
  const size_t smem = sizeof(Smem) + 1024;
  g4_status st = allow_max_dynamic_smem(ctx, (const void*)mlp_tc_kernel, smem, "mlp_tc_kernel smem");
  if (st != G4_OK) return st;
  void* args[] = {&maps[0], &maps[1], &maps[2], &maps[3], &maps[4], &maps[5], &a};
  // Not cooperative (see launch_decoder_feedforward): one CTA per SM, and its shared memory
  // excludes a second CTA, so every CTA is resident while others wait for its words.
  return launch_kernel(ctx, (const void*)mlp_tc_kernel, dim3(G), dim3(kThreads), smem, args, false,
                       "launch mlp_tc_kernel");
}

}  // namespace g4
