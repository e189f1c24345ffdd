// Batched prefill of decoder_feedforward (ops::decoder_feedforward, src/ops.rs:213-253,
// for n tokens at once) on the 5th-generation tensor cores.
//
// The reference prefills one position per dispatch (src/host/generate.rs:194-211).  Here
// the MLP block of n tokens runs as two block-scaled FP4 GEMMs
// (tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16, f32 accumulators in
// tensor memory) on the checkpoint's NVFP4 weights, unchanged:
//   1. quant (x)  : per token, RMSNorm(residual, pre_ff) -> bf16 -> P NVFP4 pieces;
//   2. gemm (gate/up): D[128 weight rows][128 tokens], rows = 64 gate + the same 64 up
//                   rows, K = 3840; epilogue gate = bf16(bf16(acc/g) * gs_gate), likewise
//                   up, h = bf16(bf16(gelu_tanh(gate)) * up) written bf16 [n][L];
//   3. quant (h)  : per token, h -> P NVFP4 pieces;
//   4. gemm (down): D[128 rows][128 tokens], K = 15360; y = acc/g in f32 [n][H];
//   5. tail       : per token, y = bf16(bf16(y) * gs_down),
//                   residual = bf16(bf16(residual + RMSNorm(y, post_ff)) * layer_scalar).
// Tensor parallel: gate/up hold the rank's intermediate rows, down its k-slice; the
// ranks' f32 y are summed (NCCL all-reduce) before the tail.
//
// Activation pieces.  The MMA's second operand is NVFP4 too, so a token's activation row
// x is written as P NVFP4 rows sharing one per-token scale g = 6*448 / max|x| (computed
// as reciprocal(max|x|) * 2688, the weight quantiser's recipe): with y_0 = x*g,
//   s_p[b] = e4m3(max_b|y_p| / 6)  (p = 0: e4m3(max_b|x| / 6 * g), the weight recipe),
//   c_p    = e2m1(y_p / s_p),      y_{p+1} = y_p - c_p * s_p,
// and x ~= (sum_p c_p * s_p) / g.  The MMA adds the P pieces' products into the same
// accumulator (they share the weight tile), the epilogue multiplies by 1/g.  One piece
// leaves ~10 % relative error per activation (the MLP output then misses the reference's
// bf16 tolerance); two pieces ~1 %, three ~0.1 %.
//
// GEMM kernel: persistent CTAs over (weight tile, token tile) pairs, token tiles
// innermost so the CTAs working at one time share weight tiles in L2.  Warp 0 moves each
// 256-k stage (weights 128 x 128 B and, per piece, tokens 128 x 128 B, 128-byte swizzle;
// their block scales 128 x 16 B each) with TMA into a shared-memory ring; warps 4-7 write
// each stage's scales into tensor memory in the layout the block-scaled MMA reads; warp 1
// issues the MMAs (4 per stage and piece, K = 64 each) into one of two accumulators;
// warps 8-11 run the epilogue of the other accumulator meanwhile.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {
namespace pf {

constexpr int kThreads = 384;  // 12 warps
constexpr int kTile = 128;     // weight rows and tokens per tile
constexpr int kKStage = 256;   // k per stage (128 bytes of E2M1 codes per row)
constexpr int kMaxPieces = 3;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSf = 256;  // scales after the two 128-column accumulators
constexpr uint32_t kBarEpi = 1;
// M = 128, N = 128, both operands E2M1, scales E4M3
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kTile >> 3) << 17) | (8u << 24);

template <int P>
struct Cfg {
  static constexpr int kStages = P == 1 ? 6 : (P == 2 ? 4 : 3);  // 216 KB of ring each
  static constexpr uint32_t kStageTx = 16384 + 2048 + P * (16384 + 2048);
  static constexpr uint32_t kSfCols = 16 * (1 + P);  // TMEM scale columns per stage
  static_assert(kColSf + kStages * kSfCols <= kTmemCols, "tensor memory columns");
};

template <int P>
struct __align__(1024) Smem {
  static constexpr int S = Cfg<P>::kStages;
  uint8_t a[S][16384];           // weight rows, 128 x 128 B, 128-byte swizzle
  uint8_t b[S][P][16384];        // token rows per piece, 128 x 128 B, 128-byte swizzle
  uint8_t sfa[S][2048];          // weight block scales [128][16 B]
  uint8_t sfb[S][P][2048];       // token block scales per piece [128][16 B]
  uint16_t gate[2][16][64];      // gate/up epilogue, 16 tokens at a time (double-buffered):
  uint16_t up[2][16][64];        //   bf16 values [token][intermediate row]
  float ginv[kTile];             // this tile's per-token 1/g
  uint64_t full[S], sfready[S], empty[S];
  uint64_t dfull[2], dempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

struct GemmArgs {
  int mode;              // 0: gate/up -> h (bf16), 1: down -> y (f32, scaled by 1/g)
  int n_tok;
  int m_tiles;           // weight row tiles
  int k_stages;
  const float* ginv;     // [n_tok] 1/g of the activation rows
  const float* gs_gate;  // mode 0: reciprocal global scales of gate and up
  const float* gs_up;
  uint16_t* h;           // mode 0: [n_tok][h_ld]
  int h_ld;
  float* y;              // mode 1: [n_tok][H]
  Scratch* scr;
  uint64_t budget_ns;
};

__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1u) << 16) |
         (static_cast<uint64_t>(1024u >> 4) << 32) | (static_cast<uint64_t>(1u) << 46) |
         (static_cast<uint64_t>(2u) << 61);
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                       uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                       uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
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
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// One stage's block scales of 128 rows ([128][16 B] in shared memory) into tensor memory:
// lane l of the warp's lane quarter, column 4 s + j = the 4 scales (64-k step s) of row
// l + 32 j.
__device__ __forceinline__ void write_sf(const uint8_t* rows16, uint32_t taddr, int lane) {
  uint4 rw[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) rw[j] = *reinterpret_cast<const uint4*>(rows16 + (lane + 32 * j) * 16);
  const uint32_t r[16] = {rw[0].x, rw[1].x, rw[2].x, rw[3].x, rw[0].y, rw[1].y, rw[2].y, rw[3].y,
                          rw[0].z, rw[1].z, rw[2].z, rw[3].z, rw[0].w, rw[1].w, rw[2].w, rw[3].w};
  tc_st16(taddr, r);
}
// bf16 round-to-nearest-even with integer operations (the epilogue's conversions would
// otherwise saturate the SM's conversion pipe, which also runs tanh): bit-identical to
// cvt.rn.bf16.f32 for every finite value and infinity; a NaN stays a quiet NaN.
__device__ __forceinline__ uint32_t bf16_rne_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t r = (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
  return (f != f) ? ((u >> 16) | 0x40u) : r;
}
__device__ __forceinline__ float rne_bf16(float f) { return __uint_as_float(bf16_rne_bits(f) << 16); }
__device__ __forceinline__ uint32_t pack_rne(float a, float b) { return bf16_rne_bits(a) | (bf16_rne_bits(b) << 16); }

// bar.red.or over a named barrier: true on every participating thread if `pred` is true
// on any (a decision all of them take together).
__device__ __forceinline__ bool named_bar_any(uint32_t id, uint32_t threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(threads)
      : "memory");
  return r != 0u;
}

template <int P>
__global__ void __launch_bounds__(kThreads, 1) pf_gemm_kernel(const __grid_constant__ CUtensorMap ma0,
                                                              const __grid_constant__ CUtensorMap ma1,
                                                              const __grid_constant__ CUtensorMap msa0,
                                                              const __grid_constant__ CUtensorMap msa1,
                                                              const __grid_constant__ CUtensorMap mb,
                                                              const __grid_constant__ CUtensorMap msb,
                                                              const __grid_constant__ GemmArgs args) {
  constexpr int S = Cfg<P>::kStages;
  constexpr uint32_t kSfCols = Cfg<P>::kSfCols;
  extern __shared__ uint8_t pf_raw[];
  Smem<P>& sm = *reinterpret_cast<Smem<P>*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles_tok = (args.n_tok + kTile - 1) / kTile;
  const int n_tiles = args.m_tiles * n_tiles_tok;
  const int KS = args.k_stages;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.sfready[i], 4);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.dfull[i], 1);
      mbar_init(&sm.dempty[i], 4);
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort_flag = 0;
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
  pdl_wait();  // activations and 1/g come from the previous kernels
  const uint64_t deadline = global_ns() + args.budget_ns;
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;
  auto fail = [&]() {
    atomicOr(&args.scr->status, DEV_ERR_TIMEOUT_MBAR);
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_last_policy();  // weight and token tiles are each read by several CTAs
      uint32_t kc = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        const int mt = t / n_tiles_tok, nt = t % n_tiles_tok;
        for (int ks = 0; ks < KS; ++ks, ++kc) {
          const uint32_t st = kc % S;
          if (kc >= S && !mbar_wait_suspend(&sm.empty[st], ((kc / S) - 1) & 1u, deadline)) {
            fail();
            ok = false;
            break;
          }
          if (*abort_flag) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[st], Cfg<P>::kStageTx);
          const int x = ks * (kKStage / 2), xs = ks * (kKStage / 16);
          if (args.mode == 0) {  // 64 gate rows then the same 64 up rows
            tma_2d(sm.a[st], &ma0, x, 64 * mt, &sm.full[st], pol);
            tma_2d(sm.a[st] + 8192, &ma1, x, 64 * mt, &sm.full[st], pol);
            tma_2d(sm.sfa[st], &msa0, xs, 64 * mt, &sm.full[st], pol);
            tma_2d(sm.sfa[st] + 1024, &msa1, xs, 64 * mt, &sm.full[st], pol);
          } else {
            tma_2d(sm.a[st], &ma0, x, kTile * mt, &sm.full[st], pol);
            tma_2d(sm.sfa[st], &msa0, xs, kTile * mt, &sm.full[st], pol);
          }
#pragma unroll
          for (int p = 0; p < P; ++p) {
            tma_3d(sm.b[st][p], &mb, x, kTile * nt, p, &sm.full[st], pol);
            tma_3d(sm.sfb[st][p], &msb, xs, kTile * nt, p, &sm.full[st], pol);
          }
          issued = kc + 1;
        }
      }
      // no copy may still be in flight when the CTA exits
      for (uint32_t j = issued > static_cast<uint32_t>(S) ? issued - S : 0u; j < issued; ++j)
        if (!mbar_wait_suspend(&sm.full[j % S], (j / S) & 1u, deadline + args.budget_ns)) break;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t kc = 0, ti = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++ti) {
        const uint32_t buf = ti & 1u;
        if (ti >= 2) {
          if (!mbar_wait(&sm.dempty[buf], ((ti >> 1) - 1) & 1u, deadline, true)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
        }
        const uint32_t d = tbase + buf * kTile;
        for (int ks = 0; ks < KS; ++ks, ++kc) {
          const uint32_t st = kc % S;
          if (!mbar_wait(&sm.sfready[st], (kc / S) & 1u, deadline, true)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = desc_sw128(smem_u32(sm.a[st]));
          const uint32_t sfa = tbase + kColSf + kSfCols * st;
#pragma unroll
          for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int p = 0; p < P; ++p) {
              const uint64_t db = desc_sw128(smem_u32(sm.b[st][p]));
              tc_mma(d, da + 2u * s, db + 2u * s, sfa + 4u * s, sfa + 16u * (1 + p) + 4u * s,
                     (ks == 0 && s == 0 && p == 0) ? 0u : 1u);
            }
          }
          tc_commit(&sm.empty[st]);
        }
        if (!ok) break;
        tc_commit(&sm.dfull[buf]);
      }
      // every MMA has finished before tensor memory is released
      tc_commit(&sm.mma_done);
      mbar_wait(&sm.mma_done, 0u, deadline + args.budget_ns);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------------- block scales -> TMEM
    // Lane l of warp 4+q writes TMEM lane 32q + l, the same in all four lane quarters.
    // Stage st's columns: weight scales at kColSf + kSfCols*st (+4 s + j: 64-k step s of
    // row l + 32 j), piece p's token scales 16 (1 + p) further.
    const uint32_t q = static_cast<uint32_t>(warp & 3);
    uint32_t kc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
      for (int ks = 0; ks < KS; ++ks, ++kc) {
        const uint32_t st = kc % S;
        const bool got = __all_sync(0xffffffffu, mbar_wait(&sm.full[st], (kc / S) & 1u, deadline));
        if (!got) {
          if (lane == 0) fail();
          ok = false;
          break;
        }
        const uint32_t col = tbase + kColSf + kSfCols * st + ((32u * q) << 16);
        write_sf(sm.sfa[st], col, lane);
#pragma unroll
        for (int p = 0; p < P; ++p) write_sf(sm.sfb[st][p], col + 16u * (1 + p), lane);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.sfready[st]);
      }
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3, m = 32 * q + lane;  // this thread's accumulator row (TMEM lane)
    const int etid = tid - 256;                 // 0..127
    float gs_gate = 0.f, gs_up = 0.f;
    if (args.mode == 0) {
      gs_gate = __ldg(args.gs_gate);
      gs_up = __ldg(args.gs_up);
    }
    uint32_t ti = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++ti) {
      const int mt = t / n_tiles_tok, nt = t % n_tiles_tok;
      const uint32_t buf = ti & 1u;
      {
        const int n = kTile * nt + etid;
        sm.ginv[etid] = (n < args.n_tok) ? args.ginv[n] : 0.f;
      }
      const bool got = mbar_wait(&sm.dfull[buf], (ti >> 1) & 1u, deadline);
      if (!got) fail();
      if (named_bar_any(kBarEpi, 128, !got || *abort_flag)) break;
      tc_fence_after();
      const uint32_t dcol = tbase + buf * kTile + ((32u * q) << 16);
      if (args.mode == 0) {
        // Accumulator rows 0..63 are gate rows, 64..127 the same intermediate rows' up, so
        // gate and up of one h meet in shared memory, 16 tokens at a time: every thread
        // stores its row's 16 scaled values, then h = bf16(bf16(gelu(gate)) * up) for the
        // chunk's 64 rows x 16 tokens, a warp writing 64 consecutive bf16 of one token.
        // Chunks alternate buffers, so one barrier per chunk keeps writers behind readers.
        const float gs = (m < 64) ? gs_gate : gs_up;
        const int j = m & 63;
        const int jp = etid & 31, r0 = etid >> 5;
        uint16_t* hcol = args.h + static_cast<size_t>(64 * mt + 2 * jp);
        // the whole row leaves tensor memory first, so the accumulator is free for the
        // tile after next while the exchange runs
        uint32_t hv[kTile / 2];
#pragma unroll
        for (int c = 0; c < kTile / 16; ++c) {
          float v[16];
          tc_ld16(dcol + 16u * c, v);
#pragma unroll
          for (int i = 0; i < 16; i += 2)
            hv[8 * c + i / 2] = pack_rne(rne_bf16(v[i] * sm.ginv[16 * c + i]) * gs,
                                         rne_bf16(v[i + 1] * sm.ginv[16 * c + i + 1]) * gs);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.dempty[buf]);
#pragma unroll
        for (int c = 0; c < kTile / 16; ++c) {
          uint16_t(*dst)[64] = (m < 64) ? sm.gate[c & 1] : sm.up[c & 1];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            dst[i][j] = static_cast<uint16_t>(hv[8 * c + i / 2] & 0xFFFFu);
            dst[i + 1][j] = static_cast<uint16_t>(hv[8 * c + i / 2] >> 16);
          }
          named_bar_sync(kBarEpi, 128);
#pragma unroll
          for (int i = r0; i < 16; i += 4) {
            const int tok = kTile * nt + 16 * c + i;
            if (tok < args.n_tok) {
              const uint32_t g2 = *reinterpret_cast<const uint32_t*>(&sm.gate[c & 1][i][2 * jp]);
              const uint32_t u2 = *reinterpret_cast<const uint32_t*>(&sm.up[c & 1][i][2 * jp]);
              const float h0 = rne_bf16(gelu_tanh(__uint_as_float(g2 << 16))) * __uint_as_float(u2 << 16);
              const float h1 = rne_bf16(gelu_tanh(__uint_as_float(g2 & 0xFFFF0000u))) * __uint_as_float(u2 & 0xFFFF0000u);
              *reinterpret_cast<uint32_t*>(hcol + static_cast<size_t>(tok) * args.h_ld) = pack_rne(h0, h1);
            }
          }
        }
      } else {
        // y[token][row] = acc / g in f32 (the global scale and bf16 roundings follow the
        // cross-rank sum, in the tail)
        float* ycol = args.y + (kTile * mt + m);
#pragma unroll
        for (int c = 0; c < kTile / 16; ++c) {
          float v[16];
          tc_ld16(dcol + 16u * c, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int tok = kTile * nt + 16 * c + i;
            if (tok < args.n_tok) ycol[static_cast<size_t>(tok) * H] = v[i] * sm.ginv[16 * c + i];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.dempty[buf]);
      }
      named_bar_sync(kBarEpi, 128);  // smem (gate/up rows, 1/g) free for the next tile
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------- activation pieces
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\t.reg .b16 h;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tmov.b16 h, {t, 0};\n\t"
      "cvt.u32.u16 %0, h;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t e4m3_byte(float v) {
  uint16_t s;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(s) : "f"(v), "f"(v));
  return s & 0xFFu;
}

constexpr int kQThreads = 256;  // the tail kernel

template <int T, bool kMax>
__device__ __forceinline__ float block_reduce(float val, float* red) {
  val = kMax ? warp_max(val) : warp_sum(val);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = val;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int w = 0; w < T / 32; ++w) r = kMax ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

// y / s correctly rounded, given rcp = RN(1 / s): q0 = RN(y * rcp) is within an ulp of the
// quotient, the remainder y - q0 * s is exact in one FMA, and one correction step gives
// the correctly rounded quotient (Markstein's division theorem; the divisors here are
// E4M3 values, the dividends normal f32 well inside the range).
__device__ __forceinline__ float div_by(float y, float s, float rcp) {
  const float q0 = __fmul_rn(y, rcp);
  return __fmaf_rn(__fmaf_rn(-q0, s, y), rcp, q0);
}

// Per token: x (bf16 [K]; with norm_w, RMSNorm'ed and rounded to bf16 first) -> n_pieces
// NVFP4 pieces (see the file comment): codes [piece][token][K/2] (low nibble first) at
// piece stride code_pstride, scales [piece][token][scale_ld] at piece stride
// scale_pstride, and 1/g.  A zero (or non-finite) row gets all codes and scales 0 and
// 1/g = 0.  One CTA of T threads per token; thread t handles the 16-element blocks
// t, t + T, ... (at most NB of them), held as bf16 pairs in registers.
template <int T, int NB>
__global__ void __launch_bounds__(T, 768 / T) pf_quant_kernel(const uint16_t* __restrict__ x, int K,
                                                     const uint16_t* __restrict__ norm_w, int n_pieces,
                                                     uint8_t* __restrict__ codes, size_t code_pstride,
                                                     uint8_t* __restrict__ scales, int scale_ld,
                                                     size_t scale_pstride, float* __restrict__ ginv) {
  __shared__ float red[T / 32];
  const int tok = blockIdx.x, tid = threadIdx.x;
  const int nb = K / 16;
  const uint16_t* row = x + static_cast<size_t>(tok) * K;
  pdl_wait();
  uint32_t w[NB][8];
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int b = tid + i * T;
    if (b < nb) {
      const uint4 w0 = *reinterpret_cast<const uint4*>(row + 16 * b);
      const uint4 w1 = *reinterpret_cast<const uint4*>(row + 16 * b + 8);
      w[i][0] = w0.x, w[i][1] = w0.y, w[i][2] = w0.z, w[i][3] = w0.w;
      w[i][4] = w1.x, w[i][5] = w1.y, w[i][6] = w1.z, w[i][7] = w1.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) w[i][e] = 0u;
    }
  }
  auto lo = [](uint32_t v) { return bf16_to_f32(static_cast<uint16_t>(v & 0xFFFFu)); };
  auto hi = [](uint32_t v) { return bf16_to_f32(static_cast<uint16_t>(v >> 16)); };
  if (norm_w != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NB; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float a = lo(w[i][e]), c = hi(w[i][e]);
        ss = __fadd_rn(ss, __fmul_rn(a, a));
        ss = __fadd_rn(ss, __fmul_rn(c, c));
      }
    const float r = rms_factor(block_reduce<T, false>(ss, red), K);
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int b = tid + i * T;
      if (b < nb) {
        const uint4 n0 = __ldg(reinterpret_cast<const uint4*>(norm_w + 16 * b));
        const uint4 n1 = __ldg(reinterpret_cast<const uint4*>(norm_w + 16 * b + 8));
        const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e)
          w[i][e] = pack_bf16x2(__fmul_rn(__fmul_rn(lo(w[i][e]), r), lo(nw[e])),
                                __fmul_rn(__fmul_rn(hi(w[i][e]), r), hi(nw[e])));
      }
    }
  }
  // block maxima on the bf16 bit patterns (|x| orders like its low 15 bits)
  uint32_t bm[NB], am = 0u;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    uint32_t m2 = 0u;
#pragma unroll
    for (int e = 0; e < 8; ++e) m2 = __vmaxu2(m2, w[i][e] & 0x7FFF7FFFu);
    bm[i] = max(m2 & 0xFFFFu, m2 >> 16);
    am = max(am, bm[i]);
  }
  const float amax = block_reduce<T, true>(bf16_to_f32(static_cast<uint16_t>(am)), red);
  const bool zero = !(amax > 0.f) || !isfinite(amax);
  const float g = zero ? 1.0f : __fmul_rn(__frcp_rn(amax), 2688.0f);
  if (tid == 0) ginv[tok] = zero ? 0.f : __frcp_rn(g);
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int b = tid + i * T;
    if (b >= nb) continue;
    float y[16];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      y[2 * e] = __fmul_rn(lo(w[i][e]), g);
      y[2 * e + 1] = __fmul_rn(hi(w[i][e]), g);
    }
    // piece 0: the weight recipe, e4m3(max_b|x| / 6 * g)
    float smax = __fmul_rn(__fdiv_rn(bf16_to_f32(static_cast<uint16_t>(bm[i])), 6.0f), g);
    for (int p = 0; p < n_pieces; ++p) {
      if (p > 0) {
        smax = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) smax = fmaxf(smax, fabsf(y[e]));
        smax = __fdiv_rn(smax, 6.0f);
      }
      const uint32_t sc = zero ? 0u : e4m3_byte(fminf(smax, 448.0f));
      const float sf = e4m3_value(sc);
      uint32_t packed[2] = {0u, 0u};
      if (sf > 0.f) {
        const float rcp = __frcp_rn(sf);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const uint32_t two = e2m1x2(div_by(y[e], sf, rcp), div_by(y[e + 1], sf, rcp));
          const uint32_t hv = cvt_e2m1x2(two);  // the two code values, exact in f16
          y[e] = __fsub_rn(y[e], __fmul_rn(__half2float(__ushort_as_half(static_cast<uint16_t>(hv))), sf));
          y[e + 1] = __fsub_rn(y[e + 1], __fmul_rn(__half2float(__ushort_as_half(static_cast<uint16_t>(hv >> 16))), sf));
          packed[e >> 3] |= two << (8 * ((e >> 1) & 3));
        }
      }
      *reinterpret_cast<uint2*>(codes + p * code_pstride + static_cast<size_t>(tok) * (K / 2) + 8 * b) =
          make_uint2(packed[0], packed[1]);
      scales[p * scale_pstride + static_cast<size_t>(tok) * scale_ld + b] = static_cast<uint8_t>(sc);
    }
  }
}

// Per token: y = bf16(bf16(y32) * gs_down) (y32: the down projection's sums over every
// rank, already divided by g), residual = bf16(bf16(residual + RMSNorm(y, post_w)) * layer_scalar).
__global__ void __launch_bounds__(kQThreads) pf_tail_kernel(const float* __restrict__ y32,
                                                            const float* __restrict__ gs_down,
                                                            const uint16_t* __restrict__ post_w,
                                                            const uint16_t* __restrict__ layer_scalar,
                                                            uint16_t* __restrict__ residual) {
  __shared__ float red[kQThreads / 32];
  const int tok = blockIdx.x, tid = threadIdx.x;
  pdl_wait();
  constexpr int kPer = (H + kQThreads - 1) / kQThreads;
  const float gs = __ldg(gs_down);
  float yv[kPer], ss = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int c = tid + i * kQThreads;
    yv[i] = (c < H) ? round_bf16(__fmul_rn(round_bf16(y32[static_cast<size_t>(tok) * H + c]), gs)) : 0.f;
    ss = __fadd_rn(ss, __fmul_rn(yv[i], yv[i]));
  }
  const float r = rms_factor(block_reduce<kQThreads, false>(ss, red), H);
  const float ls = bf16_to_f32(layer_scalar[0]);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int c = tid + i * kQThreads;
    if (c < H) {
      uint16_t* rp = residual + static_cast<size_t>(tok) * H + c;
      const float nb = round_bf16(__fmul_rn(__fmul_rn(yv[i], r), bf16_to_f32(post_w[c])));
      const float s = round_bf16(__fadd_rn(bf16_to_f32(*rp), nb));
      *rp = f32_to_bf16(__fmul_rn(s, ls));
    }
  }
}

// Copies block scales [rows][cols] into [rows][ld] (ld = cols rounded up to 16 bytes,
// the TMA row-stride unit), zeroing the padding.
__global__ void pf_pad_scales_kernel(const uint8_t* __restrict__ src, int cols, uint8_t* __restrict__ dst, int ld,
                                     int rows) {
  pdl_wait();  // the previous call's down GEMM may still read dst
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(rows) * ld) return;
  const int r = static_cast<int>(i / ld), c = static_cast<int>(i % ld);
  dst[i] = (c < cols) ? src[static_cast<size_t>(r) * cols + c] : 0;
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
// Byte matrix [planes][rows][cols] (row stride ld, plane stride plane_ld; planes == 0:
// 2-D), box [1][box_rows][box_cols]; rows past `rows` read as zeros.
static bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                     uint32_t box_cols, bool swizzle, uint64_t planes = 0, uint64_t plane_ld = 0) {
  EncodeFn fn = encoder();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {cols, rows, planes};
  const cuuint64_t strides[2] = {ld, plane_ld};
  const cuuint32_t box[3] = {box_cols, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, planes ? 3 : 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int P>
static g4_status launch_gemm(g4_ctx* ctx, CUtensorMap (&m)[6], const GemmArgs& ga, const char* what) {
  const void* fn = reinterpret_cast<const void*>(&pf_gemm_kernel<P>);
  const size_t smem = sizeof(Smem<P>) + 1024;
  static_assert(sizeof(Smem<P>) + 1024 <= 232448, "shared memory per CTA");
  g4_status st = allow_max_dynamic_smem(ctx, fn, smem, what);
  if (st != G4_OK) return st;
  const int tiles = ga.m_tiles * ((ga.n_tok + kTile - 1) / kTile);
  GemmArgs a_copy = ga;
  void* a[] = {&m[0], &m[1], &m[2], &m[3], &m[4], &m[5], &a_copy};
  return launch_kernel(ctx, fn, dim3(tiles < ctx->sm_count ? tiles : ctx->sm_count), dim3(kThreads), smem, a, false,
                       what);
}
// The quantiser instance for rows of nb 16-element blocks: T threads x NB blocks >= nb.
static g4_status launch_quant(g4_ctx* ctx, int nb, int n, void** a, const char* what) {
  const void* fn;
  int threads = 128;
  if (nb <= 128) fn = reinterpret_cast<const void*>(&pf_quant_kernel<128, 1>);
  else if (nb <= 256) fn = reinterpret_cast<const void*>(&pf_quant_kernel<128, 2>);
  else if (nb <= 512) fn = reinterpret_cast<const void*>(&pf_quant_kernel<128, 4>);
  else if (nb <= 1024) fn = reinterpret_cast<const void*>(&pf_quant_kernel<256, 4>), threads = 256;
  else return fail(ctx, G4_ERR_UNSUPPORTED, "prefill: row too long for the quantiser");
  return launch_kernel(ctx, fn, dim3(n), dim3(threads), 0, a, false, what);
}
static g4_status launch_gemm_p(g4_ctx* ctx, int pieces, CUtensorMap (&m)[6], const GemmArgs& ga, const char* what) {
  switch (pieces) {
    case 1: return launch_gemm<1>(ctx, m, ga, what);
    case 2: return launch_gemm<2>(ctx, m, ga, what);
    default: return launch_gemm<3>(ctx, m, ga, what);
  }
}

}  // namespace pf

static inline int round16(int v) { return (v + 15) & ~15; }

// Grows the context's prefill scratch to n tokens (kept until the context is destroyed).
// Padding bytes of the scale rows are zeroed here and never written again.
static g4_status prefill_scratch(g4_ctx* ctx, int n, int lrows) {
  PrefillBuffers& p = ctx->prefill;
  if (p.cap >= n) return G4_OK;
  cudaFree(p.xq);
  cudaFree(p.h);
  cudaFree(p.hq);
  cudaFree(p.y);
  cudaFree(p.ginv);
  cudaFree(p.down_sf);
  p = PrefillBuffers{};
  const size_t t = static_cast<size_t>(n), np = pf::kMaxPieces;
  const size_t xq_bytes = np * t * (H / 2 + H / 16);
  const size_t hq_bytes = np * t * (lrows / 2 + round16(lrows / 16));
  g4_status st = check_cuda(ctx, cudaMalloc(&p.xq, xq_bytes), "prefill scratch");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&p.h, t * lrows * 2), "prefill scratch");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&p.hq, hq_bytes), "prefill scratch");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&p.y, t * H * 4), "prefill scratch");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&p.ginv, t * 2 * 4), "prefill scratch");
  if (st == G4_OK && (lrows / 16) % 16 != 0)
    st = check_cuda(ctx, cudaMalloc(&p.down_sf, static_cast<size_t>(H) * round16(lrows / 16)), "prefill scratch");
  if (st == G4_OK) st = check_cuda(ctx, cudaMemsetAsync(p.hq, 0, hq_bytes, ctx->stream), "prefill scratch");
  if (st == G4_OK) p.cap = n;
  return st;
}

g4_status launch_prefill_feedforward(g4_ctx* ctx, int n, uint16_t* residual, const uint16_t* pre_w,
                                     const uint8_t* up_p, const uint8_t* gate_p, const uint8_t* down_p,
                                     const uint8_t* up_s, const uint8_t* gate_s, const uint8_t* down_s,
                                     const float* up_gs, const float* gate_gs, const float* down_gs,
                                     const uint16_t* post_w, const uint16_t* layer_scalar) {
  using namespace pf;
  const int world = ctx->tp_world;
  if (L % (64 * world) != 0) return fail(ctx, G4_ERR_UNSUPPORTED, "prefill: unsupported tensor-parallel world");
  const int pieces = ctx->prefill_pieces;
  if (pieces < 1 || pieces > kMaxPieces) return fail(ctx, G4_ERR_BAD_ARG, "prefill: bad activation piece count");
  const int lrows = L / world;  // this rank's intermediate rows
  const int hsld = round16(lrows / 16);
  g4_status st = prefill_scratch(ctx, n, lrows);
  if (st != G4_OK) return st;
  PrefillBuffers& p = ctx->prefill;
  const size_t cap = static_cast<size_t>(p.cap);
  // per buffer: [piece][cap][codes] then [piece][cap][scales]; the scale padding bytes stay
  // the zeros written at allocation whatever n a call uses
  uint8_t* xq_codes = p.xq;
  uint8_t* xq_scales = p.xq + kMaxPieces * cap * (H / 2);
  uint8_t* hq_codes = p.hq;
  uint8_t* hq_scales = p.hq + kMaxPieces * cap * (lrows / 2);
  float* ginv_x = p.ginv;
  float* ginv_h = p.ginv + cap;
  // 1. RMSNorm + NVFP4 pieces of the normed activations
  {
    int K = H, np = pieces, sld = H / 16;
    size_t cps = cap * (H / 2), sps = cap * (H / 16);
    const uint16_t* x = residual;
    void* a[] = {(void*)&x,   (void*)&K,         (void*)&pre_w, (void*)&np,  (void*)&xq_codes,
                 (void*)&cps, (void*)&xq_scales, (void*)&sld,   (void*)&sps, (void*)&ginv_x};
    if ((st = launch_quant(ctx, H / 16, n, a, "prefill norm+quant")) != G4_OK) return st;
  }
  // 2. gate/up GEMM with the GeGLU epilogue -> h
  {
    CUtensorMap m[6];
    bool ok = make_map(&m[0], gate_p, lrows, H / 2, H / 2, 64, 128, true) &&
              make_map(&m[1], up_p, lrows, H / 2, H / 2, 64, 128, true) &&
              make_map(&m[2], gate_s, lrows, H / 16, H / 16, 64, 16, false) &&
              make_map(&m[3], up_s, lrows, H / 16, H / 16, 64, 16, false) &&
              make_map(&m[4], xq_codes, n, H / 2, H / 2, kTile, 128, true, pieces, cap * (H / 2)) &&
              make_map(&m[5], xq_scales, n, H / 16, H / 16, kTile, 16, false, pieces, cap * (H / 16));
    if (!ok) return fail(ctx, G4_ERR_CUDA, "cuTensorMapEncodeTiled failed (prefill gate/up)");
    GemmArgs ga = {};
    ga.mode = 0;
    ga.n_tok = n;
    ga.m_tiles = lrows / 64;
    ga.k_stages = H / kKStage;
    ga.ginv = ginv_x;
    ga.gs_gate = gate_gs;
    ga.gs_up = up_gs;
    ga.h = p.h;
    ga.h_ld = lrows;
    ga.scr = ctx->buf.scratch;
    ga.budget_ns = ctx->wait_budget_ns;
    if ((st = launch_gemm_p(ctx, pieces, m, ga, "prefill gate/up gemm")) != G4_OK) return st;
  }
  // 3. NVFP4 pieces of h (this rank's columns)
  {
    int K = lrows, np = pieces, sld = hsld;
    size_t cps = cap * (lrows / 2), sps = cap * hsld;
    const uint16_t* x = p.h;
    const uint16_t* nw = nullptr;
    void* a[] = {(void*)&x,   (void*)&K,         (void*)&nw,  (void*)&np,  (void*)&hq_codes,
                 (void*)&cps, (void*)&hq_scales, (void*)&sld, (void*)&sps, (void*)&ginv_h};
    if ((st = launch_quant(ctx, lrows / 16, n, a, "prefill h quant")) != G4_OK) return st;
  }
  // 4. down GEMM -> y (f32, this rank's k-slice)
  {
    const uint8_t* dsf = down_s;
    if (hsld != lrows / 16) {  // scale rows are not a whole number of 16 bytes: pad them
      int cols = lrows / 16, ld = hsld, rows = H;
      uint8_t* dst = p.down_sf;
      void* a[] = {(void*)&down_s, (void*)&cols, (void*)&dst, (void*)&ld, (void*)&rows};
      const int total = H * hsld;
      if ((st = launch_kernel(ctx, (const void*)pf_pad_scales_kernel, dim3((total + 255) / 256), dim3(256), 0, a,
                              false, "prefill scale padding")) != G4_OK)
        return st;
      dsf = p.down_sf;
    }
    CUtensorMap m[6];
    bool ok = make_map(&m[0], down_p, H, lrows / 2, lrows / 2, kTile, 128, true) &&
              make_map(&m[2], dsf, H, hsld, hsld, kTile, 16, false) &&
              make_map(&m[4], hq_codes, n, lrows / 2, lrows / 2, kTile, 128, true, pieces, cap * (lrows / 2)) &&
              make_map(&m[5], hq_scales, n, hsld, hsld, kTile, 16, false, pieces, cap * hsld);
    m[1] = m[0];
    m[3] = m[2];
    if (!ok) return fail(ctx, G4_ERR_CUDA, "cuTensorMapEncodeTiled failed (prefill down)");
    GemmArgs ga = {};
    ga.mode = 1;
    ga.n_tok = n;
    ga.m_tiles = H / kTile;
    ga.k_stages = (lrows + kKStage - 1) / kKStage;  // a partial last stage reads zeros past the end
    ga.ginv = ginv_h;
    ga.y = p.y;
    ga.scr = ctx->buf.scratch;
    ga.budget_ns = ctx->wait_budget_ns;
    if ((st = launch_gemm_p(ctx, pieces, m, ga, "prefill down gemm")) != G4_OK) return st;
  }
  // 5. sum the ranks' partial projections, then post-FF RMSNorm, residual add, layer scalar
  if (world > 1 && (st = allreduce_f32(ctx, p.y, static_cast<size_t>(n) * H)) != G4_OK) return st;
  {
    const float* y = p.y;
    void* a[] = {(void*)&y, (void*)&down_gs, (void*)&post_w, (void*)&layer_scalar, (void*)&residual};
    return launch_kernel(ctx, (const void*)pf_tail_kernel, dim3(n), dim3(kQThreads), 0, a, false, "prefill tail");
  }
}

}  // namespace g4
