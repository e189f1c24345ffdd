// decoder_feedforward: the NVFP4 GeGLU MLP block of one decode token, ONE persistent
// launch of one CTA per SM (drop-in for ops::decoder_feedforward, src/ops.rs:213-253).
//
//   phase 0  stage:   x = RMSNorm(residual, pre_ff)           (src/device/shared/rmsnorm.rs)
//   phase 0  items:   8 gate rows + the same 8 up rows per item;
//                     epilogue h = bf16(gelu_tanh(bf16(bf16(g)*gs_g)) * bf16(bf16(u)*gs_u))
//                     (mlp.rs:13-155 projection, :218-334 GeGLU; tanh per the oracle)
//   grid wait:        every CTA's h rows are visible (bounded spin, error flag on timeout)
//   phase 1  stage:   h as scaled f16 (max |h| gathered with atomicMax in phase 0)
//   phase 1  items:   two units of 8/dq whole down rows, each row cut into dq K segments
//                     (TP1: 2 rows x 4 segments of 3840 per unit, 4 rows per item;
//                     mlp.rs:339-437); one f32 sum per row to scratch
//   final (last CTA): y = bf16(bf16(sum)*gs_d); residual = bf16(bf16(residual +
//                     RMSNorm(y, post_ff)) * layer_scalar)   (ops.rs:248-252, residual.rs)
//
// The producer warp never waits for the grid: it streams phase-1 down weights while the
// last gate/up items of other CTAs finish, so the phase boundary costs no HBM time.
// Under tensor parallelism CTA 0 first sums the ranks' partial y in a one-shot
// all-reduce over NVLink peer memory (peer_allreduce), then runs the same tail on the
// full vector; without peer access the partial y goes to an NCCL all-reduce and a
// one-CTA epilogue kernel instead.
#include <mutex>

#include "g4_internal.h"
#include "g4_stream.cuh"

namespace g4 {

struct MlpOp {
  static constexpr Fmt kFmt = Fmt::NVFP4;
  static constexpr int kPhases = 2;

  uint16_t* residual;
  const uint16_t* pre_w;
  const uint16_t* post_w;
  const uint16_t* layer_scalar;
  const uint8_t* up_p;
  const uint8_t* gate_p;
  const uint8_t* down_p;
  const uint8_t* up_s;
  const uint8_t* gate_s;
  const uint8_t* down_s;
  const float* up_gs;
  const float* gate_gs;
  const float* down_gs;
  Scratch* scr;
  float* part;
  uint16_t* hbuf;
  float* ybuf;      // TP over NCCL: f32 partial y for the all-reduce (nullptr: fused tail)
  PeerXch xch;      // TP over peer memory (world <= 1: not in use)
  int lrows;        // local intermediate rows (L / tp)
  int dq;           // down: K segments per row (pseudo-rows per real row)
  UnitGeom g0, g1;  // gate/up: 8 rows x 3840 K; down: 8/dq rows x full K

  // down: a unit is 8/dq whole rows, an item two units (A, B) = 16/dq rows
  __device__ int down_rows() const { return 8 / dq; }
  __device__ int items(int ph) const { return ph == 0 ? lrows / 8 : H / (2 * down_rows()); }
  __device__ UnitGeom geom(int ph) const { return ph == 0 ? g0 : g1; }
  __device__ UnitDesc unit(int ph, int it, int half) const {
    UnitDesc u;
    if (ph == 0) {
      const uint8_t* p = half ? up_p : gate_p;
      const uint8_t* s = half ? up_s : gate_s;
      u.codes = p + static_cast<size_t>(it) * 8 * (H / 2);
      u.scales = s + static_cast<size_t>(it) * 8 * (H / 16);
      u.code_stride = H / 2;
      u.scale_stride = H / 16;
    } else {
      const size_t cstride = lrows / 2, sstride = lrows / 16;
      const size_t row0 = static_cast<size_t>(2 * it + half) * down_rows();
      u.codes = down_p + row0 * cstride;
      u.scales = down_s + row0 * sstride;
      u.code_stride = static_cast<uint32_t>(cstride);
      u.scale_stride = static_cast<uint32_t>(sstride);
    }
    return u;
  }
  __device__ uint32_t* status() const { return &scr->status; }
  __device__ uint32_t* done_counter() const { return &scr->mlp_done; }
  // At kernel start CTA c pulls line c of the pre-FF norm weight (read by every CTA's
  // staging) and, for the fused tail, line c of post_w (CTA 0: the scalars) into L2.
  __device__ void prefetch_l2(int cta, int lane) const {
    constexpr int kBytes = H * 2, kLines = kBytes / 128 + 1;
    if (cta >= kLines) return;
    const int off = min(cta * 128, kBytes - 1);
    if (lane == 0) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(pre_w) + off);
    if (ybuf != nullptr) return;  // TP: the tail runs in its own kernel after the all-reduce
    if (lane == 1) prefetch_l2_keep(reinterpret_cast<const uint8_t*>(post_w) + off);
    if (lane == 2 && cta == 0) {
      prefetch_l2_keep(layer_scalar);
      prefetch_l2_keep(down_gs);
    }
  }
  __device__ bool has_final() const { return true; }

  __device__ void stage(StreamSmem& sm, uint8_t* xbuf, int ph, int tid, const XLayout& xl) const {
    uint16_t* xs = reinterpret_cast<uint16_t*>(xbuf);
    if (ph == 0) {
      const int e = stage_rmsnorm(residual, pre_w, H, xs, true, sm.scratch, xl);
      if (tid == 0) {
        sm.xexp = e;
        sm.scratch[40] = __ldg(gate_gs);
        sm.scratch[41] = __ldg(up_gs);
      }
    } else {
      // h and its max were published before the grid barrier (acquired by its thread 0,
      // then bar.sync): plain L2 loads, 8 h values per 16-byte load, all issued together.
      constexpr int kG = 4;  // lrows <= kG * 8 * kConsumerThreads
      static_assert(kG * 8 * kConsumerThreads >= L, "phase-1 staging must cover L");
      uint4 hv[kG];
#pragma unroll
      for (int k = 0; k < kG; ++k) {
        const int gi = tid + k * kConsumerThreads;
        if (gi * 8 < lrows) hv[k] = __ldcg(reinterpret_cast<const uint4*>(hbuf) + gi);
      }
      const float amax = __uint_as_float(__ldcg(&scr->mlp_amax));
      const int e = f16_scale_exponent(amax);
      const float sc = ldexpf(1.0f, e);
#pragma unroll
      for (int k = 0; k < kG; ++k) {
        const int gi = tid + k * kConsumerThreads;
        if (gi * 8 < lrows) {
          const uint32_t w[4] = {hv[k].x, hv[k].y, hv[k].z, hv[k].w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[i] = pack_u16x2(f32_to_f16(bf16_to_f32(static_cast<uint16_t>(w[i] & 0xFFFFu)) * sc),
                              f32_to_f16(bf16_to_f32(static_cast<uint16_t>(w[i] >> 16)) * sc));
          *reinterpret_cast<uint4*>(xs + x_pos(static_cast<uint32_t>(gi) * 8u, xl)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      if (tid == 0) sm.xexp = e;
    }
  }

  __device__ bool between_phases(StreamSmem& sm, int ph, uint64_t deadline) const {
    return grid_wait(&scr->mlp_sync, gridDim.x, deadline, &scr->status, sm);
  }

  __device__ void item_epilogue(StreamSmem& sm, int ph, int it, int lane, float v) const {
    const float unscale = ldexpf(1.0f, -sm.xexp);
    if (ph == 0) {
      const float up = __shfl_down_sync(0xffffffffu, v, 8);
      float hv = 0.f;
      if (lane < 8) {
        const float g2 = round_bf16(round_bf16(v * unscale) * sm.scratch[40]);
        const float u2 = round_bf16(round_bf16(up * unscale) * sm.scratch[41]);
        hv = round_bf16(round_bf16(gelu_tanh(g2)) * u2);
        hbuf[it * 8 + lane] = f32_to_bf16(hv);
      }
      const float m = warp_max(fabsf(hv));
      if (lane == 0) atomicMax(&scr->mlp_amax, __float_as_uint(m));
    } else {
      const float y = sum_pseudo_rows(v, lane, dq);
      if (lane < 2 * down_rows()) part[it * 2 * down_rows() + lane] = y * unscale;
    }
  }

  // Thread tid < H/8 owns outputs [8*tid, 8*tid + 8): it issues all of its loads (the
  // down sums, the residual, the post-FF norm weight) before any math, so the tail of
  // the launch pays one memory latency, not one per output.
  __device__ void final_epilogue(StreamSmem& sm, uint8_t*, int tid) const {
    const bool mine = tid < H / 8;
    float y[8];
    uint4 rv = make_uint4(0u, 0u, 0u, 0u), wv = rv;
    if (mine) {
      const float4 p0 = __ldcg(reinterpret_cast<const float4*>(part) + 2 * tid);
      const float4 p1 = __ldcg(reinterpret_cast<const float4*>(part) + 2 * tid + 1);
      y[0] = p0.x, y[1] = p0.y, y[2] = p0.z, y[3] = p0.w, y[4] = p1.x, y[5] = p1.y, y[6] = p1.z, y[7] = p1.w;
      if (ybuf == nullptr) {
        rv = *reinterpret_cast<const uint4*>(residual + 8 * tid);
        wv = __ldg(reinterpret_cast<const uint4*>(post_w) + tid);
      }
    }
    if (ybuf != nullptr) {
      if (mine) {
        reinterpret_cast<float4*>(ybuf)[2 * tid] = make_float4(y[0], y[1], y[2], y[3]);
        reinterpret_cast<float4*>(ybuf)[2 * tid + 1] = make_float4(y[4], y[5], y[6], y[7]);
      }
    } else if (xch.world <= 1 || peer_allreduce(xch, &scr->xch_epoch, y, tid, &scr->status, sm)) {
      const float gsd = __ldg(down_gs);
      float ss = 0.f;
      if (mine) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float d2 = round_bf16(round_bf16(y[i]) * gsd);
          y[i] = d2;
          ss = __fadd_rn(ss, __fmul_rn(d2, d2));
        }
      }
      const float r = rms_factor(consumer_sum(ss, sm.scratch), H);
      const float ls = bf16_to_f32(layer_scalar[0]);
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
            const float r2 = round_bf16(__fadd_rn(res, nb));
            h2[j] = f32_to_bf16(__fmul_rn(r2, ls));
          }
          o[i] = pack_u16x2(h2[0], h2[1]);
        }
        *reinterpret_cast<uint4*>(residual + 8 * tid) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (tid == 0) {
      scr->mlp_sync = 0u;
      scr->mlp_amax = 0u;
    }
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    mlp_kernel(const MlpOp op, const StreamLayout lay, uint32_t slot_bytes, uint64_t budget_ns) {
  stream_body(op, lay, slot_bytes, budget_ns);
}

// TP epilogue after the all-reduce of y (one CTA): the same math as the fused tail.
__global__ void __launch_bounds__(1024) mlp_tp_epilogue_kernel(const float* __restrict__ y, const float* down_gs,
                                                               const uint16_t* __restrict__ post_w,
                                                               const uint16_t* __restrict__ layer_scalar,
                                                               uint16_t* __restrict__ residual) {
  __shared__ float red[32];
  __shared__ float yb[H];
  const float gsd = __ldg(down_gs);
  float ss = 0.f;
  for (int n = threadIdx.x; n < H; n += blockDim.x) {
    const float d2 = round_bf16(round_bf16(y[n]) * gsd);
    yb[n] = d2;
    ss = __fadd_rn(ss, __fmul_rn(d2, d2));
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) tot += red[w];
  const float r = rms_factor(tot, H);
  const float ls = bf16_to_f32(layer_scalar[0]);
  for (int n = threadIdx.x; n < H; n += blockDim.x) {
    const float nb = round_bf16(__fmul_rn(__fmul_rn(yb[n], r), bf16_to_f32(post_w[n])));
    const float r2 = round_bf16(__fadd_rn(bf16_to_f32(residual[n]), nb));
    residual[n] = f32_to_bf16(__fmul_rn(r2, ls));
  }
}

static constexpr uint32_t kMlpSlots = 8;

g4_status launch_decoder_feedforward(g4_ctx* ctx, uint16_t* residual, const uint16_t* pre_w, const uint8_t* up_p,
                                     const uint8_t* gate_p, const uint8_t* down_p, const uint8_t* up_s,
                                     const uint8_t* gate_s, const uint8_t* down_s, const float* up_gs,
                                     const float* gate_gs, const float* down_gs, const uint16_t* post_w,
                                     const uint16_t* layer_scalar) {
  if (mlp_tc_enabled(ctx))
    return launch_decoder_feedforward_tc(ctx, residual, pre_w, up_p, gate_p, down_p, up_s, gate_s, down_s, up_gs,
                                         gate_gs, down_gs, post_w, layer_scalar);
  MlpOp op;
  op.residual = residual;
  op.pre_w = pre_w;
  op.post_w = post_w;
  op.layer_scalar = layer_scalar;
  op.up_p = up_p;
  op.gate_p = gate_p;
  op.down_p = down_p;
  op.up_s = up_s;
  op.gate_s = gate_s;
  op.down_s = down_s;
  op.up_gs = up_gs;
  op.gate_gs = gate_gs;
  op.down_gs = down_gs;
  op.scr = ctx->buf.scratch;
  op.part = ctx->buf.part;
  op.hbuf = ctx->buf.hbuf;
  const bool tp_nccl = ctx->tp_world > 1 && ctx->peers.world <= 1;
  op.ybuf = tp_nccl ? ctx->buf.ybuf : nullptr;
  op.xch = ctx->peers;
  op.lrows = L / ctx->tp_world;
  // down rows hold lrows K elements: cut into dq segments of 3840 (one segment when smaller)
  op.dq = (op.lrows % 3840 == 0) ? op.lrows / 3840 : 1;
  op.g0 = make_geom(Fmt::NVFP4, H / 2, 1);
  op.g1 = make_geom(Fmt::NVFP4, op.lrows / 2 / op.dq, op.dq);
  if (!geom_ok(op.g0, H / 2, H / 16) || !geom_ok(op.g1, op.lrows / 2, op.lrows / 16))
    return fail(ctx, G4_ERR_UNSUPPORTED, "MLP shard geometry");
  const uint32_t slot_bytes = op.g0.slot_bytes > op.g1.slot_bytes ? op.g0.slot_bytes : op.g1.slot_bytes;
  // activation buffer: h as f16 (phase 1) or the f32 down-projection sums (final epilogue)
  const uint32_t x_bytes = static_cast<uint32_t>(op.lrows * 2 > H * 4 ? op.lrows * 2 : H * 4);
  const StreamLayout lay = make_layout(slot_bytes, kMlpSlots, x_bytes);
  {
    const g4_status st = allow_max_dynamic_smem(ctx, (const void*)mlp_kernel, lay.total, "mlp_kernel smem");
    if (st != G4_OK) return st;
  }
  const uint64_t budget = ctx->wait_budget_ns;
  void* args[] = {(void*)&op, (void*)&lay, (void*)&slot_bytes, (void*)&budget};
  // Not a cooperative launch, so that the next launch's CTAs can take SMs as this one's
  // exit (programmatic dependent launch).  The grid barrier between the phases needs
  // every CTA resident at some point, which holds without the cooperative guarantee:
  // the grid is one CTA per SM, a CTA's shared memory excludes a second one, and CTAs
  // waiting at the barrier only wait for SMs held by work that finishes on its own.  Its
  // bounded wait turns anything else into a device status error, not a hang.
  g4_status st = launch_kernel(ctx, (const void*)mlp_kernel, dim3(ctx->sm_count), dim3(kThreads), lay.total, args,
                               false, "launch mlp_kernel");
  if (st != G4_OK) return st;
  if (tp_nccl) {
    st = allreduce_f32(ctx, ctx->buf.ybuf, H);
    if (st != G4_OK) return st;
    mlp_tp_epilogue_kernel<<<1, 1024, 0, ctx->stream>>>(ctx->buf.ybuf, down_gs, post_w, layer_scalar, residual);
    st = check_cuda(ctx, cudaGetLastError(), "launch mlp_tp_epilogue");
  }
  return st;
}

}  // namespace g4

// ======================================================================= no-alloc variant
// g4_decoder_feedforward_noalloc runs mlp_kernel above with its scratch in one fixed
// array of this translation unit instead of a context's cudaMalloc'd buffers, for hosts
// that own all device memory and forbid a library from allocating.  Layout of the
// array (every offset a multiple of 256 bytes):
//   [0, 1 KiB)            Scratch counters and the device status word
//   [1 KiB, +H*4)         f32 down-projection sums, one per output row
//   [16 KiB, +max*2)      bf16 intermediate vector h
namespace {

constexpr size_t kNoAllocPartOff = 1024;
constexpr size_t kNoAllocHOff = kNoAllocPartOff + static_cast<size_t>(g4::H) * 4;
constexpr size_t kNoAllocBytes = kNoAllocHOff + static_cast<size_t>(G4_NOALLOC_MAX_INTERMEDIATE) * 2;
static_assert(sizeof(g4::Scratch) <= kNoAllocPartOff, "counter block overflows its 1 KiB");
static_assert(kNoAllocHOff % 256 == 0, "h must stay 256-byte aligned");
static_assert(kNoAllocBytes == G4_NOALLOC_SCRATCH_BYTES, "header states the array size");

// In host code this name only identifies the array; its device address comes from
// cudaGetSymbolAddress on each device.
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

struct NoAllocDevice {
  bool ready = false;             // set up successfully (a failed set-up is retried)
  unsigned char* base = nullptr;  // this device's address of g_noalloc_scratch
  int sm_count = 0;
  int smem_dyn_max = 0;           // dynamic shared memory mlp_kernel may use per launch
  bool coop = false;
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current (under g_noalloc_mu; a failure leaves the
// device not ready, so the next call tries again).  Allocates nothing: the array belongs
// to the module image the runtime loaded on this device.  It also raises mlp_kernel's
// dynamic shared-memory limit to the opt-in maximum minus the kernel's static shared
// memory: the same value the context path sets, so neither path lowers it under the other.
cudaError_t noalloc_setup(NoAllocDevice& d, int dev) {
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  int coop = 0, optin = 0, sms = 0;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess)
    return e;
  cudaFuncAttributes fa = {};
  if ((e = cudaFuncGetAttributes(&fa, (const void*)g4::mlp_kernel)) != cudaSuccess) return e;
  const int dyn_max = optin - static_cast<int>(fa.sharedSizeBytes);
  if (dyn_max <= 0) return cudaErrorInvalidConfiguration;
  if ((e = cudaFuncSetAttribute((const void*)g4::mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_max)) !=
      cudaSuccess)
    return e;
  d.sm_count = sms;
  d.smem_dyn_max = dyn_max;
  d.coop = coop != 0;
  d.base = static_cast<unsigned char*>(ptr);
  d.ready = true;
  return cudaSuccess;
}

bool noalloc_aligned(const void* p, uintptr_t a) {
  return p != nullptr && reinterpret_cast<uintptr_t>(p) % a == 0;
}

}  // namespace

extern "C" g4_status g4_decoder_feedforward_noalloc(
    g4_stream_t stream, uint32_t intermediate_size, g4_bf16* residual, const g4_bf16* pre_ff_rms_weight,
    const g4_f4x2* up_weight_packed, const g4_f4x2* gate_weight_packed, const g4_f4x2* down_weight_packed,
    const g4_f8e4m3* up_weight_scale, const g4_f8e4m3* gate_weight_scale, const g4_f8e4m3* down_weight_scale,
    const float* up_global_scale, const float* gate_global_scale, const float* down_global_scale,
    const g4_bf16* post_ff_rms_weight, const g4_bf16* layer_scalar) {
  using namespace g4;
  // sizes first: nothing below runs for a call that the scratch array cannot hold
  const uint32_t n = intermediate_size;
  if (n > G4_NOALLOC_MAX_INTERMEDIATE) return G4_ERR_TOO_LARGE;
  if (n == 0) return G4_ERR_BAD_ARG;
  const uint32_t dq = (n % 3840u == 0u) ? n / 3840u : 1u;
  MlpOp op;
  op.lrows = static_cast<int>(n);
  op.dq = static_cast<int>(dq);
  op.g0 = make_geom(Fmt::NVFP4, H / 2, 1);
  op.g1 = make_geom(Fmt::NVFP4, n / 2u / dq, dq);
  // the shapes the kernel's down-phase geometry is built and tested for
  const bool shape_ok = (n <= 3840u && n % 128u == 0u) || n == 7680u || n == 15360u;
  if (!shape_ok || !geom_ok(op.g0, H / 2, H / 16) || !geom_ok(op.g1, n / 2u, n / 16u)) return G4_ERR_UNSUPPORTED;
  const void* p16[] = {residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed, down_weight_packed,
                       up_weight_scale, gate_weight_scale, down_weight_scale, post_ff_rms_weight, layer_scalar};
  for (const void* p : p16)
    if (!noalloc_aligned(p, 16)) return G4_ERR_BAD_ARG;
  const void* p4[] = {up_global_scale, gate_global_scale, down_global_scale};
  for (const void* p : p4)
    if (!noalloc_aligned(p, 4)) return G4_ERR_BAD_ARG;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G4_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return G4_ERR_UNSUPPORTED;
  NoAllocDevice& d = g_noalloc_dev[dev];
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!d.ready && noalloc_setup(d, dev) != cudaSuccess) {
      (void)cudaGetLastError();
      return G4_ERR_CUDA;
    }
  }
  if (!d.coop) return G4_ERR_UNSUPPORTED;

  const uint32_t slot_bytes = op.g0.slot_bytes > op.g1.slot_bytes ? op.g0.slot_bytes : op.g1.slot_bytes;
  const uint32_t x_bytes = (n * 2u > static_cast<uint32_t>(H) * 4u) ? n * 2u : static_cast<uint32_t>(H) * 4u;
  const StreamLayout lay = make_layout(slot_bytes, kMlpSlots, x_bytes);
  if (lay.total > static_cast<uint32_t>(d.smem_dyn_max)) return G4_ERR_UNSUPPORTED;

  op.residual = residual;
  op.pre_w = pre_ff_rms_weight;
  op.post_w = post_ff_rms_weight;
  op.layer_scalar = layer_scalar;
  op.up_p = up_weight_packed;
  op.gate_p = gate_weight_packed;
  op.down_p = down_weight_packed;
  op.up_s = up_weight_scale;
  op.gate_s = gate_weight_scale;
  op.down_s = down_weight_scale;
  op.up_gs = up_global_scale;
  op.gate_gs = gate_global_scale;
  op.down_gs = down_global_scale;
  op.scr = reinterpret_cast<Scratch*>(d.base);
  op.part = reinterpret_cast<float*>(d.base + kNoAllocPartOff);
  op.hbuf = reinterpret_cast<uint16_t*>(d.base + kNoAllocHOff);
  op.ybuf = nullptr;
  op.xch = PeerXch{};

  // The counters and status word must start at zero; a call that gave up on a device
  // wait may have left them set.
  if (cudaMemsetAsync(d.base, 0, sizeof(Scratch), stream) != cudaSuccess) return G4_ERR_CUDA;
  const uint64_t budget = 2000000000ull;  // the context default: 2 s per device-side wait
  void* args[] = {(void*)&op, (void*)&lay, (void*)&slot_bytes, (void*)&budget};
  if (cudaLaunchCooperativeKernel((const void*)mlp_kernel, dim3(d.sm_count), dim3(kThreads), args, lay.total,
                                  stream) != cudaSuccess)
    return G4_ERR_CUDA;
  return G4_OK;
}
