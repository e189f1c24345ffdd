// Small kernels of the decode path: token embedding, device argmax, dequant checks.
#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {

// ops::embed_token (src/ops.rs:9-36): out = bf16(row * bf16(EMBED_SCALE)), the row at a
// device-resident byte offset into the [W, H] table.  The oracle multiplies by the
// scale rounded to bf16 (Gemma4TextScaledWordEmbedding: embed_scale.to(weight.dtype)).
__global__ void embed_kernel(const uint16_t* __restrict__ table, const int32_t* __restrict__ offset,
                             long long table_elems, uint16_t* __restrict__ out, uint32_t* status) {
  const long long e0 = static_cast<long long>(__ldg(offset)) / 2;
  if (e0 < 0 || e0 + H > table_elems || (e0 % H) != 0) {
    if (threadIdx.x == 0) atomicOr(status, DEV_ERR_BAD_OFFSET);
    return;
  }
  const float scale = round_bf16(EMBED_SCALE);
  for (int i = threadIdx.x; i < H; i += blockDim.x) out[i] = f32_to_bf16(bf16_to_f32(table[e0 + i]) * scale);
}

// First index of the maximum of a bf16 vector (ties -> lowest index, like torch.argmax).
__global__ void __launch_bounds__(1024) argmax_kernel(const uint16_t* __restrict__ x, int n, int32_t* out) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  float best = -CUDART_INF_F;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x * 8; i < n; i += blockDim.x * 8) {
    if (i + 8 <= n) {
      const uint4 w = *reinterpret_cast<const uint4*>(x + i);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf16_to_f32(static_cast<uint16_t>(ww[j] & 0xFFFFu));
        const float b = bf16_to_f32(static_cast<uint16_t>(ww[j] >> 16));
        if (a > best) { best = a; idx = i + 2 * j; }
        if (b > best) { best = b; idx = i + 2 * j + 1; }
      }
    } else {
      for (int j = i; j < n; ++j) {
        const float a = bf16_to_f32(x[j]);
        if (a > best) { best = a; idx = j; }
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
  }
  if ((threadIdx.x & 31) == 0) { bv[threadIdx.x >> 5] = best; bi[threadIdx.x >> 5] = idx; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = bv[0];
    int id = bi[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (bv[w] > b || (bv[w] == b && bi[w] < id)) { b = bv[w]; id = bi[w]; }
    *out = (id == 0x7fffffff) ? 0 : id;
  }
}

// Dequantisation through the same conversions the GEMV kernels use.
__global__ void dequant_nvfp4_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scale, int rows,
                                     int cols, uint16_t* __restrict__ out) {
  const long long pairs = static_cast<long long>(rows) * cols / 2;
  for (long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; p < pairs;
       p += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = 2 * p;
    const long long r = e / cols, c = e % cols;
    const uint32_t codes = cvt_e2m1x2(packed[p]);
    const uint32_t s = cvt_e4m3x2(static_cast<uint16_t>(scale[r * (cols / 16) + c / 16]));
    const uint32_t v = hmul2_u32(codes, dup_lo(s));
    const __half2 h = *reinterpret_cast<const __half2*>(&v);
    out[e] = f32_to_bf16(__low2float(h));
    out[e + 1] = f32_to_bf16(__high2float(h));
  }
}

__global__ void dequant_fp8_kernel(const uint8_t* __restrict__ w, long long count, uint16_t* __restrict__ out) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = f32_to_bf16(e4m3_value(w[i]));
}

g4_status launch_embed(g4_ctx* ctx, const uint16_t* table, const int32_t* offset, uint16_t* out) {
  embed_kernel<<<1, 480, 0, ctx->stream>>>(table, offset, static_cast<long long>(W) * H, out, &ctx->buf.scratch->status);
  return check_cuda(ctx, cudaGetLastError(), "embed_token");
}
g4_status launch_argmax(g4_ctx* ctx, const uint16_t* x, int n, int32_t* out) {
  argmax_kernel<<<1, 1024, 0, ctx->stream>>>(x, n, out);
  return check_cuda(ctx, cudaGetLastError(), "argmax");
}
g4_status launch_dequant_nvfp4(g4_ctx* ctx, const uint8_t* p, const uint8_t* s, int rows, int cols, uint16_t* out) {
  dequant_nvfp4_kernel<<<4 * ctx->sm_count, 256, 0, ctx->stream>>>(p, s, rows, cols, out);
  return check_cuda(ctx, cudaGetLastError(), "dequant_nvfp4");
}
g4_status launch_dequant_fp8(g4_ctx* ctx, const uint8_t* w, long long count, uint16_t* out) {
  dequant_fp8_kernel<<<4 * ctx->sm_count, 256, 0, ctx->stream>>>(w, count, out);
  return check_cuda(ctx, cudaGetLastError(), "dequant_fp8");
}

}  // namespace g4
