// Top-k / top-p (nucleus) sampling on the device (src/host/sampling.rs:20-72), replacing
// the logits read-back and host sampling of src/host/generate.rs:135-143.
//
// The reference: keep the top (top_k + |banned|) logits, sort them descending, drop
// banned ids (unless that leaves none), keep top_k, p_i = exp((l_i - l_0) / T) / sum,
// nucleus = the shortest prefix whose running sum reaches top_p, threshold = u * (sum of
// the nucleus), and the first id whose running sum reaches the threshold (the last one
// otherwise).  Here:
//   1. select: CTA c sorts the 64-bit keys of its 2048 logits (bitonic, in shared
//      memory) and writes its top kk = top_k + |banned| keys; key = (the bf16 logit's
//      order-preserving bits << 32) | ~global index, so equal logits rank by lower index
//      (the reference's unstable sort leaves their order open);
//   2. (tensor parallel) each rank reduces its candidates to its top kk, the ranks'
//      candidates are all-gathered (NCCL), so every rank sees the same kk * world keys;
//   3. sample: one CTA sorts the candidates, keeps the global top kk, and one thread runs
//      the reference's sequential f32 arithmetic on them (at most 128 values) with the
//      uniform draw u read from device memory.
// All three steps are deterministic; every rank of a TP group draws the same id.
#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {
namespace smp {

constexpr int kChunk = 2048;        // logits per select CTA
constexpr int kSelThreads = 512;
constexpr int kMaxKeep = 128;       // top_k + |banned|
constexpr int kMaxCand = 16384;     // keys the sample CTA sorts
constexpr int kSampleThreads = 1024;

__device__ __forceinline__ uint64_t make_key(uint16_t bits, uint32_t index) {
  const uint32_t ord = (bits & 0x8000u) ? (~static_cast<uint32_t>(bits) & 0xFFFFu) : (bits | 0x8000u);
  return (static_cast<uint64_t>(ord) << 32) | (0xFFFFFFFFu - index);
}
__device__ __forceinline__ uint32_t key_index(uint64_t key) { return 0xFFFFFFFFu - static_cast<uint32_t>(key); }
__device__ __forceinline__ float key_logit(uint64_t key) {
  const uint32_t ord = static_cast<uint32_t>(key >> 32);
  const uint16_t bits = (ord & 0x8000u) ? static_cast<uint16_t>(ord & 0x7FFFu) : static_cast<uint16_t>(~ord & 0xFFFFu);
  return bf16_to_f32(bits);
}

// In-place bitonic sort of n (a power of two) keys in shared memory, descending.
__device__ void bitonic_desc(uint64_t* k, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));  // first element of the pair
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;          // direction of this sub-sequence
        const uint64_t a = k[lo], b = k[hi];
        if ((a < b) == desc) {
          k[lo] = b;
          k[hi] = a;
        }
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(const uint16_t* __restrict__ logits, int n,
                                                             uint32_t base, int kk, uint64_t* __restrict__ cand) {
  __shared__ uint64_t keys[kChunk];
  pdl_wait();  // the logits come from the previous kernel
  const int c0 = blockIdx.x * kChunk;
  for (int i = threadIdx.x; i < kChunk; i += kSelThreads) {
    const int j = c0 + i;
    keys[i] = (j < n) ? make_key(logits[j], base + static_cast<uint32_t>(j)) : 0ull;
  }
  bitonic_desc(keys, kChunk);
  for (int i = threadIdx.x; i < kk; i += kSelThreads) cand[static_cast<size_t>(blockIdx.x) * kk + i] = keys[i];
}

// The decode runtime's draw for the step at `pos`: splitmix64 of seed + pos * golden
// ratio, top 24 bits as a float in [0, 1) (the same construction as a uniform f32 from
// 24 random bits; reproducible on the host).
__device__ __forceinline__ float draw_uniform(uint64_t seed, int pos) {
  uint64_t z = seed + static_cast<uint64_t>(static_cast<uint32_t>(pos)) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

struct SampleArgs {
  int m;           // candidate keys
  int kk;          // top_k + banned (kept before filtering)
  int top_k;
  int n_banned;
  int32_t banned[kMaxKeep];
  float temperature;
  float top_p;
  int reduce;      // 1: write the top kk keys to out_keys (a rank's share), 0: sample
  const int32_t* draw_pos;  // non-null: u = draw_uniform(seed, *draw_pos) instead of *uniform
  uint64_t seed;
};

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const uint64_t* __restrict__ cand,
                                                                const float* __restrict__ uniform,
                                                                uint64_t* __restrict__ out_keys,
                                                                int32_t* __restrict__ out_index,
                                                                const __grid_constant__ SampleArgs a) {
  extern __shared__ uint64_t sk[];
  pdl_wait();
  int n2 = 1;
  while (n2 < a.m) n2 <<= 1;
  for (int i = threadIdx.x; i < n2; i += kSampleThreads) sk[i] = (i < a.m) ? cand[i] : 0ull;
  bitonic_desc(sk, n2);
  if (a.reduce) {
    for (int i = threadIdx.x; i < a.kk; i += kSampleThreads) out_keys[i] = sk[i];
    return;
  }
  if (threadIdx.x != 0) return;
  // the reference's arithmetic, in its order (src/host/sampling.rs:20-72)
  int ids[kMaxKeep];
  float lg[kMaxKeep];
  int cnt = 0;
  for (int i = 0; i < a.kk; ++i) {
    const int id = static_cast<int>(key_index(sk[i]));
    bool ban = false;
    for (int b = 0; b < a.n_banned; ++b) ban = ban || (a.banned[b] == id);
    if (!ban) {
      ids[cnt] = id;
      lg[cnt] = key_logit(sk[i]);
      ++cnt;
    }
  }
  if (cnt == 0) {  // every candidate banned: keep them all
    for (int i = 0; i < a.kk; ++i) {
      ids[i] = static_cast<int>(key_index(sk[i]));
      lg[i] = key_logit(sk[i]);
    }
    cnt = a.kk;
  }
  if (cnt > a.top_k) cnt = a.top_k;
  const float t = fmaxf(a.temperature, 1e-5f);
  float p[kMaxKeep];
  float sum = 0.f;
  for (int i = 0; i < cnt; ++i) {
    p[i] = expf(__fdiv_rn(__fsub_rn(lg[i], lg[0]), t));
    sum = __fadd_rn(sum, p[i]);
  }
  for (int i = 0; i < cnt; ++i) p[i] = __fdiv_rn(p[i], sum);
  int nucleus = cnt;
  float cum = 0.f;
  for (int i = 0; i < cnt; ++i) {
    cum = __fadd_rn(cum, p[i]);
    if (cum >= a.top_p) {
      nucleus = i + 1;
      break;
    }
  }
  float nsum = 0.f;
  for (int i = 0; i < nucleus; ++i) nsum = __fadd_rn(nsum, p[i]);
  const float u = a.draw_pos != nullptr ? draw_uniform(a.seed, *a.draw_pos) : *uniform;
  const float threshold = __fmul_rn(u, nsum);
  int pick = ids[nucleus - 1];
  float acc = 0.f;
  for (int i = 0; i < nucleus; ++i) {
    acc = __fadd_rn(acc, p[i]);
    if (acc >= threshold) {
      pick = ids[i];
      break;
    }
  }
  *out_index = pick;
}

}  // namespace smp

g4_status launch_sample(g4_ctx* ctx, const uint16_t* logits, int n, float temperature, int top_k, float top_p,
                        const int32_t* banned, int n_banned, const float* uniform, int32_t* out_index,
                        const int32_t* draw_pos, uint64_t seed) {
  using namespace smp;
  const int kk = top_k + n_banned < n * ctx->tp_world ? top_k + n_banned : n * ctx->tp_world;
  const int grid = (n + kChunk - 1) / kChunk;
  if (static_cast<size_t>(grid) * kk > kMaxCand || kk > kMaxKeep)
    return fail(ctx, G4_ERR_UNSUPPORTED, "sampling: too many candidates (top_k + banned <= 128, n <= 262144)");
  uint64_t* cand = ctx->buf.cand;
  uint64_t* share = cand + kMaxCand;                 // [kMaxKeep] this rank's top kk
  uint64_t* gathered = share + kMaxKeep;             // [kMaxTp * kMaxKeep]
  const uint32_t base = static_cast<uint32_t>(ctx->tp_rank) * static_cast<uint32_t>(n);
  int kk_sel = kk < n ? kk : n;  // a rank holds at most n candidates
  {
    void* args[] = {(void*)&logits, (void*)&n, (void*)&base, (void*)&kk_sel, (void*)&cand};
    g4_status st = launch_kernel(ctx, (const void*)select_kernel, dim3(grid), dim3(kSelThreads), 0, args, false,
                                 "sampling select");
    if (st != G4_OK) return st;
  }
  SampleArgs sa = {};
  sa.kk = kk;
  sa.top_k = top_k;
  sa.n_banned = n_banned;
  for (int i = 0; i < n_banned; ++i) sa.banned[i] = banned[i];
  sa.temperature = temperature;
  sa.top_p = top_p;
  sa.draw_pos = draw_pos;
  sa.seed = seed;
  const void* fn = (const void*)sample_kernel;
  g4_status st = allow_max_dynamic_smem(ctx, fn, kMaxCand * 8, "sampling");
  if (st != G4_OK) return st;
  const uint64_t* src = cand;
  sa.m = grid * kk_sel;
  if (ctx->tp_world > 1) {
    // this rank's top kk, then every rank's, gathered
    SampleArgs ra = sa;
    ra.kk = kk_sel;
    ra.reduce = 1;
    uint64_t* no_keys = share;
    int32_t* no_index = nullptr;
    void* a1[] = {(void*)&src, (void*)&uniform, (void*)&no_keys, (void*)&no_index, (void*)&ra};
    if ((st = launch_kernel(ctx, fn, dim3(1), dim3(kSampleThreads), kMaxCand * 8, a1, false, "sampling reduce")) !=
        G4_OK)
      return st;
    if ((st = allgather_u64n(ctx, share, gathered, kk_sel)) != G4_OK) return st;
    src = gathered;
    sa.m = kk_sel * ctx->tp_world;
  }
  sa.reduce = 0;
  uint64_t* keys_out = nullptr;
  void* a2[] = {(void*)&src, (void*)&uniform, (void*)&keys_out, (void*)&out_index, (void*)&sa};
  size_t smem = 8;
  while (smem < static_cast<size_t>(sa.m) * 8) smem <<= 1;
  if (smem < 8 * 2) smem = 16;
  return launch_kernel(ctx, fn, dim3(1), dim3(kSampleThreads), smem, a2, false, "sampling");
}

}  // namespace g4
