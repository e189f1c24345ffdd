// Decode runtime: the reference's host-side decode step on this library's kernels.
//
//  g4_model     the per-layer weight set of src/host/load.rs:10-87 (MlpWeights,
//               SlidingLayer, FullLayer, Model), filled by checkpoint tensor name; layer i
//               is a full-attention layer iff i % 6 == 5 (load.rs:369-376).
//  g4_workspace src/host/runtime.rs:135-211 (Workspace): RoPE tables built as rope_data
//               does (:271-299), the per-layer KV caches (sliding ring [Ts, Ns, Ds]; full
//               layers one contiguous [rows, Df] array whose 512-row pages are the
//               reference's page tensors), the current mask row, the device-resident
//               offsets of set_position_offsets (:213-228), the decode scratch of Decode
//               (:301-309) and the logits.
//  one step     Decode::run / run_layers / sliding / full / mlp (:311-513): embed_token,
//               48 x {project_qkv, attention, attention_output, decoder_feedforward},
//               final_norm_and_logits, then a device argmax (replacing the logits read-back
//               and host sampling of src/host/generate.rs:130-143) that also advances the
//               position.  Everything position-dependent is read from device memory, so a
//               step is captured once as a CUDA graph and replayed for every position.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {

// launchers of the other translation units
g4_status launch_qkv(g4_ctx*, bool, bool, const uint16_t*, const uint8_t* const[3], const uint8_t* const[3],
                     const uint16_t* const[3], const float* const[3], const uint16_t*, const uint16_t*,
                     const uint16_t*, const int32_t*, const int32_t*, const uint16_t*, const uint16_t*, uint16_t*,
                     uint16_t*, uint16_t*, long long);
g4_status launch_oproj(g4_ctx*, bool, bool, const uint16_t*, const float*, const uint16_t*, const uint8_t*,
                       const uint8_t*, const uint16_t*, const float*, uint16_t*);
g4_status launch_lm_head(g4_ctx*, const uint16_t*, const uint16_t*, const uint16_t*, uint16_t*);
g4_status launch_sliding_attention(g4_ctx*, const uint16_t*, const uint16_t*, const uint16_t*, const float*,
                                   uint16_t*);
g4_status launch_full_rows(g4_ctx*, const uint16_t*, const uint16_t*, const uint16_t*, const int32_t*, int, float*,
                           uint16_t*);
g4_status launch_embed(g4_ctx*, const uint16_t*, const int32_t*, uint16_t*);

// ------------------------------------------------------------------ weight set
enum LayerTensor {
  kInputNorm, kPostAttnNorm, kPreFfNorm, kPostFfNorm, kLayerScalar,
  kQW, kQS, kKW, kKS, kVW, kVS, kOW, kOS, kQNorm, kKNorm,
  kUpP, kUpS, kUpG, kGateP, kGateS, kGateG, kDownP, kDownS, kDownG,
  kLayerTensors
};

// Checkpoint names below "model.language_model.layers.<i>." (load.rs:240-339).
const char* const kLayerSuffix[kLayerTensors] = {
    "input_layernorm.weight", "post_attention_layernorm.weight", "pre_feedforward_layernorm.weight",
    "post_feedforward_layernorm.weight", "layer_scalar",
    "self_attn.q_proj.weight", "self_attn.q_proj.weight_scale", "self_attn.k_proj.weight",
    "self_attn.k_proj.weight_scale", "self_attn.v_proj.weight", "self_attn.v_proj.weight_scale",
    "self_attn.o_proj.weight", "self_attn.o_proj.weight_scale", "self_attn.q_norm.weight",
    "self_attn.k_norm.weight",
    "mlp.up_proj.weight_packed", "mlp.up_proj.weight_scale", "mlp.up_proj.weight_global_scale",
    "mlp.gate_proj.weight_packed", "mlp.gate_proj.weight_scale", "mlp.gate_proj.weight_global_scale",
    "mlp.down_proj.weight_packed", "mlp.down_proj.weight_scale", "mlp.down_proj.weight_global_scale"};

const char* const kLayerPrefix = "model.language_model.layers.";
const char* const kEmbedName = "model.language_model.embed_tokens.weight";
const char* const kFinalNormName = "model.language_model.norm.weight";

struct TensorRef {
  const void* ptr = nullptr;
  uint64_t bytes = 0;
};
struct LayerRefs {
  TensorRef t[kLayerTensors];
};

bool layer_is_full(int i) { return i % 6 == 5; }

// Device bytes of a layer tensor as the kernels take it on a rank of `world` (0: the
// tensor does not exist in this layer type).  Global scales are the reciprocal f32 the
// reference loader uploads (load.rs:171-191); the layer scalar is replicated to [8]
// (load.rs:99-111).
uint64_t layer_tensor_bytes(int kind, bool full, int world) {
  const uint64_t n = static_cast<uint64_t>(world);
  const uint64_t q = (full ? QF : QS) / n, d = full ? DF : DS;
  switch (kind) {
    case kInputNorm: case kPostAttnNorm: case kPreFfNorm: case kPostFfNorm: return H * 2ull;
    case kLayerScalar: return 16;
    case kQW: return q * H;
    case kQS: return q * 2;
    case kKW: return (full ? PF : PS / n) * static_cast<uint64_t>(H);
    case kKS: return (full ? PF : PS / n) * 2ull;
    case kVW: return full ? 0 : (PS / n) * static_cast<uint64_t>(H);
    case kVS: return full ? 0 : (PS / n) * 2ull;
    case kOW: return H * q;
    case kOS: return H * 2ull;
    case kQNorm: case kKNorm: return d * 2;
    case kUpP: case kGateP: return (L / n) * (H / 2ull);
    case kUpS: case kGateS: return (L / n) * (H / 16ull);
    case kDownP: return H * (L / n / 2);
    case kDownS: return H * (L / n / 16);
    case kUpG: case kGateG: case kDownG: return 4;
    default: return 0;
  }
}

// ------------------------------------------------------------------ step state
// Device-resident state of the decode loop.  The offsets are the reference's i32 BYTE
// offsets (runtime.rs:213-228; kv_off_f addresses the whole contiguous page array).
struct StepState {
  int32_t token;        // token embedded at this step
  int32_t pos;          // position of this step
  int32_t embed_off, kv_off_s, kv_off_f, rope_off_s, rope_off_f, n_rows_f;
  int32_t start_pos;    // prompt[k] is the token at position start_pos + k
  int32_t prompt_end;   // start_pos + prompt length
  int32_t n_generated;  // tokens appended to `generated` so far
  int32_t max_new;      // capacity of `generated`
  int32_t last_pred;    // greedy prediction of the last finished step
  int32_t status;       // bit 0: a step started at an invalid position or token
  int32_t pad[2];
};
static_assert(sizeof(StepState) == 64, "step state is one 64-byte block");

constexpr int kArgmaxCtas = 128;

__global__ void __launch_bounds__(1024) step_begin_kernel(StepState* st, float* mask_s, int max_pos, int nkv) {
  pdl_wait();  // the previous step's last kernel advanced the state
  const int pos = st->pos, tok = st->token;
  const bool ok = pos >= 0 && pos < max_pos && tok >= 0 && tok < W;
  const int row = min(pos, TS - 1);  // mask_s[min(pos, Ts-1)] (runtime.rs:155,357)
  for (int c = threadIdx.x; c < TS; c += blockDim.x) mask_s[c] = (ok && c <= row) ? 1.0f : 0.0f;
  if (threadIdx.x == 0) {
    if (ok) {
      st->embed_off = tok * H * 2;
      st->kv_off_s = (pos % TS) * nkv * DS * 2;
      st->kv_off_f = pos * DF * 2;
      st->rope_off_s = pos * DS * 2;
      st->rope_off_f = pos * DF * 2;
      st->n_rows_f = pos + 1;
    } else {
      // negative offsets: every kernel flags them and skips its reads and writes
      st->status |= 1;
      st->embed_off = st->kv_off_s = st->kv_off_f = st->rope_off_s = st->rope_off_f = -2;
      st->n_rows_f = 0;
    }
  }
}

// Monotone key of (bf16 value, index): larger value first, then lower index (torch.argmax).
__device__ __forceinline__ uint64_t argmax_key(uint32_t b, uint32_t idx) {
  const uint32_t ord = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return (static_cast<uint64_t>(ord) << 32) | (0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t x = __shfl_xor_sync(0xffffffffu, v, o);
    v = x > v ? x : v;
  }
  return v;
}

// The greedy token and the position advance (src/host/generate.rs:233-298 without the
// host round trip): inside the prompt the next input is the next prompt token, after it
// the prediction, which is also appended to `generated`.
__device__ void finish_step(StepState* st, uint64_t best, const int32_t* prompt, int32_t* generated,
                            int32_t* pred_log, int max_pos) {
  const int32_t pred = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
  const int p1 = st->pos + 1;
  const int k = st->pos - st->start_pos;
  if (k >= 0 && k < max_pos) pred_log[k] = pred;
  int next;
  if (p1 < st->prompt_end) {
    next = prompt[p1 - st->start_pos];
  } else {
    next = pred;
    if (st->n_generated < st->max_new) generated[st->n_generated] = pred;
    st->n_generated += 1;
  }
  st->last_pred = pred;
  st->token = next;
  st->pos = p1;
}

// Argmax of this rank's logits slice: kArgmaxCtas CTAs each reduce a slice, the last to
// finish reduces their candidates; on one GPU it finishes the step, under tensor
// parallelism it leaves the rank's candidate for the all-gather.
__global__ void __launch_bounds__(256) argmax_step_kernel(const uint16_t* logits, int n, uint32_t base,
                                                          uint64_t* cand, uint32_t* ticket, StepState* st,
                                                          const int32_t* prompt, int32_t* generated,
                                                          int32_t* pred_log, int max_pos, int world,
                                                          uint64_t* gather_in) {
  __shared__ uint64_t red[8];
  __shared__ int last;
  pdl_wait();
  const int per = ((n + gridDim.x - 1) / gridDim.x + 7) & ~7;
  const int b0 = blockIdx.x * per, b1 = min(n, b0 + per);
  uint64_t best = 0;
  for (int i = b0 + threadIdx.x * 8; i < b1; i += blockDim.x * 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(logits + i);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t k0 = argmax_key(ww[j] & 0xFFFFu, base + i + 2 * j);
      const uint64_t k1 = argmax_key(ww[j] >> 16, base + i + 2 * j + 1);
      best = k0 > best ? k0 : best;
      best = k1 > best ? k1 : best;
    }
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) best = red[w] > best ? red[w] : best;
    cand[blockIdx.x] = best;
    __threadfence();
    last = atom_add_acq_rel_gpu(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x >= 32) return;
  __threadfence();
  uint64_t b = 0;
  for (int c = threadIdx.x; c < static_cast<int>(gridDim.x); c += 32) {
    const uint64_t x = __ldcg(reinterpret_cast<const unsigned long long*>(cand) + c);
    b = x > b ? x : b;
  }
  b = warp_max_u64(b);
  if (threadIdx.x == 0) {
    if (world == 1)
      finish_step(st, b, prompt, generated, pred_log, max_pos);
    else
      gather_in[0] = b;
    *ticket = 0u;
  }
}

// Top-k / top-p mode: the sampled token (every rank drew the same) finishes the step.
__global__ void sample_finish_kernel(const int32_t* picked, StepState* st, const int32_t* prompt,
                                     int32_t* generated, int32_t* pred_log, int max_pos) {
  pdl_wait();
  if (threadIdx.x != 0) return;
  const uint64_t key = 0xFFFFFFFFu - static_cast<uint32_t>(*picked);  // finish_step's key of `picked`
  finish_step(st, key, prompt, generated, pred_log, max_pos);
}

__global__ void step_finish_kernel(const uint64_t* gathered, int world, StepState* st, const int32_t* prompt,
                                   int32_t* generated, int32_t* pred_log, int max_pos) {
  pdl_wait();
  if (threadIdx.x != 0) return;
  uint64_t b = 0;
  for (int r = 0; r < world; ++r) b = gathered[r] > b ? gathered[r] : b;
  finish_step(st, b, prompt, generated, pred_log, max_pos);
}

// RoPE tables exactly as rope_data (runtime.rs:271-299): f32 angle pos / theta^(2i/dim),
// cos and -sin (low half) / +sin (high half), identity beyond the rotated angles, bf16.
static uint16_t host_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return static_cast<uint16_t>((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}
static void rope_data(int dim, float theta, int rotated_dim, std::vector<uint16_t>& cos_t,
                      std::vector<uint16_t>& sin_t) {
  const int half = dim / 2, rhalf = rotated_dim / 2;
  cos_t.resize(static_cast<size_t>(E) * dim);
  sin_t.resize(static_cast<size_t>(E) * dim);
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = powf(theta, static_cast<float>(2 * i) / static_cast<float>(dim));
  for (int pos = 0; pos < E; ++pos) {
    uint16_t* c = cos_t.data() + static_cast<size_t>(pos) * dim;
    uint16_t* s = sin_t.data() + static_cast<size_t>(pos) * dim;
    for (int i = 0; i < half; ++i) {
      if (i < rhalf) {
        const float f = static_cast<float>(pos) / inv[i];
        const float cf = cosf(f), sf = sinf(f);
        c[i] = c[i + half] = host_bf16(cf);
        s[i] = host_bf16(-sf);
        s[i + half] = host_bf16(sf);
      } else {
        c[i] = c[i + half] = host_bf16(1.0f);
        s[i] = s[i + half] = host_bf16(0.0f);
      }
    }
  }
}

}  // namespace g4

using namespace g4;

struct g4_model {
  int n_layers = 0;
  std::vector<LayerRefs> layers;
  TensorRef embed, final_norm;
  std::vector<void*> owned;  // device buffers a loader allocated for this model
  int owned_device = -1;
  std::string last_error;
};

struct g4_workspace {
  int device = 0, n_layers = 0, max_pos = 0, cap_rows = 0, world = 1, rank = 0;
  uint16_t *cos_s = nullptr, *sin_s = nullptr, *cos_f = nullptr, *sin_f = nullptr;
  std::vector<uint16_t*> kc, vc;
  std::vector<uint64_t> cache_bytes;
  float* mask_s = nullptr;
  StepState* st = nullptr;
  int32_t *prompt = nullptr, *generated = nullptr;
  int32_t* pred_log = nullptr;  // greedy prediction of every step since the last begin
  uint16_t *x = nullptr, *q_s = nullptr, *q_f = nullptr, *attn_s = nullptr, *attn_f = nullptr;
  float *attn_max = nullptr, *attn_sum = nullptr;
  uint16_t* logits = nullptr;
  uint64_t* cand = nullptr;  // [kArgmaxCtas] candidates, then [kMaxTp] gather in/out
  uint32_t* ticket = nullptr;
  int32_t* picked = nullptr;  // the sampled token of the step (top-k / top-p mode)
  // sampling (g4_workspace_set_sampling): top_k == 0 is greedy
  int sample_k = 0;
  float sample_t = 1.0f, sample_p = 1.0f;
  std::vector<int32_t> sample_banned;
  uint64_t sample_seed = 0;
  std::vector<void*> allocs;
  cudaGraphExec_t exec = nullptr;
  const g4_model* graph_model = nullptr;
  cudaStream_t graph_stream = nullptr;
  int steps_planned = 0;
};

namespace g4 {
void model_adopt(g4_model* m, const std::vector<void*>& ptrs, int device) {
  m->owned.insert(m->owned.end(), ptrs.begin(), ptrs.end());
  m->owned_device = device;
}
}  // namespace g4

namespace {

g4_status model_fail(g4_model* m, g4_status code, const std::string& msg) {
  if (m) m->last_error = msg;
  return code;
}

// Checks that every tensor of every layer is set with the bytes a rank of `world` takes.
g4_status validate_model(g4_ctx* ctx, const g4_model* m, int world) {
  if (m->embed.ptr == nullptr || m->embed.bytes != static_cast<uint64_t>(W) * H * 2)
    return fail(ctx, G4_ERR_BAD_ARG, std::string(kEmbedName) + " missing or not [262144, 3840] bf16");
  if (m->final_norm.ptr == nullptr || m->final_norm.bytes != H * 2ull)
    return fail(ctx, G4_ERR_BAD_ARG, std::string(kFinalNormName) + " missing or not [3840] bf16");
  for (int i = 0; i < m->n_layers; ++i) {
    const bool full = layer_is_full(i);
    for (int k = 0; k < kLayerTensors; ++k) {
      const uint64_t want = layer_tensor_bytes(k, full, world);
      const TensorRef& t = m->layers[i].t[k];
      if (want == 0) continue;
      const std::string name = std::string(kLayerPrefix) + std::to_string(i) + "." + kLayerSuffix[k];
      if (t.ptr == nullptr) return fail(ctx, G4_ERR_BAD_ARG, name + " is not set");
      if (t.bytes != want)
        return fail(ctx, G4_ERR_BAD_ARG,
                    name + " has " + std::to_string(t.bytes) + " bytes, expected " + std::to_string(want) +
                        " for tensor-parallel world " + std::to_string(world));
    }
  }
  return G4_OK;
}

void free_workspace(g4_workspace* ws) {
  if (ws->exec) cudaGraphExecDestroy(ws->exec);
  for (void* p : ws->allocs) cudaFree(p);
  delete ws;
}

const void* P(const LayerRefs& l, int k) { return l.t[k].ptr; }
const uint8_t* P8(const LayerRefs& l, int k) { return static_cast<const uint8_t*>(l.t[k].ptr); }
const uint16_t* P16(const LayerRefs& l, int k) { return static_cast<const uint16_t*>(l.t[k].ptr); }
const float* PF32(const LayerRefs& l, int k) { return static_cast<const float*>(l.t[k].ptr); }

// One decode step (Decode::run, runtime.rs:312-347) issued on the context's stream.
g4_status issue_step(g4_ctx* ctx, g4_workspace* ws, const g4_model* m) {
  StepState* st = ws->st;
  g4_status s;
  {
    int maxp = ws->max_pos, nkv = NS / ws->world;
    void* a[] = {(void*)&st, (void*)&ws->mask_s, (void*)&maxp, (void*)&nkv};
    s = launch_kernel(ctx, (const void*)step_begin_kernel, dim3(1), dim3(1024), 0, a, false, "step begin");
    if (s != G4_OK) return s;
  }
  const uint16_t* embed = static_cast<const uint16_t*>(m->embed.ptr);
  if ((s = launch_embed(ctx, embed, &st->embed_off, ws->x)) != G4_OK) return s;
  for (int i = 0; i < m->n_layers; ++i) {
    const LayerRefs& l = m->layers[i];
    const uint8_t* bs[3] = {nullptr, nullptr, nullptr};
    const float* gs[3] = {nullptr, nullptr, nullptr};
    if (!layer_is_full(i)) {  // runtime.rs:349-408
      const uint8_t* w[3] = {P8(l, kQW), P8(l, kKW), P8(l, kVW)};
      const uint16_t* rs[3] = {P16(l, kQS), P16(l, kKS), P16(l, kVS)};
      s = launch_qkv(ctx, false, false, ws->x, w, bs, rs, gs, P16(l, kInputNorm), P16(l, kQNorm), P16(l, kKNorm),
                     &st->kv_off_s, &st->rope_off_s, ws->cos_s, ws->sin_s, ws->kc[i], ws->vc[i], ws->q_s, 0);
      if (s == G4_OK) s = launch_sliding_attention(ctx, ws->q_s, ws->kc[i], ws->vc[i], ws->mask_s, ws->attn_s);
      if (s == G4_OK)
        s = launch_oproj(ctx, false, false, ws->attn_s, nullptr, P16(l, kPostAttnNorm), P8(l, kOW), nullptr,
                         P16(l, kOS), nullptr, ws->x);
    } else {  // runtime.rs:410-482, every page in one launch
      const uint8_t* w[3] = {P8(l, kQW), P8(l, kKW), nullptr};
      const uint16_t* rs[3] = {P16(l, kQS), P16(l, kKS), nullptr};
      s = launch_qkv(ctx, true, false, ws->x, w, bs, rs, gs, P16(l, kInputNorm), P16(l, kQNorm), P16(l, kKNorm),
                     &st->kv_off_f, &st->rope_off_f, ws->cos_f, ws->sin_f, ws->kc[i], ws->vc[i], ws->q_f,
                     static_cast<long long>(ws->cap_rows) * DF);
      if (s == G4_OK)
        s = launch_full_rows(ctx, ws->q_f, ws->kc[i], ws->vc[i], &st->n_rows_f, ws->cap_rows, ws->attn_sum,
                             ws->attn_f);
      if (s == G4_OK)
        s = launch_oproj(ctx, true, false, ws->attn_f, ws->attn_sum, P16(l, kPostAttnNorm), P8(l, kOW), nullptr,
                         P16(l, kOS), nullptr, ws->x);
    }
    if (s == G4_OK)  // runtime.rs:484-512
      s = launch_decoder_feedforward(ctx, ws->x, P16(l, kPreFfNorm), P8(l, kUpP), P8(l, kGateP), P8(l, kDownP),
                                     P8(l, kUpS), P8(l, kGateS), P8(l, kDownS), PF32(l, kUpG), PF32(l, kGateG),
                                     PF32(l, kDownG), P16(l, kPostFfNorm), P16(l, kLayerScalar));
    if (s != G4_OK) return s;
  }
  // final_norm_and_logits on this rank's vocab slice of the tied table (runtime.rs:342-346)
  const int vrows = W / ws->world;
  s = launch_lm_head(ctx, ws->x, static_cast<const uint16_t*>(m->final_norm.ptr),
                     embed + static_cast<size_t>(ws->rank) * vrows * H, ws->logits);
  if (s != G4_OK) return s;
  if (ws->sample_k > 0) {
    // top-k / top-p with the step's own draw (seed, position), then the step advance
    s = launch_sample(ctx, ws->logits, vrows, ws->sample_t, ws->sample_k, ws->sample_p, ws->sample_banned.data(),
                      static_cast<int>(ws->sample_banned.size()), nullptr, ws->picked, &st->pos, ws->sample_seed);
    if (s != G4_OK) return s;
    int maxp = ws->max_pos;
    void* b[] = {(void*)&ws->picked, (void*)&st, (void*)&ws->prompt, (void*)&ws->generated, (void*)&ws->pred_log,
                 (void*)&maxp};
    return launch_kernel(ctx, (const void*)sample_finish_kernel, dim3(1), dim3(32), 0, b, false, "sample finish");
  }
  {
    const uint16_t* lg = ws->logits;
    int n = vrows, world = ws->world, maxp = ws->max_pos;
    uint32_t base = static_cast<uint32_t>(ws->rank) * vrows;
    uint64_t* cand = ws->cand;
    uint64_t* gin = ws->cand + kArgmaxCtas;
    void* a[] = {(void*)&lg, (void*)&n, (void*)&base, (void*)&cand, (void*)&ws->ticket, (void*)&st,
                 (void*)&ws->prompt, (void*)&ws->generated, (void*)&ws->pred_log, (void*)&maxp, (void*)&world,
                 (void*)&gin};
    s = launch_kernel(ctx, (const void*)argmax_step_kernel, dim3(kArgmaxCtas), dim3(256), 0, a, false, "argmax");
    if (s != G4_OK || world == 1) return s;
    uint64_t* gout = gin + 1;
    if ((s = allgather_u64(ctx, gin, gout)) != G4_OK) return s;
    void* b[] = {(void*)&gout, (void*)&world, (void*)&st, (void*)&ws->prompt, (void*)&ws->generated,
                 (void*)&ws->pred_log, (void*)&maxp};
    return launch_kernel(ctx, (const void*)step_finish_kernel, dim3(1), dim3(32), 0, b, false, "step finish");
  }
}

// The whole step as one CUDA graph, captured on first use (and again when the model or
// the stream changes).  Capture needs a stream other than the legacy default stream.
g4_status ensure_graph(g4_ctx* ctx, g4_workspace* ws, const g4_model* m) {
  if (ws->exec != nullptr && ws->graph_model == m && ws->graph_stream == ctx->stream) return G4_OK;
  if (ws->exec != nullptr) {
    cudaGraphExecDestroy(ws->exec);
    ws->exec = nullptr;
  }
  if (ctx->stream == nullptr)
    return fail(ctx, G4_ERR_UNSUPPORTED, "graph replay needs a non-default stream (g4_ctx_set_stream)");
  g4_status s = check_cuda(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeRelaxed), "begin capture");
  if (s != G4_OK) return s;
  const g4_status si = issue_step(ctx, ws, m);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
  if (si != G4_OK) {
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();
    return si;
  }
  if ((s = check_cuda(ctx, e, "end capture")) != G4_OK) return s;
  s = check_cuda(ctx, cudaGraphInstantiate(&ws->exec, g, 0), "instantiate step graph");
  cudaGraphDestroy(g);
  if (s != G4_OK) return s;
  ws->graph_model = m;
  ws->graph_stream = ctx->stream;
  return G4_OK;
}

g4_status set_state(g4_ctx* ctx, g4_workspace* ws, int token, int pos, int start_pos, int prompt_end, int max_new) {
  StepState h = {};
  h.token = token;
  h.pos = pos;
  h.start_pos = start_pos;
  h.prompt_end = prompt_end;
  h.max_new = max_new;
  h.last_pred = -1;
  // pageable source: the copy is staged before the call returns
  return check_cuda(ctx, cudaMemcpyAsync(ws->st, &h, sizeof(h), cudaMemcpyHostToDevice, ctx->stream), "set state");
}

}  // namespace

extern "C" {

g4_status g4_model_create(int n_layers, g4_model** out) {
  if (out == nullptr) return G4_ERR_BAD_ARG;
  *out = nullptr;
  if (n_layers < 1 || n_layers > G4_LAYERS) return G4_ERR_BAD_ARG;
  g4_model* m = new g4_model();
  m->n_layers = n_layers;
  m->layers.resize(n_layers);
  *out = m;
  return G4_OK;
}

g4_status g4_model_destroy(g4_model* m) {
  if (m == nullptr) return G4_ERR_BAD_ARG;
  if (!m->owned.empty()) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->owned_device);
    for (void* p : m->owned) cudaFree(p);
    cudaSetDevice(prev);
  }
  delete m;
  return G4_OK;
}

const char* g4_model_last_error(const g4_model* m) { return m ? m->last_error.c_str() : "null model"; }

int g4_model_layer_is_full(int layer) { return layer_is_full(layer) ? 1 : 0; }

g4_status g4_model_set_tensor(g4_model* m, const char* name, const void* device_ptr, uint64_t bytes) {
  if (m == nullptr || name == nullptr) return G4_ERR_BAD_ARG;
  if (device_ptr == nullptr || (reinterpret_cast<uintptr_t>(device_ptr) & 15u) != 0)
    return model_fail(m, G4_ERR_BAD_ARG, std::string(name) + ": pointer is null or not 16-byte aligned");
  const std::string n(name);
  if (n == kEmbedName) {
    m->embed = {device_ptr, bytes};
    return G4_OK;
  }
  if (n == kFinalNormName) {
    m->final_norm = {device_ptr, bytes};
    return G4_OK;
  }
  const size_t pl = std::strlen(kLayerPrefix);
  if (n.compare(0, pl, kLayerPrefix) == 0) {
    size_t i = pl;
    int layer = 0;
    bool digits = false;
    while (i < n.size() && n[i] >= '0' && n[i] <= '9' && layer < 1000) {
      layer = layer * 10 + (n[i] - '0');
      ++i;
      digits = true;
    }
    if (digits && i < n.size() && n[i] == '.') {
      const std::string suffix = n.substr(i + 1);
      if (layer >= m->n_layers)
        return model_fail(m, G4_ERR_BAD_ARG, n + ": layer index beyond the model's " + std::to_string(m->n_layers));
      for (int k = 0; k < kLayerTensors; ++k) {
        if (suffix == kLayerSuffix[k]) {
          if (layer_tensor_bytes(k, layer_is_full(layer), 1) == 0)
            return model_fail(m, G4_ERR_BAD_ARG, n + ": full-attention layers have no such tensor");
          m->layers[layer].t[k] = {device_ptr, bytes};
          return G4_OK;
        }
      }
    }
  }
  return model_fail(m, G4_ERR_BAD_ARG, n + ": not a tensor of the text decoder");
}

g4_status g4_workspace_create(g4_ctx* ctx, const g4_model* m, int max_positions, g4_workspace** out) {
  if (ctx == nullptr || m == nullptr || out == nullptr) return G4_ERR_BAD_ARG;
  *out = nullptr;
  if (max_positions < 1 || max_positions > G4_E)
    return fail(ctx, G4_ERR_BAD_ARG, "max_positions must be in [1, 32768]");
  g4_status s = validate_model(ctx, m, ctx->tp_world);
  if (s != G4_OK) return s;
  if ((s = check_cuda(ctx, cudaSetDevice(ctx->device), "cudaSetDevice")) != G4_OK) return s;
  g4_workspace* ws = new g4_workspace();
  ws->device = ctx->device;
  ws->n_layers = m->n_layers;
  ws->max_pos = max_positions;
  ws->cap_rows = (max_positions + TF - 1) / TF * TF;  // whole pages
  ws->world = ctx->tp_world;
  ws->rank = ctx->tp_rank;
  auto alloc = [&](void** p, size_t bytes, const char* what) -> bool {
    if (s != G4_OK) return false;
    s = check_cuda(ctx, cudaMalloc(p, bytes), what);
    if (s == G4_OK) {
      ws->allocs.push_back(*p);
      s = check_cuda(ctx, cudaMemset(*p, 0, bytes), what);
    }
    return s == G4_OK;
  };
  alloc((void**)&ws->cos_s, static_cast<size_t>(E) * DS * 2, "rope cos_s");
  alloc((void**)&ws->sin_s, static_cast<size_t>(E) * DS * 2, "rope sin_s");
  alloc((void**)&ws->cos_f, static_cast<size_t>(E) * DF * 2, "rope cos_f");
  alloc((void**)&ws->sin_f, static_cast<size_t>(E) * DF * 2, "rope sin_f");
  ws->kc.assign(m->n_layers, nullptr);
  ws->vc.assign(m->n_layers, nullptr);
  ws->cache_bytes.assign(m->n_layers, 0);
  for (int i = 0; i < m->n_layers && s == G4_OK; ++i) {
    const size_t bytes = layer_is_full(i) ? static_cast<size_t>(ws->cap_rows) * DF * 2
                                          : static_cast<size_t>(TS) * (NS / ws->world) * DS * 2;
    ws->cache_bytes[i] = bytes;
    alloc((void**)&ws->kc[i], bytes, "k cache");
    alloc((void**)&ws->vc[i], bytes, "v cache");
  }
  alloc((void**)&ws->mask_s, TS * 4, "mask row");
  alloc((void**)&ws->st, sizeof(StepState), "step state");
  alloc((void**)&ws->prompt, static_cast<size_t>(max_positions) * 4, "prompt");
  alloc((void**)&ws->generated, static_cast<size_t>(max_positions) * 4, "generated");
  alloc((void**)&ws->pred_log, static_cast<size_t>(max_positions) * 4, "prediction log");
  alloc((void**)&ws->x, H * 2, "x");
  alloc((void**)&ws->q_s, NS * GS * DS * 2, "q_s");
  alloc((void**)&ws->q_f, GF * DF * 2, "q_f");
  alloc((void**)&ws->attn_s, NS * GS * DS * 2, "attn_s");
  alloc((void**)&ws->attn_f, GF * DF * 2, "attn_f");
  alloc((void**)&ws->attn_max, GF * 4, "attn_max");
  alloc((void**)&ws->attn_sum, GF * 4, "attn_sum");
  alloc((void**)&ws->logits, static_cast<size_t>(W / ws->world) * 2, "logits");
  alloc((void**)&ws->cand, (kArgmaxCtas + 2 * kMaxTp) * 8, "argmax candidates");
  alloc((void**)&ws->ticket, 4, "argmax ticket");
  alloc((void**)&ws->picked, 4, "sampled token");
  if (s == G4_OK) {
    std::vector<uint16_t> c, sn;
    rope_data(DS, 10000.0f, DS, c, sn);  // runtime.rs:153
    s = check_cuda(ctx, cudaMemcpy(ws->cos_s, c.data(), c.size() * 2, cudaMemcpyHostToDevice), "rope upload");
    if (s == G4_OK)
      s = check_cuda(ctx, cudaMemcpy(ws->sin_s, sn.data(), sn.size() * 2, cudaMemcpyHostToDevice), "rope upload");
    rope_data(DF, 1000000.0f, 128, c, sn);  // runtime.rs:154: first 128 of 512 dims rotated
    if (s == G4_OK)
      s = check_cuda(ctx, cudaMemcpy(ws->cos_f, c.data(), c.size() * 2, cudaMemcpyHostToDevice), "rope upload");
    if (s == G4_OK)
      s = check_cuda(ctx, cudaMemcpy(ws->sin_f, sn.data(), sn.size() * 2, cudaMemcpyHostToDevice), "rope upload");
  }
  if (s == G4_OK) s = check_cuda(ctx, cudaDeviceSynchronize(), "workspace init");
  if (s != G4_OK) {
    free_workspace(ws);
    return s;
  }
  *out = ws;
  return G4_OK;
}

g4_status g4_workspace_set_sampling(g4_workspace* ws, float temperature, int top_k, float top_p,
                                    const int32_t* banned, int n_banned, uint64_t seed) {
  if (ws == nullptr) return G4_ERR_BAD_ARG;
  if (top_k < 0 || n_banned < 0 || top_k + n_banned > 128 || (n_banned > 0 && banned == nullptr)) return G4_ERR_BAD_ARG;
  if (top_k > 0 && (!(top_p > 0.f) || !(top_p <= 1.f) || !(temperature >= 0.f) || !std::isfinite(temperature)))
    return G4_ERR_BAD_ARG;
  ws->sample_k = top_k;
  ws->sample_t = temperature;
  ws->sample_p = top_p;
  ws->sample_banned.assign(banned, banned + n_banned);
  ws->sample_seed = seed;
  if (ws->exec != nullptr) {  // the step graph changes: capture it again on next use
    cudaSetDevice(ws->device);
    cudaGraphExecDestroy(ws->exec);
    ws->exec = nullptr;
  }
  return G4_OK;
}

g4_status g4_workspace_destroy(g4_workspace* ws) {
  if (ws == nullptr) return G4_ERR_BAD_ARG;
  cudaSetDevice(ws->device);
  free_workspace(ws);
  return G4_OK;
}

g4_status g4_workspace_kv_cache(g4_workspace* ws, int layer, g4_bf16** k, g4_bf16** v, uint64_t* bytes) {
  if (ws == nullptr || layer < 0 || layer >= ws->n_layers || k == nullptr || v == nullptr || bytes == nullptr)
    return G4_ERR_BAD_ARG;
  *k = ws->kc[layer];
  *v = ws->vc[layer];
  *bytes = ws->cache_bytes[layer];
  return G4_OK;
}

g4_status g4_workspace_logits(g4_workspace* ws, const g4_bf16** logits, int* count) {
  if (ws == nullptr || logits == nullptr || count == nullptr) return G4_ERR_BAD_ARG;
  *logits = ws->logits;
  *count = W / ws->world;
  return G4_OK;
}

g4_status g4_workspace_hidden(g4_workspace* ws, const g4_bf16** x) {
  if (ws == nullptr || x == nullptr) return G4_ERR_BAD_ARG;
  *x = ws->x;
  return G4_OK;
}

g4_status g4_decode_run(g4_ctx* ctx, g4_workspace* ws, const g4_model* m, int32_t token, int32_t pos) {
  if (ctx == nullptr || ws == nullptr || m == nullptr || m->n_layers != ws->n_layers) return G4_ERR_BAD_ARG;
  if (pos < 0 || pos >= ws->max_pos || token < 0 || token >= G4_W)
    return fail(ctx, G4_ERR_BAD_ARG, "token or position out of range");
  g4_status s = set_state(ctx, ws, token, pos, pos, pos + 1, 0);
  return s != G4_OK ? s : issue_step(ctx, ws, m);
}

g4_status g4_decode_begin(g4_ctx* ctx, g4_workspace* ws, const int32_t* prompt, int prompt_len, int start_pos,
                          int max_new) {
  if (ctx == nullptr || ws == nullptr || prompt == nullptr) return G4_ERR_BAD_ARG;
  if (prompt_len < 1 || start_pos < 0 || max_new < 0 ||
      static_cast<long long>(start_pos) + prompt_len + max_new - 1 > ws->max_pos)
    return fail(ctx, G4_ERR_BAD_ARG, "prompt, start position and new tokens must fit the workspace's positions");
  for (int i = 0; i < prompt_len; ++i)
    if (prompt[i] < 0 || prompt[i] >= G4_W) return fail(ctx, G4_ERR_BAD_ARG, "prompt token out of range");
  g4_status s = check_cuda(ctx, cudaMemcpyAsync(ws->prompt, prompt, static_cast<size_t>(prompt_len) * 4,
                                                cudaMemcpyHostToDevice, ctx->stream),
                           "prompt upload");
  if (s == G4_OK) s = set_state(ctx, ws, prompt[0], start_pos, start_pos, start_pos + prompt_len, max_new);
  ws->steps_planned = prompt_len + max_new - 1;
  return s;
}

g4_status g4_decode_steps(g4_ctx* ctx, g4_workspace* ws, const g4_model* m, int n_steps, int use_graph) {
  if (ctx == nullptr || ws == nullptr || m == nullptr || n_steps < 0 || m->n_layers != ws->n_layers)
    return G4_ERR_BAD_ARG;
  if (use_graph) {
    g4_status s = ensure_graph(ctx, ws, m);
    if (s != G4_OK) return s;
    for (int i = 0; i < n_steps; ++i)
      if ((s = check_cuda(ctx, cudaGraphLaunch(ws->exec, ctx->stream), "step graph launch")) != G4_OK) return s;
    return G4_OK;
  }
  for (int i = 0; i < n_steps; ++i) {
    const g4_status s = issue_step(ctx, ws, m);
    if (s != G4_OK) return s;
  }
  return G4_OK;
}

g4_status g4_decode_tokens(g4_ctx* ctx, g4_workspace* ws, int32_t* out, int max_out, int* n_out) {
  if (ctx == nullptr || ws == nullptr || n_out == nullptr || (max_out > 0 && out == nullptr)) return G4_ERR_BAD_ARG;
  StepState h = {};
  g4_status s = check_cuda(ctx, cudaMemcpyAsync(&h, ws->st, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream), "state");
  if (s == G4_OK) s = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "decode sync");
  if (s != G4_OK) return s;
  const int n = h.n_generated < h.max_new ? h.n_generated : h.max_new;
  const int k = n < max_out ? n : max_out;
  if (k > 0 && (s = check_cuda(ctx, cudaMemcpy(out, ws->generated, static_cast<size_t>(k) * 4, cudaMemcpyDeviceToHost),
                               "tokens")) != G4_OK)
    return s;
  *n_out = k;
  if (h.status != 0) return fail(ctx, G4_ERR_BAD_ARG, "a step ran at a position or token out of range");
  uint32_t bits = 0;
  return g4_ctx_poll_device_status(ctx, &bits);
}

g4_status g4_decode_predictions(g4_ctx* ctx, g4_workspace* ws, int32_t* out, int max_out, int* n_out) {
  if (ctx == nullptr || ws == nullptr || n_out == nullptr || (max_out > 0 && out == nullptr)) return G4_ERR_BAD_ARG;
  StepState h = {};
  g4_status s = check_cuda(ctx, cudaMemcpyAsync(&h, ws->st, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream), "state");
  if (s == G4_OK) s = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "decode sync");
  if (s != G4_OK) return s;
  int n = h.pos - h.start_pos;
  n = n < 0 ? 0 : (n > ws->max_pos ? ws->max_pos : n);
  const int k = n < max_out ? n : max_out;
  if (k > 0 && (s = check_cuda(ctx, cudaMemcpy(out, ws->pred_log, static_cast<size_t>(k) * 4, cudaMemcpyDeviceToHost),
                               "predictions")) != G4_OK)
    return s;
  *n_out = k;
  return G4_OK;
}

g4_status g4_decode_last_prediction(g4_ctx* ctx, g4_workspace* ws, int32_t* token, int32_t* next_pos) {
  if (ctx == nullptr || ws == nullptr || token == nullptr || next_pos == nullptr) return G4_ERR_BAD_ARG;
  StepState h = {};
  g4_status s = check_cuda(ctx, cudaMemcpyAsync(&h, ws->st, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream), "state");
  if (s == G4_OK) s = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "decode sync");
  if (s != G4_OK) return s;
  *token = h.last_pred;
  *next_pos = h.pos;
  return G4_OK;
}

g4_status g4_generate_greedy(g4_ctx* ctx, g4_workspace* ws, const g4_model* m, const int32_t* prompt, int prompt_len,
                             int start_pos, int max_new, int use_graph, int32_t* out_tokens) {
  g4_status s = g4_decode_begin(ctx, ws, prompt, prompt_len, start_pos, max_new);
  if (s == G4_OK) s = g4_decode_steps(ctx, ws, m, prompt_len + max_new - 1, use_graph);
  int n = 0;
  if (s == G4_OK) s = g4_decode_tokens(ctx, ws, out_tokens, max_new, &n);
  if (s == G4_OK && n != max_new) return fail(ctx, G4_ERR_CUDA, "decode produced fewer tokens than asked");
  return s;
}

}  // extern "C"
