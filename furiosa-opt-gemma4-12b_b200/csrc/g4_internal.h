// Host-side context and device scratch layout shared by the g4b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "g4.h"

struct ncclComm;

namespace g4 {

// Device scratch owned by a context.  Counters are zero at creation and every kernel
// that uses one returns it to zero before it exits, so launches (and CUDA-graph
// replays) need no host-side reset.
struct Scratch {
  uint32_t status;            // DEV_ERR_* bits raised by kernels (sticky until polled)
  uint32_t mlp_sync;          // MLP: CTAs that finished the gate/up phase
  uint32_t mlp_done;          // MLP: CTAs that finished the down phase
  uint32_t mlp_amax;          // MLP: bits of max |h| over the intermediate vector
  uint32_t proj_done;         // o-proj: CTAs done
  uint32_t lm_done;           // (reserved)
  uint32_t xch_epoch;         // TP: launches that used the peer exchange (same on every rank)
  uint32_t tc_epoch;          // tensor-core MLP: launches finished (tags the values CTAs exchange)
  uint32_t head_count[64];    // qkv: completed items per head group
  uint32_t attn_count[64];    // split-KV attention: completed chunks per kv head
  uint32_t attn_done;         // paged attention: CTAs done
  uint32_t pad1[31];
};

constexpr size_t kPartFloats = 16 * 3840 * 2;     // row-parallel partial sums
constexpr size_t kHeadFloats = 8192 + 512 + 8192; // raw projection rows (qkv)
constexpr size_t kHFloats = 15360;                // MLP intermediate (bf16 stored)
constexpr size_t kAttnFloats = 512 * (2 * 16 + 16 * 512) + 4096;  // 512 chunks of 16 heads
constexpr size_t kTcTiles = 15360 / 64 + 3840 / 128;              // gate/up tiles + down tiles
constexpr size_t kTcSegFloats = 3840;                             // the down projection's H sums
constexpr size_t kTcPartWords = kTcTiles * 8 * 128;                // tagged segment partials (both phases)
constexpr size_t kCandWords = 16384 + 128 + 8 * 128;              // sampling: candidates, a rank's share, gathered

// Tensor-parallel one-shot all-reduce over peer memory.  Each rank owns one exchange
// buffer of 64-bit words, word[2][kMaxTp][3840]: two halves used by alternate launches,
// one [3840] slot per source rank.  A word carries one f32 value (low half) and the
// number of the launch that sent it (high half), so a reader knows a value has arrived
// without any fence or separate flag.
constexpr int kMaxTp = 8;
constexpr size_t kXchWords = 2 * static_cast<size_t>(kMaxTp) * 3840;
constexpr size_t kXchBytes = kXchWords * 8;

// This rank's view of every rank's exchange buffer (its own included); world <= 1 means
// the peer exchange is not in use.
struct PeerXch {
  uint64_t* buf[kMaxTp];
  int rank;
  int world;
};

struct DeviceBuffers {
  Scratch* scratch = nullptr;
  float* part = nullptr;     // [kPartFloats]
  float* rows = nullptr;     // [kHeadFloats]
  uint16_t* hbuf = nullptr;  // [kHFloats] bf16
  float* ybuf = nullptr;     // [3840] f32 (TP all-reduce buffer)
  float* attn = nullptr;     // [kAttnFloats] split-KV partials
  uint64_t* xch = nullptr;   // [kXchWords] TP peer exchange (this rank's, IPC-exported)
  float* tc_seg = nullptr;   // [kTcSegFloats] tensor-core MLP: the down projection's 3840 sums
  // Tensor-core MLP values exchanged between CTAs, each word tagged with the launch that
  // wrote it (zero at creation): segment partials {f32, tag} and h {bf16, tag}.
  uint64_t* tc_ptag = nullptr;  // [kTcPartWords]
  uint32_t* tc_htag = nullptr;  // [kHFloats]
  uint64_t* cand = nullptr;     // [kCandWords] sampling candidates (g4_sample.cu)
};

// Batched prefill feed-forward scratch, grown to the largest token count seen and kept
// until the context is destroyed: NVFP4 activations (codes then block scales), h in bf16,
// the down projection's output, and the per-token 1/g of both quantised activations.
struct PrefillBuffers {
  int cap = 0;
  uint8_t* xq = nullptr;     // [cap][H/2] codes, then [cap][H/16] scales
  uint16_t* h = nullptr;     // [cap][lrows] (lrows: this rank's intermediate rows)
  uint8_t* hq = nullptr;     // [cap][lrows/2] codes, then [cap][ld] scales (ld: lrows/16 rounded up to 16)
  float* y = nullptr;        // [cap][H] the down projection's f32 sums
  float* ginv = nullptr;     // [2][cap]
  uint8_t* down_sf = nullptr;  // [H][ld] the down weights' scales re-laid out (when their rows
                               // are not a multiple of 16 bytes: 8-way tensor parallel)
};

}  // namespace g4

struct g4_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  int tp_rank = 0;
  int tp_world = 1;
  ncclComm* comm = nullptr;
  uint64_t wait_budget_ns = 2000000000ull;  // 2 s
  g4::DeviceBuffers buf;
  std::string last_error;
  bool coop_ok = true;
  bool pdl_ok = true;  // programmatic dependent launch accepted by the runtime
  bool cluster_ok = true;  // thread-block cluster launches accepted
  // The K cache and device offset of the last attention projection launched on this
  // context: sliding attention over that cache re-reads the row it wrote after waiting
  // for its predecessor (the other rows it copies before).
  const uint16_t* qkv_kc = nullptr;
  const int32_t* qkv_kv_off = nullptr;
  int mlp_kernel = 0;  // G4_MLP_AUTO / G4_MLP_STREAM / G4_MLP_TENSOR
  g4::PeerXch peers = {};  // TP exchange buffers mapped from every rank (world 0: NCCL path)
  g4::PrefillBuffers prefill;
  int prefill_pieces = 2;  // NVFP4 pieces per prefill activation (1..3)
};

namespace g4 {

g4_status fail(g4_ctx* ctx, g4_status code, const std::string& msg);
g4_status check_cuda(g4_ctx* ctx, cudaError_t err, const char* what);
bool aligned16(const void* p);

// Launchers implemented in the kernel translation units.
g4_status launch_decoder_feedforward(g4_ctx* ctx, uint16_t* residual, const uint16_t* pre_w,
                                     const uint8_t* up_p, const uint8_t* gate_p, const uint8_t* down_p,
                                     const uint8_t* up_s, const uint8_t* gate_s, const uint8_t* down_s,
                                     const float* up_gs, const float* gate_gs, const float* down_gs,
                                     const uint16_t* post_w, const uint16_t* layer_scalar);
g4_status allreduce_f32(g4_ctx* ctx, float* buf, size_t count);
// Hands device buffers a loader allocated for `model` to it: freed by g4_model_destroy.
void model_adopt(g4_model* model, const std::vector<void*>& ptrs, int device);
// Every rank's one 64-bit word into out[world] (NCCL all-gather on the context's stream).
g4_status allgather_u64(g4_ctx* ctx, const uint64_t* in, uint64_t* out);
// Every rank's `count` 64-bit words into out[world][count].
g4_status allgather_u64n(g4_ctx* ctx, const uint64_t* in, uint64_t* out, int count);
// Top-k / top-p sampling of this rank's logits[n] (g4_sample.cu).
// draw_pos non-null: the draw is derived on the device from (seed, *draw_pos) instead of
// read from `uniform` (the decode runtime's per-position draw).
g4_status launch_sample(g4_ctx* ctx, const uint16_t* logits, int n, float temperature, int top_k, float top_p,
                        const int32_t* banned, int n_banned, const float* uniform, int32_t* out_index,
                        const int32_t* draw_pos = nullptr, uint64_t seed = 0);
bool mlp_tc_enabled(const g4_ctx* ctx);
g4_status launch_decoder_feedforward_tc(g4_ctx* ctx, uint16_t* residual, const uint16_t* pre_w,
                                        const uint8_t* up_p, const uint8_t* gate_p, const uint8_t* down_p,
                                        const uint8_t* up_s, const uint8_t* gate_s, const uint8_t* down_s,
                                        const float* up_gs, const float* gate_gs, const float* down_gs,
                                        const uint16_t* post_w, const uint16_t* layer_scalar);
// n tokens' MLP block at once on the tensor cores (g4_prefill.cu).
g4_status launch_prefill_feedforward(g4_ctx* ctx, int n, uint16_t* residual, const uint16_t* pre_w,
                                     const uint8_t* up_p, const uint8_t* gate_p, const uint8_t* down_p,
                                     const uint8_t* up_s, const uint8_t* gate_s, const uint8_t* down_s,
                                     const float* up_gs, const float* gate_gs, const float* down_gs,
                                     const uint16_t* post_w, const uint16_t* layer_scalar);

// Raises `fn`'s dynamic shared-memory limit to the device's opt-in maximum, once per
// (kernel, device): every launch, whatever its layout (`need` bytes, checked), then fits,
// and no context can lower the limit under another.
g4_status allow_max_dynamic_smem(g4_ctx* ctx, const void* fn, size_t need, const char* what);

// Launches `fn` on the context's stream, optionally cooperative.  The launch allows
// programmatic dependent launch: the kernel may start while the previous kernel on the
// stream finishes, so it must execute griddepcontrol.wait before touching anything that
// kernel wrote (weights, never written by these kernels, may be read before).  If the
// runtime rejects that attribute once, the context launches without it from then on.
// cluster_x > 1 launches clusters of that many CTAs along x.
g4_status launch_kernel(g4_ctx* ctx, const void* fn, dim3 grid, dim3 block, size_t smem, void** args,
                        bool cooperative, const char* what, unsigned cluster_x = 0);

}  // namespace g4
