/*
 * g4.h - C ABI of the B200 (sm_100a) Gemma-4-12B text-decoder hot path.
 *
 * Each `g4_<op>` entry point is the drop-in for the `#[device]` function of the same
 * name in the reference crate's `src/ops.rs`.  The reference launches those as
 * `launch(ops::<op>, (ctx, &a, &mut b, ...)).await` (src/host/runtime.rs:316-511); here
 * the same call is `g4_<op>(ctx, a, b, ...)` with:
 *   - the SAME argument order as the ops.rs signature (the `ctx` first, then tensors);
 *   - device pointers in the reference's dtypes and row-major layouts (shapes below,
 *     named by the reference's axes, src/axes.rs: H=3840 L=15360 W=262144 Ns=8 Gs=2
 *     Ds=256 Qs=4096 Ps=2048 Ts=1024 Gf=16 Df=512 Qf=8192 Pf=512 Tf=512 E=32768);
 *   - `&mut` tensors written in place exactly where the reference writes them;
 *   - offsets kept as device-resident int32 BYTE offsets (src/host/runtime.rs:213-228),
 *     so a whole decode step can be captured in a CUDA graph and replayed;
 *   - work issued asynchronously on the context's stream (g4_ctx_set_stream), in stream
 *     order, like the reference's awaited launches;
 *   - a g4_status return instead of the reference's panics.
 *
 * Storage formats (identical to the reference checkpoint, src/host/load.rs:10-191):
 *   bf16   : uint16 bit patterns.
 *   f8e4m3 : one byte per element (OCP E4M3FN).
 *   f4e2m1 : NVFP4 codes packed two per byte, LOW nibble = even element
 *            (scripts/fixture_prng.py:153-168), a [N, K] matrix stored as [N, K/2] bytes.
 *   NVFP4 block scale : one f8e4m3 per 16 consecutive K elements, [N, K/16].
 *   NVFP4 global scale: one f32, already the RECIPROCAL of the checkpoint value
 *            (src/host/load.rs:171-191), multiplied into the projection result.
 *
 * Threading: one g4_ctx per host thread, like the reference's non-Send
 * `Context::acquire()` guard (src/api/worker.rs:73-99).  Pointers must be 16-byte
 * aligned (cudaMalloc gives 256).  Shapes are the reference's fixed axes unless an
 * entry point says otherwise; under tensor parallelism (g4_ctx_init_tp) the weight
 * arguments are this rank's shard, as documented per entry point.
 *
 * Overlap between consecutive calls: kernels are launched with programmatic dependent
 * launch, and before waiting for the previous kernel on the stream they read only data
 * that kernel cannot be writing -- weights and norm weights, and KV-cache rows other
 * than the newest (sliding attention: the row the context's last attention projection
 * wrote into that cache; full attention: the last row of the range), which they read again
 * after the wait.  A kernel of the caller's own
 * that precedes a g4 call on the same stream is waited for as usual unless it triggers
 * programmatic completion early itself (griddepcontrol.launch_dependents), in which case
 * it must not be writing weights or cache rows the next g4 call reads.
 */
#ifndef G4_B200_API_H_
#define G4_B200_API_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t g4_bf16;   /* bfloat16 bits                                  */
typedef uint8_t g4_f8e4m3;  /* E4M3FN byte                                    */
typedef uint8_t g4_f4x2;    /* two E2M1 codes, low nibble = even element      */
typedef struct CUstream_st* g4_stream_t; /* same type as cudaStream_t          */
typedef struct g4_ctx g4_ctx;

typedef enum g4_status {
  G4_OK = 0,
  G4_ERR_BAD_ARG = 1,     /* null/misaligned pointer, bad size or rank          */
  G4_ERR_CUDA = 2,        /* a CUDA runtime call or kernel launch failed        */
  G4_ERR_NCCL = 3,        /* an NCCL call failed                                */
  G4_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up                 */
  G4_ERR_UNSUPPORTED = 5, /* configuration not built into this library          */
  G4_ERR_TOO_LARGE = 6    /* a size exceeds a fixed limit (no-alloc entry point) */
} g4_status;

/* Model constants (src/lib.rs:19-22, src/axes.rs:4-29). */
#define G4_H 3840
#define G4_L 15360
#define G4_W 262144
#define G4_NS 8
#define G4_GS 2
#define G4_DS 256
#define G4_QS 4096
#define G4_PS 2048
#define G4_TS 1024
#define G4_GF 16
#define G4_DF 512
#define G4_QF 8192
#define G4_PF 512
#define G4_TF 512
#define G4_E 32768
#define G4_LAYERS 48

/* ------------------------------------------------------------------------------ */
/* Context (replaces furiosa_opt_std::Context; no reference entry point)           */
/* ------------------------------------------------------------------------------ */

/* Create a context on CUDA device `device`: allocates this context's scratch
 * (partial sums, completion counters, intermediate activations).  Replaces
 * `Context::acquire()` (src/api/worker.rs:85). */
g4_status g4_ctx_create(int device, g4_ctx** out);
g4_status g4_ctx_destroy(g4_ctx* ctx);
/* Stream all subsequent entry points of this context are issued on (default: the
 * legacy default stream). */
g4_status g4_ctx_set_stream(g4_ctx* ctx, g4_stream_t stream);
/* Tensor parallelism: this context becomes rank `rank` of `world` (1, 2, 4 or 8).
 * `nccl_id` points to the 128-byte ncclUniqueId rank 0 created (g4_nccl_unique_id)
 * and broadcast out of band.  After this, projection entry points take this rank's
 * weight shard (column-parallel gate/up/q/k/v rows, row-parallel down/o K-slices)
 * and all-reduce the row-parallel partial sums before their RMSNorm epilogue.
 * The all-reduce runs inside the MLP / o-proj kernel over NVLink peer memory: each
 * rank's exchange buffer (480 KiB) is mapped into every other rank's process with
 * CUDA IPC, so the ranks must be separate processes with peer access.  Otherwise, or
 * when any rank has G4B200_TP_EXCHANGE=nccl in its environment, every rank agrees to
 * use an NCCL all-reduce and a separate epilogue kernel instead.  The ranks must issue
 * the same sequence of MLP / o-proj calls, and destroy their contexts only after all
 * ranks' launches have finished.  (The reference runs on one chip and has no
 * counterpart; src/lib.rs:17.) */
g4_status g4_nccl_unique_id(uint8_t out_id[128]);
g4_status g4_ctx_init_tp(g4_ctx* ctx, int rank, int world, const uint8_t nccl_id[128]);
/* 1 if this context's MLP / o-proj kernels all-reduce over peer memory, 0 if they use
 * the NCCL fallback or the context is not tensor-parallel.  No reference counterpart. */
g4_status g4_ctx_tp_peer_exchange(const g4_ctx* ctx, int* out_enabled);
/* Message of the last failing call on this context (never NULL). */
const char* g4_ctx_last_error(const g4_ctx* ctx);
/* Time limit, in microseconds, of every bounded device-side wait (mbarrier, grid-wide
 * and cross-GPU waits inside fused kernels); default 2 s.  A wait that runs out sets a
 * bit in the context's device status word and its kernel returns early. */
g4_status g4_ctx_set_wait_budget(g4_ctx* ctx, uint32_t timeout_us);
/* Which kernel runs decoder_feedforward on this context (no reference counterpart):
 * G4_MLP_AUTO (the default; G4B200_MLP_KERNEL=stream in the environment switches it) or
 * G4_MLP_TENSOR run the tcgen05 block-scaled FP4 kernel on one GPU and on 2-GPU
 * tensor-parallel contexts that exchange over peer memory; G4_MLP_STREAM (CUDA-core NVFP4
 * decode + mma.sync) runs the other tensor-parallel contexts and can be asked for
 * anywhere.  Same results within f32 rounding of the dot products. */
enum { G4_MLP_AUTO = 0, G4_MLP_STREAM = 1, G4_MLP_TENSOR = 2 };
g4_status g4_ctx_set_mlp_kernel(g4_ctx* ctx, int kind);

/* How many NVFP4 pieces represent each activation in g4_decoder_feedforward_prefill
 * (no reference counterpart): 1 (plain NVFP4 activations, fastest; ~10 % relative error
 * per activation), 2 (the default; ~1 %, within the reference's bf16 tolerance on the
 * MLP output) or 3 (~0.1 %).  The tensor-core work grows with the count. */
g4_status g4_ctx_set_prefill_pieces(g4_ctx* ctx, int pieces);
/* Synchronise the context's stream, then read and clear the device status word
 * (0 = no kernel reported a timeout or an out-of-range device offset).  Returns
 * G4_ERR_TIMEOUT / G4_ERR_BAD_ARG when a bit was set. */
g4_status g4_ctx_poll_device_status(g4_ctx* ctx, uint32_t* out_bits);
/* Library build id string ("g4b200 <version> sm_100a"). */
const char* g4_version(void);

/* ------------------------------------------------------------------------------ */
/* Text entry points (src/ops.rs)                                                   */
/* ------------------------------------------------------------------------------ */

/* ops::embed_token (src/ops.rs:9-36): out[H] = bf16(table[row] * bf16(61.967734)),
 * row = *offset / (H*2), `offset` a device int32 byte offset into table[W,H]. */
g4_status g4_embed_token(g4_ctx* ctx, const g4_bf16* embedding_table, const int32_t* offset,
                         g4_bf16* out);

/* ops::copy_hidden_state (src/ops.rs:38-42): out[H] = x[H]. */
g4_status g4_copy_hidden_state(g4_ctx* ctx, const g4_bf16* x, g4_bf16* out);

/* ops::sliding_project_qkv (src/ops.rs:44-84).  Input RMSNorm; FP8 Q[Qs,H], K[Ps,H],
 * V[Ps,H] projections with per-row bf16 scales; per-head q/k RMSNorm (weights [Ds]),
 * unweighted v RMSNorm; RoPE (theta 1e4, full head) from cos/sin[E,Ds] rows at the
 * byte offset *rope_offset (sin low half pre-negated, src/host/runtime.rs:271-299);
 * q_out[Ns,Gs,Ds]; k,v scattered into the ring caches[Ts,Ns,Ds] at byte offset
 * *kv_offset.  TP: Q/K/V rows are the rank's heads (Qs/N, Ps/N rows), caches and
 * q_out the rank's heads. */
g4_status g4_sliding_project_qkv(g4_ctx* ctx, const g4_bf16* x, const g4_f8e4m3* q_weight,
                                 const g4_f8e4m3* k_weight, const g4_f8e4m3* v_weight,
                                 const g4_bf16* q_weight_scale, const g4_bf16* k_weight_scale,
                                 const g4_bf16* v_weight_scale, const g4_bf16* input_rms_weight,
                                 const g4_bf16* q_rms_weight, const g4_bf16* k_rms_weight,
                                 const int32_t* kv_offset, const int32_t* rope_offset,
                                 const g4_bf16* cos, const g4_bf16* sin, g4_bf16* k_cache,
                                 g4_bf16* v_cache, g4_bf16* q_out);

/* ops::full_project_qkv (src/ops.rs:86-124).  Full-attention (MQA) geometry: FP8
 * Q[Qf,H], K[Pf,H]; V = unweighted RMSNorm of the raw K projection; partial RoPE
 * (theta 1e6, first quarter of the angles) over Df; writes q_out[Gf,Df] and one row
 * of the page caches[Tf,Df] at byte offset *kv_offset.  TP: Q rows are the rank's
 * heads; K/V (one head) is computed redundantly on every rank. */
g4_status g4_full_project_qkv(g4_ctx* ctx, const g4_bf16* x, const g4_f8e4m3* q_weight,
                              const g4_f8e4m3* k_weight, const g4_bf16* q_weight_scale,
                              const g4_bf16* k_weight_scale, const g4_bf16* input_rms_weight,
                              const g4_bf16* q_rms_weight, const g4_bf16* k_rms_weight,
                              const int32_t* kv_offset, const int32_t* rope_offset,
                              const g4_bf16* cos, const g4_bf16* sin, g4_bf16* k_cache,
                              g4_bf16* v_cache, g4_bf16* q_out);

/* ops::sliding_attention (src/ops.rs:126-136): GQA (2 q heads per kv head), scale
 * 1.0, softmax over the ring slots whose f32 mask[Ts] is > 0, out[Ns,Gs,Ds]. */
g4_status g4_sliding_attention(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k,
                               const g4_bf16* v, const float* mask, g4_bf16* out);

/* ops::sliding_attention_output (src/ops.rs:138-158): residual[H] +=
 * RMSNorm(bf16(Wo[H,Qs]·x * o_scale)).  TP: Wo is the rank's K-slice [H, Qs/N]
 * (passed with row stride Qs/N) and x the rank's heads. */
g4_status g4_sliding_attention_output(g4_ctx* ctx, const g4_bf16* x,
                                      const g4_bf16* post_attn_rms_weight,
                                      const g4_f8e4m3* o_weight, const g4_bf16* o_weight_scale,
                                      g4_bf16* residual);

/* ops::full_attention_first_page (src/ops.rs:160-172): one 512-row page of MQA
 * attention for the 16 q heads; initialises running_max[Gf], running_sum[Gf] and the
 * UNNORMALISED out[Gf,Df] (bf16). */
g4_status g4_full_attention_first_page(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k,
                                       const g4_bf16* v, const float* mask, float* running_max,
                                       float* running_sum, g4_bf16* out);

/* ops::full_attention_page (src/ops.rs:174-186): online-softmax update of
 * running_max/running_sum/out with one more page. */
g4_status g4_full_attention_page(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k,
                                 const g4_bf16* v, const float* mask, float* running_max,
                                 float* running_sum, g4_bf16* out);

/* ops::full_attention_output (src/ops.rs:188-211): x/running_sum per head, FP8
 * o-proj Wo[H,Qf], RMSNorm, residual add in place.  TP: Wo is the rank's K-slice. */
g4_status g4_full_attention_output(g4_ctx* ctx, const g4_bf16* x, const float* running_sum,
                                   const g4_bf16* post_attn_rms_weight,
                                   const g4_f8e4m3* o_weight, const g4_bf16* o_weight_scale,
                                   g4_bf16* residual);

/* ops::decoder_feedforward (src/ops.rs:213-253), the primary hot path:
 *   x = RMSNorm(residual, pre_ff); h = gelu_tanh(bf16(bf16(Wg·x)*gs_g)) * bf16(bf16(Wu·x)*gs_u);
 *   y = bf16(bf16(Wd·h)*gs_d); residual = bf16(bf16(residual + RMSNorm(y, post_ff)) * layer_scalar[0])
 * with NVFP4 weights (packed codes + E4M3 block-16 scales + reciprocal f32 global
 * scales), in place on residual[H].  layer_scalar is bf16 [8] (replicated,
 * src/host/load.rs:99-111).  TP: up/gate are the rank's L/N rows ([L/N,H/2] codes,
 * [L/N,H/16] scales), down the rank's K-slice ([H, L/N] as [H, L/(2N)] codes with
 * row stride L/(2N), scales [H, L/(16N)]). */
g4_status g4_decoder_feedforward(g4_ctx* ctx, g4_bf16* residual, const g4_bf16* pre_ff_rms_weight,
                                 const g4_f4x2* up_weight_packed, const g4_f4x2* gate_weight_packed,
                                 const g4_f4x2* down_weight_packed,
                                 const g4_f8e4m3* up_weight_scale,
                                 const g4_f8e4m3* gate_weight_scale,
                                 const g4_f8e4m3* down_weight_scale, const float* up_global_scale,
                                 const float* gate_global_scale, const float* down_global_scale,
                                 const g4_bf16* post_ff_rms_weight, const g4_bf16* layer_scalar);

/* ops::final_norm_and_logits (src/ops.rs:255-312): out[W] = bf16(tanh(l/30)*30),
 * l = bf16(lm_head[W,H] · RMSNorm(input, rms_weight)).  TP: lm_head is the rank's
 * vocab slice [W/N, H] and out the rank's W/N logits. */
g4_status g4_final_norm_and_logits(g4_ctx* ctx, const g4_bf16* input, const g4_bf16* rms_weight,
                                   const g4_bf16* lm_head_weight, g4_bf16* out);

/* ------------------------------------------------------------------------------ */
/* B200 additions (no single reference entry point; each names what it replaces)    */
/* ------------------------------------------------------------------------------ */

/* Batched prefill of ops::decoder_feedforward (src/ops.rs:213-253) for n_tokens
 * positions at once, replacing the reference's one-position-per-dispatch prefill
 * (src/host/generate.rs:194-211) for the MLP block.  residual is [n_tokens][H] bf16,
 * updated in place; the weights are those of g4_decoder_feedforward (TP: the same
 * shards).  The block runs as two block-scaled FP4 GEMMs on the tensor cores: the
 * normed activations and h are quantised per token to NVFP4 with the weights' recipe
 * (g = 6*448/max|row|, E4M3 scale per 16, E2M1 codes), so each token's result is the
 * reference MLP applied to NVFP4-quantised activations.  Scratch for n_tokens is
 * allocated by the context on first use and kept until g4_ctx_destroy; the call
 * synchronises the device when it grows.  TP: each rank computes its intermediate
 * rows and the ranks' down-projection sums are all-reduced in f32 over NCCL. */
#define G4_PREFILL_MAX_TOKENS 65536
g4_status g4_decoder_feedforward_prefill(g4_ctx* ctx, int n_tokens, g4_bf16* residual,
                                         const g4_bf16* pre_ff_rms_weight,
                                         const g4_f4x2* up_weight_packed,
                                         const g4_f4x2* gate_weight_packed,
                                         const g4_f4x2* down_weight_packed,
                                         const g4_f8e4m3* up_weight_scale,
                                         const g4_f8e4m3* gate_weight_scale,
                                         const g4_f8e4m3* down_weight_scale,
                                         const float* up_global_scale, const float* gate_global_scale,
                                         const float* down_global_scale,
                                         const g4_bf16* post_ff_rms_weight, const g4_bf16* layer_scalar);

/* All pages of one full-attention layer in ONE split-KV launch (replaces the host loop
 * of full_attention_first_page/_page dispatches, src/host/runtime.rs:438-459).
 * k_pages/v_pages: DEVICE arrays of n_pages page pointers ([Tf,Df] bf16 each); rows
 * [0, last_row] of the last page and every row of earlier pages are attended.
 * Writes the NORMALISED output into out[Gf,Df] and 1.0 into running_sum[Gf], so
 * g4_full_attention_output consumes it unchanged. */
g4_status g4_full_attention_paged(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* const* k_pages,
                                  const g4_bf16* const* v_pages, int n_pages, int last_row,
                                  float* running_sum, g4_bf16* out);

/* Greedy sampling on the device (replaces the 512 KB logits read-back and host
 * argmax of src/host/generate.rs:130-143): *out_index = first index of the maximum
 * of logits[n] (bf16). */
g4_status g4_argmax_bf16(g4_ctx* ctx, const g4_bf16* logits, int n, int32_t* out_index);

/* Top-k / top-p sampling on the device (src/host/sampling.rs:20-72; replaces the
 * logits read-back and host sampling of src/host/generate.rs:135-143): keep the
 * (top_k + n_banned) largest logits, drop the `banned` ids (distinct; host array) unless
 * that drops all, keep top_k, p = softmax((l - l_max) / max(temperature, 1e-5)), the
 * nucleus = the shortest prefix whose running sum reaches top_p, and *out_index = the
 * first id whose running sum reaches (*uniform) x (nucleus sum).  `uniform` is a device
 * f32 in [0, 1) (the host's draw).  Equal logits rank by lower id.  1 <= top_k,
 * top_k + n_banned <= 128, 0 < top_p <= 1.  TP: logits is the rank's vocab slice of n
 * entries (ids rank*n ...); every rank gets the same id. */
g4_status g4_sample_top_k_top_p(g4_ctx* ctx, const g4_bf16* logits, int n, float temperature, int top_k,
                                float top_p, const int32_t* banned, int n_banned, const float* uniform,
                                int32_t* out_index);

/* Bit-exact dequantisation checks (scripts/generate_references.py:207-216,622-626):
 * out[n,k] = bf16(e2m1(codes) * e4m3(scale[n, k/16])) and out[n,k] = bf16(e4m3(w)). */
g4_status g4_dequant_nvfp4(g4_ctx* ctx, const g4_f4x2* packed, const g4_f8e4m3* block_scale,
                           int rows, int cols, g4_bf16* out);
g4_status g4_dequant_fp8(g4_ctx* ctx, const g4_f8e4m3* weight, int64_t count, g4_bf16* out);

/* NVFP4 variants of the attention projections (the same GEMV
 * engine with E2M1 codes, E4M3 block-16 scales and an f32 reciprocal global scale in
 * place of the FP8 per-row scales).  Argument order follows the FP8 entry points with
 * each (weight, weight_scale) pair replaced by (packed codes, block scales, global
 * scale). */
g4_status g4_sliding_project_qkv_nvfp4(
    g4_ctx* ctx, const g4_bf16* x, const g4_f4x2* q_weight, const g4_f4x2* k_weight,
    const g4_f4x2* v_weight, const g4_f8e4m3* q_block_scale, const g4_f8e4m3* k_block_scale,
    const g4_f8e4m3* v_block_scale, const float* q_global_scale, const float* k_global_scale,
    const float* v_global_scale, const g4_bf16* input_rms_weight, const g4_bf16* q_rms_weight,
    const g4_bf16* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
    const g4_bf16* cos, const g4_bf16* sin, g4_bf16* k_cache, g4_bf16* v_cache, g4_bf16* q_out);

g4_status g4_sliding_attention_output_nvfp4(g4_ctx* ctx, const g4_bf16* x,
                                            const g4_bf16* post_attn_rms_weight,
                                            const g4_f4x2* o_weight,
                                            const g4_f8e4m3* o_block_scale,
                                            const float* o_global_scale, g4_bf16* residual);

/* NVFP4 variants of the full-attention (MQA) projections: as
 * g4_full_project_qkv / g4_full_attention_output with each FP8 (weight, row scale) pair
 * replaced by (packed E2M1 codes [N, K/2], E4M3 block scales [N, K/16], reciprocal f32
 * global scale).  TP as the FP8 entry points. */
g4_status g4_full_project_qkv_nvfp4(g4_ctx* ctx, const g4_bf16* x, const g4_f4x2* q_weight, const g4_f4x2* k_weight,
                                    const g4_f8e4m3* q_block_scale, const g4_f8e4m3* k_block_scale,
                                    const float* q_global_scale, const float* k_global_scale,
                                    const g4_bf16* input_rms_weight, const g4_bf16* q_rms_weight,
                                    const g4_bf16* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                                    const g4_bf16* cos, const g4_bf16* sin, g4_bf16* k_cache, g4_bf16* v_cache,
                                    g4_bf16* q_out);
g4_status g4_full_attention_output_nvfp4(g4_ctx* ctx, const g4_bf16* x, const float* running_sum,
                                         const g4_bf16* post_attn_rms_weight, const g4_f4x2* o_weight,
                                         const g4_f8e4m3* o_block_scale, const float* o_global_scale,
                                         g4_bf16* residual);

/* GQA decode attention of the sliding geometry over a cache of any length (BASELINE
 * config 3's synthetic 16 q heads over 8 KV heads of 256): q[Ns,Gs,Ds], k/v[n_rows,Ns,Ds],
 * mask[n_rows] f32 (> 0 = attended), out[Ns,Gs,Ds]; n_rows a multiple of 64 up to 32768.
 * g4_sliding_attention is this at n_rows = Ts.  TP: the rank's heads. */
g4_status g4_attention_gqa(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k, const g4_bf16* v, const float* mask,
                           int n_rows, g4_bf16* out);

/* ------------------------------------------------------------------------------ */
/* Decode runtime (src/host/load.rs Model, src/host/runtime.rs Workspace / Decode)  */
/* ------------------------------------------------------------------------------ */

/* The text decoder's weight set (MlpWeights / SlidingLayer / FullLayer / Model,
 * src/host/load.rs:10-87) as device pointers registered by checkpoint tensor name:
 *   model.language_model.embed_tokens.weight         bf16 [W, H] (tied lm_head; every rank
 *                                                     holds the whole table)
 *   model.language_model.norm.weight                 bf16 [H]
 *   model.language_model.layers.<i>.<suffix>, suffix one of
 *     input_layernorm.weight, post_attention_layernorm.weight,
 *     pre_feedforward_layernorm.weight, post_feedforward_layernorm.weight   bf16 [H]
 *     layer_scalar                                   bf16 [8] (the scalar replicated,
 *                                                     load.rs:99-111)
 *     self_attn.{q,k,v,o}_proj.weight                f8e4m3 [N, K] (no v_proj in full layers)
 *     self_attn.{q,k,v,o}_proj.weight_scale          bf16 [N] per-row scale
 *     self_attn.{q,k}_norm.weight                    bf16 [D]
 *     mlp.{up,gate,down}_proj.weight_packed          u8 [N, K/2] E2M1 codes
 *     mlp.{up,gate,down}_proj.weight_scale           f8e4m3 [N, K/16]
 *     mlp.{up,gate,down}_proj.weight_global_scale    f32 [1], the RECIPROCAL of the
 *                                                     checkpoint value (load.rs:171-191)
 * Layer i is a full-attention layer iff i % 6 == 5 (load.rs:369-376).  Under tensor
 * parallelism each tensor is the rank's shard as the per-op entry points take it.  The
 * model only records pointers (it never frees them) unless a loader filled it.
 * g4_model_create needs no GPU; sizes are checked by g4_workspace_create. */
typedef struct g4_model g4_model;
g4_status g4_model_create(int n_layers, g4_model** out);
g4_status g4_model_destroy(g4_model* model);
g4_status g4_model_set_tensor(g4_model* model, const char* name, const void* device_ptr, uint64_t bytes);
const char* g4_model_last_error(const g4_model* model);
/* load_model (src/host/load.rs:357-386) for the text decoder: memory-maps a safetensors
 * checkpoint, checks every tensor's dtype and shape as the reference loader does
 * (load.rs:89-191: BF16 norms and row scales [N, 1], F8_E4M3 projections, U8 NVFP4 codes
 * [N, K/2], F8_E4M3 block scales [N, K/16], scalar F32 global scales that must be finite
 * and non-zero), copies this context's tensor-parallel shard of each to the device (the
 * global scale as its reciprocal, the layer scalar replicated to [8]) and returns a model
 * that owns those buffers.  Errors name the tensor (g4_ctx_last_error). */
g4_status g4_model_load_safetensors(g4_ctx* ctx, const char* path, int n_layers, g4_model** out);
/* The same checks without a GPU: G4_OK if the file holds an n_layers text decoder that
 * can be cut for `world` ranks; otherwise G4_ERR_BAD_ARG and the reason in msg. */
g4_status g4_checkpoint_check(const char* path, int n_layers, int world, char* msg, uint64_t msg_len);
/* 1 if layer `layer` is a full-attention layer (load.rs:369-376), else 0. */
int g4_model_layer_is_full(int layer);

/* Workspace (src/host/runtime.rs:135-211): RoPE tables (rope_data, :271-299), every
 * layer's KV cache (sliding: ring [Ts, Ns/N, Ds]; full: [ceil(max_positions/512)*512, Df],
 * i.e. the reference's 512-row pages back to back), the current mask row, the
 * device-resident byte offsets (:213-228), the decode scratch of Decode (:301-309) and
 * the logits [W/N].  Checks that every tensor of `model` is set with the shard size of
 * the context's tensor-parallel world. */
typedef struct g4_workspace g4_workspace;
g4_status g4_workspace_create(g4_ctx* ctx, const g4_model* model, int max_positions, g4_workspace** out);
/* Sampling mode of the decode steps (src/host/generate.rs:214-297 with
 * src/host/sampling.rs): top_k == 0 is greedy (the default); otherwise every step
 * draws its token by g4_sample_top_k_top_p's rule with the draw u derived on the device
 * from (seed, position) (splitmix64 of seed + pos * 0x9E3779B97F4A7C15, top 24 bits / 2^24),
 * so a run is reproducible and every TP rank draws the same token.  Predictions logged by
 * g4_decode_predictions are the drawn tokens.  Takes effect at the next step. */
g4_status g4_workspace_set_sampling(g4_workspace* ws, float temperature, int top_k, float top_p,
                                    const int32_t* banned, int n_banned, uint64_t seed);
g4_status g4_workspace_destroy(g4_workspace* ws);
/* Device pointers of layer `layer`'s K and V caches and their size in bytes each. */
g4_status g4_workspace_kv_cache(g4_workspace* ws, int layer, g4_bf16** k, g4_bf16** v, uint64_t* bytes);
/* This rank's logits [W/N] of the last step and the hidden state x [H] (device). */
g4_status g4_workspace_logits(g4_workspace* ws, const g4_bf16** logits, int* count);
g4_status g4_workspace_hidden(g4_workspace* ws, const g4_bf16** x);

/* Decode::run (src/host/runtime.rs:312-347): embed `token`, run every layer at position
 * `pos` (writing that position's K/V), final norm and logits into the workspace, then the
 * device argmax (g4_decode_last_prediction reads it).  Asynchronous on the context's
 * stream. */
g4_status g4_decode_run(g4_ctx* ctx, g4_workspace* ws, const g4_model* model, int32_t token, int32_t pos);
/* Greedy decoding with the position and token kept on the device (replaces the host loop
 * of src/host/generate.rs:194-298: prefill one position per step, read logits, sample):
 *   g4_decode_begin  uploads prompt[prompt_len] for positions start_pos.. and resets the
 *                    state; g4_decode_steps runs n steps (use_graph: one CUDA graph of the
 *                    whole step, captured on first use, replayed per step; needs a
 *                    non-default stream); each step's input is the next prompt token while
 *                    the prompt lasts, then the previous step's argmax, which is recorded;
 *   g4_decode_tokens synchronises and copies up to max_out recorded tokens to the host;
 *   g4_generate_greedy runs prompt_len + max_new - 1 steps and returns max_new tokens. */
g4_status g4_decode_begin(g4_ctx* ctx, g4_workspace* ws, const int32_t* prompt, int prompt_len, int start_pos,
                          int max_new);
g4_status g4_decode_steps(g4_ctx* ctx, g4_workspace* ws, const g4_model* model, int n_steps, int use_graph);
g4_status g4_decode_tokens(g4_ctx* ctx, g4_workspace* ws, int32_t* out, int max_out, int* n_out);
/* The greedy prediction of every step since g4_decode_begin (prompt positions included),
 * in step order, up to max_out; and the last step's prediction with the next position. */
g4_status g4_decode_predictions(g4_ctx* ctx, g4_workspace* ws, int32_t* out, int max_out, int* n_out);
g4_status g4_decode_last_prediction(g4_ctx* ctx, g4_workspace* ws, int32_t* token, int32_t* next_pos);
g4_status g4_generate_greedy(g4_ctx* ctx, g4_workspace* ws, const g4_model* model, const int32_t* prompt,
                             int prompt_len, int start_pos, int max_new, int use_graph, int32_t* out_tokens);

/* ------------------------------------------------------------------------------ */
/* Allocation-free decoder_feedforward (no counterpart in the reference)            */
/* ------------------------------------------------------------------------------ */

/* Scratch this entry point owns: one fixed array in the library's device image, on
 * every GPU that loads the library, held until the process exits. */
#define G4_NOALLOC_MAX_INTERMEDIATE 15360 /* rows of up/gate = K of down       */
#define G4_NOALLOC_SCRATCH_BYTES 47104    /* 46 KiB: 1 KiB counters, f32 [H], bf16 [max intermediate] */

/* The decoder_feedforward math of g4_decoder_feedforward (same formula, in place on
 * residual[H]) for callers that cannot allocate device memory.  It always runs the
 * streaming kernel (CUDA-core NVFP4 decode + mma.sync, the kernel a context runs with
 * G4_MLP_STREAM), whose scratch fits the fixed array below; a single-GPU context
 * defaults to the tcgen05 kernel, so the two agree within f32 rounding, not bit for bit.  It has no
 * counterpart in the reference.  A g4_ctx needs cudaMalloc for its scratch, which some
 * hosts do not allow: serving engines that hand every free byte of HBM to their own
 * pool at start-up (a later cudaMalloc fails or fragments that pool), plugin hooks that
 * must not allocate on the per-call path, and latency-critical loops that cannot take
 * the device-wide synchronisation a cudaMalloc/cudaFree may cause.  This entry point
 * instead keeps its scratch (counters, the down-projection sums and the intermediate
 * vector h) in the fixed array above and calls no allocating routine.
 *
 *   stream            : a stream of the CURRENT device (NULL = its default stream).
 *   intermediate_size : rows of up/gate and K of down: exactly G4_L (the model's
 *                       layer), 7680, or a multiple of 128 up to 3840 (single-GPU only,
 *                       no all-reduce).  > G4_NOALLOC_MAX_INTERMEDIATE returns
 *                       G4_ERR_TOO_LARGE; every other size returns G4_ERR_UNSUPPORTED.
 *   weights           : as g4_decoder_feedforward with L = intermediate_size
 *                       (up/gate [n, H/2] codes, [n, H/16] scales; down [H, n/2] codes,
 *                       [H, n/16] scales).
 *
 * The first call on a device sets up that device (looks up the array's device address,
 * the SM count and the launch limits); make that first call before any stream capture
 * starts.  Every call on a device shares the one array and leaves its contents behind;
 * each call first clears, on `stream`, the counter block that must start at zero.
 * Calls that can overlap on the GPU (different streams without ordering between them,
 * or different host threads) race on the array and give wrong results: order them.
 * Device-side wait timeouts are not reported here (there is no context to poll). */
g4_status g4_decoder_feedforward_noalloc(
    g4_stream_t stream, uint32_t intermediate_size, g4_bf16* residual,
    const g4_bf16* pre_ff_rms_weight, const g4_f4x2* up_weight_packed,
    const g4_f4x2* gate_weight_packed, const g4_f4x2* down_weight_packed,
    const g4_f8e4m3* up_weight_scale, const g4_f8e4m3* gate_weight_scale,
    const g4_f8e4m3* down_weight_scale, const float* up_global_scale,
    const float* gate_global_scale, const float* down_global_scale,
    const g4_bf16* post_ff_rms_weight, const g4_bf16* layer_scalar);

#ifdef __cplusplus
}
#endif

#endif /* G4_B200_API_H_ */
