#include <cmath>
// The C ABI of include/g4.h: argument validation and dispatch to the kernel launchers.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "g4_internal.h"
#include "g4_common.cuh"

namespace g4 {

g4_status fail(g4_ctx* ctx, g4_status code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}
g4_status check_cuda(g4_ctx* ctx, cudaError_t err, const char* what) {
  if (err == cudaSuccess) return G4_OK;
  return fail(ctx, G4_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}
g4_status allow_max_dynamic_smem(g4_ctx* ctx, const void* fn, size_t need, const char* what) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, ctx->device})) return G4_OK;
  int optin = 0;
  g4_status st = check_cuda(ctx, cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device),
                            "cudaDeviceGetAttribute(smem opt-in)");
  if (st != G4_OK) return st;
  // the opt-in maximum covers static and dynamic shared memory together
  cudaFuncAttributes fa = {};
  st = check_cuda(ctx, cudaFuncGetAttributes(&fa, fn), "cudaFuncGetAttributes");
  if (st != G4_OK) return st;
  const int dyn_max = optin - static_cast<int>(fa.sharedSizeBytes);
  if (dyn_max <= 0 || need > static_cast<size_t>(dyn_max))
    return fail(ctx, G4_ERR_UNSUPPORTED, std::string(what) + ": shared memory layout too large");
  st = check_cuda(ctx, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_max), what);
  if (st == G4_OK) done.insert({fn, ctx->device});
  return st;
}

g4_status launch_kernel(g4_ctx* ctx, const void* fn, dim3 grid, dim3 block, size_t smem, void** args,
                        bool cooperative, const char* what, unsigned cluster_x) {
  cudaLaunchAttribute attrs[3];
  unsigned n = 0;
  if (cooperative) {
    attrs[n].id = cudaLaunchAttributeCooperative;
    attrs[n].val.cooperative = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster_x;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  const unsigned base = n;
  if (ctx->pdl_ok) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess && n > base) {
    (void)cudaGetLastError();
    cfg.numAttrs = base;
    e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e == cudaSuccess) ctx->pdl_ok = false;  // the launch attribute was what failed
  }
  if (e != cudaSuccess) (void)cudaGetLastError();
  return check_cuda(ctx, e, what);
}

bool aligned16(const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// NCCL is resolved at run time, only when tensor parallelism is used: a process that
// already loaded an NCCL (e.g. torch's bundled one) keeps using that copy, and a
// single-GPU process never loads one.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

static NcclApi& nccl() {
  static NcclApi api;
  static bool tried = false;
  if (tried) return api;
  tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) return api;
  api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
  api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
  api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
  api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
  api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
  api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
  api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.comm_destroy &&
           api.error_string;
  return api;
}

g4_status allreduce_f32(g4_ctx* ctx, float* buf, size_t count) {
  if (ctx->comm == nullptr || !nccl().ok) return fail(ctx, G4_ERR_NCCL, "tensor parallelism without a communicator");
  const ncclResult_t r =
      nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum, reinterpret_cast<ncclComm_t>(ctx->comm), ctx->stream);
  if (r != ncclSuccess) return fail(ctx, G4_ERR_NCCL, std::string("ncclAllReduce: ") + nccl().error_string(r));
  return G4_OK;
}

g4_status allgather_u64n(g4_ctx* ctx, const uint64_t* in, uint64_t* out, int count) {
  if (ctx->comm == nullptr || !nccl().ok) return fail(ctx, G4_ERR_NCCL, "tensor parallelism without a communicator");
  const ncclResult_t r = nccl().all_gather(in, out, static_cast<size_t>(count), ncclUint64,
                                           reinterpret_cast<ncclComm_t>(ctx->comm), ctx->stream);
  if (r != ncclSuccess) return fail(ctx, G4_ERR_NCCL, std::string("ncclAllGather: ") + nccl().error_string(r));
  return G4_OK;
}

g4_status allgather_u64(g4_ctx* ctx, const uint64_t* in, uint64_t* out) {
  if (ctx->comm == nullptr || !nccl().ok) return fail(ctx, G4_ERR_NCCL, "tensor parallelism without a communicator");
  const ncclResult_t r =
      nccl().all_gather(in, out, 1, ncclUint64, reinterpret_cast<ncclComm_t>(ctx->comm), ctx->stream);
  if (r != ncclSuccess) return fail(ctx, G4_ERR_NCCL, std::string("ncclAllGather: ") + nccl().error_string(r));
  return G4_OK;
}

// Maps every rank's TP exchange buffer into this process (CUDA IPC handles swapped with
// an NCCL all-gather), so that the MLP and o-proj kernels all-reduce their partial
// outputs themselves over NVLink.  The ranks then agree (NCCL min) on whether all of
// them succeeded: any rank without peer access, or with G4B200_TP_EXCHANGE=nccl in its
// environment, puts every rank on the NCCL all-reduce path instead.  Returns G4_OK in
// both cases; an error only if the NCCL calls themselves fail.
static void close_peer_exchange(g4_ctx* ctx) {
  for (int p = 0; p < kMaxTp; ++p) {
    if (ctx->peers.buf[p] != nullptr && p != ctx->tp_rank) cudaIpcCloseMemHandle(ctx->peers.buf[p]);
    ctx->peers.buf[p] = nullptr;
  }
  ctx->peers.world = 0;
}

static g4_status setup_peer_exchange(g4_ctx* ctx) {
  const int world = ctx->tp_world, rank = ctx->tp_rank;
  const ncclComm_t comm = reinterpret_cast<ncclComm_t>(ctx->comm);
  const char* env = std::getenv("G4B200_TP_EXCHANGE");
  bool ok = !(env != nullptr && std::strcmp(env, "nccl") == 0);
  cudaIpcMemHandle_t mine = {};
  if (ok) ok = cudaMalloc(&ctx->buf.xch, kXchBytes) == cudaSuccess;
  if (ok) ok = cudaMemset(ctx->buf.xch, 0, kXchBytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (ok) ok = cudaIpcGetMemHandle(&mine, ctx->buf.xch) == cudaSuccess;
  if (!ok) (void)cudaGetLastError();
  // [world] handles gathered in the row-parallel partial buffer (unused until the first
  // launch), then the agreement flag after them
  static_assert(sizeof(cudaIpcMemHandle_t) * kMaxTp + 4 <= kPartFloats * 4, "staging fits");
  uint8_t* stage = reinterpret_cast<uint8_t*>(ctx->buf.part);
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  // (a pageable host-to-device copy may return before its DMA lands: synchronize before
  // NCCL reads it on another stream)
  g4_status st = check_cuda(ctx, cudaMemcpy(stage + rank * hb, &mine, hb, cudaMemcpyHostToDevice), "xch: stage");
  if (st == G4_OK) st = check_cuda(ctx, cudaDeviceSynchronize(), "xch: stage sync");
  if (st != G4_OK) return st;
  ncclResult_t r = nccl().all_gather(stage + rank * hb, stage, hb, ncclUint8, comm, ctx->stream);
  if (r != ncclSuccess) return fail(ctx, G4_ERR_NCCL, std::string("ncclAllGather: ") + nccl().error_string(r));
  cudaIpcMemHandle_t all[kMaxTp];
  st = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "xch: gather");
  if (st == G4_OK) st = check_cuda(ctx, cudaMemcpy(all, stage, hb * world, cudaMemcpyDeviceToHost), "xch: read");
  if (st != G4_OK) return st;
  ctx->peers = PeerXch{};
  for (int p = 0; p < world && ok; ++p) {
    if (p == rank) {
      ctx->peers.buf[p] = ctx->buf.xch;
      continue;
    }
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      (void)cudaGetLastError();
      ok = false;
    } else {
      ctx->peers.buf[p] = static_cast<uint64_t*>(ptr);
    }
  }
  int32_t* flag = reinterpret_cast<int32_t*>(stage + hb * kMaxTp);
  const int32_t mine_ok = ok ? 1 : 0;
  int32_t all_ok = 0;
  st = check_cuda(ctx, cudaMemcpy(flag, &mine_ok, 4, cudaMemcpyHostToDevice), "xch: flag");
  if (st == G4_OK) st = check_cuda(ctx, cudaDeviceSynchronize(), "xch: flag sync");
  if (st != G4_OK) return st;
  r = nccl().all_reduce(flag, flag, 1, ncclInt32, ncclMin, comm, ctx->stream);
  if (r != ncclSuccess) return fail(ctx, G4_ERR_NCCL, std::string("ncclAllReduce: ") + nccl().error_string(r));
  st = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "xch: agree");
  if (st == G4_OK) st = check_cuda(ctx, cudaMemcpy(&all_ok, flag, 4, cudaMemcpyDeviceToHost), "xch: agree read");
  if (st != G4_OK) return st;
  if (all_ok == 1) {
    ctx->peers.rank = rank;
    ctx->peers.world = world;
  } else {
    close_peer_exchange(ctx);
  }
  return G4_OK;
}

// launchers (other translation units)
g4_status launch_qkv(g4_ctx*, bool, bool, const uint16_t*, const uint8_t* const[3], const uint8_t* const[3],
                     const uint16_t* const[3], const float* const[3], const uint16_t*, const uint16_t*,
                     const uint16_t*, const int32_t*, const int32_t*, const uint16_t*, const uint16_t*, uint16_t*,
                     uint16_t*, uint16_t*, long long);
g4_status launch_oproj(g4_ctx*, bool, bool, const uint16_t*, const float*, const uint16_t*, const uint8_t*,
                       const uint8_t*, const uint16_t*, const float*, uint16_t*);
g4_status launch_lm_head(g4_ctx*, const uint16_t*, const uint16_t*, const uint16_t*, uint16_t*);
g4_status launch_sliding_attention(g4_ctx*, const uint16_t*, const uint16_t*, const uint16_t*, const float*,
                                   uint16_t*);
g4_status launch_full_page(g4_ctx*, bool, const uint16_t*, const uint16_t*, const uint16_t*, const float*, float*,
                           float*, uint16_t*);
g4_status launch_full_paged(g4_ctx*, const uint16_t*, const uint16_t* const*, const uint16_t* const*, int, int,
                            float*, uint16_t*);
g4_status launch_embed(g4_ctx*, const uint16_t*, const int32_t*, uint16_t*);
g4_status launch_gqa_attention(g4_ctx*, const uint16_t*, const uint16_t*, const uint16_t*, const float*, int,
                               uint16_t*);
g4_status launch_argmax(g4_ctx*, const uint16_t*, int, int32_t*);
g4_status launch_dequant_nvfp4(g4_ctx*, const uint8_t*, const uint8_t*, int, int, uint16_t*);
g4_status launch_dequant_fp8(g4_ctx*, const uint8_t*, long long, uint16_t*);

}  // namespace g4

using namespace g4;

#define G4_CHECK_CTX(ctx) \
  if ((ctx) == nullptr) return G4_ERR_BAD_ARG
// Every listed pointer must be non-null and 16-byte aligned.
#define G4_REQUIRE_PTRS(ctx, ...)                                                          \
  do {                                                                                     \
    const void* _ptrs[] = {__VA_ARGS__};                                                   \
    for (size_t _i = 0; _i < sizeof(_ptrs) / sizeof(_ptrs[0]); ++_i)                       \
      if (!aligned16(_ptrs[_i]))                                                           \
        return fail(ctx, G4_ERR_BAD_ARG, "argument " + std::to_string(_i) +                \
                                             " is null or not 16-byte aligned");           \
  } while (0)
// Scalars/offsets need only natural alignment.
#define G4_REQUIRE_SCALARS(ctx, ...)                                                       \
  do {                                                                                     \
    const void* _ptrs[] = {__VA_ARGS__};                                                   \
    for (size_t _i = 0; _i < sizeof(_ptrs) / sizeof(_ptrs[0]); ++_i)                       \
      if (_ptrs[_i] == nullptr || (reinterpret_cast<uintptr_t>(_ptrs[_i]) & 3u))           \
        return fail(ctx, G4_ERR_BAD_ARG, "scalar argument " + std::to_string(_i) +         \
                                             " is null or misaligned");                    \
  } while (0)

extern "C" {

const char* g4_version(void) { return "g4b200 0.1.0 sm_100a"; }

g4_status g4_ctx_create(int device, g4_ctx** out) {
  if (out == nullptr) return G4_ERR_BAD_ARG;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return G4_ERR_CUDA;
  g4_ctx* ctx = new g4_ctx();
  ctx->device = device;
  g4_status st = check_cuda(ctx, cudaSetDevice(device), "cudaSetDevice");
  if (st == G4_OK)
    st = check_cuda(ctx, cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device), "sm count");
  int major = 0;
  if (st == G4_OK) st = check_cuda(ctx, cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "cc");
  if (st == G4_OK && major != 10) st = fail(ctx, G4_ERR_UNSUPPORTED, "g4b200 needs a compute capability 10.0 GPU");
  DeviceBuffers& b = ctx->buf;
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.scratch, sizeof(Scratch)), "cudaMalloc scratch");
  if (st == G4_OK) st = check_cuda(ctx, cudaMemset(b.scratch, 0, sizeof(Scratch)), "cudaMemset scratch");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.part, kPartFloats * 4), "cudaMalloc part");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.rows, kHeadFloats * 4), "cudaMalloc rows");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.hbuf, kHFloats * 2), "cudaMalloc hbuf");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.ybuf, 3840 * 4), "cudaMalloc ybuf");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.attn, kAttnFloats * 4), "cudaMalloc attn");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.tc_seg, kTcSegFloats * 4), "cudaMalloc tc_seg");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.tc_ptag, kTcPartWords * 8), "cudaMalloc tc_ptag");
  if (st == G4_OK) st = check_cuda(ctx, cudaMemset(b.tc_ptag, 0, kTcPartWords * 8), "cudaMemset tc_ptag");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.tc_htag, kHFloats * 4), "cudaMalloc tc_htag");
  if (st == G4_OK) st = check_cuda(ctx, cudaMalloc(&b.cand, kCandWords * 8), "cudaMalloc cand");
  if (st == G4_OK) st = check_cuda(ctx, cudaMemset(b.tc_htag, 0, kHFloats * 4), "cudaMemset tc_htag");
  if (st == G4_OK) st = check_cuda(ctx, cudaDeviceSynchronize(), "ctx init");
  if (st != G4_OK) {
    g4_ctx_destroy(ctx);
    return st;
  }
  *out = ctx;
  return G4_OK;
}

g4_status g4_ctx_destroy(g4_ctx* ctx) {
  G4_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  close_peer_exchange(ctx);
  if (ctx->comm && nccl().ok) nccl().comm_destroy(reinterpret_cast<ncclComm_t>(ctx->comm));
  cudaFree(ctx->buf.scratch);
  cudaFree(ctx->buf.part);
  cudaFree(ctx->buf.rows);
  cudaFree(ctx->buf.hbuf);
  cudaFree(ctx->buf.ybuf);
  cudaFree(ctx->buf.attn);
  cudaFree(ctx->buf.xch);
  cudaFree(ctx->buf.tc_seg);
  cudaFree(ctx->buf.tc_ptag);
  cudaFree(ctx->buf.tc_htag);
  cudaFree(ctx->buf.cand);
  cudaFree(ctx->prefill.xq);
  cudaFree(ctx->prefill.h);
  cudaFree(ctx->prefill.hq);
  cudaFree(ctx->prefill.y);
  cudaFree(ctx->prefill.ginv);
  cudaFree(ctx->prefill.down_sf);
  delete ctx;
  return G4_OK;
}

g4_status g4_ctx_set_stream(g4_ctx* ctx, g4_stream_t stream) {
  G4_CHECK_CTX(ctx);
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  return G4_OK;
}

g4_status g4_nccl_unique_id(uint8_t out_id[128]) {
  if (out_id == nullptr) return G4_ERR_BAD_ARG;
  ncclUniqueId id;
  if (!nccl().ok || nccl().get_unique_id(&id) != ncclSuccess) return G4_ERR_NCCL;
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(out_id, &id, 128);
  return G4_OK;
}

g4_status g4_ctx_init_tp(g4_ctx* ctx, int rank, int world, const uint8_t nccl_id[128]) {
  G4_CHECK_CTX(ctx);
  if (!(world == 1 || world == 2 || world == 4 || world == 8) || rank < 0 || rank >= world)
    return fail(ctx, G4_ERR_BAD_ARG, "tensor-parallel world must be 1, 2, 4 or 8 and 0 <= rank < world");
  ctx->tp_rank = rank;
  ctx->tp_world = world;
  if (world == 1) return G4_OK;
  if (nccl_id == nullptr) return fail(ctx, G4_ERR_BAD_ARG, "nccl_id is null");
  ncclUniqueId id;
  std::memcpy(&id, nccl_id, 128);
  cudaSetDevice(ctx->device);
  ncclComm_t comm = nullptr;
  if (!nccl().ok) return fail(ctx, G4_ERR_NCCL, "libnccl.so.2 could not be loaded");
  const ncclResult_t r = nccl().comm_init_rank(&comm, world, id, rank);
  if (r != ncclSuccess) return fail(ctx, G4_ERR_NCCL, std::string("ncclCommInitRank: ") + nccl().error_string(r));
  ctx->comm = reinterpret_cast<ncclComm*>(comm);
  return setup_peer_exchange(ctx);
}

g4_status g4_ctx_tp_peer_exchange(const g4_ctx* ctx, int* out_enabled) {
  if (ctx == nullptr || out_enabled == nullptr) return G4_ERR_BAD_ARG;
  *out_enabled = ctx->peers.world > 1 ? 1 : 0;
  return G4_OK;
}

const char* g4_ctx_last_error(const g4_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

g4_status g4_ctx_set_wait_budget(g4_ctx* ctx, uint32_t timeout_us) {
  G4_CHECK_CTX(ctx);
  if (timeout_us == 0) return fail(ctx, G4_ERR_BAD_ARG, "wait budget must be positive");
  ctx->wait_budget_ns = static_cast<uint64_t>(timeout_us) * 1000ull;
  return G4_OK;
}

g4_status g4_ctx_set_mlp_kernel(g4_ctx* ctx, int kind) {
  G4_CHECK_CTX(ctx);
  if (kind != G4_MLP_AUTO && kind != G4_MLP_STREAM && kind != G4_MLP_TENSOR)
    return fail(ctx, G4_ERR_BAD_ARG, "mlp kernel must be G4_MLP_AUTO, G4_MLP_STREAM or G4_MLP_TENSOR");
  ctx->mlp_kernel = kind;
  return G4_OK;
}

g4_status g4_ctx_set_prefill_pieces(g4_ctx* ctx, int pieces) {
  G4_CHECK_CTX(ctx);
  if (pieces < 1 || pieces > 3) return fail(ctx, G4_ERR_BAD_ARG, "prefill pieces must be 1, 2 or 3");
  ctx->prefill_pieces = pieces;
  return G4_OK;
}

g4_status g4_ctx_poll_device_status(g4_ctx* ctx, uint32_t* out_bits) {
  G4_CHECK_CTX(ctx);
  if (out_bits == nullptr) return fail(ctx, G4_ERR_BAD_ARG, "out_bits is null");
  g4_status st = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "poll: stream sync");
  if (st != G4_OK) return st;
  uint32_t bits = 0;
  st = check_cuda(ctx, cudaMemcpy(&bits, &ctx->buf.scratch->status, 4, cudaMemcpyDeviceToHost), "poll: read");
  if (st != G4_OK) return st;
  st = check_cuda(ctx, cudaMemset(&ctx->buf.scratch->status, 0, 4), "poll: clear");
  if (st != G4_OK) return st;
  *out_bits = bits;
  if (bits & (DEV_ERR_TIMEOUT_MBAR | DEV_ERR_TIMEOUT_GRID | DEV_ERR_TIMEOUT_PEER))
    return fail(ctx, G4_ERR_TIMEOUT, "a bounded device-side wait timed out (status " + std::to_string(bits) + ")");
  if (bits & DEV_ERR_BAD_OFFSET) return fail(ctx, G4_ERR_BAD_ARG, "a device-resident offset was out of range");
  return G4_OK;
}

g4_status g4_embed_token(g4_ctx* ctx, const g4_bf16* embedding_table, const int32_t* offset, g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, embedding_table, out);
  G4_REQUIRE_SCALARS(ctx, offset);
  return launch_embed(ctx, embedding_table, offset, out);
}

g4_status g4_copy_hidden_state(g4_ctx* ctx, const g4_bf16* x, g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, out);
  return check_cuda(ctx, cudaMemcpyAsync(out, x, G4_H * 2, cudaMemcpyDeviceToDevice, ctx->stream),
                    "copy_hidden_state");
}

g4_status g4_sliding_project_qkv(g4_ctx* ctx, const g4_bf16* x, const g4_f8e4m3* q_weight, const g4_f8e4m3* k_weight,
                                 const g4_f8e4m3* v_weight, const g4_bf16* q_weight_scale,
                                 const g4_bf16* k_weight_scale, const g4_bf16* v_weight_scale,
                                 const g4_bf16* input_rms_weight, const g4_bf16* q_rms_weight,
                                 const g4_bf16* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                                 const g4_bf16* cos, const g4_bf16* sin, g4_bf16* k_cache, g4_bf16* v_cache,
                                 g4_bf16* q_out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, q_weight, k_weight, v_weight, input_rms_weight, q_rms_weight, k_rms_weight, cos, sin,
                  k_cache, v_cache, q_out);
  G4_REQUIRE_SCALARS(ctx, q_weight_scale, k_weight_scale, v_weight_scale, kv_offset, rope_offset);
  const uint8_t* w[3] = {q_weight, k_weight, v_weight};
  const uint8_t* bs[3] = {nullptr, nullptr, nullptr};
  const uint16_t* rs[3] = {q_weight_scale, k_weight_scale, v_weight_scale};
  const float* gs[3] = {nullptr, nullptr, nullptr};
  return launch_qkv(ctx, false, false, x, w, bs, rs, gs, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset,
                    rope_offset, cos, sin, k_cache, v_cache, q_out, 0);
}

g4_status g4_sliding_project_qkv_nvfp4(g4_ctx* ctx, const g4_bf16* x, const g4_f4x2* q_weight,
                                       const g4_f4x2* k_weight, const g4_f4x2* v_weight,
                                       const g4_f8e4m3* q_block_scale, const g4_f8e4m3* k_block_scale,
                                       const g4_f8e4m3* v_block_scale, const float* q_global_scale,
                                       const float* k_global_scale, const float* v_global_scale,
                                       const g4_bf16* input_rms_weight, const g4_bf16* q_rms_weight,
                                       const g4_bf16* k_rms_weight, const int32_t* kv_offset,
                                       const int32_t* rope_offset, const g4_bf16* cos, const g4_bf16* sin,
                                       g4_bf16* k_cache, g4_bf16* v_cache, g4_bf16* q_out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, q_weight, k_weight, v_weight, q_block_scale, k_block_scale, v_block_scale,
                  input_rms_weight, q_rms_weight, k_rms_weight, cos, sin, k_cache, v_cache, q_out);
  G4_REQUIRE_SCALARS(ctx, q_global_scale, k_global_scale, v_global_scale, kv_offset, rope_offset);
  const uint8_t* w[3] = {q_weight, k_weight, v_weight};
  const uint8_t* bs[3] = {q_block_scale, k_block_scale, v_block_scale};
  const uint16_t* rs[3] = {nullptr, nullptr, nullptr};
  const float* gs[3] = {q_global_scale, k_global_scale, v_global_scale};
  return launch_qkv(ctx, false, true, x, w, bs, rs, gs, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset,
                    rope_offset, cos, sin, k_cache, v_cache, q_out, 0);
}

g4_status g4_full_project_qkv(g4_ctx* ctx, const g4_bf16* x, const g4_f8e4m3* q_weight, const g4_f8e4m3* k_weight,
                              const g4_bf16* q_weight_scale, const g4_bf16* k_weight_scale,
                              const g4_bf16* input_rms_weight, const g4_bf16* q_rms_weight,
                              const g4_bf16* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                              const g4_bf16* cos, const g4_bf16* sin, g4_bf16* k_cache, g4_bf16* v_cache,
                              g4_bf16* q_out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, q_weight, k_weight, input_rms_weight, q_rms_weight, k_rms_weight, cos, sin, k_cache,
                  v_cache, q_out);
  G4_REQUIRE_SCALARS(ctx, q_weight_scale, k_weight_scale, kv_offset, rope_offset);
  const uint8_t* w[3] = {q_weight, k_weight, nullptr};
  const uint8_t* bs[3] = {nullptr, nullptr, nullptr};
  const uint16_t* rs[3] = {q_weight_scale, k_weight_scale, nullptr};
  const float* gs[3] = {nullptr, nullptr, nullptr};
  return launch_qkv(ctx, true, false, x, w, bs, rs, gs, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset,
                    rope_offset, cos, sin, k_cache, v_cache, q_out, 0);
}

g4_status g4_full_project_qkv_nvfp4(g4_ctx* ctx, const g4_bf16* x, const g4_f4x2* q_weight, const g4_f4x2* k_weight,
                                    const g4_f8e4m3* q_block_scale, const g4_f8e4m3* k_block_scale,
                                    const float* q_global_scale, const float* k_global_scale,
                                    const g4_bf16* input_rms_weight, const g4_bf16* q_rms_weight,
                                    const g4_bf16* k_rms_weight, const int32_t* kv_offset, const int32_t* rope_offset,
                                    const g4_bf16* cos, const g4_bf16* sin, g4_bf16* k_cache, g4_bf16* v_cache,
                                    g4_bf16* q_out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, q_weight, k_weight, q_block_scale, k_block_scale, input_rms_weight, q_rms_weight,
                  k_rms_weight, cos, sin, k_cache, v_cache, q_out);
  G4_REQUIRE_SCALARS(ctx, q_global_scale, k_global_scale, kv_offset, rope_offset);
  const uint8_t* w[3] = {q_weight, k_weight, nullptr};
  const uint8_t* bs[3] = {q_block_scale, k_block_scale, nullptr};
  const uint16_t* rs[3] = {nullptr, nullptr, nullptr};
  const float* gs[3] = {q_global_scale, k_global_scale, nullptr};
  return launch_qkv(ctx, true, true, x, w, bs, rs, gs, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset,
                    rope_offset, cos, sin, k_cache, v_cache, q_out, 0);
}

g4_status g4_attention_gqa(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k, const g4_bf16* v, const float* mask,
                           int n_rows, g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, q, k, v, mask, out);
  if (n_rows < 64 || n_rows > G4_E || n_rows % 64 != 0)
    return fail(ctx, G4_ERR_BAD_ARG, "n_rows must be a multiple of 64 in [64, 32768]");
  return launch_gqa_attention(ctx, q, k, v, mask, n_rows, out);
}

g4_status g4_sliding_attention(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k, const g4_bf16* v, const float* mask,
                               g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, q, k, v, mask, out);
  return launch_sliding_attention(ctx, q, k, v, mask, out);
}

g4_status g4_sliding_attention_output(g4_ctx* ctx, const g4_bf16* x, const g4_bf16* post_attn_rms_weight,
                                      const g4_f8e4m3* o_weight, const g4_bf16* o_weight_scale,
                                      g4_bf16* residual) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, post_attn_rms_weight, o_weight, o_weight_scale, residual);
  return launch_oproj(ctx, false, false, x, nullptr, post_attn_rms_weight, o_weight, nullptr, o_weight_scale, nullptr,
                      residual);
}

g4_status g4_sliding_attention_output_nvfp4(g4_ctx* ctx, const g4_bf16* x, const g4_bf16* post_attn_rms_weight,
                                            const g4_f4x2* o_weight, const g4_f8e4m3* o_block_scale,
                                            const float* o_global_scale, g4_bf16* residual) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, post_attn_rms_weight, o_weight, o_block_scale, residual);
  G4_REQUIRE_SCALARS(ctx, o_global_scale);
  return launch_oproj(ctx, false, true, x, nullptr, post_attn_rms_weight, o_weight, o_block_scale, nullptr,
                      o_global_scale, residual);
}

g4_status g4_full_attention_output_nvfp4(g4_ctx* ctx, const g4_bf16* x, const float* running_sum,
                                         const g4_bf16* post_attn_rms_weight, const g4_f4x2* o_weight,
                                         const g4_f8e4m3* o_block_scale, const float* o_global_scale,
                                         g4_bf16* residual) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, post_attn_rms_weight, o_weight, o_block_scale, residual);
  G4_REQUIRE_SCALARS(ctx, running_sum, o_global_scale);
  return launch_oproj(ctx, true, true, x, running_sum, post_attn_rms_weight, o_weight, o_block_scale, nullptr,
                      o_global_scale, residual);
}

g4_status g4_full_attention_first_page(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k, const g4_bf16* v,
                                       const float* mask, float* running_max, float* running_sum, g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, q, k, v, mask, out);
  G4_REQUIRE_SCALARS(ctx, running_max, running_sum);
  return launch_full_page(ctx, true, q, k, v, mask, running_max, running_sum, out);
}

g4_status g4_full_attention_page(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* k, const g4_bf16* v, const float* mask,
                                 float* running_max, float* running_sum, g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, q, k, v, mask, out);
  G4_REQUIRE_SCALARS(ctx, running_max, running_sum);
  return launch_full_page(ctx, false, q, k, v, mask, running_max, running_sum, out);
}

g4_status g4_full_attention_paged(g4_ctx* ctx, const g4_bf16* q, const g4_bf16* const* k_pages,
                                  const g4_bf16* const* v_pages, int n_pages, int last_row, float* running_sum,
                                  g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, q, out);
  G4_REQUIRE_SCALARS(ctx, k_pages, v_pages, running_sum);
  if (n_pages < 1 || n_pages > G4_E / G4_TF || last_row < 0 || last_row >= G4_TF)
    return fail(ctx, G4_ERR_BAD_ARG, "n_pages must be in [1, 64] and last_row in [0, 511]");
  return launch_full_paged(ctx, q, k_pages, v_pages, n_pages, last_row, running_sum, out);
}

g4_status g4_full_attention_output(g4_ctx* ctx, const g4_bf16* x, const float* running_sum,
                                   const g4_bf16* post_attn_rms_weight, const g4_f8e4m3* o_weight,
                                   const g4_bf16* o_weight_scale, g4_bf16* residual) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, x, post_attn_rms_weight, o_weight, o_weight_scale, residual);
  G4_REQUIRE_SCALARS(ctx, running_sum);
  return launch_oproj(ctx, true, false, x, running_sum, post_attn_rms_weight, o_weight, nullptr, o_weight_scale,
                      nullptr, residual);
}

g4_status g4_decoder_feedforward(g4_ctx* ctx, g4_bf16* residual, const g4_bf16* pre_ff_rms_weight,
                                 const g4_f4x2* up_weight_packed, const g4_f4x2* gate_weight_packed,
                                 const g4_f4x2* down_weight_packed, const g4_f8e4m3* up_weight_scale,
                                 const g4_f8e4m3* gate_weight_scale, const g4_f8e4m3* down_weight_scale,
                                 const float* up_global_scale, const float* gate_global_scale,
                                 const float* down_global_scale, const g4_bf16* post_ff_rms_weight,
                                 const g4_bf16* layer_scalar) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed, down_weight_packed,
                  up_weight_scale, gate_weight_scale, down_weight_scale, post_ff_rms_weight, layer_scalar);
  G4_REQUIRE_SCALARS(ctx, up_global_scale, gate_global_scale, down_global_scale);
  return launch_decoder_feedforward(ctx, residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                                    down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
                                    up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight,
                                    layer_scalar);
}

g4_status g4_decoder_feedforward_prefill(g4_ctx* ctx, int n_tokens, g4_bf16* residual,
                                         const g4_bf16* pre_ff_rms_weight, const g4_f4x2* up_weight_packed,
                                         const g4_f4x2* gate_weight_packed, const g4_f4x2* down_weight_packed,
                                         const g4_f8e4m3* up_weight_scale, const g4_f8e4m3* gate_weight_scale,
                                         const g4_f8e4m3* down_weight_scale, const float* up_global_scale,
                                         const float* gate_global_scale, const float* down_global_scale,
                                         const g4_bf16* post_ff_rms_weight, const g4_bf16* layer_scalar) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed, down_weight_packed,
                  up_weight_scale, gate_weight_scale, down_weight_scale, post_ff_rms_weight, layer_scalar);
  G4_REQUIRE_SCALARS(ctx, up_global_scale, gate_global_scale, down_global_scale);
  if (n_tokens <= 0 || n_tokens > G4_PREFILL_MAX_TOKENS)
    return fail(ctx, G4_ERR_BAD_ARG, "n_tokens must be in [1, G4_PREFILL_MAX_TOKENS]");
  return launch_prefill_feedforward(ctx, n_tokens, residual, pre_ff_rms_weight, up_weight_packed,
                                    gate_weight_packed, down_weight_packed, up_weight_scale, gate_weight_scale,
                                    down_weight_scale, up_global_scale, gate_global_scale, down_global_scale,
                                    post_ff_rms_weight, layer_scalar);
}

g4_status g4_final_norm_and_logits(g4_ctx* ctx, const g4_bf16* input, const g4_bf16* rms_weight,
                                   const g4_bf16* lm_head_weight, g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, input, rms_weight, lm_head_weight, out);
  return launch_lm_head(ctx, input, rms_weight, lm_head_weight, out);
}

g4_status g4_sample_top_k_top_p(g4_ctx* ctx, const g4_bf16* logits, int n, float temperature, int top_k,
                                float top_p, const int32_t* banned, int n_banned, const float* uniform,
                                int32_t* out_index) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, logits);
  G4_REQUIRE_SCALARS(ctx, uniform, out_index);
  if (n <= 0 || n > 262144) return fail(ctx, G4_ERR_BAD_ARG, "n must be in [1, 262144]");
  if (top_k < 1 || n_banned < 0 || top_k + n_banned > 128)
    return fail(ctx, G4_ERR_BAD_ARG, "need top_k >= 1 and top_k + n_banned <= 128");
  if (n_banned > 0 && banned == nullptr) return fail(ctx, G4_ERR_BAD_ARG, "banned is null");
  if (!(top_p > 0.f) || !(top_p <= 1.f)) return fail(ctx, G4_ERR_BAD_ARG, "top_p must be in (0, 1]");
  if (!(temperature >= 0.f) || !std::isfinite(temperature)) return fail(ctx, G4_ERR_BAD_ARG, "bad temperature");
  return launch_sample(ctx, logits, n, temperature, top_k, top_p, banned, n_banned, uniform, out_index);
}

g4_status g4_argmax_bf16(g4_ctx* ctx, const g4_bf16* logits, int n, int32_t* out_index) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, logits);
  G4_REQUIRE_SCALARS(ctx, out_index);
  if (n <= 0) return fail(ctx, G4_ERR_BAD_ARG, "n must be positive");
  return launch_argmax(ctx, logits, n, out_index);
}

g4_status g4_dequant_nvfp4(g4_ctx* ctx, const g4_f4x2* packed, const g4_f8e4m3* block_scale, int rows, int cols,
                           g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, packed, block_scale, out);
  if (rows <= 0 || cols <= 0 || cols % 16 != 0) return fail(ctx, G4_ERR_BAD_ARG, "cols must be a positive multiple of 16");
  return launch_dequant_nvfp4(ctx, packed, block_scale, rows, cols, out);
}

g4_status g4_dequant_fp8(g4_ctx* ctx, const g4_f8e4m3* weight, int64_t count, g4_bf16* out) {
  G4_CHECK_CTX(ctx);
  G4_REQUIRE_PTRS(ctx, weight, out);
  if (count <= 0) return fail(ctx, G4_ERR_BAD_ARG, "count must be positive");
  return launch_dequant_fp8(ctx, weight, count, out);
}

}  // extern "C"
