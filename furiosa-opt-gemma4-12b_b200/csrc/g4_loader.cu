// Checkpoint loader: the text decoder's tensors of a safetensors file into a g4_model,
// cut for this context's tensor-parallel rank (src/host/load.rs:89-386 on one chip).
//
// The file is memory-mapped; its JSON header gives each tensor's dtype, shape and byte
// range.  Every tensor the decoder needs is checked against the dtype and shape the
// reference loader demands (load_bf16 / load_f8 / load_f4 / load_bf16_column /
// read_f32, load.rs:89-191) and then copied to the device in the format the kernels
// take: the NVFP4 global scale as its reciprocal (load.rs:171-191, rejecting 0 and
// non-finite values), the layer scalar replicated to [8] (load.rs:99-111), FP8 row
// scales [N, 1] as [N].  Under tensor parallelism rows (column-parallel q/k/v, gate/up)
// or columns (row-parallel o-proj, down, with their block scales) of the rank are
// copied with one 2-D copy; the full layers' single K head and the embedding table are
// copied whole.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "g4_internal.h"

namespace {

struct StInfo {
  std::string dtype;
  std::vector<uint64_t> shape;
  uint64_t begin = 0, end = 0;
};

// Minimal JSON reader for a safetensors header: an object whose members are either
// tensor records {"dtype": str, "shape": [int], "data_offsets": [int, int]} or the
// "__metadata__" object of strings (skipped).
struct Json {
  const char* p;
  const char* e;
  std::string err;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return fail("expected a string");
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return fail("bad escape");
        const char c = *p;
        out.push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c);
        ++p;
        continue;
      }
      out.push_back(*p++);
    }
    if (p >= e) return fail("unterminated string");
    ++p;
    return true;
  }
  bool num(uint64_t& v) {
    ws();
    if (p >= e || *p < '0' || *p > '9') return fail("expected an unsigned integer");
    v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      if (v > (UINT64_MAX - 9) / 10) return fail("integer overflow");
      v = v * 10 + static_cast<uint64_t>(*p++ - '0');
    }
    return true;
  }
  bool ints(std::vector<uint64_t>& out) {
    out.clear();
    if (!lit('[')) return fail("expected '['");
    if (lit(']')) return true;
    do {
      uint64_t v;
      if (!num(v)) return false;
      out.push_back(v);
    } while (lit(','));
    return lit(']') || fail("expected ']'");
  }
  bool skip_value() {  // strings, numbers, nested objects/arrays of them
    ws();
    if (p >= e) return fail("unexpected end");
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      ++p;
      if (lit(close)) return true;
      do {
        if (open == '{') {
          std::string k;
          if (!str(k) || !lit(':')) return fail("bad object");
        }
        if (!skip_value()) return false;
      } while (lit(','));
      return lit(close) || fail("unterminated container");
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
    return true;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  bool header(std::map<std::string, StInfo>& out) {
    if (!lit('{')) return fail("header is not an object");
    if (lit('}')) return true;
    do {
      std::string name;
      if (!str(name) || !lit(':')) return fail("bad member");
      if (name == "__metadata__") {
        if (!skip_value()) return false;
        continue;
      }
      StInfo t;
      if (!lit('{')) return fail("tensor record is not an object");
      if (!lit('}')) {
        do {
          std::string k;
          if (!str(k) || !lit(':')) return fail("bad tensor record");
          if (k == "dtype") {
            if (!str(t.dtype)) return false;
          } else if (k == "shape") {
            if (!ints(t.shape)) return false;
          } else if (k == "data_offsets") {
            std::vector<uint64_t> o;
            if (!ints(o)) return false;
            if (o.size() != 2 || o[1] < o[0]) return fail("bad data_offsets");
            t.begin = o[0];
            t.end = o[1];
          } else if (!skip_value()) {
            return false;
          }
        } while (lit(','));
        if (!lit('}')) return fail("unterminated tensor record");
      }
      out[name] = t;
    } while (lit(','));
    return lit('}') || fail("unterminated header");
  }
};

uint64_t dtype_size(const std::string& d) {
  if (d == "U8" || d == "I8" || d == "F8_E4M3" || d == "F8_E5M2" || d == "BOOL") return 1;
  if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  return 0;
}

// How one tensor is cut for a rank and converted.
enum class Cut { Whole, Rows, Cols };
enum class Conv { None, Reciprocal, Replicate8 };
struct Need {
  std::string name;
  std::string dtype;
  std::vector<uint64_t> shape;  // as stored in the checkpoint
  Cut cut;
  Conv conv;
};

struct File {
  int fd = -1;
  void* map = nullptr;
  size_t size = 0;
  const uint8_t* data = nullptr;  // start of the tensor data
  uint64_t data_size = 0;
  std::map<std::string, StInfo> tensors;
  ~File() {
    if (map != nullptr && map != MAP_FAILED) munmap(map, size);
    if (fd >= 0) close(fd);
  }
};

bool open_file(File& f, const char* path, std::string& err) {
  f.fd = open(path, O_RDONLY);
  if (f.fd < 0) {
    err = std::string(path) + ": cannot open";
    return false;
  }
  struct stat sb;
  if (fstat(f.fd, &sb) != 0 || sb.st_size < 8) {
    err = std::string(path) + ": not a safetensors file (too short)";
    return false;
  }
  f.size = static_cast<size_t>(sb.st_size);
  f.map = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
  if (f.map == MAP_FAILED) {
    err = std::string(path) + ": mmap failed";
    return false;
  }
  const uint8_t* b = static_cast<const uint8_t*>(f.map);
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | b[i];
  if (hlen > f.size - 8 || hlen > (100ull << 20)) {
    err = std::string(path) + ": header length out of range";
    return false;
  }
  Json j{reinterpret_cast<const char*>(b + 8), reinterpret_cast<const char*>(b + 8 + hlen), {}};
  if (!j.header(f.tensors)) {
    err = std::string(path) + ": bad header JSON (" + j.err + ")";
    return false;
  }
  f.data = b + 8 + hlen;
  f.data_size = f.size - 8 - hlen;
  for (const auto& kv : f.tensors) {
    const StInfo& t = kv.second;
    uint64_t n = dtype_size(t.dtype);
    for (uint64_t d : t.shape) n *= d;
    if (t.end > f.data_size || t.end - t.begin != n || n == 0) {
      err = kv.first + ": data_offsets do not match its dtype and shape or lie outside the file";
      return false;
    }
  }
  return true;
}

std::string shape_str(const std::vector<uint64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

// The tensors of an n-layer text decoder, with the dtype/shape load.rs expects.
std::vector<Need> needed(int n_layers) {
  using V = std::vector<uint64_t>;
  const uint64_t H = G4_H, L = G4_L;
  std::vector<Need> out;
  out.push_back({"model.language_model.embed_tokens.weight", "BF16", V{G4_W, H}, Cut::Whole, Conv::None});
  out.push_back({"model.language_model.norm.weight", "BF16", V{H}, Cut::Whole, Conv::None});
  for (int i = 0; i < n_layers; ++i) {
    const std::string p = "model.language_model.layers." + std::to_string(i) + ".";
    const bool full = i % 6 == 5;
    const uint64_t q = full ? G4_QF : G4_QS, k = full ? G4_PF : G4_PS, d = full ? G4_DF : G4_DS;
    for (const char* nm : {"input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                           "post_feedforward_layernorm"})
      out.push_back({p + nm + ".weight", "BF16", V{H}, Cut::Whole, Conv::None});
    out.push_back({p + "layer_scalar", "BF16", V{1}, Cut::Whole, Conv::Replicate8});
    out.push_back({p + "self_attn.q_proj.weight", "F8_E4M3", V{q, H}, Cut::Rows, Conv::None});
    out.push_back({p + "self_attn.q_proj.weight_scale", "BF16", V{q, 1}, Cut::Rows, Conv::None});
    const Cut kc = full ? Cut::Whole : Cut::Rows;  // the MQA head is replicated
    out.push_back({p + "self_attn.k_proj.weight", "F8_E4M3", V{k, H}, kc, Conv::None});
    out.push_back({p + "self_attn.k_proj.weight_scale", "BF16", V{k, 1}, kc, Conv::None});
    if (!full) {
      out.push_back({p + "self_attn.v_proj.weight", "F8_E4M3", V{k, H}, Cut::Rows, Conv::None});
      out.push_back({p + "self_attn.v_proj.weight_scale", "BF16", V{k, 1}, Cut::Rows, Conv::None});
    }
    out.push_back({p + "self_attn.o_proj.weight", "F8_E4M3", V{H, q}, Cut::Cols, Conv::None});
    out.push_back({p + "self_attn.o_proj.weight_scale", "BF16", V{H, 1}, Cut::Whole, Conv::None});
    out.push_back({p + "self_attn.q_norm.weight", "BF16", V{d}, Cut::Whole, Conv::None});
    out.push_back({p + "self_attn.k_norm.weight", "BF16", V{d}, Cut::Whole, Conv::None});
    for (const char* nm : {"up_proj", "gate_proj"}) {
      out.push_back({p + "mlp." + nm + ".weight_packed", "U8", V{L, H / 2}, Cut::Rows, Conv::None});
      out.push_back({p + "mlp." + nm + ".weight_scale", "F8_E4M3", V{L, H / 16}, Cut::Rows, Conv::None});
      out.push_back({p + "mlp." + nm + ".weight_global_scale", "F32", V{}, Cut::Whole, Conv::Reciprocal});
    }
    out.push_back({p + "mlp.down_proj.weight_packed", "U8", V{H, L / 2}, Cut::Cols, Conv::None});
    out.push_back({p + "mlp.down_proj.weight_scale", "F8_E4M3", V{H, L / 16}, Cut::Cols, Conv::None});
    out.push_back({p + "mlp.down_proj.weight_global_scale", "F32", V{}, Cut::Whole, Conv::Reciprocal});
  }
  return out;
}

uint64_t numel(const std::vector<uint64_t>& s) {
  uint64_t n = 1;
  for (uint64_t d : s) n *= d;
  return n;
}

// Checks every needed tensor's presence, dtype and shape (a scalar f32 may be [] or [1],
// as read_f32 only checks it holds 4 bytes, load.rs:163-169).
bool check_all(const File& f, const std::vector<Need>& need, int world, std::string& err) {
  for (const Need& n : need) {
    auto it = f.tensors.find(n.name);
    if (it == f.tensors.end()) {
      err = n.name + ": missing from the checkpoint";
      return false;
    }
    const StInfo& t = it->second;
    const bool scalar = n.conv == Conv::Reciprocal;
    const bool shape_ok = scalar ? (numel(t.shape) == 1) : (t.shape == n.shape);
    if (t.dtype != n.dtype || !shape_ok) {
      err = n.name + " is " + t.dtype + " " + shape_str(t.shape) + ", expected " + n.dtype + " " +
            (scalar ? std::string("scalar") : shape_str(n.shape));
      return false;
    }
    if ((n.cut == Cut::Rows && n.shape[0] % world) || (n.cut == Cut::Cols && n.shape[1] % world)) {
      err = n.name + ": cannot be cut for tensor-parallel world " + std::to_string(world);
      return false;
    }
    if (n.conv == Conv::Reciprocal) {
      float v;
      std::memcpy(&v, f.data + t.begin, 4);
      if (v == 0.0f || !std::isfinite(v)) {  // load.rs:171-181
        err = "invalid NVFP4 global scale " + n.name + ": " + std::to_string(v);
        return false;
      }
    }
  }
  return true;
}

}  // namespace

extern "C" {

g4_status g4_checkpoint_check(const char* path, int n_layers, int world, char* msg, uint64_t msg_len) {
  std::string err;
  g4_status st = G4_OK;
  if (path == nullptr || n_layers < 1 || n_layers > G4_LAYERS || !(world == 1 || world == 2 || world == 4 || world == 8)) {
    err = "bad arguments";
    st = G4_ERR_BAD_ARG;
  } else {
    File f;
    if (!open_file(f, path, err) || !check_all(f, needed(n_layers), world, err)) st = G4_ERR_BAD_ARG;
  }
  if (msg != nullptr && msg_len > 0) {
    std::snprintf(msg, static_cast<size_t>(msg_len), "%s", err.c_str());
  }
  return st;
}

g4_status g4_model_load_safetensors(g4_ctx* ctx, const char* path, int n_layers, g4_model** out) {
  if (ctx == nullptr || path == nullptr || out == nullptr) return G4_ERR_BAD_ARG;
  *out = nullptr;
  if (n_layers < 1 || n_layers > G4_LAYERS) return g4::fail(ctx, G4_ERR_BAD_ARG, "n_layers must be in [1, 48]");
  const int world = ctx->tp_world, rank = ctx->tp_rank;
  std::string err;
  File f;
  const std::vector<Need> need = needed(n_layers);
  if (!open_file(f, path, err) || !check_all(f, need, world, err)) return g4::fail(ctx, G4_ERR_BAD_ARG, err);
  g4_status st = g4::check_cuda(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  if (st != G4_OK) return st;
  g4_model* m = nullptr;
  if ((st = g4_model_create(n_layers, &m)) != G4_OK) return st;
  std::vector<void*> owned;
  auto done = [&](g4_status s) {
    g4::model_adopt(m, owned, ctx->device);
    if (s != G4_OK) {
      g4_model_destroy(m);
      return s;
    }
    *out = m;
    return G4_OK;
  };
  for (const Need& n : need) {
    const StInfo& t = f.tensors.at(n.name);
    const uint8_t* src = f.data + t.begin;
    const uint64_t es = dtype_size(t.dtype);
    uint64_t bytes = t.end - t.begin;
    std::vector<uint8_t> host;  // converted copies
    if (n.conv == Conv::Reciprocal) {
      float v;
      std::memcpy(&v, src, 4);
      v = 1.0f / v;
      host.resize(4);
      std::memcpy(host.data(), &v, 4);
      src = host.data();
      bytes = 4;
    } else if (n.conv == Conv::Replicate8) {
      host.resize(16);
      for (int i = 0; i < 8; ++i) std::memcpy(host.data() + 2 * i, src, 2);
      src = host.data();
      bytes = 16;
    }
    uint64_t rows = 1, row_bytes = bytes;
    if (n.cut == Cut::Rows) {
      rows = n.shape[0] / world;
      row_bytes = bytes / n.shape[0];
      src += static_cast<uint64_t>(rank) * rows * row_bytes;
      bytes = rows * row_bytes;
    }
    void* dst = nullptr;
    if (n.cut == Cut::Cols) {
      const uint64_t full_pitch = n.shape[1] * es, part = full_pitch / world;
      bytes = n.shape[0] * part;
      st = g4::check_cuda(ctx, cudaMalloc(&dst, bytes), "cudaMalloc (checkpoint tensor)");
      if (st != G4_OK) return done(st);
      owned.push_back(dst);
      st = g4::check_cuda(ctx,
                          cudaMemcpy2D(dst, part, src + static_cast<uint64_t>(rank) * part, full_pitch, part,
                                       n.shape[0], cudaMemcpyHostToDevice),
                          "cudaMemcpy2D (checkpoint tensor)");
    } else {
      st = g4::check_cuda(ctx, cudaMalloc(&dst, bytes), "cudaMalloc (checkpoint tensor)");
      if (st != G4_OK) return done(st);
      owned.push_back(dst);
      st = g4::check_cuda(ctx, cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "cudaMemcpy (checkpoint tensor)");
    }
    if (st != G4_OK) return done(st);
    if ((st = g4_model_set_tensor(m, n.name.c_str(), dst, bytes)) != G4_OK)
      return done(g4::fail(ctx, st, g4_model_last_error(m)));
  }
  return done(G4_OK);
}

}  // extern "C"
