// gsv_file.cpp — the GSV1 weight container (GPT-SoVITS-native
// src/runtime/gsv_loader.hpp:50-114; format per tools/convert.py:3-28) read
// on the host and registered with the device engines.
//
// Layout, all little-endian: magic "GSV1", u32 version (1), u32 flags (bit 0:
// fp16 segments present), u16 + utf8 model name, u32 + utf8 config JSON, u32
// tensor count, then per tensor: u16 + utf8 name, u16 rank + rank x u32
// dims, u16 source dtype (1 fp32, 2 fp16), u64 fp32 offset, u64 fp32 bytes,
// u64 fp16 offset, u64 fp16 bytes (0 = no fp16 copy).  Data blocks start on
// 64-byte boundaries.  The file is mapped read-only; tensor pointers stay
// valid until gsvk_gsv_close.
//
// Validation follows the reference loader: magic / version / truncation of
// the header, per entry a rank <= 8, a known dtype, segment sizes that match
// the shape (an fp16-only "slim" tensor may omit its fp32 copy), 64-byte
// aligned in-bounds segments, an element count below 2^40, and flag bit 0
// equal to whether any fp16 segment exists.  A bad file fails with
// GSVK_ERR_INVALID and a message naming the entry.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "gsvk_internal.hpp"

struct gsvk_gsv {
  int fd = -1;
  void* map = nullptr;
  uint64_t size = 0;
  uint32_t flags = 0;
  std::string name, config;
  struct Entry {
    std::string name;
    uint32_t rank = 0;
    uint32_t dims[8] = {};
    int dtype = 1;
    uint64_t numel = 0;
    uint64_t f32_off = 0, f32_bytes = 0, f16_off = 0, f16_bytes = 0;
  };
  std::vector<Entry> entries;
};

using namespace gsvk;

namespace {

constexpr uint64_t kAlign = 64;
constexpr uint64_t kMaxNumel = 1ull << 40;

template <typename T>
T rd(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof v);
  return v;
}

void close_file(gsvk_gsv* f) {
  if (f->map) munmap(f->map, f->size);
  if (f->fd >= 0) ::close(f->fd);
  f->map = nullptr;
  f->fd = -1;
}

// Parses the mapped bytes; returns GSVK_OK or GSVK_ERR_INVALID with a message.
int parse(gsvk_gsv* f) {
  const uint8_t* base = static_cast<const uint8_t*>(f->map);
  const uint8_t* p = base;
  const uint8_t* const end = base + f->size;
  auto left = [&] { return static_cast<uint64_t>(end - p); };
  if (f->size < 12 || std::memcmp(base, "GSV1", 4) != 0)
    return fail(GSVK_ERR_INVALID, "gsv: magic is not GSV1");
  if (rd<uint32_t>(base + 4) != 1)
    return fail(GSVK_ERR_INVALID, "gsv: unsupported version %u", rd<uint32_t>(base + 4));
  f->flags = rd<uint32_t>(base + 8);
  p = base + 12;
  if (left() < 2) return fail(GSVK_ERR_INVALID, "gsv: header truncated (name length)");
  const uint16_t name_len = rd<uint16_t>(p);
  p += 2;
  if (left() < name_len) return fail(GSVK_ERR_INVALID, "gsv: header truncated (name)");
  f->name.assign(reinterpret_cast<const char*>(p), name_len);
  p += name_len;
  if (left() < 4) return fail(GSVK_ERR_INVALID, "gsv: header truncated (config length)");
  const uint32_t cfg_len = rd<uint32_t>(p);
  p += 4;
  if (left() < cfg_len) return fail(GSVK_ERR_INVALID, "gsv: header truncated (config)");
  f->config.assign(reinterpret_cast<const char*>(p), cfg_len);
  p += cfg_len;
  if (left() < 4) return fail(GSVK_ERR_INVALID, "gsv: header truncated (tensor count)");
  const uint32_t n = rd<uint32_t>(p);
  p += 4;
  bool any_f16 = false;
  f->entries.reserve(n < 1u << 20 ? n : 1u << 20);
  for (uint32_t i = 0; i < n; ++i) {
    gsvk_gsv::Entry e;
    if (left() < 2) return fail(GSVK_ERR_INVALID, "gsv: entry %u truncated (name length)", i);
    const uint16_t nl = rd<uint16_t>(p);
    p += 2;
    if (left() < nl) return fail(GSVK_ERR_INVALID, "gsv: entry %u truncated (name)", i);
    e.name.assign(reinterpret_cast<const char*>(p), nl);
    p += nl;
    if (left() < 2) return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) truncated (rank)", i, e.name.c_str());
    e.rank = rd<uint16_t>(p);
    p += 2;
    if (e.rank > 8) return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) rank %u > 8", i, e.name.c_str(), e.rank);
    if (left() < 4ull * e.rank)
      return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) truncated (dims)", i, e.name.c_str());
    e.numel = 1;
    for (uint32_t r = 0; r < e.rank; ++r) {
      e.dims[r] = rd<uint32_t>(p + 4 * r);
      e.numel *= e.dims[r];
      if (e.numel > kMaxNumel)
        return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) has too many elements", i, e.name.c_str());
    }
    p += 4ull * e.rank;
    if (left() < 34)
      return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) truncated (dtype/offsets)", i, e.name.c_str());
    e.dtype = rd<uint16_t>(p);
    if (e.dtype != 1 && e.dtype != 2)
      return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) unknown dtype %d", i, e.name.c_str(), e.dtype);
    e.f32_off = rd<uint64_t>(p + 2);
    e.f32_bytes = rd<uint64_t>(p + 10);
    e.f16_off = rd<uint64_t>(p + 18);
    e.f16_bytes = rd<uint64_t>(p + 26);
    p += 34;
    const bool has16 = e.f16_bytes != 0;
    if (has16 ? (e.f32_bytes != 0 && e.f32_bytes != e.numel * 4) : e.f32_bytes != e.numel * 4)
      return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) fp32 segment size does not match the shape",
                  i, e.name.c_str());
    if (has16 && e.f16_bytes != e.numel * 2)
      return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) fp16 segment size does not match the shape",
                  i, e.name.c_str());
    if (e.f32_bytes && (e.f32_off % kAlign || e.f32_off > f->size || e.f32_bytes > f->size - e.f32_off))
      return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) fp32 segment unaligned or out of the file",
                  i, e.name.c_str());
    if (has16 && (e.f16_off % kAlign || e.f16_off > f->size || e.f16_bytes > f->size - e.f16_off))
      return fail(GSVK_ERR_INVALID, "gsv: entry %u (%s) fp16 segment unaligned or out of the file",
                  i, e.name.c_str());
    any_f16 = any_f16 || has16;
    f->entries.push_back(std::move(e));
  }
  if (((f->flags & 1u) != 0) != any_f16)
    return fail(GSVK_ERR_INVALID, "gsv: flag bit 0 disagrees with the fp16 segments present");
  return GSVK_OK;
}

// --------------------------------------------------------------- tiny JSON
// Enough JSON to read numbers out of nested objects of the config (the
// reference parses it with its own mini_json, src/runtime/mini_json.hpp).
struct Json {
  const char* p;
  const char* e;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool skip_string() {
    if (p >= e || *p != '"') return false;
    for (++p; p < e; ++p) {
      if (*p == '\\') {
        ++p;
        continue;
      }
      if (*p == '"') {
        ++p;
        return true;
      }
    }
    return false;
  }
  bool skip_value(int depth = 0) {
    ws();
    if (p >= e || depth > 64) return false;
    if (*p == '"') return skip_string();
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      ++p;
      ws();
      if (p < e && *p == close) {
        ++p;
        return true;
      }
      for (;;) {
        if (close == '}') {
          ws();
          if (!skip_string()) return false;
          ws();
          if (p >= e || *p != ':') return false;
          ++p;
        }
        if (!skip_value(depth + 1)) return false;
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == close) {
          ++p;
          return true;
        }
        return false;
      }
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') ++p;
    return true;
  }
  // Positions p at the value of `key` in the object starting at p.
  bool find(const char* key) {
    ws();
    if (p >= e || *p != '{') return false;
    ++p;
    const size_t kl = std::strlen(key);
    for (;;) {
      ws();
      if (p >= e || *p != '"') return false;
      const char* k0 = p + 1;
      if (!skip_string()) return false;
      const bool hit = static_cast<size_t>(p - 1 - k0) == kl && std::memcmp(k0, key, kl) == 0;
      ws();
      if (p >= e || *p != ':') return false;
      ++p;
      ws();
      if (hit) return true;
      if (!skip_value()) return false;
      ws();
      if (p < e && *p == ',') {
        ++p;
        continue;
      }
      return false;
    }
  }
};

bool json_number(const std::string& s, const char* const* path, int depth, double* out) {
  Json j{s.data(), s.data() + s.size()};
  for (int i = 0; i < depth; ++i)
    if (!j.find(path[i])) return false;
  char buf[64];
  size_t n = 0;
  while (j.p < j.e && n < sizeof buf - 1 && std::strchr("+-0123456789.eE", *j.p)) buf[n++] = *j.p++;
  buf[n] = 0;
  if (!n) return false;
  char* endp = nullptr;
  *out = std::strtod(buf, &endp);
  return endp == buf + n;
}

const gsvk_gsv::Entry* find_entry(const gsvk_gsv* f, const char* name) {
  for (const auto& e : f->entries)
    if (e.name == name) return &e;
  return nullptr;
}

void fill(const gsvk_gsv* f, const gsvk_gsv::Entry& e, gsvk_gsv_tensor* t) {
  const uint8_t* base = static_cast<const uint8_t*>(f->map);
  t->name = e.name.c_str();
  t->rank = e.rank;
  for (int r = 0; r < 8; ++r) t->dims[r] = r < static_cast<int>(e.rank) ? e.dims[r] : 0;
  t->src_dtype = e.dtype;
  t->numel = e.numel;
  t->f32 = e.f32_bytes ? reinterpret_cast<const float*>(base + e.f32_off) : nullptr;
  t->f16 = e.f16_bytes ? reinterpret_cast<const uint16_t*>(base + e.f16_off) : nullptr;
}

}  // namespace

extern "C" {

int gsvk_gsv_open(const char* path, gsvk_gsv_t* out) {
  if (!path || !out) return fail(GSVK_ERR_INVALID, "gsv_open: null argument");
  *out = nullptr;
  auto* f = new gsvk_gsv();
  f->fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (f->fd < 0) {
    const int err = errno;
    delete f;
    return fail(GSVK_ERR_INVALID, "gsv_open: cannot open %s: %s", path, std::strerror(err));
  }
  struct stat st {};
  if (fstat(f->fd, &st) != 0 || st.st_size <= 0) {
    close_file(f);
    delete f;
    return fail(GSVK_ERR_INVALID, "gsv_open: %s is empty or cannot be read", path);
  }
  f->size = static_cast<uint64_t>(st.st_size);
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
  if (m == MAP_FAILED) {
    const int err = errno;
    close_file(f);
    delete f;
    return fail(GSVK_ERR_INVALID, "gsv_open: mmap of %s failed: %s", path, std::strerror(err));
  }
  f->map = m;
  if (int rc = parse(f)) {
    close_file(f);
    delete f;
    return rc;
  }
  *out = f;
  return GSVK_OK;
}

int gsvk_gsv_close(gsvk_gsv_t f) {
  if (!f) return GSVK_OK;
  close_file(f);
  delete f;
  return GSVK_OK;
}

size_t gsvk_gsv_count(gsvk_gsv_t f) { return f ? f->entries.size() : 0; }

const char* gsvk_gsv_model_name(gsvk_gsv_t f) { return f ? f->name.c_str() : nullptr; }

const char* gsvk_gsv_config(gsvk_gsv_t f, size_t* len) {
  if (!f) return nullptr;
  if (len) *len = f->config.size();
  return f->config.c_str();
}

int gsvk_gsv_tensor_at(gsvk_gsv_t f, size_t i, gsvk_gsv_tensor* out) {
  if (!f || !out) return fail(GSVK_ERR_INVALID, "gsv_tensor_at: null argument");
  if (i >= f->entries.size()) return fail(GSVK_ERR_INVALID, "gsv_tensor_at: index %zu >= %zu", i, f->entries.size());
  fill(f, f->entries[i], out);
  return GSVK_OK;
}

int gsvk_gsv_find(gsvk_gsv_t f, const char* name, gsvk_gsv_tensor* out) {
  if (!f || !name || !out) return fail(GSVK_ERR_INVALID, "gsv_find: null argument");
  const auto* e = find_entry(f, name);
  if (!e) return fail(GSVK_ERR_INVALID, "gsv_find: no tensor named %s", name);
  fill(f, *e, out);
  return GSVK_OK;
}

int gsvk_t2s_create_from_gsv(gsvk_gsv_t f, int cap, gsvk_t2s_t* out) {
  if (!f || !out) return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: null argument");
  *out = nullptr;
  // dimensions from the embedded checkpoint config (t2s_engine.cpp:545-563)
  static const char* const kModel[] = {"model_config", "model"};
  auto dim = [&](const char* key, double* v) {
    const char* path[] = {kModel[0], kModel[1], key};
    return json_number(f->config, path, 3, v);
  };
  double hidden, head, units, layers, vocab, emb = -1, eos = -1;
  if (!dim("hidden_dim", &hidden) || !dim("head", &head) || !dim("linear_units", &units) ||
      !dim("n_layer", &layers) || !dim("vocab_size", &vocab))
    return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: config lacks model_config.model "
                                  "hidden_dim / head / linear_units / n_layer / vocab_size");
  if (dim("embedding_dim", &emb) && emb != hidden)
    return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: embedding_dim != hidden_dim");
  if (dim("EOS", &eos) && eos != vocab - 1)
    return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: EOS != vocab_size - 1");
  const int L = static_cast<int>(layers), D = static_cast<int>(hidden), F = static_cast<int>(units),
            V = static_cast<int>(vocab);
  gsvk_t2s_config cfg{};
  cfg.n_layers = L;
  cfg.d_model = D;
  cfg.n_heads = static_cast<int>(head);
  cfg.ffn = F;
  cfg.vocab = V;
  cfg.ln_eps = 1e-5f;  // layer_norm_eps (t2s_engine.hpp:47)
  cfg.cap = cap;
  // tensors (t2s_engine.cpp:565-630): fp16 matrices, fp32 vectors; the
  // per-layer tensors are gathered into the [L][...] blocks the engine takes
  auto need = [&](const std::string& name, uint64_t numel, bool f16,
                  const gsvk_gsv::Entry** e) -> int {
    *e = find_entry(f, name.c_str());
    if (!*e) return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: missing %s", name.c_str());
    if ((*e)->numel != numel)
      return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: %s has %llu elements, expected %llu",
                  name.c_str(), (unsigned long long)(*e)->numel, (unsigned long long)numel);
    if (f16 && !(*e)->f16_bytes)
      return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: %s has no fp16 segment", name.c_str());
    if (!f16 && !(*e)->f32_bytes)
      return fail(GSVK_ERR_INVALID, "t2s_create_from_gsv: %s has no fp32 segment", name.c_str());
    return GSVK_OK;
  };
  const uint8_t* base = static_cast<const uint8_t*>(f->map);
  std::vector<uint16_t> wqkv((size_t)L * 3 * D * D), wout((size_t)L * D * D), w1((size_t)L * F * D),
      w2((size_t)L * D * F);
  std::vector<float> bqkv((size_t)L * 3 * D), bout((size_t)L * D), b1((size_t)L * F),
      b2((size_t)L * D), n1g((size_t)L * D), n1b((size_t)L * D), n2g((size_t)L * D), n2b((size_t)L * D);
  const gsvk_gsv::Entry* e = nullptr;
  auto take16 = [&](const std::string& name, uint64_t numel, uint16_t* dst) -> int {
    if (int rc = need(name, numel, true, &e)) return rc;
    std::memcpy(dst, base + e->f16_off, numel * 2);
    return GSVK_OK;
  };
  auto take32 = [&](const std::string& name, uint64_t numel, float* dst) -> int {
    if (int rc = need(name, numel, false, &e)) return rc;
    std::memcpy(dst, base + e->f32_off, numel * 4);
    return GSVK_OK;
  };
  for (int l = 0; l < L; ++l) {
    const std::string p = "h.layers." + std::to_string(l) + ".", ps = p + "self_attn.";
    int rc;
    if ((rc = take16(ps + "in_proj_weight", 3ull * D * D, &wqkv[(size_t)l * 3 * D * D])) ||
        (rc = take32(ps + "in_proj_bias", 3ull * D, &bqkv[(size_t)l * 3 * D])) ||
        (rc = take16(ps + "out_proj.weight", 1ull * D * D, &wout[(size_t)l * D * D])) ||
        (rc = take32(ps + "out_proj.bias", D, &bout[(size_t)l * D])) ||
        (rc = take16(p + "linear1.weight", 1ull * F * D, &w1[(size_t)l * F * D])) ||
        (rc = take32(p + "linear1.bias", F, &b1[(size_t)l * F])) ||
        (rc = take16(p + "linear2.weight", 1ull * D * F, &w2[(size_t)l * D * F])) ||
        (rc = take32(p + "linear2.bias", D, &b2[(size_t)l * D])) ||
        (rc = take32(p + "norm1.weight", D, &n1g[(size_t)l * D])) ||
        (rc = take32(p + "norm1.bias", D, &n1b[(size_t)l * D])) ||
        (rc = take32(p + "norm2.weight", D, &n2g[(size_t)l * D])) ||
        (rc = take32(p + "norm2.bias", D, &n2b[(size_t)l * D])))
      return rc;
  }
  const gsvk_gsv::Entry *pred = nullptr, *emb_a = nullptr, *alpha = nullptr;
  int rc;
  if ((rc = need("ar_predict_layer.weight", (uint64_t)V * D, true, &pred)) ||
      (rc = need("ar_audio_embedding.word_embeddings.weight", (uint64_t)V * D, true, &emb_a)) ||
      (rc = need("ar_audio_position.alpha", 1, false, &alpha)))
    return rc;
  cfg.alpha_audio = *reinterpret_cast<const float*>(base + alpha->f32_off);
  gsvk_t2s_host_weights w{};
  w.wqkv = wqkv.data();
  w.bqkv = bqkv.data();
  w.wout = wout.data();
  w.bout = bout.data();
  w.w1 = w1.data();
  w.b1 = b1.data();
  w.w2 = w2.data();
  w.b2 = b2.data();
  w.n1g = n1g.data();
  w.n1b = n1b.data();
  w.n2g = n2g.data();
  w.n2b = n2b.data();
  w.wpred = reinterpret_cast<const uint16_t*>(base + pred->f16_off);
  w.audio_emb = reinterpret_cast<const uint16_t*>(base + emb_a->f16_off);
  return gsvk_t2s_create(&cfg, &w, out);
}

}  // extern "C"
