// GGUF loading for libl3g: l3g_model_load_gguf() maps the file, parses it
// like internal/gguf/gguf.go and reads the hyperparameters like
// readHyperParams (internal/llama/model.go:168-219), then hands the tensor
// views to l3g_model_load().
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "l3g.h"
#include "l3g_internal.h"

namespace {

// value types, gguf.go:25-39
enum : uint32_t {
  T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64
};

struct Value {
  uint32_t type = 0;
  uint64_t u = 0;  // unsigned scalars
  double f = 0;    // floating scalars
  std::string s;
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
};

struct Cursor {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  bool need(size_t k) {
    if (!ok || pos + k > n) ok = false;
    return ok;
  }
  template <typename T>
  T get() {
    T v{};
    if (need(sizeof(T))) {
      std::memcpy(&v, p + pos, sizeof(T));
      pos += sizeof(T);
    }
    return v;
  }
  // readString, gguf.go:247-260
  std::string str() {
    const uint64_t len = get<uint64_t>();
    if (len > (1ull << 30)) ok = false;
    if (!need(len)) return {};
    std::string s(reinterpret_cast<const char*>(p + pos), len);
    pos += len;
    return s;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case T_U8: case T_I8: case T_BOOL: return 1;
    case T_U16: case T_I16: return 2;
    case T_U32: case T_I32: case T_F32: return 4;
    case T_U64: case T_I64: case T_F64: return 8;
    default: return 0;
  }
}

// readValue, gguf.go:262-380 (arrays are skipped: no hyperparameter is one)
bool read_value(Cursor& c, uint32_t t, Value& v) {
  v.type = t;
  switch (t) {
    case T_U8: v.u = c.get<uint8_t>(); break;
    case T_I8: v.u = (uint64_t)(int64_t)c.get<int8_t>(); break;
    case T_U16: v.u = c.get<uint16_t>(); break;
    case T_I16: v.u = (uint64_t)(int64_t)c.get<int16_t>(); break;
    case T_U32: v.u = c.get<uint32_t>(); break;
    case T_I32: v.u = (uint64_t)(int64_t)c.get<int32_t>(); break;
    case T_U64: v.u = c.get<uint64_t>(); break;
    case T_I64: v.u = (uint64_t)c.get<int64_t>(); break;
    case T_F32: v.f = c.get<float>(); break;
    case T_F64: v.f = c.get<double>(); break;
    case T_BOOL: v.u = c.get<uint8_t>() != 0; break;
    case T_STR: v.s = c.str(); break;
    case T_ARR: {
      const uint32_t et = c.get<uint32_t>();
      const uint64_t n = c.get<uint64_t>();
      if (n > (1ull << 28)) return false;  // gguf.go:311-313
      if (et == T_STR) {
        for (uint64_t i = 0; i < n && c.ok; ++i) c.str();
      } else if (size_t sz = scalar_size(et)) {
        if (!c.need(sz * n)) return false;
        c.pos += sz * n;
      } else {
        Value tmp;
        for (uint64_t i = 0; i < n && c.ok; ++i)
          if (!read_value(c, et, tmp)) return false;
      }
      break;
    }
    default:
      return false;
  }
  return c.ok;
}

size_t tensor_bytes(uint32_t type, const std::vector<uint64_t>& dims) {
  uint64_t n = 1;
  for (uint64_t d : dims) n *= d;
  switch (type) {
    case L3G_TYPE_F32: return n * 4;
    case L3G_TYPE_F16: return n * 2;
    case L3G_TYPE_Q8_0: return dims.empty() || dims[0] % 32 ? 0 : n / 32 * 34;
    default: return 0;
  }
}

}  // namespace

extern "C" int l3g_model_load_gguf(const char* path, const l3g_options* opt, l3g_model** out) {
  if (!path || !out) return l3g_fail(L3G_E_INVALID, "null argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return l3g_fail(L3G_E_FORMAT, "open %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    close(fd);
    return l3g_fail(L3G_E_FORMAT, "not a gguf file (too short)");
  }
  const size_t size = (size_t)st.st_size;
  void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return l3g_fail(L3G_E_FORMAT, "mmap %s: %s", path, strerror(errno));
  const uint8_t* base = static_cast<const uint8_t*>(map);
  int rc = L3G_OK;
  do {
    Cursor c{base, size};
    if (std::memcmp(base, "GGUF", 4) != 0) {  // gguf.go:68-74
      rc = l3g_fail(L3G_E_FORMAT, "not a gguf file (magic=\"%.4s\")", (const char*)base);
      break;
    }
    c.pos = 4;
    c.get<uint32_t>();  // version
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    std::map<std::string, Value> kv;
    uint32_t alignment = 32;  // gguf.go:178
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
      std::string key = c.str();
      const uint32_t t = c.get<uint32_t>();
      Value v;
      if (!read_value(c, t, v)) {
        rc = l3g_fail(L3G_E_FORMAT, "read kv \"%s\": unsupported or truncated value", key.c_str());
        break;
      }
      if (key == "general.alignment" && t == T_U32) alignment = (uint32_t)v.u;  // :192-196
      kv[key] = v;
    }
    if (rc) break;
    std::vector<TensorInfo> tis;
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
      TensorInfo ti;
      ti.name = c.str();
      const uint32_t nd = c.get<uint32_t>();
      if (nd > 4) c.ok = false;
      for (uint32_t d = 0; d < nd && c.ok; ++d) ti.dims.push_back(c.get<uint64_t>());
      ti.type = c.get<uint32_t>();
      ti.offset = c.get<uint64_t>();
      tis.push_back(ti);
    }
    if (!c.ok) {
      rc = l3g_fail(L3G_E_FORMAT, "truncated gguf header");
      break;
    }
    size_t data_off = c.pos;  // computeDataOffset, gguf.go:225-233
    if (alignment > 0 && data_off % alignment) data_off += alignment - data_off % alignment;

    // GetU32 (gguf.go:391-405): UINT32, or UINT64 that fits
    auto get_u32 = [&](const char* k, int32_t* dst) {
      auto it = kv.find(k);
      if (it == kv.end()) return false;
      if (it->second.type == T_U32 || (it->second.type == T_U64 && it->second.u <= 0xffffffffull)) {
        *dst = (int32_t)it->second.u;
        return true;
      }
      return false;
    };
    // GetF32 (gguf.go:425-432): FLOAT32 only
    auto get_f32 = [&](const char* k, float* dst) {
      auto it = kv.find(k);
      if (it == kv.end() || it->second.type != T_F32) return false;
      *dst = (float)it->second.f;
      return true;
    };
    l3g_hparams hp{};
    get_u32("llama.vocab_size", &hp.vocab_size);
    get_u32("llama.block_count", &hp.n_layers);
    get_u32("llama.embedding_length", &hp.n_emb);
    get_u32("llama.feed_forward_length", &hp.n_ff);
    get_u32("llama.attention.head_count", &hp.n_heads);
    get_u32("llama.attention.head_count_kv", &hp.n_heads_kv);
    if (!get_f32("llama.norm_rms_eps", &hp.rms_eps)) hp.rms_eps = 1e-5f;
    if (!get_f32("llama.rope.freq_base", &hp.rope_base)) hp.rope_base = 10000.0f;
    get_u32("llama.rope.dimension_count", &hp.rope_dim);
    if (!get_u32("llama.context_length", &hp.ctx_len)) hp.ctx_len = 2048;
    if (hp.vocab_size == 0 || hp.n_layers == 0 || hp.n_emb == 0 || hp.n_heads == 0 ||
        hp.n_ff == 0) {
      rc = l3g_fail(L3G_E_FORMAT, "missing required llama.* hyperparams in gguf");
      break;
    }
    if (hp.n_heads_kv == 0) hp.n_heads_kv = hp.n_heads;
    if (hp.rope_dim == 0) hp.rope_dim = hp.n_emb / hp.n_heads;

    std::vector<l3g_tensor> ts(tis.size());
    for (size_t i = 0; i < tis.size(); ++i) {
      const TensorInfo& ti = tis[i];
      const size_t nb = tensor_bytes(ti.type, ti.dims);
      const uint64_t abs = data_off + ti.offset;  // TensorAbsOffset, gguf.go:484-486
      if (abs > size) {  // reader.go:27-30
        rc = l3g_fail(L3G_E_FORMAT, "tensor \"%s\" offset out of range", ti.name.c_str());
        break;
      }
      if (nb && abs + nb > size) {
        rc = l3g_fail(L3G_E_FORMAT, "tensor \"%s\" truncated", ti.name.c_str());
        break;
      }
      l3g_tensor& t = ts[i];
      t.name = ti.name.c_str();
      t.type = ti.type;
      t.n_dims = (uint32_t)ti.dims.size();
      for (size_t d = 0; d < ti.dims.size(); ++d) t.dims[d] = ti.dims[d];
      t.data = base + abs;
      t.nbytes = nb;
    }
    if (rc) break;
    rc = l3g_model_load(&hp, ts.data(), (int32_t)ts.size(), opt, out);
  } while (false);
  munmap(map, size);
  return rc;
}
