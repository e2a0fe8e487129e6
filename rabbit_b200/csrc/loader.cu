// loader.cu -- checkpoint (.safetensors) -> HBM expert tables: the replacement for rabbit's
// expert streaming tier. Host code only (no kernels): shard headers are parsed once, tensors are
// read with pread straight into host staging and uploaded through the layer's own upload entry
// points, so every byte-count check of those applies as well.
//
// Reference behaviour restated here:
// * Shards::open_multi (src/safetensors.rs:248-349): every `*.safetensors` file of the given
//   directories, sorted by file name; per file an 8-byte little-endian header length (rejected
//   when larger than the file), a JSON object of `name -> {dtype, shape, data_offsets}` (the
//   `__metadata__` entry skipped), offsets relative to the end of the header and checked
//   against the file size; a name seen again later wins.
// * ExpertNaming::tensor_specs / packed_suffix (src/expert_cache.rs:66-210): the tensor names of
//   one routed expert per checkpoint convention, gate then up then down.
// * qt_load_mxfp4 + mxfp4_from_raw (src/expert_cache.rs:1232-1256): `{base}{suffix}` and
//   `{base}.weight_scale` read verbatim, lengths rows*ceil(cols/2) and rows*ceil(cols/32).
// * qt_load with a `.qs` sidecar (src/glm52/model.rs:137-156) + QT::from_packed_grouped
//   (src/quant.rs:266-275): offset-binary int4 bytes + an f32 scale per group.
#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "rmoe.h"

// The library-wide error text (rmoe_last_error) lives in api.cu.
void rmoe_set_error(const char* msg);

namespace {

rmoe_status lfail(rmoe_status s, const char* fmt, ...) {
  char buf[768];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  rmoe_set_error(buf);
  return s;
}

struct StTensor {
  std::string name;
  int file = 0;
  uint64_t offset = 0;  // absolute byte offset in its file
  uint64_t nbytes = 0;
  std::string dtype;
  std::vector<uint64_t> shape;
};

// ---- a small JSON reader for safetensors headers (objects, arrays, strings, numbers, literals)
struct Json {
  const char* p;
  const char* end;
  std::string err;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  bool expect(char c) {
    ws();
    if (p < end && *p == c) {
      p++;
      return true;
    }
    err = std::string("expected '") + c + "'";
    return false;
  }
  bool string(std::string& out) {
    ws();
    if (p >= end || *p != '"') {
      err = "expected a string";
      return false;
    }
    p++;
    out.clear();
    while (p < end && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= end) break;
        const char e = *p++;
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (end - p < 4) {
              err = "bad \\u escape";
              return false;
            }
            unsigned v = 0;
            for (int i = 0; i < 4; i++) {
              const char h = *p++;
              v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : (h | 32) - 'a' + 10);
            }
            if (v < 0x80) {
              out += static_cast<char>(v);
            } else if (v < 0x800) {
              out += static_cast<char>(0xC0 | (v >> 6));
              out += static_cast<char>(0x80 | (v & 63));
            } else {
              out += static_cast<char>(0xE0 | (v >> 12));
              out += static_cast<char>(0x80 | ((v >> 6) & 63));
              out += static_cast<char>(0x80 | (v & 63));
            }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (p >= end) {
      err = "unterminated string";
      return false;
    }
    p++;
    return true;
  }
  bool u64(uint64_t& v) {
    ws();
    if (p >= end || *p < '0' || *p > '9') {
      err = "expected an unsigned integer";
      return false;
    }
    v = 0;
    while (p < end && *p >= '0' && *p <= '9') {
      const uint64_t d = static_cast<uint64_t>(*p++ - '0');
      if (v > (UINT64_MAX - d) / 10) {
        err = "integer overflow";
        return false;
      }
      v = v * 10 + d;
    }
    if (p < end && (*p == '.' || *p == 'e' || *p == 'E' || *p == '-')) {
      err = "expected an unsigned integer";
      return false;
    }
    return true;
  }
  bool skip() {  // any value
    ws();
    if (p >= end) {
      err = "unexpected end";
      return false;
    }
    if (*p == '"') {
      std::string s;
      return string(s);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      p++;
      ws();
      if (p < end && *p == close) {
        p++;
        return true;
      }
      for (;;) {
        if (obj) {
          std::string k;
          if (!string(k) || !expect(':')) return false;
        }
        if (!skip()) return false;
        ws();
        if (p < end && *p == ',') {
          p++;
          continue;
        }
        return expect(close);
      }
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') p++;
    return true;
  }
  bool u64_array(std::vector<uint64_t>& out) {
    out.clear();
    if (!expect('[')) return false;
    ws();
    if (p < end && *p == ']') {
      p++;
      return true;
    }
    for (;;) {
      uint64_t v;
      if (!u64(v)) return false;
      out.push_back(v);
      ws();
      if (p < end && *p == ',') {
        p++;
        continue;
      }
      return expect(']');
    }
  }
};

bool read_exact_at(int fd, uint64_t off, void* dst, uint64_t n) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  while (n) {
    const ssize_t r = pread(fd, d, n > (1u << 30) ? (1u << 30) : n, static_cast<off_t>(off));
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    d += r;
    off += static_cast<uint64_t>(r);
    n -= static_cast<uint64_t>(r);
  }
  return true;
}

}  // namespace

struct rmoe_shards {
  std::vector<int> fds;
  std::vector<std::string> paths;
  std::vector<StTensor> tensors;
  std::unordered_map<std::string, size_t> index;
  ~rmoe_shards() {
    for (int fd : fds) close(fd);
  }
  const StTensor* find(const std::string& n) const {
    auto it = index.find(n);
    return it == index.end() ? nullptr : &tensors[it->second];
  }
};

namespace {

rmoe_status parse_file(rmoe_shards* sh, const std::string& path) {
  const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return lfail(RMOE_IO_ERROR, "%s: %s", path.c_str(), strerror(errno));
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    return lfail(RMOE_IO_ERROR, "%s: %s", path.c_str(), strerror(errno));
  }
  const uint64_t file_len = static_cast<uint64_t>(st.st_size);
  uint8_t hb[8];
  if (file_len < 8 || !read_exact_at(fd, 0, hb, 8)) {
    close(fd);
    return lfail(RMOE_IO_ERROR, "%s: bad safetensors header: file shorter than its length prefix", path.c_str());
  }
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | hb[i];
  if (hlen > file_len) {
    close(fd);
    return lfail(RMOE_IO_ERROR, "%s: bad safetensors header: header length %llu exceeds file size %llu", path.c_str(),
                 static_cast<unsigned long long>(hlen), static_cast<unsigned long long>(file_len));
  }
  std::vector<char> h(hlen);
  if (hlen && !read_exact_at(fd, 8, h.data(), hlen)) {
    close(fd);
    return lfail(RMOE_IO_ERROR, "%s: short read of the header", path.c_str());
  }
  const uint64_t data_start = 8 + hlen;
  const int file_index = static_cast<int>(sh->fds.size());
  sh->fds.push_back(fd);
  sh->paths.push_back(path);
  Json js{h.data(), h.data() + h.size(), {}};
  auto bad = [&](const std::string& what) {
    return lfail(RMOE_IO_ERROR, "%s: bad safetensors header: %s", path.c_str(), what.c_str());
  };
  if (!js.expect('{')) return bad("top-level value is not an object");
  js.ws();
  if (js.p < js.end && *js.p == '}') return RMOE_OK;
  for (;;) {
    std::string name;
    if (!js.string(name) || !js.expect(':')) return bad(js.err);
    if (name == "__metadata__") {
      if (!js.skip()) return bad(js.err);
    } else {
      StTensor t;
      t.name = name;
      t.file = file_index;
      bool have_dtype = false, have_shape = false, have_off = false;
      std::vector<uint64_t> offs;
      if (!js.expect('{')) return bad(name + ": " + js.err);
      js.ws();
      if (js.p < js.end && *js.p != '}') {
        for (;;) {
          std::string key;
          if (!js.string(key) || !js.expect(':')) return bad(name + ": " + js.err);
          if (key == "dtype") {
            if (!js.string(t.dtype)) return bad(name + ": " + js.err);
            have_dtype = true;
          } else if (key == "shape") {
            if (!js.u64_array(t.shape)) return bad(name + ": shape: " + js.err);
            have_shape = true;
          } else if (key == "data_offsets") {
            if (!js.u64_array(offs)) return bad(name + ": data_offsets: " + js.err);
            have_off = true;
          } else if (!js.skip()) {
            return bad(name + ": " + js.err);
          }
          js.ws();
          if (js.p < js.end && *js.p == ',') {
            js.p++;
            continue;
          }
          if (!js.expect('}')) return bad(name + ": " + js.err);
          break;
        }
      } else {
        js.p++;
      }
      if (!have_dtype) return bad(name + ": missing dtype");
      if (!have_off) return bad(name + ": missing data_offsets");
      if (!have_shape) return bad(name + ": missing shape");
      if (offs.size() != 2) return bad(name + ": data_offsets must have 2 elements");
      if (offs[1] < offs[0]) return bad(name + ": data_offsets end precedes start");
      if (data_start + offs[1] > file_len) return bad(name + ": data_offsets end extends past end of file");
      t.offset = data_start + offs[0];
      t.nbytes = offs[1] - offs[0];
      auto it = sh->index.find(name);
      if (it != sh->index.end()) {
        sh->tensors[it->second] = t;  // a later shard's tensor of the same name wins
      } else {
        sh->index.emplace(name, sh->tensors.size());
        sh->tensors.push_back(std::move(t));
      }
    }
    js.ws();
    if (js.p < js.end && *js.p == ',') {
      js.p++;
      continue;
    }
    if (!js.expect('}')) return bad(js.err);
    break;
  }
  return RMOE_OK;
}

// One tensor read in full into a host buffer.
rmoe_status read_tensor(const rmoe_shards* sh, const std::string& name, std::vector<uint8_t>& out) {
  const StTensor* t = sh->find(name);
  if (!t) return lfail(RMOE_MISSING_TENSOR, "missing tensor: %s", name.c_str());
  out.resize(t->nbytes);
  if (t->nbytes && !read_exact_at(sh->fds[t->file], t->offset, out.data(), t->nbytes))
    return lfail(RMOE_IO_ERROR, "%s: short read from %s", name.c_str(), sh->paths[t->file].c_str());
  return RMOE_OK;
}

size_t div_up(size_t a, size_t b) { return (a + b - 1) / b; }

// One quantized matrix of an expert as the layer takes it: data + scale bytes.
struct QtBytes {
  std::vector<uint8_t> data, scale;
};

// The base name's MXFP4 pair ({base}{suffix}, {base}.weight_scale), lengths checked.
rmoe_status load_mxfp4(const rmoe_shards* sh, const std::string& base, const char* suffix, size_t rows, size_t cols,
                       QtBytes& q) {
  const std::string packed = base + suffix, scale = base + ".weight_scale";
  rmoe_status s = read_tensor(sh, packed, q.data);
  if (s != RMOE_OK) return s;
  if ((s = read_tensor(sh, scale, q.scale)) != RMOE_OK) return s;
  if (q.data.size() != rows * div_up(cols, 2))
    return lfail(RMOE_SHAPE_MISMATCH, "%s: expected %zu bytes, got %zu", packed.c_str(), rows * div_up(cols, 2),
                 q.data.size());
  if (q.scale.size() != rows * div_up(cols, 32))
    return lfail(RMOE_SHAPE_MISMATCH, "%s: expected %zu bytes, got %zu", scale.c_str(), rows * div_up(cols, 32),
                 q.scale.size());
  return RMOE_OK;
}

// A `{name}` int4 matrix with its `{name}.qs` f32 group scales (rabbit's pre-quantized format).
rmoe_status load_grouped(const rmoe_shards* sh, const std::string& name, size_t rows, size_t cols, size_t gs,
                         QtBytes& q) {
  const std::string qs = name + ".qs";
  if (!sh->find(qs)) {
    if (sh->find(name))
      return lfail(RMOE_NOT_SUPPORTED,
                   "%s: a plain float tensor (no .qs sidecar): the reference quantizes those at load; "
                   "store the expert pre-quantized (int4 bytes + .qs scales) or as an MXFP4 pair",
                   name.c_str());
    return lfail(RMOE_MISSING_TENSOR, "missing tensor: %s", name.c_str());
  }
  rmoe_status s = read_tensor(sh, name, q.data);
  if (s != RMOE_OK) return s;
  if ((s = read_tensor(sh, qs, q.scale)) != RMOE_OK) return s;
  const StTensor* t = sh->find(qs);
  if (t->dtype != "F32") return lfail(RMOE_NOT_SUPPORTED, "%s: scales stored as %s (F32 expected)", qs.c_str(), t->dtype.c_str());
  const size_t ng = div_up(cols, gs);
  if (q.data.size() != rows * div_up(cols, 2) || q.scale.size() != rows * ng * 4)
    return lfail(RMOE_SHAPE_MISMATCH,
                 "%s: packed format mismatch: data %zu bytes, scale %zu floats for a %zu x %zu matrix, group size %zu",
                 name.c_str(), q.data.size(), q.scale.size() / 4, rows, cols, gs);
  return RMOE_OK;
}

bool is_mxfp4_naming(int naming) { return naming == RMOE_NAMING_KIMI_K3_MXFP4 || naming == RMOE_NAMING_QWEN38_MXFP4; }

// (tensor name, rows, cols) of one routed expert in read order: gate, up, down (fused: gate_up, down).
bool expert_specs(int naming, int layer, int eid, size_t inter, size_t hidden,
                  std::vector<std::pair<std::string, std::pair<size_t, size_t>>>& out) {
  char pre[256];
  out.clear();
  auto add = [&](const char* suffix, size_t r, size_t c) { out.push_back({std::string(pre) + suffix, {r, c}}); };
  switch (naming) {
    case RMOE_NAMING_GLM52:
      snprintf(pre, sizeof(pre), "model.layers.%d.mlp.experts.%d.", layer, eid);
      add("gate_proj.weight", inter, hidden);
      add("up_proj.weight", inter, hidden);
      add("down_proj.weight", hidden, inter);
      return true;
    case RMOE_NAMING_GLM52_FUSED_GATE_UP:
      snprintf(pre, sizeof(pre), "model.layers.%d.mlp.experts.%d.", layer, eid);
      add("gate_up_proj.weight", 2 * inter, hidden);
      add("down_proj.weight", hidden, inter);
      return true;
    case RMOE_NAMING_KIMI_LINEAR:
      snprintf(pre, sizeof(pre), "model.layers.%d.block_sparse_moe.experts.%d.", layer, eid);
      add("w1.weight", inter, hidden);
      add("w3.weight", inter, hidden);
      add("w2.weight", hidden, inter);
      return true;
    case RMOE_NAMING_KIMI_K3:
      snprintf(pre, sizeof(pre), "language_model.model.layers.%d.block_sparse_moe.experts.%d.", layer, eid);
      add("w1.weight", inter, hidden);
      add("w3.weight", inter, hidden);
      add("w2.weight", hidden, inter);
      return true;
    case RMOE_NAMING_KIMI_K3_MXFP4:  // base names: the loader appends the packed / scale suffixes
      snprintf(pre, sizeof(pre), "language_model.model.layers.%d.block_sparse_moe.experts.%d.", layer, eid);
      add("w1", inter, hidden);
      add("w3", inter, hidden);
      add("w2", hidden, inter);
      return true;
    case RMOE_NAMING_QWEN38_MXFP4:
      snprintf(pre, sizeof(pre), "model.layers.%d.mlp.experts.%d.", layer, eid);
      add("gate_proj", inter, hidden);
      add("up_proj", inter, hidden);
      add("down_proj", hidden, inter);
      return true;
    default:
      return false;
  }
}

// One matrix of the layer's weight format from `name`: an MXFP4 pair when the layer is MXFP4
// (`name` a base name, or `name` = base + ".weight" whose ".weight_scale" sidecar exists), a
// grouped-int4 `.qs` pair otherwise.
rmoe_status load_matrix(const rmoe_shards* sh, const rmoe_layer_desc& d, const std::string& name, bool base_name,
                        const char* suffix, size_t rows, size_t cols, QtBytes& q) {
  if (d.weight_format == RMOE_FMT_MXFP4) {
    if (base_name) return load_mxfp4(sh, name, suffix, rows, cols, q);
    const std::string base = name.size() > 7 && name.compare(name.size() - 7, 7, ".weight") == 0
                                 ? name.substr(0, name.size() - 7)
                                 : name;
    if (sh->find(base + ".weight_scale")) return load_mxfp4(sh, base, ".weight", rows, cols, q);
    if (sh->find(name + ".qs"))
      return lfail(RMOE_NOT_SUPPORTED, "%s: grouped int4 (.qs) tensor for an MXFP4 layer", name.c_str());
    if (sh->find(name))
      return lfail(RMOE_NOT_SUPPORTED,
                   "%s: a plain float tensor: the reference quantizes those at load; store it as an MXFP4 pair",
                   name.c_str());
    return lfail(RMOE_MISSING_TENSOR, "missing tensor: %s", name.c_str());
  }
  if (base_name) return lfail(RMOE_NOT_SUPPORTED, "%s: MXFP4 checkpoint naming for an int4 layer", name.c_str());
  if (d.scale_dtype != RMOE_F32)
    return lfail(RMOE_NOT_SUPPORTED, "%s: the checkpoint's .qs scales are f32; create the layer with scale_dtype RMOE_F32",
                 name.c_str());
  return load_grouped(sh, name, rows, cols, static_cast<size_t>(d.group_size), q);
}

rmoe_status read_f32_vector(const rmoe_shards* sh, const std::string& name, size_t expected, std::vector<float>& out,
                            std::vector<uint16_t>* bf16_out = nullptr) {
  const StTensor* t = sh->find(name);
  if (!t) return lfail(RMOE_MISSING_TENSOR, "missing tensor: %s", name.c_str());
  std::vector<uint8_t> raw;
  rmoe_status s = read_tensor(sh, name, raw);
  if (s != RMOE_OK) return s;
  const size_t esz = t->dtype == "F32" ? 4 : (t->dtype == "BF16" || t->dtype == "F16") ? 2 : 0;
  if (!esz) return lfail(RMOE_NOT_SUPPORTED, "%s: dtype %s (F32, BF16 or F16 expected)", name.c_str(), t->dtype.c_str());
  const size_t n = raw.size() / esz;
  if (n != expected || raw.size() % esz)
    return lfail(RMOE_SHAPE_MISMATCH, "%s: expected %zu elements, got %zu", name.c_str(), expected, n);
  if (bf16_out && t->dtype == "BF16") {  // kept as stored (the router takes bf16 directly)
    bf16_out->resize(n);
    memcpy(bf16_out->data(), raw.data(), raw.size());
    out.clear();
    return RMOE_OK;
  }
  out.resize(n);
  for (size_t i = 0; i < n; i++) {
    if (esz == 4) {
      memcpy(&out[i], raw.data() + 4 * i, 4);
    } else {
      uint16_t hbits;
      memcpy(&hbits, raw.data() + 2 * i, 2);
      uint32_t f;
      if (t->dtype == "BF16") {
        f = static_cast<uint32_t>(hbits) << 16;
      } else {  // IEEE binary16 -> binary32 (exact)
        const uint32_t sign = (hbits & 0x8000u) << 16, ex = (hbits >> 10) & 31, man = hbits & 1023;
        if (ex == 0) {
          if (man == 0) {
            f = sign;
          } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do {
              e++;
              m <<= 1;
            } while (!(m & 1024));
            f = sign | ((112 - e) << 23) | ((m & 1023) << 13);
          }
        } else if (ex == 31) {
          f = sign | 0x7F800000u | (man << 13);
        } else {
          f = sign | ((ex + 112) << 23) | (man << 13);
        }
      }
      memcpy(&out[i], &f, 4);
    }
  }
  return RMOE_OK;
}

}  // namespace

extern "C" rmoe_status rmoe_shards_open(const char* const* dirs, int32_t n_dirs, rmoe_shards** out) {
  if (!out || (!dirs && n_dirs > 0) || n_dirs < 0) return lfail(RMOE_INVALID_ARG, "rmoe_shards_open: null argument");
  *out = nullptr;
  std::vector<std::pair<std::string, std::string>> files;  // (file name, path)
  for (int i = 0; i < n_dirs; i++) {
    if (!dirs[i]) return lfail(RMOE_INVALID_ARG, "rmoe_shards_open: null directory %d", i);
    DIR* d = opendir(dirs[i]);
    if (!d) return lfail(RMOE_IO_ERROR, "%s: %s", dirs[i], strerror(errno));
    while (dirent* e = readdir(d)) {
      const std::string n = e->d_name;
      if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0)
        files.push_back({n, std::string(dirs[i]) + "/" + n});
    }
    closedir(d);
  }
  std::stable_sort(files.begin(), files.end(),
                   [](const auto& a, const auto& b) { return a.first < b.first; });
  rmoe_shards* sh = new (std::nothrow) rmoe_shards();
  if (!sh) return lfail(RMOE_OUT_OF_MEMORY, "rmoe_shards_open: host allocation");
  for (const auto& f : files) {
    rmoe_status s = parse_file(sh, f.second);
    if (s != RMOE_OK) {
      delete sh;
      return s;
    }
  }
  *out = sh;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_shards_close(rmoe_shards* sh) {
  delete sh;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_shards_count(const rmoe_shards* sh, int64_t* n_tensors) {
  if (!sh || !n_tensors) return lfail(RMOE_INVALID_ARG, "rmoe_shards_count: null argument");
  *n_tensors = static_cast<int64_t>(sh->tensors.size());
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_shards_tensor(const rmoe_shards* sh, const char* name, char* dtype, uint64_t* shape,
                                          int32_t* ndim, uint64_t* nbytes) {
  if (!sh || !name) return lfail(RMOE_INVALID_ARG, "rmoe_shards_tensor: null argument");
  const StTensor* t = sh->find(name);
  if (!t) return lfail(RMOE_MISSING_TENSOR, "missing tensor: %s", name);
  if (dtype) {
    memset(dtype, 0, RMOE_DTYPE_NAME_BYTES);
    strncpy(dtype, t->dtype.c_str(), RMOE_DTYPE_NAME_BYTES - 1);
  }
  if (ndim) *ndim = static_cast<int32_t>(t->shape.size());
  if (shape)
    for (size_t i = 0; i < t->shape.size() && i < RMOE_MAX_TENSOR_DIMS; i++) shape[i] = t->shape[i];
  if (nbytes) *nbytes = t->nbytes;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_shards_read_raw(const rmoe_shards* sh, const char* name, void* dst, size_t dst_bytes) {
  if (!sh || !name || (!dst && dst_bytes)) return lfail(RMOE_INVALID_ARG, "rmoe_shards_read_raw: null argument");
  const StTensor* t = sh->find(name);
  if (!t) return lfail(RMOE_MISSING_TENSOR, "missing tensor: %s", name);
  if (t->nbytes != dst_bytes)
    return lfail(RMOE_SHAPE_MISMATCH, "%s: tensor holds %llu bytes, buffer %zu", name,
                 static_cast<unsigned long long>(t->nbytes), dst_bytes);
  if (dst_bytes && !read_exact_at(sh->fds[t->file], t->offset, dst, dst_bytes))
    return lfail(RMOE_IO_ERROR, "%s: short read from %s", name, sh->paths[t->file].c_str());
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_load_expert(rmoe_layer* layer, const rmoe_shards* sh, int32_t naming, int32_t layer_index,
                                        int32_t eid) {
  if (!layer || !sh) return lfail(RMOE_INVALID_ARG, "rmoe_load_expert: null argument");
  rmoe_layer_desc d{};
  rmoe_status s = rmoe_layer_get_desc(layer, &d);
  if (s != RMOE_OK) return s;
  std::vector<std::pair<std::string, std::pair<size_t, size_t>>> specs;
  if (!expert_specs(naming, layer_index, eid, static_cast<size_t>(d.moe_inter), static_cast<size_t>(d.hidden), specs))
    return lfail(RMOE_INVALID_ARG, "rmoe_load_expert: naming %d", naming);
  const bool mx = is_mxfp4_naming(naming);
  const char* suffix = naming == RMOE_NAMING_QWEN38_MXFP4 ? ".weight" : ".weight_packed";
  std::vector<QtBytes> q(specs.size());
  for (size_t i = 0; i < specs.size(); i++) {
    s = load_matrix(sh, d, specs[i].first, mx, suffix, specs[i].second.first, specs[i].second.second, q[i]);
    if (s != RMOE_OK) return s;
  }
  if (specs.size() == 2)
    return rmoe_upload_expert_fused(layer, eid, q[0].data.data(), q[0].data.size(), q[0].scale.data(), q[0].scale.size(),
                                    q[1].data.data(), q[1].data.size(), q[1].scale.data(), q[1].scale.size());
  return rmoe_upload_expert(layer, eid, q[0].data.data(), q[0].data.size(), q[0].scale.data(), q[0].scale.size(),
                            q[1].data.data(), q[1].data.size(), q[1].scale.data(), q[1].scale.size(),
                            q[2].data.data(), q[2].data.size(), q[2].scale.data(), q[2].scale.size());
}

extern "C" rmoe_status rmoe_load_moe_weights(rmoe_layer* layer, const rmoe_shards* sh, int32_t family,
                                             int32_t layer_index) {
  if (!layer || !sh) return lfail(RMOE_INVALID_ARG, "rmoe_load_moe_weights: null argument");
  if (family != RMOE_FAMILY_QWEN38 && family != RMOE_FAMILY_GLM52)
    return lfail(RMOE_INVALID_ARG, "rmoe_load_moe_weights: family %d", family);
  rmoe_layer_desc d{};
  rmoe_status s = rmoe_layer_get_desc(layer, &d);
  if (s != RMOE_OK) return s;
  char mp[128];
  snprintf(mp, sizeof(mp), "model.layers.%d.mlp.", layer_index);
  const std::string p = mp;
  const size_t E = static_cast<size_t>(d.n_experts), H = static_cast<size_t>(d.router_hidden ? d.router_hidden : d.hidden);
  // router [E, H] (src/qwen38/model.rs:320, src/glm52/model.rs:249), kept bf16 when stored bf16
  {
    std::vector<float> r;
    std::vector<uint16_t> rb;
    if ((s = read_f32_vector(sh, p + "gate.weight", E * H, r, &rb)) != RMOE_OK) return s;
    s = rb.empty() ? rmoe_upload_router(layer, r.data(), RMOE_F32, r.size() * 4)
                   : rmoe_upload_router(layer, rb.data(), RMOE_BF16, rb.size() * 2);
    if (s != RMOE_OK) return s;
  }
  if (family == RMOE_FAMILY_GLM52) {  // selection-only correction bias (src/glm52/model.rs:250)
    std::vector<float> b;
    if ((s = read_f32_vector(sh, p + "gate.e_score_correction_bias", E, b)) != RMOE_OK) return s;
    if ((s = rmoe_upload_router_bias(layer, b.data(), b.size())) != RMOE_OK) return s;
  }
  if (d.shared_inter <= 0) return RMOE_OK;
  const size_t Is = static_cast<size_t>(d.shared_inter), Hd = static_cast<size_t>(d.hidden);
  const std::string sp = p + (family == RMOE_FAMILY_QWEN38 ? "shared_expert." : "shared_experts.");
  QtBytes g, u, dn;
  if ((s = load_matrix(sh, d, sp + "gate_proj.weight", false, nullptr, Is, Hd, g)) != RMOE_OK) return s;
  if ((s = load_matrix(sh, d, sp + "up_proj.weight", false, nullptr, Is, Hd, u)) != RMOE_OK) return s;
  if ((s = load_matrix(sh, d, sp + "down_proj.weight", false, nullptr, Hd, Is, dn)) != RMOE_OK) return s;
  std::vector<float> sg;
  if (family == RMOE_FAMILY_QWEN38 && d.shared_gated) {  // shared_expert_gate.weight [1, H] (:321)
    if ((s = read_f32_vector(sh, p + "shared_expert_gate.weight", Hd, sg)) != RMOE_OK) return s;
  }
  return rmoe_upload_shared(layer, g.data.data(), g.data.size(), g.scale.data(), g.scale.size(), u.data.data(),
                            u.data.size(), u.scale.data(), u.scale.size(), dn.data.data(), dn.data.size(),
                            dn.scale.data(), dn.scale.size(), sg.empty() ? nullptr : sg.data());
}
