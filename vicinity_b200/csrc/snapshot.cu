// Directory snapshots in the reference's format: vg_ivfpq_save mirrors
// IVFPQIndex::save_to_dir (src/ivf_pq/search.rs:945-1015) and vg_ivfpq_load
// mirrors IVFPQIndex::load_from_dir (search.rs:1034-1084).
//
// Files (all little-endian):
//   manifest.json     serde JSON of IVFPQManifest (manifest.rs:44-62)
//   centroids.bin     f32 [num_centroids][dimension]
//   doc_ids.bin       u32 [num_vectors]
//   codes.bin         u8  [num_vectors][num_codebooks], insertion order
//   list_offsets.bin  u64 [num_clusters + 1]   (file_storage.rs:39-72;
//   list_codes.bin    u8  list-contiguous codes  written, not read by load)
//   clusters.bin      "VICIVF1\0", u64 count, per cluster u64 filter
//                     bitmask, u64 length, u32 ids (persistence.rs:51-69)
//   raw_vectors.bin   f32 [num_vectors][dimension] when raw vectors are kept
// Every file is written to a temporary name, flushed, synced and renamed into
// place, then the directory is synced (persistence.rs:71-110).
//
// This file is host code only: it parses and writes the files and hands a
// SnapshotState to index.cu, which owns the device layout.
#include <cerrno>
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <algorithm>
#include <cctype>
#include <chrono>
#include <atomic>
#include <sys/file.h>
#include <dirent.h>
#include <string>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

#include "snapshot.h"
#include "vicinity_gpu.h"

namespace {

using vg::SnapshotState;

constexpr uint32_t kFormatVersion = 1;  // persistence.rs:9
constexpr char kClusterMagic[8] = {'V', 'I', 'C', 'I', 'V', 'F', '1', '\0'};

int fail(int code, const std::string &msg) {
  vg::set_last_error(msg.c_str());
  return code;
}

int io_fail(int err, const std::string &what) {
  return fail(err == ENOENT ? VG_ERR_NOT_FOUND : VG_ERR_IO, what + ": " + std::strerror(err));
}

int format_fail(const std::string &msg) { return fail(VG_ERR_FORMAT, msg); }

// ---- a small JSON reader -----------------------------------------------------

struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  std::string text;  // number token or decoded string
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal *get(const char *key) const {
    for (const auto &kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char *p, *end;
  std::string err;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail_at(const char *what) {
    if (err.empty()) err = what;
    return false;
  }
  bool lit(const char *s) {
    const size_t n = std::strlen(s);
    if (static_cast<size_t>(end - p) < n || std::memcmp(p, s, n) != 0) return fail_at("invalid literal");
    p += n;
    return true;
  }
  static void put_utf8(std::string &o, uint32_t c) {
    if (c < 0x80) {
      o += static_cast<char>(c);
    } else if (c < 0x800) {
      o += static_cast<char>(0xC0 | (c >> 6));
      o += static_cast<char>(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
      o += static_cast<char>(0xE0 | (c >> 12));
      o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (c & 0x3F));
    } else {
      o += static_cast<char>(0xF0 | (c >> 18));
      o += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
      o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (c & 0x3F));
    }
  }
  bool hex4(uint32_t &v) {
    if (end - p < 4) return fail_at("truncated \\u escape");
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else return fail_at("bad \\u escape");
    }
    return true;
  }
  bool string(std::string &o) {
    if (p >= end || *p != '"') return fail_at("expected string");
    ++p;
    while (p < end && *p != '"') {
      const unsigned char c = static_cast<unsigned char>(*p++);
      if (c < 0x20) return fail_at("control character in string");
      if (c != '\\') {
        o += static_cast<char>(c);
        continue;
      }
      if (p >= end) return fail_at("truncated escape");
      const char e = *p++;
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t v = 0;
          if (!hex4(v)) return false;
          if (v >= 0xD800 && v < 0xDC00) {
            uint32_t lo = 0;
            if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return fail_at("unpaired surrogate");
            p += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail_at("unpaired surrogate");
            v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
          } else if (v >= 0xDC00 && v < 0xE000) {
            return fail_at("unpaired surrogate");
          }
          put_utf8(o, v);
          break;
        }
        default: return fail_at("bad escape");
      }
    }
    if (p >= end) return fail_at("unterminated string");
    ++p;
    return true;
  }
  bool number(std::string &o) {
    const char *s = p;
    if (p < end && *p == '-') ++p;
    if (p >= end || !(*p >= '0' && *p <= '9')) return fail_at("bad number");
    if (*p == '0') ++p;
    else while (p < end && *p >= '0' && *p <= '9') ++p;
    if (p < end && *p == '.') {
      ++p;
      if (p >= end || !(*p >= '0' && *p <= '9')) return fail_at("bad number");
      while (p < end && *p >= '0' && *p <= '9') ++p;
    }
    if (p < end && (*p == 'e' || *p == 'E')) {
      ++p;
      if (p < end && (*p == '+' || *p == '-')) ++p;
      if (p >= end || !(*p >= '0' && *p <= '9')) return fail_at("bad number");
      while (p < end && *p >= '0' && *p <= '9') ++p;
    }
    o.assign(s, p);
    return true;
  }
  bool value(JVal &v) {
    if (++depth > 64) return fail_at("nesting too deep");
    ws();
    if (p >= end) return fail_at("unexpected end of input");
    bool ok = true;
    switch (*p) {
      case '{': {
        v.kind = JVal::Obj;
        ++p;
        ws();
        if (p < end && *p == '}') {
          ++p;
          break;
        }
        for (;;) {
          ws();
          std::string key;
          if (!string(key)) return false;
          ws();
          if (p >= end || *p != ':') return fail_at("expected ':'");
          ++p;
          v.obj.emplace_back(std::move(key), JVal{});
          if (!value(v.obj.back().second)) return false;
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == '}') {
            ++p;
            break;
          }
          return fail_at("expected ',' or '}'");
        }
        break;
      }
      case '[': {
        v.kind = JVal::Arr;
        ++p;
        ws();
        if (p < end && *p == ']') {
          ++p;
          break;
        }
        for (;;) {
          v.arr.emplace_back();
          if (!value(v.arr.back())) return false;
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == ']') {
            ++p;
            break;
          }
          return fail_at("expected ',' or ']'");
        }
        break;
      }
      case '"': v.kind = JVal::Str; ok = string(v.text); break;
      case 't': v.kind = JVal::Bool; v.b = true; ok = lit("true"); break;
      case 'f': v.kind = JVal::Bool; v.b = false; ok = lit("false"); break;
      case 'n': v.kind = JVal::Null; ok = lit("null"); break;
      default: v.kind = JVal::Num; ok = number(v.text); break;
    }
    --depth;
    return ok;
  }
};

bool parse_json(const std::string &text, JVal &out, std::string &err) {
  JParser ps{text.data(), text.data() + text.size()};
  if (!ps.value(out)) {
    err = ps.err;
    return false;
  }
  ps.ws();
  if (ps.p != ps.end) {
    err = "trailing characters";
    return false;
  }
  return true;
}

// Typed field access in serde's terms: a missing or mistyped field is a
// format error naming the field.
struct Fields {
  const JVal &o;
  std::string where, err;
  const JVal *need(const char *key, JVal::Kind kind) {
    const JVal *v = o.kind == JVal::Obj ? o.get(key) : nullptr;
    if (!v) {
      if (err.empty()) err = "missing field `" + std::string(key) + "` in " + where;
      return nullptr;
    }
    if (v->kind != kind) {
      if (err.empty()) err = "invalid type for `" + std::string(key) + "` in " + where;
      return nullptr;
    }
    return v;
  }
  bool u64(const char *key, uint64_t &out) {
    const JVal *v = need(key, JVal::Num);
    if (!v) return false;
    const std::string &t = v->text;
    if (t.empty() || t[0] == '-' || t.find_first_of(".eE") != std::string::npos) {
      if (err.empty()) err = "`" + std::string(key) + "` is not an unsigned integer in " + where;
      return false;
    }
    errno = 0;
    out = std::strtoull(t.c_str(), nullptr, 10);
    if (errno == ERANGE) {
      if (err.empty()) err = "`" + std::string(key) + "` overflows u64 in " + where;
      return false;
    }
    return true;
  }
  bool boolean(const char *key, bool &out) {
    const JVal *v = need(key, JVal::Bool);
    if (v) out = v->b;
    return v != nullptr;
  }
};

bool f32_array(const JVal &a, std::vector<float> &out, std::string &err, const char *what) {
  if (a.kind != JVal::Arr) {
    err = std::string(what) + " is not an array";
    return false;
  }
  out.resize(a.arr.size());
  for (size_t i = 0; i < a.arr.size(); ++i) {
    if (a.arr[i].kind != JVal::Num) {
      err = std::string(what) + " holds a non-number";
      return false;
    }
    out[i] = std::strtof(a.arr[i].text.c_str(), nullptr);
  }
  return true;
}

bool read_product(const JVal &q, SnapshotState &st, std::string &err) {
  Fields f{q, "quantizer"};
  uint64_t dim = 0, m = 0, ks = 0, dsub = 0;
  if (!f.u64("dimension", dim) || !f.u64("num_codebooks", m) || !f.u64("codebook_size", ks) ||
      !f.u64("subvector_dim", dsub)) {
    err = f.err;
    return false;
  }
  const JVal *cb = f.need("codebooks", JVal::Arr);
  if (!cb) {
    err = f.err;
    return false;
  }
  if (!f32_array(*cb, st.codebooks, err, "quantizer codebooks")) return false;
  if (dim != st.dim || m != st.params.num_codebooks || ks != st.params.codebook_size || m == 0 ||
      dsub * m != dim) {
    err = "quantizer shape does not match the manifest";
    return false;
  }
  return true;
}

// ---- binary files -------------------------------------------------------------

int read_file(const std::string &path, std::string &out) {
  FILE *f = std::fopen(path.c_str(), "rb");
  if (!f) return io_fail(errno, path);
  out.clear();
  char buf[1 << 16];
  size_t got;
  while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) out.append(buf, got);
  const bool bad = std::ferror(f) != 0;
  const int e = errno;
  std::fclose(f);
  if (bad) return io_fail(e, path);
  return VG_OK;
}

template <class T>
int read_exact(const std::string &path, size_t count, std::vector<T> &out) {
  std::string raw;
  if (int s = read_file(path, raw)) return s;
  if (raw.size() != count * sizeof(T))  // persistence.rs:120-176
    return format_fail(path + " size mismatch: expected " + std::to_string(count * sizeof(T)) + " bytes, got " +
                       std::to_string(raw.size()));
  out.resize(count);
  if (count) std::memcpy(out.data(), raw.data(), raw.size());
  return VG_OK;
}

int read_clusters(const std::string &path, size_t expected, size_t n, SnapshotState &st) {
  std::string raw;
  if (int s = read_file(path, raw)) return s;
  size_t pos = 0;
  auto take = [&](void *dst, size_t bytes) {
    if (raw.size() - pos < bytes) return false;
    std::memcpy(dst, raw.data() + pos, bytes);
    pos += bytes;
    return true;
  };
  char magic[8];
  if (!take(magic, 8)) return format_fail("truncated IVF-PQ cluster file");
  if (std::memcmp(magic, kClusterMagic, 8) != 0) return format_fail("invalid IVF-PQ cluster file magic");
  uint64_t count = 0;
  if (!take(&count, 8)) return format_fail("truncated IVF-PQ cluster file");
  if (count != expected)
    return format_fail("cluster count mismatch: expected " + std::to_string(expected) + ", got " +
                       std::to_string(count));
  st.list_offsets.assign(1, 0);
  st.bitmasks.clear();
  st.list_ids.clear();
  for (uint64_t c = 0; c < count; ++c) {
    uint64_t mask = 0, len = 0;
    if (!take(&mask, 8) || !take(&len, 8)) return format_fail("truncated IVF-PQ cluster file");
    if (len > n)
      return format_fail("cluster length " + std::to_string(len) + " exceeds vector count " + std::to_string(n));
    const size_t base = st.list_ids.size();
    st.list_ids.resize(base + len);
    if (len && !take(st.list_ids.data() + base, len * 4)) return format_fail("truncated IVF-PQ cluster file");
    for (size_t i = base; i < base + len; ++i)
      if (st.list_ids[i] >= n)
        return format_fail("cluster id " + std::to_string(st.list_ids[i]) + " exceeds vector count " +
                           std::to_string(n));
    st.bitmasks.push_back(mask);
    st.list_offsets.push_back(st.list_ids.size());
  }
  if (pos != raw.size()) return format_fail("trailing bytes in IVF-PQ cluster file");
  return VG_OK;
}

struct Writer {
  std::string dir;
  int seq = 0;
  int put(const char *name, const void *data, size_t bytes) {
    const std::string path = dir + "/" + name;
    const std::string tmp = path + ".tmp." + std::to_string(getpid()) + "." + std::to_string(seq++);
    const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return io_fail(errno, tmp);
    const char *c = static_cast<const char *>(data);
    size_t done = 0;
    while (done < bytes) {
      const ssize_t w = ::write(fd, c + done, bytes - done);
      if (w < 0) {
        if (errno == EINTR) continue;
        const int e = errno;
        ::close(fd);
        ::unlink(tmp.c_str());
        return io_fail(e, tmp);
      }
      done += static_cast<size_t>(w);
    }
    if (::fsync(fd) != 0 || ::close(fd) != 0) {
      const int e = errno;
      ::unlink(tmp.c_str());
      return io_fail(e, tmp);
    }
    if (std::rename(tmp.c_str(), path.c_str()) != 0) {
      const int e = errno;
      ::unlink(tmp.c_str());
      return io_fail(e, path);
    }
    return VG_OK;
  }
};

int make_dirs(const std::string &dir) {
  std::string cur;
  for (size_t i = 0; i <= dir.size(); ++i) {
    if (i == dir.size() || (dir[i] == '/' && i > 0)) {
      cur = dir.substr(0, i);
      if (::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST) return io_fail(errno, cur);
    }
  }
  struct stat sb;
  if (::stat(dir.c_str(), &sb) != 0) return io_fail(errno, dir);
  if (!S_ISDIR(sb.st_mode)) return io_fail(ENOTDIR, dir);
  return VG_OK;
}

// ---- manifest writer ----------------------------------------------------------

void json_string(std::string &o, const std::string &s) {
  o += '"';
  for (const unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          std::snprintf(b, sizeof(b), "\\u%04x", c);
          o += b;
        } else {
          o += static_cast<char>(c);
        }
    }
  }
  o += '"';
}

bool json_f32_array(std::string &o, const std::vector<float> &v) {
  o += '[';
  char b[32];
  for (size_t i = 0; i < v.size(); ++i) {
    if (!std::isfinite(v[i])) return false;
    // 9 significant digits identify every f32 exactly
    std::snprintf(b, sizeof(b), "%.9g", static_cast<double>(v[i]));
    if (i) o += ',';
    o += b;
  }
  o += ']';
  return true;
}

bool manifest_text(const SnapshotState &st, std::string &o, bool generation_components = false) {
  const auto &p = st.params;
  auto u = [](uint64_t v) { return std::to_string(v); };
  o = "{\n";
  o += "  \"version\": " + u(kFormatVersion) + ",\n";
  o += "  \"dimension\": " + u(st.dim) + ",\n";
  o += "  \"num_vectors\": " + u(st.num_vectors) + ",\n";
  o += "  \"num_centroids\": " + u(st.num_centroids) + ",\n";
  o += std::string("  \"raw_vectors_present\": ") + (st.vectors.empty() ? "false" : "true") + ",\n";
  o += "  \"params\": {\n";
  o += "    \"num_clusters\": " + u(p.num_clusters) + ",\n";
  o += "    \"nprobe\": " + u(p.nprobe) + ",\n";
  o += "    \"num_codebooks\": " + u(p.num_codebooks) + ",\n";
  o += "    \"codebook_size\": " + u(p.codebook_size) + ",\n";
  o += std::string("    \"use_opq\": ") + (p.use_opq ? "true" : "false") + ",\n";
  o += "    \"seed\": " + u(p.seed) + "\n";
  o += "  },\n";
  std::string pq = "{\"dimension\": " + u(st.dim) + ", \"num_codebooks\": " + u(p.num_codebooks) +
                   ", \"codebook_size\": " + u(p.codebook_size) +
                   ", \"subvector_dim\": " + u(st.dim / p.num_codebooks) + ", \"codebooks\": ";
  if (!json_f32_array(pq, st.codebooks)) return false;
  pq += "}";
  if (st.optimized) {  // opq.rs:31-41
    std::string rot;
    if (st.rotation.empty()) {
      rot = "null";
    } else if (!json_f32_array(rot, st.rotation)) {
      return false;
    }
    o += "  \"quantizer\": {\"Optimized\": {\"dimension\": " + u(st.dim) + ", \"num_codebooks\": " +
         u(p.num_codebooks) + ", \"codebook_size\": " + u(p.codebook_size) + ", \"rotation\": " + rot +
         ", \"pq\": " + pq + "}},\n";
  } else {
    o += "  \"quantizer\": {\"Product\": " + pq + "},\n";
  }
  o += "  \"filter_field\": ";
  if (st.has_filter_field) json_string(o, st.filter_field);
  else o += "null";
  o += ",\n  \"filter_metadata\": [";
  for (size_t i = 0; i < st.metadata.size(); ++i) {
    o += i ? ",\n    " : "\n    ";
    o += "{\"doc_id\": " + u(st.metadata[i].first) + ", \"metadata\": " + st.metadata[i].second + "}";
  }
  o += st.metadata.empty() ? "]" : "\n  ]";
  if (generation_components) {  // manifest.rs:64-77: the payload files of a generation
    o += ",\n  \"generation_components\": [\"centroids.bin\", \"clusters.bin\", \"codes.bin\", \"doc_ids.bin\", "
         "\"list_codes.bin\", \"list_offsets.bin\"";
    if (!st.vectors.empty()) o += ", \"raw_vectors.bin\"";
    o += "]";
  }
  o += "\n}\n";
  return true;
}

// Re-serialise a parsed metadata object compactly (it is stored as text).
void json_dump(std::string &o, const JVal &v) {
  switch (v.kind) {
    case JVal::Null: o += "null"; break;
    case JVal::Bool: o += v.b ? "true" : "false"; break;
    case JVal::Num: o += v.text; break;
    case JVal::Str: json_string(o, v.text); break;
    case JVal::Arr:
      o += '[';
      for (size_t i = 0; i < v.arr.size(); ++i) {
        if (i) o += ',';
        json_dump(o, v.arr[i]);
      }
      o += ']';
      break;
    case JVal::Obj:
      o += '{';
      for (size_t i = 0; i < v.obj.size(); ++i) {
        if (i) o += ',';
        json_string(o, v.obj[i].first);
        o += ':';
        json_dump(o, v.obj[i].second);
      }
      o += '}';
      break;
  }
}

int parse_manifest(const std::string &text, SnapshotState &st) {
  JVal root;
  std::string err;
  if (!parse_json(text, root, err)) return format_fail("manifest.json: " + err);
  if (root.kind != JVal::Obj) return format_fail("manifest.json: not an object");
  Fields f{root, "manifest"};
  uint64_t version = 0, dim = 0, n = 0, nc = 0;
  bool raw = false;
  if (!f.u64("version", version) || !f.u64("dimension", dim) || !f.u64("num_vectors", n) ||
      !f.u64("num_centroids", nc) || !f.boolean("raw_vectors_present", raw))
    return format_fail("manifest.json: " + f.err);
  // persistence.rs:178-203
  if (version != kFormatVersion) return format_fail("unsupported IVF-PQ format version " + std::to_string(version));
  if (dim == 0) return format_fail("IVF-PQ manifest has zero dimension");
  if (n == 0) return format_fail("IVF-PQ manifest has zero vectors");
  if (nc == 0) return format_fail("IVF-PQ manifest has zero centroids");
  st.dim = dim;
  st.num_vectors = n;
  st.num_centroids = nc;
  const JVal *params = f.need("params", JVal::Obj);
  if (!params) return format_fail("manifest.json: " + f.err);
  Fields pf{*params, "params"};
  uint64_t L = 0, nprobe = 0, M = 0, ks = 0, seed = 0;
  bool opq = false;
  if (!pf.u64("num_clusters", L) || !pf.u64("nprobe", nprobe) || !pf.u64("num_codebooks", M) ||
      !pf.u64("codebook_size", ks) || !pf.boolean("use_opq", opq) || !pf.u64("seed", seed))
    return format_fail("manifest.json: " + pf.err);
  st.params.num_clusters = L;
  st.params.nprobe = nprobe;
  st.params.num_codebooks = M;
  st.params.codebook_size = ks;
  st.params.use_opq = opq ? 1 : 0;
  st.params.seed = seed;
  const JVal *q = f.need("quantizer", JVal::Obj);
  if (!q) return format_fail("manifest.json: " + f.err);
  if (q->obj.size() != 1) return format_fail("manifest.json: quantizer must name exactly one variant");
  const std::string &variant = q->obj[0].first;
  const JVal &qv = q->obj[0].second;
  if (variant == "Product") {
    if (!read_product(qv, st, err)) return format_fail("manifest.json: " + err);
  } else if (variant == "Optimized") {
    st.optimized = true;
    Fields of{qv, "Optimized quantizer"};
    const JVal *pq = of.need("pq", JVal::Obj);
    if (!pq) return format_fail("manifest.json: " + of.err);
    if (!read_product(*pq, st, err)) return format_fail("manifest.json: " + err);
    const JVal *rot = qv.get("rotation");
    if (!rot) return format_fail("manifest.json: missing field `rotation` in Optimized quantizer");
    if (rot->kind != JVal::Null) {
      if (!f32_array(*rot, st.rotation, err, "OPQ rotation")) return format_fail("manifest.json: " + err);
      if (st.rotation.size() != dim * dim) return format_fail("manifest.json: OPQ rotation is not dimension x dimension");
    }
  } else {
    return format_fail("manifest.json: unknown quantizer variant `" + variant + "`");
  }
  // optional fields (serde defaults, manifest.rs:53-61)
  if (const JVal *ff = root.get("filter_field")) {
    if (ff->kind == JVal::Str) {
      st.has_filter_field = true;
      st.filter_field = ff->text;
    } else if (ff->kind != JVal::Null) {
      return format_fail("manifest.json: invalid type for `filter_field`");
    }
  }
  if (const JVal *fm = root.get("filter_metadata")) {
    if (fm->kind != JVal::Arr) return format_fail("manifest.json: invalid type for `filter_metadata`");
    for (const JVal &e : fm->arr) {
      Fields ef{e, "filter_metadata entry"};
      uint64_t doc = 0;
      if (!ef.u64("doc_id", doc) || doc > 0xffffffffull) return format_fail("manifest.json: " + ef.err);
      const JVal *md = ef.need("metadata", JVal::Obj);
      if (!md) return format_fail("manifest.json: " + ef.err);
      std::string txt;
      json_dump(txt, *md);
      st.metadata.emplace_back(static_cast<uint32_t>(doc), std::move(txt));
    }
    if (!st.metadata.empty() && !st.has_filter_field)  // search.rs:1068-1073
      return format_fail("IVF-PQ manifest has filter metadata without filter_field");
  }
  if (const JVal *gc = root.get("generation_components")) {  // manifest.rs:64-98
    if (gc->kind != JVal::Null) {
      std::vector<std::string> expect = {"centroids.bin", "clusters.bin", "codes.bin",
                                         "doc_ids.bin", "list_codes.bin", "list_offsets.bin"};
      if (raw) expect.push_back("raw_vectors.bin");
      bool same = gc->kind == JVal::Arr && gc->arr.size() == expect.size();
      for (size_t i = 0; same && i < expect.size(); ++i)
        same = gc->arr[i].kind == JVal::Str && gc->arr[i].text == expect[i];
      if (!same) return format_fail("IVF-PQ generation component inventory mismatch");
    }
  }
  st.vectors.clear();
  if (raw) st.vectors.resize(1);  // marker, replaced by raw_vectors.bin
  return VG_OK;
}

// A MetadataValue in serde form: one of {"Int": i64}, {"Float": f64},
// {"Str": string}, {"Bool": bool}.
bool metadata_value(const JVal &v, std::string &tag) {
  if (v.kind != JVal::Obj || v.obj.size() != 1) return false;
  tag = v.obj[0].first;
  const JVal &x = v.obj[0].second;
  if (tag == "Int") return x.kind == JVal::Num && x.text.find_first_of(".eE") == std::string::npos;
  if (tag == "Float") return x.kind == JVal::Num;
  if (tag == "Str") return x.kind == JVal::Str;
  if (tag == "Bool") return x.kind == JVal::Bool;
  return false;
}

// Category of an Int value: 0..63, else the reference's error.
int int_category(const JVal &v, const std::string &tag, int *category, bool at_search) {
  if (tag != "Int")
    return fail(VG_ERR_INVALID_PARAMETER, "category ID must be an integer in 0..63 for bitmask filtering");
  errno = 0;
  const long long n = std::strtoll(v.obj[0].second.text.c_str(), nullptr, 10);
  if (errno == ERANGE || n < 0 || n >= 64)
    return fail(VG_ERR_INVALID_PARAMETER,
                "category ID " + v.obj[0].second.text + " exceeds bitmask limit of 63" +
                    (at_search ? std::string() : std::string("; use an integer in 0..63")));
  *category = static_cast<int>(n);
  return VG_OK;
}

// Snapshot of ix into directory d (search.rs:945-1016); with generation
// components the manifest lists the payload files (a generation's layout).
int save_dir(const vg_index *ix, const std::string &d, bool components) {
  SnapshotState st;
  if (int s = vg::snapshot_export(ix, st)) return s;
  std::string manifest;
  if (!manifest_text(st, manifest, components)) return fail(VG_ERR_INVALID_PARAMETER, "non-finite value in the quantizer");
  if (int s = make_dirs(d)) return s;
  // list-contiguous codes for the file searcher (file_storage.rs:39-72)
  const size_t M = st.params.num_codebooks;
  std::vector<uint64_t> list_offsets(st.list_offsets.size());
  std::vector<uint8_t> list_codes(st.list_ids.size() * M);
  for (size_t i = 0; i < st.list_offsets.size(); ++i) list_offsets[i] = st.list_offsets[i] * M;
  for (size_t p = 0; p < st.list_ids.size(); ++p)
    std::memcpy(list_codes.data() + p * M, st.codes.data() + static_cast<size_t>(st.list_ids[p]) * M, M);
  std::string clusters(kClusterMagic, 8);
  const uint64_t L = st.bitmasks.size();
  clusters.append(reinterpret_cast<const char *>(&L), 8);
  for (size_t l = 0; l < L; ++l) {
    const uint64_t len = st.list_offsets[l + 1] - st.list_offsets[l];
    clusters.append(reinterpret_cast<const char *>(&st.bitmasks[l]), 8);
    clusters.append(reinterpret_cast<const char *>(&len), 8);
    clusters.append(reinterpret_cast<const char *>(st.list_ids.data() + st.list_offsets[l]), len * 4);
  }
  Writer w{d};
  int s = w.put("manifest.json", manifest.data(), manifest.size());
  if (!s) s = w.put("centroids.bin", st.centroids.data(), st.centroids.size() * 4);
  if (!s) s = w.put("doc_ids.bin", st.doc_ids.data(), st.doc_ids.size() * 4);
  if (!s) s = w.put("codes.bin", st.codes.data(), st.codes.size());
  if (!s) s = w.put("list_offsets.bin", list_offsets.data(), list_offsets.size() * 8);
  if (!s) s = w.put("list_codes.bin", list_codes.data(), list_codes.size());
  if (!s) s = w.put("clusters.bin", clusters.data(), clusters.size());
  if (!s && !st.vectors.empty()) s = w.put("raw_vectors.bin", st.vectors.data(), st.vectors.size() * 4);
  if (s) return s;
  const int fd = ::open(d.c_str(), O_RDONLY | O_DIRECTORY);
  if (fd < 0) return io_fail(errno, d);
  const int r = ::fsync(fd);
  const int e = errno;
  ::close(fd);
  if (r != 0) return io_fail(e, d);
  return VG_OK;
}

// Every file of a directory snapshot read and checked against its manifest
// (persistence.rs:178-203, search.rs:1034-1084), host side only.
int read_snapshot(const std::string &d, SnapshotState &st) {
  std::string text;
  if (int s = read_file(d + "/manifest.json", text)) return s;
  if (int s = parse_manifest(text, st)) return s;
  const bool raw = !st.vectors.empty();
  const size_t n = st.num_vectors, dim = st.dim, M = st.params.num_codebooks;
  if (int s = read_exact(d + "/doc_ids.bin", n, st.doc_ids)) return s;
  if (int s = read_exact(d + "/centroids.bin", st.num_centroids * dim, st.centroids)) return s;
  if (int s = read_exact(d + "/codes.bin", n * M, st.codes)) return s;
  if (int s = read_clusters(d + "/clusters.bin", st.params.num_clusters, n, st)) return s;
  if (raw) {
    if (int s = read_exact(d + "/raw_vectors.bin", n * dim, st.vectors)) return s;
  } else {
    st.vectors.clear();
  }
  return VG_OK;
}

// ---- generations (persistence/generation.rs) ---------------------------------
// A generation root holds generations/<id>/ snapshot directories and a CURRENT
// file naming the published one; each generation carries GENERATION.json, an
// inventory of its files with length and CRC-32.

// CRC-32 (IEEE 802.3: reflected polynomial 0xEDB88320, initial value and
// final xor 0xFFFFFFFF), table-driven.
uint32_t crc32_update(uint32_t crc, const unsigned char *p, size_t n) {
  static uint32_t table[256];
  static bool ready = false;
  if (!ready) {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int b = 0; b < 8; ++b) c = (c & 1u) ? (c >> 1) ^ 0xEDB88320u : c >> 1;
      table[i] = c;
    }
    ready = true;
  }
  for (size_t i = 0; i < n; ++i) crc = table[(crc ^ p[i]) & 0xFFu] ^ (crc >> 8);
  return crc;
}

struct GenFile {
  std::string path;  // relative, '/' separated
  uint64_t length = 0;
  uint32_t crc32 = 0;
};

int checksum_file(const std::string &path, uint64_t &length, uint32_t &crc) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return io_fail(errno, path);
  std::vector<unsigned char> buf(1 << 16);
  uint32_t c = 0xFFFFFFFFu;
  uint64_t len = 0;
  for (;;) {
    const ssize_t r = ::read(fd, buf.data(), buf.size());
    if (r < 0) {
      const int e = errno;
      if (e == EINTR) continue;
      ::close(fd);
      return io_fail(e, path);
    }
    if (r == 0) break;
    c = crc32_update(c, buf.data(), static_cast<size_t>(r));
    len += static_cast<uint64_t>(r);
  }
  ::close(fd);
  length = len;
  crc = ~c;
  return VG_OK;
}

// Regular files below `dir` (recursively) except the inventory itself;
// symlinks and other entries are errors (generation.rs:409-455).
int collect_files(const std::string &root, const std::string &rel, std::vector<GenFile> &files) {
  const std::string dir = rel.empty() ? root : root + "/" + rel;
  DIR *dp = ::opendir(dir.c_str());
  if (!dp) return io_fail(errno, dir);
  std::vector<std::string> names;
  while (struct dirent *e = ::readdir(dp)) {
    const std::string name = e->d_name;
    if (name != "." && name != "..") names.push_back(name);
  }
  ::closedir(dp);
  for (const std::string &name : names) {
    const std::string r = rel.empty() ? name : rel + "/" + name;
    struct stat sb;
    if (::lstat((root + "/" + r).c_str(), &sb) != 0) return io_fail(errno, root + "/" + r);
    if (S_ISLNK(sb.st_mode)) return format_fail("generation contains symlink " + root + "/" + r);
    if (S_ISDIR(sb.st_mode)) {
      if (int s = collect_files(root, r, files)) return s;
    } else if (S_ISREG(sb.st_mode)) {
      if (r == "GENERATION.json") continue;
      GenFile f;
      f.path = r;
      if (int s = checksum_file(root + "/" + r, f.length, f.crc32)) return s;
      files.push_back(std::move(f));
    } else {
      return format_fail("generation contains unsupported entry " + root + "/" + r);
    }
  }
  return VG_OK;
}

int fsync_path(const std::string &path, bool directory) {
  const int fd = ::open(path.c_str(), directory ? (O_RDONLY | O_DIRECTORY) : O_RDONLY);
  if (fd < 0) return io_fail(errno, path);
  const int r = ::fsync(fd);
  const int e = errno;
  ::close(fd);
  return r == 0 ? VG_OK : io_fail(e, path);
}

// CURRENT's generation id, or "" when there is no CURRENT (not_found set).
int read_current(const std::string &root, std::string &id, bool &not_found) {
  not_found = false;
  id.clear();
  std::string text;
  const std::string path = root + "/CURRENT";
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    if (errno == ENOENT) {
      not_found = true;
      return VG_OK;
    }
    return io_fail(errno, path);
  }
  ::close(fd);
  if (int s = read_file(path, text)) return s;
  size_t a = 0, b = text.size();
  while (a < b && std::isspace(static_cast<unsigned char>(text[a]))) ++a;
  while (b > a && std::isspace(static_cast<unsigned char>(text[b - 1]))) --b;
  id = text.substr(a, b - a);
  return VG_OK;
}

// generation.rs:481-488
bool safe_generation_id(const std::string &id) {
  return !id.empty() && id != "." && id != ".." && id.find('/') == std::string::npos &&
         id.find('\\') == std::string::npos;
}

// generation.rs:191-205: the directory CURRENT names, which must be a real
// directory below generations/.
int open_current(const std::string &root, std::string &dir) {
  std::string id;
  bool none = false;
  if (int s = read_current(root, id, none)) return s;
  if (none) return fail(VG_ERR_NOT_FOUND, "no CURRENT generation pointer in " + root);
  if (!safe_generation_id(id)) return format_fail("CURRENT must contain one safe generation basename");
  dir = root + "/generations/" + id;
  struct stat sb;
  if (::lstat(dir.c_str(), &sb) != 0) return io_fail(errno, dir);
  if (S_ISLNK(sb.st_mode) || !S_ISDIR(sb.st_mode))
    return format_fail("current generation " + dir + " is not a directory");
  return VG_OK;
}

std::string inventory_text(const std::vector<GenFile> &files) {  // serde_json pretty form
  std::string o = "{\n  \"version\": 1,\n  \"files\": [";
  for (size_t i = 0; i < files.size(); ++i) {
    o += i ? ",\n    {\n" : "\n    {\n";
    o += "      \"path\": ";
    json_string(o, files[i].path);
    o += ",\n      \"length\": " + std::to_string(files[i].length) + ",\n";
    o += "      \"crc32\": " + std::to_string(files[i].crc32) + "\n    }";
  }
  o += files.empty() ? "]\n}" : "\n  ]\n}";
  return o;
}

int write_whole(const std::string &path, const std::string &data) {
  const int fd = ::open(path.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
  if (fd < 0) return io_fail(errno, path);
  size_t off = 0;
  while (off < data.size()) {
    const ssize_t w = ::write(fd, data.data() + off, data.size() - off);
    if (w < 0) {
      if (errno == EINTR) continue;
      const int e = errno;
      ::close(fd);
      return io_fail(e, path);
    }
    off += static_cast<size_t>(w);
  }
  const int r = ::fsync(fd);
  const int e = errno;
  ::close(fd);
  return r == 0 ? VG_OK : io_fail(e, path);
}

std::atomic<uint64_t> g_generation_sequence{0};

// generation.rs:472-479
std::string unique_generation_id() {
  const auto nanos = std::chrono::duration_cast<std::chrono::nanoseconds>(
                         std::chrono::system_clock::now().time_since_epoch())
                         .count();
  return std::to_string(nanos) + "-" + std::to_string(::getpid()) + "-" +
         std::to_string(g_generation_sequence.fetch_add(1));
}

// generation.rs:285-365: every file of dir against its GENERATION.json.
int verify_generation_dir(const std::string &dir) {
  std::string text;
  {
    const std::string path = dir + "/GENERATION.json";
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
      if (errno == ENOENT) return format_fail("generation inventory " + path + " is missing");
      return io_fail(errno, path);
    }
    ::close(fd);
    if (int s = read_file(path, text)) return s;
  }
  JVal root;
  std::string err;
  if (!parse_json(text, root, err) || root.kind != JVal::Obj)
    return format_fail("invalid generation inventory: " + (err.empty() ? std::string("not an object") : err));
  Fields f{root, "inventory"};
  uint64_t version = 0;
  if (!f.u64("version", version)) return format_fail("invalid generation inventory: " + f.err);
  if (version != 1) return format_fail("unsupported generation inventory version " + std::to_string(version));
  const JVal *arr = f.need("files", JVal::Arr);
  if (!arr) return format_fail("invalid generation inventory: " + f.err);
  std::vector<GenFile> listed;
  for (const JVal &e : arr->arr) {
    Fields ef{e, "inventory file"};
    const JVal *path = ef.need("path", JVal::Str);
    GenFile g;
    uint64_t crc = 0;
    if (!path || !ef.u64("length", g.length) || !ef.u64("crc32", crc) || crc > 0xffffffffull)
      return format_fail("invalid generation inventory: " + ef.err);
    g.path = path->text;
    g.crc32 = static_cast<uint32_t>(crc);
    if (g.path.empty() || g.path[0] == '/' || g.path.find('\\') != std::string::npos ||
        g.path.find("..") != std::string::npos)
      return format_fail("invalid generation file path " + g.path);
    if (g.path == "GENERATION.json") return format_fail("GENERATION.json cannot inventory itself");
    listed.push_back(std::move(g));
  }
  for (size_t i = 1; i < listed.size(); ++i)
    if (!(listed[i - 1].path < listed[i].path))
      return format_fail("generation inventory paths must be strictly sorted and unique");
  std::vector<GenFile> actual;
  if (int s = collect_files(dir, "", actual)) return s;
  for (const GenFile &a : actual) {
    auto it = std::lower_bound(listed.begin(), listed.end(), a,
                               [](const GenFile &x, const GenFile &y) { return x.path < y.path; });
    if (it == listed.end() || it->path != a.path)
      return format_fail("generation file " + a.path + " is absent from GENERATION.json inventory");
    if (it->length != a.length)
      return format_fail("generation file " + a.path + " length mismatch: expected " + std::to_string(it->length) +
                         ", got " + std::to_string(a.length));
    if (it->crc32 != a.crc32)
      return format_fail("generation file " + a.path + " checksum mismatch: expected " + std::to_string(it->crc32) +
                         ", got " + std::to_string(a.crc32));
  }
  if (listed.size() != actual.size())
    return format_fail("GENERATION.json lists a file that is missing from the generation");
  return VG_OK;
}

// search.rs:916-935 with GenerationWriter (generation.rs:30-140): stage the
// snapshot, check it, inventory it, then publish it under the advisory lock
// by renaming it into generations/ and replacing CURRENT atomically.
int save_generation(const vg_index *ix, const std::string &root) {
  const std::string gens = root + "/generations";
  if (int s = make_dirs(gens)) return s;
  std::string expected;
  bool none = false;
  if (int s = read_current(root, expected, none)) return s;
  const std::string id = unique_generation_id();
  const std::string staging = gens + "/.staging-" + id;
  if (::mkdir(staging.c_str(), 0755) != 0) return io_fail(errno, staging);
  if (int s = save_dir(ix, staging, true)) return s;
  {  // search.rs:1018-1031: the staged snapshot must read back
    SnapshotState st;
    std::string text;
    if (int s = read_file(staging + "/manifest.json", text)) return s;
    if (text.find("\"generation_components\"") == std::string::npos)
      return format_fail("IVF-PQ generation manifest is missing its component inventory");
    if (int s = read_snapshot(staging, st)) return s;
  }
  const std::string lock_path = root + "/.PUBLISH.lock";
  const int lock = ::open(lock_path.c_str(), O_WRONLY | O_CREAT, 0644);
  if (lock < 0) return io_fail(errno, lock_path);
  struct LockGuard {
    int fd;
    ~LockGuard() {
      ::flock(fd, LOCK_UN);
      ::close(fd);
    }
  };
  if (::flock(lock, LOCK_EX | LOCK_NB) != 0) {
    const int e = errno;
    ::close(lock);
    if (e == EWOULDBLOCK) return fail(VG_ERR_IO, "lock failed on " + lock_path + ": another generation publisher holds the advisory lock");
    return io_fail(e, lock_path);
  }
  LockGuard guard{lock};
  std::string now;
  if (int s = read_current(root, now, none)) return s;
  if (now != expected)
    return fail(VG_ERR_IO, "lock failed on " + root + "/CURRENT: CURRENT changed while this generation was being built");
  std::vector<GenFile> files;
  if (int s = collect_files(staging, "", files)) return s;
  std::sort(files.begin(), files.end(), [](const GenFile &a, const GenFile &b) { return a.path < b.path; });
  if (int s = write_whole(staging + "/GENERATION.json", inventory_text(files))) return s;
  if (int s = fsync_path(staging, true)) return s;
  const std::string published = gens + "/" + id;
  if (::rename(staging.c_str(), published.c_str()) != 0) return io_fail(errno, published);
  if (int s = fsync_path(gens, true)) return s;
  const std::string tmp = root + "/.CURRENT.tmp." + std::to_string(::getpid()) + "." +
                          std::to_string(g_generation_sequence.fetch_add(1));
  if (int s = write_whole(tmp, id + "\n")) {
    ::unlink(tmp.c_str());
    return s;
  }
  if (::rename(tmp.c_str(), (root + "/CURRENT").c_str()) != 0) {
    const int e = errno;
    ::unlink(tmp.c_str());
    return io_fail(e, root + "/CURRENT");
  }
  return fsync_path(root, true);
}

}  // namespace

namespace vg {

int parse_metadata(const char *json, const std::string &field, int *category, std::string *canonical) {
  JVal root;
  std::string err;
  if (!json || !parse_json(json, root, err)) return fail(VG_ERR_INVALID_PARAMETER, "metadata is not valid JSON: " + err);
  if (root.kind != JVal::Obj) return fail(VG_ERR_INVALID_PARAMETER, "metadata must be a JSON object");
  *category = -1;
  for (const auto &kv : root.obj) {
    std::string tag;
    if (!metadata_value(kv.second, tag))
      return fail(VG_ERR_INVALID_PARAMETER, "metadata value of `" + kv.first +
                                                "` must be {\"Int\"|\"Float\"|\"Str\"|\"Bool\": value}");
    if (kv.first == field)
      if (int s = int_category(kv.second, tag, category, false)) return s;
  }
  canonical->clear();
  json_dump(*canonical, root);
  return VG_OK;
}

int parse_filter_category(const char *value_json, int *category) {
  JVal v;
  std::string err, tag;
  if (!value_json || !parse_json(value_json, v, err) || !metadata_value(v, tag))
    return fail(VG_ERR_INVALID_PARAMETER, "filter value must be {\"Int\"|\"Float\"|\"Str\"|\"Bool\": value}");
  return int_category(v, tag, category, true);
}

}  // namespace vg

extern "C" {

int vg_ivfpq_save(const vg_index *ix, const char *dir) {
  if (!ix || !dir || !*dir) return fail(VG_ERR_INVALID_PARAMETER, "null index or directory");
  return save_dir(ix, std::string(dir), false);
}

int vg_ivfpq_save_generation(const vg_index *ix, const char *root) {
  if (!ix || !root || !*root) return fail(VG_ERR_INVALID_PARAMETER, "null index or directory");
  return save_generation(ix, std::string(root));
}

int vg_ivfpq_load_generation(const char *root, int device, vg_index **out) {
  if (!root || !*root || !out) return fail(VG_ERR_INVALID_PARAMETER, "null directory or output");
  *out = nullptr;
  std::string dir;
  if (int s = open_current(std::string(root), dir)) return s;
  return vg_ivfpq_load(dir.c_str(), device, out);
}

int vg_generation_current(const char *root, char *out, size_t len) {
  if (!root || !*root || !out || len == 0) return fail(VG_ERR_INVALID_PARAMETER, "null directory or output");
  std::string dir;
  if (int s = open_current(std::string(root), dir)) return s;
  if (dir.size() + 1 > len) return fail(VG_ERR_INVALID_PARAMETER, "output buffer too small for the generation path");
  std::memcpy(out, dir.c_str(), dir.size() + 1);
  return VG_OK;
}

int vg_verify_generation(const char *dir) {
  if (!dir || !*dir) return fail(VG_ERR_INVALID_PARAMETER, "null directory");
  return verify_generation_dir(std::string(dir));
}

int vg_ivfpq_load(const char *dir, int device, vg_index **out) {
  if (!dir || !*dir || !out) return fail(VG_ERR_INVALID_PARAMETER, "null directory or output");
  *out = nullptr;
  SnapshotState st;
  if (int s = read_snapshot(std::string(dir), st)) return s;
  const size_t dim = st.dim;
  vg_index *ix = nullptr;
  if (int s = vg_ivfpq_create(dim, &st.params, device, &ix)) {
    if (s == VG_ERR_CUDA || s == VG_ERR_OUT_OF_MEMORY) return s;
    // a shape the index rejects describes an invalid snapshot
    char why[512];
    vg_last_error(why, sizeof(why));
    return fail(VG_ERR_FORMAT, std::string("IVF-PQ snapshot parameters are invalid: ") + why);
  }
  if (int s = vg::snapshot_adopt(ix, st)) {
    vg_ivfpq_destroy(ix);
    return s;
  }
  *out = ix;
  return VG_OK;
}

}  // extern "C"
