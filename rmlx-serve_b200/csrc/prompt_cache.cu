// Prompt cache save/load (crates/rmlx-serve-cache/src/prompt_cache.rs:63-210):
// a sequence's K/V as a safetensors file with one [seq_len, head_dim] tensor
// per (layer, head, keys|values) named layer_{l}_head_{h}_{keys|values}, and
// optional string metadata under "__metadata__".
//
// The file is written as the safetensors crate serialises it (the reference
// calls safetensors::tensor::serialize, Cargo.lock pins safetensors 0.4.5):
//   u64 little-endian header length N, N bytes of compact JSON, tensor data;
//   the JSON holds "__metadata__" first (when given), then the tensors in
//   data order, each {"dtype":..,"shape":[..],"data_offsets":[begin,end]};
//   tensors are ordered by dtype and then by name (bytewise), and the JSON
//   is padded with spaces to a multiple of 8 bytes.
//
// Device side: save gathers the sequence's rows of every layer through the
// pool's own gather (dequantised for a quantised pool), load writes them
// into caller-allocated blocks with the pool's append (quantising for a
// quantised pool).  Heads are named by their global index (head_offset + h),
// so a pool that holds a shard of the heads reads its own heads from a file
// that holds all of them.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "kv_pool_internal.cuh"

using namespace rmlx;

namespace {

const char* st_dtype(int dt) {
  switch (dt) {
    case RMLX_F32: return "F32";
    case RMLX_F16: return "F16";
    case RMLX_BF16: return "BF16";
  }
  return nullptr;
}
int esize(int dt) { return dt == RMLX_F32 ? 4 : 2; }

std::string tensor_name(int l, int h, bool values) {
  return "layer_" + std::to_string(l) + "_head_" + std::to_string(h) + (values ? "_values" : "_keys");
}

// JSON string as serde_json writes it: ", \ and control characters escaped,
// everything else (UTF-8 included) verbatim.
void json_str(std::string& o, const std::string& s) {
  static const char* hex = "0123456789abcdef";
  o += '"';
  for (unsigned char ch : s) {
    switch (ch) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\b': o += "\\b"; break;
      case '\f': o += "\\f"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (ch < 0x20) {
          o += "\\u00";
          o += hex[ch >> 4];
          o += hex[ch & 15];
        } else {
          o += (char)ch;
        }
    }
  }
  o += '"';
}

// ---- minimal JSON reader for safetensors headers --------------------------
struct JVal {
  enum Kind { NUL, NUM, STR, ARR, OBJ } kind = NUL;
  int64_t num = 0;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* e;
  std::string err;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail_(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  static void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 63));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 63));
      o += (char)(0x80 | (cp & 63));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 63));
      o += (char)(0x80 | ((cp >> 6) & 63));
      o += (char)(0x80 | (cp & 63));
    }
  }
  bool hex4(uint32_t& v) {
    if (e - p < 4) return fail_("truncated \\u escape");
    v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else return fail_("bad \\u escape");
    }
    return true;
  }
  bool string(std::string& o) {
    if (p >= e || *p != '"') return fail_("expected string");
    ++p;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return fail_("truncated escape");
        char c = *p++;
        switch (c) {
          case '"': o += '"'; break;
          case '\\': o += '\\'; break;
          case '/': o += '/'; break;
          case 'b': o += '\b'; break;
          case 'f': o += '\f'; break;
          case 'n': o += '\n'; break;
          case 'r': o += '\r'; break;
          case 't': o += '\t'; break;
          case 'u': {
            uint32_t cp;
            if (!hex4(cp)) return false;
            if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
              uint32_t lo;
              if (e - p < 2 || p[0] != '\\' || p[1] != 'u') return fail_("lone surrogate");
              p += 2;
              if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail_("bad surrogate pair");
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            }
            put_utf8(o, cp);
            break;
          }
          default: return fail_("bad escape");
        }
      } else {
        o += *p++;
      }
    }
    if (p >= e) return fail_("unterminated string");
    ++p;
    return true;
  }
  bool value(JVal& v, int depth) {
    if (depth > 8) return fail_("header nested too deeply");
    ws();
    if (p >= e) return fail_("unexpected end of header");
    if (*p == '{') {
      v.kind = JVal::OBJ;
      ++p;
      ws();
      if (p < e && *p == '}') {
        ++p;
        return true;
      }
      for (;;) {
        ws();
        std::string k;
        if (!string(k)) return false;
        ws();
        if (p >= e || *p != ':') return fail_("expected ':'");
        ++p;
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == '}') {
          ++p;
          return true;
        }
        return fail_("expected ',' or '}'");
      }
    }
    if (*p == '[') {
      v.kind = JVal::ARR;
      ++p;
      ws();
      if (p < e && *p == ']') {
        ++p;
        return true;
      }
      for (;;) {
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.arr.push_back(std::move(x));
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == ']') {
          ++p;
          return true;
        }
        return fail_("expected ',' or ']'");
      }
    }
    if (*p == '"') {
      v.kind = JVal::STR;
      return string(v.str);
    }
    if (*p == '-' || (*p >= '0' && *p <= '9')) {
      v.kind = JVal::NUM;
      bool neg = *p == '-';
      if (neg) ++p;
      if (p >= e || *p < '0' || *p > '9') return fail_("bad number");
      uint64_t x = 0;
      while (p < e && *p >= '0' && *p <= '9') {
        if (x > (uint64_t)INT64_MAX / 10) return fail_("number too large");
        x = x * 10 + (uint64_t)(*p++ - '0');
      }
      if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return fail_("non-integer number in header");
      if (x > (uint64_t)INT64_MAX) return fail_("number too large");
      v.num = neg ? -(int64_t)x : (int64_t)x;
      return true;
    }
    if (e - p >= 4 && !strncmp(p, "null", 4)) {
      p += 4;
      return true;
    }
    return fail_("unexpected character in header");
  }
};

struct Entry {
  int layer, head;
  bool values;
  int64_t rows, cols, begin, end;
};

struct Header {
  int dtype = -1;  // common dtype of the entries, -1 when there are none
  std::vector<Entry> entries;
  std::string metadata_json;  // the "__metadata__" object as JSON ("" when absent)
  int64_t data_start = 0, file_size = 0;
};

bool parse_name(const std::string& n, int& l, int& h, bool& values) {
  // layer_{l}_head_{h}_{keys|values}
  unsigned long a, b;
  char tail[16];
  int used = 0;
  if (sscanf(n.c_str(), "layer_%lu_head_%lu_%15s%n", &a, &b, tail, &used) != 3 || used != (int)n.size()) return false;
  if (std::string(tail) == "keys") values = false;
  else if (std::string(tail) == "values") values = true;
  else return false;
  if (a > 1000000 || b > 1000000) return false;
  // reject leading zeros / signs so that names map one-to-one to indices
  if (n != tensor_name((int)a, (int)b, values)) return false;
  l = (int)a;
  h = (int)b;
  return true;
}

rmlx_status read_header(FILE* f, Header& hd) {
  if (fseek(f, 0, SEEK_END) != 0) return fail(RMLX_E_BAD_ARG, "cannot seek prompt cache file");
  hd.file_size = ftell(f);
  rewind(f);
  uint8_t lenb[8];
  if (hd.file_size < 8 || fread(lenb, 1, 8, f) != 8) return fail(RMLX_E_BAD_ARG, "prompt cache file too short");
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | lenb[i];
  if (n > (uint64_t)(hd.file_size - 8) || n > (100u << 20)) return fail(RMLX_E_BAD_ARG, "bad safetensors header length");
  std::string js((size_t)n, '\0');
  if (n && fread(&js[0], 1, (size_t)n, f) != n) return fail(RMLX_E_BAD_ARG, "cannot read safetensors header");
  hd.data_start = 8 + (int64_t)n;
  JParser jp{js.data(), js.data() + js.size(), {}};
  JVal root;
  if (!jp.value(root, 0)) return fail(RMLX_E_BAD_ARG, "safetensors header: %s", jp.err.c_str());
  jp.ws();
  if (jp.p != jp.e || root.kind != JVal::OBJ) return fail(RMLX_E_BAD_ARG, "safetensors header is not one JSON object");
  const int64_t data_len = hd.file_size - hd.data_start;
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      if (kv.second.kind != JVal::OBJ) return fail(RMLX_E_BAD_ARG, "__metadata__ must be an object");
      std::string o = "{";
      bool first = true;
      for (auto& m : kv.second.obj) {
        if (m.second.kind != JVal::STR) return fail(RMLX_E_BAD_ARG, "__metadata__ values must be strings");
        if (!first) o += ',';
        first = false;
        json_str(o, m.first);
        o += ':';
        json_str(o, m.second.str);
      }
      hd.metadata_json = o + "}";
      continue;
    }
    Entry en;
    if (!parse_name(kv.first, en.layer, en.head, en.values))
      return fail(RMLX_E_BAD_ARG, "tensor '%s' is not layer_{l}_head_{h}_{keys|values}", kv.first.c_str());
    const JVal& t = kv.second;
    const JVal *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
    if (t.kind != JVal::OBJ || !dt || !sh || !off || dt->kind != JVal::STR || sh->kind != JVal::ARR ||
        off->kind != JVal::ARR || off->arr.size() != 2)
      return fail(RMLX_E_BAD_ARG, "tensor '%s': bad entry", kv.first.c_str());
    int d = -1;
    for (int c : {RMLX_F32, RMLX_F16, RMLX_BF16})
      if (dt->str == st_dtype(c)) d = c;
    if (d < 0) return fail(RMLX_E_BAD_ARG, "tensor '%s': dtype %s is not F32, F16 or BF16", kv.first.c_str(),
                           dt->str.c_str());
    if (hd.dtype >= 0 && d != hd.dtype) return fail(RMLX_E_BAD_ARG, "tensors of different dtypes");
    hd.dtype = d;
    if (sh->arr.size() != 2 || sh->arr[0].kind != JVal::NUM || sh->arr[1].kind != JVal::NUM || sh->arr[0].num < 0 ||
        sh->arr[1].num < 0)
      return fail(RMLX_E_BAD_ARG, "tensor '%s': shape must be [seq_len, head_dim]", kv.first.c_str());
    en.rows = sh->arr[0].num;
    en.cols = sh->arr[1].num;
    if (off->arr[0].kind != JVal::NUM || off->arr[1].kind != JVal::NUM)
      return fail(RMLX_E_BAD_ARG, "tensor '%s': bad data_offsets", kv.first.c_str());
    en.begin = off->arr[0].num;
    en.end = off->arr[1].num;
    if (en.rows > (int64_t)1 << 31 || en.cols > (int64_t)1 << 20 || en.begin < 0 || en.end < en.begin ||
        en.end > data_len || en.end - en.begin != en.rows * en.cols * esize(d))
      return fail(RMLX_E_BAD_ARG, "tensor '%s': data_offsets do not match its shape or the file", kv.first.c_str());
    hd.entries.push_back(en);
  }
  return RMLX_OK;
}

struct FileCloser {
  void operator()(FILE* f) const {
    if (f) fclose(f);
  }
};
using FilePtr = std::unique_ptr<FILE, FileCloser>;

// Shape of a file as a cache: layers [0, L), heads [0, H) by the largest
// indices present, counted from 0 as load_prompt_cache does (an empty file
// is 1 layer x 1 head, prompt_cache.rs:151-167); one seq_len and head_dim.
rmlx_status file_shape(const Header& hd, int32_t* L, int32_t* H, int32_t* seq, int32_t* dim) {
  int ml = 0, mh = 0;
  int64_t rows = -1, cols = -1;
  for (auto& en : hd.entries) {
    ml = std::max(ml, en.layer);
    mh = std::max(mh, en.head);
    if (rows >= 0 && (en.rows != rows || en.cols != cols))
      return fail(RMLX_E_BAD_ARG, "tensors of different shapes");
    rows = en.rows;
    cols = en.cols;
  }
  *L = ml + 1;
  *H = mh + 1;
  *seq = (int32_t)std::max<int64_t>(rows, 0);
  *dim = (int32_t)std::max<int64_t>(cols, 0);
  return RMLX_OK;
}

// Host arrays [layers][heads][seq_len][head_dim] for keys and values.
rmlx_status write_file(const char* path, int32_t L, int32_t H, int32_t head_offset, int32_t seq, int32_t D, int32_t dt,
                       const uint8_t* keys, const uint8_t* values, const char* const* mk, const char* const* mv,
                       int32_t nmeta) {
  const int64_t tbytes = (int64_t)seq * D * esize(dt);
  struct T {
    std::string name;
    const uint8_t* data;
  };
  std::vector<T> ts;
  if (seq > 0) {  // the reference writes no tensor for an empty layer (prompt_cache.rs:79)
    for (int l = 0; l < L; ++l)
      for (int h = 0; h < H; ++h)
        for (int v = 0; v < 2; ++v)
          ts.push_back({tensor_name(l, head_offset + h, v == 1),
                        (v ? values : keys) + ((int64_t)l * H + h) * tbytes});
  }
  std::sort(ts.begin(), ts.end(), [](const T& a, const T& b) { return a.name < b.name; });
  std::string js = "{";
  bool first = true;
  if (nmeta > 0) {
    js += "\"__metadata__\":{";
    for (int i = 0; i < nmeta; ++i) {
      if (i) js += ',';
      json_str(js, mk[i]);
      js += ':';
      json_str(js, mv[i]);
    }
    js += '}';
    first = false;
  }
  int64_t off = 0;
  for (auto& t : ts) {
    if (!first) js += ',';
    first = false;
    json_str(js, t.name);
    js += ":{\"dtype\":\"";
    js += st_dtype(dt);
    js += "\",\"shape\":[" + std::to_string(seq) + "," + std::to_string(D) + "],\"data_offsets\":[" +
          std::to_string(off) + "," + std::to_string(off + tbytes) + "]}";
    off += tbytes;
  }
  js += '}';
  js.append((8 - js.size() % 8) % 8, ' ');
  FilePtr f(fopen(path, "wb"));
  if (!f) return fail(RMLX_E_BAD_ARG, "cannot open '%s' for writing", path);
  uint8_t lenb[8];
  uint64_t n = js.size();
  for (int i = 0; i < 8; ++i) lenb[i] = (uint8_t)(n >> (8 * i));
  bool ok = fwrite(lenb, 1, 8, f.get()) == 8 && fwrite(js.data(), 1, js.size(), f.get()) == js.size();
  for (auto& t : ts) ok = ok && fwrite(t.data, 1, (size_t)tbytes, f.get()) == (size_t)tbytes;
  if (!ok) return fail(RMLX_E_BAD_ARG, "write to '%s' failed", path);
  if (fclose(f.release()) != 0) return fail(RMLX_E_BAD_ARG, "write to '%s' failed", path);
  return RMLX_OK;
}

rmlx_status read_file(const char* path, int32_t L, int32_t H, int32_t head_offset, int32_t D, int32_t dt,
                      uint8_t* keys, uint8_t* values, size_t cap, int32_t* seq_out) {
  FilePtr f(fopen(path, "rb"));
  if (!f) return fail(RMLX_E_BAD_ARG, "cannot open '%s'", path);
  Header hd;
  rmlx_status s = read_header(f.get(), hd);
  if (s != RMLX_OK) return s;
  int32_t fl, fh, seq, dim;
  if ((s = file_shape(hd, &fl, &fh, &seq, &dim)) != RMLX_OK) return s;
  if (hd.entries.empty()) {
    *seq_out = 0;
    return RMLX_OK;
  }
  if (hd.dtype != dt) return fail(RMLX_E_BAD_ARG, "file dtype %s differs from the cache's", st_dtype(hd.dtype));
  if (dim != D) return fail(RMLX_E_BAD_ARG, "file head_dim %d differs from the cache's %d", dim, D);
  if (fl > L) return fail(RMLX_E_BAD_ARG, "file has %d layers, the cache %d", fl, L);
  const int64_t tbytes = (int64_t)seq * D * esize(dt);
  if ((uint64_t)fl * H * tbytes > cap) return fail(RMLX_E_BAD_ARG, "output buffers too small for %d tokens", seq);
  std::map<std::pair<int, int>, std::pair<const Entry*, const Entry*>> kvs;
  for (auto& en : hd.entries) {
    auto& slot = kvs[{en.layer, en.head}];
    (en.values ? slot.second : slot.first) = &en;
  }
  for (int l = 0; l < fl; ++l)
    for (int h = 0; h < H; ++h) {
      auto it = kvs.find({l, head_offset + h});
      if (it == kvs.end() || !it->second.first || !it->second.second)
        return fail(RMLX_E_BAD_ARG, "file lacks the keys or values of layer %d head %d", l, head_offset + h);
      for (int v = 0; v < 2; ++v) {
        const Entry* en = v ? it->second.second : it->second.first;
        uint8_t* dst = (v ? values : keys) + ((int64_t)l * H + h) * tbytes;
        if (fseek(f.get(), (long)(hd.data_start + en->begin), SEEK_SET) != 0 ||
            (tbytes && fread(dst, 1, (size_t)tbytes, f.get()) != (size_t)tbytes))
          return fail(RMLX_E_BAD_ARG, "cannot read tensor data of '%s'", path);
      }
    }
  *seq_out = seq;
  return RMLX_OK;
}

struct DevBuf {
  void* p = nullptr;
  cudaStream_t st = nullptr;
  ~DevBuf() {
    if (p) cudaFreeAsync(p, st);
  }
};

}  // namespace

extern "C" {

rmlx_status rmlx_prompt_cache_write(const char* path, int32_t num_layers, int32_t num_kv_heads, int32_t head_offset,
                                    int32_t seq_len, int32_t head_dim, int32_t dtype, const void* keys,
                                    const void* values, const char* const* meta_keys, const char* const* meta_values,
                                    int32_t num_meta) {
  if (!path) return fail(RMLX_E_BAD_ARG, "NULL path");
  if (num_layers < 0 || num_kv_heads < 0 || head_offset < 0 || seq_len < 0 || head_dim < 0 || num_meta < 0)
    return fail(RMLX_E_BAD_ARG, "negative size");
  if (!st_dtype(dtype)) return fail(RMLX_E_BAD_ARG, "dtype must be F32, F16 or BF16");
  if (seq_len > 0 && num_layers * num_kv_heads > 0 && (!keys || !values)) return fail(RMLX_E_BAD_ARG, "NULL keys or values");
  if (num_meta > 0 && (!meta_keys || !meta_values)) return fail(RMLX_E_BAD_ARG, "NULL metadata");
  for (int i = 0; i < num_meta; ++i)
    if (!meta_keys[i] || !meta_values[i]) return fail(RMLX_E_BAD_ARG, "NULL metadata entry");
  return write_file(path, num_layers, num_kv_heads, head_offset, seq_len, head_dim, dtype,
                    static_cast<const uint8_t*>(keys), static_cast<const uint8_t*>(values), meta_keys, meta_values,
                    num_meta);
}

rmlx_status rmlx_prompt_cache_info(const char* path, int32_t* num_layers, int32_t* num_kv_heads, int32_t* seq_len,
                                   int32_t* head_dim, int32_t* dtype, char* metadata_json, size_t metadata_cap,
                                   size_t* metadata_len) {
  if (!path || !num_layers || !num_kv_heads || !seq_len || !head_dim || !dtype) return fail(RMLX_E_BAD_ARG, "NULL argument");
  FilePtr f(fopen(path, "rb"));
  if (!f) return fail(RMLX_E_BAD_ARG, "cannot open '%s'", path);
  Header hd;
  rmlx_status s = read_header(f.get(), hd);
  if (s != RMLX_OK) return s;
  if ((s = file_shape(hd, num_layers, num_kv_heads, seq_len, head_dim)) != RMLX_OK) return s;
  *dtype = hd.dtype;
  if (metadata_len) *metadata_len = hd.metadata_json.size();
  if (metadata_json && metadata_cap) {
    const size_t n = std::min(metadata_cap - 1, hd.metadata_json.size());
    memcpy(metadata_json, hd.metadata_json.data(), n);
    metadata_json[n] = '\0';
  }
  return RMLX_OK;
}

rmlx_status rmlx_prompt_cache_read(const char* path, int32_t num_layers, int32_t num_kv_heads, int32_t head_offset,
                                   int32_t head_dim, int32_t dtype, void* keys, void* values, size_t cap_bytes,
                                   int32_t* seq_len) {
  if (!path || !seq_len) return fail(RMLX_E_BAD_ARG, "NULL argument");
  if (num_layers < 0 || num_kv_heads < 0 || head_offset < 0 || head_dim <= 0) return fail(RMLX_E_BAD_ARG, "bad shape");
  if (!st_dtype(dtype)) return fail(RMLX_E_BAD_ARG, "dtype must be F32, F16 or BF16");
  if (cap_bytes && (!keys || !values)) return fail(RMLX_E_BAD_ARG, "NULL keys or values");
  return read_file(path, num_layers, num_kv_heads, head_offset, head_dim, dtype, static_cast<uint8_t*>(keys),
                   static_cast<uint8_t*>(values), cap_bytes, seq_len);
}

rmlx_status rmlx_prompt_cache_save(rmlx_kv_pool* p, const int32_t* block_ids, int32_t num_block_ids, int32_t seq_len,
                                   const char* path, const char* const* meta_keys, const char* const* meta_values,
                                   int32_t num_meta, void* stream) {
  if (!p || !path) return fail(RMLX_E_BAD_ARG, "NULL pool or path");
  const rmlx_pool_config& c = p->cfg;
  if (seq_len < 0 || num_block_ids < 0) return fail(RMLX_E_BAD_ARG, "negative seq_len or num_block_ids");
  if ((int64_t)num_block_ids * c.block_size < seq_len) return fail(RMLX_E_BAD_ARG, "block_ids hold fewer than seq_len rows");
  if (seq_len > 0 && !block_ids) return fail(RMLX_E_BAD_ARG, "NULL block_ids");
  const int L = c.num_layers, H = c.num_kv_heads, D = c.head_dim, es = esize(c.dtype);
  const size_t layer_bytes = (size_t)H * seq_len * D * es;
  std::vector<uint8_t> keys((size_t)L * layer_bytes), values((size_t)L * layer_bytes);
  if (seq_len > 0) {
    DeviceGuard dg(p->device);
    cudaStream_t st = (cudaStream_t)stream;
    DevBuf bt, lens, ok, ov;
    bt.st = lens.st = ok.st = ov.st = st;
    if (cudaMallocAsync(&bt.p, (size_t)num_block_ids * 4, st) != cudaSuccess ||
        cudaMallocAsync(&lens.p, 16, st) != cudaSuccess || cudaMallocAsync(&ok.p, layer_bytes, st) != cudaSuccess ||
        cudaMallocAsync(&ov.p, layer_bytes, st) != cudaSuccess)
      return cuda_check(cudaGetLastError(), "prompt cache save: device buffers");
    cudaMemcpyAsync(bt.p, block_ids, (size_t)num_block_ids * 4, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(lens.p, &seq_len, 4, cudaMemcpyHostToDevice, st);
    for (int l = 0; l < L; ++l) {
      rmlx_status s = rmlx_kv_gather(p, l, static_cast<int32_t*>(bt.p), num_block_ids, static_cast<int32_t*>(lens.p),
                                     1, ok.p, ov.p, stream);
      if (s != RMLX_OK) return s;
      cudaMemcpyAsync(keys.data() + l * layer_bytes, ok.p, layer_bytes, cudaMemcpyDeviceToHost, st);
      cudaMemcpyAsync(values.data() + l * layer_bytes, ov.p, layer_bytes, cudaMemcpyDeviceToHost, st);
    }
    rmlx_status s = cuda_check(cudaStreamSynchronize(st), "prompt cache save");
    if (s != RMLX_OK) return s;
    int32_t dev_err = 0;
    if ((s = rmlx_kv_pool_check(p, &dev_err)) != RMLX_OK) return s;
    if (dev_err) return fail(RMLX_E_RANGE, "block id outside the pool (device error bits %d)", dev_err);
  }
  return write_file(path, L, H, c.head_offset, seq_len, D, c.dtype, keys.data(), values.data(), meta_keys,
                    meta_values, num_meta);
}

rmlx_status rmlx_prompt_cache_load(rmlx_kv_pool* p, const char* path, const int32_t* block_ids, int32_t num_block_ids,
                                   int32_t* seq_len, void* stream) {
  if (!p || !path || !seq_len) return fail(RMLX_E_BAD_ARG, "NULL argument");
  const rmlx_pool_config& c = p->cfg;
  const int L = c.num_layers, H = c.num_kv_heads, D = c.head_dim, es = esize(c.dtype);
  int32_t fl, fh, seq, dim, dt;
  rmlx_status s = rmlx_prompt_cache_info(path, &fl, &fh, &seq, &dim, &dt, nullptr, 0, nullptr);
  if (s != RMLX_OK) return s;
  if ((int64_t)num_block_ids * c.block_size < seq) return fail(RMLX_E_BAD_ARG, "block_ids hold fewer than %d rows", seq);
  if (seq > 0 && !block_ids) return fail(RMLX_E_BAD_ARG, "NULL block_ids");
  for (int64_t i = 0; i < (seq + c.block_size - 1) / c.block_size; ++i)
    if (block_ids[i] < 0 || block_ids[i] >= c.num_blocks) return fail(RMLX_E_RANGE, "block id %d out of range", block_ids[i]);
  const size_t layer_bytes = (size_t)H * seq * D * es;
  std::vector<uint8_t> keys((size_t)L * layer_bytes), values((size_t)L * layer_bytes);
  int32_t got = 0;
  if ((s = read_file(path, L, H, c.head_offset, D, c.dtype, keys.data(), values.data(), keys.size(), &got)) != RMLX_OK)
    return s;
  *seq_len = got;
  if (got == 0) return RMLX_OK;
  // one append of all got tokens into the layers the file holds, rows taken
  // from the [layer][head][token][dim] arrays (the reference's per-head layout)
  std::vector<int32_t> slots(got);
  for (int t = 0; t < got; ++t) slots[t] = block_ids[t / c.block_size] * c.block_size + t % c.block_size;
  DeviceGuard dg(p->device);
  cudaStream_t st = (cudaStream_t)stream;
  DevBuf dk, dv, ds;
  dk.st = dv.st = ds.st = st;
  const size_t nbytes = (size_t)fl * layer_bytes;
  if (cudaMallocAsync(&dk.p, nbytes, st) != cudaSuccess || cudaMallocAsync(&dv.p, nbytes, st) != cudaSuccess ||
      cudaMallocAsync(&ds.p, (size_t)got * 4, st) != cudaSuccess)
    return cuda_check(cudaGetLastError(), "prompt cache load: device buffers");
  cudaMemcpyAsync(dk.p, keys.data(), nbytes, cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(dv.p, values.data(), nbytes, cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(ds.p, slots.data(), (size_t)got * 4, cudaMemcpyHostToDevice, st);
  s = rmlx_kv_append(p, 0, fl, dk.p, dv.p, (int64_t)H * got * D, D, (int64_t)got * D, static_cast<int32_t*>(ds.p), got,
                     stream);
  if (s != RMLX_OK) return s;
  s = cuda_check(cudaStreamSynchronize(st), "prompt cache load");  // host staging outlives the copies
  if (s != RMLX_OK) return s;
  return RMLX_OK;
}

}  // extern "C"
