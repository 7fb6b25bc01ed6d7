// Device-direct safetensors checkpoints (the io "save" / io "load" path of
// sheaf/src/interpreter/builtins/safetensors.rs:13-81,200-331).
//
// Save writes what save_safetensors writes for the same tensors, byte for
// byte: entries sorted by key, a compact JSON header whose entry fields are
// in key order ("data_offsets", "dtype", "shape"), padded with spaces so the
// data section starts 8-byte aligned, then the raw little-endian tensor
// bytes. The bytes of each device buffer go to the file through pinned
// staging (no conversion: buffers already hold the file's element type).
//
// Load parses the header (any valid safetensors file, "__metadata__"
// ignored) and streams one tensor at a time into a new device buffer. Element
// types follow decode_raw: F32, F16, BF16 and I32 keep their bytes; F64
// becomes F32; I64, U8 and BOOL become I32 (BOOL as 0 / 1: device buffers have
// no boolean type).
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "runtime.h"

struct sb_safetensors_file_s {
  struct Entry {
    std::string key, dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // relative to the data section
  };
  std::string path;
  uint64_t data_start = 0, data_len = 0;
  std::vector<Entry> entries;  // in key order
};

namespace sb {
namespace {

// ---- a small JSON reader for safetensors headers ----
struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
};

struct JsonReader {
  const std::string& t;
  size_t p = 0;
  std::string err;
  explicit JsonReader(const std::string& s) : t(s) {}
  void ws() {
    while (p < t.size() && std::isspace(static_cast<unsigned char>(t[p]))) ++p;
  }
  bool fail(const char* m) {
    if (err.empty()) err = std::string(m) + " at byte " + std::to_string(p);
    return false;
  }
  bool string(std::string* out) {
    if (p >= t.size() || t[p] != '"') return fail("expected string");
    ++p;
    std::string v;
    while (p < t.size() && t[p] != '"') {
      char ch = t[p++];
      if (ch == '\\') {
        if (p >= t.size()) return fail("bad escape");
        const char e = t[p++];
        switch (e) {
          case 'n': ch = '\n'; break;
          case 't': ch = '\t'; break;
          case 'r': ch = '\r'; break;
          case 'b': ch = '\b'; break;
          case 'f': ch = '\f'; break;
          case 'u': {  // keep ASCII code points, replace the rest
            if (p + 4 > t.size()) return fail("bad \\u escape");
            const unsigned cp = static_cast<unsigned>(std::stoul(t.substr(p, 4), nullptr, 16));
            p += 4;
            ch = cp < 0x80 ? static_cast<char>(cp) : '?';
            break;
          }
          default: ch = e;
        }
      }
      v += ch;
    }
    if (p >= t.size()) return fail("unterminated string");
    ++p;
    *out = std::move(v);
    return true;
  }
  bool value(Json* out, int depth = 0) {
    if (depth > 32) return fail("nesting too deep");
    ws();
    if (p >= t.size()) return fail("unexpected end");
    const char ch = t[p];
    if (ch == '{') {
      ++p;
      out->kind = Json::kObj;
      ws();
      if (p < t.size() && t[p] == '}') {
        ++p;
        return true;
      }
      while (true) {
        ws();
        std::string k;
        if (!string(&k)) return false;
        ws();
        if (p >= t.size() || t[p] != ':') return fail("expected ':'");
        ++p;
        Json v;
        if (!value(&v, depth + 1)) return false;
        out->obj.emplace_back(std::move(k), std::move(v));
        ws();
        if (p < t.size() && t[p] == ',') {
          ++p;
          continue;
        }
        if (p < t.size() && t[p] == '}') {
          ++p;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (ch == '[') {
      ++p;
      out->kind = Json::kArr;
      ws();
      if (p < t.size() && t[p] == ']') {
        ++p;
        return true;
      }
      while (true) {
        Json v;
        if (!value(&v, depth + 1)) return false;
        out->arr.push_back(std::move(v));
        ws();
        if (p < t.size() && t[p] == ',') {
          ++p;
          continue;
        }
        if (p < t.size() && t[p] == ']') {
          ++p;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (ch == '"') {
      out->kind = Json::kStr;
      return string(&out->str);
    }
    if (t.compare(p, 4, "true") == 0 || t.compare(p, 5, "false") == 0) {
      out->kind = Json::kBool;
      out->b = t[p] == 't';
      p += out->b ? 4 : 5;
      return true;
    }
    if (t.compare(p, 4, "null") == 0) {
      p += 4;
      return true;
    }
    size_t q = p;
    while (q < t.size() && (std::isdigit(static_cast<unsigned char>(t[q])) || t[q] == '-' || t[q] == '+' ||
                            t[q] == '.' || t[q] == 'e' || t[q] == 'E'))
      ++q;
    if (q == p) return fail("unexpected character");
    out->kind = Json::kNum;
    out->num = std::stod(t.substr(p, q - p));
    p = q;
    return true;
  }
};

size_t dtype_bytes(const std::string& d) {
  if (d == "F64" || d == "I64") return 8;
  if (d == "F32" || d == "I32") return 4;
  if (d == "F16" || d == "BF16") return 2;
  if (d == "U8" || d == "BOOL") return 1;
  return 0;
}

uint32_t elem_for(const std::string& d) {
  if (d == "F32" || d == "F64") return SB_ELEM_F32;
  if (d == "BF16") return SB_ELEM_BF16;
  if (d == "F16") return SB_ELEM_F16;
  return SB_ELEM_I32;  // I32, I64, U8, BOOL
}

const char* dtype_for(uint32_t elem) {
  switch (elem) {
    case SB_ELEM_F32: return "F32";
    case SB_ELEM_BF16: return "BF16";
    case SB_ELEM_F16: return "F16";
    case SB_ELEM_I32: return "I32";
    default: return nullptr;
  }
}

struct FileCloser {
  void operator()(FILE* f) const {
    if (f) std::fclose(f);
  }
};
using FilePtr = std::unique_ptr<FILE, FileCloser>;

// Two pinned staging chunks, so the file I/O of one overlaps the copy of
// the other.
struct Staging {
  static constexpr size_t kChunk = 32u << 20;
  void* buf[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  ~Staging() {
    for (int i = 0; i < 2; ++i) {
      if (done[i]) cudaEventDestroy(done[i]);
      if (buf[i]) cudaFreeHost(buf[i]);
    }
  }
  sb_status init() {
    for (int i = 0; i < 2; ++i) {
      SB_CUDA_TRY(cudaMallocHost(&buf[i], kChunk));
      SB_CUDA_TRY(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
    }
    return nullptr;
  }
};

sb_status parse_header(const std::string& path, sb_safetensors_file_s* f) {
  FilePtr fp(std::fopen(path.c_str(), "rb"));
  SB_RETURN_IF(!fp, SB_STATUS_NOT_FOUND, "safetensors: cannot open " + path);
  std::fseek(fp.get(), 0, SEEK_END);
  const long file_len = std::ftell(fp.get());
  std::fseek(fp.get(), 0, SEEK_SET);
  SB_RETURN_IF(file_len < 8, SB_STATUS_INVALID_ARGUMENT, "safetensors: file too small");
  unsigned char hb[8];
  SB_RETURN_IF(std::fread(hb, 1, 8, fp.get()) != 8, SB_STATUS_INVALID_ARGUMENT, "safetensors: short read");
  uint64_t hsize = 0;
  for (int i = 7; i >= 0; --i) hsize = (hsize << 8) | hb[i];
  SB_RETURN_IF(hsize > static_cast<uint64_t>(file_len) - 8, SB_STATUS_INVALID_ARGUMENT,
               "safetensors: header size " + std::to_string(hsize) + " exceeds file length " +
                   std::to_string(file_len));
  std::string header(hsize, '\0');
  SB_RETURN_IF(hsize && std::fread(&header[0], 1, hsize, fp.get()) != hsize, SB_STATUS_INVALID_ARGUMENT,
               "safetensors: short read");
  JsonReader r(header);
  Json root;
  SB_RETURN_IF(!r.value(&root) || root.kind != Json::kObj, SB_STATUS_INVALID_ARGUMENT,
               "safetensors: invalid header: " + (r.err.empty() ? std::string("not an object") : r.err));
  f->path = path;
  f->data_start = 8 + hsize;
  f->data_len = static_cast<uint64_t>(file_len) - f->data_start;
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& o = kv.second;
    SB_RETURN_IF(o.kind != Json::kObj, SB_STATUS_INVALID_ARGUMENT, "safetensors: '" + kv.first + "' must be object");
    sb_safetensors_file_s::Entry e;
    e.key = kv.first;
    bool have_dtype = false, have_shape = false, have_off = false;
    for (auto& field : o.obj) {
      if (field.first == "dtype" && field.second.kind == Json::kStr) {
        e.dtype = field.second.str;
        have_dtype = true;
      } else if (field.first == "shape" && field.second.kind == Json::kArr) {
        for (auto& d : field.second.arr) {
          SB_RETURN_IF(d.kind != Json::kNum || d.num < 0, SB_STATUS_INVALID_ARGUMENT,
                       "safetensors: '" + kv.first + "' bad shape");
          e.shape.push_back(static_cast<int64_t>(d.num));
        }
        have_shape = true;
      } else if (field.first == "data_offsets" && field.second.kind == Json::kArr && field.second.arr.size() == 2) {
        e.begin = static_cast<uint64_t>(field.second.arr[0].num);
        e.end = static_cast<uint64_t>(field.second.arr[1].num);
        have_off = true;
      }
    }
    SB_RETURN_IF(!have_dtype, SB_STATUS_INVALID_ARGUMENT, "safetensors: '" + kv.first + "' missing dtype");
    SB_RETURN_IF(!have_shape, SB_STATUS_INVALID_ARGUMENT, "safetensors: '" + kv.first + "' missing shape");
    SB_RETURN_IF(!have_off, SB_STATUS_INVALID_ARGUMENT, "safetensors: '" + kv.first + "' missing data_offsets");
    const size_t eb = dtype_bytes(e.dtype);
    SB_RETURN_IF(!eb, SB_STATUS_UNIMPLEMENTED, "safetensors: '" + kv.first + "': unsupported dtype '" + e.dtype + "'");
    SB_RETURN_IF(e.end > f->data_len || e.begin > e.end, SB_STATUS_INVALID_ARGUMENT,
                 "safetensors: '" + kv.first + "' offsets [" + std::to_string(e.begin) + ", " + std::to_string(e.end) +
                     "] exceed data length " + std::to_string(f->data_len));
    uint64_t n = 1;
    for (auto d : e.shape) n *= static_cast<uint64_t>(d);
    SB_RETURN_IF(n * eb != e.end - e.begin, SB_STATUS_INVALID_ARGUMENT,
                 "safetensors: '" + kv.first + "' shape expects " + std::to_string(n) + " elements, got " +
                     std::to_string((e.end - e.begin) / eb));
    f->entries.push_back(std::move(e));
  }
  std::sort(f->entries.begin(), f->entries.end(),
            [](const sb_safetensors_file_s::Entry& a, const sb_safetensors_file_s::Entry& b) { return a.key < b.key; });
  return nullptr;
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" {

sb_status sb_safetensors_open(const char* path, sb_safetensors_file** out) {
  SB_RETURN_IF(!path || !out, SB_STATUS_INVALID_ARGUMENT, "null argument");
  auto f = std::make_unique<sb_safetensors_file_s>();
  try {
    SB_TRY(parse_header(path, f.get()));
  } catch (const std::exception& e) {  // malformed numbers in the header
    return make_status(SB_STATUS_INVALID_ARGUMENT, std::string("safetensors: invalid header (") + e.what() + ")");
  }
  *out = f.release();
  return nullptr;
}

size_t sb_safetensors_count(const sb_safetensors_file* f) { return f ? f->entries.size() : 0; }

const char* sb_safetensors_key(const sb_safetensors_file* f, size_t index) {
  return (f && index < f->entries.size()) ? f->entries[index].key.c_str() : nullptr;
}

sb_status sb_safetensors_info(const sb_safetensors_file* f, size_t index, uint32_t* elem_type, int64_t* shape,
                              size_t shape_capacity, size_t* rank) {
  SB_RETURN_IF(!f || index >= f->entries.size(), SB_STATUS_INVALID_ARGUMENT, "bad safetensors entry");
  const auto& e = f->entries[index];
  if (elem_type) *elem_type = elem_for(e.dtype);
  if (rank) *rank = e.shape.size();
  for (size_t i = 0; i < e.shape.size() && i < shape_capacity && shape; ++i) shape[i] = e.shape[i];
  return nullptr;
}

void sb_safetensors_close(sb_safetensors_file* f) { delete f; }

sb_status sb_safetensors_read(sb_session* s, const sb_safetensors_file* f, size_t index, sb_buffer** out) {
  SB_RETURN_IF(!s || !f || !out || index >= f->entries.size(), SB_STATUS_INVALID_ARGUMENT, "bad argument");
  cudaSetDevice(s->device);
  const auto& e = f->entries[index];
  const uint32_t elem = elem_for(e.dtype);
  Buffer* b = nullptr;
  SB_TRY(buffer_create(*s, e.shape, elem, &b));
  FilePtr fp(std::fopen(f->path.c_str(), "rb"));
  if (!fp || std::fseek(fp.get(), static_cast<long>(f->data_start + e.begin), SEEK_SET) != 0) {
    buffer_release(b);
    return make_status(SB_STATUS_NOT_FOUND, "safetensors: cannot read " + f->path);
  }
  const size_t fb = dtype_bytes(e.dtype), ob = elem_size(elem);
  const uint64_t count = (e.end - e.begin) / fb;
  Staging stg;
  sb_status st = stg.init();
  // chunks of whole elements; file bytes -> staging (converted in place
  // where the element type changes) -> device
  const uint64_t per = Staging::kChunk / std::max(fb, ob);
  uint64_t done = 0;
  int slot = 0;
  std::vector<unsigned char> raw;
  while (!st && done < count) {
    const uint64_t n = std::min<uint64_t>(per, count - done);
    if (cudaEventSynchronize(stg.done[slot]) != cudaSuccess) {
      st = make_status(SB_STATUS_INTERNAL, "safetensors: staging wait failed");
      break;
    }
    unsigned char* dst = static_cast<unsigned char*>(stg.buf[slot]);
    if (fb == ob && e.dtype != "BOOL") {
      if (std::fread(dst, fb, n, fp.get()) != n) st = make_status(SB_STATUS_INVALID_ARGUMENT, "safetensors: short read");
    } else {
      raw.resize(n * fb);
      if (std::fread(raw.data(), fb, n, fp.get()) != n) {
        st = make_status(SB_STATUS_INVALID_ARGUMENT, "safetensors: short read");
        break;
      }
      for (uint64_t i = 0; i < n; ++i) {
        const unsigned char* src = raw.data() + i * fb;
        if (e.dtype == "F64") {
          double v;
          std::memcpy(&v, src, 8);
          const float x = static_cast<float>(v);
          std::memcpy(dst + 4 * i, &x, 4);
        } else if (e.dtype == "I64") {
          int64_t v;
          std::memcpy(&v, src, 8);
          const int32_t x = static_cast<int32_t>(static_cast<float>(v));  // via f32, as decode_raw
          std::memcpy(dst + 4 * i, &x, 4);
        } else {  // U8, BOOL
          const int32_t x = e.dtype == "BOOL" ? (src[0] != 0) : src[0];
          std::memcpy(dst + 4 * i, &x, 4);
        }
      }
    }
    if (st) break;
    if (cudaMemcpyAsync(static_cast<char*>(b->data()) + done * ob, dst, n * ob, cudaMemcpyHostToDevice, s->stream) !=
            cudaSuccess ||
        cudaEventRecord(stg.done[slot], s->stream) != cudaSuccess)
      st = make_status(SB_STATUS_INTERNAL, "safetensors: host-to-device copy failed");
    done += n;
    slot ^= 1;
  }
  if (!st && cudaStreamSynchronize(s->stream) != cudaSuccess)
    st = make_status(SB_STATUS_INTERNAL, "safetensors: copy failed");
  if (st) {
    cudaStreamSynchronize(s->stream);
    buffer_release(b);
    return st;
  }
  *out = static_cast<sb_buffer*>(b);
  return nullptr;
}

sb_status sb_safetensors_save(sb_session* s, const char* path, const char* const* keys, sb_buffer* const* buffers,
                              size_t count) {
  SB_RETURN_IF(!s || !path || (count && (!keys || !buffers)), SB_STATUS_INVALID_ARGUMENT, "null argument");
  cudaSetDevice(s->device);
  std::vector<std::pair<std::string, Buffer*>> items;
  for (size_t i = 0; i < count; ++i) {
    SB_RETURN_IF(!keys[i] || !buffers[i], SB_STATUS_INVALID_ARGUMENT, "null key or buffer");
    SB_RETURN_IF(!dtype_for(buffers[i]->elem), SB_STATUS_INVALID_ARGUMENT, "unsupported element type");
    items.emplace_back(keys[i], buffers[i]);
  }
  std::sort(items.begin(), items.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
  for (size_t i = 1; i < items.size(); ++i)
    SB_RETURN_IF(items[i].first == items[i - 1].first, SB_STATUS_INVALID_ARGUMENT,
                 "safetensors: duplicate key " + items[i].first);
  // header: {"key":{"data_offsets":[a,b],"dtype":"F32","shape":[..]},...}
  std::string h = "{";
  uint64_t off = 0;
  for (size_t i = 0; i < items.size(); ++i) {
    const Buffer* b = items[i].second;
    // escaped as serde_json writes strings: \" and \\, the short forms \b \f
    // \n \r \t, other control characters as \u00xx (lowercase hex)
    std::string k;
    for (char ch : items[i].first) {
      const unsigned char u = static_cast<unsigned char>(ch);
      switch (ch) {
        case '"': k += "\\\""; break;
        case '\\': k += "\\\\"; break;
        case '\b': k += "\\b"; break;
        case '\f': k += "\\f"; break;
        case '\n': k += "\\n"; break;
        case '\r': k += "\\r"; break;
        case '\t': k += "\\t"; break;
        default:
          if (u < 0x20) {
            static const char hex[] = "0123456789abcdef";
            k += "\\u00";
            k += hex[u >> 4];
            k += hex[u & 15];
          } else {
            k += ch;
          }
      }
    }
    h += (i ? ",\"" : "\"") + k + "\":{\"data_offsets\":[" + std::to_string(off) + "," +
         std::to_string(off + b->bytes()) + "],\"dtype\":\"" + dtype_for(b->elem) + "\",\"shape\":[";
    for (size_t d = 0; d < b->shape.size(); ++d) h += (d ? "," : "") + std::to_string(b->shape[d]);
    h += "]}";
    off += b->bytes();
  }
  h += "}";
  while ((8 + h.size()) % 8 != 0) h += ' ';
  const std::string tmp = std::string(path) + ".tmp";
  FilePtr fp(std::fopen(tmp.c_str(), "wb"));
  SB_RETURN_IF(!fp, SB_STATUS_NOT_FOUND, std::string("safetensors: cannot create ") + tmp);
  unsigned char hb[8];
  for (int i = 0; i < 8; ++i) hb[i] = static_cast<unsigned char>((static_cast<uint64_t>(h.size()) >> (8 * i)) & 0xFF);
  bool ok = std::fwrite(hb, 1, 8, fp.get()) == 8 && std::fwrite(h.data(), 1, h.size(), fp.get()) == h.size();
  Staging stg;
  SB_TRY(stg.init());
  // device -> staging (async) -> file; the write of one chunk overlaps the
  // copy of the next
  struct Pending {
    size_t bytes = 0;
    bool live = false;
  } pend[2];
  int slot = 0;
  for (auto& it : items) {
    const Buffer* b = it.second;
    const char* src = static_cast<const char*>(b->data());
    for (size_t done = 0; ok && done < b->bytes();) {
      const size_t n = std::min(Staging::kChunk, b->bytes() - done);
      if (pend[slot].live) {  // write out the chunk this slot still holds
        ok = cudaEventSynchronize(stg.done[slot]) == cudaSuccess &&
             std::fwrite(stg.buf[slot], 1, pend[slot].bytes, fp.get()) == pend[slot].bytes;
        pend[slot].live = false;
        if (!ok) break;
      }
      ok = cudaMemcpyAsync(stg.buf[slot], src + done, n, cudaMemcpyDeviceToHost, s->stream) == cudaSuccess &&
           cudaEventRecord(stg.done[slot], s->stream) == cudaSuccess;
      pend[slot] = Pending{n, true};
      done += n;
      // keep file order: the other slot's chunk (issued earlier) goes first
      const int other = slot ^ 1;
      if (ok && pend[other].live) {
        ok = cudaEventSynchronize(stg.done[other]) == cudaSuccess &&
             std::fwrite(stg.buf[other], 1, pend[other].bytes, fp.get()) == pend[other].bytes;
        pend[other].live = false;
      }
      slot = other;
    }
    if (!ok) break;
  }
  for (int k = 0; k < 2 && ok; ++k) {  // the last chunk in flight
    const int sl = slot ^ 1 ^ k;
    if (pend[sl].live) {
      ok = cudaEventSynchronize(stg.done[sl]) == cudaSuccess &&
           std::fwrite(stg.buf[sl], 1, pend[sl].bytes, fp.get()) == pend[sl].bytes;
      pend[sl].live = false;
    }
  }
  cudaStreamSynchronize(s->stream);
  ok = ok && std::fflush(fp.get()) == 0;
  fp.reset();
  if (!ok) {
    std::remove(tmp.c_str());
    return make_status(SB_STATUS_INTERNAL, std::string("safetensors: writing ") + path + " failed");
  }
  SB_RETURN_IF(std::rename(tmp.c_str(), path) != 0, SB_STATUS_INTERNAL,
               std::string("safetensors: cannot move the file into place at ") + path);
  return nullptr;
}

}  // extern "C"
