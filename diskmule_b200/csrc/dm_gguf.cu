// dm_gguf.cu -- GGUF tensor index and expert slices (include/diskmule_gguf.h). Host code.
//
// The parse restates GgufFile::read_from_with_arrays (src/gguf.rs:460-607): a bounded
// reader over the file image, the same entry / length limits (src/gguf.rs:18-27), the
// same validation order and the same error texts (GgufError, src/gguf.rs:33-142), so a
// file the reference refuses is refused here with the same reason. The index is read
// from a read-only mapping of the whole file (TensorSource, src/gguf.rs:610-723).
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/diskmule_gguf.h"
#include "dm_internal.cuh"

using dmi::fail;

namespace {

constexpr uint32_t kDefaultAlignment = 32;
constexpr uint64_t kMaxMetadataEntries = 1000000;
constexpr uint64_t kMaxTensors = 1000000;
constexpr uint64_t kMaxKeyBytes = 64 * 1024;
constexpr uint64_t kMaxNameBytes = 1024 * 1024;
constexpr uint64_t kMaxValueStringBytes = 64ull * 1024 * 1024;
constexpr uint64_t kMaxArrayElements = 16000000;
constexpr uint64_t kMaxCapturedArrayElements = 1000000;
constexpr uint64_t kMaxCapturedArrayBytes = 256ull * 1024 * 1024;
constexpr uint32_t kMaxDimensions = 4;

// GGML type -> (elements per block, bytes per block) (TensorType::layout, src/gguf.rs:321-342)
bool ggml_layout(uint32_t kind, uint64_t *elems, uint64_t *bytes, const char **name) {
  struct L {
    uint32_t id;
    uint64_t e, b;
    const char *n;
  };
  static const L table[] = {
      {0, 1, 4, "F32"},      {1, 1, 2, "F16"},      {2, 32, 18, "Q4_0"},  {3, 32, 20, "Q4_1"},
      {6, 32, 22, "Q5_0"},   {7, 32, 24, "Q5_1"},   {8, 32, 34, "Q8_0"},  {9, 32, 40, "Q8_1"},
      {10, 256, 84, "Q2_K"}, {11, 256, 110, "Q3_K"}, {12, 256, 144, "Q4_K"},
      {13, 256, 176, "Q5_K"}, {14, 256, 210, "Q6_K"}, {15, 256, 292, "Q8_K"},
      {24, 1, 1, "I8"},      {25, 1, 2, "I16"},     {26, 1, 4, "I32"},    {27, 1, 8, "I64"},
      {28, 1, 8, "F64"},     {30, 1, 2, "BF16"},
  };
  for (const L &l : table)
    if (l.id == kind) {
      *elems = l.e;
      *bytes = l.b;
      if (name) *name = l.n;
      return true;
    }
  return false;
}

struct Value {
  uint32_t type = 0;           // GGUF value type
  uint64_t u = 0;              // integer bits (unsigned view)
  int64_t i = 0;               // signed view for the signed types
  double f = 0;                // f32 / f64
  std::string s;               // string
  uint32_t element_type = 0;   // arrays
  uint64_t length = 0;
  bool captured = false;
  std::vector<uint8_t> packed;          // captured numeric array
  std::vector<std::string> strings;     // captured string array
  std::vector<const char *> string_ptrs;
};

struct Tensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t kind = 0;
  uint64_t offset = 0, absolute = 0, byte_len = 0;
};

// A parse failure: a dm_status and the reference's error text.
struct ParseError {
  int32_t status;
  std::string message;
};

std::string fmt(const char *f, ...) {
  char buf[640];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof(buf), f, ap);
  va_end(ap);
  return buf;
}

// BoundedReader (src/gguf.rs:1036-1133): every read is checked against the file length.
struct Reader {
  const uint8_t *data;
  uint64_t len;
  uint64_t pos = 0;

  bool need(uint64_t n, const char *field, ParseError *err) {
    if (n > len - std::min(pos, len)) {
      *err = {DM_ERR_FORMAT, fmt("GGUF is truncated at byte %llu while reading %s",
                                 (unsigned long long)pos, field)};
      return false;
    }
    return true;
  }
  template <class T>
  bool read(T *out, const char *field, ParseError *err) {
    if (!need(sizeof(T), field, err)) return false;
    memcpy(out, data + pos, sizeof(T));  // little-endian host
    pos += sizeof(T);
    return true;
  }
  bool skip(uint64_t n, const char *field, ParseError *err) {
    if (!need(n, field, err)) return false;
    pos += n;
    return true;
  }
  bool read_string(std::string *out, const char *field, uint64_t limit, ParseError *err) {
    uint64_t n;
    if (!read(&n, field, err)) return false;
    if (n > limit) {
      *err = {DM_ERR_FORMAT, fmt("%s length %llu exceeds the inspection limit %llu", field,
                                 (unsigned long long)n, (unsigned long long)limit)};
      return false;
    }
    const uint64_t start = pos;
    if (!need(n, field, err)) return false;
    out->assign((const char *)data + pos, (size_t)n);
    pos += n;
    if (!valid_utf8(*out)) {
      *err = {DM_ERR_FORMAT, fmt("invalid UTF-8 in %s at byte %llu", field, (unsigned long long)start)};
      return false;
    }
    return true;
  }
  static bool valid_utf8(const std::string &s) {
    const unsigned char *p = (const unsigned char *)s.data();
    const size_t n = s.size();
    size_t i = 0;
    while (i < n) {
      const unsigned c = p[i];
      if (c < 0x80) {
        i++;
        continue;
      }
      int extra;
      uint32_t cp;
      if ((c >> 5) == 6) {
        extra = 1;
        cp = c & 0x1f;
      } else if ((c >> 4) == 14) {
        extra = 2;
        cp = c & 0x0f;
      } else if ((c >> 3) == 30) {
        extra = 3;
        cp = c & 0x07;
      } else {
        return false;
      }
      if (i + extra >= n) return false;
      for (int k = 1; k <= extra; k++) {
        if ((p[i + k] >> 6) != 2) return false;
        cp = (cp << 6) | (p[i + k] & 0x3f);
      }
      if ((extra == 1 && cp < 0x80) || (extra == 2 && cp < 0x800) || (extra == 3 && cp < 0x10000) ||
          cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff))
        return false;
      i += extra + 1;
    }
    return true;
  }
};

bool count_limit(const char *field, uint64_t count, uint64_t limit, ParseError *err) {
  if (count > limit) {
    *err = {DM_ERR_FORMAT, fmt("%s count %llu exceeds the inspection limit %llu", field,
                               (unsigned long long)count, (unsigned long long)limit)};
    return false;
  }
  return true;
}

uint64_t scalar_bytes(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
  }
}

// read_metadata_value / read_metadata_array / skip_metadata_value (src/gguf.rs:736-986)
bool read_scalar(Reader &in, uint32_t t, uint64_t kind_offset, Value *v, const char *field,
                 ParseError *err) {
  v->type = t;
  switch (t) {
    case 0: { uint8_t x; if (!in.read(&x, field, err)) return false; v->u = x; v->i = x; return true; }
    case 1: { uint8_t x; if (!in.read(&x, field, err)) return false; v->i = (int8_t)x; v->u = (uint64_t)v->i; return true; }
    case 2: { uint16_t x; if (!in.read(&x, field, err)) return false; v->u = x; v->i = x; return true; }
    case 3: { uint16_t x; if (!in.read(&x, field, err)) return false; v->i = (int16_t)x; v->u = (uint64_t)v->i; return true; }
    case 4: { uint32_t x; if (!in.read(&x, field, err)) return false; v->u = x; v->i = x; return true; }
    case 5: { uint32_t x; if (!in.read(&x, field, err)) return false; v->i = (int32_t)x; v->u = (uint64_t)v->i; return true; }
    case 6: { uint32_t x; if (!in.read(&x, field, err)) return false; float f; memcpy(&f, &x, 4); v->f = f; return true; }
    case 7: {
      uint8_t x;
      if (!in.read(&x, field, err)) return false;
      if (x > 1) {
        *err = {DM_ERR_FORMAT, fmt("invalid GGUF boolean value %u at byte %llu", x,
                                   (unsigned long long)(in.pos - 1))};
        return false;
      }
      v->u = x;
      return true;
    }
    case 10: { uint64_t x; if (!in.read(&x, field, err)) return false; v->u = x; v->i = (int64_t)x; return true; }
    case 11: { uint64_t x; if (!in.read(&x, field, err)) return false; v->i = (int64_t)x; v->u = x; return true; }
    case 12: { uint64_t x; if (!in.read(&x, field, err)) return false; memcpy(&v->f, &x, 8); return true; }
    default:
      *err = {DM_ERR_FORMAT, fmt("unknown GGUF metadata value type %u at byte %llu", t,
                                 (unsigned long long)kind_offset)};
      return false;
  }
}

bool read_value(Reader &in, uint32_t kind, uint64_t kind_offset, const std::string &key,
                bool capture, Value *v, ParseError *err) {
  if (kind == 8) {
    v->type = 8;
    return in.read_string(&v->s, "metadata string", kMaxValueStringBytes, err);
  }
  if (kind != 9) return read_scalar(in, kind, kind_offset, v, "metadata value", err);
  v->type = 9;
  const uint64_t element_offset = in.pos;
  uint32_t et;
  if (!in.read(&et, "metadata array element type", err)) return false;
  if (et == 9) {
    *err = {DM_ERR_FORMAT, fmt("nested GGUF metadata arrays are not supported at byte %llu",
                               (unsigned long long)element_offset)};
    return false;
  }
  uint64_t n;
  if (!in.read(&n, "metadata array length", err)) return false;
  if (!count_limit("metadata array element", n, kMaxArrayElements, err)) return false;
  v->element_type = et;
  v->length = n;
  if (!capture) {
    for (uint64_t j = 0; j < n; j++) {
      if (et == 8) {
        std::string tmp;
        if (!in.read_string(&tmp, "metadata array string", kMaxValueStringBytes, err)) return false;
      } else if (et == 7) {
        Value b;
        if (!read_scalar(in, 7, element_offset, &b, "BOOL metadata array element", err)) return false;
      } else {
        const uint64_t sb = scalar_bytes(et);
        if (!sb) {
          *err = {DM_ERR_FORMAT, fmt("unknown GGUF metadata value type %u at byte %llu", et,
                                     (unsigned long long)element_offset)};
          return false;
        }
        if (!in.skip(sb, "metadata array element", err)) return false;
      }
    }
    return true;
  }
  if (n > kMaxCapturedArrayElements) {
    *err = {DM_ERR_FORMAT,
            fmt("captured metadata array \"%s\" is too large (%llu elements; limit %llu)",
                key.c_str(), (unsigned long long)n, (unsigned long long)kMaxCapturedArrayElements)};
    return false;
  }
  v->captured = true;
  if (et == 8) {
    uint64_t retained = n * sizeof(std::string);
    for (uint64_t j = 0; j < n; j++) {
      std::string s;
      if (!in.read_string(&s, "metadata array string", kMaxValueStringBytes, err)) return false;
      retained += s.size();
      if (retained > kMaxCapturedArrayBytes) {
        *err = {DM_ERR_FORMAT, fmt("captured metadata array \"%s\" exceeds the %llu-byte memory budget",
                                   key.c_str(), (unsigned long long)kMaxCapturedArrayBytes)};
        return false;
      }
      v->strings.push_back(std::move(s));
    }
    for (const std::string &s : v->strings) v->string_ptrs.push_back(s.c_str());
    return true;
  }
  const uint64_t sb = scalar_bytes(et);
  if (!sb) {
    *err = {DM_ERR_FORMAT, fmt("unknown GGUF metadata value type %u at byte %llu", et,
                               (unsigned long long)element_offset)};
    return false;
  }
  if (n * sb > kMaxCapturedArrayBytes) {
    *err = {DM_ERR_FORMAT, fmt("captured metadata array \"%s\" exceeds the %llu-byte memory budget",
                               key.c_str(), (unsigned long long)kMaxCapturedArrayBytes)};
    return false;
  }
  if (et == 7) {
    for (uint64_t j = 0; j < n; j++) {
      Value b;
      if (!read_scalar(in, 7, in.pos, &b, "BOOL metadata array element", err)) return false;
      v->packed.push_back((uint8_t)b.u);
    }
    return true;
  }
  if (!in.need(n * sb, "metadata array element", err)) return false;
  v->packed.assign(in.data + in.pos, in.data + in.pos + n * sb);
  in.pos += n * sb;
  return true;
}

}  // namespace

struct dm_gguf {
  std::vector<uint8_t> copy;  // in-memory images (dm_gguf_parse)
  const uint8_t *data = nullptr;
  uint64_t len = 0;
  int fd = -1;
  void *map = nullptr;
  uint32_t version = 0, alignment = kDefaultAlignment;
  uint64_t data_offset = 0;
  std::map<std::string, Value> metadata;
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, size_t> index;
};

namespace {

bool parse(dm_gguf *g, const std::set<std::string> &capture, const char *path, ParseError *err) {
  Reader in{g->data, g->len};
  if (g->len < 4 || memcmp(g->data, "GGUF", 4) != 0) {
    if (g->len < 4 && !in.need(4, "GGUF magic", err)) return false;
    *err = {DM_ERR_FORMAT, fmt("%s is not a GGUF file", path)};
    return false;
  }
  in.pos = 4;
  if (!in.read(&g->version, "GGUF version", err)) return false;
  if (g->version != 2 && g->version != 3) {
    *err = {DM_ERR_FORMAT, fmt("unsupported GGUF version %u; DiskMule supports versions 2 and 3",
                               g->version)};
    return false;
  }
  uint64_t tensor_count, metadata_count;
  if (!in.read(&tensor_count, "tensor count", err)) return false;
  if (!count_limit("tensor", tensor_count, kMaxTensors, err)) return false;
  if (!in.read(&metadata_count, "metadata count", err)) return false;
  if (!count_limit("metadata", metadata_count, kMaxMetadataEntries, err)) return false;
  for (uint64_t m = 0; m < metadata_count; m++) {
    std::string key;
    if (!in.read_string(&key, "metadata key", kMaxKeyBytes, err)) return false;
    const uint64_t kind_offset = in.pos;
    uint32_t kind;
    if (!in.read(&kind, "metadata value type", err)) return false;
    Value v;
    if (!read_value(in, kind, kind_offset, key, capture.count(key) > 0, &v, err)) return false;
    if (!g->metadata.emplace(key, std::move(v)).second) {
      *err = {DM_ERR_FORMAT, fmt("duplicate GGUF metadata key \"%s\"", key.c_str())};
      return false;
    }
  }
  auto al = g->metadata.find("general.alignment");
  if (al != g->metadata.end()) {
    if (al->second.type != 4) {
      *err = {DM_ERR_FORMAT, "invalid general.alignment value 0; expected a nonzero power of two"};
      return false;
    }
    g->alignment = (uint32_t)al->second.u;
  }
  if (g->alignment == 0 || (g->alignment & (g->alignment - 1))) {
    *err = {DM_ERR_FORMAT, fmt("invalid general.alignment value %u; expected a nonzero power of two",
                               g->alignment)};
    return false;
  }
  std::set<std::string> names;
  for (uint64_t t = 0; t < tensor_count; t++) {
    Tensor ti;
    if (!in.read_string(&ti.name, "tensor name", kMaxNameBytes, err)) return false;
    if (!names.insert(ti.name).second) {
      *err = {DM_ERR_FORMAT, fmt("duplicate tensor name \"%s\"", ti.name.c_str())};
      return false;
    }
    uint32_t nd;
    if (!in.read(&nd, "tensor dimension count", err)) return false;
    if (nd > kMaxDimensions) {
      *err = {DM_ERR_FORMAT, fmt("tensor \"%s\" has invalid dimension count %u; maximum is %u",
                                 ti.name.c_str(), nd, kMaxDimensions)};
      return false;
    }
    for (uint32_t d = 0; d < nd; d++) {
      uint64_t dim;
      if (!in.read(&dim, "tensor dimension", err)) return false;
      if (dim == 0) {
        *err = {DM_ERR_FORMAT, fmt("tensor \"%s\" has a zero-sized dimension", ti.name.c_str())};
        return false;
      }
      ti.dims.push_back(dim);
    }
    if (!in.read(&ti.kind, "tensor type", err)) return false;
    uint64_t be, bb;
    const char *kname = "";
    if (!ggml_layout(ti.kind, &be, &bb, &kname)) {
      *err = {DM_ERR_UNSUPPORTED_TENSOR_TYPE, fmt("unsupported GGML tensor type %u for tensor \"%s\"",
                                                  ti.kind, ti.name.c_str())};
      return false;
    }
    if (!in.read(&ti.offset, "tensor offset", err)) return false;
    // tensor_byte_len (src/gguf.rs:988-1009): element count, block shape, bytes
    uint64_t elements = 1;
    for (uint64_t dim : ti.dims) {
      if (elements > UINT64_MAX / dim) {
        *err = {DM_ERR_OVERFLOW, "integer overflow while calculating tensor element count"};
        return false;
      }
      elements *= dim;
    }
    if (!ti.dims.empty() && ti.dims[0] % be) {
      *err = {DM_ERR_FORMAT,
              fmt("tensor \"%s\" first dimension %llu is not divisible by the %llu-element block "
                  "size for %s", ti.name.c_str(), (unsigned long long)ti.dims[0],
                  (unsigned long long)be, kname)};
      return false;
    }
    const uint64_t blocks = elements / be;
    if (blocks > UINT64_MAX / bb) {
      *err = {DM_ERR_OVERFLOW, "integer overflow while calculating tensor byte length"};
      return false;
    }
    ti.byte_len = blocks * bb;
    g->tensors.push_back(std::move(ti));
  }
  const uint64_t mask = g->alignment - 1;
  if (in.pos > UINT64_MAX - mask) {
    *err = {DM_ERR_OVERFLOW, "integer overflow while calculating GGUF data alignment"};
    return false;
  }
  g->data_offset = (in.pos + mask) & ~mask;
  if (g->data_offset > g->len) {
    *err = {DM_ERR_FORMAT, fmt("GGUF is truncated at byte %llu while reading aligned tensor data section",
                               (unsigned long long)in.pos)};
    return false;
  }
  for (Tensor &ti : g->tensors) {
    if (ti.offset % g->alignment) {
      *err = {DM_ERR_FORMAT, fmt("tensor \"%s\" offset %llu is not aligned to %u bytes",
                                 ti.name.c_str(), (unsigned long long)ti.offset, g->alignment)};
      return false;
    }
    if (ti.offset > UINT64_MAX - g->data_offset) {
      *err = {DM_ERR_OVERFLOW, "integer overflow while calculating absolute tensor offset"};
      return false;
    }
    ti.absolute = g->data_offset + ti.offset;
    if (ti.byte_len > UINT64_MAX - ti.absolute) {
      *err = {DM_ERR_OVERFLOW, "integer overflow while calculating tensor byte range"};
      return false;
    }
    const uint64_t end = ti.absolute + ti.byte_len;
    if (end > g->len) {
      *err = {DM_ERR_FORMAT, fmt("tensor \"%s\" byte range %llu..%llu exceeds the %llu-byte GGUF file",
                                 ti.name.c_str(), (unsigned long long)ti.absolute,
                                 (unsigned long long)end, (unsigned long long)g->len)};
      return false;
    }
  }
  // validate_non_overlapping (src/gguf.rs:1019-1034)
  std::vector<const Tensor *> ordered;
  for (const Tensor &ti : g->tensors) ordered.push_back(&ti);
  std::stable_sort(ordered.begin(), ordered.end(),
                   [](const Tensor *a, const Tensor *b) { return a->absolute < b->absolute; });
  uint64_t previous_end = 0;
  for (const Tensor *ti : ordered) {
    if (ti->absolute < previous_end) {
      *err = {DM_ERR_FORMAT, fmt("tensor \"%s\" overlaps an earlier tensor at byte %llu",
                                 ti->name.c_str(), (unsigned long long)ti->absolute)};
      return false;
    }
    previous_end = ti->absolute + ti->byte_len;
  }
  for (size_t i = 0; i < g->tensors.size(); i++) g->index.emplace(g->tensors[i].name, i);
  return true;
}

std::set<std::string> capture_set(const char *keys) {
  std::set<std::string> out;
  if (!keys) return out;
  std::string s(keys);
  size_t start = 0;
  while (start <= s.size()) {
    size_t end = s.find('\n', start);
    if (end == std::string::npos) end = s.size();
    if (end > start) out.insert(s.substr(start, end - start));
    start = end + 1;
  }
  return out;
}

int32_t finish(dm_gguf *g, const char *capture, const char *path, dm_gguf **out) {
  ParseError err{DM_OK, ""};
  if (!parse(g, capture_set(capture), path, &err)) {
    dm_gguf_close(g);
    return fail(err.status, "%s", err.message.c_str());
  }
  *out = g;
  return DM_OK;
}

const Value *find_value(const dm_gguf *g, const char *key) {
  if (!g || !key) return nullptr;
  auto it = g->metadata.find(key);
  return it == g->metadata.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

int32_t dm_gguf_open(const char *path, const char *capture_arrays, dm_gguf **out) {
  if (!path || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(DM_ERR_IO, "could not read GGUF: %s (%s)", strerror(errno), path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    const int e = errno;
    close(fd);
    return fail(DM_ERR_IO, "could not read GGUF: %s (%s)", strerror(e), path);
  }
  dm_gguf *g = new dm_gguf();
  g->fd = fd;
  g->len = (uint64_t)st.st_size;
  if (g->len > 0) {
    void *m = mmap(nullptr, (size_t)g->len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
      const int e = errno;
      dm_gguf_close(g);
      return fail(DM_ERR_IO, "could not read GGUF: %s (%s)", strerror(e), path);
    }
    g->map = m;
    g->data = (const uint8_t *)m;
  }
  return finish(g, capture_arrays, path, out);
}

int32_t dm_gguf_parse(const void *bytes, uint64_t length, const char *capture_arrays,
                      dm_gguf **out) {
  if ((!bytes && length) || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  dm_gguf *g = new dm_gguf();
  g->copy.assign((const uint8_t *)bytes, (const uint8_t *)bytes + length);
  g->data = g->copy.data();
  g->len = length;
  return finish(g, capture_arrays, "<memory>", out);
}

void dm_gguf_close(dm_gguf *g) {
  if (!g) return;
  if (g->map) munmap(g->map, (size_t)g->len);
  if (g->fd >= 0) close(g->fd);
  delete g;
}

int32_t dm_gguf_header(const dm_gguf *g, uint32_t *version, uint32_t *alignment,
                       uint64_t *data_offset, uint64_t *file_len) {
  if (!g) return fail(DM_ERR_INVALID_ARGUMENT, "null GGUF handle");
  if (version) *version = g->version;
  if (alignment) *alignment = g->alignment;
  if (data_offset) *data_offset = g->data_offset;
  if (file_len) *file_len = g->len;
  return DM_OK;
}

int64_t dm_gguf_tensor_count(const dm_gguf *g) { return g ? (int64_t)g->tensors.size() : 0; }

int32_t dm_gguf_find_tensor(const dm_gguf *g, const char *name, int64_t *index) {
  if (!g || !name || !index) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  auto it = g->index.find(name);
  if (it == g->index.end())
    return fail(DM_ERR_FORMAT, "tensor \"%s\" was not found in the GGUF index", name);
  *index = (int64_t)it->second;
  return DM_OK;
}

int32_t dm_gguf_tensor(const dm_gguf *g, int64_t index, dm_gguf_tensor_info *out) {
  if (!g || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (index < 0 || (uint64_t)index >= g->tensors.size())
    return fail(DM_ERR_INVALID_ARGUMENT, "tensor index %lld out of range", (long long)index);
  const Tensor &t = g->tensors[(size_t)index];
  memset(out, 0, sizeof(*out));
  out->name = t.name.c_str();
  out->n_dims = (uint32_t)t.dims.size();
  for (size_t d = 0; d < t.dims.size(); d++) out->dims[d] = t.dims[d];
  out->type = (int32_t)t.kind;
  out->offset = t.offset;
  out->absolute_offset = t.absolute;
  out->byte_len = t.byte_len;
  return DM_OK;
}

int32_t dm_gguf_tensor_bytes(const dm_gguf *g, int64_t index, const void **data,
                             uint64_t *length) {
  if (!g || !data || !length) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (index < 0 || (uint64_t)index >= g->tensors.size())
    return fail(DM_ERR_INVALID_ARGUMENT, "tensor index %lld out of range", (long long)index);
  const Tensor &t = g->tensors[(size_t)index];
  *data = g->data + t.absolute;
  *length = t.byte_len;
  return DM_OK;
}

int32_t dm_gguf_read_tensor_at(const dm_gguf *g, const char *name, uint64_t offset,
                               void *destination, uint64_t length) {
  if (!g || !name || (!destination && length)) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  auto it = g->index.find(name);
  if (it == g->index.end())
    return fail(DM_ERR_FORMAT, "tensor \"%s\" was not found in the GGUF index", name);
  const Tensor &t = g->tensors[it->second];
  if (offset > UINT64_MAX - length)
    return fail(DM_ERR_OVERFLOW, "integer overflow while calculating tensor read range");
  const uint64_t end = offset + length;
  if (end > t.byte_len)
    return fail(DM_ERR_FORMAT, "requested range %llu..%llu exceeds tensor \"%s\" length %llu",
                (unsigned long long)offset, (unsigned long long)end, name,
                (unsigned long long)t.byte_len);
  uint64_t at = t.absolute + offset;
  uint8_t *dst = (uint8_t *)destination;
  if (g->fd < 0) {
    memcpy(dst, g->data + at, (size_t)length);
    return DM_OK;
  }
  // read_exact_at (src/gguf.rs:929-945): positional reads, retried on EINTR
  while (length > 0) {
    const ssize_t n = pread(g->fd, dst, (size_t)std::min<uint64_t>(length, 1ull << 30), (off_t)at);
    if (n < 0) {
      if (errno == EINTR) continue;
      return fail(DM_ERR_IO, "could not read GGUF: %s", strerror(errno));
    }
    if (n == 0) return fail(DM_ERR_IO, "could not read GGUF: unexpected end of file");
    dst += n;
    at += (uint64_t)n;
    length -= (uint64_t)n;
  }
  return DM_OK;
}

int32_t dm_gguf_metadata_type(const dm_gguf *g, const char *key, uint32_t *type,
                              uint32_t *element_type, uint64_t *length) {
  const Value *v = find_value(g, key);
  if (!v) return fail(DM_ERR_FORMAT, "metadata key \"%s\" is not present", key ? key : "");
  if (type) *type = v->type;
  if (element_type) *element_type = v->type == 9 ? v->element_type : 0;
  if (length) *length = v->type == 9 ? v->length : (v->type == 8 ? v->s.size() : 1);
  return DM_OK;
}

int32_t dm_gguf_metadata_u64(const dm_gguf *g, const char *key, uint64_t *value) {
  const Value *v = find_value(g, key);
  if (!v) return fail(DM_ERR_FORMAT, "metadata key \"%s\" is not present", key ? key : "");
  if (!value) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  switch (v->type) {
    case 0: case 2: case 4: case 10: case 7: *value = v->u; return DM_OK;
    case 1: case 3: case 5: case 11:
      if (v->i < 0) return fail(DM_ERR_FORMAT, "metadata \"%s\" is negative", key);
      *value = (uint64_t)v->i;
      return DM_OK;
    default: return fail(DM_ERR_FORMAT, "metadata \"%s\" is not an integer", key);
  }
}

int32_t dm_gguf_metadata_f64(const dm_gguf *g, const char *key, double *value) {
  const Value *v = find_value(g, key);
  if (!v) return fail(DM_ERR_FORMAT, "metadata key \"%s\" is not present", key ? key : "");
  if (!value) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (v->type != 6 && v->type != 12) return fail(DM_ERR_FORMAT, "metadata \"%s\" is not a float", key);
  *value = v->f;
  return DM_OK;
}

int32_t dm_gguf_metadata_string(const dm_gguf *g, const char *key, char *buffer, uint64_t capacity) {
  const Value *v = find_value(g, key);
  if (!v) return fail(DM_ERR_FORMAT, "metadata key \"%s\" is not present", key ? key : "");
  if (v->type != 8) return fail(DM_ERR_FORMAT, "metadata \"%s\" is not a string", key);
  if (!buffer || capacity < v->s.size() + 1)
    return fail(DM_ERR_OUTPUT_LENGTH, "metadata \"%s\" needs %zu bytes", key, v->s.size() + 1);
  memcpy(buffer, v->s.c_str(), v->s.size() + 1);
  return DM_OK;
}

int32_t dm_gguf_metadata_array(const dm_gguf *g, const char *key, uint32_t *element_type,
                               uint64_t *length, const void **values) {
  const Value *v = find_value(g, key);
  if (!v) return fail(DM_ERR_FORMAT, "metadata key \"%s\" is not present", key ? key : "");
  if (v->type != 9) return fail(DM_ERR_FORMAT, "metadata \"%s\" is not an array", key);
  if (!v->captured)
    return fail(DM_ERR_FORMAT, "metadata array \"%s\" was not captured (list it when opening)", key);
  if (element_type) *element_type = v->element_type;
  if (length) *length = v->length;
  if (values)
    *values = v->element_type == 8 ? (const void *)v->string_ptrs.data()
                                   : (const void *)v->packed.data();
  return DM_OK;
}

int32_t dm_gguf_expert_layout(const dm_gguf *g, const char *gate_up, const char *down,
                              int32_t expert_count, dm_expert_layer_layout *out) {
  if (!g || !gate_up || !down || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  int64_t gi, di;
  int32_t rc = dm_gguf_find_tensor(g, gate_up, &gi);
  if (rc != DM_OK) return rc;
  rc = dm_gguf_find_tensor(g, down, &di);
  if (rc != DM_OK) return rc;
  const Tensor &gt = g->tensors[(size_t)gi], &dt = g->tensors[(size_t)di];
  // bytes_per_expert (src/gemma4/metal.rs:1101-1117)
  for (const Tensor *t : {&gt, &dt})
    if (expert_count <= 0 || t->byte_len % (uint64_t)expert_count)
      return fail(DM_ERR_FORMAT,
                  "invalid expert cache layout: %s byte length %llu is not divisible by %d experts",
                  t->name.c_str(), (unsigned long long)t->byte_len, expert_count);
  out->expert_count = expert_count;
  out->gate_up_offset = gt.absolute;
  out->gate_up_bytes = gt.byte_len / (uint64_t)expert_count;
  out->down_offset = dt.absolute;
  out->down_bytes = dt.byte_len / (uint64_t)expert_count;
  return DM_OK;
}

}  // extern "C"
