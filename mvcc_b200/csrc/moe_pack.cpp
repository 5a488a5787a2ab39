// moe_pack.cpp -- the .mvccq pack reader declared in include/moe_pack.h.
//
// The file is mapped read-only; its JSON header (convert.py:200-211 writes it, pack.hpp:127-139 reads it) is parsed
// by the small recursive-descent reader below into a table of tensor entries, each checked against the file size and
// its own dtype x shape. A layer's MoE block tensors are then looked up by the names convert.py:366-415 gives them,
// checked against the geometry qwen.cu:161-165 reads, and copied into one device region.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "moe_pack.h"

namespace moe {
void note_pack_bytes(uint64_t n);  // moe_stats_get's counter (moe_api.cu)
}  // namespace moe

namespace {

// ----------------------------------------------------------------------------------------------- JSON reader

struct JNode {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<JNode> items;                          // array elements
  std::vector<std::pair<std::string, JNode>> fields;  // object members in file order

  const JNode* field(const char* key) const {
    for (const auto& f : fields)
      if (f.first == key) return &f.second;
    return nullptr;
  }
};

// Reads one JSON document (RFC 8259) from [p, end). Nesting is bounded so a hostile header cannot exhaust the stack.
class JReader {
 public:
  JReader(const char* p, const char* end) : p_(p), end_(end) {}

  bool document(JNode& out) {
    if (!value(out, 0)) return false;
    skip_space();
    if (p_ != end_) return fail("trailing bytes after the header object");
    return true;
  }
  const std::string& error() const { return err_; }

 private:
  static constexpr int kMaxDepth = 64;
  const char* p_;
  const char* end_;
  std::string err_;

  bool fail(const char* what) {
    if (err_.empty()) err_ = what;
    return false;
  }
  void skip_space() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool literal(const char* word) {
    const size_t n = strlen(word);
    if ((size_t)(end_ - p_) < n || memcmp(p_, word, n) != 0) return fail("unknown literal");
    p_ += n;
    return true;
  }

  bool value(JNode& out, int depth) {
    if (depth > kMaxDepth) return fail("header nested too deeply");
    skip_space();
    if (p_ >= end_) return fail("header ends inside a value");
    switch (*p_) {
      case '{': return object(out, depth);
      case '[': return array(out, depth);
      case '"': out.kind = JNode::kStr; return string(out.str);
      case 't': out.kind = JNode::kBool; out.b = true; return literal("true");
      case 'f': out.kind = JNode::kBool; out.b = false; return literal("false");
      case 'n': out.kind = JNode::kNull; return literal("null");
      default: out.kind = JNode::kNum; return number(out.num);
    }
  }

  bool object(JNode& out, int depth) {
    out.kind = JNode::kObj;
    ++p_;  // '{'
    skip_space();
    if (p_ < end_ && *p_ == '}') { ++p_; return true; }
    for (;;) {
      skip_space();
      if (p_ >= end_ || *p_ != '"') return fail("object key is not a string");
      std::string key;
      if (!string(key)) return false;
      skip_space();
      if (p_ >= end_ || *p_ != ':') return fail("missing ':' after an object key");
      ++p_;
      out.fields.emplace_back(std::move(key), JNode());
      if (!value(out.fields.back().second, depth + 1)) return false;
      skip_space();
      if (p_ < end_ && *p_ == ',') { ++p_; continue; }
      if (p_ < end_ && *p_ == '}') { ++p_; return true; }
      return fail("missing ',' or '}' in an object");
    }
  }

  bool array(JNode& out, int depth) {
    out.kind = JNode::kArr;
    ++p_;  // '['
    skip_space();
    if (p_ < end_ && *p_ == ']') { ++p_; return true; }
    for (;;) {
      out.items.emplace_back();
      if (!value(out.items.back(), depth + 1)) return false;
      skip_space();
      if (p_ < end_ && *p_ == ',') { ++p_; continue; }
      if (p_ < end_ && *p_ == ']') { ++p_; return true; }
      return fail("missing ',' or ']' in an array");
    }
  }

  static void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
      s += (char)cp;
    } else if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xF0 | (cp >> 18));
      s += (char)(0x80 | ((cp >> 12) & 0x3F));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
  }

  bool hex4(uint32_t& v) {
    if (end_ - p_ < 4) return fail("short \\u escape");
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail("bad hex digit in a \\u escape");
    }
    return true;
  }

  bool string(std::string& s) {
    ++p_;  // opening quote
    for (;;) {
      if (p_ >= end_) return fail("header ends inside a string");
      const char c = *p_++;
      if (c == '"') return true;
      if ((unsigned char)c < 0x20) return fail("control character inside a string");
      if (c != '\\') { s += c; continue; }
      if (p_ >= end_) return fail("header ends inside an escape");
      const char e = *p_++;
      switch (e) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
            uint32_t lo;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("lone surrogate in a string");
            p_ += 2;
            if (!hex4(lo)) return false;
            if (lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair in a string");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(s, cp);
          break;
        }
        default: return fail("unknown escape in a string");
      }
    }
  }

  bool number(double& v) {
    const char* q = p_;
    while (q < end_ && *q != '\0' && strchr("+-0123456789.eE", *q) != nullptr) ++q;
    if (q == p_) return fail("unexpected character in the header");
    const std::string text(p_, q);
    char* stop = nullptr;
    v = strtod(text.c_str(), &stop);
    if (stop != text.c_str() + text.size()) return fail("malformed number in the header");
    p_ = q;
    return true;
  }
};

// ----------------------------------------------------------------------------------------------- pack

struct Entry {
  uint64_t off = 0, nbytes = 0;
  std::string dtype;
  std::vector<int64_t> shape;
};

size_t dtype_size(const std::string& d) {
  if (d == "bf16" || d == "f16") return 2;
  if (d == "f32") return 4;
  if (d == "u8" || d == "i8") return 1;
  return 0;  // unknown to this reader: size not checked
}

constexpr int kBlockTensors = 9;
constexpr size_t kDevAlign = 256;

}  // namespace

struct moe_pack {
  int fd = -1;
  void* base = MAP_FAILED;
  size_t size = 0;
  moe_pack_geometry geo{};
  std::map<std::string, Entry> tensors;  // ordered by name
  std::vector<const std::string*> names;
  std::string err;
  std::map<std::pair<int, int>, std::vector<uint16_t>> dequant;  // (layer, block tensor) -> bf16 rows of an int8 pack

  int set_err(int code, const char* fmt, ...) __attribute__((format(printf, 3, 4))) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    err = buf;
    return code;
  }
  const uint8_t* bytes() const { return static_cast<const uint8_t*>(base); }
};

namespace {

constexpr int kInvalid = (int)cudaErrorInvalidValue;
constexpr int kNotSupported = (int)cudaErrorNotSupported;

bool as_int(const JNode* n, int32_t& out) {
  if (!n || n->kind != JNode::kNum) return false;
  if (!(n->num >= -2147483648.0 && n->num <= 2147483647.0) || n->num != (double)(int64_t)n->num) return false;
  out = (int32_t)n->num;
  return true;
}

// Parses the header text and fills pack->geo and pack->tensors. Returns "" or the reason.
std::string parse_header(moe_pack* pk, const char* text, size_t n, uint64_t data_start) {
  JNode root;
  JReader rd(text, text + n);
  if (!rd.document(root)) return "header JSON: " + rd.error();
  if (root.kind != JNode::kObj) return "header JSON is not an object";
  const JNode* cfg = root.field("config");
  const JNode* tens = root.field("tensors");
  if (!cfg || cfg->kind != JNode::kObj) return "header has no \"config\" object";
  if (!tens || tens->kind != JNode::kObj) return "header has no \"tensors\" object";

  moe_pack_geometry& g = pk->geo;
  const struct { const char* key; int32_t* dst; } ints[] = {
      {"hidden", &g.H}, {"layers", &g.L}, {"experts", &g.E}, {"topk", &g.TOPK}, {"inter", &g.I},
      {"shared_inter", &g.Is}};
  for (const auto& f : ints)
    if (!as_int(cfg->field(f.key), *f.dst) || *f.dst < 1)
      return std::string("config.") + f.key + " is missing or not a positive integer";
  const JNode* grp = cfg->field("group");
  g.G = 128;
  if (grp && (!as_int(grp, g.G) || g.G < 2)) return "config.group is not an integer >= 2";
  const JNode* eps = cfg->field("eps");
  if (!eps || eps->kind != JNode::kNum || !(eps->num > 0.0)) return "config.eps is missing or not positive";
  g.eps = (float)eps->num;
  if (g.H % 2 || g.I % 2 || g.H % g.G || g.I % g.G) return "config: hidden and inter must be even multiples of group";

  for (const auto& f : tens->fields) {
    const JNode& t = f.second;
    const JNode* off = t.field("off");
    const JNode* nb = t.field("nbytes");
    const JNode* dt = t.field("dtype");
    const JNode* sh = t.field("shape");
    if (!off || off->kind != JNode::kNum || !nb || nb->kind != JNode::kNum || !dt || dt->kind != JNode::kStr || !sh ||
        sh->kind != JNode::kArr)
      return "tensor " + f.first + ": entry needs off, nbytes, dtype and shape";
    if (off->num < 0 || nb->num < 0 || off->num > 9.0e15 || nb->num > 9.0e15 || off->num != (double)(uint64_t)off->num ||
        nb->num != (double)(uint64_t)nb->num)
      return "tensor " + f.first + ": off/nbytes are not byte counts";
    Entry e;
    e.off = (uint64_t)off->num;
    e.nbytes = (uint64_t)nb->num;
    e.dtype = dt->str;
    if (sh->items.size() > 6) return "tensor " + f.first + ": more than 6 dimensions";
    uint64_t elems = 1;
    for (const auto& d : sh->items) {
      if (d.kind != JNode::kNum || d.num < 0 || d.num > 9.0e15 || d.num != (double)(int64_t)d.num)
        return "tensor " + f.first + ": shape holds a non-integer";
      e.shape.push_back((int64_t)d.num);
      elems = elems * (uint64_t)d.num;
    }
    if (e.off < data_start || e.off > pk->size || e.nbytes > pk->size - e.off)
      return "tensor " + f.first + ": blob lies outside the file's data area";
    const size_t isz = dtype_size(e.dtype);
    if (isz && elems * isz != e.nbytes) return "tensor " + f.first + ": nbytes disagrees with dtype x shape";
    pk->tensors[f.first] = std::move(e);
  }
  for (const auto& kv : pk->tensors) pk->names.push_back(&kv.first);
  return "";
}

struct Want {
  const char* suffix;
  const char* dtype;
  int ndim;
  int64_t dims[3];
  bool int8_ok;  // may be stored as int8 rows + fp16 group scales (convert.py --dense int8)
};

// The nine block tensors of one layer, in the order moe_layer_weights lists its pointers, with the shapes
// qwen.cu:181-190 reads (Model::linear checks [N,K] of the shared expert, qwen.cu:137-155).
void block_wants(const moe_pack_geometry& g, Want w[kBlockTensors]) {
  const int64_t H = g.H, E = g.E, I = g.I, Is = g.Is, G = g.G;
  const Want all[kBlockTensors] = {
      {"rms2", "bf16", 1, {H, 0, 0}, false},
      {"router", "bf16", 2, {E, H, 0}, false},
      {"exp.gate_up.q", "u8", 3, {E, 2 * I, H / 2}, false},
      {"exp.gate_up.s", "f16", 3, {E, 2 * I, H / G}, false},
      {"exp.down.q", "u8", 3, {E, H, I / 2}, false},
      {"exp.down.s", "f16", 3, {E, H, I / G}, false},
      {"shared.gate_up", "bf16", 2, {2 * Is, H, 0}, true},
      {"shared.down", "bf16", 2, {H, Is, 0}, true},
      {"shared.gate", "bf16", 1, {H, 0, 0}, false},
  };
  for (int i = 0; i < kBlockTensors; ++i) w[i] = all[i];
}

// Where one block tensor comes from: a stored tensor of the wanted dtype (`e`), or -- for the shared expert of an
// int8 pack -- int8 rows `q8` [N,K] with fp16 scales `s8` [N, K/group] (quant_int8_rows, convert.py:159-169) that
// the loader dequantizes to bf16.
struct Src {
  const Entry* e = nullptr;
  const Entry* q8 = nullptr;
  const Entry* s8 = nullptr;
  int64_t rows = 0, cols = 0, group = 0;
  uint64_t nbytes() const { return e ? e->nbytes : (uint64_t)(rows * cols * 2); }
};

std::string dims_text(const std::vector<int64_t>& v) {
  std::string t;
  for (size_t d = 0; d < v.size(); ++d) t += (d ? "," : "") + std::to_string(v[d]);
  return t;
}

bool shape_is(const Entry& e, const char* dtype, int ndim, const int64_t* dims) {
  bool ok = e.dtype == dtype && (int)e.shape.size() == ndim;
  for (int d = 0; ok && d < ndim; ++d) ok = e.shape[d] == dims[d];
  return ok;
}

// Looks up and checks layer `layer`'s block tensors; fills src[] in moe_layer_weights order.
int find_block(moe_pack* pk, int layer, Src src[kBlockTensors]) {
  if (layer < 0 || layer >= pk->geo.L)
    return pk->set_err(kInvalid, "layer %d is outside the pack's %d layers", layer, pk->geo.L);
  Want want[kBlockTensors];
  block_wants(pk->geo, want);
  const std::string pre = "L" + std::to_string(layer) + ".";
  for (int i = 0; i < kBlockTensors; ++i) {
    const Want& wt = want[i];
    const std::string name = pre + wt.suffix;
    src[i] = Src();
    auto it = pk->tensors.find(name);
    if (it == pk->tensors.end() && wt.int8_ok && pk->tensors.count(name + ".q8")) {
      auto sq = pk->tensors.find(name + ".s8");
      if (sq == pk->tensors.end()) return pk->set_err(kInvalid, "pack has %s.q8 but no %s.s8", name.c_str(), name.c_str());
      const Entry& q = pk->tensors.at(name + ".q8");
      const Entry& sc = sq->second;
      const int64_t N = wt.dims[0], K = wt.dims[1];
      if (!shape_is(q, "i8", 2, wt.dims))
        return pk->set_err(kInvalid, "tensor %s.q8 is %s [%s], expected i8 [%lld,%lld]", name.c_str(), q.dtype.c_str(),
                           dims_text(q.shape).c_str(), (long long)N, (long long)K);
      if (sc.dtype != "f16" || sc.shape.size() != 2 || sc.shape[0] != N || sc.shape[1] < 1 || K % sc.shape[1])
        return pk->set_err(kInvalid, "tensor %s.s8 is %s [%s], expected f16 [%lld, K/group]", name.c_str(),
                           sc.dtype.c_str(), dims_text(sc.shape).c_str(), (long long)N);
      src[i].q8 = &q;
      src[i].s8 = &sc;
      src[i].rows = N;
      src[i].cols = K;
      src[i].group = K / sc.shape[1];
      continue;
    }
    if (it == pk->tensors.end()) return pk->set_err(kInvalid, "pack has no tensor %s", name.c_str());
    const Entry& e = it->second;
    if (!shape_is(e, wt.dtype, wt.ndim, wt.dims)) {
      std::vector<int64_t> exp(wt.dims, wt.dims + wt.ndim);
      return pk->set_err(kInvalid, "tensor %s is %s [%s], expected %s [%s]", name.c_str(), e.dtype.c_str(),
                         dims_text(e.shape).c_str(), wt.dtype, dims_text(exp).c_str());
    }
    src[i].e = &e;
  }
  return 0;
}

// IEEE 754 binary16 bits -> float (normal, subnormal, infinity and NaN encodings).
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  uint32_t bits;
  if (ex == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (ex != 0) {
    bits = sign | ((ex + 112u) << 23) | (man << 13);  // rebias 15 -> 127
  } else {
    float f = std::ldexp((float)man, -24);  // subnormal: man * 2^-24, exact in float
    memcpy(&bits, &f, 4);
    bits |= sign;
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// float -> bf16 bits, round to nearest, ties to even (NaN kept quiet).
uint16_t float_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// bf16(q * scale) row by row: the int8 value times its group's fp16 scale is exact in fp32 (8 + 11 significant
// bits), so the single rounding is the one to bf16.
void dequant_i8_rows(const int8_t* q, const uint16_t* sc, int64_t rows, int64_t cols, int64_t group, uint16_t* out) {
  const int64_t groups = cols / group;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t g = 0; g < groups; ++g) {
      const float s = half_bits_to_float(sc[r * groups + g]);
      const int8_t* qq = q + r * cols + g * group;
      uint16_t* o = out + r * cols + g * group;
      for (int64_t k = 0; k < group; ++k) o[k] = float_to_bf16_rne((float)qq[k] * s);
    }
}

// Whether the shared expert of a --dense int8 pack can also be handed to the block as int8 (both matrices stored as
// q8 + s8 with one group size, a multiple of 32); its group size in *group. False for a bf16 pack.
bool int8_shared(const Src src[kBlockTensors], int64_t* group) {
  const Src& gu = src[6];
  const Src& dn = src[7];
  if (!gu.q8 || !dn.q8 || gu.group != dn.group || gu.group % 32 || gu.group <= 0) return false;
  *group = gu.group;
  return true;
}

void fill_weights(const moe_pack_geometry& g, const void* const ptr[kBlockTensors], moe_layer_weights* w) {
  memset(w, 0, sizeof *w);
  w->rms2 = static_cast<const uint16_t*>(ptr[0]);
  w->router = static_cast<const uint16_t*>(ptr[1]);
  w->exp_gu_q = static_cast<const uint8_t*>(ptr[2]);
  w->exp_gu_s = static_cast<const uint16_t*>(ptr[3]);
  w->exp_dn_q = static_cast<const uint8_t*>(ptr[4]);
  w->exp_dn_s = static_cast<const uint16_t*>(ptr[5]);
  w->shared_gate_up = static_cast<const uint16_t*>(ptr[6]);
  w->shared_down = static_cast<const uint16_t*>(ptr[7]);
  w->shared_gate = static_cast<const uint16_t*>(ptr[8]);
  w->H = g.H;
  w->E = g.E;
  w->TOPK = g.TOPK;
  w->I = g.I;
  w->Is = g.Is;
  w->G = g.G;
  w->eps = g.eps;
  w->router_bias = nullptr;
}

size_t align_up(size_t x) { return (x + kDevAlign - 1) / kDevAlign * kDevAlign; }

void copy_err(char* err, size_t err_len, const std::string& msg) {
  if (!err || err_len == 0) return;
  snprintf(err, err_len, "%s", msg.c_str());
}

}  // namespace

namespace {

// Host bytes of block tensor i: the blob in the mapping, or (int8 shared expert) its bf16 rows, dequantised once per
// (layer, tensor) and kept until the pack is closed.
const void* host_block_bytes(moe_pack* pk, int layer, int i, const Src& src) {
  if (src.e) return pk->bytes() + src.e->off;
  std::vector<uint16_t>& rows = pk->dequant[{layer, i}];
  if (rows.empty()) {
    rows.resize((size_t)(src.rows * src.cols));
    dequant_i8_rows(reinterpret_cast<const int8_t*>(pk->bytes() + src.q8->off),
                    reinterpret_cast<const uint16_t*>(pk->bytes() + src.s8->off), src.rows, src.cols, src.group,
                    rows.data());
  }
  return rows.data();
}

}  // namespace

extern "C" {

moe_pack* moe_pack_open(const char* path, char* err, size_t err_len) {
  if (!path) {
    copy_err(err, err_len, "path is NULL");
    return nullptr;
  }
  moe_pack* pk = new moe_pack();
  std::string why;
  pk->fd = ::open(path, O_RDONLY | O_CLOEXEC);
  struct stat st;
  if (pk->fd < 0) {
    why = std::string("cannot open ") + path + ": " + strerror(errno);
  } else if (fstat(pk->fd, &st) != 0 || !S_ISREG(st.st_mode)) {
    why = std::string(path) + " is not a regular file";
  } else if (st.st_size < 16) {
    why = std::string(path) + " is too short for a pack header";
  } else {
    pk->size = (size_t)st.st_size;
    pk->base = mmap(nullptr, pk->size, PROT_READ, MAP_SHARED, pk->fd, 0);
    if (pk->base == MAP_FAILED) {
      why = std::string("mmap failed: ") + strerror(errno);
    } else if (memcmp(pk->bytes(), "MVCCQ001", 8) != 0) {
      why = std::string(path) + ": bad magic (not an MVCCQ001 pack)";
    } else {
      uint64_t hlen = 0;
      for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | pk->bytes()[8 + i];  // little-endian u64
      if (hlen > pk->size - 16) {
        why = std::string(path) + ": header length runs past the end of the file";
      } else {
        why = parse_header(pk, reinterpret_cast<const char*>(pk->bytes()) + 16, (size_t)hlen, 16 + hlen);
        if (!why.empty()) why = std::string(path) + ": " + why;
      }
    }
  }
  if (!why.empty()) {
    copy_err(err, err_len, why);
    moe_pack_close(pk);
    return nullptr;
  }
  copy_err(err, err_len, "");
  return pk;
}

void moe_pack_close(moe_pack* pk) {
  if (!pk) return;
  if (pk->base != MAP_FAILED) munmap(pk->base, pk->size);
  if (pk->fd >= 0) ::close(pk->fd);
  delete pk;
}

const char* moe_pack_last_error(const moe_pack* pk) { return pk ? pk->err.c_str() : "pack is NULL"; }

int moe_pack_geometry_get(moe_pack* pk, moe_pack_geometry* geo) {
  if (!pk || !geo) return kInvalid;
  pk->err.clear();
  *geo = pk->geo;
  return 0;
}

int moe_pack_tensor_count(const moe_pack* pk) { return pk ? (int)pk->names.size() : 0; }

const char* moe_pack_tensor_name(const moe_pack* pk, int i) {
  if (!pk || i < 0 || i >= (int)pk->names.size()) return nullptr;
  return pk->names[i]->c_str();
}

int moe_pack_tensor(moe_pack* pk, const char* name, moe_pack_tensor_info* info) {
  if (!pk || !name || !info) return kInvalid;
  pk->err.clear();
  auto it = pk->tensors.find(name);
  if (it == pk->tensors.end()) return pk->set_err(kInvalid, "pack has no tensor %s", name);
  const Entry& e = it->second;
  memset(info, 0, sizeof *info);
  info->off = e.off;
  info->nbytes = e.nbytes;
  info->host = pk->bytes() + e.off;
  info->ndim = (int32_t)e.shape.size();
  for (size_t d = 0; d < e.shape.size(); ++d) info->shape[d] = e.shape[d];
  snprintf(info->dtype, sizeof info->dtype, "%s", e.dtype.c_str());
  return 0;
}

int moe_pack_layer_host(moe_pack* pk, int layer, moe_layer_weights* w) {
  if (!pk || !w) return kInvalid;
  pk->err.clear();
  Src src[kBlockTensors];
  if (int rc = find_block(pk, layer, src)) return rc;
  const void* ptr[kBlockTensors];
  for (int i = 0; i < kBlockTensors; ++i) ptr[i] = host_block_bytes(pk, layer, i, src[i]);
  fill_weights(pk->geo, ptr, w);
  int64_t g8 = 0;
  if (int8_shared(src, &g8)) {  // the int8 rows and scales as stored, in the mapping
    w->shared_gate_up_q8 = reinterpret_cast<const int8_t*>(pk->bytes() + src[6].q8->off);
    w->shared_gate_up_s8 = reinterpret_cast<const uint16_t*>(pk->bytes() + src[6].s8->off);
    w->shared_down_q8 = reinterpret_cast<const int8_t*>(pk->bytes() + src[7].q8->off);
    w->shared_down_s8 = reinterpret_cast<const uint16_t*>(pk->bytes() + src[7].s8->off);
    w->shared_group = (int32_t)g8;
  }
  return 0;
}

size_t moe_pack_layer_bytes(moe_pack* pk, int layer) {
  if (!pk) return 0;
  pk->err.clear();
  Src src[kBlockTensors];
  if (find_block(pk, layer, src)) return 0;
  size_t total = 0;
  for (int i = 0; i < kBlockTensors; ++i) total += align_up((size_t)src[i].nbytes());
  int64_t g8 = 0;
  if (int8_shared(src, &g8))
    for (int i = 6; i <= 7; ++i) total += align_up(src[i].q8->nbytes) + align_up(src[i].s8->nbytes);
  return total;
}

int moe_pack_upload_layer(moe_pack* pk, int layer, void* dev, size_t dev_bytes, moe_layer_weights* w,
                          moe_stream_t stream) {
  if (!pk || !w) return kInvalid;
  pk->err.clear();
  Src src[kBlockTensors];
  if (int rc = find_block(pk, layer, src)) return rc;
  size_t need = 0;
  for (int i = 0; i < kBlockTensors; ++i) need += align_up((size_t)src[i].nbytes());
  int64_t g8 = 0;
  const bool i8 = int8_shared(src, &g8);
  if (i8)
    for (int i = 6; i <= 7; ++i) need += align_up(src[i].q8->nbytes) + align_up(src[i].s8->nbytes);
  if (!dev || reinterpret_cast<uintptr_t>(dev) % kDevAlign)
    return pk->set_err(kInvalid, "device region must be %zu-byte aligned", kDevAlign);
  if (dev_bytes < need) return pk->set_err(kInvalid, "device region holds %zu bytes, layer needs %zu", dev_bytes, need);
  const void* ptr[kBlockTensors];
  size_t at = 0;
  for (int i = 0; i < kBlockTensors; ++i) {
    uint8_t* dst = static_cast<uint8_t*>(dev) + at;
    const size_t n = (size_t)src[i].nbytes();
    // Pageable source (the mapping, or the dequantised rows of an int8 shared expert): the call returns after the
    // bytes are staged, so the source may be released afterwards.
    const bool cached = pk->dequant.count({layer, i}) != 0;
    const cudaError_t e =
        cudaMemcpyAsync(dst, host_block_bytes(pk, layer, i, src[i]), n, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (!src[i].e && !cached) pk->dequant.erase({layer, i});  // rows made only for this copy: already staged
    if (e != cudaSuccess) return pk->set_err((int)e, "host-to-device copy failed: %s", cudaGetErrorString(e));
    ptr[i] = dst;
    at += align_up(n);
    moe::note_pack_bytes(n);
  }
  fill_weights(pk->geo, ptr, w);
  if (i8) {
    // the int8 shared expert as stored (its bf16 rows above serve the paths that read bf16): q8 then s8 of gate_up,
    // then of down, each 256-byte aligned after the nine block tensors
    const void* dst8[4];
    const Entry* e8[4] = {src[6].q8, src[6].s8, src[7].q8, src[7].s8};
    for (int j = 0; j < 4; ++j) {
      uint8_t* dst = static_cast<uint8_t*>(dev) + at;
      const cudaError_t e =
          cudaMemcpyAsync(dst, pk->bytes() + e8[j]->off, e8[j]->nbytes, cudaMemcpyHostToDevice, (cudaStream_t)stream);
      if (e != cudaSuccess) return pk->set_err((int)e, "host-to-device copy failed: %s", cudaGetErrorString(e));
      dst8[j] = dst;
      at += align_up(e8[j]->nbytes);
      moe::note_pack_bytes(e8[j]->nbytes);
    }
    w->shared_gate_up_q8 = static_cast<const int8_t*>(dst8[0]);
    w->shared_gate_up_s8 = static_cast<const uint16_t*>(dst8[1]);
    w->shared_down_q8 = static_cast<const int8_t*>(dst8[2]);
    w->shared_down_s8 = static_cast<const uint16_t*>(dst8[3]);
    w->shared_group = (int32_t)g8;
  }
  return 0;
}

}  // extern "C"
