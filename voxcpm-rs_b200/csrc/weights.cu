// Checkpoint ingestion (reference src/weights.rs): safetensors files and PyTorch zip
// checkpoints (.pth / .pt) parsed on the host, weight_norm pairs materialised, and the
// upstream VoxCPM2 key layout mapped onto the library's model objects.
//
//   * safetensors: 8-byte little-endian header length, a JSON header {name: {dtype, shape,
//     data_offsets}} and the raw little-endian tensor bytes; the file is memory-mapped.
//   * PyTorch zip (torch.save): a stored (uncompressed) zip, zip64 when large, holding
//     <archive>/data.pkl (pickle protocol 2) and one file per storage (<archive>/data/<key>).
//     A small pickle machine rebuilds the state dict: _rebuild_tensor_v2 / _rebuild_parameter
//     over persistent storage ids; nested dicts are flattened with '.', and the container
//     prefixes "state_dict." / "model_state_dict." / "module." are stripped as
//     strip_pth_top_level does (weights.rs:400-411).  Only contiguous tensors are accepted.
//   * weight_norm (weights.rs:447-471): w[o, ...] = g[o] * v[o, ...] / max(||v[o, :]||, 1e-12).
//   * q/k/v and gate/up are uploaded as the separate tensors the checkpoint stores; the
//     library concatenates them along `out` as fuse_qkv / fuse_gate_up do (weights.rs:637-772).
//     Already-fused qkv_proj / gate_up_proj tensors are accepted too.
//   * AudioVAE keys follow the checkpoint's nn.Sequential numbering (remap_audiovae_key,
//     weights.rs:140-262): decoder.model.0 / 1 = first dw / pw conv, 2.. = decoder blocks
//     (block.0 snake, block.1 transposed conv, block.2-4 residual units whose block.0-3 are
//     snake1, conv1, snake2, conv2), then snake_out and the last conv; sr_cond_model.<2+i>.
// Weights are stored as the library keeps them: bf16 (round to nearest even) for matrices
// and convolution kernels, f32 for norms, biases, snake alphas and SR tables.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "runtime.cuh"

using namespace vx;

namespace {

thread_local std::string g_weights_err;

int werr(int code, const std::string& msg) {
  g_weights_err = msg;
  return code;
}

struct WTensor {
  std::string name;
  int dtype = -1;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
};

int dtype_size(int dt) {
  switch (dt) {
    case VX_DT_F64: case VX_DT_I64: return 8;
    case VX_DT_F32: case VX_DT_I32: return 4;
    case VX_DT_F16: case VX_DT_BF16: case VX_DT_I16: return 2;
    case VX_DT_I8: case VX_DT_U8: case VX_DT_BOOL: return 1;
  }
  return 0;
}

float half_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = s;
    } else {  // subnormal: value = m * 2^-24
      float f = (float)m * 5.9604644775390625e-8f;
      std::memcpy(&bits, &f, 4);
      bits |= s;
    }
  } else if (e == 31) {
    bits = s | 0x7f800000u | (m << 13);
  } else {
    bits = s | ((e + 112) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  const uint32_t r = 0x7fffu + ((u >> 16) & 1u);  // round to nearest, ties to even
  return (uint16_t)((u + r) >> 16);
}

float elem_f32(const uint8_t* p, int dt, size_t i) {
  switch (dt) {
    case VX_DT_F32: { float f; std::memcpy(&f, p + 4 * i, 4); return f; }
    case VX_DT_F64: { double d; std::memcpy(&d, p + 8 * i, 8); return (float)d; }
    case VX_DT_BF16: { uint16_t h; std::memcpy(&h, p + 2 * i, 2); uint32_t u = (uint32_t)h << 16; float f; std::memcpy(&f, &u, 4); return f; }
    case VX_DT_F16: { uint16_t h; std::memcpy(&h, p + 2 * i, 2); return half_to_f32(h); }
    case VX_DT_I64: { int64_t v; std::memcpy(&v, p + 8 * i, 8); return (float)v; }
    case VX_DT_I32: { int32_t v; std::memcpy(&v, p + 4 * i, 4); return (float)v; }
    case VX_DT_I16: { int16_t v; std::memcpy(&v, p + 2 * i, 2); return (float)v; }
    case VX_DT_I8: return (float)(int8_t)p[i];
    case VX_DT_U8: case VX_DT_BOOL: return (float)p[i];
  }
  return 0.f;
}

// ------------------------------------------------------------------------------ JSON

struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonParser {
  const char* p;
  const char* e;
  int depth = 0;
  bool fail = false;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool str(std::string* out) {
    if (p >= e || *p != '"') return false;
    ++p;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return false;
        const char c = *p++;
        switch (c) {
          case 'n': out->push_back('\n'); break;
          case 't': out->push_back('\t'); break;
          case 'r': out->push_back('\r'); break;
          case 'b': out->push_back('\b'); break;
          case 'f': out->push_back('\f'); break;
          case 'u': {
            if (e - p < 4) return false;
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10 : h >= 'A' && h <= 'F' ? h - 'A' + 10 : 0);
            }
            if (v < 0x80) {
              out->push_back((char)v);
            } else if (v < 0x800) {
              out->push_back((char)(0xc0 | (v >> 6)));
              out->push_back((char)(0x80 | (v & 0x3f)));
            } else {
              out->push_back((char)(0xe0 | (v >> 12)));
              out->push_back((char)(0x80 | ((v >> 6) & 0x3f)));
              out->push_back((char)(0x80 | (v & 0x3f)));
            }
            break;
          }
          default: out->push_back(c);
        }
      } else {
        out->push_back(*p++);
      }
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool value(Json* v) {
    if (++depth > 64) return false;
    ws();
    if (p >= e) return false;
    bool ok = true;
    if (*p == '{') {
      v->kind = Json::OBJ;
      ++p;
      ws();
      if (p < e && *p == '}') {
        ++p;
      } else {
        while (ok) {
          ws();
          std::string k;
          if (!str(&k)) return false;
          ws();
          if (p >= e || *p != ':') return false;
          ++p;
          v->obj.emplace_back(k, Json());
          if (!value(&v->obj.back().second)) return false;
          ws();
          if (p < e && *p == ',') { ++p; continue; }
          if (p < e && *p == '}') { ++p; break; }
          return false;
        }
      }
    } else if (*p == '[') {
      v->kind = Json::ARR;
      ++p;
      ws();
      if (p < e && *p == ']') {
        ++p;
      } else {
        while (true) {
          v->arr.emplace_back();
          if (!value(&v->arr.back())) return false;
          ws();
          if (p < e && *p == ',') { ++p; continue; }
          if (p < e && *p == ']') { ++p; break; }
          return false;
        }
      }
    } else if (*p == '"') {
      v->kind = Json::STR;
      ok = str(&v->str);
    } else if (e - p >= 4 && !std::strncmp(p, "true", 4)) {
      v->kind = Json::BOOL; v->num = 1; p += 4;
    } else if (e - p >= 5 && !std::strncmp(p, "false", 5)) {
      v->kind = Json::BOOL; p += 5;
    } else if (e - p >= 4 && !std::strncmp(p, "null", 4)) {
      v->kind = Json::NUL; p += 4;
    } else {
      v->kind = Json::NUM;
      const char* s = p;
      while (p < e && (std::strchr("+-0123456789.eE", *p) != nullptr)) ++p;
      if (p == s) return false;
      v->num = std::strtod(std::string(s, p).c_str(), nullptr);
    }
    --depth;
    return ok;
  }
};

// ------------------------------------------------------------------------------ zip

struct ZipEntry {
  std::string name;
  uint64_t offset = 0;  // of the stored data
  uint64_t size = 0;
};

template <typename T>
bool rd(const uint8_t* base, size_t len, uint64_t off, T* v) {
  if (off + sizeof(T) > len) return false;
  std::memcpy(v, base + off, sizeof(T));
  return true;
}

int zip_entries(const uint8_t* b, size_t len, std::vector<ZipEntry>* out) {
  // end of central directory: signature 0x06054b50 within the last 64 KB + 22 bytes
  if (len < 22) return werr(VX_ERR_CONFIG, "zip: file too short");
  int64_t eocd = -1;
  for (int64_t i = (int64_t)len - 22; i >= 0 && i >= (int64_t)len - 22 - 65535; --i) {
    uint32_t sig;
    rd(b, len, (uint64_t)i, &sig);
    if (sig == 0x06054b50u) { eocd = i; break; }
  }
  if (eocd < 0) return werr(VX_ERR_CONFIG, "zip: no end-of-central-directory record");
  uint16_t n16 = 0;
  uint32_t cd_size32 = 0, cd_off32 = 0;
  rd(b, len, eocd + 10, &n16);
  rd(b, len, eocd + 12, &cd_size32);
  rd(b, len, eocd + 16, &cd_off32);
  uint64_t n = n16, cd_off = cd_off32;
  if (n16 == 0xffff || cd_off32 == 0xffffffffu || cd_size32 == 0xffffffffu) {
    // zip64: locator just before the EOCD record points at the zip64 EOCD record
    uint32_t lsig = 0;
    uint64_t z64 = 0;
    if (eocd < 20 || !rd(b, len, eocd - 20, &lsig) || lsig != 0x07064b50u || !rd(b, len, eocd - 20 + 8, &z64))
      return werr(VX_ERR_CONFIG, "zip: missing zip64 locator");
    uint32_t zsig = 0;
    if (!rd(b, len, z64, &zsig) || zsig != 0x06064b50u) return werr(VX_ERR_CONFIG, "zip: bad zip64 record");
    rd(b, len, z64 + 32, &n);
    rd(b, len, z64 + 48, &cd_off);
  }
  uint64_t p = cd_off;
  for (uint64_t k = 0; k < n; ++k) {
    uint32_t sig = 0;
    if (!rd(b, len, p, &sig) || sig != 0x02014b50u) return werr(VX_ERR_CONFIG, "zip: bad central directory entry");
    uint16_t method = 0, nlen = 0, xlen = 0, clen = 0;
    uint32_t csize = 0, usize = 0, loff = 0;
    rd(b, len, p + 10, &method);
    rd(b, len, p + 20, &csize);
    rd(b, len, p + 24, &usize);
    rd(b, len, p + 28, &nlen);
    rd(b, len, p + 30, &xlen);
    rd(b, len, p + 32, &clen);
    rd(b, len, p + 42, &loff);
    if (p + 46 + nlen > len) return werr(VX_ERR_CONFIG, "zip: truncated entry name");
    ZipEntry z;
    z.name.assign(reinterpret_cast<const char*>(b + p + 46), nlen);
    uint64_t size = usize, off = loff, csz = csize;
    // zip64 extra field (id 1): the 0xffffffff fields in order usize, csize, offset
    uint64_t x = p + 46 + nlen, xe = x + xlen;
    while (x + 4 <= xe) {
      uint16_t id = 0, sz = 0;
      rd(b, len, x, &id);
      rd(b, len, x + 2, &sz);
      if (id == 1) {
        uint64_t q = x + 4;
        if (usize == 0xffffffffu) { rd(b, len, q, &size); q += 8; }
        if (csize == 0xffffffffu) { rd(b, len, q, &csz); q += 8; }
        if (loff == 0xffffffffu) { rd(b, len, q, &off); q += 8; }
      }
      x += 4 + sz;
    }
    if (method != 0 || csz != size) return werr(VX_ERR_CONFIG, "zip: compressed entry " + z.name + " (only stored entries)");
    uint32_t lsig = 0;
    uint16_t lnlen = 0, lxlen = 0;
    if (!rd(b, len, off, &lsig) || lsig != 0x04034b50u) return werr(VX_ERR_CONFIG, "zip: bad local header");
    rd(b, len, off + 26, &lnlen);
    rd(b, len, off + 28, &lxlen);
    z.offset = off + 30 + lnlen + lxlen;
    z.size = size;
    if (z.offset + z.size > len) return werr(VX_ERR_CONFIG, "zip: entry past the end of the file");
    out->push_back(z);
    p += 46 + nlen + xlen + clen;
  }
  return VX_OK;
}

// ------------------------------------------------------------------------------ pickle

struct PVal;
using PRef = std::shared_ptr<PVal>;
struct PVal {
  enum Kind { NONE, BOOL, INT, FLOAT, STR, TUPLE, LIST, DICT, GLOBAL, STORAGE, TENSOR, MARK, OTHER } kind = NONE;
  int64_t i = 0;
  double f = 0;
  std::string s, s2;                 // STR; GLOBAL module, name; STORAGE key
  std::vector<PRef> items;           // TUPLE / LIST
  std::vector<std::pair<PRef, PRef>> dict;
  int dtype = -1;                    // STORAGE / TENSOR
  PRef storage;                      // TENSOR
  int64_t offset = 0;
  std::vector<int64_t> shape, stride;
};

PRef mk(PVal::Kind k) {
  auto v = std::make_shared<PVal>();
  v->kind = k;
  return v;
}

int storage_dtype(const std::string& cls) {
  static const std::pair<const char*, int> t[] = {
      {"FloatStorage", VX_DT_F32}, {"HalfStorage", VX_DT_F16}, {"BFloat16Storage", VX_DT_BF16},
      {"DoubleStorage", VX_DT_F64}, {"LongStorage", VX_DT_I64}, {"IntStorage", VX_DT_I32},
      {"ShortStorage", VX_DT_I16}, {"CharStorage", VX_DT_I8}, {"ByteStorage", VX_DT_U8}, {"BoolStorage", VX_DT_BOOL}};
  for (auto& e : t)
    if (cls == e.first) return e.second;
  return -1;
}

bool int_list(const PRef& v, std::vector<int64_t>* out) {
  if (!v || (v->kind != PVal::TUPLE && v->kind != PVal::LIST)) return false;
  for (auto& x : v->items) {
    if (x->kind != PVal::INT) return false;
    out->push_back(x->i);
  }
  return true;
}

int unpickle(const uint8_t* b, size_t len, PRef* result) {
  std::vector<PRef> st;
  std::vector<size_t> marks;
  std::map<uint64_t, PRef> memo;
  size_t p = 0;
  auto need = [&](size_t n) { return p + n <= len; };
  auto pop = [&]() -> PRef {
    if (st.empty()) return nullptr;
    PRef v = st.back();
    st.pop_back();
    return v;
  };
  auto pop_mark = [&](std::vector<PRef>* items) -> bool {
    if (marks.empty()) return false;
    const size_t m = marks.back();
    marks.pop_back();
    if (m > st.size()) return false;
    items->assign(st.begin() + m, st.end());
    st.resize(m);
    return true;
  };
  auto rd_str = [&](size_t n, std::string* s) -> bool {
    if (!need(n)) return false;
    s->assign(reinterpret_cast<const char*>(b + p), n);
    p += n;
    return true;
  };
  auto line = [&](std::string* s) -> bool {
    const size_t q = p;
    while (p < len && b[p] != '\n') ++p;
    if (p >= len) return false;
    s->assign(reinterpret_cast<const char*>(b + q), p - q);
    ++p;
    return true;
  };
  const char* bad = "pickle: malformed data";
  for (int guard = 0; guard < (1 << 28); ++guard) {
    if (p >= len) return werr(VX_ERR_CONFIG, "pickle: no STOP");
    const uint8_t op = b[p++];
    switch (op) {
      case 0x80: if (!need(1)) return werr(VX_ERR_CONFIG, bad); p += 1; break;        // PROTO
      case 0x95: if (!need(8)) return werr(VX_ERR_CONFIG, bad); p += 8; break;        // FRAME
      case '.': *result = pop(); return *result ? VX_OK : werr(VX_ERR_CONFIG, bad);  // STOP
      case '(': marks.push_back(st.size()); break;                                   // MARK
      case '}': st.push_back(mk(PVal::DICT)); break;
      case ']': st.push_back(mk(PVal::LIST)); break;
      case ')': st.push_back(mk(PVal::TUPLE)); break;
      case 'N': st.push_back(mk(PVal::NONE)); break;
      case 0x88: case 0x89: { auto v = mk(PVal::BOOL); v->i = op == 0x88; st.push_back(v); break; }
      case 'K': { if (!need(1)) return werr(VX_ERR_CONFIG, bad); auto v = mk(PVal::INT); v->i = b[p]; p += 1; st.push_back(v); break; }
      case 'M': { uint16_t x; if (!rd(b, len, p, &x)) return werr(VX_ERR_CONFIG, bad); p += 2; auto v = mk(PVal::INT); v->i = x; st.push_back(v); break; }
      case 'J': { int32_t x; if (!rd(b, len, p, &x)) return werr(VX_ERR_CONFIG, bad); p += 4; auto v = mk(PVal::INT); v->i = x; st.push_back(v); break; }
      case 0x8a: {  // LONG1
        if (!need(1)) return werr(VX_ERR_CONFIG, bad);
        const int n = b[p++];
        if (n > 8 || !need(n)) return werr(VX_ERR_CONFIG, "pickle: long integer too wide");
        int64_t x = 0;
        for (int i = 0; i < n; ++i) x |= (int64_t)b[p + i] << (8 * i);
        if (n > 0 && n < 8 && (b[p + n - 1] & 0x80)) x -= (int64_t)1 << (8 * n);
        p += n;
        auto v = mk(PVal::INT);
        v->i = x;
        st.push_back(v);
        break;
      }
      case 'G': {  // BINFLOAT (big endian)
        if (!need(8)) return werr(VX_ERR_CONFIG, bad);
        uint64_t u = 0;
        for (int i = 0; i < 8; ++i) u = (u << 8) | b[p + i];
        p += 8;
        auto v = mk(PVal::FLOAT);
        std::memcpy(&v->f, &u, 8);
        st.push_back(v);
        break;
      }
      case 'X': case 0x8c: case 0x8d: case 'T': case 'U': case 'B': case 'C': {  // strings / bytes
        uint64_t n = 0;
        if (op == 'X' || op == 'T' || op == 'B') { uint32_t x; if (!rd(b, len, p, &x)) return werr(VX_ERR_CONFIG, bad); n = x; p += 4; }
        else if (op == 0x8d) { if (!rd(b, len, p, &n)) return werr(VX_ERR_CONFIG, bad); p += 8; }
        else { if (!need(1)) return werr(VX_ERR_CONFIG, bad); n = b[p++]; }
        auto v = mk(PVal::STR);
        if (!rd_str(n, &v->s)) return werr(VX_ERR_CONFIG, bad);
        st.push_back(v);
        break;
      }
      case 'c': {  // GLOBAL module\nname\n
        auto v = mk(PVal::GLOBAL);
        if (!line(&v->s) || !line(&v->s2)) return werr(VX_ERR_CONFIG, bad);
        st.push_back(v);
        break;
      }
      case 0x93: {  // STACK_GLOBAL
        PRef name = pop(), mod = pop();
        if (!name || !mod) return werr(VX_ERR_CONFIG, bad);
        auto v = mk(PVal::GLOBAL);
        v->s = mod->s;
        v->s2 = name->s;
        st.push_back(v);
        break;
      }
      case 'q': { if (!need(1) || st.empty()) return werr(VX_ERR_CONFIG, bad); memo[b[p]] = st.back(); p += 1; break; }
      case 'r': { uint32_t k; if (!rd(b, len, p, &k) || st.empty()) return werr(VX_ERR_CONFIG, bad); memo[k] = st.back(); p += 4; break; }
      case 0x94: { if (st.empty()) return werr(VX_ERR_CONFIG, bad); const uint64_t k = memo.size(); memo[k] = st.back(); break; }
      case 'h': case 'j': {
        uint64_t k = 0;
        if (op == 'h') { if (!need(1)) return werr(VX_ERR_CONFIG, bad); k = b[p++]; }
        else { uint32_t x; if (!rd(b, len, p, &x)) return werr(VX_ERR_CONFIG, bad); k = x; p += 4; }
        auto it = memo.find(k);
        if (it == memo.end()) return werr(VX_ERR_CONFIG, "pickle: memo miss");
        st.push_back(it->second);
        break;
      }
      case 't': { auto v = mk(PVal::TUPLE); if (!pop_mark(&v->items)) return werr(VX_ERR_CONFIG, bad); st.push_back(v); break; }
      case 'l': { auto v = mk(PVal::LIST); if (!pop_mark(&v->items)) return werr(VX_ERR_CONFIG, bad); st.push_back(v); break; }
      case 'd': {
        std::vector<PRef> it;
        if (!pop_mark(&it) || it.size() % 2) return werr(VX_ERR_CONFIG, bad);
        auto v = mk(PVal::DICT);
        for (size_t i = 0; i < it.size(); i += 2) v->dict.emplace_back(it[i], it[i + 1]);
        st.push_back(v);
        break;
      }
      case 0x85: case 0x86: case 0x87: {
        const int n = op - 0x84;
        if ((int)st.size() < n) return werr(VX_ERR_CONFIG, bad);
        auto v = mk(PVal::TUPLE);
        v->items.assign(st.end() - n, st.end());
        st.resize(st.size() - n);
        st.push_back(v);
        break;
      }
      case 'a': { PRef x = pop(); if (!x || st.empty()) return werr(VX_ERR_CONFIG, bad); st.back()->items.push_back(x); break; }
      case 'e': {
        std::vector<PRef> it;
        if (!pop_mark(&it) || st.empty()) return werr(VX_ERR_CONFIG, bad);
        for (auto& x : it) st.back()->items.push_back(x);
        break;
      }
      case 's': {
        PRef v = pop(), k = pop();
        if (!v || !k || st.empty()) return werr(VX_ERR_CONFIG, bad);
        st.back()->dict.emplace_back(k, v);
        break;
      }
      case 'u': {
        std::vector<PRef> it;
        if (!pop_mark(&it) || it.size() % 2 || st.empty()) return werr(VX_ERR_CONFIG, bad);
        for (size_t i = 0; i < it.size(); i += 2) st.back()->dict.emplace_back(it[i], it[i + 1]);
        break;
      }
      case 'b': { if (!pop() || st.empty()) return werr(VX_ERR_CONFIG, bad); break; }  // BUILD: state ignored
      case 'Q': {  // BINPERSID: ('storage', <class>, key, location, numel)
        PRef pid = pop();
        if (!pid || pid->kind != PVal::TUPLE || pid->items.size() < 5 || pid->items[1]->kind != PVal::GLOBAL)
          return werr(VX_ERR_CONFIG, "pickle: unsupported persistent id");
        auto v = mk(PVal::STORAGE);
        v->dtype = storage_dtype(pid->items[1]->s2);
        v->s = pid->items[2]->s;
        v->i = pid->items[4]->kind == PVal::INT ? pid->items[4]->i : 0;
        if (v->dtype < 0) return werr(VX_ERR_CONFIG, "pickle: unsupported storage " + pid->items[1]->s2);
        st.push_back(v);
        break;
      }
      case 'R': case 0x81: {  // REDUCE / NEWOBJ
        PRef args = pop(), fn = pop();
        if (!args || !fn) return werr(VX_ERR_CONFIG, bad);
        PRef out;
        const std::string q = fn->kind == PVal::GLOBAL ? fn->s + "." + fn->s2 : "";
        if (q == "collections.OrderedDict" || q == "builtins.dict") {
          out = mk(PVal::DICT);
        } else if (q == "torch._utils._rebuild_tensor_v2" || q == "torch._utils._rebuild_tensor") {
          if (args->items.size() < 4 || args->items[0]->kind != PVal::STORAGE || args->items[1]->kind != PVal::INT)
            return werr(VX_ERR_CONFIG, "pickle: bad tensor record");
          out = mk(PVal::TENSOR);
          out->storage = args->items[0];
          out->dtype = out->storage->dtype;
          out->offset = args->items[1]->i;
          if (!int_list(args->items[2], &out->shape) || !int_list(args->items[3], &out->stride))
            return werr(VX_ERR_CONFIG, "pickle: bad tensor shape");
        } else if (q == "torch._utils._rebuild_parameter" || q == "torch._utils._rebuild_parameter_with_state") {
          if (args->items.empty()) return werr(VX_ERR_CONFIG, bad);
          out = args->items[0];
        } else {
          out = mk(PVal::OTHER);
        }
        st.push_back(out);
        break;
      }
      default: {
        char m[64];
        snprintf(m, sizeof(m), "pickle: unsupported opcode 0x%02x", op);
        return werr(VX_ERR_CONFIG, m);
      }
    }
  }
  return werr(VX_ERR_CONFIG, "pickle: too long");
}

}  // namespace

struct vx_weights {
  void* map = nullptr;
  size_t map_len = 0;
  std::vector<WTensor> tensors;
  std::map<std::string, int> index;
};

namespace {

int add_tensor(vx_weights* w, WTensor t) {
  size_t n = 1;
  for (int64_t d : t.shape) {
    if (d < 0) return werr(VX_ERR_CONFIG, "negative dimension in " + t.name);
    n *= (size_t)d;
  }
  if (n * dtype_size(t.dtype) != t.nbytes) return werr(VX_ERR_CONFIG, "size mismatch for " + t.name);
  if (w->index.count(t.name)) return werr(VX_ERR_CONFIG, "duplicate tensor " + t.name);
  w->index[t.name] = (int)w->tensors.size();
  w->tensors.push_back(std::move(t));
  return VX_OK;
}

int parse_safetensors(vx_weights* w) {
  const uint8_t* b = static_cast<const uint8_t*>(w->map);
  uint64_t hlen = 0;
  if (!rd(b, w->map_len, 0, &hlen) || 8 + hlen > w->map_len) return werr(VX_ERR_CONFIG, "safetensors: bad header length");
  JsonParser jp{reinterpret_cast<const char*>(b + 8), reinterpret_cast<const char*>(b + 8 + hlen)};
  Json root;
  if (!jp.value(&root) || root.kind != Json::OBJ) return werr(VX_ERR_CONFIG, "safetensors: bad JSON header");
  const uint8_t* data = b + 8 + hlen;
  const size_t dlen = w->map_len - 8 - hlen;
  static const std::pair<const char*, int> dts[] = {{"F32", VX_DT_F32}, {"F16", VX_DT_F16}, {"BF16", VX_DT_BF16},
                                                    {"F64", VX_DT_F64}, {"I64", VX_DT_I64}, {"I32", VX_DT_I32},
                                                    {"I16", VX_DT_I16}, {"I8", VX_DT_I8}, {"U8", VX_DT_U8},
                                                    {"BOOL", VX_DT_BOOL}};
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const Json* dt = kv.second.get("dtype");
    const Json* sh = kv.second.get("shape");
    const Json* of = kv.second.get("data_offsets");
    if (!dt || !sh || !of || dt->kind != Json::STR || sh->kind != Json::ARR || of->kind != Json::ARR || of->arr.size() != 2)
      return werr(VX_ERR_CONFIG, "safetensors: bad entry " + kv.first);
    WTensor t;
    t.name = kv.first;
    for (auto& d : dts)
      if (dt->str == d.first) t.dtype = d.second;
    if (t.dtype < 0) return werr(VX_ERR_CONFIG, "safetensors: unsupported dtype " + dt->str);
    for (auto& d : sh->arr) t.shape.push_back((int64_t)d.num);
    const uint64_t o0 = (uint64_t)of->arr[0].num, o1 = (uint64_t)of->arr[1].num;
    if (o1 < o0 || o1 > dlen) return werr(VX_ERR_CONFIG, "safetensors: offsets out of range for " + kv.first);
    t.data = data + o0;
    t.nbytes = o1 - o0;
    const int rc = add_tensor(w, std::move(t));
    if (rc) return rc;
  }
  return VX_OK;
}

void flatten(vx_weights* w, const PRef& v, const std::string& prefix, std::map<std::string, PRef>* out) {
  if (v->kind == PVal::DICT) {
    for (auto& kv : v->dict)
      if (kv.first->kind == PVal::STR) flatten(w, kv.second, prefix.empty() ? kv.first->s : prefix + "." + kv.first->s, out);
  } else if (v->kind == PVal::TENSOR) {
    (*out)[prefix] = v;
  }
}

std::string strip_top(const std::string& n) {
  for (const char* pre : {"state_dict.", "model_state_dict.", "module."})
    if (n.compare(0, std::strlen(pre), pre) == 0) return n.substr(std::strlen(pre));
  return n;
}

int parse_torch_zip(vx_weights* w) {
  const uint8_t* b = static_cast<const uint8_t*>(w->map);
  std::vector<ZipEntry> ents;
  int rc = zip_entries(b, w->map_len, &ents);
  if (rc) return rc;
  const ZipEntry* pkl = nullptr;
  std::string root;
  for (auto& e : ents) {
    const size_t k = e.name.rfind("/data.pkl");
    if (k != std::string::npos && k + 9 == e.name.size()) {
      pkl = &e;
      root = e.name.substr(0, k + 1);
    }
  }
  if (!pkl) return werr(VX_ERR_CONFIG, "torch zip: no data.pkl");
  std::map<std::string, const ZipEntry*> files;
  for (auto& e : ents) files[e.name] = &e;
  PRef top;
  rc = unpickle(b + pkl->offset, pkl->size, &top);
  if (rc) return rc;
  std::map<std::string, PRef> flat;
  flatten(w, top, "", &flat);
  for (auto& kv : flat) {
    const PVal& t = *kv.second;
    auto f = files.find(root + "data/" + t.storage->s);
    if (f == files.end()) return werr(VX_ERR_CONFIG, "torch zip: missing storage " + t.storage->s);
    // contiguous only
    int64_t expect = 1;
    for (int i = (int)t.shape.size() - 1; i >= 0; --i) {
      if (t.shape[i] != 1 && (i >= (int)t.stride.size() || t.stride[i] != expect))
        return werr(VX_ERR_CONFIG, "torch zip: non-contiguous tensor " + kv.first);
      expect *= t.shape[i];
    }
    WTensor wt;
    wt.name = strip_top(kv.first);
    wt.dtype = t.dtype;
    wt.shape = t.shape;
    const size_t es = dtype_size(t.dtype);
    wt.nbytes = (size_t)expect * es;
    if ((uint64_t)t.offset * es + wt.nbytes > f->second->size)
      return werr(VX_ERR_CONFIG, "torch zip: tensor past its storage " + kv.first);
    wt.data = b + f->second->offset + (size_t)t.offset * es;
    rc = add_tensor(w, std::move(wt));
    if (rc) return rc;
  }
  return VX_OK;
}

// ------------------------------------------------------------------------------ readers

const WTensor* find(const vx_weights* w, const std::string& name) {
  auto it = w->index.find(name);
  return it == w->index.end() ? nullptr : &w->tensors[it->second];
}

size_t numel(const WTensor& t) {
  size_t n = 1;
  for (int64_t d : t.shape) n *= (size_t)d;
  return n;
}

void convert(const WTensor& t, int out_dt, void* out) {
  const size_t n = numel(t);
  if (out_dt == VX_DT_F32) {
    float* o = static_cast<float*>(out);
    for (size_t i = 0; i < n; ++i) o[i] = elem_f32(t.data, t.dtype, i);
  } else if (t.dtype == VX_DT_BF16) {
    std::memcpy(out, t.data, n * 2);
  } else {
    uint16_t* o = static_cast<uint16_t*>(out);
    for (size_t i = 0; i < n; ++i) o[i] = f32_to_bf16(elem_f32(t.data, t.dtype, i));
  }
}

// A weight by name: the tensor itself, or its weight_norm pair (<stem>.weight_g / _v) when
// `name` ends in ".weight".  Returns the element count through *n, the shape through *shape.
int get_weight(const vx_weights* w, const std::string& name, int out_dt, std::vector<uint8_t>* buf,
               std::vector<int64_t>* shape) {
  const int es = out_dt == VX_DT_F32 ? 4 : 2;
  if (const WTensor* t = find(w, name)) {
    buf->resize(numel(*t) * es);
    convert(*t, out_dt, buf->data());
    *shape = t->shape;
    return VX_OK;
  }
  const std::string stem = name.size() > 7 && name.compare(name.size() - 7, 7, ".weight") == 0
                               ? name.substr(0, name.size() - 7) : name;
  const WTensor* g = find(w, stem + ".weight_g");
  const WTensor* v = find(w, stem + ".weight_v");
  if (!g || !v) return werr(VX_ERR_ARG, "missing weight " + name);
  if (v->shape.empty() || numel(*g) != (size_t)v->shape[0])
    return werr(VX_ERR_SHAPE, "weight_norm: g does not match v's first dimension for " + stem);
  const size_t co = (size_t)v->shape[0], inner = numel(*v) / co;
  buf->resize(numel(*v) * es);
  for (size_t o = 0; o < co; ++o) {
    double ss = 0.0;
    for (size_t j = 0; j < inner; ++j) {
      const double x = elem_f32(v->data, v->dtype, o * inner + j);
      ss += x * x;
    }
    const float norm = std::max((float)std::sqrt(ss), 1e-12f);
    const float scale = elem_f32(g->data, g->dtype, o) / norm;
    for (size_t j = 0; j < inner; ++j) {
      const float x = elem_f32(v->data, v->dtype, o * inner + j) * scale;
      if (out_dt == VX_DT_F32)
        reinterpret_cast<float*>(buf->data())[o * inner + j] = x;
      else
        reinterpret_cast<uint16_t*>(buf->data())[o * inner + j] = f32_to_bf16(x);
    }
  }
  *shape = v->shape;
  return VX_OK;
}

size_t prod(const std::vector<int64_t>& s) {
  size_t n = 1;
  for (int64_t d : s) n *= (size_t)d;
  return n;
}

// Loader helper: named weights converted to host buffers, checked against an element count.
struct Loader {
  const vx_weights* w;
  vx_ctx* ctx;
  std::vector<std::vector<uint8_t>> keep;
  int rc = VX_OK;
  const void* get(const std::string& name, int dt, size_t expect) {
    if (rc) return nullptr;
    keep.emplace_back();
    std::vector<int64_t> shape;
    const int r = get_weight(w, name, dt, &keep.back(), &shape);
    if (r) {
      rc = fail(ctx, r, "%s", g_weights_err.c_str());
      return nullptr;
    }
    if (prod(shape) != expect) {
      rc = fail(ctx, VX_ERR_SHAPE, "%s: %zu elements, expected %zu", name.c_str(), prod(shape), expect);
      return nullptr;
    }
    return keep.back().data();
  }
  const uint16_t* bf(const std::string& n, size_t e) { return static_cast<const uint16_t*>(get(n, VX_DT_BF16, e)); }
  const float* f32(const std::string& n, size_t e) { return static_cast<const float*>(get(n, VX_DT_F32, e)); }
};

int load_lm(vx_lm* lm, const vx_weights* w, const std::string& P, bool is_dit, vx_dit* dit) {
  int L, H, I, qs, ks, V;
  lm_dims(lm, &L, &H, &I, &qs, &ks, &V);
  vx_ctx* ctx = lm_ctx(lm);
  for (int l = 0; l < L; ++l) {
    Loader ld{w, ctx};
    const std::string p = P + "layers." + std::to_string(l) + ".";
    const uint16_t *q, *k, *v, *gate, *up;
    if (find(w, p + "self_attn.qkv_proj.weight")) {  // already fused (q | k | v along out)
      const uint16_t* qkv = ld.bf(p + "self_attn.qkv_proj.weight", (size_t)(qs + 2 * ks) * H);
      q = qkv;
      k = qkv ? qkv + (size_t)qs * H : nullptr;
      v = qkv ? qkv + (size_t)(qs + ks) * H : nullptr;
    } else {
      q = ld.bf(p + "self_attn.q_proj.weight", (size_t)qs * H);
      k = ld.bf(p + "self_attn.k_proj.weight", (size_t)ks * H);
      v = ld.bf(p + "self_attn.v_proj.weight", (size_t)ks * H);
    }
    const uint16_t* o = ld.bf(p + "self_attn.o_proj.weight", (size_t)H * qs);
    if (find(w, p + "mlp.gate_up_proj.weight")) {
      const uint16_t* gu = ld.bf(p + "mlp.gate_up_proj.weight", (size_t)2 * I * H);
      gate = gu;
      up = gu ? gu + (size_t)I * H : nullptr;
    } else {
      gate = ld.bf(p + "mlp.gate_proj.weight", (size_t)I * H);
      up = ld.bf(p + "mlp.up_proj.weight", (size_t)I * H);
    }
    const uint16_t* down = ld.bf(p + "mlp.down_proj.weight", (size_t)H * I);
    const float* ln_in = ld.f32(p + "input_layernorm.weight", H);
    const float* ln_post = ld.f32(p + "post_attention_layernorm.weight", H);
    if (ld.rc) return ld.rc;
    const int rc = is_dit ? vx_dit_load_layer(dit, l, q, k, v, o, gate, up, down, ln_in, ln_post)
                          : vx_lm_load_layer(lm, l, q, k, v, o, gate, up, down, ln_in, ln_post);
    if (rc) return rc;
  }
  Loader ld{w, ctx};
  const float* norm = ld.f32(P + "norm.weight", H);
  if (ld.rc) return ld.rc;
  int rc = is_dit ? vx_dit_load_norm(dit, norm) : vx_lm_load_norm(lm, norm);
  if (rc) return rc;
  if (V > 0 && !is_dit) {
    const uint16_t* e = ld.bf(P + "embed_tokens.weight", (size_t)V * H);
    if (ld.rc) return ld.rc;
    rc = vx_lm_load_embed(lm, e);
  }
  return rc;
}

}  // namespace

extern "C" {

const char* vx_weights_last_error(void) { return g_weights_err.c_str(); }

int vx_weights_open(const char* path, vx_weights** out) {
  if (!path || !out) return VX_ERR_ARG;
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return werr(VX_ERR_ARG, std::string("cannot open ") + path);
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
    close(fd);
    return werr(VX_ERR_CONFIG, std::string("not a checkpoint: ") + path);
  }
  void* m = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return werr(VX_ERR_OOM, std::string("mmap failed: ") + path);
  vx_weights* w = new vx_weights();
  w->map = m;
  w->map_len = (size_t)sb.st_size;
  const uint8_t* b = static_cast<const uint8_t*>(m);
  const int rc = (b[0] == 'P' && b[1] == 'K') ? parse_torch_zip(w) : parse_safetensors(w);
  if (rc) {
    vx_weights_close(w);
    return rc;
  }
  *out = w;
  return VX_OK;
}

void vx_weights_close(vx_weights* w) {
  if (!w) return;
  if (w->map) munmap(w->map, w->map_len);
  delete w;
}

int vx_weights_count(const vx_weights* w) { return w ? (int)w->tensors.size() : 0; }

const char* vx_weights_name(const vx_weights* w, int i) {
  return (w && i >= 0 && i < (int)w->tensors.size()) ? w->tensors[i].name.c_str() : nullptr;
}

int vx_weights_find(const vx_weights* w, const char* name) {
  if (!w || !name) return -1;
  auto it = w->index.find(name);
  return it == w->index.end() ? -1 : it->second;
}

int vx_weights_info(const vx_weights* w, int i, int* dtype, int64_t* shape, int max_dims) {
  if (!w || i < 0 || i >= (int)w->tensors.size()) return -1;
  const WTensor& t = w->tensors[i];
  if (dtype) *dtype = t.dtype;
  for (int d = 0; d < (int)t.shape.size() && d < max_dims; ++d) shape[d] = t.shape[d];
  return (int)t.shape.size();
}

int vx_weights_read(const vx_weights* w, const char* name, int out_dtype, void* out, size_t n_elems) {
  if (!w || !name || !out || (out_dtype != VX_DT_F32 && out_dtype != VX_DT_BF16)) return VX_ERR_ARG;
  std::vector<uint8_t> buf;
  std::vector<int64_t> shape;
  const int rc = get_weight(w, name, out_dtype, &buf, &shape);
  if (rc) return rc;
  if (prod(shape) != n_elems) return werr(VX_ERR_SHAPE, std::string("element count mismatch for ") + name);
  std::memcpy(out, buf.data(), buf.size());
  return VX_OK;
}

int vx_lm_load_weights(vx_lm* lm, const vx_weights* w, const char* prefix) {
  if (!lm || !w) return VX_ERR_ARG;
  return load_lm(lm, w, prefix ? prefix : "", false, nullptr);
}

int vx_dit_load_weights(vx_dit* d, const vx_weights* w, const char* prefix) {
  if (!d || !w) return VX_ERR_ARG;
  const std::string P = prefix ? prefix : "";
  int H, C;
  vx_lm* dec = dit_decoder(d, &H, &C);
  Loader ld{w, dit_ctx(d)};
  const uint16_t* in_w = ld.bf(P + "in_proj.weight", (size_t)H * C);
  const float* in_b = ld.f32(P + "in_proj.bias", H);
  const uint16_t* cond_w = ld.bf(P + "cond_proj.weight", (size_t)H * C);
  const float* cond_b = ld.f32(P + "cond_proj.bias", H);
  const uint16_t* out_w = ld.bf(P + "out_proj.weight", (size_t)C * H);
  const float* out_b = ld.f32(P + "out_proj.bias", C);
  const uint16_t* t1w = ld.bf(P + "time_mlp.linear_1.weight", (size_t)H * H);
  const float* t1b = ld.f32(P + "time_mlp.linear_1.bias", H);
  const uint16_t* t2w = ld.bf(P + "time_mlp.linear_2.weight", (size_t)H * H);
  const float* t2b = ld.f32(P + "time_mlp.linear_2.bias", H);
  const uint16_t* d1w = ld.bf(P + "delta_time_mlp.linear_1.weight", (size_t)H * H);
  const float* d1b = ld.f32(P + "delta_time_mlp.linear_1.bias", H);
  const uint16_t* d2w = ld.bf(P + "delta_time_mlp.linear_2.weight", (size_t)H * H);
  const float* d2b = ld.f32(P + "delta_time_mlp.linear_2.bias", H);
  if (ld.rc) return ld.rc;
  int rc = vx_dit_load(d, in_w, in_b, cond_w, cond_b, out_w, out_b, t1w, t1b, t2w, t2b, d1w, d1b, d2w, d2b);
  if (rc) return rc;
  return load_lm(dec, w, P + "decoder.", true, d);
}

int vx_vae_load_weights(vx_vae* v, const vx_weights* w, const char* prefix) {
  if (!v || !w) return VX_ERR_ARG;
  const std::string P = std::string(prefix ? prefix : "") + "decoder.";
  VaeDims vd;
  vae_dims(v, &vd);
  Loader ld{w, vae_ctx(v)};
  const size_t L = vd.latent, D = vd.dim;
  const uint16_t* dw_w = ld.bf(P + "model.0.weight", L * 7);
  const float* dw_b = ld.f32(P + "model.0.bias", L);
  const uint16_t* pw_w = ld.bf(P + "model.1.weight", D * L);
  const float* pw_b = ld.f32(P + "model.1.bias", D);
  if (ld.rc) return ld.rc;
  int rc = vx_vae_load_first(v, dw_w, dw_b, pw_w, pw_b);
  if (rc) return rc;
  for (int i = 0; i < vd.nblocks; ++i) {
    Loader lb{w, vae_ctx(v)};
    const size_t ci = D >> i, co = D >> (i + 1), s = vd.rates[i];
    const std::string b = P + "model." + std::to_string(2 + i) + ".block.";
    vx_vae_block_weights bw = {};
    bw.alpha = lb.f32(b + "0.alpha", ci);
    bw.up_w = lb.bf(b + "1.weight", ci * co * 2 * s);
    bw.up_b = lb.f32(b + "1.bias", co);
    for (int u = 0; u < 3; ++u) {
      const std::string r = b + std::to_string(2 + u) + ".block.";
      bw.res_alpha1[u] = lb.f32(r + "0.alpha", co);
      bw.res_w1[u] = lb.bf(r + "1.weight", co * 7);
      bw.res_b1[u] = lb.f32(r + "1.bias", co);
      bw.res_alpha2[u] = lb.f32(r + "2.alpha", co);
      bw.res_w2[u] = lb.bf(r + "3.weight", co * co);
      bw.res_b2[u] = lb.f32(r + "3.bias", co);
    }
    if (vd.n_buckets > 0) {
      const std::string c = P + "sr_cond_model." + std::to_string(2 + i) + ".";
      bw.sr_scale = lb.f32(c + "scale_embed.weight", (size_t)vd.n_buckets * ci);
      bw.sr_bias = lb.f32(c + "bias_embed.weight", (size_t)vd.n_buckets * ci);
    }
    if (lb.rc) return lb.rc;
    rc = vx_vae_load_block(v, i, &bw);
    if (rc) return rc;
  }
  const size_t cl = D >> vd.nblocks;
  const float* a_out = ld.f32(P + "model." + std::to_string(2 + vd.nblocks) + ".alpha", cl);
  const uint16_t* last_w = ld.bf(P + "model." + std::to_string(3 + vd.nblocks) + ".weight", cl * 7);
  const float* last_b = ld.f32(P + "model." + std::to_string(3 + vd.nblocks) + ".bias", 1);
  if (ld.rc) return ld.rc;
  return vx_vae_load_out(v, a_out, last_w, last_b);
}

int vx_voxcpm2_load_weights(vx_voxcpm2* m, const vx_weights* w) {
  if (!m || !w) return VX_ERR_ARG;
  vx_lm *base, *res, *enc;
  vx_dit* dit;
  int dm[6];
  voxcpm2_parts(m, &base, &res, &enc, &dit, dm);
  const size_t H = dm[0], He = dm[1], Hd = dm[2], D = dm[3], Lq = dm[5];
  int rc = load_lm(base, w, "base_lm.", false, nullptr);
  if (!rc) rc = load_lm(res, w, "residual_lm.", false, nullptr);
  if (!rc) rc = load_lm(enc, w, "feat_encoder.encoder.", false, nullptr);
  if (!rc) rc = vx_dit_load_weights(dit, w, "feat_decoder.estimator.");
  if (rc) return rc;
  Loader ld{w, lm_ctx(base)};
  vx_voxcpm2_weights vw = {};
  vw.special_token = ld.f32("feat_encoder.special_token", He);
  vw.enc_in_w = ld.bf("feat_encoder.in_proj.weight", He * D);
  vw.enc_in_b = ld.f32("feat_encoder.in_proj.bias", He);
  vw.enc_to_lm_w = ld.bf("enc_to_lm_proj.weight", H * He);
  vw.enc_to_lm_b = ld.f32("enc_to_lm_proj.bias", H);
  vw.lm_to_dit_w = ld.bf("lm_to_dit_proj.weight", Hd * H);
  vw.lm_to_dit_b = ld.f32("lm_to_dit_proj.bias", Hd);
  vw.res_to_dit_w = ld.bf("res_to_dit_proj.weight", Hd * H);
  vw.res_to_dit_b = ld.f32("res_to_dit_proj.bias", Hd);
  vw.fusion_w = ld.bf("fusion_concat_proj.weight", 2 * H * H);
  vw.fusion_b = ld.f32("fusion_concat_proj.bias", H);
  vw.stop_proj_w = ld.bf("stop_proj.weight", H * H);
  vw.stop_proj_b = ld.f32("stop_proj.bias", H);
  vw.stop_head_w = ld.bf("stop_head.weight", 2 * H);
  vw.fsq_in_w = ld.bf("fsq_layer.in_proj.weight", Lq * H);
  vw.fsq_in_b = ld.f32("fsq_layer.in_proj.bias", Lq);
  vw.fsq_out_w = ld.bf("fsq_layer.out_proj.weight", H * Lq);
  vw.fsq_out_b = ld.f32("fsq_layer.out_proj.bias", H);
  if (ld.rc) return ld.rc;
  return vx_voxcpm2_load(m, &vw);
}

}  // extern "C"
