// kq_pack.h -- host-side reader of a Kindi Q4 pack (a repacked GGUF directory), for
// kq_pack_read_config / kq_model_load_pack.
//
// The pack is the reference's on-disk format (scripts/kindi_q4/kindi/q4pack.py:86-180):
//   kindi_pack.json  manifest: pack_format "kindi-q4-v1", head "output.weight", hadamard_block 1,
//                    `dimensions`, and `files` {name: {size, sha256}} for every other file
//   index.json       {"tensors": {gguf name: record}}; a Q4_K/Q6_K record has rows, ne0 (columns),
//                    type 12/14, offset (a multiple of 16 KiB into weights.bin), bytes =
//                    rows * ne0/256 * block bytes, padded_bytes = bytes rounded up to 16 KiB; a
//                    float record has type 0 and f32_off (a multiple of 4 into f32.bin)
//   weights.bin      the quantised matrices, each in the 8-row interleave [R/8][C/256][8][block]
//                    (q4pack.py:151-158, q4kernels.h:8-10), zero padded to 16 KiB
//   f32.bin          the float tensors (norm weights)
// Everything is validated before any device allocation, as verify_pack does (q4pack.py:86-108):
// the manifest fields, bare file names, file sizes, SHA-256 digests (unless KINDI_Q4_VERIFY=size),
// the exact tensor set, every shape, type, offset and span.
//
// The reference's manifest profile is its hybrid GDN / attention model; this runtime runs the
// dense GQA decoder, so `dimensions` describes that: layers, width, ffn, heads, kv_heads, head_dim,
// rope_dim (= head_dim, full-width rotary), rope_base, optional norm_eps (1e-6) and
// full_attention_interval (must be 1: every layer is attention). A hybrid pack is rejected.
#pragma once
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <sys/stat.h>
#include <utility>
#include <vector>

#include "../../include/kq.h"

namespace kqpack {

// ------------------------------------------------------------------------------ JSON
struct JVal {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } k = NUL;
  bool b = false;
  double n = 0.0;
  std::string s;
  std::vector<JVal> a;
  std::vector<std::pair<std::string, JVal>> o;
  const JVal* get(const char* key) const {
    if (k != OBJ) return nullptr;
    for (const auto& kv : o)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

// A strict recursive-descent parser for the manifest and index (RFC 8259 grammar; \u escapes
// outside ASCII are kept as UTF-8). Depth is bounded.
class JParser {
 public:
  JParser(const char* p, size_t n) : p_(p), e_(p + n) {}
  bool parse(JVal& v, std::string& err) {
    ws();
    if (!value(v, 0)) { err = "malformed JSON (" + err_ + ")"; return false; }
    ws();
    if (p_ != e_) { err = "malformed JSON (trailing data)"; return false; }
    return true;
  }

 private:
  const char *p_, *e_;
  std::string err_;
  void ws() { while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_; }
  bool fail(const char* m) { err_ = m; return false; }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if ((size_t)(e_ - p_) < n || std::memcmp(p_, w, n)) return false;
    p_ += n;
    return true;
  }
  static void utf8(std::string& out, unsigned cp) {
    if (cp < 0x80) out += (char)cp;
    else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 63)); }
    else if (cp < 0x10000) { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63)); }
    else { out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 63)); out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63)); }
  }
  bool hex4(unsigned& v) {
    if (e_ - p_ < 4) return false;
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  bool str(std::string& out) {
    if (p_ >= e_ || *p_ != '"') return fail("expected a string");
    ++p_;
    while (p_ < e_ && *p_ != '"') {
      const unsigned char c = (unsigned char)*p_++;
      if (c < 0x20) return fail("control character in a string");
      if (c != '\\') { out += (char)c; continue; }
      if (p_ >= e_) return fail("unterminated escape");
      const char x = *p_++;
      switch (x) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          unsigned cp;
          if (!hex4(cp)) return fail("bad \\u escape");
          if (cp >= 0xD800 && cp < 0xDC00) {   // surrogate pair
            unsigned lo;
            if (e_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') return fail("unpaired surrogate");
            p_ += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail("unpaired surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(out, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p_ >= e_) return fail("unterminated string");
    ++p_;
    return true;
  }
  bool num(double& v) {
    const char* s = p_;
    if (p_ < e_ && *p_ == '-') ++p_;
    if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return fail("bad number");
    if (*p_ == '0') ++p_;
    else while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    if (p_ < e_ && *p_ == '.') {
      ++p_;
      if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return fail("bad number");
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
      ++p_;
      if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) return fail("bad number");
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    v = std::strtod(std::string(s, p_).c_str(), nullptr);
    return true;
  }
  bool value(JVal& v, int depth) {
    if (depth > 64) return fail("nesting too deep");
    if (p_ >= e_) return fail("unexpected end");
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v.k = JVal::OBJ;
      ws();
      if (p_ < e_ && *p_ == '}') { ++p_; return true; }
      for (;;) {
        ws();
        std::string key;
        if (!str(key)) return false;
        ws();
        if (p_ >= e_ || *p_ != ':') return fail("expected ':'");
        ++p_;
        ws();
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.o.emplace_back(std::move(key), std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') { ++p_; continue; }
        if (p_ < e_ && *p_ == '}') { ++p_; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p_;
      v.k = JVal::ARR;
      ws();
      if (p_ < e_ && *p_ == ']') { ++p_; return true; }
      for (;;) {
        ws();
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.a.push_back(std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') { ++p_; continue; }
        if (p_ < e_ && *p_ == ']') { ++p_; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') { v.k = JVal::STR; return str(v.s); }
    if (lit("true")) { v.k = JVal::BOOL; v.b = true; return true; }
    if (lit("false")) { v.k = JVal::BOOL; v.b = false; return true; }
    if (lit("null")) { v.k = JVal::NUL; return true; }
    v.k = JVal::NUM;
    return num(v.n);
  }
};

// ------------------------------------------------------------------------------ SHA-256
// FIPS 180-4 SHA-256 over a file, streamed in 4 MiB reads (the manifest's digests).
class Sha256 {
 public:
  Sha256() { reset(); }
  void reset() {
    static const uint32_t H0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    std::memcpy(h_, H0, sizeof h_);
    len_ = 0;
    nbuf_ = 0;
  }
  void update(const uint8_t* d, size_t n) {
    len_ += n;
    if (nbuf_) {
      const size_t t = std::min(n, (size_t)64 - nbuf_);
      std::memcpy(buf_ + nbuf_, d, t);
      nbuf_ += t; d += t; n -= t;
      if (nbuf_ == 64) { block(buf_); nbuf_ = 0; }
    }
    while (n >= 64) { block(d); d += 64; n -= 64; }
    if (n) { std::memcpy(buf_, d, n); nbuf_ = n; }
  }
  std::string hex() {
    const uint64_t bits = len_ * 8;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (nbuf_ != 56) update(&zero, 1);
    uint8_t lb[8];
    for (int i = 0; i < 8; ++i) lb[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(lb, 8);
    static const char* hx = "0123456789abcdef";
    std::string out;
    for (int i = 0; i < 8; ++i)
      for (int j = 3; j >= 0; --j) {
        const uint8_t b = (uint8_t)(h_[i] >> (8 * j));
        out += hx[b >> 4];
        out += hx[b & 15];
      }
    return out;
  }

 private:
  uint32_t h_[8];
  uint64_t len_;
  uint8_t buf_[64];
  size_t nbuf_;
  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const uint8_t* p) {
    static const uint32_t K[64] = {
        0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
        0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
        0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
        0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
        0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
        0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
        0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
        0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25), ch = (e & f) ^ (~e & g);
      const uint32_t t1 = h + S1 + ch + K[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22), mj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + mj;
      h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d; h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
  }
};

inline bool file_sha256(const std::string& path, std::string& out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  std::vector<uint8_t> buf((size_t)4 << 20);
  Sha256 h;
  size_t n;
  while ((n = std::fread(buf.data(), 1, buf.size(), f)) > 0) h.update(buf.data(), n);
  const bool ok = !std::ferror(f);
  std::fclose(f);
  if (ok) out = h.hex();
  return ok;
}

// ------------------------------------------------------------------------------ the pack
constexpr uint64_t PAGE = 16384;   // tensor alignment in weights.bin (q4pack.py PAGE)

struct Tensor {
  int type = 0;                    // 0 float, 12 Q4_K, 14 Q6_K
  long long rows = 0, cols = 0;
  uint64_t offset = 0, bytes = 0, padded = 0;   // quantised
  uint64_t f32_off = 0;                         // float
};

struct Pack {
  std::string dir;
  kq_config cfg{};
  std::map<std::string, Tensor> t;
  std::string ffn_norm_name;       // "ffn_norm.weight" or "post_attention_norm.weight"
  uint64_t weights_size = 0, f32_size = 0;
};

inline bool read_small(const std::string& path, std::string& out, size_t cap) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  out.clear();
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) {
    out.append(buf, n);
    if (out.size() > cap) { std::fclose(f); return false; }
  }
  std::fclose(f);
  return true;
}

inline bool as_int(const JVal* v, long long& out) {
  if (!v || v->k != JVal::NUM || !(std::fabs(v->n) < 9.007199254740992e15) || v->n != std::floor(v->n)) return false;
  out = (long long)v->n;
  return true;
}

inline int block_bytes_of(int type) { return type == KQ_Q4_K ? 144 : 210; }

// Reads and validates the pack in `dir` (no device work). Returns 0, or -1 with `err` set.
inline int read_pack(const char* dir, int ctx, Pack& P, std::string& err) {
  if (!dir || !*dir) { err = "null pack directory"; return -1; }
  P = Pack();
  P.dir = dir;
  const std::string base = P.dir + "/";
  std::string text;
  if (!read_small(base + "kindi_pack.json", text, (size_t)1 << 22)) { err = "cannot read kindi_pack.json in " + P.dir; return -1; }
  JVal man;
  if (!JParser(text.data(), text.size()).parse(man, err)) { err = "kindi_pack.json: " + err; return -1; }
  const JVal* fmt = man.get("pack_format");
  if (!fmt || fmt->k != JVal::STR || fmt->s != "kindi-q4-v1") { err = "Unsupported pack"; return -1; }
  const JVal* head = man.get("head");
  long long hb = 0;
  if (!head || head->k != JVal::STR || head->s != "output.weight" || !as_int(man.get("hadamard_block"), hb) || hb != 1) {
    err = "Unsupported Q4 profile (head must be output.weight, hadamard_block 1)";
    return -1;
  }
  // ---- dimensions: the dense GQA profile
  const JVal* dims = man.get("dimensions");
  if (!dims || dims->k != JVal::OBJ) { err = "Unsupported Q4 profile (no dimensions)"; return -1; }
  long long fai = 1;
  if (dims->get("full_attention_interval") && !as_int(dims->get("full_attention_interval"), fai)) fai = -1;
  if (fai != 1 || dims->get("state_size") || dims->get("gdn_inner")) {
    err = "Unsupported Q4 profile: hybrid GDN / attention packs are not supported (full_attention_interval must be 1)";
    return -1;
  }
  long long layers, width, ffn, heads, kvh, hd, rdim;
  if (!as_int(dims->get("layers"), layers) || !as_int(dims->get("width"), width) || !as_int(dims->get("ffn"), ffn) ||
      !as_int(dims->get("heads"), heads) || !as_int(dims->get("kv_heads"), kvh) || !as_int(dims->get("head_dim"), hd) ||
      !as_int(dims->get("rope_dim"), rdim)) {
    err = "Unsupported Q4 profile (dimensions need integer layers, width, ffn, heads, kv_heads, head_dim, rope_dim)";
    return -1;
  }
  const JVal* rb = dims->get("rope_base");
  if (!rb || rb->k != JVal::NUM || !(rb->n > 0)) { err = "Unsupported Q4 profile (rope_base)"; return -1; }
  double eps = 1e-6;
  if (const JVal* ev = dims->get("norm_eps")) {
    if (ev->k != JVal::NUM || !(ev->n > 0)) { err = "Unsupported Q4 profile (norm_eps)"; return -1; }
    eps = ev->n;
  }
  if (rdim != hd) { err = "Unsupported Q4 profile: partial rotary (rope_dim != head_dim)"; return -1; }
  const long long lim = 1 << 20;
  if (layers < 1 || layers > 4096 || width < 1 || width > lim || ffn < 1 || ffn > lim || heads < 1 || heads > 4096 ||
      kvh < 1 || kvh > heads || hd < 1 || hd > 4096) {
    err = "Unsupported Q4 profile (dimensions out of range)";
    return -1;
  }
  // ---- files: bare names, sizes, digests
  const JVal* files = man.get("files");
  if (!files || files->k != JVal::OBJ) { err = "Invalid manifest (no files)"; return -1; }
  const char* mode = std::getenv("KINDI_Q4_VERIFY");
  const std::string vm = mode ? mode : "full";
  if (vm != "full" && vm != "size") { err = "KINDI_Q4_VERIFY must be full or size"; return -1; }
  std::set<std::string> listed;
  for (const auto& kv : files->o) {
    const std::string& name = kv.first;
    if (name.empty() || name == "." || name == ".." || name.find('/') != std::string::npos || name.find('\\') != std::string::npos) {
      err = "Invalid manifest path";
      return -1;
    }
    long long size;
    if (!as_int(kv.second.get("size"), size) || size < 0) { err = "Invalid manifest record: " + name; return -1; }
    struct stat st;
    if (::stat((base + name).c_str(), &st) != 0 || (long long)st.st_size != size) { err = "Pack size mismatch: " + name; return -1; }
    if (vm == "full") {
      const JVal* sha = kv.second.get("sha256");
      std::string got;
      if (!sha || sha->k != JVal::STR) { err = "Invalid manifest record (sha256): " + name; return -1; }
      if (!file_sha256(base + name, got)) { err = "cannot read " + name; return -1; }
      if (got != sha->s) { err = "Pack checksum mismatch: " + name; return -1; }
    }
    if (name == "weights.bin") P.weights_size = (uint64_t)size;
    if (name == "f32.bin") P.f32_size = (uint64_t)size;
    listed.insert(name);
  }
  for (const char* must : {"weights.bin", "f32.bin", "index.json"})
    if (!listed.count(must)) { err = std::string("Invalid manifest: ") + must + " is not listed"; return -1; }
  // ---- index
  if (!read_small(base + "index.json", text, (size_t)1 << 26)) { err = "cannot read index.json"; return -1; }
  JVal idx;
  if (!JParser(text.data(), text.size()).parse(idx, err)) { err = "index.json: " + err; return -1; }
  const JVal* tens = idx.get("tensors");
  if (!tens || tens->k != JVal::OBJ) { err = "index.json has no tensors"; return -1; }
  for (const auto& kv : tens->o) {
    Tensor T;
    long long ty, rows, cols;
    if (!as_int(kv.second.get("type"), ty) || !as_int(kv.second.get("rows"), rows) || !as_int(kv.second.get("ne0"), cols) ||
        rows < 1 || cols < 1) {
      err = "Invalid tensor record: " + kv.first;
      return -1;
    }
    T.type = (int)ty; T.rows = rows; T.cols = cols;
    if (ty == KQ_Q4_K || ty == KQ_Q6_K) {
      long long off, bytes, padded;
      if (!as_int(kv.second.get("offset"), off) || !as_int(kv.second.get("bytes"), bytes) ||
          !as_int(kv.second.get("padded_bytes"), padded)) {
        err = "Invalid tensor record: " + kv.first;
        return -1;
      }
      const long long expected = rows * (cols / 256) * block_bytes_of((int)ty);
      if (rows % 8 || cols % 256 || expected != bytes) { err = "Invalid packed tensor dimensions: " + kv.first; return -1; }
      if (off < 0 || (uint64_t)off % PAGE || (uint64_t)padded != ((uint64_t)bytes + PAGE - 1) / PAGE * PAGE ||
          (uint64_t)off + (uint64_t)padded > P.weights_size) {
        err = "Invalid packed tensor span: " + kv.first;
        return -1;
      }
      T.offset = (uint64_t)off; T.bytes = (uint64_t)bytes; T.padded = (uint64_t)padded;
    } else if (ty == 0) {
      long long off;
      if (!as_int(kv.second.get("f32_off"), off) || off < 0 || off % 4 ||
          (uint64_t)off + (uint64_t)rows * (uint64_t)cols * 4 > P.f32_size) {
        err = "Invalid float tensor span: " + kv.first;
        return -1;
      }
      T.f32_off = (uint64_t)off;
    } else {
      err = "Invalid tensor type: " + kv.first;
      return -1;
    }
    if (P.t.count(kv.first)) { err = "Duplicate tensor: " + kv.first; return -1; }
    P.t[kv.first] = T;
  }
  // ---- the exact tensor set of the dense decoder, with shapes and storage
  const bool post = P.t.count("blk.0.post_attention_norm.weight") > 0;
  P.ffn_norm_name = post ? "post_attention_norm.weight" : "ffn_norm.weight";
  const auto out_it = P.t.find("output.weight");
  if (out_it == P.t.end()) { err = "Missing/extra tensors for the dense decoder (output.weight)"; return -1; }
  const long long vocab = out_it->second.rows;
  std::map<std::string, std::pair<long long, long long>> want = {
      {"token_embd.weight", {vocab, width}}, {"output.weight", {vocab, width}}, {"output_norm.weight", {1, width}}};
  for (long long l = 0; l < layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    want[p + "attn_norm.weight"] = {1, width};
    want[p + P.ffn_norm_name] = {1, width};
    want[p + "attn_q.weight"] = {heads * hd, width};
    want[p + "attn_k.weight"] = {kvh * hd, width};
    want[p + "attn_v.weight"] = {kvh * hd, width};
    want[p + "attn_output.weight"] = {width, heads * hd};
    want[p + "ffn_gate.weight"] = {ffn, width};
    want[p + "ffn_up.weight"] = {ffn, width};
    want[p + "ffn_down.weight"] = {width, ffn};
  }
  if (want.size() != P.t.size()) { err = "Missing/extra tensors for the dense decoder"; return -1; }
  for (const auto& w : want) {
    const auto it = P.t.find(w.first);
    if (it == P.t.end()) { err = "Missing/extra tensors for the dense decoder: " + w.first; return -1; }
    if (it->second.rows != w.second.first || it->second.cols != w.second.second) { err = "Unexpected shape: " + w.first; return -1; }
    const bool is_float = w.second.first == 1;
    if ((it->second.type == 0) != is_float) { err = "Unexpected tensor storage: " + w.first; return -1; }
  }
  // ---- the configuration; one quantisation type per tensor kind across the layers
  kq_config& c = P.cfg;
  kq_config_default(&c);
  c.dim = (int)width; c.n_layers = (int)layers; c.n_heads = (int)heads; c.n_kv_heads = (int)kvh; c.head_dim = (int)hd;
  c.ffn = (int)ffn; c.vocab = (int)vocab; c.ctx = ctx; c.rope_theta = (float)rb->n; c.eps = (float)eps;
  c.t_emb = P.t["token_embd.weight"].type;
  c.t_out = P.t["output.weight"].type;
  struct KindType { const char* name; int* field; };
  const KindType kinds[] = {{"attn_q.weight", &c.t_q}, {"attn_k.weight", &c.t_k}, {"attn_v.weight", &c.t_v},
                            {"attn_output.weight", &c.t_o}, {"ffn_gate.weight", &c.t_gate}, {"ffn_up.weight", &c.t_up},
                            {"ffn_down.weight", &c.t_down}};
  for (const KindType& k : kinds) {
    *k.field = P.t[std::string("blk.0.") + k.name].type;
    for (long long l = 1; l < layers; ++l)
      if (P.t["blk." + std::to_string(l) + "." + k.name].type != *k.field) {
        err = std::string("mixed quantisation types across layers are not supported: ") + k.name;
        return -1;
      }
  }
  return 0;
}

}  // namespace kqpack
