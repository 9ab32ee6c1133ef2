/*
 * gguf.cpp — GGUF reader (see gguf.h) and synthetic LLaMA GGUF writer.
 */
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <thread>

#include "ulb_common.h"

namespace ulbe {

enum { GV_U8, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STR, GV_ARR, GV_U64, GV_I64, GV_F64 };

size_t gguf_type_nbytes(int type, uint64_t n) {
  /* (units of n, bytes per unit); 0 for an unsupported type, a partial block or a size that
     does not fit 64 bits */
  uint64_t unit = 0, per = 0;
  switch (type) {
    case 0: unit = 1; per = 4; break;      /* F32  */
    case 1: unit = 1; per = 2; break;      /* F16  */
    case 2: unit = 32; per = 18; break;    /* Q4_0 */
    case 12: unit = 256; per = 144; break; /* Q4_K */
    case 8: unit = 32; per = 34; break;    /* Q8_0 */
    case 14: unit = 256; per = 210; break; /* Q6_K */
    default: return 0;
  }
  if (n % unit) return 0;
  uint64_t bytes = 0;
  if (__builtin_mul_overflow(n / unit, per, &bytes)) return 0;
  return (size_t)bytes;
}

namespace {
struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool bad = false;
  uint64_t u(int n) {
    if (bad || p + n > end) { bad = true; return 0; }
    uint64_t v = 0;
    memcpy(&v, p, n);
    p += n;
    return v;
  }
  std::string s() {
    uint64_t len = u(8);
    if (bad || len > (uint64_t)(end - p)) { bad = true; return {}; }
    std::string r((const char*)p, (size_t)len);
    p += len;
    return r;
  }
};
int gv_size(int t) {
  switch (t) {
    case GV_U8: case GV_I8: case GV_BOOL: return 1;
    case GV_U16: case GV_I16: return 2;
    case GV_U32: case GV_I32: case GV_F32: return 4;
    case GV_U64: case GV_I64: case GV_F64: return 8;
  }
  return -1;
}
double scalar(Reader& r, int t) {
  uint64_t raw = r.u(gv_size(t));
  switch (t) {
    case GV_I8: return (double)(int8_t)raw;
    case GV_I16: return (double)(int16_t)raw;
    case GV_I32: return (double)(int32_t)raw;
    case GV_I64: return (double)(int64_t)raw;
    case GV_F32: { float f; uint32_t v = (uint32_t)raw; memcpy(&f, &v, 4); return f; }
    case GV_F64: { double f; memcpy(&f, &raw, 8); return f; }
    default: return (double)raw;
  }
}
}  // namespace

GGUFFile::~GGUFFile() {
  if (map_) munmap(map_, map_len_);
}

bool GGUFFile::open(const std::string& path, std::string* err) {
  auto fail = [&](const std::string& m) {
    if (err) *err = path + ": " + m;
    return false;
  };
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return fail("cannot open");
  struct stat st;
  if (fstat(fd, &st) != 0) { ::close(fd); return fail("cannot stat"); }
  map_len_ = (size_t)st.st_size;
  file_bytes = map_len_;
  if (map_len_ < 24) { ::close(fd); return fail("too short for a GGUF header"); }
  map_ = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) { map_ = nullptr; return fail("mmap failed"); }
  Reader r{(const uint8_t*)map_, (const uint8_t*)map_ + map_len_};
  if (memcmp(r.p, "GGUF", 4) != 0) return fail("bad magic");
  r.p += 4;
  version = (uint32_t)r.u(4);
  if (version < 2 || version > 3) return fail("unsupported GGUF version " + std::to_string(version));
  const uint64_t n_t = r.u(8), n_kv = r.u(8);
  if (n_t > 1000000 || n_kv > 1000000) return fail("implausible tensor / kv counts");
  for (uint64_t i = 0; i < n_kv && !r.bad; ++i) {
    std::string key = r.s();
    int t = (int)r.u(4);
    if (t == GV_STR) { str_[key] = r.s(); continue; }
    if (t == GV_ARR) {
      int et = (int)r.u(4);
      uint64_t cnt = r.u(8);
      if (cnt > (uint64_t)(r.end - r.p)) return fail("truncated array " + key);
      if (et == GV_STR) {
        std::vector<std::string>& v = strarr_[key];
        v.reserve(cnt);
        for (uint64_t j = 0; j < cnt && !r.bad; ++j) v.push_back(r.s());
      } else if (gv_size(et) > 0) {
        std::vector<double>& v = numarr_[key];
        v.reserve(cnt);
        for (uint64_t j = 0; j < cnt && !r.bad; ++j) v.push_back(scalar(r, et));
      } else {
        return fail("unsupported nested array in " + key);
      }
      continue;
    }
    if (gv_size(t) < 0) return fail("unknown metadata value type " + std::to_string(t));
    num_[key] = scalar(r, t);
  }
  if (r.bad) return fail("truncated metadata");
  alignment = (uint64_t)num("general.alignment", 32);
  if (alignment == 0 || (alignment & (alignment - 1))) alignment = 32;
  tensors.resize(n_t);
  for (uint64_t i = 0; i < n_t; ++i) {
    GGUFTensor& t = tensors[i];
    t.name = r.s();
    t.n_dims = (int)r.u(4);
    if (r.bad || t.n_dims < 1 || t.n_dims > 4) return fail("bad tensor info");
    uint64_t n = 1;
    bool wrap = false;
    for (int j = 0; j < t.n_dims; ++j) {
      t.ne[j] = r.u(8);
      wrap |= __builtin_mul_overflow(n, t.ne[j], &n);
    }
    if (wrap) return fail("tensor " + t.name + ": element count overflows 64 bits");
    t.type = (int)r.u(4);
    t.offset = r.u(8);
    t.nbytes = gguf_type_nbytes(t.type, n);
    if (!t.nbytes && n)
      return fail("tensor " + t.name + ": unsupported type " + std::to_string(t.type) +
                  " (or a size that is not whole blocks / overflows)");
  }
  if (r.bad) return fail("truncated tensor infos");
  const size_t hdr = (size_t)(r.p - (const uint8_t*)map_);
  const size_t data = (hdr + alignment - 1) / alignment * alignment;
  for (GGUFTensor& t : tensors) {
    /* three separate comparisons: no sum of file-supplied values can wrap around */
    if (data > map_len_ || t.offset > map_len_ - data || t.nbytes > map_len_ - data - t.offset)
      return fail("tensor " + t.name + " extends past the end of the file");
    t.data = (const uint8_t*)map_ + data + t.offset;
  }
  return true;
}

const GGUFTensor* GGUFFile::find(const std::string& name) const {
  for (const GGUFTensor& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

double GGUFFile::num(const std::string& key, double dflt) const {
  auto it = num_.find(key);
  return it == num_.end() ? dflt : it->second;
}

std::string GGUFFile::str(const std::string& key, const std::string& dflt) const {
  auto it = str_.find(key);
  return it == str_.end() ? dflt : it->second;
}

const std::vector<std::string>* GGUFFile::str_array(const std::string& key) const {
  auto it = strarr_.find(key);
  return it == strarr_.end() ? nullptr : &it->second;
}

const std::vector<double>* GGUFFile::num_array(const std::string& key) const {
  auto it = numarr_.find(key);
  return it == numarr_.end() ? nullptr : &it->second;
}

/* ------------------------------------------------------------------ quantisers */

/* GGUF reference Q4_0 quantiser: d = (value of max |x|) / -8, q = min(15, trunc(x/d + 8.5)) */
void quantize_q4_0(const float* x, uint64_t n, uint8_t* out) {
  for (uint64_t b = 0; b < n / 32; ++b) {
    const float* v = x + b * 32;
    float amax = 0.f, mx = 0.f;
    for (int i = 0; i < 32; ++i)
      if (std::fabs(v[i]) > amax) { amax = std::fabs(v[i]); mx = v[i]; }
    const float d = mx / -8.0f;
    const float id = d != 0.f ? 1.0f / d : 0.f;
    uint8_t* blk = out + b * 18;
    const uint16_t dh = ulb_f2h(d);
    memcpy(blk, &dh, 2);
    for (int i = 0; i < 16; ++i) {
      const float a = v[i] * id;
      const float c = v[i + 16] * id;
      int qa = (int)std::trunc(a + 8.5f), qc = (int)std::trunc(c + 8.5f);
      qa = std::min(15, std::max(0, qa));
      qc = std::min(15, std::max(0, qc));
      blk[2 + i] = (uint8_t)(qa | (qc << 4));
    }
  }
}

/*
 * Q4_K quantiser (this project's own; any valid encoding decodes bit-exactly): per 32-weight
 * sub-block j, min_j = min(0, min x), scale_j = (max x - min_j) / 15; super-block
 * d = max scale / 63, dmin = max(-min) / 63 (stored fp16); 6-bit sc_j = round(scale_j / d),
 * m_j = round(-min_j / dmin); q = clamp(round((x + dmin*m_j) / (d*sc_j)), 0, 15).
 */
/* Q8_0 block (34 B): fp16 d, 32 x int8; d = amax / 127, q = round(x / d). */
void quantize_q8_0(const float* x, uint64_t n, uint8_t* out) {
  for (uint64_t b = 0; b < n / 32; ++b) {
    const float* v = x + b * 32;
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(v[i]));
    const uint16_t dh = ulb_f2h(amax / 127.f);
    const float d = ulb_h2f(dh), id = d != 0.f ? 1.f / d : 0.f;
    uint8_t* blk = out + b * 34;
    memcpy(blk, &dh, 2);
    for (int i = 0; i < 32; ++i) {
      const int q = (int)std::lrint(v[i] * id);
      blk[2 + i] = (uint8_t)(int8_t)std::min(127, std::max(-127, q));
    }
  }
}

/* Q6_K super-block (210 B): ql[128] low nibbles, qh[64] high bit pairs, int8 scales[16] (one
 * per 16 weights), fp16 d; weight i = d * scales[i / 16] * (q_i - 32).  Weight i of half
 * h = i / 128 (r = i % 128, k = r / 32, l = r % 32) keeps its low nibble in
 * ql[64h + l + 32 (k & 1)] (low nibble for k < 2, high for k >= 2) and its top two bits in
 * bits 2k, 2k + 1 of qh[32h + l].  Scales: sub-block amax / 31 over d = max / 127. */
void quantize_q6_k(const float* x, uint64_t n, uint8_t* out) {
  for (uint64_t b = 0; b < n / 256; ++b) {
    const float* v = x + b * 256;
    float sub[16], smax = 0.f;
    for (int j = 0; j < 16; ++j) {
      float amax = 0.f;
      for (int i = 0; i < 16; ++i) amax = std::max(amax, std::fabs(v[16 * j + i]));
      sub[j] = amax / 31.f;
      smax = std::max(smax, sub[j]);
    }
    uint8_t* blk = out + b * 210;
    memset(blk, 0, 210);
    const uint16_t dh = ulb_f2h(smax / 127.f);
    const float d = ulb_h2f(dh);
    memcpy(blk + 208, &dh, 2);
    for (int j = 0; j < 16; ++j) {
      const int sc = d != 0.f ? std::min(127, (int)std::lrint(sub[j] / d)) : 0;
      blk[192 + j] = (uint8_t)(int8_t)sc;
      const float step = d * (float)sc;
      for (int e = 0; e < 16; ++e) {
        const int i = 16 * j + e;
        int q = step != 0.f ? (int)std::lrint(v[i] / step) + 32 : 32;
        q = std::min(63, std::max(0, q));
        const int h = i / 128, r = i % 128, k = r / 32, l = r % 32;
        uint8_t& lo = blk[64 * h + l + 32 * (k & 1)];
        lo |= (uint8_t)((q & 15) << (k >= 2 ? 4 : 0));
        blk[128 + 32 * h + l] |= (uint8_t)((q >> 4) << (2 * k));
      }
    }
  }
}

void quantize_q4_k(const float* x, uint64_t n, uint8_t* out) {
  for (uint64_t b = 0; b < n / 256; ++b) {
    const float* v = x + b * 256;
    float scale[8], minv[8];
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; ++j) {
      float lo = 0.f, hi = -INFINITY;
      for (int i = 0; i < 32; ++i) { lo = std::min(lo, v[32 * j + i]); hi = std::max(hi, v[32 * j + i]); }
      scale[j] = (hi - lo) / 15.0f;
      minv[j] = -lo;
      max_scale = std::max(max_scale, scale[j]);
      max_min = std::max(max_min, minv[j]);
    }
    const uint16_t dh = ulb_f2h(max_scale / 63.0f), mh = ulb_f2h(max_min / 63.0f);
    const float df = ulb_h2f(dh), mf = ulb_h2f(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
      sc[j] = df > 0.f ? std::min(63, (int)std::lrint(scale[j] / df)) : 0;
      mn[j] = mf > 0.f ? std::min(63, (int)std::lrint(minv[j] / mf)) : 0;
    }
    uint8_t* blk = out + b * 144;
    memcpy(blk, &dh, 2);
    memcpy(blk + 2, &mh, 2);
    uint8_t* s12 = blk + 4;
    for (int j = 0; j < 4; ++j) {
      s12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      s12[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
      s12[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; ++j) {
      const float s = df * (float)sc[j], m = mf * (float)mn[j];
      for (int i = 0; i < 32; ++i) {
        int qi = 0;
        if (s > 0.f) qi = std::min(15, std::max(0, (int)std::lrint((v[32 * j + i] + m) / s)));
        q[32 * j + i] = (uint8_t)qi;
      }
    }
    uint8_t* qs = blk + 16;
    for (int c = 0; c < 4; ++c)
      for (int l = 0; l < 32; ++l) qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
  }
}

/* ------------------------------------------------------------------ synthetic writer */
static uint64_t fnv1a64(const std::string& s) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char ch : s) { h ^= ch; h *= 1099511628211ull; }
  return h;
}

static inline void normals4(uint64_t seed, uint64_t nh, uint64_t blk, double z[4]) {
  const ulb_u32x4 r = ulb_philox4x32_10((uint32_t)blk, (uint32_t)(blk >> 32), 0x53594E54u /* "SYNT" */, 0u,
                                        (uint32_t)(seed ^ nh), (uint32_t)((seed ^ nh) >> 32));
  const double two32 = 4294967296.0, two_pi = 6.283185307179586476925286766559;
  for (int p = 0; p < 2; ++p) {
    const double u1 = ((double)r.v[2 * p] + 1.0) / two32; /* (0, 1] */
    const double u2 = (double)r.v[2 * p + 1] / two32;
    const double rad = std::sqrt(-2.0 * std::log(u1));
    z[2 * p] = rad * std::cos(two_pi * u2);
    z[2 * p + 1] = rad * std::sin(two_pi * u2);
  }
}

double synth_normal(uint64_t seed, const std::string& name, uint64_t i) {
  double z[4];
  normals4(seed, fnv1a64(name), i / 4, z);
  return z[i % 4];
}

static void parallel_for(uint64_t n, int threads, const std::function<void(uint64_t, uint64_t)>& fn) {
  threads = std::max(1, threads);
  if (threads == 1 || n < 4096) { fn(0, n); return; }
  std::vector<std::thread> ts;
  const uint64_t chunk = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const uint64_t a = t * chunk, b = std::min(n, a + chunk);
    if (a >= b) break;
    ts.emplace_back(fn, a, b);
  }
  for (auto& th : ts) th.join();
}

namespace {
struct PlannedTensor {
  std::string name;
  int type;
  int n_dims;
  uint64_t ne[2];
  enum Fill { NORMAL, ONES } fill;
  uint64_t offset = 0;
  size_t nbytes = 0;
};

void put_str(std::vector<uint8_t>& b, const std::string& s) {
  const uint64_t n = s.size();
  b.insert(b.end(), (const uint8_t*)&n, (const uint8_t*)&n + 8);
  b.insert(b.end(), s.begin(), s.end());
}
template <typename T>
void put(std::vector<uint8_t>& b, T v) {
  b.insert(b.end(), (const uint8_t*)&v, (const uint8_t*)&v + sizeof(T));
}
void kv_u32(std::vector<uint8_t>& b, const std::string& k, uint32_t v) { put_str(b, k); put<uint32_t>(b, GV_U32); put(b, v); }
void kv_f32(std::vector<uint8_t>& b, const std::string& k, float v) { put_str(b, k); put<uint32_t>(b, GV_F32); put(b, v); }
void kv_u64(std::vector<uint8_t>& b, const std::string& k, uint64_t v) { put_str(b, k); put<uint32_t>(b, GV_U64); put(b, v); }
void kv_str(std::vector<uint8_t>& b, const std::string& k, const std::string& v) { put_str(b, k); put<uint32_t>(b, GV_STR); put_str(b, v); }
void kv_bool(std::vector<uint8_t>& b, const std::string& k, bool v) {
  put_str(b, k);
  put<uint32_t>(b, GV_BOOL);
  put<uint8_t>(b, v ? 1 : 0);
}
void kv_arr_str(std::vector<uint8_t>& b, const std::string& k, const std::vector<std::string>& v) {
  put_str(b, k);
  put<uint32_t>(b, GV_ARR);
  put<uint32_t>(b, GV_STR);
  put<uint64_t>(b, v.size());
  for (const std::string& x : v) put_str(b, x);
}
template <class T>
void kv_arr_num(std::vector<uint8_t>& b, const std::string& k, uint32_t gv, const std::vector<T>& v) {
  put_str(b, k);
  put<uint32_t>(b, GV_ARR);
  put<uint32_t>(b, gv);
  put<uint64_t>(b, v.size());
  for (const T& x : v) put(b, x);
}
}  // namespace

bool write_synthetic_gguf(const std::string& path, const SynthSpec& sp, int threads, std::string* err) {
  auto fail = [&](const std::string& m) {
    if (err) *err = m;
    return false;
  };
  if (sp.n_layer <= 0 || sp.d_model <= 0 || sp.n_head <= 0 || sp.n_head_kv <= 0 || sp.d_ff <= 0 || sp.n_vocab <= 0)
    return fail("synthetic spec: non-positive dimension");
  if (sp.d_model % sp.n_head || sp.n_head % sp.n_head_kv) return fail("synthetic spec: head split");
  if (sp.wtype != 2 && sp.wtype != 12) return fail("synthetic spec: wtype must be 2 (Q4_0) or 12 (Q4_K)");
  if (!sp.vocab.empty() && (sp.scores.size() != sp.vocab.size() || sp.token_types.size() != sp.vocab.size()))
    return fail("synthetic spec: vocab, scores and token_types differ in length");
  const int out_type = sp.out_type >= 0 ? sp.out_type : sp.wtype;
  auto qtype_ok = [](int t) { return t == 2 || t == 8 || t == 12 || t == 14; };
  if (!qtype_ok(out_type)) return fail("synthetic spec: out_type must be Q4_0, Q8_0, Q4_K or Q6_K");
  if (sp.embd_type != 0 && sp.embd_type != 1 && !qtype_ok(sp.embd_type))
    return fail("synthetic spec: embd_type must be F32, F16, Q4_0, Q8_0, Q4_K or Q6_K");
  if (sp.d_model % 256 && (out_type == 12 || out_type == 14 || sp.embd_type == 12 || sp.embd_type == 14))
    return fail("synthetic spec: d_model must be a multiple of 256 for K-quant token_embd / output");
  const int blk = sp.wtype == 2 ? 32 : 256;
  const int hd = sp.d_model / sp.n_head;
  const uint64_t nq = (uint64_t)sp.n_head * hd, nkv = (uint64_t)sp.n_head_kv * hd;
  if (sp.d_model % blk || sp.d_ff % blk || nq % blk) return fail("synthetic spec: dims must be multiples of the block size");
  const int v_type = sp.v_type >= 0 ? sp.v_type : sp.wtype, o_type = sp.o_type >= 0 ? sp.o_type : sp.wtype,
            down_type = sp.down_type >= 0 ? sp.down_type : sp.wtype;
  auto blk_of = [](int t) { return t == 2 || t == 8 ? 32 : 256; };
  if (!qtype_ok(v_type) || !qtype_ok(o_type) || !qtype_ok(down_type))
    return fail("synthetic spec: v_type / o_type / down_type must be Q4_0, Q8_0, Q4_K or Q6_K");
  if (sp.d_model % blk_of(v_type) || nq % blk_of(o_type) || sp.d_ff % blk_of(down_type))
    return fail("synthetic spec: the inner dimension of attn_v / attn_output / ffn_down is not whole blocks");
  std::vector<PlannedTensor> plan;
  plan.push_back({"token_embd.weight", sp.embd_type, 2, {(uint64_t)sp.d_model, (uint64_t)sp.n_vocab}, PlannedTensor::NORMAL});
  for (int l = 0; l < sp.n_layer; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    const uint64_t d = sp.d_model, f = sp.d_ff;
    plan.push_back({p + "attn_norm.weight", 0, 1, {d, 1}, PlannedTensor::ONES});
    plan.push_back({p + "attn_q.weight", sp.wtype, 2, {d, nq}, PlannedTensor::NORMAL});
    plan.push_back({p + "attn_k.weight", sp.wtype, 2, {d, nkv}, PlannedTensor::NORMAL});
    plan.push_back({p + "attn_v.weight", v_type, 2, {d, nkv}, PlannedTensor::NORMAL});
    plan.push_back({p + "attn_output.weight", o_type, 2, {nq, d}, PlannedTensor::NORMAL});
    plan.push_back({p + "ffn_norm.weight", 0, 1, {d, 1}, PlannedTensor::ONES});
    plan.push_back({p + "ffn_gate.weight", sp.wtype, 2, {d, f}, PlannedTensor::NORMAL});
    plan.push_back({p + "ffn_up.weight", sp.wtype, 2, {d, f}, PlannedTensor::NORMAL});
    plan.push_back({p + "ffn_down.weight", down_type, 2, {f, d}, PlannedTensor::NORMAL});
  }
  plan.push_back({"output_norm.weight", 0, 1, {(uint64_t)sp.d_model, 1}, PlannedTensor::ONES});
  if (!sp.tied)
    plan.push_back({"output.weight", out_type, 2, {(uint64_t)sp.d_model, (uint64_t)sp.n_vocab}, PlannedTensor::NORMAL});
  const uint64_t align = 32;
  uint64_t off = 0;
  for (PlannedTensor& t : plan) {
    t.nbytes = gguf_type_nbytes(t.type, t.ne[0] * t.ne[1]);
    t.offset = off;
    off = (off + t.nbytes + align - 1) / align * align;
  }
  std::vector<uint8_t> h;
  h.insert(h.end(), {'G', 'G', 'U', 'F'});
  put<uint32_t>(h, 3);
  put<uint64_t>(h, plan.size());
  const bool with_vocab = !sp.vocab.empty();
  const int n_flags = with_vocab ? (sp.add_bos >= 0) + (sp.add_space_prefix >= 0) : 0;
  const int n_merges = with_vocab && !sp.merges.empty() ? 1 : 0;
  const int n_pre = with_vocab && !sp.tok_pre.empty() ? 1 : 0;
  put<uint64_t>(h, 14 + (with_vocab ? 7 : 0) + n_flags + n_merges + n_pre);
  kv_str(h, "general.architecture", "llama");
  kv_str(h, "general.name", sp.name);
  kv_u32(h, "general.alignment", (uint32_t)align);
  kv_u32(h, "llama.block_count", sp.n_layer);
  kv_u32(h, "llama.embedding_length", sp.d_model);
  kv_u32(h, "llama.feed_forward_length", sp.d_ff);
  kv_u32(h, "llama.attention.head_count", sp.n_head);
  kv_u32(h, "llama.attention.head_count_kv", sp.n_head_kv);
  kv_f32(h, "llama.attention.layer_norm_rms_epsilon", sp.rms_eps);
  kv_f32(h, "llama.rope.freq_base", sp.rope_base);
  kv_u32(h, "llama.rope.dimension_count", hd);
  kv_u32(h, "llama.context_length", sp.ctx_len);
  kv_u32(h, "llama.vocab_size", sp.n_vocab);
  kv_u64(h, "ulb.synthetic.seed", sp.seed);
  if (with_vocab) {
    kv_str(h, "tokenizer.ggml.model", n_merges ? "gpt2" : "llama");
    if (n_merges) kv_arr_str(h, "tokenizer.ggml.merges", sp.merges);
    if (n_pre) kv_str(h, "tokenizer.ggml.pre", sp.tok_pre);
    kv_arr_str(h, "tokenizer.ggml.tokens", sp.vocab);
    kv_arr_num<float>(h, "tokenizer.ggml.scores", GV_F32, sp.scores);
    kv_arr_num<int32_t>(h, "tokenizer.ggml.token_type", GV_I32, sp.token_types);
    kv_u32(h, "tokenizer.ggml.bos_token_id", 1);
    kv_u32(h, "tokenizer.ggml.eos_token_id", 2);
    kv_u32(h, "tokenizer.ggml.unknown_token_id", 0);
    if (sp.add_bos >= 0) kv_bool(h, "tokenizer.ggml.add_bos_token", sp.add_bos != 0);
    if (sp.add_space_prefix >= 0) kv_bool(h, "tokenizer.ggml.add_space_prefix", sp.add_space_prefix != 0);
  }
  for (const PlannedTensor& t : plan) {
    put_str(h, t.name);
    put<uint32_t>(h, t.n_dims);
    for (int j = 0; j < t.n_dims; ++j) put<uint64_t>(h, t.ne[j]);
    put<uint32_t>(h, t.type);
    put<uint64_t>(h, t.offset);
  }
  while (h.size() % align) h.push_back(0);
  FILE* f = fopen((path + ".tmp").c_str(), "wb");
  if (!f) return fail("cannot create " + path);
  bool ok = fwrite(h.data(), 1, h.size(), f) == h.size();
  uint64_t written = 0;
  std::vector<uint8_t> buf;
  std::vector<float> vals;
  for (const PlannedTensor& t : plan) {
    if (!ok) break;
    const uint64_t n = t.ne[0] * t.ne[1];
    buf.assign(t.nbytes, 0);
    const uint64_t nh = fnv1a64(t.name);
    if (t.fill == PlannedTensor::ONES) {
      for (uint64_t i = 0; i < n; ++i) reinterpret_cast<float*>(buf.data())[i] = 1.0f;
    } else if (t.type == 1) {
      uint16_t* o = reinterpret_cast<uint16_t*>(buf.data());
      parallel_for((n + 3) / 4, threads, [&](uint64_t a, uint64_t b) {
        for (uint64_t q = a; q < b; ++q) {
          double z[4];
          normals4(sp.seed, nh, q, z);
          for (int e = 0; e < 4 && q * 4 + e < n; ++e) o[q * 4 + e] = ulb_f2h((float)(sp.stddev * z[e]));
        }
      });
    } else if (t.type == 0) {
      float* o = reinterpret_cast<float*>(buf.data());
      parallel_for((n + 3) / 4, threads, [&](uint64_t a, uint64_t b) {
        for (uint64_t q = a; q < b; ++q) {
          double z[4];
          normals4(sp.seed, nh, q, z);
          for (int e = 0; e < 4 && q * 4 + e < n; ++e) o[q * 4 + e] = (float)(sp.stddev * z[e]);
        }
      });
    } else {
      /* quantised: block by block, the same N(0, stddev) values whatever the type */
      const int tb = t.type == 2 || t.type == 8 ? 32 : 256;
      const size_t bb = gguf_type_nbytes(t.type, (uint64_t)tb);
      const uint64_t nblk = n / tb;
      parallel_for(nblk, threads, [&](uint64_t a, uint64_t b) {
        std::vector<float> v(tb);
        for (uint64_t q = a; q < b; ++q) {
          for (int e = 0; e < tb; e += 4) {
            double z[4];
            normals4(sp.seed, nh, (q * tb + e) / 4, z);
            for (int k = 0; k < 4; ++k) v[e + k] = (float)(sp.stddev * z[k]);
          }
          uint8_t* o = buf.data() + q * bb;
          if (t.type == 2) quantize_q4_0(v.data(), tb, o);
          else if (t.type == 12) quantize_q4_k(v.data(), tb, o);
          else if (t.type == 8) quantize_q8_0(v.data(), tb, o);
          else quantize_q6_k(v.data(), tb, o);
        }
      });
    }
    while (written < t.offset && ok) { ok = fputc(0, f) != EOF; ++written; }
    ok = ok && fwrite(buf.data(), 1, buf.size(), f) == buf.size();
    written += buf.size();
  }
  ok = fclose(f) == 0 && ok;
  if (!ok) return fail("write failed: " + path);
  if (rename((path + ".tmp").c_str(), path.c_str()) != 0) return fail("rename failed: " + path);
  return true;
}

}  // namespace ulbe
