// format.cpp -- .qora-tts reader and seeded synthetic writer (host only).
//
// Reader: the talker and predictor sections of save.rs:262-409 (load_model /
// load_talker / load_predictor), reading only headers and lengths and seeking
// over payloads so the upload can stream them straight to the device.
// Writer: the save.rs:23-137 byte layout filled with seeded synthetic values
// (the decoder section is written empty so that the file stays loadable by
// save::load_model).
#include "format.h"

#include <math.h>
#include <stdio.h>
#include <string.h>

#include <memory>

namespace qtts {

namespace {

struct File {
  FILE* f = nullptr;
  ~File() {
    if (f) fclose(f);
  }
};

struct Reader {
  FILE* f;
  uint64_t size;
  bool bad = false;
  std::string msg;
  void fail(const std::string& m) {
    if (!bad) msg = m;
    bad = true;
  }
  uint64_t tell() { return (uint64_t)ftello(f); }
  void bytes(void* p, size_t n) {
    if (bad) {
      memset(p, 0, n);
      return;
    }
    if (fread(p, 1, n, f) != n) {
      fail("unexpected end of file");
      memset(p, 0, n);
    }
  }
  uint32_t u32() { uint32_t v; bytes(&v, 4); return v; }
  uint64_t u64() { uint64_t v; bytes(&v, 8); return v; }
  uint8_t u8() { uint8_t v; bytes(&v, 1); return v; }
  void skip(uint64_t n) {
    if (bad) return;
    const uint64_t at = tell();
    if (n > size || at + n > size) {
      fail("payload runs past the end of the file");
      return;
    }
    if (fseeko(f, (off_t)n, SEEK_CUR) != 0) fail("seek failed");
  }
  HVec vec(uint64_t elem) {  // u64 len + payload (gemv.rs:575-594)
    HVec v;
    v.len = u64();
    if (bad) return v;
    if (v.len > (1ull << 40) / elem) {
      fail("vector length out of range");
      return v;
    }
    v.bytes = v.len * elem;
    v.off = tell();
    skip(v.bytes);
    return v;
  }
  HWeight weight(int fmt) {  // read_weight_io gemv.rs:635-650
    HWeight w;
    w.fmt = fmt;
    w.k = u64();
    w.n = u64();
    if (bad) return w;
    if (w.k == 0 || w.n == 0 || w.k > (1u << 24) || w.n > (1u << 24)) {
      fail("weight dimensions out of range");
      return w;
    }
    if (fmt == 1) {
      HVec a = vec(1), b = vec(2);
      w.off_a = a.off; w.bytes_a = a.bytes;
      w.off_b = b.off; w.bytes_b = b.bytes;
      if (!bad && (w.n % 32 != 0 || a.len != w.k * w.n / 2 || b.len != w.k * w.n / 32))
        fail("Q4 weight length does not match k*n");
    } else if (fmt == 0) {
      HVec a = vec(2);
      w.off_a = a.off; w.bytes_a = a.bytes;
      if (!bad && a.len != w.k * w.n) fail("F16 weight length does not match k*n");
    } else {
      fail("Unknown format");
    }
    return w;
  }
};

bool check_w(Reader& r, const HWeight& w, uint64_t k, uint64_t n, const char* what) {
  if (r.bad) return false;
  if (w.k != k || w.n != n) {
    char b[160];
    snprintf(b, sizeof b, "%s is [%llu,%llu], expected [%llu,%llu]", what, (unsigned long long)w.k,
             (unsigned long long)w.n, (unsigned long long)k, (unsigned long long)n);
    r.fail(b);
    return false;
  }
  return true;
}

void read_layer(Reader& r, int fmt, HLayer& L) {
  L.q = r.weight(fmt); L.k = r.weight(fmt); L.v = r.weight(fmt); L.o = r.weight(fmt);
  L.q_norm = r.vec(2); L.k_norm = r.vec(2);
  L.gate = r.weight(fmt); L.up = r.weight(fmt); L.down = r.weight(fmt);
  L.in_norm = r.vec(2); L.post_norm = r.vec(2);
}

bool check_layer(Reader& r, const HLayer& L, int hidden, int heads, int kvh, int hd, int inter, const char* who) {
  char w[64];
  snprintf(w, sizeof w, "%s q_proj", who);
  if (!check_w(r, L.q, hidden, (uint64_t)heads * hd, w)) return false;
  snprintf(w, sizeof w, "%s k_proj", who);
  if (!check_w(r, L.k, hidden, (uint64_t)kvh * hd, w)) return false;
  snprintf(w, sizeof w, "%s v_proj", who);
  if (!check_w(r, L.v, hidden, (uint64_t)kvh * hd, w)) return false;
  snprintf(w, sizeof w, "%s o_proj", who);
  if (!check_w(r, L.o, (uint64_t)heads * hd, hidden, w)) return false;
  snprintf(w, sizeof w, "%s gate_proj", who);
  if (!check_w(r, L.gate, hidden, inter, w)) return false;
  snprintf(w, sizeof w, "%s up_proj", who);
  if (!check_w(r, L.up, hidden, inter, w)) return false;
  snprintf(w, sizeof w, "%s down_proj", who);
  if (!check_w(r, L.down, inter, hidden, w)) return false;
  if (L.q_norm.len != (uint64_t)hd || L.k_norm.len != (uint64_t)hd || L.in_norm.len != (uint64_t)hidden ||
      L.post_norm.len != (uint64_t)hidden) {
    r.fail(std::string(who) + " norm vector length mismatch");
    return false;
  }
  return true;
}

// The speech-decoder section (save.rs:446-552 load_decoder_weights).  Its
// codebook / pre-conv / transformer tensors are recorded when asked for (the
// GPU decoder stage reads them); the upsample and Vocos stages are walked
// without reading payloads, so that a file save::load_model would reject is
// rejected here too.
HConv1d conv1d(Reader& r) {  // save.rs:411-422
  HConv1d c;
  c.in = r.u32(); c.out = r.u32(); c.k = r.u32(); c.stride = r.u32(); c.pad = r.u32(); c.dil = r.u32();
  c.w = r.vec(4); c.b = r.vec(4);
  return c;
}
void skip_conv_t1d(Reader& r) {  // save.rs:424-434
  for (int i = 0; i < 5; ++i) r.u32();
  r.vec(4); r.vec(4);
}
void skip_dw_conv(Reader& r) {  // save.rs:436-444
  for (int i = 0; i < 3; ++i) r.u32();
  r.vec(4); r.vec(4);
}
void read_decoder(Reader& r, HDecoder* out) {
  HDecoder d;
  d.hidden = r.u32(); d.heads = r.u32(); d.head_dim = r.u32();
  d.inter = r.u32(); d.window = r.u32(); d.cb_dim = r.u32();
  d.cb0 = r.vec(4); d.proj0 = r.vec(4);
  uint32_t n = r.u32();
  if (!r.bad && n > 4096) r.fail("bad decoder codebook count");
  for (uint32_t i = 0; i < n && !r.bad; ++i) d.cb_rest.push_back(r.vec(4));
  d.proj_rest = r.vec(4);
  d.pre_conv = conv1d(r);
  d.in_w = r.vec(4); d.in_b = r.vec(4);
  n = r.u32();
  if (!r.bad && n > 4096) r.fail("bad decoder layer count");
  for (uint32_t i = 0; i < n && !r.bad; ++i) {
    HDecLayer L;
    L.q = r.vec(4); L.k = r.vec(4); L.v = r.vec(4); L.o = r.vec(4);
    L.gate = r.vec(4); L.up = r.vec(4); L.down = r.vec(4);
    L.in_norm = r.vec(4); L.post_norm = r.vec(4); L.attn_scale = r.vec(4); L.mlp_scale = r.vec(4);
    d.layers.push_back(L);
  }
  d.norm = r.vec(4); d.out_w = r.vec(4); d.out_b = r.vec(4);
  n = r.u32();
  if (!r.bad && n > 4096) r.fail("bad decoder upsample count");
  for (uint32_t i = 0; i < n && !r.bad; ++i) {
    r.u32();
    skip_conv_t1d(r);
    skip_dw_conv(r);
    for (int j = 0; j < 7; ++j) r.vec(4);
  }
  conv1d(r);
  n = r.u32();
  if (!r.bad && n > 4096) r.fail("bad vocos block count");
  for (uint32_t i = 0; i < n && !r.bad; ++i) {
    r.vec(4); r.vec(4);
    skip_conv_t1d(r);
    const uint32_t nr = r.u32();
    if (!r.bad && nr > 4096) r.fail("bad vocos residual count");
    for (uint32_t j = 0; j < nr && !r.bad; ++j) {
      r.vec(4); r.vec(4); conv1d(r); r.vec(4); r.vec(4); conv1d(r);
    }
  }
  r.vec(4); r.vec(4);
  conv1d(r);
  d.rope_cos = r.vec(4); d.rope_sin = r.vec(4);
  if (out && !r.bad) *out = std::move(d);
}

}  // namespace

int parse_model(const char* path, HModel* out, std::string* err, HDecoder* dec) {
  File fh;
  fh.f = fopen(path, "rb");
  if (!fh.f) {
    if (err) *err = std::string("cannot open ") + path;
    return QTTS_ERR_IO;
  }
  fseeko(fh.f, 0, SEEK_END);
  Reader r{fh.f, (uint64_t)ftello(fh.f)};
  fseeko(fh.f, 0, SEEK_SET);
  HModel m;
  m.file_size = r.size;
  char magic[4];
  r.bytes(magic, 4);
  if (!r.bad && memcmp(magic, "QTTS", 4) != 0) r.fail("Invalid magic (expected QTTS)");
  const uint32_t ver = r.u32();
  if (!r.bad && ver != 1) r.fail("unsupported version (expected 1)");
  const int fmt = r.u8();
  if (!r.bad && fmt != 0 && fmt != 1) r.fail("Unknown format");
  qtts_dims& d = m.d;
  d.fmt = fmt;
  // load_talker (save.rs:300-351)
  d.t_layers = (int)r.u32(); d.t_hidden = (int)r.u32(); d.t_text_hidden = (int)r.u32();
  d.t_heads = (int)r.u32(); d.t_kv_heads = (int)r.u32(); d.t_head_dim = (int)r.u32();
  m.t_kv_groups = (int)r.u32();
  m.t_nsec = (int)r.u32();
  if (!r.bad && (d.t_layers <= 0 || d.t_layers > 1024 || d.t_hidden <= 0 || d.t_hidden > 65536 ||
                 d.t_heads <= 0 || d.t_kv_heads <= 0 || d.t_heads % d.t_kv_heads || d.t_head_dim <= 0 ||
                 m.t_nsec < 0 || m.t_nsec > 3 || m.t_kv_groups != d.t_heads / d.t_kv_heads))
    r.fail("bad talker header");
  for (int i = 0; i < m.t_nsec && !r.bad; ++i) d.t_sec[i] = (int)r.u32();
  if (!r.bad) {
    m.tl.resize(d.t_layers);
    for (int l = 0; l < d.t_layers && !r.bad; ++l) read_layer(r, fmt, m.tl[l]);
  }
  m.codec_emb = r.weight(fmt);
  m.text_emb = r.weight(fmt);
  m.fc1 = r.weight(fmt);
  m.fc1_b = r.vec(4);
  m.fc2 = r.weight(fmt);
  m.fc2_b = r.vec(4);
  m.codec_head = r.weight(fmt);
  m.t_final = r.vec(2);
  m.t_cos = r.vec(4);
  m.t_sin = r.vec(4);
  if (!r.bad) {
    d.t_inter = (int)m.tl[0].gate.n;
    d.t_vocab = (int)m.codec_head.n;
    d.t_text_vocab = (int)m.text_emb.k;
    for (int l = 0; l < d.t_layers && !r.bad; ++l)
      check_layer(r, m.tl[l], d.t_hidden, d.t_heads, d.t_kv_heads, d.t_head_dim, d.t_inter, "talker");
    check_w(r, m.codec_emb, m.codec_emb.k, d.t_hidden, "codec_embedding");
    check_w(r, m.text_emb, m.text_emb.k, d.t_text_hidden, "text_embedding");
    check_w(r, m.fc1, d.t_text_hidden, m.fc1.n, "text_proj_fc1");
    check_w(r, m.fc2, m.fc1.n, d.t_hidden, "text_proj_fc2");
    check_w(r, m.codec_head, d.t_hidden, m.codec_head.n, "codec_head");
    if (!r.bad && (m.fc1_b.len != m.fc1.n || m.fc2_b.len != m.fc2.n || m.t_final.len != (uint64_t)d.t_hidden))
      r.fail("talker bias / norm length mismatch");
    const uint64_t half = (uint64_t)d.t_head_dim / 2;
    if (!r.bad && (m.t_cos.len != m.t_sin.len || m.t_cos.len % half)) r.fail("talker rope table length mismatch");
    d.t_max_pos = r.bad ? 0 : (int)(m.t_cos.len / half);
  }
  // load_predictor (save.rs:353-409)
  d.p_layers = (int)r.u32(); d.p_hidden = (int)r.u32(); d.p_heads = (int)r.u32();
  d.p_kv_heads = (int)r.u32(); d.p_head_dim = (int)r.u32();
  m.p_kv_groups = (int)r.u32();
  if (!r.bad && (d.p_layers <= 0 || d.p_layers > 1024 || d.p_hidden <= 0 || d.p_heads <= 0 || d.p_kv_heads <= 0 ||
                 d.p_heads % d.p_kv_heads || m.p_kv_groups != d.p_heads / d.p_kv_heads))
    r.fail("bad predictor header");
  m.has_proj = r.u8() == 1;
  if (m.has_proj) {
    m.input_proj = r.weight(fmt);
    m.input_proj_b = r.vec(4);
  }
  const uint32_t n_emb = r.u32();
  if (!r.bad && (n_emb == 0 || n_emb > 64)) r.fail("bad codec embedding count");
  if (!r.bad) {
    m.p_emb.resize(n_emb);
    for (uint32_t g = 0; g < n_emb && !r.bad; ++g) m.p_emb[g] = r.weight(fmt);
    m.pl.resize(d.p_layers);
    for (int l = 0; l < d.p_layers && !r.bad; ++l) read_layer(r, fmt, m.pl[l]);
    const uint32_t n_lm = r.u32();
    if (!r.bad && (n_lm == 0 || n_lm > 64)) r.fail("bad lm_head count");
    if (!r.bad) {
      m.lm.resize(n_lm);
      for (uint32_t g = 0; g < n_lm && !r.bad; ++g) m.lm[g] = r.weight(fmt);
    }
    m.p_final = r.vec(2);
    m.p_cos = r.vec(4);
    m.p_sin = r.vec(4);
  }
  if (!r.bad) {
    d.p_inter = (int)m.pl[0].gate.n;
    d.p_vocab = (int)m.lm[0].n;
    d.p_groups = (int)m.lm.size();
    for (int l = 0; l < d.p_layers && !r.bad; ++l)
      check_layer(r, m.pl[l], d.p_hidden, d.p_heads, d.p_kv_heads, d.p_head_dim, d.p_inter, "predictor");
    if (m.has_proj) {
      check_w(r, m.input_proj, d.t_hidden, d.p_hidden, "input_proj");
      if (!r.bad && m.input_proj_b.len != (uint64_t)d.p_hidden) r.fail("input_proj bias length mismatch");
    } else if (!r.bad && d.p_hidden != d.t_hidden) {
      r.fail("predictor without input_proj needs equal hidden sizes");
    }
    for (size_t g = 0; g < m.p_emb.size() && !r.bad; ++g)
      check_w(r, m.p_emb[g], m.p_emb[g].k, d.t_hidden, "predictor codec_embedding");
    for (size_t g = 0; g < m.lm.size() && !r.bad; ++g) check_w(r, m.lm[g], d.p_hidden, d.p_vocab, "lm_head");
    // code_predictor.rs:257 and :285 index codec_embeddings[0 .. lm_heads.len())
    if (!r.bad && m.p_emb.size() < m.lm.size()) r.fail("fewer codec embeddings than lm_heads");
    if (!r.bad && m.lm.size() + 1 > 16) r.fail("more than 15 lm_heads");
    if (!r.bad && m.p_final.len != (uint64_t)d.p_hidden) r.fail("predictor final norm length mismatch");
    const uint64_t half = (uint64_t)d.p_head_dim / 2;
    if (!r.bad && (m.p_cos.len != m.p_sin.len || m.p_cos.len % half)) r.fail("predictor rope table length mismatch");
    d.p_max_pos = r.bad ? 0 : (int)(m.p_cos.len / half);
  }
  if (!r.bad) read_decoder(r, dec);
  if (r.bad) {
    if (err) *err = r.msg;
    return QTTS_ERR_FORMAT;
  }
  *out = std::move(m);
  return QTTS_OK;
}

// ---------------------------------------------------------------------------
// synthetic writer -- splitmix64 streams + Box-Muller, one stream per tensor
namespace {
uint64_t sm64(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
double u01(uint64_t* s) { return ((double)(sm64(s) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
double gauss(uint64_t* s) {
  const double u1 = u01(s), u2 = u01(s);
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}
uint64_t stream_seed(uint64_t seed, uint64_t id) {
  uint64_t s = seed ^ (id * 0xD1B54A32D192ED03ull);
  (void)sm64(&s);
  return s;
}
uint16_t f2h(float f) {  // round to nearest even (half 2.x from_f32)
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0));
  const int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    const int shift = 14 - e;
    uint32_t hm = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
    return (uint16_t)(sign | hm);
  }
  const uint32_t hm = man >> 13, rem = man & 0x1fffu;
  uint16_t o = (uint16_t)(sign | ((uint32_t)e << 10) | hm);
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) o++;
  return o;
}

struct Writer {
  FILE* f;
  uint64_t seed;
  uint64_t id = 0;
  bool bad = false;
  std::vector<uint8_t> buf = std::vector<uint8_t>(1u << 22);
  void bytes(const void* p, size_t n) {
    if (fwrite(p, 1, n, f) != n) bad = true;
  }
  void u32(uint32_t v) { bytes(&v, 4); }
  void u64(uint64_t v) { bytes(&v, 8); }
  void u8(uint8_t v) { bytes(&v, 1); }
  void q4(uint64_t k, uint64_t n) {
    uint64_t s = stream_seed(seed, ++id);
    u64(k); u64(n);
    const uint64_t nb = k * n / 2;
    u64(nb);
    for (uint64_t done = 0; done < nb;) {
      const uint64_t m = nb - done < buf.size() ? nb - done : buf.size();
      for (uint64_t i = 0; i < m; i += 8) {
        const uint64_t r = sm64(&s);
        memcpy(buf.data() + i, &r, (m - i) < 8 ? (m - i) : 8);
      }
      bytes(buf.data(), m);
      done += m;
    }
    const uint64_t ns = k * n / 32;
    u64(ns);
    uint16_t* sb = reinterpret_cast<uint16_t*>(buf.data());
    for (uint64_t done = 0; done < ns;) {
      const uint64_t m = ns - done < buf.size() / 2 ? ns - done : buf.size() / 2;
      for (uint64_t i = 0; i < m; ++i) sb[i] = f2h((float)fabs(gauss(&s) * 0.02));
      bytes(sb, m * 2);
      done += m;
    }
  }
  void f16w(uint64_t k, uint64_t n) {
    uint64_t s = stream_seed(seed, ++id);
    u64(k); u64(n); u64(k * n);
    for (uint64_t i = 0; i < k * n; ++i) {
      const uint16_t h = f2h((float)(gauss(&s) * 0.02));
      bytes(&h, 2);
    }
  }
  void weight(int fmt, uint64_t k, uint64_t n) {
    if (fmt == 1) q4(k, n);
    else f16w(k, n);
  }
  void norm(uint64_t n) {
    ++id;
    u64(n);
    const uint16_t one = 0x3c00;
    for (uint64_t i = 0; i < n; ++i) bytes(&one, 2);
  }
  void bias(uint64_t n) {
    uint64_t s = stream_seed(seed, ++id);
    u64(n);
    for (uint64_t i = 0; i < n; ++i) {
      const float v = (float)(gauss(&s) * 0.02);
      bytes(&v, 4);
    }
  }
  void f32vec(const std::vector<float>& v) {
    ++id;
    u64(v.size());
    bytes(v.data(), v.size() * 4);
  }
  void gvec(uint64_t n, double mean, double sd) {  // write_f32_vec_io of mean + sd * N(0, 1)
    uint64_t s = stream_seed(seed, ++id);
    u64(n);
    float* fb = reinterpret_cast<float*>(buf.data());
    for (uint64_t done = 0; done < n;) {
      const uint64_t m = n - done < buf.size() / 4 ? n - done : buf.size() / 4;
      for (uint64_t i = 0; i < m; ++i) fb[i] = (float)(mean + sd * gauss(&s));
      bytes(fb, m * 4);
      done += m;
    }
  }
  void empty_vec() { u64(0); }
  void empty_conv1d() {
    for (int i = 0; i < 6; ++i) u32(0);
    empty_vec();
    empty_vec();
  }
};

// rope.rs:11-41 (talker, sections) and loader.rs:399-408 (predictor).
void rope_tables(int hd, int max_pos, const int* sec, int nsec, std::vector<float>& c, std::vector<float>& s,
                 double theta = 1000000.0) {
  const int half = hd / 2;
  c.assign((size_t)max_pos * half, 0.0f);
  s.assign((size_t)max_pos * half, 0.0f);
  int off = 0;
  for (int q = 0; q < nsec; ++q) {
    for (int i = 0; i < sec[q]; ++i) {
      const int dd = off + i;
      const double freq = 1.0 / pow(theta, (double)(2 * dd) / (double)hd);
      for (int p = 0; p < max_pos; ++p) {
        const double a = (double)p * freq;
        c[(size_t)p * half + dd] = (float)cos(a);
        s[(size_t)p * half + dd] = (float)sin(a);
      }
    }
    off += sec[q];
  }
}
}  // namespace

void dims_1p7b(qtts_dims* d) {
  memset(d, 0, sizeof(*d));
  d->t_layers = 28; d->t_hidden = 2048; d->t_text_hidden = 2048; d->t_heads = 16; d->t_kv_heads = 8;
  d->t_head_dim = 128; d->t_inter = 6144; d->t_vocab = 3072; d->t_text_vocab = 151936; d->t_max_pos = 32768;
  d->t_sec[0] = 24; d->t_sec[1] = 20; d->t_sec[2] = 20;
  d->p_layers = 5; d->p_hidden = 1024; d->p_heads = 16; d->p_kv_heads = 8; d->p_head_dim = 128;
  d->p_inter = 3072; d->p_vocab = 2048; d->p_groups = 15; d->p_max_pos = 65536; d->fmt = 1;
}

void dims_tiny(qtts_dims* d) {
  memset(d, 0, sizeof(*d));
  d->t_layers = 2; d->t_hidden = 512; d->t_text_hidden = 512; d->t_heads = 4; d->t_kv_heads = 2;
  d->t_head_dim = 128; d->t_inter = 1024; d->t_vocab = 3072; d->t_text_vocab = 151936; d->t_max_pos = 4096;
  d->t_sec[0] = 24; d->t_sec[1] = 20; d->t_sec[2] = 20;
  d->p_layers = 2; d->p_hidden = 256; d->p_heads = 2; d->p_kv_heads = 1; d->p_head_dim = 128;
  d->p_inter = 512; d->p_vocab = 2048; d->p_groups = 15; d->p_max_pos = 64; d->fmt = 1;
}

// The synthetic speech decoder (decoder.rs:21-108 shapes of the 12 Hz
// tokenizer's decoder): 16 codebooks of 2048 x 256, hidden 512, 16 heads of 64,
// MLP 1024, window 72, 8 layers, latent 1024, RoPE theta 10000 over 8192
// positions.  Values: codebooks N(0, 1); projections N(0, 1/fan_in); biases
// N(0, 0.02); norm weights 1 + N(0, 0.1); layer scales 0.05 + N(0, 0.01).
constexpr uint32_t kDecHidden = 512, kDecHeads = 16, kDecHeadDim = 64, kDecInter = 1024, kDecWindow = 72,
                   kDecCbDim = 256, kDecEntries = 2048, kDecLayers = 8, kDecLatent = 1024, kDecRopePos = 8192;
void write_decoder(Writer& w) {
  const uint32_t H = kDecHidden, A = kDecHeads * kDecHeadDim;
  w.u32(H); w.u32(kDecHeads); w.u32(kDecHeadDim); w.u32(kDecInter); w.u32(kDecWindow); w.u32(kDecCbDim);
  w.gvec((uint64_t)kDecEntries * kDecCbDim, 0.0, 1.0);
  w.gvec((uint64_t)kDecCbDim * 512, 0.0, 1.0 / sqrt((double)kDecCbDim));
  w.u32(15);
  for (int g = 0; g < 15; ++g) w.gvec((uint64_t)kDecEntries * kDecCbDim, 0.0, 1.0);
  w.gvec((uint64_t)kDecCbDim * 512, 0.0, 1.0 / sqrt((double)kDecCbDim));
  // pre-conv: CausalConv1d(512 -> 1024, k = 3), weight [out][in][k]
  w.u32(512); w.u32(kDecLatent); w.u32(3); w.u32(1); w.u32(0); w.u32(1);
  w.gvec((uint64_t)kDecLatent * 512 * 3, 0.0, 1.0 / sqrt(512.0 * 3.0));
  w.gvec(kDecLatent, 0.0, 0.02);
  w.gvec((uint64_t)kDecLatent * H, 0.0, 1.0 / sqrt((double)kDecLatent));
  w.gvec(H, 0.0, 0.02);
  w.u32(kDecLayers);
  for (uint32_t l = 0; l < kDecLayers; ++l) {
    for (int m = 0; m < 3; ++m) w.gvec((uint64_t)H * A, 0.0, 1.0 / sqrt((double)H));  // q, k, v
    w.gvec((uint64_t)A * H, 0.0, 1.0 / sqrt((double)A));                             // o
    w.gvec((uint64_t)H * kDecInter, 0.0, 1.0 / sqrt((double)H));                     // gate
    w.gvec((uint64_t)H * kDecInter, 0.0, 1.0 / sqrt((double)H));                     // up
    w.gvec((uint64_t)kDecInter * H, 0.0, 1.0 / sqrt((double)kDecInter));             // down
    w.gvec(H, 1.0, 0.1); w.gvec(H, 1.0, 0.1);                                         // norms
    w.gvec(H, 0.05, 0.01); w.gvec(H, 0.05, 0.01);                                     // layer scales
  }
  w.gvec(H, 1.0, 0.1);
  w.gvec((uint64_t)H * kDecLatent, 0.0, 1.0 / sqrt((double)H));
  w.gvec(kDecLatent, 0.0, 0.02);
  w.u32(0);                      // no upsample stages
  w.empty_conv1d(); w.u32(0);    // no Vocos stages
  w.empty_vec(); w.empty_vec(); w.empty_conv1d();
  const int sec1[1] = {(int)kDecHeadDim / 2};
  std::vector<float> c, s;
  rope_tables((int)kDecHeadDim, (int)kDecRopePos, sec1, 1, c, s, 10000.0);
  w.f32vec(c); w.f32vec(s);
}

int synth_write(const char* path, const qtts_dims& d, uint64_t seed, std::string* err, bool with_decoder) {
  if (d.t_layers <= 0 || d.p_layers <= 0 || d.t_heads % d.t_kv_heads || d.p_heads % d.p_kv_heads ||
      d.t_hidden % 32 || d.p_hidden % 32 || d.t_inter % 32 || d.p_inter % 32 || d.t_vocab % 32 || d.p_vocab % 32 ||
      (d.fmt != 0 && d.fmt != 1) || d.t_sec[0] + d.t_sec[1] + d.t_sec[2] != d.t_head_dim / 2) {
    if (err) *err = "invalid dimensions for a synthetic model";
    return QTTS_ERR_BADARG;
  }
  File fh;
  fh.f = fopen(path, "wb");
  if (!fh.f) {
    if (err) *err = std::string("cannot create ") + path;
    return QTTS_ERR_IO;
  }
  setvbuf(fh.f, nullptr, _IOFBF, 1 << 23);
  Writer w{fh.f, seed};
  const int fmt = d.fmt;
  w.bytes("QTTS", 4); w.u32(1); w.u8((uint8_t)fmt);  // save.rs:31-35
  const uint64_t tq = (uint64_t)d.t_heads * d.t_head_dim, tkv = (uint64_t)d.t_kv_heads * d.t_head_dim;
  w.u32(d.t_layers); w.u32(d.t_hidden); w.u32(d.t_text_hidden); w.u32(d.t_heads); w.u32(d.t_kv_heads);
  w.u32(d.t_head_dim); w.u32(d.t_heads / d.t_kv_heads); w.u32(3);
  for (int i = 0; i < 3; ++i) w.u32(d.t_sec[i]);
  for (int l = 0; l < d.t_layers; ++l) {  // save.rs:62-74
    w.weight(fmt, d.t_hidden, tq); w.weight(fmt, d.t_hidden, tkv); w.weight(fmt, d.t_hidden, tkv);
    w.weight(fmt, tq, d.t_hidden);
    w.norm(d.t_head_dim); w.norm(d.t_head_dim);
    w.weight(fmt, d.t_hidden, d.t_inter); w.weight(fmt, d.t_hidden, d.t_inter); w.weight(fmt, d.t_inter, d.t_hidden);
    w.norm(d.t_hidden); w.norm(d.t_hidden);
  }
  w.weight(fmt, d.t_vocab, d.t_hidden);
  w.weight(fmt, d.t_text_vocab, d.t_text_hidden);
  w.weight(fmt, d.t_text_hidden, d.t_text_hidden);
  w.bias(d.t_text_hidden);
  w.weight(fmt, d.t_text_hidden, d.t_hidden);
  w.bias(d.t_hidden);
  w.weight(fmt, d.t_hidden, d.t_vocab);
  w.norm(d.t_hidden);
  {
    std::vector<float> c, s;
    rope_tables(d.t_head_dim, d.t_max_pos, d.t_sec, 3, c, s);
    w.f32vec(c); w.f32vec(s);
  }
  const uint64_t pq = (uint64_t)d.p_heads * d.p_head_dim, pkv = (uint64_t)d.p_kv_heads * d.p_head_dim;
  w.u32(d.p_layers); w.u32(d.p_hidden); w.u32(d.p_heads); w.u32(d.p_kv_heads); w.u32(d.p_head_dim);
  w.u32(d.p_heads / d.p_kv_heads);
  if (d.p_hidden != d.t_hidden) {
    w.u8(1);
    w.weight(fmt, d.t_hidden, d.p_hidden);
    w.bias(d.p_hidden);
  } else {
    w.u8(0);
  }
  w.u32(d.p_groups);
  for (int g = 0; g < d.p_groups; ++g) w.weight(fmt, d.p_vocab, d.t_hidden);
  for (int l = 0; l < d.p_layers; ++l) {
    w.weight(fmt, d.p_hidden, pq); w.weight(fmt, d.p_hidden, pkv); w.weight(fmt, d.p_hidden, pkv);
    w.weight(fmt, pq, d.p_hidden);
    w.norm(d.p_head_dim); w.norm(d.p_head_dim);
    w.weight(fmt, d.p_hidden, d.p_inter); w.weight(fmt, d.p_hidden, d.p_inter); w.weight(fmt, d.p_inter, d.p_hidden);
    w.norm(d.p_hidden); w.norm(d.p_hidden);
  }
  w.u32(d.p_groups);
  for (int g = 0; g < d.p_groups; ++g) w.weight(fmt, d.p_hidden, d.p_vocab);
  w.norm(d.p_hidden);
  {
    const int sec1[1] = {d.p_head_dim / 2};
    std::vector<float> c, s;
    rope_tables(d.p_head_dim, d.p_max_pos, sec1, 1, c, s);
    w.f32vec(c); w.f32vec(s);
  }
  if (with_decoder) {
    write_decoder(w);
  } else {
    // empty speech-decoder section (save.rs:171-256 layout)
    for (int i = 0; i < 6; ++i) w.u32(0);
    w.empty_vec(); w.empty_vec(); w.u32(0); w.empty_vec();
    w.empty_conv1d();
    w.empty_vec(); w.empty_vec(); w.u32(0);
    w.empty_vec(); w.empty_vec(); w.empty_vec();
    w.u32(0);
    w.empty_conv1d(); w.u32(0);
    w.empty_vec(); w.empty_vec(); w.empty_conv1d();
    w.empty_vec(); w.empty_vec();
  }
  if (fflush(fh.f) != 0) w.bad = true;
  if (w.bad) {
    if (err) *err = "write failed";
    return QTTS_ERR_IO;
  }
  return QTTS_OK;
}

}  // namespace qtts
