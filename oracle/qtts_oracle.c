/*
 * qtts_oracle.c -- CPU restatement of the QORA-TTS 1.7B per-frame decode loop.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline).  Nothing
 * in the product links or calls this file.  PARITY UNPINNED: the reference
 * Rust crate cannot be built here and ships no golden vectors for this path;
 * see qtts_oracle.h for the arithmetic conventions that keep this file
 * bit-faithful to the Rust source.
 *
 * Reference paths below are relative to the qora-tts crate root.
 */
#define _GNU_SOURCE
#include "qtts_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* f16 <-> f32 (half 2.x)                                                    */
/* ------------------------------------------------------------------------ */

float oq_h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do { man <<= 1; e++; } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t oq_f2h(float f) { /* round to nearest even */
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    int shift = 14 - e;
    uint32_t half_man = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (half_man & 1u))) half_man++;
    return (uint16_t)(sign | half_man);
  }
  uint32_t half_man = man >> 13;
  uint32_t rem = man & 0x1fffu;
  uint16_t out = (uint16_t)(sign | ((uint32_t)e << 10) | half_man);
  if (rem > 0x1000u || (rem == 0x1000u && (half_man & 1u))) out++;
  return out;
}

/* ------------------------------------------------------------------------ */
/* seeded synthetic data (splitmix64 + Box-Muller)                           */
/* ------------------------------------------------------------------------ */

static uint64_t sm64(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static double u01(uint64_t* s) { return ((double)(sm64(s) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
static double gauss(uint64_t* s) {
  double u1 = u01(s), u2 = u01(s);
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}
static uint64_t stream_seed(uint64_t seed, uint64_t id) {
  uint64_t s = seed ^ (id * 0xD1B54A32D192ED03ull);
  (void)sm64(&s);
  return s;
}

void oq_rand_normal(uint64_t seed, float* out, size_t n, float stddev) {
  uint64_t s = stream_seed(seed, 0x6e6f726dull);
  for (size_t i = 0; i < n; i++) out[i] = (float)(gauss(&s) * stddev);
}
void oq_rand_tokens(uint64_t seed, uint32_t* out, size_t n, uint32_t vocab) {
  uint64_t s = stream_seed(seed, 0x746f6bull);
  for (size_t i = 0; i < n; i++) out[i] = (uint32_t)(sm64(&s) % vocab);
}
void oq_rand_bytes(uint64_t seed, uint8_t* out, size_t n) {
  uint64_t s = stream_seed(seed, 0x627974ull);
  size_t i = 0;
  for (; i + 8 <= n; i += 8) { uint64_t r = sm64(&s); memcpy(out + i, &r, 8); }
  if (i < n) { uint64_t r = sm64(&s); memcpy(out + i, &r, n - i); }
}
void oq_rand_scales(uint64_t seed, uint16_t* out, size_t n, float stddev) {
  uint64_t s = stream_seed(seed, 0x73636cull);
  for (size_t i = 0; i < n; i++) out[i] = oq_f2h((float)fabs(gauss(&s) * stddev));
}

/* ------------------------------------------------------------------------ */
/* thread policy (gemv.rs:268-272)                                           */
/* ------------------------------------------------------------------------ */

static int g_threads = 8;
void oq_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int oq_get_threads(void) { return g_threads; }

/* ------------------------------------------------------------------------ */
/* Q4 / F16 kernels (gemv.rs)                                                */
/* ------------------------------------------------------------------------ */

/* gemv.rs:222-261 gemv_q4_inner: LUT scatter-add over rows [k0,k1). */
static void gemv_q4_inner(const float* input, const uint8_t* packed, const uint16_t* scales,
                          size_t n, size_t k0, size_t k1, float* out) {
  const size_t gpr = n / 32, ppg = 16, ppr = gpr * ppg;
  for (size_t j = 0; j < n; j++) out[j] = 0.0f;
  for (size_t ki = k0; ki < k1; ki++) {
    float iv = input[ki];
    if (iv == 0.0f) continue; /* :233 */
    size_t sb = ki * gpr, pb = ki * ppr;
    for (size_t g = 0; g < gpr; g++) {
      float s = oq_h2f(scales[sb + g]) * iv; /* :239 */
      if (s == 0.0f) continue;             /* :240 */
      float lut[16] = {s * -8.0f, s * -7.0f, s * -6.0f, s * -5.0f, s * -4.0f, s * -3.0f,
                       s * -2.0f, s * -1.0f, 0.0f,      s,         s * 2.0f,  s * 3.0f,
                       s * 4.0f,  s * 5.0f,  s * 6.0f,  s * 7.0f};
      const uint8_t* p = packed + pb + g * ppg;
      float* o = out + g * 32;
      for (size_t j = 0; j < ppg; j++) {
        uint8_t b = p[j];
        o[j * 2] += lut[b & 0x0f];    /* :254 low nibble = even column */
        o[j * 2 + 1] += lut[b >> 4];  /* :255 */
      }
    }
  }
}

typedef struct {
  const float* x; const uint8_t* packed; const uint16_t* scales;
  size_t n, k0, k1; float* out;
} gq_job;
static void* gq_thread(void* a) {
  gq_job* j = (gq_job*)a;
  gemv_q4_inner(j->x, j->packed, j->scales, j->n, j->k0, j->k1, j->out);
  return NULL;
}

/* gemv.rs:263-309 gemv_q4: K split over spawned threads, partials summed in
 * thread order. */
void oq_gemv_q4(const float* x, const uint8_t* packed, const uint16_t* scales, size_t k,
                size_t n, float* y) {
  int nt = (k * n >= 4000000) ? g_threads : 1;
  if (nt <= 1) { gemv_q4_inner(x, packed, scales, n, 0, k, y); return; }
  size_t chunk = (k + nt - 1) / nt;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nt);
  gq_job* jobs = (gq_job*)malloc(sizeof(gq_job) * nt);
  float* parts = (float*)malloc(sizeof(float) * n * nt);
  for (int t = 0; t < nt; t++) {
    size_t k0 = (size_t)t * chunk, k1 = (size_t)(t + 1) * chunk;
    if (k1 > k) k1 = k;
    if (k0 > k1) k0 = k1; /* Rust range k0..k1 with k0 > k1 is empty */
    jobs[t] = (gq_job){x, packed, scales, n, k0, k1, parts + (size_t)t * n};
    pthread_create(&th[t], NULL, gq_thread, &jobs[t]);
  }
  for (size_t j = 0; j < n; j++) y[j] = 0.0f;
  for (int t = 0; t < nt; t++) {
    pthread_join(th[t], NULL);
    const float* p = parts + (size_t)t * n;
    for (size_t j = 0; j < n; j++) y[j] += p[j];
  }
  free(parts); free(jobs); free(th);
}

/* gemv.rs:311-375 gemm_q4: every row is a full-K gemv_q4_inner (the row
 * split over threads does not change any row's summation order). */
void oq_gemm_q4(const float* x, size_t seq, const uint8_t* packed, const uint16_t* scales,
                size_t k, size_t n, float* y) {
  for (size_t t = 0; t < seq; t++) gemv_q4_inner(x + t * k, packed, scales, n, 0, k, y + t * n);
}

/* gemv.rs:183-196 gemv_f16 */
void oq_gemv_f16(const float* x, const uint16_t* w, size_t k, size_t n, float* y) {
  for (size_t j = 0; j < n; j++) y[j] = 0.0f;
  for (size_t ki = 0; ki < k; ki++) {
    float iv = x[ki];
    const uint16_t* row = w + ki * n;
    for (size_t j = 0; j < n; j++) y[j] += iv * oq_h2f(row[j]);
  }
}

/* gemv.rs:92-130 quantize_f32_to_q4 */
void oq_quantize_q4(const float* data, size_t k, size_t n, uint8_t* packed, uint16_t* scales) {
  size_t gpr = n / 32;
  for (size_t ki = 0; ki < k; ki++) {
    for (size_t g = 0; g < gpr; g++) {
      size_t gi = ki * gpr + g, c0 = g * 32;
      float absmax = 0.0f;
      for (size_t j = 0; j < 32; j++) {
        float v = fabsf(data[ki * n + c0 + j]);
        if (v > absmax) absmax = v;
      }
      float scale = absmax / 7.0f;
      scales[gi] = oq_f2h(scale);
      float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
      for (size_t j = 0; j < 32; j += 2) {
        float v0 = data[ki * n + c0 + j], v1 = data[ki * n + c0 + j + 1];
        float r0 = roundf(v0 * inv), r1 = roundf(v1 * inv); /* Rust round: half away from 0 */
        r0 = r0 < -8.0f ? -8.0f : (r0 > 7.0f ? 7.0f : r0);
        r1 = r1 < -8.0f ? -8.0f : (r1 > 7.0f ? 7.0f : r1);
        /* f32::clamp keeps NaN and Rust's `as u8` maps NaN to 0 (saturating
         * cast); a C cast of NaN is undefined, so spell it out */
        uint8_t q0 = r0 != r0 ? 0 : (uint8_t)(r0 + 8.0f), q1 = r1 != r1 ? 0 : (uint8_t)(r1 + 8.0f);
        packed[gi * 16 + j / 2] = (uint8_t)(q0 | (q1 << 4));
      }
    }
  }
}

/* gemv.rs:378-400 embed_lookup_q4 (= talker.rs:119-142) */
void oq_embed_q4(const uint8_t* packed, const uint16_t* scales, size_t n, size_t row, float* out) {
  size_t gpr = n / 32;
  for (size_t g = 0; g < gpr; g++) {
    float scale = oq_h2f(scales[row * gpr + g]);
    const uint8_t* p = packed + row * gpr * 16 + g * 16;
    for (size_t j = 0; j < 16; j++) {
      int q0 = (p[j] & 0x0f) - 8, q1 = ((p[j] >> 4) & 0x0f) - 8;
      out[g * 32 + j * 2] = scale * (float)q0;
      out[g * 32 + j * 2 + 1] = scale * (float)q1;
    }
  }
}

/* gemv.rs:408-417 rms_norm_f16 */
void oq_rms_norm_f16(const float* x, const uint16_t* gamma, size_t n, float* out) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
  float inv = 1.0f / sqrtf(ss / (float)n + 1e-6f);
  for (size_t i = 0; i < n; i++) out[i] = x[i] * inv * oq_h2f(gamma[i]);
}

/* gemv.rs:434-445 softmax_raw */
void oq_softmax_raw(float* s, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++) mx = fmaxf(mx, s[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) { s[i] = expf(s[i] - mx); sum += s[i]; }
  float inv = 1.0f / sum;
  for (size_t i = 0; i < n; i++) s[i] *= inv;
}

/* gemv.rs:449-451 silu */
float oq_silu(float x) { return x / (1.0f + expf(-x)); }

/* rope.rs:11-41 build_mrope_tables */
void oq_build_mrope_tables(int head_dim, int max_pos, double theta, const int* sec, int n_sec,
                           float* cos_t, float* sin_t) {
  int half = head_dim / 2, off = 0;
  for (int s = 0; s < n_sec; s++) {
    for (int i = 0; i < sec[s]; i++) {
      int d = off + i;
      double freq = 1.0 / pow(theta, (double)(2 * d) / (double)head_dim);
      for (int p = 0; p < max_pos; p++) {
        double a = (double)p * freq;
        cos_t[(size_t)p * half + d] = (float)cos(a);
        sin_t[(size_t)p * half + d] = (float)sin(a);
      }
    }
    off += sec[s];
  }
}

/* loader.rs:399-408 (predictor table, standard rope) */
void oq_build_rope_tables(int head_dim, int max_pos, double theta, float* cos_t, float* sin_t) {
  int half = head_dim / 2;
  for (int i = 0; i < half; i++) {
    double freq = 1.0 / pow(theta, (double)(2 * i) / (double)head_dim);
    for (int p = 0; p < max_pos; p++) {
      double a = (double)p * freq;
      cos_t[(size_t)p * half + i] = (float)cos(a);
      sin_t[(size_t)p * half + i] = (float)sin(a);
    }
  }
}

/* ------------------------------------------------------------------------ */
/* model structures (talker.rs:19-56, code_predictor.rs:14-46)               */
/* ------------------------------------------------------------------------ */

typedef struct {
  int fmt;
  uint64_t k, n;
  uint8_t* packed;   /* Q4 */
  uint16_t* scales;  /* Q4 */
  uint16_t* data;    /* F16 */
} ow;

typedef struct {
  ow q, k, v, o, gate, up, down;
  uint16_t *q_norm, *k_norm, *in_norm, *post_norm;
} ol;

struct oq_model {
  oq_dims d;
  /* talker */
  int t_kv_groups, t_nsec;
  ol* tl;
  ow codec_emb, text_emb, fc1, fc2, codec_head;
  float *fc1_b, *fc2_b;
  uint16_t* t_final_norm;
  float *t_cos, *t_sin;
  uint64_t t_rope_len;
  /* predictor */
  int p_kv_groups, has_proj;
  ow input_proj;
  float* input_proj_b;
  int n_emb, n_lm;
  ow* p_emb;
  ol* pl;
  ow* lm;
  uint16_t* p_final_norm;
  float *p_cos, *p_sin;
  uint64_t p_rope_len;
};

static void gemv_w(const ow* w, const float* x, float* y) { /* gemv.rs:149-154 */
  if (w->fmt == 1) oq_gemv_q4(x, w->packed, w->scales, w->k, w->n, y);
  else oq_gemv_f16(x, w->data, w->k, w->n, y);
}
static void gemm_w(const ow* w, const float* x, size_t seq, float* y) { /* gemv.rs:157-162 */
  if (w->fmt == 1) oq_gemm_q4(x, seq, w->packed, w->scales, w->k, w->n, y);
  else for (size_t t = 0; t < seq; t++) oq_gemv_f16(x + t * w->k, w->data, w->k, w->n, y + t * w->n);
}
static void embed_w(const ow* w, size_t row, size_t hidden, float* out) { /* talker.rs:119-150 */
  if (w->fmt == 1) oq_embed_q4(w->packed, w->scales, hidden, row, out);
  else for (size_t i = 0; i < hidden; i++) out[i] = oq_h2f(w->data[row * hidden + i]);
}

/* ------------------------------------------------------------------------ */
/* synthetic writer: the save.rs:48-137 byte layout                         */
/* ------------------------------------------------------------------------ */

typedef struct { FILE* f; uint64_t seed; uint64_t id; int err; } wctx;
static void w_bytes(wctx* c, const void* p, size_t n) { if (fwrite(p, 1, n, c->f) != n) c->err = 1; }
static void w_u32(wctx* c, uint32_t v) { w_bytes(c, &v, 4); }
static void w_u64(wctx* c, uint64_t v) { w_bytes(c, &v, 8); }
static void w_u8(wctx* c, uint8_t v) { w_bytes(c, &v, 1); }

#define WCHUNK (1u << 22)
/* write_weight_io (gemv.rs:558-573): Q4 = k, n, len+packed, len+scales */
static void w_q4(wctx* c, uint64_t k, uint64_t n) {
  uint64_t s = stream_seed(c->seed, ++c->id);
  w_u64(c, k); w_u64(c, n);
  uint64_t nb = k * n / 2;
  w_u64(c, nb);
  uint8_t* buf = (uint8_t*)malloc(WCHUNK);
  for (uint64_t done = 0; done < nb;) {
    uint64_t m = nb - done < WCHUNK ? nb - done : WCHUNK;
    for (uint64_t i = 0; i < m; i += 8) { uint64_t r = sm64(&s); memcpy(buf + i, &r, (m - i) < 8 ? (m - i) : 8); }
    w_bytes(c, buf, m);
    done += m;
  }
  uint64_t ns = k * n / 32;
  w_u64(c, ns);
  uint16_t* sb = (uint16_t*)buf;
  for (uint64_t done = 0; done < ns;) {
    uint64_t m = ns - done < WCHUNK / 2 ? ns - done : WCHUNK / 2;
    for (uint64_t i = 0; i < m; i++) sb[i] = oq_f2h((float)fabs(gauss(&s) * 0.02));
    w_bytes(c, sb, m * 2);
    done += m;
  }
  free(buf);
}
/* F16 weight: k, n, len + N(0,0.02) f16 data */
static void w_f16w(wctx* c, uint64_t k, uint64_t n) {
  uint64_t s = stream_seed(c->seed, ++c->id);
  w_u64(c, k); w_u64(c, n); w_u64(c, k * n);
  for (uint64_t i = 0; i < k * n; i++) { uint16_t h = oq_f2h((float)(gauss(&s) * 0.02)); w_bytes(c, &h, 2); }
}
static void w_weight(wctx* c, int fmt, uint64_t k, uint64_t n) { if (fmt == 1) w_q4(c, k, n); else w_f16w(c, k, n); }
/* Test fixture, not a reference format: a Q4 weight whose column j equals
 * column j % period in every row (one scale per row for all its groups, the
 * nibbles of the first `period` columns repeated), so a projection through
 * it gives bit-equal outputs on every column of a residue class.  Used for
 * the predictor heads to exercise argmax ties (code_predictor.rs:328-334). */
static int g_tie_period = 0;
void oq_set_tie_period(int period) { g_tie_period = period > 0 ? period : 0; }
static void w_q4_tied(wctx* c, uint64_t k, uint64_t n, int period) {
  uint64_t s = stream_seed(c->seed, ++c->id);
  w_u64(c, k); w_u64(c, n);
  w_u64(c, k * n / 2);
  uint8_t* row = (uint8_t*)malloc(n / 2);
  uint8_t nib[64];
  for (uint64_t r = 0; r < k; r++) {
    for (int j = 0; j < period; j++) nib[j] = (uint8_t)(sm64(&s) & 15u);
    for (uint64_t j = 0; j < n; j += 2) row[j / 2] = (uint8_t)(nib[j % period] | (nib[(j + 1) % period] << 4));
    w_bytes(c, row, n / 2);
  }
  free(row);
  w_u64(c, k * n / 32);
  for (uint64_t r = 0; r < k; r++) {
    const uint16_t h = oq_f2h((float)fabs(gauss(&s) * 0.02));
    for (uint64_t g = 0; g < n / 32; g++) w_bytes(c, &h, 2);
  }
}
static void w_norm(wctx* c, uint64_t n) { /* write_f16_vec_io of ones */
  ++c->id;
  w_u64(c, n);
  for (uint64_t i = 0; i < n; i++) { uint16_t one = 0x3c00; w_bytes(c, &one, 2); }
}
static void w_bias(wctx* c, uint64_t n) { /* write_f32_vec_io of N(0,0.02) */
  uint64_t s = stream_seed(c->seed, ++c->id);
  w_u64(c, n);
  for (uint64_t i = 0; i < n; i++) { float v = (float)(gauss(&s) * 0.02); w_bytes(c, &v, 4); }
}
static void w_f32vec(wctx* c, const float* v, uint64_t n) { ++c->id; w_u64(c, n); w_bytes(c, v, n * 4); }
static void w_gvec(wctx* c, uint64_t n, double mean, double sd) { /* write_f32_vec_io of mean + sd*N(0,1) */
  uint64_t s = stream_seed(c->seed, ++c->id);
  w_u64(c, n);
  for (uint64_t i = 0; i < n; i++) { float v = (float)(mean + sd * gauss(&s)); w_bytes(c, &v, 4); }
}
static void w_empty_vec(wctx* c) { w_u64(c, 0); }
static void w_empty_conv1d(wctx* c) { for (int i = 0; i < 6; i++) w_u32(c, 0); w_empty_vec(c); w_empty_vec(c); }

void oq_dims_1p7b(oq_dims* d) {
  memset(d, 0, sizeof(*d));
  d->t_layers = 28; d->t_hidden = 2048; d->t_text_hidden = 2048; d->t_heads = 16;
  d->t_kv_heads = 8; d->t_head_dim = 128; d->t_inter = 6144; d->t_vocab = 3072;
  d->t_text_vocab = 151936; d->t_max_pos = 32768;
  d->t_sec[0] = 24; d->t_sec[1] = 20; d->t_sec[2] = 20;
  d->p_layers = 5; d->p_hidden = 1024; d->p_heads = 16; d->p_kv_heads = 8; d->p_head_dim = 128;
  d->p_inter = 3072; d->p_vocab = 2048; d->p_groups = 15; d->p_max_pos = 65536; d->fmt = 1;
}

void oq_dims_tiny(oq_dims* d) {
  memset(d, 0, sizeof(*d));
  d->t_layers = 2; d->t_hidden = 512; d->t_text_hidden = 512; d->t_heads = 4;
  d->t_kv_heads = 2; d->t_head_dim = 128; d->t_inter = 1024; d->t_vocab = 3072;
  d->t_text_vocab = 151936; d->t_max_pos = 4096;
  d->t_sec[0] = 24; d->t_sec[1] = 20; d->t_sec[2] = 20;
  d->p_layers = 2; d->p_hidden = 256; d->p_heads = 2; d->p_kv_heads = 1; d->p_head_dim = 128;
  d->p_inter = 512; d->p_vocab = 2048; d->p_groups = 15; d->p_max_pos = 64; d->fmt = 1;
}

/* The synthetic speech decoder, decoder.rs:21-108 shapes (12 Hz tokenizer
 * decoder): 16 codebooks of 2048 x 256, hidden 512, 16 heads of 64, MLP 1024,
 * window 72, 8 layers, latent 1024, RoPE theta 10000 over 8192 positions;
 * upsample and Vocos stages empty (they are not restated here).  Values:
 * codebooks N(0,1), projections N(0,1/fan_in), biases N(0,0.02), norm weights
 * 1 + N(0,0.1), layer scales 0.05 + N(0,0.01); save.rs:171-256 order. */
static void w_decoder(wctx* c) {
  const uint32_t H = OQ_DEC_HIDDEN, A = OQ_DEC_HEADS * OQ_DEC_HEAD_DIM;
  w_u32(c, H); w_u32(c, OQ_DEC_HEADS); w_u32(c, OQ_DEC_HEAD_DIM); w_u32(c, OQ_DEC_INTER);
  w_u32(c, OQ_DEC_WINDOW); w_u32(c, OQ_DEC_CB_DIM);
  w_gvec(c, (uint64_t)OQ_DEC_ENTRIES * OQ_DEC_CB_DIM, 0.0, 1.0);
  w_gvec(c, (uint64_t)OQ_DEC_CB_DIM * 512, 0.0, 1.0 / sqrt((double)OQ_DEC_CB_DIM));
  w_u32(c, 15);
  for (int g = 0; g < 15; g++) w_gvec(c, (uint64_t)OQ_DEC_ENTRIES * OQ_DEC_CB_DIM, 0.0, 1.0);
  w_gvec(c, (uint64_t)OQ_DEC_CB_DIM * 512, 0.0, 1.0 / sqrt((double)OQ_DEC_CB_DIM));
  w_u32(c, 512); w_u32(c, OQ_DEC_LATENT); w_u32(c, 3); w_u32(c, 1); w_u32(c, 0); w_u32(c, 1);
  w_gvec(c, (uint64_t)OQ_DEC_LATENT * 512 * 3, 0.0, 1.0 / sqrt(512.0 * 3.0));
  w_gvec(c, OQ_DEC_LATENT, 0.0, 0.02);
  w_gvec(c, (uint64_t)OQ_DEC_LATENT * H, 0.0, 1.0 / sqrt((double)OQ_DEC_LATENT));
  w_gvec(c, H, 0.0, 0.02);
  w_u32(c, OQ_DEC_LAYERS);
  for (int l = 0; l < OQ_DEC_LAYERS; l++) {
    for (int m = 0; m < 3; m++) w_gvec(c, (uint64_t)H * A, 0.0, 1.0 / sqrt((double)H));
    w_gvec(c, (uint64_t)A * H, 0.0, 1.0 / sqrt((double)A));
    w_gvec(c, (uint64_t)H * OQ_DEC_INTER, 0.0, 1.0 / sqrt((double)H));
    w_gvec(c, (uint64_t)H * OQ_DEC_INTER, 0.0, 1.0 / sqrt((double)H));
    w_gvec(c, (uint64_t)OQ_DEC_INTER * H, 0.0, 1.0 / sqrt((double)OQ_DEC_INTER));
    w_gvec(c, H, 1.0, 0.1); w_gvec(c, H, 1.0, 0.1);
    w_gvec(c, H, 0.05, 0.01); w_gvec(c, H, 0.05, 0.01);
  }
  w_gvec(c, H, 1.0, 0.1);
  w_gvec(c, (uint64_t)H * OQ_DEC_LATENT, 0.0, 1.0 / sqrt((double)H));
  w_gvec(c, OQ_DEC_LATENT, 0.0, 0.02);
  w_u32(c, 0);
  w_empty_conv1d(c); w_u32(c, 0);
  w_empty_vec(c); w_empty_vec(c); w_empty_conv1d(c);
  size_t n = (size_t)OQ_DEC_ROPE_POS * (OQ_DEC_HEAD_DIM / 2);
  float* cs = (float*)malloc(n * 4); float* sn = (float*)malloc(n * 4);
  oq_build_rope_tables(OQ_DEC_HEAD_DIM, OQ_DEC_ROPE_POS, 10000.0, cs, sn);
  w_f32vec(c, cs, n); w_f32vec(c, sn, n);
  free(cs); free(sn);
}

int oq_synth_write(const char* path, const oq_dims* d, uint64_t seed) { return oq_synth_write_ex(path, d, seed, 0); }

int oq_synth_write_ex(const char* path, const oq_dims* d, uint64_t seed, unsigned flags) {
  wctx c = {fopen(path, "wb"), seed, 0, 0};
  if (!c.f) return -1;
  setvbuf(c.f, NULL, _IOFBF, 1 << 23);
  const int fmt = d->fmt;
  w_bytes(&c, "QTTS", 4); w_u32(&c, 1); w_u8(&c, (uint8_t)fmt); /* save.rs:31-35 */
  /* save_talker (save.rs:48-89) */
  int tq = d->t_heads * d->t_head_dim, tkv = d->t_kv_heads * d->t_head_dim;
  w_u32(&c, d->t_layers); w_u32(&c, d->t_hidden); w_u32(&c, d->t_text_hidden);
  w_u32(&c, d->t_heads); w_u32(&c, d->t_kv_heads); w_u32(&c, d->t_head_dim);
  w_u32(&c, d->t_heads / d->t_kv_heads); w_u32(&c, 3);
  for (int i = 0; i < 3; i++) w_u32(&c, d->t_sec[i]);
  for (int l = 0; l < d->t_layers; l++) {
    w_weight(&c, fmt, d->t_hidden, tq); w_weight(&c, fmt, d->t_hidden, tkv);
    w_weight(&c, fmt, d->t_hidden, tkv); w_weight(&c, fmt, tq, d->t_hidden);
    w_norm(&c, d->t_head_dim); w_norm(&c, d->t_head_dim);
    w_weight(&c, fmt, d->t_hidden, d->t_inter); w_weight(&c, fmt, d->t_hidden, d->t_inter);
    w_weight(&c, fmt, d->t_inter, d->t_hidden);
    w_norm(&c, d->t_hidden); w_norm(&c, d->t_hidden);
  }
  w_weight(&c, fmt, d->t_vocab, d->t_hidden);                 /* codec_embedding */
  w_weight(&c, fmt, d->t_text_vocab, d->t_text_hidden);       /* text_embedding */
  w_weight(&c, fmt, d->t_text_hidden, d->t_text_hidden);      /* text_proj_fc1 */
  w_bias(&c, d->t_text_hidden);
  w_weight(&c, fmt, d->t_text_hidden, d->t_hidden);           /* text_proj_fc2 */
  w_bias(&c, d->t_hidden);
  w_weight(&c, fmt, d->t_hidden, d->t_vocab);                 /* codec_head */
  w_norm(&c, d->t_hidden);                                    /* final_norm */
  {
    size_t n = (size_t)d->t_max_pos * (d->t_head_dim / 2);
    float* cs = (float*)malloc(n * 4); float* sn = (float*)malloc(n * 4);
    oq_build_mrope_tables(d->t_head_dim, d->t_max_pos, 1000000.0, d->t_sec, 3, cs, sn);
    w_f32vec(&c, cs, n); w_f32vec(&c, sn, n);
    free(cs); free(sn);
  }
  /* save_predictor (save.rs:91-137) */
  int pq = d->p_heads * d->p_head_dim, pkv = d->p_kv_heads * d->p_head_dim;
  w_u32(&c, d->p_layers); w_u32(&c, d->p_hidden); w_u32(&c, d->p_heads);
  w_u32(&c, d->p_kv_heads); w_u32(&c, d->p_head_dim); w_u32(&c, d->p_heads / d->p_kv_heads);
  if (d->p_hidden != d->t_hidden) {
    w_u8(&c, 1);
    w_weight(&c, fmt, d->t_hidden, d->p_hidden);
    w_bias(&c, d->p_hidden);
  } else {
    w_u8(&c, 0);
  }
  w_u32(&c, d->p_groups);
  for (int g = 0; g < d->p_groups; g++) w_weight(&c, fmt, d->p_vocab, d->t_hidden);
  for (int l = 0; l < d->p_layers; l++) {
    w_weight(&c, fmt, d->p_hidden, pq); w_weight(&c, fmt, d->p_hidden, pkv);
    w_weight(&c, fmt, d->p_hidden, pkv); w_weight(&c, fmt, pq, d->p_hidden);
    w_norm(&c, d->p_head_dim); w_norm(&c, d->p_head_dim);
    w_weight(&c, fmt, d->p_hidden, d->p_inter); w_weight(&c, fmt, d->p_hidden, d->p_inter);
    w_weight(&c, fmt, d->p_inter, d->p_hidden);
    w_norm(&c, d->p_hidden); w_norm(&c, d->p_hidden);
  }
  w_u32(&c, d->p_groups);
  for (int g = 0; g < d->p_groups; g++) {
    if (fmt == 1 && g_tie_period > 0 && g_tie_period <= 64) w_q4_tied(&c, d->p_hidden, d->p_vocab, g_tie_period);
    else w_weight(&c, fmt, d->p_hidden, d->p_vocab);
  }
  w_norm(&c, d->p_hidden);
  {
    size_t n = (size_t)d->p_max_pos * (d->p_head_dim / 2);
    float* cs = (float*)malloc(n * 4); float* sn = (float*)malloc(n * 4);
    oq_build_rope_tables(d->p_head_dim, d->p_max_pos, 1000000.0, cs, sn);
    w_f32vec(&c, cs, n); w_f32vec(&c, sn, n);
    free(cs); free(sn);
  }
  if (flags & OQ_SYNTH_DECODER) {
    w_decoder(&c);
  } else {
    /* An empty speech-decoder section in the save.rs:171-256 layout, so that
     * save::load_model parses the file. */
    for (int i = 0; i < 6; i++) w_u32(&c, 0);
    w_empty_vec(&c); w_empty_vec(&c); w_u32(&c, 0); w_empty_vec(&c);
    w_empty_conv1d(&c);
    w_empty_vec(&c); w_empty_vec(&c); w_u32(&c, 0);
    w_empty_vec(&c); w_empty_vec(&c); w_empty_vec(&c);
    w_u32(&c, 0);
    w_empty_conv1d(&c); w_u32(&c, 0);
    w_empty_vec(&c); w_empty_vec(&c); w_empty_conv1d(&c);
    w_empty_vec(&c); w_empty_vec(&c);
  }
  int err = c.err;
  if (fclose(c.f) != 0) err = 1;
  return err ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* loader (save.rs:262-409; gemv.rs:596-650)                                */
/* ------------------------------------------------------------------------ */

typedef struct { FILE* f; int err; char* msg; int msglen; } rctx;
static void r_fail(rctx* r, const char* what) {
  if (!r->err && r->msg) snprintf(r->msg, r->msglen, "%s", what);
  r->err = 1;
}
static void r_bytes(rctx* r, void* p, size_t n) {
  if (r->err) { memset(p, 0, n); return; }
  if (fread(p, 1, n, r->f) != n) { r_fail(r, "unexpected end of file"); memset(p, 0, n); }
}
static uint32_t r_u32(rctx* r) { uint32_t v; r_bytes(r, &v, 4); return v; }
static uint64_t r_u64(rctx* r) { uint64_t v; r_bytes(r, &v, 8); return v; }
static void* r_vec(rctx* r, size_t elem, uint64_t* len_out) {
  uint64_t len = r_u64(r);
  if (r->err) { *len_out = 0; return NULL; }
  if (len > (1ull << 36) / elem) { r_fail(r, "vector length out of range"); *len_out = 0; return NULL; }
  void* p = malloc(len * elem + 16);
  if (!p) { r_fail(r, "out of memory"); *len_out = 0; return NULL; }
  r_bytes(r, p, len * elem);
  *len_out = len;
  return p;
}
static ow r_weight(rctx* r, int fmt) { /* read_weight_io gemv.rs:635-650 */
  ow w;
  memset(&w, 0, sizeof(w));
  w.fmt = fmt;
  w.k = r_u64(r); w.n = r_u64(r);
  uint64_t l1, l2;
  if (fmt == 1) {
    w.packed = (uint8_t*)r_vec(r, 1, &l1);
    w.scales = (uint16_t*)r_vec(r, 2, &l2);
    if (!r->err && (l1 != w.k * w.n / 2 || l2 != w.k * w.n / 32 || w.n % 32))
      r_fail(r, "Q4 weight length mismatch");
  } else if (fmt == 0) {
    w.data = (uint16_t*)r_vec(r, 2, &l1);
    if (!r->err && l1 != w.k * w.n) r_fail(r, "F16 weight length mismatch");
  } else {
    r_fail(r, "Unknown format");
  }
  return w;
}
static void free_w(ow* w) { free(w->packed); free(w->scales); free(w->data); }
static uint16_t* r_f16(rctx* r, uint64_t expect) {
  uint64_t l;
  uint16_t* p = (uint16_t*)r_vec(r, 2, &l);
  if (!r->err && l != expect) r_fail(r, "f16 vector length mismatch");
  return p;
}
static float* r_f32(rctx* r, uint64_t* len) { return (float*)r_vec(r, 4, len); }

static void read_layer(rctx* r, int fmt, ol* L, int hd, int hidden) {
  L->q = r_weight(r, fmt); L->k = r_weight(r, fmt); L->v = r_weight(r, fmt); L->o = r_weight(r, fmt);
  L->q_norm = r_f16(r, hd); L->k_norm = r_f16(r, hd);
  L->gate = r_weight(r, fmt); L->up = r_weight(r, fmt); L->down = r_weight(r, fmt);
  L->in_norm = r_f16(r, hidden); L->post_norm = r_f16(r, hidden);
}
static void free_layer(ol* L) {
  free_w(&L->q); free_w(&L->k); free_w(&L->v); free_w(&L->o);
  free_w(&L->gate); free_w(&L->up); free_w(&L->down);
  free(L->q_norm); free(L->k_norm); free(L->in_norm); free(L->post_norm);
}

/* the talker and predictor sections; the stream is left at the decoder section */
static oq_model* load_lm(rctx* r) {
  oq_model* m = (oq_model*)calloc(1, sizeof(oq_model));
  char magic[4];
  r_bytes(r, magic, 4);
  if (!r->err && memcmp(magic, "QTTS", 4) != 0) r_fail(r, "Invalid magic (expected QTTS)");
  uint32_t ver = r_u32(r);
  if (!r->err && ver != 1) r_fail(r, "unsupported version");
  uint8_t fmt = 0;
  r_bytes(r, &fmt, 1);
  oq_dims* d = &m->d;
  d->fmt = fmt;
  /* load_talker save.rs:300-351 */
  d->t_layers = r_u32(r); d->t_hidden = r_u32(r); d->t_text_hidden = r_u32(r);
  d->t_heads = r_u32(r); d->t_kv_heads = r_u32(r); d->t_head_dim = r_u32(r);
  m->t_kv_groups = r_u32(r);
  m->t_nsec = r_u32(r);
  if (!r->err && (m->t_nsec > 3 || d->t_layers > 4096 || d->t_layers == 0))
    r_fail(r, "bad talker header");
  for (int i = 0; i < m->t_nsec && !r->err; i++) d->t_sec[i] = r_u32(r);
  if (!r->err) {
    m->tl = (ol*)calloc(d->t_layers, sizeof(ol));
    for (int l = 0; l < d->t_layers && !r->err; l++)
      read_layer(r, fmt, &m->tl[l], d->t_head_dim, d->t_hidden);
  }
  m->codec_emb = r_weight(r, fmt);
  m->text_emb = r_weight(r, fmt);
  m->fc1 = r_weight(r, fmt);
  uint64_t l;
  m->fc1_b = r_f32(r, &l);
  m->fc2 = r_weight(r, fmt);
  m->fc2_b = r_f32(r, &l);
  m->codec_head = r_weight(r, fmt);
  m->t_final_norm = r_f16(r, d->t_hidden);
  m->t_cos = r_f32(r, &m->t_rope_len);
  m->t_sin = r_f32(r, &l);
  if (!r->err) {
    d->t_inter = m->tl[0].gate.n; d->t_vocab = m->codec_head.n;
    d->t_text_vocab = m->text_emb.k;
    d->t_max_pos = (int)(m->t_rope_len / (d->t_head_dim / 2));
  }
  /* load_predictor save.rs:353-409 */
  d->p_layers = r_u32(r); d->p_hidden = r_u32(r); d->p_heads = r_u32(r);
  d->p_kv_heads = r_u32(r); d->p_head_dim = r_u32(r); m->p_kv_groups = r_u32(r);
  uint8_t hp = 0;
  r_bytes(r, &hp, 1);
  m->has_proj = hp == 1;
  if (m->has_proj) { m->input_proj = r_weight(r, fmt); m->input_proj_b = r_f32(r, &l); }
  m->n_emb = r_u32(r);
  if (!r->err && (m->n_emb > 64 || d->p_layers > 4096 || d->p_layers == 0)) r_fail(r, "bad predictor header");
  if (!r->err) {
    m->p_emb = (ow*)calloc(m->n_emb, sizeof(ow));
    for (int g = 0; g < m->n_emb; g++) m->p_emb[g] = r_weight(r, fmt);
    m->pl = (ol*)calloc(d->p_layers, sizeof(ol));
    for (int i = 0; i < d->p_layers && !r->err; i++) read_layer(r, fmt, &m->pl[i], d->p_head_dim, d->p_hidden);
    m->n_lm = r_u32(r);
    if (!r->err && m->n_lm > 64) r_fail(r, "bad lm_head count");
    if (!r->err) {
      m->lm = (ow*)calloc(m->n_lm, sizeof(ow));
      for (int g = 0; g < m->n_lm; g++) m->lm[g] = r_weight(r, fmt);
    }
    m->p_final_norm = r_f16(r, d->p_hidden);
    m->p_cos = r_f32(r, &m->p_rope_len);
    m->p_sin = r_f32(r, &l);
  }
  if (r->err) { oq_free(m); return NULL; }
  d->p_inter = m->pl[0].gate.n; d->p_vocab = m->lm[0].n; d->p_groups = m->n_lm;
  d->p_max_pos = (int)(m->p_rope_len / (d->p_head_dim / 2));
  return m;
}


oq_model* oq_load(const char* path, char* err, int errlen) {
  rctx r = {fopen(path, "rb"), 0, err, errlen};
  if (!r.f) { if (err) snprintf(err, errlen, "cannot open %s", path); return NULL; }
  setvbuf(r.f, NULL, _IOFBF, 1 << 23);
  oq_model* m = load_lm(&r);
  fclose(r.f);
  return m;
}

void oq_free(oq_model* m) {
  if (!m) return;
  if (m->tl) for (int l = 0; l < m->d.t_layers; l++) free_layer(&m->tl[l]);
  free(m->tl);
  free_w(&m->codec_emb); free_w(&m->text_emb); free_w(&m->fc1); free_w(&m->fc2); free_w(&m->codec_head);
  free(m->fc1_b); free(m->fc2_b); free(m->t_final_norm); free(m->t_cos); free(m->t_sin);
  if (m->has_proj) { free_w(&m->input_proj); free(m->input_proj_b); }
  if (m->p_emb) for (int g = 0; g < m->n_emb; g++) free_w(&m->p_emb[g]);
  free(m->p_emb);
  if (m->pl) for (int l = 0; l < m->d.p_layers; l++) free_layer(&m->pl[l]);
  free(m->pl);
  if (m->lm) for (int g = 0; g < m->n_lm; g++) free_w(&m->lm[g]);
  free(m->lm);
  free(m->p_final_norm); free(m->p_cos); free(m->p_sin);
  free(m);
}

void oq_get_dims(const oq_model* m, oq_dims* d) { *d = m->d; }

/* ------------------------------------------------------------------------ */
/* KV cache (gemv.rs:77-86): per layer f32 [seq, kv_heads, head_dim]         */
/* ------------------------------------------------------------------------ */

struct oq_kv { int layers, stride; int* len; int* cap; float** k; float** v; };

oq_kv* oq_kv_new(int layers, int kv_heads, int head_dim) {
  oq_kv* kv = (oq_kv*)calloc(1, sizeof(oq_kv));
  kv->layers = layers; kv->stride = kv_heads * head_dim;
  kv->len = (int*)calloc(layers, sizeof(int)); kv->cap = (int*)calloc(layers, sizeof(int));
  kv->k = (float**)calloc(layers, sizeof(float*)); kv->v = (float**)calloc(layers, sizeof(float*));
  return kv;
}
void oq_kv_free(oq_kv* kv) {
  if (!kv) return;
  for (int l = 0; l < kv->layers; l++) { free(kv->k[l]); free(kv->v[l]); }
  free(kv->k); free(kv->v); free(kv->len); free(kv->cap); free(kv);
}
void oq_kv_clear(oq_kv* kv) { for (int l = 0; l < kv->layers; l++) kv->len[l] = 0; }
int oq_kv_len(const oq_kv* kv, int layer) { return kv->len[layer]; }
static void kv_append(oq_kv* kv, int l, const float* k, const float* v, int n) {
  if (kv->len[l] + n > kv->cap[l]) {
    int nc = kv->cap[l] ? kv->cap[l] : 512;
    while (nc < kv->len[l] + n) nc *= 2;
    kv->k[l] = (float*)realloc(kv->k[l], sizeof(float) * (size_t)nc * kv->stride);
    kv->v[l] = (float*)realloc(kv->v[l], sizeof(float) * (size_t)nc * kv->stride);
    kv->cap[l] = nc;
  }
  memcpy(kv->k[l] + (size_t)kv->len[l] * kv->stride, k, sizeof(float) * (size_t)n * kv->stride);
  memcpy(kv->v[l] + (size_t)kv->len[l] * kv->stride, v, sizeof(float) * (size_t)n * kv->stride);
  kv->len[l] += n;
}
oq_kv* oq_talker_kv_new(const oq_model* m) { return oq_kv_new(m->d.t_layers, m->d.t_kv_heads, m->d.t_head_dim); }
oq_kv* oq_predictor_kv_new(const oq_model* m) { return oq_kv_new(m->d.p_layers, m->d.p_kv_heads, m->d.p_head_dim); }

/* ------------------------------------------------------------------------ */
/* shared layer pieces                                                       */
/* ------------------------------------------------------------------------ */

/* talker.rs:89-99 / code_predictor.rs:84-93 apply_qk_norm */
static void qk_norm(float* x, int heads, int hd, const uint16_t* g) {
  for (int h = 0; h < heads; h++) {
    float* s = x + h * hd;
    float ss = 0.0f;
    for (int d = 0; d < hd; d++) ss += s[d] * s[d];
    float inv = 1.0f / sqrtf(ss / (float)hd + 1e-6f);
    for (int d = 0; d < hd; d++) s[d] = s[d] * inv * oq_h2f(g[d]);
  }
}

/* rope.rs:51-93 apply_mrope_interleaved with position_ids = [p,p,p]: the
 * per-section gather collapses to row p of the table (sections tile 0..half);
 * the rotation is split-half (:79-92).  Returns -1 where the Rust indexing
 * would panic (p beyond the table). */
static int mrope(float* x, int heads, int hd, int p, const oq_model* m) {
  int half = hd / 2;
  if ((uint64_t)(p + 1) * half > m->t_rope_len) return -1;
  const float* c = m->t_cos + (size_t)p * half;
  const float* s = m->t_sin + (size_t)p * half;
  for (int h = 0; h < heads; h++) {
    float* b = x + h * hd;
    for (int i = 0; i < half; i++) {
      float x1 = b[i], x2 = b[half + i];
      b[i] = x1 * c[i] - x2 * s[i];
      b[half + i] = x2 * c[i] + x1 * s[i];
    }
  }
  return 0;
}

/* code_predictor.rs:97-121 apply_rope_split (silently skips positions past
 * the table, :107) */
static void rope_split(float* x, int heads, int hd, int p, const oq_model* m) {
  int half = hd / 2;
  uint64_t off = (uint64_t)p * half;
  if (off + half > m->p_rope_len) return;
  const float* c = m->p_cos + off;
  const float* s = m->p_sin + off;
  for (int h = 0; h < heads; h++) {
    float* b = x + h * hd;
    for (int i = 0; i < half; i++) {
      float x1 = b[i], x2 = b[half + i];
      b[i] = x1 * c[i] - x2 * s[i];
      b[half + i] = x2 * c[i] + x1 * s[i];
    }
  }
}

/* GQA attention of one query row against cache rows [0, len) --
 * talker.rs:305-331 (decode) / :415-437 (prefill, len = t1+1). */
static void attend(const float* q, const float* K, const float* V, int len, int heads,
                   int kv_heads, int hd, float* out) {
  int groups = heads / kv_heads, stride = kv_heads * hd;
  float scale = 1.0f / sqrtf((float)hd);
  float* sc = (float*)malloc(sizeof(float) * (len > 0 ? len : 1));
  for (int i = 0; i < heads * hd; i++) out[i] = 0.0f;
  for (int h = 0; h < heads; h++) {
    int kh = h / groups;
    const float* qv = q + h * hd;
    for (int s = 0; s < len; s++) {
      const float* kr = K + (size_t)s * stride + kh * hd;
      float dot = 0.0f;
      for (int d = 0; d < hd; d++) dot += qv[d] * kr[d];
      sc[s] = dot * scale;
    }
    oq_softmax_raw(sc, len);
    float* o = out + h * hd;
    for (int s = 0; s < len; s++) {
      const float* vr = V + (size_t)s * stride + kh * hd;
      float p = sc[s];
      for (int d = 0; d < hd; d++) o[d] += p * vr[d];
    }
  }
  free(sc);
}

/* ------------------------------------------------------------------------ */
/* talker (talker.rs)                                                        */
/* ------------------------------------------------------------------------ */

/* talker.rs:105-116 embed_text_token */
void oq_embed_text_token(const oq_model* m, uint32_t tok, float* out) {
  const oq_dims* d = &m->d;
  float* raw = (float*)malloc(sizeof(float) * d->t_text_hidden);
  float* h = (float*)malloc(sizeof(float) * m->fc1.n);
  embed_w(&m->text_emb, tok, d->t_text_hidden, raw);
  gemv_w(&m->fc1, raw, h);
  for (uint64_t j = 0; j < m->fc1.n; j++) h[j] += m->fc1_b[j];
  for (uint64_t j = 0; j < m->fc1.n; j++) h[j] = oq_silu(h[j]);
  gemv_w(&m->fc2, h, out);
  for (uint64_t j = 0; j < m->fc2.n; j++) out[j] += m->fc2_b[j];
  free(raw); free(h);
}

/* talker.rs:152-154 embed_codec_token */
void oq_embed_codec_token(const oq_model* m, uint32_t tok, float* out) {
  embed_w(&m->codec_emb, tok, m->d.t_hidden, out);
}

/* talker.rs:627-629 apply_codec_head */
void oq_apply_codec_head(const oq_model* m, const float* h, float* logits) {
  gemv_w(&m->codec_head, h, logits);
}

/* talker.rs:263-360 forward_with_embedding */
int oq_forward_with_embedding(const oq_model* m, const float* emb, oq_kv* kv, int position,
                              float* out) {
  const oq_dims* d = &m->d;
  const int H = d->t_hidden, hd = d->t_head_dim;
  const int qd = d->t_heads * hd, kd = d->t_kv_heads * hd, I = d->t_inter;
  float* x = (float*)malloc(sizeof(float) * H);
  float* xn = (float*)malloc(sizeof(float) * H);
  float* q = (float*)malloc(sizeof(float) * qd);
  float* kn = (float*)malloc(sizeof(float) * kd);
  float* vn = (float*)malloc(sizeof(float) * kd);
  float* at = (float*)malloc(sizeof(float) * qd);
  float* ao = (float*)malloc(sizeof(float) * H);
  float* g = (float*)malloc(sizeof(float) * I);
  float* u = (float*)malloc(sizeof(float) * I);
  int rc = 0;
  memcpy(x, emb, sizeof(float) * H);
  for (int l = 0; l < d->t_layers; l++) {
    const ol* L = &m->tl[l];
    oq_rms_norm_f16(x, L->in_norm, H, xn);
    gemv_w(&L->q, xn, q); gemv_w(&L->k, xn, kn); gemv_w(&L->v, xn, vn);
    qk_norm(q, d->t_heads, hd, L->q_norm);
    qk_norm(kn, d->t_kv_heads, hd, L->k_norm);
    if (mrope(q, d->t_heads, hd, position, m) || mrope(kn, d->t_kv_heads, hd, position, m)) { rc = -1; break; }
    kv_append(kv, l, kn, vn, 1);
    attend(q, kv->k[l], kv->v[l], kv->len[l], d->t_heads, d->t_kv_heads, hd, at);
    gemv_w(&L->o, at, ao);
    for (int j = 0; j < H; j++) x[j] += ao[j];
    oq_rms_norm_f16(x, L->post_norm, H, xn);
    gemv_w(&L->gate, xn, g); gemv_w(&L->up, xn, u);
    for (int j = 0; j < I; j++) g[j] = oq_silu(g[j]) * u[j];
    gemv_w(&L->down, g, ao);
    for (int j = 0; j < H; j++) x[j] += ao[j];
  }
  if (rc == 0) {
    oq_rms_norm_f16(x, m->t_final_norm, H, out);
    gemv_w(&m->codec_head, out, out + H);
  }
  free(x); free(xn); free(q); free(kn); free(vn); free(at); free(ao); free(g); free(u);
  return rc;
}

/* Shared body of talker.rs:364-462 prefill_talker_raw and
 * code_predictor.rs:338-431 prefill_code_predictor (same recipe; the talker
 * uses mrope at positions 0..seq-1, the predictor split rope at t). */
static int prefill_layers(const oq_model* m, int is_talker, const float* x_in, int seq, oq_kv* kv,
                          float* last_hidden) {
  const oq_dims* d = &m->d;
  const int H = is_talker ? d->t_hidden : d->p_hidden;
  const int heads = is_talker ? d->t_heads : d->p_heads;
  const int kvh = is_talker ? d->t_kv_heads : d->p_kv_heads;
  const int hd = is_talker ? d->t_head_dim : d->p_head_dim;
  const int nl = is_talker ? d->t_layers : d->p_layers;
  const int I = is_talker ? d->t_inter : d->p_inter;
  const int qd = heads * hd, kd = kvh * hd;
  const size_t S = (size_t)seq;
  float* x = (float*)malloc(sizeof(float) * S * H);
  float* xn = (float*)malloc(sizeof(float) * S * H);
  float* q = (float*)malloc(sizeof(float) * S * qd);
  float* k = (float*)malloc(sizeof(float) * S * kd);
  float* v = (float*)malloc(sizeof(float) * S * kd);
  float* at = (float*)malloc(sizeof(float) * S * qd);
  float* ao = (float*)malloc(sizeof(float) * S * H);
  float* g = (float*)malloc(sizeof(float) * S * I);
  float* u = (float*)malloc(sizeof(float) * S * I);
  int rc = 0;
  memcpy(x, x_in, sizeof(float) * S * H);
  for (int l = 0; l < nl && rc == 0; l++) {
    const ol* L = is_talker ? &m->tl[l] : &m->pl[l];
    for (int t = 0; t < seq; t++) oq_rms_norm_f16(x + t * H, L->in_norm, H, xn + t * H);
    gemm_w(&L->q, xn, S, q); gemm_w(&L->k, xn, S, k); gemm_w(&L->v, xn, S, v);
    for (int t = 0; t < seq; t++) {
      qk_norm(q + (size_t)t * qd, heads, hd, L->q_norm);
      qk_norm(k + (size_t)t * kd, kvh, hd, L->k_norm);
      if (!is_talker) {
        rope_split(q + (size_t)t * qd, heads, hd, t, m);
        rope_split(k + (size_t)t * kd, kvh, hd, t, m);
      }
    }
    if (is_talker) {
      for (int t = 0; t < seq && rc == 0; t++)
        if (mrope(q + (size_t)t * qd, heads, hd, t, m) || mrope(k + (size_t)t * kd, kvh, hd, t, m)) rc = -1;
      if (rc) break;
    }
    int base = kv->len[l];
    kv_append(kv, l, k, v, seq);
    for (int t1 = 0; t1 < seq; t1++) {
      /* cache rows [0, base + t1] -- base is 0 on the reference's path */
      attend(q + (size_t)t1 * qd, kv->k[l], kv->v[l], base + t1 + 1, heads, kvh, hd, at + (size_t)t1 * qd);
    }
    kv->len[l] = base + seq;
    gemm_w(&L->o, at, S, ao);
    for (size_t j = 0; j < S * H; j++) x[j] += ao[j];
    for (int t = 0; t < seq; t++) oq_rms_norm_f16(x + t * H, L->post_norm, H, xn + t * H);
    gemm_w(&L->gate, xn, S, g); gemm_w(&L->up, xn, S, u);
    for (size_t j = 0; j < S * I; j++) g[j] = oq_silu(g[j]) * u[j];
    gemm_w(&L->down, g, S, ao);
    for (size_t j = 0; j < S * H; j++) x[j] += ao[j];
  }
  if (rc == 0)
    oq_rms_norm_f16(x + (size_t)(seq - 1) * H, is_talker ? m->t_final_norm : m->p_final_norm, H, last_hidden);
  free(x); free(xn); free(q); free(k); free(v); free(at); free(ao); free(g); free(u);
  return rc;
}

int oq_prefill_talker_raw(const oq_model* m, const float* x, int seq, oq_kv* kv, float* last_hidden) {
  return prefill_layers(m, 1, x, seq, kv, last_hidden);
}

/* ------------------------------------------------------------------------ */
/* code predictor (code_predictor.rs)                                        */
/* ------------------------------------------------------------------------ */

/* code_predictor.rs:51-61 project_input */
static void project_input(const oq_model* m, const float* in, float* out) {
  if (m->has_proj) {
    gemv_w(&m->input_proj, in, out);
    for (int j = 0; j < m->d.p_hidden; j++) out[j] += m->input_proj_b[j];
  } else {
    memcpy(out, in, sizeof(float) * m->d.p_hidden);
  }
}

/* code_predictor.rs:328-334 sample_argmax: Iterator::max_by keeps the LAST of
 * equal maxima. */
uint32_t oq_sample_argmax(const float* logits, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  for (size_t i = 1; i < n; i++)
    if (!(logits[i] < logits[best])) best = i; /* i wins on >= */
  return (uint32_t)best;
}

/* code_predictor.rs:434-506 decode_one_code_predictor_token */
static void decode_one(const oq_model* m, const float* emb, oq_kv* kv, float* out) {
  const oq_dims* d = &m->d;
  const int H = d->p_hidden, hd = d->p_head_dim, qd = d->p_heads * hd, kd = d->p_kv_heads * hd;
  const int I = d->p_inter;
  float* x = (float*)malloc(sizeof(float) * H);
  float* xn = (float*)malloc(sizeof(float) * H);
  float* q = (float*)malloc(sizeof(float) * qd);
  float* kn = (float*)malloc(sizeof(float) * kd);
  float* vn = (float*)malloc(sizeof(float) * kd);
  float* at = (float*)malloc(sizeof(float) * qd);
  float* ao = (float*)malloc(sizeof(float) * H);
  float* g = (float*)malloc(sizeof(float) * I);
  float* u = (float*)malloc(sizeof(float) * I);
  memcpy(x, emb, sizeof(float) * H);
  for (int l = 0; l < d->p_layers; l++) {
    const ol* L = &m->pl[l];
    int off = kv->len[l];
    oq_rms_norm_f16(x, L->in_norm, H, xn);
    gemv_w(&L->q, xn, q); gemv_w(&L->k, xn, kn); gemv_w(&L->v, xn, vn);
    qk_norm(q, d->p_heads, hd, L->q_norm);
    qk_norm(kn, d->p_kv_heads, hd, L->k_norm);
    rope_split(q, d->p_heads, hd, off, m);
    rope_split(kn, d->p_kv_heads, hd, off, m);
    kv_append(kv, l, kn, vn, 1);
    attend(q, kv->k[l], kv->v[l], kv->len[l], d->p_heads, d->p_kv_heads, hd, at);
    gemv_w(&L->o, at, ao);
    for (int j = 0; j < H; j++) x[j] += ao[j];
    oq_rms_norm_f16(x, L->post_norm, H, xn);
    gemv_w(&L->gate, xn, g); gemv_w(&L->up, xn, u);
    for (int j = 0; j < I; j++) g[j] = oq_silu(g[j]) * u[j];
    gemv_w(&L->down, g, ao);
    for (int j = 0; j < H; j++) x[j] += ao[j];
  }
  oq_rms_norm_f16(x, m->p_final_norm, H, out);
  free(x); free(xn); free(q); free(kn); free(vn); free(at); free(ao); free(g); free(u);
}

/* code_predictor.rs:218-273 generate_acoustic_codes */
void oq_generate_acoustic_codes(const oq_model* m, const float* talker_hidden,
                                const float* semantic_embed, oq_kv* pkv, uint32_t* codes) {
  const int H = m->d.p_hidden, V = m->d.p_vocab, E = m->d.t_hidden;
  oq_kv_clear(pkv); /* :227-231 */
  float* in2 = (float*)malloc(sizeof(float) * 2 * H);
  float* h = (float*)malloc(sizeof(float) * H);
  float* lg = (float*)malloc(sizeof(float) * V);
  float* emb = (float*)malloc(sizeof(float) * E);
  float* pe = (float*)malloc(sizeof(float) * H);
  project_input(m, talker_hidden, in2);       /* :235 */
  project_input(m, semantic_embed, in2 + H);  /* :236 */
  prefill_layers(m, 0, in2, 2, pkv, h);       /* :244 */
  gemv_w(&m->lm[0], h, lg);                   /* :247 */
  codes[0] = oq_sample_argmax(lg, V);
  for (int g = 1; g < m->n_lm; g++) {         /* :253-270 */
    embed_w(&m->p_emb[g - 1], codes[g - 1], m->p_emb[g - 1].n, emb);
    project_input(m, emb, pe);
    decode_one(m, pe, pkv, h);
    gemv_w(&m->lm[g], h, lg);
    codes[g] = oq_sample_argmax(lg, V);
  }
  free(in2); free(h); free(lg); free(emb); free(pe);
}

/* code_predictor.rs:280-293 get_acoustic_embeddings_sum */
void oq_acoustic_embed_sum(const oq_model* m, const uint32_t* codes, float* out) {
  const int E = (int)m->p_emb[0].n;
  float* e = (float*)malloc(sizeof(float) * E);
  for (int j = 0; j < E; j++) out[j] = 0.0f;
  for (int g = 0; g < m->n_lm; g++) {
    embed_w(&m->p_emb[g], codes[g], E, e);
    for (int j = 0; j < E; j++) out[j] += e[j];
  }
  free(e);
}

/* ------------------------------------------------------------------------ */
/* generation (generate_new.rs)                                              */
/* ------------------------------------------------------------------------ */

enum {
  IM_START = 151644, ASSISTANT = 77091, NEWLINE = 198, TTS_PAD = 151671, TTS_BOS = 151672,
  TTS_EOS = 151673, CODEC_THINK = 2154, CODEC_THINK_BOS = 2156, CODEC_THINK_EOS = 2157,
  CODEC_PAD = 2148, CODEC_BOS = 2149
};

/* generate_new.rs:16-22 simple_rand (xorshift64) */
float oq_simple_rand(uint64_t* st) {
  *st ^= *st << 13;
  *st ^= *st >> 7;
  *st ^= *st << 17;
  return (float)(*st) / (float)UINT64_MAX;
}

typedef struct { size_t i; float p; } ip_t;
/* stable merge sort by p descending (slice::sort_by is stable) */
static void msort(ip_t* a, ip_t* tmp, size_t n) {
  if (n < 2) return;
  size_t h = n / 2;
  msort(a, tmp, h);
  msort(a + h, tmp, n - h);
  size_t i = 0, j = h, k = 0;
  while (i < h && j < n) {
    if (a[j].p > a[i].p) tmp[k++] = a[j++]; /* b.1.partial_cmp(&a.1): take right only if strictly greater */
    else tmp[k++] = a[i++];
  }
  while (i < h) tmp[k++] = a[i++];
  while (j < n) tmp[k++] = a[j++];
  memcpy(a, tmp, sizeof(ip_t) * n);
}

/* generate_new.rs:329-391 sample_token */
uint32_t oq_sample_token(const float* logits, size_t n, const oq_params* p, const uint32_t* prev,
                         uint64_t* rng) {
  float* s = (float*)malloc(sizeof(float) * n);
  memcpy(s, logits, sizeof(float) * n);
  if (p->repetition_penalty != 1.0f) {          /* :333-343 */
    for (int i = 0; i < 16; i++) {
      uint32_t t = prev[i];
      if ((size_t)t < n) {
        if (s[t] > 0.0f) s[t] /= p->repetition_penalty;
        else s[t] *= p->repetition_penalty;
      }
    }
  }
  if (p->temperature != 1.0f)                    /* :346-350 */
    for (size_t i = 0; i < n; i++) s[i] /= p->temperature;
  float mx = -INFINITY;                          /* :353-360 */
  for (size_t i = 0; i < n; i++) mx = fmaxf(mx, s[i]);
  for (size_t i = 0; i < n; i++) s[i] = expf(s[i] - mx);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) sum += s[i];
  for (size_t i = 0; i < n; i++) s[i] /= sum;
  if (p->top_k > 0 && (size_t)p->top_k < n) {   /* :363-378 */
    ip_t* a = (ip_t*)malloc(sizeof(ip_t) * n);
    ip_t* tmp = (ip_t*)malloc(sizeof(ip_t) * n);
    for (size_t i = 0; i < n; i++) a[i] = (ip_t){i, s[i]};
    msort(a, tmp, n);
    for (size_t r = (size_t)p->top_k; r < n; r++) s[a[r].i] = 0.0f;
    float s2 = 0.0f;
    for (size_t i = 0; i < n; i++) s2 += s[i];
    if (s2 > 0.0f)
      for (size_t i = 0; i < n; i++) s[i] /= s2;
    free(a); free(tmp);
  }
  float r = oq_simple_rand(rng);                 /* :381-390 */
  float cum = 0.0f;
  uint32_t out = 0;
  for (size_t i = 0; i < n; i++) {
    cum += s[i];
    if (r < cum) { out = (uint32_t)i; break; }
  }
  free(s);
  return out;
}

/* generate_new.rs:84-188 prefill_custom_voice.  full_prompt (a benchmark
 * mode of this build, not of the reference): the remaining text tokens
 * 1..n_text-1 follow as prefill rows embed_text(tok) + embed_codec(CODEC_PAD),
 * so prompts of different lengths leave caches of different lengths; the
 * frame loop's trailing text then holds TTS_EOS only. */
static int prefill_rows(const oq_model* m, const uint32_t* text, int n_text, uint32_t speaker_id,
                        uint32_t language_id, const float* voice, int full_prompt, oq_kv* kv,
                        float* last_hidden, float* logits) {
  const int H = m->d.t_hidden;
  const int extra = (full_prompt && n_text > 1) ? n_text - 1 : 0;
  float* x = (float*)calloc((size_t)(10 + extra) * H, sizeof(float));
  float* a = (float*)malloc(sizeof(float) * H);
  float* b = (float*)malloc(sizeof(float) * H);
  int seq = 0;
  const uint32_t role[3] = {IM_START, ASSISTANT, NEWLINE};
  for (int i = 0; i < 3; i++) oq_embed_text_token(m, role[i], x + (size_t)(seq++) * H);
  if (voice) {
    const uint32_t pc[4] = {CODEC_THINK, CODEC_THINK_BOS, language_id, CODEC_THINK_EOS};
    float* pad = (float*)malloc(sizeof(float) * H);
    float* bos = (float*)malloc(sizeof(float) * H);
    oq_embed_text_token(m, TTS_PAD, pad);
    oq_embed_text_token(m, TTS_BOS, bos);
    for (int i = 0; i < 4; i++) {
      oq_embed_codec_token(m, pc[i], a);
      float* o = x + (size_t)(seq++) * H;
      for (int j = 0; j < H; j++) o[j] = a[j] + pad[j];
    }
    memcpy(x + (size_t)(seq++) * H, voice, sizeof(float) * H);
    oq_embed_codec_token(m, CODEC_PAD, a);
    {
      float* o = x + (size_t)(seq++) * H;
      for (int j = 0; j < H; j++) o[j] = a[j] + bos[j];
    }
    if (n_text > 0) {
      oq_embed_codec_token(m, CODEC_BOS, a);
      oq_embed_text_token(m, text[0], b);
      float* o = x + (size_t)(seq++) * H;
      for (int j = 0; j < H; j++) o[j] = a[j] + b[j];
    }
    free(pad); free(bos);
  } else {
    const uint32_t ct[6] = {CODEC_THINK, CODEC_THINK_BOS, language_id, CODEC_THINK_EOS, speaker_id, CODEC_PAD};
    float* pad = (float*)malloc(sizeof(float) * H);
    float* bos = (float*)malloc(sizeof(float) * H);
    oq_embed_text_token(m, TTS_PAD, pad);
    oq_embed_text_token(m, TTS_BOS, bos);
    for (int i = 0; i < 6; i++) {
      oq_embed_codec_token(m, ct[i], a);
      const float* ov = i < 5 ? pad : bos;
      float* o = x + (size_t)(seq++) * H;
      for (int j = 0; j < H; j++) o[j] = a[j] + ov[j];
    }
    if (n_text > 0) {
      oq_embed_codec_token(m, CODEC_BOS, a);
      oq_embed_text_token(m, text[0], b);
      float* o = x + (size_t)(seq++) * H;
      for (int j = 0; j < H; j++) o[j] = a[j] + b[j];
    }
    free(pad); free(bos);
  }
  if (extra) {
    oq_embed_codec_token(m, CODEC_PAD, a);
    for (int i = 1; i < n_text; i++) {
      oq_embed_text_token(m, text[i], b);
      float* o = x + (size_t)(seq++) * H;
      for (int j = 0; j < H; j++) o[j] = b[j] + a[j];
    }
  }
  int rc = oq_prefill_talker_raw(m, x, seq, kv, last_hidden);
  if (rc == 0) oq_apply_codec_head(m, last_hidden, logits);
  free(x); free(a); free(b);
  return rc ? rc : seq;
}

int oq_prefill_custom_voice(const oq_model* m, const uint32_t* text, int n_text, uint32_t speaker_id,
                            uint32_t language_id, const float* voice, oq_kv* kv, float* last_hidden,
                            float* logits) {
  return prefill_rows(m, text, n_text, speaker_id, language_id, voice, 0, kv, last_hidden, logits);
}

/* generate_new.rs:191-300 generate_speech (frame loop; audio decode out of
 * scope) with teacher forcing and dumps for parity work.  flags: bit 0
 * ignore EOS (benchmarks), bit 1 full_prompt (see prefill_rows). */
int oq_generate(const oq_model* m, const uint32_t* text, int n_text, uint32_t speaker_id,
                uint32_t language_id, const float* voice, const oq_params* p, uint64_t seed,
                int flags, const uint32_t* forced, uint32_t* codes_out, float* logits_dump,
                float* hidden_dump) {
  const int ignore_eos = flags & 1, full_prompt = (flags >> 1) & 1;
  const int H = m->d.t_hidden, V = m->d.t_vocab, G = m->n_lm;
  oq_kv* tkv = oq_talker_kv_new(m);
  oq_kv* pkv = oq_predictor_kv_new(m);
  float* hidden = (float*)malloc(sizeof(float) * H);
  float* res = (float*)malloc(sizeof(float) * (H + V));
  float* logits = (float*)malloc(sizeof(float) * V);
  float* sem = (float*)malloc(sizeof(float) * H);
  float* acs = (float*)malloc(sizeof(float) * H);
  int rc = prefill_rows(m, text, n_text, speaker_id, language_id, voice, full_prompt, tkv, hidden, logits);
  int frames = 0;
  if (rc < 0) goto done;
  int position = rc;                                              /* :216 (9 or 10 rows) */
  int n_trail = (!full_prompt && n_text > 1 ? n_text - 1 : 0) + 1; /* :314-326 */
  float* trail = (float*)malloc(sizeof(float) * (size_t)n_trail * H);
  for (int i = 1; i < n_trail; i++) oq_embed_text_token(m, text[i], trail + (size_t)(i - 1) * H);
  oq_embed_text_token(m, TTS_EOS, trail + (size_t)(n_trail - 1) * H);
  float* tts_pad = (float*)malloc(sizeof(float) * H);
  oq_embed_text_token(m, TTS_PAD, tts_pad);
  uint32_t prev[16] = {0};
  uint64_t rng = seed;
  uint32_t ac[64];
  for (int f = 0; f < p->max_codes; f++) {                        /* :242 */
    if (logits_dump) memcpy(logits_dump + (size_t)f * V, logits, sizeof(float) * V);
    if (hidden_dump) memcpy(hidden_dump + (size_t)f * H, hidden, sizeof(float) * H);
    uint32_t tok = oq_sample_token(logits, V, p, prev, &rng);
    if (codes_out) codes_out[(size_t)f * 16] = tok;
    if (forced) tok = forced[(size_t)f * 16];
    if (tok == p->codec_eos_id && !ignore_eos) break;
    prev[0] = tok;
    oq_embed_codec_token(m, tok, sem);
    oq_generate_acoustic_codes(m, hidden, sem, pkv, ac);
    for (int g = 0; g < G; g++) {
      if (codes_out) codes_out[(size_t)f * 16 + 1 + g] = ac[g];
      if (forced) ac[g] = forced[(size_t)f * 16 + 1 + g];
      prev[g + 1] = ac[g];
    }
    oq_acoustic_embed_sum(m, ac, acs);
    for (int j = 0; j < H; j++) sem[j] += acs[j];
    const float* ta = f < n_trail ? trail + (size_t)f * H : tts_pad;
    for (int j = 0; j < H; j++) sem[j] += ta[j];
    if (oq_forward_with_embedding(m, sem, tkv, position, res)) { frames = -1; break; }
    memcpy(hidden, res, sizeof(float) * H);
    memcpy(logits, res + H, sizeof(float) * V);
    position++;
    frames = f + 1;
  }
  free(trail); free(tts_pad);
done:
  oq_kv_free(tkv); oq_kv_free(pkv);
  free(hidden); free(res); free(logits); free(sem); free(acs);
  return rc < 0 ? rc : frames;
}

/* CPU-baseline helper: time `frames` full frame steps (sample + predictor +
 * fusion + talker step) on a talker KV pre-filled to kv_len positions with
 * seeded values; returns seconds per frame.  Timing is value-independent. */
double oq_time_frames(const oq_model* m, int kv_len, int frames, uint64_t seed) {
  const oq_dims* d = &m->d;
  const int H = d->t_hidden, V = d->t_vocab, stride = d->t_kv_heads * d->t_head_dim;
  oq_kv* tkv = oq_talker_kv_new(m);
  oq_kv* pkv = oq_predictor_kv_new(m);
  float* fill = (float*)malloc(sizeof(float) * (size_t)kv_len * stride);
  oq_rand_normal(seed, fill, (size_t)kv_len * stride, 1.0f);
  for (int l = 0; l < d->t_layers; l++) kv_append(tkv, l, fill, fill, kv_len);
  free(fill);
  float* hidden = (float*)malloc(sizeof(float) * H);
  float* logits = (float*)malloc(sizeof(float) * V);
  float* res = (float*)malloc(sizeof(float) * (H + V));
  float* sem = (float*)malloc(sizeof(float) * H);
  float* acs = (float*)malloc(sizeof(float) * H);
  oq_rand_normal(seed + 1, hidden, H, 1.0f);
  oq_rand_normal(seed + 2, logits, V, 4.0f);
  oq_params p = {frames, 0.8f, 50, 1.05f, 2150, 2149};
  uint32_t prev[16] = {0}, ac[64];
  uint64_t rng = seed | 1;
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (int f = 0; f < frames; f++) {
    uint32_t tok = oq_sample_token(logits, V, &p, prev, &rng);
    prev[0] = tok;
    oq_embed_codec_token(m, tok, sem);
    oq_generate_acoustic_codes(m, hidden, sem, pkv, ac);
    for (int g = 0; g < m->n_lm; g++) prev[g + 1] = ac[g];
    oq_acoustic_embed_sum(m, ac, acs);
    for (int j = 0; j < H; j++) sem[j] += acs[j];
    oq_forward_with_embedding(m, sem, tkv, kv_len + f, res);
    memcpy(hidden, res, sizeof(float) * H);
    memcpy(logits, res + H, sizeof(float) * V);
  }
  clock_gettime(CLOCK_MONOTONIC, &t1);
  oq_kv_free(tkv); oq_kv_free(pkv);
  free(hidden); free(logits); free(res); free(sem); free(acs);
  return ((t1.tv_sec - t0.tv_sec) + 1e-9 * (t1.tv_nsec - t0.tv_nsec)) / (frames > 0 ? frames : 1);
}

/* ------------------------------------------------------------------------ */
/* speech decoder, codes -> transformer output: decoder.rs:142-335 and the  */
/* conv.rs:114-191 pre-conv (decode_to_audio decoder.rs:394-424, steps 1-3); */
/* reader save.rs:446-552 (the upsample / Vocos stages are read and dropped) */
/* ------------------------------------------------------------------------ */

typedef struct { uint32_t in, out, k, stride, pad, dil; float* w; float* b; uint64_t wl, bl; } oconv;
typedef struct { float *q, *k, *v, *o, *gate, *up, *down, *in_norm, *post_norm, *attn_scale, *mlp_scale; } odl;
struct oq_decoder {
  uint32_t hidden, heads, head_dim, inter, window, cb_dim, entries;
  float* cb0; float* proj0; float* cb_rest[15]; float* proj_rest;
  oconv pre;
  float *in_w, *in_b, *norm, *out_w, *out_b, *rope_cos, *rope_sin;
  uint64_t rope_len;
  int n_layers;
  odl* L;
};

static oconv r_conv1d(rctx* r) { /* save.rs:411-422 */
  oconv c;
  memset(&c, 0, sizeof(c));
  c.in = r_u32(r); c.out = r_u32(r); c.k = r_u32(r); c.stride = r_u32(r); c.pad = r_u32(r); c.dil = r_u32(r);
  c.w = r_f32(r, &c.wl); c.b = r_f32(r, &c.bl);
  return c;
}
static void drop_vec(rctx* r) { uint64_t l; free(r_f32(r, &l)); }
static void drop_conv(rctx* r, int hdr) { for (int i = 0; i < hdr; i++) r_u32(r); drop_vec(r); drop_vec(r); }
static float* r_f32n(rctx* r, uint64_t expect, const char* what) {
  uint64_t l = 0;
  float* v = r_f32(r, &l);
  if (!r->err && l != expect) r_fail(r, what);
  return v;
}

void oq_decoder_free(oq_decoder* d) {
  if (!d) return;
  free(d->cb0); free(d->proj0); free(d->proj_rest);
  for (int g = 0; g < 15; g++) free(d->cb_rest[g]);
  free(d->pre.w); free(d->pre.b);
  free(d->in_w); free(d->in_b); free(d->norm); free(d->out_w); free(d->out_b);
  free(d->rope_cos); free(d->rope_sin);
  if (d->L)
    for (int l = 0; l < d->n_layers; l++) {
      odl* L = &d->L[l];
      free(L->q); free(L->k); free(L->v); free(L->o); free(L->gate); free(L->up); free(L->down);
      free(L->in_norm); free(L->post_norm); free(L->attn_scale); free(L->mlp_scale);
    }
  free(d->L);
  free(d);
}

oq_decoder* oq_decoder_load(const char* path, char* err, int errlen) {
  rctx r = {fopen(path, "rb"), 0, err, errlen};
  if (!r.f) { if (err) snprintf(err, errlen, "cannot open %s", path); return NULL; }
  setvbuf(r.f, NULL, _IOFBF, 1 << 23);
  oq_model* m = load_lm(&r);
  if (!m) { fclose(r.f); return NULL; }
  oq_free(m);
  oq_decoder* d = (oq_decoder*)calloc(1, sizeof(oq_decoder));
  d->hidden = r_u32(&r); d->heads = r_u32(&r); d->head_dim = r_u32(&r);
  d->inter = r_u32(&r); d->window = r_u32(&r); d->cb_dim = r_u32(&r);
  if (!r.err && (d->hidden == 0 || d->heads == 0 || d->head_dim == 0 || d->inter == 0 || d->cb_dim == 0))
    r_fail(&r, "the file has no speech decoder");
  const uint64_t A = (uint64_t)d->heads * d->head_dim, H = d->hidden;
  uint64_t l = 0;
  d->cb0 = r_f32(&r, &l);
  if (!r.err && (l == 0 || l % d->cb_dim)) r_fail(&r, "codebook length");
  d->entries = (uint32_t)(l / (d->cb_dim ? d->cb_dim : 1));
  d->proj0 = r_f32n(&r, (uint64_t)d->cb_dim * 512, "codebook projection length");
  uint32_t nr = r_u32(&r);
  if (!r.err && nr != 15) r_fail(&r, "expected 15 rest codebooks");
  for (uint32_t g = 0; g < nr && g < 15 && !r.err; g++)
    d->cb_rest[g] = r_f32n(&r, (uint64_t)d->entries * d->cb_dim, "codebook length");
  d->proj_rest = r_f32n(&r, (uint64_t)d->cb_dim * 512, "codebook projection length");
  d->pre = r_conv1d(&r);
  if (!r.err && (d->pre.in != 512 || d->pre.out != 1024 || d->pre.k == 0 || d->pre.dil == 0 ||
                 d->pre.wl != (uint64_t)d->pre.out * d->pre.in * d->pre.k || d->pre.bl != d->pre.out))
    r_fail(&r, "pre-conv shape");
  d->in_w = r_f32n(&r, 1024 * H, "transformer input projection length");
  d->in_b = r_f32n(&r, H, "transformer input bias length");
  d->n_layers = (int)r_u32(&r);
  if (!r.err && (d->n_layers <= 0 || d->n_layers > 64)) r_fail(&r, "bad decoder layer count");
  if (!r.err) {
    d->L = (odl*)calloc(d->n_layers, sizeof(odl));
    for (int i = 0; i < d->n_layers && !r.err; i++) {
      odl* L = &d->L[i];
      L->q = r_f32n(&r, H * A, "q_proj length"); L->k = r_f32n(&r, H * A, "k_proj length");
      L->v = r_f32n(&r, H * A, "v_proj length"); L->o = r_f32n(&r, A * H, "o_proj length");
      L->gate = r_f32n(&r, H * d->inter, "gate_proj length"); L->up = r_f32n(&r, H * d->inter, "up_proj length");
      L->down = r_f32n(&r, (uint64_t)d->inter * H, "down_proj length");
      L->in_norm = r_f32n(&r, H, "norm length"); L->post_norm = r_f32n(&r, H, "norm length");
      L->attn_scale = r_f32n(&r, H, "layer scale length"); L->mlp_scale = r_f32n(&r, H, "layer scale length");
    }
  }
  d->norm = r_f32n(&r, H, "norm length");
  d->out_w = r_f32n(&r, H * 1024, "transformer output projection length");
  d->out_b = r_f32n(&r, 1024, "transformer output bias length");
  uint32_t nu = r_u32(&r);
  if (!r.err && nu > 4096) r_fail(&r, "bad decoder upsample count");
  for (uint32_t i = 0; i < nu && !r.err; i++) {
    r_u32(&r); drop_conv(&r, 5); drop_conv(&r, 3);
    for (int j = 0; j < 7; j++) drop_vec(&r);
  }
  drop_conv(&r, 6);
  uint32_t nb = r_u32(&r);
  if (!r.err && nb > 4096) r_fail(&r, "bad vocos block count");
  for (uint32_t i = 0; i < nb && !r.err; i++) {
    drop_vec(&r); drop_vec(&r); drop_conv(&r, 5);
    uint32_t nres = r_u32(&r);
    if (!r.err && nres > 4096) r_fail(&r, "bad vocos residual count");
    for (uint32_t j = 0; j < nres && !r.err; j++) {
      drop_vec(&r); drop_vec(&r); drop_conv(&r, 6); drop_vec(&r); drop_vec(&r); drop_conv(&r, 6);
    }
  }
  drop_vec(&r); drop_vec(&r); drop_conv(&r, 6);
  d->rope_cos = r_f32(&r, &d->rope_len);
  d->rope_sin = r_f32n(&r, d->rope_len, "rope table length");
  fclose(r.f);
  if (r.err) { oq_decoder_free(d); return NULL; }
  return d;
}

/* decoder.rs:527-538 f32_gemv: weight [k][n], zero inputs skipped */
static void dec_gemv(const float* in, const float* w, size_t k, size_t n, float* out) {
  for (size_t j = 0; j < n; j++) out[j] = 0.0f;
  for (size_t ki = 0; ki < k; ki++) {
    float iv = in[ki];
    if (iv == 0.0f) continue;
    const float* wr = w + ki * n;
    for (size_t j = 0; j < n; j++) out[j] += iv * wr[j];
  }
}
/* decoder.rs:541-553 f32_gemv_bias */
static void dec_gemv_bias(const float* in, const float* w, size_t k, size_t n, const float* bias, float* out) {
  memcpy(out, bias, n * sizeof(float));
  for (size_t ki = 0; ki < k; ki++) {
    float iv = in[ki];
    if (iv == 0.0f) continue;
    const float* wr = w + ki * n;
    for (size_t j = 0; j < n; j++) out[j] += iv * wr[j];
  }
}
/* decoder.rs:515-525 rms_norm_f32 */
static void dec_rms(const float* x, const float* g, size_t n, float eps, float* out) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
  float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; i++) out[i] = x[i] * inv * g[i];
}
/* decoder.rs:556-578 apply_rope_split_half */
static void dec_rope(float* x, int heads, int hd, int pos, const float* c, const float* s, uint64_t len) {
  int half = hd / 2;
  uint64_t off = (uint64_t)pos * half;
  if (off + half > len) return;
  for (int h = 0; h < heads; h++) {
    float* b = x + (size_t)h * hd;
    for (int i = 0; i < half; i++) {
      float x0 = b[i], x1 = b[half + i], cc = c[off + i], ss = s[off + i];
      b[i] = x0 * cc - x1 * ss;
      b[half + i] = x1 * cc + x0 * ss;
    }
  }
}

int oq_decode_latent(const oq_decoder* d, const uint32_t* codes, int T, float* out) {
  const size_t cb = d->cb_dim, H = d->hidden, A = (size_t)d->heads * d->head_dim, I = d->inter;
  if (T <= 0) return 0;
  for (int g = 0; g < 16; g++)
    for (int t = 0; t < T; t++)
      if (codes[(size_t)g * T + t] >= d->entries) return -1;
  /* codebook_lookup decoder.rs:142-187 -> vq [512][T] */
  float* vq = (float*)calloc((size_t)512 * T, sizeof(float));
  float* proj = (float*)malloc(512 * sizeof(float));
  float* se = (float*)malloc(cb * sizeof(float));
  for (int t = 0; t < T; t++) {
    dec_gemv(d->cb0 + (size_t)codes[t] * cb, d->proj0, cb, 512, proj);
    for (int c = 0; c < 512; c++) vq[(size_t)c * T + t] += proj[c];
  }
  for (int t = 0; t < T; t++) {
    for (size_t e = 0; e < cb; e++) se[e] = 0.0f;
    for (int g = 0; g < 15; g++) {
      const float* emb = d->cb_rest[g] + (size_t)codes[(size_t)(g + 1) * T + t] * cb;
      for (size_t e = 0; e < cb; e++) se[e] += emb[e];
    }
    dec_gemv(se, d->proj_rest, cb, 512, proj);
    for (int c = 0; c < 512; c++) vq[(size_t)c * T + t] += proj[c];
  }
  /* causal_conv1d conv.rs:114-191 (left pad (k-1)*dilation) -> [1024][T] */
  const oconv* pc = &d->pre;
  float* pre = (float*)malloc((size_t)pc->out * T * sizeof(float));
  {
    const size_t pad = (size_t)(pc->k - 1) * pc->dil, ick = (size_t)pc->in * pc->k;
    for (uint32_t oc = 0; oc < pc->out; oc++)
      for (int o = 0; o < T; o++) {
        float sum = pc->b[oc];
        for (uint32_t ic = 0; ic < pc->in; ic++) {
          const float* wr = pc->w + oc * ick + (size_t)ic * pc->k;
          for (uint32_t k = 0; k < pc->k; k++) {
            size_t in_pos = (size_t)o + (size_t)k * pc->dil;
            if (in_pos >= pad) {
              size_t idx = in_pos - pad;
              if (idx < (size_t)T) sum += vq[(size_t)ic * T + idx] * wr[k];
            }
          }
        }
        pre[(size_t)oc * T + o] = sum;
      }
  }
  /* decoder_transformer decoder.rs:195-335 */
  const size_t D = 1024;
  float* xrow = (float*)malloc(D * T * sizeof(float));
  for (size_t c = 0; c < D; c++)
    for (int t = 0; t < T; t++) xrow[(size_t)t * D + c] = pre[c * T + t];
  float* x = (float*)malloc(H * T * sizeof(float));
  for (int t = 0; t < T; t++) dec_gemv_bias(xrow + (size_t)t * D, d->in_w, D, H, d->in_b, x + (size_t)t * H);
  float* q = (float*)malloc(A * T * sizeof(float));
  float* k = (float*)malloc(A * T * sizeof(float));
  float* v = (float*)malloc(A * T * sizeof(float));
  float* xn = (float*)malloc(H * sizeof(float));
  float* ao = (float*)malloc(A * sizeof(float));
  float* oo = (float*)malloc(H * sizeof(float));
  float* sc = (float*)malloc((size_t)(d->window + 1) * sizeof(float));
  float* gt = (float*)malloc(I * sizeof(float));
  float* up = (float*)malloc(I * sizeof(float));
  const int hd = (int)d->head_dim;
  const float scale = 1.0f / sqrtf((float)hd);
  for (int li = 0; li < d->n_layers; li++) {
    const odl* L = &d->L[li];
    for (int t = 0; t < T; t++) {
      dec_rms(x + (size_t)t * H, L->in_norm, H, 1e-5f, xn);
      dec_gemv(xn, L->q, H, A, q + (size_t)t * A);
      dec_gemv(xn, L->k, H, A, k + (size_t)t * A);
      dec_gemv(xn, L->v, H, A, v + (size_t)t * A);
    }
    for (int t = 0; t < T; t++) {
      dec_rope(q + (size_t)t * A, (int)d->heads, hd, t, d->rope_cos, d->rope_sin, d->rope_len);
      dec_rope(k + (size_t)t * A, (int)d->heads, hd, t, d->rope_cos, d->rope_sin, d->rope_len);
    }
    for (int t = 0; t < T; t++) {
      int start = (t + 1 > (int)d->window) ? t + 1 - (int)d->window : 0;
      int L_ = t + 1 - start;
      for (size_t e = 0; e < A; e++) ao[e] = 0.0f;
      for (int h = 0; h < (int)d->heads; h++) {
        const float* qq = q + (size_t)t * A + (size_t)h * hd;
        for (int s = 0; s < L_; s++) {
          const float* kk = k + (size_t)(start + s) * A + (size_t)h * hd;
          float dot = 0.0f;
          for (int e = 0; e < hd; e++) dot += qq[e] * kk[e];
          sc[s] = dot * scale;
        }
        oq_softmax_raw(sc, (size_t)L_);
        for (int s = 0; s < L_; s++) {
          const float* vv = v + (size_t)(start + s) * A + (size_t)h * hd;
          float p = sc[s];
          for (int e = 0; e < hd; e++) ao[(size_t)h * hd + e] += p * vv[e];
        }
      }
      dec_gemv(ao, L->o, A, H, oo);
      for (size_t j = 0; j < H; j++) x[(size_t)t * H + j] += oo[j] * L->attn_scale[j];
    }
    for (int t = 0; t < T; t++) {
      dec_rms(x + (size_t)t * H, L->post_norm, H, 1e-5f, xn);
      dec_gemv(xn, L->gate, H, I, gt);
      dec_gemv(xn, L->up, H, I, up);
      for (size_t j = 0; j < I; j++) {
        float g = gt[j];
        gt[j] = (g / (1.0f + expf(-g))) * up[j];
      }
      dec_gemv(gt, L->down, I, H, oo);
      for (size_t j = 0; j < H; j++) x[(size_t)t * H + j] += oo[j] * L->mlp_scale[j];
    }
  }
  float* orow = (float*)malloc(D * sizeof(float));
  for (int t = 0; t < T; t++) {
    dec_rms(x + (size_t)t * H, d->norm, H, 1e-5f, xn);
    dec_gemv_bias(xn, d->out_w, H, D, d->out_b, orow);
    for (size_t c = 0; c < D; c++) out[c * T + t] = orow[c];
  }
  free(vq); free(proj); free(se); free(pre); free(xrow); free(x); free(q); free(k); free(v);
  free(xn); free(ao); free(oo); free(sc); free(gt); free(up); free(orow);
  return 0;
}
