/*
 * qtts_oracle.h -- CPU restatement of the QORA-TTS per-frame decode loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path
 * is compared against (and the timed CPU baseline in bench.py).  The product
 * (libqtts_b200.so) never links, loads or calls it.
 *
 * PARITY UNPINNED: the reference (a Rust crate) cannot be compiled in this
 * image (no cargo/rustc) and its own tests hold no golden vectors for this
 * path, so this restatement is pinned only by transcription review and by
 * the self-consistency tests under tests/.  Every function cites the
 * reference file:line it restates.
 *
 * Arithmetic conventions (they decide bit-exactness against the reference):
 *   - all activations f32, sequential left-to-right summation exactly as the
 *     Rust loops / iter().sum() do; compiled with -ffp-contract=off;
 *   - f16 -> f32 is exact (half 2.x to_f32); f32 -> f16 is round-to-nearest-
 *     even (half 2.x from_f32), used only when writing synthetic weights;
 *   - exp is glibc expf (Rust's f32::exp lowers to the platform libm).
 */
#ifndef QTTS_ORACLE_H
#define QTTS_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Dimensions of a synthetic model (talker + code predictor). */
typedef struct {
  int t_layers, t_hidden, t_text_hidden, t_heads, t_kv_heads, t_head_dim;
  int t_inter, t_vocab, t_text_vocab, t_max_pos;
  int t_sec[3];
  int p_layers, p_hidden, p_heads, p_kv_heads, p_head_dim, p_inter, p_vocab;
  int p_groups, p_max_pos;
  int fmt; /* 1 = Q4 (the only format the synthetic writer emits), 0 = F16 */
} oq_dims;

typedef struct {
  int max_codes;
  float temperature;
  int top_k;
  float repetition_penalty;
  uint32_t codec_eos_id;
  uint32_t codec_bos_id;
} oq_params;

typedef struct oq_model oq_model;
typedef struct oq_kv oq_kv;

/* -- f16 helpers (half 2.x semantics) -- */
float oq_h2f(uint16_t h);
uint16_t oq_f2h(float f);

/* -- synthetic weights in the .qora-tts layout (save.rs:23-137) -- */
int oq_synth_write(const char* path, const oq_dims* d, uint64_t seed);
/* flags: OQ_SYNTH_DECODER writes a full-size synthetic speech decoder
 * (codebooks, pre-conv, transformer, RoPE; upsample / Vocos stages empty). */
#define OQ_SYNTH_DECODER 1u
int oq_synth_write_ex(const char* path, const oq_dims* d, uint64_t seed, unsigned flags);
/* decoder shapes of the synthetic file (decoder.rs:21-108) */
#define OQ_DEC_HIDDEN 512
#define OQ_DEC_HEADS 16
#define OQ_DEC_HEAD_DIM 64
#define OQ_DEC_INTER 1024
#define OQ_DEC_WINDOW 72
#define OQ_DEC_CB_DIM 256
#define OQ_DEC_ENTRIES 2048
#define OQ_DEC_LAYERS 8
#define OQ_DEC_LATENT 1024
#define OQ_DEC_ROPE_POS 8192

/* -- speech decoder, codes -> transformer output (decoder.rs:142-335 with
 * the conv.rs:114-191 pre-conv, the first three steps of decode_to_audio
 * decoder.rs:394-424) -- */
typedef struct oq_decoder oq_decoder;
oq_decoder* oq_decoder_load(const char* path, char* err, int errlen);
void oq_decoder_free(oq_decoder* d);
/* codes: [16][T] (codes[g][t], the reference's &[Vec<u32>]); out: the
 * transformer output [1024][T] channel-first.  Returns 0, or -1 for a code
 * past its codebook (the reference panics on that index). */
int oq_decode_latent(const oq_decoder* d, const uint32_t* codes, int T, float* out);
/* Test fixture: predictor heads written with column j == column j % period
 * (0 = the ordinary synthetic heads); applies to later oq_synth_write calls. */
void oq_set_tie_period(int period);
void oq_dims_1p7b(oq_dims* d);
void oq_dims_tiny(oq_dims* d);
/* seeded synthetic inputs shared by tests and bench */
void oq_rand_normal(uint64_t seed, float* out, size_t n, float stddev);
void oq_rand_tokens(uint64_t seed, uint32_t* out, size_t n, uint32_t vocab);
void oq_rand_bytes(uint64_t seed, uint8_t* out, size_t n);
void oq_rand_scales(uint64_t seed, uint16_t* out, size_t n, float stddev);

/* -- model I/O (save.rs:262-409) -- */
oq_model* oq_load(const char* path, char* err, int errlen);
void oq_free(oq_model* m);
void oq_get_dims(const oq_model* m, oq_dims* d);
/* thread policy of gemv.rs:268-272 (num_threads when k*n >= 4e6) */
void oq_set_threads(int n);
int oq_get_threads(void);

/* -- numeric kernels (gemv.rs) -- */
void oq_gemv_q4(const float* x, const uint8_t* packed, const uint16_t* scales,
                size_t k, size_t n, float* y);                 /* gemv.rs:263 */
void oq_gemm_q4(const float* x, size_t seq, const uint8_t* packed,
                const uint16_t* scales, size_t k, size_t n, float* y); /* :311 */
void oq_gemv_f16(const float* x, const uint16_t* w, size_t k, size_t n, float* y);
void oq_quantize_q4(const float* data, size_t k, size_t n, uint8_t* packed,
                    uint16_t* scales);                          /* gemv.rs:92 */
void oq_embed_q4(const uint8_t* packed, const uint16_t* scales, size_t n,
                 size_t row, float* out);                       /* gemv.rs:378 */
void oq_rms_norm_f16(const float* x, const uint16_t* gamma, size_t n, float* out);
void oq_softmax_raw(float* s, size_t n);
float oq_silu(float x);
void oq_build_mrope_tables(int head_dim, int max_pos, double theta,
                           const int* sec, int n_sec, float* cos_t, float* sin_t);
void oq_build_rope_tables(int head_dim, int max_pos, double theta, float* cos_t,
                          float* sin_t);

/* -- KV cache (gemv.rs:77-86) -- */
oq_kv* oq_kv_new(int layers, int kv_heads, int head_dim);
void oq_kv_free(oq_kv* kv);
void oq_kv_clear(oq_kv* kv);
int oq_kv_len(const oq_kv* kv, int layer);

/* -- model forward (talker.rs, code_predictor.rs) -- */
oq_kv* oq_talker_kv_new(const oq_model* m);
oq_kv* oq_predictor_kv_new(const oq_model* m);
void oq_embed_text_token(const oq_model* m, uint32_t tok, float* out);
void oq_embed_codec_token(const oq_model* m, uint32_t tok, float* out);
/* out = normed_hidden[H] ++ logits[V] */
int oq_forward_with_embedding(const oq_model* m, const float* emb, oq_kv* kv,
                              int position, float* out);
int oq_prefill_talker_raw(const oq_model* m, const float* x, int seq, oq_kv* kv,
                          float* last_hidden);
void oq_apply_codec_head(const oq_model* m, const float* h, float* logits);
void oq_generate_acoustic_codes(const oq_model* m, const float* talker_hidden,
                                const float* semantic_embed, oq_kv* pkv,
                                uint32_t* codes15);
void oq_acoustic_embed_sum(const oq_model* m, const uint32_t* codes15, float* out);
uint32_t oq_sample_argmax(const float* logits, size_t n);

/* -- generation loop (generate_new.rs) -- */
float oq_simple_rand(uint64_t* state);
uint32_t oq_sample_token(const float* logits, size_t n, const oq_params* p,
                         const uint32_t* prev16, uint64_t* rng);
/* prefill_custom_voice: returns seq_len, writes last_hidden[H], logits[V] */
int oq_prefill_custom_voice(const oq_model* m, const uint32_t* text, int n_text,
                            uint32_t speaker_id, uint32_t language_id,
                            const float* voice_emb /*nullable*/, oq_kv* kv,
                            float* last_hidden, float* logits);
/* The frame loop of generate_new.rs:191-300 without the audio decoder.
 *   forced   nullable [max_codes*16]: teacher forcing (codes that drive the
 *            next step; the oracle's own choices still land in codes_out)
 *   logits_dump nullable [max_codes*V]: logits sampled at each frame
 *   hidden_dump nullable [max_codes*H]: talker hidden fed to the predictor
 *   flags    bit 0: ignore EOS (benchmarks with random weights); bit 1:
 *            full prompt (a benchmark mode of this build: text tokens
 *            1..n-1 prefilled as embed_text + embed_codec(CODEC_PAD) rows,
 *            trailing text = TTS_EOS, then TTS_PAD)
 * Returns the number of frames produced (EOS stops unless ignored). */
int oq_generate(const oq_model* m, const uint32_t* text, int n_text,
                uint32_t speaker_id, uint32_t language_id, const float* voice_emb,
                const oq_params* p, uint64_t seed, int flags,
                const uint32_t* forced, uint32_t* codes_out, float* logits_dump,
                float* hidden_dump);

/* time one frame step at a pre-filled KV length (CPU baseline helper) */
double oq_time_frames(const oq_model* m, int kv_len, int frames, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
