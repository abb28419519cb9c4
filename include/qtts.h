/*
 * qtts.h -- C ABI of the B200-native QORA-TTS 1.7B decode loop
 * (libqtts_b200.so).
 *
 * Every entry point returns an int status (QTTS_OK = 0, negative = error;
 * qtts_last_error() gives the message of the calling thread's last failure).
 * Host buffers are caller-owned; pointers named *_dev are device pointers.
 * A model is read-only and may be shared across threads; a session belongs to
 * one thread at a time.  Reference citations are paths inside the qora-tts
 * crate (src/...), the Rust functions each entry point replaces.
 */
#ifndef QTTS_H
#define QTTS_H
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QTTS_API __attribute__((visibility("default")))
#else
#define QTTS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define QTTS_OK 0
#define QTTS_ERR_BADARG (-1)
#define QTTS_ERR_OOM (-2)
#define QTTS_ERR_CUDA (-3)
#define QTTS_ERR_TIMEOUT (-4)
#define QTTS_ERR_FORMAT (-5)
#define QTTS_ERR_IO (-6)
#define QTTS_ERR_STATE (-7)
#define QTTS_ERR_NODEV (-8)
#define QTTS_ERR_RANGE (-9)

typedef struct qtts_model qtts_model;
typedef struct qtts_session qtts_session;
typedef struct qtts_decoder qtts_decoder;

/* Model dimensions as stored in the .qora-tts headers (save.rs:49-59,92-97). */
typedef struct {
  int t_layers, t_hidden, t_text_hidden, t_heads, t_kv_heads, t_head_dim;
  int t_inter, t_vocab, t_text_vocab, t_max_pos;
  int t_sec[3];
  int p_layers, p_hidden, p_heads, p_kv_heads, p_head_dim, p_inter, p_vocab;
  int p_groups, p_max_pos;
  int fmt; /* save.rs:34 format_id: 1 = Q4, 0 = F16 */
} qtts_dims;

/* generate_new.rs:38-45 TTSParams (max_codes is a qtts_generate argument). */
typedef struct {
  float temperature;
  int top_k;
  float repetition_penalty;
  uint32_t codec_eos_id;
} qtts_sample_params;

/* One utterance of generate_new.rs:191-202 generate_speech, after
 * tokenization (tokenizer.rs:16 is out of scope: callers pass token ids). */
typedef struct {
  const uint32_t* text; /* token ids */
  int n_text;
  uint32_t speaker_id;
  uint32_t language_id;
  const float* voice; /* nullable: 2048-d speaker embedding (main.rs:209-217) */
  uint64_t seed;      /* xorshift64 state, generate_new.rs:233 */
  qtts_sample_params params;
} qtts_utterance;

/* qtts_generate flags */
#define QTTS_IGNORE_EOS 1u /* run all max_frames (benchmarks with random weights) */
/* Benchmark mode of this library (not a reference mode): after the
 * generate_new.rs:94-173 prefill rows, text tokens 1..n_text-1 are prefilled
 * as embed_text(tok) + embed_codec(CODEC_PAD) rows, so utterances with
 * different prompt lengths decode over KV caches of different lengths; the
 * frames' trailing text is then TTS_EOS followed by TTS_PAD. */
#define QTTS_FULL_PROMPT 2u

QTTS_API const char* qtts_last_error(void);
QTTS_API int qtts_version(void);

/* ---- .qora-tts file (host only; no GPU needed) ---------------------------- */
/* Parse and validate the talker + predictor sections: save.rs:262-409. */
QTTS_API int qtts_file_probe(const char* path, qtts_dims* out);
/* Write a seeded synthetic model in the save.rs:23-137 byte layout (talker,
 * predictor and an empty decoder section): Q4 bytes uniform, scales
 * f16(|N(0,0.02)|), norms 1, biases N(0,0.02), RoPE tables per rope.rs:11-41
 * and loader.rs:399-408.  Replaces offline compress_model.rs:35-82. */
QTTS_API int qtts_synth_write(const char* path, const qtts_dims* dims, uint64_t seed);
/* flags: QTTS_SYNTH_DECODER writes a full-size synthetic speech decoder
 * section (decoder.rs:21-108 shapes: 16 codebooks of 2048 x 256, pre-conv,
 * 8 transformer layers of hidden 512 / 16 heads of 64 / MLP 1024 / window
 * 72, RoPE tables; the upsample and Vocos stages written empty) instead of
 * an empty one.  The talker and predictor bytes are the same as without. */
#define QTTS_SYNTH_DECODER 1u
QTTS_API int qtts_synth_write_ex(const char* path, const qtts_dims* dims, uint64_t seed, unsigned flags);
QTTS_API void qtts_dims_1p7b(qtts_dims* out);
QTTS_API void qtts_dims_tiny(qtts_dims* out);

/* ---- model ------------------------------------------------------------------ */
/* save.rs:262 load_model + one upload to HBM in the on-disk layout. */
QTTS_API int qtts_model_load(const char* path, int device, qtts_model** out);
QTTS_API int qtts_model_free(qtts_model* m);
QTTS_API int qtts_model_dims(const qtts_model* m, qtts_dims* out);
QTTS_API size_t qtts_model_device_bytes(const qtts_model* m);

/* ---- session: device KV caches + activations for up to max_batch utterances */
/* gemv.rs:79-86 empty_kv_cache, as paged device KV (16 positions / page). */
QTTS_API int qtts_session_create(qtts_model* m, int max_batch, int max_positions, qtts_session** out);
/* Opt-in session modes (no counterpart in the reference, whose caches are
 * f32 Vec<f32>, gemv.rs:77-86).  QTTS_SESSION_KV_F16: the talker and
 * predictor K/V caches hold f16 (round to nearest even) instead of f32,
 * halving their bytes and the attention's HBM traffic; every other value,
 * the attention arithmetic included, stays f32.  Results then differ from
 * the reference's by the cache rounding (logits within 1e-2 of the largest
 * logit on the parity cases); qtts_session_create is _ex with flags 0. */
#define QTTS_SESSION_KV_F16 1u
QTTS_API int qtts_session_create_ex(qtts_model* m, int max_batch, int max_positions, unsigned flags,
                                    qtts_session** out);
QTTS_API int qtts_session_free(qtts_session* s);
QTTS_API int qtts_session_reset(qtts_session* s);
QTTS_API void* qtts_session_stream(qtts_session* s); /* cudaStream_t the session launches on */
/* No counterpart in the reference (it has no failure detection: it panics).
 * Bound, in nanoseconds, on the device wait in which the one-row GEMV's
 * cluster root collects its peers' split-K partials (default 1 s; takes
 * effect for the next generation or per-call step).  A wait that runs out
 * makes the call return QTTS_ERR_TIMEOUT, and keeps waiting for at most 1 s
 * more so that no peer's transfer is left in flight into the waiting CTA;
 * the outputs of such a call are undefined.  A short budget exercises the
 * timeout path without a GPU fault. */
QTTS_API int qtts_session_set_wait_budget(qtts_session* s, uint64_t ns);

/* ---- per-call reference API (slot 0 of the session, batch 1) ------------- */
QTTS_API int qtts_embed_text(qtts_session* s, uint32_t token, float* out);  /* talker.rs:105 */
QTTS_API int qtts_embed_codec(qtts_session* s, uint32_t token, float* out); /* talker.rs:152 */
/* talker.rs:364-462 prefill_talker_raw (+ talker.rs:627 apply_codec_head):
 * emb [n][H] host; hidden_out [H], logits_out [V] (either may be NULL). */
QTTS_API int qtts_prefill(qtts_session* s, const float* emb, int n, float* hidden_out, float* logits_out);
/* talker.rs:263-360 forward_with_embedding: out = normed hidden [H] ++ logits [V]. */
QTTS_API int qtts_talker_step(qtts_session* s, const float* emb, int position, float* out);
/* code_predictor.rs:218-273 generate_acoustic_codes -> codes[p_groups]. */
QTTS_API int qtts_predict_acoustic(qtts_session* s, const float* talker_hidden, const float* semantic_embed,
                          uint32_t* codes);
/* code_predictor.rs:280-293 get_acoustic_embeddings_sum. */
QTTS_API int qtts_acoustic_embed_sum(qtts_session* s, const uint32_t* codes, float* out);
/* generate_new.rs:329-391 sample_token on the GPU (bit-exact given the same
 * logits and rng state); *rng is advanced as the reference advances it. */
QTTS_API int qtts_sample(qtts_session* s, const float* logits, int n, const qtts_sample_params* p,
                const uint32_t* prev16, uint64_t* rng, uint32_t* out);

/* ---- batched generation (generate_new.rs:191-300 frame loop, one CUDA graph
 * per frame for all utterances) ------------------------------------------- */
/* forced: nullable [n_utt][max_frames][16] teacher-forcing codes (they drive
 * the next steps; the GPU's own choices are still written to codes_out).
 * codes_out [n_utt][max_frames][16]; frames_out [n_utt]; logits_dump
 * nullable [n_utt][max_frames][V]; hidden_dump nullable [n_utt][max_frames][H]. */
QTTS_API int qtts_generate(qtts_session* s, int n_utt, const qtts_utterance* utts, int max_frames,
                  unsigned flags, const uint32_t* forced, uint32_t* codes_out, int* frames_out,
                  float* logits_dump, float* hidden_dump);
/* The same loop split in three for timing: begin = prefill + trailing text;
 * frames = n_frames graph replays (asynchronous on the session stream);
 * end = wait and copy results out. */
QTTS_API int qtts_generate_begin(qtts_session* s, int n_utt, const qtts_utterance* utts, int max_frames,
                        unsigned flags, const uint32_t* forced);
QTTS_API int qtts_generate_frames(qtts_session* s, int n_frames);
QTTS_API int qtts_generate_end(qtts_session* s, uint32_t* codes_out, int* frames_out, float* logits_dump,
                      float* hidden_dump);
/* Number of kernels one frame launches (CUDA-graph nodes). */
QTTS_API int qtts_frame_kernel_count(qtts_session* s);
/* Frame graphs this session has captured.  qtts_generate / _begin reuse the
 * last one while the batch size, max_frames, trailing-text rows, forcing and
 * dump options are unchanged (the per-generation buffers are grow-only). */
QTTS_API int qtts_frame_graph_captures(qtts_session* s);

/* ---- speech decoder, first stage (codes -> transformer output) ------------
 * The reference runs decode_to_audio (decoder.rs:394-513) on the CPU; its
 * first three steps -- codebook_lookup (decoder.rs:142-187), the causal
 * pre-conv (conv.rs:114-191) and decoder_transformer (decoder.rs:195-335) --
 * run here on the GPU over all frames of an utterance at once.  The
 * upsample / Vocos stages that follow stay with the caller. */
/* save.rs:446-552 load_decoder_weights (the decoder section of a .qora-tts
 * file), uploaded to `device`; QTTS_ERR_FORMAT if the section is empty. */
QTTS_API int qtts_decoder_load(const char* path, int device, qtts_decoder** out);
QTTS_API int qtts_decoder_free(qtts_decoder* d);
QTTS_API void* qtts_decoder_stream(qtts_decoder* d); /* cudaStream_t of the decoder */
/* codes [16][n_frames] host (codes[g][t], the reference's &[Vec<u32>]);
 * out [1024][n_frames] host, channel-first like decoder_transformer's
 * result.  QTTS_ERR_RANGE for a code past its codebook (the reference
 * panics on that index). */
QTTS_API int qtts_decode_latent(qtts_decoder* d, const uint32_t* codes, int n_frames, float* out);
/* The same on device buffers, asynchronous on the decoder's stream; a bad
 * code is reported by the next qtts_decoder_sync. */
QTTS_API int qtts_decode_latent_dev(qtts_decoder* d, const uint32_t* codes, int n_frames, float* out);
QTTS_API int qtts_decoder_sync(qtts_decoder* d);

/* ---- profiling (no counterpart in the reference) -------------------------- */
/* Kernel families of the frame plan. */
#define QTTS_FAMILY_Q4MV_DEC 1  /* q4mv_dec_kernel: one-row CUDA-core Q4 GEMV */
#define QTTS_FAMILY_Q4MV_ROWS 2 /* q4mv_rows_kernel: multi-row CUDA-core Q4 GEMV (shapes the others do not take) */
#define QTTS_FAMILY_TC_PROJ 3   /* tc_proj_kernel: tcgen05 Q4 projection */
#define QTTS_FAMILY_ATTN 4      /* attn_kernel: GQA over the paged cache */
#define QTTS_FAMILY_Q4MV_BATCH 5 /* q4mv_batch_kernel: 3-15-row CUDA-core Q4 GEMV */
/* Device time of one frame's launches of one family, captured without the
 * frame's other launches (same order, parameters and dependent-launch links)
 * and replayed `reps` times between CUDA events on the session stream.  Needs
 * a generation begun on the session; the replays rewrite the current frame's
 * cache entries, activations and codes, so that generation ends (the next
 * qtts_generate / _begin starts afresh).  Outputs: ms per replay, launches
 * per replay, their useful FLOPs (2*M*k*n per projection matrix) and their
 * Q4 weight bytes (k*n*0.5625 per matrix). */
QTTS_API int qtts_frame_family_time(qtts_session* s, int family, int reps, float* ms_per_replay, int* launches,
                                    double* flops, double* weight_bytes);

/* ---- kernels on device pointers (gemv.rs:149 gemv / :157 gemm) ------------ */
/* y[m][n] = sum_k x[m][k] * W[k][n] for a Q4 g32 weight in the on-disk
 * [k][n] layout (packed k*n/2 bytes, low nibble = even column; scales
 * k*n/32 f16).  scratch_dev: split-K tile counters and partials,
 * qtts_q4_gemv_scratch_bytes() bytes, zero-filled before its first use (every
 * call leaves the counters at zero again).  m >= 16 with 16-byte aligned x/y,
 * k % 4 == 0 and n % 64 == 0 runs on the tensor cores (tcgen05). */
QTTS_API size_t qtts_q4_gemv_scratch_bytes(int k, int n, int m);
QTTS_API int qtts_q4_gemv_dev(const uint8_t* packed_dev, const uint16_t* scales_dev, int k, int n,
                     const float* x_dev, int m, float* y_dev, void* scratch_dev,
                     size_t scratch_bytes, void* stream);
/* No counterpart in the reference.  qtts_q4_gemv_dev for callers that cannot
 * allocate device memory: a real-time audio thread that may not block inside
 * a driver allocation, or a host whose GPU memory is already owned by another
 * framework's caching allocator, where a fresh cudaMalloc can fail or
 * fragment that pool.  The split-K scratch (tile counters, then partial sums)
 * comes from a static device array of QTTS_Q4_GEMV_NOALLOC_SCRATCH_BYTES that
 * every GPU loading the library holds until exit; the caller passes only
 * inputs and outputs, and the call allocates nothing.  The first call on a
 * device looks up the array's device address and sets the kernels' shared-
 * memory attributes, so make that first call before any stream capture.
 * Under CUDA's lazy module loading that first call may also load this
 * library's device code, which reserves the array inside the driver: make
 * it once per device as a warm-up, off the real-time thread.  The address
 * and attributes are kept for the life of the process, so the entry point
 * must not be used across a cudaDeviceReset of that device.
 * Every call on a device shares the array, which keeps the last call's
 * contents: the counters are cleared on each call and the partial sums are
 * rewritten before they are read, but calls that overlap on the GPU (other
 * streams or threads) race on it and must be serialised by the caller.
 * Shapes whose scratch exceeds the array return QTTS_ERR_RANGE. */
#define QTTS_Q4_GEMV_NOALLOC_SCRATCH_BYTES (4u << 20)
QTTS_API int qtts_q4_gemv_dev_noalloc(const uint8_t* packed_dev, const uint16_t* scales_dev, int k, int n,
                                      const float* x_dev, int m, float* y_dev, void* stream);
/* Same contract with host buffers (copies in, runs, copies out). */
QTTS_API int qtts_q4_gemv(const uint8_t* packed, const uint16_t* scales, int k, int n, const float* x,
                 int m, float* y);
/* The exp the code-0 sampler uses (Rust f32::exp at generate_new.rs:355,
 * i.e. glibc expf), element-wise on device pointers, for validation. */
QTTS_API int qtts_expf_dev(const float* x_dev, float* y_dev, int n, void* stream);
/* gemv.rs:183-196 gemv_f16 on device pointers. */
QTTS_API int qtts_f16_gemv_dev(const uint16_t* w_dev, int k, int n, const float* x_dev, int m, float* y_dev,
                      void* stream);
/* gemv.rs:378-400 dequant of the whole matrix: out[k][n] = f32(scale)*(q-8). */
QTTS_API int qtts_q4_dequant_dev(const uint8_t* packed_dev, const uint16_t* scales_dev, int k, int n,
                        float* out_dev, void* stream);
/* gemv.rs:92-130 quantize_f32_to_q4 on device pointers: data[k][n] f32 ->
 * packed[k*n/2] (low nibble = even column) + scales[k*n/32] f16, the on-disk
 * layout, bit-identical to the reference (scale = f16(absmax/7), q =
 * clamp(round(v/scale), -8, 7) + 8, NaN -> 0).  n % 32 == 0; data 16-byte
 * aligned, packed and scales 2-byte aligned. */
QTTS_API int qtts_q4_quantize_dev(const float* data_dev, int k, int n, uint8_t* packed_dev, uint16_t* scales_dev,
                                  void* stream);
/* Same with host buffers (copies in, runs, copies out). */
QTTS_API int qtts_q4_quantize(const float* data, int k, int n, uint8_t* packed, uint16_t* scales);

#ifdef __cplusplus
}
#endif
#endif
