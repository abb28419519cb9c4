// format.h -- .qora-tts file layout (save.rs:23-137, 262-409; gemv.rs:558-650).
#pragma once
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/qtts.h"

namespace qtts {

// A Weight record (gemv.rs:558-573): Q4 = k, n, len+packed, len+f16 scales;
// F16 = k, n, len+f16 data.  Offsets are payload byte offsets in the file.
struct HWeight {
  int fmt = 1;
  uint64_t k = 0, n = 0;
  uint64_t off_a = 0, bytes_a = 0;  // packed (Q4) or data (F16)
  uint64_t off_b = 0, bytes_b = 0;  // scales (Q4)
};
struct HVec {  // u64 length + raw little-endian payload
  uint64_t off = 0, bytes = 0, len = 0;
};
struct HLayer {
  HWeight q, k, v, o, gate, up, down;
  HVec q_norm, k_norm, in_norm, post_norm;
};
struct HModel {
  qtts_dims d{};
  int t_kv_groups = 0, p_kv_groups = 0, t_nsec = 0;
  std::vector<HLayer> tl, pl;
  HWeight codec_emb, text_emb, fc1, fc2, codec_head, input_proj;
  HVec fc1_b, fc2_b, t_final, t_cos, t_sin, input_proj_b, p_final, p_cos, p_sin;
  std::vector<HWeight> p_emb, lm;
  bool has_proj = false;
  uint64_t file_size = 0;
};

// The speech decoder's codebook / pre-conv / transformer part of the decoder
// section (save.rs:446-552 load_decoder_weights; decoder.rs:21-108 shapes):
// payload offsets of its f32 vectors, the rest of the section walked only.
struct HConv1d {
  uint32_t in = 0, out = 0, k = 0, stride = 0, pad = 0, dil = 0;
  HVec w, b;
};
struct HDecLayer {
  HVec q, k, v, o, gate, up, down, in_norm, post_norm, attn_scale, mlp_scale;
};
struct HDecoder {
  uint32_t hidden = 0, heads = 0, head_dim = 0, inter = 0, window = 0, cb_dim = 0;
  HVec cb0, proj0, proj_rest;
  std::vector<HVec> cb_rest;
  HConv1d pre_conv;
  HVec in_w, in_b, norm, out_w, out_b, rope_cos, rope_sin;
  std::vector<HDecLayer> layers;
};

// Parse the talker and predictor sections, checking every length against the
// header dimensions (and, with `dec`, record the decoder's tensors).  Returns
// QTTS_OK or QTTS_ERR_IO / QTTS_ERR_FORMAT.
int parse_model(const char* path, HModel* out, std::string* err, HDecoder* dec = nullptr);
// with_decoder: a full-size synthetic speech decoder (codebooks, pre-conv,
// transformer, RoPE tables; upsample and Vocos stages empty) instead of an
// empty decoder section.
int synth_write(const char* path, const qtts_dims& d, uint64_t seed, std::string* err, bool with_decoder = false);
void dims_1p7b(qtts_dims* d);
void dims_tiny(qtts_dims* d);

}  // namespace qtts
