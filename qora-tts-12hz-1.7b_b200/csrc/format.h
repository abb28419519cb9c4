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

// Parse the talker and predictor sections, checking every length against the
// header dimensions.  Returns QTTS_OK or QTTS_ERR_IO / QTTS_ERR_FORMAT.
int parse_model(const char* path, HModel* out, std::string* err);
int synth_write(const char* path, const qtts_dims& d, uint64_t seed, std::string* err);
void dims_1p7b(qtts_dims* d);
void dims_tiny(qtts_dims* d);

}  // namespace qtts
