// engine.h -- device model, sessions and per-frame launch plans.
#pragma once
#include <cuda_runtime.h>

#include <functional>
#include <string>
#include <vector>

#include "../../include/qtts.h"
#include "format.h"
#include "kernels.h"
#include "misc.h"

namespace qtts {

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
// One tensor-core projection over M input rows from weights given only as
// expanded operand tiles (Q4Mat::wx set; k, n): out[M][ldo] = X * W (+ bias)
// for EPI_STORE, or silu(X * W0) * (X * W1) for the paired EPI_SWIGLU.  Rows
// above 64 are split once into xs_buf (tc_xsplit_scratch_bytes(M, k)).
// Errors of the launch; device-side ones set bits of err_flag.
// x_split_pre: the input rows already split by their producer (X unused
// then); xs_out: the EPI_SWIGLU result also written split (for a next
// projection of K = n).
int tc_project_expanded(const Q4Mat* mats, int nmat, int epi, const float* X, long ldx, int M, float* out, long ldo,
                        const float* bias, uint8_t* xs_buf, size_t xs_bytes, const uint8_t* x_split_pre,
                        uint8_t* xs_out, int* err_flag, cudaStream_t st);

struct DLayer {
  Q4Mat q, k, v, o, gate, up, down;
  const __half *q_norm = nullptr, *k_norm = nullptr, *in_norm = nullptr, *post_norm = nullptr;
};

// The model in HBM: every Weight keeps its on-disk bytes (packed + f16
// scales), norms stay f16, biases and RoPE tables f32 -- one arena.
struct Model {
  qtts_dims d{};
  int device = 0;
  int sm_count = 148;
  char* arena = nullptr;
  size_t bytes = 0;
  std::vector<DLayer> tl, pl;
  Q4Mat codec_emb, text_emb, fc1, fc2, codec_head, input_proj;
  const float *fc1_b = nullptr, *fc2_b = nullptr, *input_proj_b = nullptr;
  const float *t_cos = nullptr, *t_sin = nullptr, *p_cos = nullptr, *p_sin = nullptr;
  const __half *t_final = nullptr, *p_final = nullptr;
  std::vector<Q4Mat> p_emb, lm;
  Q4Mat* d_group_emb = nullptr;  // device copy of p_emb for the fusion kernel
  uint8_t* wx_arena = nullptr;   // predictor layer weights expanded for the tensor cores (optional)
  size_t wx_bytes = 0;
  bool has_proj = false;
};

using Op = std::function<cudaError_t(cudaStream_t)>;

struct Session {
  Model* m = nullptr;
  int maxB = 0, maxP = 0, pages_per_sess = 0;
  cudaStream_t st = nullptr;
  // caches
  float* kv_pool = nullptr;   // talker [pages][layers][2][kvh][16][128]
  int* page_table = nullptr;  // [maxB][pages_per_sess]
  float* pkv_pool = nullptr;  // predictor, one page per slot
  int kv_f16 = 0;             // both caches hold f16 elements (QTTS_SESSION_KV_F16)
  // per-slot state
  SlotState* slots = nullptr;
  // activations
  int rows = 0;  // row capacity of q/attn/h/xpre (10 * maxB)
  float *x = nullptr, *pin = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr;
  size_t h_floats = 0;  // capacity of h
  float *px = nullptr, *px1 = nullptr, *logits = nullptr, *xpre = nullptr, *hid1 = nullptr;
  // scratch
  float* part = nullptr;
  size_t part_floats = 0;
  unsigned* counters = nullptr;
  size_t n_counters = 0;
  unsigned* counters2 = nullptr;
  unsigned long long* keys = nullptr;
  uint8_t* xs_buf = nullptr;  // input rows split into tensor-core operand tiles (row blocks > 64 rows)
  uint8_t* xs_buf2 = nullptr; // the same, written by the producers of the o and down inputs
  size_t xs_bytes = 0;
  float* apart = nullptr;
  size_t apart_floats = 0;
  unsigned* acounters = nullptr;
  size_t n_acounters = 0;
  int* err_flag = nullptr;
  uint32_t* codes_plain = nullptr;  // [maxB][16]
  // per-call API
  int kvlen0 = 0;
  float* io = nullptr;  // staging [io_floats]
  // per-256-column sums of squares of residual rows (talker, predictor
  // prefill rows, predictor decode rows), row stride kSsqLd
  float *ssq_t = nullptr, *ssq_p = nullptr, *ssq_p1 = nullptr;
  size_t io_floats = 0;
  // generation
  int B = 0, max_frames = 0, max_trail = 0;
  unsigned flags = 0;
  uint32_t* codes = nullptr;
  uint32_t* forced = nullptr;
  float* trail = nullptr;
  float* tts_pad = nullptr;
  float* tp = nullptr;
  float* tp_h1 = nullptr;
  uint32_t* tp_tok = nullptr;
  RowRecipe* recipes = nullptr;
  int* trail_idx = nullptr;
  float* voices = nullptr;
  float* dump_logits = nullptr;
  float* dump_hidden = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  int frame_kernels = 0;
  bool generating = false;
  // Per-generation device buffers (codes, forcing, text rows, dumps, ...),
  // grow-only: a buffer moves only when a generation needs more than it
  // holds, which bumps buf_epoch.  The frame graph bakes in pointers, so it
  // is reused across generations while graph_key (batch, frames, trailing
  // rows, forcing and dumps, buffer epoch) is unchanged.
  struct GenBuf {
    void* p = nullptr;
    size_t bytes = 0;
  };
  static constexpr int kGenBufs = 11;
  GenBuf gen[kGenBufs];
  unsigned long buf_epoch = 0;
  struct GraphKey {
    int B = -1, F = -1, max_trail = -1, forced = 0, dump_logits = 0, dump_hidden = 0;
    unsigned long epoch = 0;
    unsigned long long wait_ns = 0;
    bool operator==(const GraphKey& o) const {
      return B == o.B && F == o.F && max_trail == o.max_trail && forced == o.forced &&
             dump_logits == o.dump_logits && dump_hidden == o.dump_hidden && epoch == o.epoch &&
             wait_ns == o.wait_ns;
    }
  };
  GraphKey graph_key;
  int graph_captures = 0;  // frame graphs captured by this session (cache misses)
  // budget of the one-row GEMV's split-K cluster wait (tests of the timeout
  // path set it short); part of the frame graph's key
  unsigned long long wait_ns = 1000000000ull;
};

}  // namespace qtts
