// engine.cu -- model upload, sessions, launch plans and the C ABI.
//
// The reference decode loop (generate_new.rs:242-300) is expressed as a list
// of kernel launches per frame, built once per generation and captured into a
// CUDA graph; every per-frame quantity (positions, frame index, codes, rng)
// lives in device memory, so the graph replays unchanged frame after frame
// with no host round trip.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <memory>
#include <mutex>
#include <tuple>
#include <cmath>
#include <string>
#include <vector>

#include "engine.h"

namespace qtts {

static thread_local std::string g_err;
void set_error(const std::string& msg) { g_err = msg; }

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define CK(call)                                                                          \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)
#define RC(call)                  \
  do {                            \
    int r_ = (call);              \
    if (r_ != QTTS_OK) return r_; \
  } while (0)

static inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

// generate_new.rs:25-36 token constants
enum : uint32_t {
  IM_START = 151644, ASSISTANT = 77091, NEWLINE = 198, TTS_PAD = 151671, TTS_BOS = 151672,
  TTS_EOS = 151673, CODEC_THINK = 2154, CODEC_THINK_BOS = 2156, CODEC_THINK_EOS = 2157,
  CODEC_PAD = 2148, CODEC_BOS = 2149
};

// ---------------------------------------------------------------------------
// model upload (save.rs:262-409 -> HBM)
// ---------------------------------------------------------------------------
namespace {
struct Piece {
  uint64_t file_off, bytes;
  size_t dev_off;
};
struct Layout {
  size_t total = 0;
  std::vector<Piece> pieces;
  size_t add(uint64_t file_off, uint64_t bytes) {
    const size_t at = total;
    pieces.push_back({file_off, bytes, at});
    total += (bytes + 255) & ~(size_t)255;
    return at;
  }
};
struct WOff {
  size_t a, b;
  int k, n;
};
WOff lay_w(Layout& L, const HWeight& w) { return {L.add(w.off_a, w.bytes_a), L.add(w.off_b, w.bytes_b), (int)w.k, (int)w.n}; }
size_t lay_v(Layout& L, const HVec& v) { return L.add(v.off, v.bytes); }
Q4Mat mk(char* base, const WOff& o) {
  Q4Mat q;
  q.packed = reinterpret_cast<const uint8_t*>(base + o.a);
  q.scales = reinterpret_cast<const __half*>(base + o.b);
  q.k = o.k;
  q.n = o.n;
  return q;
}
struct LOff {
  WOff q, k, v, o, gate, up, down;
  size_t qn, kn, in, post;
};
LOff lay_layer(Layout& L, const HLayer& h) {
  LOff o;
  o.q = lay_w(L, h.q); o.k = lay_w(L, h.k); o.v = lay_w(L, h.v); o.o = lay_w(L, h.o);
  o.qn = lay_v(L, h.q_norm); o.kn = lay_v(L, h.k_norm);
  o.gate = lay_w(L, h.gate); o.up = lay_w(L, h.up); o.down = lay_w(L, h.down);
  o.in = lay_v(L, h.in_norm); o.post = lay_v(L, h.post_norm);
  return o;
}
DLayer mk_layer(char* base, const LOff& o) {
  DLayer d;
  d.q = mk(base, o.q); d.k = mk(base, o.k); d.v = mk(base, o.v); d.o = mk(base, o.o);
  d.gate = mk(base, o.gate); d.up = mk(base, o.up); d.down = mk(base, o.down);
  d.q_norm = reinterpret_cast<const __half*>(base + o.qn);
  d.k_norm = reinterpret_cast<const __half*>(base + o.kn);
  d.in_norm = reinterpret_cast<const __half*>(base + o.in);
  d.post_norm = reinterpret_cast<const __half*>(base + o.post);
  return d;
}
}  // namespace

void gemv_init_attributes();
void attn_init_attributes();

// For batched decode the layer projections (talker and code predictor), the
// codec head and the predictor's input_proj and group heads are expanded once into the
// tensor-core operand layout (4 bytes per weight: ~6 GB for 1.7B, of the
// GPU's 180 GB), so those launches copy operand tiles instead of
// dequantising them; the predictor's are otherwise dequantised 15 times per
// frame.  Optional: without the memory the launches dequantise in the kernel.
static void expand_weights(Model* m) {
  std::vector<Q4Mat*> mats;
  for (auto& L : m->tl)
    for (Q4Mat* w : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down}) mats.push_back(w);
  for (auto& L : m->pl)
    for (Q4Mat* w : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down}) mats.push_back(w);
  if (m->has_proj) mats.push_back(&m->input_proj);
  for (auto& w : m->lm) mats.push_back(&w);
  mats.push_back(&m->codec_head);
  mats.erase(std::remove_if(mats.begin(), mats.end(), [](const Q4Mat* w) { return w->n % 64 != 0; }), mats.end());
  size_t total = 0;
  for (Q4Mat* w : mats) total += (tc_expand_bytes(w->k, w->n) + 255) & ~(size_t)255;
  if (total == 0 || cudaMalloc(&m->wx_arena, total) != cudaSuccess) {
    cudaGetLastError();
    m->wx_arena = nullptr;
    return;
  }
  size_t off = 0;
  bool ok = true;
  for (Q4Mat* w : mats) {
    ok = ok && tc_expand(*w, m->wx_arena + off, nullptr) == cudaSuccess;
    w->wx = m->wx_arena + off;
    off += (tc_expand_bytes(w->k, w->n) + 255) & ~(size_t)255;
  }
  ok = ok && cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {  // fall back to in-kernel dequantisation
    for (Q4Mat* w : mats) w->wx = nullptr;
    cudaFree(m->wx_arena);
    m->wx_arena = nullptr;
    cudaGetLastError();
    return;
  }
  m->wx_bytes = total;
}

static int model_load(const char* path, int device, Model** out) {
  HModel hm;
  std::string err;
  int rc = parse_model(path, &hm, &err);
  if (rc != QTTS_OK) return fail(rc, err);
  if (hm.d.fmt != 1) return fail(QTTS_ERR_FORMAT, "the GPU decode path needs a Q4 model file (format_id 1)");
  if (!hm.has_proj) return fail(QTTS_ERR_FORMAT, "models without predictor input_proj (0.6B) are not supported");
  const qtts_dims& d = hm.d;
  if (d.t_head_dim != kHeadDim || d.p_head_dim != kHeadDim) return fail(QTTS_ERR_FORMAT, "head_dim must be 128");
  if (d.p_groups + 1 > kMaxGroups || d.t_vocab > 4096) return fail(QTTS_ERR_FORMAT, "unsupported vocabulary / group count");
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(QTTS_ERR_NODEV, "no such CUDA device");
  CK(cudaSetDevice(device));
  Layout L;
  std::vector<LOff> tl, pl;
  for (auto& h : hm.tl) tl.push_back(lay_layer(L, h));
  const WOff codec_emb = lay_w(L, hm.codec_emb), text_emb = lay_w(L, hm.text_emb), fc1 = lay_w(L, hm.fc1);
  const size_t fc1_b = lay_v(L, hm.fc1_b);
  const WOff fc2 = lay_w(L, hm.fc2);
  const size_t fc2_b = lay_v(L, hm.fc2_b);
  const WOff codec_head = lay_w(L, hm.codec_head);
  const size_t t_final = lay_v(L, hm.t_final), t_cos = lay_v(L, hm.t_cos), t_sin = lay_v(L, hm.t_sin);
  const WOff input_proj = lay_w(L, hm.input_proj);
  const size_t input_proj_b = lay_v(L, hm.input_proj_b);
  std::vector<WOff> pe, lm;
  for (auto& w : hm.p_emb) pe.push_back(lay_w(L, w));
  for (auto& h : hm.pl) pl.push_back(lay_layer(L, h));
  for (auto& w : hm.lm) lm.push_back(lay_w(L, w));
  const size_t p_final = lay_v(L, hm.p_final), p_cos = lay_v(L, hm.p_cos), p_sin = lay_v(L, hm.p_sin);

  Model* m = new Model();
  m->d = d;
  m->device = device;
  CK(cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, device));
  m->bytes = L.total;
  if (cudaMalloc(&m->arena, L.total) != cudaSuccess) {
    delete m;
    return fail(QTTS_ERR_OOM, "cannot allocate the weight arena");
  }
  // stream payloads file -> pinned staging -> HBM (double-buffered)
  FILE* f = fopen(path, "rb");
  const size_t chunk = 64u << 20;
  void* stage[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaStream_t st = nullptr;
  bool ok = f != nullptr;
  ok = ok && cudaMallocHost(&stage[0], chunk) == cudaSuccess && cudaMallocHost(&stage[1], chunk) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming) == cudaSuccess &&
       cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess;
  int cur = 0;
  bool used[2] = {false, false};
  for (size_t i = 0; ok && i < L.pieces.size(); ++i) {
    const Piece& p = L.pieces[i];
    uint64_t done = 0;
    if (fseeko(f, (off_t)p.file_off, SEEK_SET) != 0) ok = false;
    while (ok && done < p.bytes) {
      const size_t nb = (size_t)std::min<uint64_t>(chunk, p.bytes - done);
      if (used[cur]) ok = cudaEventSynchronize(ev[cur]) == cudaSuccess;
      if (!ok) break;
      if (fread(stage[cur], 1, nb, f) != nb) { ok = false; break; }
      ok = cudaMemcpyAsync(m->arena + p.dev_off + done, stage[cur], nb, cudaMemcpyHostToDevice, st) == cudaSuccess &&
           cudaEventRecord(ev[cur], st) == cudaSuccess;
      used[cur] = true;
      done += nb;
      cur ^= 1;
    }
  }
  if (st) ok = (cudaStreamSynchronize(st) == cudaSuccess) && ok;
  if (f) fclose(f);
  for (int i = 0; i < 2; ++i) {
    if (stage[i]) cudaFreeHost(stage[i]);
    if (ev[i]) cudaEventDestroy(ev[i]);
  }
  if (st) cudaStreamDestroy(st);
  if (!ok) {
    cudaFree(m->arena);
    delete m;
    return fail(QTTS_ERR_IO, "failed to stream the weights to the device");
  }
  char* b = m->arena;
  for (auto& o : tl) m->tl.push_back(mk_layer(b, o));
  for (auto& o : pl) m->pl.push_back(mk_layer(b, o));
  m->codec_emb = mk(b, codec_emb); m->text_emb = mk(b, text_emb); m->fc1 = mk(b, fc1); m->fc2 = mk(b, fc2);
  m->codec_head = mk(b, codec_head); m->input_proj = mk(b, input_proj);
  m->fc1_b = reinterpret_cast<const float*>(b + fc1_b);
  m->fc2_b = reinterpret_cast<const float*>(b + fc2_b);
  m->input_proj_b = reinterpret_cast<const float*>(b + input_proj_b);
  m->t_cos = reinterpret_cast<const float*>(b + t_cos);
  m->t_sin = reinterpret_cast<const float*>(b + t_sin);
  m->p_cos = reinterpret_cast<const float*>(b + p_cos);
  m->p_sin = reinterpret_cast<const float*>(b + p_sin);
  m->t_final = reinterpret_cast<const __half*>(b + t_final);
  m->p_final = reinterpret_cast<const __half*>(b + p_final);
  for (auto& o : pe) m->p_emb.push_back(mk(b, o));
  for (auto& o : lm) m->lm.push_back(mk(b, o));
  m->has_proj = hm.has_proj;
  if (cudaMalloc(&m->d_group_emb, sizeof(Q4Mat) * m->p_emb.size()) != cudaSuccess ||
      cudaMemcpy(m->d_group_emb, m->p_emb.data(), sizeof(Q4Mat) * m->p_emb.size(), cudaMemcpyHostToDevice) !=
          cudaSuccess) {
    cudaFree(m->arena);
    delete m;
    return fail(QTTS_ERR_CUDA, "cannot upload the embedding table list");
  }
  gemv_init_attributes();
  attn_init_attributes();
  tc_init_attributes();
  expand_weights(m);
  *out = m;
  return QTTS_OK;
}

// ---------------------------------------------------------------------------
// launch planning
// ---------------------------------------------------------------------------
static GemvDesc gemv_base(int epi, std::initializer_list<Q4Mat> mats, bool paired, int M) {
  GemvDesc g;
  g.epi_kind = epi;
  g.nmat = (int)mats.size();
  g.paired = paired ? 1 : 0;
  int tiles = 0, cols = 0, i = 0;
  for (const Q4Mat& q : mats) {
    g.mat[i] = q;
    g.tile0[i] = tiles;
    g.col0[i] = cols;
    if (!paired) tiles += ceil_div(q.n, kTileN);
    cols += q.n;
    ++i;
  }
  if (paired) tiles = ceil_div(g.mat[0].n, kTileN);
  g.tile0[g.nmat] = tiles;
  g.ntiles = tiles;
  g.ncols = cols;
  g.k = g.mat[0].k;
  g.M = M;
  return g;
}

// cudaOccupancyMaxActiveClusters per (kernel, cluster size, shared memory,
// block size), cached: planning asks for the same few shapes over and over.
int occupancy_clusters(const void* func, const cudaLaunchConfig_t& cfg) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, unsigned, size_t, unsigned, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  unsigned cy = 1;
  for (unsigned i = 0; i < cfg.numAttrs; ++i)
    if (cfg.attrs[i].id == cudaLaunchAttributeClusterDimension) cy = cfg.attrs[i].val.clusterDim.y;
  const auto key = std::make_tuple(func, cy, cfg.dynamicSmemBytes, cfg.blockDim.x, dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, func, &cfg) != cudaSuccess) n = 0;
  cudaGetLastError();
  cache[key] = n;
  return n;
}

// Clusters of g's launch (as launch_gemv would issue it) that fit at once.
int gemv_wave_clusters(const GemvDesc& g) {
  g_occ_query = true;
  g_occ_clusters = 0;
  launch_gemv(g, FrameCodes{}, nullptr);
  g_occ_query = false;
  return g_occ_clusters;
}

// With a cluster-reduced K split, every (tile, row block) is one cluster and
// all of them should be resident in one wave: lower S until they fit.
static void fit_split_to_wave(GemvDesc& g) {
  if (g.tc || !g.cluster) return;
  const long units = (long)g.ntiles * ceil_div(g.M, g.mb);
  for (int S = g.S; S >= 1; --S) {
    GemvDesc t = g;
    const int rps = std::min(ceil_div(ceil_div(g.k, S), 32) * 32, 2048);
    t.rows_per_split = rps;
    t.S = ceil_div(g.k, rps);
    if (t.S > S) continue;
    if (gemv_wave_clusters(t) >= units) {
      g = t;
      return;
    }
  }
}

// Batches of 3..15 rows (q4mv_batch_kernel): 8 input rows per CTA (4 for a
// gate/up pair), K slices of whole 8-row steps of at most kBatchMaxRpsNM1/NM2 rows,
// the slices of a tile in one cluster.  Starting from about two CTAs per SM,
// the largest split whose clusters all fit in one wave.
static void batch_plan(int sm_count, GemvDesc& g) {
  if (g.tc || g.M <= kDecMaxM || g.M >= kTcMinRows || g.attn_in || g.x_glu) return;
  GemvDesc t = g;
  t.batch = 1;
  t.cluster = 1;
  t.mb = g.paired ? kBatchRowsNM2 : kBatchRowsNM1;
  const long units = (long)t.ntiles * ceil_div(t.M, t.mb);
  int S0 = (int)std::lround(2.0 * sm_count / (double)units);
  S0 = std::max(1, std::min(S0, kMaxClusterSplits));
  for (int S = S0; S >= 1; --S) {
    t.rows_per_split = ceil_div(ceil_div(g.k, S), 8) * 8;
    if (t.rows_per_split > (g.paired ? kBatchMaxRpsNM2 : kBatchMaxRpsNM1)) return;  // a smaller split only grows it
    t.S = ceil_div(g.k, t.rows_per_split);
    if (t.S > S) continue;
    if (S == 1 || gemv_wave_clusters(t) >= units) {
      g = t;
      return;
    }
  }
}

// Split-K choice: about two CTAs per SM, slices of whole 32-row blocks, at
// most 2048 rows per slice (shared-memory bound of the input slice).
void choose_split(int sm_count, GemvDesc& g) {
  // up to kDecMaxM rows: one row per CTA (the decode kernel's grid.z)
  g.mb = g.M <= kDecMaxM ? 1 : (g.paired ? 2 : 4);
  const int zb = ceil_div(g.M, g.mb);
  const int target = 2 * sm_count;
  int S = (int)std::lround((double)target / (double)(g.ntiles * zb));
  S = std::max(1, std::min(std::min(S, kMaxClusterSplits), ceil_div(g.k, 32)));
  int rps = ceil_div(ceil_div(g.k, S), 32) * 32;
  rps = std::min(rps, 2048);
  g.rows_per_split = rps;
  g.S = ceil_div(g.k, rps);
}

template <class T>
static int dalloc(T** p, size_t count, std::vector<void*>* track = nullptr) {
  if (count == 0) count = 1;
  if (cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * count) != cudaSuccess)
    return fail(QTTS_ERR_OOM, "device allocation failed");
  if (cudaMemset(*p, 0, sizeof(T) * count) != cudaSuccess) return fail(QTTS_ERR_CUDA, "cudaMemset failed");
  if (track) track->push_back(*p);
  return QTTS_OK;
}

// Decode rows whose register-resident K slices fit the decode kernel only
// with more clusters than one wave holds (the talker's gate/up pair): keep
// about two CTAs per SM and reduce the slices through global memory (the
// last CTA of a tile to arrive sums them) instead of a cluster, which frees
// the CTAs from cluster placement.
static void try_global_split(Session& s, GemvDesc& g) {
  if (g.M > kDecMaxM || g.tc || gemv_uses_decode_kernel(g)) return;
  GemvDesc t = g;
  choose_split(s.m->sm_count, t);
  t.cluster = 0;
  const int nrmax = t.paired ? kDecRowsNM2 : kDecRowsNM1;
  while (t.rows_per_split > 32 * nrmax && t.S < kMaxGlobalSplits) {
    const int S = t.S + 1;
    t.rows_per_split = ceil_div(ceil_div(t.k, S), 32) * 32;
    t.S = ceil_div(t.k, t.rows_per_split);
  }
  t.part = s.part;
  if (!gemv_uses_decode_kernel(t) || (size_t)t.S * t.M * t.ncols > s.part_floats ||
      (size_t)t.ntiles * t.M > s.n_counters)
    return;
  if (gemv_uses_decode_kernel(g) && (long)t.ntiles * t.S <= (long)g.ntiles * g.S) return;
  g = t;
}

static int plan_gemv(Session& s, GemvDesc& g) {
  choose_split(s.m->sm_count, g);
  g.cluster = 1;  // split-K partials reduced over distributed shared memory
  g.pdl = 1;
  fit_split_to_wave(g);
  try_global_split(s, g);
  batch_plan(s.m->sm_count, g);
  g.err_flag = s.err_flag;
  g.wait_ns = s.wait_ns;
  if (g.M >= kTcMinRows) {
    tc_plan(s.m->sm_count, g);  // one tcgen05 kernel: prologue, GEMM, split-K, epilogue
    g.part = s.part;
    g.xs_buf = s.xs_buf;
    g.xs_bytes = s.xs_bytes;
    const size_t zt = (size_t)ceil_div(g.M, kTcRows);
    if (tc_splits(g) > 1 &&
        ((size_t)tc_splits(g) * g.M * g.ncols > s.part_floats || 2 * (size_t)g.ntiles * zt > s.n_counters))
      return fail(QTTS_ERR_OOM, "split-K scratch too small for this projection");
  }
  // the CUDA-core kernels' tile counters (the tensor-core kernel's are checked above)
  const size_t zb = (size_t)ceil_div(g.M, g.mb);
  if (!g.tc && ((size_t)g.ntiles * zb > s.n_counters || zb > 4096))
    return fail(QTTS_ERR_OOM, "tile counter array too small");
  g.counters = s.counters;
  if (g.epi_kind == EPI_ARGMAX) {
    g.epi.counters2 = s.counters2;
    g.epi.keys = s.keys;
  }
  return QTTS_OK;
}

// The projection planned last in the current op list: the next one planned
// fills in its L2-prefetch targets (GemvDesc::pf_*), so every projection
// pulls its successor's weights into L2 while it runs.
static thread_local std::shared_ptr<GemvDesc> g_prev_gemv;
static void chain_reset() { g_prev_gemv.reset(); }

static Op gemv_op(const GemvDesc& g, const FrameCodes& fc = FrameCodes{}) {
  auto sp = std::make_shared<GemvDesc>(g);
  // A launch that streams expanded tiles (4 bytes a weight) reads no Q4
  // bytes, and prefetching its tiles measured slower than none (config 5:
  // 24.0k with those of at most 32 MB, 24.9k with none; config 4 9.04k vs
  // 9.15k): its predecessor prefetches nothing.
  if (g_prev_gemv && !tc_reads_expanded(g)) {
    GemvDesc& p = *g_prev_gemv;
    const int nm = g.paired ? 2 : g.nmat;
    for (int i = 0; i < nm && i < 3; ++i) {
      const Q4Mat& w = g.mat[i];
      p.pf_ptr[2 * i] = w.packed;
      p.pf_bytes[2 * i] = (uint32_t)((size_t)w.k * w.n / 2);
      p.pf_ptr[2 * i + 1] = reinterpret_cast<const uint8_t*>(w.scales);
      p.pf_bytes[2 * i + 1] = (uint32_t)(((size_t)w.k * w.n / 32 * 2) & ~(size_t)15);
    }
  }
  g_prev_gemv = sp;
  return [sp, fc](cudaStream_t st) { return launch_gemv(*sp, fc, st); };
}

struct LayerIO {
  float* X = nullptr;
  long ldx = 0;
  int M = 0;
  RowPos rp;
  KvDesc kv;
  const float *cos = nullptr, *sin = nullptr;
  int rope_rows = 0, skip_oob = 0;
  int heads = 0, kvh = 0, inter = 0;
  int nsplit = 1;
  // per-256-column sums of squares of the residual rows (row stride kSsqLd):
  // written by every residual epilogue, read by the next RMSNorm prologue;
  // ssq_valid = 0 when the input rows came without them (host copies)
  float* ssq = nullptr;
  int ssq_valid = 0;
  // M = 1 with a short cache (the predictor): attention folded into the
  // o_proj kernel's input prologue when its K split is one head per slice
  int fuse_attn = 0;
};

// One transformer layer (talker.rs:279-349 / code_predictor.rs:448-502):
// RMSNorm+QKV+QK-norm+RoPE+KV append | attention | O+residual |
// RMSNorm+gate/up+SwiGLU | down+residual.
static int add_layer(Session& s, std::vector<Op>& ops, const DLayer& L, const LayerIO& io) {
  const int qd = io.heads * kHeadDim;
  const int nt = ceil_div(io.ldx > 0 ? L.q.k : 0, kSsqCols);  // sum-of-squares blocks of a residual row
  auto use_ssq = [&](GemvDesc& gd, bool valid) {
    if (io.ssq && valid) {
      gd.ssq_in = io.ssq; gd.ssq_ld = kSsqLd; gd.ssq_n = nt;
    }
  };
  auto emit_ssq = [&](GemvDesc& gd) {
    if (io.ssq) {
      gd.epi.ssq_out = io.ssq; gd.epi.ssq_ld = kSsqLd;
    }
  };
  GemvDesc g = gemv_base(EPI_QKV, {L.q, L.k, L.v}, false, io.M);
  g.X = io.X; g.ldx = io.ldx; g.gamma = L.in_norm;
  use_ssq(g, io.ssq_valid != 0);
  g.epi.q_out = s.q; g.epi.ldq = qd; g.epi.q_norm = L.q_norm; g.epi.k_norm = L.k_norm;
  g.epi.rope_cos = io.cos; g.epi.rope_sin = io.sin; g.epi.rope_rows = io.rope_rows; g.epi.rope_skip_oob = io.skip_oob;
  g.epi.heads = io.heads; g.epi.kv_heads = io.kvh; g.epi.kv = io.kv; g.epi.rp = io.rp; g.epi.err_flag = s.err_flag;
  RC(plan_gemv(s, g));
  ops.push_back(gemv_op(g));

  GemvDesc o = gemv_base(EPI_RESID, {L.o}, false, io.M);
  o.X = s.attn; o.ldx = qd; o.epi.out = io.X; o.epi.ldo = io.ldx;
  emit_ssq(o);
  RC(plan_gemv(s, o));
  const bool fused = io.fuse_attn && io.M <= kDecMaxM && !o.tc && o.rows_per_split == kHeadDim && o.S * kHeadDim == qd &&
                     gemv_uses_decode_kernel(o);
  if (fused) {
    o.attn_in = 1; o.attn_q = s.q; o.attn_ldq = qd; o.attn_kv = io.kv; o.attn_rp = io.rp;
    o.attn_group = io.heads / io.kvh;
  } else {
    AttnDesc a;
    a.q = s.q; a.ldq = qd; a.out = s.attn; a.ldo = qd; a.kv = io.kv; a.rp = io.rp;
    a.heads = io.heads; a.kv_heads = io.kvh; a.M = io.M; a.nsplit = io.nsplit;
    // The early L2 prefetch of the K / V rows helps while everything it pulls
    // stays resident until read (small batches, long caches).  With many rows
    // the launch's cache (up to M * kv_heads * maxP positions, K and V of
    // 512 bytes each) exceeds L2 and prefetched lines evict each other first.
    a.l2_prefetch = (double)io.M * io.kvh * s.maxP * 2.0 * kHeadDim * (s.kv_f16 ? 2 : 4) <= kAttnPrefetchMaxBytes;
    if (a.nsplit > 1) {
      const size_t need = (size_t)io.M * io.kvh * a.nsplit * (io.heads / io.kvh) * kAttnRec;
      if (need > s.apart_floats || (size_t)io.M * io.kvh > s.n_acounters)
        return fail(QTTS_ERR_OOM, "attention split scratch too small");
      a.part = s.apart;
      a.counters = s.acounters;
    }
    // o on split input rows (tensor cores, > 64 rows): the attention writes them
    if (a.nsplit == 1 && s.xs_buf2 && tc_takes_split_from_producer(o)) {
      a.xs_out = s.xs_buf2;
      a.err_flag = s.err_flag;
      o.x_split_pre = s.xs_buf2;
    }
    ops.push_back([a](cudaStream_t st) { return launch_attention(a, st); });
  }
  ops.push_back(gemv_op(o));

  GemvDesc dn = gemv_base(EPI_RESID, {L.down}, false, io.M);
  dn.X = s.h; dn.ldx = io.inter; dn.epi.out = io.X; dn.epi.ldo = io.ldx;
  emit_ssq(dn);
  RC(plan_gemv(s, dn));

  // One decode row: gate and up as two matrices of one launch (twice the
  // tiles, so more K slices fit the decode kernel's registers), SiLU on the
  // gate columns in its epilogue, the product silu(gate) * up taken by the
  // down projection's prologue (x_glu).  Otherwise the paired SwiGLU launch.
  GemvDesc gs = gemv_base(EPI_STORE, {L.gate, L.up}, false, io.M);
  gs.X = io.X; gs.ldx = io.ldx; gs.gamma = L.post_norm; gs.epi.out = s.h; gs.epi.ldo = 2L * io.inter;
  gs.epi.act_silu = 1;  // matrix 0 = gate
  use_ssq(gs, true);
  bool split_glu = false;
  if (io.M <= kDecMaxM && (size_t)2 * io.inter * io.M <= s.h_floats) {
    RC(plan_gemv(s, gs));
    GemvDesc dg = dn;
    dg.x_glu = io.inter;
    dg.ldx = 2L * io.inter;
    split_glu = gemv_uses_decode_kernel(gs) && gemv_uses_decode_kernel(dg);
    if (split_glu) dn = dg;
  }
  if (split_glu) {
    ops.push_back(gemv_op(gs));
  } else {
    GemvDesc gu = gemv_base(EPI_SWIGLU, {L.gate, L.up}, true, io.M);
    gu.X = io.X; gu.ldx = io.ldx; gu.gamma = L.post_norm; gu.epi.out = s.h; gu.epi.ldo = io.inter;
    use_ssq(gu, true);
    RC(plan_gemv(s, gu));
    // down on split input rows: the gate/up epilogue writes them (its own
    // input rows come split from the other buffer)
    if (gu.tc && s.xs_buf2 && tc_takes_split_from_producer(dn)) {
      gu.xs_out = s.xs_buf2;
      gu.xs_out_k = io.inter;
      dn.x_split_pre = s.xs_buf2;
    }
    ops.push_back(gemv_op(gu));
  }
  ops.push_back(gemv_op(dn));
  return QTTS_OK;
}

static KvDesc talker_kv(Session& s, int layer) {
  KvDesc k;
  k.pool = s.kv_pool; k.page_table = s.page_table; k.pages_per_sess = s.pages_per_sess;
  k.n_layers = s.m->d.t_layers; k.kv_heads = s.m->d.t_kv_heads; k.layer = layer; k.f16 = s.kv_f16;
  return k;
}
static KvDesc pred_kv(Session& s, int layer) {
  KvDesc k;
  k.pool = s.pkv_pool; k.page_table = nullptr; k.pages_per_sess = 1;
  k.n_layers = s.m->d.p_layers; k.kv_heads = s.m->d.p_kv_heads; k.layer = layer; k.f16 = s.kv_f16;
  return k;
}
// Attention splits of the talker cache: 32 positions per split, about four
// CTAs per SM at most.
static int talker_nsplit(Session& s, int M) {
  const int byL = ceil_div(s.maxP, 32);
  const int byPar = std::max(1, ceil_div(4L * s.m->sm_count, (long)M * s.m->d.t_kv_heads));
  return std::max(1, std::min(kMaxClusterSplits, std::min(byL, byPar)));
}

// Talker layers over rows X (decode: one row per session; prefill: seq rows).
// ssq0: sums of squares of the input rows when their producer left them.
static int add_talker(Session& s, std::vector<Op>& ops, float* X, long ldx, int M, const RowPos& rp, int nsplit,
                      bool ssq0) {
  const Model& m = *s.m;
  for (int l = 0; l < m.d.t_layers; ++l) {
    LayerIO io;
    io.X = X; io.ldx = ldx; io.M = M; io.rp = rp; io.kv = talker_kv(s, l);
    io.cos = m.t_cos; io.sin = m.t_sin; io.rope_rows = m.d.t_max_pos; io.skip_oob = 0;
    io.heads = m.d.t_heads; io.kvh = m.d.t_kv_heads; io.inter = m.d.t_inter; io.nsplit = nsplit;
    io.ssq = s.ssq_t;
    io.ssq_valid = (l > 0 || ssq0) ? 1 : 0;
    RC(add_layer(s, ops, m.tl[l], io));
  }
  return QTTS_OK;
}

// final norm + codec_head (talker.rs:353-354): logits and the normed hidden.
// Rows X are the talker residual rows whose sums of squares are in s.ssq_t
// (row r of X <-> ssq row ssq_row0 + r * ssq_rows_step).
static int add_codec_head(Session& s, std::vector<Op>& ops, const float* X, long ldx, int M, float* logits,
                          float* hid, long ldh, long ssq_row0 = 0, long ssq_rows_step = 1) {
  GemvDesc g = gemv_base(EPI_STORE, {s.m->codec_head}, false, M);
  g.X = X; g.ldx = ldx; g.gamma = s.m->t_final;
  g.ssq_in = s.ssq_t + ssq_row0 * kSsqLd; g.ssq_ld = ssq_rows_step * kSsqLd; g.ssq_n = ceil_div(s.m->d.t_hidden, kSsqCols);
  g.epi.out = logits; g.epi.ldo = s.m->d.t_vocab;
  g.xnorm_out = hid; g.ld_xnorm = ldh;
  RC(plan_gemv(s, g));
  ops.push_back(gemv_op(g));
  return QTTS_OK;
}

// Predictor expansion for B sessions (code_predictor.rs:218-273).  Inputs:
// s.pin rows (2b = talker hidden, 2b+1 = semantic embedding).  Codes go
// through FrameCodes (generation) or s.codes_plain (per-call API).
static int add_predictor(Session& s, std::vector<Op>& ops, int B, bool frame_mode, const FrameCodes& fc) {
  const Model& m = *s.m;
  const qtts_dims& d = m.d;
  const int pH = d.p_hidden;
  // project_input of both prefill rows (code_predictor.rs:235-236)
  const int pnt = ceil_div(pH, kSsqCols);
  GemvDesc pj = gemv_base(EPI_STORE, {m.input_proj}, false, 2 * B);
  pj.X = s.pin; pj.ldx = d.t_hidden; pj.epi.out = s.px; pj.epi.ldo = pH; pj.epi.bias = m.input_proj_b;
  pj.epi.ssq_out = s.ssq_p; pj.epi.ssq_ld = kSsqLd;
  RC(plan_gemv(s, pj));
  ops.push_back(gemv_op(pj));
  auto layers = [&](float* X, int M, const RowPos& rp, float* ssq) -> int {
    for (int l = 0; l < d.p_layers; ++l) {
      LayerIO io;
      io.X = X; io.ldx = pH; io.M = M; io.rp = rp; io.kv = pred_kv(s, l);
      io.cos = m.p_cos; io.sin = m.p_sin; io.rope_rows = d.p_max_pos; io.skip_oob = 1;
      io.heads = d.p_heads; io.kvh = d.p_kv_heads; io.inter = d.p_inter; io.nsplit = 1;
      io.ssq = ssq; io.ssq_valid = 1;  // every input row comes from a projection epilogue
      io.fuse_attn = (M <= kDecMaxM && d.p_groups + 1 <= kAttnInMaxPos) ? 1 : 0;
      RC(add_layer(s, ops, m.pl[l], io));
    }
    return QTTS_OK;
  };
  RowPos rp0;
  rp0.rows_per_sess = 2;  // prefill positions 0, 1 (code_predictor.rs:244, :369)
  RC(layers(s.px, 2 * B, rp0, s.ssq_p));
  auto head = [&](const float* X, long ldx, int g, const float* ssq, long ssq_ld) -> int {
    // final norm + lm_heads[g] + argmax
    GemvDesc h = gemv_base(EPI_ARGMAX, {m.lm[g]}, false, B);
    h.X = X; h.ldx = ldx; h.gamma = m.p_final;
    h.ssq_in = ssq; h.ssq_ld = ssq_ld; h.ssq_n = pnt;
    h.epi.group = g + 1; h.epi.frame_codes = frame_mode ? 1 : 0; h.epi.codes_plain = s.codes_plain;
    RC(plan_gemv(s, h));
    ops.push_back(gemv_op(h, fc));
    return QTTS_OK;
  };
  RC(head(s.px + pH, 2L * pH, 0, s.ssq_p + kSsqLd, 2L * kSsqLd));
  for (int g = 1; g < d.p_groups; ++g) {  // code_predictor.rs:253-270
    GemvDesc pe = gemv_base(EPI_STORE, {m.input_proj}, false, B);
    pe.emb = m.p_emb[g - 1];
    if (frame_mode) {
      pe.emb_idx = &s.slots[0].cur[g];
      pe.emb_idx_stride = (int)(sizeof(SlotState) / sizeof(uint32_t));
    } else {
      pe.emb_idx = s.codes_plain + g;
      pe.emb_idx_stride = kMaxGroups;
    }
    pe.epi.out = s.px1; pe.epi.ldo = pH; pe.epi.bias = m.input_proj_b;
    pe.epi.ssq_out = s.ssq_p1; pe.epi.ssq_ld = kSsqLd;
    RC(plan_gemv(s, pe));
    ops.push_back(gemv_op(pe));
    RowPos rp;
    rp.pos_const = g + 1;
    RC(layers(s.px1, B, rp, s.ssq_p1));
    RC(head(s.px1, pH, g, s.ssq_p1, kSsqLd));
  }
  return QTTS_OK;
}

// embed_text_token for rows of token ids (talker.rs:105-116):
// fc1(emb) + b1 -> silu -> fc2 + b2.
static int add_text_proj(Session& s, std::vector<Op>& ops, const uint32_t* tok_dev, int n, float* h1, float* out,
                         long ldo) {
  const Model& m = *s.m;
  GemvDesc g1 = gemv_base(EPI_STORE, {m.fc1}, false, n);
  g1.emb = m.text_emb; g1.emb_idx = tok_dev; g1.emb_idx_stride = 1;
  g1.epi.out = h1; g1.epi.ldo = m.fc1.n; g1.epi.bias = m.fc1_b; g1.epi.act_silu = 1;
  RC(plan_gemv(s, g1));
  ops.push_back(gemv_op(g1));
  GemvDesc g2 = gemv_base(EPI_STORE, {m.fc2}, false, n);
  g2.X = h1; g2.ldx = m.fc1.n;
  g2.epi.out = out; g2.epi.ldo = ldo; g2.epi.bias = m.fc2_b;
  RC(plan_gemv(s, g2));
  ops.push_back(gemv_op(g2));
  return QTTS_OK;
}

static int run_ops(Session& s, const std::vector<Op>& ops) {
  chain_reset();  // the next op list starts its own prefetch chain
  for (size_t i = 0; i < ops.size(); ++i) {
    const cudaError_t e = ops[i](s.st);
    if (e != cudaSuccess)
      return fail(QTTS_ERR_CUDA, "kernel launch (op " + std::to_string(i) + " of " + std::to_string(ops.size()) +
                                     "): " + cudaGetErrorString(e));
  }
  return QTTS_OK;
}
static int sync_check(Session& s) {
  CK(cudaStreamSynchronize(s.st));
  int flag = 0;
  CK(cudaMemcpy(&flag, s.err_flag, sizeof(int), cudaMemcpyDeviceToHost));
  if (flag) {
    CK(cudaMemset(s.err_flag, 0, sizeof(int)));
    if (flag & kErrRopeRange) return fail(QTTS_ERR_RANGE, "position beyond the talker RoPE table (rope.rs:73 would panic)");
    if (flag & kErrFp16Input) return fail(QTTS_ERR_RANGE, "tensor-core input outside the fp16 range");
    return fail(QTTS_ERR_TIMEOUT, "a bounded device wait expired (cluster peer, pipeline or grid barrier)");
  }
  return QTTS_OK;
}

// ---------------------------------------------------------------------------
// sessions
// ---------------------------------------------------------------------------

// Ends the generation in progress.  Its buffers and captured frame graph stay
// for the next generation of the same shape.
static void free_generation(Session& s) { s.generating = false; }

static void destroy_graph(Session& s) {
  if (s.graph_exec) cudaGraphExecDestroy(s.graph_exec);
  if (s.graph) cudaGraphDestroy(s.graph);
  s.graph_exec = nullptr;
  s.graph = nullptr;
  s.graph_key = Session::GraphKey{};
  s.frame_kernels = 0;
}

// Grow-only per-generation buffer `slot` of at least `bytes`.
static int gen_buf(Session& s, int slot, size_t bytes, void** out) {
  Session::GenBuf& b = s.gen[slot];
  bytes = std::max<size_t>(bytes, 16);
  if (bytes > b.bytes) {
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.bytes = 0;
    ++s.buf_epoch;
    if (cudaMalloc(&b.p, bytes) != cudaSuccess) return fail(QTTS_ERR_OOM, "device allocation failed");
    b.bytes = bytes;
  }
  *out = b.p;
  return QTTS_OK;
}
template <class T>
static int gen_alloc(Session& s, int slot, T** p, size_t count) {
  void* v = nullptr;
  RC(gen_buf(s, slot, sizeof(T) * count, &v));
  *p = static_cast<T*>(v);
  return QTTS_OK;
}

static void session_free_all(Session* s) {
  if (!s) return;
  cudaSetDevice(s->m->device);
  if (s->st) cudaStreamSynchronize(s->st);
  free_generation(*s);
  destroy_graph(*s);
  for (auto& b : s->gen)
    if (b.p) cudaFree(b.p);
  void* bufs[] = {s->kv_pool, s->page_table, s->pkv_pool, s->slots, s->x, s->pin, s->q, s->attn, s->h,
                  s->px, s->px1, s->logits, s->xpre, s->hid1, s->part, s->counters, s->counters2, s->keys,
                  s->apart, s->acounters, s->err_flag, s->codes_plain, s->io, s->ssq_t, s->ssq_p, s->ssq_p1,
                  s->xs_buf, s->xs_buf2};
  for (void* p : bufs)
    if (p) cudaFree(p);
  if (s->st) cudaStreamDestroy(s->st);
  delete s;
}

static int session_create(Model* m, int maxB, int maxP, unsigned flags, Session** out) {
  if (!m || maxB <= 0 || maxB > 4096 || maxP <= 0) return fail(QTTS_ERR_BADARG, "bad session arguments");
  if (flags & ~(unsigned)QTTS_SESSION_KV_F16) return fail(QTTS_ERR_BADARG, "unknown session flags");
  if (maxP > m->d.t_max_pos) return fail(QTTS_ERR_RANGE, "max_positions exceeds the talker RoPE table");
  CK(cudaSetDevice(m->device));
  const qtts_dims& d = m->d;
  Session* s = new Session();
  s->m = m;
  s->maxB = maxB;
  s->maxP = maxP;
  s->pages_per_sess = ceil_div(maxP, kPageSize);
  s->kv_f16 = (flags & QTTS_SESSION_KV_F16) ? 1 : 0;
  int rc = QTTS_OK;
  auto A = [&](auto** p, size_t n) {
    if (rc == QTTS_OK) rc = dalloc(p, n);
  };
  if (cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking) != cudaSuccess) rc = fail(QTTS_ERR_CUDA, "stream");
  const size_t tpage = (size_t)d.t_layers * 2 * d.t_kv_heads * kPageSize * kHeadDim;
  const size_t ppage = (size_t)d.p_layers * 2 * d.p_kv_heads * kPageSize * kHeadDim;
  const size_t kv_div = s->kv_f16 ? 2 : 1;  // f16 elements: two per float of the allocation
  A(&s->kv_pool, tpage * maxB * s->pages_per_sess / kv_div);
  A(&s->page_table, (size_t)maxB * s->pages_per_sess);
  A(&s->pkv_pool, ppage * maxB / kv_div);
  A(&s->slots, (size_t)maxB);
  s->rows = 10 * maxB;
  const int qmax = std::max(d.t_heads, d.p_heads) * kHeadDim;
  const int imax = std::max(d.t_inter, d.p_inter);
  A(&s->x, (size_t)maxB * d.t_hidden);
  A(&s->pin, (size_t)maxB * 2 * d.t_hidden);
  A(&s->q, (size_t)s->rows * qmax);
  A(&s->attn, (size_t)s->rows * qmax);
  A(&s->h, (size_t)s->rows * imax);
  s->h_floats = (size_t)s->rows * imax;
  A(&s->px, (size_t)2 * maxB * d.p_hidden);
  A(&s->px1, (size_t)maxB * d.p_hidden);
  A(&s->logits, (size_t)maxB * d.t_vocab);
  A(&s->xpre, (size_t)s->rows * d.t_hidden);
  A(&s->hid1, (size_t)maxB * d.t_hidden);
  s->part_floats = (size_t)16 << 20;
  A(&s->part, s->part_floats);
  s->n_counters = 1 << 18;
  A(&s->counters, s->n_counters);
  A(&s->counters2, (size_t)4096);
  A(&s->keys, (size_t)std::max(maxB * 10, 4096));
  s->apart_floats = (size_t)8 << 20;
  A(&s->apart, s->apart_floats);
  // split input-row tiles for the frame's tensor-core launches (up to 2 rows
  // per utterance, at most 1024 rows; larger launches split their rows in
  // the kernel): 128-row blocks x 64-deep stages x 32 KB (fp16 hi + lo),
  // over the widest input of any projection (two buffers: the split kernel
  // fills one, while the producers of the o and down inputs, attention and
  // the gate/up epilogue, write the other)
  if (2 * maxB > 64) {
    const int xrows = std::min(2 * maxB, 1024);
    const int kmax = std::max(std::max(imax, qmax), std::max(d.t_hidden, d.p_hidden));
    s->xs_bytes = (size_t)ceil_div(xrows, 128) * ceil_div(kmax, 64) * 32768;
    A(&s->xs_buf, s->xs_bytes);
    A(&s->xs_buf2, s->xs_bytes);
  }
  s->n_acounters = (size_t)s->rows * std::max(d.t_kv_heads, d.p_kv_heads);
  A(&s->acounters, s->n_acounters);
  A(&s->err_flag, (size_t)1);
  A(&s->codes_plain, (size_t)maxB * kMaxGroups);
  s->io_floats = (size_t)s->rows * d.t_hidden + 2 * d.t_hidden + d.t_vocab + 64;
  A(&s->io, s->io_floats);
  A(&s->ssq_t, (size_t)s->rows * kSsqLd);
  A(&s->ssq_p, (size_t)2 * maxB * kSsqLd);
  A(&s->ssq_p1, (size_t)maxB * kSsqLd);
  if (rc == QTTS_OK) {  // pages: slot b owns pages [b*pps, (b+1)*pps)
    std::vector<int> pt((size_t)maxB * s->pages_per_sess);
    for (size_t i = 0; i < pt.size(); ++i) pt[i] = (int)i;
    if (cudaMemcpy(s->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice) != cudaSuccess)
      rc = fail(QTTS_ERR_CUDA, "page table upload");
  }
  if (rc != QTTS_OK) {
    std::string msg = g_err;
    session_free_all(s);
    return fail(rc, msg);
  }
  *out = s;
  return QTTS_OK;
}

// ---------------------------------------------------------------------------
// generation (generate_new.rs:191-300)
// ---------------------------------------------------------------------------
static int build_frame_ops(Session& s, std::vector<Op>& ops, bool dumps) {
  chain_reset();
  const Model& m = *s.m;
  const qtts_dims& d = m.d;
  const int B = s.B, H = d.t_hidden, V = d.t_vocab;
  FrameCodes fc;
  fc.slots = s.slots; fc.codes = s.codes; fc.forced = s.forced; fc.max_frames = s.max_frames;
  SlotState* slots = s.slots;
  const int F = s.max_frames;
  if (dumps) {
    float* dl = s.dump_logits;
    float* dh = s.dump_hidden;
    const float* lg = s.logits;
    const float* pin = s.pin;
    if (dl) ops.push_back([=](cudaStream_t st) { return launch_dump(slots, B, lg, V, V, dl, F, st); });
    if (dh) ops.push_back([=](cudaStream_t st) { return launch_dump(slots, B, pin, 2L * H, H, dh, F, st); });
  }
  SampleDesc sd;
  sd.logits = s.logits; sd.ldl = V; sd.V = V; sd.B = B; sd.fc = fc;
  ops.push_back([sd](cudaStream_t st) { return launch_sample(sd, st); });
  const Q4Mat ce = m.codec_emb;
  float* sem = s.pin + H;
  ops.push_back([=](cudaStream_t st) { return launch_embed_code0(ce, slots, B, sem, 2L * H, st); });
  RC(add_predictor(s, ops, B, true, fc));
  FuseDesc fd;
  fd.x = s.x; fd.ldx = H; fd.codec_emb = m.codec_emb; fd.group_emb = m.d_group_emb; fd.n_groups = d.p_groups;
  fd.trail = s.trail; fd.max_trail = s.max_trail; fd.tts_pad = s.tts_pad; fd.B = B; fd.H = H; fd.fc = fc;
  fd.ssq_out = s.ssq_t; fd.ssq_ld = kSsqLd;
  ops.push_back([fd](cudaStream_t st) { return launch_fuse(fd, st); });
  RowPos rp;
  rp.pos_base = &s.slots[0].pos;
  rp.pos_stride = (int)(sizeof(SlotState) / sizeof(int));
  RC(add_talker(s, ops, s.x, H, B, rp, talker_nsplit(s, B), true));
  RC(add_codec_head(s, ops, s.x, H, B, s.logits, s.pin, 2L * H));
  ops.push_back([slots, B](cudaStream_t st) { return launch_frame_end(slots, B, st); });
  return QTTS_OK;
}

// Grow the row-sized session buffers (prefill rows: activations, queries,
// attention output, FFN hidden, sums of squares, attention counters, staging)
// to `rows`.  Only between generations: no captured graph refers to them.
static int ensure_rows(Session& s, int rows) {
  if (rows <= s.rows) return QTTS_OK;
  const qtts_dims& d = s.m->d;
  const int qmax = std::max(d.t_heads, d.p_heads) * kHeadDim;
  const int imax = std::max(d.t_inter, d.p_inter);
  float** bufs[] = {&s.q, &s.attn, &s.h, &s.xpre, &s.io, &s.ssq_t};
  for (float** b : bufs) {
    cudaFree(*b);
    *b = nullptr;
  }
  cudaFree(s.acounters);
  s.acounters = nullptr;
  s.rows = rows;
  ++s.buf_epoch;  // a cached frame graph refers to the old buffers
  RC(dalloc(&s.q, (size_t)rows * qmax));
  RC(dalloc(&s.attn, (size_t)rows * qmax));
  RC(dalloc(&s.h, (size_t)rows * imax));
  s.h_floats = (size_t)rows * imax;
  RC(dalloc(&s.xpre, (size_t)rows * d.t_hidden));
  s.io_floats = (size_t)rows * d.t_hidden + 2 * d.t_hidden + d.t_vocab + 64;
  RC(dalloc(&s.io, s.io_floats));
  RC(dalloc(&s.ssq_t, (size_t)rows * kSsqLd));
  s.n_acounters = (size_t)rows * std::max(d.t_kv_heads, d.p_kv_heads);
  RC(dalloc(&s.acounters, s.n_acounters));
  return QTTS_OK;
}

static int generate_begin(Session& s, int n, const qtts_utterance* u, int F, unsigned flags, const uint32_t* forced,
                          bool dump_logits, bool dump_hidden) {
  const Model& m = *s.m;
  const qtts_dims& d = m.d;
  if (n <= 0 || n > s.maxB || !u || F <= 0) return fail(QTTS_ERR_BADARG, "bad generate arguments");
  const bool full_prompt = (flags & QTTS_FULL_PROMPT) != 0;
  int max_prefill = 10;
  for (int b = 0; b < n; ++b)
    if (full_prompt && u[b].n_text > 1) max_prefill = std::max(max_prefill, 9 + u[b].n_text);
  if (max_prefill + F > s.maxP) return fail(QTTS_ERR_RANGE, "prefill + max_frames exceeds the session's max_positions");
  CK(cudaSetDevice(m.device));
  CK(cudaStreamSynchronize(s.st));
  free_generation(s);
  const int H = d.t_hidden;
  // token rows: 6 specials then each utterance's text
  std::vector<uint32_t> tok = {IM_START, ASSISTANT, NEWLINE, TTS_PAD, TTS_BOS, TTS_EOS};
  std::vector<int> text_row(n);
  int max_trail = 1, n_voice = 0;
  for (int b = 0; b < n; ++b) {
    const qtts_utterance& q = u[b];
    if (q.n_text < 0 || (q.n_text > 0 && !q.text) || q.n_text > 65536) return fail(QTTS_ERR_BADARG, "bad text");
    const qtts_sample_params& p = q.params;
    if (!(p.temperature > 0.0f) || p.top_k < 0 || !std::isfinite(p.repetition_penalty))
      return fail(QTTS_ERR_BADARG, "temperature must be > 0 (the reference divides by it), top_k >= 0");
    if ((int)q.language_id >= d.t_vocab || (!q.voice && (int)q.speaker_id >= d.t_vocab))
      return fail(QTTS_ERR_BADARG, "speaker / language id outside the codec vocabulary");
    text_row[b] = (int)tok.size();
    for (int i = 0; i < q.n_text; ++i) {
      if ((int)q.text[i] >= d.t_text_vocab) return fail(QTTS_ERR_BADARG, "text token outside the text vocabulary");
      tok.push_back(q.text[i]);
    }
    max_trail = std::max(max_trail, (full_prompt ? 0 : std::max(q.n_text - 1, 0)) + 1);
    if (q.voice) ++n_voice;
  }
  if (full_prompt) {  // all prefill rows live in xpre at once
    int rows = 0;
    for (int b = 0; b < n; ++b) rows += u[b].n_text > 0 ? 9 + u[b].n_text : 9;
    RC(ensure_rows(s, rows));
  }
  s.B = n;
  s.max_frames = F;
  s.max_trail = max_trail;
  s.flags = flags;
  const int Nt = (int)tok.size();
  RC(gen_alloc(s, 0, &s.codes, (size_t)n * F * kMaxGroups));
  s.forced = nullptr;
  if (forced) RC(gen_alloc(s, 1, &s.forced, (size_t)n * F * kMaxGroups));
  RC(gen_alloc(s, 2, &s.tp, (size_t)Nt * H));
  RC(gen_alloc(s, 3, &s.tp_h1, (size_t)Nt * m.fc1.n));
  RC(gen_alloc(s, 4, &s.tp_tok, (size_t)Nt));
  RC(gen_alloc(s, 5, &s.recipes, (size_t)n * max_prefill));
  RC(gen_alloc(s, 6, &s.trail, (size_t)n * max_trail * H));
  RC(gen_alloc(s, 7, &s.trail_idx, (size_t)n * max_trail));
  RC(gen_alloc(s, 8, &s.voices, (size_t)std::max(n_voice, 1) * H));
  s.dump_logits = nullptr;
  s.dump_hidden = nullptr;
  if (dump_logits) RC(gen_alloc(s, 9, &s.dump_logits, (size_t)n * F * d.t_vocab));
  if (dump_hidden) RC(gen_alloc(s, 10, &s.dump_hidden, (size_t)n * F * H));
  // frames an utterance never reaches (EOS) read back as zero
  CK(cudaMemsetAsync(s.codes, 0, sizeof(uint32_t) * n * F * kMaxGroups, s.st));
  if (s.dump_logits) CK(cudaMemsetAsync(s.dump_logits, 0, sizeof(float) * n * F * d.t_vocab, s.st));
  if (s.dump_hidden) CK(cudaMemsetAsync(s.dump_hidden, 0, sizeof(float) * n * F * H, s.st));
  if (forced) CK(cudaMemcpy(s.forced, forced, sizeof(uint32_t) * n * F * kMaxGroups, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(s.tp_tok, tok.data(), sizeof(uint32_t) * Nt, cudaMemcpyHostToDevice));
  // prefill recipes (generate_new.rs:94-173) and trailing text rows (:314-326)
  std::vector<RowRecipe> rec((size_t)n * max_prefill, RowRecipe{-1, -1, -1, 0});
  std::vector<int> seq(n), row0(n), trail_idx((size_t)n * max_trail, 5);
  std::vector<SlotState> slots(n);
  int vi = 0, nrows = 0;
  for (int b = 0; b < n; ++b) {
    const qtts_utterance& q = u[b];
    row0[b] = nrows;
    RowRecipe* r = &rec[(size_t)nrows];
    int t = 0;
    for (int i = 0; i < 3; ++i) r[t++] = {-1, i, -1, 0};  // role prefix
    const int lang = (int)q.language_id;
    const int pre[4] = {(int)CODEC_THINK, (int)CODEC_THINK_BOS, lang, (int)CODEC_THINK_EOS};
    for (int i = 0; i < 4; ++i) r[t++] = {pre[i], 3, -1, 0};  // codec + TTS_PAD
    if (q.voice) {
      CK(cudaMemcpy(s.voices + (size_t)vi * H, q.voice, sizeof(float) * H, cudaMemcpyHostToDevice));
      r[t++] = {-1, -1, vi++, 0};  // raw voice embedding
    } else {
      r[t++] = {(int)q.speaker_id, 3, -1, 0};
    }
    r[t++] = {(int)CODEC_PAD, 4, -1, 0};  // PAD + TTS_BOS
    if (q.n_text > 0) r[t++] = {(int)CODEC_BOS, text_row[b], -1, 0};
    if (full_prompt)  // the rest of the text as prefill rows (QTTS_FULL_PROMPT)
      for (int i = 1; i < q.n_text; ++i) r[t++] = {(int)CODEC_PAD, text_row[b] + i, -1, 0};
    seq[b] = t;
    nrows += t;
    const int ntr = (full_prompt ? 0 : std::max(q.n_text - 1, 0)) + 1;
    for (int i = 1; i < ntr; ++i) trail_idx[(size_t)b * max_trail + i - 1] = text_row[b] + i;
    trail_idx[(size_t)b * max_trail + ntr - 1] = 5;  // TTS_EOS
    SlotState& sl = slots[b];
    memset(&sl, 0, sizeof(sl));
    sl.pos = t;  // generate_new.rs:216
    sl.n_trail = ntr;
    sl.flags = (flags & QTTS_IGNORE_EOS) ? 1 : 0;
    sl.temperature = q.params.temperature;
    sl.rep_pen = q.params.repetition_penalty;
    sl.top_k = q.params.top_k;
    sl.eos = q.params.codec_eos_id;
    sl.rng = q.seed;
  }
  CK(cudaMemcpy(s.recipes, rec.data(), sizeof(RowRecipe) * rec.size(), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(s.trail_idx, trail_idx.data(), sizeof(int) * trail_idx.size(), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(s.slots, slots.data(), sizeof(SlotState) * n, cudaMemcpyHostToDevice));
  CK(cudaMemset(s.err_flag, 0, sizeof(int)));

  // prefill
  std::vector<Op> ops;
  RC(add_text_proj(s, ops, s.tp_tok, Nt, s.tp_h1, s.tp, H));
  {
    const Q4Mat ce = m.codec_emb;
    const RowRecipe* rc = s.recipes;
    const float* tp = s.tp;
    const float* vo = s.voices;
    float* xp = s.xpre;
    ops.push_back([=](cudaStream_t st) { return launch_assemble(ce, rc, nrows, tp, H, vo, H, xp, H, H, st); });
    float* tr = s.trail;
    const int* ti = s.trail_idx;
    const int ntr = n * max_trail;
    ops.push_back([=](cudaStream_t st) { return launch_gather_rows(tp, H, ti, ntr, tr, H, H, st); });
  }
  RC(run_ops(s, ops));
  ops.clear();
  s.tts_pad = s.tp + 3L * H;  // embed_text_token(TTS_PAD), generate_new.rs:222
  // prefill runs of consecutive utterances with equal sequence length
  // (9 without text, 10 with); their rows are contiguous in xpre
  int b0 = 0;
  while (b0 < n) {
    int b1 = b0;
    while (b1 < n && seq[b1] == seq[b0]) ++b1;
    const int sq = seq[b0], nb = b1 - b0;
    float* X = s.xpre + (size_t)row0[b0] * H;
    RowPos rp;
    rp.rows_per_sess = sq;
    rp.sess0 = b0;
    RC(add_talker(s, ops, X, H, nb * sq, rp, 1, false));
    RC(add_codec_head(s, ops, X + (size_t)(sq - 1) * H, (long)sq * H, nb, s.logits + (size_t)b0 * d.t_vocab,
                      s.pin + (size_t)b0 * 2 * H, 2L * H, sq - 1, sq));
    RC(run_ops(s, ops));
    ops.clear();
    b0 = b1;
  }
  RC(sync_check(s));

  // frame plan -> CUDA graph, reused while nothing it bakes in has changed
  Session::GraphKey key;
  key.B = n; key.F = F; key.max_trail = max_trail; key.forced = forced ? 1 : 0;
  key.dump_logits = dump_logits ? 1 : 0; key.dump_hidden = dump_hidden ? 1 : 0; key.epoch = s.buf_epoch;
  key.wait_ns = s.wait_ns;
  if (s.graph_exec && s.graph_key == key) {
    s.generating = true;
    return QTTS_OK;
  }
  destroy_graph(s);
  std::vector<Op> fops;
  RC(build_frame_ops(s, fops, dump_logits || dump_hidden));
  CK(cudaStreamBeginCapture(s.st, cudaStreamCaptureModeThreadLocal));
  const long launches0 = g_kernel_launches;
  int rc = run_ops(s, fops);
  s.frame_kernels = (int)(g_kernel_launches - launches0);
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(s.st, &g);
  if (rc != QTTS_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
  s.graph = g;
  CK(cudaGraphInstantiate(&s.graph_exec, g, 0));
  s.graph_key = key;
  ++s.graph_captures;
  s.generating = true;
  return QTTS_OK;
}

static int generate_frames(Session& s, int nf) {
  if (!s.generating) return fail(QTTS_ERR_STATE, "no generation in progress");
  for (int i = 0; i < nf; ++i) CK(cudaGraphLaunch(s.graph_exec, s.st));
  return QTTS_OK;
}

static int generate_end(Session& s, uint32_t* codes, int* frames_out, float* dl, float* dh) {
  if (!s.generating) return fail(QTTS_ERR_STATE, "no generation in progress");
  RC(sync_check(s));
  const int n = s.B, F = s.max_frames;
  const qtts_dims& d = s.m->d;
  if (codes) CK(cudaMemcpy(codes, s.codes, sizeof(uint32_t) * n * F * kMaxGroups, cudaMemcpyDeviceToHost));
  if (frames_out) {
    std::vector<SlotState> sl(n);
    CK(cudaMemcpy(sl.data(), s.slots, sizeof(SlotState) * n, cudaMemcpyDeviceToHost));
    for (int b = 0; b < n; ++b) frames_out[b] = std::min(sl[b].frames_out, F);
  }
  if (dl && s.dump_logits) CK(cudaMemcpy(dl, s.dump_logits, sizeof(float) * n * F * d.t_vocab, cudaMemcpyDeviceToHost));
  if (dh && s.dump_hidden) CK(cudaMemcpy(dh, s.dump_hidden, sizeof(float) * n * F * d.t_hidden, cudaMemcpyDeviceToHost));
  return QTTS_OK;
}

// Profiling: one frame's launches of kernel family `fam`, built exactly as
// the frame plan builds them (order, parameters, dependent-launch links,
// L2-prefetch targets), captured without the frame's other launches and
// replayed `reps` times between events on the session stream.  The replays
// rewrite the current frame's cache entries, activations and codes, so the
// generation in progress ends here.
static int family_time(Session& s, int fam, int reps, float* ms, int* launches, double* flops, double* wbytes) {
  if (!s.graph_exec) return fail(QTTS_ERR_STATE, "no frame plan: begin a generation first");
  if (reps <= 0 || reps > 100000) return fail(QTTS_ERR_BADARG, "bad repetition count");
  CK(cudaStreamSynchronize(s.st));
  std::vector<Op> fops, sel;
  RC(build_frame_ops(s, fops, false));
  double fl = 0.0, wb = 0.0;
  for (const Op& op : fops) {  // sort by family without launching
    g_occ_query = true;
    g_occ_family = FAM_OTHER;
    g_occ_flops = g_occ_wbytes = 0.0;
    const cudaError_t qe = op(nullptr);
    g_occ_query = false;
    if (qe != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("launch plan: ") + cudaGetErrorString(qe));
    if (g_occ_family == fam) {
      sel.push_back(op);
      fl += g_occ_flops;
      wb += g_occ_wbytes;
    }
  }
  s.generating = false;
  *ms = 0.0f;
  *launches = 0;
  *flops = fl;
  *wbytes = wb;
  if (sel.empty()) return QTTS_OK;
  CK(cudaStreamBeginCapture(s.st, cudaStreamCaptureModeThreadLocal));
  const long l0 = g_kernel_launches;
  const int rc = run_ops(s, sel);
  const int nl = (int)(g_kernel_launches - l0);
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(s.st, &g);
  if (rc != QTTS_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
  cudaGraphExec_t ge = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ie));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaError_t err = cudaEventCreate(&e0);
  if (err == cudaSuccess) err = cudaEventCreate(&e1);
  for (int i = 0; err == cudaSuccess && i < 3; ++i) err = cudaGraphLaunch(ge, s.st);  // warm-up
  if (err == cudaSuccess) err = cudaEventRecord(e0, s.st);
  for (int i = 0; err == cudaSuccess && i < reps; ++i) err = cudaGraphLaunch(ge, s.st);
  if (err == cudaSuccess) err = cudaEventRecord(e1, s.st);
  if (err == cudaSuccess) err = cudaEventSynchronize(e1);
  float t = 0.0f;
  if (err == cudaSuccess) err = cudaEventElapsedTime(&t, e0, e1);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaGraphExecDestroy(ge);
  if (err != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("family replay: ") + cudaGetErrorString(err));
  RC(sync_check(s));
  *ms = t / (float)reps;
  *launches = nl;
  return QTTS_OK;
}

// ---------------------------------------------------------------------------
// per-call reference API (slot 0)
// ---------------------------------------------------------------------------
static int text_embed(Session& s, uint32_t tok, float* out) {
  const Model& m = *s.m;
  if ((int)tok >= m.d.t_text_vocab) return fail(QTTS_ERR_BADARG, "token outside the text vocabulary");
  uint32_t* td = s.codes_plain;  // scratch for one id
  CK(cudaMemcpyAsync(td, &tok, sizeof(uint32_t), cudaMemcpyHostToDevice, s.st));
  std::vector<Op> ops;
  float* h1 = s.h;
  float* o = s.io;
  RC(add_text_proj(s, ops, td, 1, h1, o, m.d.t_hidden));
  RC(run_ops(s, ops));
  CK(cudaMemcpyAsync(out, o, sizeof(float) * m.d.t_hidden, cudaMemcpyDeviceToHost, s.st));
  return sync_check(s);
}

static int codec_embed(Session& s, uint32_t tok, float* out) {
  const Model& m = *s.m;
  if ((int)tok >= m.codec_emb.k) return fail(QTTS_ERR_BADARG, "token outside the codec vocabulary");
  CK(cudaMemcpyAsync(s.codes_plain, &tok, sizeof(uint32_t), cudaMemcpyHostToDevice, s.st));
  const cudaError_t e = launch_embed_rows(m.codec_emb, s.codes_plain, 1, s.io, m.d.t_hidden, s.st);
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
  CK(cudaMemcpyAsync(out, s.io, sizeof(float) * m.d.t_hidden, cudaMemcpyDeviceToHost, s.st));
  return sync_check(s);
}

static int prefill_call(Session& s, const float* emb, int n, float* hid, float* logits) {
  const Model& m = *s.m;
  const int H = m.d.t_hidden;
  if (!emb || n <= 0 || n > s.rows || n > s.maxP) return fail(QTTS_ERR_BADARG, "bad prefill length");
  if (s.kvlen0 != 0) return fail(QTTS_ERR_STATE, "prefill needs an empty cache (qtts_session_reset)");
  if (s.generating) free_generation(s);
  CK(cudaMemcpyAsync(s.xpre, emb, sizeof(float) * n * H, cudaMemcpyHostToDevice, s.st));
  std::vector<Op> ops;
  RowPos rp;
  rp.rows_per_sess = n;
  RC(add_talker(s, ops, s.xpre, H, n, rp, 1, false));
  RC(add_codec_head(s, ops, s.xpre + (size_t)(n - 1) * H, H, 1, s.logits, s.hid1, H, n - 1, 1));
  RC(run_ops(s, ops));
  if (hid) CK(cudaMemcpyAsync(hid, s.hid1, sizeof(float) * H, cudaMemcpyDeviceToHost, s.st));
  if (logits) CK(cudaMemcpyAsync(logits, s.logits, sizeof(float) * m.d.t_vocab, cudaMemcpyDeviceToHost, s.st));
  RC(sync_check(s));
  s.kvlen0 = n;
  return QTTS_OK;
}

static int talker_step_call(Session& s, const float* emb, int position, float* out) {
  const Model& m = *s.m;
  const int H = m.d.t_hidden, V = m.d.t_vocab;
  if (!emb || !out || position < 0) return fail(QTTS_ERR_BADARG, "bad talker step arguments");
  if (s.kvlen0 + 1 > s.maxP) return fail(QTTS_ERR_RANGE, "session KV capacity exhausted");
  if (position >= m.d.t_max_pos) return fail(QTTS_ERR_RANGE, "position beyond the talker RoPE table");
  if (s.generating) free_generation(s);
  CK(cudaMemcpyAsync(s.x, emb, sizeof(float) * H, cudaMemcpyHostToDevice, s.st));
  std::vector<Op> ops;
  RowPos rp;
  rp.pos_const = position;
  rp.kv_const = s.kvlen0;
  RC(add_talker(s, ops, s.x, H, 1, rp, talker_nsplit(s, 1), false));
  RC(add_codec_head(s, ops, s.x, H, 1, s.logits, s.hid1, H));
  RC(run_ops(s, ops));
  CK(cudaMemcpyAsync(out, s.hid1, sizeof(float) * H, cudaMemcpyDeviceToHost, s.st));
  CK(cudaMemcpyAsync(out + H, s.logits, sizeof(float) * V, cudaMemcpyDeviceToHost, s.st));
  RC(sync_check(s));
  s.kvlen0 += 1;
  return QTTS_OK;
}

static int predict_call(Session& s, const float* hidden, const float* sem, uint32_t* codes) {
  const Model& m = *s.m;
  const int H = m.d.t_hidden;
  if (!hidden || !sem || !codes) return fail(QTTS_ERR_BADARG, "null argument");
  if (s.generating) free_generation(s);
  CK(cudaMemcpyAsync(s.pin, hidden, sizeof(float) * H, cudaMemcpyHostToDevice, s.st));
  CK(cudaMemcpyAsync(s.pin + H, sem, sizeof(float) * H, cudaMemcpyHostToDevice, s.st));
  std::vector<Op> ops;
  RC(add_predictor(s, ops, 1, false, FrameCodes{}));
  RC(run_ops(s, ops));
  uint32_t c[kMaxGroups];
  CK(cudaMemcpyAsync(c, s.codes_plain, sizeof(c), cudaMemcpyDeviceToHost, s.st));
  RC(sync_check(s));
  for (int g = 0; g < m.d.p_groups; ++g) codes[g] = c[g + 1];
  return QTTS_OK;
}

static int acoustic_sum_call(Session& s, const uint32_t* codes, float* out) {
  const Model& m = *s.m;
  if (!codes || !out) return fail(QTTS_ERR_BADARG, "null argument");
  for (int g = 0; g < m.d.p_groups; ++g)
    if ((int)codes[g] >= m.p_emb[g].k) return fail(QTTS_ERR_BADARG, "code outside the predictor vocabulary");
  CK(cudaMemcpyAsync(s.codes_plain, codes, sizeof(uint32_t) * m.d.p_groups, cudaMemcpyHostToDevice, s.st));
  FuseDesc fd;
  fd.x = s.io; fd.ldx = m.d.t_hidden; fd.group_emb = m.d_group_emb; fd.n_groups = m.d.p_groups;
  fd.B = 1; fd.H = m.d.t_hidden; fd.mode = 2; fd.codes_plain = s.codes_plain;
  const cudaError_t e = launch_fuse(fd, s.st);
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
  CK(cudaMemcpyAsync(out, s.io, sizeof(float) * m.d.t_hidden, cudaMemcpyDeviceToHost, s.st));
  return sync_check(s);
}

static int sample_call(Session& s, const float* logits, int n, const qtts_sample_params* p, const uint32_t* prev,
                       uint64_t* rng, uint32_t* out) {
  if (!logits || !p || !prev || !rng || !out || n <= 0 || n > 4096) return fail(QTTS_ERR_BADARG, "bad sample arguments");
  if (!(p->temperature > 0.0f) || p->top_k < 0) return fail(QTTS_ERR_BADARG, "temperature must be > 0, top_k >= 0");
  // io layout: [logits n][prev 16][rng 2][out 1]
  float* dl = s.io;
  uint32_t* dprev = reinterpret_cast<uint32_t*>(s.io + n);
  unsigned long long* drng = reinterpret_cast<unsigned long long*>(s.io + ((n + 16 + 1) & ~1));
  uint32_t* dout = reinterpret_cast<uint32_t*>(drng + 1);
  CK(cudaMemcpyAsync(dl, logits, sizeof(float) * n, cudaMemcpyHostToDevice, s.st));
  CK(cudaMemcpyAsync(dprev, prev, sizeof(uint32_t) * 16, cudaMemcpyHostToDevice, s.st));
  CK(cudaMemcpyAsync(drng, rng, sizeof(uint64_t), cudaMemcpyHostToDevice, s.st));
  SampleDesc sd;
  sd.logits = dl; sd.ldl = n; sd.V = n; sd.B = 1; sd.standalone = 1;
  sd.temperature = p->temperature; sd.rep_pen = p->repetition_penalty; sd.top_k = p->top_k;
  sd.prev = dprev; sd.rng = drng; sd.out = dout;
  const cudaError_t e = launch_sample(sd, s.st);
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
  CK(cudaMemcpyAsync(rng, drng, sizeof(uint64_t), cudaMemcpyDeviceToHost, s.st));
  CK(cudaMemcpyAsync(out, dout, sizeof(uint32_t), cudaMemcpyDeviceToHost, s.st));
  return sync_check(s);
}

// ---------------------------------------------------------------------------
// standalone GEMV entry points
// ---------------------------------------------------------------------------
constexpr size_t kCounterBytes = 16384;  // 4096 tile counters at the head of the scratch

static int gemv_plan_standalone(int k, int n, int m, GemvDesc& g) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  gemv_init_attributes();  // the occupancy queries of the planners need them
  tc_init_attributes();
  Q4Mat w;
  w.k = k;
  w.n = n;
  g = gemv_base(EPI_STORE, {w}, false, m);
  choose_split(sms, g);
  if (m >= kTcMinRows && k % 4 == 0 && n % 64 == 0) tc_plan(sms, g);
  return QTTS_OK;
}

int tc_project_expanded(const Q4Mat* mats, int nmat, int epi, const float* X, long ldx, int M, float* out, long ldo,
                        const float* bias, uint8_t* xs_buf, size_t xs_bytes, const uint8_t* x_split_pre,
                        uint8_t* xs_out, int* err_flag, cudaStream_t st) {
  if (M < kTcMinRows || nmat < 1 || nmat > 2 || (nmat == 2) != (epi == EPI_SWIGLU))
    return fail(QTTS_ERR_BADARG, "tensor-core projection: bad shape");
  for (int i = 0; i < nmat; ++i)
    if (!mats[i].wx || mats[i].k % 4 || mats[i].n % 64) return fail(QTTS_ERR_BADARG, "tensor-core projection: bad weights");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  tc_init_attributes();
  GemvDesc g = nmat == 2 ? gemv_base(epi, {mats[0], mats[1]}, true, M) : gemv_base(epi, {mats[0]}, false, M);
  g.X = X; g.ldx = ldx;
  g.epi.out = out; g.epi.ldo = ldo; g.epi.bias = bias;
  g.err_flag = err_flag;
  g.xs_buf = xs_buf; g.xs_bytes = xs_bytes;
  g.x_split_pre = x_split_pre;
  if (xs_out) {
    if (epi != EPI_SWIGLU) return fail(QTTS_ERR_BADARG, "tensor-core projection: split output needs SwiGLU");
    g.xs_out = xs_out;
    g.xs_out_k = mats[0].n;
  }
  g.cluster = 1;
  tc_plan(sms, g);
  // more than 128 rows must take split rows: the other instance reads Q4 bytes
  if (M > kTcRows && !x_split_pre && !tc_takes_split(g))
    return fail(QTTS_ERR_BADARG, "tensor-core projection: split-row scratch too small");
  const cudaError_t e = launch_gemv(g, FrameCodes{}, st);  // (checks the operands' alignment)
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
  return QTTS_OK;
}

// Scratch layout: [tile counters 16 KB][split-K partials of either kernel]
// [split input rows of a tensor-core launch of more than 64 rows, 16-byte
// aligned]
static size_t gemv_part_bytes(const GemvDesc& g, int m, int n) {
  const size_t S = std::max(g.S > 1 ? g.S : 0, g.tc && tc_splits(g) > 1 ? tc_splits(g) : 0);
  return (sizeof(float) * S * m * n + 15) & ~(size_t)15;
}
static size_t gemv_scratch(int k, int n, int m) {
  GemvDesc g;
  gemv_plan_standalone(k, n, m, g);
  const size_t xs = g.tc && m > 64 ? tc_xsplit_scratch_bytes(m, k) : 0;
  return kCounterBytes + gemv_part_bytes(g, m, n) + xs;
}

static int gemv_dev(const uint8_t* packed, const uint16_t* scales, int k, int n, const float* x, int m, float* y,
                    void* scratch, size_t scratch_bytes, cudaStream_t st) {
  if (!packed || !scales || !x || !y || k <= 0 || n <= 0 || m <= 0 || n % 32)
    return fail(QTTS_ERR_BADARG, "bad gemv arguments (n must be a multiple of 32)");
  if (reinterpret_cast<uintptr_t>(packed) % 16 || reinterpret_cast<uintptr_t>(scales) % 2 ||
      reinterpret_cast<uintptr_t>(x) % 4 || reinterpret_cast<uintptr_t>(y) % 4 ||
      reinterpret_cast<uintptr_t>(scratch) % 16)
    return fail(QTTS_ERR_BADARG, "packed and scratch must be 16-byte aligned, x/y 4-byte, scales 2-byte");
  GemvDesc g;
  gemv_plan_standalone(k, n, m, g);
  g.mat[0].packed = packed;
  g.mat[0].scales = reinterpret_cast<const __half*>(scales);
  g.X = x; g.ldx = k;
  g.epi.out = y; g.epi.ldo = n;
  const size_t zb = (size_t)ceil_div(m, g.mb), zt = (size_t)ceil_div(m, kTcRows);
  if (g.ntiles * zb > kCounterBytes / 4 || 2 * g.ntiles * zt > kCounterBytes / 4)
    return fail(QTTS_ERR_BADARG, "too many tiles for the counter area");
  const size_t need = gemv_scratch(k, n, m);
  if (!scratch || scratch_bytes < need) return fail(QTTS_ERR_BADARG, "scratch smaller than qtts_q4_gemv_scratch_bytes()");
  g.counters = reinterpret_cast<unsigned*>(scratch);
  g.part = reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) + kCounterBytes);
  if (g.tc && m > 64) {  // the input rows split once for every column tile, as in the frame
    g.xs_buf = reinterpret_cast<uint8_t*>(scratch) + kCounterBytes + gemv_part_bytes(g, m, n);
    g.xs_bytes = tc_xsplit_scratch_bytes(m, k);
  }
  // the tensor-core kernel's float4 accesses need 16-byte aligned rows
  if (g.tc && (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 16)) g.tc = 0;
  g.cluster = 1;
  // programmatic dependent launch, as in the frame: the kernel loads its
  // weights while the previous kernel on the stream finishes and waits for it
  // before reading x or writing y
  g.pdl = 1;
  gemv_init_attributes();
  tc_init_attributes();
  fit_split_to_wave(g);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  cudaGetLastError();
  batch_plan(sms, g);
  // partial sums go through the scratch only for a K split reduced in global memory
  if (!g.tc && !g.cluster && g.S > 1 && scratch_bytes < kCounterBytes + sizeof(float) * (size_t)g.S * m * n)
    return fail(QTTS_ERR_BADARG, "scratch smaller than qtts_q4_gemv_scratch_bytes()");
  const cudaError_t e = launch_gemv(g, FrameCodes{}, st);
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
  return QTTS_OK;
}

}  // namespace qtts

// ===========================================================================
// C ABI
// ===========================================================================
using namespace qtts;

struct qtts_model {
  Model* m;
};
struct qtts_session {
  Session* s;
};

extern "C" {

const char* qtts_last_error(void) { return g_err.c_str(); }
int qtts_version(void) { return 1; }

int qtts_file_probe(const char* path, qtts_dims* out) {
  if (!path || !out) return fail(QTTS_ERR_BADARG, "null argument");
  HModel hm;
  std::string err;
  const int rc = parse_model(path, &hm, &err);
  if (rc != QTTS_OK) return fail(rc, err);
  *out = hm.d;
  return QTTS_OK;
}

int qtts_synth_write(const char* path, const qtts_dims* dims, uint64_t seed) {
  if (!path || !dims) return fail(QTTS_ERR_BADARG, "null argument");
  std::string err;
  const int rc = synth_write(path, *dims, seed, &err);
  return rc == QTTS_OK ? rc : fail(rc, err);
}
void qtts_dims_1p7b(qtts_dims* out) { dims_1p7b(out); }
void qtts_dims_tiny(qtts_dims* out) { dims_tiny(out); }

int qtts_model_load(const char* path, int device, qtts_model** out) {
  if (!path || !out) return fail(QTTS_ERR_BADARG, "null argument");
  Model* m = nullptr;
  const int rc = model_load(path, device, &m);
  if (rc != QTTS_OK) return rc;
  *out = new qtts_model{m};
  return QTTS_OK;
}

int qtts_model_free(qtts_model* h) {
  if (!h) return QTTS_OK;
  cudaSetDevice(h->m->device);
  cudaFree(h->m->arena);
  cudaFree(h->m->d_group_emb);
  if (h->m->wx_arena) cudaFree(h->m->wx_arena);
  delete h->m;
  delete h;
  return QTTS_OK;
}

int qtts_model_dims(const qtts_model* h, qtts_dims* out) {
  if (!h || !out) return fail(QTTS_ERR_BADARG, "null argument");
  *out = h->m->d;
  return QTTS_OK;
}
size_t qtts_model_device_bytes(const qtts_model* h) { return h ? h->m->bytes + h->m->wx_bytes : 0; }

int qtts_session_create_ex(qtts_model* h, int max_batch, int max_positions, unsigned flags, qtts_session** out) {
  if (!h || !out) return fail(QTTS_ERR_BADARG, "null argument");
  Session* s = nullptr;
  const int rc = session_create(h->m, max_batch, max_positions, flags, &s);
  if (rc != QTTS_OK) return rc;
  *out = new qtts_session{s};
  return QTTS_OK;
}
int qtts_session_create(qtts_model* h, int max_batch, int max_positions, qtts_session** out) {
  return qtts_session_create_ex(h, max_batch, max_positions, 0u, out);
}
int qtts_session_free(qtts_session* h) {
  if (!h) return QTTS_OK;
  session_free_all(h->s);
  delete h;
  return QTTS_OK;
}
int qtts_session_reset(qtts_session* h) {
  if (!h) return fail(QTTS_ERR_BADARG, "null argument");
  Session& s = *h->s;
  CK(cudaSetDevice(s.m->device));
  CK(cudaStreamSynchronize(s.st));
  free_generation(s);
  s.kvlen0 = 0;
  return QTTS_OK;
}
void* qtts_session_stream(qtts_session* h) { return h ? (void*)h->s->st : nullptr; }
int qtts_session_set_wait_budget(qtts_session* h, uint64_t ns) {
  if (!h || ns == 0) return fail(QTTS_ERR_BADARG, "null session or zero budget");
  h->s->wait_ns = ns;
  return QTTS_OK;
}

#define SESS(h)                                                      \
  if (!h) return fail(QTTS_ERR_BADARG, "null session");              \
  Session& s = *h->s;                                                \
  if (cudaSetDevice(s.m->device) != cudaSuccess) return fail(QTTS_ERR_CUDA, "cudaSetDevice");

int qtts_embed_text(qtts_session* h, uint32_t token, float* out) {
  SESS(h);
  if (!out) return fail(QTTS_ERR_BADARG, "null output");
  return text_embed(s, token, out);
}
int qtts_embed_codec(qtts_session* h, uint32_t token, float* out) {
  SESS(h);
  if (!out) return fail(QTTS_ERR_BADARG, "null output");
  return codec_embed(s, token, out);
}
int qtts_prefill(qtts_session* h, const float* emb, int n, float* hidden_out, float* logits_out) {
  SESS(h);
  return prefill_call(s, emb, n, hidden_out, logits_out);
}
int qtts_talker_step(qtts_session* h, const float* emb, int position, float* out) {
  SESS(h);
  return talker_step_call(s, emb, position, out);
}
int qtts_predict_acoustic(qtts_session* h, const float* talker_hidden, const float* semantic_embed, uint32_t* codes) {
  SESS(h);
  return predict_call(s, talker_hidden, semantic_embed, codes);
}
int qtts_acoustic_embed_sum(qtts_session* h, const uint32_t* codes, float* out) {
  SESS(h);
  return acoustic_sum_call(s, codes, out);
}
int qtts_sample(qtts_session* h, const float* logits, int n, const qtts_sample_params* p, const uint32_t* prev16,
                uint64_t* rng, uint32_t* out) {
  SESS(h);
  return sample_call(s, logits, n, p, prev16, rng, out);
}

int qtts_generate_begin(qtts_session* h, int n_utt, const qtts_utterance* utts, int max_frames, unsigned flags,
                        const uint32_t* forced) {
  SESS(h);
  return generate_begin(s, n_utt, utts, max_frames, flags, forced, false, false);
}
int qtts_generate_frames(qtts_session* h, int n_frames) {
  SESS(h);
  return generate_frames(s, n_frames);
}
int qtts_generate_end(qtts_session* h, uint32_t* codes_out, int* frames_out, float* logits_dump, float* hidden_dump) {
  SESS(h);
  return generate_end(s, codes_out, frames_out, logits_dump, hidden_dump);
}
int qtts_generate(qtts_session* h, int n_utt, const qtts_utterance* utts, int max_frames, unsigned flags,
                  const uint32_t* forced, uint32_t* codes_out, int* frames_out, float* logits_dump,
                  float* hidden_dump) {
  SESS(h);
  RC(generate_begin(s, n_utt, utts, max_frames, flags, forced, logits_dump != nullptr, hidden_dump != nullptr));
  RC(generate_frames(s, max_frames));
  return generate_end(s, codes_out, frames_out, logits_dump, hidden_dump);
}
int qtts_frame_kernel_count(qtts_session* h) { return h ? h->s->frame_kernels : 0; }
int qtts_frame_graph_captures(qtts_session* h) { return h ? h->s->graph_captures : 0; }
int qtts_frame_family_time(qtts_session* h, int family, int reps, float* ms, int* launches, double* flops,
                           double* weight_bytes) {
  SESS(h);
  if (!ms || !launches || !flops || !weight_bytes) return fail(QTTS_ERR_BADARG, "null output");
  if (family < FAM_Q4MV_DEC || family > FAM_ATTN) return fail(QTTS_ERR_BADARG, "unknown kernel family");
  return family_time(s, family, reps, ms, launches, flops, weight_bytes);
}

size_t qtts_q4_gemv_scratch_bytes(int k, int n, int m) {
  if (k <= 0 || n <= 0 || m <= 0) return 0;
  return gemv_scratch(k, n, m);
}
int qtts_q4_gemv_dev(const uint8_t* packed, const uint16_t* scales, int k, int n, const float* x, int m, float* y,
                     void* scratch, size_t scratch_bytes, void* stream) {
  return gemv_dev(packed, scales, k, n, x, m, y, scratch, scratch_bytes, (cudaStream_t)stream);
}
int qtts_q4_gemv(const uint8_t* packed, const uint16_t* scales, int k, int n, const float* x, int m, float* y) {
  if (!packed || !scales || !x || !y || k <= 0 || n <= 0 || m <= 0 || n % 32) return fail(QTTS_ERR_BADARG, "bad gemv arguments");
  const size_t pb = (size_t)k * n / 2, sb = (size_t)k * n / 32 * 2, xb = sizeof(float) * (size_t)m * k,
               yb = sizeof(float) * (size_t)m * n, scr = gemv_scratch(k, n, m);
  char* buf = nullptr;
  const size_t a = (pb + 255) & ~(size_t)255, b2 = (sb + 255) & ~(size_t)255, c = (xb + 255) & ~(size_t)255,
               dsz = (yb + 255) & ~(size_t)255;
  if (cudaMalloc(&buf, a + b2 + c + dsz + scr) != cudaSuccess) return fail(QTTS_ERR_OOM, "device allocation failed");
  int rc = QTTS_OK;
  if (cudaMemset(buf + a + b2 + c + dsz, 0, scr) != cudaSuccess ||
      cudaMemcpy(buf, packed, pb, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(buf + a, scales, sb, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(buf + a + b2, x, xb, cudaMemcpyHostToDevice) != cudaSuccess)
    rc = fail(QTTS_ERR_CUDA, "copy to device failed");
  if (rc == QTTS_OK)
    rc = gemv_dev(reinterpret_cast<uint8_t*>(buf), reinterpret_cast<uint16_t*>(buf + a), k, n,
                  reinterpret_cast<float*>(buf + a + b2), m, reinterpret_cast<float*>(buf + a + b2 + c),
                  buf + a + b2 + c + dsz, scr, nullptr);
  if (rc == QTTS_OK && cudaMemcpy(y, buf + a + b2 + c, yb, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = fail(QTTS_ERR_CUDA, "copy from device failed");
  cudaFree(buf);
  return rc;
}
int qtts_expf_dev(const float* x, float* y, int n, void* stream) {
  if (!x || !y || n < 0) return fail(QTTS_ERR_BADARG, "bad expf arguments");
  const cudaError_t e = launch_expf(x, y, n, (cudaStream_t)stream);
  return e == cudaSuccess ? QTTS_OK : fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
}
int qtts_f16_gemv_dev(const uint16_t* w, int k, int n, const float* x, int m, float* y, void* stream) {
  if (!w || !x || !y || k <= 0 || n <= 0 || m <= 0 || n % 2) return fail(QTTS_ERR_BADARG, "bad f16 gemv arguments");
  const cudaError_t e = launch_f16_gemv(reinterpret_cast<const __half*>(w), k, n, x, m, y, (cudaStream_t)stream);
  return e == cudaSuccess ? QTTS_OK : fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
}
int qtts_q4_dequant_dev(const uint8_t* packed, const uint16_t* scales, int k, int n, float* out, void* stream) {
  if (!packed || !scales || !out || k <= 0 || n <= 0 || n % 32) return fail(QTTS_ERR_BADARG, "bad dequant arguments");
  Q4Mat q;
  q.packed = packed;
  q.scales = reinterpret_cast<const __half*>(scales);
  q.k = k;
  q.n = n;
  const cudaError_t e = launch_dequant(q, out, (cudaStream_t)stream);
  return e == cudaSuccess ? QTTS_OK : fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
}
int qtts_q4_quantize_dev(const float* data, int k, int n, uint8_t* packed, uint16_t* scales, void* stream) {
  if (!data || !packed || !scales || k <= 0 || n <= 0 || n % 32) return fail(QTTS_ERR_BADARG, "bad quantize arguments");
  if ((reinterpret_cast<uintptr_t>(data) & 15u) || (reinterpret_cast<uintptr_t>(packed) & 1u) ||
      (reinterpret_cast<uintptr_t>(scales) & 1u))
    return fail(QTTS_ERR_BADARG, "quantize: data must be 16-byte aligned, packed and scales 2-byte aligned");
  const cudaError_t e = launch_q4_quantize(data, (size_t)k, (size_t)n, packed, scales, (cudaStream_t)stream);
  return e == cudaSuccess ? QTTS_OK : fail(QTTS_ERR_CUDA, cudaGetErrorString(e));
}
int qtts_q4_quantize(const float* data, int k, int n, uint8_t* packed, uint16_t* scales) {
  if (!data || !packed || !scales || k <= 0 || n <= 0 || n % 32) return fail(QTTS_ERR_BADARG, "bad quantize arguments");
  const size_t db = sizeof(float) * (size_t)k * n, pb = (size_t)k * n / 2, sb = (size_t)k * n / 32 * 2;
  const size_t a = (db + 255) & ~(size_t)255, b = (pb + 255) & ~(size_t)255;
  char* buf = nullptr;
  if (cudaMalloc(&buf, a + b + sb) != cudaSuccess) return fail(QTTS_ERR_OOM, "device allocation failed");
  int rc = QTTS_OK;
  if (cudaMemcpy(buf, data, db, cudaMemcpyHostToDevice) != cudaSuccess) rc = fail(QTTS_ERR_CUDA, "copy to device failed");
  if (rc == QTTS_OK)
    rc = qtts_q4_quantize_dev(reinterpret_cast<float*>(buf), k, n, reinterpret_cast<uint8_t*>(buf + a),
                              reinterpret_cast<uint16_t*>(buf + a + b), nullptr);
  if (rc == QTTS_OK && (cudaMemcpy(packed, buf + a, pb, cudaMemcpyDeviceToHost) != cudaSuccess ||
                        cudaMemcpy(scales, buf + a + b, sb, cudaMemcpyDeviceToHost) != cudaSuccess))
    rc = fail(QTTS_ERR_CUDA, "copy from device failed");
  cudaFree(buf);
  return rc;
}

}  // extern "C"
