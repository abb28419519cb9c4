// kernels.h -- descriptors and launchers of the QORA-TTS sm_100a kernels.
// Shared by the kernel translation units and the engine (host C++).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace qtts {

constexpr int kHeadDim = 128;      // head_dim of talker and predictor (config.json)
constexpr int kPageSize = 16;      // KV positions per page
constexpr int kTileN = 256;        // GEMV columns per CTA tile (8 Q4 groups of 32)
constexpr int kGemvThreads = 256;  // 8 warps
constexpr int kMaxGroups = 16;     // codes per frame (1 semantic + 15 acoustic)
constexpr int kAttnRec = 4 + 128;  // attention split record: m, l, pad, acc[128]

// One Q4 g32 weight in its on-disk [k][n] layout (gemv.rs:26-31).
struct Q4Mat {
  const uint8_t* packed = nullptr;  // k*n/2 bytes, low nibble = even column
  const __half* scales = nullptr;   // k*n/32 f16, groups of 32 along n
  int k = 0, n = 0;
  // optional: the weights expanded once into the tensor-core operand layout
  // (fp16 hi / lo blocks per 128-column tile and 64-row stage, tc_expand)
  const uint8_t* wx = nullptr;
};

// Paged KV addressing.  A page holds kPageSize positions of every layer:
//   pool[page][layer][K|V][kv_head][pos % 16][128]  (f32, the reference's
//   precision; f16 elements when `f16` is set, an opt-in session mode)
// page = page_table[sess * pages_per_sess + pos / 16] (or = sess when
// page_table is null: one page per session, the predictor cache).
struct KvDesc {
  float* pool = nullptr;  // element i at pool + i, or at (__half*)pool + i (f16)
  const int* page_table = nullptr;
  int pages_per_sess = 0;
  int n_layers = 0;
  int kv_heads = 0;
  int layer = 0;
  int f16 = 0;
};

// Row -> (session, position) mapping shared by the QKV epilogue and the
// attention kernel: s = m / rows_per_sess, r = m % rows_per_sess,
// session = sess0 + s, rope position = (pos_base ? pos_base[session *
// pos_stride] : pos_const) + r, cache index = kv_const + r when kv_const >= 0
// (talker.rs:277,299: K/V append at cached_len, RoPE at `position`), else the
// rope position.  A row attends cache entries [0, cache index].
struct RowPos {
  int rows_per_sess = 1;
  const int* pos_base = nullptr;
  int pos_stride = 1;
  int pos_const = 0;
  int kv_const = -1;
  int sess0 = 0;
};

__host__ __device__ __forceinline__ void row_pos(const RowPos& rp, int m, int& sess, int& pos, int& kvpos) {
  const int s = m / rp.rows_per_sess;
  const int r = m - s * rp.rows_per_sess;
  sess = rp.sess0 + s;
  pos = (rp.pos_base ? rp.pos_base[sess * rp.pos_stride] : rp.pos_const) + r;
  kvpos = rp.kv_const >= 0 ? rp.kv_const + r : pos;
}

enum EpiKind : int {
  EPI_STORE = 0,    // out = v (+bias) (optionally silu)
  EPI_RESID = 1,    // out += v
  EPI_SWIGLU = 2,   // paired gate/up: out = silu(gate) * up
  EPI_QKV = 3,      // q|k|v: per-head QK-norm + RoPE; q -> q_out, k/v -> KV cache
  EPI_ARGMAX = 4,   // argmax over n, last index wins on ties -> code
};

struct EpiDesc {
  // STORE / RESID / SWIGLU
  float* out = nullptr;
  long ldo = 0;
  const float* bias = nullptr;
  int act_silu = 0;  // bit a: SiLU on the columns of matrix a (after the bias)
  // QKV
  float* q_out = nullptr;
  long ldq = 0;
  const __half* q_norm = nullptr;
  const __half* k_norm = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int rope_rows = 0;
  int rope_skip_oob = 0;  // predictor: rotation skipped past the table (code_predictor.rs:107)
  int heads = 0, kv_heads = 0;
  KvDesc kv;
  RowPos rp;
  int* err_flag = nullptr;
  // STORE / RESID: per-tile sums of squares of the written row values,
  // ssq_out[m * ssq_ld + t]: sum of squares of the row's kSsqCols-column
  // block t, consumed by the next RMSNorm prologue
  float* ssq_out = nullptr;
  long ssq_ld = 0;
  // ARGMAX: keys[m] accumulates (order_key(v) << 32 | col); the last tile
  // finalises codes (see FrameCodes).
  unsigned long long* keys = nullptr;
  unsigned* counters2 = nullptr;
  int group = 0;         // code slot written (1..15)
  int frame_codes = 0;   // 1 = write through FrameCodes (generation); 0 = codes_plain
  uint32_t* codes_plain = nullptr;  // [M][16]
};

struct GemvDesc {
  int epi_kind = EPI_STORE;
  int nmat = 1;     // matrices in this launch (<= 3)
  int paired = 0;   // 1: both matrices cover the same columns (gate/up)
  Q4Mat mat[3];
  int tile0[4] = {0, 0, 0, 0};  // first tile of each matrix (concatenated mode)
  int col0[4] = {0, 0, 0, 0};   // first concatenated column of each matrix
  int ntiles = 0;
  int ncols = 0;                // concatenated columns (partial row stride)
  int k = 0;
  int S = 1;                    // K splits (grid.y)
  int rows_per_split = 0;
  int M = 1;                    // activation rows
  int mb = 1;                   // rows per CTA (grid.z = ceil(M / mb))
  // input rows
  const float* X = nullptr;
  long ldx = 0;
  const __half* gamma = nullptr;  // RMSNorm prologue (gemv.rs:408-417)
  // sum of squares of each input row as ssq_n tile partials written by the
  // producer (ssq_in[m * ssq_ld + t]); null = reduce the full row here
  const float* ssq_in = nullptr;
  long ssq_ld = 0;
  int ssq_n = 0;
  // embedding-gather prologue: row m = dequant(emb row emb_idx[m*emb_idx_stride])
  Q4Mat emb;
  const uint32_t* emb_idx = nullptr;
  int emb_idx_stride = 1;
  float* xnorm_out = nullptr;  // optional copy of the normalised rows
  long ld_xnorm = 0;
  // split-K reduction: cluster = 1 reduces the S partials of a tile over
  // distributed shared memory (the S CTAs form one cluster, S <= 16);
  // cluster = 0 goes through global scratch (part + counters).
  int cluster = 0;
  int pdl = 0;
  float* part = nullptr;        // [S][M][ncols]
  unsigned* counters = nullptr; // [ntiles * zblocks], left at zero
  // tensor-core path (tc_gemm.cu): tc = 1 runs the projection as one
  // tcgen05 kernel with K slices of tc_ks 64-deep stages reduced inside a
  // thread-block cluster
  // attention prologue (M = 1, short KV): the input rows [r0, r0 + 128) of a
  // K slice are the attention output of query head r0 / 128 over the cache
  int attn_in = 0;
  const float* attn_q = nullptr;  // rotated queries [M][heads * 128], row stride attn_ldq
  long attn_ldq = 0;
  KvDesc attn_kv;
  RowPos attn_rp;
  int attn_group = 1;             // query heads per KV head
  int tc = 0;
  int tc_ks = 0;
  // tensor-core launches of more than 64 rows per block: session scratch
  // for the input rows split once into operand tiles (tc_xsplit_kernel),
  // and, set for the projection kernel at launch, the split tiles
  uint8_t* xs_buf = nullptr;
  size_t xs_bytes = 0;
  const uint8_t* x_split = nullptr;
  // split tiles of this launch's input written by its producer (no split
  // kernel), and split tiles of this launch's output for its consumer
  // (SwiGLU epilogue of the tensor-core kernel), xs_out_k columns wide
  const uint8_t* x_split_pre = nullptr;
  uint8_t* xs_out = nullptr;
  int xs_out_k = 0;
  // weights of the next projection in the frame (packed and scales of up to
  // three matrices), pulled into L2 by this launch's CTAs as they start
  const uint8_t* pf_ptr[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  uint32_t pf_bytes[6] = {0, 0, 0, 0, 0, 0};
  int* err_flag = nullptr;      // bit 4: a bounded wait expired; bit 8: input outside the fp16 range
  // budget of the decode kernel's split-K wait (the root's wait for its
  // cluster peers' partials), 1 s unless a test of the timeout path sets it
  unsigned long long wait_ns = 1000000000ull;
  // GLU input (decode kernel only): x[r] = X[r] * X[x_glu + r], the SwiGLU
  // product of a row holding silu(gate) in [0, x_glu) and up in [x_glu, 2 x_glu)
  int x_glu = 0;
  // batch kernel (3..15 rows on the CUDA cores): mb rows per CTA, the K
  // slices of a tile reduced row by row inside their cluster
  int batch = 0;
  EpiDesc epi;
};
// err_flag bits shared by the kernels (the session's flag word)
constexpr int kErrRopeRange = 1;     // a position beyond the talker RoPE table
constexpr int kErrWaitExpired = 4;   // a bounded device wait ran out
constexpr int kErrFp16Input = 8;     // a tensor-core input outside the fp16 range
constexpr int kMaxClusterSplits = 16;
constexpr int kMaxGlobalSplits = 64;  // decode kernel, split-K reduced through global memory
constexpr int kAttnInMaxPos = 32;  // cache positions the attention prologue handles
// M = 1 decode kernel: weight rows a lane keeps in registers (32 rows per
// step of the 8 warps x 4 row offsets), per matrix count
constexpr int kDecRowsNM1 = 12;  // rows per split <= 384
constexpr int kDecMaxM = 2;      // decode kernel: input rows per launch (one per grid.z)
constexpr int kDecRowsNM2 = 6;   // rows per split <= 192
// batch kernel: input rows per CTA (one matrix / a gate-up pair) and the
// largest K slice it stages in shared memory (one matrix / a pair)
constexpr int kBatchRowsNM1 = 8;
constexpr int kBatchRowsNM2 = 4;
constexpr int kBatchMaxRpsNM1 = 768;
constexpr int kBatchMaxRpsNM2 = 512;
constexpr int kSsqLd = 64;       // row stride of the sum-of-squares partials
constexpr int kSsqCols = 128;    // columns summed per partial (rows up to 64 * 128 wide)

// Frame bookkeeping shared by the sampler / argmax epilogue / fusion.
struct SlotState {
  int pos;          // next talker position (KV length before the step)
  int frame;        // frames produced so far
  int n_trail;      // trailing text rows
  int done;         // EOS seen
  int frames_out;   // frames recorded
  int flags;
  float temperature;
  float rep_pen;
  int top_k;
  uint32_t eos;
  unsigned long long rng;
  uint32_t prev[16];  // repetition-penalty history (generate_new.rs:231,252,267)
  uint32_t cur[16];   // codes driving the current frame (after forcing)
};

struct FrameCodes {
  SlotState* slots = nullptr;
  uint32_t* codes = nullptr;       // [B][max_frames][16] chosen codes
  const uint32_t* forced = nullptr;// [B][max_frames][16] or null
  int max_frames = 0;
};

// ---- launch helper: programmatic dependent launch + cluster shape ----
// PDL lets a kernel start (and prefetch its weights) while its predecessor
// finishes; the kernel's griddepcontrol.wait orders all dependent reads.
// kernels launched through launch_k by this thread (frame-plan kernel counts)
inline thread_local long g_kernel_launches = 0;
// Occupancy query mode: with g_occ_query set, launch_k launches nothing and
// stores in g_occ_clusters how many clusters of the launch fit on the device
// at once (cudaOccupancyMaxActiveClusters), so planners can size one wave.
inline thread_local bool g_occ_query = false;
inline thread_local int g_occ_clusters = 0;
// Kernel family of the last launch issued in occupancy-query mode, and the
// algorithmic work of a projection launch (useful FLOPs 2*M*k*n, Q4 weight
// bytes k*n*0.5625): lets the profiling entry point sort a frame's launches
// by family without launching them.
enum KernelFamily : int {
  FAM_OTHER = 0, FAM_Q4MV_DEC = 1, FAM_Q4MV_ROWS = 2, FAM_TC_PROJ = 3, FAM_ATTN = 4, FAM_Q4MV_BATCH = 5
};
inline thread_local int g_occ_family = FAM_OTHER;
inline thread_local double g_occ_flops = 0.0, g_occ_wbytes = 0.0;
int occupancy_clusters(const void* func, const cudaLaunchConfig_t& cfg);
struct LaunchOpts {
  bool pdl = false;
  unsigned cluster_y = 1;  // CTAs of one cluster along grid.y
};
template <typename Kern, typename... Args>
inline cudaError_t launch_k(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, LaunchOpts o,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  unsigned n = 0;
  if (o.cluster_y > 1) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = 1;
    at[n].val.clusterDim.y = o.cluster_y;
    at[n].val.clusterDim.z = 1;
    ++n;
  }
  if (o.pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  if (g_occ_query) {
    g_occ_clusters = occupancy_clusters(reinterpret_cast<const void*>(kern), cfg);
    return cudaSuccess;
  }
  ++g_kernel_launches;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ---- launchers (return cudaError_t of the launch) ----
size_t gemv_smem_bytes(const GemvDesc& d);
cudaError_t launch_gemv(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st);
bool gemv_uses_decode_kernel(const GemvDesc& d);  // M = 1 plan served by gemv_dec_kernel

// tensor-core path (tc_gemm.cu)
constexpr int kTcRows = 128;     // MMA tile rows (TMEM lanes)
constexpr int kTcCols = 128;     // CTA tile columns per matrix
constexpr int kTcK = 64;         // K per pipeline stage
constexpr int kTcMinRows = 16;   // projections with M >= this take the tensor cores
void tc_plan(int sm_count, GemvDesc& g);   // sets tc = 1 and tc_ks (K split fitted to one wave)
int tc_splits(const GemvDesc& d);          // K slices of a planned launch
size_t tc_smem_bytes(int nm);
cudaError_t launch_tc(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st);
// Expanded tensor-core operands of a Q4 weight: bytes needed, and the
// expansion (one launch; the blocks are what the projection's converters write).
size_t tc_expand_bytes(int k, int n);
cudaError_t tc_expand(const Q4Mat& w, uint8_t* out, cudaStream_t st);
// f32 weights w[k][ld] (columns col0 .. col0 + n) into the same operand
// tiles, split hi + lo to ~22 significand bits (the speech decoder's
// projections)
cudaError_t tc_expand_f32(const float* w, int k, int n, long ld, int col0, uint8_t* out, cudaStream_t st);
void tc_init_attributes();



struct AttnDesc {
  const float* q = nullptr;  // row m: heads*128
  long ldq = 0;
  float* out = nullptr;
  long ldo = 0;
  KvDesc kv;
  RowPos rp;
  int heads = 0, kv_heads = 0;
  int M = 1;
  int nsplit = 1;
  float* part = nullptr;        // [M][kv_heads][nsplit][G][kAttnRec]
  unsigned* counters = nullptr; // [M][kv_heads]
  int l2_prefetch = 1;          // pull the CTA's K / V rows into L2 before the dependent-launch wait
  // the output rows also as split tiles for the o projection (heads * 128
  // wide; one position slice only), and the flag word for values past fp16
  uint8_t* xs_out = nullptr;
  int* err_flag = nullptr;
};
// largest cache (K + V bytes over all rows of a launch) whose rows the
// attention kernel prefetches into L2 (126 MB) before its dependency wait
constexpr double kAttnPrefetchMaxBytes = 48.0 * (1 << 20);
cudaError_t launch_attention(const AttnDesc& d, cudaStream_t st);
bool tc_takes_split(const GemvDesc& d);
bool tc_takes_split_from_producer(const GemvDesc& d);
bool tc_reads_expanded(const GemvDesc& d);
size_t tc_xsplit_scratch_bytes(int M, int k);

struct SampleDesc {
  const float* logits = nullptr;  // [B][ldl]
  long ldl = 0;
  int V = 0;
  int B = 0;
  FrameCodes fc;
  unsigned long long* argmax_keys = nullptr;  // [16][B] reset here for the frame
  int n_keys = 0;
  // standalone mode (qtts_sample): params/prev/rng given explicitly
  int standalone = 0;
  float temperature = 1.0f, rep_pen = 1.0f;
  int top_k = 0;
  const uint32_t* prev = nullptr;
  unsigned long long* rng = nullptr;
  uint32_t* out = nullptr;
};
cudaError_t launch_sample(const SampleDesc& d, cudaStream_t st);

// Frame input fusion (generate_new.rs:255,271-286):
// x[b] = (emb_codec(code0) + sum_g emb_g(code_{g+1})) + text_add[b]
struct FuseDesc {
  float* x = nullptr;            // [B][H]
  long ldx = 0;
  float* sem_out = nullptr;      // optional copy of emb_codec(code0) [B][lds]
  long lds = 0;
  Q4Mat codec_emb;               // talker codec embedding [V][H]
  const Q4Mat* group_emb = nullptr;  // device array of p_groups matrices [pV][H]
  int n_groups = 0;
  const float* trail = nullptr;  // [B][max_trail][H]
  int max_trail = 0;
  const float* tts_pad = nullptr;  // [H]
  int B = 0, H = 0;
  float* ssq_out = nullptr;      // per-128-column sums of squares of x [B][ssq_ld]
  long ssq_ld = 0;
  FrameCodes fc;
  int mode = 0;                  // 0: full frame fusion; 1: semantic only (sem_out); 2: acoustic sum only
  const uint32_t* codes_plain = nullptr;  // mode 1/2 standalone codes
};
cudaError_t launch_fuse(const FuseDesc& d, cudaStream_t st);

// Gather dequantised Q4 rows: out[i] = row idx[i] of mat (gemv.rs:378-400).
cudaError_t launch_embed_rows(const Q4Mat& mat, const uint32_t* idx, int count, float* out, long ldo,
                              cudaStream_t st);
// Semantic embedding of the current code0: out[b] = emb(slots[b].cur[0]).
cudaError_t launch_embed_code0(const Q4Mat& mat, const SlotState* slots, int B, float* out, long ldo,
                               cudaStream_t st);
// Elementwise: out[r] = a[r] + b[r] (prefill overlays), rows of n floats.
cudaError_t launch_add_rows(const float* a, long lda, const float* b, long ldb, float* out, long ldo,
                            int rows, int n, cudaStream_t st);
cudaError_t launch_frame_end(SlotState* slots, int B, cudaStream_t st);
cudaError_t launch_dequant(const Q4Mat& m, float* out, cudaStream_t st);
// f32 [k][n] -> Q4 g32 (gemv.rs:92-130), bit-identical to the reference.
cudaError_t launch_q4_quantize(const float* data, size_t k, size_t n, uint8_t* packed, uint16_t* scales,
                               cudaStream_t st);
cudaError_t launch_f16_gemv(const __half* w, int k, int n, const float* x, int m, float* y,
                            cudaStream_t st);

}  // namespace qtts
