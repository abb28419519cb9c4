// decoder.cu -- the speech decoder's first stage on the GPU: 16 code streams
// of T frames -> the transformer output [1024][T] that the upsample / Vocos
// stages consume.  The reference runs it on the CPU, frame by frame:
// codebook_lookup (decoder.rs:142-187), the causal pre-conv
// (conv.rs:114-191, called at decoder.rs:404), decoder_transformer
// (decoder.rs:195-335) -- steps 1-3 of decode_to_audio (decoder.rs:394-424).
//
// Layout: every activation is frame-major [T][channels] (one row per frame),
// so each projection is one GEMM over all T frames; the result is written
// channel-first [1024][T] like the reference's return value.
//
//   gather          codes -> E0 = codebook 0 row, S = sum of the 15 other rows
//                   (in group order, as decoder.rs:163-169)
//   gemm            VQ = E0 * P0, VQ += S * Pr (decoder.rs:151-156, 171-175)
//   gemm (3 taps)   the causal conv as a GEMM over [x(t-2) | x(t-1) | x(t)]
//                   with its weights re-laid [tap][in][out] at load
//   gemm            x = pre * W_in + b_in
//   per layer:      rmsnorm; gemm q|k|v (weights concatenated at load);
//                   rope; windowed attention; gemm o with x += o * attn_scale;
//                   rmsnorm; gemm gate|up; silu(g) * u; gemm down with
//                   x += d * mlp_scale
//   rmsnorm, gemm   out^T = norm(x) * W_out + b_out
//
// Arithmetic is f32 throughout (the weights are f32 in the file).  The
// GEMM is a CUDA-core tiled kernel (64 x 64 tiles, 4 x 4 per thread,
// double-buffered 32-deep K steps), its
// accumulation starting from the bias as f32_gemv_bias does; attention
// keeps the reference's summation orders (sequential dot products, the
// softmax sum in position order, the weighted V sum in position order).
#include <cuda_fp16.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "engine.h"
#include "format.h"
#include "kernels.h"

namespace qtts {

namespace {

constexpr int kBM = 64, kBN = 64, kBK = 32, kGemmThreads = 256;
constexpr int kDecMaxWindow = 128;  // attention window held in shared memory
constexpr int kDecGroups = 16;      // codebooks per frame (1 + 15)
constexpr unsigned kDecErrCode = 1u;  // err bit of a bad code (the projection kernel sets bits 4 and 8)

struct DecGemm {
  const float* A;
  long lda;
  int M, K, N;
  int taps, cin;       // taps > 1: A(m, kk) = A[(m + kk / cin - (taps - 1)) * lda + kk % cin], zero above row 0
  const float* B;      // [K][N]
  const float* bias;   // [N] or null: the sums start from it
  const float* scale;  // [N] (mode 2)
  float* C;
  long ldc;
  int mode;   // 0: C = acc; 1: C += acc; 2: C += acc * scale[n]
  int trans;  // store at C[n * ldc + m]
  // with mode 1 and N = 512: the finished rows also as the causal 3-tap
  // conv's split operand rows (K 1536): row m into rows m + 2 - j at columns
  // j * 512 + n, the taps before frame 0 as zeros
  uint8_t* conv_xs;
  int* err;
};

// One 64 x 64 output tile per CTA, 4 x 4 per thread.  K runs in 32-deep
// steps through two shared-memory buffers: the next step's A and B tiles are
// loaded into registers before this step's FMAs and stored into the other
// buffer after them, so each step's global round trip overlaps the math of
// the step before.
__global__ void __launch_bounds__(kGemmThreads) dec_gemm_kernel(const DecGemm g) {
  __shared__ __align__(16) float As[2][kBK][kBM + 4];
  __shared__ __align__(16) float Bs[2][kBK][kBN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  float acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = n0 + tx * 4 + j;
    const float b0 = (g.bias && n < g.N) ? g.bias[n] : 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][j] = b0;
  }
  const int ar = tid >> 3, ac = (tid & 7) * 4;   // A tile: rows ar, ar + 32; k chunk ac
  const int br = tid >> 4, bc = (tid & 15) * 4;  // B tile: k rows br, br + 16; column chunk bc
  float4 ra[2], rb[2];
  auto load = [&](int k0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = m0 + ar + 32 * h, kk = k0 + ac;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < g.M && kk < g.K) {
        long row = m;
        int col = kk;
        if (g.taps > 1) {
          row = (long)m + kk / g.cin - (g.taps - 1);
          col = kk % g.cin;
        }
        if (row >= 0) v = *reinterpret_cast<const float4*>(g.A + row * g.lda + col);
      }
      ra[h] = v;
      const int kb = k0 + br + 16 * h, n = n0 + bc;
      rb[h] = (kb < g.K && n < g.N) ? *reinterpret_cast<const float4*>(g.B + (long)kb * g.N + n)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      As[buf][ac + 0][ar + 32 * h] = ra[h].x;
      As[buf][ac + 1][ar + 32 * h] = ra[h].y;
      As[buf][ac + 2][ar + 32 * h] = ra[h].z;
      As[buf][ac + 3][ar + 32 * h] = ra[h].w;
      *reinterpret_cast<float4*>(&Bs[buf][br + 16 * h][bc]) = rb[h];
    }
  };
  const int nk = (g.K + kBK - 1) / kBK;
  load(0);
  store(0);
  __syncthreads();
  for (int kt = 0; kt < nk; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nk) load((kt + 1) * kBK);
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < nk) store(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= g.N) continue;
      float* c = g.trans ? g.C + (long)n * g.ldc + m : g.C + (long)m * g.ldc + n;
      if (g.mode == 0) *c = acc[i][j];
      else if (g.mode == 1) *c += acc[i][j];
      else *c += acc[i][j] * g.scale[n];
      if (g.conv_xs) {
        const float v = *c;
#pragma unroll
        for (int tap = 0; tap < 3; ++tap)
          if (m + 2 - tap < g.M) xs_store1(g.conv_xs, 3 * 512, m + 2 - tap, tap * 512 + n, v);
        if (m == 0) {  // frame 0 sees no frames before it, frame 1 one
          xs_store1(g.conv_xs, 3 * 512, 0, n, 0.0f);
          xs_store1(g.conv_xs, 3 * 512, 0, 512 + n, 0.0f);
          if (g.M > 1) xs_store1(g.conv_xs, 3 * 512, 1, n, 0.0f);
        }
        if (fabsf(v) > 65504.0f) atomicOr(g.err, kErrFp16Input);
      }
    }
  }
}

// codes [16][T] -> E0 [T][cb] (codebook 0 row), S [T][cb] (rows of
// codebooks 1..15 summed in group order from 0, decoder.rs:163-169)
__global__ void dec_gather_kernel(const uint32_t* codes, int T, int entries, int cb, const float* cb0,
                                  const float* cb_rest, float* E0, float* S, unsigned* err) {
  const int t = blockIdx.x;
  __shared__ uint32_t idx[kDecGroups];
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  if (threadIdx.x < kDecGroups) {
    const uint32_t c = codes[(size_t)threadIdx.x * T + t];
    idx[threadIdx.x] = c;
    if (c >= (uint32_t)entries) atomicOr(&bad, 1);
  }
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) atomicOr(err, kDecErrCode);
    return;
  }
  for (int d = threadIdx.x; d < cb; d += blockDim.x) {
    E0[(size_t)t * cb + d] = cb0[(size_t)idx[0] * cb + d];
    float s = 0.0f;
    for (int g = 0; g < kDecGroups - 1; ++g) s += cb_rest[((size_t)g * entries + idx[g + 1]) * cb + d];
    S[(size_t)t * cb + d] = s;
  }
}

// rms_norm_f32 (decoder.rs:515-525): y = x * (1 / sqrt(sum x^2 / n + eps)) * gamma,
// a warp per row, lane l holding columns 4l + 128 j (n % 128 == 0); with xs,
// also written as the next projection's split operand rows (err bit 8 for a
// value outside the fp16 range).  With add, the layer-scaled residual that
// precedes the norm is applied first, in place: x += add * add_scale
// (decoder.rs:286-288, 313-315).
__global__ void dec_rmsnorm_kernel(float* X, int M, int n, const float* gamma, float eps, float* Y, uint8_t* xs,
                                   int* err, const float* add, const float* add_scale) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= M) return;
  float* x = X + (size_t)row * n;
  float ss = 0.0f;
  for (int c = 4 * lane; c < n; c += 128) {
    float4 v = *reinterpret_cast<const float4*>(x + c);
    if (add) {
      const float4 a = *reinterpret_cast<const float4*>(add + (size_t)row * n + c);
      const float4 sc = *reinterpret_cast<const float4*>(add_scale + c);
      v = make_float4(v.x + a.x * sc.x, v.y + a.y * sc.y, v.z + a.z * sc.z, v.w + a.w * sc.w);
      *reinterpret_cast<float4*>(x + c) = v;
    }
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  bool big = false;
  for (int c = 4 * lane; c < n; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(x + c), g = *reinterpret_cast<const float4*>(gamma + c);
    const float4 y = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
    *reinterpret_cast<float4*>(Y + (size_t)row * n + c) = y;
    if (xs) {
      xs_store4(xs, n, row, c, y);
      big = big || fp16_overflow4(y);
    }
  }
  if (big) atomicOr(err, kErrFp16Input);
}

// apply_rope_split_half (decoder.rs:556-578) on the q and k parts of a
// q|k|v row, position = frame; positions past the table are left as they are
__global__ void dec_rope_kernel(float* QKV, int T, int heads, int hd, const float* cs, const float* sn,
                                long table_len) {
  const int half = hd / 2, per = heads * half;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * per * 2) return;
  const int which = (int)(i / ((long)T * per));  // 0: q, 1: k
  const long r = i % ((long)T * per);
  const int t = (int)(r / per), h = (int)(r % per) / half, e = (int)(r % half);
  const long off = (long)t * half;
  if (off + half > table_len) return;
  float* b = QKV + (size_t)t * 3 * heads * hd + (size_t)which * heads * hd + (size_t)h * hd;
  const float x0 = b[e], x1 = b[half + e], c = cs[off + e], s = sn[off + e];
  b[e] = x0 * c - x1 * s;
  b[half + e] = x1 * c + x0 * s;
}

// causal sliding-window attention (decoder.rs:258-289).  A CTA takes
// kAttnFrames consecutive frames of one head and stages the K and V rows of
// their joint window (up to kAttnFrames + window - 1 positions) in shared
// memory with coalesced row loads; K rows are padded to 65 floats so that
// lanes reading different rows hit different banks.  Per frame (a warp
// each, in turn): lane j scores positions j, j + 32, ... (sequential 64-term
// dot products), lane 0 runs softmax_raw (gemv.rs:434-445) in position
// order, then lane d accumulates dimensions d and d + 32 over the positions
// in order.
constexpr int kAttnFrames = 16;
constexpr int kAttnWarps = 8;  // frames of a block taken warp by warp
// floats of the padded K rows, rounded up to a multiple of 4 so that the V
// rows after them start on a 16-byte boundary
__host__ __device__ constexpr size_t attn_k_floats(int window) {
  return ((size_t)(kAttnFrames + window - 1) * (64 + 1) + 3) & ~(size_t)3;
}
template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) dec_attn_kernel(const float* QKV, int T, int heads, int window, float* out,
                                                       uint8_t* xs, int* err) {
  static_assert(HD == 64, "two dimensions per lane");
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, t0 = blockIdx.x * kAttnFrames;
  const int t1 = min(T, t0 + kAttnFrames);  // frames [t0, t1)
  const int w0 = t0 + 1 > window ? t0 + 1 - window : 0;  // first position any of them sees
  const int nw = t1 - w0;                                 // positions [w0, t1)
  const int rows = kAttnFrames + window - 1;               // the largest joint window
  float* sK = sm;                                         // [rows][HD + 1]
  float* sV = sK + attn_k_floats(window);                 // [rows][HD], 16-byte aligned (float4 stores)
  float* sP = sV + (size_t)rows * HD;                     // [kAttnWarps][window]
  float* sQ = sP + kAttnWarps * window;                   // [kAttnFrames][HD]: the block's q rows
  const long ld = 3L * heads * HD;
  for (int i = threadIdx.x; i < (t1 - t0) * HD; i += blockDim.x)
    sQ[i] = QKV[(size_t)(t0 + i / HD) * ld + (size_t)h * HD + i % HD];
  for (int i = threadIdx.x; i < nw * (HD / 4); i += blockDim.x) {
    const int r = i / (HD / 4), c4 = i % (HD / 4);
    const float* row = QKV + (size_t)(w0 + r) * ld + (size_t)h * HD;
    const float4 k = *reinterpret_cast<const float4*>(row + (size_t)heads * HD + 4 * c4);
    const float4 v = *reinterpret_cast<const float4*>(row + (size_t)2 * heads * HD + 4 * c4);
    float* kd = sK + (size_t)r * (HD + 1) + 4 * c4;
    kd[0] = k.x; kd[1] = k.y; kd[2] = k.z; kd[3] = k.w;
    *reinterpret_cast<float4*>(sV + (size_t)r * HD + 4 * c4) = v;
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf((float)HD);
  float* p = sP + warp * window;
  for (int t = t0 + warp; t < t1; t += kAttnWarps) {
    const float* qs = sQ + (size_t)(t - t0) * HD;
    const int start = t + 1 > window ? t + 1 - window : 0, L = t + 1 - start;
    float mx = -INFINITY;
    for (int s = lane; s < L; s += 32) {
      const float* k = sK + (size_t)(start + s - w0) * (HD + 1);
      float dot = 0.0f;
#pragma unroll 16
      for (int e = 0; e < HD; ++e) dot += qs[e] * k[e];
      p[s] = dot * scale;
      mx = fmaxf(mx, p[s]);
    }
    // softmax_raw: the max is order-free; the exponentials in parallel; their
    // sum in position order on lane 0, as the reference adds them
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int s = lane; s < L; s += 32) p[s] = expf(p[s] - mx);
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0) {
      float sum = 0.0f;
      for (int s = 0; s < L; ++s) sum += p[s];
      inv = 1.0f / sum;
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int s = lane; s < L; s += 32) p[s] *= inv;
    __syncwarp();
    float a0 = 0.0f, a1 = 0.0f;
    for (int s = 0; s < L; ++s) {
      const float* v = sV + (size_t)(start + s - w0) * HD;
      const float ps = p[s];
      a0 += ps * v[lane];
      a1 += ps * v[lane + 32];
    }
    out[(size_t)t * heads * HD + (size_t)h * HD + lane] = a0;
    out[(size_t)t * heads * HD + (size_t)h * HD + lane + 32] = a1;
    if (xs) {  // the o projection's split operand rows
      xs_store1(xs, heads * HD, t, h * HD + lane, a0);
      xs_store1(xs, heads * HD, t, h * HD + lane + 32, a1);
      if (fmaxf(fabsf(a0), fabsf(a1)) > 65504.0f) atomicOr(err, kErrFp16Input);
    }
    __syncwarp();  // p is rewritten for this warp's next frame
  }
}
size_t attn_smem(int window) {
  return (attn_k_floats(window) + (size_t)(kAttnFrames + window - 1) * 64 + kAttnWarps * (size_t)window +
          (size_t)kAttnFrames * 64) * sizeof(float);
}

// [T][n] -> [n][T] (the channel-first result), through a 32 x 33 tile
__global__ void dec_transpose_kernel(const float* in, int T, int n, float* out) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, t0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int t = t0 + r, c = c0 + threadIdx.x;
    if (t < T && c < n) tile[r][threadIdx.x] = in[(size_t)t * n + c];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int c = c0 + r, t = t0 + threadIdx.x;
    if (t < T && c < n) out[(size_t)c * T + t] = tile[threadIdx.x][r];
  }
}

// the MLP's silu(gate) * up (decoder.rs:307-311) on a gate|up row
__global__ void dec_swiglu_kernel(const float* GU, int T, int I, float* Hout) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * I) return;
  const long t = i / I, j = i % I;
  const float g = GU[t * 2 * I + j], u = GU[t * 2 * I + I + j];
  Hout[i] = (g / (1.0f + expf(-g))) * u;
}

cudaError_t gemm(cudaStream_t st, const DecGemm& g) {
  if (g.M <= 0) return cudaSuccess;
  const dim3 grid((g.N + kBN - 1) / kBN, (g.M + kBM - 1) / kBM);
  ++g_kernel_launches;
  dec_gemm_kernel<<<grid, kGemmThreads, 0, st>>>(g);
  return cudaGetLastError();
}

}  // namespace

// ---------------------------------------------------------------------------
// host side

struct DecLayerDev {
  float *wqkv, *wo, *wgu, *wdown, *in_norm, *post_norm, *attn_scale, *mlp_scale;
  Q4Mat tqkv, to, tg, tu, td;  // the same weights as tensor-core operand tiles (wx)
};
struct Decoder {
  int device = 0;
  uint32_t hidden = 0, heads = 0, head_dim = 0, inter = 0, window = 0, cb_dim = 0, entries = 0;
  long rope_len = 0;
  std::vector<void*> allocs;
  float *cb0 = nullptr, *cb_rest = nullptr, *proj0 = nullptr, *proj_rest = nullptr;
  float *pre_w = nullptr, *pre_b = nullptr, *in_w = nullptr, *in_b = nullptr;
  float *norm = nullptr, *out_w = nullptr, *out_b = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
  std::vector<DecLayerDev> layers;
  bool tc = false;  // the layer projections run on the tensor cores (T >= kTcMinRows)
  Q4Mat tin;        // input projection tiles
  Q4Mat tpre, tout; // pre-conv ([tap][in] x out) and output projection tiles
  // grow-only scratch for T frames
  int cap_T = 0;
  float *E0 = nullptr, *S = nullptr, *vq = nullptr, *pre = nullptr, *x = nullptr, *xn = nullptr, *qkv = nullptr,
        *ao = nullptr, *gu = nullptr, *h = nullptr, *tmp = nullptr;
  uint8_t* xs = nullptr;  // split input rows of the tensor-core projections
  size_t xs_bytes = 0;
  uint8_t *xs2a = nullptr, *xs2b = nullptr;  // the same, written by the rows' producers (alternating)
  uint32_t* codes = nullptr;
  float* out = nullptr;
  int cap_io = 0;
  unsigned* err = nullptr;
  cudaStream_t st = nullptr;
  ~Decoder() {
    if (st) cudaStreamSynchronize(st);
    for (void* p : allocs)
      if (p) cudaFree(p);
    cudaFree(E0); cudaFree(xs); cudaFree(xs2a); cudaFree(xs2b); cudaFree(codes); cudaFree(out);
    if (st) cudaStreamDestroy(st);
  }
};

}  // namespace qtts

struct qtts_decoder {
  qtts::Decoder* d;
};

namespace qtts {
namespace {

int read_vec(FILE* f, const HVec& v, std::vector<float>& out) {
  out.resize(v.len);
  if (v.len == 0) return QTTS_OK;
  if (fseeko(f, (off_t)v.off, SEEK_SET) != 0 || fread(out.data(), 4, v.len, f) != v.len)
    return fail(QTTS_ERR_IO, "decoder tensor read failed");
  return QTTS_OK;
}

int upload(Decoder& D, const std::vector<float>& h, float** dev) {
  *dev = nullptr;
  if (h.empty()) return fail(QTTS_ERR_FORMAT, "empty decoder tensor");
  if (cudaMalloc(reinterpret_cast<void**>(dev), h.size() * 4) != cudaSuccess)
    return fail(QTTS_ERR_OOM, "device allocation failed");
  D.allocs.push_back(*dev);
  if (cudaMemcpy(*dev, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(QTTS_ERR_CUDA, "decoder upload failed");
  return QTTS_OK;
}

int check_len(const HVec& v, uint64_t n, const char* what) {
  if (v.len != n) return fail(QTTS_ERR_FORMAT, std::string("decoder ") + what + " length mismatch");
  return QTTS_OK;
}

#define DRC(x)                 \
  do {                         \
    const int rc_ = (x);       \
    if (rc_ != QTTS_OK) return rc_; \
  } while (0)

int decoder_load(const char* path, int device, Decoder* D) {
  HModel hm;
  HDecoder hd;
  std::string err;
  int rc = parse_model(path, &hm, &err, &hd);
  if (rc != QTTS_OK) return fail(rc, err);
  if (hd.hidden == 0 || hd.heads == 0 || hd.head_dim == 0 || hd.cb_dim == 0 || hd.layers.empty())
    return fail(QTTS_ERR_FORMAT, "the file has no speech decoder");
  if (hd.head_dim != 64) return fail(QTTS_ERR_FORMAT, "decoder head_dim must be 64");
  if (hd.window == 0 || hd.window > (uint32_t)kDecMaxWindow) return fail(QTTS_ERR_FORMAT, "decoder window out of range");
  if (hd.hidden % 64 || hd.inter % 64 || hd.cb_dim % 4) return fail(QTTS_ERR_FORMAT, "decoder dims not multiples of 64");
  const uint64_t H = hd.hidden, A = (uint64_t)hd.heads * hd.head_dim, I = hd.inter, cb = hd.cb_dim;
  if (hd.cb0.len == 0 || hd.cb0.len % cb) return fail(QTTS_ERR_FORMAT, "decoder codebook length");
  const uint64_t entries = hd.cb0.len / cb;
  if (hd.cb_rest.size() != kDecGroups - 1) return fail(QTTS_ERR_FORMAT, "expected 15 rest codebooks");
  for (auto& v : hd.cb_rest) DRC(check_len(v, entries * cb, "codebook"));
  DRC(check_len(hd.proj0, cb * 512, "codebook projection"));
  DRC(check_len(hd.proj_rest, cb * 512, "codebook projection"));
  const HConv1d& pc = hd.pre_conv;
  if (pc.in != 512 || pc.out != 1024 || pc.k == 0 || pc.k > 8 || pc.dil != 1)
    return fail(QTTS_ERR_FORMAT, "decoder pre-conv shape");
  DRC(check_len(pc.w, (uint64_t)pc.out * pc.in * pc.k, "pre-conv weight"));
  DRC(check_len(pc.b, pc.out, "pre-conv bias"));
  DRC(check_len(hd.in_w, 1024 * H, "input projection"));
  DRC(check_len(hd.in_b, H, "input bias"));
  for (auto& L : hd.layers) {
    DRC(check_len(L.q, H * A, "q_proj")); DRC(check_len(L.k, H * A, "k_proj")); DRC(check_len(L.v, H * A, "v_proj"));
    DRC(check_len(L.o, A * H, "o_proj")); DRC(check_len(L.gate, H * I, "gate_proj")); DRC(check_len(L.up, H * I, "up_proj"));
    DRC(check_len(L.down, I * H, "down_proj")); DRC(check_len(L.in_norm, H, "norm")); DRC(check_len(L.post_norm, H, "norm"));
    DRC(check_len(L.attn_scale, H, "layer scale")); DRC(check_len(L.mlp_scale, H, "layer scale"));
  }
  DRC(check_len(hd.norm, H, "norm"));
  DRC(check_len(hd.out_w, H * 1024, "output projection"));
  DRC(check_len(hd.out_b, 1024, "output bias"));
  const uint64_t half = hd.head_dim / 2;
  if (hd.rope_cos.len == 0 || hd.rope_cos.len % half || hd.rope_sin.len != hd.rope_cos.len)
    return fail(QTTS_ERR_FORMAT, "decoder rope table length");

  if (cudaSetDevice(device) != cudaSuccess) return fail(QTTS_ERR_NODEV, "cudaSetDevice failed");
  D->device = device;
  D->hidden = hd.hidden; D->heads = hd.heads; D->head_dim = hd.head_dim; D->inter = hd.inter;
  D->window = hd.window; D->cb_dim = hd.cb_dim; D->entries = (uint32_t)entries;
  D->rope_len = (long)hd.rope_cos.len;
  if (cudaStreamCreateWithFlags(&D->st, cudaStreamNonBlocking) != cudaSuccess) return fail(QTTS_ERR_CUDA, "stream");
  if (cudaFuncSetAttribute(dec_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)attn_smem((int)hd.window)) != cudaSuccess)
    return fail(QTTS_ERR_CUDA, "decoder attention shared memory");
  if (cudaMalloc(reinterpret_cast<void**>(&D->err), 4) != cudaSuccess) return fail(QTTS_ERR_OOM, "device allocation failed");
  D->allocs.push_back(D->err);
  cudaMemset(D->err, 0, 4);

  FILE* f = fopen(path, "rb");
  if (!f) return fail(QTTS_ERR_IO, std::string("cannot open ") + path);
  struct Closer { FILE* f; ~Closer() { fclose(f); } } closer{f};
  std::vector<float> a, b;
  float wmax = 0.0f;  // largest |weight| of the projections that may take the tensor cores
  auto track = [&](const std::vector<float>& v) {
    for (float x : v) wmax = std::max(wmax, fabsf(x));
  };
  DRC(read_vec(f, hd.cb0, a)); DRC(upload(*D, a, &D->cb0));
  {
    std::vector<float> all;
    all.reserve(entries * cb * (kDecGroups - 1));
    for (auto& v : hd.cb_rest) {
      DRC(read_vec(f, v, a));
      all.insert(all.end(), a.begin(), a.end());
    }
    DRC(upload(*D, all, &D->cb_rest));
  }
  DRC(read_vec(f, hd.proj0, a)); DRC(upload(*D, a, &D->proj0));
  DRC(read_vec(f, hd.proj_rest, a)); DRC(upload(*D, a, &D->proj_rest));
  {  // [out][in][k] -> [k][in][out]: the conv as a GEMM over k taps of the input rows
    DRC(read_vec(f, pc.w, a));
    b.assign(a.size(), 0.0f);
    for (uint32_t oc = 0; oc < pc.out; ++oc)
      for (uint32_t ic = 0; ic < pc.in; ++ic)
        for (uint32_t k = 0; k < pc.k; ++k)
          b[((size_t)k * pc.in + ic) * pc.out + oc] = a[((size_t)oc * pc.in + ic) * pc.k + k];
    DRC(upload(*D, b, &D->pre_w));
    DRC(read_vec(f, pc.b, a)); DRC(upload(*D, a, &D->pre_b));
  }
  DRC(read_vec(f, hd.in_w, a)); track(a); DRC(upload(*D, a, &D->in_w));
  DRC(read_vec(f, hd.in_b, a)); DRC(upload(*D, a, &D->in_b));
  for (auto& L : hd.layers) {
    DecLayerDev dl{};
    std::vector<float> q, k, v;
    DRC(read_vec(f, L.q, q)); DRC(read_vec(f, L.k, k)); DRC(read_vec(f, L.v, v));
    track(q); track(k); track(v);
    b.assign(H * 3 * A, 0.0f);  // row kk: q | k | v
    for (uint64_t r = 0; r < H; ++r) {
      memcpy(&b[r * 3 * A], &q[r * A], A * 4);
      memcpy(&b[r * 3 * A + A], &k[r * A], A * 4);
      memcpy(&b[r * 3 * A + 2 * A], &v[r * A], A * 4);
    }
    DRC(upload(*D, b, &dl.wqkv));
    DRC(read_vec(f, L.o, a)); track(a); DRC(upload(*D, a, &dl.wo));
    DRC(read_vec(f, L.gate, q)); DRC(read_vec(f, L.up, k));
    track(q); track(k);
    b.assign(H * 2 * I, 0.0f);  // row kk: gate | up
    for (uint64_t r = 0; r < H; ++r) {
      memcpy(&b[r * 2 * I], &q[r * I], I * 4);
      memcpy(&b[r * 2 * I + I], &k[r * I], I * 4);
    }
    DRC(upload(*D, b, &dl.wgu));
    DRC(read_vec(f, L.down, a)); track(a); DRC(upload(*D, a, &dl.wdown));
    DRC(read_vec(f, L.in_norm, a)); DRC(upload(*D, a, &dl.in_norm));
    DRC(read_vec(f, L.post_norm, a)); DRC(upload(*D, a, &dl.post_norm));
    DRC(read_vec(f, L.attn_scale, a)); DRC(upload(*D, a, &dl.attn_scale));
    DRC(read_vec(f, L.mlp_scale, a)); DRC(upload(*D, a, &dl.mlp_scale));
    D->layers.push_back(dl);
  }
  DRC(read_vec(f, hd.norm, a)); DRC(upload(*D, a, &D->norm));
  DRC(read_vec(f, hd.out_w, a)); DRC(upload(*D, a, &D->out_w));
  DRC(read_vec(f, hd.out_b, a)); DRC(upload(*D, a, &D->out_b));
  DRC(read_vec(f, hd.rope_cos, a)); DRC(upload(*D, a, &D->rope_cos));
  DRC(read_vec(f, hd.rope_sin, a)); DRC(upload(*D, a, &D->rope_sin));
  // The layer projections (and the input projection) also as tensor-core
  // operand tiles: fp16 hi + lo of each f32 weight (~22 significand bits),
  // while every weight is inside the fp16 range
  if (wmax < 60000.0f) {
    auto expand = [&](const float* w, uint32_t k, uint32_t n, long ld, int col0, Q4Mat* m) {
      uint8_t* t = nullptr;
      if (cudaMalloc(reinterpret_cast<void**>(&t), tc_expand_bytes((int)k, (int)n)) != cudaSuccess)
        return fail(QTTS_ERR_OOM, "device allocation failed");
      D->allocs.push_back(t);
      if (tc_expand_f32(w, (int)k, (int)n, ld, col0, t, D->st) != cudaSuccess)
        return fail(QTTS_ERR_CUDA, "decoder weight expansion failed");
      m->k = (int)k;
      m->n = (int)n;
      m->wx = t;
      return (int)QTTS_OK;
    };
    DRC(expand(D->in_w, 1024, (uint32_t)H, (long)H, 0, &D->tin));
    DRC(expand(D->pre_w, 3 * 512, 1024, 1024, 0, &D->tpre));
    DRC(expand(D->out_w, (uint32_t)H, 1024, 1024, 0, &D->tout));
    for (DecLayerDev& L : D->layers) {
      DRC(expand(L.wqkv, (uint32_t)H, (uint32_t)(3 * A), (long)(3 * A), 0, &L.tqkv));
      DRC(expand(L.wo, (uint32_t)A, (uint32_t)H, (long)H, 0, &L.to));
      DRC(expand(L.wgu, (uint32_t)H, (uint32_t)I, (long)(2 * I), 0, &L.tg));
      DRC(expand(L.wgu, (uint32_t)H, (uint32_t)I, (long)(2 * I), (int)I, &L.tu));
      DRC(expand(L.wdown, (uint32_t)I, (uint32_t)H, (long)H, 0, &L.td));
    }
    if (cudaStreamSynchronize(D->st) != cudaSuccess) return fail(QTTS_ERR_CUDA, "decoder weight expansion failed");
    D->tc = true;
  }
  return QTTS_OK;
}

int ensure_scratch(Decoder& D, int T) {
  if (T <= D.cap_T) return QTTS_OK;
  if (D.st) cudaStreamSynchronize(D.st);
  cudaFree(D.E0);
  cudaFree(D.xs);
  cudaFree(D.xs2a);
  cudaFree(D.xs2b);
  D.E0 = nullptr;
  D.xs = D.xs2a = D.xs2b = nullptr;
  D.cap_T = 0;
  const size_t H = D.hidden, A = (size_t)D.heads * D.head_dim, I = D.inter, cb = D.cb_dim;
  const size_t per = 2 * cb + 512 + 1024 + 2 * H + 3 * A + A + 2 * I + I + H;
  if (D.tc) {  // the largest K of the tensor-core projections: 1024 (input, o) or the MLP width (down)
    // the largest K of the tensor-core projections: the pre-conv's 3 x 512
    D.xs_bytes = tc_xsplit_scratch_bytes(T, (int)std::max<size_t>(std::max<size_t>(3 * 512, A), I));
    if (cudaMalloc(reinterpret_cast<void**>(&D.xs), D.xs_bytes) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&D.xs2a), D.xs_bytes) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&D.xs2b), D.xs_bytes) != cudaSuccess)
      return fail(QTTS_ERR_OOM, "device allocation failed");
  }
  float* base = nullptr;
  if (cudaMalloc(reinterpret_cast<void**>(&base), per * (size_t)T * 4) != cudaSuccess)
    return fail(QTTS_ERR_OOM, "device allocation failed");
  float* p = base;
  auto take = [&](size_t n) { float* r = p; p += n * (size_t)T; return r; };
  D.E0 = take(cb); D.S = take(cb); D.vq = take(512); D.pre = take(1024); D.x = take(H); D.xn = take(H);
  D.qkv = take(3 * A); D.ao = take(A); D.gu = take(2 * I); D.h = take(I); D.tmp = take(H);
  D.cap_T = T;
  return QTTS_OK;
}

cudaError_t rms(Decoder& D, float* X, int T, int n, const float* gamma, float* Y, uint8_t* xs = nullptr,
               const float* add = nullptr, const float* add_scale = nullptr) {
  ++g_kernel_launches;
  dec_rmsnorm_kernel<<<(T + 7) / 8, 256, 0, D.st>>>(X, T, n, gamma, 1e-5f, Y, xs, reinterpret_cast<int*>(D.err),
                                                    add, add_scale);
  return cudaGetLastError();
}

// The whole stage for T frames on D.st: codes (device [16][T]) -> out
// (device [1024][T]).  Launch-time errors only; a bad code is recorded in
// D.err by the gather kernel.
int decode_dev(Decoder& D, const uint32_t* codes, int T, float* out) {
  DRC(ensure_scratch(D, T));
  const int H = (int)D.hidden, A = (int)(D.heads * D.head_dim), I = (int)D.inter, cb = (int)D.cb_dim;
  cudaError_t e = cudaSuccess;
  auto ok = [&](cudaError_t x) { if (e == cudaSuccess) e = x; };
  ++g_kernel_launches;
  dec_gather_kernel<<<T, 256, 0, D.st>>>(codes, T, (int)D.entries, cb, D.cb0, D.cb_rest, D.E0, D.S, D.err);
  ok(cudaGetLastError());
  DecGemm g{};
  g.taps = 1; g.cin = 1;
  auto plain = [&](const float* Ain, int K, const float* B, int N, float* C, const float* bias, int mode,
                   const float* scale) {
    DecGemm t = g;
    t.A = Ain; t.lda = K; t.M = T; t.K = K; t.N = N; t.B = B; t.bias = bias; t.scale = scale;
    t.C = C; t.ldc = N; t.mode = mode; t.trans = 0;
    ok(gemm(D.st, t));
  };
  // the pre-conv and every projection from the input projection on run on
  // the tensor cores from T >= 16 frames (the projection kernel's smallest
  // row block); the codebook projections stay on the CUDA cores
  const bool tc = D.tc && T >= kTcMinRows;
  int* tc_err = reinterpret_cast<int*>(D.err);
  auto proj = [&](const Q4Mat* mats, int nmat, int epi, const float* X, int ldx, float* C, int ldo,
                  const float* bias, const uint8_t* pre = nullptr, uint8_t* xs_out = nullptr) {
    return tc_project_expanded(mats, nmat, epi, X, ldx, T, C, ldo, bias, D.xs, D.xs_bytes, pre, xs_out, tc_err,
                               D.st);
  };
  plain(D.E0, cb, D.proj0, 512, D.vq, nullptr, 0, nullptr);
  if (tc) {
    // the finished codebook rows go out as the causal conv's split operand
    // rows (3 taps of 512), and the conv is a tensor-core projection
    DecGemm t = g;
    t.A = D.S; t.lda = cb; t.M = T; t.K = cb; t.N = 512; t.B = D.proj_rest; t.C = D.vq; t.ldc = 512; t.mode = 1;
    t.conv_xs = D.xs2a; t.err = tc_err;
    ok(gemm(D.st, t));
    DRC(proj(&D.tpre, 1, EPI_STORE, D.vq, 3 * 512, D.pre, 1024, D.pre_b, D.xs2a));
  } else {
    plain(D.S, cb, D.proj_rest, 512, D.vq, nullptr, 1, nullptr);
    DecGemm t = g;  // causal conv: 3 taps of 512 input channels
    t.A = D.vq; t.lda = 512; t.M = T; t.K = 3 * 512; t.N = 1024; t.taps = 3; t.cin = 512;
    t.B = D.pre_w; t.bias = D.pre_b; t.C = D.pre; t.ldc = 1024; t.mode = 0;
    ok(gemm(D.st, t));
  }
  // above 64 frames every layer projection takes its rows split by their
  // producer (RMSNorm, attention, the gate|up epilogue) from one of two
  // buffers that alternate, instead of a split launch of its own
  uint8_t* xa = (tc && T > 64) ? D.xs2a : nullptr;
  uint8_t* xb = (tc && T > 64) ? D.xs2b : nullptr;
  // On the tensor-core path o and down write their products to tmp and the
  // next RMSNorm applies the layer-scaled residual x += tmp * scale first.
  const float* pending = nullptr;  // the layer scale of a residual not yet applied
  if (tc) DRC(proj(&D.tin, 1, EPI_STORE, D.pre, 1024, D.x, H, D.in_b));
  else plain(D.pre, 1024, D.in_w, H, D.x, D.in_b, 0, nullptr);
  for (const DecLayerDev& L : D.layers) {
    ok(rms(D, D.x, T, H, L.in_norm, D.xn, xa, pending ? D.tmp : nullptr, pending));
    pending = nullptr;
    if (tc) DRC(proj(&L.tqkv, 1, EPI_STORE, D.xn, H, D.qkv, 3 * A, nullptr, xa));
    else plain(D.xn, H, L.wqkv, 3 * A, D.qkv, nullptr, 0, nullptr);
    {
      const long n = (long)T * D.heads * (D.head_dim / 2) * 2;
      ++g_kernel_launches;
      dec_rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, D.st>>>(D.qkv, T, (int)D.heads, (int)D.head_dim,
                                                                    D.rope_cos, D.rope_sin, D.rope_len);
      ok(cudaGetLastError());
    }
    ++g_kernel_launches;
    dec_attn_kernel<64><<<dim3((unsigned)((T + kAttnFrames - 1) / kAttnFrames), D.heads), kAttnWarps * 32,
                          attn_smem((int)D.window),
                          D.st>>>(
        D.qkv, T, (int)D.heads, (int)D.window, D.ao, xb, tc_err);
    ok(cudaGetLastError());
    if (tc) {
      DRC(proj(&L.to, 1, EPI_STORE, D.ao, A, D.tmp, H, nullptr, xb));
      pending = L.attn_scale;
    } else {
      plain(D.ao, A, L.wo, H, D.x, nullptr, 2, L.attn_scale);
    }
    ok(rms(D, D.x, T, H, L.post_norm, D.xn, xa, pending ? D.tmp : nullptr, pending));
    pending = nullptr;
    if (tc) {
      const Q4Mat gu[2] = {L.tg, L.tu};  // silu(gate) * up in the projection's epilogue
      DRC(proj(gu, 2, EPI_SWIGLU, D.xn, H, D.h, I, nullptr, xa, xb));
      DRC(proj(&L.td, 1, EPI_STORE, D.h, I, D.tmp, H, nullptr, xb));
      pending = L.mlp_scale;
    } else {
      plain(D.xn, H, L.wgu, 2 * I, D.gu, nullptr, 0, nullptr);
      const long n = (long)T * I;
      ++g_kernel_launches;
      dec_swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, D.st>>>(D.gu, T, I, D.h);
      ok(cudaGetLastError());
      plain(D.h, I, L.wdown, H, D.x, nullptr, 2, L.mlp_scale);
    }
  }
  ok(rms(D, D.x, T, H, D.norm, D.xn, xa, pending ? D.tmp : nullptr, pending));
  if (tc) {  // frame-major into the free pre-conv buffer, then channel-first [1024][T]
    DRC(proj(&D.tout, 1, EPI_STORE, D.xn, H, D.pre, 1024, D.out_b, xa));
    ++g_kernel_launches;
    dec_transpose_kernel<<<dim3(1024 / 32, (unsigned)((T + 31) / 32)), dim3(32, 8), 0, D.st>>>(D.pre, T, 1024, out);
    ok(cudaGetLastError());
  } else {
    DecGemm t = g;  // channel-first output [1024][T]
    t.A = D.xn; t.lda = H; t.M = T; t.K = H; t.N = 1024; t.B = D.out_w; t.bias = D.out_b;
    t.C = out; t.ldc = T; t.mode = 0; t.trans = 1;
    ok(gemm(D.st, t));
  }
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("decoder launch: ") + cudaGetErrorString(e));
  return QTTS_OK;
}

int check_err(Decoder& D) {
  unsigned h = 0;
  if (cudaMemcpyAsync(&h, D.err, 4, cudaMemcpyDeviceToHost, D.st) != cudaSuccess ||
      cudaStreamSynchronize(D.st) != cudaSuccess)
    return fail(QTTS_ERR_CUDA, std::string("decoder: ") + cudaGetErrorString(cudaGetLastError()));
  if (h) {
    cudaMemsetAsync(D.err, 0, 4, D.st);
    cudaStreamSynchronize(D.st);
    if (h & kDecErrCode) return fail(QTTS_ERR_RANGE, "decoder: a code index is past its codebook");
    if (h & kErrWaitExpired) return fail(QTTS_ERR_TIMEOUT, "decoder: a bounded device wait expired");
    return fail(QTTS_ERR_RANGE, "decoder: a tensor-core input outside the fp16 range");
  }
  return QTTS_OK;
}

}  // namespace
}  // namespace qtts

using qtts::fail;

int qtts_decoder_load(const char* path, int device, qtts_decoder** out) {
  if (!path || !out) return fail(QTTS_ERR_BADARG, "null argument");
  *out = nullptr;
  auto* D = new qtts::Decoder();
  const int rc = qtts::decoder_load(path, device, D);
  if (rc != QTTS_OK) {
    delete D;
    return rc;
  }
  *out = new qtts_decoder{D};
  return QTTS_OK;
}

int qtts_decoder_free(qtts_decoder* h) {
  if (!h) return QTTS_OK;
  cudaSetDevice(h->d->device);
  delete h->d;
  delete h;
  return QTTS_OK;
}

void* qtts_decoder_stream(qtts_decoder* h) { return h ? h->d->st : nullptr; }

int qtts_decode_latent_dev(qtts_decoder* h, const uint32_t* codes, int n_frames, float* out) {
  if (!h || !codes || !out || n_frames <= 0) return fail(QTTS_ERR_BADARG, "bad decoder arguments");
  if (cudaSetDevice(h->d->device) != cudaSuccess) return fail(QTTS_ERR_NODEV, "cudaSetDevice failed");
  return qtts::decode_dev(*h->d, codes, n_frames, out);
}

int qtts_decoder_sync(qtts_decoder* h) {
  if (!h) return fail(QTTS_ERR_BADARG, "null argument");
  if (cudaSetDevice(h->d->device) != cudaSuccess) return fail(QTTS_ERR_NODEV, "cudaSetDevice failed");
  return qtts::check_err(*h->d);
}

int qtts_decode_latent(qtts_decoder* h, const uint32_t* codes, int n_frames, float* out) {
  if (!h || !codes || !out || n_frames <= 0) return fail(QTTS_ERR_BADARG, "bad decoder arguments");
  qtts::Decoder& D = *h->d;
  if (cudaSetDevice(D.device) != cudaSuccess) return fail(QTTS_ERR_NODEV, "cudaSetDevice failed");
  for (long i = 0; i < (long)qtts::kDecGroups * n_frames; ++i)
    if (codes[i] >= D.entries) return fail(QTTS_ERR_RANGE, "decoder: a code index is past its codebook");
  if (n_frames > D.cap_io) {
    cudaStreamSynchronize(D.st);
    cudaFree(D.codes);
    cudaFree(D.out);
    D.codes = nullptr;
    D.out = nullptr;
    D.cap_io = 0;
    if (cudaMalloc(reinterpret_cast<void**>(&D.codes), (size_t)qtts::kDecGroups * n_frames * 4) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&D.out), (size_t)1024 * n_frames * 4) != cudaSuccess)
      return fail(QTTS_ERR_OOM, "device allocation failed");
    D.cap_io = n_frames;
  }
  if (cudaMemcpyAsync(D.codes, codes, (size_t)qtts::kDecGroups * n_frames * 4, cudaMemcpyHostToDevice, D.st) !=
      cudaSuccess)
    return fail(QTTS_ERR_CUDA, "decoder: code upload failed");
  const int rc = qtts::decode_dev(D, D.codes, n_frames, D.out);
  if (rc != QTTS_OK) return rc;
  if (cudaMemcpyAsync(out, D.out, (size_t)1024 * n_frames * 4, cudaMemcpyDeviceToHost, D.st) != cudaSuccess)
    return fail(QTTS_ERR_CUDA, "decoder: output copy failed");
  return qtts::check_err(D);
}

int qtts_synth_write_ex(const char* path, const qtts_dims* dims, uint64_t seed, unsigned flags) {
  if (!path || !dims) return fail(QTTS_ERR_BADARG, "null argument");
  if (flags & ~(unsigned)QTTS_SYNTH_DECODER) return fail(QTTS_ERR_BADARG, "unknown synth flags");
  std::string err;
  const int rc = qtts::synth_write(path, *dims, seed, &err, (flags & QTTS_SYNTH_DECODER) != 0);
  if (rc != QTTS_OK) return fail(rc, err);
  return QTTS_OK;
}
