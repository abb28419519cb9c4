// misc.cu -- embedding gathers, frame-input fusion, prefill row assembly,
// frame bookkeeping, whole-matrix dequant and the F16 GEMV (sm_100a).
#include "common.cuh"
#include "kernels.h"
#include "misc.h"

#include <algorithm>

namespace qtts {

constexpr int kMaxGridY = 65535;  // grid.y limit: row kernels loop over the rest

namespace {
constexpr LaunchOpts kPdl = {true, 1};
}  // namespace

// ---- frame input (generate_new.rs:255, 271-286) ---------------------------
// x[b][j] = (sem[j] + acs[j]) + text[j], with acs = ((0 + e_0) + e_1) ... + e_14
// accumulated in group order exactly like get_acoustic_embeddings_sum
// (code_predictor.rs:280-293).  Element-wise, so bit-identical to the CPU.
__global__ void fuse_kernel(const FuseDesc d) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d.H) return;  // H is a multiple of 256 whenever ssq_out is set (checked at launch)
  const uint32_t* codes;
  int f = 0, ntr = 0;
  if (d.codes_plain) {
    codes = d.codes_plain + (size_t)b * kMaxGroups;
  } else {
    const SlotState& sl = d.fc.slots[b];
    codes = sl.cur;
    f = sl.frame;
    ntr = sl.n_trail;
  }
  if (d.mode == 2) {  // acoustic sum only (codes[0..n_groups))
    float acs = 0.0f;
    for (int g = 0; g < d.n_groups; ++g) {
      const Q4Mat& E = d.group_emb[g];
      const uint32_t c = codes[g];
      acs = acs + q4_value(E.packed + (size_t)c * (E.n / 2), E.scales + (size_t)c * (E.n / 32), j);
    }
    d.x[(size_t)b * d.ldx + j] = acs;
    return;
  }
  const uint32_t c0 = codes[0];
  const float sem = q4_value(d.codec_emb.packed + (size_t)c0 * (d.codec_emb.n / 2),
                             d.codec_emb.scales + (size_t)c0 * (d.codec_emb.n / 32), j);
  if (d.sem_out) d.sem_out[(size_t)b * d.lds + j] = sem;
  if (d.mode == 1) return;
  float acs = 0.0f;
  for (int g = 0; g < d.n_groups; ++g) {
    const Q4Mat& E = d.group_emb[g];
    const uint32_t c = codes[g + 1];
    acs = acs + q4_value(E.packed + (size_t)c * (E.n / 2), E.scales + (size_t)c * (E.n / 32), j);
  }
  const float* ta = (f < ntr) ? d.trail + ((size_t)b * d.max_trail + f) * d.H : d.tts_pad;
  const float xv = (sem + acs) + ta[j];
  d.x[(size_t)b * d.ldx + j] = xv;
  if (d.ssq_out) {  // sums of squares of this tile's two 128-column blocks for the next RMSNorm
    __shared__ float sred[8];
    float q = xv * xv;
#pragma unroll
    for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = q;
    __syncthreads();
    if ((threadIdx.x & 127) == 0) {
      const int w0 = (threadIdx.x >> 5) & 4;
      d.ssq_out[(size_t)b * d.ssq_ld + blockIdx.x * 2 + (threadIdx.x >> 7)] =
          (sred[w0] + sred[w0 + 1]) + (sred[w0 + 2] + sred[w0 + 3]);
    }
  }
}

cudaError_t launch_fuse(const FuseDesc& d, cudaStream_t st) {
  if (d.B <= 0 || d.H <= 0 || (d.ssq_out && d.H % 256)) return cudaErrorInvalidValue;
  const dim3 grid((d.H + 255) / 256, d.B);
  return launch_k(fuse_kernel, dim3(grid), dim3(256), 0, st, kPdl, d);
}

// ---- gathers ----------------------------------------------------------------
__global__ void embed_rows_kernel(const Q4Mat m, const uint32_t* idx, int count, float* out, long ldo) {
  pdl_launch_dependents();
  pdl_wait();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m.n) return;
  for (int i = blockIdx.y; i < count; i += gridDim.y) {  // rows past grid.y's 65535 limit loop
    const uint32_t r = idx[i];
    out[(size_t)i * ldo + j] = q4_value(m.packed + (size_t)r * (m.n / 2), m.scales + (size_t)r * (m.n / 32), j);
  }
}
cudaError_t launch_embed_rows(const Q4Mat& mat, const uint32_t* idx, int count, float* out, long ldo,
                              cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  const dim3 grid((mat.n + 255) / 256, std::min(count, kMaxGridY));
  return launch_k(embed_rows_kernel, dim3(grid), dim3(256), 0, st, kPdl, mat, idx, count, out, ldo);
}

__global__ void embed_code0_kernel(const Q4Mat m, const SlotState* slots, float* out, long ldo) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m.n) return;
  const uint32_t r = slots[b].cur[0];
  out[(size_t)b * ldo + j] = q4_value(m.packed + (size_t)r * (m.n / 2), m.scales + (size_t)r * (m.n / 32), j);
}
cudaError_t launch_embed_code0(const Q4Mat& mat, const SlotState* slots, int B, float* out, long ldo,
                               cudaStream_t st) {
  const dim3 grid((mat.n + 255) / 256, B);
  return launch_k(embed_code0_kernel, dim3(grid), dim3(256), 0, st, kPdl, mat, slots, out, ldo);
}

__global__ void add_rows_kernel(const float* a, long lda, const float* b, long ldb, float* out, long ldo, int rows,
                                int n) {
  pdl_launch_dependents();
  pdl_wait();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) out[(size_t)r * ldo + j] = a[(size_t)r * lda + j] + b[(size_t)r * ldb + j];
}
cudaError_t launch_add_rows(const float* a, long lda, const float* b, long ldb, float* out, long ldo, int rows,
                            int n, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid((n + 255) / 256, std::min(rows, kMaxGridY));
  return launch_k(add_rows_kernel, dim3(grid), dim3(256), 0, st, kPdl, a, lda, b, ldb, out, ldo, rows, n);
}

// Prefill rows of generate_new.rs:94-173: each row is codec_emb(tok) +
// text_proj(row), the raw voice embedding, or a text_proj row alone.
__global__ void assemble_kernel(const Q4Mat codec, const RowRecipe* rec, const float* tp, long ldtp,
                                const float* voice, long ldv, float* out, long ldo, int H, int rows) {
  pdl_launch_dependents();
  pdl_wait();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= H) return;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const RowRecipe q = rec[r];
    float v;
    if (q.voice >= 0) {
      v = voice[(size_t)q.voice * ldv + j];
    } else if (q.codec >= 0) {
      const float c = q4_value(codec.packed + (size_t)q.codec * (codec.n / 2),
                               codec.scales + (size_t)q.codec * (codec.n / 32), j);
      v = (q.tp >= 0) ? c + tp[(size_t)q.tp * ldtp + j] : c;
    } else {
      v = tp[(size_t)q.tp * ldtp + j];
    }
    out[(size_t)r * ldo + j] = v;
  }
}
cudaError_t launch_assemble(const Q4Mat& codec, const RowRecipe* rec, int rows, const float* tp, long ldtp,
                            const float* voice, long ldv, float* out, long ldo, int H, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid((H + 255) / 256, std::min(rows, kMaxGridY));
  return launch_k(assemble_kernel, dim3(grid), dim3(256), 0, st, kPdl, codec, rec, tp, ldtp, voice, ldv, out, ldo, H,
                  rows);
}

__global__ void gather_rows_kernel(const float* src, long lds, const int* idx, float* out, long ldo, int rows, int n) {
  pdl_launch_dependents();
  pdl_wait();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) out[(size_t)r * ldo + j] = src[(size_t)idx[r] * lds + j];
}
cudaError_t launch_gather_rows(const float* src, long lds, const int* idx, int rows, float* out, long ldo, int n,
                               cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid((n + 255) / 256, std::min(rows, kMaxGridY));
  return launch_k(gather_rows_kernel, dim3(grid), dim3(256), 0, st, kPdl, src, lds, idx, out, ldo, rows, n);
}

// ---- frame bookkeeping --------------------------------------------------------
__global__ void frame_end_kernel(SlotState* slots, int B) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  SlotState& s = slots[b];
  if (!s.done) {
    s.pos += 1;
    s.frame += 1;
    s.frames_out = s.frame;
  }
}
cudaError_t launch_frame_end(SlotState* slots, int B, cudaStream_t st) {
  return launch_k(frame_end_kernel, dim3((B + 127) / 128), dim3(128), 0, st, kPdl, slots, B);
}

// Copy logits / talker hidden of the current frame into dump buffers.
__global__ void dump_kernel(const SlotState* slots, const float* src, long lds, int n, float* dst, int max_frames) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const int f = slots[b].frame;
  if (f >= max_frames || slots[b].done) return;
  dst[((size_t)b * max_frames + f) * n + j] = src[(size_t)b * lds + j];
}
cudaError_t launch_dump(const SlotState* slots, int B, const float* src, long lds, int n, float* dst, int max_frames,
                        cudaStream_t st) {
  const dim3 grid((n + 255) / 256, B);
  return launch_k(dump_kernel, dim3(grid), dim3(256), 0, st, kPdl, slots, src, lds, n, dst, max_frames);
}

// ---- whole-matrix dequant (gemv.rs:378-400 applied to every row) --------------
__global__ void dequant_kernel(const Q4Mat m, float* out) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t total = (size_t)m.k * m.n / 2;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / (m.n / 2), cb = i % (m.n / 2);
    const uint8_t b = m.packed[i];
    const float s = h2f(m.scales[r * (m.n / 32) + (2 * cb) / 32]);
    out[r * m.n + 2 * cb] = s * (float)((int)(b & 0xF) - 8);
    out[r * m.n + 2 * cb + 1] = s * (float)((int)(b >> 4) - 8);
  }
}
cudaError_t launch_dequant(const Q4Mat& m, float* out, cudaStream_t st) {
  return launch_k(dequant_kernel, dim3(1184), dim3(256), 0, st, kPdl, m, out);
}

// ---- the sampler's exp, element-wise ----------------------------------------------
__global__ void expf_kernel(const float* x, float* y, int n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = expf_glibc(x[i]);
}
cudaError_t launch_expf(const float* x, float* y, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  expf_kernel<<<std::min((n + 255) / 256, 4096), 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

// ---- F16 GEMV (gemv.rs:183-196) -------------------------------------------------
// One thread per (row m, column pair); sequential over k like the reference
// loop, so each output is the reference's own summation order.
__global__ void f16_gemv_kernel(const __half* w, int k, int n, const float* x, int m, float* y) {
  pdl_launch_dependents();
  pdl_wait();
  const int j2 = blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * j2 >= n) return;
  for (int row = blockIdx.y; row < m; row += gridDim.y) {
    const float* xr = x + (size_t)row * k;
    float a0 = 0.0f, a1 = 0.0f;
    for (int kk = 0; kk < k; ++kk) {
      const __half2 wv = *reinterpret_cast<const __half2*>(w + (size_t)kk * n + 2 * j2);
      const float xv = xr[kk];
      a0 = __fadd_rn(a0, __fmul_rn(xv, __low2float(wv)));
      a1 = __fadd_rn(a1, __fmul_rn(xv, __high2float(wv)));
    }
    y[(size_t)row * n + 2 * j2] = a0;
    y[(size_t)row * n + 2 * j2 + 1] = a1;
  }
}
cudaError_t launch_f16_gemv(const __half* w, int k, int n, const float* x, int m, float* y, cudaStream_t st) {
  if (n % 2) return cudaErrorInvalidValue;
  if (m <= 0) return cudaSuccess;
  const dim3 grid((n / 2 + 127) / 128, std::min(m, kMaxGridY));
  return launch_k(f16_gemv_kernel, dim3(grid), dim3(128), 0, st, kPdl, w, k, n, x, m, y);
}

}  // namespace qtts
