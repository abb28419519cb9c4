// gemv.cu -- Q4 g32 dequant + GEMV/skinny-GEMM for sm_100a with fused
// prologues (RMSNorm, embedding gather) and epilogues (bias/SiLU, residual,
// SwiGLU, QK-norm + RoPE + KV append, argmax).
//
// Replaces gemv.rs:222-309 (gemv_q4_inner / gemv_q4) and gemv.rs:311-375
// (gemm_q4) and fuses the per-step glue of talker.rs:279-349 and
// code_predictor.rs:448-505 around them.
//
// Work decomposition.  The weight is [k][n] with groups of 32 along n, so an
// output column needs all k rows.  A CTA owns a 256-column tile (8 groups)
// and a contiguous slice of rows (split-K).  A warp load covers 4 rows x 128
// bytes (lane = (row quad, group)); a lane keeps 32 column accumulators per
// input row in registers.  Rows of the slice are interleaved across the 8
// warps.  After the slice, lanes reduce over their 4 row offsets with
// shuffles, warps reduce through shared memory, and the CTA writes its
// partial.  The last CTA of each tile (atomic ticket) sums the partials in
// split order -- the result is deterministic -- and runs the epilogue.
#include "common.cuh"
#include "kernels.h"

namespace qtts {

namespace {

__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

__device__ __forceinline__ float block_sum_256(float v, float* sbuf) {
  // all 256 threads participate; sbuf >= 8 floats
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sbuf[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += sbuf[w];
  return t;
}

__device__ __forceinline__ float* kv_row(const KvDesc& kv, int sess, int pos, int which, int h) {
  const int page = kv.page_table ? kv.page_table[sess * kv.pages_per_sess + pos / kPageSize] : sess;
  const size_t blk = (((size_t)page * kv.n_layers + kv.layer) * 2 + which) * kv.kv_heads + h;
  return kv.pool + (blk * kPageSize + (pos % kPageSize)) * kHeadDim;
}

}  // namespace

template <int MB, int NM, int EPI>
__global__ void __launch_bounds__(kGemvThreads) gemv_q4_kernel(const GemvDesc d, const FrameCodes fc) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y, zb = blockIdx.z;
  const int RPS = d.rows_per_split;
  float* xs = sm;                               // [MB][RPS]
  float* red = xs + MB * RPS;                   // [8][NM][MB][256]
  float* sbuf = red + 8 * NM * MB * kTileN;     // 64 floats
  float* ybuf = sbuf + 64;                      // [MB][256] (QKV epilogue)

  int mat = 0;
  if (NM == 1) {
    while (mat + 1 < d.nmat && tile >= d.tile0[mat + 1]) ++mat;
  }
  const int tcol = (NM == 2 ? tile : tile - d.tile0[mat]) * kTileN;
  const int n = d.mat[mat].n;
  const int r0 = split * RPS;
  const int r1 = min(d.k, r0 + RPS);
  const int R = max(0, r1 - r0);
  const int m0 = zb * MB;
  const int mcnt = min(MB, d.M - m0);

  // ---- prologue: rows [m0, m0+mcnt) x k-slice [r0, r1) -> shared memory
  for (int mm = 0; mm < MB; ++mm) {
    float* xd = xs + mm * RPS;
    if (mm >= mcnt) {
      for (int i = tid; i < R; i += kGemvThreads) xd[i] = 0.0f;
      continue;
    }
    const int m = m0 + mm;
    if (d.emb_idx) {
      const uint32_t row = d.emb_idx[(size_t)m * d.emb_idx_stride];
      const uint8_t* prow = d.emb.packed + (size_t)row * (d.emb.n / 2);
      const __half* srow = d.emb.scales + (size_t)row * (d.emb.n / 32);
      for (int i = tid; i < R; i += kGemvThreads) xd[i] = q4_value(prow, srow, r0 + i);
    } else {
      const float* xr = d.X + (size_t)m * d.ldx;
      if (d.gamma) {
        float ss = 0.0f;
        for (int i = tid; i < d.k; i += kGemvThreads) ss += xr[i] * xr[i];
        ss = block_sum_256(ss, sbuf);
        const float inv = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
        for (int i = tid; i < R; i += kGemvThreads) xd[i] = xr[r0 + i] * inv * h2f(d.gamma[r0 + i]);
        if (d.xnorm_out && tile == 0)
          for (int i = tid; i < R; i += kGemvThreads) d.xnorm_out[(size_t)m * d.ld_xnorm + r0 + i] = xd[i];
      } else {
        for (int i = tid; i < R; i += kGemvThreads) xd[i] = xr[r0 + i];
      }
    }
  }
  __syncthreads();

  // ---- main loop: stream the Q4 slice, accumulate 32 columns per lane
  const int rr = lane >> 3, gi = lane & 7;
  const int gcol = tcol + gi * 32;
  const bool gval = gcol < n;
  const size_t rowbytes = (size_t)n / 2;
  const int ngr = n / 32;
  float2 acc[NM][MB][16];
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int b = 0; b < MB; ++b)
#pragma unroll
      for (int c = 0; c < 16; ++c) acc[a][b][c] = make_float2(0.0f, 0.0f);

  constexpr int U = (NM * MB >= 4) ? 2 : 4;
  for (int rb = warp * 4 + rr; rb < R; rb += 32 * U) {
    uint4 w[U][NM];
    float s[U][NM];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int rbu = rb + 32 * u;
      const bool ok = gval && rbu < R;
#pragma unroll
      for (int a = 0; a < NM; ++a) {
        const Q4Mat& Mt = d.mat[NM == 2 ? a : mat];
        if (ok) {
          const size_t r = (size_t)(r0 + rbu);
          w[u][a] = ld_stream16(Mt.packed + r * rowbytes + gcol / 2);
          s[u][a] = h2f(Mt.scales[r * ngr + gcol / 32]);
        } else {
          w[u][a] = make_uint4(0, 0, 0, 0);
          s[u][a] = 0.0f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int rbu = rb + 32 * u;
      if (rbu < R) {
#pragma unroll
        for (int mm = 0; mm < MB; ++mm) {
          const float xv = xs[mm * RPS + rbu];
#pragma unroll
          for (int a = 0; a < NM; ++a) {
            const SxPack p = make_sx(s[u][a] * xv);  // s = scale * x (gemv.rs:239)
            q4_word_fma(w[u][a].x, p, &acc[a][mm][0]);
            q4_word_fma(w[u][a].y, p, &acc[a][mm][4]);
            q4_word_fma(w[u][a].z, p, &acc[a][mm][8]);
            q4_word_fma(w[u][a].w, p, &acc[a][mm][12]);
          }
        }
      }
    }
  }

  // ---- reduce the 4 row offsets of a warp, then the 8 warps
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int mm = 0; mm < MB; ++mm)
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float2 v = acc[a][mm][c];
        v.x += __shfl_xor_sync(0xffffffffu, v.x, 8);
        v.y += __shfl_xor_sync(0xffffffffu, v.y, 8);
        v.x += __shfl_xor_sync(0xffffffffu, v.x, 16);
        v.y += __shfl_xor_sync(0xffffffffu, v.y, 16);
        acc[a][mm][c] = v;
      }
  if (rr == 0) {
#pragma unroll
    for (int a = 0; a < NM; ++a)
#pragma unroll
      for (int mm = 0; mm < MB; ++mm) {
        float4* dst = reinterpret_cast<float4*>(red + ((warp * NM + a) * MB + mm) * kTileN + gi * 32);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          dst[c] = make_float4(acc[a][mm][2 * c].x, acc[a][mm][2 * c].y, acc[a][mm][2 * c + 1].x,
                               acc[a][mm][2 * c + 1].y);
      }
  }
  __syncthreads();
  float v[NM][MB];
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      float t = 0.0f;
#pragma unroll
      for (int w8 = 0; w8 < 8; ++w8) t += red[((w8 * NM + a) * MB + mm) * kTileN + tid];
      v[a][mm] = t;
    }

  const int col = tcol + tid;  // column within the matrix
  const bool cval = col < n;

  // ---- split-K: deterministic last-CTA reduction
  if (d.S > 1) {
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const int cg = d.col0[NM == 2 ? a : mat] + col;
#pragma unroll
      for (int mm = 0; mm < MB; ++mm)
        if (cval && mm < mcnt) d.part[((size_t)split * d.M + m0 + mm) * d.ncols + cg] = v[a][mm];
    }
    __threadfence();
    __syncthreads();
    __shared__ unsigned s_ticket;
    unsigned* ctr = d.counters + (size_t)tile * gridDim.z + zb;
    if (tid == 0) s_ticket = atomicAdd(ctr, 1u);
    __syncthreads();
    if (s_ticket != (unsigned)(d.S - 1)) return;
    __threadfence();
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const int cg = d.col0[NM == 2 ? a : mat] + col;
#pragma unroll
      for (int mm = 0; mm < MB; ++mm) {
        float t = 0.0f;
        if (cval && mm < mcnt)
          for (int sp = 0; sp < d.S; ++sp) t += ld_cg(d.part + ((size_t)sp * d.M + m0 + mm) * d.ncols + cg);
        v[a][mm] = t;
      }
    }
    if (tid == 0) *ctr = 0u;
  }

  // ---- epilogues
  const EpiDesc& e = d.epi;
  if (EPI == EPI_STORE) {
    const int cg = d.col0[mat] + col;
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      if (!cval || mm >= mcnt) continue;
      float val = v[0][mm];
      if (e.bias) val = val + e.bias[cg];
      if (e.act_silu) val = silu_ref(val);
      e.out[(size_t)(m0 + mm) * e.ldo + cg] = val;
    }
  } else if (EPI == EPI_RESID) {
    const int cg = d.col0[mat] + col;
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      if (!cval || mm >= mcnt) continue;
      float* o = e.out + (size_t)(m0 + mm) * e.ldo + cg;
      *o = *o + v[0][mm];
    }
  } else if (EPI == EPI_SWIGLU) {
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      if (!cval || mm >= mcnt) continue;
      e.out[(size_t)(m0 + mm) * e.ldo + col] = silu_ref(v[0][mm]) * v[NM - 1][mm];
    }
  } else if (EPI == EPI_QKV) {
    // mat 0 = q, 1 = k, 2 = v; heads of 128 columns never straddle a tile.
    const int h = col / kHeadDim, dd = col % kHeadDim, hl = tid / kHeadDim;
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      const int m = m0 + mm;
      const bool live = mm < mcnt;
      int sess = 0, pos = 0, kvp = 0;
      if (live) row_pos(e.rp, m, sess, pos, kvp);
      if (mat == 2) {
        if (live && cval) {
          KvDesc kv = e.kv;
          kv_row(kv, sess, kvp, 1, h)[dd] = v[0][mm];
        }
        continue;
      }
      // QK-norm (talker.rs:89-99): per head of 128 = 4 warps
      float x = (live && cval) ? v[0][mm] : 0.0f;
      float sq = x * x;
#pragma unroll
      for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      __syncthreads();
      if (lane == 0) sbuf[warp] = sq;
      __syncthreads();
      const float ss = sbuf[hl * 4 + 0] + sbuf[hl * 4 + 1] + sbuf[hl * 4 + 2] + sbuf[hl * 4 + 3];
      const float inv = 1.0f / sqrtf(ss / (float)kHeadDim + 1e-6f);
      const __half* g = (mat == 0) ? e.q_norm : e.k_norm;
      const float y = x * inv * h2f(g[dd]);
      ybuf[mm * kTileN + tid] = y;
      __syncthreads();
      // split-half RoPE (rope.rs:79-92, code_predictor.rs:108-120)
      const int half = kHeadDim / 2, i = dd % half;
      const float x1 = ybuf[mm * kTileN + hl * kHeadDim + i];
      const float x2 = ybuf[mm * kTileN + hl * kHeadDim + half + i];
      float outv = y;
      if (live && cval) {
        if (pos < e.rope_rows && pos >= 0) {
          const float c = e.rope_cos[(size_t)pos * half + i];
          const float sn = e.rope_sin[(size_t)pos * half + i];
          outv = (dd < half) ? (x1 * c - x2 * sn) : (x2 * c + x1 * sn);
        } else if (!e.rope_skip_oob && e.err_flag) {
          atomicOr(e.err_flag, 1);
        }
        if (mat == 0) {
          e.q_out[(size_t)m * e.ldq + col] = outv;
        } else {
          KvDesc kv = e.kv;
          kv_row(kv, sess, kvp, 0, h)[dd] = outv;
        }
      }
    }
  } else if (EPI == EPI_ARGMAX) {
    __shared__ unsigned long long s_key[8];
    __shared__ unsigned s_last;
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      unsigned long long key = 0ull;
      if (cval && mm < mcnt) key = ((unsigned long long)f32_order_key(v[0][mm]) << 32) | (unsigned)col;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      __syncthreads();
      if (lane == 0) s_key[warp] = key;
      __syncthreads();
      if (tid == 0 && mm < mcnt) {
        unsigned long long best = s_key[0];
        for (int w8 = 1; w8 < 8; ++w8) best = s_key[w8] > best ? s_key[w8] : best;
        atomicMax(e.keys + m0 + mm, best);
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(e.counters2 + zb, 1u);
    __syncthreads();
    if (s_last != (unsigned)(d.ntiles - 1)) return;
    __threadfence();
    if (tid < mcnt) {
      const int m = m0 + tid;
      const unsigned long long key = atomicExch(e.keys + m, 0ull);
      const uint32_t code = (uint32_t)(key & 0xffffffffull);
      if (e.frame_codes) {
        SlotState& sl = fc.slots[m];
        const int f = sl.frame;
        const size_t at = ((size_t)m * fc.max_frames + f) * kMaxGroups + e.group;
        uint32_t used = code;
        if (f < fc.max_frames) {
          fc.codes[at] = code;
          if (fc.forced) used = fc.forced[at];
        }
        sl.cur[e.group] = used;
        sl.prev[e.group] = used;
      } else {
        e.codes_plain[(size_t)m * kMaxGroups + e.group] = code;
      }
    }
    if (tid == 0) e.counters2[zb] = 0u;
  }
}

// ---------------------------------------------------------------------------
size_t gemv_smem_bytes(const GemvDesc& d) {
  const int NM = d.paired ? 2 : 1;
  return sizeof(float) * ((size_t)d.mb * d.rows_per_split + 8 * NM * d.mb * kTileN + 64 + d.mb * kTileN);
}

template <int MB, int NM, int EPI>
static cudaError_t launch_t(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  const size_t smem = gemv_smem_bytes(d);
  const dim3 grid(d.ntiles, d.S, (d.M + MB - 1) / MB);
  gemv_q4_kernel<MB, NM, EPI><<<grid, kGemvThreads, smem, st>>>(d, fc);
  return cudaGetLastError();
}

template <int MB, int NM, int EPI>
static void set_attr() {
  cudaFuncSetAttribute(gemv_q4_kernel<MB, NM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
}

// Opt every instantiation into large dynamic shared memory once per device
// (outside any stream capture).
void gemv_init_attributes() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
  set_attr<1, 1, EPI_STORE>(); set_attr<2, 1, EPI_STORE>(); set_attr<4, 1, EPI_STORE>();
  set_attr<1, 1, EPI_RESID>(); set_attr<2, 1, EPI_RESID>(); set_attr<4, 1, EPI_RESID>();
  set_attr<1, 1, EPI_QKV>(); set_attr<2, 1, EPI_QKV>(); set_attr<4, 1, EPI_QKV>();
  set_attr<1, 1, EPI_ARGMAX>(); set_attr<2, 1, EPI_ARGMAX>(); set_attr<4, 1, EPI_ARGMAX>();
  set_attr<1, 2, EPI_SWIGLU>(); set_attr<2, 2, EPI_SWIGLU>();
  cudaGetLastError();
  done[dev] = true;
}

template <int EPI>
static cudaError_t launch_mb(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  if (d.paired) {
    if (EPI != EPI_SWIGLU) return cudaErrorInvalidValue;
    if (d.mb == 1) return launch_t<1, 2, EPI_SWIGLU>(d, fc, st);
    if (d.mb == 2) return launch_t<2, 2, EPI_SWIGLU>(d, fc, st);
    return cudaErrorInvalidValue;
  }
  if (EPI == EPI_SWIGLU) return cudaErrorInvalidValue;
  constexpr int E = EPI == EPI_SWIGLU ? EPI_STORE : EPI;
  if (d.mb == 1) return launch_t<1, 1, E>(d, fc, st);
  if (d.mb == 2) return launch_t<2, 1, E>(d, fc, st);
  if (d.mb == 4) return launch_t<4, 1, E>(d, fc, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  if (d.ntiles <= 0 || d.S <= 0 || d.M <= 0 || d.rows_per_split <= 0) return cudaErrorInvalidValue;
  switch (d.epi_kind) {
    case EPI_STORE: return launch_mb<EPI_STORE>(d, fc, st);
    case EPI_RESID: return launch_mb<EPI_RESID>(d, fc, st);
    case EPI_SWIGLU: return launch_mb<EPI_SWIGLU>(d, fc, st);
    case EPI_QKV: return launch_mb<EPI_QKV>(d, fc, st);
    case EPI_ARGMAX: return launch_mb<EPI_ARGMAX>(d, fc, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qtts
