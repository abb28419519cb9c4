// epilogue.cuh -- the projection epilogues shared by the CUDA-core GEMV
// kernels (gemv.cu) and the tensor-core GEMM (tc_gemm.cu): bias/SiLU store,
// residual add (+ per-tile sums of squares for the next RMSNorm), SwiGLU,
// QK-norm + RoPE + KV append, and the argmax of the greedy heads -- the
// per-step glue of talker.rs:279-349 and code_predictor.rs:448-505.
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace qtts {
namespace {

// L2 prefetch of the next projection's weights: every CTA of the launch takes
// an equal 16-byte-aligned share of each region and thread 0 issues one bulk
// prefetch per region (no registers, no shared memory, no completion to wait
// for).  DRAM then streams the next layer's weights while this one computes.
__device__ __forceinline__ void prefetch_next_weights(const GemvDesc& d) {
  if (threadIdx.x != 0) return;
  const unsigned nctas = gridDim.x * gridDim.y * gridDim.z;
  const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const uint32_t bytes = d.pf_bytes[i];
    if (!d.pf_ptr[i] || bytes == 0) continue;
    const uint32_t share = ((bytes + nctas - 1) / nctas + 15u) & ~15u;
    const uint32_t b0 = cta * share;
    if (b0 >= bytes) continue;
    const uint32_t n = min(share, bytes - b0) & ~15u;
    if (n == 0) continue;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(d.pf_ptr[i] + b0), "r"(n) : "memory");
  }
}

// RMSNorm scale of a row from the producer's per-tile sums of squares.
// The partial sums are loaded 16 at a time before any is added (one memory
// round trip per 16 tiles instead of one per few), then added in tile order;
// the zero padding adds exactly nothing.
__device__ __forceinline__ float inv_rms_from_ssq(const GemvDesc& d, int m) {
  const float* p = d.ssq_in + (size_t)m * d.ssq_ld;
  float ss = 0.0f;
  for (int t0 = 0; t0 < d.ssq_n; t0 += 16) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = t0 + j < d.ssq_n ? p[t0 + j] : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) ss += v[j];
  }
  return 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
}

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

// Final code of row m once every tile has folded its maximum into keys[m]
// (the key is (order key << 32) | column, so the last index wins ties):
// record it for the frame (teacher forcing substitutes the forced code) or
// in the plain code array, and reset the key.
__device__ __forceinline__ void argmax_finalize_row(const EpiDesc& e, const FrameCodes& fc, int m) {
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

// Sum over the thread's half of a 256-thread block (threads 0-127 / 128-255).
__device__ __forceinline__ float block_sum_half(float v, float* sbuf) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sbuf[warp] = v;
  __syncthreads();
  const int w0 = warp & 4;
  return (sbuf[w0] + sbuf[w0 + 1]) + (sbuf[w0 + 2] + sbuf[w0 + 3]);
}

// ---------------------------------------------------------------------------
// QKV epilogue inputs of one thread (column tcol + tid of matrix mat, input
// row m) gathered during the decode kernel's prologue, so the epilogue makes
// no dependent global round trip: the QK-norm weight (before the wait: a
// weight), the rope position (issued with the inputs), then the RoPE factors
// and the destination (issued once the position has arrived, consumed only
// after the reduction).
struct QkvPre {
  bool on = false;
  float g = 0.0f;                   // q_norm / k_norm weight of the column
  int m = 0, r = 0;                 // input row; its index within the session's rows
  int pos_raw = 0;                  // pos_base entry (or pos_const)
  int sess = 0, pos = 0, kvp = 0;
  int page = 0;                     // KV page of (sess, kvp)
  bool rope_ok = false;             // pos inside the RoPE table
  float c = 0.0f, sn = 0.0f;        // cos / sin of (pos, column % 64)
};
__device__ __forceinline__ void qkv_pre_weights(QkvPre& q, const GemvDesc& d, int mat, int col) {
  if (mat == 2 || col >= d.mat[mat].n) return;
  q.g = h2f((mat == 0 ? d.epi.q_norm : d.epi.k_norm)[col % kHeadDim]);
}
__device__ __forceinline__ void qkv_pre_pos(QkvPre& q, const GemvDesc& d, int m) {
  const RowPos& rp = d.epi.rp;  // row_pos, split in two loads' halves
  const int sl = m / rp.rows_per_sess;
  q.m = m;
  q.r = m - sl * rp.rows_per_sess;
  q.sess = rp.sess0 + sl;
  q.pos_raw = rp.pos_base ? rp.pos_base[q.sess * rp.pos_stride] : rp.pos_const;
}
// Loads whose results are consumed only in the epilogue (no stall here).
__device__ __forceinline__ void qkv_pre_rest(QkvPre& q, const GemvDesc& d, int mat, int col) {
  const EpiDesc& e = d.epi;
  q.pos = q.pos_raw + q.r;
  q.kvp = e.rp.kv_const >= 0 ? e.rp.kv_const + q.r : q.pos;
  if (col >= d.mat[mat].n) return;
  if (mat != 0) q.page = kv_page(e.kv, q.sess, q.kvp);
  if (mat == 2) return;
  const int half = kHeadDim / 2, i = (col % kHeadDim) % half;
  q.rope_ok = q.pos < e.rope_rows && q.pos >= 0;
  if (q.rope_ok) {
    q.c = e.rope_cos[(size_t)q.pos * half + i];
    q.sn = e.rope_sin[(size_t)q.pos * half + i];
  }
}
// Store of the column's value: to q_out, or to its K / V cache element.
__device__ __forceinline__ void qkv_put(const QkvPre& q, const EpiDesc& e, int mat, int col, float v) {
  if (mat == 0) {
    e.q_out[(size_t)q.m * e.ldq + col] = v;
    return;
  }
  kv_store1(e.kv, kv_elem(e.kv, q.page, q.kvp, mat == 2 ? 1 : 0, col / kHeadDim) + col % kHeadDim, v);
}

// ---------------------------------------------------------------------------
// Epilogues, run by the root CTA of a tile with v[a][mm] = column tcol+tid of
// matrix a for input row m0+mm.  All 256 threads take part.
template <int MB, int NM, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvDesc& d, const FrameCodes& fc, float (&v)[NM][MB], int mat,
                                              int tile, int tcol, int m0, int mcnt, int zb, float* sbuf,
                                              float* ybuf, const float* res_pre = nullptr,
                                              const QkvPre* qp = nullptr) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = d.mat[mat].n;
  const int col = tcol + tid;
  const bool cval = col < n;
  const EpiDesc& e = d.epi;
  if (EPI == EPI_STORE || EPI == EPI_RESID) {
    const int cgl = d.col0[mat] + col;
    const int ltile = (NM == 2 ? tile : tile - d.tile0[mat]);
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      float val = 0.0f;
      if (cval && mm < mcnt) {
        if (EPI == EPI_STORE) {
          val = v[0][mm];
          if (e.bias) val = val + e.bias[cgl];
          if ((e.act_silu >> mat) & 1) val = silu_ref(val);
          e.out[(size_t)(m0 + mm) * e.ldo + cgl] = val;
        } else {
          float* o = e.out + (size_t)(m0 + mm) * e.ldo + cgl;
          val = (res_pre ? res_pre[mm] : *o) + v[0][mm];  // residual loaded ahead by the caller when given
          *o = val;
        }
      }
      if (e.ssq_out) {  // uniform branch: every thread takes part in the half-tile sums
        const float ss = block_sum_half(val * val, sbuf);
        const int hb = ltile * 2 + (tid >> 7);  // 128-column block of the row
        if ((tid & 127) == 0 && mm < mcnt && tcol + (tid & 128) < n) e.ssq_out[(size_t)(m0 + mm) * e.ssq_ld + hb] = ss;
      }
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
    if (MB == 1 && qp && qp->on) {  // one row, everything it needs preloaded
      if (mat == 2) {
        if (cval) qkv_put(*qp, e, mat, col, v[0][0]);
        return;
      }
      const float x = cval ? v[0][0] : 0.0f;
      float sq = x * x;
#pragma unroll
      for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      __syncthreads();
      if (lane == 0) sbuf[warp] = sq;
      __syncthreads();
      const float ss = sbuf[hl * 4 + 0] + sbuf[hl * 4 + 1] + sbuf[hl * 4 + 2] + sbuf[hl * 4 + 3];
      const float inv = 1.0f / sqrtf(ss / (float)kHeadDim + 1e-6f);
      const float y = x * inv * qp->g;
      ybuf[tid] = y;
      __syncthreads();
      const int half = kHeadDim / 2, i = dd % half;
      const float x1 = ybuf[hl * kHeadDim + i];
      const float x2 = ybuf[hl * kHeadDim + half + i];
      if (cval) {
        float outv = y;
        if (qp->rope_ok) {
          outv = (dd < half) ? (x1 * qp->c - x2 * qp->sn) : (x2 * qp->c + x1 * qp->sn);
        } else if (!e.rope_skip_oob && e.err_flag) {
          atomicOr(e.err_flag, kErrRopeRange);
        }
        qkv_put(*qp, e, mat, col, outv);
      }
      return;
    }
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      const int m = m0 + mm;
      const bool live = mm < mcnt;
      int sess = 0, pos = 0, kvp = 0;
      if (live) row_pos(e.rp, m, sess, pos, kvp);
      if (mat == 2) {
        if (live && cval) kv_store1(e.kv, kv_at(e.kv, sess, kvp, 1, h) + dd, v[0][mm]);
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
          atomicOr(e.err_flag, kErrRopeRange);
        }
        if (mat == 0) {
          e.q_out[(size_t)m * e.ldq + col] = outv;
        } else {
          kv_store1(e.kv, kv_at(e.kv, sess, kvp, 0, h) + dd, outv);
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
    if (tid < mcnt) argmax_finalize_row(e, fc, m0 + tid);
    if (tid == 0) e.counters2[zb] = 0u;
  }
}

}  // namespace
}  // namespace qtts
