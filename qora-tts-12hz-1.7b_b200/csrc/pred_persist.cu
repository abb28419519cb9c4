// pred_persist.cu -- the code predictor of one utterance (batch 1) as one
// persistent cooperative kernel.
//
// generate_acoustic_codes (code_predictor.rs:218-273) is 15 dependent group
// steps, each input_proj + 5 layers + lm_head + argmax: ~400 dependent
// projections per frame whose 44 MB of weights stay in L2.  As separate
// kernels every one of them pays a launch and a completion; here one CTA per
// SM runs them all as phases separated by a grid barrier (a global counter,
// every spin bounded), which is what bounds this path.
//
// Phases of one group step (M = 2 rows for the prefill step, positions 0 and
// 1; M = 1 row at position g + 1 afterwards):
//   PROJ    input_proj of [talker hidden, semantic embedding] or of the
//           embedding row of the previous group's code (code_predictor.rs:235,
//           :256-258), K-split partials;
//   per layer (code_predictor.rs:448-505):
//   QKV     residual row = previous residual + sum of the producer's partials
//           (+ bias after PROJ), RMSNorm, q|k|v projection partials;
//   ATTN    one CTA per query head: sums its q/k/v partials, QK-norm,
//           split-half RoPE, appends k/v to the predictor KV page, causal
//           attention over positions [0, pos];
//   O       o_proj partials;
//   GATEUP  residual + o, RMSNorm, gate|up partials;
//   DOWN    silu(gate) * up, down_proj partials;
//   HEAD    final norm, lm_head[g] in 32-column units, argmax folded into an
//           atomicMax key ((order key << 32) | column: the last index wins
//           ties, code_predictor.rs:328-334).
// A projection phase splits its work into (column tile, K slice) units; the
// consumer phase sums the K slices in slice order (deterministic).
#include "common.cuh"
#include "kernels.h"

namespace qtts {

namespace {

constexpr int kThreads = kPPThreads;
constexpr unsigned kSpinLimit = 1u << 22;  // grid-barrier polls before giving up (~0.2 s)

__device__ __forceinline__ float u16_h2f(unsigned short s) { return __half2float(__ushort_as_half(s)); }
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier number `phase` (1-based) over a counter zeroed before the
// launch; every CTA of the cooperative grid takes part.
__device__ __forceinline__ void grid_sync(const PredPersistDesc& d, unsigned phase) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(d.bar, 1u);
    const unsigned target = phase * gridDim.x;
    unsigned it = 0;
    while (ld_acquire(d.bar) < target) {
      if (++it > kSpinLimit) {
        atomicOr(d.err_flag, kErrGridBarrier);
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
  }
  __syncthreads();
}

__device__ __forceinline__ float block_sum(float v, float* sred) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sred[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < kThreads / 32; ++w) t += sred[w];
  return t;
}

// The weight rows a thread reads for one unit, loaded ahead of time (before
// the grid barrier that precedes the unit's phase: weights never depend on an
// earlier phase).  Thread: 32-column chunk t % CW, row lane t / CW, rows
// r0 + rl + j * RL.
constexpr int kPre = 4;
struct WPre {
  uint4 w[kPre];
  unsigned short s[kPre];
};
__device__ __forceinline__ void prefetch_unit(const Q4Mat& W, int c0, int TW, int r0, int r1, WPre& pre) {
  const int CW = TW / 32, RL = kThreads / CW;
  const int t = threadIdx.x, chunk = t % CW, rl = t / CW;
  const int col = c0 + chunk * 32;
  const uint8_t* wp = W.packed + col / 2;
  const unsigned short* sp = reinterpret_cast<const unsigned short*>(W.scales) + col / 32;
  const size_t wrow = (size_t)W.n / 2, srow = (size_t)W.n / 32;
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int r = r0 + rl + j * RL;
    if (r < r1) {
      pre.w[j] = __ldg(reinterpret_cast<const uint4*>(wp + (size_t)r * wrow));
      pre.s[j] = __ldg(sp + (size_t)r * srow);
    }
  }
}

// One (column tile, K slice) unit: out[m][c] = sum_{r in [r0, r1)} xs[m][r - r0] * W[r][c0 + c]
// for c < TW, m < M, the first kPre rows of the thread from `pre` when given.
template <int M>
__device__ void gemv_unit(const Q4Mat& W, int c0, int TW, int r0, int r1, const WPre& pre, bool use_pre,
                          const float* xs, int xld, float* red, float* out, int ldo) {
  const int CW = TW / 32, RL = kThreads / CW;
  const int t = threadIdx.x, chunk = t % CW, rl = t / CW;
  float2 acc[M][16];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int c = 0; c < 16; ++c) acc[m][c] = make_float2(0.0f, 0.0f);
  const int col = c0 + chunk * 32;
  const uint8_t* wp = W.packed + col / 2;
  const unsigned short* sp = reinterpret_cast<const unsigned short*>(W.scales) + col / 32;
  const size_t wrow = (size_t)W.n / 2, srow = (size_t)W.n / 32;
  auto row = [&](int r, const uint4& w, unsigned short s16) {
    const float s = u16_h2f(s16);
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const SxPack p = make_sx(s * xs[m * xld + (r - r0)]);  // (scale * x) * (q - 8), gemv.rs:239
      q4_word_fma(w.x, p, &acc[m][0]);
      q4_word_fma(w.y, p, &acc[m][4]);
      q4_word_fma(w.z, p, &acc[m][8]);
      q4_word_fma(w.w, p, &acc[m][12]);
    }
  };
  if (use_pre) {
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int r = r0 + rl + j * RL;
      if (r < r1) row(r, pre.w[j], pre.s[j]);
    }
  }
#pragma unroll 4
  for (int r = r0 + rl + (use_pre ? kPre * RL : 0); r < r1; r += RL)
    row(r, __ldg(reinterpret_cast<const uint4*>(wp + (size_t)r * wrow)), __ldg(sp + (size_t)r * srow));
  // reduce the row lanes: first the 32 / CW lanes of a warp (butterfly over
  // the lane bits above the chunk bits), then the 8 warps through shared memory
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int c = 0; c < 16; ++c)
      for (int o = CW; o < 32; o <<= 1) {
        acc[m][c].x += __shfl_xor_sync(0xffffffffu, acc[m][c].x, o);
        acc[m][c].y += __shfl_xor_sync(0xffffffffu, acc[m][c].y, o);
      }
  const int warp = t >> 5, lane = t & 31;
  if (lane < CW) {  // lane == chunk of this warp's first row lane
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float4* dst = reinterpret_cast<float4*>(red + ((size_t)warp * M + m) * TW + chunk * 32);
#pragma unroll
      for (int c = 0; c < 8; ++c)
        dst[c] = make_float4(acc[m][2 * c].x, acc[m][2 * c].y, acc[m][2 * c + 1].x, acc[m][2 * c + 1].y);
    }
  }
  __syncthreads();
  for (int i = t; i < M * TW; i += kThreads) {
    const int m = i / TW, c = i % TW;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) v += red[((size_t)w * M + m) * TW + c];
    out[(size_t)m * ldo + c] = v;
  }
  __syncthreads();
}

// Sum of the S (<= kSMax) K-slice partials p[s * stride] in slice order, every
// load issued before the first add (one L2 round trip, not S).
constexpr int kSMax = 8;
__device__ __forceinline__ float sum_slices(const float* p, size_t stride, int S) {
  float v[kSMax];
#pragma unroll
  for (int s = 0; s < kSMax; ++s) v[s] = s < S ? __ldcg(p + s * stride) : 0.0f;
  float t = v[0];
#pragma unroll
  for (int s = 1; s < kSMax; ++s)
    if (s < S) t += v[s];
  return t;
}

struct Mats {  // up to three matrices side by side (concatenated columns)
  const Q4Mat* m[3];
  int nmat;
  int col0[4];
  __device__ int find(int col, int& local) const {
    int i = 0;
    while (i + 1 < nmat && col >= col0[i + 1]) ++i;
    local = col - col0[i];
    return i;
  }
};

// A projection phase: matrices, K, concatenated columns, tile width, K slices.
struct PhaseW {
  Mats W;
  int k, ncols, TW, S;
  __device__ int units() const { return (ncols / TW) * S; }
  // unit u -> matrix, local first column, rows [r0, r1), tile, slice
  __device__ const Q4Mat& unit(int u, int& c0, int& r0, int& r1, int& tile, int& s) const {
    const int tiles = ncols / TW, rps = (k + S - 1) / S;
    tile = u % tiles;
    s = u / tiles;
    r0 = s * rps;
    r1 = min(k, r0 + rps);
    const int mi = W.find(tile * TW, c0);
    return *W.m[mi];
  }
};

}  // namespace

// Grid: at most one CTA per SM (cooperative), kThreads threads, kPPSmem bytes.
__global__ void __launch_bounds__(kThreads, 1) pred_persist_kernel(const __grid_constant__ PredPersistDesc d) {
  pdl_wait();
  extern __shared__ __align__(16) float psm[];
  float* red = psm;                        // [8192 * 2] row-lane reduction
  float* xs = red + 8192 * 2;              // [2][kPPMaxSlice] unit input slice
  float* xfull = xs + 2 * kPPMaxSlice;     // [2][kPPMaxHidden] residual rows
  float* sred = xfull + 2 * kPPMaxHidden;  // [32] block sums
  float* sinv = sred + 32;                 // [2]
  float* qkv = sinv + 4;                   // [3][2][128] q, k, v of the current rows (ATTN)
  float* sc = qkv + 3 * 2 * kHeadDim;      // [2][kPPMaxPos] attention scores
  __shared__ uint32_t s_code;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pH = d.pH, qn = d.heads * kHeadDim, kn = d.kvh * kHeadDim, qkvn = qn + 2 * kn;
  const int G = d.heads / d.kvh;
  unsigned phase = 0;

  // partial-sum regions
  float* P_proj = d.part;
  float* P_qkv = P_proj + (size_t)d.s_proj * 2 * pH;
  float* P_o = P_qkv + (size_t)d.s_qkv * 2 * qkvn;
  float* P_gu = P_o + (size_t)d.s_o * 2 * pH;
  float* P_down = P_gu + (size_t)d.s_gu * 2 * 2 * d.inter;
  float* Xa = d.X;                 // layer input rows [2][pH]
  float* Xb = d.X + 2 * pH;        // rows after attention [2][pH]

  // projection phase over the units of (tiles x S), input slice built by `fill`
  WPre pre;  // weights of this CTA's first unit of the coming phase
  auto prefetch = [&](const PhaseW& ph) {
    if ((int)blockIdx.x < ph.units()) {
      int c0, r0, r1, tile, s;
      const Q4Mat& W = ph.unit(blockIdx.x, c0, r0, r1, tile, s);
      prefetch_unit(W, c0, ph.TW, r0, r1, pre);
    }
  };
  auto proj_phase = [&](const PhaseW& ph, int M, float* P, auto&& fill) {
    const int k = ph.k, ncols = ph.ncols, TW = ph.TW, units = ph.units(), rps = (k + ph.S - 1) / ph.S;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int c0, r0, r1, tile, s;
      const Q4Mat& Wm = ph.unit(u, c0, r0, r1, tile, s);
      for (int i0 = tid; i0 < M * rps; i0 += 2 * kThreads) {  // two elements' loads in flight
        float v[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int i = i0 + e * kThreads, m = i / rps, r = r0 + i % rps;
          v[e] = (i < M * rps && r < r1) ? fill(m, r) : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int i = i0 + e * kThreads, m = i / rps, r = r0 + i % rps;
          if (i < M * rps && r < r1) xs[m * kPPMaxSlice + (r - r0)] = v[e];
        }
      }
      __syncthreads();
      float* out = P + (size_t)s * M * ncols + tile * TW;
      // the two prefill rows run as two one-row passes (the second re-reads the
      // unit's weights from L2); keeps the unit's accumulators at one row
      for (int m = 0; m < M; ++m)
        gemv_unit<1>(Wm, c0, TW, r0, r1, pre, m == 0 && u == (int)blockIdx.x, xs + m * kPPMaxSlice, kPPMaxSlice,
                     red, out + (size_t)m * ncols, ncols);
    }
  };
  // residual rows into shared memory: base (may be null) + sum of S partial
  // slices (+ bias), optional write-back by CTA 0, 1/rms per row
  auto residual = [&](int M, const float* base, const float* P, int S, int ldp, const float* bias, float* wb) {
    constexpr int E = 4;  // elements per thread per batch, all loads in flight together
    for (int i0 = tid; i0 < M * pH; i0 += kThreads * E) {
      float bv[E], tv[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = i0 + e * kThreads;
        const int m = i / pH, c = i % pH;
        const bool ok = i < M * pH;
        bv[e] = (ok && base) ? __ldcg(base + (size_t)m * pH + c) : 0.0f;
        tv[e] = ok ? sum_slices(P + (size_t)m * ldp + c, (size_t)M * ldp, S) : 0.0f;
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = i0 + e * kThreads;
        if (i < M * pH) {
          const int m = i / pH, c = i % pH;
          float t = tv[e];
          if (bias) t = t + bias[c];
          const float v = base ? bv[e] + t : t;
          xfull[m * kPPMaxHidden + c] = v;
          if (wb && blockIdx.x == 0) wb[(size_t)m * pH + c] = v;
        }
      }
    }
    __syncthreads();
    for (int m = 0; m < M; ++m) {
      float ss = 0.0f;
      for (int c = tid; c < pH; c += kThreads) ss += xfull[m * kPPMaxHidden + c] * xfull[m * kPPMaxHidden + c];
      ss = block_sum(ss, sred);
      if (tid == 0) sinv[m] = 1.0f / sqrtf(ss / (float)pH + 1e-6f);  // gemv.rs:408-417
    }
    __syncthreads();
  };
  // the group code chosen by the last HEAD phase: record it, return the one used
  auto take_code = [&](int group, int parity) -> uint32_t {
    if (tid == 0) {
      const unsigned long long key = ld_acquire_u64(d.keys + parity);
      const uint32_t code = (uint32_t)(key & 0xffffffffull);
      uint32_t used = code;
      if (d.frame_mode) {
        SlotState& sl = d.fc.slots[0];
        const int f = sl.frame;
        const size_t at = (size_t)f * kMaxGroups + group;
        if (f < d.fc.max_frames) {
          if (d.fc.forced) used = d.fc.forced[at];
          if (blockIdx.x == 0) d.fc.codes[at] = code;
        }
        if (blockIdx.x == 0) {
          sl.cur[group] = used;
          sl.prev[group] = used;
        }
      } else if (blockIdx.x == 0) {
        d.codes_plain[group] = code;
      }
      s_code = used;
    }
    __syncthreads();
    return s_code;
  };

  const float scale = 1.0f / sqrtf((float)kHeadDim);
  // the projection phases (matrices, K, columns, tile width, K slices)
  auto ph_proj = [&]() { return PhaseW{Mats{{&d.proj, nullptr, nullptr}, 1, {0, pH, 0, 0}}, d.t_hidden, pH, 128, d.s_proj}; };
  auto ph_qkv = [&](int l) {
    return PhaseW{Mats{{&d.L[l].q, &d.L[l].k, &d.L[l].v}, 3, {0, qn, qn + kn, qkvn}}, pH, qkvn, 128, d.s_qkv};
  };
  auto ph_o = [&](int l) { return PhaseW{Mats{{&d.L[l].o, nullptr, nullptr}, 1, {0, pH, 0, 0}}, qn, pH, 128, d.s_o}; };
  auto ph_gu = [&](int l) {
    return PhaseW{Mats{{&d.L[l].gate, &d.L[l].up, nullptr}, 2, {0, d.inter, 2 * d.inter, 0}}, pH, 2 * d.inter, 128,
                  d.s_gu};
  };
  auto ph_down = [&](int l) {
    return PhaseW{Mats{{&d.L[l].down, nullptr, nullptr}, 1, {0, pH, 0, 0}}, d.inter, pH, 128, d.s_down};
  };
  auto ph_head = [&](int g) {
    return PhaseW{Mats{{&d.lm[g], nullptr, nullptr}, 1, {0, d.lm[g].n, 0, 0}}, pH, d.lm[g].n, 32, 1};
  };
  prefetch(ph_proj());
  for (int step = 0; step < d.groups; ++step) {
    const int M = step == 0 ? 2 : 1;
    const int pos0 = step == 0 ? 0 : step + 1;
    // ---- PROJ (code_predictor.rs:235-236, :256-258)
    {
      const PhaseW W = ph_proj();
      if (step == 0) {
        proj_phase(W, 2, P_proj, [&](int m, int r) { return d.pin[(size_t)m * d.t_hidden + r]; });
      } else {
        const uint32_t code = take_code(step, (step - 1) & 1);
        if (blockIdx.x == 0 && tid == 0) d.keys[step & 1] = 0ull;  // next HEAD's key
        const Q4Mat& E = d.emb[step - 1];
        const uint8_t* prow = E.packed + (size_t)code * (E.n / 2);
        const __half* srow = E.scales + (size_t)code * (E.n / 32);
        proj_phase(W, 1, P_proj, [&](int, int r) { return q4_value(prow, srow, r); });
      }
      prefetch(ph_qkv(0));
      grid_sync(d, ++phase);
    }
    for (int l = 0; l < d.layers; ++l) {
      const PPLayer& L = d.L[l];
      // ---- QKV
      if (l == 0)
        residual(M, nullptr, P_proj, d.s_proj, pH, d.proj_b, Xa);
      else
        residual(M, Xb, P_down, d.s_down, pH, nullptr, Xa);
      proj_phase(ph_qkv(l), M, P_qkv, [&](int m, int r) {
        return xfull[m * kPPMaxHidden + r] * sinv[m] * h2f(L.in_norm[r]);
      });
      prefetch(ph_o(l));  // held through the attention phase
      grid_sync(d, ++phase);
      // ---- ATTN: CTA h handles query head h
      for (int h = blockIdx.x; h < d.heads; h += gridDim.x) {
        const int hk = h / G;
        {
          float tv[3];
#pragma unroll
          for (int e = 0; e < 3; ++e) {
            const int i = tid + e * kThreads;
            const int which = i / (M * kHeadDim), m = (i / kHeadDim) % M, c = i % kHeadDim;
            const int col = which == 0 ? h * kHeadDim + c : qn + (which - 1) * kn + hk * kHeadDim + c;
            tv[e] = i < 3 * M * kHeadDim ? sum_slices(P_qkv + (size_t)m * qkvn + col, (size_t)M * qkvn, d.s_qkv) : 0.0f;
          }
#pragma unroll
          for (int e = 0; e < 3; ++e) {
            const int i = tid + e * kThreads;
            const int which = i / (M * kHeadDim), m = (i / kHeadDim) % M, c = i % kHeadDim;
            if (i < 3 * M * kHeadDim) qkv[(which * 2 + m) * kHeadDim + c] = tv[e];
          }
        }
        __syncthreads();
        // QK-norm (code_predictor.rs:84-93) and split-half RoPE (:97-121) of q and k
        for (int which = 0; which < 2; ++which) {
          for (int m = 0; m < M; ++m) {
            float* v = qkv + (which * 2 + m) * kHeadDim;
            float ss = tid < kHeadDim ? v[tid] * v[tid] : 0.0f;
            ss = block_sum(ss, sred);
            const float inv = 1.0f / sqrtf(ss / (float)kHeadDim + 1e-6f);
            const __half* g = which == 0 ? L.q_norm : L.k_norm;
            float y = 0.0f;
            if (tid < kHeadDim) y = v[tid] * inv * h2f(g[tid]);
            __syncthreads();
            if (tid < kHeadDim) v[tid] = y;
            __syncthreads();
            const int pos = pos0 + m, half = kHeadDim / 2;
            float o = 0.0f;
            if (tid < kHeadDim) {
              const int i = tid % half;
              const float x1 = v[i], x2 = v[half + i];
              o = v[tid];
              if (pos < d.rope_rows) {
                const float c = d.cos[(size_t)pos * half + i], sn = d.sin[(size_t)pos * half + i];
                o = tid < half ? (x1 * c - x2 * sn) : (x2 * c + x1 * sn);
              }
            }
            __syncthreads();
            if (tid < kHeadDim) v[tid] = o;
            __syncthreads();
          }
        }
        // append k, v of the current rows (the first query head of the group writes)
        if (h % G == 0) {
          for (int i = tid; i < 2 * M * kHeadDim; i += kThreads) {
            const int which = i / (M * kHeadDim), m = (i / kHeadDim) % M, c = i % kHeadDim;
            const int pos = pos0 + m;
            float* row = d.kv + ((((size_t)l * 2 + which) * d.kvh + hk) * kPageSize + pos) * kHeadDim;
            row[c] = qkv[((1 + which) * 2 + m) * kHeadDim + c];
          }
        }
        // causal attention of each row over positions [0, pos]
        for (int m = 0; m < M; ++m) {
          const int pos = pos0 + m;
          const float* q = qkv + m * kHeadDim;
          for (int j = warp; j <= pos; j += kThreads / 32) {
            const float* kr = j >= pos0 ? qkv + (2 + (j - pos0)) * kHeadDim
                                        : d.kv + ((((size_t)l * 2 + 0) * d.kvh + hk) * kPageSize + j) * kHeadDim;
            float dot = 0.0f;
            for (int c = lane; c < kHeadDim; c += 32) dot += q[c] * kr[c];
#pragma unroll
            for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0) sc[m * kPPMaxPos + j] = dot * scale;
          }
          __syncthreads();
          if (tid == 0) {  // softmax_raw (gemv.rs:430-447): max, exp, * (1 / sum)
            float mx = -INFINITY;
            for (int j = 0; j <= pos; ++j) mx = fmaxf(mx, sc[m * kPPMaxPos + j]);
            float sum = 0.0f;
            for (int j = 0; j <= pos; ++j) {
              const float e = expf(sc[m * kPPMaxPos + j] - mx);
              sc[m * kPPMaxPos + j] = e;
              sum += e;
            }
            const float inv = 1.0f / sum;
            for (int j = 0; j <= pos; ++j) sc[m * kPPMaxPos + j] *= inv;
          }
          __syncthreads();
          if (tid < kHeadDim) {
            float o = 0.0f;
            for (int j = 0; j <= pos; ++j) {
              const float* vr = j >= pos0 ? qkv + (4 + (j - pos0)) * kHeadDim
                                          : d.kv + ((((size_t)l * 2 + 1) * d.kvh + hk) * kPageSize + j) * kHeadDim;
              o += sc[m * kPPMaxPos + j] * vr[tid];
            }
            d.attn[(size_t)m * qn + h * kHeadDim + tid] = o;
          }
          __syncthreads();
        }
      }
      grid_sync(d, ++phase);
      // ---- O
      proj_phase(ph_o(l), M, P_o, [&](int m, int r) { return __ldcg(d.attn + (size_t)m * qn + r); });
      prefetch(ph_gu(l));
      grid_sync(d, ++phase);
      // ---- GATEUP: residual + o, RMSNorm
      residual(M, Xa, P_o, d.s_o, pH, nullptr, Xb);
      proj_phase(ph_gu(l), M, P_gu, [&](int m, int r) {
        return xfull[m * kPPMaxHidden + r] * sinv[m] * h2f(L.post_norm[r]);
      });
      prefetch(ph_down(l));
      grid_sync(d, ++phase);
      // ---- DOWN: silu(gate) * up (gemv.rs:449-451)
      {
        const int ldp = 2 * d.inter;
        proj_phase(ph_down(l), M, P_down, [&](int m, int r) {
          const float g = sum_slices(P_gu + (size_t)m * ldp + r, (size_t)M * ldp, d.s_gu);
          const float u = sum_slices(P_gu + (size_t)m * ldp + d.inter + r, (size_t)M * ldp, d.s_gu);
          return silu_ref(g) * u;
        });
      }
      if (l + 1 < d.layers)
        prefetch(ph_qkv(l + 1));
      else
        prefetch(ph_head(step));
      grid_sync(d, ++phase);
    }
    // ---- HEAD: final norm of the last row, lm_head[step], argmax key
    residual(M, Xb, P_down, d.s_down, pH, nullptr, nullptr);
    {
      const int m_last = M - 1;
      const Q4Mat& W = d.lm[step];
      const int TW = 32, units = W.n / TW;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        for (int r = tid; r < pH; r += kThreads)
          xs[r] = xfull[m_last * kPPMaxHidden + r] * sinv[m_last] * h2f(d.final_norm[r]);
        __syncthreads();
        float* out = sc;  // 32 logits
        gemv_unit<1>(W, u * TW, TW, 0, pH, pre, u == (int)blockIdx.x, xs, kPPMaxSlice, red, out, TW);
        if (warp == 0) {
          const float v = out[lane];
          unsigned long long key = ((unsigned long long)f32_order_key(v) << 32) | (unsigned)(u * TW + lane);
#pragma unroll
          for (int o = 16; o; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
          }
          if (lane == 0) atomicMax(d.keys + (step & 1), key);
        }
        __syncthreads();
      }
    }
    if (step + 1 < d.groups) prefetch(ph_proj());
    grid_sync(d, ++phase);
  }
  take_code(d.groups, (d.groups - 1) & 1);
  pdl_launch_dependents();
}

size_t pred_persist_part_floats(const PredPersistDesc& d) {
  const size_t qkvn = (size_t)(d.heads + 2 * d.kvh) * kHeadDim;
  return 2 * ((size_t)d.s_proj * d.pH + (size_t)d.s_qkv * qkvn + (size_t)d.s_o * d.pH + (size_t)d.s_gu * 2 * d.inter +
              (size_t)d.s_down * d.pH);
}

// Shapes the kernel handles: 128-column tiles, unit K slices and the hidden
// row within shared memory, positions within one KV page.
bool pred_persist_supported(const PredPersistDesc& d) {
  auto slice = [](int k, int s) { return (k + s - 1) / s; };
  return d.layers > 0 && d.layers <= kPPMaxLayers && d.groups > 0 && d.groups <= kMaxGroups - 1 &&
         d.heads % d.kvh == 0 && d.pH % 128 == 0 && d.inter % 128 == 0 && d.pH <= kPPMaxHidden &&
         d.pH <= kPPMaxSlice && d.groups < kPageSize && d.groups < kPPMaxPos &&  // last position = groups
         slice(d.t_hidden, d.s_proj) <= kPPMaxSlice && slice(d.pH, d.s_qkv) <= kPPMaxSlice &&
         slice(d.heads * kHeadDim, d.s_o) <= kPPMaxSlice && slice(d.pH, d.s_gu) <= kPPMaxSlice &&
         slice(d.inter, d.s_down) <= kPPMaxSlice && d.lm[0].n % 32 == 0 && d.s_proj <= kSMax &&
         d.s_qkv <= kSMax && d.s_o <= kSMax && d.s_gu <= kSMax && d.s_down <= kSMax && 3 * 2 * kHeadDim <= 3 * kThreads;
}

cudaError_t launch_pred_persist(const PredPersistDesc& d, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPPSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  unsigned n = 0;
  at[n].id = cudaLaunchAttributeCooperative;
  at[n].val.cooperative = 1;
  ++n;
  if (pdl_enabled()) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  if (g_occ_query) {
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, pred_persist_kernel, kThreads, kPPSmem) != cudaSuccess)
      nb = 0;
    g_occ_clusters = nb;
    return cudaSuccess;
  }
  ++g_kernel_launches;
  return cudaLaunchKernelEx(&cfg, pred_persist_kernel, d);
}

void pred_persist_init_attributes() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
  cudaFuncSetAttribute(pred_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPPSmem);
  cudaGetLastError();
  done[dev] = true;
}

}  // namespace qtts
