// sample.cu -- code-0 sampler (generate_new.rs:329-391) and the xorshift64
// draw (generate_new.rs:16-22), one CTA per utterance.
//
// Bit-exactness with the reference, given the same logits and rng state:
//   * repetition penalty, temperature, max-subtract, division by the sum,
//     renormalisation and the cumulative walk are the same IEEE f32
//     operations in the same order (sums are sequential in index order, as
//     iter().sum() is);
//   * exp is the glibc-identical expf_glibc (common.cuh);
//   * top-k is the stable descending sort of the reference expressed as a
//     selection: keep p_i iff fewer than k elements precede it in
//     (p desc, index asc) order.  The k-th value is found with a 4-pass
//     8-bit radix select over the f32 bits (p >= 0 so the bits order like
//     the values); ties at the threshold keep the lowest indices.
// The sequential sums run on one thread (they cannot be reassociated without
// changing the bits); everything else is parallel.
#include "common.cuh"
#include "kernels.h"

namespace qtts {

namespace {
constexpr int kThreads = 1024;
constexpr int kMaxV = 4096;

__device__ __forceinline__ float block_max(float v, float* sbuf) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sbuf[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < kThreads / 32; ++w) t = fmaxf(t, sbuf[w]);
  return t;
}

// exclusive prefix sum over the block of one value per thread
__device__ __forceinline__ int block_excl_scan(int v, int* sbuf, int* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) sbuf[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = sbuf[lane];
    int s = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    sbuf[32 + lane] = s - w;  // exclusive warp offsets
    if (lane == 31) sbuf[64] = s;
  }
  __syncthreads();
  *total = sbuf[64];
  return sbuf[32 + warp] + x - v;
}
}  // namespace

__global__ void __launch_bounds__(kThreads) sample_kernel(const SampleDesc d) {
  __shared__ float p[kMaxV];
  __shared__ int kidx[kMaxV];
  __shared__ unsigned hist[256];
  __shared__ float sbuf[64];
  __shared__ int ibuf[96];
  __shared__ float s_sum;
  __shared__ unsigned s_prefix, s_need;
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int b = blockIdx.x;
  const int V = d.V;

  float T, rep;
  int topk;
  const uint32_t* prev;
  SlotState* sl = nullptr;
  if (d.standalone) {
    T = d.temperature; rep = d.rep_pen; topk = d.top_k; prev = d.prev;
  } else {
    sl = d.fc.slots + b;
    T = sl->temperature; rep = sl->rep_pen; topk = sl->top_k; prev = sl->prev;
  }

  const float* lg = d.logits + (size_t)b * d.ldl;
  for (int i = tid; i < V; i += kThreads) p[i] = lg[i];
  __syncthreads();
  if (tid == 0 && rep != 1.0f) {  // generate_new.rs:333-343, duplicates re-applied
    for (int i = 0; i < 16; ++i) {
      const uint32_t t = prev[i];
      if ((int)t < V && t < (uint32_t)V) {
        const float s = p[t];
        p[t] = (s > 0.0f) ? __fdiv_rn(s, rep) : __fmul_rn(s, rep);
      }
    }
  }
  __syncthreads();
  if (T != 1.0f)  // :346-350
    for (int i = tid; i < V; i += kThreads) p[i] = __fdiv_rn(p[i], T);
  float mx = -INFINITY;  // :353 fold(NEG_INFINITY, f32::max)
  for (int i = tid; i < V; i += kThreads) mx = fmaxf(mx, p[i]);
  mx = block_max(mx, sbuf);
  for (int i = tid; i < V; i += kThreads) p[i] = expf_glibc(__fsub_rn(p[i], mx));
  __syncthreads();
  if (tid == 0) {  // :357 sequential sum
    float s = 0.0f;
    for (int i = 0; i < V; ++i) s = __fadd_rn(s, p[i]);
    s_sum = s;
  }
  __syncthreads();
  const float sum1 = s_sum;
  for (int i = tid; i < V; i += kThreads) p[i] = __fdiv_rn(p[i], sum1);
  __syncthreads();

  const bool filter = topk > 0 && topk < V;  // :363
  int nkeep = 0;
  if (filter) {
    // radix select of the topk-th largest bit pattern
    unsigned prefix = 0, mask = 0, need = (unsigned)topk;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
      __syncthreads();
      for (int i = tid; i < V; i += kThreads) {
        const unsigned u = __float_as_uint(p[i]);
        if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid < 32) {
        // lane l owns buckets 255-8l .. 248-8l (descending)
        unsigned c = 0;
        for (int j = 0; j < 8; ++j) c += hist[255 - 8 * tid - j];
        unsigned inc = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned y = __shfl_up_sync(0xffffffffu, inc, o);
          if (tid >= o) inc += y;
        }
        const unsigned before = inc - c;
        const unsigned hit = __ballot_sync(0xffffffffu, inc >= need);
        const int first = __ffs(hit) - 1;
        if (tid == first) {
          unsigned run = before;
          for (int j = 0; j < 8; ++j) {
            const int bk = 255 - 8 * tid - j;
            if (run + hist[bk] >= need) {
              s_prefix = prefix | ((unsigned)bk << shift);
              s_need = need - run;
              break;
            }
            run += hist[bk];
          }
        }
      }
      __syncthreads();
      prefix = s_prefix;
      need = s_need;
      mask |= 255u << shift;
    }
    // keep: u > vk, or u == vk among the first `need` equal ones by index
    const unsigned vk = prefix;
    constexpr int PER = kMaxV / kThreads;
    const int i0 = tid * PER;
    int eq = 0;
    for (int j = 0; j < PER; ++j) {
      const int i = i0 + j;
      if (i < V && __float_as_uint(p[i]) == vk) ++eq;
    }
    int tot;
    int eqr = block_excl_scan(eq, ibuf, &tot);
    int kept = 0;
    bool keepv[PER];
    for (int j = 0; j < PER; ++j) {
      const int i = i0 + j;
      bool k = false;
      if (i < V) {
        const unsigned u = __float_as_uint(p[i]);
        if (u > vk) k = true;
        else if (u == vk) { k = (unsigned)eqr < need; ++eqr; }
      }
      keepv[j] = k;
      kept += k;
    }
    int at = block_excl_scan(kept, ibuf, &tot);
    nkeep = tot;
    for (int j = 0; j < PER; ++j) {
      const int i = i0 + j;
      if (i < V) {
        if (keepv[j]) kidx[at++] = i;
        else p[i] = 0.0f;  // :367-369
      }
    }
    __syncthreads();
  }

  if (tid == 0) {
    uint32_t tok = 0;
    unsigned long long st = d.standalone ? *d.rng : sl->rng;
    st ^= st << 13;  // generate_new.rs:16-22
    st ^= st >> 7;
    st ^= st << 17;
    const float r = __fdiv_rn(__ull2float_rn(st), 18446744073709551616.0f);
    if (filter) {
      float s2 = 0.0f;  // :372 (zeros contribute nothing)
      for (int j = 0; j < nkeep; ++j) s2 = __fadd_rn(s2, p[kidx[j]]);
      float cum = 0.0f;
      for (int j = 0; j < nkeep; ++j) {
        float q = p[kidx[j]];
        if (s2 > 0.0f) q = __fdiv_rn(q, s2);
        cum = __fadd_rn(cum, q);
        if (r < cum) { tok = (uint32_t)kidx[j]; break; }
      }
    } else {
      float cum = 0.0f;
      for (int i = 0; i < V; ++i) {
        cum = __fadd_rn(cum, p[i]);
        if (r < cum) { tok = (uint32_t)i; break; }
      }
    }
    if (d.standalone) {
      *d.rng = st;
      *d.out = tok;
    } else {
      sl->rng = st;
      const int f = sl->frame;
      uint32_t used = tok;
      if (f < d.fc.max_frames) {
        const size_t at = ((size_t)b * d.fc.max_frames + f) * kMaxGroups;
        d.fc.codes[at] = tok;
        if (d.fc.forced) used = d.fc.forced[at];
      }
      sl->cur[0] = used;
      sl->prev[0] = used;
      if (!(sl->flags & 1) && used == sl->eos && !sl->done) {  // generate_new.rs:246
        sl->done = 1;
        sl->frames_out = f;
      }
    }
  }
}

cudaError_t launch_sample(const SampleDesc& d, cudaStream_t st) {
  if (d.V <= 0 || d.V > kMaxV || d.B <= 0) return cudaErrorInvalidValue;
  LaunchOpts o;
  o.pdl = true;
  return launch_k(sample_kernel, dim3(d.B), dim3(kThreads), 0, st, o, d);
}

}  // namespace qtts
