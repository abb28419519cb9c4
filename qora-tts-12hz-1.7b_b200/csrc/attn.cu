// attn.cu -- GQA attention over the paged f32 KV cache (sm_100a).
//
// Replaces the per-head loops of talker.rs:305-331 (decode), talker.rs:410-438
// (causal prefill) and code_predictor.rs:379-407 / :466-491 (predictor).  A
// query row m attends cache positions [0, pos(m)] of its session; the score is
// q.k / sqrt(128) and the output sum_p softmax(score)_p v_p.  The reference
// normalises with a max-subtracted softmax over all scores; this kernel uses
// the equivalent online form (running max, rescaled sums), so results agree
// to float rounding.
//
// Grid: (M * kv_heads, nsplit).  A CTA of 4 warps takes one KV head (and its
// G = heads/kv_heads query heads) over one slice of positions; warps stride
// over positions, a lane owns 4 of the 128 dims.  Slices are combined by the
// last CTA of the (row, head) in slice order (deterministic).
#include "common.cuh"
#include "kernels.h"

namespace qtts {

namespace {
__device__ __forceinline__ const float* kv_row_c(const KvDesc& kv, int sess, int pos, int which, int h) {
  const int page = kv.page_table ? kv.page_table[sess * kv.pages_per_sess + pos / kPageSize] : sess;
  const size_t blk = (((size_t)page * kv.n_layers + kv.layer) * 2 + which) * kv.kv_heads + h;
  return kv.pool + (blk * kPageSize + (pos % kPageSize)) * kHeadDim;
}
}  // namespace

template <int G>
__global__ void __launch_bounds__(128) attn_kernel(const AttnDesc d) {
  constexpr int NW = 4;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.x / d.kv_heads, h = blockIdx.x % d.kv_heads;
  const int split = blockIdx.y;
  int sess, pos, kvp;
  row_pos(d.rp, m, sess, pos, kvp);
  const int L = kvp + 1;  // cache entries [0, kvp] (talker.rs:301-302)
  const int chunk = (L + d.nsplit - 1) / d.nsplit;
  const int p0 = split * chunk, p1 = min(L, p0 + chunk);
  const float scale = 1.0f / sqrtf((float)kHeadDim);  // talker.rs:305

  float4 q[G];
#pragma unroll
  for (int g = 0; g < G; ++g)
    q[g] = *reinterpret_cast<const float4*>(d.q + (size_t)m * d.ldq + (h * G + g) * kHeadDim + 4 * lane);
  float mx[G], l[G];
  float4 acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    mx[g] = -INFINITY;
    l[g] = 0.0f;
    acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  constexpr int U = 4;
  for (int pb = p0 + warp; pb < p1; pb += NW * U) {
    float4 k4[U], v4[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = pb + NW * u;
      if (p < p1) {
        k4[u] = *reinterpret_cast<const float4*>(kv_row_c(d.kv, sess, p, 0, h) + 4 * lane);
        v4[u] = *reinterpret_cast<const float4*>(kv_row_c(d.kv, sess, p, 1, h) + 4 * lane);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = pb + NW * u;
      if (p >= p1) break;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float dot = q[g].x * k4[u].x + q[g].y * k4[u].y + q[g].z * k4[u].z + q[g].w * k4[u].w;
#pragma unroll
        for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float s = dot * scale;
        const float mn = fmaxf(mx[g], s);
        const float corr = expf(mx[g] - mn);
        const float pe = expf(s - mn);
        l[g] = l[g] * corr + pe;
        acc[g].x = acc[g].x * corr + pe * v4[u].x;
        acc[g].y = acc[g].y * corr + pe * v4[u].y;
        acc[g].z = acc[g].z * corr + pe * v4[u].z;
        acc[g].w = acc[g].w * corr + pe * v4[u].w;
        mx[g] = mn;
      }
    }
  }

  // combine the 4 warps
  __shared__ float s_m[NW][G], s_l[NW][G];
  __shared__ float4 s_acc[NW][G][32];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      s_m[warp][g] = mx[g];
      s_l[warp][g] = l[g];
    }
    s_acc[warp][g][lane] = acc[g];
  }
  __syncthreads();
  // thread t < G*32 finalises (g = t/32, dims 4*(t%32)..)
  const int nsp = d.nsplit;
  // per (split, g) record: m, l, 2 pad, acc[128] -- 132 floats keeps the
  // float4 accumulator stores 16-byte aligned
  const size_t rec = kAttnRec;
  float* part = d.part ? d.part + ((size_t)(m * d.kv_heads + h) * nsp) * G * rec : nullptr;
  if (tid < G * 32) {
    const int g = tid / 32, ln = tid % 32;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, s_m[w][g]);
    float lt = 0.0f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < NW; ++w) {
      const float f = (s_l[w][g] > 0.0f) ? expf(s_m[w][g] - M) : 0.0f;
      lt += s_l[w][g] * f;
      const float4 x = s_acc[w][g][ln];
      a.x += x.x * f; a.y += x.y * f; a.z += x.z * f; a.w += x.w * f;
    }
    if (nsp == 1) {
      float4 o = make_float4(a.x / lt, a.y / lt, a.z / lt, a.w / lt);
      *reinterpret_cast<float4*>(d.out + (size_t)m * d.ldo + (h * G + g) * kHeadDim + 4 * ln) = o;
    } else {
      float* r = part + ((size_t)split * G + g) * rec;
      if (ln == 0) { r[0] = M; r[1] = lt; }
      *reinterpret_cast<float4*>(r + 4 + 4 * ln) = a;
    }
  }
  if (nsp == 1) return;
  __threadfence();
  __syncthreads();
  __shared__ unsigned s_ticket;
  unsigned* ctr = d.counters + (size_t)m * d.kv_heads + h;
  if (tid == 0) s_ticket = atomicAdd(ctr, 1u);
  __syncthreads();
  if (s_ticket != (unsigned)(nsp - 1)) return;
  __threadfence();
  if (tid < G * 32) {
    const int g = tid / 32, ln = tid % 32;
    float M = -INFINITY;
    for (int sp = 0; sp < nsp; ++sp) M = fmaxf(M, __ldcg(part + ((size_t)sp * G + g) * rec));
    float lt = 0.0f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsp; ++sp) {
      const float* r = part + ((size_t)sp * G + g) * rec;
      const float ls = __ldcg(r + 1);
      if (!(ls > 0.0f)) continue;
      const float f = expf(__ldcg(r) - M);
      lt += ls * f;
      const float4 x = __ldcg(reinterpret_cast<const float4*>(r + 4) + ln);
      a.x += x.x * f; a.y += x.y * f; a.z += x.z * f; a.w += x.w * f;
    }
    float4 o = make_float4(a.x / lt, a.y / lt, a.z / lt, a.w / lt);
    *reinterpret_cast<float4*>(d.out + (size_t)m * d.ldo + (h * G + g) * kHeadDim + 4 * ln) = o;
  }
  if (tid == 0) *ctr = 0u;
}

cudaError_t launch_attention(const AttnDesc& d, cudaStream_t st) {
  if (d.kv_heads <= 0 || d.heads % d.kv_heads) return cudaErrorInvalidValue;
  if (d.nsplit > 1 && (!d.part || !d.counters)) return cudaErrorInvalidValue;
  const int G = d.heads / d.kv_heads;
  const dim3 grid(d.M * d.kv_heads, d.nsplit);
  switch (G) {
    case 1: attn_kernel<1><<<grid, 128, 0, st>>>(d); break;
    case 2: attn_kernel<2><<<grid, 128, 0, st>>>(d); break;
    case 4: attn_kernel<4><<<grid, 128, 0, st>>>(d); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace qtts
