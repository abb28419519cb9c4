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
// root CTA of the (row, head) cluster over distributed shared memory, in
// slice order (deterministic).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace qtts {

// F16: the cache's element type (KvDesc::f16), fixed per instance so that the
// position loop carries no type test.
template <int G, bool F16>
__global__ void __launch_bounds__(128) attn_kernel(const AttnDesc d) {
  pdl_launch_dependents();
  const KvDesc& kv = d.kv;
  constexpr int NW = 4;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.x / d.kv_heads, h = blockIdx.x % d.kv_heads;
  const int split = blockIdx.y;
  if (tid == 0 && d.l2_prefetch) {
    // Before the wait: pull this CTA's K / V rows into L2 (one bulk prefetch
    // per page and K / V).  A hint only: the position is read through L2 and
    // may be a step old, and rows the q/k/v step is writing are refetched by
    // the loads after the wait; every address stays inside the pool.
    const RowPos& rp = d.rp;
    const int sl = m / rp.rows_per_sess, r = m - sl * rp.rows_per_sess;
    const int ss = rp.sess0 + sl;
    const int ps = (rp.pos_base ? __ldcg(rp.pos_base + ss * rp.pos_stride) : rp.pos_const) + r;
    const int kvi = rp.kv_const >= 0 ? rp.kv_const + r : ps;
    if (kvi >= 0 && kvi < kv.pages_per_sess * kPageSize) {
      const int Lp = kvi + 1, ch = (Lp + d.nsplit - 1) / d.nsplit;
      const int q0 = split * ch, q1 = min(Lp, q0 + ch);
      for (int pg = q0 / kPageSize; pg * kPageSize < q1; ++pg) {
        const int a = max(q0, pg * kPageSize), b = min(q1, (pg + 1) * kPageSize);
        for (int which = 0; which < 2; ++which)
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(kv_addr(kv, kv_at(kv, ss, a, which, h), F16)),
                       "r"((uint32_t)((b - a) * kHeadDim * (F16 ? 2 : 4)))
                       : "memory");
      }
    }
  }
  pdl_wait();
  int sess, pos, kvp;
  row_pos(d.rp, m, sess, pos, kvp);
  const int L = kvp + 1;  // cache entries [0, kvp] (talker.rs:301-302)
  const int chunk = (L + d.nsplit - 1) / d.nsplit;
  const int p0 = split * chunk, p1 = min(L, p0 + chunk);
  const float scale = 1.0f / sqrtf((float)kHeadDim);  // talker.rs:305

  // per (virtual) warp softmax state for the combine
  constexpr int NVW = F16 ? 2 * NW : NW;
  __shared__ float s_m[NVW][G], s_l[NVW][G];
  __shared__ float4 s_acc[NVW][G][32];
  if constexpr (F16) {
    // f16 caches: a half-warp per position (lane j = lane % 16 holds
    // dimensions 8j..8j+7, one 16-byte load per row), so a warp keeps as many
    // bytes in flight per load as the f32 loop; the two halves are separate
    // online-softmax streams (virtual warps vw = 2 warp + half) over
    // positions pw + half + 8u, pw = p0 + 2 warp + 32 t.
    const int hh = lane >> 4, j = lane & 15, vw = 2 * warp + hh;
    float4 qa[G], qb[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float* qr = d.q + (size_t)m * d.ldq + (h * G + g) * kHeadDim + 8 * j;
      qa[g] = *reinterpret_cast<const float4*>(qr);
      qb[g] = *reinterpret_cast<const float4*>(qr + 4);
    }
    float mx[G], l[G];
    float4 aa[G], ab[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      mx[g] = -INFINITY;
      l[g] = 0.0f;
      aa[g] = make_float4(0.f, 0.f, 0.f, 0.f);
      ab[g] = aa[g];
    }
    constexpr int U = 4;
    const bool b3 = (lane & 8) != 0, b2 = (lane & 4) != 0;
    auto h8 = [](const uint4& w, float (&f)[8]) {
      const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&v[t]));
        f[2 * t] = x.x;
        f[2 * t + 1] = x.y;
      }
    };
    for (int pw = p0 + 2 * warp; pw < p1; pw += 2 * NW * U) {
      uint4 k8[U], v8[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int p = pw + hh + 2 * NW * u;
        if (p < p1) {
          k8[u] = *reinterpret_cast<const uint4*>(kv_addr(kv, kv_at(kv, sess, p, 0, h) + 8 * j, true));
          v8[u] = *reinterpret_cast<const uint4*>(kv_addr(kv, kv_at(kv, sess, p, 1, h) + 8 * j, true));
        } else {
          k8[u] = make_uint4(0u, 0u, 0u, 0u);
          v8[u] = k8[u];
        }
      }
      // every k row converted once for all G heads, every v row once for all
      float dp[G][U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float kf[8];
        h8(k8[u], kf);
#pragma unroll
        for (int g = 0; g < G; ++g)
          dp[g][u] = ((qa[g].x * kf[0] + qa[g].y * kf[1]) + (qa[g].z * kf[2] + qa[g].w * kf[3])) +
                     ((qb[g].x * kf[4] + qb[g].y * kf[5]) + (qb[g].z * kf[6] + qb[g].w * kf[7]));
      }
      float pe[G][U];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        // 16-lane sums of the 4 dots, transposed: after xor 8 and xor 4 the
        // lane bits (3, 2) name the position u kept, xor 2 and xor 1 finish it
        float a0 = b3 ? dp[g][2] : dp[g][0], a1 = b3 ? dp[g][3] : dp[g][1];
        a0 += __shfl_xor_sync(0xffffffffu, b3 ? dp[g][0] : dp[g][2], 8);
        a1 += __shfl_xor_sync(0xffffffffu, b3 ? dp[g][1] : dp[g][3], 8);
        float c = b2 ? a1 : a0;
        c += __shfl_xor_sync(0xffffffffu, b2 ? a0 : a1, 4);
        c += __shfl_xor_sync(0xffffffffu, c, 2);
        c += __shfl_xor_sync(0xffffffffu, c, 1);
        float mn = mx[g];
#pragma unroll
        for (int u = 0; u < U; ++u) {  // position u of this half sits at lane 16 hh + 4u
          pe[g][u] = __shfl_sync(0xffffffffu, c, (lane & 16) + 4 * u) * scale;
          if (pw + hh + 2 * NW * u >= p1) pe[g][u] = -INFINITY;
          mn = fmaxf(mn, pe[g][u]);
        }
        // a half whose positions all lie past p1 keeps mn = -inf: no update
        const float corr = mn == -INFINITY ? 1.0f : expf(mx[g] - mn);
        float lsum = l[g] * corr;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          pe[g][u] = mn == -INFINITY ? 0.0f : expf(pe[g][u] - mn);  // 0 past p1
          lsum += pe[g][u];
        }
        l[g] = lsum;
        mx[g] = mn;
        aa[g] = make_float4(aa[g].x * corr, aa[g].y * corr, aa[g].z * corr, aa[g].w * corr);
        ab[g] = make_float4(ab[g].x * corr, ab[g].y * corr, ab[g].z * corr, ab[g].w * corr);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float vf[8];
        h8(v8[u], vf);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float e = pe[g][u];
          aa[g].x += e * vf[0]; aa[g].y += e * vf[1]; aa[g].z += e * vf[2]; aa[g].w += e * vf[3];
          ab[g].x += e * vf[4]; ab[g].y += e * vf[5]; ab[g].z += e * vf[6]; ab[g].w += e * vf[7];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (j == 0) {
        s_m[vw][g] = mx[g];
        s_l[vw][g] = l[g];
      }
      s_acc[vw][g][2 * j] = aa[g];
      s_acc[vw][g][2 * j + 1] = ab[g];
    }
  } else {
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

    // Each warp takes U positions per step (pb, pb + NW, ...).  The U partial
    // dot products of a lane are reduced together: two transposing butterfly
    // rounds leave lane group j = lane / 8 with position j's sum over 16 and
    // then 8 lanes, three more rounds finish it (6 shuffles for 4 dots instead
    // of 20), and lane 8 j broadcasts it.  The online softmax then updates once
    // per step: one rescale for the block's max, one exp per position.
    constexpr int U = 4;
    const bool hi16 = (lane & 16) != 0, hi8 = (lane & 8) != 0;
    for (int pb = p0 + warp; pb < p1; pb += NW * U) {
      float4 k4[U], v4[U];
  #pragma unroll
      for (int u = 0; u < U; ++u) {
        const int p = pb + NW * u;
        if (p < p1) {
          k4[u] = kv_load4(kv, kv_at(kv, sess, p, 0, h) + 4 * lane, F16);
          v4[u] = kv_load4(kv, kv_at(kv, sess, p, 1, h) + 4 * lane, F16);
        } else {
          k4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          v4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
  #pragma unroll
      for (int g = 0; g < G; ++g) {
        float dp[U];
  #pragma unroll
        for (int u = 0; u < U; ++u) dp[u] = q[g].x * k4[u].x + q[g].y * k4[u].y + q[g].z * k4[u].z + q[g].w * k4[u].w;
        // step 1 (xor 16): lanes < 16 keep positions 0, 1; lanes >= 16 keep 2, 3
        float a0 = hi16 ? dp[2] : dp[0], a1 = hi16 ? dp[3] : dp[1];
        const float b0 = hi16 ? dp[0] : dp[2], b1 = hi16 ? dp[1] : dp[3];
        a0 += __shfl_xor_sync(0xffffffffu, b0, 16);
        a1 += __shfl_xor_sync(0xffffffffu, b1, 16);
        // step 2 (xor 8): lane group j = lane / 8 keeps position j
        float c = hi8 ? a1 : a0;
        c += __shfl_xor_sync(0xffffffffu, hi8 ? a0 : a1, 8);
        c += __shfl_xor_sync(0xffffffffu, c, 4);
        c += __shfl_xor_sync(0xffffffffu, c, 2);
        c += __shfl_xor_sync(0xffffffffu, c, 1);
        float sc[U];
        float mn = mx[g];
  #pragma unroll
        for (int u = 0; u < U; ++u) {
          sc[u] = __shfl_sync(0xffffffffu, c, 8 * u) * scale;
          if (pb + NW * u >= p1) sc[u] = -INFINITY;
          mn = fmaxf(mn, sc[u]);
        }
        const float corr = expf(mx[g] - mn);
        float lsum = l[g] * corr;
        float4 a4 = make_float4(acc[g].x * corr, acc[g].y * corr, acc[g].z * corr, acc[g].w * corr);
  #pragma unroll
        for (int u = 0; u < U; ++u) {
          const float pe = expf(sc[u] - mn);  // 0 for the positions past p1
          lsum += pe;
          a4.x += pe * v4[u].x; a4.y += pe * v4[u].y; a4.z += pe * v4[u].z; a4.w += pe * v4[u].w;
        }
        l[g] = lsum;
        acc[g] = a4;
        mx[g] = mn;
      }
    }

    // combine the 4 warps
  #pragma unroll
    for (int g = 0; g < G; ++g) {
      if (lane == 0) {
        s_m[warp][g] = mx[g];
        s_l[warp][g] = l[g];
      }
      s_acc[warp][g][lane] = acc[g];
    }
  }
  __syncthreads();
  // thread t < G*32 finalises (g = t/32, dims 4*(t%32)..)
  const int nsp = d.nsplit;
  // per (g) record of this CTA: m, l, 2 pad, acc[128] -- 132 floats keeps
  // the float4 accumulator stores 16-byte aligned
  __shared__ __align__(16) float s_rec[G][kAttnRec];
  if (tid < G * 32) {
    const int g = tid / 32, ln = tid % 32;
    float M = -INFINITY;
    for (int w = 0; w < NVW; ++w) M = fmaxf(M, s_m[w][g]);
    float lt = 0.0f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < NVW; ++w) {
      const float f = (s_l[w][g] > 0.0f) ? expf(s_m[w][g] - M) : 0.0f;
      lt += s_l[w][g] * f;
      const float4 x = s_acc[w][g][ln];
      a.x += x.x * f; a.y += x.y * f; a.z += x.z * f; a.w += x.w * f;
    }
    if (nsp == 1) {
      float4 o = make_float4(a.x / lt, a.y / lt, a.z / lt, a.w / lt);
      *reinterpret_cast<float4*>(d.out + (size_t)m * d.ldo + (h * G + g) * kHeadDim + 4 * ln) = o;
      if (d.xs_out) {  // the o projection's input rows, split for its tensor-core kernel
        xs_store4(d.xs_out, d.heads * kHeadDim, m, (h * G + g) * kHeadDim + 4 * ln, o);
        if (fp16_overflow4(o) && d.err_flag) atomicOr(d.err_flag, kErrFp16Input);
      }
    } else {
      if (ln == 0) { s_rec[g][0] = M; s_rec[g][1] = lt; }
      *reinterpret_cast<float4*>(&s_rec[g][4 + 4 * ln]) = a;
    }
  }
  if (nsp == 1) return;
  // the nsplit CTAs of this (row, head) form one cluster: the root combines
  // the slices over distributed shared memory in slice order
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  const bool root = cl.block_rank() == 0;
  if (root && tid < G * 32) {
    const int g = tid / 32, ln = tid % 32;
    float M = -INFINITY;
    for (int sp = 0; sp < nsp; ++sp) M = fmaxf(M, cl.map_shared_rank(&s_rec[g][0], sp)[0]);
    float lt = 0.0f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsp; ++sp) {
      const float* r = cl.map_shared_rank(&s_rec[g][0], sp);
      const float ls = r[1];
      if (!(ls > 0.0f)) continue;
      const float f = expf(r[0] - M);
      lt += ls * f;
      const float4 x = reinterpret_cast<const float4*>(r + 4)[ln];
      a.x += x.x * f; a.y += x.y * f; a.z += x.z * f; a.w += x.w * f;
    }
    float4 o = make_float4(a.x / lt, a.y / lt, a.z / lt, a.w / lt);
    *reinterpret_cast<float4*>(d.out + (size_t)m * d.ldo + (h * G + g) * kHeadDim + 4 * ln) = o;
  }
  cl.sync();  // peers keep their records until the root has read them
}

cudaError_t launch_attention(const AttnDesc& d, cudaStream_t st) {
  if (d.kv_heads <= 0 || d.heads % d.kv_heads) return cudaErrorInvalidValue;
  if (d.nsplit < 1 || d.nsplit > kMaxClusterSplits) return cudaErrorInvalidValue;
  const int G = d.heads / d.kv_heads;
  const dim3 grid(d.M * d.kv_heads, d.nsplit);
  LaunchOpts o;
  o.pdl = true;
  o.cluster_y = (unsigned)d.nsplit;
  if (g_occ_query) g_occ_family = FAM_ATTN;
  const bool f16 = d.kv.f16 != 0;
  switch (G) {
    case 1: return launch_k(f16 ? attn_kernel<1, true> : attn_kernel<1, false>, grid, dim3(128), 0, st, o, d);
    case 2: return launch_k(f16 ? attn_kernel<2, true> : attn_kernel<2, false>, grid, dim3(128), 0, st, o, d);
    case 4: return launch_k(f16 ? attn_kernel<4, true> : attn_kernel<4, false>, grid, dim3(128), 0, st, o, d);
    default: return cudaErrorInvalidValue;
  }
}

void attn_init_attributes() {
  for (auto* k : {attn_kernel<1, false>, attn_kernel<2, false>, attn_kernel<4, false>, attn_kernel<1, true>,
                  attn_kernel<2, true>, attn_kernel<4, true>})
    cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaGetLastError();
}

}  // namespace qtts
