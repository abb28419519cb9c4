// phase.cu -- the one-row (batch-1) decode layer as two cluster-local phases.
//
// A transformer layer of the talker (talker.rs:279-349) or the code
// predictor (code_predictor.rs:448-502) at one input row has four global
// dependencies when every projection is its own kernel (q/k/v -> attention
// -> o -> gate/up -> down).  Here it runs as two kernels whose internal
// dependencies stay inside a thread-block cluster:
//
//   phase A (attention block), one cluster per KV head j: RMSNorm of the
//     residual row, the q (2 query heads of j) / k / v columns as a K-split
//     over the cluster's ranks summed over distributed shared memory, QK-norm
//     + split-half RoPE (every rank, redundantly), K/V append (rank 0), the
//     attention over the cache split by positions across the ranks and
//     combined over distributed shared memory, and finally rank r's columns
//     of o over the 256 rows that belong to j's heads: parts_out[j] = KV
//     head j's share of the o projection.
//   phase B (MLP block), one CTA per 32 U intermediate columns: RMSNorm of
//     r + sum_j parts[j], gate and up over all H rows, silu(gate) * up, those
//     rows of down over all H columns; the C CTAs of a cluster sum their
//     partial rows over distributed shared memory: parts_out[cluster].
//
// The residual row is never written by a projection: every phase reads
// r = base + sum_p parts[p] (p in order, deterministic), CTA 0 writes r for
// the next phase, and the phase's own output stays in partial rows.  Weights
// never depend on an earlier kernel, so each CTA loads its slice (registers,
// or shared memory by cp.async for phase B's gate/up) before the
// programmatic-dependent-launch wait, and every phase pulls the next phase's
// weights into L2 as it starts.  All arithmetic is f32.
#include "common.cuh"
#include "kernels.h"

namespace qtts {

namespace {

constexpr int kT = kPhaseThreads;

__device__ __forceinline__ uint32_t sm_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsm(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_dsm(uint32_t a, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
// Cluster barrier (every thread of every CTA of the cluster), release /
// acquire: shared-memory and global writes before it are visible after it.
__device__ __forceinline__ void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void cl_sync() {
  cl_arrive();
  cl_wait();
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ float u16f(unsigned short s) { return __half2float(__ushort_as_half(s)); }
// Physical index of column col of a 256-column row whose 32-column groups
// store their 4-column chunk c at chunk (c + group) % 8.
__device__ __forceinline__ int rot_col(int col) { return (col & ~31) | ((col + 4 * (col >> 5)) & 31); }

// This CTA's share of up to 8 regions, pulled into L2 by thread 0.
__device__ __forceinline__ void prefetch_l2(const uint8_t* const (&ptr)[8], const uint32_t (&bytes)[8]) {
  if (threadIdx.x != 0) return;
  const unsigned nctas = gridDim.x * gridDim.y, cta = blockIdx.x * gridDim.y + blockIdx.y;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (!ptr[i] || bytes[i] == 0) continue;
    const uint32_t share = ((bytes[i] + nctas - 1) / nctas + 15u) & ~15u;
    const uint32_t b0 = cta * share;
    if (b0 >= bytes[i]) continue;
    const uint32_t n = min(share, bytes[i] - b0) & ~15u;
    if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr[i] + b0), "r"(n) : "memory");
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float block_sum(float v, float* sbuf) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sbuf[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kT / 32; ++w) t += sbuf[w];
  return t;
}

// r = base + sum_p parts[p] into xr[H] (parts added in order p = 0, 1, ...,
// loads of four parts in flight at a time); the first CTA of the grid also
// writes r to in.out.  Returns 1 / rms(r) (gemv.rs:408-417).
__device__ __forceinline__ float load_resid(const PhaseResid& in, int H, float* xr, float* sbuf) {
  constexpr int MT = kPhaseMaxH / kT;
  const int tid = threadIdx.x;
  float v[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int i = tid + kT * t;
    v[t] = i < H ? in.base[i] : 0.0f;
  }
  for (int p0 = 0; p0 < in.nparts; p0 += 4) {
    float w[4][MT];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int i = tid + kT * t;
        w[q][t] = (p0 + q < in.nparts && i < H) ? in.parts[(size_t)(p0 + q) * H + i] : 0.0f;
      }
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int t = 0; t < MT; ++t)
        if (p0 + q < in.nparts) v[t] += w[q][t];
  }
  const bool writer = in.out && blockIdx.x == 0 && blockIdx.y == 0;
  float ss = 0.0f;
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int i = tid + kT * t;
    if (i < H) {
      xr[i] = v[t];
      ss += v[t] * v[t];
      if (writer) in.out[i] = v[t];
    }
  }
  ss = block_sum(ss, sbuf);  // also orders the xr writes before any read
  return 1.0f / sqrtf(ss / (float)H + 1e-6f);
}

__device__ __forceinline__ void fma_chunk(const uint4& w, unsigned short s, float x, float2* acc) {
  const SxPack p = make_sx(u16f(s) * x);  // (scale * x) * (q - 8), gemv.rs:239
  q4_word_fma(w.x, p, &acc[0]);
  q4_word_fma(w.y, p, &acc[4]);
  q4_word_fma(w.z, p, &acc[8]);
  q4_word_fma(w.w, p, &acc[12]);
}

__device__ __forceinline__ const float* kvp_row(const KvDesc& kv, int sess, int pos, int which, int h) {
  const int page = kv.page_table ? kv.page_table[sess * kv.pages_per_sess + pos / kPageSize] : sess;
  const size_t blk = (((size_t)page * kv.n_layers + kv.layer) * 2 + which) * kv.kv_heads + h;
  return kv.pool + (blk * kPageSize + (pos % kPageSize)) * kHeadDim;
}

}  // namespace

// Shared-memory floats of phase A: residual row, CTA reduction [8][512],
// partial and reduced q|k|v (512 each), normed and rotated q|k (384 each),
// per-warp attention state, the CTA's attention record, attention output,
// scratch.
__host__ __device__ constexpr int attn_phase_floats(int H) {
  return H + 8 * 512 + 512 + 512 + 384 + 384 + 2 * 8 + 2 * 8 + 8 * 2 * 128 + 2 * kAttnRec + 256 + 32;
}

// ===========================================================================
// Phase A.  Grid (kvh, C), cluster (1, C, 1), 256 threads; NR = H / (32 C).
template <int NR>
__global__ void __launch_bounds__(kT) attn_phase_kernel(const __grid_constant__ AttnPhaseDesc d) {
  extern __shared__ __align__(16) float sm[];
  const int H = d.H, C = (int)gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j = blockIdx.x, rank = blockIdx.y;  // KV head; rank in the cluster (the cluster spans grid.y)
  constexpr int RPC = 32 * NR;                 // rows of the K split per rank = o columns per rank
  const int r0 = rank * RPC;
  float* xr = sm;                     // [H]
  float* red = xr + H;                // [8][512]
  float* part = red + 8 * 512;        // [512] this CTA's partial q|k|v
  float* full = part + 512;           // [512] reduced q0|q1|k|v
  float* qk = full + 512;             // [384] QK-normed q0|q1|k
  float* qr = qk + 384;               // [384] rotated q0|q1|k
  float* wm = qr + 384;               // [8][2] per-warp running max
  float* wl = wm + 16;                // [8][2] per-warp running sum
  float* wacc = wl + 16;              // [8][2][128] per-warp accumulators
  float* rec = wacc + 8 * 2 * 128;    // [2][kAttnRec] this CTA's record (m, l, pad, acc[128])
  float* aout = rec + 2 * kAttnRec;   // [256] attention output of the two heads
  float* sbuf = aout + 256;           // [32]

  prefetch_l2(d.pf_ptr, d.pf_bytes);
  // ---- weights before the dependent-launch wait (never written by a kernel)
  const int rr = lane >> 3, gi = lane & 7;
  // fields picked one by one: a reference to either parameter would make
  // the compiler copy the parameter block to local memory
  const uint8_t* kv_packed = gi < 4 ? d.k.packed : d.v.packed;
  const unsigned short* kv_scales = reinterpret_cast<const unsigned short*>(gi < 4 ? d.k.scales : d.v.scales);
  const int kv_n = gi < 4 ? d.k.n : d.v.n;
  const int qcol = j * 2 * kHeadDim + gi * 32, kvcol = j * kHeadDim + (gi & 3) * 32;
  uint4 wq[NR], wkv[NR];
  unsigned short sq[NR], skv[NR];
  float gv[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    const size_t row = (size_t)(r0 + warp * 4 + rr + 32 * i);
    wq[i] = ld_stream16(d.q.packed + row * (d.q.n / 2) + qcol / 2);
    sq[i] = __ldg(reinterpret_cast<const unsigned short*>(d.q.scales) + row * (d.q.n / 32) + qcol / 32);
    wkv[i] = ld_stream16(kv_packed + row * (kv_n / 2) + kvcol / 2);
    skv[i] = __ldg(kv_scales + row * (kv_n / 32) + kvcol / 32);
    gv[i] = h2f(d.gamma[row]);
  }
  // o: rows [256 j, 256 j + 256), columns [r0, r0 + RPC); lane = (group og,
  // row offset oro), a warp covers 32 / NR rows per step, NR steps
  const int og = lane % NR, oro = lane / NR;
  uint4 wo[NR];
  unsigned short so[NR];
#pragma unroll
  for (int s = 0; s < NR; ++s) {
    const size_t orow = (size_t)(j * 2 * kHeadDim + s * (256 / NR) + warp * (32 / NR) + oro);
    const int ocol = r0 + og * 32;
    wo[s] = ld_stream16(d.o.packed + orow * (H / 2) + ocol / 2);
    so[s] = __ldg(reinterpret_cast<const unsigned short*>(d.o.scales) + orow * (H / 32) + ocol / 32);
  }
  const float gqk = h2f(tid < 256 ? d.q_norm[tid & 127] : d.k_norm[tid & 127]);
  const float gk = h2f(d.k_norm[tid & 127]);
  pdl_wait();

  // ---- residual row, RMSNorm, this lane's inputs
  const float inv = load_resid(d.in, H, xr, sbuf);
  float xv[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) xv[i] = xr[r0 + warp * 4 + rr + 32 * i] * inv * gv[i];

  // ---- q | k v columns of this rank's rows
  float2 acc[2][16];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int c = 0; c < 16; ++c) acc[t][c] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    fma_chunk(wq[i], sq[i], xv[i], acc[0]);
    fma_chunk(wkv[i], skv[i], xv[i], acc[1]);
  }
  pdl_launch_dependents();
  // the 4 row offsets of a warp, then the 8 warps (lanes rr = 0 store)
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      float2 v = acc[t][c];
      v.x += __shfl_xor_sync(0xffffffffu, v.x, 8);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, 8);
      v.x += __shfl_xor_sync(0xffffffffu, v.x, 16);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, 16);
      acc[t][c] = v;
    }
  if (rr == 0) {
    // chunk c of lane gi's 32 columns goes to chunk (c + gi) % 8 of its
    // group, so the 8 storing lanes hit different banks (rot_col undoes it)
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      float4* dst = reinterpret_cast<float4*>(red + warp * 512 + t * 256 + gi * 32);
#pragma unroll
      for (int c = 0; c < 8; ++c)
        dst[(c + gi) & 7] = make_float4(acc[t][2 * c].x, acc[t][2 * c].y, acc[t][2 * c + 1].x, acc[t][2 * c + 1].y);
    }
  }
  __syncthreads();
  const int pc = rot_col(tid);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w * 512 + h * 256 + pc];
    part[h * 256 + tid] = s;
  }
  cl_sync();  // every rank's partial is written (and every rank is running)

  // ---- rank r sums columns [r SL, (r+1) SL) over the ranks (in rank order)
  // and stores them into every rank's `full`
  const int SL = 512 / C;
  if (tid < SL) {
    const int col = rank * SL + tid;
    const uint32_t pa = sm_u32(part + col);
    float pv[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) pv[p] = p < C ? ld_dsm(map_rank(pa, (uint32_t)p)) : 0.0f;
    float s = pv[0];
#pragma unroll
    for (int p = 1; p < 16; ++p)
      if (p < C) s += pv[p];
    const uint32_t fa = sm_u32(full + col);
    for (int p = 0; p < C; ++p) st_dsm(map_rank(fa, (uint32_t)p), s);
  }
  cl_sync();  // `full` is complete on every rank

  // ---- QK-norm (talker.rs:89-99) and split-half RoPE (rope.rs:79-92)
  int sess, pos, kvp;
  row_pos(d.rp, 0, sess, pos, kvp);
  const int dd = tid & 127;
  {
    const float xa = full[tid];                          // q0 (tid < 128) or q1
    const float xk = tid < 128 ? full[256 + tid] : 0.0f;  // k
    const float sa = warp_sum(xa * xa), sk = warp_sum(xk * xk);
    if (lane == 0) {
      sbuf[warp] = sa;
      sbuf[8 + warp] = sk;
    }
    __syncthreads();
    const int hb = (tid >> 7) * 4;
    const float ia = 1.0f / sqrtf((sbuf[hb] + sbuf[hb + 1] + sbuf[hb + 2] + sbuf[hb + 3]) / (float)kHeadDim + 1e-6f);
    const float ik = 1.0f / sqrtf((sbuf[8] + sbuf[9] + sbuf[10] + sbuf[11]) / (float)kHeadDim + 1e-6f);
    qk[tid] = xa * ia * gqk;
    if (tid < 128) qk[256 + tid] = xk * ik * gk;
  }
  __syncthreads();
  const bool rope_ok = pos >= 0 && pos < d.rope_rows;
  {
    const int half = kHeadDim / 2, i = dd % half;
    float c = 0.0f, s = 0.0f;
    if (rope_ok) {
      c = d.rope_cos[(size_t)pos * half + i];
      s = d.rope_sin[(size_t)pos * half + i];
    }
    for (int e = tid; e < 384; e += kT) {
      const int hb = (e >> 7) * kHeadDim;
      const float y = qk[e];
      float o = y;
      if (rope_ok) {
        const float x1 = qk[hb + i], x2 = qk[hb + half + i];
        o = (dd < half) ? (x1 * c - x2 * s) : (x2 * c + x1 * s);
      }
      qr[e] = o;
    }
  }
  if (!rope_ok && !d.rope_skip_oob && d.err_flag && j == 0 && rank == 0 && tid == 0) atomicOr(d.err_flag, kErrRopeRange);
  __syncthreads();
  if (rank == 0 && tid < 128) {  // the cache entry of this step (talker.rs:299-302)
    KvDesc kv = d.kv;
    const_cast<float*>(kvp_row(kv, sess, kvp, 0, j))[tid] = qr[256 + tid];
    const_cast<float*>(kvp_row(kv, sess, kvp, 1, j))[tid] = full[384 + tid];
  }

  // ---- attention of the 2 query heads over this rank's positions
  // (talker.rs:305-331): online max / sum, a lane owns 4 of the 128 dims
  {
    const int L = kvp + 1, chunk = (L + C - 1) / C;
    const int p0 = rank * chunk, p1 = min(L, p0 + chunk);
    const float scale = 1.0f / sqrtf((float)kHeadDim);
    const float4 q0 = reinterpret_cast<const float4*>(qr)[lane];
    const float4 q1 = reinterpret_cast<const float4*>(qr + kHeadDim)[lane];
    float mx[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    float4 a[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    for (int p = p0 + warp; p < p1; p += 8) {
      float4 k4, v4;
      if (p == kvp) {  // this step's entry, from shared memory
        k4 = reinterpret_cast<const float4*>(qr + 256)[lane];
        v4 = reinterpret_cast<const float4*>(full + 384)[lane];
      } else {
        k4 = reinterpret_cast<const float4*>(kvp_row(d.kv, sess, p, 0, j))[lane];
        v4 = reinterpret_cast<const float4*>(kvp_row(d.kv, sess, p, 1, j))[lane];
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const float4 q = g ? q1 : q0;
        const float sc = warp_sum(q.x * k4.x + q.y * k4.y + q.z * k4.z + q.w * k4.w) * scale;
        const float mn = fmaxf(mx[g], sc);
        const float corr = expf(mx[g] - mn), pe = expf(sc - mn);
        l[g] = l[g] * corr + pe;
        a[g] = make_float4(a[g].x * corr + pe * v4.x, a[g].y * corr + pe * v4.y, a[g].z * corr + pe * v4.z,
                           a[g].w * corr + pe * v4.w);
        mx[g] = mn;
      }
    }
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      if (lane == 0) {
        wm[warp * 2 + g] = mx[g];
        wl[warp * 2 + g] = l[g];
      }
      reinterpret_cast<float4*>(wacc + (warp * 2 + g) * 128)[lane] = a[g];
    }
    __syncthreads();
    if (tid < 64) {  // the 8 warps of this rank -> its record
      const int g = tid >> 5, ln = tid & 31;
      float M = -INFINITY;
      for (int w = 0; w < 8; ++w)
        if (wl[w * 2 + g] > 0.0f) M = fmaxf(M, wm[w * 2 + g]);
      float lt = 0.0f;
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int w = 0; w < 8; ++w) {
        const float lw = wl[w * 2 + g];
        if (!(lw > 0.0f)) continue;
        const float f = expf(wm[w * 2 + g] - M);
        lt += lw * f;
        const float4 x = reinterpret_cast<const float4*>(wacc + (w * 2 + g) * 128)[ln];
        s4.x += x.x * f; s4.y += x.y * f; s4.z += x.z * f; s4.w += x.w * f;
      }
      if (ln == 0) {
        rec[g * kAttnRec] = M;
        rec[g * kAttnRec + 1] = lt;
      }
      reinterpret_cast<float4*>(rec + g * kAttnRec + 4)[ln] = s4;
    }
  }
  cl_sync();  // every rank's record is written

  // ---- combine the ranks' records (every rank, in rank order)
  {
    const int g = tid >> 7;
    const uint32_t ra = sm_u32(rec + g * kAttnRec);
    float m[16], lv[16], av[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      if (p < C) {
        const uint32_t b = map_rank(ra, (uint32_t)p);
        m[p] = ld_dsm(b);
        lv[p] = ld_dsm(b + 4);
        av[p] = ld_dsm(b + 16 + 4 * dd);
      } else {
        m[p] = -INFINITY;
        lv[p] = 0.0f;
        av[p] = 0.0f;
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int p = 0; p < 16; ++p)
      if (lv[p] > 0.0f) M = fmaxf(M, m[p]);
    float lt = 0.0f, s = 0.0f;
#pragma unroll
    for (int p = 0; p < 16; ++p)
      if (lv[p] > 0.0f) {
        const float f = expf(m[p] - M);
        lt += lv[p] * f;
        s += av[p] * f;
      }
    aout[tid] = s / lt;
  }
  cl_arrive();  // this rank's reads of its peers are done; wait before exiting
  __syncthreads();

  // ---- o: columns [r0, r0 + RPC) over the 256 rows of j's heads
  float2 oacc[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) oacc[c] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int s = 0; s < NR; ++s) fma_chunk(wo[s], so[s], aout[s * (256 / NR) + warp * (32 / NR) + oro], oacc);
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    float2 v = oacc[c];
#pragma unroll
    for (int o = NR; o < 32; o <<= 1) {
      v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
    }
    oacc[c] = v;
  }
  if (oro == 0) {
    float4* dst = reinterpret_cast<float4*>(red + warp * RPC + og * 32);
#pragma unroll
    for (int c = 0; c < 8; ++c) dst[c] = make_float4(oacc[2 * c].x, oacc[2 * c].y, oacc[2 * c + 1].x, oacc[2 * c + 1].y);
  }
  __syncthreads();
  if (tid < RPC) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w * RPC + tid];
    d.parts_out[(size_t)j * H + r0 + tid] = s;
  }
  cl_wait();
}

// Shared-memory bytes of phase B: gate/up packed slices [H][2U][16 B] and
// scales [H][2U], residual row, warp partials [8][64 U], gate|up values,
// silu(gate) * up, down partials [8192 / H][H], the CTA's partial row,
// scratch.
__host__ __device__ constexpr size_t mlp_phase_bytes(int H, int U) {
  return (size_t)H * 2 * U * 16 + (((size_t)H * 2 * U * 2 + 15) & ~(size_t)15) +
         4 * ((size_t)H + 8 * 64 * U + 64 * U + 32 * U + 8192 + H + 32);
}

// ===========================================================================
// Phase B.  Grid (clusters, C), cluster (1, C, 1), 256 threads; CTA u =
// blockIdx.x * C + blockIdx.y owns intermediate columns [32 U u, 32 U (u+1)).
// NS = 32 U / (8192 / H): row steps of down per thread.
template <int U, int NS>
__global__ void __launch_bounds__(kT) mlp_phase_kernel(const __grid_constant__ MlpPhaseDesc d) {
  extern __shared__ __align__(16) uint8_t smb[];
  const int H = d.H, I = d.I, C = (int)gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.y, u = blockIdx.x * C + blockIdx.y;
  const int c0 = u * 32 * U;
  constexpr int SLOTS = 2 * U;                  // (gate | up) x U groups of 32 columns
  uint8_t* wgu = smb;                           // [H][SLOTS][16]
  unsigned short* sgu = reinterpret_cast<unsigned short*>(smb + (size_t)H * SLOTS * 16);  // [H][SLOTS]
  float* xr = reinterpret_cast<float*>(smb + (size_t)H * SLOTS * 16 + (((size_t)H * SLOTS * 2 + 15) & ~(size_t)15));
  float* redg = xr + H;           // [8][64 U]
  float* gu = redg + 8 * 64 * U;  // [64 U] gate | up
  float* hb = gu + 64 * U;        // [32 U] silu(gate) * up
  float* yred = hb + 32 * U;      // [8192 / H][H]
  float* ypart = yred + 8192;     // [H] this CTA's partial down row (read by the peers)
  float* sbuf = ypart + H;        // [32]

  prefetch_l2(d.pf_ptr, d.pf_bytes);
  // ---- weights before the dependent-launch wait: gate/up slices by
  // cp.async into shared memory, their scales and the down slice in registers
  {
    const int nch = H * SLOTS;
    for (int c = tid; c < nch; c += kT) {
      const int row = c / SLOTS, slot = c % SLOTS, mat = slot / U, g = slot % U;
      const uint8_t* wp = mat ? d.up.packed : d.gate.packed;
      const unsigned short* ws = reinterpret_cast<const unsigned short*>(mat ? d.up.scales : d.gate.scales);
      cp16(sm_u32(wgu + (size_t)c * 16), wp + (size_t)row * (I / 2) + (c0 + 32 * g) / 2);
      sgu[c] = __ldg(ws + (size_t)row * (I / 32) + (c0 + 32 * g) / 32);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const int RO = 8192 / H, GR = H / 32;  // down: threads per column group, column groups
  const int dg = tid % GR, ro = tid / GR;
  uint4 wd[NS];
  unsigned short sd[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const size_t row = (size_t)(c0 + ro + RO * s);
    wd[s] = ld_stream16(d.down.packed + row * (H / 2) + dg * 16);
    sd[s] = __ldg(reinterpret_cast<const unsigned short*>(d.down.scales) + row * (H / 32) + dg);
  }
  pdl_wait();

  // ---- residual row r = base + sum_j parts[j], RMSNorm into xr
  const float inv = load_resid(d.in, H, xr, sbuf);
  for (int i = tid; i < H; i += kT) xr[i] = xr[i] * inv * h2f(d.gamma[i]);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // ---- gate / up: thread = (slot, row offset), 256 / SLOTS rows per pass
  const int slot = tid % SLOTS, rg = tid / SLOTS;
  constexpr int RP = kT / SLOTS;
  float2 acc[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) acc[c] = make_float2(0.0f, 0.0f);
  for (int row = rg; row < H; row += RP) {
    const uint4 w = *reinterpret_cast<const uint4*>(wgu + ((size_t)row * SLOTS + slot) * 16);
    fma_chunk(w, sgu[row * SLOTS + slot], xr[row], acc);
  }
  pdl_launch_dependents();
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    float2 v = acc[c];
#pragma unroll
    for (int o = SLOTS; o < 32; o <<= 1) {
      v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
      v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
    }
    acc[c] = v;
  }
  if (lane < SLOTS) {
    float4* dst = reinterpret_cast<float4*>(redg + warp * 64 * U + lane * 32);
#pragma unroll
    for (int c = 0; c < 8; ++c) dst[c] = make_float4(acc[2 * c].x, acc[2 * c].y, acc[2 * c + 1].x, acc[2 * c + 1].y);
  }
  __syncthreads();
  if (tid < 64 * U) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += redg[w * 64 * U + tid];
    gu[tid] = s;
  }
  __syncthreads();
  if (tid < 32 * U) hb[tid] = silu_ref(gu[tid]) * gu[32 * U + tid];  // gemv.rs:449-451, talker.rs:339-349
  __syncthreads();

  // ---- down: rows [c0, c0 + 32 U) over all H columns
  float2 dacc[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) dacc[c] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int s = 0; s < NS; ++s) fma_chunk(wd[s], sd[s], hb[ro + RO * s], dacc);
  {
    float4* dst = reinterpret_cast<float4*>(yred + (size_t)ro * H + dg * 32);
#pragma unroll
    for (int c = 0; c < 8; ++c) dst[c] = make_float4(dacc[2 * c].x, dacc[2 * c].y, dacc[2 * c + 1].x, dacc[2 * c + 1].y);
  }
  __syncthreads();
  for (int c = tid; c < H; c += kT) {
    float s = 0.0f;
    for (int q = 0; q < RO; ++q) s += yred[(size_t)q * H + c];
    ypart[c] = s;
  }
  cl_sync();  // every CTA's partial row is written

  // ---- rank r sums columns [r H / C, (r+1) H / C) over the cluster
  const int HC = H / C;
  if (tid < HC) {
    const int col = rank * HC + tid;
    const uint32_t pa = sm_u32(ypart + col);
    float pv[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) pv[p] = p < C ? ld_dsm(map_rank(pa, (uint32_t)p)) : 0.0f;
    float s = pv[0];
#pragma unroll
    for (int p = 1; p < 16; ++p)
      if (p < C) s += pv[p];
    d.parts_out[(size_t)blockIdx.x * H + col] = s;
  }
  cl_sync();  // peers keep their shared memory until every rank has read it
}

// ---------------------------------------------------------------------------
bool attn_phase_supported(int H, int heads, int kvh, int* C) {
  if (heads != 2 * kvh || kvh <= 0 || H > kPhaseMaxH || H % 256) return false;
  for (int c : {16, 8}) {
    const int nr = H / (32 * c);
    if (H % (32 * c) == 0 && (nr == 1 || nr == 2 || nr == 4)) {
      *C = c;
      return true;
    }
  }
  return false;
}

bool mlp_phase_supported(int H, int I, int* U, int* C) {
  if (!(H == 256 || H == 512 || H == 1024 || H == 2048)) return false;
  const int u = H >= 2048 ? 2 : 1;
  if (I % (32 * u)) return false;
  const int ncta = I / (32 * u);
  int c = 0;
  if (ncta % 16 == 0) c = 16;
  else if (ncta % 8 == 0) c = 8;
  else return false;
  if (mlp_phase_bytes(H, u) > 227 * 1024) return false;
  *U = u;
  *C = c;
  return true;
}

size_t attn_phase_smem(const AttnPhaseDesc& d) { return sizeof(float) * (size_t)attn_phase_floats(d.H); }
size_t mlp_phase_smem(const MlpPhaseDesc& d) { return mlp_phase_bytes(d.H, d.U); }

static LaunchOpts phase_opts(int C) {
  LaunchOpts o;
  o.pdl = true;
  o.cluster_y = (unsigned)C;
  return o;
}

cudaError_t launch_attn_phase(const AttnPhaseDesc& d, cudaStream_t st) {
  int C = 0;
  if (!attn_phase_supported(d.H, 2 * d.kvh, d.kvh, &C) || C != d.C || d.in.nparts > kPhaseMaxParts ||
      (d.in.nparts && !d.in.parts) || !d.in.base || !d.parts_out)
    return cudaErrorInvalidValue;
  if (g_occ_query) {
    g_occ_family = FAM_PHASE;
    const double kn = (double)d.H * (d.q.n + d.k.n + d.v.n) + (double)d.o.k * d.o.n;
    g_occ_flops = 2.0 * kn;
    g_occ_wbytes = 0.5625 * kn;
  }
  const dim3 grid(d.kvh, C);
  const size_t smem = attn_phase_smem(d);
  switch (d.H / (32 * C)) {
    case 1: return launch_k(attn_phase_kernel<1>, grid, dim3(kT), smem, st, phase_opts(C), d);
    case 2: return launch_k(attn_phase_kernel<2>, grid, dim3(kT), smem, st, phase_opts(C), d);
    case 4: return launch_k(attn_phase_kernel<4>, grid, dim3(kT), smem, st, phase_opts(C), d);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_mlp_phase(const MlpPhaseDesc& d, cudaStream_t st) {
  int U = 0, C = 0;
  if (!mlp_phase_supported(d.H, d.I, &U, &C) || U != d.U || C != d.C || d.in.nparts > kPhaseMaxParts ||
      (d.in.nparts && !d.in.parts) || !d.in.base || !d.parts_out)
    return cudaErrorInvalidValue;
  if (g_occ_query) {
    g_occ_family = FAM_PHASE;
    const double kn = 3.0 * d.H * d.I;
    g_occ_flops = 2.0 * kn;
    g_occ_wbytes = 0.5625 * kn;
  }
  const dim3 grid(d.I / (32 * U) / C, C);
  const size_t smem = mlp_phase_smem(d);
  const int NS = 32 * U / (8192 / d.H);
  if (U == 2 && NS == 16) return launch_k(mlp_phase_kernel<2, 16>, grid, dim3(kT), smem, st, phase_opts(C), d);
  if (U == 1 && NS == 4) return launch_k(mlp_phase_kernel<1, 4>, grid, dim3(kT), smem, st, phase_opts(C), d);
  if (U == 1 && NS == 2) return launch_k(mlp_phase_kernel<1, 2>, grid, dim3(kT), smem, st, phase_opts(C), d);
  if (U == 1 && NS == 1) return launch_k(mlp_phase_kernel<1, 1>, grid, dim3(kT), smem, st, phase_opts(C), d);
  return cudaErrorInvalidValue;
}

// Large dynamic shared memory and 16-CTA clusters, once per device (outside
// any stream capture).
void phase_init_attributes() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
  auto attrs = [](const void* f, size_t smem) {
    cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  };
  const size_t sa = sizeof(float) * (size_t)attn_phase_floats(kPhaseMaxH);
  attrs(reinterpret_cast<const void*>(attn_phase_kernel<1>), sa);
  attrs(reinterpret_cast<const void*>(attn_phase_kernel<2>), sa);
  attrs(reinterpret_cast<const void*>(attn_phase_kernel<4>), sa);
  attrs(reinterpret_cast<const void*>(mlp_phase_kernel<2, 16>), mlp_phase_bytes(2048, 2));
  attrs(reinterpret_cast<const void*>(mlp_phase_kernel<1, 4>), mlp_phase_bytes(1024, 1));
  attrs(reinterpret_cast<const void*>(mlp_phase_kernel<1, 2>), mlp_phase_bytes(512, 1));
  attrs(reinterpret_cast<const void*>(mlp_phase_kernel<1, 1>), mlp_phase_bytes(256, 1));
  cudaGetLastError();
  done[dev] = true;
}

}  // namespace qtts
