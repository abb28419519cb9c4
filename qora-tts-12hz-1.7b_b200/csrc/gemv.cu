// gemv.cu -- Q4 g32 dequant + GEMV/skinny-GEMM for sm_100a with fused
// prologues (RMSNorm, embedding gather) and epilogues (bias/SiLU, residual,
// SwiGLU, QK-norm + RoPE + KV append, argmax).
//
// Replaces gemv.rs:222-309 (gemv_q4_inner / gemv_q4) and gemv.rs:311-375
// (gemm_q4) and fuses the per-step glue of talker.rs:279-349 and
// code_predictor.rs:448-505 around them.
//
// Work decomposition (both kernels).  The weight is [k][n] with groups of 32
// along n, so an output column needs all k rows.  A CTA owns a 256-column
// tile (8 groups) and a contiguous slice of rows (split-K).  A warp load
// covers 4 rows x 128 bytes (lane = (row offset rr, group gi)); a lane keeps
// 32 column accumulators per input row.  The S CTAs of a tile form a
// thread-block cluster and reduce their partials in split order
// (deterministic).
//
// q4mv_dec_kernel (one input row, the batch-1 decode path) is shaped for
// latency: every weight row of a lane is loaded into registers before the
// programmatic-dependent-launch wait (weights are never written by an earlier
// kernel; the next kernel is released once this one's FMAs are done), the
// RMSNorm scale comes from per-tile sums of squares left by the
// producer of the row, the CTA reduces through shared memory, and the
// cluster reduction pushes each partial straight into the root CTA's shared
// memory followed by a single cluster barrier.
//
// q4mv_rows_kernel (M rows, MB per CTA) serves prefill and small batches.
#include <cooperative_groups.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace qtts {

namespace {

__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// mbarrier with one arrival (the root's expect-tx), made visible to the
// cluster before the CTA's barrier.cluster.arrive.relaxed.
__device__ __forceinline__ void mbar_init_cluster(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n\tfence.mbarrier_init.release.cluster;" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_expect_arrive(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Remote 4-byte store into a peer CTA's shared memory that completes 4
// transaction bytes on the peer's mbarrier.
__device__ __forceinline__ void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(raddr), "f"(v),
               "r"(rbar)
               : "memory");
}
// Phase-0 wait with cluster-scope acquire (the peers' st.async data), bounded
// by limit_ns of %globaltimer (1 s unless the launch's budget is shorter);
// false when it ran out.  A budget below 1 s polls with the non-blocking
// test_wait and reads the clock on every try (try_wait may suspend the
// thread until the data arrives, which a short budget would never see).
constexpr unsigned long long kWaitNs = 1000000000ull;
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, unsigned long long limit_ns) {
  const uint32_t a = smem_addr(bar);
  const bool short_budget = limit_ns < kWaitNs;
  unsigned long long t0 = 0;
  for (unsigned it = 0;; ++it) {
    uint32_t done;
    if (short_budget) {
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(done)
          : "r"(a)
          : "memory");
    } else {
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(done)
          : "r"(a)
          : "memory");
    }
    if (done) return true;
    if ((it & 255u) == 0 || short_budget) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (it == 0) t0 = t;
      else if (t - t0 > limit_ns) return false;
    }
  }
}


// Weight words + raw f16 scales of U row-steps of one lane (NM matrices).
template <int U, int NM>
struct WBatch {
  uint4 w[U][NM];
  unsigned short s[U][NM];
};

template <int U, int NM>
__device__ __forceinline__ void load_batch(WBatch<U, NM>& b, const GemvDesc& d, int mat, int r0, int R, int rb,
                                           int gcol, bool gval, size_t rowbytes, int ngr) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int rbu = rb + 32 * u;
    const bool ok = gval && rbu < R;
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const Q4Mat& Mt = d.mat[NM == 2 ? a : mat];
      if (ok) {
        const size_t r = (size_t)(r0 + rbu);
        b.w[u][a] = ld_stream16(Mt.packed + r * rowbytes + gcol / 2);
        b.s[u][a] = __ldg(reinterpret_cast<const unsigned short*>(Mt.scales) + r * ngr + gcol / 32);
      } else {
        b.w[u][a] = make_uint4(0, 0, 0, 0);
        b.s[u][a] = 0;
      }
    }
  }
}

__device__ __forceinline__ float u16_h2f(unsigned short s) { return __half2float(__ushort_as_half(s)); }

// One 256-column row of a reduction buffer, written by the 8 lanes gi = 0..7
// of a 4-row warp slice (32 columns each).  Lane gi writes its 16-byte chunk c
// at chunk (c + gi) % 8 of its group, so the 8 lanes of a store phase hit 8
// different bank groups instead of one; red_col gives the physical index of
// logical column col.
__device__ __forceinline__ void red_store(float* row, int gi, const float2 (&acc)[16]) {
  float4* dst = reinterpret_cast<float4*>(row + gi * 32);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    dst[(c + gi) & 7] = make_float4(acc[2 * c].x, acc[2 * c].y, acc[2 * c + 1].x, acc[2 * c + 1].y);
}
__device__ __forceinline__ int red_col(int col) { return (col & ~31) | ((col + 4 * (col >> 5)) & 31); }

}  // namespace

// Floats of shared memory before the split-K partial buffer: the CTA
// reduction buffer [8 warps][4 row offsets][NM][256].
__host__ __device__ inline int dec_front_floats(int NM) { return 8 * 4 * NM * kTileN; }

// ===========================================================================
// Decode kernel: M <= kDecMaxM input rows, one per blockIdx.z
template <int NM, int EPI, int NR>
__global__ void __launch_bounds__(kGemvThreads) q4mv_dec_kernel(const GemvDesc d, const FrameCodes fc) {
  extern __shared__ __align__(16) float sm[];
  const bool clustered = d.cluster && d.S > 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y, m = blockIdx.z;  // input row m
  float* red = sm;                                  // [8 warps][4 rr][NM][256]
  float* pbuf = sm + dec_front_floats(NM);          // [S][NM][256] partials pushed to the root
  float* sbuf = pbuf + kMaxClusterSplits * NM * kTileN;  // 64 floats
  float* ybuf = sbuf + 64;                          // [256]
  uint64_t* mbar = reinterpret_cast<uint64_t*>(ybuf + kTileN);  // root: partials landed
  if (clustered) {
    if (split == 0 && tid == 0) mbar_init_cluster(mbar);
    cluster_arrive_relaxed();  // the wait below precedes any DSMEM store
  }
  prefetch_next_weights(d);

  int mat = 0;
  if (NM == 1) {
    while (mat + 1 < d.nmat && tile >= d.tile0[mat + 1]) ++mat;
  }
  const int tcol = (NM == 2 ? tile : tile - d.tile0[mat]) * kTileN;
  const int n = d.mat[mat].n;
  const int r0 = split * d.rows_per_split;
  const int R = max(0, min(d.k, r0 + d.rows_per_split) - r0);
  const int rr = lane >> 3, gi = lane & 7;
  const int gcol = tcol + gi * 32;
  const bool gval = gcol < n;
  const int rb0 = warp * 4 + rr;

  // every weight row of this lane and, for an RMSNorm prologue, the norm
  // weights of its rows, before waiting on the previous kernel
  WBatch<NR, NM> wb;
  load_batch<NR, NM>(wb, d, mat, r0, R, rb0, gcol, gval, (size_t)n / 2, n / 32);
  // Prologue forms compiled per epilogue (the host rejects other pairings):
  // the embedding gather feeds STORE launches (input_proj, text fc1), the
  // attention and GLU inputs feed RESID launches (O, down), RMSNorm feeds the
  // rest.  Keeping the unused forms out keeps each instance's code small: a
  // batch-1 frame cycles through a few instances, and instruction fetch is a
  // top stall of these short kernels.
  constexpr bool kEmb = EPI == EPI_STORE, kAttn = EPI == EPI_RESID, kGlu = EPI == EPI_RESID,
                 kNorm = EPI != EPI_RESID;
  const bool norm_in = kNorm && d.gamma && !d.emb_idx && !d.attn_in;
  float gv[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    const int rb = rb0 + 32 * i;
    gv[i] = (norm_in && rb < R) ? h2f(d.gamma[r0 + rb]) : 0.0f;
  }
  // The CTA that runs the epilogue: the cluster's root, or (global split-K,
  // the last CTA of a tile to arrive) any of them, so all gather its inputs.
  const bool may_epi = !clustered || split == 0;
  QkvPre qp;  // QKV root CTA: what its epilogue reads, gathered in the prologue
  if (EPI == EPI_QKV && may_epi) {
    qp.on = true;
    qkv_pre_weights(qp, d, mat, tcol + tid);
  }
  pdl_wait();
  if (EPI == EPI_QKV && qp.on) qkv_pre_pos(qp, d, m);

  // the residual this CTA's epilogue will add (root CTA, EPI_RESID): loaded
  // now, alongside the inputs, instead of after the reduction
  float res_pre[1] = {0.0f};
  if (EPI == EPI_RESID && may_epi) {
    const int col = tcol + tid;
    if (col < n) res_pre[0] = d.epi.out[(size_t)m * d.epi.ldo + d.col0[mat] + col];
  }
  // Input values of this lane's rows.  Every load of a prologue is issued
  // before the first of them is used (one dependent round trip), and the
  // wait on the cluster barrier (every CTA of the cluster running, so DSMEM
  // is live) overlaps them.
  float xv[NR];
  if (kEmb && d.emb_idx) {
    const uint32_t row = d.emb_idx[(size_t)m * d.emb_idx_stride];
    const uint8_t* prow = d.emb.packed + (size_t)row * (d.emb.n / 2);
    const __half* srow = d.emb.scales + (size_t)row * (d.emb.n / 32);
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int rb = rb0 + 32 * i;
      xv[i] = rb < R ? q4_value(prow, srow, r0 + rb) : 0.0f;
    }
    if (clustered) cluster_wait();
    if (EPI == EPI_QKV && qp.on) qkv_pre_rest(qp, d, mat, tcol + tid);
  } else if (kAttn && d.attn_in) {
    // this K slice is query head h = r0 / 128: its attention output over
    // cache positions [0, kvp] (code_predictor.rs:467-491) is the input slice
    float* obuf = ybuf;        // [128] attention output
    float* sc = ybuf + 128;    // [kAttnInMaxPos] scores, then weights
    const int h = r0 / kHeadDim, hk = h / d.attn_group;
    int sess, pos, kvp;
    row_pos(d.attn_rp, m, sess, pos, kvp);
    const int L = kvp + 1;
    constexpr int kPw = kAttnInMaxPos / (kGemvThreads / 32);  // positions per warp
    const float4 q = *reinterpret_cast<const float4*>(d.attn_q + (size_t)m * d.attn_ldq + h * kHeadDim + 4 * lane);
    float4 kk[kPw];
#pragma unroll
    for (int t = 0; t < kPw; ++t) {
      const int j = warp + t * (kGemvThreads / 32);
      kk[t] = j < L ? kv_load4(d.attn_kv, kv_at(d.attn_kv, sess, j, 0, hk) + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float vc[kAttnInMaxPos];  // V column tid of every position (threads < 128)
#pragma unroll
    for (int j = 0; j < kAttnInMaxPos; ++j)
      vc[j] = (j < L && tid < kHeadDim) ? kv_load1(d.attn_kv, kv_at(d.attn_kv, sess, j, 1, hk) + tid) : 0.0f;
    if (clustered) cluster_wait();
    if (EPI == EPI_QKV && qp.on) qkv_pre_rest(qp, d, mat, tcol + tid);
    const float scale = 1.0f / sqrtf((float)kHeadDim);
#pragma unroll
    for (int t = 0; t < kPw; ++t) {
      const int j = warp + t * (kGemvThreads / 32);
      float dot = q.x * kk[t].x + q.y * kk[t].y + q.z * kk[t].z + q.w * kk[t].w;
#pragma unroll
      for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (lane == 0 && j < L) sc[j] = dot * scale;
    }
    __syncthreads();
    if (warp == 0) {  // max-subtracted softmax over the L <= 32 scores
      const float s = lane < L ? sc[lane] : -INFINITY;
      float mx = s;
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float e = lane < L ? expf(s - mx) : 0.0f;
      float sum = e;
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane < L) sc[lane] = e * (1.0f / sum);
    }
    __syncthreads();
    if (tid < kHeadDim) {
      float o = 0.0f;
#pragma unroll
      for (int j = 0; j < kAttnInMaxPos; ++j)
        if (j < L) o += sc[j] * vc[j];
      obuf[tid] = o;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int rb = rb0 + 32 * i;
      xv[i] = rb < R ? obuf[rb] : 0.0f;
    }
  } else {
    const float* xr = d.X + (size_t)m * d.ldx;
    float xg[NR];  // GLU: the up half of the row
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int rb = rb0 + 32 * i;
      xv[i] = rb < R ? xr[r0 + rb] : 0.0f;
      xg[i] = (kGlu && d.x_glu && rb < R) ? xr[d.x_glu + r0 + rb] : 0.0f;
    }
    // the producer's per-tile sums of squares (at most 16 tiles here)
    const bool ssq16 = kNorm && d.gamma && d.ssq_in && d.ssq_n <= 16;
    float sv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) sv[j] = (ssq16 && j < d.ssq_n) ? d.ssq_in[(size_t)m * d.ssq_ld + j] : 0.0f;
    if (clustered) cluster_wait();
    if (EPI == EPI_QKV && qp.on) qkv_pre_rest(qp, d, mat, tcol + tid);
    if (kNorm && d.gamma) {
      float inv;
      if (ssq16) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) ss += sv[j];  // tile order; the zero padding adds nothing
        inv = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
      } else if (d.ssq_in) {
        inv = inv_rms_from_ssq(d, m);
      } else {
        float ss = 0.0f;
        for (int i = tid; i < d.k; i += kGemvThreads) ss += xr[i] * xr[i];
        ss = block_sum_256(ss, sbuf);
        inv = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
      }
#pragma unroll
      for (int i = 0; i < NR; ++i) xv[i] = xv[i] * inv * gv[i];  // gemv.rs:414
    }
    if (kGlu && d.x_glu) {
#pragma unroll
      for (int i = 0; i < NR; ++i) xv[i] = xv[i] * xg[i];  // silu(gate) * up (gemv.rs:449-451)
    }
    if (d.xnorm_out && tile == 0 && gi == 0) {
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const int rb = rb0 + 32 * i;
        if (rb < R) d.xnorm_out[(size_t)m * d.ld_xnorm + r0 + rb] = xv[i];
      }
    }
  }

  float2 acc[NM][16];
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int c = 0; c < 16; ++c) acc[a][c] = make_float2(0.0f, 0.0f);
  const WBatch<NR, NM>& wr = wb;
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    if (rb0 + 32 * i < R) {
#pragma unroll
      for (int a = 0; a < NM; ++a) {
        const SxPack p = make_sx(u16_h2f(wr.s[i][a]) * xv[i]);  // s = scale * x (gemv.rs:239)
        q4_word_fma(wr.w[i][a].x, p, &acc[a][0]);
        q4_word_fma(wr.w[i][a].y, p, &acc[a][4]);
        q4_word_fma(wr.w[i][a].z, p, &acc[a][8]);
        q4_word_fma(wr.w[i][a].w, p, &acc[a][12]);
      }
    }
  }

  // Release the next kernel only now: its CTAs then prefetch their weights
  // while this one reduces, without crowding out this kernel's own loads.
  pdl_launch_dependents();
  // CTA reduction through shared memory: 32 (warp, rr) partials per column
  // (group-rotated rows: red_store / red_col)
#pragma unroll
  for (int a = 0; a < NM; ++a) red_store(red + ((warp * 4 + rr) * NM + a) * kTileN, gi, acc[a]);
  __syncthreads();
  float v[NM][1];
  const int pc = red_col(tid);
#pragma unroll
  for (int a = 0; a < NM; ++a) {
    float t = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) t += red[(j * NM + a) * kTileN + pc];
    v[a][0] = t;
  }

  if (clustered) {
    // Split-K: every other CTA of the cluster pushes its partial into the
    // root's shared memory with st.async, which completes bytes on the root's
    // mbarrier, and leaves; only the root waits (no second cluster barrier).
    const int rank = split;  // the cluster spans grid.y
    if (rank != 0) {
      const uint32_t rp = dsmem_map(smem_addr(pbuf), 0), rm = dsmem_map(smem_addr(mbar), 0);
#pragma unroll
      for (int a = 0; a < NM; ++a) st_async_f32(rp + 4u * (uint32_t)((rank * NM + a) * kTileN + tid), v[a][0], rm);
      return;
    }
    if (tid == 0) mbar_expect_arrive(mbar, (uint32_t)((d.S - 1) * NM * kTileN * sizeof(float)));
    // Within the launch's budget; past it the error is recorded and the
    // wait goes on (bounded by 1 s), so that no peer's push is still in
    // flight into this CTA when it moves on.
    if (!mbar_wait_cluster(mbar, d.wait_ns)) {
      if (tid == 0 && d.err_flag) atomicOr(d.err_flag, kErrWaitExpired);
      if (!mbar_wait_cluster(mbar, kWaitNs)) return;  // a peer never delivered: write nothing
    }
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      float pv[kMaxClusterSplits];  // every partial loaded before the first add
#pragma unroll
      for (int sp = 1; sp < kMaxClusterSplits; ++sp) pv[sp] = sp < d.S ? pbuf[(sp * NM + a) * kTileN + tid] : 0.0f;
      float t = v[a][0];  // split 0 first, then the others in split order
#pragma unroll
      for (int sp = 1; sp < kMaxClusterSplits; ++sp)
        if (sp < d.S) t += pv[sp];
      v[a][0] = t;
    }
  }
  else if (d.S > 1) {
    // Global split-K (no cluster): each slice writes its partials, the last
    // CTA of the tile to arrive sums all slices in split order
    // (deterministic) and runs the epilogue.
    const bool cv = tcol + tid < n;
#pragma unroll
    for (int a = 0; a < NM; ++a)
      if (cv) d.part[((size_t)split * d.M + m) * d.ncols + d.col0[NM == 2 ? a : mat] + tcol + tid] = v[a][0];
    __threadfence();
    __syncthreads();
    unsigned* ctr = d.counters + (size_t)tile * gridDim.z + m;
    if (tid == 0) *reinterpret_cast<volatile unsigned*>(sbuf) = atomicAdd(ctr, 1u);
    __syncthreads();
    if (*reinterpret_cast<volatile unsigned*>(sbuf) != (unsigned)(d.S - 1)) return;
    __syncthreads();  // every thread has read the ticket before sbuf is reused
    __threadfence();
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const size_t c = (size_t)d.col0[NM == 2 ? a : mat] + tcol + tid;
      float t = 0.0f;
      for (int sp0 = 0; sp0 < d.S; sp0 += 16) {  // 16 slices' loads in flight, added in split order
        float pv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          pv[j] = (sp0 + j < d.S && cv) ? __ldcg(d.part + ((size_t)(sp0 + j) * d.M + m) * d.ncols + c) : 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (sp0 + j < d.S) t += pv[j];
      }
      v[a][0] = t;
    }
    if (tid == 0) *ctr = 0u;  // ready for the next launch
  }
  gemv_epilogue<1, NM, EPI>(d, fc, v, mat, tile, tcol, m, 1, m, sbuf, ybuf, EPI == EPI_RESID ? res_pre : nullptr,
                            EPI == EPI_QKV ? &qp : nullptr);
}

// ===========================================================================
// general kernel: M rows, MB per CTA (prefill, batched decode)
template <int MB, int NM, int EPI>
__global__ void __launch_bounds__(kGemvThreads) q4mv_rows_kernel(const GemvDesc d, const FrameCodes fc) {
  pdl_launch_dependents();
  prefetch_next_weights(d);
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

  const int rr = lane >> 3, gi = lane & 7;
  const int gcol = tcol + gi * 32;
  const bool gval = gcol < n;
  const size_t rowbytes = (size_t)n / 2;
  const int ngr = n / 32;
  constexpr int U = (NM * MB >= 4) ? 2 : 4;

  // first weight batch: issued before waiting on the previous kernel
  WBatch<U, NM> cur;
  const int rb0 = warp * 4 + rr;
  load_batch<U, NM>(cur, d, mat, r0, R, rb0, gcol, gval, rowbytes, ngr);
  pdl_wait();

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
        float inv;
        if (d.ssq_in) {
          inv = inv_rms_from_ssq(d, m);
        } else {
          float ss = 0.0f;
          for (int i = tid; i < d.k; i += kGemvThreads) ss += xr[i] * xr[i];
          ss = block_sum_256(ss, sbuf);
          inv = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
        }
        for (int i = tid; i < R; i += kGemvThreads) xd[i] = xr[r0 + i] * inv * h2f(d.gamma[r0 + i]);
        if (d.xnorm_out && tile == 0)
          for (int i = tid; i < R; i += kGemvThreads) d.xnorm_out[(size_t)m * d.ld_xnorm + r0 + i] = xd[i];
      } else {
        for (int i = tid; i < R; i += kGemvThreads) xd[i] = xr[r0 + i];
      }
    }
  }
  __syncthreads();

  // ---- main loop: stream the Q4 slice (double-buffered), 32 columns per lane
  float2 acc[NM][MB][16];
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int b = 0; b < MB; ++b)
#pragma unroll
      for (int c = 0; c < 16; ++c) acc[a][b][c] = make_float2(0.0f, 0.0f);

  for (int rb = rb0; rb < R; rb += 32 * U) {
    WBatch<U, NM> nxt;
    const bool more = rb + 32 * U < R;
    if (more) load_batch<U, NM>(nxt, d, mat, r0, R, rb + 32 * U, gcol, gval, rowbytes, ngr);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int rbu = rb + 32 * u;
      if (rbu < R) {
#pragma unroll
        for (int mm = 0; mm < MB; ++mm) {
          const float xv = xs[mm * RPS + rbu];
#pragma unroll
          for (int a = 0; a < NM; ++a) {
            const SxPack p = make_sx(u16_h2f(cur.s[u][a]) * xv);  // s = scale * x (gemv.rs:239)
            q4_word_fma(cur.w[u][a].x, p, &acc[a][mm][0]);
            q4_word_fma(cur.w[u][a].y, p, &acc[a][mm][4]);
            q4_word_fma(cur.w[u][a].z, p, &acc[a][mm][8]);
            q4_word_fma(cur.w[u][a].w, p, &acc[a][mm][12]);
          }
        }
      }
    }
    if (more) cur = nxt;
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
      for (int mm = 0; mm < MB; ++mm) red_store(red + ((warp * NM + a) * MB + mm) * kTileN, gi, acc[a][mm]);
  }
  __syncthreads();
  float v[NM][MB];
  const int pc = red_col(tid);
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      float t = 0.0f;
#pragma unroll
      for (int w8 = 0; w8 < 8; ++w8) t += red[((w8 * NM + a) * MB + mm) * kTileN + pc];
      v[a][mm] = t;
    }

  const int col = tcol + tid;
  const bool cval = col < n;

  // ---- split-K reduction (deterministic, split order)
  if (d.S > 1 && d.cluster) {
    cg::cluster_group cl = cg::this_cluster();
    __syncthreads();  // every warp has read `red`
#pragma unroll
    for (int a = 0; a < NM; ++a)
#pragma unroll
      for (int mm = 0; mm < MB; ++mm) red[(a * MB + mm) * kTileN + tid] = v[a][mm];
    cl.sync();
    const bool root = cl.block_rank() == 0;
    if (root) {
#pragma unroll
      for (int a = 0; a < NM; ++a)
#pragma unroll
        for (int mm = 0; mm < MB; ++mm) {
          float t = 0.0f;
          for (int sp = 0; sp < d.S; ++sp) t += cl.map_shared_rank(red, sp)[(a * MB + mm) * kTileN + tid];
          v[a][mm] = t;
        }
    }
    cl.sync();  // peers keep their shared memory until the root has read it
    if (!root) return;
  } else if (d.S > 1) {
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const int cg0 = d.col0[NM == 2 ? a : mat] + col;
#pragma unroll
      for (int mm = 0; mm < MB; ++mm)
        if (cval && mm < mcnt) d.part[((size_t)split * d.M + m0 + mm) * d.ncols + cg0] = v[a][mm];
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
      const int cg0 = d.col0[NM == 2 ? a : mat] + col;
#pragma unroll
      for (int mm = 0; mm < MB; ++mm) {
        float t = 0.0f;
        if (cval && mm < mcnt)
          for (int sp = 0; sp < d.S; ++sp) t += ld_cg(d.part + ((size_t)sp * d.M + m0 + mm) * d.ncols + cg0);
        v[a][mm] = t;
      }
    }
    if (tid == 0) *ctr = 0u;
  }
  gemv_epilogue<MB, NM, EPI>(d, fc, v, mat, tile, tcol, m0, mcnt, zb, sbuf, ybuf);
}

// ===========================================================================
// Batch kernel: 3..15 input rows (small decode batches), MB per CTA.
//
// The CTA's weight slice (RPS rows x 256 columns of each matrix) and its
// group scales are staged in shared memory before the dependency wait, so
// the whole slice is in flight at once.  Thread (warp w, lane l) owns the 8
// columns of weight word l (group l / 4) and the slice rows w, w + 8, ...:
// each word is dequantised once and applied to all MB input rows.  The 8
// warps' partials are reduced through shared memory; row mm of the tile then
// belongs to cluster rank mm % S, which receives the other ranks' partials
// of that row by st.async, adds them in split order (deterministic) and runs
// the epilogue for it.
__host__ __device__ inline size_t batch_main_bytes(int NM, int MB, int rps) {
  const size_t front = (size_t)rps * (NM * (128 + 16) + MB * 8);  // words, scales, (x, x) pairs
  const size_t red = (size_t)8 * NM * MB * kTileN * sizeof(float);  // warp partials (reuse the front)
  return front > red ? front : red;
}
__host__ __device__ inline size_t batch_recv_bytes(int NM, int MB, int S) {
  return (size_t)S * ((MB + S - 1) / S) * NM * kTileN * sizeof(float);
}

namespace {
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
}  // namespace

template <int MB, int NM, int EPI>
#ifndef QTTS_BATCH_MINB
#define QTTS_BATCH_MINB 1
#endif
__global__ void __launch_bounds__(kGemvThreads, QTTS_BATCH_MINB) q4mv_batch_kernel(const GemvDesc d, const FrameCodes fc) {
  extern __shared__ __align__(16) unsigned char smb[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y, zb = blockIdx.z;
  const int S = d.S, RPS = d.rows_per_split;
  const bool clustered = S > 1;  // the S slices of a tile form one cluster
  const int RO = (MB + S - 1) / S;  // rows of the tile a rank may own
  uint32_t* wsm = reinterpret_cast<uint32_t*>(smb);                                    // [NM][RPS][32]
  unsigned short* ssm = reinterpret_cast<unsigned short*>(smb + (size_t)NM * RPS * 128);  // [NM][RPS][8]
  float2* xsm = reinterpret_cast<float2*>(smb + (size_t)NM * RPS * 144);                // [RPS][MB]
  float* red = reinterpret_cast<float*>(smb);                                          // [8][NM][MB][256]
  float* recv = reinterpret_cast<float*>(smb + batch_main_bytes(NM, MB, RPS));          // [S][RO][NM][256]
  float* sbuf = recv + (size_t)S * RO * NM * kTileN;                                   // 64 floats
  float* ybuf = sbuf + 64;                                                             // [256]
  uint64_t* mbar = reinterpret_cast<uint64_t*>(ybuf + kTileN);                         // this rank's rows landed
  const int m0 = zb * MB, mcnt = min(MB, d.M - m0);
  const int nown = split < mcnt ? (mcnt - split + S - 1) / S : 0;  // rows split, split + S, ...
  if (clustered) {
    if (tid == 0) mbar_init_cluster(mbar);
    cluster_arrive_relaxed();  // the wait below precedes any DSMEM store
  }
  prefetch_next_weights(d);

  int mat = 0;
  if (NM == 1) {
    while (mat + 1 < d.nmat && tile >= d.tile0[mat + 1]) ++mat;
  }
  const int tcol = (NM == 2 ? tile : tile - d.tile0[mat]) * kTileN;
  const int n = d.mat[mat].n;
  const int r0 = split * RPS;
  const int R = max(0, min(d.k, r0 + RPS) - r0);
  const size_t rowbytes = (size_t)n / 2;
  const int ngr = n / 32;

  // Weight slice -> shared memory by cp.async, zero-filled past the slice or
  // the matrix (weights are never written by an earlier kernel: issued before
  // the dependency wait, they land while the prologue runs)
#pragma unroll
  for (int a = 0; a < NM; ++a) {
    const Q4Mat& Mt = d.mat[NM == 2 ? a : mat];
    for (int e = tid; e < RPS * 8; e += kGemvThreads) {
      const int r = e >> 3, c = e & 7;
      const bool ok = r < R && tcol + 32 * c < n;
      const uint8_t* src = ok ? Mt.packed + (size_t)(r0 + r) * rowbytes + tcol / 2 + 16 * c : Mt.packed;
      cp_async16(smem_addr(wsm + ((size_t)a * RPS * 8 + e) * 4), src, ok ? 16u : 0u);
    }
  }
  // group scales: 16 bytes (8 groups) per slice row by cp.async when the
  // scale rows are 16-byte aligned (n a multiple of 256), else plain loads
  const bool sc16 = (n & 255) == 0;
#pragma unroll
  for (int a = 0; a < NM; ++a) {
    const unsigned short* sc = reinterpret_cast<const unsigned short*>(d.mat[NM == 2 ? a : mat].scales);
    if (sc16 && (reinterpret_cast<uintptr_t>(sc) & 15) == 0) {
      for (int r = tid; r < RPS; r += kGemvThreads) {
        const bool ok = r < R;
        cp_async16(smem_addr(ssm + ((size_t)a * RPS + r) * 8), ok ? sc + (size_t)(r0 + r) * ngr + tcol / 32 : sc,
                   ok ? 16u : 0u);
      }
    } else {
      for (int e0 = tid; e0 < RPS * 8; e0 += 8 * kGemvThreads) {
        unsigned short t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int e = e0 + u * kGemvThreads, r = e >> 3, gg = e & 7;
          t[u] = (r < R && tcol + 32 * gg < n) ? __ldg(sc + (size_t)(r0 + r) * ngr + tcol / 32 + gg)
                                              : (unsigned short)0;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (e0 + u * kGemvThreads < RPS * 8) ssm[(size_t)a * RPS * 8 + e0 + u * kGemvThreads] = t[u];
      }
    }
  }
  cp_async_commit();
  pdl_wait();

  // ---- prologue: rows [m0, m0 + mcnt) x K slice [r0, r0 + R) -> (x, x)
  // pairs; thread i takes slice row i of every input row, all loads first
  float inv[MB];
#pragma unroll
  for (int mm = 0; mm < MB; ++mm) inv[mm] = 1.0f;
  if (!d.emb_idx && d.gamma) {  // RMSNorm scale of each row
    if (d.ssq_in) {
#pragma unroll
      for (int mm = 0; mm < MB; ++mm)
        if (mm < mcnt) inv[mm] = inv_rms_from_ssq(d, m0 + mm);
    } else {
      for (int mm = 0; mm < mcnt; ++mm) {  // uniform: every thread takes part in the row sum
        const float* xr = d.X + (size_t)(m0 + mm) * d.ldx;
        float ss = 0.0f;
        for (int i = tid; i < d.k; i += kGemvThreads) ss += xr[i] * xr[i];
        ss = block_sum_256(ss, sbuf);
        const float t = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
#pragma unroll
        for (int q = 0; q < MB; ++q)
          if (q == mm) inv[q] = t;
      }
    }
  }
  for (int i = tid; i < RPS; i += kGemvThreads) {
    float x[MB];
    const bool in = i < R;
    if (d.emb_idx) {
#pragma unroll
      for (int mm = 0; mm < MB; ++mm) {
        x[mm] = 0.0f;
        if (in && mm < mcnt) {
          const uint32_t row = d.emb_idx[(size_t)(m0 + mm) * d.emb_idx_stride];
          x[mm] = q4_value(d.emb.packed + (size_t)row * (d.emb.n / 2), d.emb.scales + (size_t)row * (d.emb.n / 32),
                           r0 + i);
        }
      }
    } else {
#pragma unroll
      for (int mm = 0; mm < MB; ++mm) x[mm] = (in && mm < mcnt) ? d.X[(size_t)(m0 + mm) * d.ldx + r0 + i] : 0.0f;
      if (d.gamma) {
        const float gm = in ? h2f(d.gamma[r0 + i]) : 0.0f;
#pragma unroll
        for (int mm = 0; mm < MB; ++mm) {
          x[mm] = x[mm] * inv[mm] * gm;  // gemv.rs:414
          if (d.xnorm_out && tile == 0 && in && mm < mcnt) d.xnorm_out[(size_t)(m0 + mm) * d.ld_xnorm + r0 + i] = x[mm];
        }
      }
    }
    float4* xd = reinterpret_cast<float4*>(xsm + (size_t)i * MB);
#pragma unroll
    for (int q = 0; q < MB / 2; ++q) xd[q] = make_float4(x[2 * q], x[2 * q], x[2 * q + 1], x[2 * q + 1]);
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- main loop: one staged row per step, 8 columns x MB rows per thread
  float2 acc[NM][MB][4];
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int b = 0; b < MB; ++b)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[a][b][j] = make_float2(0.0f, 0.0f);
  const int g = lane >> 2;
  const int nsteps = (R + 7) >> 3;  // rows past the slice in the last step are zero
#pragma unroll 4
  for (int i = 0; i < nsteps; ++i) {
    const int r = warp + 8 * i;
    float2 xx[MB];
    const float4* xp = reinterpret_cast<const float4*>(xsm + (size_t)r * MB);
#pragma unroll
    for (int q = 0; q < MB / 2; ++q) {
      const float4 t = xp[q];
      xx[2 * q] = make_float2(t.x, t.y);
      xx[2 * q + 1] = make_float2(t.z, t.w);
    }
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const uint32_t w = wsm[((size_t)a * RPS + r) * 32 + lane];
      const float s = u16_h2f(ssm[((size_t)a * RPS + r) * 8 + g]);
      // Weight values s * (q - 8), exact in f32 (an f16 scale times a 4-bit
      // integer): nibble j of byte b is column 2b + j (low nibble first,
      // gemv.rs:124); 0x43000000 | q << 16 is the float 128 + q, and one
      // fused multiply-add (128 + q) * s - 136 * s, its product exact and
      // 136 * s exact, rounds nothing.
      const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
      const float2 ss = make_float2(s, s), cc = make_float2(-136.0f * s, -136.0f * s);
      float2 wv[4];
#pragma unroll
      for (int b = 0; b < 4; ++b)
        wv[b] = __ffma2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x43000000u, 0x7054u | (b << 8))),
                                       __uint_as_float(__byte_perm(hi, 0x43000000u, 0x7054u | (b << 8)))),
                           ss, cc);
#pragma unroll
      for (int mm = 0; mm < MB; ++mm)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][mm][b] = __ffma2_rn(wv[b], xx[mm], acc[a][mm][b]);
    }
  }

  // Release the next kernel only now (as the decode kernel does).
  pdl_launch_dependents();
  // ---- CTA reduction over the 8 warps.  Lane l's 8 columns are two 16-byte
  // chunks, stored in swapped order when bit 2 of l is set, so that the 8
  // lanes of a store phase hit 8 different bank groups.
  __syncthreads();  // every warp is done with the staged slice (red reuses it)
  {
    const int sw = (lane >> 2) & 1;
#pragma unroll
    for (int a = 0; a < NM; ++a)
#pragma unroll
      for (int mm = 0; mm < MB; ++mm) {
        float4* dst = reinterpret_cast<float4*>(red + ((size_t)(warp * NM + a) * MB + mm) * kTileN + 8 * lane);
        dst[sw] = make_float4(acc[a][mm][0].x, acc[a][mm][0].y, acc[a][mm][1].x, acc[a][mm][1].y);
        dst[sw ^ 1] = make_float4(acc[a][mm][2].x, acc[a][mm][2].y, acc[a][mm][3].x, acc[a][mm][3].y);
      }
  }
  __syncthreads();
  const int pc = tid ^ (((tid >> 5) & 1) << 2);  // physical index of column tid
  float v[NM][MB];
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      float pv[8];
#pragma unroll
      for (int w8 = 0; w8 < 8; ++w8) pv[w8] = red[((size_t)(w8 * NM + a) * MB + mm) * kTileN + pc];
      float t = 0.0f;
#pragma unroll
      for (int w8 = 0; w8 < 8; ++w8) t += pv[w8];  // warp order
      v[a][mm] = t;
    }

  // ---- split-K: row mm's partial goes to rank mm % S (slot [split][mm / S])
  if (clustered) cluster_wait();  // every rank's mbarrier is initialised, its CTA running
  {
    int o = 0, ro = 0;  // rank and slot of row mm (mm % S, mm / S)
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      if (mm < mcnt) {
#pragma unroll
        for (int a = 0; a < NM; ++a) {
          const int idx = ((split * RO + ro) * NM + a) * kTileN + tid;
          if (o == split) {
            recv[idx] = v[a][mm];  // read back below by this same thread
          } else {
            st_async_f32(dsmem_map(smem_addr(recv + idx), (uint32_t)o), v[a][mm],
                         dsmem_map(smem_addr(mbar), (uint32_t)o));
          }
        }
      }
      if (++o == S) {
        o = 0;
        ++ro;
      }
    }
  }
  if (nown == 0) return;
  if (clustered) {
    if (tid == 0) mbar_expect_arrive(mbar, (uint32_t)((S - 1) * nown * NM * kTileN * sizeof(float)));
    // within the launch's budget; past it the error is recorded and the wait
    // goes on (bounded by 1 s) so that no peer's push is still in flight
    if (!mbar_wait_cluster(mbar, d.wait_ns)) {
      if (tid == 0 && d.err_flag) atomicOr(d.err_flag, kErrWaitExpired);
      if (!mbar_wait_cluster(mbar, kWaitNs)) return;  // a peer never delivered: write nothing
    }
  }
  for (int ro = 0; ro < nown; ++ro) {
    const int m = m0 + split + ro * S;
    float v1[NM][1];
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      float t = 0.0f;
      for (int sp = 0; sp < S; ++sp) t += recv[((sp * RO + ro) * NM + a) * kTileN + tid];  // split order
      v1[a][0] = t;
    }
    gemv_epilogue<1, NM, EPI>(d, fc, v1, mat, tile, tcol, m, 1, m, sbuf, ybuf);
  }
}

// ---------------------------------------------------------------------------
static bool use_dec(const GemvDesc& d) {
  const int nrmax = d.paired ? kDecRowsNM2 : kDecRowsNM1;
  return d.M <= kDecMaxM && d.mb == 1 && d.S <= (d.cluster ? kMaxClusterSplits : kMaxGlobalSplits) &&
         d.rows_per_split <= 32 * nrmax;
}

static bool use_batch(const GemvDesc& d) {
  return d.batch && (d.paired ? d.mb == kBatchRowsNM2 : (d.mb == kBatchRowsNM1 || d.mb == kBatchRowsNM1 / 2)) &&
         d.S >= 1 && d.S <= kMaxClusterSplits &&
         d.rows_per_split % 8 == 0 && d.rows_per_split <= (d.paired ? kBatchMaxRpsNM2 : kBatchMaxRpsNM1) && (long)d.S * d.rows_per_split >= d.k &&
         (d.S == 1 || d.cluster);
}

size_t gemv_smem_bytes(const GemvDesc& d) {
  const int NM = d.paired ? 2 : 1;
  if (d.batch)
    return batch_main_bytes(NM, d.mb, d.rows_per_split) + batch_recv_bytes(NM, d.mb, d.S) +
           sizeof(float) * (64 + kTileN) + 16;
  if (use_dec(d))
    return sizeof(float) * ((size_t)dec_front_floats(NM) +
                            (size_t)kMaxClusterSplits * NM * kTileN + 64 + kTileN + 4);
  return sizeof(float) * ((size_t)d.mb * d.rows_per_split + 8 * NM * d.mb * kTileN + 64 + d.mb * kTileN);
}

static LaunchOpts opts(const GemvDesc& d) {
  LaunchOpts o;
  o.pdl = d.pdl != 0;
  o.cluster_y = (d.cluster && d.S > 1) ? (unsigned)d.S : 1u;
  return o;
}

template <int MB, int NM, int EPI>
static cudaError_t launch_t(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  const dim3 grid(d.ntiles, d.S, (d.M + MB - 1) / MB);
  return launch_k(q4mv_rows_kernel<MB, NM, EPI>, grid, dim3(kGemvThreads), gemv_smem_bytes(d), st, opts(d), d, fc);
}

template <int MB, int NM, int EPI>
static cudaError_t launch_b(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  const dim3 grid(d.ntiles, d.S, (d.M + MB - 1) / MB);
  return launch_k(q4mv_batch_kernel<MB, NM, EPI>, grid, dim3(kGemvThreads), gemv_smem_bytes(d), st, opts(d), d,
                  fc);
}

template <int NM, int EPI, int NR>
static cudaError_t launch_dec(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  const dim3 grid(d.ntiles, d.S, d.M);
  return launch_k(q4mv_dec_kernel<NM, EPI, NR>, grid, dim3(kGemvThreads), gemv_smem_bytes(d), st, opts(d), d,
                  fc);
}

template <int NM, int EPI>
static cudaError_t dispatch_dec(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  const int nr = (d.rows_per_split + 31) / 32;
  if (NM == 2) {
    if (nr <= 2) return launch_dec<2, EPI, 2>(d, fc, st);
    if (nr <= 4) return launch_dec<2, EPI, 4>(d, fc, st);
    return launch_dec<2, EPI, kDecRowsNM2>(d, fc, st);
  }
  // residual projections (O and down) share one instance: fewer distinct
  // kernels in a layer's instruction stream
  if (nr <= 4 && EPI != EPI_RESID) return launch_dec<1, EPI, 4>(d, fc, st);
  if (nr <= 8) return launch_dec<1, EPI, 8>(d, fc, st);
  return launch_dec<1, EPI, kDecRowsNM1>(d, fc, st);
}

template <int MB, int NM, int EPI>
static void set_attr() {
  cudaFuncSetAttribute(q4mv_rows_kernel<MB, NM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
  cudaFuncSetAttribute(q4mv_rows_kernel<MB, NM, EPI>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}
template <int NM, int EPI, int NR>
static void set_attr_dec() {
  cudaFuncSetAttribute(q4mv_dec_kernel<NM, EPI, NR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
  cudaFuncSetAttribute(q4mv_dec_kernel<NM, EPI, NR>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}
template <int MB, int NM, int EPI>
static void set_attr_b() {
  cudaFuncSetAttribute(q4mv_batch_kernel<MB, NM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaFuncSetAttribute(q4mv_batch_kernel<MB, NM, EPI>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}
template <int EPI>
static void set_attr_dec_nm1() {
  set_attr_dec<1, EPI, 4>(); set_attr_dec<1, EPI, 8>(); set_attr_dec<1, EPI, kDecRowsNM1>();
}

// Opt every instantiation into large dynamic shared memory and 16-CTA
// clusters once per device (outside any stream capture).
void gemv_init_attributes() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
  set_attr<1, 1, EPI_STORE>(); set_attr<2, 1, EPI_STORE>(); set_attr<4, 1, EPI_STORE>();
  set_attr<1, 1, EPI_RESID>(); set_attr<2, 1, EPI_RESID>(); set_attr<4, 1, EPI_RESID>();
  set_attr<1, 1, EPI_QKV>(); set_attr<2, 1, EPI_QKV>(); set_attr<4, 1, EPI_QKV>();
  set_attr<1, 1, EPI_ARGMAX>(); set_attr<2, 1, EPI_ARGMAX>(); set_attr<4, 1, EPI_ARGMAX>();
  set_attr<1, 2, EPI_SWIGLU>(); set_attr<2, 2, EPI_SWIGLU>();
  set_attr_dec_nm1<EPI_STORE>(); set_attr_dec_nm1<EPI_RESID>(); set_attr_dec_nm1<EPI_QKV>();
  set_attr_dec_nm1<EPI_ARGMAX>();
  set_attr_dec<2, EPI_SWIGLU, 2>(); set_attr_dec<2, EPI_SWIGLU, 4>(); set_attr_dec<2, EPI_SWIGLU, kDecRowsNM2>();
  set_attr_b<kBatchRowsNM1, 1, EPI_STORE>(); set_attr_b<kBatchRowsNM1, 1, EPI_RESID>();
  set_attr_b<kBatchRowsNM1, 1, EPI_QKV>(); set_attr_b<kBatchRowsNM1, 1, EPI_ARGMAX>();
  set_attr_b<kBatchRowsNM1 / 2, 1, EPI_STORE>(); set_attr_b<kBatchRowsNM1 / 2, 1, EPI_RESID>();
  set_attr_b<kBatchRowsNM1 / 2, 1, EPI_QKV>(); set_attr_b<kBatchRowsNM1 / 2, 1, EPI_ARGMAX>();
  set_attr_b<kBatchRowsNM2, 2, EPI_SWIGLU>();
  cudaGetLastError();
  done[dev] = true;
}

template <int EPI>
static cudaError_t launch_mb(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  if (d.batch) {
    if (!use_batch(d)) return cudaErrorInvalidValue;
    if (d.paired) return EPI == EPI_SWIGLU ? launch_b<kBatchRowsNM2, 2, EPI_SWIGLU>(d, fc, st) : cudaErrorInvalidValue;
    if (EPI == EPI_SWIGLU) return cudaErrorInvalidValue;
    constexpr int E = EPI == EPI_SWIGLU ? EPI_STORE : EPI;
    if (d.mb == kBatchRowsNM1 / 2) return launch_b<kBatchRowsNM1 / 2, 1, E>(d, fc, st);
    return launch_b<kBatchRowsNM1, 1, E>(d, fc, st);
  }
  if (d.paired) {
    if (EPI != EPI_SWIGLU) return cudaErrorInvalidValue;
    if (use_dec(d)) return dispatch_dec<2, EPI_SWIGLU>(d, fc, st);
    if (d.mb == 1) return launch_t<1, 2, EPI_SWIGLU>(d, fc, st);
    if (d.mb == 2) return launch_t<2, 2, EPI_SWIGLU>(d, fc, st);
    return cudaErrorInvalidValue;
  }
  if (EPI == EPI_SWIGLU) return cudaErrorInvalidValue;
  constexpr int E = EPI == EPI_SWIGLU ? EPI_STORE : EPI;
  if (use_dec(d)) return dispatch_dec<1, E>(d, fc, st);
  if (d.mb == 1) return launch_t<1, 1, E>(d, fc, st);
  if (d.mb == 2) return launch_t<2, 1, E>(d, fc, st);
  if (d.mb == 4) return launch_t<4, 1, E>(d, fc, st);
  return cudaErrorInvalidValue;
}

bool gemv_uses_decode_kernel(const GemvDesc& d) { return !d.tc && !d.batch && use_dec(d); }

cudaError_t launch_gemv(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  if (g_occ_query) {  // family and algorithmic work of this launch (profiling)
    g_occ_family = d.tc ? FAM_TC_PROJ : d.batch ? FAM_Q4MV_BATCH : (use_dec(d) ? FAM_Q4MV_DEC : FAM_Q4MV_ROWS);
    g_occ_flops = g_occ_wbytes = 0.0;
    for (int i = 0; i < (d.paired ? 2 : d.nmat); ++i) {
      const double kn = (double)d.mat[i].k * d.mat[i].n;
      g_occ_flops += 2.0 * d.M * kn;
      g_occ_wbytes += kn * 0.5625;
    }
  }
  if (d.batch && (d.tc || d.attn_in || d.x_glu)) return cudaErrorInvalidValue;
  if (d.attn_in && (d.tc || !use_dec(d) || d.rows_per_split != kHeadDim || d.epi_kind != EPI_RESID))
    return cudaErrorInvalidValue;  // the attention prologue lives in the decode kernel only
  if (d.x_glu && (d.tc || !use_dec(d) || d.gamma || d.emb_idx || d.attn_in || d.paired || d.epi_kind != EPI_RESID))
    return cudaErrorInvalidValue;  // the GLU prologue lives in the decode kernel's plain input path
  if (!d.tc && !d.batch && use_dec(d) &&
      ((d.emb_idx && d.epi_kind != EPI_STORE) || (d.gamma && d.epi_kind == EPI_RESID)))
    return cudaErrorInvalidValue;  // prologue forms the decode kernel compiles per epilogue
  if (d.tc) return launch_tc(d, fc, st);
  if (d.ntiles <= 0 || d.S <= 0 || d.M <= 0 || d.rows_per_split <= 0) return cudaErrorInvalidValue;
  if (d.cluster && d.S > kMaxClusterSplits) return cudaErrorInvalidValue;
  if (!d.cluster && d.S > 1 && (!d.part || !d.counters)) return cudaErrorInvalidValue;
  if (d.ssq_in && (d.ssq_n <= 0 || d.ssq_ld < d.ssq_n)) return cudaErrorInvalidValue;
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
