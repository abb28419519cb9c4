// tc_gemm.cu -- batched Q4 projections on the sm_100a tensor cores (tcgen05).
//
// Serves a projection with M >= kTcMinRows input rows (batched decode,
// prefill): gemm_q4 of gemv.rs:311-375 as a real GEMM, with the same
// prologues and epilogues as the CUDA-core kernels of gemv.cu.  Three kernels
// per projection:
//
//  1. xsplit_kernel: the RMSNorm / embedding-gather prologue, writing the
//     input rows as two fp16 operands hi + lo (hi = fp16(x), lo = fp16(x - hi),
//     x = hi + lo to ~22 bits) already in the UMMA K-major core-matrix order,
//     one 32 KB block (hi | lo) per (128-row block, 64-deep K stage), so that a
//     stage of A is one bulk copy.
//  2. tc_gemm_kernel: a CTA owns one 128-column tile (of both matrices of a
//     gate/up pair) and one K slice.  Per 64-deep stage a bulk copy brings
//     the A block (mbarrier complete_tx), the 128 threads dequantise the Q4
//     tile into fp16 hi + lo in the UMMA MN-major core-matrix order (the Q4
//     value (q-8)*scale has at most 14 significant bits, so hi + lo holds it
//     exactly), and one thread issues hi*hi + hi*lo + lo*hi tcgen05.mma
//     (kind::f16, f32 accumulate in TMEM) and commits them to the stage's
//     mbarrier.  Two stages are in flight: the MMAs of stage i run while the
//     threads dequantise stage i+1, and the A block of stage i+2 is fetched
//     as soon as the MMAs of stage i have drained.  The accumulator is read
//     back with tcgen05.ld and stored as this slice's partial.  Every
//     mbarrier wait is bounded in time: on expiry the kernel records an
//     error, drains (bounded) its own copies and MMAs, frees its TMEM and
//     returns.
//  3. tc_epilogue_kernel: sums the K-slice partials in slice order
//     (deterministic) and runs the epilogue of epilogue.cuh.
//
// Shared-memory operand layout (no swizzle, 16-byte core-matrix rows):
//   A (K-major):  row r, k-chunk c (8 elements) at (r/8)*1024 + c*128 + (r%8)*16
//                 -> LBO 128 B (next 8-deep K chunk), SBO 1024 B (next 8 rows)
//   B (MN-major): k row j, column group g (8 columns) at g*1024 + (j/8)*128 + (j%8)*16
//                 -> LBO 128 B (next 8-deep K group), SBO 1024 B (next 8 columns)
// A 16-deep MMA step advances both start addresses by 256 B.
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace qtts {

namespace {

constexpr int TM = kTcRows;     // rows per MMA tile (TMEM lanes)
constexpr int TN = kTcCols;     // columns per CTA tile (per matrix)
constexpr int TK = kTcK;        // K per stage
constexpr int STAGES = 2;
constexpr int A_BYTES = TM * TK * 2;  // 16 KB per operand half
constexpr int B_BYTES = TN * TK * 2;  // 16 KB per operand half
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s bound on any wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Parity wait bounded by kWaitNs; true when the phase completed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (unsigned it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 255u) == 0) {
      const unsigned long long t = globaltimer();
      if (it == 0) t0 = t;
      else if (t - t0 > kWaitNs) return false;
    }
  }
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// SMEM matrix descriptor: start >> 4, LBO 128 B, SBO 1024 B, version 1, no swizzle.
__device__ __forceinline__ uint64_t sdesc(const void* p) {
  const uint64_t start = (smem_u32(p) >> 4) & 0x3FFFu;
  return start | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46);
}
// Instruction descriptor, kind::f16: D f32, A fp16 K-major, B fp16 MN-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) |
                            ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void split_h(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

// 128-column tile t of the launch -> matrix, first column within it.
__device__ __forceinline__ int tc_tile(const GemvDesc& d, int t, int NMv, int& tcol) {
  const int t256 = t >> 1;
  int mat = 0;
  if (NMv == 1) {
    while (mat + 1 < d.nmat && t256 >= d.tile0[mat + 1]) ++mat;
  }
  tcol = ((NMv == 2 ? t256 : t256 - d.tile0[mat]) * 2 + (t & 1)) * TN;
  return mat;
}

}  // namespace

// ---------------------------------------------------------------------------
// 1. prologue + operand split.  Grid (nks, ceil(M/TM)), 128 threads; thread r
// converts row r of the (row block, K stage) block.
__global__ void __launch_bounds__(128) xsplit_kernel(const GemvDesc d) {
  pdl_launch_dependents();
  pdl_wait();
  const int ks = blockIdx.x, mb = blockIdx.y, r = threadIdx.x;
  const int m = mb * TM + r;
  const int nks = (d.k + TK - 1) / TK;
  const int k0 = ks * TK;
  __half* hi = d.xsplit + ((size_t)(mb * nks + ks) * 2) * (TM * TK);
  __half* lo = hi + TM * TK;
  float xv[TK];
#pragma unroll
  for (int j = 0; j < TK; ++j) xv[j] = 0.0f;
  if (m < d.M) {
    if (d.emb_idx) {
      const uint32_t row = d.emb_idx[(size_t)m * d.emb_idx_stride];
      const uint8_t* prow = d.emb.packed + (size_t)row * (d.emb.n / 2);
      const __half* srow = d.emb.scales + (size_t)row * (d.emb.n / 32);
#pragma unroll
      for (int j = 0; j < TK; ++j)
        if (k0 + j < d.k) xv[j] = q4_value(prow, srow, k0 + j);
    } else {
      const float* xr = d.X + (size_t)m * d.ldx;
      if (d.gamma) {
        float inv;
        if (d.ssq_in) {
          inv = inv_rms_from_ssq(d, m);
        } else {
          float ss = 0.0f;
          for (int i = 0; i < d.k; ++i) ss += xr[i] * xr[i];
          inv = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
        }
#pragma unroll
        for (int j = 0; j < TK; ++j)
          if (k0 + j < d.k) xv[j] = xr[k0 + j] * inv * h2f(d.gamma[k0 + j]);  // gemv.rs:408-417
        if (d.xnorm_out) {
#pragma unroll
          for (int j = 0; j < TK; ++j)
            if (k0 + j < d.k) d.xnorm_out[(size_t)m * d.ld_xnorm + k0 + j] = xv[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < TK; ++j)
          if (k0 + j < d.k) xv[j] = xr[k0 + j];
      }
    }
  }
  const int grp = r >> 3, rl = r & 7;
#pragma unroll
  for (int c = 0; c < TK / 8; ++c) {
    __align__(16) __half h8[8];
    __align__(16) __half l8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) split_h(xv[c * 8 + j], h8[j], l8[j]);
    const size_t off = (size_t)grp * 512 + (size_t)c * 64 + rl * 8;  // halves
    *reinterpret_cast<uint4*>(hi + off) = *reinterpret_cast<const uint4*>(h8);
    *reinterpret_cast<uint4*>(lo + off) = *reinterpret_cast<const uint4*>(l8);
  }
}

// ---------------------------------------------------------------------------
// 2. the tensor-core GEMM.  Grid (2 * ntiles, S, ceil(M/TM)), 128 threads.
template <int NM>
__global__ void __launch_bounds__(128, 1) tc_gemm_kernel(const GemvDesc d) {
  extern __shared__ __align__(1024) uint8_t tsm[];
  // per stage: A hi | A lo | B hi (NM matrices) | B lo (NM matrices); then barriers
  constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * NM * B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tsm + STAGES * STAGE_BYTES);
  uint64_t* a_full = bars;             // [STAGES] A block landed
  uint64_t* mma_done = bars + STAGES;  // [STAGES] MMAs of the stage drained
  uint64_t* fin = bars + 2 * STAGES;   // every MMA drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int split = blockIdx.y, mb = blockIdx.z;
  int tcol;
  const int mat = tc_tile(d, blockIdx.x, NM, tcol);
  const int n = d.mat[mat].n;
  const int nks = (d.k + TK - 1) / TK;
  const int ks0 = split * d.tc_ks;
  const int nst = max(0, min(nks, ks0 + d.tc_ks) - ks0);
  if (tcol >= n || nst == 0) return;  // empty half tile (n % 256 != 0) or empty slice

  if (tid == 0) {
    for (int s = 0; s < 2 * STAGES + 1; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_wait();  // the operands are ready; TMEM is taken only after this
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)(NM * TN)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // B producer: thread -> k row br of the stage, 64-column half bh; threads
  // 8j..8j+7 hold 8 consecutive k rows (conflict-free 16-byte smem stores)
  const int br = (tid & 7) | ((tid >> 4) << 3), bh = (tid >> 3) & 1;
  const int kg = br >> 3, kr = br & 7;
  auto load_b = [&](int ks, int a, uint4 (&w)[2], unsigned short (&s)[2]) {
    const Q4Mat& Mt = d.mat[NM == 2 ? a : mat];
    const int row = ks * TK + br;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int col = tcol + bh * 64 + g * 32;
      if (col < n && row < d.k) {
        w[g] = ld_stream16(Mt.packed + (size_t)row * (n / 2) + col / 2);
        s[g] = __ldg(reinterpret_cast<const unsigned short*>(Mt.scales) + (size_t)row * (n / 32) + col / 32);
      } else {
        w[g] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // q = 8 -> 0
        s[g] = 0;
      }
    }
  };
  auto store_b = [&](uint8_t* bhi, uint8_t* blo, const uint4 (&w)[2], const unsigned short (&s)[2]) {
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const float sc = __half2float(__ushort_as_half(s[g]));
      const uint32_t words[4] = {w[g].x, w[g].y, w[g].z, w[g].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // 8 columns per 32-bit word, low nibble first
        __align__(16) __half h8[8];
        __align__(16) __half l8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int qv = (int)((words[q] >> (4 * j)) & 0xFu) - 8;
          split_h(sc * (float)qv, h8[j], l8[j]);
        }
        const int cg8 = bh * 8 + g * 4 + q;  // 8-column group within the tile
        const int off = cg8 * 1024 + kg * 128 + kr * 16;
        *reinterpret_cast<uint4*>(bhi + off) = *reinterpret_cast<const uint4*>(h8);
        *reinterpret_cast<uint4*>(blo + off) = *reinterpret_cast<const uint4*>(l8);
      }
    }
  };
  const size_t ablk = (size_t)2 * TM * TK;  // halves per (row block, stage)
  const __half* abase = d.xsplit + ((size_t)mb * nks + ks0) * ablk;

  // thread 0's bookkeeping of outstanding A copies (for the error drain)
  unsigned a_uses[STAGES] = {0u, 0u};  // completed a_full waits per buffer
  bool a_pend[STAGES] = {false, false};

  uint4 wn[NM][2];
  unsigned short sn[NM][2];
#pragma unroll
  for (int a = 0; a < NM; ++a) load_b(ks0, a, wn[a], sn[a]);
  if (tid == 0) {
    for (int i = 0; i < min(STAGES, nst); ++i) {
      mbar_expect_tx(&a_full[i], 2 * A_BYTES);
      bulk_g2s(tsm + i * STAGE_BYTES, abase + (size_t)i * ablk, 2 * A_BYTES, &a_full[i]);
      a_pend[i] = true;
    }
  }
  bool ok = true;
  for (int i = 0; i < nst; ++i) {
    const int b = i % STAGES;
    uint8_t* st = tsm + b * STAGE_BYTES;
    uint4 w[NM][2];
    unsigned short s[NM][2];
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      w[a][0] = wn[a][0]; w[a][1] = wn[a][1];
      s[a][0] = sn[a][0]; s[a][1] = sn[a][1];
    }
    if (i + 1 < nst) {
#pragma unroll
      for (int a = 0; a < NM; ++a) load_b(ks0 + i + 1, a, wn[a], sn[a]);
    }
    // this buffer's B was read by the MMAs of stage i - STAGES
    bool w_ok = true;
    if (i >= STAGES) w_ok = mbar_wait(&mma_done[b], (unsigned)((i / STAGES) - 1) & 1u);
    if (!__syncthreads_and(w_ok)) { ok = false; break; }
#pragma unroll
    for (int a = 0; a < NM; ++a)
      store_b(st + 2 * A_BYTES + a * B_BYTES, st + 2 * A_BYTES + (NM + a) * B_BYTES, w[a], s[a]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // st.shared -> visible to tcgen05.mma
    __syncthreads();
    bool t_ok = true;
    if (tid == 0) {
      t_ok = mbar_wait(&a_full[b], a_uses[b] & 1u);
      if (t_ok) {
        ++a_uses[b];
        a_pend[b] = false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint8_t* ahi = st;
        const uint8_t* alo = st + A_BYTES;
#pragma unroll
        for (int a = 0; a < NM; ++a) {
          const uint8_t* bhi = st + 2 * A_BYTES + a * B_BYTES;
          const uint8_t* blo = st + 2 * A_BYTES + (NM + a) * B_BYTES;
          const uint32_t dt = tmem + (uint32_t)(a * TN);
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk) {
            umma(dt, sdesc(ahi + kk * 256), sdesc(bhi + kk * 256), (i > 0 || kk > 0) ? 1u : 0u);
            umma(dt, sdesc(ahi + kk * 256), sdesc(blo + kk * 256), 1u);
            umma(dt, sdesc(alo + kk * 256), sdesc(bhi + kk * 256), 1u);
          }
        }
        umma_commit(&mma_done[b]);
        // the previous stage's MMAs have had a dequantise period to drain:
        // refill its A buffer with stage i - 1 + STAGES
        if (i >= 1 && i - 1 + STAGES < nst) {
          const int pb = (i - 1) % STAGES;
          t_ok = mbar_wait(&mma_done[pb], (unsigned)((i - 1) / STAGES) & 1u);
          if (t_ok) {
            mbar_expect_tx(&a_full[pb], 2 * A_BYTES);
            bulk_g2s(tsm + pb * STAGE_BYTES, abase + (size_t)(i - 1 + STAGES) * ablk, 2 * A_BYTES, &a_full[pb]);
            a_pend[pb] = true;
          }
        }
      }
    }
    if (!__syncthreads_and(t_ok)) { ok = false; break; }
  }
  // drain: the commit tracks every earlier tcgen05.mma of thread 0
  if (tid == 0) umma_commit(fin);
  const bool fin_ok = mbar_wait(fin, 0);
  if (tid == 0) {
    if (!ok) {  // wait (bounded) for A copies still in flight into this CTA's shared memory
      for (int b = 0; b < STAGES; ++b)
        if (a_pend[b]) mbar_wait(&a_full[b], a_uses[b] & 1u);
    }
    if ((!ok || !fin_ok) && d.err_flag) atomicOr(d.err_flag, 4);
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  // accumulator -> partial [split][m][ncols]: thread = TMEM lane = output row
  const int m = mb * TM + tid;
  if (ok && fin_ok) {
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const int c0 = d.col0[NM == 2 ? a : mat] + tcol;
#pragma unroll
      for (int cc = 0; cc < TN / 32; ++cc) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(a * TN + cc * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
              "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
              "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (m < d.M) {
          float* dst = d.part + ((size_t)split * d.M + m) * d.ncols + c0 + cc * 32;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (tcol + cc * 32 + q * 4 < n)
              *reinterpret_cast<float4*>(dst + q * 4) =
                  make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                              __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
        }
      }
    }
  }
  pdl_launch_dependents();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(NM * TN)));
}

// ---------------------------------------------------------------------------
// 3. partial sum (slice order) + epilogue.  Grid (ntiles, 1, ceil(M/MB)).
template <int MB, int NM, int EPI>
__global__ void __launch_bounds__(kGemvThreads) tc_epilogue_kernel(const GemvDesc d, const FrameCodes fc, int S) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float sbuf[64];
  __shared__ float ybuf[MB * kTileN];
  const int tile = blockIdx.x, zb = blockIdx.z, tid = threadIdx.x;
  int mat = 0;
  if (NM == 1) {
    while (mat + 1 < d.nmat && tile >= d.tile0[mat + 1]) ++mat;
  }
  const int tcol = (NM == 2 ? tile : tile - d.tile0[mat]) * kTileN;
  const int n = d.mat[mat].n;
  const int m0 = zb * MB, mcnt = min(MB, d.M - m0);
  const int col = tcol + tid;
  float v[NM][MB];
#pragma unroll
  for (int a = 0; a < NM; ++a)
#pragma unroll
    for (int mm = 0; mm < MB; ++mm) {
      float t = 0.0f;
      if (col < n && mm < mcnt) {
        const size_t c = (size_t)d.col0[NM == 2 ? a : mat] + col;
        for (int sp = 0; sp < S; ++sp) t += __ldcg(d.part + ((size_t)sp * d.M + m0 + mm) * d.ncols + c);
      }
      v[a][mm] = t;
    }
  gemv_epilogue<MB, NM, EPI>(d, fc, v, mat, tile, tcol, m0, mcnt, zb, sbuf, ybuf);
}

// ---------------------------------------------------------------------------
size_t tc_smem_bytes(int nm) { return (size_t)STAGES * (2 * A_BYTES + 2 * nm * B_BYTES) + 128; }

size_t tc_xsplit_halves(int M, int k) {
  return (size_t)((M + TM - 1) / TM) * TM * (size_t)((k + TK - 1) / TK) * TK * 2;
}

int tc_splits(const GemvDesc& d) { return ((d.k + TK - 1) / TK + d.tc_ks - 1) / d.tc_ks; }

void tc_plan(int sm_count, GemvDesc& g) {
  const long nks = (g.k + TK - 1) / TK;
  const long ctas = 2L * g.ntiles * ((g.M + TM - 1) / TM);  // 128-column tiles x row blocks
  const long S = std::max(1L, std::min(nks, (sm_count + ctas - 1) / ctas));
  g.tc_ks = (int)((nks + S - 1) / S);
  g.tc = 1;
}

template <int MB, int NM, int EPI>
static cudaError_t launch_epi(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  LaunchOpts o;
  o.pdl = d.pdl != 0;
  const dim3 grid(d.ntiles, 1, (d.M + MB - 1) / MB);
  return launch_k(tc_epilogue_kernel<MB, NM, EPI>, grid, dim3(kGemvThreads), 0, st, o, d, fc, tc_splits(d));
}

cudaError_t launch_tc(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  if (!d.xsplit || !d.part || d.tc_ks <= 0 || d.M <= 0 || d.k <= 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(d.xsplit) % 16) return cudaErrorMisalignedAddress;
  const int nks = (d.k + TK - 1) / TK;
  const int S = tc_splits(d);
  const int zt = (d.M + TM - 1) / TM;
  LaunchOpts o;
  o.pdl = d.pdl != 0;
  cudaError_t e = launch_k(xsplit_kernel, dim3(nks, zt), dim3(128), 0, st, o, d);
  if (e != cudaSuccess) return e;
  const dim3 grid(2 * d.ntiles, S, zt);
  e = d.paired ? launch_k(tc_gemm_kernel<2>, grid, dim3(128), tc_smem_bytes(2), st, o, d)
               : launch_k(tc_gemm_kernel<1>, grid, dim3(128), tc_smem_bytes(1), st, o, d);
  if (e != cudaSuccess) return e;
  if (d.paired) return launch_epi<2, 2, EPI_SWIGLU>(d, fc, st);
  switch (d.epi_kind) {
    case EPI_STORE: return launch_epi<4, 1, EPI_STORE>(d, fc, st);
    case EPI_RESID: return launch_epi<4, 1, EPI_RESID>(d, fc, st);
    case EPI_QKV: return launch_epi<4, 1, EPI_QKV>(d, fc, st);
    case EPI_ARGMAX: return launch_epi<4, 1, EPI_ARGMAX>(d, fc, st);
    default: return cudaErrorInvalidValue;
  }
}

// Opt the GEMM into its dynamic shared memory once per device (outside any
// stream capture).
void tc_init_attributes() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
  cudaFuncSetAttribute(tc_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes(1));
  cudaFuncSetAttribute(tc_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes(2));
  cudaGetLastError();
  done[dev] = true;
}

}  // namespace qtts
