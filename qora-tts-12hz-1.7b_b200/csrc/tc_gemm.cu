// tc_gemm.cu -- batched Q4 projections on the sm_100a tensor cores (tcgen05).
//
// Serves a projection with M >= kTcMinRows input rows (batched decode,
// prefill): gemm_q4 of gemv.rs:311-375 as a real GEMM, with the prologues of
// the CUDA-core kernels (RMSNorm with the producer's sums of squares,
// embedding gather) and the same epilogues, in ONE kernel per projection.
//
// Work split.  A CTA (16 warps, one CTA per SM) owns one 128-column tile (of
// both matrices of a gate/up pair), one 128-row block of the input rows and
// one K slice; the S K-slices of a tile form a thread-block cluster (1, S, 1),
// with S chosen so that every cluster of the launch is resident in one wave.
//
// Main loop, per 64-deep K stage (2-4 operand stages in flight):
//   * the raw Q4 tile of the stage (packed bytes + f16 scales) has been
//     streaming into a shared-memory ring by cp.async 3-5 stages ahead;
//   * warps 0-6 dequantise it (a thread per 16-byte chunk of 32 columns) and
//     warps 7-14 normalise the input rows (held in registers one stage
//     ahead) and take the leftover chunks word by word, into
//     shared memory: X = the normalised input rows, W = the Q4 weights, each as
//     two fp16 operands hi + lo with lo = fp16((v - hi) * 2^11).  The Q4 value
//     (q-8)*scale has at most 14 significant bits, so hi + lo holds it
//     exactly; an f32 input keeps ~22 bits.  Carrying lo scaled by 2^11 keeps
//     it clear of the fp16 subnormal range.
//   * the converters arrive on the stage's "full" mbarrier; warp 15 waits on
//     it and issues the tcgen05.mma (kind::f16, f32 accumulators in TMEM)
//     with the weights as operand A (M = the tile's 128 columns) and the
//     input rows as operand B (N = the CTA's rows rounded up to 16):
//     D_main += W_hi*X_hi, D_cross += W_lo*X_hi + W_hi*X_lo, committing them
//     to the stage's "done" mbarrier, while the converters (synchronised
//     among themselves by a named barrier) already convert the next stage.
// Result = D_main + 2^-11 * D_cross (the dropped lo*lo term is ~2^-22).
//
// Expanded weights (WX instances): when every matrix of the launch carries
// the tiles tc_expand wrote at load, one thread bulk-copies each stage's
// 32 KB hi/lo tiles per matrix straight into the operand buffer (the first
// stages before the dependent-launch wait, the others once the buffer's
// MMAs are done) and the MMA warp also waits on that copy's mbarrier; the
// converters then only split the input rows.
//
// Epilogue: the accumulators go TMEM -> registers -> shared memory; the S
// CTAs of the cluster then each take a slice of the rows, sum the S partials
// over distributed shared memory in slice order (deterministic), and run the
// projection's epilogue with one warp per row: bias/SiLU store, residual add
// with per-128-column sums of squares, SwiGLU, per-head QK-norm + RoPE + KV
// append (a head is one 128-column tile), or the greedy argmax.
//
// Shared-memory operand layout (no swizzle, 16-byte core-matrix rows):
//   X (K-major):  row r, k-chunk c (8 elements) at (r/8)*1024 + c*128 + (r%8)*16
//                 -> LBO 128 B (next 8-deep K chunk), SBO 1024 B (next 8 rows)
//   W (MN-major): k row j, column group g (8 columns) at g*1024 + (j/8)*128 + (j%8)*16
//                 -> LBO 128 B (next 8-deep K group), SBO 1024 B (next 8 columns);
//                 a 16-byte row holds the group's columns in the order
//                 0,4,1,5,2,6,3,7 (tc_col maps accumulator lanes back)
// A 16-deep MMA step advances both start addresses by 256 B.
//
// Every mbarrier wait is bounded in time; on expiry the kernel records an
// error flag, waits (bounded) for its own copies and MMAs, frees its TMEM
// and still takes part in the cluster barriers, so no CTA is left waiting.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace qtts {

namespace {

constexpr int TM = kTcRows;  // rows per MMA tile (TMEM lanes)
constexpr int TN = kTcCols;  // columns per CTA tile (per matrix)
constexpr int TK = kTcK;     // K per stage
constexpr int kBConv = 224;           // warps 0-6 dequantise the weights
constexpr int kConv = 480;            // + warps 7-14 split the input rows
constexpr int kMmaWarp = kConv / 32;  // warp 15 issues the tensor-core MMAs
constexpr int kThreads = kConv + 32;
constexpr int A_BYTES = TM * TK * 2;  // 16 KB per operand half
constexpr int B_BYTES = TN * TK * 2;  // 16 KB per operand half
constexpr int kRedLd = TN + 4;        // staging row stride (floats)
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr float kLoScale = 2048.0f;
constexpr float kLoUnscale = 1.0f / 2048.0f;
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s bound on any wait
constexpr int kErrTimeout = kErrWaitExpired, kErrFp16Range = kErrFp16Input;      // err_flag bits

constexpr int kRawRow = 80;                       // raw packed row stride: 64 B + pad (conflict-free 16 B reads)
constexpr int kRawMat = TK * kRawRow + TK * 8;     // one matrix's raw stage: packed rows + 4 f16 scales per row

// CMP (compact): expanded weights and one input-row pass -- X halves of 64
// rows and no raw ring, which leaves room for a fourth single-matrix stage.
template <int NM, bool CMP = false>
struct TcCfg {
  static constexpr int XB = CMP ? A_BYTES / 2 : A_BYTES;    // bytes per input-row operand half
  static constexpr int STAGES = NM == 1 ? (CMP ? 4 : 3) : 2;  // operand stages (fp16 hi/lo, UMMA layout)
  static constexpr int RS = CMP ? 2 : (NM == 1 ? 5 : 3);     // raw weight stages in flight (cp.async ring)
  static constexpr int STAGE_BYTES = 2 * XB + 2 * NM * B_BYTES;
  static constexpr int PIPE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int RAW_STAGE = NM * kRawMat;
  static constexpr int RAW_BYTES = CMP ? 0 : RS * RAW_STAGE;  // the compact form has no raw ring
  static constexpr int RED_BYTES = NM * TM * kRedLd * 4;     // epilogue staging, over the operand stages
  static_assert(RED_BYTES <= PIPE_BYTES, "staging must fit the operand stages");
  static constexpr int AUX = PIPE_BYTES + RAW_BYTES;
  static constexpr int SMEM = AUX + 1024;  // + barriers, TMEM slot, 1/rms, flags
  static constexpr uint32_t TMEM_COLS = NM * 2 * TN;  // main + cross per matrix
};

// global -> shared asynchronous copies (cp.async); src_size < size zero-fills
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_size) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_size) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_size) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_size) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_dsmem4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
// Barrier 1 over the converter threads, AND-reducing a status.
__device__ __forceinline__ bool conv_sync_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kConv)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Bulk copy global -> this CTA's shared memory (no multicast), completing its
// bytes on the CTA's mbarrier; addresses and size multiples of 16 bytes.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
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
// SMEM matrix descriptor: start >> 4, LBO 128 B, SBO 1024 B, version 1, no swizzle.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  return ((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46);
}
// Instruction descriptor, kind::f16: D f32, A = the weights (fp16, MN-major:
// the 128 columns of the tile are the MMA's M), B = the input rows (fp16,
// K-major: N = the CTA's rows rounded up to 16), so a block of 64 rows costs
// half the tensor-pipe cycles of a 128-row tile.
__device__ __forceinline__ uint32_t idesc_rows(int nrows) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (1u << 15) | (0u << 16) | ((uint32_t)(nrows >> 3) << 17) |
         ((uint32_t)(TN >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// f32 pair -> fp16 hi pair and fp16 (residual * 2^11) pair (common.cuh)
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) { split_pair(a, b, hi, lo); }
static_assert(kXsRows == TM && kXsK == TK && kXsHalf == A_BYTES && kSplitLoScale == kLoScale,
              "split tiles are the input-row operand halves");

// 8 dequantised weights of one 32-bit word (nibble i = column i of the word,
// gemv.rs:124) as hi / lo 16-byte core-matrix rows.  One shift + LOP3 turns
// nibbles p and p + 4 into the half2 (1024 + q_p, 1024 + q_{p+4}), so a row
// holds the columns in the order 0,4,1,5,2,6,3,7; the MMA's M rows may come in
// any order, and the epilogue maps the accumulator lanes back (tc_col).
__device__ __forceinline__ void dequant_word(uint32_t w, __half2 s2, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
  const __half2 sc = __float2half2_rn(kLoScale);
  const __half2 k1032 = __float2half2_rn(1032.0f);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    uint32_t bits = ((w >> (4 * p)) & 0x000F000Fu) | 0x64006400u;  // 1024 + q per half
    const __half2 q = __hsub2(*reinterpret_cast<__half2*>(&bits), k1032);  // q - 8, exact
    const __half2 hh = __hmul2(q, s2);                      // fp16(q * scale)
    const __half2 rr = __hfma2(q, s2, __hneg2(hh));          // exact residual
    h[p] = h2_bits(hh);
    l[p] = h2_bits(__hmul2(rr, sc));
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}
// Column of the tile held by accumulator lane c (the MMA's M row c): rows
// store each 8-column group in the order 0,4,1,5,2,6,3,7.
__device__ __forceinline__ int tc_col(int c) { return (c & ~7) | ((c & 7) >> 1) | ((c & 1) << 2); }

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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Input rows of one stage held in registers by an input-row thread: pass p
// covers row (at & 63) + 64 p, 16 consecutive k starting at 16 * ((at >> 6) & 3).
template <int NP>
struct ARegs {
  float x[NP][16];
  uint4 g[2];  // the RMSNorm weights of the 16-deep k slice (same for every row)
};

}  // namespace

// ---------------------------------------------------------------------------
// Grid (2 * ntiles, S, ceil(M / 128)), cluster (1, S, 1), 512 threads.
template <int NM, int EPI, int NP, bool WX>
__global__ void __launch_bounds__(kThreads, 1) tc_proj_kernel(const GemvDesc d, const FrameCodes fc) {
  using C = TcCfg<NM, WX && NP == 1>;
  extern __shared__ __align__(1024) uint8_t tsm[];
  static_assert(C::STAGES <= 4, "barrier area holds 4 stages");
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(tsm + C::AUX);  // [STAGES] MMAs of the stage drained
  uint64_t* full = mma_done + 4;                                     // [STAGES] operands of the stage written
  uint64_t* wfull = full + 4;                                        // [STAGES] (WX) weight tiles of the stage landed
  uint64_t* fin = wfull + 4;                                         // every MMA drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tsm + C::AUX + 104);
  unsigned* s_flag = reinterpret_cast<unsigned*>(tsm + C::AUX + 112);
  float* s_inv = reinterpret_cast<float*>(tsm + C::AUX + 128);  // [128]
  float* red = reinterpret_cast<float*>(tsm);                   // epilogue staging [NM][128][kRedLd]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mb = blockIdx.z;
  int tcol;
  const int mat = tc_tile(d, blockIdx.x, NM, tcol);
  const int n = d.mat[mat].n;
  if (tcol >= n) return;  // empty half tile (n % 256 != 0): the whole cluster leaves together
  prefetch_next_weights(d);
  const int nks = (d.k + TK - 1) / TK;
  const int ks0 = blockIdx.y * d.tc_ks;
  const int nst = min(nks, ks0 + d.tc_ks) - ks0;  // >= 1 by construction of tc_ks
  const int m0 = mb * TM;
  const int Mv = min(TM, d.M - m0);
  const uint32_t tsm_a = smem_u32(tsm);
  // Row blocks of more than 64 rows may get their input rows split once for
  // all column tiles (tc_xsplit_kernel, or the rows' producer): the stage's
  // two X operand halves then arrive by one bulk copy, and every converter
  // warp dequantises weights -- or, with expanded weights, the stage is bulk
  // copies only (weights and rows on the same mbarrier) and nothing converts.
  const bool xs = NP == 2 && d.x_split != nullptr;

  // ---- raw weight tiles stream into the ring RS - 1 stages ahead; the
  // weights are never written by an earlier kernel, so this starts before
  // the programmatic-dependent-launch wait
  const uint32_t raw_a = tsm_a + C::PIPE_BYTES;
  // A thread's raw chunks are fixed for the whole kernel (chunk c = tid + j *
  // kConv of NM * 384: 256 packed 16-byte chunks, then 128 4-byte scale pairs
  // per matrix); per stage only the source row moves, by TK rows.
  struct RawChunk {
    const uint8_t* src0;  // row `row` of the tile's columns
    size_t stride;        // bytes per TK rows
    uint32_t dst;         // offset in a raw stage
    int row;              // row within the stage
    bool on, pk;          // chunk exists; packed (16 bytes) or scales (4 bytes)
  };
  RawChunk rc[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = tid + j * kConv;
    rc[j].on = tid < kConv && c < NM * 384;
    const int a = rc[j].on ? c / 384 : 0, cc = c % 384;
    const Q4Mat& Mt = d.mat[NM == 2 ? a : mat];
    rc[j].pk = cc < 256;
    if (rc[j].pk) {  // 16 bytes = 32 columns of packed nibbles
      const int ch = cc & 3;
      rc[j].row = cc >> 2;
      rc[j].on = rc[j].on && tcol + ch * 32 < n;
      rc[j].src0 = Mt.packed + (size_t)rc[j].row * (n / 2) + tcol / 2 + ch * 16;
      rc[j].stride = (size_t)TK * (n / 2);
      rc[j].dst = (uint32_t)(a * kRawMat + rc[j].row * kRawRow + ch * 16);
    } else {         // 4 bytes = 2 f16 scales = 64 columns
      const int h = (cc - 256) & 1;
      rc[j].row = (cc - 256) >> 1;
      rc[j].on = rc[j].on && tcol + h * 64 < n;
      rc[j].src0 = reinterpret_cast<const uint8_t*>(Mt.scales + (size_t)rc[j].row * (n / 32) + tcol / 32 + h * 2);
      rc[j].stride = (size_t)TK * (n / 32) * 2;
      rc[j].dst = (uint32_t)(a * kRawMat + TK * kRawRow + rc[j].row * 8 + h * 4);
    }
  }
  // Chunks past K or past n are zero-filled (source size 0) from a valid address.
  auto issue_b = [&](int ks, int slot) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (j * kConv >= NM * 384) break;
      const bool v = rc[j].on && ks * TK + rc[j].row < d.k;
      const uint8_t* src = v ? rc[j].src0 + (size_t)ks * rc[j].stride : d.mat[0].packed;
      const uint32_t dst = raw_a + slot * C::RAW_STAGE + rc[j].dst;
      if (tid + j * kConv < NM * 384) {
        if (rc[j].pk) cp_async16(dst, src, v ? 16u : 0u);
        else cp_async4(dst, src, v ? 4u : 0u);
      }
    }
  };
  if (!WX && tid < kConv) {
    for (int j = 0; j < C::RS - 1; ++j) {
      if (j < nst) issue_b(ks0 + j, j);
      cp_async_commit();
    }
  }
  // WX: the stage's expanded weight tiles (16 KB hi + 16 KB lo per matrix,
  // block (tile, stage) of the matrix's expansion) by bulk copies into the
  // operand buffer, completing on wfull[buffer]; one thread issues them
  const int nks_all = (d.k + TK - 1) / TK;
  auto issue_w = [&](int i) {
    const int b = i % C::STAGES;
    const uint32_t st_a = tsm_a + (uint32_t)(b * C::STAGE_BYTES);
    // with split rows the stage's row copy (issued later, after the
    // dependent-launch wait for the first stages) completes on the same phase
    mbar_expect_tx(&wfull[b], (uint32_t)(NM * 2 * B_BYTES + (xs ? 2 * C::XB : 0)));
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      const Q4Mat& Mt = d.mat[NM == 2 ? a : mat];
      const uint8_t* src = Mt.wx + ((size_t)(tcol / TN) * nks_all + (ks0 + i)) * (2 * B_BYTES);
      bulk_g2s(st_a + 2 * C::XB + a * B_BYTES, src, B_BYTES, &wfull[b]);
      bulk_g2s(st_a + 2 * C::XB + (NM + a) * B_BYTES, src + B_BYTES, B_BYTES, &wfull[b]);
    }
  };
  // pre-split input rows: block (row block mb, stage) of the split tiles,
  // hi then lo, straight into the stage's X halves, completing on wfull
  auto issue_xs = [&](int i) {
    const int b = i % C::STAGES;
    if (!WX) mbar_expect_tx(&wfull[b], (uint32_t)(2 * C::XB));  // (WX: counted by issue_w)
    bulk_g2s(tsm_a + (uint32_t)(b * C::STAGE_BYTES), d.x_split + ((size_t)mb * nks_all + (ks0 + i)) * (2 * C::XB),
             (uint32_t)(2 * C::XB), &wfull[b]);
  };

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&mma_done[s], 1);
      mbar_init(&full[s], kConv);
    }
    mbar_init(fin, 1);
    if (WX || xs)
      for (int s = 0; s < C::STAGES; ++s) mbar_init(&wfull[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *s_flag = 0u;
    // the weights never depend on an earlier kernel: the first stages' tiles
    // are requested before the dependent-launch wait
    if (WX)
      for (int j = 0; j < C::STAGES && j < nst; ++j) issue_w(j);
  }
  int w_issued = (WX && tid == 0) ? min(C::STAGES, nst) : 0;  // stages whose weight copies were issued
  // rows [Mv, Nr) of every input-row buffer stay zero for the whole kernel
  // (the MMAs read Nr rows; rows past Nr are never read)
  const int Nr = (Mv + 15) & ~15;
  const uint32_t idesc = idesc_rows(Nr);
  if (!xs && Mv < Nr) {  // (the split tiles carry their zero rows)
    const int zrows = Nr - Mv;
    for (int i = tid; i < C::STAGES * 2 * zrows * (TK / 8); i += kThreads) {
      // rows fastest: 8 consecutive threads fill 8 different 16-byte bank groups
      const int r = Mv + i % zrows, c = (i / zrows) % (TK / 8), h = i / (zrows * (TK / 8));  // h: stage*2 + half
      uint8_t* base = tsm + (h >> 1) * C::STAGE_BYTES + (h & 1) * C::XB;
      *reinterpret_cast<uint4*>(base + (r >> 3) * 1024 + c * 128 + (r & 7) * 16) = make_uint4(0, 0, 0, 0);
    }
  }
  // ---- input rows of a stage (warps 7-14): registers one stage ahead ->
  // shared memory (split).  Thread: row (at & 63) + 64 p, 16-deep k slice at / 64.
  // the embedding gather and the normed-row copy serve STORE launches only
  // (input_proj, text fc1, codec head); other kinds compile without them
  constexpr bool kEmb = EPI == EPI_STORE;
  const bool a_thr = tid >= kBConv && tid < kConv;
  const int at = tid - kBConv, arow = at & 63, akc = (at >> 6) & 3;
  const int npass = NP == 1 ? 1 : (Mv > 64 ? 2 : 1);  // NP: passes compiled (1: blocks of <= 64 rows)
  const bool g16 = d.gamma && (reinterpret_cast<uintptr_t>(d.gamma) & 15u) == 0;
  auto load_a = [&](int ks, ARegs<NP>& R) {
    const int kk0 = ks * TK + akc * 16;
    if (g16 && kk0 + 16 <= d.k && !(kEmb && d.emb_idx)) {  // with the rows, one stage ahead
      R.g[0] = __ldg(reinterpret_cast<const uint4*>(d.gamma + kk0));
      R.g[1] = __ldg(reinterpret_cast<const uint4*>(d.gamma + kk0) + 1);
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int r = arow + 64 * p;
      if (p < npass && r < Mv) {
        const int m = m0 + r;
        if (kEmb && d.emb_idx) {
          const uint32_t er = d.emb_idx[(size_t)m * d.emb_idx_stride];
          const uint8_t* prow = d.emb.packed + (size_t)er * (d.emb.n / 2);
          const __half* srow = d.emb.scales + (size_t)er * (d.emb.n / 32);
#pragma unroll
          for (int j = 0; j < 16; ++j) R.x[p][j] = (kk0 + j < d.k) ? q4_value(prow, srow, kk0 + j) : 0.0f;
        } else {
          const float* xr = d.X + (size_t)m * d.ldx + kk0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 v = (kk0 + 4 * q < d.k) ? __ldg(reinterpret_cast<const float4*>(xr) + q)
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            R.x[p][4 * q] = v.x; R.x[p][4 * q + 1] = v.y; R.x[p][4 * q + 2] = v.z; R.x[p][4 * q + 3] = v.w;
          }
        }
      }
    }
  };
  pdl_wait();  // activations, norms' sums of squares and KV of earlier kernels are ready
  // the first stage's input rows are issued now, so their round trip overlaps
  // the TMEM allocation and the 1/rms loads below
  ARegs<NP> an;
  if (a_thr && !xs) load_a(ks0, an);
  if (xs && tid == 0) {  // the split tiles come from the kernel just before: after the wait
    for (int j = 0; j < C::STAGES && j < nst; ++j) issue_xs(j);
    w_issued = min(C::STAGES, nst);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // 1 / rms of each row (gemv.rs:408-417; applied by the split kernel instead)
  if (d.gamma && !xs) {
    if (d.ssq_in) {
      for (int r = tid; r < Mv; r += kThreads) s_inv[r] = inv_rms_from_ssq(d, m0 + r);
    } else {
      for (int r = warp; r < Mv; r += kThreads / 32) {
        const float* xr = d.X + (size_t)(m0 + r) * d.ldx;
        float ss = 0.0f;
        for (int i = lane; i < d.k; i += 32) ss += xr[i] * xr[i];
        ss = warp_sum(ss);
        if (lane == 0) s_inv[r] = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  float amax = 0.0f;
  auto store_a = [&](int ks, const ARegs<NP>& R, uint8_t* ahi, uint8_t* alo) {
    const int kk0 = ks * TK + akc * 16;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int r = arow + 64 * p;
      if (p < npass && r < Mv) {
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = R.x[p][j];
        if (d.gamma && !(kEmb && d.emb_idx)) {
          const float inv = s_inv[r];
          if (kk0 + 16 <= d.k && g16) {  // the two 16-byte loads issued with the rows
            const __half2* g2 = reinterpret_cast<const __half2*>(R.g);
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // (x * inv) * gamma, pairwise in f32x2 (gemv.rs:414)
              const float2 t = __fmul2_rn(__fmul2_rn(make_float2(y[2 * j], y[2 * j + 1]), make_float2(inv, inv)),
                                          __half22float2(g2[j]));
              y[2 * j] = t.x;
              y[2 * j + 1] = t.y;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = (kk0 + j < d.k) ? y[j] * inv * h2f(d.gamma[kk0 + j]) : 0.0f;
          }
          if (kEmb && d.xnorm_out && blockIdx.x == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (kk0 + j < d.k) d.xnorm_out[(size_t)(m0 + r) * d.ld_xnorm + kk0 + j] = y[j];
          }
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {  // two 8-deep k chunks
          uint32_t h[4], l[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            amax = fmaxf(amax, fmaxf(fabsf(y[c * 8 + 2 * q]), fabsf(y[c * 8 + 2 * q + 1])));
            split2(y[c * 8 + 2 * q], y[c * 8 + 2 * q + 1], h[q], l[q]);
          }
          const int off = (r >> 3) * 1024 + (akc * 2 + c) * 128 + (r & 7) * 16;
          *reinterpret_cast<uint4*>(ahi + off) = make_uint4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<uint4*>(alo + off) = make_uint4(l[0], l[1], l[2], l[3]);
        }
      }
    }
  };


  // Raw stage chunk q = (matrix q >> 8, 16-byte chunk ch = (q >> 6) & 3 of the
  // row, row q & 63): 32 columns, 4 words, one f16 scale.  Consecutive q are
  // consecutive rows, so a warp's 16-byte loads are conflict-free (80-byte
  // row stride) and each of its operand stores fills 512 contiguous bytes.
  // Word k of chunk ch is the 8-column group g8 = 4 ch + k, stored at
  // g8 * 1024 + (row / 8) * 128 + (row % 8) * 16 (hi; lo NM operands later).
  auto chunk_at = [&](int slot, int q, const uint8_t*& raw, uint8_t*& dst, uint8_t* stb) {
    const int a = q >> 8, ch = (q >> 6) & 3, brow = q & 63;
    const uint8_t* base = tsm + C::PIPE_BYTES + slot * C::RAW_STAGE + a * kRawMat;
    raw = base + brow * kRawRow + ch * 16;
    dst = stb + a * B_BYTES + ch * 4096 + (brow >> 3) * 128 + (brow & 7) * 16;
    return __half2half2(__ushort_as_half(*reinterpret_cast<const unsigned short*>(base + TK * kRawRow + brow * 8 + ch * 2)));
  };
  auto store_chunk = [&](uint8_t* stb, int slot, int q) {
    const uint8_t* raw;
    uint8_t* dst;
    const __half2 s2 = chunk_at(slot, q, raw, dst, stb);
    const uint4 w4 = *reinterpret_cast<const uint4*>(raw);
    const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint4 hi, lo;
      dequant_word(wv[k], s2, hi, lo);
      *reinterpret_cast<uint4*>(dst + k * 1024) = hi;
      *reinterpret_cast<uint4*>(dst + NM * B_BYTES + k * 1024) = lo;
    }
  };
  auto store_word = [&](uint8_t* stb, int slot, int q, int k) {  // word k of chunk q
    const uint8_t* raw;
    uint8_t* dst;
    const __half2 s2 = chunk_at(slot, q, raw, dst, stb);
    uint4 hi, lo;
    dequant_word(*reinterpret_cast<const uint32_t*>(raw + 4 * k), s2, hi, lo);
    *reinterpret_cast<uint4*>(dst + k * 1024) = hi;
    *reinterpret_cast<uint4*>(dst + NM * B_BYTES + k * 1024) = lo;
  };
  // Chunks per stage: NM * 256.  The weight warps take NM chunks each; the
  // 32 NM chunks left go to the input-row threads one word each (after their
  // rows, which take about as long as 3-4 words).
  constexpr int kChunksRem = NM * 256 - kBConv * NM;

  bool ok = true;
  if (tid < kConv) {
    // ---- converters (the input-row threads hold stage 0's rows in `an`)
    for (int i = 0; i < nst; ++i) {
      const int b = i % C::STAGES;
      uint8_t* st = tsm + b * C::STAGE_BYTES;
      const ARegs<NP> ac = an;
      if (a_thr && !xs && i + 1 < nst) load_a(ks0 + i + 1, an);  // input rows one stage ahead
      cp_async_wait<C::RS - 2>();  // this thread's raw copies of stage i have landed
      // this operand buffer was read by the MMAs of stage i - STAGES
      bool w_ok = true;
      if (i >= C::STAGES) w_ok = mbar_wait(&mma_done[b], (unsigned)((i / C::STAGES) - 1) & 1u);
      if (WX && tid == 0 && i >= C::STAGES && w_ok) {  // the buffer's MMAs are done
        issue_w(i);
        w_issued = i + 1;
      }
      if (xs && tid == 0 && i >= C::STAGES && w_ok) {
        issue_xs(i);
        w_issued = i + 1;
      }
      // publishes every converter's raw copies of stage i; every conversion of
      // stage i - 1 is done, so its raw slot takes stage i + RS - 1
      if (!conv_sync_and(w_ok)) { ok = false; break; }
      if (!WX && i + C::RS - 1 < nst) issue_b(ks0 + i + C::RS - 1, (i + C::RS - 1) % C::RS);
      cp_async_commit();
      if (xs) {  // weights only, every converter thread: a chunk each, and the
        // chunks past the threads (a gate/up pair: 32) one word each over as many threads
        if (!WX) {
          if (tid < NM * 256) store_chunk(st + 2 * C::XB, i % C::RS, tid);
          constexpr int kXsRem = NM * 256 - kConv;
          if (kXsRem > 0 && tid < 4 * kXsRem)
            store_word(st + 2 * C::XB, i % C::RS, kConv + tid % (kXsRem > 0 ? kXsRem : 1),
                       tid / (kXsRem > 0 ? kXsRem : 1));
        }
      } else if (a_thr) {
        store_a(ks0 + i, ac, st, st + C::XB);
        if (!WX && at < 4 * kChunksRem) store_word(st + 2 * C::XB, i % C::RS, kBConv * NM + at % kChunksRem, at / kChunksRem);
      } else if (!WX && tid < kBConv) {
#pragma unroll
        for (int j = 0; j < NM; ++j) store_chunk(st + 2 * C::XB, i % C::RS, tid + j * kBConv);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // st.shared -> visible to tcgen05.mma
      mbar_arrive(&full[b]);
    }
  } else if (warp == kMmaWarp) {
    // ---- MMA issue
    for (int i = 0; i < nst; ++i) {
      const int b = i % C::STAGES;
      bool f_ok = mbar_wait(&full[b], (unsigned)(i / C::STAGES) & 1u);
      if ((WX || xs) && f_ok) f_ok = mbar_wait(&wfull[b], (unsigned)(i / C::STAGES) & 1u);
      if (!__all_sync(0xffffffffu, f_ok)) { ok = false; break; }
      if (lane == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t xhi = tsm_a + b * C::STAGE_BYTES, xlo = xhi + C::XB;  // input rows (MMA operand B)
#pragma unroll
        for (int a = 0; a < NM; ++a) {
          // weights (MMA operand A)
          const uint32_t whi = xhi + 2 * C::XB + a * B_BYTES, wlo = xhi + 2 * C::XB + (NM + a) * B_BYTES;
          const uint32_t dm = tmem + (uint32_t)(a * 2 * TN), dc = dm + TN;
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk) {
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            umma(dm, sdesc(whi + kk * 256), sdesc(xhi + kk * 256), idesc, acc);
            umma(dc, sdesc(wlo + kk * 256), sdesc(xhi + kk * 256), idesc, acc);
            umma(dc, sdesc(whi + kk * 256), sdesc(xlo + kk * 256), idesc, 1u);
          }
        }
        umma_commit(&mma_done[b]);
      }
      __syncwarp();
    }
    // the commit tracks every earlier tcgen05.mma of this thread
    if (lane == 0) umma_commit(fin);
  }
  cp_async_wait<0>();  // no copy may land after the ring is reused for staging
  if ((WX || xs) && tid == 0) {  // nor a weight (or split-row) copy (bounded; all have landed unless a wait timed out)
    for (int j = max(0, w_issued - C::STAGES); j < w_issued; ++j)
      if (!mbar_wait(&wfull[j % C::STAGES], (unsigned)(j / C::STAGES) & 1u)) atomicOr(s_flag, (unsigned)kErrTimeout);
  }
  pdl_launch_dependents();
  __syncthreads();
  const bool fin_ok = mbar_wait(fin, 0);
  if (amax > 65504.0f) atomicOr(s_flag, (unsigned)kErrFp16Range);
  if (!ok || !fin_ok) atomicOr(s_flag, (unsigned)kErrTimeout);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  const bool good = (*s_flag & kErrTimeout) == 0;

  // ---- accumulators -> shared staging.  TMEM lane = column of the tile,
  // TMEM column = input row.  Warp: lane quarter w % 4 (columns), 32-row block
  // w / 4; a store instruction writes 32 consecutive columns of one row.
  {
    const int lq = warp & 3, rb = warp >> 2;
    if (good && rb * 32 < Mv) {
      const int c = tc_col(lq * 32 + lane);
#pragma unroll
      for (int a = 0; a < NM; ++a) {
        float vm[32], vc[32];
        const uint32_t ta = tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(a * 2 * TN + rb * 32);
        tmem_ld32(ta, vm);
        tmem_ld32(ta + TN, vc);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float* dst = red + ((size_t)a * TM + rb * 32) * kRedLd + c;
#pragma unroll
        for (int j = 0; j < 32; ++j) dst[(size_t)j * kRedLd] = vm[j] + vc[j] * kLoUnscale;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  if (tid == 0 && *s_flag && d.err_flag) atomicOr(d.err_flag, (int)*s_flag);

  cluster_sync_all();  // every K slice's staging is complete

  // ---- this CTA's slice of rows: sum the S partials over the cluster, then
  // the epilogue with one warp per row
  const int S = (int)gridDim.y;
  const uint32_t rank = cluster_rank();
  const int R = (Mv + S - 1) / S;
  const int rb = (int)rank * R, re = min(Mv, rb + R);
  const EpiDesc& e = d.epi;
  const int cc = lane * 4;    // this lane's 4 columns within the tile
  const int col = tcol + cc;  // column within the matrix
  const bool cval = col < n;  // n % 32 == 0: all 4 valid or none
  // Pass 1: the sums go into this CTA's own staging rows [rb, re), which no
  // peer reads (each reads only the rows of its own slice).
  for (int r = rb + warp; good && r < re; r += kThreads / 32) {
#pragma unroll
    for (int a = 0; a < NM; ++a) {
      float* row = red + ((size_t)a * TM + r) * kRedLd + cc;
      const uint32_t la = smem_u32(row);
      float4 part[kMaxSplits];
#pragma unroll
      for (int p = 0; p < kMaxSplits; ++p)  // all loads in flight before the ordered sum
        if (p < S) part[p] = ld_dsmem4(dsmem_addr(la, (uint32_t)p));
      float4 t4 = part[0];
#pragma unroll
      for (int p = 1; p < kMaxSplits; ++p)
        if (p < S) {
          t4.x += part[p].x; t4.y += part[p].y; t4.z += part[p].z; t4.w += part[p].w;
        }
      *reinterpret_cast<float4*>(row) = t4;
    }
  }
  // This CTA's reads of its peers' staging are done: arrive now and wait at
  // the very end, so the barrier's latency overlaps the epilogue.
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  // Pass 2: the epilogue, one warp per row (the warp that summed the row).
  if (EPI == EPI_QKV && good) {
    // q / k / v: mat 0 = q, 1 = k, 2 = v; the tile is head tcol / 128.  The
    // rows' positions and KV pages are loaded up front (lane j: the warp's
    // j-th row), and the RoPE factors of the next row while this one is
    // processed, so the chain of dependent loads is paid about once per warp.
    const int h = tcol / kHeadDim, half = kHeadDim / 2;
    const int nrw = re > rb + warp ? (re - rb - warp + 15) / 16 : 0;  // this warp's rows (<= 8)
    int p_sess = 0, p_pos = 0, p_kvp = 0, p_page = 0;
    if (lane < nrw) {
      row_pos(e.rp, m0 + rb + warp + 16 * lane, p_sess, p_pos, p_kvp);
      p_page = (mat == 2 || mat == 1) ? kv_page(e.kv, p_sess, p_kvp) : 0;
    }
    float gv[4] = {0.f, 0.f, 0.f, 0.f};
    if (mat != 2) {
      const __half* gn = (mat == 0) ? e.q_norm : e.k_norm;
#pragma unroll
      for (int j = 0; j < 4; ++j) gv[j] = h2f(gn[cc + j]);
    }
    auto rope_ld = [&](int pos, float4& c4, float4& s4) {
      if (mat != 2 && pos < e.rope_rows && pos >= 0) {
        c4 = __ldg(reinterpret_cast<const float4*>(e.rope_cos + (size_t)pos * half + (cc % half)));
        s4 = __ldg(reinterpret_cast<const float4*>(e.rope_sin + (size_t)pos * half + (cc % half)));
      }
    };
    float4 cn = make_float4(0.f, 0.f, 0.f, 0.f), sn4 = cn;
    if (nrw > 0) rope_ld(__shfl_sync(0xffffffffu, p_pos, 0), cn, sn4);
    for (int jr = 0; jr < nrw; ++jr) {
      const int r = rb + warp + 16 * jr, m = m0 + r;
      const int pos = __shfl_sync(0xffffffffu, p_pos, jr), kvp = __shfl_sync(0xffffffffu, p_kvp, jr);
      const int page = __shfl_sync(0xffffffffu, p_page, jr);
      const float4 c4 = cn, s4 = sn4;
      if (jr + 1 < nrw) rope_ld(__shfl_sync(0xffffffffu, p_pos, jr + 1), cn, sn4);
      const float4 acc0 = *reinterpret_cast<const float4*>(red + (size_t)r * kRedLd + cc);
      if (mat == 2) {
        kv_store4(e.kv, kv_elem(e.kv, page, kvp, 1, h) + cc, acc0);
        continue;
      }
      const float vv[4] = {acc0.x, acc0.y, acc0.z, acc0.w};
      const float ss = warp_sum((vv[0] * vv[0] + vv[1] * vv[1]) + (vv[2] * vv[2] + vv[3] * vv[3]));
      const float inv = 1.0f / sqrtf(ss / (float)kHeadDim + 1e-6f);  // talker.rs:89-99
      float y[4], pr[4], o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = vv[j] * inv * gv[j];
#pragma unroll
      for (int j = 0; j < 4; ++j) pr[j] = __shfl_xor_sync(0xffffffffu, y[j], 16);  // column +- 64
      const bool in_range = pos < e.rope_rows && pos >= 0;
      const float cf[4] = {c4.x, c4.y, c4.z, c4.w}, sf[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {  // split-half RoPE (rope.rs:79-92)
        const int dd = cc + j;
        const float x1 = dd < half ? y[j] : pr[j];
        const float x2 = dd < half ? pr[j] : y[j];
        o[j] = y[j];
        if (in_range) o[j] = (dd < half) ? (x1 * cf[j] - x2 * sf[j]) : (x2 * cf[j] + x1 * sf[j]);
      }
      if (!in_range && !e.rope_skip_oob && e.err_flag && lane == 0) atomicOr(e.err_flag, kErrRopeRange);
      if (mat == 0)
        *reinterpret_cast<float4*>(e.q_out + (size_t)m * e.ldq + col) = make_float4(o[0], o[1], o[2], o[3]);
      else
        kv_store4(e.kv, kv_elem(e.kv, page, kvp, 0, h) + cc, make_float4(o[0], o[1], o[2], o[3]));
    }
  }
  for (int r = rb + warp; EPI != EPI_QKV && good && r < re; r += kThreads / 32) {
    float4 acc[NM];
#pragma unroll
    for (int a = 0; a < NM; ++a) acc[a] = *reinterpret_cast<const float4*>(red + ((size_t)a * TM + r) * kRedLd + cc);
    const int m = m0 + r;
    if (EPI == EPI_STORE || EPI == EPI_RESID) {
      float vv[4] = {acc[0].x, acc[0].y, acc[0].z, acc[0].w};
      const int cgl = d.col0[mat] + col;
      if (cval) {
        float* o = e.out + (size_t)m * e.ldo + cgl;
        if (EPI == EPI_STORE) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (e.bias) vv[j] = vv[j] + e.bias[cgl + j];
            if ((e.act_silu >> mat) & 1) vv[j] = silu_ref(vv[j]);
          }
        } else {
          const float4 ov = *reinterpret_cast<const float4*>(o);
          vv[0] = ov.x + vv[0]; vv[1] = ov.y + vv[1]; vv[2] = ov.z + vv[2]; vv[3] = ov.w + vv[3];
        }
        *reinterpret_cast<float4*>(o) = make_float4(vv[0], vv[1], vv[2], vv[3]);
      }
      if (e.ssq_out) {
        const float ss = warp_sum(cval ? (vv[0] * vv[0] + vv[1] * vv[1]) + (vv[2] * vv[2] + vv[3] * vv[3]) : 0.0f);
        if (lane == 0) e.ssq_out[(size_t)m * e.ssq_ld + tcol / kSsqCols] = ss;
      }
    } else if (EPI == EPI_SWIGLU) {
      if (cval) {
        const float g[4] = {acc[0].x, acc[0].y, acc[0].z, acc[0].w};
        const float u[4] = {acc[NM - 1].x, acc[NM - 1].y, acc[NM - 1].z, acc[NM - 1].w};
        const float4 hv =
            make_float4(silu_ref(g[0]) * u[0], silu_ref(g[1]) * u[1], silu_ref(g[2]) * u[2], silu_ref(g[3]) * u[3]);
        *reinterpret_cast<float4*>(e.out + (size_t)m * e.ldo + col) = hv;
        if (d.xs_out) {  // the down projection's input rows, split for its tensor-core kernel
          xs_store4(d.xs_out, d.xs_out_k, m, col, hv);
          if (fp16_overflow4(hv) && d.err_flag) atomicOr(d.err_flag, kErrFp16Range);
        }
      }
    } else if (EPI == EPI_ARGMAX) {
      const float vv[4] = {acc[0].x, acc[0].y, acc[0].z, acc[0].w};
      unsigned long long key = 0ull;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const unsigned long long kj = cval ? (((unsigned long long)f32_order_key(vv[j]) << 32) | (unsigned)(col + j)) : 0ull;
        key = kj > key ? kj : key;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (lane == 0) atomicMax(e.keys + m, key);
    }
  }
  // peers keep their staging until every CTA has read its slice
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (EPI == EPI_ARGMAX) {
    __shared__ unsigned s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned total = (unsigned)(((n + TN - 1) / TN) * S);  // CTAs of this row block
      s_last = atomicAdd(e.counters2 + mb, 1u) == total - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      for (int r = tid; r < Mv; r += kThreads) argmax_finalize_row(e, fc, m0 + r);
      if (tid == 0) e.counters2[mb] = 0u;
    }
  }
}

// ---------------------------------------------------------------------------
size_t tc_smem_bytes(int nm) { return nm == 2 ? (size_t)TcCfg<2>::SMEM : (size_t)TcCfg<1>::SMEM; }

int tc_splits(const GemvDesc& d) { return ((d.k + TK - 1) / TK + d.tc_ks - 1) / d.tc_ks; }

// K slices: the largest S (at most a portable cluster of 8, at most the
// 64-deep stages there are) whose clusters (one per tile and row block) are
// all resident in one wave; S = 1 always is.
void tc_plan(int sm_count, GemvDesc& g) {
  const long nks = (g.k + TK - 1) / TK;
  long tiles = 0;
  if (g.paired) {
    tiles = (g.mat[0].n + TN - 1) / TN;
  } else {
    for (int i = 0; i < g.nmat; ++i) tiles += (g.mat[i].n + TN - 1) / TN;
  }
  const long units = tiles * ((g.M + TM - 1) / TM);
  g.tc = 1;
  g.tc_ks = (int)nks;
  // Launches of more than 64 rows split K at most 4 ways: their reduction
  // moves twice the rows per slice, and under waves side by side the SMs a
  // launch leaves free go to the other wave (config 5: +1.7%; at 64 rows the
  // full split stays faster, config 4: 9.09k vs 8.05k frames/s with the cap)
  const long smax = g.M > TM / 2 ? 4 : kMaxSplits;
  for (long S = std::min<long>(smax, std::min<long>(nks, std::max<long>(1, sm_count / units))); S > 1; --S) {
    GemvDesc t = g;
    t.tc_ks = (int)((nks + S - 1) / S);
    if (tc_splits(t) != S) continue;
    g_occ_query = true;
    g_occ_clusters = 0;
    launch_tc(t, FrameCodes{}, nullptr);
    g_occ_query = false;
    // the empty half tiles of an odd 128-column count are clusters too
    const long clusters = 2L * g.ntiles * ((g.M + TM - 1) / TM);
    if (g_occ_clusters >= clusters) {
      g.tc_ks = t.tc_ks;
      return;
    }
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Operand and output layouts the kernel's vector and asynchronous accesses
// need (4-byte scale copies: rows of n / 32 scales start 4-byte aligned).
bool tc_layout_ok(const GemvDesc& d) {
  for (int i = 0; i < (d.paired ? 2 : d.nmat); ++i)
    if (d.mat[i].n % 64 || !al16(d.mat[i].packed) || (reinterpret_cast<uintptr_t>(d.mat[i].scales) & 3u)) return false;
  if (!d.emb_idx && (!al16(d.X) || d.ldx % 4 || d.k % 4)) return false;
  const EpiDesc& e = d.epi;
  if (d.epi_kind != EPI_ARGMAX && d.epi_kind != EPI_QKV && (!al16(e.out) || e.ldo % 4)) return false;
  if (d.epi_kind == EPI_QKV && (!al16(e.q_out) || e.ldq % 4 || !al16(e.kv.pool))) return false;
  return true;
}

template <int NM, int EPI, int NP, bool WX = false>
static cudaError_t launch_np(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  const int S = tc_splits(d);
  LaunchOpts o;
  o.pdl = d.pdl != 0;
  o.cluster_y = (unsigned)S;
  const dim3 grid(2 * d.ntiles, S, (d.M + TM - 1) / TM);
  return launch_k(tc_proj_kernel<NM, EPI, NP, WX>, grid, dim3(kThreads), (size_t)TcCfg<NM, WX && NP == 1>::SMEM, st,
                  o, d, fc);
}

// ---------------------------------------------------------------------------
// Input rows split once for a projection whose column tiles would each split
// them again (row blocks of more than 64 rows): block (row block rb of 128
// rows, stage ks of 64) at (rb * nks + ks) * 2 * A_BYTES holds the fp16 hi
// then the fp16 (lo * 2^11) operand half, K-major core matrices, exactly as
// the projection kernel's input-row threads write them: the same RMSNorm
// (1/rms from the producer's sums of squares or over the row, then x * inv *
// gamma pairwise), the same split; rows past M and k past K are zero.
// 512 threads: row r = tid % 128, 16-deep slice tid / 128 of the stage.
__global__ void __launch_bounds__(512) tc_xsplit_kernel(const GemvDesc d, uint8_t* out) {
  __shared__ float s_inv[TM];
  pdl_launch_dependents();
  const int ks = blockIdx.x, rb = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = tid & (TM - 1), akc = tid >> 7;
  const int m = rb * TM + r, kk0 = ks * TK + akc * 16;
  const int nks = (d.k + TK - 1) / TK;
  const bool g16 = d.gamma && kk0 + 16 <= d.k && (reinterpret_cast<uintptr_t>(d.gamma) & 15u) == 0;
  uint4 g4[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  if (g16) {  // norm weights never depend on an earlier kernel: before the wait
    g4[0] = __ldg(reinterpret_cast<const uint4*>(d.gamma + kk0));
    g4[1] = __ldg(reinterpret_cast<const uint4*>(d.gamma + kk0) + 1);
  }
  pdl_wait();
  // every load is issued before the first is used: the row slice, then the
  // producer's sums of squares of the block's rows
  float y[16];
  const bool live = m < d.M;
  if (d.emb_idx) {  // gathered Q4 embedding rows (gemv.rs:393-396), as the STORE prologue reads them
    const uint32_t er = live ? d.emb_idx[(size_t)m * d.emb_idx_stride] : 0u;
    const uint8_t* prow = d.emb.packed + (size_t)er * (d.emb.n / 2);
    const __half* srow = d.emb.scales + (size_t)er * (d.emb.n / 32);
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = (live && kk0 + j < d.k) ? q4_value(prow, srow, kk0 + j) : 0.0f;
  } else {
    const float* xr = d.X + (size_t)(live ? m : 0) * d.ldx + kk0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = (live && kk0 + 4 * q < d.k) ? __ldg(reinterpret_cast<const float4*>(xr) + q)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
      y[4 * q] = v.x; y[4 * q + 1] = v.y; y[4 * q + 2] = v.z; y[4 * q + 3] = v.w;
    }
  }
  if (d.gamma) {
    if (d.ssq_in) {
      if (tid < TM && rb * TM + tid < d.M) s_inv[tid] = inv_rms_from_ssq(d, rb * TM + tid);
    } else {
      for (int rr = warp; rr < TM; rr += 16) {
        if (rb * TM + rr >= d.M) break;
        const float* xr = d.X + (size_t)(rb * TM + rr) * d.ldx;
        float ss = 0.0f;
        for (int i = lane; i < d.k; i += 32) ss += xr[i] * xr[i];
        ss = warp_sum(ss);
        if (lane == 0) s_inv[rr] = 1.0f / sqrtf(ss / (float)d.k + 1e-6f);
      }
    }
    __syncthreads();
    if (live) {
      const float inv = s_inv[r];
      if (g16) {
        const __half2* g2 = reinterpret_cast<const __half2*>(g4);
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // (x * inv) * gamma, pairwise in f32x2 (gemv.rs:414)
          const float2 t = __fmul2_rn(__fmul2_rn(make_float2(y[2 * j], y[2 * j + 1]), make_float2(inv, inv)),
                                      __half22float2(g2[j]));
          y[2 * j] = t.x;
          y[2 * j + 1] = t.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = (kk0 + j < d.k) ? y[j] * inv * h2f(d.gamma[kk0 + j]) : 0.0f;
      }
    }
  }
  if (d.xnorm_out && live) {  // the normed rows the launch also hands on (the codec head's hidden)
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (kk0 + j < d.k) d.xnorm_out[(size_t)m * d.ld_xnorm + kk0 + j] = y[j];
  }
  float amax = 0.0f;
  uint8_t* hi = out + ((size_t)rb * nks + ks) * (2 * A_BYTES);
#pragma unroll
  for (int c = 0; c < 2; ++c) {  // two 8-deep k chunks
    uint32_t h[4], l[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      amax = fmaxf(amax, fmaxf(fabsf(y[c * 8 + 2 * q]), fabsf(y[c * 8 + 2 * q + 1])));
      split2(y[c * 8 + 2 * q], y[c * 8 + 2 * q + 1], h[q], l[q]);
    }
    const int off = (r >> 3) * 1024 + (akc * 2 + c) * 128 + (r & 7) * 16;
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(hi + A_BYTES + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
  if (amax > 65504.0f && d.err_flag) atomicOr(d.err_flag, kErrFp16Range);
}

// Bytes of split tiles a launch of M rows over K needs.
static size_t tc_xsplit_bytes(int M, int k) {
  return (size_t)((M + TM - 1) / TM) * ((k + TK - 1) / TK) * (2 * A_BYTES);
}
size_t tc_xsplit_scratch_bytes(int M, int k) { return tc_xsplit_bytes(M, k); }

// Whether a planned launch runs the tensor-core instance that reads split
// input rows (the branch of launch_t below): its producer may then write
// them directly.
bool tc_takes_split(const GemvDesc& d) {
  // gathered embedding rows: the STORE launches without a norm (input_proj);
  // normed rows handed on: the STORE launches that keep them (codec head)
  const bool emb = d.emb_idx != nullptr;
  if (emb && (d.epi_kind != EPI_STORE || d.gamma || d.xnorm_out)) return false;
  if (d.xnorm_out && (d.epi_kind != EPI_STORE || !d.gamma)) return false;
  if (!d.tc || !d.xs_buf || (!emb && !d.X) || d.M <= TM / 2 || (reinterpret_cast<uintptr_t>(d.xs_buf) & 15u))
    return false;
  return tc_xsplit_bytes(d.M, d.k) <= d.xs_bytes;
}

// Whether the producer of a planned launch's input rows (attention, the
// gate/up epilogue) may write them split for it: as tc_takes_split, and at
// any row count, since no extra launch is involved (config 4, 64 rows: o and
// down then bulk-copy their rows instead of splitting them in the K loop,
// 9.14k -> 9.21k frames/s).
bool tc_takes_split_from_producer(const GemvDesc& d) {
  if (!d.tc || !d.xs_buf || d.emb_idx || d.xnorm_out || !d.X || (reinterpret_cast<uintptr_t>(d.xs_buf) & 15u))
    return false;
  return tc_xsplit_bytes(d.M, d.k) <= d.xs_bytes;
}

// Whether a tensor-core launch of `d` streams the expanded weight tiles (the
// choice launch_t makes below): every matrix expanded, and a row block of at
// most 64 rows, split input rows, or at most 128 rows.
bool tc_reads_expanded(const GemvDesc& d) {
  if (!d.tc) return false;
  for (int i = 0; i < (d.paired ? 2 : d.nmat); ++i)
    if (!d.mat[i].wx) return false;
  return d.M <= TM || d.x_split_pre != nullptr || tc_takes_split(d);
}

template <int NM, int EPI>
static cudaError_t launch_t(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  // Row blocks of more than 64 rows take their input rows split once per
  // projection (or by their producer) whenever the session's scratch holds
  // them: the instance with 128-row operand halves then dequantises weights
  // with every converter warp (at 128 rows this beat the expanded tiles by
  // 12-16%; at 64 rows the expanded tiles win).  Row blocks of at most 64 rows
  // run the instance compiled for one input-row pass; with every matrix
  // expanded (tc_expand), the one fed by bulk copies.
  bool wx = true;
  for (int i = 0; i < (NM == 2 ? 2 : d.nmat); ++i) wx = wx && d.mat[i].wx != nullptr;
  if (d.x_split_pre) {  // the producer of the input rows wrote them split
    GemvDesc e = d;
    e.x_split = d.x_split_pre;
    return wx ? launch_np<NM, EPI, 2, true>(e, fc, st) : launch_np<NM, EPI, 2>(e, fc, st);
  }
  if (tc_takes_split(d)) {
    GemvDesc e = d;
    e.x_split = d.xs_buf;
    if (!g_occ_query) {
      const dim3 grid((d.k + TK - 1) / TK, (d.M + TM - 1) / TM);
      LaunchOpts o;
      o.pdl = d.pdl != 0;
      const cudaError_t err = launch_k(tc_xsplit_kernel, grid, dim3(512), 0, st, o, d, d.xs_buf);
      if (err != cudaSuccess) return err;
    }
    return wx ? launch_np<NM, EPI, 2, true>(e, fc, st) : launch_np<NM, EPI, 2>(e, fc, st);
  }
  if (d.M <= TM / 2) {
    if (wx) return launch_np<NM, EPI, 1, true>(d, fc, st);
    return launch_np<NM, EPI, 1>(d, fc, st);
  }
  if (wx && d.M <= TM) return launch_np<NM, EPI, 2, true>(d, fc, st);
  return launch_np<NM, EPI, 2>(d, fc, st);
}

cudaError_t launch_tc(const GemvDesc& d, const FrameCodes& fc, cudaStream_t st) {
  if (d.tc_ks <= 0 || d.M <= 0 || d.k <= 0 || tc_splits(d) > kMaxSplits) return cudaErrorInvalidValue;
  if (!tc_layout_ok(d)) return cudaErrorMisalignedAddress;
  if (d.epi_kind != EPI_STORE && (d.emb_idx || d.xnorm_out)) return cudaErrorInvalidValue;
  if (d.epi_kind == EPI_ARGMAX && (d.M + TM - 1) / TM > 4096) return cudaErrorInvalidValue;
  if (d.paired) return d.epi_kind == EPI_SWIGLU ? launch_t<2, EPI_SWIGLU>(d, fc, st) : cudaErrorInvalidValue;
  switch (d.epi_kind) {
    case EPI_STORE: return launch_t<1, EPI_STORE>(d, fc, st);
    case EPI_RESID: return launch_t<1, EPI_RESID>(d, fc, st);
    case EPI_QKV: return launch_t<1, EPI_QKV>(d, fc, st);
    case EPI_ARGMAX: return launch_t<1, EPI_ARGMAX>(d, fc, st);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// Weight expansion for the WX instances: block (tile t of 128 columns, stage
// ks of 64 rows) at ((t * nks) + ks) * 32 KB holds the 16 KB hi then 16 KB lo
// fp16 operand tiles exactly as store_chunk writes them (rows past k and
// columns past n zero); a thread per 16-byte packed chunk.
__global__ void tc_expand_kernel(const Q4Mat w, uint8_t* out) {
  const int nt = (w.n + TN - 1) / TN, nks = (w.k + TK - 1) / TK;
  const size_t nchunks = (size_t)nt * nks * 256;
  for (size_t c = (size_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunks; c += (size_t)gridDim.x * blockDim.x) {
    const int q = (int)(c & 255);
    const size_t blk = c >> 8;
    const int ks = (int)(blk % nks), t = (int)(blk / nks);
    const int ch = (q >> 6) & 3, brow = q & 63;
    const int row = ks * TK + brow, col = t * TN + ch * 32;
    uint4 w4 = make_uint4(0, 0, 0, 0);
    unsigned short sc = 0;
    if (row < w.k && col < w.n) {
      w4 = *reinterpret_cast<const uint4*>(w.packed + (size_t)row * (w.n / 2) + col / 2);
      sc = reinterpret_cast<const unsigned short*>(w.scales)[(size_t)row * (w.n / 32) + col / 32];
    }
    const __half2 s2 = __half2half2(__ushort_as_half(sc));
    uint8_t* dst = out + blk * (2 * B_BYTES) + ch * 4096 + (brow >> 3) * 128 + (brow & 7) * 16;
    const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint4 hi, lo;
      dequant_word(wv[k], s2, hi, lo);
      *reinterpret_cast<uint4*>(dst + k * 1024) = hi;
      *reinterpret_cast<uint4*>(dst + B_BYTES + k * 1024) = lo;
    }
  }
}

// The same expansion from f32 weights w[k][ld] (columns col0 .. col0 + n):
// hi = fp16(w), lo = fp16((w - hi) * 2^11).  Unlike the Q4 values this split
// is not exact: it keeps ~22 of the 24 significand bits (|w| < 65504).  A
// thread per row and 8-column group of a block.
__global__ void tc_expand_f32_kernel(const float* w, int k, int n, long ld, int col0, uint8_t* out) {
  const int nt = (n + TN - 1) / TN, nks = (k + TK - 1) / TK;
  const size_t items = (size_t)nt * nks * TK * (TN / 8);
  for (size_t c = (size_t)blockIdx.x * blockDim.x + threadIdx.x; c < items; c += (size_t)gridDim.x * blockDim.x) {
    const int g8 = (int)(c % (TN / 8));
    const int brow = (int)((c / (TN / 8)) % TK);
    const size_t blk = c / ((size_t)(TN / 8) * TK);
    const int ks = (int)(blk % nks), t = (int)(blk / nks);
    const int row = ks * TK + brow, cb = t * TN + g8 * 8;
    uint32_t h[4], l[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {  // half2 p holds columns p and p + 4 of the group
      float v[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int col = cb + p + 4 * q;
        v[q] = (row < k && col < n) ? w[(size_t)row * ld + col0 + col] : 0.0f;
      }
      const __half2 hh = __floats2half2_rn(v[0], v[1]);
      const float2 hf = __half22float2(hh);
      h[p] = h2_bits(hh);
      l[p] = h2_bits(__floats2half2_rn((v[0] - hf.x) * kLoScale, (v[1] - hf.y) * kLoScale));
    }
    uint8_t* dst = out + blk * (2 * B_BYTES) + g8 * 1024 + (brow >> 3) * 128 + (brow & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(dst + B_BYTES) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

cudaError_t tc_expand_f32(const float* w, int k, int n, long ld, int col0, uint8_t* out, cudaStream_t st) {
  if (!w || !out || k <= 0 || n <= 0 || n % 64 || !al16(out)) return cudaErrorInvalidValue;
  const size_t items = (size_t)((n + TN - 1) / TN) * ((k + TK - 1) / TK) * TK * (TN / 8);
  const unsigned grid = (unsigned)std::min<size_t>((items + 255) / 256, 148 * 8);
  tc_expand_f32_kernel<<<grid, 256, 0, st>>>(w, k, n, ld, col0, out);
  return cudaGetLastError();
}

size_t tc_expand_bytes(int k, int n) {
  return (size_t)((n + TN - 1) / TN) * ((k + TK - 1) / TK) * (2 * B_BYTES);
}

cudaError_t tc_expand(const Q4Mat& w, uint8_t* out, cudaStream_t st) {
  if (!w.packed || !w.scales || !out || w.k <= 0 || w.n <= 0 || w.n % 64 || !al16(w.packed) || !al16(out))
    return cudaErrorInvalidValue;
  const size_t nchunks = tc_expand_bytes(w.k, w.n) / (2 * B_BYTES) * 256;
  const unsigned grid = (unsigned)std::min<size_t>((nchunks + 255) / 256, 148 * 8);
  tc_expand_kernel<<<grid, 256, 0, st>>>(w, out);
  return cudaGetLastError();
}

// Opt the kernels into their dynamic shared memory once per device (outside
// any stream capture).
void tc_init_attributes() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_STORE, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_STORE, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_RESID, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_RESID, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_QKV, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_QKV, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_ARGMAX, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_ARGMAX, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<2, EPI_SWIGLU, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<2>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<2, EPI_SWIGLU, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<2>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_STORE, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_RESID, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_QKV, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_ARGMAX, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<2, EPI_SWIGLU, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<2>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_STORE, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_RESID, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_QKV, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<1, EPI_ARGMAX, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<1>::SMEM);
  cudaFuncSetAttribute(tc_proj_kernel<2, EPI_SWIGLU, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<2>::SMEM);
  cudaGetLastError();
  done[dev] = true;
}

}  // namespace qtts
