// common.cuh -- device helpers shared by the QORA-TTS sm_100a kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace qtts {

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }  // exact (half::to_f32)

// Programmatic dependent launch: let the next kernel in the stream launch now;
// wait until the previous kernel has completed and its writes are visible.
// Both are no-ops for kernels launched without the PDL attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 16-byte read-only streaming load (weights are read once per frame).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Q4 group-32 accumulate of one 32-bit word (8 columns, low nibble first as
// gemv.rs:124/254).  A nibble q sitting at bit 4p (p <= 4) is turned into the
// exact float 2^23 + q*2^(4p) by OR-ing the exponent of 2^23 onto it; one
// subtraction of 2^23 + 8*2^(4p) then yields (q-8)*2^(4p) exactly, and the
// pre-scaled multiplier sx*2^(-4p) restores (q-8)*sx in the FMA.  Nibbles 5..7
// are read from w >> 12.  Pairs of columns go through the sm_100 f32x2 FMA.
struct SxPack {
  float2 a, b, c, d;  // multipliers for column pairs (0,1) (2,3) (4,5) (6,7)
};
__device__ __forceinline__ SxPack make_sx(float sx) {
  const float s0 = sx, s1 = sx * 0.0625f, s2 = sx * 0.00390625f, s3 = sx * 0.000244140625f,
              s4 = sx * 1.52587890625e-05f;
  SxPack p;
  p.a = make_float2(s0, s1);  // nibbles 0,1 at p = 0,1
  p.b = make_float2(s2, s3);  // nibbles 2,3 at p = 2,3
  p.c = make_float2(s4, s2);  // nibble 4 at p = 4, nibble 5 at p = 2 of w>>12
  p.d = make_float2(s3, s4);  // nibbles 6,7 at p = 3,4 of w>>12
  return p;
}
__device__ __forceinline__ float magic_nib(uint32_t w, uint32_t mask) {
  return __uint_as_float((w & mask) | 0x4B000000u);
}
__device__ __forceinline__ void q4_word_fma(uint32_t w, const SxPack& s, float2* acc) {
  const uint32_t h = w >> 12;
  const float2 C01 = make_float2(-8388616.0f, -8388736.0f);
  const float2 C23 = make_float2(-8390656.0f, -8421376.0f);
  const float2 C42 = make_float2(-8912896.0f, -8390656.0f);
  const float2 C34 = make_float2(-8421376.0f, -8912896.0f);
  float2 d0 = __fadd2_rn(make_float2(magic_nib(w, 0xFu), magic_nib(w, 0xF0u)), C01);
  float2 d1 = __fadd2_rn(make_float2(magic_nib(w, 0xF00u), magic_nib(w, 0xF000u)), C23);
  float2 d2 = __fadd2_rn(make_float2(magic_nib(w, 0xF0000u), magic_nib(h, 0xF00u)), C42);
  float2 d3 = __fadd2_rn(make_float2(magic_nib(h, 0xF000u), magic_nib(h, 0xF0000u)), C34);
  acc[0] = __ffma2_rn(d0, s.a, acc[0]);
  acc[1] = __ffma2_rn(d1, s.b, acc[1]);
  acc[2] = __ffma2_rn(d2, s.c, acc[2]);
  acc[3] = __ffma2_rn(d3, s.d, acc[3]);
}

// ---- input rows split for the tensor-core projection ----------------------
// An f32 pair becomes the fp16 pair hi = fp16(x) and the fp16 pair
// lo = fp16((x - hi) * 2^11): x - hi is exact in f32 and so is the scaling,
// and the 2^11 keeps lo clear of the fp16 subnormals (sm_100 f32x2 ops).
constexpr float kSplitLoScale = 2048.0f;
__device__ __forceinline__ uint32_t half2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// ---- paged KV cache elements (KvDesc): f32, or f16 rounded to nearest even
__device__ __forceinline__ int kv_page(const KvDesc& kv, int sess, int pos) {
  return kv.page_table ? kv.page_table[sess * kv.pages_per_sess + pos / kPageSize] : sess;
}
// element index of (page, position, K = 0 / V = 1, kv head), dimension 0
__device__ __forceinline__ size_t kv_elem(const KvDesc& kv, int page, int pos, int which, int h) {
  const size_t blk = (((size_t)page * kv.n_layers + kv.layer) * 2 + which) * kv.kv_heads + h;
  return (blk * kPageSize + (pos % kPageSize)) * kHeadDim;
}
__device__ __forceinline__ size_t kv_at(const KvDesc& kv, int sess, int pos, int which, int h) {
  return kv_elem(kv, kv_page(kv, sess, pos), pos, which, h);
}
// (`f16` = kv.f16, or a constant in kernels specialised on the element type)
__device__ __forceinline__ const void* kv_addr(const KvDesc& kv, size_t i, bool f16) {
  return f16 ? static_cast<const void*>(reinterpret_cast<const __half*>(kv.pool) + i)
             : static_cast<const void*>(kv.pool + i);
}
__device__ __forceinline__ void kv_store1(const KvDesc& kv, size_t i, float v) {
  if (kv.f16) reinterpret_cast<__half*>(kv.pool)[i] = __float2half_rn(v);
  else kv.pool[i] = v;
}
__device__ __forceinline__ float kv_load1(const KvDesc& kv, size_t i) {
  return kv.f16 ? __half2float(reinterpret_cast<const __half*>(kv.pool)[i]) : kv.pool[i];
}
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  hi = half2_bits(h);
  const float2 r = __fmul2_rn(__ffma2_rn(hf, make_float2(-1.0f, -1.0f), make_float2(a, b)),
                              make_float2(kSplitLoScale, kSplitLoScale));
  lo = half2_bits(__floats2half2_rn(r.x, r.y));
}
// four consecutive elements (i % 4 == 0)
__device__ __forceinline__ void kv_store4(const KvDesc& kv, size_t i, float4 v) {
  if (kv.f16) {
    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(kv.pool) + i) =
        make_uint2(half2_bits(__floats2half2_rn(v.x, v.y)), half2_bits(__floats2half2_rn(v.z, v.w)));
  } else {
    *reinterpret_cast<float4*>(kv.pool + i) = v;
  }
}
__device__ __forceinline__ float4 kv_load4(const KvDesc& kv, size_t i, bool f16) {
  if (f16) {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(kv.pool) + i);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  return *reinterpret_cast<const float4*>(kv.pool + i);
}
__device__ __forceinline__ float4 kv_load4(const KvDesc& kv, size_t i) { return kv_load4(kv, i, kv.f16 != 0); }
// Split tiles of a projection's input rows (K wide): block (row m / 128,
// column c / 64) of 32 KB holds the hi half then the lo half, each K-major
// core matrices of 8 rows x 16 bytes, row r and column j of the block at
// (r / 8) * 1024 + (j / 8) * 128 + (r % 8) * 16 + (j % 8) * 2.
constexpr int kXsRows = 128, kXsK = 64, kXsHalf = kXsRows * kXsK * 2;
// Row m, columns c..c+3 (c % 4 == 0) of value v; the producer of a row
// writes all of its K columns.
__device__ __forceinline__ void xs_store4(uint8_t* buf, int K, int m, int c, float4 v) {
  const int nks = (K + kXsK - 1) / kXsK, r = m & (kXsRows - 1), j = c & (kXsK - 1);
  uint8_t* p = buf + ((size_t)(m / kXsRows) * nks + c / kXsK) * (2 * kXsHalf) + (r >> 3) * 1024 + (j >> 3) * 128 +
               (r & 7) * 16 + (j & 7) * 2;
  uint32_t h0, l0, h1, l1;
  split_pair(v.x, v.y, h0, l0);
  split_pair(v.z, v.w, h1, l1);
  *reinterpret_cast<uint2*>(p) = make_uint2(h0, h1);
  *reinterpret_cast<uint2*>(p + kXsHalf) = make_uint2(l0, l1);
}
// One element (row m, column c) of the same tiles, split as split_pair does.
__device__ __forceinline__ void xs_store1(uint8_t* buf, int K, int m, int c, float v) {
  const int nks = (K + kXsK - 1) / kXsK, r = m & (kXsRows - 1), j = c & (kXsK - 1);
  uint8_t* p = buf + ((size_t)(m / kXsRows) * nks + c / kXsK) * (2 * kXsHalf) + (r >> 3) * 1024 + (j >> 3) * 128 +
               (r & 7) * 16 + (j & 7) * 2;
  const __half h = __float2half_rn(v);
  *reinterpret_cast<__half*>(p) = h;
  *reinterpret_cast<__half*>(p + kXsHalf) = __float2half_rn(__fmul_rn(__fsub_rn(v, __half2float(h)), kSplitLoScale));
}
__device__ __forceinline__ bool fp16_overflow4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))) > 65504.0f;
}

// Dequantised value of column j of a Q4 row (gemv.rs:393-396): f32(scale)*(q-8).
__device__ __forceinline__ float q4_value(const uint8_t* packed_row, const __half* scales_row, int j) {
  const uint8_t b = packed_row[j >> 1];
  const int q = (j & 1) ? (b >> 4) : (b & 0xF);
  return h2f(scales_row[j >> 5]) * (float)(q - 8);
}

// SiLU exactly as gemv.rs:449-451 writes it (x / (1 + exp(-x))).
__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// Orderable 32-bit key of an f32 (total order of non-NaN values).  -0.0 is
// first turned into +0.0 (x + 0 rounds -0 to +0), so the two zeros share a
// key as they compare equal under partial_cmp (code_predictor.rs:328-334).
__device__ __forceinline__ uint32_t f32_order_key(float f) {
  uint32_t u = __float_as_uint(__fadd_rn(f, 0.0f));
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// expf with glibc's bits.  Rust's f32::exp calls the platform libm; on the
// x86-64 hosts of this image glibc (2.28+) resolves expf to its FMA variant of
// the ARM optimized-routines method: x*N/ln2 = k + r (N = 32), 2^(k/N) from a
// 32-entry table, 2^(r/N) from a cubic, all in double, with the multiply
// x*N/ln2 contracted into both its uses.  This restatement reproduces that
// evaluation order with explicit round-to-nearest double ops; it was checked
// bit-for-bit against the host expf on every float in [-110, 90].
// Table entries: bits of the correctly rounded 2^(i/32) minus (i << 47).
// Method, table layout and polynomial coefficients: the expf of ARM's
// optimized-routines project (licence: MIT OR Apache-2.0 WITH
// LLVM-exception), the code glibc imported for its expf; the values here
// were recomputed (exp2l) and the steps restated from that published method.
__device__ __constant__ uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

__device__ __forceinline__ float expf_glibc(float x) {
  const uint32_t ux = __float_as_uint(x);
  const uint32_t abstop = (ux >> 20) & 0x7ff;
  if (abstop >= 0x42b) {  // |x| >= 88 (top 12 bits of 88.0f) or nan
    if (ux == 0xff800000u) return 0.0f;
    if (abstop >= 0x7f8) return x + x;
    if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
    if (x < -0x1.9fe368p6f) return 0.0f;
  }
  const double InvLn2N = 0x1.71547652b82fep+0 * 32.0;
  const double Shift = 0x1.8p+52;
  const double C0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0;
  const double C1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0;
  const double C2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double xd = (double)x;
  double kd = __fma_rn(InvLn2N, xd, Shift);
  const uint64_t ki = (uint64_t)__double_as_longlong(kd);
  kd = __dsub_rn(kd, Shift);
  const double r = __fma_rn(InvLn2N, xd, -kd);
  uint64_t t = kExp2Tab[ki % 32];
  t += ki << 47;
  const double s = __longlong_as_double((long long)t);
  const double z = __fma_rn(C0, r, C1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(C2, r, 1.0);
  y = __fma_rn(z, r2, y);
  y = __dmul_rn(y, s);
  return __double2float_rn(y);
}

}  // namespace qtts
