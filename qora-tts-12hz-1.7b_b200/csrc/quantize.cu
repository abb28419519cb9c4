// quantize.cu -- f32 -> Q4 g32 quantisation on the GPU (sm_100a).
//
// Replaces quantize_f32_to_q4 (gemv.rs:92-130), the conversion the
// reference's converter applies to every projection before writing the
// .qora-tts file: per group of 32 consecutive columns of a row,
//   absmax = max |v|            (NaN never wins: `v > absmax` is false)
//   scale  = absmax / 7          (f32, correctly rounded), stored as f16 (RNE)
//   inv    = scale > 0 ? 1 / scale : 0   (f32, correctly rounded)
//   q      = clamp(round(v * inv), -8, 7) + 8   (round: half away from zero;
//            NaN -> 0, Rust's saturating `as u8`)
// packed byte j of the group = q[2j] | q[2j+1] << 4 (low nibble = even column).
//
// The rows are contiguous and n % 32 == 0, so the matrix is a flat sequence
// of k*n/32 groups: group g is data[32g, 32g+32), packed[16g, 16g+16),
// scales[g].  HBM-bound: 128 bytes read and 18 written per group.  A warp
// takes 4 groups per 512-byte load (8 lanes x float4 per group) and keeps
// kUnits such loads in flight; the max over a group is 3 xor-shuffles among
// its 8 lanes (max is order-independent, so this equals the sequential scan).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace qtts {

namespace {
constexpr int kQThreads = 256;
constexpr int kUnits = 4;  // 512-byte loads in flight per warp

__device__ __forceinline__ uint32_t q4_code(float v, float inv) {
  float r = roundf(__fmul_rn(v, inv));  // f32 product, no contraction; half away from zero
  if (r != r) return 0u;                // NaN (0 * inf, NaN input): `NaN as u8` is 0
  r = fminf(fmaxf(r, -8.0f), 7.0f);
  return (uint32_t)(int)(r + 8.0f);
}
}  // namespace

__global__ void __launch_bounds__(kQThreads) q4_quantize_kernel(const float* __restrict__ data, size_t ngroups,
                                                                uint8_t* __restrict__ packed,
                                                                uint16_t* __restrict__ scales) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const size_t warp = ((size_t)blockIdx.x * kQThreads + threadIdx.x) >> 5;
  const size_t nwarps = ((size_t)gridDim.x * kQThreads) >> 5;
  const size_t nunits = (ngroups + 3) / 4;
  for (size_t u0 = warp * kUnits; u0 < nunits; u0 += nwarps * kUnits) {
    float4 v[kUnits];
#pragma unroll
    for (int i = 0; i < kUnits; ++i) {  // every load issued before the first is used
      const size_t g = (u0 + i) * 4 + (lane >> 3);
      v[i] = g < ngroups ? __ldcs(reinterpret_cast<const float4*>(data + g * 32) + sub)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kUnits; ++i) {
      const size_t g = (u0 + i) * 4 + (lane >> 3);
      // starting from 0 keeps NaN out of the max (fmaxf returns the non-NaN operand)
      float a = fmaxf(fmaxf(fmaxf(fmaxf(0.0f, fabsf(v[i].x)), fabsf(v[i].y)), fabsf(v[i].z)), fabsf(v[i].w));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
      const float scale = __fdiv_rn(a, 7.0f);
      const float inv = scale > 0.0f ? __frcp_rn(scale) : 0.0f;
      if (g < ngroups) {
        const uint32_t b = q4_code(v[i].x, inv) | (q4_code(v[i].y, inv) << 4) | (q4_code(v[i].z, inv) << 8) |
                           (q4_code(v[i].w, inv) << 12);
        __stcs(reinterpret_cast<unsigned short*>(packed + g * 16) + sub, (unsigned short)b);
        if (sub == 0) __stcs(reinterpret_cast<unsigned short*>(scales) + g, __half_as_ushort(__float2half_rn(scale)));
      }
    }
  }
}

cudaError_t launch_q4_quantize(const float* data, size_t k, size_t n, uint8_t* packed, uint16_t* scales,
                               cudaStream_t st) {
  const size_t ngroups = k * n / 32;
  if (ngroups == 0) return cudaSuccess;
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  int nsm = (dev >= 0 && dev < 64) ? sms[dev] : 0;
  if (nsm == 0) {
    if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || nsm <= 0) nsm = 148;
    if (dev >= 0 && dev < 64) sms[dev] = nsm;
  }
  // one wave of 8 CTAs per SM at most; each warp covers kUnits * 4 groups per pass
  const size_t per_cta = (size_t)(kQThreads / 32) * kUnits * 4;
  const size_t want = (ngroups + per_cta - 1) / per_cta;
  const unsigned grid = (unsigned)std::min<size_t>(want, (size_t)nsm * 8);
  return launch_k(q4_quantize_kernel, dim3(grid), dim3(kQThreads), 0, st, LaunchOpts{true, 1}, data, ngroups, packed,
                  scales);
}

}  // namespace qtts
