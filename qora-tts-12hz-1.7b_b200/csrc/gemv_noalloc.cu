// gemv_noalloc.cu -- the Q4 GEMV entry point that allocates nothing.
//
// qtts_q4_gemv_dev needs a caller-provided scratch buffer for its split-K
// partial sums.  Callers that cannot allocate device memory (a real-time
// audio thread that may not block inside a driver allocation, or a process
// whose GPU memory belongs to another framework's caching allocator) call
// qtts_q4_gemv_dev_noalloc instead: the same kernel and split plan, with the
// scratch taken from the static device array below.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "engine.h"

namespace qtts {

void choose_split(int sm_count, GemvDesc& g);
void gemv_init_attributes();

namespace {

constexpr size_t kNoallocBytes = QTTS_Q4_GEMV_NOALLOC_SCRATCH_BYTES;  // 4 MiB per device
constexpr size_t kNoallocCounterBytes = 16384;                       // 4096 tile counters

// Split-K scratch shared by every call on a device: [tile counters | partial
// sums].  Host code must not use this name as an address: it is a host-side
// stand-in; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

std::mutex g_mu;
void* g_addr[64] = {};  // device address of g_noalloc_scratch, per device
int g_sms[64] = {};

// Once per device, with that device current: resolve the array's device
// address and opt the GEMV kernels into large shared memory.
int noalloc_setup(int dev, void** addr, int* sms) {
  if (dev < 0 || dev >= 64) return fail(QTTS_ERR_NODEV, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(QTTS_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
    gemv_init_attributes();
    g_sms[dev] = n;
    g_addr[dev] = p;
  }
  *addr = g_addr[dev];
  *sms = g_sms[dev];
  return QTTS_OK;
}

}  // namespace
}  // namespace qtts

using namespace qtts;

extern "C" int qtts_q4_gemv_dev_noalloc(const uint8_t* packed, const uint16_t* scales, int k, int n,
                                        const float* x, int m, float* y, void* stream) {
  if (!packed || !scales || !x || !y || k <= 0 || n <= 0 || m <= 0 || n % 32)
    return fail(QTTS_ERR_BADARG, "bad gemv arguments (n must be a multiple of 32)");
  if (reinterpret_cast<uintptr_t>(packed) % 16 || reinterpret_cast<uintptr_t>(scales) % 2 ||
      reinterpret_cast<uintptr_t>(x) % 4 || reinterpret_cast<uintptr_t>(y) % 4)
    return fail(QTTS_ERR_BADARG, "packed must be 16-byte aligned, x/y 4-byte, scales 2-byte");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(QTTS_ERR_NODEV, "no current CUDA device");
  void* base = nullptr;
  int sms = 0;
  const int rc = noalloc_setup(dev, &base, &sms);
  if (rc != QTTS_OK) return rc;

  GemvDesc g;
  g.epi_kind = EPI_STORE;
  g.nmat = 1;
  g.mat[0].packed = packed;
  g.mat[0].scales = reinterpret_cast<const __half*>(scales);
  g.mat[0].k = k;
  g.mat[0].n = n;
  g.ntiles = (n + kTileN - 1) / kTileN;
  g.tile0[1] = g.ntiles;
  g.ncols = n;
  g.k = k;
  g.M = m;
  choose_split(sms, g);
  const size_t zb = (size_t)((m + g.mb - 1) / g.mb);
  const size_t counter_bytes = (size_t)g.ntiles * zb * sizeof(unsigned);
  const size_t part_bytes = g.S > 1 ? sizeof(float) * (size_t)g.S * m * n : 0;
  if (counter_bytes > kNoallocCounterBytes || part_bytes > kNoallocBytes - kNoallocCounterBytes)
    return fail(QTTS_ERR_RANGE, "shape needs " + std::to_string(counter_bytes) + " counter bytes and " +
                                    std::to_string(part_bytes) + " partial-sum bytes; the static scratch holds " +
                                    std::to_string(kNoallocCounterBytes) + " + " +
                                    std::to_string(kNoallocBytes - kNoallocCounterBytes));
  g.counters = reinterpret_cast<unsigned*>(base);
  g.part = reinterpret_cast<float*>(reinterpret_cast<char*>(base) + kNoallocCounterBytes);
  g.X = x;
  g.ldx = k;
  g.epi.out = y;
  g.epi.ldo = n;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the tile counters must start at zero; the partial sums are written before read
  cudaError_t e = cudaMemsetAsync(base, 0, counter_bytes, st);
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  e = launch_gemv(g, FrameCodes{}, st);
  if (e != cudaSuccess) return fail(QTTS_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return QTTS_OK;
}
