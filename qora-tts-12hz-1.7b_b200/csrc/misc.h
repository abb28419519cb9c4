// misc.h -- prefill assembly and gather launchers (misc.cu).
#pragma once
#include "kernels.h"

namespace qtts {

// One prefill row of generate_new.rs:94-173.
struct RowRecipe {
  int codec;  // codec token (talker codec_embedding row) or -1
  int tp;     // text-projection row or -1
  int voice;  // voice embedding index (raw row) or -1
  int pad;
};

cudaError_t launch_assemble(const Q4Mat& codec, const RowRecipe* rec, int rows, const float* tp, long ldtp,
                            const float* voice, long ldv, float* out, long ldo, int H, cudaStream_t st);
cudaError_t launch_gather_rows(const float* src, long lds, const int* idx, int rows, float* out, long ldo, int n,
                               cudaStream_t st);
cudaError_t launch_expf(const float* x, float* y, int n, cudaStream_t st);
cudaError_t launch_dump(const SlotState* slots, int B, const float* src, long lds, int n, float* dst, int max_frames,
                        cudaStream_t st);

}  // namespace qtts
