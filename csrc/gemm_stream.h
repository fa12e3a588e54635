// Persistent stream-K W4A16 GEMM for decode batches (gemm_stream.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace cb {

struct StreamPlan {
  int MT;              // token tile (16, 32 or 64)
  int tpp, kstep;      // row tiles per pair, k-blocks per step
  int pairs, ksteps;   // iteration space: pairs * ksteps steps
  int ctas, ub, ur;    // persistent CTAs; steps per CTA (ub, or ub + 1 for the first ur)
  long long ws_floats; // split-pair partials (fp32)
  int counters;        // per (row tile, lane quarter) arrival counters
};

StreamPlan stream_plan(int M, int N, int K, int num_sms);
// Sets the shared-memory attribute of every instantiation on the current
// device (stream_launch does it on first use; callers that must not do it
// inside a call, like the allocation-free entry point, do it at set-up).
cudaError_t stream_set_attrs();
bool stream_eligible(int M, int N, int K);
// x [M, K] bf16 (row stride ldx), wblob the pre-tiled INT4 blob of W [N, K],
// out [M, ldo] bf16 (N columns, N/2 for SiLU), residual [M, ldr] for the
// residual epilogue.  ws: stream_plan().ws_floats floats; counters: zero on
// entry, zero again on exit.
void stream_launch(const void* x, int64_t ldx, const uint8_t* wblob, void* out, int64_t ldo,
                   const void* residual, int64_t ldr, int M, int N, int K, int group_size,
                   int epilogue, float* ws, int* counters, int* status, cudaStream_t stream,
                   unsigned long long* trace = nullptr);

}  // namespace cb
