// Small-M W4A16 GEMM (decode, 1..16 tokens): shared declarations.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace cb {

constexpr int kGemvMaxM = 16;
// Epilogue codes (same values as the tcgen05 GEMM's).
enum GemvEpilogue : int { kGvEpiStore = 0, kGvEpiSilu = 1, kGvEpiResid = 2 };

bool gemv_eligible(int64_t M);
int64_t gemv_workspace_floats(int64_t M, int64_t N, int64_t K, int64_t forced_splits);
// Launch on `stream`.  x [M, K] bf16 (row stride ldx), wblob the pre-tiled
// INT4 blob of W [N, K], out [M, ldo] bf16; ws / counters: split-K scratch
// (counters zero on entry, zero again on exit).
void gemv_launch(const void* x, int64_t ldx, const uint8_t* wblob, void* out, int64_t ldo,
                 const void* residual, int64_t ldr, int M, int N, int K, int group_size,
                 int epilogue, float* ws, int* counters, int* status, int forced_splits,
                 cudaStream_t stream);

}  // namespace cb
