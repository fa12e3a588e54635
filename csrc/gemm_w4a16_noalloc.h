// W4A16 GEMM entry point that allocates no device memory.
//
// This entry point has no counterpart in the reference.  It exists for
// callers that cannot call cudaMalloc (or any allocating routine) at the time
// they run the GEMM:
//   * host applications that reserve all device memory up front and hand a
//     kernel library only the buffers they planned (inference servers with a
//     fixed memory budget, plugins inside another runtime): an allocation
//     behind their back can fail or break that budget;
//   * code in C, C++ or another language that uses this library without
//     PyTorch, and so without PyTorch's caching allocator to draw scratch from;
//   * latency-critical paths, where cudaMalloc / cudaFree can synchronise the
//     device and take unbounded time.
// The regular entry point (the Python `w4a16_gemm`) takes its scratch from a
// caller-visible workspace tensor; this one takes it from a fixed device
// array built into the library instead.  Both choose the same kernel for a
// shape: the small-M kernel for decode batches of up to 8 rows, the split-K
// tcgen05 kernel above.
//
// Scratch: one file-scope device array of CB_NOALLOC_SCRATCH_BYTES (about
// 24 MiB).  Every GPU that loads the library holds one copy until the process
// exits.  All calls on a device share it and it keeps the last call's
// contents; the call clears what must start at zero.  Calls whose GPU work
// overlaps (on different streams, or from different host threads without
// ordering between their streams) race on the scratch and give wrong results:
// order them on one stream.
//
// Set-up: the first call on each device looks up the array's device address
// (cudaGetSymbolAddress), sets the kernel's shared-memory attribute and loads
// the tensor-map encoder.  Make that first call before any stream capture.
// The device is the current device of the calling thread; all pointers must
// be memory of that device.
//
// Operands (same layout and numerics as `w4a16_gemm`):
//   x        [M, K] bf16, row stride ldx elements (ldx*2 a multiple of 16,
//            x 16-byte aligned);
//   wblob    the pre-tiled INT4 weight blob of W [N, K] (group 128 or 32);
//   out      [M, ldo] bf16; N columns, or N/2 for the SiLU epilogue;
//   residual [M, ldr] bf16 for the residual-add epilogue, else NULL;
//   epilogue 0 store, 1 SiLU(gate)*up over interleaved gate/up rows,
//            2 residual add;
//   status   optional device int (zero it before the call): receives the
//            first error code if a bounded wait inside the kernel gave up.
//            With NULL the code goes to a word of the scratch array that the
//            next call clears: a kernel-side timeout is then DISCARDED, so
//            callers that need to detect one must pass a status word;
//   stream   a cudaStream_t (NULL = legacy default stream);
//   err      optional host buffer of err_len bytes for a message on failure.
// Limits: K and N multiples of 128; the fp32 partials of the chosen kernel
// must fit CB_NOALLOC_MAX_WS_FLOATS floats and its counters
// CB_NOALLOC_MAX_COUNTERS (N up to 524288 rows); larger sizes are rejected
// with CB_NOALLOC_ETOOBIG.
// Returns CB_NOALLOC_OK once the kernel is enqueued.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define CB_NOALLOC_MAX_WS_FLOATS (6u << 20)
#define CB_NOALLOC_MAX_COUNTERS 16384u
#define CB_NOALLOC_SCRATCH_BYTES \
  (CB_NOALLOC_MAX_WS_FLOATS * 4u + CB_NOALLOC_MAX_COUNTERS * 4u + 256u)

enum {
  CB_NOALLOC_OK = 0,
  CB_NOALLOC_EINVAL = 1,   // bad argument (shape, alignment, epilogue)
  CB_NOALLOC_ETOOBIG = 2,  // the plan's scratch exceeds the fixed maximum
  CB_NOALLOC_ECUDA = 3     // a CUDA call failed (message in err)
};

int cb_w4a16_gemm_noalloc(const void* x, long long ldx, const void* wblob, void* out,
                          long long ldo, const void* residual, long long ldr, int M, int N,
                          int K, int group_size, int epilogue, int* status, void* stream,
                          char* err, int err_len);

#ifdef __cplusplus
}
#endif
