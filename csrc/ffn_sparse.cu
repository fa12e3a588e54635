// Activation-sparse SwiGLU FFN for one token (optional path, off by default).
//
// Gate first, then up and down only on the "active" intermediate lanes:
// lane i is active when |silu(gate_i)| >= tau_i * max_j |silu(gate_j)|
// (one global tau, or per-channel tau from offline calibration); inactive
// lanes contribute nothing.  The down projection runs in AXPY form over a
// transposed, re-quantised down weight [I, H] (groups along H), so an
// inactive lane's row is never read:
//     y[h] = sum_{r active} silu(g_r) * up_r * downT[r, h]
// (the reference's CPU kernels: crates/cascadia-int4-gemm/src/
// ffn_sparsity.rs:106-186 build_active_mask, :253 rows-subset GEMV,
// ffn_axpy.rs:167-273 AXPY down, :342 transpose_requantize_down).
//
// Weights use the plain INT4 layout: packed int32 [rows, K/8] (nibble e of
// word w is column 8w + e, value nibble - 8) and scales [rows, K/gs].
//
// Kernels (all bounded, no waits on other CTAs):
//   int4_rows_gemv_kernel  one warp per (listed) row: dot(x, dequant(row))
//   ffn_mask_kernel        one CTA: silu, max, threshold, ordered compaction
//   ffn_axpy_kernel        column slices x row groups, fp32 atomics into y
//   ffn_finish_kernel      out = bf16(y + residual), y reset to zero
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {

using bf16 = __nv_bfloat16;

struct RowsGemvArgs {
  const int* packed;       // [rows, K/8]
  const bf16* scales;      // [rows, K/gs]
  const bf16* x;           // [K]
  const int* rows;         // compacted row list (nullptr: rows 0..n-1)
  const int* count;        // number of listed rows (nullptr: n)
  const float* mul;        // optional per-listed-row factor (silu(gate) of the lane)
  float* out;              // [n] fp32, out[k] for the k-th listed row
  int n, K, gs;
};

__global__ void __launch_bounds__(256) int4_rows_gemv_kernel(const RowsGemvArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = blockIdx.x * 8 + warp;
  const int n = a.count != nullptr ? *a.count : a.n;
  if (k >= n) return;
  const int r = a.rows != nullptr ? a.rows[k] : k;
  const int words = a.K / 8;
  const int* pw = a.packed + (size_t)r * words;
  const bf16* ps = a.scales + (size_t)r * (a.K / a.gs);
  float acc = 0.f;
  for (int w = lane; w < words; w += 32) {
    const uint32_t v = (uint32_t)pw[w];
    const float s = __bfloat162float(ps[(8 * w) / a.gs]);
    const uint4 xv = *reinterpret_cast<const uint4*>(a.x + 8 * w);
    const bf16* xe = reinterpret_cast<const bf16*>(&xv);
    float d = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      d += (float)((int)((v >> (4 * e)) & 15u) - 8) * __bfloat162float(xe[e]);
    acc += d * s;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) a.out[k] = a.mul != nullptr ? acc * a.mul[k] : acc;
}

// One CTA of 1024 threads.  Writes the active lanes in ascending order
// (block-wide exclusive scan per 1024-lane chunk), their silu(gate) values,
// and the count.
__global__ void __launch_bounds__(1024) ffn_mask_kernel(const float* __restrict__ gate, int I,
                                                        const float* __restrict__ tau,
                                                        float tau_all, int* __restrict__ active,
                                                        float* __restrict__ silu_act,
                                                        int* __restrict__ count) {
  __shared__ float red[32];
  __shared__ int scan[32];
  __shared__ int base;
  grid_dep_launch();
  grid_dep_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float mx = 0.f;
  for (int i = tid; i < I; i += 1024) {
    const float g = gate[i];
    mx = fmaxf(mx, fabsf(g / (1.f + __expf(-g))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  if (tid == 0) base = 0;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < 32; ++w) mx = fmaxf(mx, red[w]);
  for (int c0 = 0; c0 < I; c0 += 1024) {
    const int i = c0 + tid;
    float sv = 0.f;
    bool on = false;
    if (i < I) {
      const float g = gate[i];
      sv = g / (1.f + __expf(-g));
      const float t = tau != nullptr ? tau[i] : tau_all;
      on = t <= 0.f || fabsf(sv) >= t * mx;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, on);
    if (lane == 0) scan[warp] = __popc(bal);
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += scan[w];
    const int pos = base + before + __popc(bal & ((1u << lane) - 1u));
    if (on) {
      active[pos] = i;
      silu_act[pos] = sv;
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < 32; ++w) tot += scan[w];
      base += tot;
    }
    __syncthreads();
  }
  if (tid == 0) *count = base;
}

struct AxpyArgs {
  const int* packed;       // downT [I, H/8]
  const bf16* scales;      // [I, H/gs]
  const int* active;       // [count]
  const int* count;
  const float* act;        // [count]: silu(g) * up of each listed lane
  float* y;                // [H] fp32 accumulator (zero on entry)
  int H, gs;
};

__global__ void __launch_bounds__(256) ffn_axpy_kernel(const AxpyArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  const int w = blockIdx.x * 256 + threadIdx.x;  // packed word = 8 columns
  if (w >= a.H / 8) return;
  const int n = *a.count;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int k = blockIdx.y; k < n; k += gridDim.y) {
    const int r = a.active[k];
    const float f = a.act[k] * __bfloat162float(a.scales[(size_t)r * (a.H / a.gs) + (8 * w) / a.gs]);
    const uint32_t v = (uint32_t)a.packed[(size_t)r * (a.H / 8) + w];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += f * (float)((int)((v >> (4 * e)) & 15u) - 8);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) atomicAdd(&a.y[8 * w + e], acc[e]);
}

__global__ void ffn_finish_kernel(float* __restrict__ y, const bf16* __restrict__ residual,
                                  bf16* __restrict__ out, int H) {
  grid_dep_launch();
  grid_dep_wait();
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H) return;
  float v = y[h];
  if (residual != nullptr) v += __bfloat162float(residual[h]);
  out[h] = __float2bfloat16(v);
  y[h] = 0.f;
}

// ---------------------------------------------------------------- host side

static void rows_gemv(const torch::Tensor& packed, const torch::Tensor& scales, const bf16* x,
                      const int* rows, const int* count, const float* mul, float* out, int n,
                      int K, int gs, cudaStream_t s) {
  RowsGemvArgs a;
  a.packed = packed.data_ptr<int>();
  a.scales = reinterpret_cast<const bf16*>(scales.data_ptr());
  a.x = x;
  a.rows = rows;
  a.count = count;
  a.mul = mul;
  a.out = out;
  a.n = n;
  a.K = K;
  a.gs = gs;
  launch_kernel(int4_rows_gemv_kernel, dim3((unsigned)((n + 7) / 8)), dim3(256), 0, s, a);
}

// x [1, H] bf16 -> out [1, H] bf16 (+ residual).  work: int32 [2 * I + 1]
// (active list, count), fp32 [3 * I + H] (gate, silu(gate) of the listed
// lanes, act, y accumulator; y must be zero on the first call and is left
// zero).  tau: per-channel [I] fp32 or None (then tau_all).
void ffn_sparse_forward(torch::Tensor x, torch::Tensor gate_packed, torch::Tensor gate_scales,
                        torch::Tensor up_packed, torch::Tensor up_scales,
                        torch::Tensor downT_packed, torch::Tensor downT_scales,
                        c10::optional<torch::Tensor> tau, double tau_all,
                        c10::optional<torch::Tensor> residual, torch::Tensor out,
                        torch::Tensor iwork, torch::Tensor fwork, int64_t group_size,
                        int64_t down_group_size) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.size(0) == 1 &&
                  x.is_contiguous(), "x must be one contiguous bf16 row");
  const int H = (int)x.size(1);
  const int I = (int)gate_packed.size(0);
  const int gs = (int)group_size;
  TORCH_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
  TORCH_CHECK(gate_packed.size(1) * 8 == H && up_packed.size(0) == I && downT_packed.size(0) == I &&
                  downT_packed.size(1) * 8 == H, "weights: gate/up [I, H/8], downT [I, H/8]");
  TORCH_CHECK(H % gs == 0 && gs % 8 == 0 && H % down_group_size == 0 && down_group_size % 8 == 0,
              "group sizes must be multiples of 8 dividing the hidden size");
  TORCH_CHECK(iwork.numel() >= 2 * I + 1 && fwork.numel() >= 3 * I + H, "work buffers too small");
  TORCH_CHECK(!tau.has_value() || (tau->numel() == I && tau->scalar_type() == at::kFloat),
              "tau: fp32 [I]");
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  int* active = iwork.data_ptr<int>();
  int* count = active + I;
  float* gate = fwork.data_ptr<float>();
  float* silu_g = gate + I;
  float* act = silu_g + I;
  float* y = act + I;
  const bf16* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  rows_gemv(gate_packed, gate_scales, xp, nullptr, nullptr, nullptr, gate, I, H, gs, s);
  launch_kernel(ffn_mask_kernel, dim3(1), dim3(1024), 0, s, (const float*)gate, I,
                tau.has_value() ? (const float*)tau->data_ptr<float>() : (const float*)nullptr,
                (float)tau_all, active, silu_g, count);
  rows_gemv(up_packed, up_scales, xp, active, count, silu_g, act, I, H, gs, s);
  AxpyArgs a;
  a.packed = downT_packed.data_ptr<int>();
  a.scales = reinterpret_cast<const bf16*>(downT_scales.data_ptr());
  a.active = active;
  a.count = count;
  a.act = act;
  a.y = y;
  a.H = H;
  a.gs = (int)down_group_size;
  const int cols = (H / 8 + 255) / 256;
  launch_kernel(ffn_axpy_kernel, dim3((unsigned)cols, 64), dim3(256), 0, s, a);
  launch_kernel(ffn_finish_kernel, dim3((unsigned)((H + 255) / 256)), dim3(256), 0, s, y,
                residual.has_value() ? (const bf16*)residual->data_ptr() : (const bf16*)nullptr,
                reinterpret_cast<bf16*>(out.data_ptr()), H);
}

}  // namespace cb
