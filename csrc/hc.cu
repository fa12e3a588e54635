// DeepSeek-V4 Hyper-Connections pre-mix, one kernel per sublayer input.
//
// The residual stream holds `hc` copies of each token's hidden vector.  For
// every token this kernel
//   1. computes the inverse RMS of the flattened copies [hc * dim],
//   2. the (2 + hc) * hc mixing logits  m = (copies . fn_j) * rms^-1,
//   3. pre  = sigmoid(m[:hc] * s0 + b[:hc]) + eps,
//      post = 2 sigmoid(m[hc:2hc] * s1 + b[hc:2hc]),
//      comb = row softmax(m[2hc:] * s2 + b[2hc:]) + eps, then column
//             normalise and (iters - 1) rounds of row + column normalisation
//             (Sinkhorn), every division by (sum + eps),
//   4. the reduced sublayer input y[d] = bf16(sum_h pre[h] * copies[h][d]).
// One CTA per token: the copies row is staged in shared memory, one warp per
// group of mixing rows computes the dots, warp 0 runs the Sinkhorn on the
// hc x hc matrix in registers / shared memory, then all threads reduce.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {
namespace {

constexpr int kHcThreads = 256;
constexpr int kHcMax = 8;  // hc <= 8: (2 + hc) * hc <= 80 mixing rows

__global__ void __launch_bounds__(kHcThreads) hc_pre_kernel(
    const float* __restrict__ copies, const float* __restrict__ fn, const float* __restrict__ base,
    const float* __restrict__ scale, int hc, int dim, int iters, float hc_eps, float norm_eps,
    float* __restrict__ y, float* __restrict__ post_out, float* __restrict__ comb_out,
    float* __restrict__ pre_out) {
  grid_dep_launch();
  grid_dep_wait();
  extern __shared__ float sh[];
  const int t = blockIdx.x;
  const int n = hc * dim;
  const int nm = (2 + hc) * hc;
  float* row = sh;                 // [n]
  float* mix = sh + n;             // [nm]
  float* red = mix + nm;           // [32]
  __shared__ float s_pre[kHcMax];
  const float* src = copies + (size_t)t * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = src[i];
    row[i] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    v = warp_sum(v);
    if (lane == 0) red[0] = 1.f / sqrtf(v / (float)n + norm_eps);
  }
  __syncthreads();
  const float r = red[0];
  // Mixing logits: one warp per row, rows strided over the warps.
  for (int j = warp; j < nm; j += blockDim.x >> 5) {
    const float* w = fn + (size_t)j * n;
    float acc = 0.f;
    for (int i = lane; i < n; i += 32) acc += row[i] * w[i];
    acc = warp_sum(acc);
    if (lane == 0) mix[j] = acc * r;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float c[kHcMax * kHcMax];
    for (int j = 0; j < hc; ++j) {
      const float p = 1.f / (1.f + expf(-(mix[j] * scale[0] + base[j]))) + hc_eps;
      s_pre[j] = p;
      pre_out[(size_t)t * hc + j] = p;
      post_out[(size_t)t * hc + j] =
          2.f / (1.f + expf(-(mix[hc + j] * scale[1] + base[hc + j])));
    }
    for (int j = 0; j < hc; ++j) {
      float m = -INFINITY;
      for (int k = 0; k < hc; ++k) {
        const int i = j * hc + k;
        c[i] = mix[2 * hc + i] * scale[2] + base[2 * hc + i];
        m = fmaxf(m, c[i]);
      }
      float s = 0.f;
      for (int k = 0; k < hc; ++k) {
        c[j * hc + k] = expf(c[j * hc + k] - m);
        s += c[j * hc + k];
      }
      for (int k = 0; k < hc; ++k) c[j * hc + k] = c[j * hc + k] / s + hc_eps;
    }
    auto col_norm = [&]() {
      for (int k = 0; k < hc; ++k) {
        float s = 0.f;
        for (int j = 0; j < hc; ++j) s += c[j * hc + k];
        for (int j = 0; j < hc; ++j) c[j * hc + k] /= s + hc_eps;
      }
    };
    col_norm();
    for (int it = 1; it < iters; ++it) {
      for (int j = 0; j < hc; ++j) {
        float s = 0.f;
        for (int k = 0; k < hc; ++k) s += c[j * hc + k];
        for (int k = 0; k < hc; ++k) c[j * hc + k] /= s + hc_eps;
      }
      col_norm();
    }
    for (int i = 0; i < hc * hc; ++i) comb_out[(size_t)t * hc * hc + i] = c[i];
  }
  __syncthreads();
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    float acc = 0.f;
    for (int h = 0; h < hc; ++h) acc += s_pre[h] * row[h * dim + d];
    y[(size_t)t * dim + d] = __bfloat162float(__float2bfloat16(acc));
  }
}

}  // namespace

// copies [T, hc, dim] fp32; fn [(2+hc)*hc, hc*dim]; base [(2+hc)*hc]; scale [3].
// Returns y [T, dim] (bf16 values in fp32), post [T, hc], comb [T, hc, hc], pre [T, hc].
std::vector<torch::Tensor> hc_pre(torch::Tensor copies, torch::Tensor fn, torch::Tensor base,
                                  torch::Tensor scale, int64_t iters, double hc_eps,
                                  double norm_eps) {
  TORCH_CHECK(copies.is_cuda() && copies.scalar_type() == at::kFloat && copies.dim() == 3 &&
                  copies.is_contiguous(),
              "hc_pre: copies fp32 [T, hc, dim] contiguous");
  const int T = (int)copies.size(0), hc = (int)copies.size(1), dim = (int)copies.size(2);
  TORCH_CHECK(hc >= 1 && hc <= kHcMax, "hc_pre: hc in 1..8");
  const int nm = (2 + hc) * hc;
  TORCH_CHECK(fn.is_contiguous() && fn.scalar_type() == at::kFloat && fn.size(0) == nm &&
                  fn.size(1) == hc * dim && base.numel() == nm && scale.numel() == 3,
              "hc_pre: parameter shapes");
  const c10::cuda::CUDAGuard guard(copies.device());
  auto opt = copies.options();
  auto y = torch::empty({T, dim}, opt);
  auto post = torch::empty({T, hc}, opt);
  auto comb = torch::empty({T, hc, hc}, opt);
  auto pre = torch::empty({T, hc}, opt);
  if (T == 0) return {y, post, comb, pre};
  const size_t smem = (size_t)(hc * dim + nm + 32) * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "hc_pre: hc * dim too large for one CTA");
  if (smem > 48 * 1024) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(hc_pre_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
  }
  auto b = base.to(at::kFloat).contiguous();
  auto s = scale.to(at::kFloat).contiguous();
  launch_kernel(hc_pre_kernel, dim3(T), dim3(kHcThreads), smem, at::cuda::getCurrentCUDAStream(),
                copies.data_ptr<float>(), fn.data_ptr<float>(), b.data_ptr<float>(),
                s.data_ptr<float>(), hc, dim, (int)iters, (float)hc_eps, (float)norm_eps,
                y.data_ptr<float>(), post.data_ptr<float>(), comb.data_ptr<float>(),
                pre.data_ptr<float>());
  return {y, post, comb, pre};
}

}  // namespace cb
