// Sparse-MoE routing kernels for sm_100a.
//
// * moe_topk_gate: router logits (x . Wg^T, bf16 weights, fp32 math), score
//   function and top-k in one kernel, one CTA per token:
//     softmax routing (Qwen3-MoE): p = softmax(logits), take the top-k p,
//       optionally renormalise them to sum 1;
//     sigmoid routing (Kimi-K2 / DeepSeek-V3 "noaux_tc"): s = sigmoid(logits),
//       choose the top-k of s + bias, weight with s (not the bias),
//       optionally renormalise, then multiply by routed_scaling_factor.
//   Reference: crates/cascadia-int4-gemm/src/shell.rs:261-298 (K2.6 router),
//   crates/cascadia-engine-sparse-moe/src/glm/gate.rs:24-89.
// * moe_permute: counting sort of the (token, slot) pairs by expert ->
//   expert offsets and the permuted order, plus the gather of the activation
//   rows into expert-contiguous order for the grouped expert GEMM.
// * moe_combine: out[t] = sum_j w[t, j] * Y[pos(t, j)] (+ optional add),
//   summed in slot order, so the result does not depend on the order rows
//   were placed within an expert.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {

using bf16 = __nv_bfloat16;

constexpr int kGateThreads = 256;
constexpr int kMaxExperts = 512;
constexpr int kMaxTopK = 16;

// Grid (T, G): CTA (t, g) computes the logits of experts [32g, 32g + 32)
// for token t (one warp per 4 experts, 16-byte loads) into the fp32
// workspace; the last CTA of token t (per-token counter, left at zero again)
// then applies the score function and picks the top-k.  Splitting the
// experts over G CTAs puts T * G CTAs on the router GEMV instead of T.
constexpr int kGateExpertsPerCta = 32;

__global__ void __launch_bounds__(kGateThreads) moe_topk_gate_kernel(
    const bf16* __restrict__ x, int ldx, const bf16* __restrict__ wg,
    const float* __restrict__ bias, int H, int E, int k, int scoring, int norm_topk,
    float routed_scale, int* __restrict__ topk_ids, float* __restrict__ topk_w,
    float* __restrict__ logits, int* __restrict__ counters) {
  __shared__ float s_score[kMaxExperts];
  __shared__ float s_sel[kMaxExperts];
  __shared__ float s_red_v[32];
  __shared__ int s_red_i[32];
  __shared__ int s_last;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const bf16* xr = x + (size_t)t * ldx;
  // 1. logits of this CTA's experts.
  const int e0 = blockIdx.y * kGateExpertsPerCta;
  const int e1 = min(E, e0 + kGateExpertsPerCta);
  // Each warp computes kGatePerWarp experts side by side: one load of x
  // per step serves all of them and their weight loads are independent.
  constexpr int kGatePerWarp = kGateExpertsPerCta / (kGateThreads / 32);
  const int ew0 = e0 + warp * kGatePerWarp;
  float acc[kGatePerWarp];
#pragma unroll
  for (int j = 0; j < kGatePerWarp; ++j) acc[j] = 0.f;
#pragma unroll 2
  for (int i = lane * 8; i < H; i += 32 * 8) {
    const uint4 xu = *reinterpret_cast<const uint4*>(xr + i);
    const bf16* xv = reinterpret_cast<const bf16*>(&xu);
    float xf[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) xf[q] = __bfloat162float(xv[q]);
#pragma unroll
    for (int j = 0; j < kGatePerWarp; ++j) {
      if (ew0 + j < e1) {
        const uint4 wu = *reinterpret_cast<const uint4*>(wg + (size_t)(ew0 + j) * H + i);
        const bf16* wv = reinterpret_cast<const bf16*>(&wu);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[j] += xf[q] * __bfloat162float(wv[q]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kGatePerWarp; ++j) {
    const float v = warp_sum(acc[j]);
    if (lane == 0 && ew0 + j < e1) logits[(size_t)t * E + ew0 + j] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&counters[t], 1);
    s_last = prev == (int)gridDim.y - 1;
    if (s_last) counters[t] = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_score[e] = __ldcg(&logits[(size_t)t * E + e]);
  __syncthreads();
  // 2. score function.
  if (scoring == 0) {
    float mx = -INFINITY;
    for (int e = threadIdx.x; e < E; e += blockDim.x) mx = fmaxf(mx, s_score[e]);
    mx = warp_max(mx);
    if (lane == 0) s_red_v[warp] = mx;
    __syncthreads();
    mx = lane < nw ? s_red_v[lane] : -INFINITY;
    mx = warp_max(mx);
    __syncthreads();
    float sum = 0.f;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float p = __expf(s_score[e] - mx);
      s_score[e] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    if (lane == 0) s_red_v[warp] = sum;
    __syncthreads();
    sum = lane < nw ? s_red_v[lane] : 0.f;
    sum = warp_sum(sum);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      s_score[e] /= sum;
      s_sel[e] = s_score[e];
    }
  } else {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float sg = 1.f / (1.f + __expf(-s_score[e]));
      s_score[e] = sg;
      s_sel[e] = sg + (bias != nullptr ? bias[e] : 0.f);
    }
  }
  __syncthreads();
  // 3. top-k by repeated block argmax over s_sel (ties -> lowest expert id).
  __shared__ int s_ids[kMaxTopK];
  __shared__ float s_w[kMaxTopK];
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float v = s_sel[e];
      if (v > best || (v == best && e < bi)) {
        best = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      s_red_v[warp] = best;
      s_red_i[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float b = -INFINITY;
      int id = 0x7fffffff;
      for (int w = 0; w < nw; ++w)
        if (s_red_v[w] > b || (s_red_v[w] == b && s_red_i[w] < id)) {
          b = s_red_v[w];
          id = s_red_i[w];
        }
      s_ids[j] = id;
      s_w[j] = s_score[id];
      s_sel[id] = -INFINITY;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float sum = 0.f;
    for (int j = 0; j < k; ++j) sum += s_w[j];
    const float inv = (norm_topk && sum > 0.f) ? 1.f / sum : 1.f;
    for (int j = 0; j < k; ++j) {
      topk_ids[t * k + j] = s_ids[j];
      topk_w[t * k + j] = s_w[j] * inv * routed_scale;
    }
  }
}

void moe_topk_gate(torch::Tensor x, torch::Tensor wg, c10::optional<torch::Tensor> bias,
                   int64_t k, int64_t scoring, bool norm_topk, double routed_scale,
                   torch::Tensor topk_ids, torch::Tensor topk_w, torch::Tensor logits,
                   torch::Tensor counters) {
  const int T = (int)x.size(0);
  const int H = (int)x.size(1);
  const int E = (int)wg.size(0);
  TORCH_CHECK(E <= kMaxExperts && k <= kMaxTopK && k <= E, "unsupported expert count / top-k");
  TORCH_CHECK(H % 8 == 0 && x.stride(1) == 1 && wg.is_contiguous(), "layout");
  TORCH_CHECK(logits.numel() >= (int64_t)T * E && counters.numel() >= T, "gate workspace");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  const dim3 grid(T, (E + kGateExpertsPerCta - 1) / kGateExpertsPerCta);
  moe_topk_gate_kernel<<<grid, kGateThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), (int)x.stride(0),
      reinterpret_cast<const bf16*>(wg.data_ptr()),
      bias.has_value() ? bias->data_ptr<float>() : nullptr, H, E, (int)k, (int)scoring,
      norm_topk ? 1 : 0, (float)routed_scale, topk_ids.data_ptr<int>(), topk_w.data_ptr<float>(),
      logits.data_ptr<float>(), counters.data_ptr<int>());
  CB_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ permute
// One CTA: histogram of expert ids, exclusive scan -> offsets [E+1], then a
// parallel scatter -> perm[pos] = t*k + j and inv[t*k + j] = pos.  The order
// of rows within one expert is whatever the shared-memory atomics give: the
// grouped GEMM computes every row independently and moe_combine sums in slot
// order, so the layer output does not depend on it.
__global__ void moe_permute_kernel(const int* __restrict__ ids, int n, int E,
                                   int* __restrict__ offsets, int* __restrict__ perm,
                                   int* __restrict__ inv) {
  __shared__ int cnt[kMaxExperts + 1];
  __shared__ int cur[kMaxExperts];
  __shared__ int wsum[32];
  for (int e = threadIdx.x; e <= E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) atomicAdd(&cnt[ids[i]], 1);
  __syncthreads();
  // Exclusive scan of cnt[0..E) with one element per thread (E <= 1024).
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = threadIdx.x < E ? cnt[threadIdx.x] : 0;
  int incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int ws = lane < nw ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, ws, o);
      if (lane >= o) ws += v;
    }
    if (lane < nw) wsum[lane] = ws;  // inclusive over warps
  }
  __syncthreads();
  const int excl = incl - c + (warp > 0 ? wsum[warp - 1] : 0);
  if (threadIdx.x < E) {
    offsets[threadIdx.x] = excl;
    cur[threadIdx.x] = excl;
  }
  if (threadIdx.x == 0) offsets[E] = n;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int pos = atomicAdd(&cur[ids[i]], 1);
    perm[pos] = i;
    inv[i] = pos;
  }
}

// Gather x rows into expert order: xp[pos] = x[perm[pos] / k].
__global__ void moe_gather_kernel(const bf16* __restrict__ x, int ldx, const int* __restrict__ perm,
                                  int k, int H, bf16* __restrict__ xp) {
  const int pos = blockIdx.x;
  const int t = perm[pos] / k;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * ldx);
  uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)pos * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

void moe_permute(torch::Tensor topk_ids, int64_t E, torch::Tensor offsets, torch::Tensor perm,
                 torch::Tensor inv, c10::optional<torch::Tensor> x,
                 c10::optional<torch::Tensor> xp) {
  const int n = (int)topk_ids.numel();
  TORCH_CHECK(E <= kMaxExperts, "too many experts");
  const c10::cuda::CUDAGuard guard(topk_ids.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  moe_permute_kernel<<<1, 1024, 0, stream>>>(topk_ids.data_ptr<int>(), n, (int)E,
                                             offsets.data_ptr<int>(), perm.data_ptr<int>(),
                                             inv.data_ptr<int>());
  CB_CUDA_CHECK(cudaGetLastError());
  if (x.has_value() && n > 0) {
    const int k = (int)topk_ids.size(1);
    const int H = (int)x->size(1);
    moe_gather_kernel<<<n, 128, 0, stream>>>(reinterpret_cast<const bf16*>(x->data_ptr()),
                                             (int)x->stride(0), perm.data_ptr<int>(), k, H,
                                             reinterpret_cast<bf16*>(xp->data_ptr()));
    CB_CUDA_CHECK(cudaGetLastError());
  }
}

// ------------------------------------------------------------------ combine
// out[t] = sum_j w[t, j] * y[inv[t*k + j]] (+ add[t]), fp32 accumulation.
// out[t] = add[t] + sum_j w[t, j] * y[inv[t, j]]
//          (+ shared[t], scaled by sigmoid(shared_gate[t]) when given)
__global__ void moe_combine_kernel(const bf16* __restrict__ y, const int* __restrict__ inv,
                                   const float* __restrict__ w, int k, int H,
                                   const bf16* __restrict__ add, int ld_add,
                                   const bf16* __restrict__ shared, int ld_shared,
                                   const float* __restrict__ shared_gate,
                                   bf16* __restrict__ out, int ldo) {
  grid_dep_launch();
  grid_dep_wait();
  const int t = blockIdx.x;
  const float sg = shared_gate != nullptr ? 1.f / (1.f + __expf(-shared_gate[t])) : 1.f;
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int pos = inv[t * k + j];
      const float wt = w[t * k + j];
      const uint4 u = *reinterpret_cast<const uint4*>(y + (size_t)pos * H + i * 8);
      const bf16* v = reinterpret_cast<const bf16*>(&u);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wt * __bfloat162float(v[q]);
    }
    if (shared != nullptr) {
      const uint4 u = *reinterpret_cast<const uint4*>(shared + (size_t)t * ld_shared + i * 8);
      const bf16* v = reinterpret_cast<const bf16*>(&u);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += sg * __bfloat162float(v[q]);
    }
    if (add != nullptr) {
      const uint4 u = *reinterpret_cast<const uint4*>(add + (size_t)t * ld_add + i * 8);
      const bf16* v = reinterpret_cast<const bf16*>(&u);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(v[q]);
    }
    uint4 o;
    bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16(acc[q]);
    *reinterpret_cast<uint4*>(out + (size_t)t * ldo + i * 8) = o;
  }
}

void moe_combine(torch::Tensor y, torch::Tensor inv, torch::Tensor w, c10::optional<torch::Tensor> add,
                 torch::Tensor out, c10::optional<torch::Tensor> shared,
                 c10::optional<torch::Tensor> shared_gate) {
  const int T = (int)w.size(0);
  const int k = (int)w.size(1);
  const int H = (int)y.size(1);
  TORCH_CHECK(H % 8 == 0 && y.is_contiguous(), "y must be contiguous [rows, H], H % 8 == 0");
  TORCH_CHECK(!shared.has_value() || (shared->stride(1) == 1 && shared->size(0) >= T),
              "shared: [T, H] rows");
  TORCH_CHECK(!shared_gate.has_value() || (shared_gate->scalar_type() == at::kFloat &&
                                           shared_gate->numel() >= T),
              "shared_gate: fp32 [T]");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(y.device());
  launch_kernel(moe_combine_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                reinterpret_cast<const bf16*>(y.data_ptr()), (const int*)inv.data_ptr<int>(),
                (const float*)w.data_ptr<float>(), k, H,
                add.has_value() ? reinterpret_cast<const bf16*>(add->data_ptr()) : (const bf16*)nullptr,
                add.has_value() ? (int)add->stride(0) : 0,
                shared.has_value() ? reinterpret_cast<const bf16*>(shared->data_ptr()) : (const bf16*)nullptr,
                shared.has_value() ? (int)shared->stride(0) : 0,
                shared_gate.has_value() ? (const float*)shared_gate->data_ptr<float>() : (const float*)nullptr,
                reinterpret_cast<bf16*>(out.data_ptr()), (int)out.stride(0));
}

}  // namespace cb
