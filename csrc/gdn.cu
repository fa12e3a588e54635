// Gated DeltaNet (linear attention of the Qwen3.5 / Qwen3.6 hybrid layers)
// on sm_100a.
//
// The layer keeps, per sequence and value head h, a recurrent state matrix
// S[dk][dv] (fp32) instead of a KV cache, plus a (kernel_width - 1)-row
// causal-convolution state.  Per token (k-head kh = h / (Hv / Hk)):
//
//   q = l2norm(q_kh) / sqrt(dk),   k = l2norm(k_kh)
//   g = exp(-exp(A_log[h]) * softplus(a[h] + dt_bias[h])),  beta = sigmoid(b[h])
//   S = g * S;   u = beta * (v - S^T k);   S = S + k u^T;   o = S^T q
//   y = rmsnorm(o) * w * silu(z)
//
// (the recurrence of the reference's OpenVINO GatedDeltaNet graphs,
// crates/cascadia-engine-openvino/src/qwen36.rs:1-25 runs them as stateful
// IRs; the published model definition is the oracle in the tests).
//
// Kernels:
//   gdn_conv_kernel       depthwise causal conv (width KW) + SiLU over the
//                         mixed q|k|v channels, in place, conv state updated;
//                         one thread per channel walks its sequence's tokens.
//   gdn_recurrent_kernel  one CTA per (sequence, value head), 128 threads:
//                         thread j keeps column j of S in registers for all
//                         of the sequence's tokens (loaded and stored once),
//                         q/k normalisation, gating and the gated RMSNorm of
//                         the output are fused in.  Decode (one token per
//                         sequence) and prefill use the same kernel.
//   sigmoid_gate_kernel   out = x * sigmoid(gate) (gated full-attention
//                         output of the same models).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {

using bf16 = __nv_bfloat16;

constexpr int kGdnKW = 4;       // conv kernel width
constexpr int kGdnDK = 128;     // key head dim
constexpr int kGdnDV = 128;     // value head dim

struct GdnConvArgs {
  bf16* x;                 // [T, ldx]: channels [0, C) convolved in place
  int ldx;
  const bf16* w;           // [C, KW]
  bf16* state;             // [slots, KW - 1, C]
  const int* seq_start;    // [B + 1] token offsets
  const int* block_tables; // [B, bt_stride]: the first block of a sequence names
  int bt_stride;           //   its state slot through block_slot
  const int* block_slot;   // [num_blocks]
  int C;
};

__global__ void __launch_bounds__(256) gdn_conv_kernel(const GdnConvArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= a.C) return;
  const int t0 = a.seq_start[b], t1 = a.seq_start[b + 1];
  const int slot = a.block_slot[a.block_tables[(size_t)b * a.bt_stride]];
  bf16* st = a.state + (size_t)slot * (kGdnKW - 1) * a.C + c;
  float w[kGdnKW], h[kGdnKW - 1];
#pragma unroll
  for (int j = 0; j < kGdnKW; ++j) w[j] = __bfloat162float(a.w[(size_t)c * kGdnKW + j]);
#pragma unroll
  for (int j = 0; j < kGdnKW - 1; ++j) h[j] = __bfloat162float(st[(size_t)j * a.C]);
  for (int t = t0; t < t1; ++t) {
    bf16* p = a.x + (size_t)t * a.ldx + c;
    const float xt = __bfloat162float(*p);
    float acc = xt * w[kGdnKW - 1];
#pragma unroll
    for (int j = 0; j < kGdnKW - 1; ++j) acc += h[j] * w[j];
    // The convolution output is rounded to bf16 before the activation, as
    // the bf16 model computes it.
    acc = __bfloat162float(__float2bfloat16(acc));
    *p = __float2bfloat16(acc / (1.f + __expf(-acc)));
#pragma unroll
    for (int j = 0; j < kGdnKW - 2; ++j) h[j] = h[j + 1];
    h[kGdnKW - 2] = xt;
  }
#pragma unroll
  for (int j = 0; j < kGdnKW - 1; ++j) st[(size_t)j * a.C] = __float2bfloat16(h[j]);
}

struct GdnArgs {
  const bf16* qkv;       // [T, ldq]: q (Hk*DK) | k (Hk*DK) | v (Hv*DV), after the conv
  int ldq;
  const bf16* z;         // [T, ldz]: output gate, Hv*DV
  int ldz;
  const bf16* ab;        // [T, ldab]: b (Hv) then a (Hv)
  int ldab;
  const float* a_log;    // [Hv]
  const float* dt_bias;  // [Hv]
  const bf16* norm_w;    // [DV]
  float* state;          // [slots, Hv, DK, DV]
  const int* seq_start;  // [B + 1]
  const int* block_tables;
  int bt_stride;
  const int* block_slot;
  bf16* out;             // [T, ldo]: Hv*DV
  int ldo;
  int Hk, Hv;
  float eps;
};

__device__ __forceinline__ float gdn_block_sum2(float& x, float& y, float* red) {
  // Sums two values over the 128 threads of the CTA (4 warps); returns x.
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    x += __shfl_xor_sync(0xffffffffu, x, o);
    y += __shfl_xor_sync(0xffffffffu, y, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[2 * w] = x;
    red[2 * w + 1] = y;
  }
  __syncthreads();
  x = red[0] + red[2] + red[4] + red[6];
  y = red[1] + red[3] + red[5] + red[7];
  return x;
}

__global__ void __launch_bounds__(128) gdn_recurrent_kernel(const GdnArgs a) {
  __shared__ float qs[kGdnDK], ks[kGdnDK];
  __shared__ float red[2][8];
  grid_dep_launch();
  grid_dep_wait();
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int j = threadIdx.x;  // value column (and key row while loading q/k)
  const int kh = h / (a.Hv / a.Hk);
  const int t0 = a.seq_start[b], t1 = a.seq_start[b + 1];
  if (t0 >= t1) return;
  const int slot = a.block_slot[a.block_tables[(size_t)b * a.bt_stride]];
  float* S = a.state + ((size_t)slot * a.Hv + h) * kGdnDK * kGdnDV + j;
  float s[kGdnDK];
#pragma unroll
  for (int i = 0; i < kGdnDK; ++i) s[i] = S[(size_t)i * kGdnDV];
  const float A = -__expf(a.a_log[h]);
  const float dtb = a.dt_bias[h];
  const float nw = __bfloat162float(a.norm_w[j]);
  const float qscale = rsqrtf((float)kGdnDK);
  int rb = 0;
  for (int t = t0; t < t1; ++t) {
    const bf16* row = a.qkv + (size_t)t * a.ldq;
    float qv = __bfloat162float(row[kh * kGdnDK + j]);
    float kv = __bfloat162float(row[(a.Hk + kh) * kGdnDK + j]);
    const float vv = __bfloat162float(row[2 * a.Hk * kGdnDK + h * kGdnDV + j]);
    const float zv = __bfloat162float(a.z[(size_t)t * a.ldz + h * kGdnDV + j]);
    const float bb = __bfloat162float(a.ab[(size_t)t * a.ldab + h]);
    const float aa = __bfloat162float(a.ab[(size_t)t * a.ldab + a.Hv + h]);
    float sq = qv * qv, sk = kv * kv;
    gdn_block_sum2(sq, sk, red[rb]);
    rb ^= 1;  // the other buffer next time: no barrier needed before reuse
    qs[j] = qv * rsqrtf(sq + 1e-6f) * qscale;
    ks[j] = kv * rsqrtf(sk + 1e-6f);
    __syncthreads();
    const float x = aa + dtb;
    const float sp = x > 20.f ? x : log1pf(__expf(x));  // softplus
    const float g = __expf(A * sp);
    const float beta = 1.f / (1.f + __expf(-bb));
    // kv_mem = (g S)^T k, four partial sums for ILP.
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll
    for (int i = 0; i < kGdnDK; i += 4) {
      m0 += s[i] * ks[i];
      m1 += s[i + 1] * ks[i + 1];
      m2 += s[i + 2] * ks[i + 2];
      m3 += s[i + 3] * ks[i + 3];
    }
    const float u = beta * (vv - g * ((m0 + m1) + (m2 + m3)));
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
    for (int i = 0; i < kGdnDK; i += 4) {
      s[i] = g * s[i] + ks[i] * u;
      s[i + 1] = g * s[i + 1] + ks[i + 1] * u;
      s[i + 2] = g * s[i + 2] + ks[i + 2] * u;
      s[i + 3] = g * s[i + 3] + ks[i + 3] * u;
      o0 += s[i] * qs[i];
      o1 += s[i + 1] * qs[i + 1];
      o2 += s[i + 2] * qs[i + 2];
      o3 += s[i + 3] * qs[i + 3];
    }
    // The core output is bf16 in the model; then the gated RMSNorm.
    const float o = __bfloat162float(__float2bfloat16((o0 + o1) + (o2 + o3)));
    float so = o * o, dummy = 0.f;
    gdn_block_sum2(so, dummy, red[rb]);
    rb ^= 1;
    const float nrm = __bfloat162float(__float2bfloat16(o * rsqrtf(so / kGdnDV + a.eps)));
    const float y = nw * nrm * (zv / (1.f + __expf(-zv)));
    a.out[(size_t)t * a.ldo + h * kGdnDV + j] = __float2bfloat16(y);
    // qs/ks are rewritten next token only after its first block sum, whose
    // barrier every thread reaches after finishing this token.
  }
#pragma unroll
  for (int i = 0; i < kGdnDK; ++i) S[(size_t)i * kGdnDV] = s[i];
}

__global__ void sigmoid_gate_kernel(bf16* __restrict__ x, int ldx, const bf16* __restrict__ gate,
                                    int ldg, int n) {
  grid_dep_launch();
  grid_dep_wait();
  const int t = blockIdx.y;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) * 8; i < n; i += gridDim.x * blockDim.x * 8) {
    uint4 xv = *reinterpret_cast<const uint4*>(x + (size_t)t * ldx + i);
    const uint4 gv = *reinterpret_cast<const uint4*>(gate + (size_t)t * ldg + i);
    bf16* xe = reinterpret_cast<bf16*>(&xv);
    const bf16* ge = reinterpret_cast<const bf16*>(&gv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float g = __bfloat162float(ge[e]);
      xe[e] = __float2bfloat16(__bfloat162float(xe[e]) / (1.f + __expf(-g)));
    }
    *reinterpret_cast<uint4*>(x + (size_t)t * ldx + i) = xv;
  }
}

// ---------------------------------------------------------------- host side

void gdn_conv(torch::Tensor x, int64_t C, torch::Tensor w, torch::Tensor state,
              torch::Tensor seq_start, torch::Tensor block_tables, torch::Tensor block_slot) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "x");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.size(0) == C &&
                  w.size(1) == kGdnKW, "conv weight must be bf16 [C, 4]");
  TORCH_CHECK(state.scalar_type() == at::kBFloat16 && state.is_contiguous() &&
                  state.size(1) == kGdnKW - 1 && state.size(2) == C,
              "conv state must be bf16 [slots, 3, C]");
  TORCH_CHECK(seq_start.scalar_type() == at::kInt && block_tables.scalar_type() == at::kInt &&
                  block_slot.scalar_type() == at::kInt && block_tables.stride(1) == 1,
              "int32 seq_start / block tables / block_slot");
  const int B = (int)seq_start.numel() - 1;
  TORCH_CHECK(block_tables.size(0) >= B, "one block-table row per sequence");
  if (B == 0 || x.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  GdnConvArgs a;
  a.x = reinterpret_cast<bf16*>(x.data_ptr());
  a.ldx = (int)x.stride(0);
  a.w = reinterpret_cast<const bf16*>(w.data_ptr());
  a.state = reinterpret_cast<bf16*>(state.data_ptr());
  a.seq_start = seq_start.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = (int)block_tables.stride(0);
  a.block_slot = block_slot.data_ptr<int>();
  a.C = (int)C;
  launch_kernel(gdn_conv_kernel, dim3((unsigned)((C + 255) / 256), (unsigned)B), dim3(256), 0,
                at::cuda::getCurrentCUDAStream(), a);
}

void gdn_recurrent(torch::Tensor qkv, torch::Tensor z, torch::Tensor ab, torch::Tensor a_log,
                   torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor state,
                   torch::Tensor seq_start, torch::Tensor block_tables, torch::Tensor block_slot,
                   torch::Tensor out, int64_t Hk, int64_t Hv, double eps) {
  TORCH_CHECK(qkv.stride(1) == 1 && z.stride(1) == 1 && ab.stride(1) == 1 && out.stride(1) == 1,
              "inner strides must be 1");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.size(1) == Hv &&
                  state.size(2) == kGdnDK && state.size(3) == kGdnDV,
              "state must be fp32 [slots, Hv, 128, 128]");
  TORCH_CHECK(Hv % Hk == 0, "value heads must be a multiple of key heads");
  TORCH_CHECK(a_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat &&
                  norm_w.scalar_type() == at::kBFloat16 && norm_w.numel() == kGdnDV,
              "A_log / dt_bias fp32, norm weight bf16 [128]");
  TORCH_CHECK(seq_start.scalar_type() == at::kInt && block_tables.scalar_type() == at::kInt &&
                  block_slot.scalar_type() == at::kInt && block_tables.stride(1) == 1,
              "int32 seq_start / block tables / block_slot");
  const int B = (int)seq_start.numel() - 1;
  TORCH_CHECK(block_tables.size(0) >= B, "one block-table row per sequence");
  if (B == 0 || qkv.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(qkv.device());
  GdnArgs a;
  a.qkv = reinterpret_cast<const bf16*>(qkv.data_ptr());
  a.ldq = (int)qkv.stride(0);
  a.z = reinterpret_cast<const bf16*>(z.data_ptr());
  a.ldz = (int)z.stride(0);
  a.ab = reinterpret_cast<const bf16*>(ab.data_ptr());
  a.ldab = (int)ab.stride(0);
  a.a_log = a_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.norm_w = reinterpret_cast<const bf16*>(norm_w.data_ptr());
  a.state = state.data_ptr<float>();
  a.seq_start = seq_start.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = (int)block_tables.stride(0);
  a.block_slot = block_slot.data_ptr<int>();
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.ldo = (int)out.stride(0);
  a.Hk = (int)Hk;
  a.Hv = (int)Hv;
  a.eps = (float)eps;
  launch_kernel(gdn_recurrent_kernel, dim3((unsigned)Hv, (unsigned)B), dim3(128), 0,
                at::cuda::getCurrentCUDAStream(), a);
}

void sigmoid_gate(torch::Tensor x, torch::Tensor gate) {
  const int T = (int)x.size(0);
  const int n = (int)x.size(1);
  TORCH_CHECK(x.stride(1) == 1 && gate.stride(1) == 1 && gate.size(1) >= n && n % 8 == 0,
              "sigmoid_gate: matching rows, width a multiple of 8");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (gate.stride(0) * 2) % 16 == 0 &&
                  (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(gate.data_ptr()) & 15) == 0,
              "sigmoid_gate: rows must be 16-byte aligned");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  const int blocks = std::max(1, std::min(8, n / (256 * 8)));
  launch_kernel(sigmoid_gate_kernel, dim3((unsigned)blocks, (unsigned)T), dim3(256), 0,
                at::cuda::getCurrentCUDAStream(), reinterpret_cast<bf16*>(x.data_ptr()),
                (int)x.stride(0), reinterpret_cast<const bf16*>(gate.data_ptr()),
                (int)gate.stride(0), n);
}

}  // namespace cb
