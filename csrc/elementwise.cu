// Memory-bound helper kernels: embedding gather, RMSNorm (+ residual add),
// RoPE with the paged-KV write, greedy argmax, full sampling and the greedy
// speculative-decoding verify step.
//
// Reference math restated here:
//   RMSNorm      crates/cascadia-int4-gemm/src/shell.rs:371-394
//   RoPE + llama3 scaling (tables built on the host)  crates/cascadia-engine-openvino/src/rotary.rs:111-185
//   sampling     crates/cascadia-engine-sparse-moe/src/sampling.rs:52-187
//   spec accept  crates/cascadia-engine-sparse-moe/src/spec_decode.rs:28 (count_accepted)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <curand_kernel.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ embedding
__global__ void embedding_kernel(const int* __restrict__ ids, const bf16* __restrict__ table,
                                 bf16* __restrict__ out, int H, int ldo, int vocab_lo,
                                 int vocab_hi) {
  grid_dep_launch();
  grid_dep_wait();
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool mine = id >= vocab_lo && id < vocab_hi;  // vocab-parallel shards
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)(id - vocab_lo) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * ldo);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = mine ? src[i] : make_uint4(0, 0, 0, 0);
}

void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t vocab_lo) {
  const int T = (int)ids.size(0);
  const int H = (int)table.size(1);
  TORCH_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(ids.device());
  launch_kernel(embedding_kernel, dim3(T), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
                ids.data_ptr<int>(), reinterpret_cast<const bf16*>(table.data_ptr()),
                reinterpret_cast<bf16*>(out.data_ptr()), H, (int)out.stride(0), (int)vocab_lo,
                (int)(vocab_lo + table.size(0)));
}

// ------------------------------------------------------------------ RMSNorm
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float r = l < nw ? red[l] : 0.f;
  r = warp_sum(r);
  __syncthreads();
  return r;
}

// out = rmsnorm(x (+ residual)) * w ; if residual != null it is updated in
// place with x + residual first (the pre-norm residual stream).
template <int MAXV>
__global__ void rmsnorm_kernel(const bf16* __restrict__ x, int ldx, bf16* __restrict__ residual,
                               int ldr, const bf16* __restrict__ w, bf16* __restrict__ out, int ldo,
                               int H, float eps) {
  __shared__ float red[32];
  grid_dep_launch();
  grid_dep_wait();
  const int row = blockIdx.x;
  const int nvec = H / 8;
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      uint4 xv = reinterpret_cast<const uint4*>(x + (size_t)row * ldx)[i];
      const bf16* xe = reinterpret_cast<const bf16*>(&xv);
      if (residual != nullptr) {
        uint4 rv = reinterpret_cast<const uint4*>(residual + (size_t)row * ldr)[i];
        const bf16* re = reinterpret_cast<const bf16*>(&rv);
        uint4 nv;
        bf16* ne = reinterpret_cast<bf16*>(&nv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ne[e] = __float2bfloat16(__bfloat162float(xe[e]) + __bfloat162float(re[e]));
          v[k][e] = __bfloat162float(ne[e]);
        }
        reinterpret_cast<uint4*>(residual + (size_t)row * ldr)[i] = nv;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] = __bfloat162float(xe[e]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      uint4 wv = reinterpret_cast<const uint4*>(w)[i];
      const bf16* we = reinterpret_cast<const bf16*>(&wv);
      uint4 ov;
      bf16* oe = reinterpret_cast<bf16*>(&ov);
#pragma unroll
      for (int e = 0; e < 8; ++e) oe[e] = __float2bfloat16(v[k][e] * inv * __bfloat162float(we[e]));
      reinterpret_cast<uint4*>(out + (size_t)row * ldo)[i] = ov;
    }
  }
}

void rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w,
             torch::Tensor out, double eps) {
  const int M = (int)x.size(0);
  const int H = (int)x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8192 * 2, "unsupported hidden size");
  TORCH_CHECK(x.stride(1) == 1 && out.stride(1) == 1, "inner stride must be 1");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  const int threads = std::min(1024, std::max(32, ((H / 8 + 31) / 32) * 32));
  bf16* res = residual.has_value() ? reinterpret_cast<bf16*>(residual->data_ptr()) : nullptr;
  const int ldr = residual.has_value() ? (int)residual->stride(0) : 0;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_kernel(H / 8 <= threads ? rmsnorm_kernel<1> : rmsnorm_kernel<2>, dim3(M),
                dim3(threads), 0, stream, reinterpret_cast<const bf16*>(x.data_ptr()),
                (int)x.stride(0), res, ldr, reinterpret_cast<const bf16*>(w.data_ptr()),
                reinterpret_cast<bf16*>(out.data_ptr()), (int)out.stride(0), H, (float)eps);
  CB_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ RoPE + KV
// qkv: [T, (Hq + 2*Hkv) * D] (q heads, then k heads, then v heads).
// cos_sin: [max_pos, rot] fp32, first rot/2 columns cos, last rot/2 sin.
// Non-interleaved (rotate-half, Llama/Qwen) or interleaved pairs (GLM).
// Vectorised: one thread rotates 8 pairs (two 16-byte loads / stores).
__device__ __forceinline__ void load8(const bf16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const bf16* e = reinterpret_cast<const bf16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(e[i]);
}
__device__ __forceinline__ void store8(bf16* p, const float (&v)[8]) {
  uint4 u;
  bf16* e = reinterpret_cast<bf16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = __float2bfloat16(v[i]);
  *reinterpret_cast<uint4*>(p) = u;
}

__global__ void rope_kv_kernel(bf16* __restrict__ qkv, int ldq, const int* __restrict__ positions,
                               const float* __restrict__ cos_sin, const int* __restrict__ slots,
                               bf16* __restrict__ k_cache, bf16* __restrict__ v_cache, int layer,
                               int NB, int Hq, int Hkv, int D, int rot, int interleaved) {
  grid_dep_launch();
  grid_dep_wait();
  const int t = blockIdx.x;
  const int pos = positions[t];
  const int slot = slots[t];
  bf16* row = qkv + (size_t)t * ldq;
  const float* cs = cos_sin + (size_t)pos * rot;
  const int half = rot / 2;
  const int pieces = half / 8;  // 8 pairs per thread
  const int nrot = (Hq + Hkv) * pieces;
  const size_t cache_row =
      slot >= 0 ? ((((size_t)layer * NB + slot / 16) * Hkv) * 16 + (slot % 16)) * (size_t)D : 0;
  for (int idx = threadIdx.x; idx < nrot; idx += blockDim.x) {
    const int hh = idx / pieces;
    const int i0 = (idx % pieces) * 8;
    bf16* hp = row + (size_t)hh * D;
    float x0[8], x1[8], c[8], sn[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      c[k] = cs[i0 + k];
      sn[k] = cs[half + i0 + k];
    }
    if (!interleaved) {
      load8(hp + i0, x0);
      load8(hp + half + i0, x1);
    } else {
      float a[8], b[8];
      load8(hp + 2 * i0, a);
      load8(hp + 2 * i0 + 8, b);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        x0[k] = a[2 * k];
        x1[k] = a[2 * k + 1];
        x0[4 + k] = b[2 * k];
        x1[4 + k] = b[2 * k + 1];
      }
    }
    float y0[8], y1[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      y0[k] = x0[k] * c[k] - x1[k] * sn[k];
      y1[k] = x1[k] * c[k] + x0[k] * sn[k];
    }
    bf16* dst;
    if (hh < Hq) {
      dst = hp;
    } else {
      if (slot < 0) continue;
      dst = k_cache + cache_row + (size_t)(hh - Hq) * 16 * D;
    }
    if (!interleaved) {
      store8(dst + i0, y0);
      store8(dst + half + i0, y1);
    } else {
      float a[8], b[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        a[2 * k] = y0[k];
        a[2 * k + 1] = y1[k];
        b[2 * k] = y0[4 + k];
        b[2 * k + 1] = y1[4 + k];
      }
      store8(dst + 2 * i0, a);
      store8(dst + 2 * i0 + 8, b);
    }
  }
  if (slot < 0) return;
  // Non-rotated part of K (partial rotary) and all of V, 8 values per thread.
  const int vec_per_head = D / 8;
  for (int idx = threadIdx.x; idx < Hkv * vec_per_head; idx += blockDim.x) {
    const int kh = idx / vec_per_head;
    const int d = (idx % vec_per_head) * 8;
    const size_t base = cache_row + (size_t)kh * 16 * D + d;
    *reinterpret_cast<uint4*>(v_cache + base) =
        *reinterpret_cast<const uint4*>(row + (size_t)(Hq + Hkv + kh) * D + d);
    if (d >= rot)
      *reinterpret_cast<uint4*>(k_cache + base) =
          *reinterpret_cast<const uint4*>(row + (size_t)(Hq + kh) * D + d);
  }
}

void rope_kv_write(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                   torch::Tensor slots, torch::Tensor k_cache, torch::Tensor v_cache, int64_t layer,
                   int64_t Hq, int64_t Hkv, int64_t D, int64_t rot, bool interleaved) {
  const int T = (int)qkv.size(0);
  if (T == 0) return;
  TORCH_CHECK(qkv.stride(1) == 1, "qkv inner stride must be 1");
  TORCH_CHECK(rot % 16 == 0 && D % 8 == 0, "rotary dim must be a multiple of 16");
  TORCH_CHECK((qkv.stride(0) * 2) % 16 == 0, "qkv rows must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(qkv.device());
  launch_kernel(rope_kv_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                reinterpret_cast<bf16*>(qkv.data_ptr()), (int)qkv.stride(0),
                positions.data_ptr<int>(), cos_sin.data_ptr<float>(), slots.data_ptr<int>(),
                reinterpret_cast<bf16*>(k_cache.data_ptr()),
                reinterpret_cast<bf16*>(v_cache.data_ptr()), (int)layer, (int)k_cache.size(1),
                (int)Hq, (int)Hkv, (int)D, (int)rot, interleaved ? 1 : 0);
}

// ------------------------------------------------------------------ q/k norm
// Per-head RMSNorm of the q and k heads of a fused qkv row, in place (Qwen3's
// q_norm / k_norm, applied before RoPE).  One warp per head; D <= 1024 (each
// lane holds up to four 8-element chunks).
__global__ void head_rmsnorm_kernel(bf16* __restrict__ qkv, int ldq, const bf16* __restrict__ qw,
                                    const bf16* __restrict__ kw, int Hq, int Hkv, int D,
                                    float eps) {
  grid_dep_launch();
  grid_dep_wait();
  const int t = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nw = blockDim.x / 32;
  for (int hh = warp; hh < Hq + Hkv; hh += nw) {
    bf16* hp = qkv + (size_t)t * ldq + (size_t)hh * D;
    const bf16* w = hh < Hq ? qw : kw;
    float v[4][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d0 = c * 256 + lane * 8;
      if (d0 < D) {
        load8(hp + d0, v[c]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += v[c][k] * v[c][k];
      }
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d0 = c * 256 + lane * 8;
      if (d0 < D) {
        float wv[8];
        load8(w + d0, wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[c][k] = v[c][k] * inv * wv[k];
        store8(hp + d0, v[c]);
      }
    }
  }
}

void head_rmsnorm(torch::Tensor qkv, torch::Tensor q_w, torch::Tensor k_w, int64_t Hq,
                  int64_t Hkv, int64_t D, double eps) {
  const int T = (int)qkv.size(0);
  if (T == 0) return;
  TORCH_CHECK(qkv.stride(1) == 1 && (qkv.stride(0) * 2) % 16 == 0, "qkv rows must be aligned");
  TORCH_CHECK(D % 8 == 0 && D <= 1024, "head_rmsnorm: D must be a multiple of 8, <= 1024");
  const c10::cuda::CUDAGuard guard(qkv.device());
  launch_kernel(head_rmsnorm_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                reinterpret_cast<bf16*>(qkv.data_ptr()), (int)qkv.stride(0),
                reinterpret_cast<const bf16*>(q_w.data_ptr()),
                reinterpret_cast<const bf16*>(k_w.data_ptr()), (int)Hq, (int)Hkv, (int)D,
                (float)eps);
}

// ------------------------------------------------------------------ argmax
// Row-wise argmax over [M, V] logits; ties resolve to the lowest index (the
// reference's strict `>` scan).  Optionally returns the max value too, which
// lets vocab-parallel shards merge with a tiny all-gather.
template <typename T>
__global__ void argmax_kernel(const T* __restrict__ logits, int ld, int V, int* __restrict__ out_idx,
                              float* __restrict__ out_val, int idx_offset) {
  grid_dep_launch();
  grid_dep_wait();
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  constexpr int VEC = 16 / sizeof(T);
  const bool vec_ok = (V % VEC == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (vec_ok) {
    // 16-byte loads; indices visited in increasing order per thread, so the
    // lowest-index tie rule is preserved by the strict comparisons.
    for (int i = threadIdx.x * VEC; i < V; i += blockDim.x * VEC) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        float v;
        if constexpr (std::is_same<T, float>::value) v = e[k];
        else v = __bfloat162float(e[k]);
        if (v > best) {
          best = v;
          bi = i + k;
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      float v;
      if constexpr (std::is_same<T, float>::value) v = x[i];
      else v = __bfloat162float(x[i]);
      if (v > best || (v == best && i < bi)) {
        best = v;
        bi = i;
      }
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
  __shared__ float sv[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = l < nw ? sv[l] : -INFINITY;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (l == 0) {
      out_idx[row] = bi == 0x7fffffff ? idx_offset : bi + idx_offset;
      if (out_val != nullptr) out_val[row] = best;
    }
  }
}

void argmax(torch::Tensor logits, torch::Tensor out_idx, c10::optional<torch::Tensor> out_val,
            int64_t idx_offset) {
  const int M = (int)logits.size(0);
  const int V = (int)logits.size(1);
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  float* ov = out_val.has_value() ? out_val->data_ptr<float>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == at::kFloat) {
    launch_kernel(argmax_kernel<float>, dim3(M), dim3(1024), 0, stream,
                  logits.data_ptr<float>(), (int)logits.stride(0), V, out_idx.data_ptr<int>(), ov,
                  (int)idx_offset);
  } else {
    launch_kernel(argmax_kernel<bf16>, dim3(M), dim3(1024), 0, stream,
                  reinterpret_cast<const bf16*>(logits.data_ptr()), (int)logits.stride(0), V,
                  out_idx.data_ptr<int>(), ov, (int)idx_offset);
  }
}

// ------------------------------------------------------------------ sampling
// params per row (float[8]): temperature, top_p, top_k, freq_pen, pres_pen,
// rep_pen, rep_window, unused.  history: int32 [M, Hmax] with hist_len [M].
// work: fp32 scratch [M, V].  seeds: int64 [M] (Philox key), offsets int64 [M].
constexpr int kSampThreads = 1024;

__device__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
  return warp_sum(r);
}
__device__ float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = l < (int)(blockDim.x >> 5) ? red[l] : -INFINITY;
  return warp_max(r);
}
__device__ int block_reduce_count(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  int r = l < (int)(blockDim.x >> 5) ? red[l] : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

// Largest threshold tau (over non-negative floats, by bit pattern) such that
// pred(tau) holds, where pred is monotone (true for small tau).
template <typename Pred>
__device__ float bit_search(Pred pred) {
  uint32_t lo = 0u;  // invariant: pred(as_float(lo)) true
#pragma unroll 1
  for (int bit = 30; bit >= 0; --bit) {
    const uint32_t cand = lo | (1u << bit);
    if (pred(__uint_as_float(cand))) lo = cand;
  }
  return __uint_as_float(lo);
}

template <typename T>
__global__ void __launch_bounds__(kSampThreads) sample_kernel(
    const T* __restrict__ logits, int ld, int V, const float* __restrict__ params,
    const int* __restrict__ history, int hist_ld, const int* __restrict__ hist_len,
    float* __restrict__ work, const int64_t* __restrict__ seeds,
    const int64_t* __restrict__ offsets, int* __restrict__ out) {
  __shared__ float redf[32];
  __shared__ int redi[32];
  __shared__ float s_scan[kSampThreads];
  const int row = blockIdx.x;
  const float* p = params + row * 8;
  const float temp = p[0], top_p = p[1];
  const int top_k = (int)p[2];
  const float fpen = p[3], ppen = p[4], rpen = p[5];
  const int rwin = (int)p[6];
  const T* x = logits + (size_t)row * ld;
  float* wk = work + (size_t)row * V;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v;
    if constexpr (std::is_same<T, float>::value) v = x[i];
    else v = __bfloat162float(x[i]);
    wk[i] = v;
  }
  __syncthreads();
  // Penalties over the history (prompt + generated), applied once per
  // distinct token with its counts, which equals the reference's
  // per-occurrence loop.
  const int hl = hist_len != nullptr ? hist_len[row] : 0;
  const bool any_pen = (fabsf(rpen - 1.f) > 1.1920929e-07f) || fpen != 0.f || ppen != 0.f;
  if (any_pen && hl > 0) {
    const int* hs = history + (size_t)row * hist_ld;
    const int wstart = (rwin == 0) ? 0 : max(0, hl - rwin);
    for (int j = threadIdx.x; j < hl; j += blockDim.x) {
      const int tok = hs[j];
      bool first = true;
      for (int k = 0; k < j; ++k)
        if (hs[k] == tok) {
          first = false;
          break;
        }
      if (!first || tok < 0 || tok >= V) continue;
      int cnt = 0, cnt_w = 0;
      for (int k = j; k < hl; ++k)
        if (hs[k] == tok) {
          ++cnt;
          if (k >= wstart) ++cnt_w;
        }
      float l = wk[tok];
      if (fabsf(rpen - 1.f) > 1.1920929e-07f) {
        for (int c = 0; c < cnt_w; ++c) l = l > 0.f ? l / rpen : l * rpen;
      }
      l -= fpen * (float)cnt;
      l -= ppen;
      wk[tok] = l;
    }
  }
  __syncthreads();
  // Greedy when temperature <= 0.
  if (temp <= 0.f) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = wk[i];
      if (v > best || (v == best && i < bi)) {
        best = v;
        bi = i;
      }
    }
    const float bmax = block_reduce_max(best, redf);
    int cand = (best == bmax) ? bi : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) redi[threadIdx.x >> 5] = cand;
    __syncthreads();
    if (threadIdx.x < 32) {
      int r = threadIdx.x < (int)(blockDim.x >> 5) ? redi[threadIdx.x] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) r = min(r, __shfl_xor_sync(0xffffffffu, r, o));
      if (threadIdx.x == 0) out[row] = r == 0x7fffffff ? 0 : r;
    }
    return;
  }
  // Softmax with temperature.
  const float inv_t = 1.f / temp;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, wk[i] * inv_t);
  mx = block_reduce_max(mx, redf);
  float sum = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float e = __expf(wk[i] * inv_t - mx);
    wk[i] = e;
    sum += e;
  }
  sum = block_reduce_sum(sum, redf);
  __syncthreads();
  // Keep-threshold: entries with prob >= tau survive (tau = 0 keeps all).
  float tau = 0.f;
  float kept_sum = sum;
  if (top_k > 0 && top_k < V) {
    // k-th largest value: largest tau with count(p >= tau) >= k.
    tau = bit_search([&](float t) {
      int c = 0;
      for (int i = threadIdx.x; i < V; i += blockDim.x) c += wk[i] >= t ? 1 : 0;
      return block_reduce_count(c, redi) >= top_k;
    });
    float s2 = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) s2 += wk[i] >= tau ? wk[i] : 0.f;
    kept_sum = block_reduce_sum(s2, redf);
  }
  if (top_p > 0.f && top_p < 1.f) {
    // Smallest prefix (by descending prob) with mass >= top_p * kept_sum:
    // largest tau2 >= tau with mass(p >= tau2) >= top_p * kept_sum.
    const float target = top_p * kept_sum;
    const float tau_k = tau;
    const float tau2 = bit_search([&](float t) {
      const float tt = fmaxf(t, tau_k);
      float s3 = 0.f;
      for (int i = threadIdx.x; i < V; i += blockDim.x) s3 += wk[i] >= tt ? wk[i] : 0.f;
      return block_reduce_sum(s3, redf) >= target;
    });
    tau = fmaxf(tau, tau2);
    float s4 = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) s4 += wk[i] >= tau ? wk[i] : 0.f;
    kept_sum = block_reduce_sum(s4, redf);
  }
  // Categorical draw in index order (as the reference's cumulative scan).
  __shared__ float s_u;
  if (threadIdx.x == 0) {
    curandStatePhilox4_32_10_t st;
    curand_init((unsigned long long)seeds[row], 0ull, (unsigned long long)offsets[row], &st);
    s_u = curand_uniform(&st) * kept_sum;
  }
  const int chunk = (V + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * chunk;
  const int i1 = min(V, i0 + chunk);
  float local = 0.f;
  for (int i = i0; i < i1; ++i) local += wk[i] >= tau ? wk[i] : 0.f;
  s_scan[threadIdx.x] = local;
  __syncthreads();
  // Inclusive scan (Hillis-Steele) over the per-thread chunk sums.
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    const float v = threadIdx.x >= (unsigned)off ? s_scan[threadIdx.x - off] : 0.f;
    __syncthreads();
    s_scan[threadIdx.x] += v;
    __syncthreads();
  }
  const float u = s_u;
  const float before = threadIdx.x > 0 ? s_scan[threadIdx.x - 1] : 0.f;
  const float after = s_scan[threadIdx.x];
  __shared__ int s_pick;
  if (threadIdx.x == 0) s_pick = -1;
  __syncthreads();
  if (before < u && after >= u) {
    float cum = before;
    int pick = i1 - 1;
    for (int i = i0; i < i1; ++i) {
      const float pv = wk[i] >= tau ? wk[i] : 0.f;
      cum += pv;
      if (cum >= u && pv > 0.f) {
        pick = i;
        break;
      }
    }
    atomicMax(&s_pick, pick);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int r = s_pick;
    if (r < 0) {  // rounding left u beyond the total: last kept token
      r = V - 1;
      while (r > 0 && !(wk[r] >= tau && wk[r] > 0.f)) --r;
    }
    out[row] = r;
  }
}

void sample(torch::Tensor logits, torch::Tensor params, c10::optional<torch::Tensor> history,
            c10::optional<torch::Tensor> hist_len, torch::Tensor work, torch::Tensor seeds,
            torch::Tensor offsets, torch::Tensor out) {
  const int M = (int)logits.size(0);
  const int V = (int)logits.size(1);
  if (M == 0) return;
  TORCH_CHECK(work.numel() >= (int64_t)M * V, "work buffer too small");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int* hs = history.has_value() ? history->data_ptr<int>() : nullptr;
  const int hld = history.has_value() ? (int)history->stride(0) : 0;
  const int* hl = hist_len.has_value() ? hist_len->data_ptr<int>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == at::kFloat) {
    sample_kernel<float><<<M, kSampThreads, 0, stream>>>(
        logits.data_ptr<float>(), (int)logits.stride(0), V, params.data_ptr<float>(), hs, hld, hl,
        work.data_ptr<float>(), seeds.data_ptr<int64_t>(), offsets.data_ptr<int64_t>(),
        out.data_ptr<int>());
  } else {
    sample_kernel<bf16><<<M, kSampThreads, 0, stream>>>(
        reinterpret_cast<const bf16*>(logits.data_ptr()), (int)logits.stride(0), V,
        params.data_ptr<float>(), hs, hld, hl, work.data_ptr<float>(), seeds.data_ptr<int64_t>(),
        offsets.data_ptr<int64_t>(), out.data_ptr<int>());
  }
  CB_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ spec verify
// target: int32 [B, k+1] greedy target tokens for rows [prev, d1..dk];
// draft: int32 [B, k].  out: int32 [B, k+2] = accepted tokens (accepted drafts
// followed by the correction/bonus token), then the count n = accepted + 1 in
// the last column.  One thread per sequence.
__global__ void spec_verify_kernel(const int* __restrict__ target, const int* __restrict__ draft,
                                   int B, int k, int* __restrict__ out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int* t = target + (size_t)b * (k + 1);
  const int* d = draft + (size_t)b * k;
  int* o = out + (size_t)b * (k + 2);
  int acc = 0;
  while (acc < k && d[acc] == t[acc]) {
    o[acc] = d[acc];
    ++acc;
  }
  o[acc] = t[acc];
  for (int i = acc + 1; i < k + 1; ++i) o[i] = -1;
  o[k + 1] = acc + 1;
}

void spec_verify(torch::Tensor target, torch::Tensor draft, torch::Tensor out) {
  const int B = (int)draft.size(0);
  const int k = (int)draft.size(1);
  TORCH_CHECK(target.is_contiguous() && draft.is_contiguous() && out.is_contiguous() &&
                  target.size(0) == B && target.size(1) == k + 1 && out.size(0) == B &&
                  out.size(1) == k + 2,
              "spec_verify: target [B, k+1], draft [B, k], out [B, k+2]");
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(target.device());
  const int threads = 128;
  spec_verify_kernel<<<(B + threads - 1) / threads, threads, 0,
                       at::cuda::getCurrentCUDAStream()>>>(
      target.data_ptr<int>(), draft.data_ptr<int>(), B, k, out.data_ptr<int>());
  CB_CUDA_CHECK(cudaGetLastError());
}

// Fused verify of one speculative round (whole vocabulary on this GPU):
// one CTA per verify row takes the argmax of its logits row (lowest index on
// ties), and the last CTA to finish among a sequence's rows compares the
// drafts with the target's picks, writes out[b] = accepted drafts, the
// correction token, -1 padding and the count (accepted + 1) in column k + 1,
// and sets kv_len[b] += count: the paged-KV length after the round (the
// forward wrote entries for every row; those past the accepted prefix are
// dropped).  picks: int32 [R] scratch; done: int32 [B], zero on entry and
// zero again on exit.
__global__ void __launch_bounds__(1024) spec_verify_fused_kernel(
    const bf16* __restrict__ logits, int ld, int V, const int* __restrict__ row_seq,
    const int* __restrict__ row_start, const int* __restrict__ draft, int k,
    int* __restrict__ picks, int* __restrict__ done, int* __restrict__ kv_len,
    int* __restrict__ out) {
  grid_dep_launch();
  grid_dep_wait();
  const int r = blockIdx.x;
  const bf16* x = logits + (size_t)r * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec_ok = (V % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (vec_ok) {
    for (int i = threadIdx.x * 8; i < V; i += blockDim.x * 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + i);
      const bf16* e = reinterpret_cast<const bf16*>(&u);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float v = __bfloat162float(e[q]);
        if (v > best) {
          best = v;
          bi = i + q;
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = __bfloat162float(x[i]);
      if (v > best) {
        best = v;
        bi = i;
      }
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
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ int s_last;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = l < nw ? sv[l] : -INFINITY;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (l == 0) {
      picks[r] = bi == 0x7fffffff ? 0 : bi;
      __threadfence();
      const int b = row_seq[r];
      const int n = row_start[b + 1] - row_start[b];
      const int old = atomicAdd(&done[b], 1);
      s_last = old == n - 1 ? 1 : 0;
    }
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  const int b = row_seq[r];
  const int r0 = row_start[b];
  const int n = row_start[b + 1] - r0;
  done[b] = 0;  // ready for the next round
  const int* d = draft + (size_t)b * k;
  int* o = out + (size_t)b * (k + 2);
  const volatile int* pk = picks;
  int acc = 0;
  while (acc < n - 1 && d[acc] == pk[r0 + acc]) {
    o[acc] = d[acc];
    ++acc;
  }
  o[acc] = pk[r0 + acc];
  for (int i = acc + 1; i < k + 1; ++i) o[i] = -1;
  o[k + 1] = acc + 1;
  kv_len[b] += acc + 1;
}

void spec_verify_fused(torch::Tensor logits, torch::Tensor row_seq, torch::Tensor row_start,
                       torch::Tensor draft, torch::Tensor picks, torch::Tensor done,
                       torch::Tensor kv_len, torch::Tensor out) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "bf16 logits");
  const int R = (int)logits.size(0);
  const int V = (int)logits.size(1);
  const int B = (int)draft.size(0);
  const int k = (int)draft.size(1);
  TORCH_CHECK(row_seq.numel() >= R && row_start.numel() >= B + 1 && picks.numel() >= R &&
                  done.numel() >= B && kv_len.numel() >= B && out.size(1) == k + 2 &&
                  draft.is_contiguous() && out.is_contiguous(),
              "spec_verify_fused: buffer sizes");
  if (R == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  launch_kernel(spec_verify_fused_kernel, dim3(R), dim3(1024), 0,
                at::cuda::getCurrentCUDAStream(),
                reinterpret_cast<const bf16*>(logits.data_ptr()), (int)logits.stride(0), V,
                row_seq.data_ptr<int>(), row_start.data_ptr<int>(), draft.data_ptr<int>(), k,
                picks.data_ptr<int>(), done.data_ptr<int>(), kv_len.data_ptr<int>(),
                out.data_ptr<int>());
}

}  // namespace cb
