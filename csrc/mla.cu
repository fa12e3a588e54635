// Multi-head latent attention (MLA, DeepSeek-V3 / Kimi-K2 shape) for decode,
// in the absorbed form: every token's cache entry is its normalised latent
// c (kv_lora_rank = 512) followed by its rotated shared rope key (64), one
// 576-wide bf16 row per token instead of per-head K and V.  With
//   q_lat[h] = W_UK[h]^T q_nope[h]   (absorbed on the host side, 512 wide)
// the kernel computes, per head h,
//   s[t] = (q_lat[h] . c[t] + q_rope[h] . k_rope[t]) * scale,
//   o_lat[h] = softmax(s) . c          (512 wide, later multiplied by W_UV[h])
// which equals the reference's per-head attention over expanded K/V
// (crates/cascadia-int4-gemm/src/shell.rs:81-341, non-absorbed).
//
// Cache layout: [layers, blocks, 16 tokens, 576] bf16; inside a block the
// 16-byte chunk j of token row r is stored at chunk j ^ (r & 7), so one bulk
// copy brings a whole block (18 KiB) into shared memory in a layout whose
// ldmatrix reads are bank-conflict free.
//
// Decode kernel: CTA = (16 heads, one sequence, one context split), 4 warps.
// Warp w owns latent/rope dims [144w, 144w + 144) for the scores (partial
// scores summed across warps through shared memory) and latent dims
// [128w, 128w + 128) of the output; every warp keeps the same online-softmax
// state.  Blocks stream through a 3-stage ring (bulk copies, bounded waits).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"
#include "mma_frag.cuh"

namespace cb {

namespace {

using bf16 = __nv_bfloat16;
constexpr int kLat = 512;
constexpr int kRope = 64;
constexpr int kRow = kLat + kRope;        // 576 values per token
constexpr int kRowBytes = kRow * 2;       // 1152
constexpr int kBlockBytes = 16 * kRowBytes;  // 18432
constexpr int kStages = 3;
constexpr float kNegBigM = -1e30f;

__device__ __forceinline__ uint32_t mla_off(int row, int chunk) {
  return (uint32_t)(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------------ rope + cache write
// Per token t: rotate the rope part of the shared key (interleaved pairs:
// (x[2i], x[2i+1]) by angle i -- the same dot products as the reference's
// de-interleave + rotate-half) and of every head's query, write the cache
// row [c (normalised latent) | rotated key] into the paged cache (swizzled),
// and write the rotated query rope into q_out[:, h, 512:576].
__global__ void mla_rope_write_kernel(const bf16* __restrict__ ckv, int ld_ckv,
                                      const bf16* __restrict__ kr, int ld_kr,
                                      const bf16* __restrict__ qrope, int ld_q, int q_head_stride,
                                      bf16* __restrict__ q_out, const int* __restrict__ positions,
                                      const float* __restrict__ cos_sin, const int* __restrict__ slots,
                                      bf16* __restrict__ cache, int layer, int NB, int heads) {
  const int t = blockIdx.x;
  const int pos = positions[t];
  const int slot = slots[t];
  const float* cs = cos_sin + (size_t)pos * kRope;  // [cos 32 | sin 32]
  // Query rope parts: heads x 32 pairs.
  for (int idx = threadIdx.x; idx < heads * (kRope / 2); idx += blockDim.x) {
    const int h = idx / (kRope / 2), i = idx % (kRope / 2);
    const bf16* src = qrope + (size_t)t * ld_q + (size_t)h * q_head_stride + 2 * i;
    const float x0 = __bfloat162float(src[0]), x1 = __bfloat162float(src[1]);
    const float c = cs[i], s = cs[kRope / 2 + i];
    bf16* dst = q_out + ((size_t)t * heads + h) * kRow + kLat + 2 * i;
    dst[0] = __float2bfloat16(x0 * c - x1 * s);
    dst[1] = __float2bfloat16(x1 * c + x0 * s);
  }
  if (slot < 0) return;
  uint8_t* blk = reinterpret_cast<uint8_t*>(cache) +
                 ((size_t)layer * NB + slot / 16) * kBlockBytes;
  const int r = slot % 16;
  // Latent: 64 chunks of 8 values.
  for (int j = threadIdx.x; j < kLat / 8; j += blockDim.x) {
    const uint4 v = *reinterpret_cast<const uint4*>(ckv + (size_t)t * ld_ckv + j * 8);
    *reinterpret_cast<uint4*>(blk + mla_off(r, j)) = v;
  }
  // Rope key: 8 chunks (threads 0..7), each rotates 4 pairs.
  if (threadIdx.x < kRope / 8) {
    const int j = threadIdx.x;
    const bf16* src = kr + (size_t)t * ld_kr + j * 8;
    uint4 o;
    bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int i = j * 4 + p;
      const float x0 = __bfloat162float(src[2 * p]), x1 = __bfloat162float(src[2 * p + 1]);
      const float c = cs[i], s = cs[kRope / 2 + i];
      oe[2 * p] = __float2bfloat16(x0 * c - x1 * s);
      oe[2 * p + 1] = __float2bfloat16(x1 * c + x0 * s);
    }
    *reinterpret_cast<uint4*>(blk + mla_off(r, kLat / 8 + j)) = o;
  }
}

// ------------------------------------------------------------------ decode
struct MlaArgs {
  const bf16* q;            // [B, heads, 576]
  const bf16* cache;        // [L, NB, 16, 576] swizzled
  const int* block_tables;  // [B, bt_stride]
  const int* seq_lens;      // [B]
  bf16* out;                // [B, heads, 512]
  float* part_o;            // [B, heads, splits, 512]
  float* part_ml;           // [B, heads, splits, 2]
  int* status;
  int heads, bt_stride, NB, layer, splits, blocks_per_split;
  float scale_log2;
  // Optional DSA selection: position p of sequence b is attended only if
  // sel[b * sel_ld + p] >= sel_thr[b] (its indexer score reaches the top-k
  // threshold).  nullptr: dense attention.
  const float* sel;
  int sel_ld;
  const float* sel_thr;
};

__global__ void __launch_bounds__(128) mla_decode_kernel(const MlaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;                                              // kStages blocks
  float* s_part = reinterpret_cast<float*>(smem + kStages * kBlockBytes);  // [2][4][16][16]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_part + 2 * 4 * 256);
  uint64_t* empty = full + kStages;
  const int hg = blockIdx.x, b = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int seq_len = a.seq_lens[b];
  const int nblk = (seq_len + 15) / 16;
  const int blk0 = sp * a.blocks_per_split;
  const int my_n = max(0, min(a.blocks_per_split, nblk - blk0));
  const int* bt = a.block_tables + (size_t)b * a.bt_stride;
  const uint8_t* cache_l = reinterpret_cast<const uint8_t*>(a.cache) + (size_t)a.layer * a.NB * kBlockBytes;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < my_n && i < kStages; ++i) {
      mbar_arrive_expect_tx(&full[i], kBlockBytes);
      bulk_g2s(ring + i * kBlockBytes, cache_l + (size_t)bt[blk0 + i] * kBlockBytes,
               kBlockBytes, &full[i]);
    }
  }

  // Query fragments of this warp's 144 score dims (9 k-steps), heads padded to 16.
  const int h_lo = hg * 16;
  uint32_t qa[9][4];
  {
    const bf16* qb = a.q + ((size_t)b * a.heads + h_lo) * kRow;
    const bool r0 = h_lo + g < a.heads, r1 = h_lo + g + 8 < a.heads;
#pragma unroll
    for (int ks = 0; ks < 9; ++ks) {
      const int c0 = warp * 144 + ks * 16 + 2 * t4;
      qa[ks][0] = r0 ? *reinterpret_cast<const uint32_t*>(qb + g * kRow + c0) : 0u;
      qa[ks][1] = r1 ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * kRow + c0) : 0u;
      qa[ks][2] = r0 ? *reinterpret_cast<const uint32_t*>(qb + g * kRow + c0 + 8) : 0u;
      qa[ks][3] = r1 ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * kRow + c0 + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {kNegBigM, kNegBigM};
  float l[2] = {0.f, 0.f};
  bool ok = true;

  for (int i = 0; i < my_n; ++i) {
    const int st = i % kStages;
    if (ok && !mbar_wait(&full[st], (i / kStages) & 1, a.status, kStatusAttnTimeout, nullptr))
      ok = false;
    const uint32_t base = smem_u32(ring + st * kBlockBytes);
    // Partial scores over this warp's dims.
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    if (ok) {
#pragma unroll
      for (int ks = 0; ks < 9; ++ks) {
        const int row = ((lane >> 4) << 3) + (lane & 7);
        const int chunk = 2 * (warp * 9 + ks) + ((lane >> 3) & 1);
        uint32_t b00, b01, b10, b11;
        ldsm_x4(base + mla_off(row, chunk), b00, b01, b10, b11);
        mma_16816(s[0], qa[ks], b00, b01);
        mma_16816(s[1], qa[ks], b10, b11);
      }
    }
    float* sp_buf = s_part + (i & 1) * 4 * 256 + warp * 256;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = g + 8 * (e >> 1), col = nt * 8 + 2 * t4 + (e & 1);
        sp_buf[row * 16 + col] = s[nt][e];
      }
    __syncthreads();
    const float* tot = s_part + (i & 1) * 4 * 256;
    const int pos0 = (blk0 + i) * 16;
    float p[2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = kNegBigM;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int row = g + 8 * r, col = nt * 8 + 2 * t4 + e;
          float v = (tot[row * 16 + col] + tot[256 + row * 16 + col] + tot[512 + row * 16 + col] +
                     tot[768 + row * 16 + col]) * a.scale_log2;
          const bool keep =
              pos0 + col < seq_len &&
              (a.sel == nullptr || a.sel[(size_t)b * a.sel_ld + pos0 + col] >= a.sel_thr[b]);
          v = keep ? v : -INFINITY;
          s[nt][2 * r + e] = v;
          mx = fmaxf(mx, v);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m[r], mx);
      const float alpha = exp2f(m[r] - m_new);
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = exp2f(s[nt][2 * r + e] - m_new);
          p[nt][2 * r + e] = pv;
          sum += pv;
        }
      l[r] = l[r] * alpha + sum;
      m[r] = m_new;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        o[nt][2 * r] *= alpha;
        o[nt][2 * r + 1] *= alpha;
      }
    }
    uint32_t pa[4];
    pa[0] = pack_bf16(p[0][0], p[0][1]);
    pa[1] = pack_bf16(p[0][2], p[0][3]);
    pa[2] = pack_bf16(p[1][0], p[1][1]);
    pa[3] = pack_bf16(p[1][2], p[1][3]);
    if (ok) {
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        const int mi = lane >> 3;
        const int row = ((mi & 1) << 3) + (lane & 7);
        const int chunk = 16 * warp + 2 * np + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(base + mla_off(row, chunk), b0, b1, b2, b3);
        mma_16816(o[2 * np], pa, b0, b1);
        mma_16816(o[2 * np + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (threadIdx.x == 0 && i + kStages < my_n) {
      // Refill this stage once all four warps have read it.
      if (ok && mbar_wait(&empty[st], (i / kStages) & 1, a.status, kStatusAttnTimeout, nullptr)) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[st], kBlockBytes);
        bulk_g2s(ring + st * kBlockBytes, cache_l + (size_t)bt[blk0 + i + kStages] * kBlockBytes,
                 kBlockBytes, &full[st]);
      } else {
        ok = false;
      }
    }
    __syncwarp();  // lane 0 of warp 0 may have waited above: reconverge before ldmatrix / mma
  }
  // Never leave with copies in flight (bounded; matters on the error path).
  if (threadIdx.x == 0 && !ok) {
    for (int i = max(0, my_n - kStages); i < my_n; ++i)
      mbar_wait(&full[i % kStages], (i / kStages) & 1, nullptr, 0, nullptr);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int h = h_lo + g + 8 * r;
    if (h >= a.heads) continue;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int d = warp * 128 + nt * 8 + 2 * t4;
      if (a.splits == 1) {
        const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
        *reinterpret_cast<uint32_t*>(a.out + ((size_t)b * a.heads + h) * kLat + d) =
            pack_bf16(o[nt][2 * r] * inv, o[nt][2 * r + 1] * inv);
      } else {
        const size_t base = ((size_t)b * a.heads + h) * a.splits + sp;
        a.part_o[base * kLat + d] = o[nt][2 * r];
        a.part_o[base * kLat + d + 1] = o[nt][2 * r + 1];
        if (warp == 0 && nt == 0 && t4 == 0) {
          a.part_ml[base * 2] = m[r];
          a.part_ml[base * 2 + 1] = l[r];
        }
      }
    }
  }
}

__global__ void mla_combine_kernel(const float* __restrict__ part_o,
                                   const float* __restrict__ part_ml, bf16* __restrict__ out,
                                   int heads, int splits) {
  const int b = blockIdx.x, h = blockIdx.y;
  const size_t base0 = ((size_t)b * heads + h) * splits;
  float M = kNegBigM;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(base0 + s) * 2]);
  for (int d = threadIdx.x; d < kLat; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float w = exp2f(part_ml[(base0 + s) * 2] - M);
      L += part_ml[(base0 + s) * 2 + 1] * w;
      O += part_o[(base0 + s) * kLat + d] * w;
    }
    out[((size_t)b * heads + h) * kLat + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
  }
}

}  // namespace

void mla_rope_write(torch::Tensor ckv, torch::Tensor kr, torch::Tensor qrope,
                    int64_t q_head_stride, torch::Tensor q_out, torch::Tensor positions,
                    torch::Tensor cos_sin, torch::Tensor slots, torch::Tensor cache,
                    int64_t layer, int64_t heads) {
  const int T = (int)ckv.size(0);
  if (T == 0) return;
  TORCH_CHECK(ckv.size(1) == kLat && kr.size(1) == kRope && cos_sin.size(1) == kRope,
              "MLA shapes: latent 512, rope 64");
  TORCH_CHECK(cache.size(-1) == kRow && cache.size(-2) == 16, "cache [L, NB, 16, 576]");
  TORCH_CHECK((ckv.stride(0) * 2) % 16 == 0 && ckv.stride(1) == 1, "latent rows 16-byte aligned");
  const c10::cuda::CUDAGuard guard(ckv.device());
  mla_rope_write_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(ckv.data_ptr()), (int)ckv.stride(0),
      reinterpret_cast<const bf16*>(kr.data_ptr()), (int)kr.stride(0),
      reinterpret_cast<const bf16*>(qrope.data_ptr()), (int)qrope.stride(0), (int)q_head_stride,
      reinterpret_cast<bf16*>(q_out.data_ptr()), positions.data_ptr<int>(),
      cos_sin.data_ptr<float>(), slots.data_ptr<int>(), reinterpret_cast<bf16*>(cache.data_ptr()),
      (int)layer, (int)cache.size(1), (int)heads);
  CB_CUDA_CHECK(cudaGetLastError());
}

void mla_decode(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables,
                torch::Tensor seq_lens, torch::Tensor out, int64_t layer, int64_t num_splits,
                int64_t blocks_per_split, torch::Tensor part_o, torch::Tensor part_ml,
                double scale, torch::Tensor status, c10::optional<torch::Tensor> sel,
                c10::optional<torch::Tensor> sel_thr) {
  const int B = (int)q.size(0);
  const int heads = (int)q.size(1);
  TORCH_CHECK(q.size(2) == kRow && q.is_contiguous(), "q [B, heads, 576] contiguous");
  TORCH_CHECK(out.is_contiguous() && out.size(2) == kLat, "out [B, heads, 512]");
  if (B == 0) return;
  MlaArgs a{};
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.cache = reinterpret_cast<const bf16*>(cache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.seq_lens = seq_lens.data_ptr<int>();
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.part_o = num_splits > 1 ? part_o.data_ptr<float>() : nullptr;
  a.part_ml = num_splits > 1 ? part_ml.data_ptr<float>() : nullptr;
  a.status = status.data_ptr<int>();
  a.heads = heads;
  a.bt_stride = (int)block_tables.stride(0);
  a.NB = (int)cache.size(1);
  a.layer = (int)layer;
  a.splits = (int)num_splits;
  a.blocks_per_split = (int)blocks_per_split;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  if (sel.has_value()) {
    TORCH_CHECK(sel_thr.has_value() && sel->scalar_type() == at::kFloat && sel->stride(1) == 1 &&
                    sel->size(0) >= B && sel_thr->scalar_type() == at::kFloat &&
                    sel_thr->numel() >= B,
                "DSA selection: fp32 scores [B, >= max len] and thresholds [B]");
    a.sel = sel->data_ptr<float>();
    a.sel_ld = (int)sel->stride(0);
    a.sel_thr = sel_thr->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int smem = kStages * kBlockBytes + 2 * 4 * 256 * 4 + 2 * kStages * 8;
  static int configured[64] = {};
  int dev = 0;
  CB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(mla_decode_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  const dim3 grid((heads + 15) / 16, B, (unsigned)num_splits);
  mla_decode_kernel<<<grid, 128, smem, stream>>>(a);
  CB_CUDA_CHECK(cudaGetLastError());
  if (num_splits > 1) {
    mla_combine_kernel<<<dim3(B, heads), 128, 0, stream>>>(a.part_o, a.part_ml, a.out, heads,
                                                          (int)num_splits);
    CB_CUDA_CHECK(cudaGetLastError());
  }
}

// ---------------------------------------------------------------- DSA indexer
// Lightning-indexer scores of the DSA sparse attention (GLM-5; reference
// glm/indexer.rs:50-190): for query token t and every position p of its
// sequence,  score[t, p] = sum_h w[t, h] * relu(q[t, h, :] . k[p, :]),
// with the per-head weights w already holding the softmax and head-count
// scales.  Keys come from the paged index-key cache [L, NB, 16, D]; positions
// at or past the token's length score -inf.  One thread per position; the
// token's H x D query is staged in shared memory as fp32.
constexpr int kDsaMaxHeads = 64;
constexpr int kDsaD = 128;

struct DsaArgs {
  const bf16* q;          // [T, H, D]
  const float* w;         // [T, H]
  const bf16* kcache;     // [L, NB, 16, D]
  const int* block_tables;
  int bt_stride;
  const int* lens;        // [T]
  float* out;             // [T, ld]
  int ld, H, NB, layer;
};

__global__ void __launch_bounds__(128) dsa_scores_kernel(const DsaArgs a) {
  __shared__ __align__(16) float qs[kDsaMaxHeads * kDsaD];
  __shared__ float ws[kDsaMaxHeads];
  grid_dep_launch();
  grid_dep_wait();
  const int t = blockIdx.y;
  const int p = blockIdx.x * 128 + threadIdx.x;
  for (int i = threadIdx.x; i < a.H * kDsaD; i += 128)
    qs[i] = __bfloat162float(a.q[(size_t)t * a.H * kDsaD + i]);
  if (threadIdx.x < a.H) ws[threadIdx.x] = a.w[(size_t)t * a.H + threadIdx.x];
  __syncthreads();
  if (p >= a.ld) return;
  const int len = a.lens[t];
  if (p >= len) {
    a.out[(size_t)t * a.ld + p] = -INFINITY;
    return;
  }
  const int blk = a.block_tables[(size_t)t * a.bt_stride + p / 16];
  const bf16* kp = a.kcache + (((size_t)a.layer * a.NB + blk) * 16 + (p % 16)) * kDsaD;
  float acc[kDsaMaxHeads];
#pragma unroll
  for (int h = 0; h < kDsaMaxHeads; ++h) acc[h] = 0.f;
#pragma unroll 1
  for (int c = 0; c < kDsaD / 8; ++c) {
    const uint4 kv = *reinterpret_cast<const uint4*>(kp + c * 8);
    const bf16* ke = reinterpret_cast<const bf16*>(&kv);
    float k8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) k8[e] = __bfloat162float(ke[e]);
#pragma unroll
    for (int h = 0; h < kDsaMaxHeads; ++h) {
      if (h < a.H) {
        const float4 q0 = *reinterpret_cast<const float4*>(&qs[h * kDsaD + c * 8]);
        const float4 q1 = *reinterpret_cast<const float4*>(&qs[h * kDsaD + c * 8 + 4]);
        acc[h] += q0.x * k8[0] + q0.y * k8[1] + q0.z * k8[2] + q0.w * k8[3] + q1.x * k8[4] +
                  q1.y * k8[5] + q1.z * k8[6] + q1.w * k8[7];
      }
    }
  }
  float sc = 0.f;
#pragma unroll
  for (int h = 0; h < kDsaMaxHeads; ++h)
    if (h < a.H) sc += ws[h] * fmaxf(acc[h], 0.f);
  a.out[(size_t)t * a.ld + p] = sc;
}

void dsa_scores(torch::Tensor q, torch::Tensor w, torch::Tensor kcache, torch::Tensor block_tables,
                torch::Tensor lens, torch::Tensor out, int64_t layer) {
  const int T = (int)q.size(0);
  const int H = (int)q.size(1);
  TORCH_CHECK(q.is_contiguous() && q.size(2) == kDsaD && H <= kDsaMaxHeads,
              "indexer q must be [T, H <= 64, 128] contiguous bf16");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.size(1) == H, "w [T, H] fp32");
  TORCH_CHECK(kcache.is_contiguous() && kcache.size(3) == kDsaD && kcache.size(2) == 16,
              "index-key cache [L, NB, 16, 128]");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.stride(1) == 1 && out.size(0) >= T,
              "out [T, ld] fp32");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && lens.scalar_type() == at::kInt, "int32");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  DsaArgs a;
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.w = w.data_ptr<float>();
  a.kcache = reinterpret_cast<const bf16*>(kcache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = (int)block_tables.stride(0);
  a.lens = lens.data_ptr<int>();
  a.out = out.data_ptr<float>();
  a.ld = (int)out.size(1);
  a.H = H;
  a.NB = (int)kcache.size(1);
  a.layer = (int)layer;
  launch_kernel(dsa_scores_kernel, dim3((unsigned)((a.ld + 127) / 128), (unsigned)T), dim3(128),
                0, at::cuda::getCurrentCUDAStream(), a);
}

}  // namespace cb
