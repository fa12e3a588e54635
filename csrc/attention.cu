// Paged-KV attention kernels for sm_100a.
//
// KV cache layout (one tensor each for K and V, all layers):
//   [num_layers, num_blocks, num_kv_heads, 16, head_dim] bf16
// so that one (layer, block, kv-head) is a contiguous 16 x head_dim tile that a
// 2-D TMA tensor map (rows = layer*blocks*heads*16 + ..., cols = head_dim,
// 128-byte swizzle, box 64 x 16) fetches straight into a bank-conflict-free
// shared-memory layout.  This replaces the reference's host-side KV ring and
// OpenVINO stateful SDPA (crates/cascadia-engine-openvino/src/runtime.rs:1067-1236,
// tools/export_shards.py:657 cached_layer_forward_sdpa) with a device block table.
//
// * attn_decode: flash-decoding.  Grid (kv_head, seq, split); each warp streams
//   its own K/V blocks through a 2-stage TMA ring and all query heads of the
//   GQA group share every K/V byte.  Splits (when the batch is too small to
//   fill the GPU) are merged by attn_decode_combine.
// * attn_prefill: causal flash attention over ragged prompts reading K/V from
//   the same paged cache (so chunked prefill and prefix reuse work unchanged).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"
#include "mma_frag.cuh"

namespace cb {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1e30f;

struct DecodeArgs {
  const __nv_bfloat16* q;
  int q_stride;  // elements between consecutive sequences' q rows
  const int* block_tables;
  int bt_stride;
  const int* seq_lens;
  __nv_bfloat16* out;
  int out_stride;
  float* part_o;   // [B, Hkv, S, G, D]
  float* part_ml;  // [B, Hkv, S, G, 2]
  int* status;
  int Hkv, G, NB;
  int layer;
  int blocks_per_split, splits;
  float scale_log2;
  // Sliding window (0: none): a query at position q sees keys k with
  // q - window < k <= q, plus the first `sinks` positions (attention sinks).
  int window, sinks;
};

// Visible 16-token blocks of a window: the sink blocks [0, nsb) then the
// window blocks from wb0 on; virtual block v maps to block block_of(v).
struct VisibleBlocks {
  int nsb, wb0, n;
  __device__ __forceinline__ int block_of(int v) const { return v < nsb ? v : wb0 + (v - nsb); }
};

__device__ __forceinline__ VisibleBlocks visible_blocks(int first_visible, int total_blocks,
                                                        int window, int sinks) {
  VisibleBlocks vb;
  if (window <= 0) {
    vb.nsb = total_blocks;
    vb.wb0 = total_blocks;
    vb.n = total_blocks;
    return vb;
  }
  vb.wb0 = min(total_blocks, max(0, first_visible) >> 4);
  vb.nsb = min((sinks + 15) >> 4, vb.wb0);
  vb.n = vb.nsb + (total_blocks - vb.wb0);
  return vb;
}

// D: head dim (q.k and the cache rows).  DV: output dims one CTA produces;
// DV < D splits the output of a head over D / DV CTAs (head_dim 512: two
// CTAs each compute all scores and half of the output), blockIdx.z =
// split * (D / DV) + half.
// WIN: a sliding window / sinks may hide positions (compiled out otherwise).
template <int D, int DV = D, bool WIN = false>
__global__ void __launch_bounds__(128) attn_decode_kernel(const __grid_constant__ CUtensorMap tk,
                                                          const __grid_constant__ CUtensorMap tv,
                                                          const DecodeArgs a) {
  constexpr int KV_BYTES = 16 * D * 2;   // one block of K
  constexpr int V_BYTES = 16 * DV * 2;   // this CTA's slice of one block of V
  constexpr int STAGE = KV_BYTES + V_BYTES;
  constexpr int NKS = D / 16;
  constexpr int HALVES = D / DV;
  // head_dim >= 256: Q fragments come from shared memory per k-step (the
  // output accumulators alone take 128 registers).
  constexpr bool QS = D > 128;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int sp = blockIdx.z / HALVES;
  const int half = blockIdx.z % HALVES;
  uint8_t* wbuf = smem + warp * 2 * STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 4 * 2 * STAGE);
  uint64_t* full = bars + warp * 2;
  uint8_t* qsm = smem + 4 * 2 * STAGE + 128;  // [16][D] bf16, chunk-swizzled (QS)
  grid_dep_launch();
  grid_dep_wait();  // q, the cache rows and the lengths come from earlier kernels

  const int seq_len = a.seq_lens[b];
  // The query is at position seq_len - 1: with a window it sees positions
  // from seq_len - window on (and the sinks).
  const VisibleBlocks vis = visible_blocks(seq_len - a.window, (seq_len + 15) >> 4,
                                           WIN ? a.window : 0, a.sinks);
  const int nblocks = vis.n;
  const int blk0 = sp * a.blocks_per_split;
  const int blk1 = min(nblocks, blk0 + a.blocks_per_split);
  // This warp handles blocks blk0 + warp, blk0 + warp + 4, ...
  const int my_n = blk1 > blk0 + warp ? (blk1 - blk0 - warp + 3) / 4 : 0;

  if (lane == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int* bt = a.block_tables + (size_t)b * a.bt_stride;
  const int row_base_layer = a.layer * a.NB;
  auto issue = [&](int i, int st) {
    const int j = WIN ? vis.block_of(blk0 + warp + 4 * i) : blk0 + warp + 4 * i;
    const int phys = bt[j];
    const int row = ((row_base_layer + phys) * a.Hkv + h) * 16;
    uint8_t* kb = wbuf + st * STAGE;
    mbar_arrive_expect_tx(&full[st], STAGE);
#pragma unroll
    for (int bx = 0; bx < D / 64; ++bx) tma_load_2d(kb + bx * 16 * 128, &tk, bx * 64, row, &full[st]);
#pragma unroll
    for (int bx = 0; bx < DV / 64; ++bx)
      tma_load_2d(kb + KV_BYTES + bx * 16 * 128, &tv, half * DV + bx * 64, row, &full[st]);
  };
  if (lane == 0) {
    if (my_n > 0) issue(0, 0);
    if (my_n > 1) issue(1, 1);
  }

  const int g = lane >> 2;
  const int t4 = lane & 3;
  // Q fragments (rows = query heads of the group, padded to 16).
  uint32_t qa[QS ? 1 : NKS][4];
  {
    const __nv_bfloat16* qb = a.q + (size_t)b * a.q_stride + (size_t)h * a.G * D;
    if constexpr (QS) {
      for (int idx = threadIdx.x; idx < 16 * (D / 8); idx += 128) {
        const int r = idx / (D / 8), c = idx % (D / 8);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < a.G) v = *reinterpret_cast<const uint4*>(qb + r * D + c * 8);
        *reinterpret_cast<uint4*>(qsm + r * D * 2 + (((c & ~7) | ((c & 7) ^ (r & 7))) << 4)) = v;
      }
      __syncthreads();
    } else {
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        const int c0 = ks * 16 + 2 * t4;
        qa[ks][0] = g < a.G ? *reinterpret_cast<const uint32_t*>(qb + g * D + c0) : 0u;
        qa[ks][1] = g + 8 < a.G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + c0) : 0u;
        qa[ks][2] = g < a.G ? *reinterpret_cast<const uint32_t*>(qb + g * D + c0 + 8) : 0u;
        qa[ks][3] =
            g + 8 < a.G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + c0 + 8) : 0u;
      }
    }
  }

  float o[DV / 8][4];
#pragma unroll
  for (int i = 0; i < DV / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {kNegBig, kNegBig};
  float l[2] = {0.f, 0.f};
  bool ok = true;

  for (int i = 0; i < my_n && ok; ++i) {
    const int st = i & 1;
    if (!mbar_wait(&full[st], (i >> 1) & 1, a.status, kStatusAttnTimeout, nullptr)) {
      ok = false;
      break;
    }
    const uint32_t kaddr = smem_u32(wbuf + st * STAGE);
    const uint32_t vaddr = kaddr + KV_BYTES;
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks) {
      const int row = ((lane >> 4) << 3) + (lane & 7);
      const int chunk = 2 * ks + ((lane >> 3) & 1);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(kaddr + sw128_off(row, chunk, 16), b00, b01, b10, b11);
      if constexpr (QS) {
        uint32_t qf[4];
        const int qr = (lane & 7) + (((lane >> 3) & 1) << 3);
        const int qc = 2 * ks + (lane >> 4);
        ldsm_x4(smem_u32(qsm) + qr * D * 2 + (((qc & ~7) | ((qc & 7) ^ (qr & 7))) << 4), qf[0],
                qf[1], qf[2], qf[3]);
        mma_16816(s[0], qf, b00, b01);
        mma_16816(s[1], qf, b10, b11);
      } else {
        mma_16816(s[0], qa[ks], b00, b01);
        mma_16816(s[1], qa[ks], b10, b11);
      }
    }
    const int j = WIN ? vis.block_of(blk0 + warp + 4 * i) : blk0 + warp + 4 * i;
    const int pos0 = j * 16;
    float p[2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = kNegBig;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int pos = pos0 + nt * 8 + 2 * t4 + e;
          float v = s[nt][2 * r + e] * a.scale_log2;
          const bool seen =
              pos < seq_len && (!WIN || pos >= seq_len - a.window || pos < a.sinks);
          v = seen ? v : -INFINITY;
          s[nt][2 * r + e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m[r], mx);
      const float alpha = exp2f(m[r] - m_new);
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = exp2f(s[nt][2 * r + e] - m_new);
          p[nt][2 * r + e] = pv;
          sum += pv;
        }
      }
      l[r] = l[r] * alpha + sum;
      m[r] = m_new;
#pragma unroll
      for (int nt = 0; nt < DV / 8; ++nt) {
        o[nt][2 * r] *= alpha;
        o[nt][2 * r + 1] *= alpha;
      }
    }
    uint32_t pa[4];
    pa[0] = pack_bf16(p[0][0], p[0][1]);
    pa[1] = pack_bf16(p[0][2], p[0][3]);
    pa[2] = pack_bf16(p[1][0], p[1][1]);
    pa[3] = pack_bf16(p[1][2], p[1][3]);
#pragma unroll
    for (int np = 0; np < DV / 16; ++np) {
      const int mi = lane >> 3;
      const int row = ((mi & 1) << 3) + (lane & 7);
      const int chunk = 2 * np + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vaddr + sw128_off(row, chunk, 16), b0, b1, b2, b3);
      mma_16816(o[2 * np], pa, b0, b1);
      mma_16816(o[2 * np + 1], pa, b2, b3);
    }
    __syncwarp();
    if (lane == 0 && i + 2 < my_n) {
      fence_proxy_async_smem();
      issue(i + 2, st);
    }
  }
  // Drain outstanding loads of this warp (error path only).
  if (!ok && lane == 0) {
    for (int i = 0; i < my_n && i < 2; ++i) mbar_wait(&full[i], 0, nullptr, 0, nullptr);
  }
  // Row sums across the quad.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
  __syncthreads();
  // Cross-warp merge through shared memory (reuse the stage buffers).
  float* sm_o = reinterpret_cast<float*>(smem);          // [4][16][DV]
  float* sm_ml = sm_o + 4 * 16 * DV;                     // [4][16][2]
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g + 8 * r;
#pragma unroll
    for (int nt = 0; nt < DV / 8; ++nt) {
      sm_o[(warp * 16 + row) * DV + nt * 8 + 2 * t4] = o[nt][2 * r];
      sm_o[(warp * 16 + row) * DV + nt * 8 + 2 * t4 + 1] = o[nt][2 * r + 1];
    }
    if (t4 == 0) {
      sm_ml[(warp * 16 + row) * 2] = m[r];
      sm_ml[(warp * 16 + row) * 2 + 1] = l[r];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < a.G * DV; idx += 128) {
    const int gg = idx / DV;
    const int d = idx % DV;
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[(w * 16 + gg) * 2]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float wt = exp2f(sm_ml[(w * 16 + gg) * 2] - M);
      L += sm_ml[(w * 16 + gg) * 2 + 1] * wt;
      O += sm_o[(w * 16 + gg) * DV + d] * wt;
    }
    if (a.splits == 1) {
      const float y = L > 0.f ? O / L : 0.f;
      a.out[(size_t)b * a.out_stride + (size_t)(h * a.G + gg) * D + half * DV + d] =
          __float2bfloat16(y);
    } else {
      const size_t base = (((size_t)b * a.Hkv + h) * a.splits + sp) * a.G + gg;
      a.part_o[base * D + half * DV + d] = O;
      if (d == 0) {
        a.part_ml[base * 2] = M;
        a.part_ml[base * 2 + 1] = L;
      }
    }
  }
}

template <int D>
__global__ void attn_decode_combine_kernel(const float* __restrict__ part_o,
                                           const float* __restrict__ part_ml,
                                           __nv_bfloat16* __restrict__ out, int out_stride, int Hkv,
                                           int G, int splits) {
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.x;
  const int hq = blockIdx.y;
  const int h = hq / G;
  const int gg = hq % G;
  const int d = threadIdx.x;
  float M = kNegBig;
  for (int s = 0; s < splits; ++s) {
    const size_t base = (((size_t)b * Hkv + h) * splits + s) * G + gg;
    M = fmaxf(M, part_ml[base * 2]);
  }
  float L = 0.f, O = 0.f;
  for (int s = 0; s < splits; ++s) {
    const size_t base = (((size_t)b * Hkv + h) * splits + s) * G + gg;
    const float w = exp2f(part_ml[base * 2] - M);
    L += part_ml[base * 2 + 1] * w;
    O += part_o[base * D + d] * w;
  }
  out[(size_t)b * out_stride + (size_t)hq * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
}

// ---------------------------------------------------------------- prefill

struct PrefillArgs {
  const __nv_bfloat16* q;  // [T, Hq, D] (row stride q_stride elements per token)
  int q_stride;
  const int4* tiles;       // per q tile: {seq, first q row, position of first row, rows}
  const int* block_tables;
  int bt_stride;
  __nv_bfloat16* out;      // [T, Hq, D] (row stride out_stride)
  int out_stride;
  int* status;
  int Hq, Hkv, G, NB, layer;
  float scale_log2;
  int window, sinks;  // as in DecodeArgs
};

// One CTA = 64 query rows (4 warps x 16) of one query head.  K/V tiles of 64
// tokens (4 paged blocks) stream through a 2-stage TMA ring.
template <int D, bool WIN = false>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const __grid_constant__ CUtensorMap tk,
                                                           const __grid_constant__ CUtensorMap tv,
                                                           const PrefillArgs a) {
  constexpr int BLK_BYTES = 16 * D * 2;
  constexpr int TILE_BYTES = 4 * BLK_BYTES;  // 64 tokens
  constexpr int STAGE = 2 * TILE_BYTES;      // K and V
  constexpr int NKS = D / 16;
  constexpr bool QS = D > 128;               // Q fragments from shared memory
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * STAGE);
  uint8_t* qsm = smem + 2 * STAGE + 128;     // [64][D] bf16, chunk-swizzled (QS)
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int hq = blockIdx.y;
  const int h = hq / a.G;
  grid_dep_launch();
  grid_dep_wait();
  const int4 tinfo = a.tiles[blockIdx.x];
  const int b = tinfo.x, qrow0 = tinfo.y, pos0 = tinfo.z, nq = tinfo.w;
  const int kv_len = pos0 + nq;  // causal: the last query sees everything before it
  // 64-token tiles with something visible to this tile's queries (with a
  // window, the first query pos0 sees from pos0 - window + 1 on).
  const int all_tiles = (kv_len + 63) / 64;
  int nst = all_tiles, wt0 = all_tiles;
  if (WIN && a.window > 0) {
    wt0 = min(all_tiles, max(0, pos0 - a.window + 1) / 64);
    nst = min((a.sinks + 63) / 64, wt0);
  }
  const int ntiles = (WIN && a.window > 0) ? nst + (all_tiles - wt0) : all_tiles;
  auto tile_of = [&](int v) { return v < nst ? v : wt0 + (v - nst); };
  const int* bt = a.block_tables + (size_t)b * a.bt_stride;

  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int vt, int st) {
    const int ti = tile_of(vt);
    uint8_t* base = smem + st * STAGE;
    const int nblk = min(4, ((kv_len - ti * 64) + 15) / 16);
    mbar_arrive_expect_tx(&full[st], nblk * 2 * BLK_BYTES);
    for (int k = 0; k < nblk; ++k) {
      const int phys = bt[ti * 4 + k];
      const int row = ((a.layer * a.NB + phys) * a.Hkv + h) * 16;
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) {
        tma_load_2d(base + k * BLK_BYTES + bx * 16 * 128, &tk, bx * 64, row, &full[st]);
        tma_load_2d(base + TILE_BYTES + k * BLK_BYTES + bx * 16 * 128, &tv, bx * 64, row,
                    &full[st]);
      }
    }
  };
  if (threadIdx.x == 0) {
    issue(0, 0);
    if (ntiles > 1) issue(1, 1);
  }

  const int g = lane >> 2;
  const int t4 = lane & 3;
  const int r_lo = warp * 16 + g;  // query rows of this thread inside the tile
  const int r_hi = r_lo + 8;
  uint32_t qa[QS ? 1 : NKS][4];
  if constexpr (QS) {
    // This warp's 16 query rows into its slab of the Q tile.
    uint8_t* slab = qsm + warp * 16 * D * 2;
    for (int idx = lane; idx < 16 * (D / 8); idx += 32) {
      const int r = idx / (D / 8), c = idx % (D / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (warp * 16 + r < nq)
        v = *reinterpret_cast<const uint4*>(a.q + (size_t)(qrow0 + warp * 16 + r) * a.q_stride +
                                            (size_t)hq * D + c * 8);
      *reinterpret_cast<uint4*>(slab + r * D * 2 + (((c & ~7) | ((c & 7) ^ (r & 7))) << 4)) = v;
    }
    __syncwarp();
  } else {
    const __nv_bfloat16* q_lo = a.q + (size_t)(qrow0 + r_lo) * a.q_stride + (size_t)hq * D;
    const __nv_bfloat16* q_hi = a.q + (size_t)(qrow0 + r_hi) * a.q_stride + (size_t)hq * D;
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks) {
      const int c0 = ks * 16 + 2 * t4;
      qa[ks][0] = r_lo < nq ? *reinterpret_cast<const uint32_t*>(q_lo + c0) : 0u;
      qa[ks][1] = r_hi < nq ? *reinterpret_cast<const uint32_t*>(q_hi + c0) : 0u;
      qa[ks][2] = r_lo < nq ? *reinterpret_cast<const uint32_t*>(q_lo + c0 + 8) : 0u;
      qa[ks][3] = r_hi < nq ? *reinterpret_cast<const uint32_t*>(q_hi + c0 + 8) : 0u;
    }
  }
  const int qpos[2] = {pos0 + r_lo, pos0 + r_hi};
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {kNegBig, kNegBig};
  float l[2] = {0.f, 0.f};
  // Last KV position any row of this warp attends to.
  const int warp_last_pos = pos0 + min(nq, warp * 16 + 16) - 1;

  for (int ti = 0; ti < ntiles; ++ti) {
    const int st = ti & 1;
    if (!mbar_wait(&full[st], (ti >> 1) & 1, a.status, kStatusAttnTimeout, &s_abort)) break;
    const uint32_t kaddr = smem_u32(smem + st * STAGE);
    const uint32_t vaddr = kaddr + TILE_BYTES;
    const int kpos0 = tile_of(ti) * 64;
    if (kpos0 <= warp_last_pos) {
      float s[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        uint32_t qf[4];
        if constexpr (QS) {
          const int qr = (lane & 7) + (((lane >> 3) & 1) << 3);
          const int qc = 2 * ks + (lane >> 4);
          ldsm_x4(smem_u32(qsm) + (warp * 16 + qr) * D * 2 +
                      (((qc & ~7) | ((qc & 7) ^ (qr & 7))) << 4),
                  qf[0], qf[1], qf[2], qf[3]);
        } else {
          qf[0] = qa[ks][0];
          qf[1] = qa[ks][1];
          qf[2] = qa[ks][2];
          qf[3] = qa[ks][3];
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of 8-token n-tiles = one 16-token block
          const int row = ((lane >> 4) << 3) + (lane & 7);  // token within block np
          const int chunk = 2 * ks + ((lane >> 3) & 1);
          uint32_t b00, b01, b10, b11;
          ldsm_x4(kaddr + np * BLK_BYTES + sw128_off(row, chunk, 16), b00, b01, b10, b11);
          mma_16816(s[2 * np], qf, b00, b01);
          mma_16816(s[2 * np + 1], qf, b10, b11);
        }
      }
      float p[8][4];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float mx = kNegBig;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int kp = kpos0 + nt * 8 + 2 * t4 + e;
            float v = s[nt][2 * r + e] * a.scale_log2;
            const bool seen = kp <= qpos[r] && kp < kv_len &&
                              (!WIN || kp > qpos[r] - a.window || kp < a.sinks);
            v = seen ? v : -INFINITY;
            s[nt][2 * r + e] = v;
            mx = fmaxf(mx, v);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m[r], mx);
        const float alpha = exp2f(m[r] - m_new);
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float pv = exp2f(s[nt][2 * r + e] - m_new);
            p[nt][2 * r + e] = pv;
            sum += pv;
          }
        }
        l[r] = l[r] * alpha + sum;
        m[r] = m_new;
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt) {
          o[nt][2 * r] *= alpha;
          o[nt][2 * r + 1] *= alpha;
        }
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 16-token k-steps = paged blocks
        uint32_t pa[4];
        pa[0] = pack_bf16(p[2 * kk][0], p[2 * kk][1]);
        pa[1] = pack_bf16(p[2 * kk][2], p[2 * kk][3]);
        pa[2] = pack_bf16(p[2 * kk + 1][0], p[2 * kk + 1][1]);
        pa[3] = pack_bf16(p[2 * kk + 1][2], p[2 * kk + 1][3]);
        if (kpos0 + kk * 16 < kv_len) {
#pragma unroll
          for (int np = 0; np < D / 16; ++np) {
            const int mi = lane >> 3;
            const int row = ((mi & 1) << 3) + (lane & 7);
            const int chunk = 2 * np + (mi >> 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vaddr + kk * BLK_BYTES + sw128_off(row, chunk, 16), b0, b1, b2, b3);
            mma_16816(o[2 * np], pa, b0, b1);
            mma_16816(o[2 * np + 1], pa, b2, b3);
          }
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && ti + 2 < ntiles) {
      fence_proxy_async_smem();
      issue(ti + 2, st);
    }
  }
  if (s_abort) return;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = r == 0 ? r_lo : r_hi;
    if (row < nq) {
      const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
      __nv_bfloat16* op = a.out + (size_t)(qrow0 + row) * a.out_stride + (size_t)hq * D;
#pragma unroll
      for (int nt = 0; nt < D / 8; ++nt) {
        *reinterpret_cast<uint32_t*>(op + nt * 8 + 2 * t4) =
            pack_bf16(o[nt][2 * r] * inv, o[nt][2 * r + 1] * inv);
      }
    }
  }
}

// ---------------------------------------------------------------- host side

static CUtensorMap kv_tmap(const torch::Tensor& cache) {
  // cache: [L, NB, Hkv, 16, D]
  const int64_t D = cache.size(4);
  const int64_t rows = cache.numel() / D;
  return make_tmap_2d_bf16(cache.data_ptr(), (uint64_t)D, (uint64_t)rows, (uint64_t)D * 2, 64, 16,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

// Stages (a K block + this CTA's slice of a V block per warp and stage) +
// barriers + the Q tile for head dims above 128 + alignment slack.
template <int D, int DV, bool WIN>
static void launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeArgs& a,
                          dim3 grid, int B, int Hq, cudaStream_t stream) {
  constexpr int kStage = 16 * D * 2 + 16 * DV * 2;
  constexpr int smem = 4 * 2 * kStage + 128 + (D > 128 ? 16 * D * 2 : 0) + 1024;
  static bool cfg = false;
  if (!cfg) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(attn_decode_kernel<D, DV, WIN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cfg = true;
  }
  const dim3 g(grid.x, grid.y, grid.z * (D / DV));
  launch_kernel(attn_decode_kernel<D, DV, WIN>, g, dim3(128), smem, stream, tk, tv, a);
  if (a.splits > 1) {
    launch_kernel(attn_decode_combine_kernel<D>, dim3(B, Hq), dim3(D), 0, stream, a.part_o,
                  a.part_ml, a.out, a.out_stride, a.Hkv, a.G, a.splits);
  }
}

// Two K/V stages of 64 tokens + barriers + the Q tile above head_dim 128.
template <int D, bool WIN>
static void launch_prefill(const CUtensorMap& tk, const CUtensorMap& tv, const PrefillArgs& a,
                           dim3 grid, cudaStream_t stream) {
  constexpr int smem = 2 * 2 * 4 * 16 * D * 2 + 128 + (D > 128 ? 64 * D * 2 : 0) + 1024;
  static bool cfg = false;
  if (!cfg) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<D, WIN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cfg = true;
  }
  launch_kernel(attn_prefill_kernel<D, WIN>, grid, dim3(128), smem, stream, tk, tv, a);
}

// q: [B, Hq*D] view (row stride arbitrary); out: [B, Hq*D].
void attn_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                 torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor out,
                 int64_t layer, int64_t num_splits, int64_t blocks_per_split,
                 torch::Tensor part_o, torch::Tensor part_ml, double scale, torch::Tensor status,
                 int64_t window, int64_t sinks) {
  TORCH_CHECK(k_cache.dim() == 5 && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "kv cache must be [L, NB, Hkv, 16, D] contiguous");
  TORCH_CHECK(k_cache.size(3) == 16, "block size must be 16");
  const int D = (int)k_cache.size(4);
  const int Hkv = (int)k_cache.size(2);
  const int B = (int)q.size(0);
  const int Hq = (int)(q.size(1) / D);
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "GQA group must be <= 16");
  TORCH_CHECK(q.stride(1) == 1 && out.stride(1) == 1, "q/out inner stride must be 1");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt,
              "int32 block tables / seq lens");
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  DecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_stride = (int)q.stride(0);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = (int)block_tables.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_stride = (int)out.stride(0);
  a.part_o = num_splits > 1 ? part_o.data_ptr<float>() : nullptr;
  a.part_ml = num_splits > 1 ? part_ml.data_ptr<float>() : nullptr;
  a.status = status.data_ptr<int>();
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.NB = (int)k_cache.size(1);
  a.layer = (int)layer;
  a.blocks_per_split = (int)blocks_per_split;
  a.splits = (int)num_splits;
  a.scale_log2 = (float)scale * kLog2e;
  a.window = (int)window;
  a.sinks = (int)sinks;
  if (num_splits > 1) {
    TORCH_CHECK(part_o.numel() >= (int64_t)B * Hkv * num_splits * a.G * D, "part_o too small");
    TORCH_CHECK(part_ml.numel() >= (int64_t)B * Hkv * num_splits * a.G * 2, "part_ml too small");
  }
  CUtensorMap tk = kv_tmap(k_cache), tv = kv_tmap(v_cache);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const dim3 grid(Hkv, B, (unsigned)num_splits);
  const bool win = window > 0;
  if (D == 128) {
    if (win) launch_decode<128, 128, true>(tk, tv, a, grid, B, Hq, stream);
    else launch_decode<128, 128, false>(tk, tv, a, grid, B, Hq, stream);
  } else if (D == 64) {
    if (win) launch_decode<64, 64, true>(tk, tv, a, grid, B, Hq, stream);
    else launch_decode<64, 64, false>(tk, tv, a, grid, B, Hq, stream);
  } else if (D == 256) {
    if (win) launch_decode<256, 256, true>(tk, tv, a, grid, B, Hq, stream);
    else launch_decode<256, 256, false>(tk, tv, a, grid, B, Hq, stream);
  } else if (D == 512) {
    // Two CTAs per head, 256 output dims each.
    if (win) launch_decode<512, 256, true>(tk, tv, a, grid, B, Hq, stream);
    else launch_decode<512, 256, false>(tk, tv, a, grid, B, Hq, stream);
  } else {
    TORCH_CHECK(false, "head_dim must be 64, 128, 256 or 512");
  }
  CB_CUDA_CHECK(cudaGetLastError());
}

// q: [T, Hq*D]; tiles: int32 [n_tiles, 4] {seq, first row, first position, rows}
void attn_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                  torch::Tensor block_tables, torch::Tensor tiles, torch::Tensor out, int64_t layer,
                  double scale, torch::Tensor status, int64_t window, int64_t sinks) {
  const int D = (int)k_cache.size(4);
  const int Hkv = (int)k_cache.size(2);
  const int Hq = (int)(q.size(1) / D);
  const int n_tiles = (int)tiles.size(0);
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.is_contiguous() && tiles.size(1) == 4,
              "tiles must be int32 [n, 4]");
  TORCH_CHECK(q.stride(1) == 1 && out.stride(1) == 1, "q/out inner stride must be 1");
  // The kernel reads each tile descriptor as one int4.
  TORCH_CHECK(reinterpret_cast<uintptr_t>(tiles.data_ptr()) % 16 == 0,
              "tiles must start on a 16-byte boundary");
  if (n_tiles == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  PrefillArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_stride = (int)q.stride(0);
  a.tiles = reinterpret_cast<const int4*>(tiles.data_ptr<int>());
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = (int)block_tables.stride(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_stride = (int)out.stride(0);
  a.status = status.data_ptr<int>();
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.NB = (int)k_cache.size(1);
  a.layer = (int)layer;
  a.scale_log2 = (float)scale * kLog2e;
  a.window = (int)window;
  a.sinks = (int)sinks;
  CUtensorMap tk = kv_tmap(k_cache), tv = kv_tmap(v_cache);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const dim3 grid(n_tiles, Hq);
  const bool win = window > 0;
  if (D == 128) {
    if (win) launch_prefill<128, true>(tk, tv, a, grid, stream);
    else launch_prefill<128, false>(tk, tv, a, grid, stream);
  } else if (D == 64) {
    if (win) launch_prefill<64, true>(tk, tv, a, grid, stream);
    else launch_prefill<64, false>(tk, tv, a, grid, stream);
  } else if (D == 256) {
    if (win) launch_prefill<256, true>(tk, tv, a, grid, stream);
    else launch_prefill<256, false>(tk, tv, a, grid, stream);
  } else {
    TORCH_CHECK(false, "head_dim must be 64, 128 or 256");
  }
  CB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace cb
