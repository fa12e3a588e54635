// Small-M W4A16 GEMM ("GEMV") for sm_100a decode: Y[M, N] = X[M, K] *
// dequant(W[N, K])^T for M <= 16 tokens, reading the same pre-tiled INT4 blob
// as the tcgen05 kernel (gemm_w4a16.cu).
//
// Why a second kernel: with 1..16 tokens every weight is used 1..16 times, so
// the work is bounded by (a) streaming the weights and (b) dequantising them;
// the multiply-adds are negligible.  The tcgen05 path pays a fixed cost per
// 128x16 MMA (A staged through tensor memory) that dominates at these sizes.
// Here the dequantised weights go straight from registers into warp-level
// MMAs (m16n8k16, fp32 accumulate), which need no staging at all.
//
// Data flow per CTA (persistent: one CTA per SM, each walking a list of
// 128-row weight tiles of one K range):
//   * one producer thread streams the tiles' k-blocks with 1-D bulk copies of
//     TWO consecutive k-blocks (16.9 KiB: on B200 an SM completes about one
//     bulk copy per ~350 ns, so copies must be >= 16 KiB to reach HBM peak)
//     into a ring of shared-memory stages, back to back across tiles;
//   * X for the CTA's K range is loaded once (one bulk copy per token row);
//   * 16 consumer warps: warp w owns weight rows 16*(w%8) .. +15 and every
//     other k-block (parity w/8).  Lane (g, c) = (lane/4, lane%4) loads the
//     16-byte chunk c (32 consecutive k) of rows g and g+8 and issues 8 MMAs
//     per k-block and n-tile of 8 tokens.  Group 128: X is converted to fp16
//     once, the MMA A operand is the exact fp16 (c + q) made by one LOP3 per
//     pair (c = 1024 or 64 by nibble position), and the row scale and the
//     offset are applied to the fp32 k-block sum.  Group 32: pairs are
//     (q-8)*scale rounded to bf16 (LOP3 + HSUB2 + HMUL2), as in the tcgen05
//     path.  The MMA's k order is a permutation of the real k order; X is
//     read with the same permutation, so the dot products are unchanged.
//   * parity partials are summed in shared memory, then either stored with
//     the fused epilogue (store / SiLU(gate)*up / residual add) or, with
//     split-K, written to the fp32 workspace; the last CTA of a tile (per-tile
//     counter) sums the splits in a fixed order.  Deterministic.
//   * every wait is bounded (2 s): on expiry the kernel records a status code,
//     stops issuing copies, waits (bounded) for its copies in flight, returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemv_w4a16.h"
#include "host_utils.h"
#include "mma_frag.cuh"

namespace cb {

namespace {

constexpr int kGvConsumerWarps = 16;
constexpr int kGvThreads = 32 * (kGvConsumerWarps + 1);
constexpr int kGvSmemBudget = 220 * 1024;
constexpr int kGvXBudget = 72 * 1024;

template <int GS>
struct GvBlob {
  static constexpr int kPacked = 8192;
  static constexpr int kScales = 128 * (128 / GS) * 2;
  static constexpr int kBytes = kPacked + kScales;
  static constexpr int kStage = 2 * kBytes;  // two k-blocks per bulk copy
};

struct GvArgs {
  const uint8_t* wblob;
  const __nv_bfloat16* x;
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;
  float* ws;
  int* counters;
  int* status;
  int M, N, K, ldx, ldo, ldr;
  int kbps, splits, stages;
  int pdl;  // launched with programmatic stream serialisation
};

__device__ __forceinline__ uint32_t deq_pair(uint32_t w, int h, __nv_bfloat162 s2) {
  const __nv_bfloat162 k136 = __floats2bfloat162_rn(136.f, 136.f);
  uint32_t v = ((w >> (4 * h)) & 0x000F000Fu) | 0x43004300u;  // bf16 (128 + q)
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  b = __hmul2(__hsub2(b, k136), s2);                          // (q - 8) * scale
  return *reinterpret_cast<uint32_t*>(&b);
}

// Group-128 path: fp16x2 (c + q_even, c + q_odd) of a nibble pair with the
// nibble placed in the fp16 mantissa under a magic exponent: bits 0-3 give
// 1024 + q, bits 4-7 give 64 + q.  Pairs 0 and 1 of a word take one LOP3
// each; pairs 2 and 3 share one right shift by 8, done as a multiply-high on
// the FMA pipe (the LOP3s keep the ALU pipe busy).  Exact.
__device__ __forceinline__ uint32_t magic_lo(uint32_t v) {
  return (v & 0x000F000Fu) | 0x64006400u;  // 1024 + q
}
__device__ __forceinline__ uint32_t magic_hi(uint32_t v) {
  return (v & 0x00F000F0u) | 0x54005400u;  // 64 + q
}

__device__ __forceinline__ void mma_16816_f16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Persistent over row tiles: CTA b works on split (b % splits) and row tiles
// b / splits, + grid / splits, ...; the producer streams all of them back to
// back, so the ring never drains between tiles and X is loaded (and, for
// group 128, converted) once per CTA.
template <int GS, int EPI, int NT>
__global__ void __launch_bounds__(kGvThreads, 1) w4a16_gemv_kernel(const GvArgs a) {
  constexpr int MP = 8 * NT;
  constexpr int kRedFloats = 8 * 32 * NT * 4;
  constexpr int kTileFloats = 128 * (MP + 1);
  constexpr int kCons = 32 * kGvConsumerWarps;
  using Blob = GvBlob<GS>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = a.K / 128;
  const int split = blockIdx.x % a.splits;
  const int cta_in_split = blockIdx.x / a.splits;
  const int ctas_per_split = gridDim.x / a.splits;
  const int row_tiles = a.N / 128;
  const int kb0 = split * a.kbps;
  const int nkb = min(a.kbps, KB - kb0);
  const int ntiles = cta_in_split < row_tiles
                         ? (row_tiles - cta_in_split + ctas_per_split - 1) / ctas_per_split
                         : 0;
  if (a.pdl) grid_dep_launch();  // dependents may become resident; they wait for our end
  if (nkb <= 0 || ntiles <= 0) {
    grid_dep_wait();
    return;
  }
  const int spt = (nkb + 1) / 2;  // stages per tile
  const int total = ntiles * spt;
  const int S = a.stages;
  const int xstride = nkb * 256 + 16;  // bytes per token row of the X tile
  const int rows = min(a.M, MP);

  uint8_t* ring = smem;
  float* red = reinterpret_cast<float*>(smem + S * Blob::kStage);  // [8 rg][32][NT*4]
  float* tile = red + kRedFloats;                                   // [128][MP + 1]
  uint8_t* xs = reinterpret_cast<uint8_t*>(tile + kTileFloats);
  float* xsum = reinterpret_cast<float*>(xs + MP * (a.kbps * 256 + 16));  // [kbps][MP]
  float* tscale = xsum + a.kbps * MP;  // per-token exponent of the fp16 X scaling
  uint64_t* bars = reinterpret_cast<uint64_t*>(tscale + 16);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* xbar = bars + 2 * S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * S + 1);
  int* s_last = reinterpret_cast<int*>(bars + 2 * S + 2);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 2 * S + 3);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGvConsumerWarps);
    }
    mbar_init(xbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Zero the padding token rows of the X tile.
  for (int i = threadIdx.x; i < (MP - rows) * (xstride / 16); i += blockDim.x) {
    const int r = rows + i / (xstride / 16);
    reinterpret_cast<uint4*>(xs + r * xstride)[i % (xstride / 16)] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();

  if (warp == kGvConsumerWarps) {
    // Producer warp: lane 0 issues all copies.
    if (lane == 0) {
      int issued = 0;
      // X is the previous kernel's output: it is copied after the wait for
      // that kernel.  With PDL the first S weight stages (constant data) are
      // issued before it.
      const int pre = a.pdl ? min(S, total) : 0;
      auto load_x = [&] {
        grid_dep_wait();
        mbar_arrive_expect_tx(xbar, (uint32_t)(rows * nkb * 256));
        for (int r = 0; r < rows; ++r)
          bulk_g2s(xs + r * xstride, a.x + (size_t)r * a.ldx + (size_t)kb0 * 128,
                   (uint32_t)(nkb * 256), xbar);
      };
      if (pre == 0) load_x();
      int slot = 0, st = 0, j = 0;
      uint32_t phase = 0;
      for (int g = 0; g < total; ++g) {
        if (g == pre && pre > 0) load_x();
        const int rt = cta_in_split + j * ctas_per_split;
        if (g >= S &&
            !mbar_wait(&empty[slot], phase ^ 1u, a.status, kStatusGemmLoadTimeout, abort_flag))
          break;
        const int nb = min(2, nkb - 2 * st);
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(nb * Blob::kBytes));
        bulk_g2s(ring + slot * Blob::kStage,
                 a.wblob + ((size_t)rt * KB + kb0 + 2 * st) * Blob::kBytes,
                 (uint32_t)(nb * Blob::kBytes), &full[slot]);
        issued = g + 1;
        if (++st == spt) {
          st = 0;
          ++j;
        }
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
      }
      if (pre > 0 && pre == total) load_x();  // every stage fitted in the ring
      // Do not leave while copies into this CTA's shared memory are in
      // flight (matters only when the consumers gave up early).
      for (int g = max(0, issued - S); g < issued; ++g)
        mbar_wait(&full[g % S], (g / S) & 1, nullptr, 0, nullptr);
      mbar_wait(xbar, 0, nullptr, 0, nullptr);
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  grid_dep_wait();  // before any global write
  const int tid = threadIdx.x;  // 0 .. kCons-1
  const int rg = warp & 7, par = warp >> 3;
  const int g = lane >> 2, c = lane & 3;
  const int r0 = rg * 16 + g, r1 = r0 + 8;
  const int sw0 = ((c ^ ((r0 >> 1) & 3)) << 4), sw1 = ((c ^ ((r1 >> 1) & 3)) << 4);
  bool ok = mbar_wait(xbar, 0, a.status, kStatusGemmMmaTimeout, abort_flag);
  const uint32_t ring_u = smem_u32(ring);
  const uint32_t xs_u = smem_u32(xs);
  if constexpr (GS == 128) {
    // X -> fp16 in place, per token scaled by 2^-e so that |x| <= 2^14
    // (exact; e = 0 unless a token has huge activations), and the offset
    // correction -sum_k (c(k) + 8) x_k per (k-block, token).
    if (tid < 16) tscale[tid] = 0.f;
    named_bar_sync(1, kCons);
    for (int e = tid; e < rows * nkb * 16; e += kCons) {
      const int tok = e / (nkb * 16), off = e % (nkb * 16);
      const uint4 v = lds128(xs_u + tok * xstride + off * 16);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
      float m = 0.f;
#pragma unroll
      for (int z = 0; z < 4; ++z) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[z]));
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
      atomicMax(reinterpret_cast<int*>(&tscale[tok]), __float_as_int(m));  // m >= 0
    }
    named_bar_sync(1, kCons);
    if (tid < MP) {
      const float mx = tscale[tid];
      tscale[tid] = mx > 16384.f ? ceilf(log2f(mx / 16384.f)) : 0.f;
    }
    named_bar_sync(1, kCons);
    for (int e = tid; e < rows * nkb * 16; e += kCons) {
      const int tok = e / (nkb * 16), off = e % (nkb * 16);
      const float sc = exp2f(-tscale[tok]);
      uint32_t* p = reinterpret_cast<uint32_t*>(xs + tok * xstride + off * 16);
#pragma unroll
      for (int z = 0; z < 4; ++z) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&p[z]));
        const __half2 hv = __floats2half2_rn(f.x * sc, f.y * sc);
        p[z] = *reinterpret_cast<const uint32_t*>(&hv);
      }
    }
    named_bar_sync(1, kCons);
    for (int e = tid; e < nkb * MP; e += kCons) {
      const int kb = e / MP, tok = e % MP;
      float sum = 0.f;
      if (tok < rows) {
        const uint32_t src = xs_u + tok * xstride + kb * 256;
#pragma unroll 4
        for (int q = 0; q < 16; ++q) {  // 8 k per 16 bytes; pair z = (k % 8) / 2
          const uint4 v = lds128(src + q * 16);
          const uint32_t u[4] = {v.x, v.y, v.z, v.w};
          const float cz[4] = {1032.f, 72.f, 1032.f, 72.f};
#pragma unroll
          for (int z = 0; z < 4; ++z) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[z]));
            sum += cz[z] * (f.x + f.y);
          }
        }
      }
      xsum[kb * MP + tok] = -sum;
    }
    named_bar_sync(1, kCons);
  }

  // Ring position, advanced incrementally (no division by the run-time S).
  int slot = 0;
  uint32_t phase = 0;
  for (int j = 0; j < ntiles; ++j) {
    const int rt = cta_in_split + j * ctas_per_split;
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[t][q] = 0.f;
    for (int st = 0; st < spt; ++st) {
      const int cur = slot;
      const uint32_t ph = phase;
      if (++slot == S) {
        slot = 0;
        phase ^= 1u;
      }
      if (!ok || !mbar_wait(&full[cur], ph, a.status, kStatusGemmMmaTimeout, abort_flag)) {
        ok = false;
        break;
      }
      const int i = 2 * st + par;
      if (i >= nkb) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[cur]);
        continue;
      }
      const uint32_t base = ring_u + cur * Blob::kStage + par * Blob::kBytes;
      const uint4 wa = lds128(base + r0 * 64 + sw0);
      const uint4 wb = lds128(base + r1 * 64 + sw1);
      uint16_t sa, sb;
      if (GS == 128) {
        sa = lds16(base + Blob::kPacked + r0 * 2);
        sb = lds16(base + Blob::kPacked + r1 * 2);
      } else {
        sa = lds16(base + Blob::kPacked + (r0 * (128 / GS) + (c * 32) / GS) * 2);
        sb = lds16(base + Blob::kPacked + (r1 * (128 / GS) + (c * 32) / GS) * 2);
      }
      const uint32_t wa_w[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t wb_w[4] = {wb.x, wb.y, wb.z, wb.w};
      uint32_t xr[NT][16];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint32_t xa = xs_u + (8 * t + g) * xstride + (i * 128 + 32 * c) * 2;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = lds128(xa + q * 16);
          xr[t][4 * q + 0] = v.x;
          xr[t][4 * q + 1] = v.y;
          xr[t][4 * q + 2] = v.z;
          xr[t][4 * q + 3] = v.w;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[cur]);
      if constexpr (GS == 128) {
        // D = sum_k (c(k) + q) x exactly (fp16 inputs, fp32 MMA); then
        // acc += scale * (D - sum_k (c(k) + 8) x) = scale * sum_k (q - 8) x.
        float d[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int q = 0; q < 4; ++q) d[t][q] = 0.f;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int wi = jj >> 1;
          uint32_t va = wa_w[wi], vb = wb_w[wi];
          if (jj & 1) {  // pairs 2, 3: nibbles at bits 8-15 of each half
            va = __umulhi(va, 1u << 24);
            vb = __umulhi(vb, 1u << 24);
          }
          const uint32_t A[4] = {magic_lo(va), magic_lo(vb), magic_hi(va), magic_hi(vb)};
#pragma unroll
          for (int t = 0; t < NT; ++t) mma_16816_f16(d[t], A, xr[t][2 * jj], xr[t][2 * jj + 1]);
        }
        const float fa = __bfloat162float(__ushort_as_bfloat16(sa));
        const float fb = __bfloat162float(__ushort_as_bfloat16(sb));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float2 xc = *reinterpret_cast<const float2*>(&xsum[i * MP + 8 * t + 2 * c]);
          acc[t][0] = fmaf(fa, d[t][0] + xc.x, acc[t][0]);
          acc[t][1] = fmaf(fa, d[t][1] + xc.y, acc[t][1]);
          acc[t][2] = fmaf(fb, d[t][2] + xc.x, acc[t][2]);
          acc[t][3] = fmaf(fb, d[t][3] + xc.y, acc[t][3]);
        }
      } else {
        const __nv_bfloat162 sa2 =
            __halves2bfloat162(__ushort_as_bfloat16(sa), __ushort_as_bfloat16(sa));
        const __nv_bfloat162 sb2 =
            __halves2bfloat162(__ushort_as_bfloat16(sb), __ushort_as_bfloat16(sb));
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int wi = jj >> 1, h0 = 2 * (jj & 1);
          const uint32_t A[4] = {deq_pair(wa_w[wi], h0, sa2), deq_pair(wb_w[wi], h0, sb2),
                                 deq_pair(wa_w[wi], h0 + 1, sa2), deq_pair(wb_w[wi], h0 + 1, sb2)};
#pragma unroll
          for (int t = 0; t < NT; ++t) mma_16816(acc[t], A, xr[t][2 * jj], xr[t][2 * jj + 1]);
        }
      }
    }
    // ---------------------------------------------------------- reduction
    // Every consumer warp reaches these barriers on every tile, also after a
    // failed wait; the abort decision is taken uniformly from a snapshot of
    // the abort flag (the producer may raise it at any time).
    named_bar_sync(1, kCons);  // previous tile's epilogue is done with red/tile
    if (tid == 0) *s_abort = *abort_flag;
    if (par == 1) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) red[(rg * 32 + lane) * NT * 4 + t * 4 + q] = acc[t][q];
    }
    named_bar_sync(1, kCons);
    if (*s_abort) break;
    if (par == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = acc[t][q] + red[(rg * 32 + lane) * NT * 4 + t * 4 + q];
        const int n = 8 * t + 2 * c;
        if constexpr (GS == 128) {  // undo the per-token X scaling
          const float e0 = exp2f(tscale[n]), e1 = exp2f(tscale[n + 1]);
          v[0] *= e0;
          v[1] *= e1;
          v[2] *= e0;
          v[3] *= e1;
        }
        tile[r0 * (MP + 1) + n] = v[0];
        tile[r0 * (MP + 1) + n + 1] = v[1];
        tile[r1 * (MP + 1) + n] = v[2];
        tile[r1 * (MP + 1) + n + 1] = v[3];
      }
    }
    named_bar_sync(1, kCons);
    const int n0 = rt * 128;
    if (a.splits > 1) {
      float* dst = a.ws + (size_t)split * a.M * a.N;
      for (int idx = tid; idx < 128 * rows; idx += kCons) {
        const int r = idx & 127, m = idx >> 7;
        __stcg(&dst[(size_t)m * a.N + n0 + r], tile[r * (MP + 1) + m]);
      }
      __threadfence();
      named_bar_sync(1, kCons);
      if (tid == 0) {
        const int old = atomicAdd(&a.counters[rt], 1);
        const int last = old == a.splits - 1;
        if (last) a.counters[rt] = 0;  // ready for the next launch
        *s_last = last;
      }
      named_bar_sync(1, kCons);
      if (!*s_last) continue;
      __threadfence();
      for (int idx = tid; idx < 128 * rows; idx += kCons) {
        const int r = idx & 127, m = idx >> 7;
        float sum = 0.f;
        for (int sp = 0; sp < a.splits; ++sp)
          sum += __ldcg(&a.ws[((size_t)sp * a.M + m) * a.N + n0 + r]);
        tile[r * (MP + 1) + m] = sum;
      }
      named_bar_sync(1, kCons);
    }
    // ---------------------------------------------------------- epilogue
    if constexpr (EPI == kGvEpiSilu) {
      for (int idx = tid; idx < 64 * rows; idx += kCons) {
        const int jj = idx & 63, m = idx >> 6;
        const float gt = tile[(2 * jj) * (MP + 1) + m];
        const float up = tile[(2 * jj + 1) * (MP + 1) + m];
        const float y = gt / (1.f + __expf(-gt)) * up;
        a.out[(size_t)m * a.ldo + rt * 64 + jj] = __float2bfloat16(y);
      }
    } else {
      for (int idx = tid; idx < 128 * rows; idx += kCons) {
        const int r = idx & 127, m = idx >> 7;
        float y = tile[r * (MP + 1) + m];
        if constexpr (EPI == kGvEpiResid)
          y += __bfloat162float(a.residual[(size_t)m * a.ldr + n0 + r]);
        a.out[(size_t)m * a.ldo + n0 + r] = __float2bfloat16(y);
      }
    }
  }
}

template <int GS>
int gv_fixed_bytes(int kbps, int MP) {
  const int red = 8 * 32 * (MP / 8) * 4 * 4 + 128 * (MP + 1) * 4;
  return red + MP * (kbps * 256 + 16) + kbps * MP * 4 + 64 + 1024;
}

template <int GS>
int gv_stages(int kbps, int MP) {
  const int s = (kGvSmemBudget - gv_fixed_bytes<GS>(kbps, MP)) / GvBlob<GS>::kStage;
  return std::max(2, std::min(10, s));
}

template <int GS>
int gv_smem(int kbps, int MP, int stages) {
  return stages * GvBlob<GS>::kStage + gv_fixed_bytes<GS>(kbps, MP);
}

int gv_max_kbps(int MP) { return std::max(1, kGvXBudget / (MP * 256)); }

// Split-K factor: at least enough splits for the X tile to fit, then fill
// the SMs with >= 4 k-blocks per CTA.
int gv_splits(int row_tiles, int KB, int MP, int forced) {
  const int sms = num_sms();
  int s = forced > 0 ? forced : 1;
  if (forced <= 0) {
    const int smin = (KB + gv_max_kbps(MP) - 1) / gv_max_kbps(MP);
    s = smin;
    double best = -1.0;
    for (int cand = smin; cand <= KB; ++cand) {
      const int kbps = (KB + cand - 1) / cand;
      const int real = (KB + kbps - 1) / kbps;
      if (kbps < 4 && cand > smin) break;
      const long ctas = (long)row_tiles * real;
      const long waves = (ctas + sms - 1) / sms;
      const double eff = (double)ctas / (double)(waves * sms);
      if (eff > best + 1e-9) {
        best = eff;
        s = real;
      }
      if (waves > 1 && ctas > 2L * sms) break;
    }
  }
  const int kbps = (KB + s - 1) / s;
  return (KB + kbps - 1) / kbps;
}

template <int GS, int EPI, int NT>
void gv_launch_t(const GvArgs& a, dim3 grid, int smem, cudaStream_t stream) {
  // The shared-memory attribute is per device: set it once for each.
  static int configured[64] = {};
  int dev = 0;
  CB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(w4a16_gemv_kernel<GS, EPI, NT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kGvSmemBudget + 4096));
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  if (a.pdl) {
    launch_kernel(w4a16_gemv_kernel<GS, EPI, NT>, grid, dim3(kGvThreads), (size_t)smem, stream, a);
    return;
  }
  w4a16_gemv_kernel<GS, EPI, NT><<<grid, kGvThreads, smem, stream>>>(a);
  CB_CUDA_CHECK(cudaGetLastError());
}

template <int GS, int EPI>
void gv_launch_nt(int NT, const GvArgs& a, dim3 grid, int smem, cudaStream_t s) {
  if (NT == 1) gv_launch_t<GS, EPI, 1>(a, grid, smem, s);
  else gv_launch_t<GS, EPI, 2>(a, grid, smem, s);
}


// ---------------------------------------------------------------- grouped
// MoE decode: every expert e multiplies its own few rows
// [offsets[e], offsets[e+1]) of a prepared activation matrix with its own
// weights (group 128).  Work units (expert, 128-row weight tile) are spread
// over persistent CTAs; a unit with more than 8 rows runs in chunks of 8.
// The activations come prepared by moe_prep_fp16 (fp16, power-of-two scaled
// per row, with the per-k-block offset corrections and the row exponent in
// `xsum`), so a unit only copies its rows in: one bulk copy for the X rows,
// one for their corrections, into a double-buffered X tile.
//
// Unit order: with `sched` (int[2], zero before the first launch) each CTA's
// producer takes the next unit from an atomic counter, so CTAs that drew
// many-row or many-tile experts do not hold up the grid; units of experts
// without rows are skipped as they are drawn.  The producer hands each
// sub-unit (expert, tile, first row, rows) to the consumers in shared memory
// beside its X buffer, and a sentinel (expert -1) ends the loop.  The last
// producer to finish resets the counter for the next launch.  Without
// `sched` CTA b takes units b, b + grid, ... in order.
struct GvgArgs {
  const uint8_t* wblob;
  long long blob_stride;     // bytes per expert
  const __half* x16;         // [R, ldx16] fp16 rows
  const float* xsum;         // [R, ldxs]: -sum (c(k) + 8) x per k-block, then the exponent
  const int* offsets;        // [E + 1]
  int R;                     // prepared rows: rows at or past R are never read
  __nv_bfloat16* out;        // [R, ldo]
  const long long* out_rows; // optional per-row destination addresses
  int* status;
  int* sched;                // optional [next unit, CTAs done]
  int E, N, K, ldx16, ldxs, ldo, stages;
};

template <int EPI>
__global__ void __launch_bounds__(kGvThreads, 1) w4a16_gemv_grouped_kernel(const GvgArgs a) {
  constexpr int MP = 8;
  constexpr int kCons = 32 * kGvConsumerWarps;
  using Blob = GvBlob<128>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = a.K / 128;
  const int RT = a.N / 128;
  const int spt = (KB + 1) / 2;
  const int S = a.stages;
  const int xbytes = MP * a.ldx16 * 2;  // one X buffer
  const int sbytes = MP * a.ldxs * 4;   // one correction buffer
  uint8_t* ring = smem;
  float* red = reinterpret_cast<float*>(smem + S * Blob::kStage);  // [8][32][4]
  float* tile = red + 8 * 32 * 4;                                   // [128][MP + 1]
  uint8_t* xs = reinterpret_cast<uint8_t*>(tile + 128 * (MP + 1));  // 2 X buffers
  float* xsm = reinterpret_cast<float*>(xs + 2 * xbytes);           // 2 correction buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(xsm) + 2 * sbytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* xfull = bars + 2 * S;
  uint64_t* xempty = bars + 2 * S + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * S + 4);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 2 * S + 5);
  int* info = reinterpret_cast<int*>(bars + 2 * S + 6);  // [2][4]: e, rt, row0, rows

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGvConsumerWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], kGvConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kGvConsumerWarps) {
    if (lane == 0) {
      int slot = 0, sub = 0, issued = 0;
      uint32_t phase = 0;
      bool go = true;
      const int total = a.E * RT;
      int u = a.sched != nullptr ? atomicAdd(a.sched, 1) : (int)blockIdx.x;
      while (go && u < total) {
        const int e = u / RT, rt = u % RT;
        const int r0 = a.offsets[e], n = min(a.offsets[e + 1], a.R) - r0;
        const uint8_t* wsrc = a.wblob + (size_t)e * a.blob_stride + (size_t)rt * KB * Blob::kBytes;
        for (int c0 = 0; c0 < n && go; c0 += MP, ++sub) {
          const int rows = min(MP, n - c0);
          const int xb = sub & 1;
          if (sub >= 2 && !mbar_wait(&xempty[xb], ((sub >> 1) - 1) & 1, a.status,
                                     kStatusGemmLoadTimeout, abort_flag)) {
            go = false;
            break;
          }
          info[4 * xb + 0] = e;
          info[4 * xb + 1] = rt;
          info[4 * xb + 2] = r0 + c0;
          info[4 * xb + 3] = rows;
          mbar_arrive_expect_tx(&xfull[xb], (uint32_t)(rows * (a.ldx16 * 2 + a.ldxs * 4)));
          bulk_g2s(xs + xb * xbytes, a.x16 + (size_t)(r0 + c0) * a.ldx16,
                   (uint32_t)(rows * a.ldx16 * 2), &xfull[xb]);
          bulk_g2s(reinterpret_cast<uint8_t*>(xsm) + xb * sbytes,
                   a.xsum + (size_t)(r0 + c0) * a.ldxs, (uint32_t)(rows * a.ldxs * 4),
                   &xfull[xb]);
          for (int st = 0; st < spt; ++st) {
            if (issued >= S &&
                !mbar_wait(&empty[slot], phase ^ 1u, a.status, kStatusGemmLoadTimeout, abort_flag)) {
              go = false;
              break;
            }
            const int nb = min(2, KB - 2 * st);
            mbar_arrive_expect_tx(&full[slot], (uint32_t)(nb * Blob::kBytes));
            bulk_g2s(ring + slot * Blob::kStage, wsrc + (size_t)(2 * st) * Blob::kBytes,
                     (uint32_t)(nb * Blob::kBytes), &full[slot]);
            ++issued;
            if (++slot == S) {
              slot = 0;
              phase ^= 1u;
            }
          }
        }
        if (go) u = a.sched != nullptr ? atomicAdd(a.sched, 1) : u + (int)gridDim.x;
      }
      // Sentinel sub-unit: the consumers leave their loop on expert -1.
      if (go) {
        const int xb = sub & 1;
        if (sub < 2 || mbar_wait(&xempty[xb], ((sub >> 1) - 1) & 1, a.status,
                                 kStatusGemmLoadTimeout, abort_flag)) {
          info[4 * xb] = -1;
          mbar_arrive(&xfull[xb]);
          ++sub;
        }
      }
      // Wait (bounded) for the copies still in flight before leaving.
      for (int g = max(0, issued - S); g < issued; ++g)
        mbar_wait(&full[g % S], (g / S) & 1, nullptr, 0, nullptr);
      for (int sb = max(0, sub - 2); sb < sub; ++sb)
        mbar_wait(&xfull[sb & 1], (sb >> 1) & 1, nullptr, 0, nullptr);
      if (a.sched != nullptr) {
        // Every producer has drawn its last unit before it counts itself
        // done, so the last one may reset the counter for the next launch.
        __threadfence();
        if (atomicAdd(a.sched + 1, 1) == (int)gridDim.x - 1) {
          atomicExch(a.sched, 0);
          atomicExch(a.sched + 1, 0);
        }
      }
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int tid = threadIdx.x;
  const int rg = warp & 7, par = warp >> 3;
  const int g = lane >> 2, c = lane & 3;
  const int r0w = rg * 16 + g, r1w = r0w + 8;
  const int sw0 = ((c ^ ((r0w >> 1) & 3)) << 4), sw1 = ((c ^ ((r1w >> 1) & 3)) << 4);
  const uint32_t ring_u = smem_u32(ring);
  const uint32_t xs_u = smem_u32(xs);
  int slot = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int sub = 0; ok; ++sub) {
    {
      const int xb = sub & 1;
      if (!mbar_wait(&xfull[xb], (sub >> 1) & 1, a.status, kStatusGemmMmaTimeout, abort_flag))
        ok = false;
      // A failed wait leaves the info unread: the barrier section below
      // then ends the loop for every warp (abort flag set).
      const int e = ok ? info[4 * xb] : -1;
      const int rt = ok ? info[4 * xb + 1] : 0;
      const int row0 = ok ? info[4 * xb + 2] : 0;
      const int rows = (ok && e >= 0) ? info[4 * xb + 3] : 0;
      const bool work = ok && e >= 0;
      const uint32_t xbase = xs_u + xb * xbytes;
      const float* cs = xsm + xb * (sbytes / 4);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int st = 0; st < spt && work && ok; ++st) {
        const int cur = slot;
        const uint32_t ph = phase;
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
        if (!mbar_wait(&full[cur], ph, a.status, kStatusGemmMmaTimeout, abort_flag)) {
          ok = false;
          break;
        }
        const int i = 2 * st + par;
        if (i >= KB) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[cur]);
          continue;
        }
        const uint32_t base = ring_u + cur * Blob::kStage + par * Blob::kBytes;
        const uint4 wa = lds128(base + r0w * 64 + sw0);
        const uint4 wb = lds128(base + r1w * 64 + sw1);
        const uint16_t sa = lds16(base + Blob::kPacked + r0w * 2);
        const uint16_t sb = lds16(base + Blob::kPacked + r1w * 2);
        uint32_t xr[16];
        if (g < rows) {
          const uint32_t xa = xbase + g * a.ldx16 * 2 + (i * 128 + 32 * c) * 2;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = lds128(xa + q * 16);
            xr[4 * q + 0] = v.x;
            xr[4 * q + 1] = v.y;
            xr[4 * q + 2] = v.z;
            xr[4 * q + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 16; ++q) xr[q] = 0u;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[cur]);
        const uint32_t wa_w[4] = {wa.x, wa.y, wa.z, wa.w};
        const uint32_t wb_w[4] = {wb.x, wb.y, wb.z, wb.w};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int wi = jj >> 1;
          uint32_t va = wa_w[wi], vb = wb_w[wi];
          if (jj & 1) {
            va = __umulhi(va, 1u << 24);
            vb = __umulhi(vb, 1u << 24);
          }
          const uint32_t A[4] = {magic_lo(va), magic_lo(vb), magic_hi(va), magic_hi(vb)};
          mma_16816_f16(d, A, xr[2 * jj], xr[2 * jj + 1]);
        }
        const float fa = __bfloat162float(__ushort_as_bfloat16(sa));
        const float fb = __bfloat162float(__ushort_as_bfloat16(sb));
        const int n0 = 2 * c, n1 = 2 * c + 1;
        const float x0 = n0 < rows ? cs[n0 * a.ldxs + i] : 0.f;
        const float x1 = n1 < rows ? cs[n1 * a.ldxs + i] : 0.f;
        acc[0] = fmaf(fa, d[0] + x0, acc[0]);
        acc[1] = fmaf(fa, d[1] + x1, acc[1]);
        acc[2] = fmaf(fb, d[2] + x0, acc[2]);
        acc[3] = fmaf(fb, d[3] + x1, acc[3]);
      }
      // Per-row exponents of the X scaling (last column of the corrections).
      const int n0 = 2 * c, n1 = 2 * c + 1;
      const float e0 = n0 < rows ? exp2f(cs[n0 * a.ldxs + KB]) : 0.f;
      const float e1 = n1 < rows ? exp2f(cs[n1 * a.ldxs + KB]) : 0.f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xempty[xb]);  // X rows of this sub-unit consumed

      // Every consumer warp reaches these barriers for every sub-unit, also
      // after a failed wait; the abort decision is uniform (snapshot).
      named_bar_sync(1, kCons);  // previous epilogue done with red / tile
      // 1: abort, 2: sentinel (no more units); the same for every warp.
      if (tid == 0) *s_abort = *abort_flag ? 1 : (e < 0 ? 2 : 0);
      if (par == 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) red[(rg * 32 + lane) * 4 + q] = acc[q];
      }
      named_bar_sync(1, kCons);
      if (*s_abort) {
        ok = false;
        break;
      }
      if (par == 0) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = acc[q] + red[(rg * 32 + lane) * 4 + q];
        tile[r0w * (MP + 1) + n0] = v[0] * e0;
        tile[r0w * (MP + 1) + n1] = v[1] * e1;
        tile[r1w * (MP + 1) + n0] = v[2] * e0;
        tile[r1w * (MP + 1) + n1] = v[3] * e1;
      }
      named_bar_sync(1, kCons);
      if constexpr (EPI == kGvEpiSilu) {
        for (int idx = tid; idx < 64 * rows; idx += kCons) {
          const int jj = idx & 63, m = idx >> 6;
          const float gt = tile[(2 * jj) * (MP + 1) + m];
          const float up = tile[(2 * jj + 1) * (MP + 1) + m];
          const int row = row0 + m;
          __nv_bfloat16* orow = a.out_rows != nullptr
                                    ? reinterpret_cast<__nv_bfloat16*>(a.out_rows[row])
                                    : a.out + (size_t)row * a.ldo;
          orow[rt * 64 + jj] = __float2bfloat16(gt / (1.f + __expf(-gt)) * up);
        }
      } else {
        for (int idx = tid; idx < 16 * rows; idx += kCons) {
          const int r8 = (idx & 15) * 8, m = idx >> 4;
          const int row = row0 + m;
          __nv_bfloat16* orow = a.out_rows != nullptr
                                    ? reinterpret_cast<__nv_bfloat16*>(a.out_rows[row])
                                    : a.out + (size_t)row * a.ldo;
          uint4 o;
          __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
          for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16(tile[(r8 + q) * (MP + 1) + m]);
          *reinterpret_cast<uint4*>(orow + rt * 128 + r8) = o;
        }
      }
    }
  }
}

// Prepared activations for the grouped small-M kernel: one CTA per row.
//   x16[r]  = fp16(x[src(r)] * 2^-e_r)  (e_r: smallest e >= 0 with max |x| <= 2^14 * 2^e)
//   xsum[r] = [-sum_{k in kb} (c(k) + 8) * x16[r][k] for kb < K/128, e_r, 0...]
// src(r) = perm[r] / k when perm is given (expert-order gather), else r.
__global__ void moe_prep_fp16_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                     const int* __restrict__ perm, int topk, int K,
                                     __half* __restrict__ x16, int ldx16,
                                     float* __restrict__ xsum, int ldxs, int rows,
                                     const int* __restrict__ rows_dev) {
  __shared__ float red[32];
  __shared__ float s_exp;
  const int nrows = rows_dev != nullptr ? min(rows, *rows_dev) : rows;
  for (int r = blockIdx.x; r < nrows; r += gridDim.x) {
  __syncthreads();
  const int src = perm != nullptr ? perm[r] / topk : r;
  const __nv_bfloat16* xr = x + (size_t)src * ldx;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m = 0.f;
  for (int i = threadIdx.x * 8; i < K; i += blockDim.x * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int q = 0; q < 8; ++q) m = fmaxf(m, fabsf(__bfloat162float(v[q])));
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mx = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    s_exp = mx > 16384.f ? ceilf(log2f(mx / 16384.f)) : 0.f;
  }
  __syncthreads();
  const float sc = exp2f(-s_exp);
  // One warp per k-block: convert its 128 values and sum the corrections.
  const int KB = K / 128;
  for (int kb = warp; kb < KB; kb += blockDim.x >> 5) {
    const int k0 = kb * 128 + lane * 4;
    const uint2 u = *reinterpret_cast<const uint2*>(xr + k0);
    const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(&u);
    const __half2 h0 = __floats2half2_rn(__bfloat162float(v[0]) * sc, __bfloat162float(v[1]) * sc);
    const __half2 h1 = __floats2half2_rn(__bfloat162float(v[2]) * sc, __bfloat162float(v[3]) * sc);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&h0);
    o.y = *reinterpret_cast<const uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(x16 + (size_t)r * ldx16 + k0) = o;
    // k % 8 = (lane * 4) % 8 + {0..3}: pairs z = (k % 8) / 2 -> c = {1032, 72, 1032, 72}
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    const float cz0 = ((lane & 1) == 0) ? 1032.f : 1032.f;  // pair (k%8)/2 = 0 or 2
    const float cz1 = 72.f;                                   // pair 1 or 3
    float sum = cz0 * (f0.x + f0.y) + cz1 * (f1.x + f1.y);
    sum = warp_sum(sum);
    if (lane == 0) xsum[(size_t)r * ldxs + kb] = -sum;
  }
  if (threadIdx.x == 0) xsum[(size_t)r * ldxs + KB] = s_exp;
  }
}
}  // namespace

bool gemv_eligible(int64_t M) { return M >= 1 && M <= kGemvMaxM; }

int64_t gemv_workspace_floats(int64_t M, int64_t N, int64_t K, int64_t forced_splits) {
  const int MP = M <= 8 ? 8 : 16;
  const int s = gv_splits((int)(N / 128), (int)(K / 128), MP, (int)forced_splits);
  return s > 1 ? (int64_t)s * M * N : 0;
}

void gemv_launch(const void* x, int64_t ldx, const uint8_t* wblob, void* out, int64_t ldo,
                 const void* residual, int64_t ldr, int M, int N, int K, int group_size,
                 int epilogue, float* ws, int* counters, int* status, int forced_splits,
                 cudaStream_t stream) {
  const int MP = M <= 8 ? 8 : 16;
  const int NT = MP / 8;
  const int KB = K / 128;
  const int row_tiles = N / 128;
  const int splits = gv_splits(row_tiles, KB, MP, forced_splits);
  const int kbps = (KB + splits - 1) / splits;
  GvArgs a{};
  a.wblob = wblob;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.ws = ws;
  a.counters = counters;
  a.status = status;
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldx = (int)ldx;
  a.ldo = (int)ldo;
  a.ldr = (int)ldr;
  a.kbps = kbps;
  a.splits = splits;
  a.pdl = pdl_flag();
  // Persistent CTAs: one per SM in total, each split gets an equal share.
  const int per_split = std::max(1, std::min(row_tiles, num_sms() / splits));
  const dim3 grid(per_split * splits, 1, 1);
  if (group_size == 128) {
    a.stages = gv_stages<128>(kbps, MP);
    const int smem = gv_smem<128>(kbps, MP, a.stages);
    if (epilogue == kGvEpiStore) gv_launch_nt<128, kGvEpiStore>(NT, a, grid, smem, stream);
    else if (epilogue == kGvEpiSilu) gv_launch_nt<128, kGvEpiSilu>(NT, a, grid, smem, stream);
    else gv_launch_nt<128, kGvEpiResid>(NT, a, grid, smem, stream);
  } else {
    a.stages = gv_stages<32>(kbps, MP);
    const int smem = gv_smem<32>(kbps, MP, a.stages);
    if (epilogue == kGvEpiStore) gv_launch_nt<32, kGvEpiStore>(NT, a, grid, smem, stream);
    else if (epilogue == kGvEpiSilu) gv_launch_nt<32, kGvEpiSilu>(NT, a, grid, smem, stream);
    else gv_launch_nt<32, kGvEpiResid>(NT, a, grid, smem, stream);
  }
}

// Prepared-activation layout of the grouped small-M kernel.
static inline int gvg_ldx16(int K) { return K + 8; }                   // halves
static inline int gvg_ldxs(int K) { return ((K / 128 + 1) + 3) / 4 * 4; }  // floats

void moe_prep_fp16(torch::Tensor x, c10::optional<torch::Tensor> perm, int64_t topk,
                   int64_t rows, torch::Tensor x16, torch::Tensor xsum,
                   c10::optional<torch::Tensor> rows_dev) {
  const int K = (int)x.size(1);
  TORCH_CHECK(K % 128 == 0 && x.stride(1) == 1 && (x.stride(0) * 2) % 16 == 0, "x layout");
  TORCH_CHECK(x16.size(1) == gvg_ldx16(K) && xsum.size(1) == gvg_ldxs(K), "prep buffers");
  if (rows == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  // Grid-stride over rows; with rows_dev (a device row count, e.g. the rows
  // an expert-parallel receive produced) only that many rows are prepared.
  const unsigned grid = (unsigned)std::min<int64_t>(rows, rows_dev.has_value() ? 592 : rows);
  moe_prep_fp16_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0),
      perm.has_value() ? perm->data_ptr<int>() : nullptr, (int)topk, K,
      reinterpret_cast<__half*>(x16.data_ptr()), (int)x16.size(1), xsum.data_ptr<float>(),
      (int)xsum.size(1), (int)rows, rows_dev.has_value() ? rows_dev->data_ptr<int>() : nullptr);
  CB_CUDA_CHECK(cudaGetLastError());
}

std::vector<int64_t> moe_prep_shape(int64_t K) { return {gvg_ldx16((int)K), gvg_ldxs((int)K)}; }

template <int EPI>
static void gvg_launch(const GvgArgs& a, int grid, int smem, cudaStream_t stream) {
  static int configured[64] = {};
  int dev = 0;
  CB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(w4a16_gemv_grouped_kernel<EPI>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kGvSmemBudget + 4096));
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  w4a16_gemv_grouped_kernel<EPI><<<grid, kGvThreads, smem, stream>>>(a);
  CB_CUDA_CHECK(cudaGetLastError());
}

// Grouped small-M W4A16 (group 128): x16 / xsum from moe_prep_fp16, rows of
// expert e are [offsets[e], offsets[e+1]); epilogue store or SiLU(gate)*up.
void w4a16_gemv_grouped(torch::Tensor x16, torch::Tensor xsum, torch::Tensor wblob,
                        torch::Tensor out, int64_t N, int64_t epilogue, torch::Tensor offsets,
                        int64_t num_groups, torch::Tensor status,
                        c10::optional<torch::Tensor> out_rows,
                        c10::optional<torch::Tensor> sched) {
  const int K = (int)(x16.size(1) - 8);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "K and N must be multiples of 128");
  TORCH_CHECK(epilogue == kGvEpiStore || epilogue == kGvEpiSilu, "store or SiLU epilogue");
  const int64_t per = (int64_t)(N / 128) * (K / 128) * GvBlob<128>::kBytes;
  TORCH_CHECK(wblob.numel() == per * num_groups, "weight blob has wrong size");
  if (num_groups == 0) return;
  TORCH_CHECK(out_rows.has_value() || out.size(0) >= std::min(x16.size(0), xsum.size(0)),
              "out has fewer rows than the prepared activations");
  TORCH_CHECK(!out_rows.has_value() || out_rows->numel() >= x16.size(0), "out_rows too short");
  const c10::cuda::CUDAGuard guard(x16.device());
  GvgArgs a{};
  a.wblob = wblob.data_ptr<uint8_t>();
  a.blob_stride = per;
  a.x16 = reinterpret_cast<const __half*>(x16.data_ptr());
  a.xsum = xsum.data_ptr<float>();
  a.offsets = offsets.data_ptr<int>();
  a.R = (int)std::min(x16.size(0), xsum.size(0));
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_rows = out_rows.has_value()
                   ? reinterpret_cast<const long long*>(out_rows->data_ptr<int64_t>())
                   : nullptr;
  a.status = status.data_ptr<int>();
  if (sched.has_value()) {
    TORCH_CHECK(sched->is_cuda() && sched->scalar_type() == at::kInt && sched->numel() >= 2,
                "sched must be a cuda int32 tensor of 2 zeros");
    a.sched = sched->data_ptr<int>();
  }
  a.E = (int)num_groups;
  a.N = (int)N;
  a.K = K;
  a.ldx16 = (int)x16.size(1);
  a.ldxs = (int)xsum.size(1);
  a.ldo = (int)out.stride(0);
  const int fixed = (8 * 32 * 4 + 128 * 9) * 4 + 2 * (8 * a.ldx16 * 2 + 8 * a.ldxs * 4) + 1024;
  a.stages = std::max(2, std::min(10, (kGvSmemBudget - fixed) / GvBlob<128>::kStage));
  const int smem = a.stages * GvBlob<128>::kStage + fixed;
  const int units = (int)num_groups * (int)(N / 128);
  const int grid = std::max(1, std::min(units, num_sms()));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (epilogue == kGvEpiSilu) gvg_launch<kGvEpiSilu>(a, grid, smem, stream);
  else gvg_launch<kGvEpiStore>(a, grid, smem, stream);
}

// Python binding: explicit small-M path (tests and the microbenchmark).
void w4a16_gemv(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                int64_t group_size, int64_t epilogue, c10::optional<torch::Tensor> residual,
                torch::Tensor ws, torch::Tensor counters, torch::Tensor status,
                int64_t forced_splits) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "x must be a 2-D cuda bf16 tensor with unit inner stride");
  const int M = (int)x.size(0);
  const int K = (int)x.size(1);
  TORCH_CHECK(gemv_eligible(M), "small-M path takes 1..", kGemvMaxM, " rows");
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "K and N must be multiples of 128");
  TORCH_CHECK(group_size == 128 || group_size == 32, "group size must be 128 or 32");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x rows must be 16-byte aligned");
  TORCH_CHECK(wblob.numel() == (int64_t)(N / 128) * (K / 128) * (8192 + 128 * (128 / group_size) * 2),
              "weight blob has wrong size");
  TORCH_CHECK(epilogue != kGvEpiResid || residual.has_value(), "residual epilogue needs residual");
  const int64_t need = gemv_workspace_floats(M, N, K, forced_splits);
  TORCH_CHECK(ws.numel() >= need, "workspace too small");
  TORCH_CHECK(need == 0 || counters.numel() >= N / 128, "counters too small");
  const c10::cuda::CUDAGuard guard(x.device());
  gemv_launch(x.data_ptr(), x.stride(0), wblob.data_ptr<uint8_t>(), out.data_ptr(), out.stride(0),
              residual.has_value() ? residual->data_ptr() : nullptr,
              residual.has_value() ? residual->stride(0) : 0, M, (int)N, K, (int)group_size,
              (int)epilogue, ws.data_ptr<float>(), counters.data_ptr<int>(), status.data_ptr<int>(),
              (int)forced_splits, at::cuda::getCurrentCUDAStream());
}

}  // namespace cb
