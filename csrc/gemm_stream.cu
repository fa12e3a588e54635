// Persistent stream-K W4A16 GEMM for decode-sized batches (M <= 64 tokens).
//
// Y[M, N] = X[M, K] (bf16) * dequant(W[N, K])^T, W symmetric INT4 with one
// bf16 scale per GS (128 or 32) K values (value = (q - 8) * scale), stored in
// the pre-tiled blob layout of quant.pack_blob: per (128-row tile, 128-wide
// k-block) 8 KiB of swizzled nibbles followed by the block's scales.
//
// Why a second kernel next to gemm_w4a16.cu's split-K kernel: at decode M
// the weight stream is the whole cost, and measured on B200
//   * tcgen05.mma kind::f16, M = 128, A in TMEM costs ~56 cycles for any
//     N <= 64 (N = 128: 64 cycles, N = 256: 128 cycles), so one SM retires a
//     128x128 k-block (8 MMAs, 8.4 KiB of INT4) per ~445 cycles: at most
//     0.86 of the measured HBM copy bandwidth over 148 SMs;
//   * an SM completes bulk copies at a rate set by their number: copies of
//     16.9 KiB (two k-blocks of one tile) stream at the HBM peak, 8.4 KiB
//     ones near half of it.
// The split-K kernel launches one CTA per (tile, split), so every CTA pays
// the pipeline fill and drain, and 1.5 waves leave SMs idle.  Here one CTA
// per SM streams a contiguous range of the GEMM's (tile pair, k-step)
// iterations without a break between tiles, so the MMA pipe stays busy.
//
// Work decomposition (host: stream_plan):
//   * a "step" is (pair of row tiles, k-step of 1 or 2 k-blocks); the X tile
//     of a k-block is loaded once per step and used by both tiles' MMAs (half
//     the L2 -> SMEM traffic of X);
//   * the steps of the whole GEMM, pair-major, are split into 148 equal
//     contiguous ranges (stream-K).  A CTA's range covers whole pairs plus at
//     most a partial pair at each end; a "unit" is the part of one pair in
//     the range;
//   * units that cover the full K range apply the epilogue directly; a pair
//     split between CTAs is reduced through an fp32 workspace: each
//     contributor writes its partial rows (slot 0 = the CTA's first unit,
//     1 = its last), bumps a per-(tile, lane quarter) counter, and the last
//     to arrive sums all contributions in contributor order (deterministic)
//     and applies the epilogue.  It resets the counter for the next launch.
//
// Warp roles (736 threads, one CTA per SM):
//   warp 0       producer: one 16.9 KiB bulk copy per tile and k-step for the
//                weights and one 3-D TMA copy (128B swizzle) for the step's X,
//                into a ring of stages;
//   warps 1, 22  MMA issuers (one thread each; warp 1 owns TMEM): job j goes
//                to issuer j % 2 and into that issuer's accumulator;
//   warps 2..17  four dequant groups (4 warps = 128 rows each): group j % 4
//                turns job j (one tile x one k-block) into (q - 8) * scale
//                bf16 and writes it with tcgen05.st into A buffer j % 4;
//   warps 18..21 epilogue: tcgen05.ld of a finished unit's accumulators
//                (two sets of two: the next unit's MMAs run while the
//                previous one drains) and the global stores.
// TMEM: 4 A buffers x 64 columns + 4 accumulators x MT columns (<= 512).
//
// Every wait is bounded (common.cuh mbar_wait): on expiry the kernel records
// a status code, raises the CTA's abort flag, drains its own copies, frees
// TMEM and returns.
#include <torch/extension.h>

#include <algorithm>

#include "common.cuh"
#include "gemm_stream.h"
#include "host_utils.h"

namespace cb {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kSGroups = 4;                       // dequant groups = A buffers
constexpr int kSDequantWarps = 4 * kSGroups;
constexpr int kSEpiWarps = 4;
constexpr int kSThreads = 32 * (3 + kSDequantWarps + kSEpiWarps);
constexpr int kSEpiWarp0 = 2 + kSDequantWarps;
constexpr int kSIssuer1Warp = kSEpiWarp0 + kSEpiWarps;  // the second MMA issuer
constexpr uint32_t kSACols = 64;                  // one 128 x 128 bf16 A tile
constexpr int kSStageBudget = 222 * 1024;

template <int GS>
struct SBlob {
  static constexpr int kPacked = 128 * 64;
  static constexpr int kBytes = kPacked + 128 * (128 / GS) * 2;
};

template <int MT, int GS>
struct SPlan {
  static constexpr int kXSub = MT * 128;                   // 64 K values x MT rows, bf16
  static constexpr int kXBytes = 2 * kXSub;                // one k-block of X
  static constexpr int kWOff = 2 * kXBytes;                // X of two k-blocks first
  static constexpr int kStageRaw = kWOff + 4 * SBlob<GS>::kBytes;  // 2 tiles x 2 k-blocks
  static constexpr int kStage = (kStageRaw + 1023) / 1024 * 1024;
  static constexpr int kSLraw = kSStageBudget / kStage;
  static constexpr int kSL = kSLraw > 8 ? 8 : kSLraw;
  static constexpr int kBarOff = kSL * kStage;
  static constexpr int kTotal = kBarOff + 1024 + 1024;     // barriers + alignment slack
  static_assert(kSL >= 2, "need at least two load stages");
  static_assert(4 * kSACols + 4 * MT <= 512, "A buffers + accumulators must fit TMEM");
};

struct StreamArgs {
  const uint8_t* wblob;
  bf16* out;
  const bf16* residual;
  float* ws;
  int* counters;
  int* status;
  int M, N, K, ldo, ldr;
  int tpp, kstep;        // tiles per pair, k-blocks per step
  int pairs, ksteps;     // steps = pairs * ksteps
  int ub, ur;            // CTA c owns steps [c*ub + min(c, ur), ...): ub or ub + 1 steps
  int pdl;
  // Optional per-CTA trace (bench/bench_gemm.py --trace), 24 words per CTA:
  // 0-7 %globaltimer stamps (start, TMEM held, first stage landed, first
  // MMA issued, last MMA issued, first unit stored, last unit stored, end);
  // 8-14 clock64 cycles each role spent waiting (issuer 0 on stages, A
  // buffers and accumulators; dequant warp 4 on stages, on A buffers and
  // working; the producer on free stages); 16-19 issuer 0's cycles issuing
  // MMAs, in per-job commits, in per-step commits and in its whole loop.
  unsigned long long* trace;
};

__device__ __forceinline__ void s_stamp(const StreamArgs& a, int k) {
  if (a.trace != nullptr) a.trace[blockIdx.x * 24 + k] = globaltimer();
}
__device__ __forceinline__ void s_put(const StreamArgs& a, int k, unsigned long long v) {
  if (a.trace != nullptr) a.trace[blockIdx.x * 24 + k] = v;
}

__device__ __forceinline__ int s_begin(int c, int ub, int ur) { return c * ub + min(c, ur); }
__device__ __forceinline__ int s_owner(int i, int ub, int ur) {
  const int t = ur * (ub + 1);
  return i < t ? i / (ub + 1) : ur + (i - t) / ub;
}

// One job = one tile of the pair x one k-block of the step.  All roles walk
// the same sequence of steps and jobs.
struct StepInfo {
  int pair, kb0, nkb, ntl;
  bool unit_first, unit_last;
};

__device__ __forceinline__ StepInfo step_info(const StreamArgs& a, int it, int s0, int s1) {
  StepInfo si;
  si.pair = it / a.ksteps;
  const int ks = it - si.pair * a.ksteps;
  const int KB = a.K >> 7;
  si.kb0 = ks * a.kstep;
  si.nkb = min(a.kstep, KB - si.kb0);
  si.ntl = min(a.tpp, (a.N >> 7) - si.pair * a.tpp);
  si.unit_first = (it == s0) || ks == 0;
  si.unit_last = (it == s1 - 1) || ks == a.ksteps - 1;
  return si;
}

// Final epilogue of CW token columns [m0, m0 + CW) of one 128-row tile: this
// thread owns weight row `row` (output column n) and holds its CW values.
template <int CW, int EPI>
__device__ __forceinline__ void s_store(const StreamArgs& a, const float (&v)[CW], int m0, int rt,
                                        int row, int lane) {
  const int n = rt * 128 + row;
  if constexpr (EPI == 1) {  // SiLU(gate) * up, gate/up rows interleaved
#pragma unroll
    for (int i = 0; i < CW; ++i) {
      const int m = m0 + i;
      const float up = __shfl_xor_sync(0xffffffffu, v[i], 1);
      if ((lane & 1) == 0 && m < a.M) {
        const float g = v[i];
        a.out[(size_t)m * a.ldo + rt * 64 + (row >> 1)] =
            __float2bfloat16(g / (1.f + __expf(-g)) * up);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < CW; ++i) {
      const int m = m0 + i;
      if (m < a.M) {
        float y = v[i];
        if constexpr (EPI == 2) y += __bfloat162float(a.residual[(size_t)m * a.ldr + n]);
        a.out[(size_t)m * a.ldo + n] = __float2bfloat16(y);
      }
    }
  }
}

template <int MT, int GS, int EPI>
__global__ void __launch_bounds__(kSThreads, 1)
    w4a16_stream_kernel(const __grid_constant__ CUtensorMap tmap_x, const StreamArgs a) {
  using Plan = SPlan<MT, GS>;
  constexpr int SL = Plan::kSL;
  constexpr int BLOB = SBlob<GS>::kBytes;
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, MT);
  constexpr uint32_t kAccCol = kSGroups * kSACols;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Plan::kBarOff);
  uint64_t* full_w = bars;                // stage landed (W + X)
  uint64_t* empty_w = bars + SL;          // stage consumed (dequant warps + MMA commit)
  uint64_t* a_full = bars + 2 * SL;       // A buffer written (4 warps)
  uint64_t* a_empty = a_full + kSGroups;  // A buffer read by the MMAs (commit)
  uint64_t* acc_full = a_empty + kSGroups;  // unit's accumulators final (2 commits)
  uint64_t* acc_empty = acc_full + 2;       // drained by the epilogue (4 warps)
  uint64_t* mma_done = acc_empty + 2;       // every MMA of an issuer completed (2)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int cta = blockIdx.x;
  const int s0 = s_begin(cta, a.ub, a.ur);
  const int s1 = s_begin(cta + 1, a.ub, a.ur);
  const int KB = a.K >> 7;

  if (tid == 0) {
    s_stamp(a, 0);
    for (int s = 0; s < SL; ++s) {
      mbar_init(&full_w[s], 1);
      // Released by every dequant warp (after reading its rows, or at once
      // when the step holds no job of its group) and by both MMA issuers.
      mbar_init(&empty_w[s], kSDequantWarps + 2);
    }
    for (int g = 0; g < kSGroups; ++g) {
      mbar_init(&a_full[g], 4);
      mbar_init(&a_empty[g], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 2);
      mbar_init(&acc_empty[b], kSEpiWarps);
      mbar_init(&mma_done[b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (tid == 0) s_stamp(a, 1);
  // TMEM is held: a dependent kernel's CTAs may now become resident.
  if (a.pdl) grid_dep_launch();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      auto load_w = [&](int it, uint8_t* st, uint64_t* bar) {
        const StepInfo si = step_info(a, it, s0, s1);
        for (int t = 0; t < si.ntl; ++t) {
          const int rt = si.pair * a.tpp + t;
          bulk_g2s(st + Plan::kWOff + t * 2 * BLOB,
                   a.wblob + ((size_t)rt * KB + si.kb0) * BLOB, si.nkb * BLOB, bar);
        }
      };
      // X of the whole step in ONE 3-D copy: 2 * kstep slices of 64 K
      // values (an SM completes copies at a rate set by their number, not
      // their size).  A box reaching past K is zero-filled and still
      // counted in full.
      auto load_x = [&](int it, uint8_t* st, uint64_t* bar) {
        const StepInfo si = step_info(a, it, s0, s1);
        tma_load_3d(st, &tmap_x, 0, 0, si.kb0 * 2, bar);
      };
      const uint32_t x_bytes = (uint32_t)(2 * a.kstep * Plan::kXSub);
      auto stage_bytes = [&](int it) {
        const StepInfo si = step_info(a, it, s0, s1);
        return (uint32_t)(si.nkb * si.ntl * BLOB) + x_bytes;
      };
      // Weights (constant) of the first stages go out before the wait for
      // the previous kernel; X (its output) only after it.
      const int pre = a.pdl ? min(s1 - s0, SL) : 0;
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = smem + i * Plan::kStage;
        mbar_arrive_expect_tx(&full_w[i], stage_bytes(s0 + i));
        load_w(s0 + i, st, &full_w[i]);
      }
      grid_dep_wait();
      for (int i = 0; i < pre; ++i) load_x(s0 + i, smem + i * Plan::kStage, &full_w[i]);
      int issued = pre;
      unsigned long long p_wait = 0;
      for (int i = pre; i < s1 - s0; ++i) {
        const int s = i % SL;
        const unsigned long long tp = a.trace ? (unsigned long long)clock64() : 0ull;
        if (!mbar_wait_sleep(&empty_w[s], ((i / SL) & 1) ^ 1, a.status,
                             kStatusGemmLoadTimeout,
                       abort_flag))
          break;
        if (a.trace) p_wait += clock64() - tp;
        uint8_t* st = smem + s * Plan::kStage;
        mbar_arrive_expect_tx(&full_w[s], stage_bytes(s0 + i));
        load_w(s0 + i, st, &full_w[s]);
        load_x(s0 + i, st, &full_w[s]);
        ++issued;
      }
      s_put(a, 14, p_wait);
      // Never leave while our copies still write into shared memory.
      for (int i = max(0, issued - SL); i < issued; ++i)
        mbar_wait_sleep(&full_w[i % SL], (i / SL) & 1, nullptr, 0, nullptr);
    }
  } else if (warp == 1 || warp == kSIssuer1Warp) {
    // ------------------------------------------------------------ MMA issuers
    // Two issuing threads: one thread issues a tcgen05.mma about every 55
    // cycles (plus ~115 per commit), two reach the tensor pipe's rate.
    // Job j goes to issuer j % 2, into the issuer's own accumulator of the
    // unit: with tile pairs that is tile j % 2, with single tiles the two
    // accumulators hold alternate k-blocks and the epilogue adds them.
    const int who = warp == 1 ? 0 : 1;
    if (lane == 0) {
      int j = 0, u = 0;
      bool ok = true, fresh = true;
      unsigned long long w_stage = 0, w_a = 0, w_acc = 0;
      long long c_issue = 0, c_commit = 0, c_step = 0;
      long long c_total = a.trace ? clock64() : 0;
      for (int it = s0; it < s1 && ok; ++it) {
        const int i = it - s0;
        const int s = i % SL;
        const StepInfo si = step_info(a, it, s0, s1);
        unsigned long long tw = a.trace ? (unsigned long long)clock64() : 0ull;
        if (si.unit_first) {
          fresh = true;
          if (!mbar_wait_sleep(&acc_empty[u & 1], ((u >> 1) & 1) ^ 1, a.status,
                               kStatusGemmMmaTimeout, abort_flag)) {
            ok = false;
            break;
          }
        }
        if (a.trace) { const unsigned long long t1 = clock64(); w_acc += t1 - tw; tw = t1; }
        if (!mbar_wait_sleep(&full_w[s], (i / SL) & 1, a.status, kStatusGemmMmaTimeout,
                             abort_flag)) {
          ok = false;
          break;
        }
        if (a.trace) { const unsigned long long t1 = clock64(); w_stage += t1 - tw; tw = t1; }
        if (i == 0 && who == 0) s_stamp(a, 2);
        // Descriptor of the step's X tile; a K step of 16 inside a 64-wide
        // slice moves 32 bytes, the next slice kXSub bytes (the address
        // field is in 16-byte units and never carries out of its 14 bits).
        const uint64_t x_desc = umma_desc_sw128(smem_u32(smem + s * Plan::kStage));
        const uint32_t d_tm = tmem_base + kAccCol + (uint32_t)(((u & 1) * 2 + who) * MT);
        for (int b = 0; b < si.nkb && ok; ++b) {
          for (int t = 0; t < si.ntl; ++t, ++j) {
            if ((j & 1) != who) continue;
            const int g = j & 3;
            const unsigned long long ta = a.trace ? (unsigned long long)clock64() : 0ull;
            if (!mbar_wait_sleep(&a_full[g], (j >> 2) & 1, a.status, kStatusGemmMmaTimeout,
                           abort_flag)) {
              ok = false;
              break;
            }
            if (a.trace) w_a += clock64() - ta;
            tc_fence_after();
            if (j == 0) s_stamp(a, 3);
            const uint32_t a_tm = tmem_base + g * kSACols;
            const uint64_t db = x_desc + (uint64_t)((b * Plan::kXBytes) >> 4);
            const long long c0 = a.trace ? clock64() : 0;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              mma_bf16_ts(d_tm, a_tm + kk * 8,
                          db + (uint64_t)((kk >> 2) * (Plan::kXSub >> 4) + (kk & 3) * 2), kIdesc,
                          (fresh && kk == 0) ? 0u : 1u);
            }
            const long long c1 = a.trace ? clock64() : 0;
            fresh = false;
            mma_commit(&a_empty[g]);
            if (a.trace) {
              c_issue += c1 - c0;
              c_commit += clock64() - c1;
            }
          }
        }
        if (!ok) break;
        const long long c2 = a.trace ? clock64() : 0;
        mma_commit(&empty_w[s]);
        if (si.unit_last) {
          mma_commit(&acc_full[u & 1]);
          ++u;
        }
        if (a.trace) c_step += clock64() - c2;
      }
      if (a.trace) c_total = clock64() - c_total;
      if (who == 0) {
        s_stamp(a, 4);
        s_put(a, 8, w_stage);
        s_put(a, 9, w_a);
        s_put(a, 10, w_acc);
        s_put(a, 16, (unsigned long long)c_issue);
        s_put(a, 17, (unsigned long long)c_commit);
        s_put(a, 18, (unsigned long long)c_step);
        s_put(a, 19, (unsigned long long)c_total);
      }
      // Also on the abort path: TMEM is freed only after the MMAs issued
      // so far have completed.
      mma_commit(&mma_done[who]);
      mbar_wait_sleep(&mma_done[who], 0, nullptr, 0, nullptr);
    }
  } else if (warp < kSEpiWarp0) {
    // ------------------------------------------------------------ dequant
    // Group g = (warp - 2) / 4 takes jobs j with j % 4 == g.  Inside the
    // group the warp's TMEM lane quarter q picks rows 32q..32q+31, one row
    // per thread: 64 packed bytes (chunk c of row r at c ^ ((r >> 1) & 3):
    // conflict-free for 8 consecutive rows) -> 128 bf16 (q - 8) * scale.
    const int grp = (warp - 2) >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const __nv_bfloat162 k136 = __floats2bfloat162_rn(136.0f, 136.0f);
    const uint32_t a_tm = tmem_base + grp * kSACols + ((uint32_t)(q * 32) << 16);
    // Every dequant warp waits for EVERY stage fill in order and releases it:
    // a stage is refilled only after all warps passed it, so a warp never
    // waits on a stage more than one phase ahead of its fills (a parity wait
    // cannot tell further phases apart).
    int j = 0;
    bool ok = true;
    unsigned long long d_stage = 0, d_aempty = 0, d_work = 0;
    for (int it = s0; it < s1 && ok; ++it) {
      const int i = it - s0;
      const int s = i % SL;
      const StepInfo si = step_info(a, it, s0, s1);
      const uint32_t w_base = smem_u32(smem + s * Plan::kStage) + Plan::kWOff;
      unsigned long long td = a.trace ? (unsigned long long)clock64() : 0ull;
      if (!mbar_wait_sleep(&full_w[s], (i / SL) & 1, a.status, kStatusGemmDequantTimeout,
                     abort_flag)) {
        ok = false;
        break;
      }
      if (a.trace) { const unsigned long long t1 = clock64(); d_stage += t1 - td; td = t1; }
      // This warp's jobs in the step (at most one: four groups, at most four
      // jobs per step): read the rows first, then release the stage.
      int jb = -1, jt = 0, jj = 0;
      for (int b = 0; b < si.nkb; ++b)
        for (int t = 0; t < si.ntl; ++t, ++j)
          if ((j & 3) == grp) {
            jb = b;
            jt = t;
            jj = j;
          }
      uint4 p[4];
      __nv_bfloat162 s2[4];
      if (jb >= 0) {
        const uint32_t wb = w_base + jt * 2 * BLOB + jb * BLOB;
#pragma unroll
        for (int c = 0; c < 4; ++c) p[c] = lds128(wb + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int si2 = GS == 128 ? r : r * (128 / GS) + (c * 32) / GS;
          const uint16_t sraw = lds16(wb + SBlob<GS>::kPacked + si2 * 2);
          s2[c] = __halves2bfloat162(__ushort_as_bfloat16(sraw), __ushort_as_bfloat16(sraw));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_w[s]);
      if (jb < 0) continue;
      if (!mbar_wait_sleep(&a_empty[grp], ((jj >> 2) & 1) ^ 1, a.status,
                           kStatusGemmDequantTimeout, abort_flag)) {
        ok = false;
        break;
      }
      if (a.trace) { const unsigned long long t1 = clock64(); d_aempty += t1 - td; td = t1; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t words[4] = {p[c].x, p[c].y, p[c].z, p[c].w};
        uint32_t o[16];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const uint32_t w = words[wi];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            uint32_t v = ((w >> (4 * h)) & 0x000F000Fu) | 0x43004300u;  // bf16 128 + q
            __nv_bfloat162 bv = *reinterpret_cast<__nv_bfloat162*>(&v);
            bv = __hmul2(__hsub2(bv, k136), s2[c]);                    // (q - 8) * scale
            o[wi * 4 + h] = *reinterpret_cast<uint32_t*>(&bv);
          }
        }
        tmem_st16(a_tm + c * 16, o);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[grp]);
      if (a.trace) d_work += clock64() - td;
    }
    if (warp == 4 && lane == 0) {
      s_put(a, 11, d_stage);
      s_put(a, 12, d_aempty);
      s_put(a, 13, d_work);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    grid_dep_wait();  // global reads and writes from here on
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int u = 0, j = 0, j_unit = 0;
    for (int it = s0; it < s1; ++it) {
      const StepInfo si = step_info(a, it, s0, s1);
      if (si.unit_first) j_unit = j;
      j += si.nkb * si.ntl;
      if (!si.unit_last) continue;
      if (!mbar_wait_sleep(&acc_full[u & 1], (u >> 1) & 1, a.status, kStatusGemmEpiTimeout,
                     abort_flag))
        break;
      tc_fence_after();
      const int p0 = si.pair * a.ksteps;       // the pair's first step
      const int p1 = p0 + a.ksteps;            // one past its last
      const bool full = max(s0, p0) == p0 && min(s1, p1) == p1;
      const int first_c = full ? cta : s_owner(p0, a.ub, a.ur);
      const int last_c = full ? cta : s_owner(p1 - 1, a.ub, a.ur);
      const int slot = s0 < p0 ? 1 : 0;        // 0: this CTA's first unit
      const uint32_t acc0 = tmem_base + kAccCol + (uint32_t)((u & 1) * 2 * MT) + lane_off;
      // Single tiles: accumulator i holds the unit's jobs of parity i.
      const bool used0 = (j - j_unit) >= 2 || (j_unit & 1) == 0;
      const bool used1 = (j - j_unit) >= 2 || (j_unit & 1) == 1;
      // 16 token columns of tile t's result (this CTA's part of the K range).
      auto load16 = [&](int t, int c0, float (&x)[16]) {
        if (a.tpp == 2) {
          tmem_ld16(acc0 + t * MT + c0, x);
          return;
        }
        if (used0) {
          tmem_ld16(acc0 + c0, x);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] = 0.f;
        }
        if (used1) {
          float y[16];
          tmem_ld16(acc0 + MT + c0, y);
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] += y[e];
        }
      };
      for (int t = 0; t < si.ntl; ++t) {
        const int rt = si.pair * a.tpp + t;
        // Partials: [MT / 4][128 rows][4] floats per (CTA, slot, tile), so
        // that a thread moves its row's values as float4s and a warp's
        // accesses are 512 contiguous bytes.
        float4* mine = reinterpret_cast<float4*>(a.ws) +
                       ((size_t)(cta * 2 + slot) * 2 + t) * (MT / 4) * 128;
#pragma unroll 1
        for (int c0 = 0; c0 < MT; c0 += 16) {
          float v[16];
          load16(t, c0, v);
          if (full) {
            s_store<16, EPI>(a, v, c0, rt, row, lane);
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              mine[(c0 / 4 + i) * 128 + row] =
                  make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        }
        if (full) continue;
        // Partial tile: publish, count, and the last contributor finishes.
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          int* ctr = a.counters + rt * 4 + q;
          const int old = atomicAdd(ctr, 1);
          last = old == last_c - first_c;
          if (last) *ctr = 0;  // ready for the next launch
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        // Sum every contribution in contributor order (deterministic), 16
        // columns at a time; a contributor's four float4 loads are issued
        // together.  This CTA's own part is re-read from TMEM.
#pragma unroll 1
        for (int c0 = 0; c0 < MT; c0 += 16) {
          float acc[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll 2
          for (int c = first_c; c <= last_c; ++c) {
            float x[16];
            if (c == cta) {
              load16(t, c0, x);
            } else {
              const int cs = s_begin(c, a.ub, a.ur) < p0 ? 1 : 0;
              const float4* src = reinterpret_cast<const float4*>(a.ws) +
                                  ((size_t)(c * 2 + cs) * 2 + t) * (MT / 4) * 128;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 f = __ldcg(src + (c0 / 4 + i) * 128 + row);
                x[4 * i] = f.x;
                x[4 * i + 1] = f.y;
                x[4 * i + 2] = f.z;
                x[4 * i + 3] = f.w;
              }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] += x[i];
          }
          s_store<16, EPI>(a, acc, c0, rt, row, lane);
        }
      }
      // Every tile read: the next-but-one unit may reuse the accumulators.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[u & 1]);
      if (warp == kSEpiWarp0 && lane == 0) s_stamp(a, u == 0 ? 5 : 6);
      ++u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (tid == 0) s_stamp(a, 7);
}

template <int MT, int GS, int EPI>
cudaError_t set_stream_attr() {
  return cudaFuncSetAttribute(w4a16_stream_kernel<MT, GS, EPI>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, SPlan<MT, GS>::kTotal);
}

template <int MT, int GS, int EPI>
void launch_stream(const CUtensorMap& tmap, const StreamArgs& a, int ctas, cudaStream_t stream) {
  using Plan = SPlan<MT, GS>;
  static bool configured[64] = {};  // the attribute is set once per device
  int dev = 0;
  CB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    CB_CUDA_CHECK((set_stream_attr<MT, GS, EPI>()));
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  launch_kernel(w4a16_stream_kernel<MT, GS, EPI>, dim3(ctas), dim3(kSThreads),
                (size_t)Plan::kTotal, stream, tmap, a);
}

template <int GS, int EPI>
void dispatch_stream(int MT, const CUtensorMap& tmap, const StreamArgs& a, int ctas,
                     cudaStream_t s) {
  switch (MT) {
    case 16: launch_stream<16, GS, EPI>(tmap, a, ctas, s); break;
    case 32: launch_stream<32, GS, EPI>(tmap, a, ctas, s); break;
    default: launch_stream<64, GS, EPI>(tmap, a, ctas, s); break;
  }
}

template <int GS>
cudaError_t set_stream_attrs_gs() {
  const cudaError_t r[] = {set_stream_attr<16, GS, 0>(), set_stream_attr<16, GS, 1>(),
                           set_stream_attr<16, GS, 2>(), set_stream_attr<32, GS, 0>(),
                           set_stream_attr<32, GS, 1>(), set_stream_attr<32, GS, 2>(),
                           set_stream_attr<64, GS, 0>(), set_stream_attr<64, GS, 1>(),
                           set_stream_attr<64, GS, 2>()};
  for (cudaError_t e : r)
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace

cudaError_t stream_set_attrs() {
  const cudaError_t e = set_stream_attrs_gs<128>();
  return e != cudaSuccess ? e : set_stream_attrs_gs<32>();
}

StreamPlan stream_plan(int M, int N, int K, int num_sms_) {
  StreamPlan p{};
  p.MT = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  const int T = N / 128, KB = K / 128;
  p.tpp = T % 2 == 0 ? 2 : 1;
  p.kstep = 2;
  auto steps = [&] {
    p.pairs = (T + p.tpp - 1) / p.tpp;
    p.ksteps = (KB + p.kstep - 1) / p.kstep;
    return (long)p.pairs * p.ksteps;
  };
  // Coarse steps (two tiles x two k-blocks) keep copies large and share X;
  // small GEMMs take finer steps so that every SM gets work.
  if (steps() < 2L * num_sms_ && p.kstep == 2 && KB > 1) p.kstep = 1;
  if (steps() < 2L * num_sms_ && p.tpp == 2) p.tpp = 1;
  const long I = steps();
  p.ctas = (int)std::min<long>(num_sms_, I);
  p.ub = (int)(I / p.ctas);
  p.ur = (int)(I % p.ctas);
  p.ws_floats = (long long)p.ctas * 2 * 2 * p.MT * 128;
  p.counters = T * 4;
  return p;
}

bool stream_eligible(int M, int N, int K) {
  return M >= 1 && M <= 64 && N % 128 == 0 && K % 128 == 0 && N > 0 && K > 0;
}

void stream_launch(const void* x, int64_t ldx, const uint8_t* wblob, void* out, int64_t ldo,
                   const void* residual, int64_t ldr, int M, int N, int K, int group_size,
                   int epilogue, float* ws, int* counters, int* status, cudaStream_t stream,
                   unsigned long long* trace) {
  const StreamPlan p = stream_plan(M, N, K, num_sms());
  StreamArgs a{};
  a.wblob = wblob;
  a.out = static_cast<bf16*>(out);
  a.residual = static_cast<const bf16*>(residual);
  a.ws = ws;
  a.counters = counters;
  a.status = status;
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldo = (int)ldo;
  a.ldr = (int)ldr;
  a.tpp = p.tpp;
  a.kstep = p.kstep;
  a.pairs = p.pairs;
  a.ksteps = p.ksteps;
  a.ub = p.ub;
  a.ur = p.ur;
  a.pdl = pdl_flag();
  a.trace = trace;
  const CUtensorMap tmap = make_tmap_kchunks_bf16(const_cast<void*>(x), (uint64_t)K, (uint64_t)M,
                                                  (uint64_t)ldx * 2, (uint32_t)p.MT,
                                                  (uint32_t)(2 * p.kstep));
  if (group_size == 128) {
    if (epilogue == 0) dispatch_stream<128, 0>(p.MT, tmap, a, p.ctas, stream);
    else if (epilogue == 1) dispatch_stream<128, 1>(p.MT, tmap, a, p.ctas, stream);
    else dispatch_stream<128, 2>(p.MT, tmap, a, p.ctas, stream);
  } else {
    if (epilogue == 0) dispatch_stream<32, 0>(p.MT, tmap, a, p.ctas, stream);
    else if (epilogue == 1) dispatch_stream<32, 1>(p.MT, tmap, a, p.ctas, stream);
    else dispatch_stream<32, 2>(p.MT, tmap, a, p.ctas, stream);
  }
}

}  // namespace cb
