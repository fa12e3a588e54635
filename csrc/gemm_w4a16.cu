// W4A16 GEMM for sm_100a: Y[M, N] = X[M, K] (bf16) * dequant(W[N, K])^T.
//
// W is symmetric INT4 with one bf16 scale per `GS` (128 or 32) consecutive
// K values of a row: value = (q - 8) * scale.  This is the weight format of
// the reference's `cascadia shard` INT4_SYM group-128 layers
// (tools/export_shards.py:1432-1438, crates/cascadia-ov-genai-shim/cpp/gemv_offload.cpp:1-8)
// and of its group-32 expert files (crates/cascadia-int4-gemm/src/kernel.rs:46-70).
//
// Design (swap-AB, tcgen05):
//   * The MMA computes D^T[128 weight rows, MT tokens] = W_tile * X_tile^T with
//     the dequantised weight tile as operand A (M=128) and the activations as
//     operand B (N=MT in 16..256), so decode batches of 1..64 tokens map onto
//     narrow N instead of wasting a 128-row M.
//   * Weights live in a pre-tiled "blob" layout: for each (128-row tile,
//     128-wide k-block) one contiguous 8 KiB block of packed nibbles followed by
//     its scales, fetched with one cp.async.bulk.  Activations are fetched with
//     a 2-D TMA tensor map (128-byte swizzle) straight into the UMMA layout.
//     All of shared memory is this load ring (3..16 stages), so >= 48 KiB of
//     weights are in flight per SM.
//   * The dequantised A tiles live in TENSOR memory: four dequant groups (4
//     warps each, one row per thread, ~2 instructions per weight) write
//     (q - 8) * scale as bf16 with tcgen05.st into four 64-column A buffers, and
//     the MMA reads A from TMEM (tcgen05.mma ... [a_tmem], b_desc).  Four
//     buffers let dequantisation run up to four k-blocks ahead of the MMA, so
//     MMA completion latency never stalls the weight stream.
//   * Warp roles: warp 0 issues TMA, warp 1 owns TMEM and issues tcgen05.mma,
//     warps 2..17 dequantise and later run the epilogue (tcgen05.ld).
//   * Split-K over k-blocks fills the 148 SMs for decode shapes.  Partials go
//     to an fp32 workspace; the last CTA of a tile (per-tile counter) sums the
//     splits in a fixed order, so results are deterministic run to run.
//   * Fused epilogues: plain store, SiLU(gate)*up for interleaved gate/up tiles,
//     and residual add.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <mutex>

#include "gemv_w4a16.h"

#include "common.cuh"
#include "host_utils.h"

namespace cb {

enum Epilogue : int { kEpiStore = 0, kEpiSilu = 1, kEpiResid = 2 };

constexpr int kGroups = 4;                 // dequant groups (A buffers in TMEM)
constexpr int kDequantWarps = 4 * kGroups; // each group: 4 warps = 128 rows
constexpr int kDequantThreads = kDequantWarps * 32;
constexpr int kMaxIssuers = 4;                             // MMA issuing warps
constexpr int kThreads = 64 + kDequantThreads + 32 * (kMaxIssuers - 1);
constexpr int kMmaExtraWarp = 2 + kDequantWarps;           // issuers 1.. live here
constexpr uint32_t kACols = 64;            // TMEM columns of one 128x128 bf16 A tile
constexpr uint32_t kAccCol = kGroups * kACols;  // accumulator starts after the A buffers

template <int GS>
struct BlobInfo {
  static constexpr int kPacked = 128 * 64;                 // 128 rows x 128 nibbles
  static constexpr int kScales = 128 * (128 / GS) * 2;     // bf16
  static constexpr int kBytes = kPacked + kScales;
};

template <int MT, int GS>
struct SmemPlan {
  static constexpr int kXBytes = 2 * MT * 128;  // one k-block of X: two 64-wide K sub-tiles
  // A stage holds TWO consecutive k-blocks: their X tiles, then both weight
  // blobs, which are adjacent in the blob layout and arrive with ONE bulk
  // copy of 16.9 KiB (an SM completes about one bulk copy per ~350 ns, so
  // 8.4 KiB copies cap the weight stream near 3.5 TB/s; 16.9 KiB ones do not).
  static constexpr int kBlobOff = 2 * kXBytes;
  static constexpr int kStageRaw = kBlobOff + 2 * BlobInfo<GS>::kBytes;
  static constexpr int kStage = (kStageRaw + 1023) / 1024 * 1024;
  static constexpr int kBudget = 210 * 1024;
  // Stage count: even, so that every use of a stage is consumed by the same
  // two dequant groups (k-block it goes to group it % 4 and stage
  // (it / 2) % kSL); a group then never waits on a barrier more than one
  // phase ahead of what it observed, which the parity test could not tell
  // apart.
  static constexpr int kSLraw = (kBudget / kStage) / 2 * 2;
  static constexpr int kSL = kSLraw > 8 ? 8 : kSLraw;
  // Independent TMEM accumulators the MMAs rotate over (dependent MMAs into
  // one accumulator serialise on its read-modify-write latency).
  static constexpr int kNAcc = MT <= 32 ? 8 : MT <= 64 ? 4 : 2;
  // MMA issuing warps (one accumulator each): one per dequant group when the
  // accumulators fit next to the A buffers in TMEM.
  static constexpr int kIssuers = MT <= 64 ? 4 : 2;
  static constexpr int kLOff = 0;
  static constexpr int kBarOff = kSL * kStage;
  static constexpr int kTileBytes = 128 * (MT + 1) * 4;
  static_assert(kSL >= 2 && kSL % 2 == 0, "load stages must be a positive even number");
  static_assert(kNAcc * MT <= 256, "accumulators must fit next to the A buffers in TMEM");
  static_assert(kTileBytes <= kBarOff, "epilogue tile must fit in the stage area");
  static constexpr int kTotal = kBarOff + 1024 + 1024;  // barriers + alignment slack
};

struct GemmArgs {
  const uint8_t* wblob;
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;
  float* ws;
  int* counters;
  int* status;
  int M, N, K;
  int ldo, ldr;
  int kb_per_split, splits;
  // Grouped mode (MoE experts): blockIdx.z = expert * group_tiles + tile; the
  // expert's token rows are [group_offsets[e], group_offsets[e + 1]) of X and
  // Y, its weights start at wblob + e * group_blob_stride.
  const int* group_offsets;
  long long group_blob_stride;
  int group_tiles;
  // Diagnostics only: when set, 8 %globaltimer stamps per CTA (start, after
  // set-up, first weights in, all copies issued, last MMA issued,
  // accumulators ready, partials written, end).
  unsigned long long* trace;
  // out (and residual) rows are 16-byte aligned: vectorised epilogue.
  int vec_out;
  // Optional: output row m is stored at out_rows[m] instead of out + m * ldo
  // (expert parallelism: result rows go straight to the source rank's
  // return region in peer memory).
  const long long* out_rows;
  // Launched with programmatic stream serialisation: the producer issues the
  // first stages' weight copies (constant data) before griddepcontrol.wait.
  int pdl;
  // Tensor-parallel push (row-parallel GEMM, store epilogue), npeer > 0:
  // every output tile is stored into each rank's receive slot for this rank
  // (peer_out[q] + row * ldo, plain P2P stores over NVLink) instead of out,
  // and the last tile of the launch to finish raises this rank's flag in
  // every rank's signal pad (peer_sig[q][my_rank] = *push_epoch + 1), after
  // a system-scope fence.
  __nv_bfloat16* peer_out[8];
  int* peer_sig[8];
  int npeer, my_rank;
  int* push_done;          // local: tiles finished in this launch (self-resetting)
  const int* push_epoch;   // local: last completed all-reduce epoch
  // Fused RoPE + paged-KV write (the q/k/v projection, store epilogue),
  // rope_on: head_dim 128 = one 128-row tile per head.  Tile rt < hq is a
  // q head: rotated (pairs d, d + 64) at rope_pos[m] and stored to out.  A
  // k head is rotated and written to the K cache row of slot rope_slots[m],
  // a v head written to the V cache; neither is stored to out.
  int rope_on, rope_hq, rope_hkv, rope_nb;
  const int* rope_pos;
  const float* rope_cs;     // [max_pos, 128] fp32: cos (64) then sin (64)
  const int* rope_slots;
  __nv_bfloat16* rope_kc;   // this layer's K cache [blocks, hkv, 16, 128]
  __nv_bfloat16* rope_vc;
};

__device__ __forceinline__ __nv_bfloat16* gemm_out_row(const GemmArgs& a, int gm) {
  return a.out_rows != nullptr ? reinterpret_cast<__nv_bfloat16*>(a.out_rows[gm])
                               : a.out + (size_t)gm * a.ldo;
}

__device__ __forceinline__ void gemm_stamp(const GemmArgs& a, int k) {
  if (a.trace != nullptr) {
    const size_t cta = ((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    a.trace[cta * 8 + k] = globaltimer();
  }
}

template <int MT, int GS, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmArgs args) {
  using Plan = SmemPlan<MT, GS>;
  constexpr int SL = Plan::kSL;
  constexpr int BLOB = BlobInfo<GS>::kBytes;
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, MT);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align the dynamic smem base to 1024 bytes (128B-swizzle atoms).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* l_smem = smem + Plan::kLOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Plan::kBarOff);
  uint64_t* full_l = bars;
  uint64_t* empty_l = bars + SL;
  uint64_t* full_a = bars + 2 * SL;
  uint64_t* empty_a = bars + 2 * SL + kGroups;
  uint64_t* acc_full = bars + 2 * SL + 2 * kGroups;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * SL + 2 * kGroups + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* is_last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* acc_ok = reinterpret_cast<volatile int*>(tmem_slot + 3);
  float* tile = reinterpret_cast<float*>(smem);  // reused after the main loop

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rt = blockIdx.x;     // 128-row weight tile
  const int split = blockIdx.y;  // k split
  const int tt = blockIdx.z;     // token tile
  const int KB = args.K / 128;
  const int kb0 = split * args.kb_per_split;
  const int kb1 = min(KB, kb0 + args.kb_per_split);
  const int nkb = kb1 - kb0;
  // Token rows of this CTA: [m0, m_lim).  Grouped mode reads the expert's
  // range from device memory; an empty tile leaves before touching anything.
  int m0 = tt * MT, m_lim = args.M;
  const uint8_t* wbase = args.wblob;
  if (args.group_offsets != nullptr) {
    grid_dep_wait();  // the offsets come from the previous kernel
    const int e = blockIdx.z / args.group_tiles;
    const int lt = blockIdx.z % args.group_tiles;
    m0 = args.group_offsets[e] + lt * MT;
    m_lim = args.group_offsets[e + 1];
    wbase = args.wblob + (size_t)e * (size_t)args.group_blob_stride;
    if (m0 >= m_lim) return;
  }

  if (tid == 0) {
    gemm_stamp(args, 0);
    for (int s = 0; s < SL; ++s) {
      mbar_init(&full_l[s], 1);
      // Per k-block of the stage: the consuming dequant group's 4 warps + an
      // MMA commit.  (A final stage holding one k-block never completes: no
      // one waits for it again.)
      mbar_init(&empty_l[s], 2 * (4 + 1));
    }
    for (int g = 0; g < kGroups; ++g) {
      mbar_init(&full_a[g], 4);
      mbar_init(&empty_a[g], 1);
    }
    mbar_init(acc_full, SmemPlan<MT, GS>::kIssuers);  // every MMA issuer commits
    *abort_flag = 0;
    *is_last_flag = 0;
    *acc_ok = 1;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_acc = tmem_base + kAccCol;
  if (tid == 0) gemm_stamp(args, 1);
  // TMEM is held: a dependent kernel's CTAs may now become resident (they
  // cannot take this CTA's columns before it frees them, and it never waits
  // for them).
  if (args.pdl) grid_dep_launch();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      const uint8_t* wsrc = wbase + ((size_t)rt * KB + kb0) * BLOB;
      const int nst = (nkb + 1) / 2;
      auto load_x = [&](int sti, uint8_t* st, uint64_t* bar) {
        const int nb = min(2, nkb - 2 * sti);
        for (int b = 0; b < nb; ++b) {
          const int k = (kb0 + 2 * sti + b) * 128;
          tma_load_2d(st + b * Plan::kXBytes, &tmap_x, k, m0, bar);
          tma_load_2d(st + b * Plan::kXBytes + MT * 128, &tmap_x, k + 64, m0, bar);
        }
      };
      // Weights of the first stages go out before the wait for the previous
      // kernel; X (its output) only after it.
      const int pre = args.pdl ? min(nst, SL) : 0;
      for (int sti = 0; sti < pre; ++sti) {
        const int nb = min(2, nkb - 2 * sti);
        mbar_arrive_expect_tx(&full_l[sti], nb * (Plan::kXBytes + BLOB));
        bulk_g2s(l_smem + sti * Plan::kStage + Plan::kBlobOff, wsrc + (size_t)(2 * sti) * BLOB,
                 nb * BLOB, &full_l[sti]);
      }
      grid_dep_wait();
      for (int sti = 0; sti < pre; ++sti) load_x(sti, l_smem + sti * Plan::kStage, &full_l[sti]);
      int issued = pre;
      for (int sti = pre; sti < nst; ++sti) {
        const int s = sti % SL;
        const uint32_t ph = (sti / SL) & 1;
        if (!mbar_wait(&empty_l[s], ph ^ 1, args.status, kStatusGemmLoadTimeout, abort_flag)) break;
        uint8_t* st = l_smem + s * Plan::kStage;
        const int nb = min(2, nkb - 2 * sti);
        mbar_arrive_expect_tx(&full_l[s], nb * (Plan::kXBytes + BLOB));
        bulk_g2s(st + Plan::kBlobOff, wsrc + (size_t)(2 * sti) * BLOB, nb * BLOB, &full_l[s]);
        load_x(sti, st, &full_l[s]);
        ++issued;
      }
      gemm_stamp(args, 3);
      // Drain: never leave the CTA while our copies still write into smem.
      for (int sti = max(0, issued - SL); sti < issued; ++sti) {
        mbar_wait(&full_l[sti % SL], (sti / SL) & 1, nullptr, 0, nullptr);
      }
    }
  } else if (warp == 1 || warp >= kMmaExtraWarp) {
    // ------------------------------------------------------------ MMA issuers
    // Several issuing warps take k-blocks round-robin, each into its own
    // accumulator: the issue latency of one thread (measured ~64 cycles per
    // tcgen05.mma) does not bound the k-block rate.
    constexpr int NI = Plan::kIssuers;
    const int who = warp == 1 ? 0 : warp - kMmaExtraWarp + 1;
    if (lane == 0 && who < NI) {
      for (int it = who; it < nkb; it += NI) {
        const int s = (it >> 1) % SL;
        const uint32_t phl = ((it >> 1) / SL) & 1;
        const int g = it % kGroups;
        const uint32_t pha = (it / kGroups) & 1;
        if (!mbar_wait(&full_a[g], pha, args.status, kStatusGemmMmaTimeout, abort_flag)) break;
        if (!mbar_wait(&full_l[s], phl, args.status, kStatusGemmMmaTimeout, abort_flag)) break;
        tc_fence_after();
        const uint32_t a_tm = tmem_base + g * kACols;
        const uint32_t x_addr = smem_u32(l_smem + s * Plan::kStage + (it & 1) * Plan::kXBytes);
        const uint32_t d_tm = tmem_acc + who * MT;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t db = umma_desc_sw128(x_addr + (kk >> 2) * (MT * 128) + (kk & 3) * 32);
          mma_bf16_ts(d_tm, a_tm + kk * 8, db, kIdesc, (it < NI && kk == 0) ? 0u : 1u);
        }
        mma_commit(&empty_a[g]);
        mma_commit(&empty_l[s]);
      }
      if (who == 0) gemm_stamp(args, 4);
      mma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------ dequant
    // Group g (warps 2+4g .. 5+4g) handles k-blocks it = g, g+4, ...; inside a
    // group the warp's TMEM lane quarter q picks rows 32q..32q+31, one row per
    // thread.  The thread reads its row's 64 packed bytes (chunk c of row r is
    // stored at c ^ ((r >> 1) & 3): bank-conflict free for 8 consecutive
    // rows), converts 128 nibbles to bf16 (q - 8) * scale and writes the 64
    // bf16x2 columns of its lane into the group's A buffer in TMEM.
    const int t = tid - 64;
    const int grp = t >> 7;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const __nv_bfloat162 k136 = __floats2bfloat162_rn(136.0f, 136.0f);
    const uint32_t l_base = smem_u32(l_smem) + Plan::kBlobOff;
    const uint32_t a_tm = tmem_base + grp * kACols + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    for (int it = grp; it < nkb && ok; it += kGroups) {
      const int s = (it >> 1) % SL;
      const uint32_t phl = ((it >> 1) / SL) & 1;
      const uint32_t pha = (it / kGroups) & 1;
      if (!mbar_wait(&full_l[s], phl, args.status, kStatusGemmDequantTimeout, abort_flag)) {
        ok = false;
        break;
      }
      if (t == 0 && it == 0) gemm_stamp(args, 2);
      const uint32_t wb = l_base + s * Plan::kStage + (it & 1) * BLOB;
      uint4 p[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) p[c] = lds128(wb + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
      __nv_bfloat162 s2[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int si = GS == 128 ? r : r * (128 / GS) + (c * 32) / GS;
        const uint16_t sraw = lds16(wb + BlobInfo<GS>::kPacked + si * 2);
        s2[c] = __halves2bfloat162(__ushort_as_bfloat16(sraw), __ushort_as_bfloat16(sraw));
      }
      // The W part of the stage has been read: release it (the MMA still
      // needs the X part; it commits to the same barrier).
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_l[s]);
      if (!mbar_wait(&empty_a[grp], pha ^ 1, args.status, kStatusGemmDequantTimeout, abort_flag)) {
        ok = false;
        break;
      }
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
            uint32_t v = ((w >> (4 * h)) & 0x000F000Fu) | 0x43004300u;  // bf16 (128 + q)
            __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
            b = __hmul2(__hsub2(b, k136), s2[c]);                      // (q - 8) * scale
            o[wi * 4 + h] = *reinterpret_cast<uint32_t*>(&b);
          }
        }
        tmem_st16(a_tm + c * 16, o);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_a[grp]);
    }

    // ------------------------------------------------------------ epilogue
    grid_dep_wait();  // global reads and writes from here on
    const bool have_acc =
        ok && nkb > 0 && mbar_wait(acc_full, 0, args.status, kStatusGemmEpiTimeout, abort_flag);
    if (!have_acc) *acc_ok = 0;  // made uniform after the next barrier
    if (t == 0) gemm_stamp(args, 5);
    const int cg = grp;                   // which quarter of the MT columns
    const int row = r;                    // weight row inside the tile
    const int n0 = rt * 128;
    const int m_base = m0;
    const int Mpad = gridDim.z * MT;
    constexpr int CQ = MT / 4;            // columns per warp
    tc_fence_after();

    // Phase 1: TMEM -> (workspace | smem tile).  Each thread owns one row.
    float* dst_ws = args.ws;
    if (have_acc) {
      const uint32_t lane_addr = tmem_acc + ((uint32_t)(q * 32) << 16);
      constexpr int CW = CQ >= 16 ? 16 : CQ;
#pragma unroll 1
      for (int c0 = cg * CQ; c0 < (cg + 1) * CQ; c0 += CW) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        // One accumulator per MMA issuer that received a k-block.
        const int nacc = min(Plan::kIssuers, nkb);
#pragma unroll 1
        for (int ai = 0; ai < nacc; ++ai) {
          const uint32_t ad = lane_addr + ai * MT + c0;
          if constexpr (CW == 16) {
            float u[16];
            tmem_ld16(ad, u);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] += u[i];
          } else if constexpr (CW == 8) {
            float u[8];
            tmem_ld8(ad, u);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] += u[i];
          } else {
            float u[4];
            tmem_ld4(ad, u);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] += u[i];
          }
        }
        if (args.splits == 1) {
#pragma unroll
          for (int i = 0; i < CW; ++i) tile[row * (MT + 1) + c0 + i] = v[i];
        } else {
#pragma unroll
          for (int i = 0; i < CW; ++i)
            dst_ws[((size_t)split * Mpad + m_base + c0 + i) * args.N + n0 + row] = v[i];
        }
      }
    }
    tc_fence_before();
    named_bar_sync(1, kDequantThreads);
    if (t == 0) gemm_stamp(args, 6);
    // Every dequant thread takes the same branch (barriers below).  With
    // split-K the counter protocol still runs, so the per-tile counters stay
    // consistent for the next launch.
    if (!*acc_ok && args.splits == 1) {
      // Nothing to write (error path); leave outputs untouched.
    } else {
      bool do_final = true;
      if (args.splits > 1) {
        __threadfence();
        named_bar_sync(1, kDequantThreads);
        if (t == 0) {
          const int tile_id = tt * gridDim.x + rt;
          const int old = atomicAdd(&args.counters[tile_id], 1);
          const int last = (old == args.splits - 1) ? 1 : 0;
          if (last) args.counters[tile_id] = 0;  // ready for the next launch
          *is_last_flag = last;
        }
        named_bar_sync(1, kDequantThreads);
        do_final = *is_last_flag != 0;
        if (do_final) {
          __threadfence();
          // Sum the splits with 16-byte loads, a batch of U splits in flight
          // at once: a load-then-add chain per element would pay the L2
          // latency (~0.7 us) once per element row (13 us at MT = 64).
          constexpr int IT = (32 * MT) / kDequantThreads;  // float4s per thread
          float4 acc[IT];
#pragma unroll
          for (int i = 0; i < IT; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
          constexpr int U = IT >= 8 ? 1 : IT >= 4 ? 2 : 4;  // splits per batch of loads
          for (int sp0 = 0; sp0 < args.splits; sp0 += U) {
            float4 v[U][IT];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
              for (int i = 0; i < IT; ++i) {
                const int idx = t + i * kDequantThreads;
                const int r4 = (idx & 31) * 4, m = idx >> 5;
                v[u][i] = sp0 + u < args.splits
                              ? __ldcg(reinterpret_cast<const float4*>(
                                    &dst_ws[((size_t)(sp0 + u) * Mpad + m_base + m) * args.N +
                                            n0 + r4]))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
              for (int i = 0; i < IT; ++i) {
                acc[i].x += v[u][i].x;
                acc[i].y += v[u][i].y;
                acc[i].z += v[u][i].z;
                acc[i].w += v[u][i].w;
              }
          }
#pragma unroll
          for (int i = 0; i < IT; ++i) {
            const int idx = t + i * kDequantThreads;
            const int r4 = (idx & 31) * 4, m = idx >> 5;
            tile[(r4 + 0) * (MT + 1) + m] = acc[i].x;
            tile[(r4 + 1) * (MT + 1) + m] = acc[i].y;
            tile[(r4 + 2) * (MT + 1) + m] = acc[i].z;
            tile[(r4 + 3) * (MT + 1) + m] = acc[i].w;
          }
          named_bar_sync(1, kDequantThreads);
        }
      }
      // Phase 2: smem tile -> global with the fused epilogue.
      if (do_final) {
        if constexpr (EPI == kEpiSilu) {
          for (int idx = t; idx < 64 * MT; idx += kDequantThreads) {
            const int j = idx & 63;
            const int m = idx >> 6;
            const int gm = m_base + m;
            if (gm < m_lim) {
              const float g = tile[(2 * j) * (MT + 1) + m];
              const float u = tile[(2 * j + 1) * (MT + 1) + m];
              const float y = g / (1.f + __expf(-g)) * u;
              gemm_out_row(args, gm)[rt * 64 + j] = __float2bfloat16(y);
            }
          }
        } else if (EPI == kEpiStore && args.rope_on) {
          const int hh = rt;
          const bool isq = hh < args.rope_hq;
          const bool isk = !isq && hh < args.rope_hq + args.rope_hkv;
          const int kvh = isq ? 0 : (isk ? hh - args.rope_hq : hh - args.rope_hq - args.rope_hkv);
          for (int idx = t; idx < 64 * MT; idx += kDequantThreads) {
            const int j = idx & 63, m = idx >> 6;
            const int gm = m_base + m;
            if (gm >= m_lim) continue;
            // The unfused path rotates the bf16 GEMM output: round first.
            const float x0 = __bfloat162float(__float2bfloat16(tile[j * (MT + 1) + m]));
            const float x1 = __bfloat162float(__float2bfloat16(tile[(j + 64) * (MT + 1) + m]));
            float y0 = x0, y1 = x1;
            if (isq || isk) {
              const float* cs = args.rope_cs + (size_t)args.rope_pos[gm] * 128;
              const float c = cs[j], sn = cs[64 + j];
              y0 = x0 * c - x1 * sn;
              y1 = x1 * c + x0 * sn;
            }
            __nv_bfloat16* dst;
            if (isq) {
              dst = gemm_out_row(args, gm) + n0;
            } else {
              const int slot = args.rope_slots[gm];
              if (slot < 0) continue;
              dst = (isk ? args.rope_kc : args.rope_vc) +
                    ((((size_t)(slot / 16) * args.rope_hkv + kvh) * 16) + slot % 16) * 128;
            }
            dst[j] = __float2bfloat16(y0);
            dst[64 + j] = __float2bfloat16(y1);
          }
        } else if (args.npeer > 0) {
          // Push to every rank's slot: 16 consecutive threads write one
          // row's 256 contiguous bytes, so that a warp's P2P stores are two
          // full 256-byte row pieces (NVLink carries them as a few large
          // writes instead of one 16-byte write per thread).
          for (int idx = t; idx < 16 * MT; idx += kDequantThreads) {
            const int r8 = (idx & 15) * 8, m = idx >> 4;
            const int gm = m_base + m;
            if (gm < m_lim) {
              uint4 o;
              __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
              for (int e = 0; e < 8; ++e) oe[e] = __float2bfloat16(tile[(r8 + e) * (MT + 1) + m]);
              for (int q = 0; q < args.npeer; ++q)
                *reinterpret_cast<uint4*>(args.peer_out[q] + (size_t)gm * args.ldo + n0 + r8) = o;
            }
          }
        } else if (args.vec_out) {
          // 8 outputs (16 bytes) per thread and step, token index fastest
          // (conflict-free tile reads); residual loads all issued up front.
          constexpr int IT = (16 * MT + kDequantThreads - 1) / kDequantThreads;
          uint4 res[IT];
          if constexpr (EPI == kEpiResid) {
#pragma unroll
            for (int i = 0; i < IT; ++i) {
              const int idx = t + i * kDequantThreads;
              const int m = idx % MT, r8 = (idx / MT) * 8;
              const int gm = m_base + m;
              res[i] = (idx < 16 * MT && gm < m_lim)
                           ? *reinterpret_cast<const uint4*>(
                                 &args.residual[(size_t)gm * args.ldr + n0 + r8])
                           : make_uint4(0, 0, 0, 0);
            }
          }
#pragma unroll
          for (int i = 0; i < IT; ++i) {
            const int idx = t + i * kDequantThreads;
            const int m = idx % MT, r8 = (idx / MT) * 8;
            const int gm = m_base + m;
            if (idx < 16 * MT && gm < m_lim) {
              uint4 o;
              __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
              const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&res[i]);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                float y = tile[(r8 + e) * (MT + 1) + m];
                if constexpr (EPI == kEpiResid) y += __bfloat162float(re[e]);
                oe[e] = __float2bfloat16(y);
              }
              *reinterpret_cast<uint4*>(gemm_out_row(args, gm) + n0 + r8) = o;
            }
          }
        } else {
          for (int idx = t; idx < 128 * MT; idx += kDequantThreads) {
            const int rr = idx & 127;
            const int m = idx >> 7;
            const int gm = m_base + m;
            if (gm < m_lim) {
              float y = tile[rr * (MT + 1) + m];
              if constexpr (EPI == kEpiResid)
                y += __bfloat162float(args.residual[(size_t)gm * args.ldr + n0 + rr]);
              if (args.npeer > 0) {
                for (int q = 0; q < args.npeer; ++q)
                  args.peer_out[q][(size_t)gm * args.ldo + n0 + rr] = __float2bfloat16(y);
              } else {
                gemm_out_row(args, gm)[n0 + rr] = __float2bfloat16(y);
              }
            }
          }
        }
        if (args.npeer > 0) {
          // This tile is in every rank's slot: count it; the launch's last
          // tile raises the flag in every rank's pad.
          __threadfence_system();
          named_bar_sync(1, kDequantThreads);
          if (t == 0) {
            const int total = (int)(gridDim.x * gridDim.z);
            const int old = atomicAdd(args.push_done, 1);
            if (old == total - 1) {
              *args.push_done = 0;  // ready for the next launch
              const int e = *reinterpret_cast<const volatile int*>(args.push_epoch) + 1;
              __threadfence_system();
              for (int q = 0; q < args.npeer; ++q) {
                asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(args.peer_sig[q] +
                                                                          args.my_rank),
                             "r"(e)
                             : "memory");
              }
            }
          }
        }
      }
    }
  }

  if (tid == 64) gemm_stamp(args, 7);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side

template <int MT, int GS, int EPI>
void launch_w4a16(const CUtensorMap& tmap, const GemmArgs& a, dim3 grid, cudaStream_t stream) {
  using Plan = SmemPlan<MT, GS>;
  static bool configured = false;  // per instantiation; attribute is per-function
  if (!configured) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(w4a16_gemm_kernel<MT, GS, EPI>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Plan::kTotal));
    configured = true;
  }
  if (a.pdl) {
    launch_kernel(w4a16_gemm_kernel<MT, GS, EPI>, grid, dim3(kThreads), Plan::kTotal, stream, tmap,
                  a);
    return;
  }
  w4a16_gemm_kernel<MT, GS, EPI><<<grid, kThreads, Plan::kTotal, stream>>>(tmap, a);
  CB_CUDA_CHECK(cudaGetLastError());
}

template <int GS, int EPI>
void dispatch_mt(int MT, const CUtensorMap& tmap, const GemmArgs& a, dim3 grid, cudaStream_t s) {
  switch (MT) {
    case 16: launch_w4a16<16, GS, EPI>(tmap, a, grid, s); break;
    case 32: launch_w4a16<32, GS, EPI>(tmap, a, grid, s); break;
    case 64: launch_w4a16<64, GS, EPI>(tmap, a, grid, s); break;
    default: launch_w4a16<128, GS, EPI>(tmap, a, grid, s); break;
  }
}

static int pick_mt(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  return 128;
}

// Number of k-splits.  Every split adds a pipeline fill and a share of the
// fp32 partial reduction, so the rule (fitted to graph-timed sweeps of the
// Llama-3.1-8B shapes at TP = 1, 2, 4 and 8, M = 64, on B200) keeps splits
// few: none once the row tiles nearly fill the SMs or K is short, otherwise
// enough to approach one CTA per SM with at least 4 k-blocks per split,
// at most 4 splits for 24+ tiles and 8 below.  Measured examples (us):
// gate_up 14336x4096 (112 tiles) 17.6 unsplit vs 33.8 at 4 splits; qkv
// 1536x4096 (12 tiles) 17.2 unsplit vs 10.5 at 8; o 4096x1024 7.6 unsplit
// vs 9.1 at 2.
static int pick_splits(int tiles, int KB, int num_sms) {
  if (tiles >= (num_sms * 2) / 3 || KB <= 8) return 1;
  int s = std::min(8, std::min(num_sms / std::max(1, tiles), KB / 4));
  if (tiles >= 24) s = std::min(s, 4);
  return std::max(1, s);
}

struct GemmPlanInfo {
  int MT, splits, kbps, token_tiles, row_tiles;
};

static GemmPlanInfo plan_gemm(int M, int N, int K, int forced_splits) {
  GemmPlanInfo p;
  p.MT = pick_mt(M);
  p.token_tiles = (M + p.MT - 1) / p.MT;
  p.row_tiles = N / 128;
  const int KB = K / 128;
  int splits = forced_splits > 0 ? forced_splits
                                  : pick_splits(p.row_tiles * p.token_tiles, KB, num_sms());
  splits = std::max(1, std::min(splits, KB));
  p.kbps = (KB + splits - 1) / splits;
  p.splits = (KB + p.kbps - 1) / p.kbps;
  return p;
}

// Workspace floats needed for a GEMM of this shape (0 when no split).
static int vec_rows_ok(const torch::Tensor& out, const c10::optional<torch::Tensor>& residual) {
  auto ok = [](const torch::Tensor& t) {
    return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0 && t.stride(0) % 8 == 0;
  };
  return ok(out) && (!residual.has_value() || ok(*residual)) ? 1 : 0;
}

// Diagnostics: per-CTA phase stamps of the tcgen05 kernel (nullptr = off).
static unsigned long long* g_gemm_trace = nullptr;

void w4a16_set_trace(c10::optional<torch::Tensor> buf) {
  g_gemm_trace = buf.has_value()
                     ? reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>())
                     : nullptr;
}

// Decode batches of up to CASCADIA_GEMV_MAX_M (default 8) rows run the
// small-M kernel (gemv_w4a16.cu); 0 disables it.
static int gemv_max_m() {
  static const int v = [] {
    const char* e = std::getenv("CASCADIA_GEMV_MAX_M");
    return e ? std::atoi(e) : 8;
  }();
  return v;
}

// Programmatic dependent launch for the kernels launched from now on (a
// CUDA graph keeps the setting it was captured with).
void set_pdl(bool on) { pdl_flag() = on ? 1 : 0; }
bool pdl_enabled() { return pdl_flag() != 0; }

// Which kernel runs a GEMM.  `forced`: 0 chooses; > 0 the split-K kernel
// with that many k-splits; -2 the small-M kernel (tests and microbenchmarks
// compare the kernels on one shape).
enum GemmPath : int { kPathSplitK = 0, kPathSmallM = 2 };

static GemmPath choose_path(int64_t M, int64_t N, int64_t K, int64_t forced) {
  (void)N;
  (void)K;
  if (forced > 0) return kPathSplitK;
  if (forced == -2) return gemv_eligible(M) ? kPathSmallM : kPathSplitK;
  if (M <= gemv_max_m() && gemv_eligible(M)) return kPathSmallM;
  return kPathSplitK;
}

int64_t w4a16_workspace_floats(int64_t M, int64_t N, int64_t K, int64_t forced_splits) {
  switch (choose_path(M, N, K, forced_splits)) {
    case kPathSmallM: return gemv_workspace_floats(M, N, K, 0);
    default: break;
  }
  GemmPlanInfo p = plan_gemm((int)M, (int)N, (int)K, (int)forced_splits);
  if (p.splits == 1) return 0;
  return (int64_t)p.splits * p.token_tiles * p.MT * N;
}

// Counters any path may use for an [M, N] output (zero between launches):
// split-K one per (token tile, row tile), the small-M kernel one per row
// tile (at least four per row tile are reserved).
int64_t w4a16_counter_count(int64_t M, int64_t N) {
  const int MT = pick_mt((int)M);
  return (int64_t)std::max<int64_t>((M + MT - 1) / MT, 4) * (N / 128);
}

// x: [M, K] bf16 (row stride K).  wblob: uint8 blob.  out: [M, ldo] bf16.
// epilogue: 0 store, 1 silu(gate)*up (out has N/2 columns), 2 residual add.
void w4a16_gemm(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                int64_t group_size, int64_t epilogue, c10::optional<torch::Tensor> residual,
                torch::Tensor ws, torch::Tensor counters, torch::Tensor status,
                int64_t forced_splits) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16, "x must be cuda bf16");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be 2-D with unit inner stride");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1, "out must be bf16");
  const int M = (int)x.size(0);
  const int K = (int)x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "K and N must be multiples of 128");
  TORCH_CHECK(group_size == 128 || group_size == 32, "group size must be 128 or 32");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0, "x row stride must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x must be 16-byte aligned");
  const int64_t blob_bytes =
      (int64_t)(N / 128) * (K / 128) * (8192 + 128 * (128 / group_size) * 2);
  TORCH_CHECK(wblob.numel() == blob_bytes, "weight blob has wrong size");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(epilogue != kEpiResid || residual.has_value(), "residual epilogue needs residual");
  const GemmPath path = choose_path(M, N, K, forced_splits);
  if (path == kPathSmallM) {
    const int64_t need = gemv_workspace_floats(M, N, K, 0);
    TORCH_CHECK(ws.numel() >= need, "workspace too small");
    TORCH_CHECK(need == 0 || counters.numel() >= N / 128, "counters too small");
    gemv_launch(x.data_ptr(), x.stride(0), wblob.data_ptr<uint8_t>(), out.data_ptr(),
                out.stride(0), residual.has_value() ? residual->data_ptr() : nullptr,
                residual.has_value() ? residual->stride(0) : 0, M, (int)N, K, (int)group_size,
                (int)epilogue, ws.data_ptr<float>(), counters.data_ptr<int>(),
                status.data_ptr<int>(), 0, at::cuda::getCurrentCUDAStream());
    return;
  }
  GemmPlanInfo p = plan_gemm(M, (int)N, K, (int)forced_splits);
  if (p.splits > 1) {
    TORCH_CHECK(ws.numel() >= (int64_t)p.splits * p.token_tiles * p.MT * N, "workspace too small");
    TORCH_CHECK(counters.numel() >= (int64_t)p.token_tiles * p.row_tiles, "counters too small");
  }
  GemmArgs a{};
  a.wblob = wblob.data_ptr<uint8_t>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.residual = residual.has_value()
                   ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr())
                   : nullptr;
  a.ldr = residual.has_value() ? (int)residual->stride(0) : 0;
  a.ws = p.splits > 1 ? ws.data_ptr<float>() : nullptr;
  a.counters = p.splits > 1 ? counters.data_ptr<int>() : nullptr;
  a.status = status.data_ptr<int>();
  a.M = M;
  a.N = (int)N;
  a.K = K;
  a.ldo = (int)out.stride(0);
  a.kb_per_split = p.kbps;
  a.splits = p.splits;
  a.trace = g_gemm_trace;
  a.vec_out = vec_rows_ok(out, residual);
  a.pdl = pdl_flag();

  CUtensorMap tmap = make_tmap_2d_bf16(x.data_ptr(), (uint64_t)K, (uint64_t)M,
                                       (uint64_t)x.stride(0) * 2, 64, (uint32_t)p.MT,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  dim3 grid(p.row_tiles, p.splits, p.token_tiles);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (group_size == 128) {
    if (epilogue == kEpiStore) dispatch_mt<128, kEpiStore>(p.MT, tmap, a, grid, stream);
    else if (epilogue == kEpiSilu) dispatch_mt<128, kEpiSilu>(p.MT, tmap, a, grid, stream);
    else dispatch_mt<128, kEpiResid>(p.MT, tmap, a, grid, stream);
  } else {
    if (epilogue == kEpiStore) dispatch_mt<32, kEpiStore>(p.MT, tmap, a, grid, stream);
    else if (epilogue == kEpiSilu) dispatch_mt<32, kEpiSilu>(p.MT, tmap, a, grid, stream);
    else dispatch_mt<32, kEpiResid>(p.MT, tmap, a, grid, stream);
  }
}

// The q/k/v projection with RoPE and the paged-KV write fused into its
// epilogue (see GemmArgs::rope_on): out receives the rotated q heads only;
// k_cache / v_cache are [layers, blocks, hkv, 16, 128], `layer` selects the
// layer.  Head dim 128, full rotation, rotate-half pairs, the tcgen05 kernel
// (M above the small-M threshold, the caller checks).
void w4a16_gemm_rope_kv(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                        int64_t group_size, torch::Tensor ws, torch::Tensor counters,
                        torch::Tensor status, torch::Tensor positions, torch::Tensor cos_sin,
                        torch::Tensor slots, torch::Tensor k_cache, torch::Tensor v_cache,
                        int64_t layer, int64_t hq, int64_t hkv) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "x");
  const int M = (int)x.size(0);
  const int K = (int)x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0 && N == (hq + 2 * hkv) * 128,
              "rope_kv: N must be (hq + 2 hkv) * 128");
  TORCH_CHECK(k_cache.dim() == 5 && k_cache.size(4) == 128 && k_cache.size(3) == 16 &&
                  k_cache.size(2) == hkv && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  v_cache.sizes() == k_cache.sizes(),
              "rope_kv: caches [layers, blocks, hkv, 16, 128]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == 128 &&
                  cos_sin.is_contiguous(),
              "rope_kv: cos_sin fp32 [max_pos, 128]");
  TORCH_CHECK(positions.numel() >= M && slots.numel() >= M &&
                  positions.scalar_type() == at::kInt && slots.scalar_type() == at::kInt,
              "rope_kv: int32 positions / slots");
  TORCH_CHECK(out.size(0) == M && out.size(1) >= hq * 128 && out.stride(1) == 1, "rope_kv: out");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x must be 16-byte aligned");
  const int64_t blob_bytes =
      (int64_t)(N / 128) * (K / 128) * (8192 + 128 * (128 / group_size) * 2);
  TORCH_CHECK(wblob.numel() == blob_bytes, "weight blob has wrong size");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  GemmPlanInfo p = plan_gemm(M, (int)N, K, 0);
  if (p.splits > 1) {
    TORCH_CHECK(ws.numel() >= (int64_t)p.splits * p.token_tiles * p.MT * N, "workspace too small");
    TORCH_CHECK(counters.numel() >= (int64_t)p.token_tiles * p.row_tiles, "counters too small");
  }
  GemmArgs a{};
  a.wblob = wblob.data_ptr<uint8_t>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ws = p.splits > 1 ? ws.data_ptr<float>() : nullptr;
  a.counters = p.splits > 1 ? counters.data_ptr<int>() : nullptr;
  a.status = status.data_ptr<int>();
  a.M = M;
  a.N = (int)N;
  a.K = K;
  a.ldo = (int)out.stride(0);
  a.kb_per_split = p.kbps;
  a.splits = p.splits;
  a.trace = g_gemm_trace;
  a.pdl = pdl_flag();
  const int64_t layer_elems = k_cache.size(1) * hkv * 16 * 128;
  a.rope_on = 1;
  a.rope_hq = (int)hq;
  a.rope_hkv = (int)hkv;
  a.rope_nb = (int)k_cache.size(1);
  a.rope_pos = positions.data_ptr<int>();
  a.rope_cs = cos_sin.data_ptr<float>();
  a.rope_slots = slots.data_ptr<int>();
  a.rope_kc = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()) + layer * layer_elems;
  a.rope_vc = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()) + layer * layer_elems;
  CUtensorMap tmap = make_tmap_2d_bf16(x.data_ptr(), (uint64_t)K, (uint64_t)M,
                                       (uint64_t)x.stride(0) * 2, 64, (uint32_t)p.MT,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  dim3 grid(p.row_tiles, p.splits, p.token_tiles);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (group_size == 128) dispatch_mt<128, kEpiStore>(p.MT, tmap, a, grid, stream);
  else dispatch_mt<32, kEpiStore>(p.MT, tmap, a, grid, stream);
}

// Row-parallel GEMM of one tensor-parallel rank with the push epilogue (see
// GemmArgs::npeer): out_ptrs / sig_ptrs are int64 host tensors of `world`
// device addresses (every rank's receive slot for this rank, every rank's
// signal pad), ldo the slot's row pitch.  Always the split-K tcgen05 kernel.
void w4a16_gemm_push(torch::Tensor x, torch::Tensor wblob, int64_t N, int64_t group_size,
                     torch::Tensor out_ptrs, int64_t ldo, torch::Tensor sig_ptrs, int64_t my_rank,
                     torch::Tensor push_done, torch::Tensor push_epoch, torch::Tensor ws,
                     torch::Tensor counters, torch::Tensor status) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "x");
  TORCH_CHECK(out_ptrs.device().is_cpu() && sig_ptrs.device().is_cpu(), "pointer lists on host");
  const int world = (int)out_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= 8 && sig_ptrs.numel() == world, "1..8 ranks");
  const int M = (int)x.size(0);
  const int K = (int)x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "K and N must be multiples of 128");
  TORCH_CHECK(ldo % 8 == 0 && ldo >= N, "slot row pitch");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x must be 16-byte aligned");
  const int64_t blob_bytes =
      (int64_t)(N / 128) * (K / 128) * (8192 + 128 * (128 / group_size) * 2);
  TORCH_CHECK(wblob.numel() == blob_bytes, "weight blob has wrong size");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  GemmPlanInfo p = plan_gemm(M, (int)N, K, 0);
  if (p.splits > 1) {
    TORCH_CHECK(ws.numel() >= (int64_t)p.splits * p.token_tiles * p.MT * N, "workspace too small");
    TORCH_CHECK(counters.numel() >= (int64_t)p.token_tiles * p.row_tiles, "counters too small");
  }
  GemmArgs a{};
  a.wblob = wblob.data_ptr<uint8_t>();
  a.ws = p.splits > 1 ? ws.data_ptr<float>() : nullptr;
  a.counters = p.splits > 1 ? counters.data_ptr<int>() : nullptr;
  a.status = status.data_ptr<int>();
  a.M = M;
  a.N = (int)N;
  a.K = K;
  a.ldo = (int)ldo;
  a.kb_per_split = p.kbps;
  a.splits = p.splits;
  a.trace = g_gemm_trace;
  a.pdl = pdl_flag();
  auto op = out_ptrs.accessor<int64_t, 1>();
  auto sp = sig_ptrs.accessor<int64_t, 1>();
  bool aligned = true;
  for (int q = 0; q < world; ++q) {
    a.peer_out[q] = reinterpret_cast<__nv_bfloat16*>(op[q]);
    a.peer_sig[q] = reinterpret_cast<int*>(sp[q]);
    aligned = aligned && (op[q] % 16 == 0);
  }
  a.vec_out = aligned ? 1 : 0;
  a.npeer = world;
  a.my_rank = (int)my_rank;
  a.push_done = push_done.data_ptr<int>();
  a.push_epoch = push_epoch.data_ptr<int>();
  CUtensorMap tmap = make_tmap_2d_bf16(x.data_ptr(), (uint64_t)K, (uint64_t)M,
                                       (uint64_t)x.stride(0) * 2, 64, (uint32_t)p.MT,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  dim3 grid(p.row_tiles, p.splits, p.token_tiles);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (group_size == 128) dispatch_mt<128, kEpiStore>(p.MT, tmap, a, grid, stream);
  else dispatch_mt<32, kEpiStore>(p.MT, tmap, a, grid, stream);
}

// Grouped (MoE) GEMM: x holds the tokens of all experts in expert order,
// group_offsets [E + 1] (device) gives each expert's row range, wblob holds E
// weight blobs of identical shape back to back.  max_rows_per_group bounds
// the tiles launched per expert (CTAs of empty tiles exit at once).
void w4a16_gemm_grouped(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                        int64_t group_size, int64_t epilogue, torch::Tensor group_offsets,
                        int64_t num_groups, int64_t max_rows_per_group, torch::Tensor status,
                        c10::optional<torch::Tensor> out_rows) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "x");
  TORCH_CHECK(epilogue != kEpiResid, "grouped GEMM supports store and SiLU epilogues");
  const int M = (int)x.size(0);
  const int K = (int)x.size(1);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "K and N must be multiples of 128");
  const int64_t per =
      (int64_t)(N / 128) * (K / 128) * (8192 + 128 * (128 / group_size) * 2);
  TORCH_CHECK(wblob.numel() == per * num_groups, "weight blob has wrong size");
  if (M == 0 || num_groups == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  const int MT = pick_mt((int)std::max<int64_t>(1, max_rows_per_group));
  const int tiles = (int)((max_rows_per_group + MT - 1) / MT);
  GemmArgs a{};
  a.wblob = wblob.data_ptr<uint8_t>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.status = status.data_ptr<int>();
  a.M = M;
  a.N = (int)N;
  a.K = K;
  a.ldo = (int)out.stride(0);
  a.kb_per_split = K / 128;
  a.splits = 1;
  a.group_offsets = group_offsets.data_ptr<int>();
  a.group_blob_stride = per;
  a.group_tiles = tiles;
  a.vec_out = vec_rows_ok(out, c10::nullopt);
  a.pdl = pdl_flag();
  if (out_rows.has_value()) {
    TORCH_CHECK(out_rows->scalar_type() == at::kLong && out_rows->numel() >= M,
                "out_rows: int64 row addresses, one per row of x");
    // Row addresses must keep 16-byte alignment for the vectorised epilogue.
    TORCH_CHECK(N % 8 == 0, "out_rows needs N % 8 == 0");
    a.out_rows = reinterpret_cast<const long long*>(out_rows->data_ptr<int64_t>());
  }
  CUtensorMap tmap = make_tmap_2d_bf16(x.data_ptr(), (uint64_t)K, (uint64_t)M,
                                       (uint64_t)x.stride(0) * 2, 64, (uint32_t)MT,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  dim3 grid((unsigned)(N / 128), 1, (unsigned)(num_groups * tiles));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (group_size == 128) {
    if (epilogue == kEpiStore) dispatch_mt<128, kEpiStore>(MT, tmap, a, grid, stream);
    else dispatch_mt<128, kEpiSilu>(MT, tmap, a, grid, stream);
  } else {
    if (epilogue == kEpiStore) dispatch_mt<32, kEpiStore>(MT, tmap, a, grid, stream);
    else dispatch_mt<32, kEpiSilu>(MT, tmap, a, grid, stream);
  }
}

// [path, MT, a, b, c, d]: split-K (0): splits, k-blocks per split, token
// tiles, row tiles; small-M (2): zeros.
std::vector<int64_t> w4a16_plan(int64_t M, int64_t N, int64_t K, int64_t forced_splits) {
  const GemmPath path = choose_path(M, N, K, forced_splits);
  if (path == kPathSmallM) return {2, 0, 0, 0, 0, 0};
  GemmPlanInfo p = plan_gemm((int)M, (int)N, (int)K, (int)forced_splits);
  return {0, p.MT, p.splits, p.kbps, p.token_tiles, p.row_tiles};
}

}  // namespace cb

// ------------------------------------------------------------------ no-alloc entry point
// The C entry point declared in gemm_w4a16_noalloc.h: the kernel that
// w4a16_gemm picks for the shape (small-M or split-K),
// with its scratch (fp32 partials, counters and a status word) in a fixed
// file-scope device array instead of caller tensors.
#include "gemm_w4a16_noalloc.h"

#include <cstring>

namespace {

constexpr size_t kNaWsBytes = size_t(CB_NOALLOC_MAX_WS_FLOATS) * 4;
constexpr size_t kNaCounterBytes = size_t(CB_NOALLOC_MAX_COUNTERS) * 4;
constexpr size_t kNaStatusOff = kNaWsBytes + kNaCounterBytes;
static_assert(kNaStatusOff + 256 == CB_NOALLOC_SCRATCH_BYTES, "scratch layout");

}  // namespace

// In host code this name is only a stand-in: the device address comes from
// cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char cb_noalloc_scratch[CB_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNaMaxDevices = 64;
std::mutex g_na_mu;
unsigned char* g_na_base[kNaMaxDevices] = {};

void na_error(char* err, int err_len, const std::string& msg) {
  if (err == nullptr || err_len <= 0) return;
  const size_t n = std::min(msg.size(), (size_t)err_len - 1);
  std::memcpy(err, msg.data(), n);
  err[n] = '\0';
}

template <int GS, int EPI>
cudaError_t na_set_attrs() {
  cudaError_t e = cudaSuccess;
  auto set = [&](const void* f, int bytes) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  };
  set((const void*)cb::w4a16_gemm_kernel<16, GS, EPI>, cb::SmemPlan<16, GS>::kTotal);
  set((const void*)cb::w4a16_gemm_kernel<32, GS, EPI>, cb::SmemPlan<32, GS>::kTotal);
  set((const void*)cb::w4a16_gemm_kernel<64, GS, EPI>, cb::SmemPlan<64, GS>::kTotal);
  set((const void*)cb::w4a16_gemm_kernel<128, GS, EPI>, cb::SmemPlan<128, GS>::kTotal);
  return e;
}

// Set-up for the current device (once): scratch address, the kernels'
// shared-memory attributes (they are per device) and the tensor-map encoder.
cudaError_t na_setup(int dev, unsigned char** base, std::string* why) {
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (g_na_base[dev] != nullptr) {
    *base = g_na_base[dev];
    return cudaSuccess;
  }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, cb_noalloc_scratch);
  if (e != cudaSuccess) {
    *why = "cudaGetSymbolAddress";
    return e;
  }
  const cudaError_t attrs[] = {
      na_set_attrs<128, cb::kEpiStore>(), na_set_attrs<128, cb::kEpiSilu>(),
      na_set_attrs<128, cb::kEpiResid>(), na_set_attrs<32, cb::kEpiStore>(),
      na_set_attrs<32, cb::kEpiSilu>(),  na_set_attrs<32, cb::kEpiResid>()};
  for (cudaError_t a : attrs)
    if (a != cudaSuccess) {
      *why = "cudaFuncSetAttribute";
      return a;
    }
  try {
    (void)cb::encode_tiled_fn();
  } catch (const std::exception& ex) {
    *why = ex.what();
    return cudaErrorUnknown;
  }
  g_na_base[dev] = static_cast<unsigned char*>(p);
  *base = g_na_base[dev];
  return cudaSuccess;
}

bool na_aligned16(const void* p, long long ld) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ld % 8 == 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int cb_w4a16_gemm_noalloc(
    const void* x, long long ldx, const void* wblob, void* out, long long ldo,
    const void* residual, long long ldr, int M, int N, int K, int group_size, int epilogue,
    int* status, void* stream, char* err, int err_len) {
  using namespace cb;
  if (x == nullptr || wblob == nullptr || out == nullptr || M < 0 || N <= 0 || K <= 0 ||
      N % 128 != 0 || K % 128 != 0 || (group_size != 128 && group_size != 32) ||
      epilogue < kEpiStore || epilogue > kEpiResid || ldx < K ||
      ldo < (epilogue == kEpiSilu ? N / 2 : N) || (ldx * 2) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) != 0 ||
      (epilogue == kEpiResid && (residual == nullptr || ldr < N))) {
    na_error(err, err_len,
             "cb_w4a16_gemm_noalloc: invalid argument (K, N multiples of 128; group size 128 or "
             "32; x 16-byte aligned with 16-byte row pitch; residual needed for epilogue 2)");
    return CB_NOALLOC_EINVAL;
  }
  if (M == 0) return CB_NOALLOC_OK;
  // The kernel and its scratch need, exactly as w4a16_gemm chooses them.
  const GemmPath path = choose_path(M, N, K, 0);
  long long ws_floats = 0, counters = 0;
  GemmPlanInfo p{};
  if (path == kPathSmallM) {
    ws_floats = gemv_workspace_floats(M, N, K, 0);
    counters = ws_floats > 0 ? N / 128 : 0;
  } else {
    p = plan_gemm(M, N, K, 0);
    ws_floats = p.splits > 1 ? (long long)p.splits * p.token_tiles * p.MT * N : 0;
    counters = p.splits > 1 ? (long long)p.token_tiles * p.row_tiles : 0;
  }
  if (ws_floats > (long long)CB_NOALLOC_MAX_WS_FLOATS ||
      counters > (long long)CB_NOALLOC_MAX_COUNTERS) {
    na_error(err, err_len,
             "cb_w4a16_gemm_noalloc: M=" + std::to_string(M) + " N=" + std::to_string(N) +
                 " K=" + std::to_string(K) + " needs " + std::to_string(ws_floats) +
                 " scratch floats and " + std::to_string(counters) +
                 " counters; the fixed maximum is " + std::to_string(CB_NOALLOC_MAX_WS_FLOATS) +
                 " floats and " + std::to_string(CB_NOALLOC_MAX_COUNTERS) + " counters");
    return CB_NOALLOC_ETOOBIG;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess && (dev < 0 || dev >= kNaMaxDevices)) e = cudaErrorInvalidDevice;
  if (e != cudaSuccess) {
    na_error(err, err_len, std::string("cb_w4a16_gemm_noalloc: cudaGetDevice: ") +
                               cudaGetErrorString(e));
    return CB_NOALLOC_ECUDA;
  }
  unsigned char* base = nullptr;
  std::string why;
  e = na_setup(dev, &base, &why);
  if (e != cudaSuccess) {
    na_error(err, err_len, "cb_w4a16_gemm_noalloc: set-up failed in " + why + ": " +
                               cudaGetErrorString(e));
    return CB_NOALLOC_ECUDA;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* ws = reinterpret_cast<float*>(base);
  int* ctr = reinterpret_cast<int*>(base + kNaWsBytes);
  // With status == NULL the kernel's error code goes to a scratch word that
  // the next call clears: the code is discarded (the header says so).
  int* st = status != nullptr ? status : reinterpret_cast<int*>(base + kNaStatusOff);
  // What must start at zero: the counters this call uses and (when the
  // scratch word is used) the status.  The partials are written before read.
  if (counters > 0) e = cudaMemsetAsync(ctr, 0, (size_t)counters * 4, s);
  if (e == cudaSuccess && status == nullptr) e = cudaMemsetAsync(st, 0, 4, s);
  if (e != cudaSuccess) {
    na_error(err, err_len, std::string("cb_w4a16_gemm_noalloc: cudaMemsetAsync: ") +
                               cudaGetErrorString(e));
    return CB_NOALLOC_ECUDA;
  }
  try {
    if (path == kPathSmallM) {
      gemv_launch(x, ldx, static_cast<const uint8_t*>(wblob), out, ldo,
                  epilogue == kEpiResid ? residual : nullptr, epilogue == kEpiResid ? ldr : 0, M,
                  N, K, group_size, epilogue, ws, ctr, st, 0, s);
      return CB_NOALLOC_OK;
    }
    GemmArgs a{};
    a.wblob = static_cast<const uint8_t*>(wblob);
    a.out = static_cast<__nv_bfloat16*>(out);
    a.residual = epilogue == kEpiResid ? static_cast<const __nv_bfloat16*>(residual) : nullptr;
    a.ldr = epilogue == kEpiResid ? (int)ldr : 0;
    a.ws = p.splits > 1 ? ws : nullptr;
    a.counters = p.splits > 1 ? ctr : nullptr;
    a.status = st;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ldo = (int)ldo;
    a.kb_per_split = p.kbps;
    a.splits = p.splits;
    // The vectorised epilogue needs 16-byte aligned rows (as w4a16_gemm checks).
    a.vec_out = na_aligned16(out, ldo) &&
                (epilogue != kEpiResid || na_aligned16(residual, ldr)) ? 1 : 0;
    a.pdl = pdl_flag();
    CUtensorMap tmap = make_tmap_2d_bf16(const_cast<void*>(x), (uint64_t)K, (uint64_t)M,
                                         (uint64_t)ldx * 2, 64, (uint32_t)p.MT,
                                         CU_TENSOR_MAP_SWIZZLE_128B);
    const dim3 grid(p.row_tiles, p.splits, p.token_tiles);
    if (group_size == 128) {
      if (epilogue == kEpiStore) dispatch_mt<128, kEpiStore>(p.MT, tmap, a, grid, s);
      else if (epilogue == kEpiSilu) dispatch_mt<128, kEpiSilu>(p.MT, tmap, a, grid, s);
      else dispatch_mt<128, kEpiResid>(p.MT, tmap, a, grid, s);
    } else {
      if (epilogue == kEpiStore) dispatch_mt<32, kEpiStore>(p.MT, tmap, a, grid, s);
      else if (epilogue == kEpiSilu) dispatch_mt<32, kEpiSilu>(p.MT, tmap, a, grid, s);
      else dispatch_mt<32, kEpiResid>(p.MT, tmap, a, grid, s);
    }
  } catch (const std::exception& ex) {
    na_error(err, err_len, std::string("cb_w4a16_gemm_noalloc: ") + ex.what());
    return CB_NOALLOC_ECUDA;
  }
  return CB_NOALLOC_OK;
}
