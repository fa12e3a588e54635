// Dense bf16 GEMM on the 5th-generation tensor cores: Y[M, N] = X[M, K] W[N, K]^T
// (+ residual), bf16 in and out, fp32 accumulation in tensor memory.
//
// Used for the projections that stay bf16 (the attention projections of the
// sparse-MoE configs, the GLM-5 MTP input projection).  Swap-AB like the INT4
// GEMM: a 128-row weight tile is the MMA's M operand and a tile of TN tokens
// (32..256) is its N operand, so decode batches fill the instruction's wide
// side instead of padding 128 token rows.
//
// One CTA = one (128 weight rows, TN tokens, k-split) tile, 4 warps:
//   warp 0 lane 0  producer: one 2-D TMA load of the weight tile [128 x 64]
//                  and one of the activation tile [TN x 64] per stage (both
//                  128-byte swizzled, K-major), into a ring of mbarrier stages.
//                  The weight loads of the first stages go out before the
//                  programmatic-dependent-launch wait (weights are not
//                  produced by the previous kernel).
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma kind::f16 (K = 16 each) per
//                  stage, both operands from shared memory, one commit per
//                  stage releasing it, one commit when the accumulator is done.
//   all 4 warps    epilogue: warp w reads TMEM lanes 32w..32w+31 (one weight
//                  row per thread), 16 token columns per tcgen05.ld, and
//                  writes bf16 rows (+ residual); with split-K it writes fp32
//                  partials and the last CTA of the tile (atomic counter,
//                  reset by it) sums them in split order (deterministic).
// Every wait is bounded: on timeout the thread records a status code, stops
// issuing, and the CTA drains its copies and frees TMEM before leaving.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {
namespace {

constexpr int kBfThreads = 128;

// KS = 64-wide K slices per stage.  With KS > 1 each row of a weight tile
// arrives as KS x 128 contiguous bytes (a 3-D tensor map over the slices),
// which streams from HBM better than one 128-byte piece per row.
template <int TN, int KS>
struct BfPlan {
  static constexpr int kWBytes = 128 * 128 * KS;  // 128 rows x 64*KS bf16
  static constexpr int kXBytes = TN * 128 * KS;   // TN rows x 64*KS bf16
  static constexpr int kStage = kWBytes + kXBytes;
  static constexpr int kStagesRaw = (200 * 1024) / kStage;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kBarOff = kStages * kStage;
  static constexpr int kSmem = kBarOff + 256 + 1024;  // barriers + alignment slack
  static constexpr uint32_t kTmemCols = TN < 32 ? 32 : TN;
};

struct BfArgs {
  int M, N, K;
  int kb_per_split, splits;
  __nv_bfloat16* out;
  int ldo;
  const __nv_bfloat16* resid;
  int ldr;
  float* ws;
  int* counters;
  int* status;
  int pdl;
};

template <int TN, int KS, bool T3>
__global__ void __launch_bounds__(kBfThreads, 1)
    bf16_gemm_kernel(const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_x, const BfArgs a) {
  using P = BfPlan<TN, KS>;
  constexpr int S = P::kStages;
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, TN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P::kBarOff);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* acc_ok = reinterpret_cast<volatile int*>(tmem_slot + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rt = blockIdx.x, split = blockIdx.y, tt = blockIdx.z;
  const int n0 = rt * 128, m0 = tt * TN;
  const int KB = (a.K + 64 * KS - 1) / (64 * KS);  // k-blocks of 64*KS
  const int kb0 = split * a.kb_per_split;
  const int nkb = max(0, min(KB, kb0 + a.kb_per_split) - kb0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *last_flag = 0;
    *acc_ok = 1;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, P::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (a.pdl) grid_dep_launch();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
    const int pre = a.pdl ? min(nkb, S) : 0;
    // T3: 3-D maps {64, rows, K/64}; slice coordinate = k-block * KS.
    auto load = [&](const CUtensorMap* m, uint8_t* dst, int row, int kb, uint64_t* bar) {
      if constexpr (T3) tma_load_3d(dst, m, 0, row, kb * KS, bar);
      else tma_load_2d(dst, m, kb * 64, row, bar);
    };
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + i * P::kStage;
      mbar_arrive_expect_tx(&full[i], P::kStage);
      load(&tm_w, st, n0, kb0 + i, &full[i]);
    }
    grid_dep_wait();
    for (int i = 0; i < pre; ++i)
      load(&tm_x, smem + i * P::kStage + P::kWBytes, m0, kb0 + i, &full[i]);
    int issued = pre;
    for (int i = pre; i < nkb; ++i) {
      const int s = i % S;
      if (!mbar_wait(&empty[s], ((i / S) & 1) ^ 1, a.status, kStatusGemmLoadTimeout, abort_flag))
        break;
      uint8_t* st = smem + s * P::kStage;
      mbar_arrive_expect_tx(&full[s], P::kStage);
      load(&tm_w, st, n0, kb0 + i, &full[s]);
      load(&tm_x, st + P::kWBytes, m0, kb0 + i, &full[s]);
      ++issued;
    }
    // Never leave while a copy still writes into shared memory.
    for (int i = max(0, issued - S); i < issued; ++i)
      mbar_wait(&full[i % S], (i / S) & 1, nullptr, 0, nullptr);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int done = 0;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      if (!mbar_wait(&full[s], (i / S) & 1, a.status, kStatusGemmMmaTimeout, abort_flag)) break;
      tc_fence_after();
      const uint32_t w_addr = smem_u32(smem + s * P::kStage);
      const uint32_t x_addr = w_addr + P::kWBytes;
#pragma unroll
      for (int sl = 0; sl < KS; ++sl)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16_ss(tmem, umma_desc_sw128(w_addr + sl * (128 * 128) + kk * 32),
                      umma_desc_sw128(x_addr + sl * (TN * 128) + kk * 32), kIdesc,
                      (i | sl | kk) != 0 ? 1u : 0u);
        }
      mma_commit(&empty[s]);
      ++done;
    }
    if (done < nkb) *acc_ok = 0;
    mma_commit(acc_full);
  }
  __syncwarp();

  // -------------------------------------------------------------- epilogue
  grid_dep_wait();
  if (!mbar_wait(acc_full, 0, a.status, kStatusGemmEpiTimeout, abort_flag)) *acc_ok = 0;
  tc_fence_after();
  __syncthreads();
  const bool ok = *acc_ok != 0 && nkb > 0;
  const int n = n0 + tid;  // this thread's weight row (TMEM lane)
  const int Mpad = gridDim.z * TN;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
  if (ok) {
#pragma unroll 1
    for (int c0 = 0; c0 < TN; c0 += 16) {
      if (m0 + c0 >= a.M) break;  // uniform across the CTA
      __syncwarp();                  // tcgen05.ld is warp-collective
      float v[16];
      tmem_ld16(lane_addr + c0, v);
      if (n >= a.N) {
        // rows past N: nothing to write
      } else if (a.splits == 1) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int m = m0 + c0 + i;
          if (m < a.M) {
            float y = v[i];
            if (a.resid != nullptr) y += __bfloat162float(a.resid[(size_t)m * a.ldr + n]);
            a.out[(size_t)m * a.ldo + n] = __float2bfloat16(y);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          a.ws[((size_t)split * Mpad + m0 + c0 + i) * a.N + n] = v[i];
      }
    }
  }
  tc_fence_before();
  if (a.splits > 1) {
    // The counter protocol runs on the error path too, so the per-tile
    // counters are back at zero for the next launch.
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int tile_id = tt * gridDim.x + rt;
      const int old = atomicAdd(&a.counters[tile_id], 1);
      const int last = old == a.splits - 1;
      if (last) a.counters[tile_id] = 0;
      *last_flag = last;
    }
    __syncthreads();
    if (*last_flag && ok) {
      __threadfence();
      // Sum the splits for the tile: thread (r, q) owns columns
      // n0 + 4q .. n0 + 4q + 3 of token rows r, r + 4, ...  Loads are float4
      // and up to JB x SB of them are in flight per thread, so the tail costs
      // a few L2 round trips instead of one per token row and split.
      constexpr int J = TN / 4;
      constexpr int JB = J < 8 ? J : 8;
      constexpr int SB = 4;
      const int q = tid & 31, r = tid >> 5;
      const int nq = n0 + 4 * q;
      const bool vec = (a.N % 4) == 0 && nq + 3 < a.N;
#pragma unroll 1
      for (int j0 = 0; j0 < J; j0 += JB) {
        float4 acc[JB];
#pragma unroll
        for (int jj = 0; jj < JB; ++jj) acc[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
        for (int sp0 = 0; sp0 < a.splits; sp0 += SB) {
          float4 v[SB][JB];
#pragma unroll
          for (int u = 0; u < SB; ++u)
#pragma unroll
            for (int jj = 0; jj < JB; ++jj) {
              const int m = m0 + r + 4 * (j0 + jj);
              const float* src = &a.ws[((size_t)(sp0 + u) * Mpad + m) * a.N + nq];
              if (sp0 + u >= a.splits || m >= a.M || nq >= a.N) {
                v[u][jj] = make_float4(0.f, 0.f, 0.f, 0.f);
              } else if (vec) {
                v[u][jj] = __ldcg(reinterpret_cast<const float4*>(src));
              } else {
                v[u][jj].x = __ldcg(src);
                v[u][jj].y = nq + 1 < a.N ? __ldcg(src + 1) : 0.f;
                v[u][jj].z = nq + 2 < a.N ? __ldcg(src + 2) : 0.f;
                v[u][jj].w = nq + 3 < a.N ? __ldcg(src + 3) : 0.f;
              }
            }
#pragma unroll
          for (int u = 0; u < SB; ++u)
#pragma unroll
            for (int jj = 0; jj < JB; ++jj) {
              acc[jj].x += v[u][jj].x;
              acc[jj].y += v[u][jj].y;
              acc[jj].z += v[u][jj].z;
              acc[jj].w += v[u][jj].w;
            }
        }
#pragma unroll
        for (int jj = 0; jj < JB; ++jj) {
          const int m = m0 + r + 4 * (j0 + jj);
          if (m >= a.M) continue;
          const float y[4] = {acc[jj].x, acc[jj].y, acc[jj].z, acc[jj].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int nn = nq + e;
            if (nn < a.N) {
              float o = y[e];
              if (a.resid != nullptr) o += __bfloat162float(a.resid[(size_t)m * a.ldr + nn]);
              a.out[(size_t)m * a.ldo + nn] = __float2bfloat16(o);
            }
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, P::kTmemCols);
}

struct BfPlanHost {
  int TN, KS, t3, tiles_n, tiles_m, splits, kbps;
};

BfPlanHost bf16_plan(int M, int N, int K, int forced) {
  BfPlanHost p;
  p.TN = M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  p.t3 = (K % 64) == 0;
  p.KS = (p.t3 && p.TN <= 64) ? 2 : 1;
  p.tiles_n = (N + 127) / 128;
  p.tiles_m = (M + p.TN - 1) / p.TN;
  const int KB64 = (K + 63) / 64;
  const int tiles = p.tiles_n * p.tiles_m;
  int s = 1;
  if (forced > 0) {
    s = forced;
  } else if (tiles < num_sms() / 2 && KB64 >= 16) {
    s = std::min(8, std::min(num_sms() / tiles, KB64 / 8));
  }
  const int KB = (KB64 + p.KS - 1) / p.KS;  // k-blocks of 64 * KS
  s = std::max(1, std::min(s, KB));
  p.kbps = (KB + s - 1) / s;
  p.splits = (KB + p.kbps - 1) / p.kbps;  // no empty split
  return p;
}

template <int TN, int KS, bool T3>
void launch_bf16(const CUtensorMap& tw, const CUtensorMap& tx, const BfArgs& a, dim3 grid,
                 cudaStream_t stream) {
  using P = BfPlan<TN, KS>;
  static bool attr = false;
  if (!attr) {
    CB_CUDA_CHECK(cudaFuncSetAttribute(bf16_gemm_kernel<TN, KS, T3>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, P::kSmem));
    attr = true;
  }
  launch_kernel(bf16_gemm_kernel<TN, KS, T3>, grid, dim3(kBfThreads), P::kSmem, stream, tw, tx,
                a);
}

}  // namespace

// [token tile, weight-row tiles, token tiles, splits, workspace floats, counters]
std::vector<int64_t> bf16_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t splits) {
  const BfPlanHost p = bf16_plan((int)M, (int)N, (int)K, (int)splits);
  const int64_t ws = p.splits > 1 ? (int64_t)p.splits * p.tiles_m * p.TN * N : 0;
  return {p.TN, p.tiles_n, p.tiles_m, p.splits, ws, (int64_t)p.tiles_n * p.tiles_m};
}

// out[M, N] = x[M, K] @ w[N, K]^T (+ residual).  ws / counters: split-K
// scratch (fp32, counters zero on entry and on return).
void bf16_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor out,
               c10::optional<torch::Tensor> residual, torch::Tensor ws, torch::Tensor counters,
               torch::Tensor status, int64_t splits) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "bf16_gemm: bf16 tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1) && x.size(1) > 0,
              "bf16_gemm: shapes");
  const int M = (int)x.size(0), K = (int)x.size(1), N = (int)w.size(0);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "bf16_gemm: out");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && (x.stride(0) * 2) % 16 == 0 &&
                  (w.stride(0) * 2) % 16 == 0 && K % 8 == 0,
              "bf16_gemm: rows must be 16-byte multiples (K % 8 == 0)");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "bf16_gemm: x and w must start on 16-byte boundaries");
  if (M == 0 || N == 0) return;
  const BfPlanHost p = bf16_plan(M, N, K, (int)splits);
  const int64_t need_ws = p.splits > 1 ? (int64_t)p.splits * p.tiles_m * p.TN * N : 0;
  TORCH_CHECK(ws.numel() >= need_ws && counters.numel() >= (int64_t)p.tiles_n * p.tiles_m,
              "bf16_gemm: workspace too small");
  const c10::cuda::CUDAGuard guard(x.device());
  BfArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.kb_per_split = p.kbps;
  a.splits = p.splits;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = (int)out.stride(0);
  a.resid = nullptr;
  a.ldr = 0;
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->size(0) == M &&
                    residual->size(1) == N && residual->stride(1) == 1,
                "bf16_gemm: residual");
    a.resid = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ldr = (int)residual->stride(0);
  }
  a.ws = ws.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.pdl = pdl_flag();
  const dim3 grid(p.tiles_n, p.splits, p.tiles_m);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (p.t3) {
    // K-slice maps: dims {64, rows, K / 64}; one load = KS slices of a tile.
    const CUtensorMap tw = make_tmap_kchunks_bf16(w.data_ptr(), (uint64_t)K, (uint64_t)N,
                                                  (uint64_t)w.stride(0) * 2, 128, p.KS);
    const CUtensorMap tx = make_tmap_kchunks_bf16(x.data_ptr(), (uint64_t)K, (uint64_t)M,
                                                  (uint64_t)x.stride(0) * 2, p.TN, p.KS);
    switch (p.TN) {
      case 32: launch_bf16<32, 2, true>(tw, tx, a, grid, stream); break;
      case 64: launch_bf16<64, 2, true>(tw, tx, a, grid, stream); break;
      case 128: launch_bf16<128, 1, true>(tw, tx, a, grid, stream); break;
      default: launch_bf16<256, 1, true>(tw, tx, a, grid, stream); break;
    }
  } else {
    const CUtensorMap tw = make_tmap_2d_bf16(w.data_ptr(), (uint64_t)K, (uint64_t)N,
                                             (uint64_t)w.stride(0) * 2, 64, 128,
                                             CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tx = make_tmap_2d_bf16(x.data_ptr(), (uint64_t)K, (uint64_t)M,
                                             (uint64_t)x.stride(0) * 2, 64, (uint32_t)p.TN,
                                             CU_TENSOR_MAP_SWIZZLE_128B);
    switch (p.TN) {
      case 32: launch_bf16<32, 1, false>(tw, tx, a, grid, stream); break;
      case 64: launch_bf16<64, 1, false>(tw, tx, a, grid, stream); break;
      case 128: launch_bf16<128, 1, false>(tw, tx, a, grid, stream); break;
      default: launch_bf16<256, 1, false>(tw, tx, a, grid, stream); break;
    }
  }
}

}  // namespace cb
