// Tensor-parallel collectives fused with their consumer, over NVLink peer
// memory (no NCCL on this path).
//
// ar_rmsnorm: the row-parallel GEMMs (o_proj, down_proj) of every rank write
// their partial sums into a symmetric buffer (same offset on every GPU,
// mapped into every peer's address space).  This kernel then, in one launch:
//   1. signals "my partial is ready" into every peer's signal pad
//      (st.release.sys over NVLink),
//   2. waits, bounded, until every peer has signalled the same epoch,
//   3. reads the N partials of its rows straight from the peers' memory
//      (plain P2P loads), sums them in fp32, adds the residual stream and
//      applies RMSNorm, writing the updated residual and the normalised row
//      locally.
// Every rank ends with the full normalised hidden state, so the next
// column-parallel GEMM needs no all-gather.  Epochs live in device memory
// (incremented by the last CTA of each launch), so the launch is CUDA-graph
// replayable.  Two symmetric buffers alternate between consecutive
// all-reduces: a rank can only overwrite buffer b after passing the barrier
// of the following all-reduce, which every peer reaches only after it
// finished reading b.
//
// Waits are bounded (kWaitTimeoutNs); on expiry the kernel records
// kStatusPeerTimeout in the status word and leaves its outputs unwritten.
// The engine reads the status word after every step and fails the batch
// (engine.base.BatchAborted) when it is non-zero.
//
// Launched with programmatic dependent launch: the CTAs become resident
// while the GEMM that writes the partials drains, and wait for it
// (griddepcontrol.wait) before signalling the peers.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Peer data written by the peers' previous kernels: fetch from memory,
// never from L1.  The caller issues all of a row's loads before using any
// of them, so their NVLink round trips overlap.
// Sum of the 8 bf16 at `mc` over every GPU bound to the NVLink multicast
// object (the reduction runs in the NVSwitch; one 16-byte reply per load).
__device__ __forceinline__ uint4 multimem_ld_sum_bf16x8(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_cv128(const void* p) {
  uint4 v;
  asm volatile("ld.global.cv.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

constexpr int kMaxRanks = 8;
constexpr int kArThreads = 512;

struct ArArgs {
  const bf16* bufs[kMaxRanks];  // peer buffer base (this all-reduce's buffer), per rank
  int* sigs[kMaxRanks];         // peer signal pads (int[kMaxRanks]) per rank
  int* epoch;                   // local: last completed epoch
  int* done;                    // local: CTAs finished in this launch
  int* status;
  bf16* residual;               // [M, H] local residual stream (may be null)
  const bf16* w;                // RMSNorm weight (null: plain all-reduce into out)
  bf16* out;                    // [M, H]
  int rank, world, M, H, ldr, ldo;
  float eps;
  // 1: signal the peers (the partials are in each rank's own buffer);
  // 0: the producing GEMM already pushed every rank's partial into this
  // rank's slots (bufs[] are local) and raised the flags.
  int signal;
  // Multicast address of this all-reduce's buffer (NVLS), or null: with it,
  // the partials are summed by multimem.ld_reduce (one reply per 16 bytes
  // instead of one P2P load per peer).
  const bf16* mc;
};

__global__ void __launch_bounds__(kArThreads) ar_rmsnorm_kernel(const ArArgs a) {
  __shared__ int s_epoch;
  __shared__ int s_ok;
  __shared__ float red[32];
  grid_dep_launch();
  grid_dep_wait();  // the partials, the residual and the epoch of the previous launch
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile int*>(a.epoch) + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int e = s_epoch;
  // 1. signal peers (one CTA does it; the partials were written by the
  //    previous kernel on this stream, so they are complete here).
  if (a.signal && blockIdx.x == 0 && threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(a.sigs[threadIdx.x] + a.rank, e);
  }
  // 2. bounded wait for every peer's signal of this epoch.
  if (threadIdx.x < a.world) {
    const int* my = a.sigs[a.rank] + threadIdx.x;
    if (ld_acquire_sys(my) < e) {
      const uint64_t t0 = globaltimer();
      uint32_t it = 0;
      while (ld_acquire_sys(my) < e) {
        if ((++it & 1023u) == 0u && globaltimer() - t0 > kWaitTimeoutNs) {
          record_status(a.status, kStatusPeerTimeout);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    // 3. reduce rows: each thread owns 8 consecutive columns per pass.  All
    //    peers' 16-byte pieces (and the residual) are loaded first, so the
    //    NVLink round trips overlap, then summed in rank order (the same
    //    result on every rank).
    const int nvec = a.H / 8;
    for (int row = blockIdx.x; row < a.M; row += gridDim.x) {
      float ss = 0.f;
      float acc[2][8];
      int cnt = 0;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int i = threadIdx.x + k * kArThreads;
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[k][q] = 0.f;
        if (i < nvec) {
          uint4 part[kMaxRanks];
          const int np = a.mc != nullptr ? 1 : a.world;
          if (a.mc != nullptr) {
            part[0] = multimem_ld_sum_bf16x8(a.mc + (size_t)row * a.H + i * 8);
          } else {
#pragma unroll
            for (int p = 0; p < kMaxRanks; ++p)
              if (p < a.world) part[p] = ld_cv128(a.bufs[p] + (size_t)row * a.H + i * 8);
          }
          uint4 ru = make_uint4(0, 0, 0, 0);
          bf16* rp = nullptr;
          if (a.residual != nullptr) {
            rp = a.residual + (size_t)row * a.ldr + i * 8;
            ru = *reinterpret_cast<const uint4*>(rp);
          }
#pragma unroll
          for (int p = 0; p < kMaxRanks; ++p) {
            if (p < np) {
              const bf16* v = reinterpret_cast<const bf16*>(&part[p]);
#pragma unroll
              for (int q = 0; q < 8; ++q) acc[k][q] += __bfloat162float(v[q]);
            }
          }
          if (rp != nullptr) {
            bf16* re = reinterpret_cast<bf16*>(&ru);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              re[q] = __float2bfloat16(__bfloat162float(re[q]) + acc[k][q]);
              acc[k][q] = __bfloat162float(re[q]);
            }
            *reinterpret_cast<uint4*>(rp) = ru;
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) ss += acc[k][q] * acc[k][q];
          ++cnt;
        }
      }
      float inv = 1.f;
      if (a.w != nullptr) {
        float v = warp_sum(ss);
        const int wid = threadIdx.x >> 5, l = threadIdx.x & 31;
        if (l == 0) red[wid] = v;
        __syncthreads();
        float r = l < (kArThreads >> 5) ? red[l] : 0.f;
        r = warp_sum(r);
        inv = rsqrtf(r / (float)a.H + a.eps);
        __syncthreads();
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int i = threadIdx.x + k * kArThreads;
        if (i < nvec) {
          uint4 o;
          bf16* oe = reinterpret_cast<bf16*>(&o);
          if (a.w != nullptr) {
            const uint4 wu = *reinterpret_cast<const uint4*>(a.w + i * 8);
            const bf16* we = reinterpret_cast<const bf16*>(&wu);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              oe[q] = __float2bfloat16(acc[k][q] * inv * __bfloat162float(we[q]));
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16(acc[k][q]);
          }
          *reinterpret_cast<uint4*>(a.out + (size_t)row * a.ldo + i * 8) = o;
        }
      }
      (void)cnt;
    }
  }
  // 4. the last CTA of this launch advances the epoch for the next launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int d = atomicAdd(a.done, 1);
    if (d == (int)gridDim.x - 1) {
      *a.done = 0;
      __threadfence();
      *reinterpret_cast<volatile int*>(a.epoch) = e;
    }
  }
}

// bufs / sigs: int64 tensors [world] of device addresses (peer mappings).
// mc_ptr: multicast address of the symmetric buffer (0 = per-peer loads).
void ar_rmsnorm(torch::Tensor buf_ptrs, int64_t buf_offset_bytes, torch::Tensor sig_ptrs,
                torch::Tensor epoch, torch::Tensor done, torch::Tensor status, int64_t rank,
                int64_t world, int64_t M, int64_t H, c10::optional<torch::Tensor> residual,
                c10::optional<torch::Tensor> w, torch::Tensor out, double eps, int64_t mc_ptr) {
  TORCH_CHECK(world <= kMaxRanks, "at most 8 ranks");
  TORCH_CHECK(H % 8 == 0 && H / 8 <= 2 * kArThreads, "hidden size unsupported");
  TORCH_CHECK(buf_ptrs.device().is_cpu() && sig_ptrs.device().is_cpu(), "pointer lists on host");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(out.device());
  ArArgs a{};
  auto bp = buf_ptrs.accessor<int64_t, 1>();
  auto sp = sig_ptrs.accessor<int64_t, 1>();
  for (int p = 0; p < world; ++p) {
    a.bufs[p] = reinterpret_cast<const bf16*>(bp[p] + buf_offset_bytes);
    a.sigs[p] = reinterpret_cast<int*>(sp[p]);
  }
  a.epoch = epoch.data_ptr<int>();
  a.done = done.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.residual = residual.has_value() ? reinterpret_cast<bf16*>(residual->data_ptr()) : nullptr;
  a.ldr = residual.has_value() ? (int)residual->stride(0) : 0;
  a.w = w.has_value() ? reinterpret_cast<const bf16*>(w->data_ptr()) : nullptr;
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.ldo = (int)out.stride(0);
  a.rank = (int)rank;
  a.world = (int)world;
  a.M = (int)M;
  a.H = (int)H;
  a.eps = (float)eps;
  a.signal = 1;
  a.mc = mc_ptr != 0 ? reinterpret_cast<const bf16*>(mc_ptr + buf_offset_bytes) : nullptr;
  // Every CTA must be resident at once (they wait on peers): at most one per SM.
  const int grid = (int)std::min<int64_t>(M, std::min(num_sms(), 128));
  launch_kernel(ar_rmsnorm_kernel, dim3(grid), dim3(kArThreads), 0,
                at::cuda::getCurrentCUDAStream(), a);
}

// The all-reduce after a pushing GEMM (w4a16_gemm_push): slot_ptrs are the
// `world` receive slots in THIS rank's memory (slot p holds rank p's
// partial), sig_ptrs[rank] is this rank's pad that the GEMMs' last tiles
// raise.  Waits for every rank's flag, sums the slots in rank order, adds
// the residual and applies RMSNorm, like ar_rmsnorm.
void ar_rmsnorm_pushed(torch::Tensor slot_ptrs, torch::Tensor sig_ptrs, torch::Tensor epoch,
                       torch::Tensor done, torch::Tensor status, int64_t rank, int64_t world,
                       int64_t M, int64_t H, c10::optional<torch::Tensor> residual,
                       c10::optional<torch::Tensor> w, torch::Tensor out, double eps) {
  TORCH_CHECK(world <= kMaxRanks, "at most 8 ranks");
  TORCH_CHECK(H % 8 == 0 && H / 8 <= 2 * kArThreads, "hidden size unsupported");
  TORCH_CHECK(slot_ptrs.device().is_cpu() && sig_ptrs.device().is_cpu(), "pointer lists on host");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(out.device());
  ArArgs a{};
  auto bp = slot_ptrs.accessor<int64_t, 1>();
  auto sp = sig_ptrs.accessor<int64_t, 1>();
  for (int p = 0; p < world; ++p) {
    a.bufs[p] = reinterpret_cast<const bf16*>(bp[p]);
    a.sigs[p] = reinterpret_cast<int*>(sp[p]);
  }
  a.epoch = epoch.data_ptr<int>();
  a.done = done.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.residual = residual.has_value() ? reinterpret_cast<bf16*>(residual->data_ptr()) : nullptr;
  a.ldr = residual.has_value() ? (int)residual->stride(0) : 0;
  a.w = w.has_value() ? reinterpret_cast<const bf16*>(w->data_ptr()) : nullptr;
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.ldo = (int)out.stride(0);
  a.rank = (int)rank;
  a.world = (int)world;
  a.M = (int)M;
  a.H = (int)H;
  a.eps = (float)eps;
  a.signal = 0;
  a.mc = nullptr;
  const int grid = (int)std::min<int64_t>(M, std::min(num_sms(), 128));
  launch_kernel(ar_rmsnorm_kernel, dim3(grid), dim3(kArThreads), 0,
                at::cuda::getCurrentCUDAStream(), a);
}

}  // namespace cb
