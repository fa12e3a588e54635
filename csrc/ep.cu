// Expert parallelism for sparse-MoE layers over NVLink peer memory.
//
// Every rank holds E / W routed experts and its own tokens (attention is data
// parallel).  One MoE layer on rank r, with all buffers symmetric (the same
// allocation on every GPU, mapped into every peer's address space):
//
//   ep_route     (1 CTA)   top-k expert ids -> destination rank and slot of
//                          every (token, k) pair, per-destination counts;
//   ep_dispatch  (n CTAs)  P2P stores of each pair's activation row into the
//                          destination's receive region for source r, its
//                          expert id into the destination's meta array; the
//                          last CTA publishes the counts and raises r's
//                          "dispatched" flag on every peer (st.release.sys);
//   ep_recv      (1 CTA)   waits (bounded) for every source's flag, sorts the
//                          received rows by local expert (offsets for the
//                          grouped GEMM) and records, per row, where its
//                          result must go: the source's return region;
//   ep_gather    (grid)    copies the received rows into expert order;
//   grouped W4A16 GEMMs    gate/up (+SiLU), then down whose epilogue stores
//                          each result row straight into the source rank's
//                          return region (P2P, the `out_rows` table);
//   ep_finish    (1 CTA)   raises r's "returned" flag on every source;
//   ep_combine   (T CTAs)  waits for every destination's flag, then
//                          out[t] = add[t] + sum_j w[t, j] * result(t, j),
//                          summed in j order (deterministic); the last CTA
//                          advances the device epoch.
//
// Flags carry an epoch kept in device memory (CUDA-graph replayable).  A
// region is rewritten only after the reader has signalled the next layer,
// so no double buffering is needed.  Every wait is bounded: on expiry the
// kernel records kStatusPeerTimeout and carries on with zeros (the host
// aborts the batch).  No TMA touches peer memory; peer traffic is plain
// 16-byte loads and stores.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace cb {

namespace {

using bf16 = __nv_bfloat16;
constexpr int kEpMaxRanks = 8;

struct EpArgs {
  bf16* xbuf[kEpMaxRanks];  // per rank: receive regions [W][cap][H]
  bf16* rbuf[kEpMaxRanks];  // per rank: return regions [W][cap][H]
  int* meta[kEpMaxRanks];   // per rank: expert ids of received rows [W][cap]
  int* sig[kEpMaxRanks];    // per rank: [0,W) dispatched epoch, [W,2W) counts, [2W,3W) returned
  int* epoch;               // local: last completed layer epoch
  int* done;                // local: CTA completion counter (self-resetting)
  int* status;
  int rank, world, cap, H, e_local, k;
};

__device__ __forceinline__ void st_release_sys_i(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys_i(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_cv_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cv.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Bounded wait until *p >= target.
__device__ bool wait_flag(const int* p, int target, int* status) {
  if (ld_acquire_sys_i(p) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys_i(p) < target) {
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      record_status(status, kStatusPeerTimeout);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- route
__global__ void ep_route_kernel(const int* __restrict__ ids, int n, EpArgs a,
                                int* __restrict__ dest, int* __restrict__ pos,
                                int* __restrict__ send_cnt) {
  __shared__ int cnt[kEpMaxRanks];
  if (threadIdx.x < kEpMaxRanks) cnt[threadIdx.x] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int o = ids[i] / a.e_local;
    const int p = atomicAdd(&cnt[o], 1);
    dest[i] = o;
    pos[i] = p;
  }
  __syncthreads();
  if (threadIdx.x < a.world) {
    send_cnt[threadIdx.x] = cnt[threadIdx.x];
    if (cnt[threadIdx.x] > a.cap) record_status(a.status, kStatusPeerTimeout);
  }
}

// ---------------------------------------------------------------- dispatch
__global__ void ep_dispatch_kernel(const bf16* __restrict__ x, int ldx, const int* __restrict__ ids,
                                   int n, const int* __restrict__ dest, const int* __restrict__ pos,
                                   const int* __restrict__ send_cnt, EpArgs a) {
  __shared__ int s_last;
  const int i = blockIdx.x;
  if (i < n) {
    const int o = dest[i];
    const int p = pos[i];
    if (p < a.cap) {
      const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(i / a.k) * ldx);
      uint4* dst = reinterpret_cast<uint4*>(a.xbuf[o] + ((size_t)a.rank * a.cap + p) * a.H);
      for (int v = threadIdx.x; v < a.H / 8; v += blockDim.x) dst[v] = src[v];
      if (threadIdx.x == 0) a.meta[o][a.rank * a.cap + p] = ids[i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int prev = atomicAdd(a.done, 1);
    s_last = prev == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x < a.world) {
    const int e = *reinterpret_cast<volatile int*>(a.epoch) + 1;
    const int o = threadIdx.x;
    a.sig[o][a.world + a.rank] = send_cnt[o];
    __threadfence_system();
    st_release_sys_i(a.sig[o] + a.rank, e);
    if (threadIdx.x == 0) *a.done = 0;
  }
}

// ---------------------------------------------------------------- recv
// One CTA.  Outputs: offsets [e_local + 1], src_row [rows] (s * cap + p),
// out_rows [rows] (address of the result row in the source's return
// region), total [1].
constexpr int kRecvThreads = 1024;
constexpr int kMaxLocalExperts = 512;

__global__ void __launch_bounds__(kRecvThreads) ep_recv_kernel(EpArgs a, int* __restrict__ offsets,
                                                               int* __restrict__ src_row,
                                                               long long* __restrict__ out_rows,
                                                               int* __restrict__ total) {
  __shared__ int cnt_src[kEpMaxRanks];
  __shared__ int base_src[kEpMaxRanks + 1];
  __shared__ int ecnt[kMaxLocalExperts];
  __shared__ int ecur[kMaxLocalExperts];
  __shared__ int s_e;
  if (threadIdx.x == 0) s_e = *reinterpret_cast<volatile int*>(a.epoch) + 1;
  for (int e = threadIdx.x; e < a.e_local; e += blockDim.x) ecnt[e] = 0;
  __syncthreads();
  const int* my = a.sig[a.rank];
  if (threadIdx.x < a.world) {
    const int s = threadIdx.x;
    const bool ok = wait_flag(my + s, s_e, a.status);
    cnt_src[s] = ok ? min(*reinterpret_cast<volatile const int*>(my + a.world + s), a.cap) : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int s = 0; s < a.world; ++s) {
      base_src[s] = run;
      run += cnt_src[s];
    }
    base_src[a.world] = run;
    *total = run;
  }
  __syncthreads();
  const int n = base_src[a.world];
  const int* meta = a.meta[a.rank];
  const int lo = a.rank * a.e_local;
  for (int g = threadIdx.x; g < n; g += blockDim.x) {
    int s = 0;
    while (g >= base_src[s + 1]) ++s;
    const int p = g - base_src[s];
    const int le = min(max(__ldcg(&meta[s * a.cap + p]) - lo, 0), a.e_local - 1);
    atomicAdd(&ecnt[le], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < a.e_local; ++e) {
      offsets[e] = run;
      ecur[e] = run;
      run += ecnt[e];
    }
    offsets[a.e_local] = run;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < n; g += blockDim.x) {
    int s = 0;
    while (g >= base_src[s + 1]) ++s;
    const int p = g - base_src[s];
    const int le = min(max(__ldcg(&meta[s * a.cap + p]) - lo, 0), a.e_local - 1);
    const int q = atomicAdd(&ecur[le], 1);
    src_row[q] = s * a.cap + p;
    out_rows[q] = (long long)(a.rbuf[s] + ((size_t)a.rank * a.cap + p) * a.H);
  }
}

__global__ void ep_gather_kernel(EpArgs a, const int* __restrict__ src_row,
                                 const int* __restrict__ total, bf16* __restrict__ xp) {
  const int n = *total;
  const bf16* xb = a.xbuf[a.rank];
  for (int g = blockIdx.x; g < n; g += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(xb + (size_t)src_row[g] * a.H);
    uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)g * a.H);
    for (int v = threadIdx.x; v < a.H / 8; v += blockDim.x) dst[v] = ld_cv_u4(src + v);
  }
}

// ---------------------------------------------------------------- finish
__global__ void ep_finish_kernel(EpArgs a) {
  const int e = *reinterpret_cast<volatile int*>(a.epoch) + 1;
  __threadfence_system();  // the down GEMM's peer stores precede the flag
  if (threadIdx.x < a.world) st_release_sys_i(a.sig[threadIdx.x] + 2 * a.world + a.rank, e);
}

// ---------------------------------------------------------------- combine
__global__ void ep_combine_kernel(EpArgs a, int T, const int* __restrict__ dest,
                                  const int* __restrict__ pos, const float* __restrict__ w,
                                  const bf16* __restrict__ add, int ld_add, bf16* __restrict__ out,
                                  int ldo) {
  __shared__ int s_e, s_ok, s_last;
  if (threadIdx.x == 0) {
    s_e = *reinterpret_cast<volatile int*>(a.epoch) + 1;
    s_ok = 1;
  }
  __syncthreads();
  if (threadIdx.x < a.world) {
    if (!wait_flag(a.sig[a.rank] + 2 * a.world + threadIdx.x, s_e, a.status)) s_ok = 0;
  }
  __syncthreads();
  const int t = blockIdx.x;
  if (t < T) {
    const bf16* rb = a.rbuf[a.rank];
    for (int v = threadIdx.x; v < a.H / 8; v += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.f;
      for (int j = 0; j < a.k && s_ok; ++j) {
        const int i = t * a.k + j;
        const float wt = w[i];
        const uint4 u =
            ld_cv_u4(rb + ((size_t)dest[i] * a.cap + pos[i]) * a.H + (size_t)v * 8);
        const bf16* e = reinterpret_cast<const bf16*>(&u);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += wt * __bfloat162float(e[q]);
      }
      if (add != nullptr) {
        const uint4 u = *reinterpret_cast<const uint4*>(add + (size_t)t * ld_add + v * 8);
        const bf16* e = reinterpret_cast<const bf16*>(&u);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(e[q]);
      }
      uint4 o;
      bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16(acc[q]);
      *reinterpret_cast<uint4*>(out + (size_t)t * ldo + v * 8) = o;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(a.done, 1);
    s_last = prev == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *a.done = 0;
    atomicExch(a.epoch, s_e);
  }
}

EpArgs make_args(torch::Tensor xbuf_ptrs, torch::Tensor rbuf_ptrs, torch::Tensor meta_ptrs,
                 torch::Tensor sig_ptrs, torch::Tensor epoch, torch::Tensor done,
                 torch::Tensor status, int64_t rank, int64_t world, int64_t cap, int64_t H,
                 int64_t e_local, int64_t k) {
  TORCH_CHECK(world >= 1 && world <= kEpMaxRanks, "expert parallel group of 1..8 ranks");
  TORCH_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  TORCH_CHECK(e_local <= kMaxLocalExperts, "too many local experts");
  EpArgs a{};
  auto xp = xbuf_ptrs.cpu(), rp = rbuf_ptrs.cpu(), mp = meta_ptrs.cpu(), sp = sig_ptrs.cpu();
  for (int r = 0; r < world; ++r) {
    a.xbuf[r] = reinterpret_cast<bf16*>(xp.data_ptr<int64_t>()[r]);
    a.rbuf[r] = reinterpret_cast<bf16*>(rp.data_ptr<int64_t>()[r]);
    a.meta[r] = reinterpret_cast<int*>(mp.data_ptr<int64_t>()[r]);
    a.sig[r] = reinterpret_cast<int*>(sp.data_ptr<int64_t>()[r]);
  }
  a.epoch = epoch.data_ptr<int>();
  a.done = done.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.rank = (int)rank;
  a.world = (int)world;
  a.cap = (int)cap;
  a.H = (int)H;
  a.e_local = (int)e_local;
  a.k = (int)k;
  return a;
}

}  // namespace

// Route + dispatch: ids [T, k] (global expert ids), x [T, H].  dest / pos
// [T*k] int32 and send_cnt [W] are outputs kept for the combine.
void ep_dispatch(torch::Tensor x, torch::Tensor ids, torch::Tensor dest, torch::Tensor pos,
                 torch::Tensor send_cnt, torch::Tensor xbuf_ptrs, torch::Tensor rbuf_ptrs,
                 torch::Tensor meta_ptrs, torch::Tensor sig_ptrs, torch::Tensor epoch,
                 torch::Tensor done, torch::Tensor status, int64_t rank, int64_t world,
                 int64_t cap, int64_t e_local) {
  const int T = (int)ids.size(0);
  const int k = (int)ids.size(1);
  const int H = (int)x.size(1);
  EpArgs a = make_args(xbuf_ptrs, rbuf_ptrs, meta_ptrs, sig_ptrs, epoch, done, status, rank,
                       world, cap, H, e_local, k);
  TORCH_CHECK(x.stride(1) == 1 && (x.stride(0) * 2) % 16 == 0, "x rows must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int n = T * k;
  ep_route_kernel<<<1, 1024, 0, stream>>>(ids.data_ptr<int>(), n, a, dest.data_ptr<int>(),
                                          pos.data_ptr<int>(), send_cnt.data_ptr<int>());
  CB_CUDA_CHECK(cudaGetLastError());
  ep_dispatch_kernel<<<std::max(n, 1), 128, 0, stream>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), (int)x.stride(0), ids.data_ptr<int>(), n,
      dest.data_ptr<int>(), pos.data_ptr<int>(), send_cnt.data_ptr<int>(), a);
  CB_CUDA_CHECK(cudaGetLastError());
}

// Receive: wait for every source, expert-sort the received rows, gather them
// into xp [W*cap, H]; offsets [e_local+1], out_rows [W*cap] (int64), total [1].
void ep_receive(torch::Tensor xp, torch::Tensor offsets, torch::Tensor src_row,
                torch::Tensor out_rows, torch::Tensor total, torch::Tensor xbuf_ptrs,
                torch::Tensor rbuf_ptrs, torch::Tensor meta_ptrs, torch::Tensor sig_ptrs,
                torch::Tensor epoch, torch::Tensor done, torch::Tensor status, int64_t rank,
                int64_t world, int64_t cap, int64_t e_local) {
  const int H = (int)xp.size(1);
  EpArgs a = make_args(xbuf_ptrs, rbuf_ptrs, meta_ptrs, sig_ptrs, epoch, done, status, rank,
                       world, cap, H, e_local, 1);
  const c10::cuda::CUDAGuard guard(xp.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  ep_recv_kernel<<<1, kRecvThreads, 0, stream>>>(a, offsets.data_ptr<int>(), src_row.data_ptr<int>(),
                                                 reinterpret_cast<long long*>(out_rows.data_ptr<int64_t>()),
                                                 total.data_ptr<int>());
  CB_CUDA_CHECK(cudaGetLastError());
  ep_gather_kernel<<<std::min<int64_t>(world * cap, 1024), 128, 0, stream>>>(
      a, src_row.data_ptr<int>(), total.data_ptr<int>(), reinterpret_cast<bf16*>(xp.data_ptr()));
  CB_CUDA_CHECK(cudaGetLastError());
}

// Finish (results stored into the sources' return regions) + combine.
void ep_combine(torch::Tensor w, torch::Tensor dest, torch::Tensor pos,
                c10::optional<torch::Tensor> add, torch::Tensor out, torch::Tensor xbuf_ptrs,
                torch::Tensor rbuf_ptrs, torch::Tensor meta_ptrs, torch::Tensor sig_ptrs,
                torch::Tensor epoch, torch::Tensor done, torch::Tensor status, int64_t rank,
                int64_t world, int64_t cap, int64_t e_local) {
  const int T = (int)w.size(0);
  const int k = (int)w.size(1);
  const int H = (int)out.size(1);
  EpArgs a = make_args(xbuf_ptrs, rbuf_ptrs, meta_ptrs, sig_ptrs, epoch, done, status, rank,
                       world, cap, H, e_local, k);
  const c10::cuda::CUDAGuard guard(out.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  ep_finish_kernel<<<1, 32, 0, stream>>>(a);
  CB_CUDA_CHECK(cudaGetLastError());
  ep_combine_kernel<<<std::max(T, 1), 256, 0, stream>>>(
      a, T, dest.data_ptr<int>(), pos.data_ptr<int>(), w.data_ptr<float>(),
      add.has_value() ? reinterpret_cast<const bf16*>(add->data_ptr()) : nullptr,
      add.has_value() ? (int)add->stride(0) : 0, reinterpret_cast<bf16*>(out.data_ptr()),
      (int)out.stride(0));
  CB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace cb
