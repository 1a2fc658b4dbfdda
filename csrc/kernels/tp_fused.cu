// Tensor-parallel collectives fused with compute, over NVLink peer memory (sm_100a).
//
// Replaces the reference's in-process "collectives" (src/multi_gpu/tensor_parallel.rs:119-188:
// sequential to_device + add on device 0) with one process per GPU exchanging data through
// CUDA-IPC symmetric buffers:
//
//  * ipc_export / ipc_open: each rank cudaMalloc's one buffer, exports its IPC handle; every
//    rank opens every peer's handle (peer access enabled lazily by the driver).
//  * rs_norm_ag_kernel: the owner of token rows [r*R, r*R + R) waits (bounded, flag written
//    by the peers' GEMM epilogues) until every rank's partial rows have landed in its
//    reduce-scatter slots, sums them in rank order with the residual (fp32), writes the new
//    residual, applies RMSNorm, and stores the normalised row into EVERY rank's gather buffer
//    (P2P stores) - the all-gather that feeds the next GEMM.  The last CTA resets the consumed
//    flag and raises the gather flag of every rank.
//
// Waits are bounded (5 s); on expiry an error code is recorded and the kernel returns.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <cstring>

#include "common.cuh"

namespace lb {

namespace tpf {

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(int* p, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Release/acquire fence at system scope: enough to publish prior (and cumulatively
// observed) stores before a flag update; lighter than the sequentially-consistent fence.
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

struct Args {
  const bf16* rs;          // local receive buffer [world][R][H]
  const bf16* x_in;        // mode 1: local input rows [R][H] (no reduce-scatter)
  bf16* residual;          // local residual rows [R][H] (updated in place)
  const bf16* w;           // RMSNorm weight [H]
  bf16* gather[8];         // every rank's gather buffer (row-major [world*R][H])
  int* gather_flag[8];     // every rank's gather flag
  int* rs_flag;            // local: incremented once by each source rank
  int* done_counter;       // local grid-completion counter
  int world, rank, R, rows, H, mode, add_residual;
  float eps;
  int* err;
  unsigned long long* trace;  // optional: CTA 0 stamps [start, flag seen, pushed, signalled]
};

template <int VPT>
__global__ void __launch_bounds__(256) rs_norm_ag_kernel(const Args a) {
  const int row = blockIdx.x;  // local row index < rows
  __shared__ int s_ok;
  __shared__ float red[32];
  unsigned long long* tr = (a.trace != nullptr && blockIdx.x == 0) ? a.trace : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer_ns();
  if (threadIdx.x == 0) {
    int ok = 1;
    if (a.mode == 0) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t it = 0;
      while (ld_acquire_sys(a.rs_flag) < a.world) {
        if ((++it & 63u) == 0 && globaltimer_ns() - t0 > 5000000000ull) {
          record_error(a.err, kErrTimeoutPeer);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    s_ok = ok;
    if (tr) tr[1] = globaltimer_ns();
  }
  __syncthreads();
  const int nvec = a.H / 8;
  float v[VPT][8];
  float ss = 0.f;
  if (s_ok) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi >= nvec) continue;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      if (a.mode == 0) {
        for (int s = 0; s < a.world; ++s) {  // rank order: deterministic
          const uint4 raw = __ldcv(reinterpret_cast<const uint4*>(
              a.rs + (static_cast<size_t>(s) * a.R + row) * a.H) + vi);
          const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(e[j]);
        }
      } else {
        const uint4 raw = reinterpret_cast<const uint4*>(a.x_in + static_cast<size_t>(row) * a.H)[vi];
        const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __bfloat162float(e[j]);
      }
      uint4* rp = reinterpret_cast<uint4*>(a.residual + static_cast<size_t>(row) * a.H) + vi;
      if (a.add_residual) {
        const uint4 rr = *rp;
        const bf16* re = reinterpret_cast<const bf16*>(&rr);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(re[j]);
      }
      uint4 outv;
      bf16* oe = reinterpret_cast<bf16*>(&outv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        oe[j] = __float2bfloat16(acc[j]);
        v[i][j] = __bfloat162float(oe[j]);
        ss += v[i][j] * v[i][j];
      }
      *rp = outv;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / a.H + a.eps);
  if (s_ok) {
    const size_t grow = static_cast<size_t>(a.rank) * a.R + row;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi >= nvec) continue;
      const uint4 wr = reinterpret_cast<const uint4*>(a.w)[vi];
      const bf16* we = reinterpret_cast<const bf16*>(&wr);
      uint4 outv;
      bf16* oe = reinterpret_cast<bf16*>(&outv);
#pragma unroll
      for (int j = 0; j < 8; ++j) oe[j] = __float2bfloat16(v[i][j] * inv * __bfloat162float(we[j]));
      for (int d = 0; d < a.world; ++d)  // all-gather: P2P store into every rank's buffer
        reinterpret_cast<uint4*>(a.gather[d] + grow * a.H)[vi] = outv;
    }
  }
  // One system-scope fence per CTA, after the barrier that ordered all threads' gather
  // stores before it (cumulative), then the grid-completion count.
  __syncthreads();
  if (threadIdx.x == 0) {
    if (tr) tr[2] = globaltimer_ns();
    fence_acq_rel_sys();
    const int prev = atomicAdd(a.done_counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      fence_acq_rel_sys();
      if (a.mode == 0) atomicExch(a.rs_flag, 0);
      for (int d = 0; d < a.world; ++d) red_release_sys_add(a.gather_flag[d], 1);
      atomicExch(a.done_counter, 0);
      if (a.trace) a.trace[3] = globaltimer_ns();
    }
  }
}

}  // namespace tpf

// ---- IPC plumbing --------------------------------------------------------------------
// A dedicated cudaMalloc per symmetric buffer: an IPC handle names a whole allocation, so the
// buffer must not be a sub-block of the caching allocator.
int64_t ipc_alloc(int64_t bytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)));
  C10_CUDA_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)));
  return reinterpret_cast<int64_t>(p);
}

void ipc_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

at::Tensor ipc_export(int64_t ptr) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  auto t = at::empty({static_cast<int64_t>(sizeof(h))}, at::kByte);
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t ipc_open(const at::Tensor& handle) {
  TORCH_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t) && handle.device().is_cpu(), "handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) {
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

void rs_norm_ag(int64_t rs_ptr, const c10::optional<at::Tensor>& x_in, at::Tensor& residual,
                const at::Tensor& w, std::vector<int64_t> gather_ptrs,
                std::vector<int64_t> gather_flag_ptrs, int64_t rs_flag_ptr,
                int64_t done_counter_ptr, int64_t rank, int64_t R, int64_t rows, double eps,
                bool add_residual, at::Tensor& err, int64_t trace_ptr) {
  tpf::Args a = {};
  a.trace = reinterpret_cast<unsigned long long*>(trace_ptr);
  a.world = static_cast<int>(gather_ptrs.size());
  TORCH_CHECK(a.world >= 1 && a.world <= 8 && gather_flag_ptrs.size() == gather_ptrs.size(),
              "rs_norm_ag: world");
  a.rs = reinterpret_cast<const bf16*>(rs_ptr);
  a.mode = x_in.has_value() && x_in->defined() ? 1 : 0;
  a.x_in = a.mode ? reinterpret_cast<const bf16*>(x_in->data_ptr()) : nullptr;
  a.residual = reinterpret_cast<bf16*>(residual.data_ptr());
  a.w = reinterpret_cast<const bf16*>(w.data_ptr());
  for (int i = 0; i < a.world; ++i) {
    a.gather[i] = reinterpret_cast<bf16*>(gather_ptrs[i]);
    a.gather_flag[i] = reinterpret_cast<int*>(gather_flag_ptrs[i]);
  }
  a.rs_flag = reinterpret_cast<int*>(rs_flag_ptr);
  a.done_counter = reinterpret_cast<int*>(done_counter_ptr);
  a.rank = rank;
  a.R = R;
  a.rows = rows;
  a.H = residual.size(1);
  a.eps = static_cast<float>(eps);
  a.add_residual = add_residual ? 1 : 0;
  a.err = err.data_ptr<int>();
  TORCH_CHECK(a.H % 8 == 0 && residual.is_contiguous(), "rs_norm_ag: residual layout");
  if (rows <= 0) {
    TORCH_CHECK(false, "rs_norm_ag: every rank must own >= 1 row (pad the batch)");
  }
  const int vpt = (a.H / 8 + 255) / 256;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (vpt <= 1) tpf::rs_norm_ag_kernel<1><<<rows, 256, 0, st>>>(a);
  else if (vpt <= 2) tpf::rs_norm_ag_kernel<2><<<rows, 256, 0, st>>>(a);
  else if (vpt <= 4) tpf::rs_norm_ag_kernel<4><<<rows, 256, 0, st>>>(a);
  else TORCH_CHECK(false, "rs_norm_ag: hidden too large");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lb
