// Weight-streaming GEMV for decode batches of 1-4 tokens (sm_100a).
//
//   y[m, n] = sum_k x[m, k] W[n, k]     (m < MT <= 4), epilogues bf16 (+ residual), fp32,
//   and SwiGLU over gate / up rows interleaved in 64-row groups (y[m, f] = silu(g) * u).
//
// At one to four tokens a decode GEMM is a pure weight stream (1 FLOP per byte per token): the
// tensor-core split-K kernel pays tile set-up and exchanges for no math benefit and reaches
// about 56 % of HBM bandwidth at batch 1.  Here each warp streams two weight rows (for SwiGLU:
// the gate and up rows of one output feature) with 16-byte loads, 8 per row and lane in
// flight, multiplies them with the few activation rows (read through L1; every warp of the GPU
// reads the same few KB), and reduces across the warp.  No shared memory, no barriers.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {
namespace gv {

constexpr int WARPS = 8;
constexpr int UNROLL = 8;

__device__ __forceinline__ void fma8(float& acc, const uint4& w, const uint4& x) {
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&w);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fa = __bfloat1622float2(a[i]);
    const float2 fb = __bfloat1622float2(b[i]);
    acc = fmaf(fa.x, fb.x, acc);
    acc = fmaf(fa.y, fb.y, acc);
  }
}

// Streaming read of weights (read once per launch: no L1 allocation).
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// mode: 0 bf16 store (+ residual), 1 SwiGLU, 2 fp32 store.
template <int MT>
__global__ void __launch_bounds__(WARPS * 32) gemv_kernel(
    const bf16* __restrict__ x, int ldx, const bf16* __restrict__ w, int ldw, int N, int K,
    void* y, int ldy, const bf16* __restrict__ res, int ldr, int mode, int tasks) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int task = blockIdx.x * WARPS + warp;
  if (task >= tasks) return;                 // whole warp: the shuffles below stay full
  // rows of this task: SwiGLU feature f -> its gate and up rows; otherwise rows 2t, 2t + 1
  int r0, r1, f = 0;
  if (mode == 1) {
    f = task;
    r0 = (f >> 6) * 128 + (f & 63);
    r1 = r0 + 64;
  } else {
    r0 = 2 * task;
    r1 = min(r0 + 1, N - 1);
  }
  const int kv = K >> 3;                     // 16-byte vectors per row
  const uint4* w0 = reinterpret_cast<const uint4*>(w + static_cast<size_t>(r0) * ldw);
  const uint4* w1 = reinterpret_cast<const uint4*>(w + static_cast<size_t>(r1) * ldw);
  float a0[MT], a1[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) a0[m] = a1[m] = 0.f;
  int v = lane;
  for (; v + 32 * (UNROLL - 1) < kv; v += 32 * UNROLL) {
    uint4 p[UNROLL], q[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      p[u] = ld_stream(w0 + v + 32 * u);
      q[u] = ld_stream(w1 + v + 32 * u);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * ldx) +
                               v + 32 * u);
        fma8(a0[m], p[u], xv);
        fma8(a1[m], q[u], xv);
      }
    }
  }
  for (; v < kv; v += 32) {
    const uint4 p = ld_stream(w0 + v), q = ld_stream(w1 + v);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * ldx) + v);
      fma8(a0[m], p, xv);
      fma8(a1[m], q, xv);
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    a0[m] = warp_sum(a0[m]);
    a1[m] = warp_sum(a1[m]);
  }
  if (lane != 0) return;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (mode == 1) {
      const float g = a0[m];
      reinterpret_cast<bf16*>(y)[static_cast<size_t>(m) * ldy + f] =
          __float2bfloat16(g / (1.0f + __expf(-g)) * a1[m]);
    } else if (mode == 2) {
      float* out = reinterpret_cast<float*>(y) + static_cast<size_t>(m) * ldy;
      out[r0] = a0[m];
      if (r1 != r0) out[r1] = a1[m];
    } else {
      bf16* out = reinterpret_cast<bf16*>(y) + static_cast<size_t>(m) * ldy;
      float v0 = a0[m], v1 = a1[m];
      if (res != nullptr) {
        v0 += __bfloat162float(res[static_cast<size_t>(m) * ldr + r0]);
        v1 += __bfloat162float(res[static_cast<size_t>(m) * ldr + r1]);
      }
      out[r0] = __float2bfloat16(v0);
      if (r1 != r0) out[r1] = __float2bfloat16(v1);
    }
  }
}

}  // namespace gv

// C = A . W^T for A with 1..4 rows.  mode 0: bf16 (+ residual), 1: SwiGLU (N % 128 == 0,
// C [M, N/2]), 2: fp32.
void gemv_bf16(const at::Tensor& A, const at::Tensor& W, at::Tensor& C,
               const c10::optional<at::Tensor>& residual, int64_t mode) {
  TORCH_CHECK(A.is_cuda() && W.is_cuda() && C.is_cuda(), "gemv: CUDA tensors");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16, "gemv: bf16");
  TORCH_CHECK(A.dim() == 2 && W.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 &&
                  W.stride(1) == 1 && C.stride(1) == 1, "gemv: 2-D, inner stride 1");
  const int M = A.size(0), K = A.size(1), N = W.size(0);
  if (M == 0 || N == 0) return;
  TORCH_CHECK(M <= 4, "gemv: at most 4 rows");
  TORCH_CHECK(W.size(1) == K && K % 8 == 0, "gemv: K must match and be a multiple of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(A.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(W.data_ptr()) % 16 == 0 && A.stride(0) % 8 == 0 &&
                  W.stride(0) % 8 == 0, "gemv: 16-byte aligned rows");
  const bf16* res = nullptr;
  int ldr = 0;
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(mode == 0 && residual->scalar_type() == at::kBFloat16 &&
                    residual->stride(1) == 1, "gemv: residual with bf16 store only");
    res = reinterpret_cast<const bf16*>(residual->data_ptr());
    ldr = residual->stride(0);
  }
  int tasks;
  if (mode == 1) {
    TORCH_CHECK(N % 128 == 0 && C.size(1) >= N / 2 && C.scalar_type() == at::kBFloat16, "swiglu");
    tasks = N / 2;
  } else if (mode == 2) {
    TORCH_CHECK(C.scalar_type() == at::kFloat && C.size(1) >= N, "f32 out");
    tasks = (N + 1) / 2;
  } else {
    TORCH_CHECK(C.scalar_type() == at::kBFloat16 && C.size(1) >= N, "bf16 out");
    tasks = (N + 1) / 2;
  }
  TORCH_CHECK(C.size(0) >= M, "gemv: C rows");
  const int grid = (tasks + gv::WARPS - 1) / gv::WARPS;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
#define LB_GEMV(MT)                                                                        \
  C10_CUDA_CHECK(launch_k(gv::gemv_kernel<MT>, dim3(grid), dim3(gv::WARPS * 32), 0, st,    \
      nullptr, 0, reinterpret_cast<const bf16*>(A.data_ptr()), A.stride(0),                \
      reinterpret_cast<const bf16*>(W.data_ptr()), W.stride(0), N, K, C.data_ptr(),        \
      C.stride(0), res, ldr, static_cast<int>(mode), tasks))
  switch (M) {
    case 1: LB_GEMV(1); break;
    case 2: LB_GEMV(2); break;
    case 3: LB_GEMV(3); break;
    default: LB_GEMV(4); break;
  }
#undef LB_GEMV
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lb
