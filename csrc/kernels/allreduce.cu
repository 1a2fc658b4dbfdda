// Two-shot all-reduce over NVLink peer memory for tensor-parallel decode partials (sm_100a).
//
// The reference's TP "all-reduce" (src/multi_gpu/tensor_parallel.rs:119-133) copies each
// partial to device 0 and adds them serially.  This kernel replaces NCCL's ring all-reduce for
// the small (0.1-4 MB) partial sums of a decode step, where latency, not bandwidth, dominates.
// It uses no flags or handshakes: the data is its own flag.
//
//   receive buffers of every rank (CUDA IPC, opened by every peer), initialised to the
//   sentinel 0xFFFF in every bf16 lane (a NaN that is never sent: outgoing 0xFFFF lanes are
//   rewritten to the canonical NaN 0x7FFF):
//     [ epochs [NCTA] int | recv1 [2 parities][W sources][slice] | recv2 [2 parities][E] ]
//
//   epoch e (per CTA, in device memory, so the launch can live in a CUDA graph), parity e % 2:
//     push   rank r stores slice j of its partial into rank j's recv1[par][r] (peer stores);
//     RS     rank r polls recv1[par][s] of its own slice until no lane is the sentinel, sums all
//            W sources in rank order in fp32 (the owner reduces every element once, so every
//            rank ends with identical values), writes the sentinel back, stores the result in
//            its output and into every peer's recv2[par] (peer stores);
//     AG     rank r polls recv2[par] for every other slice, copies it out, writes the sentinel.
//
// Reuse: a receive slot of parity p is written again in epoch e + 2; a peer can reach that
// epoch only after finishing epoch e + 1, which needs this rank's pushes of e + 1, issued by a
// later launch than this rank's sentinel write-backs of epoch e: the write-back is performed at
// this GPU's L2 (the point of coherence of its memory) before the later launch starts, and the
// peer's next store reaches that L2 only after the peer observed a push issued by the later
// launch, so the peer's store follows the write-back in coherence order (the full argument is
// in tp_rowpar.cu, which uses the same slots discipline).  An explicit release fence at launch
// start (comm_fence_mode 1 or 2) is available; measured at TP2 on 2 MiB it costs ~7 us (every
// thread) or ~4 us (one per CTA) of an 8 us all-reduce.  Partial visibility of a 16-byte store is harmless:
// every lane is checked.  Every poll is bounded in time: on expiry the kernel records an error
// code and stops.  Peer memory is written with plain stores only; the only loads are of this
// GPU's own memory.
#include <ATen/cuda/CUDAContext.h>
#include <functional>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {
namespace ar {

constexpr int MAX_WORLD = 8;
constexpr int MAX_CTAS = 256;
constexpr int THREADS = 256;
constexpr int64_t HEADER_BYTES = ((MAX_CTAS * 4 + 255) / 256) * 256;
constexpr uint32_t SENT = 0xFFFFu;

struct Args {
  const uint4* in;                // local partial [nvec]
  uint4* out;                     // local result [nvec]
  uint4* recv1[MAX_WORLD];        // every rank's recv1 (parity 0; parity 1 follows)
  uint4* recv2[MAX_WORLD];        // every rank's recv2 (parity 0; parity 1 follows)
  int* epochs;                    // local per-CTA epochs
  int64_t nvec;                   // E / 8
  int64_t max_per;                // slice capacity (vectors) of one recv1 source
  int64_t max_vec;                // capacity (vectors) of one recv2 parity
  int world, rank;
  int fence_mode;                 // 1: every thread fences at launch start; 2: thread 0 only
  int* err;
};

__device__ __forceinline__ uint4 ld_vol(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ bool lanes_ready(const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 4; ++i) ok &= ((w[i] & 0xFFFFu) != SENT) & ((w[i] >> 16) != SENT);
  return ok;
}

__device__ __forceinline__ uint32_t canon(uint32_t w) {
  if ((w & 0xFFFFu) == SENT) w = (w & 0xFFFF0000u) | 0x7FFFu;
  if ((w >> 16) == SENT) w = (w & 0xFFFFu) | 0x7FFF0000u;
  return w;
}
__device__ __forceinline__ uint4 canon4(uint4 v) {
  return make_uint4(canon(v.x), canon(v.y), canon(v.z), canon(v.w));
}

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Poll a local slot until every lane is written; false when the kernel's time budget ran out.
__device__ __forceinline__ bool poll(const uint4* p, uint4& v, uint64_t t0) {
  uint32_t it = 0;
  while (true) {
    v = ld_vol(p);
    if (lanes_ready(v)) return true;
    if ((++it & 127u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

__device__ __forceinline__ void add8(float (&acc)[8], const uint4& v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

// Launch-start ordering (see the file comment): mode 1 = fence.acq_rel.sys in every thread,
// mode 2 = in thread 0 before the CTA barrier that precedes every store, 0 = none (measurement).
__device__ __forceinline__ void start_fence(int mode) {
  if (mode == 1 || (mode == 2 && threadIdx.x == 0)) fence_acq_rel_sys();
}

__global__ void __launch_bounds__(THREADS) allreduce_kernel(const Args a) {
  __shared__ int s_e;
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) s_e = a.epochs[blockIdx.x] + 1;
  start_fence(a.fence_mode);  // release: earlier launches' write-backs before this launch's pushes
  __syncthreads();
  const uint64_t t0 = globaltimer_ns();
  const int par = s_e & 1;
  const int W = a.world, me = a.rank;
  const int64_t per = (a.nvec + W - 1) / W;
  const int64_t step = static_cast<int64_t>(gridDim.x) * THREADS;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x;
  const uint4 sent = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
  bool ok = true;

  // ---- push: slice j of the local partial -> rank j's recv1[par][me] ----
  for (int d = 1; d < W; ++d) {
    const int j = (me + d) % W;
    const int64_t lo = j * per, hi = min(a.nvec, lo + per);
    uint4* dst = a.recv1[j] + (static_cast<int64_t>(par) * W + me) * a.max_per - lo;
#pragma unroll 4
    for (int64_t v = lo + first; v < hi; v += step) dst[v] = canon4(a.in[v]);
  }
  // ---- reduce-scatter: own slice, sources in rank order; result -> out and every recv2 ----
  {
    const int64_t lo = me * per, hi = min(a.nvec, lo + per);
    uint4* src = a.recv1[me] + static_cast<int64_t>(par) * W * a.max_per - lo;
    for (int64_t v = lo + first; v < hi && ok; v += step) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int s = 0; s < W; ++s) {
        uint4 x;
        if (s == me) {
          x = a.in[v];
        } else {
          uint4* p = src + s * a.max_per + v;
          if (!poll(p, x, t0)) { ok = false; break; }
          *p = sent;
        }
        add8(acc, x);
      }
      if (!ok) break;
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) ow[i] = pack_bf16x2(acc[2 * i], acc[2 * i + 1]);
      a.out[v] = o;
      o = canon4(o);
      for (int d = 1; d < W; ++d) {
        const int j = (me + d) % W;
        a.recv2[j][static_cast<int64_t>(par) * a.max_vec + v] = o;
      }
    }
  }
  // ---- all-gather: every other owner's slice from the local recv2 ----
  for (int d = 1; d < W && ok; ++d) {
    const int j = (me + d) % W;
    const int64_t lo = j * per, hi = min(a.nvec, lo + per);
    uint4* src = a.recv2[me] + static_cast<int64_t>(par) * a.max_vec;
    for (int64_t v = lo + first; v < hi; v += step) {
      uint4 x;
      if (!poll(src + v, x, t0)) { ok = false; break; }
      src[v] = sent;
      a.out[v] = x;
    }
  }
  if (!ok) record_error(a.err, kErrTimeoutPeer);
  __syncthreads();
  if (threadIdx.x == 0) a.epochs[blockIdx.x] = s_e;
}

// ---------------------------------------------------------------------------------------
// Fused variant for the row-parallel output of a transformer sub-layer:
//   x <- x + allreduce(y);  h <- rmsnorm(x) * w
// with the rounding of the unfused path (sum in fp32 -> bf16, add -> bf16, norm in fp32).
// Rows are owned in contiguous ranges (rank j owns rows [j * rp, (j + 1) * rp)); the owner
// reduces a row, updates its residual, pushes the new residual row to every peer (recv2)
// and normalises it; the other ranks poll the row, update their residual copy and
// normalise it too.  CTA b takes rows b, b + G, ... on every rank, so a wait only ever
// targets the same CTA slot on another rank for the same row, whose own inputs come from
// the push phase every CTA finishes first: no cycle.  The grid (and so every CTA's epoch) is
// the same as the plain kernel's, with which it shares the receive buffers.
// ---------------------------------------------------------------------------------------
constexpr int MAX_VPT = 4;   // hidden <= 8 * THREADS * MAX_VPT = 8192

struct NormArgs {
  Args b;                // in = partial [T * HV]; out unused
  uint4* x;              // residual [T * HV], updated in place
  const uint4* w;        // norm weight [HV]
  uint4* h;              // normalised output [T * HV]
  int T, HV;
  float eps;
};

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__global__ void __launch_bounds__(THREADS) allreduce_rmsnorm_kernel(const NormArgs na) {
  const Args& a = na.b;
  __shared__ int s_e;
  __shared__ float red[THREADS / 32];
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) s_e = a.epochs[blockIdx.x] + 1;
  start_fence(a.fence_mode);   // release, as in allreduce_kernel
  __syncthreads();
  const uint64_t t0 = globaltimer_ns();
  const int par = s_e & 1;
  const int W = a.world, me = a.rank;
  const int rp = (na.T + W - 1) / W;
  const int64_t per = static_cast<int64_t>(rp) * na.HV;
  const int64_t step = static_cast<int64_t>(gridDim.x) * THREADS;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x;
  const uint4 sent = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  bool ok = true;

  // ---- push: rows of owner j -> rank j's recv1[par][me] ----
  for (int d = 1; d < W; ++d) {
    const int j = (me + d) % W;
    const int64_t lo = j * per, hi = min(a.nvec, lo + per);
    uint4* dst = a.recv1[j] + (static_cast<int64_t>(par) * W + me) * a.max_per - lo;
#pragma unroll 4
    for (int64_t v = lo + first; v < hi; v += step) dst[v] = canon4(a.in[v]);
  }
  // ---- rows b, b + G, ...: reduce (owner) or receive, then residual update and norm ----
  const int64_t my_lo = me * per;
  uint4* r1 = a.recv1[me] + static_cast<int64_t>(par) * W * a.max_per;
  uint4* r2 = a.recv2[me] + static_cast<int64_t>(par) * a.max_vec;
  for (int r = blockIdx.x; r < na.T; r += gridDim.x) {
    const bool own = r / rp == me;
    float xv[MAX_VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAX_VPT; ++i) {
      const int vi = threadIdx.x + i * THREADS;
      if (vi >= na.HV) continue;
      const int64_t v = static_cast<int64_t>(r) * na.HV + vi;
      uint4 xn;
      if (own) {
        float acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0.f;
        for (int s2 = 0; s2 < W; ++s2) {
          uint4 q = zero;
          if (s2 == me) {
            q = a.in[v];
          } else if (ok) {
            uint4* p = r1 + s2 * a.max_per + (v - my_lo);
            if (poll(p, q, t0)) *p = sent;
            else { ok = false; q = zero; }
          }
          add8(acc, q);
        }
        float xr[8];
        unpack8(na.x[v], xr);
        uint32_t* xw = reinterpret_cast<uint32_t*>(&xn);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float y0 = __bfloat162float(__float2bfloat16(acc[2 * k]));
          const float y1 = __bfloat162float(__float2bfloat16(acc[2 * k + 1]));
          xw[k] = pack_bf16x2(xr[2 * k] + y0, xr[2 * k + 1] + y1);
        }
        const uint4 o = canon4(xn);
        for (int d = 1; d < W; ++d) {
          const int j = (me + d) % W;
          a.recv2[j][static_cast<int64_t>(par) * a.max_vec + v] = o;
        }
      } else {
        xn = zero;
        if (ok) {
          if (poll(r2 + v, xn, t0)) r2[v] = sent;
          else { ok = false; xn = zero; }
        }
      }
      na.x[v] = xn;
      unpack8(xn, xv[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += xv[i][k] * xv[i][k];
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < THREADS / 32; ++k) tot += red[k];
    const float inv = rsqrtf(tot / (8.f * na.HV) + na.eps);
    __syncthreads();   // red is rewritten by the next row
#pragma unroll
    for (int i = 0; i < MAX_VPT; ++i) {
      const int vi = threadIdx.x + i * THREADS;
      if (vi >= na.HV) continue;
      float wf[8];
      unpack8(na.w[vi], wf);
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        ow[k] = pack_bf16x2(xv[i][2 * k] * inv * wf[2 * k], xv[i][2 * k + 1] * inv * wf[2 * k + 1]);
      na.h[static_cast<int64_t>(r) * na.HV + vi] = o;
    }
  }
  if (!ok) record_error(a.err, kErrTimeoutPeer);
  __syncthreads();
  if (threadIdx.x == 0) a.epochs[blockIdx.x] = s_e;
}

struct Layout {
  int64_t max_vec, max_per, recv1_off, recv2_off, bytes;
};

inline Layout layout(int64_t max_elems, int64_t world) {
  Layout l;
  l.max_vec = (max_elems + 7) / 8;
  l.max_per = (l.max_vec + world - 1) / world;
  l.recv1_off = HEADER_BYTES;
  l.recv2_off = l.recv1_off + 2 * world * l.max_per * 16;
  l.bytes = l.recv2_off + 2 * l.max_vec * 16;
  return l;
}

}  // namespace ar

// Bytes of one rank's receive buffer for up to `max_elems` bf16 elements on `world` ranks.
int64_t allreduce_buffer_bytes(int64_t max_elems, int64_t world) {
  return ar::layout(max_elems, world).bytes;
}

// Zero the epochs and fill the receive slots with the sentinel (before the first call, on
// every rank, followed by a barrier).
void allreduce_prepare(int64_t base, int64_t max_elems, int64_t world) {
  const ar::Layout l = ar::layout(max_elems, world);
  uint8_t* b = reinterpret_cast<uint8_t*>(base);
  C10_CUDA_CHECK(cudaMemset(b, 0, ar::HEADER_BYTES));
  C10_CUDA_CHECK(cudaMemset(b + ar::HEADER_BYTES, 0xFF, l.bytes - ar::HEADER_BYTES));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
}

// out, inp: local [E] bf16 (contiguous, 16-byte aligned); bases: every rank's receive buffer.
void allreduce_p2p(at::Tensor& out, const at::Tensor& inp, std::vector<int64_t> bases,
                   int64_t rank, int64_t n_elems, int64_t max_elems, int64_t ctas,
                   at::Tensor& err) {
  const int world = static_cast<int>(bases.size());
  TORCH_CHECK(world >= 2 && world <= ar::MAX_WORLD, "allreduce_p2p: 2..8 ranks");
  TORCH_CHECK(n_elems % 8 == 0 && n_elems <= max_elems, "allreduce_p2p: size");
  for (const at::Tensor& t : {std::cref(out), std::cref(inp)})
    TORCH_CHECK(t.is_contiguous() && t.scalar_type() == at::kBFloat16 && t.numel() >= n_elems &&
                    reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
                "allreduce_p2p: out/inp must be contiguous 16-byte-aligned bf16");
  if (n_elems == 0) return;
  const ar::Layout l = ar::layout(max_elems, world);
  ar::Args a = {};
  for (int r = 0; r < world; ++r) {
    uint8_t* b = reinterpret_cast<uint8_t*>(bases[r]);
    a.recv1[r] = reinterpret_cast<uint4*>(b + l.recv1_off);
    a.recv2[r] = reinterpret_cast<uint4*>(b + l.recv2_off);
  }
  a.in = reinterpret_cast<const uint4*>(inp.data_ptr());
  a.out = reinterpret_cast<uint4*>(out.data_ptr());
  a.epochs = reinterpret_cast<int*>(bases[rank]);
  a.nvec = n_elems / 8;
  a.max_per = l.max_per;
  a.max_vec = l.max_vec;
  a.world = world;
  a.rank = static_cast<int>(rank);
  a.err = err.data_ptr<int>();
  const int g = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas, ar::MAX_CTAS)));
  a.fence_mode = comm_fence_mode();
  C10_CUDA_CHECK(launch_k(ar::allreduce_kernel, dim3(g), dim3(ar::THREADS), 0,
                          at::cuda::getCurrentCUDAStream(), nullptr, 0, a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// h = rmsnorm(x + allreduce(inp)) * w, x updated in place; all [T, H] bf16 contiguous.
// Returns false (nothing launched) when a row-owner slice would not fit the receive buffers.
bool allreduce_rmsnorm_p2p(at::Tensor& h, const at::Tensor& inp, at::Tensor& x,
                           const at::Tensor& w, std::vector<int64_t> bases, int64_t rank,
                           int64_t max_elems, int64_t ctas, double eps, at::Tensor& err) {
  const int world = static_cast<int>(bases.size());
  TORCH_CHECK(world >= 2 && world <= ar::MAX_WORLD, "allreduce_rmsnorm_p2p: 2..8 ranks");
  TORCH_CHECK(inp.dim() == 2 && x.sizes() == inp.sizes() && h.sizes() == inp.sizes(),
              "allreduce_rmsnorm_p2p: [T, H] shapes");
  const int64_t T = inp.size(0), H = inp.size(1);
  for (const at::Tensor& t : {std::cref(h), std::cref(inp), std::cref(x), std::cref(w)})
    TORCH_CHECK(t.is_contiguous() && t.scalar_type() == at::kBFloat16 &&
                    reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
                "allreduce_rmsnorm_p2p: contiguous 16-byte-aligned bf16 tensors");
  TORCH_CHECK(w.numel() == H && H % 8 == 0, "allreduce_rmsnorm_p2p: norm weight / hidden");
  if (H / 8 > ar::THREADS * ar::MAX_VPT || T * H > max_elems) return false;
  const ar::Layout l = ar::layout(max_elems, world);
  const int64_t rp = (T + world - 1) / world;
  if (rp * (H / 8) > l.max_per) return false;
  if (T == 0) return true;
  ar::NormArgs na = {};
  for (int r = 0; r < world; ++r) {
    uint8_t* b = reinterpret_cast<uint8_t*>(bases[r]);
    na.b.recv1[r] = reinterpret_cast<uint4*>(b + l.recv1_off);
    na.b.recv2[r] = reinterpret_cast<uint4*>(b + l.recv2_off);
  }
  na.b.in = reinterpret_cast<const uint4*>(inp.data_ptr());
  na.b.epochs = reinterpret_cast<int*>(bases[rank]);
  na.b.nvec = T * H / 8;
  na.b.max_per = l.max_per;
  na.b.max_vec = l.max_vec;
  na.b.world = world;
  na.b.rank = static_cast<int>(rank);
  na.b.err = err.data_ptr<int>();
  na.x = reinterpret_cast<uint4*>(x.data_ptr());
  na.w = reinterpret_cast<const uint4*>(w.data_ptr());
  na.h = reinterpret_cast<uint4*>(h.data_ptr());
  na.T = static_cast<int>(T);
  na.HV = static_cast<int>(H / 8);
  na.eps = static_cast<float>(eps);
  const int g = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas, ar::MAX_CTAS)));
  na.b.fence_mode = comm_fence_mode();
  C10_CUDA_CHECK(launch_k(ar::allreduce_rmsnorm_kernel, dim3(g), dim3(ar::THREADS), 0,
                          at::cuda::getCurrentCUDAStream(), nullptr, 0, na));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return true;
}

}  // namespace lb
