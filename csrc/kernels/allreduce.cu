// Two-shot all-reduce over NVLink peer memory for tensor-parallel decode partials (sm_100a).
//
// The reference's TP "all-reduce" (src/multi_gpu/tensor_parallel.rs:119-133) copies each
// partial to device 0 and adds them serially.  This kernel replaces NCCL's ring all-reduce for
// the small (0.1-4 MB) partial sums of a decode step, where latency, not bandwidth, dominates.
// It uses no flags, fences or handshakes: the data is its own flag.
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
// epoch only after this rank finished epoch e + 1 (it needs this rank's pushes of e + 2, issued
// by a later kernel), so the sentinel written back in epoch e is in place.  Partial visibility
// of a 16-byte store is harmless: every lane is checked.  Every poll is bounded in time: on
// expiry the kernel records an error code and stops.  Peer memory is written with plain stores
// only; the only loads are of this GPU's own memory.
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

__global__ void __launch_bounds__(THREADS) allreduce_kernel(const Args a) {
  __shared__ int s_e;
  if (threadIdx.x == 0) s_e = a.epochs[blockIdx.x] + 1;
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
  ar::allreduce_kernel<<<g, ar::THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lb
