// Row-parallel exchange for tensor-parallel decode/prefill over NVLink peer memory (sm_100a):
//
//     x_own <- x_own + sum_ranks(partial);   h = rmsnorm(x) * w  for every token row
//
// in ONE launch, after the row-parallel GEMM (o_proj or down_proj) of a transformer sub-layer.
// The reference's row-parallel layer is a GEMM on each shard followed by an all-reduce done as
// to_device + add on device 0 (src/multi_gpu/tensor_parallel.rs:119-133,312-345), then a
// separate residual add and RMSNorm (src/model/custom_transformer_block.rs:304-357).
//
// Ownership.  Token rows are owned in contiguous ranges: owner j holds rows
// [j * rp, min(T, (j + 1) * rp)), rp = ceil(T / world).  The residual stream is sharded the same
// way (each rank keeps only its own rows up to date), so the owner reduces, adds the residual and
// normalises each of its rows once, and only the normalised rows travel back (all-gather).  The
// bytes on NVLink are those of an all-reduce; the arithmetic of the add and the norm is split
// world ways.
//
// Data is its own flag (no flags, no handshakes).  Every receive slot holds the sentinel 0xFFFF
// in each bf16 lane until written; writers never send 0xFFFF (such a lane, a NaN, is rewritten
// to the canonical NaN 0x7FFF); readers poll their OWN memory until no lane is the sentinel,
// then write the sentinel back.  Per-rank symmetric buffer (one cudaMalloc, CUDA IPC):
//
//     [ header 256 B: epoch, done | recv1 [2 parities][world sources][RPMAX rows][H]
//                                   | recv2 [2 parities][TMAX rows][H] ]
//
// Parity = epoch & 1, where the epoch word counts row-parallel exchanges on this rank.  It is
// read by every CTA at the start of the launch and advanced by the last CTA to finish, so a
// GEMM launched next on the stream (which may push its output straight into the receive slots,
// gemm_tc.cu) sees the next parity.  Every rank performs the same exchanges in the same order,
// so epochs agree across ranks.
//
// Phases of one launch on rank `me` (CTA b, G CTAs):
//   push   (partial given locally): rows of owner j != me -> recv1_j[par][me] (peer stores);
//   own    rows b, b + G, ... of me: poll recv1_me[par][s] for every source s != me (own
//          source: the local partial, or recv1_me[par][me] written by this rank's GEMM),
//          sum in rank order (fp32, identical on every rank), round to bf16, add the residual
//          (bf16), RMSNorm, store h locally and push it to every peer's recv2[par];
//   gather rows of every other owner: poll recv2_me[par] and copy into h.
// The own phase waits only on pushes, which never wait, so no wait chain forms across ranks.
//
// Slot reuse and ordering.  A slot of parity p on rank r is written back to the sentinel by r
// (store W, launch K_e of r) and written again by a peer s in exchange e + 2 (store X, launch
// K_{e+2} of s).  W must not land after X, or the slot would read as unwritten forever (the
// bounded poll would then report a timeout) -- X must follow W in the slot's coherence order:
//   1. K_{e+1} of r starts only after K_e completed on the same stream, and a completed kernel's
//      stores are performed at r's L2, the single point of coherence of r's memory (this is
//      what lets any later kernel on the stream read them);
//   2. r's pushes of exchange e + 1 (to s) are issued by K_{e+1}, so after W was performed;
//   3. s issues X (K_{e+2}) only after K_{e+1} of s observed those pushes of r, i.e. after they
//      were performed at s's L2 -- hence after W was performed at r's L2;
//   4. X travels over NVLink to the same point of coherence (r's L2), where it is performed
//      after W, which was already performed: X follows W in coherence order.
// The same chain covers the recv2 slots.  The PTX memory model states this ordering only with
// a release fence between W and r's next pushes; that fence (fence.acq_rel.sys at launch start,
// comm_fence_mode 1 in every thread, 2 in one thread per CTA before a barrier) is available,
// but measured at TP2 (256 x 4096 bf16) it costs ~7 us (every thread) or ~4 us (per CTA) of an
// 11 us exchange, so the default relies on steps 1-4.  Every poll is bounded in time; on expiry
// the kernel records kErrTimeoutPeer and skips the rest of its waits.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {
namespace rowpar {

constexpr int MAX_WORLD = 8;
constexpr int THREADS = 256;
constexpr int MAX_VPT = 4;            // hidden <= 8 * THREADS * MAX_VPT = 8192
constexpr int64_t HEADER_BYTES = 256;
constexpr uint32_t SENT = 0xFFFFu;

struct Layout {
  int64_t rp_max, t_max, hv, recv1_off, recv2_off, bytes;
};

inline Layout layout(int64_t max_tokens, int64_t hidden, int64_t world) {
  Layout l;
  l.t_max = max_tokens;
  l.rp_max = (max_tokens + world - 1) / world;
  l.hv = hidden / 8;
  l.recv1_off = HEADER_BYTES;
  l.recv2_off = l.recv1_off + 2 * world * l.rp_max * l.hv * 16;
  l.bytes = l.recv2_off + 2 * l.t_max * l.hv * 16;
  return l;
}

struct Args {
  const uint4* partial;          // local partial [T][HV] (nullptr: pushed by the GEMM)
  uint4* recv1[MAX_WORLD];       // every rank's recv1, parity 0
  uint4* recv2[MAX_WORLD];       // every rank's recv2, parity 0
  int* epoch;                    // local header
  int* done;
  uint4* x_own;                  // residual rows of this rank [rows_me][HV], updated in place
  const uint4* w;                // norm weight [HV]
  uint4* h;                      // normalised rows, all T [T][HV]
  int T, HV, world, me, rp;
  int64_t rp_max, t_max;
  float eps;
  int* err;
  unsigned long long* trace;     // optional: CTA 0 thread 0 stamps [start, pushed, own rows
                                 // done, gathered] (globaltimer ns)
  int fence_mode;                // 1: every thread fences at launch start; 2: thread 0 only
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

// Poll a local slot until every lane is written; false when the time budget ran out.
__device__ __forceinline__ bool poll(const uint4* p, uint4& v, uint64_t t0) {
  uint32_t it = 0;
  while (true) {
    v = ld_vol(p);
    if (lanes_ready(v)) return true;
    if ((++it & 127u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ int rows_of(int j, int T, int rp) {
  return max(0, min(rp, T - j * rp));
}

__global__ void __launch_bounds__(THREADS) rowpar_norm_kernel(const Args a) {
  __shared__ int s_e;
  __shared__ float red[THREADS / 32];
  __shared__ int s_last;
  unsigned long long* tr = (a.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) ? a.trace
                                                                                       : nullptr;
  pdl_trigger();
  pdl_wait();
  if (tr) tr[0] = globaltimer_ns();
  if (threadIdx.x == 0) s_e = *a.epoch;
  // optional release fence for the slot-reuse ordering (see the file comment; mode 2: thread
  // 0, before the CTA barrier that precedes every store of the CTA)
  if (a.fence_mode == 1 || (a.fence_mode == 2 && threadIdx.x == 0)) fence_acq_rel_sys();
  __syncthreads();
  const uint64_t t0 = globaltimer_ns();
  const int par = s_e & 1;
  const int W = a.world, me = a.me, HV = a.HV, rp = a.rp;
  const int64_t src_stride = a.rp_max * HV;                 // vectors per recv1 source slot
  const uint4 sent = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  bool ok = true;

  // ---- push (local partial): rows of every other owner into its recv1[par][me] ----
  if (a.partial != nullptr) {
    const int64_t step = static_cast<int64_t>(gridDim.x) * THREADS;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x;
    for (int d = 1; d < W; ++d) {
      const int j = (me + d) % W;
      const int64_t nv = static_cast<int64_t>(rows_of(j, a.T, rp)) * HV;
      const uint4* src = a.partial + static_cast<int64_t>(j) * rp * HV;
      uint4* dst = a.recv1[j] + (static_cast<int64_t>(par) * W + me) * src_stride;
      // four loads in flight before their peer stores (the stores do not alias the partial)
      int64_t v = first;
      for (; v + 3 * step < nv; v += 4 * step) {
        uint4 t[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) t[u] = src[v + u * step];
#pragma unroll
        for (int u = 0; u < 4; ++u) dst[v + u * step] = canon4(t[u]);
      }
      for (; v < nv; v += step) dst[v] = canon4(src[v]);
    }
  }

  if (tr) tr[1] = globaltimer_ns();
  // ---- own rows: reduce (rank order) + residual + RMSNorm, push h to every peer ----
  const int my_rows = rows_of(me, a.T, rp);
  const int64_t row0 = static_cast<int64_t>(me) * rp;
  uint4* r1 = a.recv1[me] + static_cast<int64_t>(par) * W * src_stride;
  for (int i = blockIdx.x; i < my_rows; i += gridDim.x) {
    float xv[MAX_VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < MAX_VPT; ++k) {
      const int vi = threadIdx.x + k * THREADS;
      if (vi >= HV) continue;
      const int64_t off = static_cast<int64_t>(i) * HV + vi;
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      // one load of every source's slot in flight at once; only slots that are not yet
      // written are polled again (a chain of dependent polls would cost one memory latency
      // per source)
      uint4 qs[MAX_WORLD];
#pragma unroll
      for (int s = 0; s < MAX_WORLD; ++s) {
        if (s >= W) continue;
        if (s == me)
          qs[s] = a.partial != nullptr ? a.partial[(row0 + i) * HV + vi] : r1[me * src_stride + off];
        else
          qs[s] = ld_vol(r1 + s * src_stride + off);
      }
#pragma unroll
      for (int s = 0; s < MAX_WORLD; ++s) {
        if (s >= W) continue;
        uint4 q = qs[s];
        if (s != me) {
          uint4* p = r1 + s * src_stride + off;
          if (!ok) {
            q = zero;
          } else if (lanes_ready(q) || poll(p, q, t0)) {
            *p = sent;
          } else {
            ok = false;
            q = zero;
          }
        }
        float f[8];
        unpack8(q, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += f[e];
      }
      float xr[8];
      unpack8(a.x_own[off], xr);
      uint4 xn;
      uint32_t* xw = reinterpret_cast<uint32_t*>(&xn);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // rounding of the unfused path: sum -> bf16, residual add -> bf16
        const float y0 = __bfloat162float(__float2bfloat16(acc[2 * e]));
        const float y1 = __bfloat162float(__float2bfloat16(acc[2 * e + 1]));
        xw[e] = pack_bf16x2(xr[2 * e] + y0, xr[2 * e + 1] + y1);
      }
      a.x_own[off] = xn;
      unpack8(xn, xv[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += xv[k][e] * xv[k][e];
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < THREADS / 32; ++k) tot += red[k];
    const float inv = rsqrtf(tot / (8.f * HV) + a.eps);
    __syncthreads();   // red is rewritten by the next row
#pragma unroll
    for (int k = 0; k < MAX_VPT; ++k) {
      const int vi = threadIdx.x + k * THREADS;
      if (vi >= HV) continue;
      float wf[8];
      unpack8(a.w[vi], wf);
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        ow[e] = pack_bf16x2(xv[k][2 * e] * inv * wf[2 * e], xv[k][2 * e + 1] * inv * wf[2 * e + 1]);
      const int64_t g = (row0 + i) * HV + vi;
      a.h[g] = o;
      const uint4 oc = canon4(o);
      for (int d = 1; d < W; ++d) {
        const int j = (me + d) % W;
        a.recv2[j][static_cast<int64_t>(par) * a.t_max * HV + g] = oc;
      }
    }
  }

  if (tr) tr[2] = globaltimer_ns();
  // ---- gather: normalised rows of every other owner, from the local recv2 ----
  {
    uint4* r2 = a.recv2[me] + static_cast<int64_t>(par) * a.t_max * HV;
    const int64_t step = static_cast<int64_t>(gridDim.x) * THREADS;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x;
    // up to GB vectors of this thread: loads issued together, then polled where still unwritten
    constexpr int GB = 8;
    int64_t idx[GB];
    uint4 xs[GB];
    int n = 0;
    auto flush = [&]() {
#pragma unroll
      for (int u = 0; u < GB; ++u)
        if (u < n) xs[u] = ld_vol(r2 + idx[u]);
#pragma unroll
      for (int u = 0; u < GB; ++u) {
        if (u >= n || !ok) continue;
        uint4 x = xs[u];
        if (!lanes_ready(x) && !poll(r2 + idx[u], x, t0)) {
          ok = false;
          continue;
        }
        r2[idx[u]] = sent;
        a.h[idx[u]] = x;
      }
      n = 0;
    };
    for (int d = 1; d < W && ok; ++d) {
      const int j = (me + d) % W;
      const int64_t base = static_cast<int64_t>(j) * rp * HV;
      const int64_t nv = static_cast<int64_t>(rows_of(j, a.T, rp)) * HV;
      for (int64_t v = first; v < nv; v += step) {
        idx[n++] = base + v;
        if (n == GB) flush();
      }
    }
    if (ok && n > 0) flush();
  }
  if (!ok) record_error(a.err, kErrTimeoutPeer);
  if (tr) tr[3] = globaltimer_ns();
  __syncthreads();
  if (threadIdx.x == 0) {
    s_last = atomicAdd(a.done, 1) == static_cast<int>(gridDim.x) - 1;
    if (s_last) {
      *a.done = 0;
      *a.epoch = s_e + 1;   // the next exchange (and a GEMM pushing into it) uses parity ^ 1
    }
  }
}

}  // namespace rowpar

void set_pdl_launch(bool on) { set_pdl(on); }
bool pdl_launch_enabled() { return pdl_enabled(); }
void set_comm_fence_mode(int64_t mode) {
  TORCH_CHECK(mode >= 0 && mode <= 2, "fence mode 0, 1 or 2");
  comm_fence_mode() = static_cast<int>(mode);
}

int64_t rowpar_buffer_bytes(int64_t max_tokens, int64_t hidden, int64_t world) {
  TORCH_CHECK(hidden % 8 == 0 && world >= 1 && world <= rowpar::MAX_WORLD, "rowpar: shape");
  return rowpar::layout(max_tokens, hidden, world).bytes;
}

// Geometry the GEMM push epilogue needs: {recv1 offset, vectors per source slot}.
std::vector<int64_t> rowpar_geometry(int64_t max_tokens, int64_t hidden, int64_t world) {
  const rowpar::Layout l = rowpar::layout(max_tokens, hidden, world);
  return {l.recv1_off, l.rp_max, l.recv2_off, l.t_max};
}

// Zero the header and fill every receive slot with the sentinel (on every rank, then barrier).
void rowpar_prepare(int64_t base, int64_t max_tokens, int64_t hidden, int64_t world) {
  const rowpar::Layout l = rowpar::layout(max_tokens, hidden, world);
  uint8_t* b = reinterpret_cast<uint8_t*>(base);
  C10_CUDA_CHECK(cudaMemset(b, 0, rowpar::HEADER_BYTES));
  C10_CUDA_CHECK(cudaMemset(b + rowpar::HEADER_BYTES, 0xFF, l.bytes - rowpar::HEADER_BYTES));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
}

// h[T, H] = rmsnorm(x) * w for all rows, where x_own (this rank's rows [me*rp, ...), updated in
// place) += sum over ranks of the row-parallel partial.  partial: local [T, H] bf16, or None
// when the GEMM already pushed its output into the receive slots of this exchange.
void rowpar_norm(at::Tensor& h, const c10::optional<at::Tensor>& partial, at::Tensor& x_own,
                 const at::Tensor& w, std::vector<int64_t> bases, int64_t rank, int64_t T,
                 int64_t max_tokens, double eps, int64_t ctas, at::Tensor& err,
                 int64_t trace_ptr) {
  const int world = static_cast<int>(bases.size());
  TORCH_CHECK(world >= 2 && world <= rowpar::MAX_WORLD, "rowpar_norm: 2..8 ranks");
  TORCH_CHECK(T >= 1 && T <= max_tokens, "rowpar_norm: T exceeds the exchange capacity");
  const int64_t H = h.size(1);
  TORCH_CHECK(h.dim() == 2 && h.size(0) >= T && H % 8 == 0 && H / 8 <= rowpar::THREADS * rowpar::MAX_VPT,
              "rowpar_norm: h [>=T, H], H % 8 == 0, H <= 8192");
  const int64_t rp = (T + world - 1) / world;
  const int64_t my_rows = std::max<int64_t>(0, std::min<int64_t>(rp, T - rank * rp));
  TORCH_CHECK(x_own.dim() == 2 && x_own.size(0) >= my_rows && x_own.size(1) == H && w.numel() == H,
              "rowpar_norm: x_own [rows_me, H], w [H]");
  std::vector<const at::Tensor*> ts = {&h, &x_own, &w};
  if (partial.has_value() && partial->defined()) {
    TORCH_CHECK(partial->dim() == 2 && partial->size(0) >= T && partial->size(1) == H,
                "rowpar_norm: partial [T, H]");
    ts.push_back(&partial.value());
  }
  for (const at::Tensor* t : ts)
    TORCH_CHECK(t->is_contiguous() && t->scalar_type() == at::kBFloat16 &&
                    reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "rowpar_norm: contiguous 16-byte-aligned bf16 tensors");
  const rowpar::Layout l = rowpar::layout(max_tokens, H, world);
  rowpar::Args a = {};
  for (int r = 0; r < world; ++r) {
    uint8_t* b = reinterpret_cast<uint8_t*>(bases[r]);
    a.recv1[r] = reinterpret_cast<uint4*>(b + l.recv1_off);
    a.recv2[r] = reinterpret_cast<uint4*>(b + l.recv2_off);
  }
  uint8_t* mine = reinterpret_cast<uint8_t*>(bases[rank]);
  a.epoch = reinterpret_cast<int*>(mine);
  a.done = reinterpret_cast<int*>(mine + 4);
  a.partial = (partial.has_value() && partial->defined())
                  ? reinterpret_cast<const uint4*>(partial->data_ptr()) : nullptr;
  a.x_own = reinterpret_cast<uint4*>(x_own.data_ptr());
  a.w = reinterpret_cast<const uint4*>(w.data_ptr());
  a.h = reinterpret_cast<uint4*>(h.data_ptr());
  a.T = static_cast<int>(T);
  a.HV = static_cast<int>(H / 8);
  a.world = world;
  a.me = static_cast<int>(rank);
  a.rp = static_cast<int>(rp);
  a.rp_max = l.rp_max;
  a.t_max = l.t_max;
  a.eps = static_cast<float>(eps);
  a.err = err.data_ptr<int>();
  a.trace = reinterpret_cast<unsigned long long*>(trace_ptr);
  const int g = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas, 1024)));
  a.fence_mode = comm_fence_mode();
  C10_CUDA_CHECK(launch_k(rowpar::rowpar_norm_kernel, dim3(g), dim3(rowpar::THREADS), 0,
                          at::cuda::getCurrentCUDAStream(), nullptr, 0, a));
}

}  // namespace lb
