// Dense bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   C[M, N] = A[M, K] . W[N, K]^T   (+ residual)   with fused epilogues
//
// Replaces every `Linear` of the reference (cuBLAS through candle, e.g. the q/k/v/o
// projections at src/model/custom_attention.rs:265-267,671 and the MLP at
// src/model/mlp_wrapper.rs:185-195).
//
// Design (B200-first):
//  * "swap-AB": the weight tile is the MMA's 128-row A operand and the token tile is the
//    MMA's N dimension (16..256).  Decode batches of a few tokens then still issue full
//    128-row MMAs and weights are streamed exactly once.
//  * persistent CTAs (one per SM), warp-specialised: warp 0 issues TMA loads into a
//    STAGES-deep shared-memory ring, warp 1 (one thread) issues tcgen05.mma into a
//    double-buffered TMEM accumulator, warps 2..5 drain TMEM with tcgen05.ld and run the
//    epilogue while the next tile's MMAs proceed.
//  * split-K for small tile counts: fp32 partial tiles go to a workspace, the last CTA to
//    arrive on the tile's counter reduces them in fixed split order (deterministic) and
//    resets the counter for the next launch.
//  * epilogues: bf16 store (+ residual add), fp32 store (logits), and SwiGLU on
//    gate/up rows interleaved in 64-row groups (writes silu(g) * u, half width).
//  * every TMA load reads this GPU's own memory and fills one CTA's shared memory.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <mutex>

#include <cmath>
#include <cstring>

#include "cluster_rs.cuh"
#include "common.cuh"

namespace lb {

constexpr int BW = 128;        // weight rows per tile (MMA M)
constexpr int BK = 64;         // K elements per pipeline stage (one 128-byte swizzle row)
constexpr int UK = 16;         // K per tcgen05.mma kind::f16
constexpr int kThreads = 192;  // warp 0: TMA, warp 1: MMA, warps 2..5: epilogue

enum EpiMode : int { kEpiStore = 0, kEpiSwiGLU = 1, kEpiF32 = 2 };

// Tensor-parallel link of a GEMM (all zero = plain GEMM).  Consumer side: the TMA producer
// waits until *wait_flag >= wait_count (peers have pushed every row of the gathered input)
// and the last CTA resets the flag.  Producer side (scatter): output row m goes to owner
// o = m / rows_per_rank, into o's reduce-scatter slot for this rank, by P2P stores; the last
// CTA then increments every owner's flag (system-scope release).
//
// Push mode (push = 1, tp_rowpar.cu's exchange): the receive slots hold a sentinel until written
// and the data is its own flag, so there are no signals and no completion counter.  Token m goes
// to owner o = m / rows_per_rank, row m - o * rows_per_rank of slot (parity, src_rank) of o's
// receive buffer, parity = *epoch & 1 (the exchange's counter, advanced by the consuming
// rowpar_norm launch).  bf16 lanes equal to the sentinel 0xFFFF are sent as 0x7FFF; with the
// optional slot-reuse fence (push = 2) every epilogue thread executes fence.acq_rel.sys at
// kernel start.
struct TpLink {
  bf16* scatter[8];
  int* signal[8];
  int world;
  int rows_per_rank;
  int src_rank;
  long long slot_stride;  // elements between source slots in a receive buffer
  int* wait_flag;
  int wait_count;
  int* done_counter;      // local grid-completion counter (reset by the last CTA)
  int push;               // 1: sentinel-protocol push into the row-parallel exchange (2: with
                          // a release fence at kernel start)
  const int* epoch;       // push mode: this rank's exchange counter (parity = epoch & 1)
};

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_per_split, kb_total;
  void* C;
  int ldc;
  const bf16* residual;
  int ldr;
  float* ws;
  int* counters;
  int mode;
  int* err;
  unsigned long long* trace;  // optional: 8 globaltimer stamps per CTA (phase profiling)
  int vec_ok;                 // C base 16-byte aligned and ldc % 4 == 0: vector stores
  TpLink tp;
  int tma_out;                // cluster kernel: output tiles through the tensor map tmC
  int sk_q;                   // > 0: stream-K, k-blocks per CTA over the (tile, k-block) space
};

// Work of one persistent CTA, as segments (tile, split, k-block range).
//  * data-parallel / split-K: units blockIdx.x, +gridDim.x, ... of tiles x splits;
//  * stream-K (sk_q > 0): the contiguous range [b * q, (b + 1) * q) of the linearised
//    (tile, k-block) space, cut at tile boundaries.  Only a CTA's first segment can start
//    inside a tile (it then contributes a partial); a segment that starts a tile but ends
//    inside it belongs to the tile's finisher, which adds the following CTAs' partials.
struct WorkIter {
  int u, g, g1;
  __device__ __forceinline__ void begin(const GemmArgs& a) {
    if (a.sk_q > 0) {
      const long long tot = static_cast<long long>(a.m_tiles) * a.n_tiles * a.kb_total;
      g = static_cast<int>(min(static_cast<long long>(blockIdx.x) * a.sk_q, tot));
      g1 = static_cast<int>(min(static_cast<long long>(g) + a.sk_q, tot));
    } else {
      u = blockIdx.x;
    }
  }
  // tile index t (mt * n_tiles + nt), split index s (data-parallel only), k-block range.
  __device__ __forceinline__ bool next(const GemmArgs& a, int& t, int& s, int& kb0, int& kb1) {
    if (a.sk_q > 0) {
      if (g >= g1) return false;
      t = g / a.kb_total;
      kb0 = g - t * a.kb_total;
      kb1 = min(a.kb_total, kb0 + (g1 - g));
      s = 0;
      g += kb1 - kb0;
      return true;
    }
    if (u >= a.m_tiles * a.n_tiles * a.splits) return false;
    s = u % a.splits;
    t = u / a.splits;
    kb0 = s * a.kb_per_split;
    kb1 = min(kb0 + a.kb_per_split, a.kb_total);
    u += gridDim.x;
    return true;
  }
};

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

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

// Bounded wait for a flag written by peer GPUs (5 s budget).
__device__ __forceinline__ bool wait_flag_geq(const int* flag, int target, volatile int* abort_flag) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (ld_acquire_sys(flag) < target) {
    if ((++it & 63u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - t0 > 5000000000ull) return false;
    }
    __nanosleep(64);
  }
  return true;
}

template <int BT, int STAGES>
struct GemmSmem {
  static constexpr int W_BYTES = BW * BK * 2;
  static constexpr int X_BYTES = BT * BK * 2;
  static constexpr int CH = BT < 32 ? BT : 32;  // epilogue column chunk
  static constexpr int EPI_FLOATS = 64 * (CH + 1);
  static constexpr int BAR_OFF = STAGES * (W_BYTES + X_BYTES) + EPI_FLOATS * 4;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;  // barriers/flags + alignment slack
  static constexpr int TMEM_COLS = 2 * BT < 32 ? 32 : 2 * BT;
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

template <int BT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const GemmArgs a) {
  using L = GemmSmem<BT, STAGES>;
  constexpr int CH = L::CH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * L::W_BYTES;
  float* sEpi = reinterpret_cast<float*>(sX + STAGES * L::X_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_last = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* s_go = reinterpret_cast<volatile int*>(tmem_slot + 4);  // [2]
  volatile int* s_fin = reinterpret_cast<volatile int*>(tmem_slot + 6);  // [2] stream-K finisher

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // tile t -> (m tile, n tile); consecutive tiles share the token tile so that the
  // activation stays in L2 while each weight tile is streamed once.

  uint32_t issued_mask = 0, issued_parity = 0;  // producer bookkeeping for abort drain

  pdl_trigger();
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pw = policy_evict_first();
      const uint64_t px = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      WorkIter w;
      w.begin(a);
      int t, s, kb0, kb1;
      // The first work item's first weight tiles depend on no earlier kernel: issue them
      // before waiting for the previous grid (PDL); their activation tiles follow the wait.
      int pre = 0;
      {
        WorkIter w0 = w;
        int t0, s0, a0, b0;
        if (w0.next(a, t0, s0, a0, b0)) {
          pre = min(STAGES, max(0, b0 - a0));
          for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], L::W_BYTES + L::X_BYTES);
            tma_load_2d(sW + i * L::W_BYTES, &tmW, &full[i], (a0 + i) * BK,
                        (t0 % a.n_tiles) * BW, pw);
          }
        }
      }
      pdl_wait();
      int issued = 0;
      while (w.next(a, t, s, kb0, kb1)) {
        if (issued >= pre && *abort_flag) break;
        const int nt = t % a.n_tiles, mt = t / a.n_tiles;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++issued) {
          if (issued >= pre) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
              record_error(a.err, kErrTimeoutSmemEmpty);
              *abort_flag = 1;
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], L::W_BYTES + L::X_BYTES);
            tma_load_2d(sW + stage * L::W_BYTES, &tmW, &full[stage], kb * BK, nt * BW, pw);
          }
          tma_load_2d(sX + stage * L::X_BYTES, &tmX, &full[stage], kb * BK, mt * BT, px);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BW, BT);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      WorkIter w;
      w.begin(a);
      int t, s, kb0, kb1;
      for (; !*abort_flag && w.next(a, t, s, kb0, kb1); ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) {
          record_error(a.err, kErrTimeoutTmemEmpty);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BT);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            record_error(a.err, kErrTimeoutTmaFull);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wb = smem_u32(sW + stage * L::W_BYTES);
          const uint32_t xb = smem_u32(sX + stage * L::X_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UK; ++k) {
            tc_mma_f16(d_tmem, sw128_kmajor_desc(wb + k * UK * 2),
                       sw128_kmajor_desc(xb + k * UK * 2), idesc,
                       (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
      }
    }
  } else {
    // ---------------- epilogue warps ----------------
    pdl_wait();   // workspace, counters, residual and output follow the previous grid
    const int quad = warp & 3;           // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;    // weight row within the tile == TMEM lane
    const int etid = threadIdx.x - 64;   // 0..127
    int it = 0;
    WorkIter w;
    w.begin(a);
    int t, s, kb0, kb1;
    for (; w.next(a, t, s, kb0, kb1); ++it) {
      const int nt = t % a.n_tiles, mt = t / a.n_tiles;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      // One thread waits (bounded); the decision is broadcast so that all 128 epilogue
      // threads take the same path through the named barriers below.
      if (etid == 0) {
        int go = 1;
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) {
          record_error(a.err, kErrTimeoutTmemFull);
          *abort_flag = 1;
          go = 0;
        }
        s_go[it & 1] = go;
      }
      named_bar_sync(1, 128);
      if (!s_go[it & 1]) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BT);
      const int tile = t;
      const int m0 = mt * BT;
      const int n = nt * BW + row;

      auto emit = [&](const float* v, int c) {
        // v[0..CH) are columns (tokens) m0+c .. m0+c+CH-1 of weight row `row`.
        if (a.mode == kEpiSwiGLU) {
          if (row >= 64) {
#pragma unroll
            for (int j = 0; j < CH; ++j) sEpi[(row - 64) * (CH + 1) + j] = v[j];
          }
          named_bar_sync(1, 128);
          if (row < 64) {
            const int f = nt * 64 + row;
            const int nf = a.N >> 1;
            bf16* C = reinterpret_cast<bf16*>(a.C);
            if (f < nf) {
#pragma unroll
              for (int j = 0; j < CH; ++j) {
                const int m = m0 + c + j;
                if (m < a.M) {
                  const float g = v[j];
                  const float up = sEpi[row * (CH + 1) + j];
                  C[static_cast<size_t>(m) * a.ldc + f] = __float2bfloat16(silu(g) * up);
                }
              }
            }
          }
          named_bar_sync(1, 128);
        } else if (n < a.N) {
          if (a.mode == kEpiF32) {
            float* C = reinterpret_cast<float*>(a.C);
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const int m = m0 + c + j;
              if (m < a.M) C[static_cast<size_t>(m) * a.ldc + n] = v[j];
            }
          } else {
            bf16* C = reinterpret_cast<bf16*>(a.C);
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const int m = m0 + c + j;
              if (m < a.M) {
                float x = v[j];
                if (a.residual != nullptr)
                  x += __bfloat162float(a.residual[static_cast<size_t>(m) * a.ldr + n]);
                C[static_cast<size_t>(m) * a.ldc + n] = __float2bfloat16(x);
              }
            }
          }
        }
      };

      float v[CH];
      const bool sk_part = a.sk_q > 0 && kb0 > 0;                       // contributor
      const bool sk_fin = a.sk_q > 0 && kb0 == 0 && kb1 < a.kb_total;   // finisher
      if (sk_part) {
        // partial of k-blocks [kb0, kb1) -> this CTA's slot; the tile's finisher adds it
        float* wsp = a.ws + static_cast<size_t>(blockIdx.x) * BT * BW;
#pragma unroll 1
        for (int c = 0; c < BT; c += CH) {
          uint32_t r[CH];
          if constexpr (CH == 32) {
            tmem_ld32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(r));
          } else {
            tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tc_wait_ld();
          if (c + CH >= BT) {
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
          }
#pragma unroll
          for (int j = 0; j < CH; ++j) __stcg(&wsp[(c + j) * BW + row], __uint_as_float(r[j]));
        }
        __threadfence();
        named_bar_sync(1, 128);
        if (etid == 0) st_release_gpu(&a.counters[blockIdx.x], 1);
      } else if (sk_fin) {
        // contributors: the following CTAs whose ranges start inside this tile
        const long long tile_end = static_cast<long long>(t + 1) * a.kb_total;
        int c_last = blockIdx.x;
        while (c_last + 1 < static_cast<int>(gridDim.x) &&
               static_cast<long long>(c_last + 1) * a.sk_q < tile_end)
          ++c_last;
        if (etid == 0) {
          int go = 1;
          for (int c2 = blockIdx.x + 1; c2 <= c_last && go; ++c2) {
            const uint64_t t0 = globaltimer_ns();
            uint32_t spins = 0;
            while (ld_acquire_gpu(&a.counters[c2]) == 0) {
              if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
                record_error(a.err, kErrTimeoutPeer);
                *abort_flag = 1;
                go = 0;
                break;
              }
            }
            if (go) a.counters[c2] = 0;   // one consumer per contribution: re-armed for the next launch
          }
          s_fin[it & 1] = go;
        }
        named_bar_sync(1, 128);
        const bool have = s_fin[it & 1] != 0;
#pragma unroll 1
        for (int c = 0; c < BT; c += CH) {
          uint32_t r[CH];
          if constexpr (CH == 32) {
            tmem_ld32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(r));
          } else {
            tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tc_wait_ld();
          if (c + CH >= BT) {
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
          }
#pragma unroll
          for (int j = 0; j < CH; ++j) v[j] = __uint_as_float(r[j]);
          if (have) {
            // k order: this CTA's head first, then the contributors in CTA order
            for (int c2 = blockIdx.x + 1; c2 <= c_last; ++c2) {
              const float* p = a.ws + static_cast<size_t>(c2) * BT * BW;
#pragma unroll
              for (int j = 0; j < CH; ++j) v[j] += __ldcg(&p[(c + j) * BW + row]);
            }
            emit(v, c);
          }
        }
        if (!have) break;
      } else if (a.splits == 1) {
#pragma unroll 1
        for (int c = 0; c < BT; c += CH) {
          uint32_t r[CH];
          if constexpr (CH == 32) {
            tmem_ld32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(r));
          } else {
            tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tc_wait_ld();
          if (c + CH >= BT) {
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
          }
#pragma unroll
          for (int j = 0; j < CH; ++j) v[j] = __uint_as_float(r[j]);
          emit(v, c);
        }
      } else {
        // split-K: stash fp32 partial, last arriving CTA reduces in split order.
        float* wsp = a.ws + (static_cast<size_t>(tile) * a.splits + s) * BT * BW;
#pragma unroll 1
        for (int c = 0; c < BT; c += CH) {
          uint32_t r[CH];
          if constexpr (CH == 32) {
            tmem_ld32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(r));
          } else {
            tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tc_wait_ld();
          if (c + CH >= BT) {
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
          }
#pragma unroll
          for (int j = 0; j < CH; ++j) __stcg(&wsp[(c + j) * BW + row], __uint_as_float(r[j]));
        }
        __threadfence();
        named_bar_sync(1, 128);
        if (etid == 0) {
          const int prev = atomicAdd(&a.counters[tile], 1);
          *s_last = (prev == a.splits - 1) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (*s_last) {
          __threadfence();
          const float* base = a.ws + static_cast<size_t>(tile) * a.splits * BT * BW;
#pragma unroll 1
          for (int c = 0; c < BT; c += CH) {
#pragma unroll
            for (int j = 0; j < CH; ++j) v[j] = 0.f;
            for (int sp = 0; sp < a.splits; ++sp) {
              const float* p = base + static_cast<size_t>(sp) * BT * BW;
#pragma unroll
              for (int j = 0; j < CH; ++j) v[j] += __ldcg(&p[(c + j) * BW + row]);
            }
            emit(v, c);
          }
          if (etid == 0) a.counters[tile] = 0;
        }
      }
    }
  }

  __syncthreads();
  if (*abort_flag) {
    // Unwind: wait (bounded) for our own TMA loads and MMAs still in flight.
    if (warp == 0 && lane == 0) {
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s))
          if (!mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, kWaitBudgetNs))
            record_error(a.err, kErrTimeoutDrain);
    }
    if (warp == 1 && lane == 0) {
      tc_commit(drain);
      if (!mbar_wait(drain, 0, nullptr, kWaitBudgetNs)) record_error(a.err, kErrTimeoutDrain);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace lb

#include "gemm_tc2.cuh"

namespace lb {

// ======================================================================================
// Cluster split-K variant for small token counts (decode).  The S CTAs of a thread-block
// cluster own the same 128 x BT output tile and split K; the fp32 accumulators are combined
// by the push reduce-scatter of cluster_rs.cuh (16-column chunks, owner c % S, rank-order
// sum: deterministic), and each owner runs the epilogue for its chunks.  No global
// workspace, no atomics.
// ======================================================================================

// Destination row of output token m: local C, or (tensor-parallel scatter) the owner rank's
// reduce-scatter receive slot for this source rank, reached by P2P stores over NVLink.
__device__ __forceinline__ bf16* out_row(const GemmArgs& a, int m, int par) {
  if (a.tp.world > 0) {
    const int o = m / a.tp.rows_per_rank;
    const int r = m - o * a.tp.rows_per_rank;
    const long long slot = a.tp.push ? static_cast<long long>(par) * a.tp.world + a.tp.src_rank
                                     : a.tp.src_rank;
    return a.tp.scatter[o] + slot * a.tp.slot_stride + static_cast<size_t>(r) * a.ldc;
  }
  return reinterpret_cast<bf16*>(a.C) + static_cast<size_t>(m) * a.ldc;
}

// Push mode: a bf16 lane equal to the receive slots' sentinel 0xFFFF (a NaN) is sent as the
// canonical NaN 0x7FFF, so a written lane can never look unwritten.
__device__ __forceinline__ uint32_t canon_bf16x2(uint32_t w) {
  if ((w & 0xFFFFu) == 0xFFFFu) w = (w & 0xFFFF0000u) | 0x7FFFu;
  if ((w >> 16) == 0xFFFFu) w = (w & 0xFFFFu) | 0x7FFF0000u;
  return w;
}

template <int BT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_cluster_kernel(const __grid_constant__ CUtensorMap tmW,
                           const __grid_constant__ CUtensorMap tmX,
                           const __grid_constant__ CUtensorMap tmC, const GemmArgs a) {
  using L = GemmSmem<BT, STAGES>;
  constexpr int CH = L::CH;
  constexpr int TMEM_COLS = BT < 32 ? 32 : BT;
  static_assert(crs::smem_bytes(BT, 1) <= STAGES * (L::W_BYTES + L::X_BYTES) &&
                    crs::smem_bytes(BT, 8) <= STAGES * (L::W_BYTES + L::X_BYTES),
                "split-K slots");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * L::W_BYTES;
  // after the main loop: split-K slots, then the output staging tiles
  float* sSlots = reinterpret_cast<float*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* drain = tfull + 1;
  uint64_t* rbar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_go = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t S = crs::nctarank();
  const uint32_t rank = crs::ctarank();
  const int tile = blockIdx.x / S;
  float* ws_tile = a.ws + crs::ws_floats(tile, BT, S);
  const int mt = tile % a.m_tiles;
  const int nt = tile / a.m_tiles;
  const int kb0 = rank * a.kb_per_split;
  const int kb1 = min(kb0 + a.kb_per_split, a.kb_total);
  unsigned long long* tr = a.trace ? a.trace + blockIdx.x * 8 : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer_ns();
  // Push mode: release/acquire at system scope for everything of earlier launches on this
  // stream (the exchange's sentinel write-backs and polls) before this launch's peer stores.
  // Issued at kernel start by the epilogue threads (the only ones that push), where it has
  // no stores of its own to wait for and overlaps the main loop.
  if (a.tp.push == 2 && threadIdx.x >= 64) asm volatile("fence.acq_rel.sys;" ::: "memory");

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    mbar_init(rbar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  uint32_t issued_mask = 0, issued_parity = 0;
  bool mma_issued = false;
  if (tr && threadIdx.x == 0) tr[1] = globaltimer_ns();

  pdl_trigger();
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pw = policy_evict_first();
      const uint64_t px = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      // The weight tiles of the first stages depend on no earlier kernel: issue them before
      // waiting for the previous grid (PDL), the activation tiles after.
      const int pre = min(STAGES, max(0, kb1 - kb0));
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], L::W_BYTES + L::X_BYTES);
        tma_load_2d(sW + i * L::W_BYTES, &tmW, &full[i], (kb0 + i) * BK, nt * BW, pw);
      }
      pdl_wait();
      if (a.tp.wait_flag != nullptr) {
        if (!wait_flag_geq(a.tp.wait_flag, a.tp.wait_count, abort_flag)) {
          record_error(a.err, kErrTimeoutPeer);
          *abort_flag = 1;
        }
        // peers' rows were observed through the generic proxy; TMA reads via the async proxy
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0;
        if (i >= pre) {
          if (*abort_flag) break;
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            record_error(a.err, kErrTimeoutSmemEmpty);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], L::W_BYTES + L::X_BYTES);
          tma_load_2d(sW + stage * L::W_BYTES, &tmW, &full[stage], kb * BK, nt * BW, pw);
        }
        // prefetched stages still get their activation tile (after an abort too: the stage's
        // barrier expects both, and the unwind below waits for every issued stage)
        tma_load_2d(sX + stage * L::X_BYTES, &tmX, &full[stage], kb * BK, mt * BT, px);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BW, BT);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          record_error(a.err, kErrTimeoutTmaFull);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t wb = smem_u32(sW + stage * L::W_BYTES);
        const uint32_t xb = smem_u32(sX + stage * L::X_BYTES);
#pragma unroll
        for (int k = 0; k < BK / UK; ++k)
          tc_mma_f16(tmem_base, sw128_kmajor_desc(wb + k * UK * 2),
                     sw128_kmajor_desc(xb + k * UK * 2), idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        mma_issued = true;
        tc_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) tc_commit(tfull);
    }
  } else {
    // Epilogue warps: wait for the accumulator, publish the partial tile.
    pdl_wait();   // the split-K workspace, residual and output follow the previous grid
    const int etid = threadIdx.x - 64;
    if (etid == 0) {
      int go = 1;
      if (kb1 <= kb0) {
        go = 2;  // empty split: contributes zeros
      } else if (!mbar_wait(tfull, 0, abort_flag)) {
        record_error(a.err, kErrTimeoutTmemFull);
        *abort_flag = 1;
        go = 0;
      }
      s_go[0] = go;
      if (tr) tr[2] = globaltimer_ns();
    }
    named_bar_sync(1, 128);
    tc_fence_after();
    const int quad = warp & 3;
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    unsigned long long* tr2 = tr ? a.trace + (gridDim.x + blockIdx.x) * 8 : nullptr;
    crs::publish<BT>(tbase, s_go[0] == 1, sSlots, ws_tile, rank, S, quad * 32 + lane, etid, tr2);
  }

  tc_fence_before();
  if (tr && threadIdx.x == 64) tr[3] = globaltimer_ns();
  crs::sync_all();  // every partial of the cluster is in L2 / its owner's shared memory
  tc_fence_after();
  if (tr && threadIdx.x == 64) tr[4] = globaltimer_ns();

  if (warp >= 2) {
    const int e = threadIdx.x - 64;
    if (e == 0) crs::fetch<BT>(sSlots, ws_tile, rbar, rank, S);
    const int m0 = mt * BT;
    const int omode = a.mode == kEpiSwiGLU ? crs::kOutSwiGLU
                      : a.mode == kEpiF32  ? crs::kOutF32
                                           : crs::kOutBf16;
    const int x0 = omode == crs::kOutSwiGLU ? nt * 64 : nt * BW;
    const int par = a.tp.push ? (*a.tp.epoch & 1) : 0;
    // lane l: weight rows 4 l .. +3 of the chunk's token columns t0 .. t0 + 15 (acc[j])
    auto epi = [&](int oc, int t0, int l, float4 (&acc)[crs::CW]) {
      if (a.tma_out) {
        const int mf = m0 + t0, n0 = nt * BW;
        const bf16* res = a.residual != nullptr
                              ? a.residual + static_cast<size_t>(mf) * a.ldr + n0
                              : nullptr;
        uint8_t* tile = crs::out_tile(sSlots, 0, oc);
        crs::stage_out(omode, tile, l, acc, res, a.ldr, a.M - mf, a.N - n0);
        crs::store_chunk(&tmC, tile, l, x0, mf);
        return;
      }
      // per-thread stores (tensor-parallel scatter into peers' slots, or unaligned C)
      const int r0 = 4 * l;
#pragma unroll
      for (int j = 0; j < crs::CW; ++j) {
        const int m = m0 + t0 + j;
        if (a.mode == kEpiSwiGLU) {
          float4 up;
          up.x = __shfl_down_sync(0xffffffffu, acc[j].x, 16);
          up.y = __shfl_down_sync(0xffffffffu, acc[j].y, 16);
          up.z = __shfl_down_sync(0xffffffffu, acc[j].z, 16);
          up.w = __shfl_down_sync(0xffffffffu, acc[j].w, 16);
          const int f = nt * 64 + r0;
          if (l < 16 && m < a.M && f < (a.N >> 1)) {
            uint2 pk;
            pk.x = pack_bf16x2(silu(acc[j].x) * up.x, silu(acc[j].y) * up.y);
            pk.y = pack_bf16x2(silu(acc[j].z) * up.z, silu(acc[j].w) * up.w);
            *reinterpret_cast<uint2*>(out_row(a, m, par) + f) = pk;
          }
          continue;
        }
        const int n = nt * BW + r0;
        if (m >= a.M || n >= a.N) continue;
        float vv[4] = {acc[j].x, acc[j].y, acc[j].z, acc[j].w};
        if (a.mode == kEpiF32) {
          float* C = reinterpret_cast<float*>(a.C) + static_cast<size_t>(m) * a.ldc;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (n + u < a.N) C[n + u] = vv[u];
          continue;
        }
        bf16* C = out_row(a, m, par);
        if (a.residual != nullptr) {
          const bf16* R = a.residual + static_cast<size_t>(m) * a.ldr;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (n + u < a.N) vv[u] += __bfloat162float(R[n + u]);
        }
        if (n + 3 < a.N && a.vec_ok) {
          uint2 pk;
          pk.x = pack_bf16x2(vv[0], vv[1]);
          pk.y = pack_bf16x2(vv[2], vv[3]);
          if (a.tp.push) {
            pk.x = canon_bf16x2(pk.x);
            pk.y = canon_bf16x2(pk.y);
          }
          *reinterpret_cast<uint2*>(C + n) = pk;
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (n + u < a.N) C[n + u] = __float2bfloat16(vv[u]);
        }
      }
    };
    const bool ok = crs::reduce<BT>(sSlots, rbar, rank, S, e, abort_flag, epi);
    if (a.tma_out) crs::store_wait(e & 31, a.tp.done_counter != nullptr);
    if (!ok) {
      record_error(a.err, kErrTimeoutTmaFull);
      *abort_flag = 1;
      // let the bulk copies of this CTA land before its shared memory is released
      if (e == 0 && !mbar_wait(rbar, 0, nullptr, kWaitBudgetNs)) record_error(a.err, kErrTimeoutDrain);
    }
    if (tr && e == 0) tr[5] = globaltimer_ns();
  }
  __syncthreads();
  if (tr && threadIdx.x == 64) tr[6] = globaltimer_ns();
  if (a.tp.done_counter != nullptr && threadIdx.x == 0) {
    // Grid completion: the last CTA resets the consumed input flag and signals the owners.
    // One system-scope fence per CTA, after the cluster barrier that ordered every thread's
    // scatter stores before it (fences are cumulative), publishes this CTA's P2P stores.
    if (a.tp.world > 0) fence_acq_rel_sys();
    const int prev = atomicAdd(a.tp.done_counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      fence_acq_rel_sys();
      if (a.tp.wait_flag != nullptr) atomicExch(a.tp.wait_flag, 0);
      for (int o = 0; o < a.tp.world; ++o)
        if (a.tp.signal[o] != nullptr) red_release_sys_add(a.tp.signal[o], 1);
      atomicExch(a.tp.done_counter, 0);
      if (a.trace) a.trace[4095 * 8 + 7] = globaltimer_ns();
    }
  }
  if (*abort_flag) {
    if (warp == 0 && lane == 0) {
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s))
          if (!mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, kWaitBudgetNs))
            record_error(a.err, kErrTimeoutDrain);
    }
    if (warp == 1 && lane == 0 && mma_issued) {
      tc_commit(drain);
      if (!mbar_wait(drain, 0, nullptr, kWaitBudgetNs)) record_error(a.err, kErrTimeoutDrain);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ======================================================================================
// Host side
// ======================================================================================
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map (inner = contiguous dim) with 128-byte swizzle and a 64 x box_rows box.
CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swz) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                           strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(r));
  return m;
}

// Tensor map of the output for the cluster kernel's TMA-store epilogue: boxes of box_rows tokens
// x 128 columns (64 for SwiGLU), no swizzle.  False when C's base or row stride is not 16-byte
// aligned (the kernel then stores per thread).
bool make_tmap_out(const at::Tensor& C, int64_t mode, int M, int N, int box_rows, CUtensorMap* m) {
  const bool f32 = mode == kEpiF32;
  const int esz = f32 ? 4 : 2;
  const uint64_t cols = mode == kEpiSwiGLU ? N / 2 : N;
  const uint64_t stride = static_cast<uint64_t>(C.stride(0)) * esz;
  if (reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 != 0 || stride % 16 != 0 || cols == 0)
    return false;
  cuuint64_t dims[2] = {cols, static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {mode == kEpiSwiGLU ? 64u : 128u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                           2, C.data_ptr(), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BT, int STAGES>
static void launch_bt(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, int grid,
                      cudaStream_t st) {
  using L = GemmSmem<BT, STAGES>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_tc_kernel<BT, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         L::TOTAL);
    attr = true;
  }
  if (a.sk_q > 0) {
    // Stream-K: a tile's finisher waits for the partials of CTAs with higher indices, so every
    // CTA must be resident at once -- a cooperative launch guarantees it (or fails loudly)
    // instead of relying on an idle GPU.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BT, STAGES>, tw, tx, a));
    return;
  }
  C10_CUDA_CHECK(launch_k(gemm_tc_kernel<BT, STAGES>, dim3(grid), dim3(kThreads), L::TOTAL, st,
                          nullptr, 0, tw, tx, a));
}

static int pick_bt(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

// Token tile of the general GEMM: decode batches of 129-256 tokens against a narrow weight
// (<= 32 tiles of 128 rows, the tensor-parallel shards) and K <= 4096 take 128-token tiles,
// which doubles the CTAs of the cluster split-K plan.  Measured at M = 256 (us, 256 / 128):
// TP8 QKV 12.0 / 10.0, o_proj 10.0 / 7.8, down 12.2 / 11.1; TP4 QKV 12.9 / 11.2, o_proj
// 11.0 / 9.2; equal within 0.5 us on the other shard shapes and on the single-GPU o_proj.
static int pick_bt_shape(int M, int N, int K) {
  const int bt = pick_bt(M);
  if (bt == 256 && (N + BW - 1) / BW <= 32 && K <= 4096) return 128;
  return bt;
}

template <int BT, int STAGES>
static int max_active_clusters(int S) {
  using L = GemmSmem<BT, STAGES>;
  static int cache[9] = {0};
  if (S < 1 || S > 8) return 0;
  if (cache[S] == 0) {
    cudaFuncSetAttribute(gemm_tc_cluster_kernel<BT, STAGES>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S * 64);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::TOTAL;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_cluster_kernel<BT, STAGES>, &cfg) !=
        cudaSuccess) {
      cudaGetLastError();
      n = num_sms() / S;
    }
    cache[S] = std::max(1, n);
  }
  return cache[S];
}

static int active_clusters_for(int BT, int S) {
  switch (BT) {
    case 16: return max_active_clusters<16, 8>(S);
    case 32: return max_active_clusters<32, 8>(S);
    case 64: return max_active_clusters<64, 8>(S);
    case 128: return max_active_clusters<128, 6>(S);
    default: return max_active_clusters<256, 4>(S);
  }
}

// Cluster split-K factor: the largest S <= 8 whose grid (tiles x S CTAs) is co-resident in
// one wave, keeping >= 2 k-blocks per CTA.  0 = the tiles alone fill the GPU (no cluster).
// Whether the split-K receive slots of a cluster of S fit in the drained pipeline buffers.
static bool cluster_fits(int BT, int S) {
  const int stages = BT <= 64 ? 8 : BT == 128 ? 6 : 4;
  return crs::smem_bytes(BT, S) <= stages * (BW * BK * 2 + BT * BK * 2);
}

static int pick_cluster(int BT, int tiles, int kb_total) {
  if (tiles >= num_sms()) return 0;
  int best = 1;
  for (int S = 2; S <= 8; ++S) {
    if (kb_total / S < 2) break;
    if (cluster_fits(BT, S) && tiles <= active_clusters_for(BT, S)) best = S;
  }
  return best;
}

// Returns {token tile, split (>0: workspace split-K, <0: cluster split-K of -S CTAs),
// tile count, workspace floats} so Python can inspect / size workspaces.
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t bt, int64_t splits) {
  const int BT = bt > 0 ? static_cast<int>(bt)
                       : pick_bt_shape(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
  const int m_tiles = (M + BT - 1) / BT;
  const int n_tiles = (N + BW - 1) / BW;
  const int kb_total = (K + BK - 1) / BK;
  const int tiles = m_tiles * n_tiles;
  if (splits < 0 || (splits == 0 && pick_cluster(BT, tiles, kb_total) > 1)) {
    int S = splits < 0 ? static_cast<int>(-splits) : pick_cluster(BT, tiles, kb_total);
    S = std::max(1, std::min(S, std::min(8, kb_total)));
    while (S > 1 && !cluster_fits(BT, S)) --S;
    return {BT, -S, tiles, S > 1 ? crs::ws_floats(tiles, BT, S) : 0};
  }
  int sp = splits > 0 ? static_cast<int>(splits) : 1;
  sp = std::max(1, std::min(sp, kb_total));
  const int kbps = (kb_total + sp - 1) / sp;
  sp = (kb_total + kbps - 1) / kbps;  // no empty splits
  const int64_t ws_floats = sp > 1 ? static_cast<int64_t>(tiles) * sp * BT * BW : 0;
  return {BT, sp, tiles, ws_floats};
}

template <int BT, int STAGES>
static void launch_cluster(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tc,
                           const GemmArgs& a,
                           int S, cudaStream_t st) {
  using L = GemmSmem<BT, STAGES>;
  TORCH_CHECK(crs::smem_bytes(BT, S) <= STAGES * (L::W_BYTES + L::X_BYTES),
              "gemm: split-K slots exceed the pipeline buffers (BT ", BT, ", S ", S, ")");
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemm_tc_cluster_kernel<BT, STAGES>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
    attr_set = true;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  C10_CUDA_CHECK(launch_k(gemm_tc_cluster_kernel<BT, STAGES>, dim3(a.m_tiles * a.n_tiles * S),
                          dim3(kThreads), L::TOTAL, st, attr, 1, tw, tx, tc, a));
}

// SM-pair persistent GEMM (gemm_tc2.cuh): 256-row weight tiles, clusters of 2 CTAs.
template <int BT, int STAGES>
static void launch_pair(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a,
                        cudaStream_t st) {
  using L = tc2::Smem<BT, STAGES>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_tc2_kernel<BT, STAGES>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    attr = true;
  }
  const int n_tiles = (a.N + 2 * BW - 1) / (2 * BW);
  const int units = a.m_tiles * n_tiles;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr2[1];
  attr2[0].id = cudaLaunchAttributeClusterDimension;
  attr2[0].val.clusterDim.x = 2;
  attr2[0].val.clusterDim.y = 1;
  attr2[0].val.clusterDim.z = 1;
  cfg.attrs = attr2;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::TOTAL;
  // persistent grid: as many pairs as can be resident at once (SM pairs within a GPC)
  static int resident = 0;
  if (resident == 0) {
    cfg.gridDim = dim3(num_sms());
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<BT, STAGES>, &cfg) != cudaSuccess ||
        n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    resident = n;
  }
  const int pairs = std::max(1, std::min(units, resident));
  cfg.gridDim = dim3(2 * pairs);
  cfg.stream = st;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<BT, STAGES>, tw, tx, a));
}

// Token tile of the pair kernel for M tokens (0 = not worth it: the single-SM kernels win).
static int pair_bt(int M) { return M > 128 ? 256 : M > 64 ? 128 : 0; }

// C = A . W^T on SM pairs (no split-K).  bt: 128 or 256 (0 = by M).
static void gemm_pair_launch(const at::Tensor& A, const at::Tensor& W, at::Tensor& C,
                             const bf16* residual, int ldr, int64_t mode, at::Tensor& err, int BT,
                             cudaStream_t st) {
  const int M = A.size(0), K = A.size(1), N = W.size(0);
  GemmArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = (M + BT - 1) / BT;
  a.n_tiles = (N + BW - 1) / BW;
  a.splits = 1;
  a.kb_total = (K + BK - 1) / BK;
  a.kb_per_split = a.kb_total;
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.residual = residual;
  a.ldr = ldr;
  a.mode = static_cast<int>(mode);
  a.err = err.data_ptr<int>();
  a.vec_ok = (reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0) && (C.stride(0) % 4 == 0);
  const CUtensorMap tw = make_tmap_bf16_2d(W.data_ptr(), K, N, W.stride(0) * 2, BK, BW,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tx = make_tmap_bf16_2d(A.data_ptr(), K, M, A.stride(0) * 2, BK, BT / 2,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  if (BT == 256) launch_pair<256, 6>(tw, tx, a, st);
  else launch_pair<128, 8>(tw, tx, a, st);
}

// Test / benchmark entry: the SM-pair kernel regardless of the dispatch policy.
void gemm_bf16_pair(const at::Tensor& A, const at::Tensor& W, at::Tensor& C,
                    const c10::optional<at::Tensor>& residual, int64_t mode, at::Tensor& err,
                    int64_t bt) {
  TORCH_CHECK(A.is_cuda() && W.is_cuda() && C.is_cuda(), "gemm_pair: CUDA tensors");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16, "bf16 A, W");
  TORCH_CHECK(A.dim() == 2 && W.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 &&
                  W.stride(1) == 1 && C.stride(1) == 1, "gemm_pair: 2-D, inner stride 1");
  const int M = A.size(0), K = A.size(1), N = W.size(0);
  TORCH_CHECK(W.size(1) == K && K % 8 == 0, "gemm_pair: K");
  if (M == 0) return;
  if (mode == kEpiSwiGLU) {
    TORCH_CHECK(N % 128 == 0 && C.size(1) >= N / 2 && C.scalar_type() == at::kBFloat16, "swiglu");
  } else if (mode == kEpiF32) {
    TORCH_CHECK(C.scalar_type() == at::kFloat && C.size(1) >= N, "f32 out");
  } else {
    TORCH_CHECK(C.scalar_type() == at::kBFloat16 && C.size(1) >= N, "bf16 out");
  }
  TORCH_CHECK(C.size(0) >= M, "gemm_pair: C rows");
  const bf16* res = nullptr;
  int ldr = 0;
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(mode == kEpiStore && residual->scalar_type() == at::kBFloat16 &&
                    residual->stride(1) == 1, "residual");
    res = reinterpret_cast<const bf16*>(residual->data_ptr());
    ldr = residual->stride(0);
  }
  int BT = bt > 0 ? static_cast<int>(bt) : pair_bt(M);
  if (BT == 0) BT = 128;
  TORCH_CHECK(BT == 128 || BT == 256, "gemm_pair: token tile 128 or 256");
  gemm_pair_launch(A, W, C, res, ldr, mode, err, BT, at::cuda::getCurrentCUDAStream());
}

// `splits` value that selects stream-K in the persistent kernel.
constexpr int64_t kSplitsStreamK = 1000;

// Stream-K quantum: k-blocks per CTA so that ceil(total / q) CTAs (at most one per SM, all
// resident: finishers wait on contributors) share tiles x kb_total k-blocks evenly.
static int streamk_q(int tiles, int kb_total) {
  const long long tot = static_cast<long long>(tiles) * kb_total;
  const long long g = std::min<long long>(num_sms(), tot);
  return static_cast<int>((tot + g - 1) / g);
}

void gemm_bf16(const at::Tensor& A, const at::Tensor& W, at::Tensor& C,
               const c10::optional<at::Tensor>& residual, int64_t mode, at::Tensor& ws,
               at::Tensor& counters, at::Tensor& err, int64_t bt, int64_t splits,
               const c10::optional<at::Tensor>& trace) {
  TORCH_CHECK(A.is_cuda() && W.is_cuda() && C.is_cuda(), "gemm: tensors must be CUDA");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16,
              "gemm: A and W must be bf16");
  TORCH_CHECK(A.dim() == 2 && W.dim() == 2 && C.dim() == 2, "gemm: 2-D tensors expected");
  TORCH_CHECK(A.stride(1) == 1 && W.stride(1) == 1 && C.stride(1) == 1, "gemm: inner stride 1");
  const int M = A.size(0), K = A.size(1), N = W.size(0);
  TORCH_CHECK(W.size(1) == K, "gemm: K mismatch");
  TORCH_CHECK(K % 8 == 0, "gemm: K must be a multiple of 8 (16-byte TMA rows)");
  if (M == 0) return;
  if (mode == kEpiSwiGLU) {
    TORCH_CHECK(N % 128 == 0, "swiglu gemm: N must be a multiple of 128");
    TORCH_CHECK(C.size(1) >= N / 2 && C.size(0) >= M, "swiglu gemm: C too small");
    TORCH_CHECK(C.scalar_type() == at::kBFloat16, "swiglu gemm: bf16 out");
  } else if (mode == kEpiF32) {
    TORCH_CHECK(C.scalar_type() == at::kFloat && C.size(1) >= N && C.size(0) >= M, "f32 out");
  } else {
    TORCH_CHECK(C.scalar_type() == at::kBFloat16 && C.size(1) >= N && C.size(0) >= M, "bf16 out");
  }
  // Stream-K pays one fp32 partial per CTA; it wins only when every CTA covers many tiles and
  // the data-parallel tail wave would idle (measured: 2048 x 28672 x 4096, 488 -> 438 us; at
  // 3.5 tiles per CTA and below the per-thread fixup costs more than the wave it saves).
  bool stream_k = splits == kSplitsStreamK;
  if (splits == 0) {
    const int BTp = bt > 0 ? static_cast<int>(bt) : pick_bt_shape(M, N, K);
    const int tl = ((M + BTp - 1) / BTp) * ((N + BW - 1) / BW);
    const int kbt = (K + BK - 1) / BK;
    const int sms = num_sms();
    const double waves = static_cast<double>(tl) / sms;
    const double eff = waves / std::ceil(waves);
    stream_k = tl >= 8 * sms && eff < 0.95 &&
               ws.numel() >= static_cast<int64_t>(sms) * BTp * BW && counters.numel() >= sms &&
               kbt >= 4;
  }
  auto plan = gemm_plan(M, N, K, bt, stream_k ? 1 : splits);
  const int BT = plan[0];
  int sp = plan[1];
  const int tiles = plan[2];
  if (sp > 1 && (ws.numel() < plan[3] || counters.numel() < tiles)) sp = 1;
  TORCH_CHECK(sp > 0 || ws.numel() >= plan[3], "gemm: cluster split-K workspace too small (",
              ws.numel(), " < ", plan[3], " floats)");
  const int kb_total = (K + BK - 1) / BK;
  const int S = sp < 0 ? -sp : 1;
  const int nsplit = sp < 0 ? S : sp;
  const int kbps = (kb_total + nsplit - 1) / nsplit;

  GemmArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = (M + BT - 1) / BT;
  a.n_tiles = (N + BW - 1) / BW;
  a.splits = sp > 0 ? sp : 1;
  a.kb_per_split = kbps;
  a.kb_total = kb_total;
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.residual = nullptr;
  a.ldr = 0;
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(mode == kEpiStore, "residual only with bf16 store");
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1, "residual");
    a.residual = reinterpret_cast<const bf16*>(residual->data_ptr());
    a.ldr = residual->stride(0);
  }
  a.ws = (sp > 1 || sp < -1) ? ws.data_ptr<float>() : nullptr;
  a.counters = sp > 1 ? counters.data_ptr<int>() : nullptr;
  a.mode = mode;
  a.err = err.data_ptr<int>();
  a.vec_ok = (reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0) && (C.stride(0) % 4 == 0);
  TORCH_CHECK(mode != kEpiSwiGLU || a.vec_ok, "swiglu gemm: C must be 16-byte aligned, ldc % 4 == 0");
  a.trace = nullptr;
  if (trace.has_value() && trace->defined()) {
    a.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }

  const CUtensorMap tw = make_tmap_bf16_2d(W.data_ptr(), K, N, W.stride(0) * 2, BK, BW,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tx = make_tmap_bf16_2d(A.data_ptr(), K, M, A.stride(0) * 2, BK, BT,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (sp < 0) {
    CUtensorMap tc;
    std::memset(&tc, 0, sizeof(tc));
    a.tma_out = make_tmap_out(C, mode, M, N, crs::out_box_rows(BT, S), &tc) ? 1 : 0;
    switch (BT) {
      case 16: launch_cluster<16, 8>(tw, tx, tc, a, S, st); break;
      case 32: launch_cluster<32, 8>(tw, tx, tc, a, S, st); break;
      case 64: launch_cluster<64, 8>(tw, tx, tc, a, S, st); break;
      case 128: launch_cluster<128, 6>(tw, tx, tc, a, S, st); break;
      case 256: launch_cluster<256, 4>(tw, tx, tc, a, S, st); break;
      default: TORCH_CHECK(false, "gemm: unsupported token tile ", BT);
    }
    return;
  }
  const int units = a.m_tiles * a.n_tiles * a.splits;
  int grid = std::min(units, num_sms());
  if (stream_k) {
    const int q = streamk_q(tiles, kb_total);
    grid = static_cast<int>((static_cast<long long>(tiles) * kb_total + q - 1) / q);
    TORCH_CHECK(ws.numel() >= static_cast<int64_t>(grid) * BT * BW && counters.numel() >= grid,
                "gemm: stream-K workspace too small");
    a.sk_q = q;
    a.ws = ws.data_ptr<float>();
    a.counters = counters.data_ptr<int>();
  }
  switch (BT) {
    case 16: launch_bt<16, 8>(tw, tx, a, grid, st); break;
    case 32: launch_bt<32, 8>(tw, tx, a, grid, st); break;
    case 64: launch_bt<64, 8>(tw, tx, a, grid, st); break;
    case 128: launch_bt<128, 6>(tw, tx, a, grid, st); break;
    case 256: launch_bt<256, 4>(tw, tx, a, grid, st); break;
    default: TORCH_CHECK(false, "gemm: unsupported token tile ", BT);
  }
}

}  // namespace lb

namespace lb {
// Tensor-parallel GEMM (decode shapes): cluster split-K kernel with a consumer wait on the
// gathered-input flag and/or a scatter epilogue into the owners' reduce-scatter slots.
// Pointers to peer memory come from CUDA IPC handles opened by the caller.
void gemm_bf16_tp(const at::Tensor& A, const at::Tensor& W, at::Tensor& C, int64_t mode,
                  at::Tensor& err, int64_t splits, std::vector<int64_t> scatter_ptrs,
                  std::vector<int64_t> signal_ptrs, int64_t rows_per_rank, int64_t src_rank,
                  int64_t slot_stride, int64_t wait_flag_ptr, int64_t wait_count,
                  int64_t done_counter_ptr, int64_t trace_ptr,
                  const c10::optional<at::Tensor>& ws) {
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16, "bf16");
  TORCH_CHECK(A.stride(1) == 1 && W.stride(1) == 1 && C.stride(1) == 1, "inner stride 1");
  const int M = A.size(0), K = A.size(1), N = W.size(0);
  TORCH_CHECK(W.size(1) == K && K % 8 == 0, "gemm_tp: K");
  TORCH_CHECK(scatter_ptrs.size() <= 8 && signal_ptrs.size() <= 8, "gemm_tp: world <= 8");
  TORCH_CHECK(mode != kEpiF32 || scatter_ptrs.empty(), "gemm_tp: scatter is bf16 only");
  if (M == 0) return;
  const int BT = pick_bt(M);
  const int m_tiles = (M + BT - 1) / BT, n_tiles = (N + BW - 1) / BW;
  const int kb_total = (K + BK - 1) / BK;
  int S = splits > 0 ? static_cast<int>(splits) : pick_cluster(BT, m_tiles * n_tiles, kb_total);
  S = std::max(1, std::min(S, std::min(8, kb_total)));
  while (S > 1 && !cluster_fits(BT, S)) --S;
  const bool have_ws = ws.has_value() && ws->defined();
  while (S > 1 && (!have_ws || ws->numel() < crs::ws_floats(m_tiles * n_tiles, BT, S))) --S;
  GemmArgs a = {};
  a.ws = S > 1 ? ws->data_ptr<float>() : nullptr;
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = m_tiles;
  a.n_tiles = n_tiles;
  a.splits = 1;
  a.kb_per_split = (kb_total + S - 1) / S;
  a.kb_total = kb_total;
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.mode = mode;
  a.err = err.data_ptr<int>();
  a.vec_ok = (reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0) && (C.stride(0) % 4 == 0);
  a.tp.world = static_cast<int>(scatter_ptrs.size());
  for (size_t i = 0; i < scatter_ptrs.size(); ++i)
    a.tp.scatter[i] = reinterpret_cast<bf16*>(scatter_ptrs[i]);
  for (size_t i = 0; i < signal_ptrs.size(); ++i)
    a.tp.signal[i] = reinterpret_cast<int*>(signal_ptrs[i]);
  if (a.tp.world > 0) {
    TORCH_CHECK(signal_ptrs.size() == scatter_ptrs.size(), "gemm_tp: one flag per owner");
    TORCH_CHECK(a.vec_ok, "gemm_tp: scatter needs 16-byte aligned rows");
  }
  a.tp.rows_per_rank = static_cast<int>(rows_per_rank);
  a.tp.src_rank = static_cast<int>(src_rank);
  a.tp.slot_stride = slot_stride;
  a.tp.wait_flag = reinterpret_cast<int*>(wait_flag_ptr);
  a.tp.wait_count = static_cast<int>(wait_count);
  a.tp.done_counter = reinterpret_cast<int*>(done_counter_ptr);
  a.trace = reinterpret_cast<unsigned long long*>(trace_ptr);
  TORCH_CHECK(a.tp.done_counter != nullptr, "gemm_tp: needs a completion counter");
  const CUtensorMap tw = make_tmap_bf16_2d(W.data_ptr(), K, N, W.stride(0) * 2, BK, BW,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tx = make_tmap_bf16_2d(A.data_ptr(), K, M, A.stride(0) * 2, BK, BT,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  // Local output (consumer GEMM): TMA-store epilogue; scatter into peers: per-thread P2P stores.
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  a.tma_out =
      (a.tp.world == 0 && make_tmap_out(C, mode, M, N, crs::out_box_rows(BT, S), &tc)) ? 1 : 0;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  switch (BT) {
    case 16: launch_cluster<16, 8>(tw, tx, tc, a, S, st); break;
    case 32: launch_cluster<32, 8>(tw, tx, tc, a, S, st); break;
    case 64: launch_cluster<64, 8>(tw, tx, tc, a, S, st); break;
    case 128: launch_cluster<128, 6>(tw, tx, tc, a, S, st); break;
    default: launch_cluster<256, 4>(tw, tx, tc, a, S, st); break;
  }
}

// Row-parallel GEMM of a tensor-parallel layer (o_proj / down_proj) whose epilogue pushes every
// output row straight into its owner's receive slot of the row-parallel exchange (tp_rowpar.cu):
// recv1_ptrs[j] = rank j's recv1 base (parity 0), slots of rp_max rows x N columns, rows owned in
// ranges of ceil(M / world).  The exchange's rowpar_norm (partial = None) consumes them.
void gemm_bf16_rowpar(const at::Tensor& A, const at::Tensor& W, at::Tensor& err,
                      std::vector<int64_t> recv1_ptrs, int64_t rank, int64_t rp_max,
                      int64_t epoch_ptr, const c10::optional<at::Tensor>& ws, int64_t splits,
                      int64_t trace_ptr) {
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16, "bf16");
  TORCH_CHECK(A.stride(1) == 1 && W.stride(1) == 1, "inner stride 1");
  const int M = A.size(0), K = A.size(1), N = W.size(0);
  const int world = static_cast<int>(recv1_ptrs.size());
  TORCH_CHECK(W.size(1) == K && K % 8 == 0, "gemm_rowpar: K");
  TORCH_CHECK(world >= 2 && world <= 8 && rank >= 0 && rank < world, "gemm_rowpar: world");
  TORCH_CHECK(N % 8 == 0, "gemm_rowpar: N % 8 == 0 (16-byte rows)");
  const int rp = (M + world - 1) / world;
  TORCH_CHECK(rp <= rp_max, "gemm_rowpar: tokens exceed the exchange capacity");
  TORCH_CHECK(epoch_ptr != 0, "gemm_rowpar: epoch pointer");
  if (M == 0) return;
  for (int64_t p : recv1_ptrs) TORCH_CHECK(p % 16 == 0, "gemm_rowpar: 16-byte aligned slots");
  const int BT = pick_bt(M);
  const int m_tiles = (M + BT - 1) / BT, n_tiles = (N + BW - 1) / BW;
  const int kb_total = (K + BK - 1) / BK;
  int S = splits > 0 ? static_cast<int>(splits) : pick_cluster(BT, m_tiles * n_tiles, kb_total);
  S = std::max(1, std::min(S, std::min(8, kb_total)));
  while (S > 1 && !cluster_fits(BT, S)) --S;
  const bool have_ws = ws.has_value() && ws->defined();
  while (S > 1 && (!have_ws || ws->numel() < crs::ws_floats(m_tiles * n_tiles, BT, S))) --S;
  GemmArgs a = {};
  a.ws = S > 1 ? ws->data_ptr<float>() : nullptr;
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = m_tiles;
  a.n_tiles = n_tiles;
  a.splits = 1;
  a.kb_per_split = (kb_total + S - 1) / S;
  a.kb_total = kb_total;
  a.C = reinterpret_cast<void*>(recv1_ptrs[rank]);
  a.ldc = N;
  a.mode = kEpiStore;
  a.err = err.data_ptr<int>();
  a.vec_ok = 1;
  a.tp.world = world;
  for (int i = 0; i < world; ++i) a.tp.scatter[i] = reinterpret_cast<bf16*>(recv1_ptrs[i]);
  a.tp.rows_per_rank = rp;
  a.tp.src_rank = static_cast<int>(rank);
  a.tp.slot_stride = rp_max * static_cast<long long>(N);
  a.tp.push = comm_fence_mode() != 0 ? 2 : 1;   // 2: with the optional slot-reuse fence
  a.tp.epoch = reinterpret_cast<const int*>(epoch_ptr);
  a.tma_out = 0;
  a.trace = reinterpret_cast<unsigned long long*>(trace_ptr);
  const CUtensorMap tw = make_tmap_bf16_2d(W.data_ptr(), K, N, W.stride(0) * 2, BK, BW,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tx = make_tmap_bf16_2d(A.data_ptr(), K, M, A.stride(0) * 2, BK, BT,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  switch (BT) {
    case 16: launch_cluster<16, 8>(tw, tx, tc, a, S, st); break;
    case 32: launch_cluster<32, 8>(tw, tx, tc, a, S, st); break;
    case 64: launch_cluster<64, 8>(tw, tx, tc, a, S, st); break;
    case 128: launch_cluster<128, 6>(tw, tx, tc, a, S, st); break;
    default: launch_cluster<256, 4>(tw, tx, tc, a, S, st); break;
  }
}

}  // namespace lb

// ======================================================================================
// No-allocation entry point (declared in gemm_noalloc.h; no counterpart in the reference).
// The persistent split-K kernel above, with its workspace, tile counters and error word in
// one file-scope device array instead of caller- or allocator-provided memory.
// ======================================================================================
#include <cstdio>

#include "gemm_noalloc.h"

namespace {
constexpr size_t kNaCounterWords = 16384;                    // per-tile arrival counters
constexpr size_t kNaErrWords = 64;                           // error word (+ padding)
constexpr size_t kNaHeadBytes = (kNaCounterWords + kNaErrWords) * sizeof(int);
constexpr size_t kNaWsFloats = size_t(4) << 20;              // 16 MiB of fp32 partial tiles
constexpr size_t kNaScratchBytes = kNaHeadBytes + kNaWsFloats * sizeof(float);
constexpr int kNaMaxDevices = 64;
}  // namespace

// Shared by every call on a device; zero-initialised when the module loads.
static __device__ __align__(256) unsigned char lb_gemm_noalloc_scratch[kNaScratchBytes];

namespace {
std::mutex na_mu;
void* na_ptr[kNaMaxDevices] = {nullptr};

template <int BT, int STAGES>
cudaError_t na_launch(const CUtensorMap& tw, const CUtensorMap& tx, const lb::GemmArgs& a,
                      int grid, cudaStream_t st) {
  using L = lb::GemmSmem<BT, STAGES>;
  lb::gemm_tc_kernel<BT, STAGES><<<grid, lb::kThreads, L::TOTAL, st>>>(tw, tx, a);
  return cudaGetLastError();
}

template <int BT, int STAGES>
cudaError_t na_set_attr() {
  using L = lb::GemmSmem<BT, STAGES>;
  return cudaFuncSetAttribute(lb::gemm_tc_kernel<BT, STAGES>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
}

int na_fail(int code, const char* msg, cudaError_t e = cudaSuccess) {
  if (e != cudaSuccess)
    std::fprintf(stderr, "lb_gemm_bf16_noalloc: %s: %s\n", msg, cudaGetErrorString(e));
  else
    std::fprintf(stderr, "lb_gemm_bf16_noalloc: %s\n", msg);
  return code;
}
}  // namespace

extern "C" int lb_gemm_bf16_noalloc(const void* A, int lda, const void* W, int ldw, void* C,
                                    int ldc, int M, int N, int K, int splits,
                                    cudaStream_t stream) {
  using namespace lb;
  if (!A || !W || !C || M <= 0 || N <= 0 || K <= 0 || splits < 1)
    return na_fail(LB_NOALLOC_BAD_ARGS, "null pointer, non-positive size or splits < 1");
  if (K % 8 != 0 || lda < K || ldw < K || ldc < N || (lda % 8) || (ldw % 8) ||
      reinterpret_cast<uintptr_t>(A) % 16 || reinterpret_cast<uintptr_t>(W) % 16)
    return na_fail(LB_NOALLOC_BAD_ARGS,
                   "K, lda, ldw must be multiples of 8 elements and A, W 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "cudaGetDevice", e);
  if (dev < 0 || dev >= kNaMaxDevices) return na_fail(LB_NOALLOC_BAD_ARGS, "device ordinal");

  // One-time set-up per device (with that device current): scratch address + smem attribute.
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> g(na_mu);
    if (na_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, lb_gemm_noalloc_scratch);
      if (e != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "cudaGetSymbolAddress", e);
      cudaError_t e2 = na_set_attr<16, 8>();
      if (e2 == cudaSuccess) e2 = na_set_attr<32, 8>();
      if (e2 == cudaSuccess) e2 = na_set_attr<64, 8>();
      if (e2 == cudaSuccess) e2 = na_set_attr<128, 6>();
      if (e2 == cudaSuccess) e2 = na_set_attr<256, 4>();
      if (e2 != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "cudaFuncSetAttribute", e2);
      na_ptr[dev] = p;
    }
    base = na_ptr[dev];
  }

  const int BT = pick_bt(M);
  const int m_tiles = (M + BT - 1) / BT;
  const int n_tiles = (N + BW - 1) / BW;
  const int kb_total = (K + BK - 1) / BK;
  int sp = std::min(splits, kb_total);
  const int kbps = (kb_total + sp - 1) / sp;
  sp = (kb_total + kbps - 1) / kbps;
  const size_t tiles = static_cast<size_t>(m_tiles) * n_tiles;
  const size_t need = sp > 1 ? tiles * sp * BT * BW : 0;
  if (need > kNaWsFloats || (sp > 1 && tiles > kNaCounterWords)) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "M=%d N=%d K=%d splits=%d needs %zu partial floats / %zu tiles; the static "
                  "scratch holds %zu floats / %zu tiles",
                  M, N, K, splits, need, tiles, kNaWsFloats, kNaCounterWords);
    return na_fail(LB_NOALLOC_TOO_LARGE, msg);
  }

  int* counters = reinterpret_cast<int*>(base);
  int* err = counters + kNaCounterWords;
  float* ws = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + kNaHeadBytes);
  // Counters and the error word must start at zero: clear what this call uses.
  e = cudaMemsetAsync(base, 0, kNaHeadBytes, stream);
  if (e != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "cudaMemsetAsync", e);

  GemmArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = m_tiles;
  a.n_tiles = n_tiles;
  a.splits = sp;
  a.kb_per_split = kbps;
  a.kb_total = kb_total;
  a.C = C;
  a.ldc = ldc;
  a.residual = nullptr;
  a.ldr = 0;
  a.ws = sp > 1 ? ws : nullptr;
  a.counters = sp > 1 ? counters : nullptr;
  a.mode = kEpiStore;
  a.err = err;
  a.trace = nullptr;
  a.vec_ok = (reinterpret_cast<uintptr_t>(C) % 16 == 0) && (ldc % 4 == 0);

  CUtensorMap tw, tx;
  {
    cuuint64_t dw[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
    cuuint64_t sw[1] = {static_cast<cuuint64_t>(ldw) * 2};
    cuuint32_t bw[2] = {BK, BW};
    cuuint64_t dx[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    cuuint64_t sx[1] = {static_cast<cuuint64_t>(lda) * 2};
    cuuint32_t bx[2] = {BK, static_cast<cuuint32_t>(BT)};
    cuuint32_t es[2] = {1, 1};
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    cudaDriverEntryPointQueryResult q;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&enc),
                                cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || enc == nullptr)
      return na_fail(LB_NOALLOC_CUDA_ERROR, "cuTensorMapEncodeTiled unavailable", e);
    CUresult r1 = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(W), dw, sw, bw,
                      es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = enc(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(A), dx, sx, bx,
                      es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
      return na_fail(LB_NOALLOC_CUDA_ERROR, "cuTensorMapEncodeTiled failed");
  }
  int nsm = 0;
  e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "cudaDeviceGetAttribute", e);
  const int units = m_tiles * n_tiles * sp;
  const int grid = std::min(units, nsm);
  switch (BT) {
    case 16: e = na_launch<16, 8>(tw, tx, a, grid, stream); break;
    case 32: e = na_launch<32, 8>(tw, tx, a, grid, stream); break;
    case 64: e = na_launch<64, 8>(tw, tx, a, grid, stream); break;
    case 128: e = na_launch<128, 6>(tw, tx, a, grid, stream); break;
    default: e = na_launch<256, 4>(tw, tx, a, grid, stream); break;
  }
  if (e != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "kernel launch", e);
  return LB_NOALLOC_OK;
}

extern "C" int lb_gemm_bf16_noalloc_status(int* kernel_error, cudaStream_t stream) {
  if (!kernel_error) return na_fail(LB_NOALLOC_BAD_ARGS, "status: null kernel_error");
  *kernel_error = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "status: cudaGetDevice", e);
  if (dev < 0 || dev >= kNaMaxDevices) return na_fail(LB_NOALLOC_BAD_ARGS, "device ordinal");
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> g(na_mu);
    base = na_ptr[dev];
  }
  if (base == nullptr) return LB_NOALLOC_OK;  // no GEMM has run on this device yet
  // The error word sits right after the tile counters; read it behind the caller's work on
  // `stream` (a pageable destination makes the copy complete before cudaMemcpyAsync returns
  // on some paths, so the stream is synchronised explicitly either way).
  const int* err = reinterpret_cast<const int*>(base) + kNaCounterWords;
  e = cudaMemcpyAsync(kernel_error, err, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return na_fail(LB_NOALLOC_CUDA_ERROR, "status: read error word", e);
  return LB_NOALLOC_OK;
}
