// Weight-quantized GEMM on tcgen05 with dequantization fused into the producer (sm_100a).
//
//   C[M, N] = X[M, K] (bf16) . dequant(Wq)[N, K]^T,   dequant: w = q * s[g] - o[g]
//
// One kernel serves every quantized checkpoint format, after an offline repack
// (lightbulb_b200/formats/quant.py) to packed integers + per-group fp16 (scale, offset):
//   * AWQ int4 (reference src/loaders/awq.rs:162-183 -> Marlin FFI, absent):  q 0..15,
//     s = scale, o = zero * scale, group 128;
//   * GGUF Q4_K (reference QMatMul, src/model/quantizable_linear.rs:63-69):   q 0..15,
//     s = d * sc_j, o = dmin * m_j per 32-element sub-block;
//   * GGUF Q8_0: signed int8 q, s = d, o = 0, group 32.
//
// Pipeline (per CTA = one 128-row weight tile x BT tokens x one K split of a cluster):
//   warp 0      TMA: packed weight tile [128 rows x 64*QBITS/8 bytes] + activation tile
//   warps 2..5  dequant: each thread expands one weight row (64 values) into bf16 directly in
//               the 128-byte-swizzled K-major layout the MMA reads, fence.proxy.async,
//               then signals `ready`; after the main loop the same warps run the epilogue
//   warp 1      one thread issues tcgen05.mma (kind::f16, bf16 x bf16 -> fp32 in TMEM)
// Split-K partial tiles are reduced through distributed shared memory across the cluster
// (fixed rank order), exactly as in the bf16 cluster GEMM.  No multicast.
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <cstdlib>
#include <string>

#include "cluster_rs.cuh"
#include "common.cuh"

namespace lb {

namespace q {

constexpr int BW = 128, BK = 64, UK = 16, THREADS = 192;

struct Args {
  int M, N, K, m_tiles, n_tiles, kb_per_split, kb_total;
  const __half* scales;   // [N, K / group]
  const __half* offsets;  // [N, K / group]
  int group;
  void* C;
  int ldc;
  int mode;  // 0 bf16, 1 swiglu, 2 fp32
  int vec_ok;
  int* err;
  float* ws;  // split-K exchange workspace (cluster_rs.cuh)
};

template <int BT, int STAGES, int QBITS>
struct Smem {
  static constexpr int W_BYTES = BW * BK * 2;             // dequantized bf16 operand
  static constexpr int Q_BYTES = BW * BK * QBITS / 8;     // packed staging
  static constexpr int X_BYTES = BT * BK * 2;
  static constexpr int STAGE = W_BYTES + Q_BYTES + X_BYTES;
  static constexpr int CH = BT < 32 ? BT : 32;
  static constexpr int BAR_OFF = STAGES * STAGE;
  static constexpr int TOTAL = BAR_OFF + 512 + 1024;
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

template <int BT, int STAGES, int QBITS>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmC, const Args a) {
  using L = Smem<BT, STAGES, QBITS>;
  constexpr int CH = L::CH;
  constexpr int TMEM_COLS = BT < 32 ? 32 : BT;
  static_assert(crs::smem_bytes(BT, 1) <= STAGES * L::STAGE &&
                    crs::smem_bytes(BT, 8) <= STAGES * L::STAGE,
                "split-K slots");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  // stage s: [W bf16 16 KB | X BT*128 | Q staging]; W and X stay 1024-aligned
  auto sW = [&](int s) { return smem + s * L::STAGE; };
  auto sX = [&](int s) { return smem + s * L::STAGE + L::W_BYTES; };
  auto sQ = [&](int s) { return smem + s * L::STAGE + L::W_BYTES + L::X_BYTES; };
  float* sSlots = reinterpret_cast<float*>(smem);  // after the main loop: split-K slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* ready = bars + STAGES;
  uint64_t* empty = bars + 2 * STAGES;
  uint64_t* tfull = bars + 3 * STAGES;
  uint64_t* rbar = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_go = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t S = crs::nctarank(), rank = crs::ctarank();
  const int tile = blockIdx.x / S;
  const int mt = tile % a.m_tiles, nt = tile / a.m_tiles;
  float* ws_tile = a.ws + crs::ws_floats(tile, BT, S);
  const int kb0 = rank * a.kb_per_split;
  const int kb1 = min(kb0 + a.kb_per_split, a.kb_total);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(rbar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
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

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pw = policy_evict_first(), px = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          record_error(a.err, kErrTimeoutSmemEmpty);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], L::Q_BYTES + L::X_BYTES);
        tma_load_2d(sQ(stage), &tmQ, &full[stage], kb * BK * QBITS / 8, nt * BW, pw);
        tma_load_2d(sX(stage), &tmX, &full[stage], kb * BK, mt * BT, px);
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
        if (!mbar_wait(&ready[stage], phase, abort_flag)) {
          record_error(a.err, kErrTimeoutTmaFull);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t wb = smem_u32(sW(stage)), xb = smem_u32(sX(stage));
#pragma unroll
        for (int k = 0; k < BK / UK; ++k)
          tc_mma_f16(tmem_base, sw128_kmajor_desc(wb + k * UK * 2), sw128_kmajor_desc(xb + k * UK * 2),
                     idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        tc_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) tc_commit(tfull);
    }
  } else {
    // ---- dequant warps (one weight row per thread) ----
    const int row = threadIdx.x - 64;  // 0..127 (row of the weight tile)
    const int n = nt * BW + row;
    const int gpr = a.K / a.group;     // groups per weight row
    int stage = 0;
    uint32_t phase = 0;
    // Scale / offset of the (at most two) groups a 64-wide k-block touches, prefetched one
    // k-block ahead so the global-load latency overlaps the wait and the previous dequant.
    const __half* srow = a.scales + static_cast<size_t>(n < a.N ? n : 0) * gpr;
    const __half* orow = a.offsets + static_cast<size_t>(n < a.N ? n : 0) * gpr;
    // Dequantisation without int->float conversions (magic-number method): a value q held
    // in the low mantissa bits of bf16 128.0 (0x4300 | q) or fp32 2^23 (0x4B000000 | b)
    // reads as 128 + q or 2^23 + b exactly; widening bf16 -> fp32 is a shift.  4-bit: one
    // FMA with the offset pre-folded as o + 128 s (128 s is exact; the fold's rounding is
    // ~1e-5 s, far below bf16 output precision).  8-bit: 2^23 + 128 is subtracted first
    // (exact), since folding 2^23 s into the offset would cost half a quantisation step.
    //  4-bit words (repacked offline): bits [4i, 4i+4) = element 2i, bits [16+4i, 20+4i) =
    //  element 2i+1, so (w >> 4i) & 0x000F000F | 0x43004300 is the bf16 pair (2i, 2i+1).
    //  8-bit bytes are stored biased (q + 128).
    auto fetch = [&](int kb, float& s0, float& o0, float& s1, float& o1) {
      const int g0 = (kb * BK) / a.group, g1 = (kb * BK + 32) / a.group;
      s0 = __half2float(__ldg(srow + g0));
      o0 = __half2float(__ldg(orow + g0));
      s1 = __half2float(__ldg(srow + g1));
      o1 = __half2float(__ldg(orow + g1));
      if constexpr (QBITS == 4) {
        o0 += 128.f * s0;
        o1 += 128.f * s1;
      }
    };
    float ns0 = 0.f, no0 = 0.f, ns1 = 0.f, no1 = 0.f;
    if (kb0 < kb1) fetch(kb0, ns0, no0, ns1, no1);
    for (int kb = kb0; kb < kb1; ++kb) {
      const float cs0 = ns0, co0 = no0, cs1 = ns1, co1 = no1;
      if (kb + 1 < kb1) fetch(kb + 1, ns0, no0, ns1, no1);
      int go = 1;
      if (!mbar_wait(&full[stage], phase, abort_flag)) {
        record_error(a.err, kErrTimeoutTmaFull);
        *abort_flag = 1;
        go = 0;
      }
      go = __all_sync(0xffffffffu, go);
      if (!go) break;
      uint8_t* wdst = sW(stage) + row * 128;
      if constexpr (QBITS == 4) {
        const uint4* src = reinterpret_cast<const uint4*>(sQ(stage) + row * 32);
        const uint4 p0 = src[0], p1 = src[1];
        const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // word c = elements 8c .. 8c+7 = output chunk c
          const float sc = c < 4 ? cs0 : cs1, of = c < 4 ? co0 : co1;
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t t = ((w[c] >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
            const float lo = __uint_as_float(t << 16), hi = __uint_as_float(t & 0xFFFF0000u);
            o[i] = pack_bf16x2(fmaf(lo, sc, -of), fmaf(hi, sc, -of));
          }
          *reinterpret_cast<uint4*>(wdst + ((c ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(sQ(stage) + row * 64);
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 8 bytes = elements 8c .. 8c+7
          const uint4 p = src[c >> 1];
          const uint32_t w0 = (c & 1) ? p.z : p.x, w1 = (c & 1) ? p.w : p.y;
          const float sc = c < 4 ? cs0 : cs1, of = c < 4 ? co0 : co1;
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t ww = i < 2 ? w0 : w1;
            const int b = (i & 1) * 2;
            const float x0 = __uint_as_float(__byte_perm(ww, 0x4B000000u, 0x7650 + b)) - 8388736.f;
            const float x1 =
                __uint_as_float(__byte_perm(ww, 0x4B000000u, 0x7650 + b + 1)) - 8388736.f;
            o[i] = pack_bf16x2(fmaf(x0, sc, -of), fmaf(x1, sc, -of));
          }
          *reinterpret_cast<uint4*>(wdst + ((c ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      // generic-proxy smem writes -> visible to the tensor core (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      named_bar_sync(1, 128);
      if (row == 0) mbar_arrive(&ready[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // ---- accumulator ready: publish the partial tile ----
    if (row == 0) {
      int gg = 1;
      if (kb1 <= kb0) gg = 2;
      else if (*abort_flag || !mbar_wait(tfull, 0, abort_flag)) {
        record_error(a.err, kErrTimeoutTmemFull);
        *abort_flag = 1;
        gg = 0;
      }
      s_go[0] = gg;
    }
    named_bar_sync(1, 128);
    tc_fence_after();
    const int quad = warp & 3;
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    crs::publish<BT>(tbase, s_go[0] == 1, sSlots, ws_tile, rank, S, quad * 32 + lane, row);
  }

  tc_fence_before();
  crs::sync_all();  // every partial of the cluster is in L2 / its owner's shared memory
  tc_fence_after();
  if (warp >= 2) {
    const int e = threadIdx.x - 64;
    if (e == 0) crs::fetch<BT>(sSlots, ws_tile, rbar, rank, S);
    const int m0 = mt * BT;
    const int x0 = a.mode == 1 ? nt * 64 : nt * BW;
    auto epi = [&](int oc, int t0, int l, float4 (&acc)[crs::CW]) {
      uint8_t* tile = crs::out_tile(sSlots, 0, oc);
      crs::stage_out(a.mode, tile, l, acc, nullptr, 0, 0, 0);
      crs::store_chunk(&tmC, tile, l, x0, m0 + t0);
    };
    const bool ok = crs::reduce<BT>(sSlots, rbar, rank, S, e, abort_flag, epi);
    crs::store_wait(e & 31, false);
    if (!ok) {
      record_error(a.err, kErrTimeoutTmaFull);
      *abort_flag = 1;
      if (e == 0 && !mbar_wait(rbar, 0, nullptr, kWaitBudgetNs)) record_error(a.err, kErrTimeoutDrain);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace q

// ---------------------------------------------------------------------------------------------
// Small-batch path for integer-zero 4-bit weights (AWQ: w = (q - z) * s, group >= 64), M <= 32.
//
// At decode batch sizes the full-dequant kernel above is bound by the dequant instructions and
// by shared memory: every 4 KB packed k-block becomes 16 KB of bf16 written to and read back
// from shared memory, more than the SM's shared-memory bandwidth at HBM rate.  This kernel keeps
// the weights exact integers and moves the scale out of the inner loop:
//
//   y[t, n] = sum_g s[n, g] * sum_{k in g} x[t, k] * (q[n, k] - z[n, g])
//
//   * converter warps turn each packed word into bf16 pairs (128 + q) with one mask-or, subtract
//     (128 + z) with one bf16x2 subtract (exact: small integers), and store the row straight into
//     TENSOR memory with tcgen05.st -- the MMA reads its A operand (the weight tile) from TMEM, so
//     the expanded tile never touches shared memory;
//   * one thread issues tcgen05.mma (A from TMEM, the activation tile from shared memory) into
//     one of two per-group accumulators in TMEM;
//   * the same converter warps, one group behind, read a finished group accumulator (tcgen05.ld),
//     scale it by s[n, g] in fp32 and add it to the running sum in registers, then free it.
// The running sums go back to TMEM once, and the split-K exchange over the cluster (no
// multicast) and the output epilogue are those of the kernel above.
//
// Warps: 0 TMA producer, 1 MMA issuer (+ TMEM owner), 2..9 converters: warp w handles TMEM lane
// quarter (w & 3) and half (w - 2) >> 2 of each k-block's 64 columns / of the token columns.
namespace qs {

constexpr int BW = 128, BK = 64, THREADS = 320, NCONV = 8;
constexpr int TMEM_COLS = 256, ACOL = 64;  // [0, 2 BT): group accumulators; [64, 256): A stages

struct Args {
  int M, N, K, n_tiles, kb_per_split, kb_total, kpg;
  const __half* scales;   // [N, K / group]
  const __half* offsets;  // [N, K / group] = z * s
  int gpr;                // groups per weight row
  int mode;               // 0 bf16, 1 swiglu, 2 fp32
  int* err;
  float* ws;
};

// HK: 64-element halves per k-block (1 or 2).  With HK = 2 every TMA row request of the packed
// tile moves 64 bytes instead of 32.
template <int BT, int STAGES, int HK>
struct Smem {
  static constexpr int X_HALF = BT * BK * 2;        // one 64-column SW128 activation tile
  static constexpr int X_BYTES = HK * X_HALF;       // 1024-aligned (BT = 16 / 32)
  static constexpr int Q_BYTES = BW * BK * HK / 2;  // packed 4-bit tile
  static constexpr int STAGE = X_BYTES + Q_BYTES;
  static constexpr int PIPE = STAGES * STAGE;
  static constexpr int SLOTS = crs::smem_bytes(BT, 8);
  static constexpr int DATA = PIPE > SLOTS ? PIPE : SLOTS;
  static constexpr int BAR_OFF = DATA;
  static constexpr int TOTAL = BAR_OFF + 512 + 1024;
};

__device__ __forceinline__ uint32_t sub_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

template <int BT, int STAGES, int HK>
__global__ void __launch_bounds__(THREADS, 2)
    gemm_qs_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ CUtensorMap tmC, const Args a) {
  using L = Smem<BT, STAGES, HK>;
  constexpr int AW = 32 * HK;  // TMEM columns of one weight stage (2 bf16 per column)
  constexpr int HC = BT / 2;  // token columns per converter half
  static_assert(ACOL >= 2 * BT && ACOL + STAGES * AW <= TMEM_COLS, "TMEM plan");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  auto sX = [&](int s) { return smem + s * L::STAGE; };
  auto sQ = [&](int s) { return smem + s * L::STAGE + L::X_BYTES; };
  float* sSlots = reinterpret_cast<float*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* ready = bars + STAGES;
  uint64_t* empty = bars + 2 * STAGES;
  uint64_t* gfull = bars + 3 * STAGES;  // [2]
  uint64_t* gempty = gfull + 2;         // [2]
  uint64_t* rbar = gempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_go = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t S = crs::nctarank(), rank = crs::ctarank();
  const int nt = blockIdx.x / S;
  float* ws_tile = a.ws + crs::ws_floats(nt, BT, S);
  const int kb0 = rank * a.kb_per_split;
  const int kb1 = min(kb0 + a.kb_per_split, a.kb_total);
  const int ngroups = kb1 > kb0 ? (kb1 - kb0) / a.kpg : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], NCONV);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&gfull[b], 1);
      mbar_init(&gempty[b], NCONV);
    }
    mbar_init(rbar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
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

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pw = policy_evict_first(), px = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          record_error(a.err, kErrTimeoutSmemEmpty);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], L::Q_BYTES + L::X_BYTES);
        tma_load_2d(sQ(stage), &tmQ, &full[stage], kb * BK * HK / 2, nt * BW, pw);
        for (int h = 0; h < HK; ++h)
          tma_load_2d(sX(stage) + h * L::X_HALF, &tmX, &full[stage], (kb * HK + h) * BK, 0, px);
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
      for (int kb = kb0; kb < kb1; ++kb) {
        const int j = (kb - kb0) / a.kpg, r = (kb - kb0) % a.kpg;
        if (r == 0 && !mbar_wait(&gempty[j & 1], ((j >> 1) & 1) ^ 1u, abort_flag)) {
          record_error(a.err, kErrTimeoutTmemEmpty);
          *abort_flag = 1;
          break;
        }
        if (!mbar_wait(&ready[stage], phase, abort_flag)) {
          record_error(a.err, kErrTimeoutTmaFull);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t xb = smem_u32(sX(stage));
        const uint32_t acc = tmem_base + (j & 1) * BT;
        const uint32_t at = tmem_base + ACOL + stage * AW;
#pragma unroll
        for (int k = 0; k < HK * BK / 16; ++k)
          tc_mma_f16_ts(acc, at + k * 8, sw128_kmajor_desc(xb + (k >> 2) * L::X_HALF + (k & 3) * 32),
                        idesc, (r > 0 || k > 0) ? 1u : 0u);
        tc_commit(&empty[stage]);
        if (r == a.kpg - 1) tc_commit(&gfull[j & 1]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ---- converter / rescale warps ----
    const int cw = warp - 2, hf = cw >> 2, quad = warp & 3;
    const int row = quad * 32 + lane;               // TMEM lane = weight row of the tile
    const int n = min(nt * BW + row, a.N - 1);
    const uint32_t tl = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const int g0 = kb0 * BK / (a.kpg * BK);
    const __half* srow = a.scales + static_cast<size_t>(n) * a.gpr + g0;
    const __half* orow = a.offsets + static_cast<size_t>(n) * a.gpr + g0;
    float acc[HC];
#pragma unroll
    for (int c = 0; c < HC; ++c) acc[c] = 0.f;
    bool ok = true;
    // group j's scale (kept for the rescale one group later) and (128 + z) as a bf16 pair;
    // the raw values are loaded one group ahead so their latency hides behind a group's work
    __half nsh = ngroups > 0 ? srow[0] : __half(), noh = ngroups > 0 ? orow[0] : __half();
    auto group_params = [&](int j, float& sc, uint32_t& zz) {
      sc = __half2float(nsh);
      const float of = __half2float(noh);
      if (j + 1 < ngroups) {
        nsh = srow[j + 1];
        noh = orow[j + 1];
      }
      const int z = sc != 0.f ? min(15, max(0, __float2int_rn(__fdividef(of, sc)))) : 0;
      zz = (0x4300u | static_cast<uint32_t>(z)) * 0x10001u;
    };
    auto rescale = [&](int j, float sc) {
      int go = 1;
      if (!mbar_wait(&gfull[j & 1], (j >> 1) & 1, abort_flag)) {
        record_error(a.err, kErrTimeoutTmemFull);
        *abort_flag = 1;
        go = 0;
      }
      go = __all_sync(0xffffffffu, go);
      if (!go) return false;
      tc_fence_after();
      if constexpr (HC == 8) {
        uint32_t v[8];
        tmem_ld8(tl + (j & 1) * BT + hf * HC, v);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = fmaf(sc, __uint_as_float(v[c]), acc[c]);
      } else {
        uint32_t v[16];
        tmem_ld16(tl + (j & 1) * BT + hf * HC, v);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c] = fmaf(sc, __uint_as_float(v[c]), acc[c]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&gempty[j & 1]);
      return true;
    };
    int stage = 0;
    uint32_t phase = 0;
    float sc_cur = 0.f, sc_prev = 0.f;
    uint32_t zz = 0x43004300u;
    for (int kb = kb0; kb < kb1 && ok; ++kb) {
      const int j = (kb - kb0) / a.kpg, r = (kb - kb0) % a.kpg;
      if (r == 0) {
        sc_prev = sc_cur;
        group_params(j, sc_cur, zz);
      }
      int go = 1;
      if (!mbar_wait(&full[stage], phase, abort_flag)) {
        record_error(a.err, kErrTimeoutTmaFull);
        *abort_flag = 1;
        go = 0;
      }
      go = __all_sync(0xffffffffu, go);
      if (!go) {
        ok = false;
        break;
      }
      // 16 HK packed bytes = elements [32 HK hf, 32 HK (hf + 1)) of this row's 64 HK
#pragma unroll
      for (int u = 0; u < HK; ++u) {
        const uint4 p = *reinterpret_cast<const uint4*>(sQ(stage) + row * 32 * HK + (hf * HK + u) * 16);
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
        uint32_t v[16];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            v[4 * c + i] = sub_bf16x2(((w[c] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, zz);
        tmem_st16(tl + ACOL + stage * AW + (hf * HK + u) * 16, v);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[stage]);
      if (r == a.kpg - 1 && j >= 1) ok = rescale(j - 1, sc_prev);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (ok && ngroups > 0) ok = rescale(ngroups - 1, sc_cur);
    // running sums -> TMEM columns [0, BT) for the split-K exchange (every MMA has completed)
    if (ok && ngroups > 0) {
      uint32_t v[HC];
#pragma unroll
      for (int c = 0; c < HC; ++c) v[c] = __float_as_uint(acc[c]);
      if constexpr (HC == 8) tmem_st8(tl + hf * HC, v);
      else tmem_st16(tl + hf * HC, v);
      tc_wait_st();
    }
    tc_fence_before();
    if (threadIdx.x == 64) s_go[0] = (ngroups == 0) ? 2 : ((ok && !*abort_flag) ? 1 : 0);
    named_bar_sync(2, NCONV * 32);
    tc_fence_after();
    if (hf == 0) {
      // warps 2..5: the exchange of the cluster split-K (TMEM lane = quad * 32 + lane)
      crs::publish<BT>(tl, s_go[0] == 1, sSlots, ws_tile, rank, S, quad * 32 + lane,
                       threadIdx.x - 64);
    }
  }

  tc_fence_before();
  crs::sync_all();
  tc_fence_after();
  if (warp >= 2 && warp < 6) {
    const int e = threadIdx.x - 64;
    if (e == 0) crs::fetch<BT>(sSlots, ws_tile, rbar, rank, S);
    const int x0 = a.mode == 1 ? nt * 64 : nt * BW;
    auto epi = [&](int oc, int t0, int l, float4 (&accv)[crs::CW]) {
      uint8_t* tile = crs::out_tile(sSlots, 0, oc);
      crs::stage_out(a.mode, tile, l, accv, nullptr, 0, 0, 0);
      crs::store_chunk(&tmC, tile, l, x0, t0);
    };
    const bool okr = crs::reduce<BT>(sSlots, rbar, rank, S, e, abort_flag, epi);
    crs::store_wait(e & 31, false);
    if (!okr) {
      record_error(a.err, kErrTimeoutTmaFull);
      *abort_flag = 1;
      if (e == 0 && !mbar_wait(rbar, 0, nullptr, kWaitBudgetNs)) record_error(a.err, kErrTimeoutDrain);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace qs

static PFN_cuTensorMapEncodeTiled_v12000 q_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult r;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &r);
    TORCH_CHECK(p != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool make_tmap_out(const at::Tensor& C, int64_t mode, int M, int N, int box_rows, CUtensorMap* m);
CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swz);

template <int BT, int STAGES, int QBITS>
static void launch_q(const CUtensorMap& tq, const CUtensorMap& tx, const CUtensorMap& tc,
                     const q::Args& a, int S, cudaStream_t st) {
  using L = q::Smem<BT, STAGES, QBITS>;
  TORCH_CHECK(crs::smem_bytes(BT, S) <= STAGES * L::STAGE,
              "gemm_quant: split-K slots exceed the pipeline buffers (BT ", BT, ", S ", S, ")");
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(q::gemm_q_kernel<BT, STAGES, QBITS>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.m_tiles * a.n_tiles * S);
  cfg.blockDim = dim3(q::THREADS);
  cfg.dynamicSmemBytes = L::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, q::gemm_q_kernel<BT, STAGES, QBITS>, tq, tx, tc, a));
}

template <int BT, int HK>
static void launch_qs(const CUtensorMap& tq, const CUtensorMap& tx, const CUtensorMap& tc,
                      const qs::Args& a, int S, cudaStream_t st) {
  constexpr int STAGES = HK == 1 ? 6 : 3;  // TMEM: weight stages of 32 HK columns after 64
  using L = qs::Smem<BT, STAGES, HK>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(qs::gemm_qs_kernel<BT, STAGES, HK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         L::TOTAL);
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_tiles * S);
  cfg.blockDim = dim3(qs::THREADS);
  cfg.dynamicSmemBytes = L::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, qs::gemm_qs_kernel<BT, STAGES, HK>, tq, tx, tc, a));
}

// Small-batch (M <= 32) GEMM for 4-bit weights whose offsets are integer multiples of the
// scale (offset = z * s, z in 0..15: AWQ), group a multiple of 64.  Same operands as gemm_quant.
void gemm_quant_iz(const at::Tensor& X, const at::Tensor& qw, const at::Tensor& scales,
                   const at::Tensor& offsets, int64_t group, at::Tensor& C, int64_t mode,
                   int64_t splits, at::Tensor& err, at::Tensor& ws) {
  TORCH_CHECK(X.scalar_type() == at::kBFloat16 && X.stride(1) == 1, "gemm_quant_iz: X bf16");
  TORCH_CHECK(qw.scalar_type() == at::kByte && qw.is_contiguous(), "gemm_quant_iz: packed uint8");
  TORCH_CHECK(scales.scalar_type() == at::kHalf && offsets.scalar_type() == at::kHalf &&
                  scales.is_contiguous() && offsets.is_contiguous(),
              "gemm_quant_iz: contiguous fp16 scales / offsets");
  const int M = X.size(0), K = X.size(1), N = qw.size(0);
  TORCH_CHECK(M <= 32, "gemm_quant_iz: at most 32 rows");
  TORCH_CHECK(qw.size(1) * 2 == K, "gemm_quant_iz: 4-bit packed width");
  TORCH_CHECK(group >= 64 && group % 64 == 0 && K % group == 0, "gemm_quant_iz: group % 64");
  TORCH_CHECK(scales.size(0) == N && scales.size(1) == K / group, "gemm_quant_iz: scales shape");
  if (M == 0) return;
  const int BT = M <= 16 ? 16 : 32;
  qs::Args a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.n_tiles = (N + 127) / 128;
  // 128-element k-blocks (64-byte rows per TMA request) when the groups allow it
  static const bool wide_ok = []() {
    const char* e = std::getenv("LB_QS_BK");
    return !(e != nullptr && std::string(e) == "64");
  }();
  const int HK = (wide_ok && group % 128 == 0) ? 2 : 1;
  a.kb_total = K / (64 * HK);
  a.kpg = group / (64 * HK);
  a.gpr = K / group;
  const int ngroups = a.gpr;
  int S = static_cast<int>(splits);
  if (S <= 0) {
    // two CTAs per SM (TMEM: 256 columns each); at least two groups per split
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, X.get_device());
    S = 1;
    for (int s = 2; s <= 8; ++s)
      if (a.n_tiles * s <= 2 * nsm && ngroups / s >= 2) S = s;
  }
  S = std::max(1, std::min(S, std::min(8, ngroups)));
  while (S > 1 && ws.numel() < crs::ws_floats(a.n_tiles, BT, S)) --S;
  const int gps = (ngroups + S - 1) / S;
  a.kb_per_split = gps * a.kpg;
  a.ws = S > 1 ? ws.data_ptr<float>() : nullptr;
  a.scales = reinterpret_cast<const __half*>(scales.data_ptr());
  a.offsets = reinterpret_cast<const __half*>(offsets.data_ptr());
  a.mode = mode;
  a.err = err.data_ptr<int>();
  const bool vec_ok = (reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0) && (C.stride(0) % 4 == 0);
  if (mode == 1) TORCH_CHECK(N % 128 == 0 && vec_ok, "gemm_quant_iz swiglu layout");
  CUtensorMap tq;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(qw.size(1)), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(qw.stride(0))};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(32 * HK), 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = q_encode()(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qw.data_ptr(), dims, strides,
                            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "gemm_quant_iz: tensor map");
  }
  const CUtensorMap tx = make_tmap_bf16_2d(X.data_ptr(), K, M, X.stride(0) * 2, 64, BT,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tc;
  TORCH_CHECK(make_tmap_out(C, mode, M, N, crs::out_box_rows(BT, S), &tc),
              "gemm_quant_iz: C must be 16-byte aligned with a 16-byte multiple row stride");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (HK == 2) {
    if (BT == 16) launch_qs<16, 2>(tq, tx, tc, a, S, st);
    else launch_qs<32, 2>(tq, tx, tc, a, S, st);
  } else {
    if (BT == 16) launch_qs<16, 1>(tq, tx, tc, a, S, st);
    else launch_qs<32, 1>(tq, tx, tc, a, S, st);
  }
}

// X [M, K] bf16; qw [N, K*bits/8] uint8; scales / offsets [N, K/group] fp16.
void gemm_quant(const at::Tensor& X, const at::Tensor& qw, const at::Tensor& scales,
                const at::Tensor& offsets, int64_t bits, int64_t group, at::Tensor& C,
                int64_t mode, int64_t splits, at::Tensor& err, at::Tensor& ws) {
  TORCH_CHECK(X.scalar_type() == at::kBFloat16 && X.stride(1) == 1, "gemm_quant: X bf16");
  TORCH_CHECK(qw.scalar_type() == at::kByte && qw.is_contiguous(), "gemm_quant: packed uint8");
  TORCH_CHECK(scales.scalar_type() == at::kHalf && offsets.scalar_type() == at::kHalf,
              "gemm_quant: fp16 scales / offsets");
  TORCH_CHECK(bits == 4 || bits == 8, "gemm_quant: 4 or 8 bits");
  const int M = X.size(0), K = X.size(1), N = qw.size(0);
  TORCH_CHECK(qw.size(1) * 8 == K * bits, "gemm_quant: packed width");
  TORCH_CHECK(K % 64 == 0 && group >= 32 && (group % 32 == 0) && K % group == 0,
              "gemm_quant: K % 64, group in {32, 64, ...}");
  if (M == 0) return;
  const int BT = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  q::Args a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = (M + BT - 1) / BT;
  a.n_tiles = (N + 127) / 128;
  a.kb_total = K / 64;
  int S = static_cast<int>(splits);
  if (S <= 0) {
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, 0);
    const int tiles = a.m_tiles * a.n_tiles;
    S = 1;
    for (int s = 2; s <= 8; ++s)
      if (tiles * s <= nsm && a.kb_total / s >= 2) S = s;
  }
  S = std::max(1, std::min(S, std::min(8, a.kb_total)));
  {
    const int stages = BT == 128 ? 5 : BT == 256 ? 4 : 6;
    const int stage_bytes = 128 * 64 * 2 + 128 * 64 * static_cast<int>(bits) / 8 + BT * 64 * 2;
    while (S > 1 && crs::smem_bytes(BT, S) > stages * stage_bytes) --S;
    while (S > 1 && ws.numel() < crs::ws_floats(a.m_tiles * a.n_tiles, BT, S)) --S;
  }
  a.ws = S > 1 ? ws.data_ptr<float>() : nullptr;
  a.kb_per_split = (a.kb_total + S - 1) / S;
  a.scales = reinterpret_cast<const __half*>(scales.data_ptr());
  a.offsets = reinterpret_cast<const __half*>(offsets.data_ptr());
  a.group = group;
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.mode = mode;
  a.vec_ok = (reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0) && (C.stride(0) % 4 == 0);
  a.err = err.data_ptr<int>();
  if (mode == 1) TORCH_CHECK(N % 128 == 0 && a.vec_ok, "gemm_quant swiglu layout");
  CUtensorMap tq;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(qw.size(1)), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(qw.stride(0))};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(64 * bits / 8), 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = q_encode()(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qw.data_ptr(), dims, strides,
                            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "gemm_quant: tensor map");
  }
  const CUtensorMap tx = make_tmap_bf16_2d(X.data_ptr(), K, M, X.stride(0) * 2, 64, BT,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tc;
  TORCH_CHECK(make_tmap_out(C, mode, M, N, crs::out_box_rows(BT, S), &tc),
              "gemm_quant: C must be 16-byte aligned with a 16-byte multiple row stride");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
#define LB_Q(BTV, STV)                                                    \
  if (bits == 4) launch_q<BTV, STV, 4>(tq, tx, tc, a, S, st);             \
  else launch_q<BTV, STV, 8>(tq, tx, tc, a, S, st);
  switch (BT) {
    case 16: LB_Q(16, 6) break;
    case 32: LB_Q(32, 6) break;
    case 64: LB_Q(64, 6) break;
    case 128: LB_Q(128, 5) break;
    default: LB_Q(256, 4) break;
  }
#undef LB_Q
}

}  // namespace lb
