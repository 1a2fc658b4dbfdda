// Persistent bf16 GEMM on SM pairs: tcgen05.mma.cta_group::2 with 256-row weight tiles.
// Included by gemm_tc.cu (uses GemmArgs, BW, BK, UK, kThreads, the epilogue modes, silu).
//
// Why: a 128 x 256 x 16 MMA on one SM consumes 12 KB of shared-memory operands in ~135 clocks
// while the TMA writes the same amount, which is more shared-memory traffic than the SM can
// sustain; the tensor pipe then idles (the single-SM persistent kernel measured ~55 % tensor
// activity).  On an SM pair each CTA stages half of the 256 weight rows (A) and half of the
// token tile (B); one thread of the leader CTA issues the 256 x BT x 16 MMA, which reads both
// CTAs' shared memory and writes each CTA's 128 accumulator rows into that CTA's TMEM.  Per
// SM and per MMA the operand traffic drops from 12 KB to 8 KB (BT = 256).
//
// Roles (192 threads per CTA, cluster of 2):
//   warp 0  both CTAs: TMA producer.  Each CTA loads its own halves into its own shared
//           memory; every load signals the LEADER's full barrier (cta_group::2 form, no
//           multicast), whose expected byte count (both halves) the leader's producer arms.
//   warp 1  leader only: MMA issuer.  A stage is released by one commit per CTA (the leader's
//           and the peer's empty barrier); a finished accumulator by one commit per CTA to
//           each tfull barrier.
//   warps 2-5  both CTAs: epilogue from the CTA's own TMEM (128 weight rows x BT tokens), then
//           one elected arrival per CTA on the leader's tempty barrier.
// Every wait is bounded; on timeout the CTA records an error, stops issuing, waits (bounded)
// for its own copies / MMAs and meets its peer at the final cluster barrier before releasing
// TMEM.
#pragma once

namespace lb {
namespace tc2 {

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// TMA load into this CTA's shared memory, completion counted on `bar` (a shared::cluster
// address, here the leader's barrier).  Source: this GPU's own global memory.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* tmap, uint32_t bar,
                                                 int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` (shared::cluster address) when this thread's prior tcgen05 ops complete.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

template <int BT, int STAGES>
struct Smem {
  static constexpr int W_BYTES = BW * BK * 2;          // this CTA's 128 weight rows
  static constexpr int X_BYTES = (BT / 2) * BK * 2;    // this CTA's BT / 2 tokens
  static constexpr int CH = 32;                        // epilogue column chunk
  static constexpr int EPI_FLOATS = 64 * (CH + 1);
  static constexpr int BAR_OFF = STAGES * (W_BYTES + X_BYTES) + EPI_FLOATS * 4;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
  static constexpr int TMEM_COLS = 2 * BT;             // double-buffered accumulator
  static_assert(BT == 128 || BT == 256, "pair GEMM token tile");
  static_assert(TOTAL <= 227 * 1024, "pair GEMM shared memory");
};

}  // namespace tc2

template <int BT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const GemmArgs a) {
  using L = tc2::Smem<BT, STAGES>;
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
  volatile int* s_go = reinterpret_cast<volatile int*>(tmem_slot + 4);  // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = tc2::cta_rank();
  const int pair = static_cast<int>(tc2::cluster_id());
  const int npairs = static_cast<int>(tc2::num_clusters());

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2);  // one elected arrival per CTA of the pair
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
    tc2::tmem_alloc_pair(tmem_slot, L::TMEM_COLS);
    tc2::tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc2::cluster_sync();  // the peer's barriers are initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = (a.N + 2 * BW - 1) / (2 * BW);
  const int total = a.m_tiles * n_tiles;
  auto decode_unit = [&](int u, int& mt, int& nt) {
    nt = u % n_tiles;
    mt = u / n_tiles;
  };

  uint32_t issued_mask = 0, issued_parity = 0;   // leader producer: armed stages (drain)
  uint64_t last_issue_ns = 0;                    // peer producer: time of its last load

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pw = policy_evict_first();
      const uint64_t px = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; u < total && ok && !*abort_flag; u += npairs) {
        int mt, nt;
        decode_unit(u, mt, nt);
        for (int kb = 0; kb < a.kb_total; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            record_error(a.err, kErrTimeoutSmemEmpty);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t fb = tc2::peer_addr(&full[stage], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (L::W_BYTES + L::X_BYTES));
          tc2::tma_load_2d_pair(sW + stage * L::W_BYTES, &tmW, fb, kb * BK,
                                nt * 2 * BW + static_cast<int>(rank) * BW, pw);
          tc2::tma_load_2d_pair(sX + stage * L::X_BYTES, &tmX, fb, kb * BK,
                                mt * BT + static_cast<int>(rank) * (BT / 2), px);
          if (rank == 0) {
            issued_mask |= 1u << stage;
            issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          } else {
            last_issue_ns = globaltimer_ns();
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(2 * BW, BT);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int u = pair; u < total && !*abort_flag; u += npairs, ++it) {
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
        for (int kb = 0; kb < a.kb_total; ++kb) {
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
            tc2::mma_pair(d_tmem, sw128_kmajor_desc(wb + k * UK * 2),
                          sw128_kmajor_desc(xb + k * UK * 2), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc2::commit_pair(smem_u32(&empty[stage]));
          tc2::commit_pair(tc2::peer_addr(&empty[stage], 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc2::commit_pair(smem_u32(&tfull[acc]));
        tc2::commit_pair(tc2::peer_addr(&tfull[acc], 1));
      }
    }
  } else {
    // ---------------- epilogue warps: this CTA's 128 weight rows ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int etid = threadIdx.x - 64;
    int it = 0;
    for (int u = pair; u < total; u += npairs, ++it) {
      int mt, nt;
      decode_unit(u, mt, nt);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
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
      const int g128 = nt * 2 + static_cast<int>(rank);   // 128-row group of this CTA
      const int m0 = mt * BT;
      const int n = g128 * BW + row;
#pragma unroll 1
      for (int c = 0; c < BT; c += CH) {
        uint32_t r[CH];
        tmem_ld32(tbase + c, r);
        tc_wait_ld();
        if (c + CH >= BT) {
          // accumulator drained by all 128 threads -> one arrival for this CTA
          tc_fence_before();
          named_bar_sync(1, 128);
          if (etid == 0) {
            if (rank == 0) mbar_arrive(&tempty[acc]);
            else tc2::arrive_remote(tc2::peer_addr(&tempty[acc], 0));
          }
        }
        float v[CH];
#pragma unroll
        for (int j = 0; j < CH; ++j) v[j] = __uint_as_float(r[j]);
        if (a.mode == kEpiSwiGLU) {
          if (row >= 64) {
#pragma unroll
            for (int j = 0; j < CH; ++j) sEpi[(row - 64) * (CH + 1) + j] = v[j];
          }
          named_bar_sync(1, 128);
          if (row < 64) {
            const int f = g128 * 64 + row;
            const int nf = a.N >> 1;
            bf16* C = reinterpret_cast<bf16*>(a.C);
            if (f < nf) {
#pragma unroll
              for (int j = 0; j < CH; ++j) {
                const int m = m0 + c + j;
                if (m < a.M)
                  C[static_cast<size_t>(m) * a.ldc + f] =
                      __float2bfloat16(silu(v[j]) * sEpi[row * (CH + 1) + j]);
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
      }
    }
  }

  __syncthreads();
  if (*abort_flag) {
    if (warp == 0 && lane == 0) {
      if (rank == 0) {
        // the armed stages count both CTAs' bytes: their completion covers the peer's loads
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s))
            if (!mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, kWaitBudgetNs))
              record_error(a.err, kErrTimeoutDrain);
      } else if (last_issue_ns != 0) {
        // this CTA's loads signal the leader: give them a bounded grace period to land
        while (globaltimer_ns() - last_issue_ns < 2000000ull) {
        }
      }
    }
    if (warp == 1 && lane == 0 && rank == 0) {
      tc2::commit_pair(smem_u32(drain));   // same cta_group as the MMAs it tracks
      if (!mbar_wait(drain, 0, nullptr, kWaitBudgetNs)) record_error(a.err, kErrTimeoutDrain);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc2::cluster_sync();   // no remote signal or MMA into this CTA is outstanding past here
  if (warp == 1) {
    tc_fence_after();
    tc2::tmem_dealloc_pair(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace lb
