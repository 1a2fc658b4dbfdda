// Paged attention for chunked prefill and speculative verify on the 5th-generation tensor cores
// (sm_100a): S = Q K^T and O = P V run as tcgen05.mma with the accumulators in tensor memory.
//
// Reference sites replaced: the candle flash-attn / manual attention of the prefill path
// (src/model/custom_attention.rs:287-434,757-793) with its host-built masks
// (src/cache/parallel_cache_builder.rs:2232-2370).  Masks are implicit: causal index math
// against per-sequence lengths, keys read through the block table.
//
// One CTA = 128 packed query rows (token, head-in-group) of one sequence x one KV head, so the
// G query heads that share a KV head read each K/V tile once.  Keys stream in tiles of 128.
//
//   warp 0      TMA producer: Q once (a 3-D map over [tokens][heads][128] lands the packed rows
//               directly), then per key tile 8 paged blocks x 2 halves of K and of V into a
//               2-stage ring of 128-byte-swizzled tiles; block ids are validated first (an id
//               outside the pool is reported and replaced by block 0; blocks past the sequence
//               end re-load block 0, so masked keys multiply finite data).
//   warp 1      MMA issuer (one thread) and TMEM owner:
//                 S_j = Q K_j^T   -> TMEM S buffer j % 2 (fp32, 128 columns)
//                 O  += P_j V_j   (P_j read from TMEM, written over S_j as bf16; V_j from shared
//                                  memory in its natural key-major layout, an MN-major operand)
//               S_{j+1} is issued before O += P_j V_j, so the tensor core computes the next
//               scores while the softmax warps work on the current ones.
//   warps 2..5  softmax, one thread per query row (TMEM lane): mask, running max, exp2, row
//               sum, P as bf16 back into TMEM.  The running max used for P only moves when the
//               true max exceeds it by more than 2^8 (then O is rescaled in TMEM after the
//               previous P V has completed), so most tiles never touch O.  Epilogue: O / l.
// TMEM: O [0, 128), S0 [128, 256), S1 [256, 384) columns.  Every wait is bounded; on expiry the
// kernel records an error code and unwinds (TMA copies drained, TMEM freed).  No multicast.
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swz);

namespace fa {

constexpr int D = 128;          // head dim
constexpr int QT = 2;           // query tiles of 128 packed rows per CTA (ping-pong)
constexpr int BM = 128 * QT;    // packed query rows per CTA
constexpr int BN = 128;         // keys per tile
constexpr int BS = 16;          // paged block size
constexpr int THREADS = 64 + QT * 128;
constexpr int HALF = BN * 128;  // one 64-dim half of a 128-row tile (bytes)
constexpr int TILE = 2 * HALF;  // 32 KB
constexpr int KST = 2, VST = 2;
constexpr int SMEM_Q = 0;                            // [QT] tiles
constexpr int SMEM_K = QT * TILE;                    // [KST]
constexpr int SMEM_V = SMEM_K + KST * TILE;          // [VST]
constexpr int SMEM_BAR = SMEM_V + VST * TILE;
constexpr int SMEM_TOTAL = SMEM_BAR + 256 + 1024;    // + alignment slack
constexpr uint32_t TMEM_COLS = 512;                  // O_t at 128 t, S_t at 256 + 128 t
constexpr float RESCALE_THRESHOLD = 8.f;              // log2 units: P <= 2^8 between rescales

struct Args {
  bf16* out;
  int out_row_stride;
  const int* block_tables;
  int bt_stride;
  const int* seq_lens;
  const int* cu_q;
  const int* tile_seq;
  const int* tile_row0;
  int num_kv_heads, group, log2g;
  float scale_log2;
  int causal;
  int num_blocks;
  int* err;
};

// Shared-memory descriptor of an MN-major operand written by TMA with SWIZZLE_128B: 64-element
// (128-byte) rows along MN, 8-row swizzle atoms along K at SBO = 1024 bytes, the next 64 MN
// elements at LBO bytes.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Softmax arithmetic on the packed and multi-input forms of sm_100: a 3-input max, fp32 pairs
// (fma / add .f32x2: two lanes per instruction) and the hardware base-2 exponential
// (ex2.approx, denormal results flushed: P is rounded to bf16 anyway).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void unpack_f2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tma_load_3d_q(void* dst, const CUtensorMap* tmap, uint64_t* bar,
                                              int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  auto sQ = [&](int t) { return smem + SMEM_Q + t * TILE; };
  auto sK = [&](int s) { return smem + SMEM_K + s * TILE; };
  auto sV = [&](int s) { return smem + SMEM_V + s * TILE; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BAR);
  uint64_t* q_full = bars;                 // TMA Q (both tiles)
  uint64_t* k_full = bars + 1;             // [KST]
  uint64_t* k_empty = k_full + KST;        // [KST] S of every query tile done
  uint64_t* v_full = k_empty + KST;        // [VST]
  uint64_t* v_empty = v_full + VST;        // [VST] P V of every query tile done
  uint64_t* s_full = v_empty + VST;        // [QT] S_t of the current key tile (and all earlier MMAs)
  uint64_t* p_ready = s_full + QT;         // [QT] P_t in TMEM (4 softmax warps)
  uint64_t* o_full = p_ready + QT;         // last P V done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.y;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < QT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
    }
    mbar_init(o_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  pdl_trigger();
  pdl_wait();  // q, the block table, lengths and KV rows follow the previous grid

  const int seq = a.tile_seq[blockIdx.x];
  const int row0 = a.tile_row0[blockIdx.x];
  const int q_start = a.cu_q[seq];
  const int q_len = a.cu_q[seq + 1] - q_start;
  const int kv_len = a.seq_lens[seq];
  const int nrows_seq = q_len << a.log2g;
  const int nqt = row0 + 128 < nrows_seq ? QT : 1;   // query tiles holding valid rows
  const int* btab = a.block_tables + static_cast<size_t>(seq) * a.bt_stride;
  // keys this CTA needs: causal rows see keys <= kv_len - q_len + token
  int k_limit = kv_len;
  if (a.causal) {
    const int last_row = min(row0 + BM, nrows_seq) - 1;
    k_limit = min(kv_len, kv_len - q_len + (last_row >> a.log2g) + 1);
  }
  const int ntiles = k_limit > 0 ? (k_limit + BN - 1) / BN : 0;
  const int seq_blocks = (kv_len + BS - 1) / BS;

  // producer bookkeeping for the drain on abort: parity of the last load issued per stage
  int k_par[KST] = {-1, -1}, v_par[VST] = {-1, -1};
  bool q_issued = false;
  if (warp == 0) {
    if (lane == 0 && ntiles > 0) {
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(q_full, nqt * TILE);
      q_issued = true;
      for (int t = 0; t < nqt; ++t) {
        const int tok0 = q_start + ((row0 + 128 * t) >> a.log2g);
        for (int h = 0; h < 2; ++h)
          tma_load_3d_q(sQ(t) + h * HALF, &tmQ, q_full, h * 64, kvh * a.group, tok0);
      }
      auto load_tile = [&](const CUtensorMap* tm, uint8_t* dst, uint64_t* bar, int j) {
        mbar_arrive_expect_tx(bar, TILE);
        for (int b = 0; b < BN / BS; ++b) {
          const int lb = j * (BN / BS) + b;
          int blk = lb < seq_blocks ? btab[lb] : 0;
          if (static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks)) {
            record_error(a.err, kErrBounds);
            blk = 0;
          }
          const int row = (blk * a.num_kv_heads + kvh) * BS;
          for (int h = 0; h < 2; ++h) tma_load_2d(dst + h * HALF + b * BS * 128, tm, bar, h * 64, row, pol);
        }
      };
      for (int j = 0; j < ntiles; ++j) {
        const int ks = j % KST, vs = j % VST;
        if (!mbar_wait(&k_empty[ks], ((j / KST) & 1) ^ 1u, abort_flag)) {
          record_error(a.err, kErrTimeoutSmemEmpty);
          *abort_flag = 1;
          break;
        }
        load_tile(&tmK, sK(ks), &k_full[ks], j);
        k_par[ks] = (j / KST) & 1;
        if (!mbar_wait(&v_empty[vs], ((j / VST) & 1) ^ 1u, abort_flag)) {
          record_error(a.err, kErrTimeoutSmemEmpty);
          *abort_flag = 1;
          break;
        }
        load_tile(&tmV, sV(vs), &v_full[vs], j);
        v_par[vs] = (j / VST) & 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, BN);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D, 0, 1);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, abort_flag);
      // O_t += P_t V_j  (P_t over S_t in TMEM)
      auto issue_pv = [&](int t, int j) {
        if (!mbar_wait(&p_ready[t], j & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(sV(j % VST));
        const uint32_t pc = tmem_base + 256 + 128 * t;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          tc_mma_f16_ts(tmem_base + 128 * t, pc + k * 8, sw128_mnmajor_desc(vb + k * 16 * 128, HALF),
                        idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        return true;
      };
      // S_t = Q_t K_j^T
      auto issue_s = [&](int t, int j) {
        const uint32_t qb = smem_u32(sQ(t)), kb = smem_u32(sK(j % KST));
        const uint32_t sc = tmem_base + 256 + 128 * t;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * HALF + (k & 3) * 32;
          tc_mma_f16(sc, sw128_kmajor_desc(qb + off), sw128_kmajor_desc(kb + off), idesc_s,
                     k > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[t]);  // arrives once this and every earlier MMA have completed
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        ok = mbar_wait(&k_full[j % KST], (j / KST) & 1, abort_flag);
        if (ok && j > 0) ok = mbar_wait(&v_full[(j - 1) % VST], ((j - 1) / VST) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        for (int t = 0; t < nqt && ok; ++t) {
          // the previous tile's P V runs first: S_t is written over P_t, in issue order
          if (j > 0) ok = issue_pv(t, j - 1);
          if (ok) issue_s(t, j);
        }
        if (!ok) break;
        tc_commit(&k_empty[j % KST]);
        if (j > 0) tc_commit(&v_empty[(j - 1) % VST]);
      }
      if (ok) ok = mbar_wait(&v_full[(ntiles - 1) % VST], ((ntiles - 1) / VST) & 1, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < nqt && ok; ++t) ok = issue_pv(t, ntiles - 1);
      }
      if (ok) {
        tc_commit(&v_empty[(ntiles - 1) % VST]);
        tc_commit(o_full);
      } else {
        record_error(a.err, kErrTimeoutTmaFull);
        *abort_flag = 1;
      }
    }
  } else {
    // ---- softmax / epilogue: warpgroup t = query tile t, thread = query row (TMEM lane) ----
    const int t = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int pr = row0 + 128 * t + r;
    const bool valid_row = pr < nrows_seq;
    const int tok = pr >> a.log2g;
    const int qpos = kv_len - q_len + tok;
    const int klim = !valid_row ? 0 : (a.causal ? min(kv_len, qpos + 1) : kv_len);
    const uint32_t tl = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t colO = 128 * t, colS = 256 + 128 * t;
    float m_used = -INFINITY, l = 0.f;
    bool ok = t < nqt;
    for (int j = 0; j < ntiles && ok; ++j) {
      int go = mbar_wait(&s_full[t], j & 1, abort_flag) ? 1 : 0;
      go = __all_sync(0xffffffffu, go);
      if (!go) {
        if (lane == 0) record_error(a.err, kErrTimeoutTmemFull);
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld32(tl + colS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sr + 32 * c));
      tc_wait_ld();
      const int nvalid = min(BN, max(0, klim - j * BN));  // keys [j BN, j BN + nvalid) visible
      // raw scores: masked keys -> -inf (only tiles that cross a row's limit); the softmax scale
      // (> 0, order preserving) is applied to the max and folded into the exponent's FMA
      if (!__all_sync(0xffffffffu, nvalid >= BN)) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= nvalid) sr[c] = __float_as_uint(-INFINITY);
      }
      float mr = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; c += 2)
        mr = max3f(mr, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
      const float mx = mr * a.scale_log2;
      const bool need = mx > m_used + RESCALE_THRESHOLD;
      const float m_new = need ? mx : m_used;
      // s_full's arrival implies the previous P V into O_t has completed (issue order)
      if (__any_sync(0xffffffffu, need) && j > 0) {
        const float corr = need ? exp2f(m_used - m_new) : 1.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(tl + colO + 32 * c, ov);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * corr);
          tmem_st16(tl + colO + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(ov));
          tmem_st16(tl + colO + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(ov + 16));
        }
      }
      if (need) {
        l *= exp2f(m_used - m_new);  // 0 when m_used = -inf
        m_used = m_new;
      }
      const float ms = m_used == -INFINITY ? 0.f : m_used;
      const uint64_t sc2 = pack_f2(a.scale_log2, a.scale_log2), nms2 = pack_f2(-ms, -ms);
      uint64_t l2 = pack_f2(0.f, 0.f);
      // P in 32-key chunks, each stored to TMEM as soon as it is packed (P chunk q overwrites
      // S columns [16 q, 16 q + 16), whose scores are already in registers)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int e = 32 * q + 2 * c;
          float x0, x1;
          unpack_f2(fma_f2(pack_f2(__uint_as_float(sr[e]), __uint_as_float(sr[e + 1])), sc2,
                           nms2), x0, x1);
          const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
          l2 = add_f2(l2, pack_f2(p0, p1));
          pk[c] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tl + colS + 16 * q, pk);
      }
      {
        float la, lb;
        unpack_f2(l2, la, lb);
        l += la + lb;
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[t]);
    }
    // ---- epilogue: O_t / l -> out[token][head][:] ----
    if (ok && ntiles > 0) {
      int go = mbar_wait(o_full, 0, abort_flag) ? 1 : 0;
      go = __all_sync(0xffffffffu, go);
      if (go) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        bf16* dst = a.out + static_cast<size_t>(q_start + tok) * a.out_row_stride +
                    (kvh * a.group + (pr & (a.group - 1))) * D;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(tl + colO + 32 * c, ov);
          tc_wait_ld();
          if (valid_row) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(ov[8 * i]) * inv, __uint_as_float(ov[8 * i + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + 32 * c + 8 * i) = v;
            }
          }
        }
      } else {
        if (lane == 0) record_error(a.err, kErrTimeoutTmemFull);
        *abort_flag = 1;
      }
    }
  }

  // after an abort: wait (bounded) for this CTA's TMA copies still in flight
  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    bool drained = !q_issued || mbar_wait(q_full, 0, nullptr, kWaitBudgetNs);
    for (int s = 0; s < KST; ++s)
      if (k_par[s] >= 0) drained &= mbar_wait(&k_full[s], static_cast<uint32_t>(k_par[s]), nullptr, kWaitBudgetNs);
    for (int s = 0; s < VST; ++s)
      if (v_par[s] >= 0) drained &= mbar_wait(&v_full[s], static_cast<uint32_t>(v_par[s]), nullptr, kWaitBudgetNs);
    if (!drained) record_error(a.err, kErrTimeoutDrain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace fa

static PFN_cuTensorMapEncodeTiled_v12000 fa_encode() {
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

bool prefill_tc_supported(int64_t group, int64_t block_size, int64_t head_dim) {
  return head_dim == fa::D && block_size == fa::BS && group >= 1 && group <= 16 &&
         (group & (group - 1)) == 0;
}

// q [T, Hq, 128] (row stride 16-byte aligned), caches [num_blocks, Hkv, 16, 128]; the work list
// (tile_seq, tile_row0) has one entry per 256 packed rows of each sequence.
void paged_attention_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                        at::Tensor& out, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                        const at::Tensor& cu_q, const at::Tensor& tile_seq,
                        const at::Tensor& tile_row0, int64_t group, double scale, bool causal,
                        const c10::optional<at::Tensor>& err) {
  using namespace fa;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16 &&
                  v_cache.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "paged_attention_tc: bf16");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == D && q.stride(2) == 1 && q.stride(1) == D &&
                  (q.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
              "paged_attention_tc: q [T, Hq, 128], contiguous heads, 16-byte aligned rows");
  TORCH_CHECK(out.dim() == 3 && out.stride(2) == 1 && out.stride(1) == D &&
                  (out.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "paged_attention_tc: out layout");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  k_cache.sizes() == v_cache.sizes(),
              "paged_attention_tc: caches [num_blocks, Hkv, 16, 128]");
  TORCH_CHECK(prefill_tc_supported(group, k_cache.size(2), k_cache.size(3)),
              "paged_attention_tc: block size 16, head dim 128, power-of-two group <= 16");
  const int64_t rows = k_cache.size(0) * k_cache.size(1) * BS;
  TORCH_CHECK(rows < (int64_t(1) << 31), "paged_attention_tc: KV pool rows exceed int32");
  const int ntiles = tile_seq.size(0);
  if (ntiles == 0 || seq_lens.size(0) == 0) return;
  const int Hq = q.size(1), T = q.size(0);
  Args a;
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.out_row_stride = out.stride(0);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = block_tables.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.cu_q = cu_q.data_ptr<int>();
  a.tile_seq = tile_seq.data_ptr<int>();
  a.tile_row0 = tile_row0.data_ptr<int>();
  a.num_kv_heads = k_cache.size(1);
  a.group = group;
  a.log2g = 0;
  while ((1 << a.log2g) < group) ++a.log2g;
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  a.causal = causal ? 1 : 0;
  a.num_blocks = static_cast<int>(k_cache.size(0));
  a.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  CUtensorMap tq;
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(Hq),
                          static_cast<cuuint64_t>(T)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(q.stride(0) * 2)};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(group), static_cast<cuuint32_t>(128 / group)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fa_encode()(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q.data_ptr(), dims, strides,
                             box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "paged_attention_tc: q tensor map");
  }
  const CUtensorMap tk = make_tmap_bf16_2d(k_cache.data_ptr(), D, rows, D * 2, 64, BS,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tv = make_tmap_bf16_2d(v_cache.data_ptr(), D, rows, D * 2, 64, BS,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL);
    attr = true;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  dim3 grid(ntiles, a.num_kv_heads, 1);
  C10_CUDA_CHECK(launch_k(prefill_tc_kernel, grid, dim3(THREADS), SMEM_TOTAL, st, nullptr, 0, tq,
                          tk, tv, a));
}

}  // namespace lb
