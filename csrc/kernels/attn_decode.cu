// Paged decode attention, TMA-fed and warp-specialised (sm_100a).
//
// One CTA per (sequence, KV head, KV split).  Warp 0 is the producer: for each 64-key tile
// it looks up the 4 physical blocks in the block table and issues 16 TMA tile loads
// (K and V, two 64-element halves of the 128-wide head each) into a STAGES-deep ring of
// 128-byte-swizzled shared-memory tiles, signalling an mbarrier with the byte count.
// Warps 1..4 consume: each takes 16 keys of the tile, computes S = Q K^T and O += P V with
// mma.sync (the G query heads of the group packed as MMA rows), keeps an online softmax,
// and releases the stage.  At the end the 4 consumer warps merge their (m, l, O) states;
// split-KV partials (lse + normalised O) are merged by attn_combine_kernel.
//
// This replaces the reference's per-step dense attention with host masks
// (src/model/custom_attention.rs:741-858) and the CPU-only PagedAttn
// (src/model_fuel/batched.rs:932-943).  Decode attention is HBM-bound (each K/V byte is
// used once per query group), so the design goal is bytes in flight, not MMA rate.
// Every wait is bounded; on expiry the kernel records an error code and unwinds.
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swz);

namespace dec {

constexpr int D = 128;
constexpr int KT = 64;                  // keys per tile
constexpr int BS = 16;                  // paged block size this kernel is built for
constexpr int STAGES = 3;
constexpr int NCONS = 4;                // consumer warps
constexpr int THREADS = 32 * (NCONS + 1);
constexpr int HALF_BYTES = KT * 128;    // 64 keys x 64 elements x 2 bytes
constexpr int TILE_BYTES = 2 * HALF_BYTES;   // one of K or V for 64 keys
constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // K + V

struct Args {
  const bf16* q;
  int q_row_stride;
  bf16* out;
  int out_row_stride;
  const int* block_tables;
  int bt_stride;
  const int* seq_lens;
  int num_kv_heads;
  int group;
  float scale_log2;
  int num_splits;
  float* part_o;
  float* part_lse;
  int total_rows;
  int num_blocks;       // KV pool size: block ids outside [0, num_blocks) are reported
  int* err;
};

// Byte offset of (key r, 16-byte chunk c of the 256-byte head row) inside a K or V tile:
// [half][key][64 elements] with the 128-byte TMA swizzle (chunk ^ key % 8).
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
  const int half = c >> 3, cc = c & 7;
  return half * HALF_BYTES + r * 128 + ((cc ^ (r & 7)) << 4);
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(THREADS, 2)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sKV = smem;                                   // STAGES x (K tile | V tile)
  bf16* sQ = reinterpret_cast<bf16*>(smem + STAGES * STAGE_BYTES);  // 16 x 128 (swizzled)
  float* sM = reinterpret_cast<float*>(sQ + 16 * D);     // [4][16] max, [4][16] sum, [32] tot
  float* sO = sM + 160;                                  // [16][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sO + 16 * D);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  pdl_trigger();
  pdl_wait();   // q, the block table, lengths and the KV rows follow the previous grid
  const int kv_len = a.seq_lens[seq];
  const int* btab = a.block_tables + static_cast<size_t>(seq) * a.bt_stride;
  const int G = a.group;

  int k_begin = 0, k_end = kv_len;
  if (a.num_splits > 1) {
    const int per = ((kv_len + a.num_splits - 1) / a.num_splits + KT - 1) / KT * KT;
    k_begin = split * per;
    k_end = min(kv_len, k_begin + per);
  }
  const int ntiles = k_end > k_begin ? (k_end - k_begin + KT - 1) / KT : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCONS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Q rows (head g of this group, g < G) -> swizzled [16][128] (rows >= G zero).
  for (int i = threadIdx.x; i < 16 * 16; i += THREADS) {
    const int r = i >> 4, c = i & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G)
      v = *reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(seq) * a.q_row_stride +
                                          (kvh * G + r) * D + c * 8);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sQ) + r * 256 + ((c ^ (r & 7)) << 4)) = v;
  }
  __syncthreads();

  uint32_t issued_mask = 0, issued_parity = 0;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      for (int t = 0; t < ntiles; ++t) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          record_error(a.err, kErrTimeoutSmemEmpty);
          *abort_flag = 1;
          break;
        }
        const int kb = k_begin + t * KT;
        const int nblk = min(KT / BS, (k_end - kb + BS - 1) / BS);
        // Always fill all 4 block slots; slots past the sequence end re-load the tile's first
        // block so that masked keys multiply finite data (P = 0 exactly).
        mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
        uint8_t* sK = sKV + stage * STAGE_BYTES;
        uint8_t* sV = sK + TILE_BYTES;
        for (int b = 0; b < KT / BS; ++b) {
          // A block id outside the pool (a corrupted table) is reported through the error
          // word and replaced by block 0, so every TMA coordinate stays inside the tensor map.
          int blk = btab[(kb >> 4) + (b < nblk ? b : 0)];
          if (static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks)) {
            record_error(a.err, kErrBounds);
            blk = 0;
          }
          const int row = (blk * a.num_kv_heads + kvh) * BS;
          for (int h = 0; h < 2; ++h) {
            tma_load_2d(sK + h * HALF_BYTES + b * BS * 128, &tmK, &full[stage], h * 64, row, pol);
            tma_load_2d(sV + h * HALF_BYTES + b * BS * 128, &tmV, &full[stage], h * 64, row, pol);
          }
        }
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    const int cw = warp - 1;  // consumer warp: keys [16 cw, 16 cw + 16) of each tile
    const int g = lane >> 2, t4 = lane & 3;
    uint32_t qf[8][4];
    const uint32_t qbase = smem_u32(sQ);
#pragma unroll
    for (int kc = 0; kc < 8; ++kc) {
      const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = kc * 2 + (lane >> 4);
      ldsm_x4(qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3], qbase + r * 256 + ((c ^ (r & 7)) << 4));
    }
    int stage = 0;
    uint32_t phase = 0;
    for (int t = 0; t < ntiles; ++t) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag));
      if (!ok) {  // warp-uniform: ldmatrix / mma.sync below need the whole warp
        if (lane == 0) record_error(a.err, kErrTimeoutTmaFull);
        *abort_flag = 1;
        break;
      }
      const uint32_t kbase_s = smem_u32(sKV + stage * STAGE_BYTES);
      const uint32_t vbase_s = kbase_s + TILE_BYTES;
      const int key0 = cw * 16;
      const int kb = k_begin + t * KT;
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kc = 0; kc < 8; ++kc) {
        uint32_t b0, b1, b2, b3;
        const int r = key0 + (lane & 7) + (lane >> 4) * 8;
        const int c = kc * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, kbase_s + kv_off(r, c));
        mma_bf16(s[0], qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3], b0, b1);
        mma_bf16(s[1], qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3], b2, b3);
      }
      float mnew[2] = {m_r[0], m_r[1]};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = kb + key0 + j * 8 + 2 * t4 + (e & 1);
          const int h = e >> 1;
          float x = s[j][e] * a.scale_log2;
          x = (key < k_end && (g + 8 * h) < G) ? x : -INFINITY;
          s[j][e] = x;
          mnew[h] = fmaxf(mnew[h], x);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mnew[h] = fmaxf(mnew[h], __shfl_xor_sync(0xffffffffu, mnew[h], 1));
        mnew[h] = fmaxf(mnew[h], __shfl_xor_sync(0xffffffffu, mnew[h], 2));
      }
      float corr[2], ms[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        ms[h] = mnew[h] == -INFINITY ? 0.f : mnew[h];
        corr[h] = exp2f(m_r[h] - ms[h]);
        m_r[h] = mnew[h];
        l_r[h] *= corr[h];
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        o[i][0] *= corr[0];
        o[i][1] *= corr[0];
        o[i][2] *= corr[1];
        o[i][3] *= corr[1];
      }
      uint32_t pf[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float p0 = exp2f(s[j][0] - ms[0]), p1 = exp2f(s[j][1] - ms[0]);
        const float p2 = exp2f(s[j][2] - ms[1]), p3 = exp2f(s[j][3] - ms[1]);
        l_r[0] += p0 + p1;
        l_r[1] += p2 + p3;
        pf[j][0] = pack_bf16x2(p0, p1);
        pf[j][1] = pack_bf16x2(p2, p3);
      }
#pragma unroll
      for (int dn = 0; dn < 16; dn += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = key0 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dn + (lane >> 4);
        ldsm_x4_t(b0, b1, b2, b3, vbase_s + kv_off(r, c));
        mma_bf16(o[dn], pf[0][0], pf[0][1], pf[1][0], pf[1][1], b0, b1);
        mma_bf16(o[dn + 1], pf[0][0], pf[0][1], pf[1][0], pf[1][1], b2, b3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
      l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
    }
    if (t4 == 0) {
      sM[cw * 16 + g] = m_r[0];
      sM[cw * 16 + g + 8] = m_r[1];
      sM[64 + cw * 16 + g] = l_r[0];
      sM[64 + cw * 16 + g + 8] = l_r[1];
    }
  }
  for (int i = threadIdx.x; i < 16 * D; i += THREADS) sO[i] = 0.f;
  __syncthreads();
  // Merge the consumer warps' states (disjoint keys, same rows).
  if (warp > 0) {
    const int cw = warp - 1;
    const int g = lane >> 2, t4 = lane & 3;
    float sc[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + 8 * h;
      float mm = -INFINITY;
      for (int w = 0; w < NCONS; ++w) mm = fmaxf(mm, sM[w * 16 + r]);
      const float msafe = mm == -INFINITY ? 0.f : mm;
      sc[h] = exp2f(m_r[h] - msafe);
      if (cw == 0 && t4 == 0) {
        float lt = 0.f;
        for (int w = 0; w < NCONS; ++w) lt += sM[64 + w * 16 + r] * exp2f(sM[w * 16 + r] - msafe);
        sM[128 + r] = mm;
        sM[144 + r] = lt;
      }
    }
    for (int w = 0; w < NCONS; ++w) {
      if (cw == w) {
#pragma unroll
        for (int dn = 0; dn < 16; ++dn) {
          const int d = dn * 8 + 2 * t4;
          sO[g * D + d] += o[dn][0] * sc[0];
          sO[g * D + d + 1] += o[dn][1] * sc[0];
          sO[(g + 8) * D + d] += o[dn][2] * sc[1];
          sO[(g + 8) * D + d + 1] += o[dn][3] * sc[1];
        }
      }
      named_bar_sync(1, 32 * NCONS);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += THREADS) {
    const int r = i / D, d = i % D;
    const int head = kvh * G + r;
    const float lt = sM[144 + r];
    const float val = lt > 0.f ? sO[r * D + d] / lt : 0.f;
    if (a.num_splits > 1) {
      const size_t row = static_cast<size_t>(seq) * (a.num_kv_heads * G) + head;
      a.part_o[(static_cast<size_t>(split) * a.total_rows + row) * D + d] = val;
      if (d == 0)
        a.part_lse[static_cast<size_t>(split) * a.total_rows + row] =
            lt > 0.f ? sM[128 + r] + log2f(lt) : -INFINITY;
    } else {
      a.out[static_cast<size_t>(seq) * a.out_row_stride + head * D + d] = __float2bfloat16(val);
    }
  }
  // Unwind: never leave with TMA copies in flight into this CTA's shared memory.
  if (*abort_flag && warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s)
      if (issued_mask & (1u << s))
        if (!mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, kWaitBudgetNs))
          record_error(a.err, kErrTimeoutDrain);
  }
}

constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 16 * D * 2 + 160 * 4 + 16 * D * 4 + 64;

}  // namespace dec

__global__ void attn_combine_kernel(const float* part_o, const float* part_lse, bf16* out,
                                    int out_row_stride, int nrows, int heads, int splits);

void paged_decode_tma(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      at::Tensor& out, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                      int64_t group, double scale, int64_t num_splits,
                      const c10::optional<at::Tensor>& part_o,
                      const c10::optional<at::Tensor>& part_lse, at::Tensor& err) {
  using namespace dec;
  TORCH_CHECK(q.dim() == 3 && q.size(2) == D && q.stride(2) == 1 && q.stride(1) == D, "q layout");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == BS && k_cache.size(3) == D &&
                  k_cache.is_contiguous() && v_cache.is_contiguous(),
              "decode_tma: cache must be [blocks, Hkv, 16, 128] contiguous");
  TORCH_CHECK(group >= 1 && group <= 16, "decode_tma: group <= 16");
  const int B = seq_lens.size(0);
  if (B == 0) return;
  Args a;
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.q_row_stride = q.stride(0);
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.out_row_stride = out.stride(0);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = block_tables.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.num_kv_heads = k_cache.size(1);
  a.group = group;
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  a.num_splits = std::max<int64_t>(1, num_splits);
  a.part_o = nullptr;
  a.part_lse = nullptr;
  a.total_rows = q.size(0) * q.size(1);
  a.err = err.data_ptr<int>();
  a.num_blocks = static_cast<int>(k_cache.size(0));
  if (a.num_splits > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "split-KV needs workspaces");
    a.part_o = part_o->data_ptr<float>();
    a.part_lse = part_lse->data_ptr<float>();
  }
  const uint64_t rows = static_cast<uint64_t>(k_cache.size(0)) * k_cache.size(1) * BS;
  // Row coordinates are int32 (TMA) and computed in int from a checked block id.
  TORCH_CHECK(rows < (1ull << 31), "decode_tma: KV pool too large for int32 row coordinates");
  const CUtensorMap tk = make_tmap_bf16_2d(k_cache.data_ptr(), D, rows, D * 2, 64, BS,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tv = make_tmap_bf16_2d(v_cache.data_ptr(), D, rows, D * 2, 64, BS,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    attr = true;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  dim3 grid(B, a.num_kv_heads, a.num_splits);
  C10_CUDA_CHECK(launch_k(decode_kernel, grid, dim3(THREADS), SMEM, st, nullptr, 0, tk, tv, a));
  if (a.num_splits > 1) {
    const int nrows = a.total_rows;
    C10_CUDA_CHECK(launch_k(attn_combine_kernel, dim3(nrows), dim3(D), 0, st, nullptr, 0,
                            a.part_o, a.part_lse, a.out, a.out_row_stride, nrows,
                            static_cast<int>(q.size(1)), a.num_splits));
  }
}

}  // namespace lb
