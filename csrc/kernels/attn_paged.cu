// Paged attention over a block-table KV cache (decode, chunked prefill, speculative verify).
//
// Reference sites replaced: manual attention with host-built dense masks and materialised
// GQA expansion (src/model/custom_attention.rs:250-674,741-858, masks from
// src/cache/parallel_cache_builder.rs:2232-2370) and the CPU-only Fuel PagedAttn
// (src/model_fuel/batched.rs:932-943).  Masks are implicit here: causal index math against
// per-sequence lengths and block tables.
//
// Layout: k_cache / v_cache are [num_blocks, Hkv, BS, D] (one (block, head) is a contiguous
// BS*D*2-byte run).  q is [T, Hq, D] with an arbitrary row stride (it is read straight out
// of the fused QKV buffer).  Query rows are packed as (token, head-in-group) so that the G
// query heads sharing a KV head consume each K/V tile from shared memory once.
//
// Two CTA shapes over one body (templated on DECODE):
//  * prefill / verify: 4 warps x 16 rows = 64 query rows per CTA, each warp sweeps all keys.
//  * decode: one 16-row tile (<= 16 packed rows), the 4 warps split every 64-key tile
//    (16 keys each) and merge their softmax states at the end; optional split-KV across
//    CTAs with a separate combine kernel.
// Tensor-core math is mma.sync m16n8k16 (bf16 in, fp32 accumulate); decode is bound by
// HBM reads of K/V, which this layout streams with 16-byte cp.async.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

constexpr int AD = 128;      // head dim (Llama family)
constexpr int AN = 64;       // keys per tile
constexpr int AROWS = 16;    // rows per warp tile
constexpr int ATHREADS = 128;

struct AttnArgs {
  const bf16* q;
  int q_row_stride;  // elements between consecutive tokens
  const bf16* k_cache;
  const bf16* v_cache;
  bf16* out;
  int out_row_stride;
  const int* block_tables;
  int bt_stride;
  const int* seq_lens;  // total KV length per sequence (including new tokens)
  const int* cu_q;      // [num_seqs + 1] query offsets
  const int* tile_seq;  // prefill: work item -> sequence
  const int* tile_row0; // prefill: work item -> first packed row within the sequence
  int num_kv_heads;
  int group;            // query heads per KV head
  int block_size;
  float scale_log2;     // softmax scale * log2(e)
  int num_splits;       // decode split-KV
  float* part_o;        // [splits, T*Hq, D]
  float* part_lse;      // [splits, T*Hq]
  int total_rows;       // T * Hq
  int causal;
  int num_blocks;       // KV pool size: block ids outside [0, num_blocks) are rejected
  int* err;             // error word (nullptr: not reported)
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Swizzled [rows][128] bf16 tile: 16-byte chunk c of row r lives at chunk (c ^ (r & 7)).
__device__ __forceinline__ int swz(int r, int c) { return r * AD + ((c ^ (r & 7)) << 3); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Load keys [kbase, kbase + AN) of (seq, kvh) into a swizzled smem tile (zero past kv_len).
__device__ __forceinline__ void load_kv_tile(bf16* sK, bf16* sV, const AttnArgs& a,
                                             const int* btab, int kvh, int kbase, int kv_len) {
  // 64 rows x 16 chunks = 1024 chunks per tensor, 8 per thread.
#pragma unroll
  for (int i = 0; i < (AN * 16) / ATHREADS; ++i) {
    const int idx = threadIdx.x + i * ATHREADS;
    const int r = idx >> 4, c = idx & 15;
    const int key = kbase + r;
    bool ok = key < kv_len;
    const int kk = ok ? key : 0;
    int blk = btab[kk / a.block_size];
    if (static_cast<unsigned>(blk) >= static_cast<unsigned>(a.num_blocks)) {
      // corrupt block table: report, read nothing (the key is zero-filled and masked)
      if (ok && a.err != nullptr) record_error(a.err, kErrBounds);
      blk = 0;
      ok = false;
    }
    const size_t off = ((static_cast<size_t>(blk) * a.num_kv_heads + kvh) * a.block_size +
                        (kk % a.block_size)) * AD + c * 8;
    cp_async16(sK + swz(r, c), a.k_cache + off, ok);
    cp_async16(sV + swz(r, c), a.v_cache + off, ok);
  }
}

template <bool DECODE>
__global__ void __launch_bounds__(ATHREADS) paged_attn_kernel(const AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);                  // 64 x 128
  bf16* sK = sQ + 64 * AD;                                        // 2 x 64 x 128
  bf16* sV = sK + 2 * AN * AD;                                    // 2 x 64 x 128
  float* sMerge = reinterpret_cast<float*>(sV + 2 * AN * AD);     // decode merge scratch

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int kvh = blockIdx.y;

  int seq, row0, nrows_seq;
  if (DECODE) {
    seq = blockIdx.x;
    row0 = 0;
  } else {
    seq = a.tile_seq[blockIdx.x];
    row0 = a.tile_row0[blockIdx.x];
  }
  const int q_start = a.cu_q[seq];
  const int q_len = a.cu_q[seq + 1] - q_start;
  const int kv_len = a.seq_lens[seq];
  nrows_seq = q_len * a.group;
  const int* btab = a.block_tables + static_cast<size_t>(seq) * a.bt_stride;
  const int tile_rows = DECODE ? AROWS : 64;

  // ---- load Q (packed rows) ----
  for (int idx = threadIdx.x; idx < tile_rows * 16; idx += ATHREADS) {
    const int r = idx >> 4, c = idx & 15;
    const int pr = row0 + r;
    const bool ok = pr < nrows_seq;
    const int tok = ok ? pr / a.group : 0;
    const int h = kvh * a.group + (ok ? pr % a.group : 0);
    const bf16* src = a.q + static_cast<size_t>(q_start + tok) * a.q_row_stride + h * AD + c * 8;
    cp_async16(sQ + swz(r, c), src, ok);
  }

  // Key range for this CTA (decode split-KV).
  int k_begin = 0, k_end = kv_len;
  if (DECODE && a.num_splits > 1) {
    const int per = ((kv_len + a.num_splits - 1) / a.num_splits + AN - 1) / AN * AN;
    k_begin = blockIdx.z * per;
    k_end = min(kv_len, k_begin + per);
  }
  // Causal bound: the last query row of this tile sees keys < kv_len - q_len + last_tok + 1.
  int k_limit = k_end;
  if (a.causal) {
    const int last_row = min(row0 + tile_rows, nrows_seq) - 1;
    const int last_tok = last_row / a.group;
    k_limit = min(k_end, kv_len - q_len + last_tok + 1);
  }
  const int ntiles = k_limit > k_begin ? (k_limit - k_begin + AN - 1) / AN : 0;

  if (ntiles > 0) load_kv_tile(sK, sV, a, btab, kvh, k_begin, kv_len);
  cp_async_commit();

  // Per-thread state: rows (g) and (g + 8) of this warp's 16-row tile.
  const int wrow0 = DECODE ? 0 : warp * AROWS;
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  // Query position of each of this thread's two rows (for the causal mask).
  int qpos[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int pr = row0 + wrow0 + g + 8 * h;
    qpos[h] = pr < nrows_seq ? (kv_len - q_len + pr / a.group) : -1;
  }

  uint32_t qf[8][4];  // Q fragments for the 8 k-chunks of D=128
  bool q_loaded = false;

  for (int tI = 0; tI < ntiles; ++tI) {
    const int buf = tI & 1;
    if (tI + 1 < ntiles)
      load_kv_tile(sK + (buf ^ 1) * AN * AD, sV + (buf ^ 1) * AN * AD, a, btab, kvh,
                   k_begin + (tI + 1) * AN, kv_len);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (!q_loaded) {
#pragma unroll
      for (int kc = 0; kc < 8; ++kc) {
        const int r = wrow0 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kc * 2 + (lane >> 4);
        ldsm_x4(qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3], sQ + swz(r, c));
      }
      q_loaded = true;
    }
    const bf16* K = sK + buf * AN * AD;
    const bf16* V = sV + buf * AN * AD;
    const int kbase = k_begin + tI * AN;

    // Keys handled by this warp within the tile.
    constexpr int NT = DECODE ? 2 : 8;  // n-tiles of 8 keys
    const int key0 = DECODE ? warp * 16 : 0;
    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < 8; ++kc) {
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = key0 + j * 8 + (lane & 7) + (lane >> 4) * 8;
        const int c = kc * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, K + swz(r, c));
        mma_bf16(s[j], qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3], b0, b1);
        mma_bf16(s[j + 1], qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3], b2, b3);
      }
    }
    // Mask + online softmax (base-2 exponent with the scale folded in).
    float mnew[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int key = kbase + key0 + j * 8 + 2 * t4 + (e & 1);
        float x = s[j][e] * a.scale_log2;
        const bool valid = key < k_end && (!a.causal || key <= qpos[h]) && qpos[h] >= 0;
        x = valid ? x : -INFINITY;
        s[j][e] = x;
        mnew[h] = fmaxf(mnew[h], x);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mnew[h] = fmaxf(mnew[h], __shfl_xor_sync(0xffffffffu, mnew[h], 1));
      mnew[h] = fmaxf(mnew[h], __shfl_xor_sync(0xffffffffu, mnew[h], 2));
    }
    float corr[2], msafe[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      msafe[h] = mnew[h] == -INFINITY ? 0.f : mnew[h];
      corr[h] = exp2f(m_r[h] - msafe[h]);
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
    uint32_t pf[NT][2];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const float p0 = exp2f(s[j][0] - msafe[0]);
      const float p1 = exp2f(s[j][1] - msafe[0]);
      const float p2 = exp2f(s[j][2] - msafe[1]);
      const float p3 = exp2f(s[j][3] - msafe[1]);
      l_r[0] += p0 + p1;
      l_r[1] += p2 + p3;
      pf[j][0] = pack_bf16x2(p0, p1);
      pf[j][1] = pack_bf16x2(p2, p3);
    }
    // O += P V
#pragma unroll
    for (int kc = 0; kc < NT / 2; ++kc) {
      const uint32_t a0 = pf[2 * kc][0], a1 = pf[2 * kc][1];
      const uint32_t a2 = pf[2 * kc + 1][0], a3 = pf[2 * kc + 1][1];
#pragma unroll
      for (int dn = 0; dn < 16; dn += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = key0 + kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dn + (lane >> 4);
        ldsm_x4_t(b0, b1, b2, b3, V + swz(r, c));
        mma_bf16(o[dn], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[dn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Row sums across the quad.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
  }

  if (DECODE) {
    // Merge the 4 warps' partial states (same rows, disjoint keys) through shared memory.
    float* sm = sMerge;                    // [4][16] max, [4][16] sum
    float* so = sMerge + 160;              // [16][128] accumulated output
    __syncthreads();
    if (t4 == 0) {
      sm[warp * 16 + g] = m_r[0];
      sm[warp * 16 + g + 8] = m_r[1];
      sm[64 + warp * 16 + g] = l_r[0];
      sm[64 + warp * 16 + g + 8] = l_r[1];
    }
    for (int i = threadIdx.x; i < 16 * AD; i += ATHREADS) so[i] = 0.f;
    __syncthreads();
    float scale_w[2], mtot[2], ltot[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + 8 * h;
      float mm = -INFINITY;
      for (int w = 0; w < 4; ++w) mm = fmaxf(mm, sm[w * 16 + r]);
      const float ms = mm == -INFINITY ? 0.f : mm;
      float lt = 0.f;
      for (int w = 0; w < 4; ++w) lt += sm[64 + w * 16 + r] * exp2f(sm[w * 16 + r] - ms);
      scale_w[h] = exp2f(m_r[h] - ms);
      mtot[h] = mm;
      ltot[h] = lt;
    }
    for (int w = 0; w < 4; ++w) {
      if (warp == w) {
#pragma unroll
        for (int dn = 0; dn < 16; ++dn) {
          const int d = dn * 8 + 2 * t4;
          so[g * AD + d] += o[dn][0] * scale_w[0];
          so[g * AD + d + 1] += o[dn][1] * scale_w[0];
          so[(g + 8) * AD + d] += o[dn][2] * scale_w[1];
          so[(g + 8) * AD + d + 1] += o[dn][3] * scale_w[1];
        }
      }
      __syncthreads();
    }
    // Write: row r = packed (token, head); 128 threads cover 16 rows x 128 dims.
    if (warp == 0 && t4 == 0) {
      sm[128 + g] = mtot[0];
      sm[128 + g + 8] = mtot[1];
      sm[144 + g] = ltot[0];
      sm[144 + g + 8] = ltot[1];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 16 * AD; i += ATHREADS) {
      const int r = i / AD, d = i % AD;
      const int pr = row0 + r;
      if (pr >= nrows_seq) continue;
      const int tok = pr / a.group;
      const int h = kvh * a.group + pr % a.group;
      const float lt = sm[144 + r];
      if (a.num_splits > 1) {
        const size_t row = static_cast<size_t>(q_start + tok) * (a.num_kv_heads * a.group) + h;
        const size_t nrow_all = static_cast<size_t>(a.total_rows);
        a.part_o[(blockIdx.z * nrow_all + row) * AD + d] = lt > 0.f ? so[i] / lt : 0.f;
        if (d == 0) {
          const float mt = sm[128 + r];
          a.part_lse[blockIdx.z * nrow_all + row] = lt > 0.f ? (mt + log2f(lt)) : -INFINITY;
        }
      } else {
        a.out[static_cast<size_t>(q_start + tok) * a.out_row_stride + h * AD + d] =
            __float2bfloat16(lt > 0.f ? so[i] / lt : 0.f);
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int pr = row0 + wrow0 + g + 8 * h;
      if (pr >= nrows_seq) continue;
      const int tok = pr / a.group;
      const int head = kvh * a.group + pr % a.group;
      const float inv = l_r[h] > 0.f ? 1.f / l_r[h] : 0.f;
      bf16* dst = a.out + static_cast<size_t>(q_start + tok) * a.out_row_stride + head * AD;
#pragma unroll
      for (int dn = 0; dn < 16; ++dn) {
        const int d = dn * 8 + 2 * t4;
        *reinterpret_cast<uint32_t*>(dst + d) =
            pack_bf16x2(o[dn][2 * h] * inv, o[dn][2 * h + 1] * inv);
      }
    }
  }
}

// Combine split-KV partials: out = sum_s exp2(lse_s - lse) * o_s.
__global__ void attn_combine_kernel(const float* part_o, const float* part_lse, bf16* out,
                                    int out_row_stride, int nrows, int heads, int splits) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;  // token * heads + head
  const int d = threadIdx.x;   // 0..127
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_lse[static_cast<size_t>(s) * nrows + row]);
  float acc = 0.f, wsum = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float w = exp2f(part_lse[static_cast<size_t>(s) * nrows + row] - mx);
      wsum += w;
      acc += w * part_o[(static_cast<size_t>(s) * nrows + row) * AD + d];
    }
  }
  const int tok = row / heads, h = row % heads;
  out[static_cast<size_t>(tok) * out_row_stride + h * AD + d] =
      __float2bfloat16(wsum > 0.f ? acc / wsum : 0.f);
}

static int attn_smem_bytes(bool decode) {
  int b = (64 * AD + 4 * AN * AD) * 2;
  if (decode) b += (160 + 16 * AD) * 4;
  return b;
}

void paged_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                     at::Tensor& out, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                     const at::Tensor& cu_q, const c10::optional<at::Tensor>& tile_seq,
                     const c10::optional<at::Tensor>& tile_row0, int64_t group, double scale,
                     bool decode, int64_t num_splits, const c10::optional<at::Tensor>& part_o,
                     const c10::optional<at::Tensor>& part_lse, bool causal,
                     const c10::optional<at::Tensor>& err) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16,
              "paged_attention: bf16 q / cache");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == AD && q.stride(2) == 1 && q.stride(1) == AD,
              "paged_attention: q must be [T, Hq, 128] with contiguous heads");
  TORCH_CHECK(out.dim() == 3 && out.stride(2) == 1 && out.stride(1) == AD, "out layout");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == AD && k_cache.is_contiguous(), "k_cache");
  const int num_seqs = seq_lens.size(0);
  if (num_seqs == 0) return;
  AttnArgs a;
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.q_row_stride = q.stride(0);
  a.k_cache = reinterpret_cast<const bf16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const bf16*>(v_cache.data_ptr());
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.out_row_stride = out.stride(0);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = block_tables.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.cu_q = cu_q.data_ptr<int>();
  a.num_kv_heads = k_cache.size(1);
  a.block_size = k_cache.size(2);
  a.group = group;
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  a.causal = causal ? 1 : 0;
  a.num_splits = 1;
  a.part_o = nullptr;
  a.part_lse = nullptr;
  a.total_rows = q.size(0) * q.size(1);
  a.tile_seq = nullptr;
  a.tile_row0 = nullptr;
  a.num_blocks = static_cast<int>(k_cache.size(0));
  a.err = (err.has_value() && err->defined()) ? err->data_ptr<int>() : nullptr;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (decode) {
    TORCH_CHECK(group <= AROWS, "decode path packs <= 16 rows per KV head");
    const int splits = std::max<int64_t>(1, num_splits);
    if (splits > 1) {
      TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "split-KV needs workspaces");
      a.num_splits = splits;
      a.part_o = part_o->data_ptr<float>();
      a.part_lse = part_lse->data_ptr<float>();
    }
    const int smem = attn_smem_bytes(true);
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(paged_attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem);
      attr = true;
    }
    dim3 grid(num_seqs, a.num_kv_heads, splits);
    C10_CUDA_CHECK(launch_k(paged_attn_kernel<true>, grid, dim3(ATHREADS), smem, st, nullptr, 0, a));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    if (splits > 1) {
      const int nrows = q.size(0) * q.size(1);
      C10_CUDA_CHECK(launch_k(attn_combine_kernel, dim3(nrows), dim3(AD), 0, st, nullptr, 0,
                              a.part_o, a.part_lse, a.out, a.out_row_stride, nrows,
                              static_cast<int>(q.size(1)), splits));
    }
  } else {
    TORCH_CHECK(tile_seq.has_value() && tile_row0.has_value(), "prefill needs tile lists");
    a.tile_seq = tile_seq->data_ptr<int>();
    a.tile_row0 = tile_row0->data_ptr<int>();
    const int ntiles = tile_seq->size(0);
    if (ntiles == 0) return;
    const int smem = attn_smem_bytes(false);
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(paged_attn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem);
      attr = true;
    }
    dim3 grid(ntiles, a.num_kv_heads, 1);
    C10_CUDA_CHECK(launch_k(paged_attn_kernel<false>, grid, dim3(ATHREADS), smem, st, nullptr, 0, a));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

}  // namespace lb
