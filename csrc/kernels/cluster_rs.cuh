// Split-K reduce-scatter for the S CTAs of a thread-block cluster, exchanged through L2 by the
// TMA engine, and the TMA-store epilogue of the owners (sm_100a).
//
// A GEMM tile of 128 weight rows x BT tokens is computed by the S CTAs of a cluster, each over
// one K range, with the fp32 accumulator in TMEM.  The tile's token columns are cut into
// 16-wide chunks; chunk c is owned by cluster rank c % S.
//
//   publish  every CTA copies its accumulator from TMEM to shared-memory slot c of each chunk;
//            one thread bulk-stores the chunks owned by peers to a global workspace slot
//            (tile, source, chunk) and waits for the writes;
//   barrier  one cluster barrier (release / acquire): a cluster is co-scheduled, so waiting
//            for peers cannot deadlock;
//   fetch    one thread per owner bulk-loads the peers' slots of its chunks (one 8 KB copy
//            each, completion on an mbarrier);
//   reduce   owners sum the S slots in rank order (deterministic), format the output chunk in
//            shared memory (bf16 + residual, SwiGLU, or fp32) and one thread writes it with a
//            2-D TMA store (the tensor map clips the M / N edges).
//
// Measured on B200: per-thread global stores from these CTAs drained at a few GB/s per SM,
// and distributed shared memory moved 128 KB partials at ~6-15 GB/s per SM; the TMA engine
// avoids both.  No multicast.
//
// Shared layout: slots [max(chunks, owned * S)][16 columns][128 rows] fp32 (8 KB each), then
// the owner's output staging, 8 KB per owned chunk.  Slot c holds this CTA's chunk c while
// publishing; after the barrier, slot oc * S + s receives source s's part of owned chunk
// oc * S + rank (the own part is already in place: c = oc * S + rank).
#pragma once

#include "common.cuh"

namespace lb {
namespace crs {

constexpr int CW = 16;                  // token columns per chunk
constexpr int SLOT_FLOATS = CW * 128;   // one chunk of one source
constexpr int SLOT_BYTES = SLOT_FLOATS * 4;
constexpr int OUT_BYTES = 16 * 128 * 4; // staged output of one chunk (fp32 worst case)

__host__ __device__ constexpr int num_chunks(int bt) { return bt / CW; }
__host__ __device__ constexpr int owned_chunks(int bt, int rank, int S) {
  return rank < num_chunks(bt) ? (num_chunks(bt) - rank + S - 1) / S : 0;
}
__host__ __device__ constexpr int num_slots(int bt, int S) {
  return num_chunks(bt) > owned_chunks(bt, 0, S) * S ? num_chunks(bt) : owned_chunks(bt, 0, S) * S;
}
// Shared memory the exchange and the output staging need (reuses the drained pipeline).
__host__ __device__ constexpr int smem_bytes(int bt, int S) {
  return num_slots(bt, S) * SLOT_BYTES + owned_chunks(bt, 0, S) * OUT_BYTES;
}
// Global workspace floats for `tiles` output tiles split S ways.
__host__ __device__ constexpr long long ws_floats(int tiles, int bt, int S) {
  return static_cast<long long>(tiles) * S * bt * 128;
}

__device__ __forceinline__ uint32_t ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// ws_tile: this tile's workspace region, [S sources][chunks][16][128] floats.
__device__ __forceinline__ float* ws_slot(float* ws_tile, int nc, int src, int c) {
  return ws_tile + static_cast<size_t>(src * nc + c) * SLOT_FLOATS;
}

// The 128 epilogue threads (e = 0..127; `row` = this thread's TMEM lane, tbase = TMEM address
// of that lane's column 0), once the accumulator is complete and the pipeline buffers idle.
// have_acc = false publishes zeros (empty K range or failed main loop).  Uses named barrier 1.
template <int BT>
__device__ __forceinline__ void publish(uint32_t tbase, bool have_acc, float* slots,
                                        float* ws_tile, uint32_t rank, uint32_t S, int row,
                                        int e) {
  constexpr int NC = num_chunks(BT);
  constexpr int PER = NC >= 2 ? 2 : 1;  // chunks per TMEM round trip
#pragma unroll 1
  for (int c0 = 0; c0 < NC; c0 += PER) {
    uint32_t r[16 * PER];
    if (have_acc) {
      if constexpr (PER == 2) tmem_ld32(tbase + c0 * CW, r);
      else tmem_ld16(tbase + c0 * CW, r);
      tc_wait_ld();
    } else {
#pragma unroll
      for (int j = 0; j < 16 * PER; ++j) r[j] = 0u;
    }
#pragma unroll
    for (int h = 0; h < PER; ++h) {
      float* d = slots + (c0 + h) * SLOT_FLOATS + row;
#pragma unroll
      for (int j = 0; j < 16; ++j) d[j * 128] = __uint_as_float(r[16 * h + j]);
    }
  }
  // generic-proxy shared writes -> visible to the bulk copies (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  named_bar_sync(1, 128);
  if (e == 0 && S > 1) {
    for (int c = 0; c < NC; ++c)
      if (c % S != rank) bulk_store(ws_slot(ws_tile, NC, rank, c), slots + c * SLOT_FLOATS, SLOT_BYTES);
    bulk_commit();
    bulk_wait_all0();
    // the peers read these writes with bulk copies after the cluster barrier
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
}

// After the cluster barrier, one thread of each owner: fetch the peers' slots of the owned
// chunks (rbar initialised with count 1, used once).
template <int BT>
__device__ __forceinline__ void fetch(float* slots, float* ws_tile, uint64_t* rbar,
                                      uint32_t rank, uint32_t S) {
  constexpr int NC = num_chunks(BT);
  const int n_own = owned_chunks(BT, rank, S);
  if (n_own == 0 || S == 1) return;
  asm volatile("fence.proxy.async.global;" ::: "memory");
  mbar_arrive_expect_tx(rbar, n_own * (S - 1) * SLOT_BYTES);
  for (int oc = 0; oc < n_own; ++oc) {
    const int c = oc * S + rank;
    for (uint32_t s = 0; s < S; ++s)
      if (s != rank)
        bulk_load(slots + (oc * S + s) * SLOT_FLOATS, ws_slot(ws_tile, NC, s, c), SLOT_BYTES, rbar);
  }
}

// All 128 epilogue threads: wait for the fetched slots, then for each owned chunk thread e
// sums weight rows 4 (e & 31) .. +3 of token columns (e >> 5) + 4 q (q < 4) over the S sources
// in rank order and calls epi(oc, first token column of the chunk, e >> 5, e & 31, acc[4]).
// Returns false if the fetch did not complete in time.
template <int BT, class Epi>
__device__ __forceinline__ bool reduce(const float* slots, uint64_t* rbar, uint32_t rank,
                                       uint32_t S, int e, volatile int* abort_flag, Epi&& epi) {
  const int n_own = owned_chunks(BT, rank, S);
  if (n_own == 0) return true;
  const bool ok = S == 1 || mbar_wait(rbar, 0, abort_flag);
  const int ew = e >> 5, el = e & 31;
#pragma unroll 1
  for (int oc = 0; oc < n_own; ++oc) {
    float4 acc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) {
      for (uint32_t s = 0; s < S; ++s) {
        const float* slot = slots + (oc * S + s) * SLOT_FLOATS + 4 * el;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = *reinterpret_cast<const float4*>(slot + (ew + 4 * q) * 128);
          acc[q].x += v.x;
          acc[q].y += v.y;
          acc[q].z += v.z;
          acc[q].w += v.w;
        }
      }
    }
    epi(oc, (oc * S + rank) * CW, ew, el, acc);
  }
  return ok;
}

__device__ __forceinline__ float silu_c(float x) { return x / (1.0f + __expf(-x)); }

// Output modes of stage_out / the tile tensor map.
enum OutMode : int { kOutBf16 = 0, kOutSwiGLU = 1, kOutF32 = 2 };

// Format one reduced chunk into its staging tile (row-major [16 tokens][box width], the layout
// of the 2-D TMA store box).  Thread (ew, el) holds rows 4 el .. +3 of token columns ew + 4 q.
// res (optional, bf16 mode): residual at (first token of the chunk, first row of the tile);
// rows_left / cols_left bound the residual reads.
__device__ __forceinline__ void stage_out(int mode, uint8_t* out, int ew, int el,
                                          float4 (&acc)[4], const bf16* res, int ldr,
                                          int rows_left, int cols_left) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int j = ew + 4 * q;
    if (mode == kOutSwiGLU) {
      // lanes 0..15 hold gate rows 0..63, lanes 16..31 the up rows of the same features
      float4 up;
      up.x = __shfl_down_sync(0xffffffffu, acc[q].x, 16);
      up.y = __shfl_down_sync(0xffffffffu, acc[q].y, 16);
      up.z = __shfl_down_sync(0xffffffffu, acc[q].z, 16);
      up.w = __shfl_down_sync(0xffffffffu, acc[q].w, 16);
      if (el < 16) {
        uint2 pk;
        pk.x = pack_bf16x2(silu_c(acc[q].x) * up.x, silu_c(acc[q].y) * up.y);
        pk.y = pack_bf16x2(silu_c(acc[q].z) * up.z, silu_c(acc[q].w) * up.w);
        *reinterpret_cast<uint2*>(out + (j * 64 + 4 * el) * 2) = pk;
      }
    } else if (mode == kOutF32) {
      *reinterpret_cast<float4*>(out + (j * 128 + 4 * el) * 4) = acc[q];
    } else {
      float v[4] = {acc[q].x, acc[q].y, acc[q].z, acc[q].w};
      if (res != nullptr && j < rows_left) {
        const bf16* rr = res + static_cast<size_t>(j) * ldr + 4 * el;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (4 * el + u < cols_left) v[u] += __bfloat162float(rr[u]);
      }
      uint2 pk;
      pk.x = pack_bf16x2(v[0], v[1]);
      pk.y = pack_bf16x2(v[2], v[3]);
      *reinterpret_cast<uint2*>(out + (j * 128 + 4 * el) * 2) = pk;
    }
  }
}

// After every owned chunk is staged (all 128 threads): one thread stores the tiles.  x0 = first
// output column of the tile in the tensor map's units, y(oc) = first token of owned chunk oc.
// wait_all: wait until the writes are performed (a completion signal follows), else only until
// shared memory may be released.
template <int BT>
__device__ __forceinline__ void store_out(const CUtensorMap* tmap, const uint8_t* out, int e,
                                          uint32_t rank, uint32_t S, int x0, int m0,
                                          bool wait_all) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  named_bar_sync(1, 128);
  if (e != 0) return;
  const int n_own = owned_chunks(BT, rank, S);
  for (int oc = 0; oc < n_own; ++oc)
    tma_store_2d(tmap, out + oc * OUT_BYTES, x0, m0 + (oc * S + rank) * CW);
  bulk_commit();
  if (wait_all) bulk_wait_all0();
  else bulk_wait_read0();
}

}  // namespace crs
}  // namespace lb
