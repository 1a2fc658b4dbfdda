// Split-K reduce-scatter for the S CTAs of a thread-block cluster, exchanged through L2 by the
// TMA engine, and the TMA-store epilogue of the owners (sm_100a).
//
// A GEMM tile of 128 weight rows x BT tokens is computed by the S CTAs of a cluster, each over
// one K range, with the fp32 accumulator in TMEM.  The tile's token columns are cut into
// 16-wide chunks; cluster rank r owns the contiguous chunks [r * own, r * own + owned(r)),
// own = ceil(chunks / S).
//
//   publish  every CTA copies its accumulator from TMEM into shared-memory slot c of each chunk
//            c (64 columns per TMEM round trip); one thread bulk-stores each peer's contiguous
//            run of chunks to the workspace region (tile, source, chunk) -- one copy per peer --
//            and waits for the writes;
//   barrier  one cluster barrier (release / acquire): a cluster is co-scheduled, so waiting
//            for peers cannot deadlock;
//   fetch    one thread per owner bulk-loads, from every peer, that peer's slots of the owned
//            chunks (one copy per peer, completion on an mbarrier);
//   reduce   each epilogue warp takes its own owned chunks (no CTA barrier): sums the S slots in
//            rank order (deterministic), formats the chunk's output in its first slot (bf16 +
//            residual, SwiGLU, or fp32) and writes it with a 2-D TMA store (the tensor map clips
//            the M / N edges).
//
// Measured on B200: per-thread global stores from these CTAs drained at a few GB/s per SM,
// distributed shared memory moved 128 KB partials at ~6-15 GB/s per SM, and every bulk / TMA
// operation costs ~0.2 us to issue; hence few, large TMA-engine copies.  No multicast.
//
// Shared layout: slots [S * own][16 columns][128 rows] fp32 (8 KB each).  Slot c holds this
// CTA's chunk c while publishing; after the barrier, slot s * own + oc holds source s's part of
// owned chunk r * own + oc (the own part, s = r, is already in place).  The output tile of owned
// chunk oc overwrites slot oc (its source-0 part) once the owning warp has read it.
#pragma once

#include "common.cuh"

namespace lb {
namespace crs {

constexpr int CW = 16;                  // token columns per chunk
constexpr int SLOT_FLOATS = CW * 128;   // one chunk of one source
constexpr int SLOT_BYTES = SLOT_FLOATS * 4;

__host__ __device__ constexpr int num_chunks(int bt) { return bt / CW; }
__host__ __device__ constexpr int own_max(int bt, int S) { return (num_chunks(bt) + S - 1) / S; }
__host__ __device__ constexpr int owned_chunks(int bt, int rank, int S) {
  return rank * own_max(bt, S) >= num_chunks(bt)
             ? 0
             : (num_chunks(bt) - rank * own_max(bt, S) < own_max(bt, S)
                    ? num_chunks(bt) - rank * own_max(bt, S)
                    : own_max(bt, S));
}
__host__ __device__ constexpr int num_slots(int bt, int S) { return S * own_max(bt, S); }
// Shared memory the exchange and the output staging need (reuses the drained pipeline).
__host__ __device__ constexpr int smem_bytes(int bt, int S) { return num_slots(bt, S) * SLOT_BYTES; }
// Rows of one output TMA box (one chunk).
__host__ __device__ constexpr int out_box_rows(int bt, int S) { return CW; }
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
                                        int e, unsigned long long* tr = nullptr) {
  constexpr int NC = num_chunks(BT);
  constexpr int PER = NC >= 8 ? 8 : NC >= 4 ? 4 : NC;  // chunks per TMEM round trip
#pragma unroll 1
  for (int c0 = 0; c0 < NC; c0 += PER) {
    uint32_t r[16 * PER];
    if (have_acc) {
      if constexpr (PER >= 4) {
#pragma unroll
        for (int h = 0; h < PER / 2; ++h)
          tmem_ld32(tbase + c0 * CW + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(r + 32 * h));
      } else if constexpr (PER == 2) {
        tmem_ld32(tbase + c0 * CW, *reinterpret_cast<uint32_t(*)[32]>(r));
      } else {
        tmem_ld16(tbase + c0 * CW, *reinterpret_cast<uint32_t(*)[16]>(r));
      }
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
  if (tr && e == 0) tr[0] = globaltimer_ns();
  // generic-proxy shared writes -> visible to the bulk copies (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  named_bar_sync(1, 128);
  if (tr && e == 0) tr[1] = globaltimer_ns();
  if (e == 0 && S > 1) {
    const int own = own_max(BT, S);
    for (uint32_t o = 0; o < S; ++o) {
      const int n = owned_chunks(BT, o, S);
      if (o != rank && n > 0)
        bulk_store(ws_slot(ws_tile, NC, rank, o * own), slots + o * own * SLOT_FLOATS,
                   n * SLOT_BYTES);
    }
    bulk_commit();
    if (tr) tr[2] = globaltimer_ns();
    bulk_wait_all0();
    if (tr) tr[3] = globaltimer_ns();
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
  const int own = own_max(BT, S);
  asm volatile("fence.proxy.async.global;" ::: "memory");
  mbar_arrive_expect_tx(rbar, n_own * (S - 1) * SLOT_BYTES);
  for (uint32_t s = 0; s < S; ++s)
    if (s != rank)
      bulk_load(slots + s * own * SLOT_FLOATS, ws_slot(ws_tile, NC, s, rank * own),
                n_own * SLOT_BYTES, rbar);
}

// All 128 epilogue threads: wait for the fetched slots; epilogue warp w (= e >> 5) reduces the
// owned chunks oc with oc % 4 == w on its own (no CTA barrier): lane l sums weight rows
// 4 l .. +3 of the chunk's 16 token columns over the S sources in rank order, then calls
// epi(oc, first token column of the chunk, lane, acc[16]) with acc[j] = rows 4 l .. +3 of
// column j.  epi may overwrite the chunk's first slot (only this warp reads it).  Returns false
// if the fetch did not complete in time.
template <int BT, class Epi>
__device__ __forceinline__ bool reduce(const float* slots, uint64_t* rbar, uint32_t rank,
                                       uint32_t S, int e, volatile int* abort_flag, Epi&& epi) {
  const int n_own = owned_chunks(BT, rank, S);
  if (n_own == 0) return true;
  const int own = own_max(BT, S);
  const bool ok = S == 1 || mbar_wait(rbar, 0, abort_flag);
  const int w = e >> 5, l = e & 31;
#pragma unroll 1
  for (int oc = w; oc < n_own; oc += 4) {
    float4 acc[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) {
      for (uint32_t s = 0; s < S; ++s) {
        const float* slot = slots + (s * own + oc) * SLOT_FLOATS + 4 * l;
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          const float4 v = *reinterpret_cast<const float4*>(slot + j * 128);
          acc[j].x += v.x;
          acc[j].y += v.y;
          acc[j].z += v.z;
          acc[j].w += v.w;
        }
      }
    }
    __syncwarp();  // every lane has read the chunk's slots before any lane overwrites them
    epi(oc, (rank * own + oc) * CW, l, acc);
  }
  return ok;
}

__device__ __forceinline__ float silu_c(float x) { return x / (1.0f + __expf(-x)); }

// Output modes of stage_out / the tile tensor map.
enum OutMode : int { kOutBf16 = 0, kOutSwiGLU = 1, kOutF32 = 2 };

// Output staging tile of owned chunk oc: its first slot (16 tokens x box width, <= 8 KB).
__device__ __forceinline__ uint8_t* out_tile(float* slots, uint32_t own, int oc) {
  return reinterpret_cast<uint8_t*>(slots + oc * SLOT_FLOATS);
}

// Format one reduced chunk into its staging tile (row-major [16 tokens][box width], the layout
// of the 2-D TMA store box).  Lane l holds rows 4 l .. +3 of every token column j (acc[j]).
// res (optional, bf16 mode): residual at (first token of the chunk, first row of the tile);
// rows_left / cols_left bound the residual reads.
__device__ __forceinline__ void stage_out(int mode, uint8_t* out, int l, float4 (&acc)[CW],
                                          const bf16* res, int ldr, int rows_left,
                                          int cols_left) {
#pragma unroll
  for (int j = 0; j < CW; ++j) {
    if (mode == kOutSwiGLU) {
      // lanes 0..15 hold gate rows 0..63, lanes 16..31 the up rows of the same features
      float4 up;
      up.x = __shfl_down_sync(0xffffffffu, acc[j].x, 16);
      up.y = __shfl_down_sync(0xffffffffu, acc[j].y, 16);
      up.z = __shfl_down_sync(0xffffffffu, acc[j].z, 16);
      up.w = __shfl_down_sync(0xffffffffu, acc[j].w, 16);
      if (l < 16) {
        uint2 pk;
        pk.x = pack_bf16x2(silu_c(acc[j].x) * up.x, silu_c(acc[j].y) * up.y);
        pk.y = pack_bf16x2(silu_c(acc[j].z) * up.z, silu_c(acc[j].w) * up.w);
        *reinterpret_cast<uint2*>(out + (j * 64 + 4 * l) * 2) = pk;
      }
    } else if (mode == kOutF32) {
      *reinterpret_cast<float4*>(out + (j * 128 + 4 * l) * 4) = acc[j];
    } else {
      float v[4] = {acc[j].x, acc[j].y, acc[j].z, acc[j].w};
      if (res != nullptr && j < rows_left) {
        const bf16* rr = res + static_cast<size_t>(j) * ldr + 4 * l;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (4 * l + u < cols_left) v[u] += __bfloat162float(rr[u]);
      }
      uint2 pk;
      pk.x = pack_bf16x2(v[0], v[1]);
      pk.y = pack_bf16x2(v[2], v[3]);
      *reinterpret_cast<uint2*>(out + (j * 128 + 4 * l) * 2) = pk;
    }
  }
}

// Right after stage_out of chunk oc (all 32 lanes of the owning warp): lane 0 writes the tile
// with a 2-D TMA store at (x0, first token of the chunk).
__device__ __forceinline__ void store_chunk(const CUtensorMap* tmap, const uint8_t* tile, int l,
                                            int x0, int y0) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (l == 0) {
    tma_store_2d(tmap, tile, x0, y0);
    bulk_commit();
  }
}

// After a warp's last store_chunk: lane 0 waits until its stores have read shared memory
// (wait_all: until the writes are performed, when a completion signal follows).
__device__ __forceinline__ void store_wait(int l, bool wait_all) {
  if (l == 0) {
    if (wait_all) bulk_wait_all0();
    else bulk_wait_read0();
  }
}

}  // namespace crs
}  // namespace lb
