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
//   reduce   owners sum the S slots in rank order (deterministic), format the output in shared
//            memory (bf16 + residual, SwiGLU, or fp32) and one thread writes it with 2-D TMA
//            stores (one store for all owned chunks when S divides the chunk count; the tensor
//            map clips the M / N edges).
//
// Measured on B200: per-thread global stores from these CTAs drained at a few GB/s per SM,
// distributed shared memory moved 128 KB partials at ~6-15 GB/s per SM, and every bulk / TMA
// operation costs ~0.2 us to issue; hence few, large TMA-engine copies.  No multicast.
//
// Shared layout: slots [S * own][16 columns][128 rows] fp32 (8 KB each).  Slot c holds this
// CTA's chunk c while publishing; after the barrier, slot s * own + oc holds source s's part of
// owned chunk r * own + oc (the own part, s = r, is already in place).  Output tile of owned
// chunk oc: bytes [oc * T, (oc + 1) * T) from the start of the slots, T = 16 x box width x
// element size <= 8 KB, written only after every thread has read slots 0 .. oc.
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
// Rows of one output TMA box: all owned chunks at once when every rank owns the same count.
__host__ __device__ constexpr int out_box_rows(int bt, int S) {
  return num_chunks(bt) % S == 0 ? CW * own_max(bt, S) : CW;
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
                                        int e, unsigned long long* tr = nullptr) {
  constexpr int NC = num_chunks(BT);
  constexpr int PER = NC >= 4 ? 4 : NC;  // chunks per TMEM round trip
#pragma unroll 1
  for (int c0 = 0; c0 < NC; c0 += PER) {
    uint32_t r[16 * PER];
    if (have_acc) {
      if constexpr (PER == 4) {
        tmem_ld32(tbase + c0 * CW, *reinterpret_cast<uint32_t(*)[32]>(r));
        tmem_ld32(tbase + c0 * CW + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
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

// All 128 epilogue threads: wait for the fetched slots, then for each owned chunk thread e
// sums weight rows 4 (e & 31) .. +3 of token columns (e >> 5) + 4 q (q < 4) over the S sources
// in rank order and, once every thread has read the chunk's slots (named barrier 1), calls
// epi(oc, first token column of the chunk, e >> 5, e & 31, acc[4]); epi may then write the
// output tile of chunk oc.  Returns false if the fetch did not complete in time.
template <int BT, class Epi>
__device__ __forceinline__ bool reduce(const float* slots, uint64_t* rbar, uint32_t rank,
                                       uint32_t S, int e, volatile int* abort_flag, Epi&& epi,
                                       unsigned long long* tr = nullptr) {
  const int n_own = owned_chunks(BT, rank, S);
  if (n_own == 0) return true;
  const int own = own_max(BT, S);
  const bool ok = S == 1 || mbar_wait(rbar, 0, abort_flag);
  if (tr && e == 0) tr[4] = globaltimer_ns();
  const int ew = e >> 5, el = e & 31;
#pragma unroll 1
  for (int oc = 0; oc < n_own; ++oc) {
    float4 acc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) {
      for (uint32_t s = 0; s < S; ++s) {
        const float* slot = slots + (s * own + oc) * SLOT_FLOATS + 4 * el;
        float4 v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = *reinterpret_cast<const float4*>(slot + (ew + 4 * q) * 128);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[q].x += v[q].x;
          acc[q].y += v[q].y;
          acc[q].z += v[q].z;
          acc[q].w += v[q].w;
        }
      }
    }
    named_bar_sync(1, 128);  // slots 0 .. oc are read: chunk oc's output tile may be written
    epi(oc, (rank * own + oc) * CW, ew, el, acc);
  }
  if (tr && e == 0) tr[5] = globaltimer_ns();
  return ok;
}

__device__ __forceinline__ float silu_c(float x) { return x / (1.0f + __expf(-x)); }

// Output modes of stage_out / the tile tensor map.
enum OutMode : int { kOutBf16 = 0, kOutSwiGLU = 1, kOutF32 = 2 };

__host__ __device__ constexpr int out_tile_bytes(int mode) {
  return mode == kOutSwiGLU ? CW * 64 * 2 : mode == kOutF32 ? CW * 128 * 4 : CW * 128 * 2;
}
__device__ __forceinline__ uint8_t* out_tile(float* slots, int mode, int oc) {
  return reinterpret_cast<uint8_t*>(slots) + oc * out_tile_bytes(mode);
}

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
// output column of the tile in the tensor map's units, m0 = first token of the tile.  The
// tensor map's box is out_box_rows(BT, S) rows high.  wait_all: wait until the writes are
// performed (a completion signal follows), else only until shared memory may be released.
template <int BT>
__device__ __forceinline__ void store_out(const CUtensorMap* tmap, float* slots, int mode, int e,
                                          uint32_t rank, uint32_t S, int x0, int m0,
                                          bool wait_all, unsigned long long* tr = nullptr) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  named_bar_sync(1, 128);
  if (e != 0) return;
  if (tr) tr[6] = globaltimer_ns();
  const int n_own = owned_chunks(BT, rank, S);
  if (n_own == 0) return;
  const int first = m0 + rank * own_max(BT, S) * CW;
  if (out_box_rows(BT, S) > CW) {
    tma_store_2d(tmap, out_tile(slots, mode, 0), x0, first);
  } else {
    for (int oc = 0; oc < n_own; ++oc)
      tma_store_2d(tmap, out_tile(slots, mode, oc), x0, first + oc * CW);
  }
  bulk_commit();
  if (wait_all) bulk_wait_all0();
  else bulk_wait_read0();
  if (tr) tr[7] = globaltimer_ns();
}

}  // namespace crs
}  // namespace lb
