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
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_dsmem4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

template <int BT, int STAGES, int QBITS>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmX,
                  const Args a) {
  using L = Smem<BT, STAGES, QBITS>;
  constexpr int CH = L::CH;
  constexpr int TMEM_COLS = BT < 32 ? 32 : BT;
  static_assert(BW * BT * 4 <= STAGES * L::STAGE, "partial must fit");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  // stage s: [W bf16 16 KB | X BT*128 | Q staging]; W and X stay 1024-aligned
  auto sW = [&](int s) { return smem + s * L::STAGE; };
  auto sX = [&](int s) { return smem + s * L::STAGE + L::W_BYTES; };
  auto sQ = [&](int s) { return smem + s * L::STAGE + L::W_BYTES + L::X_BYTES; };
  float* sPart = reinterpret_cast<float*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* ready = bars + STAGES;
  uint64_t* empty = bars + 2 * STAGES;
  uint64_t* tfull = bars + 3 * STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_go = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t S = nctarank(), rank = ctarank();
  const int tile = blockIdx.x / S;
  const int mt = tile % a.m_tiles, nt = tile / a.m_tiles;
  const int kb0 = rank * a.kb_per_split;
  const int kb1 = min(kb0 + a.kb_per_split, a.kb_total);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
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
    for (int kb = kb0; kb < kb1; ++kb) {
      int go = 1;
      if (!mbar_wait(&full[stage], phase, abort_flag)) {
        record_error(a.err, kErrTimeoutTmaFull);
        *abort_flag = 1;
        go = 0;
      }
      go = __all_sync(0xffffffffu, go);
      if (!go) break;
      // 64 values of row `row` at k = kb*64 .. +63
      float v[64];
      if constexpr (QBITS == 4) {
        const uint4* src = reinterpret_cast<const uint4*>(sQ(stage) + row * 32);
        const uint4 p0 = src[0], p1 = src[1];
        const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i * 8 + j] = static_cast<float>((w[i] >> (4 * j)) & 0xF);
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(sQ(stage) + row * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 p = src[i];
          const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
          for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              v[i * 16 + t * 4 + j] = static_cast<float>(static_cast<int8_t>((w[t] >> (8 * j)) & 0xFF));
        }
      }
      // per-group scale / offset (group >= 32 divides 64 or is a multiple of it)
      const int k0 = kb * BK;
      uint8_t* wdst = sW(stage) + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 16-byte chunk c holds k0 + 8c .. +7
        const int g = (k0 + c * 8) / a.group;
        float sc = 0.f, of = 0.f;
        if (n < a.N) {
          sc = __half2float(a.scales[static_cast<size_t>(n) * gpr + g]);
          of = __half2float(a.offsets[static_cast<size_t>(n) * gpr + g]);
        }
        uint4 outv;
        outv.x = pack_bf16x2(v[c * 8 + 0] * sc - of, v[c * 8 + 1] * sc - of);
        outv.y = pack_bf16x2(v[c * 8 + 2] * sc - of, v[c * 8 + 3] * sc - of);
        outv.z = pack_bf16x2(v[c * 8 + 4] * sc - of, v[c * 8 + 5] * sc - of);
        outv.w = pack_bf16x2(v[c * 8 + 6] * sc - of, v[c * 8 + 7] * sc - of);
        *reinterpret_cast<uint4*>(wdst + ((c ^ (row & 7)) << 4)) = outv;
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
    // ---- accumulator -> own shared-memory partial ----
    const int quad = warp & 3, trow = quad * 32 + lane;
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
    if (s_go[0] == 1) {
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BT; c += CH) {
        uint32_t r[CH];
        if constexpr (CH == 32) tmem_ld32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(r));
        else tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < CH; ++j) sPart[(c + j) * BW + trow] = __uint_as_float(r[j]);
      }
    } else {
      for (int c = 0; c < BT; ++c) sPart[c * BW + trow] = 0.f;
    }
  }

  tc_fence_before();
  cluster_sync();

  if (warp >= 2) {
    constexpr int NQ = CH / 4;
    const int e = threadIdx.x - 64, ew = e >> 5, el = e & 31;
    const int m0 = mt * BT;
    const uint32_t my_part = smem_u32(sPart);
#pragma unroll 1
    for (int ci = rank; ci < BT / CH; ci += S) {
      const int c = ci * CH;
      float4 acc[NQ];
#pragma unroll
      for (int qq = 0; qq < NQ; ++qq) acc[qq] = make_float4(0.f, 0.f, 0.f, 0.f);
      const uint32_t coff = (c * BW + e * 4) * 4;
      for (uint32_t sp = 0; sp < S; ++sp) {
        const uint32_t b = mapa(my_part, sp) + coff;
        float4 x[NQ];
#pragma unroll
        for (int qq = 0; qq < NQ; ++qq) x[qq] = ld_dsmem4(b + qq * 128 * 16);
#pragma unroll
        for (int qq = 0; qq < NQ; ++qq) {
          acc[qq].x += x[qq].x;
          acc[qq].y += x[qq].y;
          acc[qq].z += x[qq].z;
          acc[qq].w += x[qq].w;
        }
      }
#pragma unroll
      for (int qq = 0; qq < NQ; ++qq) {
        const int m = m0 + c + 4 * qq + ew;
        const int r0 = 4 * el;
        if (a.mode == 1) {
          float4 up;
          up.x = __shfl_down_sync(0xffffffffu, acc[qq].x, 16);
          up.y = __shfl_down_sync(0xffffffffu, acc[qq].y, 16);
          up.z = __shfl_down_sync(0xffffffffu, acc[qq].z, 16);
          up.w = __shfl_down_sync(0xffffffffu, acc[qq].w, 16);
          const int f = nt * 64 + r0;
          if (el < 16 && m < a.M && f < (a.N >> 1)) {
            uint2 pk;
            pk.x = pack_bf16x2(silu_f(acc[qq].x) * up.x, silu_f(acc[qq].y) * up.y);
            pk.y = pack_bf16x2(silu_f(acc[qq].z) * up.z, silu_f(acc[qq].w) * up.w);
            *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(a.C) +
                                      static_cast<size_t>(m) * a.ldc + f) = pk;
          }
        } else {
          const int nn = nt * BW + r0;
          if (m < a.M && nn < a.N) {
            const float vv[4] = {acc[qq].x, acc[qq].y, acc[qq].z, acc[qq].w};
            if (a.mode == 2) {
              float* Cp = reinterpret_cast<float*>(a.C) + static_cast<size_t>(m) * a.ldc;
              for (int u = 0; u < 4 && nn + u < a.N; ++u) Cp[nn + u] = vv[u];
            } else {
              bf16* Cp = reinterpret_cast<bf16*>(a.C) + static_cast<size_t>(m) * a.ldc;
              if (nn + 3 < a.N && a.vec_ok) {
                uint2 pk;
                pk.x = pack_bf16x2(vv[0], vv[1]);
                pk.y = pack_bf16x2(vv[2], vv[3]);
                *reinterpret_cast<uint2*>(Cp + nn) = pk;
              } else {
                for (int u = 0; u < 4 && nn + u < a.N; ++u) Cp[nn + u] = __float2bfloat16(vv[u]);
              }
            }
          }
        }
      }
    }
  }
  cluster_sync();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace q

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

CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swz);

template <int BT, int STAGES, int QBITS>
static void launch_q(const CUtensorMap& tq, const CUtensorMap& tx, const q::Args& a, int S,
                     cudaStream_t st) {
  using L = q::Smem<BT, STAGES, QBITS>;
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
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, q::gemm_q_kernel<BT, STAGES, QBITS>, tq, tx, a));
}

// X [M, K] bf16; qw [N, K*bits/8] uint8; scales / offsets [N, K/group] fp16.
void gemm_quant(const at::Tensor& X, const at::Tensor& qw, const at::Tensor& scales,
                const at::Tensor& offsets, int64_t bits, int64_t group, at::Tensor& C,
                int64_t mode, int64_t splits, at::Tensor& err) {
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
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
#define LB_Q(BTV, STV)                                                    \
  if (bits == 4) launch_q<BTV, STV, 4>(tq, tx, a, S, st);                 \
  else launch_q<BTV, STV, 8>(tq, tx, a, S, st);
  switch (BT) {
    case 16: LB_Q(16, 6) break;
    case 32: LB_Q(32, 6) break;
    case 64: LB_Q(64, 6) break;
    case 128: LB_Q(128, 4) break;
    default: LB_Q(256, 3) break;
  }
#undef LB_Q
}

}  // namespace lb
