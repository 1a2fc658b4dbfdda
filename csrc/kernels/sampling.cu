// Token selection: greedy argmax (first max wins) or temperature + top-k + top-p + seeded
// sampling, one CTA per row, no sort.
//
// Semantics follow the reference (src/sampling.rs:28-102, src/model_fuel/engine_model.rs:25-52):
//   * temperature <= 0 -> argmax, first maximum wins (src/model_fuel/generate.rs:54-65);
//   * logits / T; top-k keeps every logit >= the k-th largest (ties kept);
//   * top-p keeps the smallest descending prefix whose softmax mass reaches p;
//   * one seeded draw from the renormalised kept distribution.
// Thresholds are found by radix selection over order-preserving 32-bit keys (4 passes of
// 8-bit digits) instead of sorting the vocabulary.  Probability mass is accumulated as
// 2^-32 fixed-point integers so the histogram sums, and hence the selected token, do not
// depend on the order of shared-memory atomics.  The uniform draw is SplitMix64 (Steele,
// Lea & Flood, 2014) of (row seed).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

constexpr int SThreads = 1024;

__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(b);
}

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

template <typename T>
__device__ __forceinline__ T block_reduce_sum(T v, T* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (blockDim.x >> 5) ? sh[l] : T(0);
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

__device__ __forceinline__ uint64_t mass_fx(float x, float mx) {
  // exp(x - mx) in [0, 1] as 2^-32 fixed point.
  return static_cast<uint64_t>(__expf(x - mx) * 4294967296.0f);
}

__global__ void __launch_bounds__(SThreads) sample_kernel(
    const float* logits, int ld, int vocab, const float* temperature, const int* top_k,
    const float* top_p, const int64_t* seeds, int* out_tokens, float* out_logprob) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const float* x = logits + static_cast<size_t>(row) * ld;
  const float T = temperature[row];
  __shared__ unsigned long long hist[256];
  __shared__ unsigned int hcount[256];
  __shared__ float fred[32];
  __shared__ unsigned long long ured[32];
  __shared__ int ired[32];
  __shared__ uint32_t s_prefix, s_mask_bits, s_sel;
  __shared__ unsigned long long s_above;

  // ---- pass 1: max and first argmax ----
  float mx = -INFINITY;
  int amx = 0x7fffffff;
  for (int i = threadIdx.x; i < vocab; i += SThreads) {
    const float v = x[i];
    if (v > mx) {
      mx = v;
      amx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o);
    const int oa = __shfl_xor_sync(0xffffffffu, amx, o);
    if (om > mx || (om == mx && oa < amx)) {
      mx = om;
      amx = oa;
    }
  }
  {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
      fred[w] = mx;
      ired[w] = amx;
    }
    __syncthreads();
    if (w == 0) {
      mx = fred[l];
      amx = ired[l];
      for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oa = __shfl_xor_sync(0xffffffffu, amx, o);
        if (om > mx || (om == mx && oa < amx)) {
          mx = om;
          amx = oa;
        }
      }
      if (l == 0) {
        fred[0] = mx;
        ired[0] = amx;
      }
    }
    __syncthreads();
    mx = fred[0];
    amx = ired[0];
    __syncthreads();
  }
  if (!(T > 0.f)) {
    if (threadIdx.x == 0) {
      out_tokens[row] = amx;
      if (out_logprob) out_logprob[row] = 0.f;
    }
    return;
  }
  const float invT = 1.f / T;
  const float smx = mx * invT;  // max of scaled logits (T > 0 preserves order)

  // ---- top-k threshold (k-th largest scaled logit) by radix selection ----
  uint32_t thr_key = 0;  // keep keys >= thr_key
  const int k = top_k[row];
  if (k > 0 && k < vocab) {
    uint32_t prefix = 0, pmask = 0;
    int remaining = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += SThreads) hcount[b] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < vocab; i += SThreads) {
        const uint32_t kk = f2key(x[i] * invT);
        if ((kk & pmask) == prefix) atomicAdd(&hcount[(kk >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int acc = 0, b = 255;
        for (; b > 0; --b) {
          if (acc + static_cast<int>(hcount[b]) >= remaining) break;
          acc += hcount[b];
        }
        s_sel = b;
        s_above = static_cast<unsigned long long>(acc);
      }
      __syncthreads();
      remaining -= static_cast<int>(s_above);
      prefix |= s_sel << shift;
      pmask |= 255u << shift;
      __syncthreads();
    }
    thr_key = prefix;
  }

  // ---- top-p threshold over the kept set ----
  uint64_t total = 0;
  for (int i = threadIdx.x; i < vocab; i += SThreads) {
    const float v = x[i] * invT;
    if (f2key(v) >= thr_key) total += mass_fx(v, smx);
  }
  total = block_reduce_sum<unsigned long long>(total, ured);
  const float p = top_p[row];
  if (p > 0.f && p < 1.f) {
    const uint64_t target = static_cast<uint64_t>(static_cast<double>(p) * static_cast<double>(total));
    uint32_t prefix = 0, pmask = 0;
    uint64_t above = 0;  // mass of keys strictly above the current prefix range
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += SThreads) hist[b] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < vocab; i += SThreads) {
        const float v = x[i] * invT;
        const uint32_t kk = f2key(v);
        if (kk >= thr_key && (kk & pmask) == prefix)
          atomicAdd(&hist[(kk >> shift) & 255u], static_cast<unsigned long long>(mass_fx(v, smx)));
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        uint64_t acc = above;
        int b = 255;
        for (; b > 0; --b) {
          if (acc + hist[b] >= target) break;
          acc += hist[b];
        }
        s_sel = b;
        s_above = acc;
      }
      __syncthreads();
      above = s_above;
      prefix |= s_sel << shift;
      pmask |= 255u << shift;
      __syncthreads();
    }
    // The bucket reached at full depth is a single key value: keep every key >= it.
    if (prefix > thr_key) thr_key = prefix;
  }

  // ---- draw: scan kept mass in index order ----
  const int per = (vocab + SThreads - 1) / SThreads;
  const int i0 = threadIdx.x * per, i1 = min(vocab, i0 + per);
  uint64_t mine = 0;
  for (int i = i0; i < i1; ++i) {
    const float v = x[i] * invT;
    if (f2key(v) >= thr_key) mine += mass_fx(v, smx);
  }
  // exclusive scan of per-thread masses (warp shuffles + warp totals)
  uint64_t incl = mine;
  const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (l >= o) incl += y;
  }
  if (l == 31) ured[w] = incl;
  __syncthreads();
  if (w == 0) {
    uint64_t v = ured[l];
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xffffffffu, v, o);
      if (l >= o) v += y;
    }
    ured[l] = v;  // inclusive warp-prefix
  }
  __syncthreads();
  const uint64_t kept_total = ured[31];
  const uint64_t excl = incl - mine + (w > 0 ? ured[w - 1] : 0ull);
  const uint64_t r = splitmix64(static_cast<uint64_t>(seeds[row]));
  const double u = static_cast<double>(r >> 11) * (1.0 / 9007199254740992.0);
  const uint64_t target = static_cast<uint64_t>(u * static_cast<double>(kept_total));
  if (threadIdx.x == 0) ired[0] = amx;  // fallback: argmax
  __syncthreads();
  if (mine > 0 && target >= excl && target < excl + mine) {
    uint64_t acc = excl;
    for (int i = i0; i < i1; ++i) {
      const float v = x[i] * invT;
      if (f2key(v) >= thr_key) {
        acc += mass_fx(v, smx);
        if (acc > target) {
          ired[0] = i;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int tok = ired[0];
    out_tokens[row] = tok;
    if (out_logprob) {
      const float v = x[tok] * invT;
      out_logprob[row] = (v - smx) - logf(static_cast<float>(kept_total) / 4294967296.0f);
    }
  }
}

void sample_tokens(const at::Tensor& logits, const at::Tensor& temperature,
                   const at::Tensor& top_k, const at::Tensor& top_p, const at::Tensor& seeds,
                   at::Tensor& out_tokens, const c10::optional<at::Tensor>& out_logprob) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "sample: f32 logits");
  const int B = logits.size(0);
  if (B == 0) return;
  float* lp = nullptr;
  if (out_logprob.has_value() && out_logprob->defined()) lp = out_logprob->data_ptr<float>();
  C10_CUDA_CHECK(launch_k(sample_kernel, dim3(B), dim3(SThreads), 0,
                          at::cuda::getCurrentCUDAStream(), nullptr, 0,
                          logits.data_ptr<float>(), static_cast<int>(logits.stride(0)),
                          static_cast<int>(logits.size(1)), temperature.data_ptr<float>(),
                          top_k.data_ptr<int>(), top_p.data_ptr<float>(),
                          seeds.data_ptr<int64_t>(), out_tokens.data_ptr<int>(), lp));
}

}  // namespace lb
