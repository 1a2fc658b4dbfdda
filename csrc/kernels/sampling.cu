// Token selection: greedy argmax (first max wins) or temperature + top-k + top-p + seeded
// sampling, one CTA per row, no sort of the vocabulary.
//
// Semantics follow the reference (src/sampling.rs:28-102, src/model_fuel/engine_model.rs:25-52):
//   * temperature <= 0 -> argmax, first maximum wins (src/model_fuel/generate.rs:54-65);
//   * logits / T; top-k keeps every logit >= the k-th largest (ties kept);
//   * top-p keeps the smallest descending prefix whose softmax mass reaches p (every logit
//     equal to the boundary one is kept);
//   * one seeded draw from the renormalised kept distribution, scanning kept tokens in index
//     order.
// Probability mass is accumulated as 2^-32 fixed-point integers so sums, and hence the selected
// token, do not depend on the order of atomics.  The uniform draw is SplitMix64 (Steele, Lea &
// Flood, 2014) of (row seed).
//
// Fast path (top-k set, the common serving case): pass 1 over the row takes the max / first
// argmax and a 4096-bin histogram of the top 12 bits of the order-preserving key of logit / T;
// the bin holding the k-th largest key bounds the candidates.  Pass 2 gathers every candidate
// (key, index) into shared memory, and the rest happens there on a few hundred entries: a
// bitonic sort by (key descending, index ascending) gives the exact top-k threshold and the
// top-p prefix, a second sort of the kept set by index gives the draw order.  Two reads of the
// row instead of ~12.  Rows without top-k, or whose candidate set exceeds CAND_CAP, take the
// general path: radix selection over the whole row (4 passes of 8-bit digits per threshold).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

constexpr int SThreads = 512;
constexpr int NBIN = 4096;       // histogram bins: top 12 bits of the key
constexpr int CAND_CAP = 4096;   // candidates held in shared memory by the fast path

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

// Block-wide argmax with first-index tie break.
__device__ __forceinline__ void block_argmax(float& mx, int& amx, float* fred, int* ired) {
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o);
    const int oa = __shfl_xor_sync(0xffffffffu, amx, o);
    if (om > mx || (om == mx && oa < amx)) {
      mx = om;
      amx = oa;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    fred[w] = mx;
    ired[w] = amx;
  }
  __syncthreads();
  if (w == 0) {
    mx = l < (blockDim.x >> 5) ? fred[l] : -INFINITY;
    amx = l < (blockDim.x >> 5) ? ired[l] : 0x7fffffff;
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

// Exclusive block scan of one 64-bit value per thread; returns the prefix, *total the sum.
__device__ __forceinline__ uint64_t block_excl_scan(uint64_t v, unsigned long long* sh,
                                                    uint64_t* total) {
  const int l = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint64_t incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (l >= o) incl += y;
  }
  __syncthreads();
  if (l == 31) sh[w] = incl;
  __syncthreads();
  if (w == 0) {
    uint64_t t = l < nw ? sh[l] : 0ull;
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xffffffffu, t, o);
      if (l >= o) t += y;
    }
    sh[l] = t;
  }
  __syncthreads();
  const uint64_t pre = incl - v + (w > 0 ? sh[w - 1] : 0ull);
  *total = sh[nw - 1];
  __syncthreads();
  return pre;
}

// In-place bitonic sort of n (a power of two <= CAND_CAP) 64-bit entries, ascending.
__device__ __forceinline__ void bitonic_sort(unsigned long long* a, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < (n >> 1); t += blockDim.x) {
        const int i = 2 * t - (t & (stride - 1));
        const int j = i + stride;
        const bool up = (i & size) == 0;
        const unsigned long long x = a[i], y = a[j];
        if ((x > y) == up) {
          a[i] = y;
          a[j] = x;
        }
      }
      __syncthreads();
    }
  }
}

// General path: thresholds by radix selection over the whole row (used when no top-k is set
// or the fast path's candidates overflow).  Returns through s_tok / s_lp (thread 0).
__device__ void select_radix(const float* x, int vocab, float invT, float smx, int k, float p,
                             int64_t seed, int amx, unsigned long long* hist,
                             unsigned int* hcount, unsigned long long* ured, int* ired,
                             int* s_tok, float* s_lp) {
  __shared__ uint32_t s_sel;
  __shared__ unsigned long long s_above;
  const int NT = blockDim.x;
  uint32_t thr_key = 0;  // keep keys >= thr_key
  if (k > 0 && k < vocab) {
    uint32_t prefix = 0, pmask = 0;
    int remaining = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += NT) hcount[b] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < vocab; i += NT) {
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
  uint64_t total = 0;
  for (int i = threadIdx.x; i < vocab; i += NT) {
    const float v = x[i] * invT;
    if (f2key(v) >= thr_key) total += mass_fx(v, smx);
  }
  total = block_reduce_sum<unsigned long long>(total, ured);
  if (p > 0.f && p < 1.f) {
    const uint64_t target = static_cast<uint64_t>(static_cast<double>(p) * static_cast<double>(total));
    uint32_t prefix = 0, pmask = 0;
    uint64_t above = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += NT) hist[b] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < vocab; i += NT) {
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
    if (prefix > thr_key) thr_key = prefix;
  }
  // draw: scan kept mass in index order (contiguous index ranges per thread)
  const int per = (vocab + NT - 1) / NT;
  const int i0 = threadIdx.x * per, i1 = min(vocab, i0 + per);
  uint64_t mine = 0;
  for (int i = i0; i < i1; ++i) {
    const float v = x[i] * invT;
    if (f2key(v) >= thr_key) mine += mass_fx(v, smx);
  }
  uint64_t kept_total = 0;
  const uint64_t excl = block_excl_scan(mine, ured, &kept_total);
  const uint64_t r = splitmix64(static_cast<uint64_t>(seed));
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
    *s_tok = ired[0];
    *s_lp = (x[ired[0]] * invT - smx) - logf(static_cast<float>(kept_total) / 4294967296.0f);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(SThreads, 2) sample_kernel(
    const float* logits, int ld, int vocab, const float* temperature, const int* top_k,
    const float* top_p, const int64_t* seeds, int* out_tokens, float* out_logprob) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ unsigned long long s_cand[];                  // CAND_CAP entries
  unsigned int* s_bins = reinterpret_cast<unsigned int*>(s_cand + CAND_CAP);  // NBIN counts
  __shared__ unsigned long long hist[256];
  __shared__ unsigned int hcount[256];
  __shared__ float fred[32];
  __shared__ unsigned long long ured[32];
  __shared__ int ired[32];
  __shared__ int s_n, s_kbin, s_tok;
  __shared__ float s_lp;
  const int NT = blockDim.x;
  const int row = blockIdx.x;
  const float* x = logits + static_cast<size_t>(row) * ld;
  const float T = temperature[row];
  const bool sampled = T > 0.f;
  const float invT = sampled ? 1.f / T : 1.f;
  const int k = top_k[row];
  const bool fast = sampled && k > 0 && k < vocab;
  const bool vec = (ld % 4 == 0) && (vocab % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(logits) % 16 == 0);

  // ---- pass 1: max / first argmax; key histogram of logit / T (fast path) ----
  if (fast)
    for (int b = threadIdx.x; b < NBIN; b += NT) s_bins[b] = 0;
  __syncthreads();
  float mx = -INFINITY;
  int amx = 0x7fffffff;
  auto see = [&](float v, int i) {
    if (v > mx) {
      mx = v;
      amx = i;
    }
    if (fast) atomicAdd(&s_bins[f2key(v * invT) >> 20], 1u);
  };
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int j = threadIdx.x; j < vocab / 4; j += NT) {
      const float4 q = x4[j];
      see(q.x, 4 * j);
      see(q.y, 4 * j + 1);
      see(q.z, 4 * j + 2);
      see(q.w, 4 * j + 3);
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += NT) see(x[i], i);
  }
  block_argmax(mx, amx, fred, ired);
  if (!sampled) {
    if (threadIdx.x == 0) {
      out_tokens[row] = amx;
      if (out_logprob) out_logprob[row] = 0.f;
    }
    return;
  }
  const float smx = mx * invT;  // max of scaled logits (T > 0 preserves order)
  const float p = top_p[row];

  // ---- fast path: the bin of the k-th largest key, then gather its candidates ----
  bool use_fast = fast;
  if (fast) {
    // thread t owns bins from the top: [NBIN - BPT (t + 1), NBIN - BPT t)
    constexpr int BPT = NBIN / SThreads;
    uint64_t local = 0;
    for (int j = 0; j < BPT; ++j) local += s_bins[NBIN - 1 - (threadIdx.x * BPT + j)];
    uint64_t tot = 0;
    const uint64_t pre = block_excl_scan(local, ured, &tot);
    if (threadIdx.x == 0) s_kbin = -1;
    __syncthreads();
    if (pre < static_cast<uint64_t>(k) && static_cast<uint64_t>(k) <= pre + local) {
      uint64_t acc = pre;
      for (int j = 0; j < BPT; ++j) {
        const int b = NBIN - 1 - (threadIdx.x * BPT + j);
        acc += s_bins[b];
        if (acc >= static_cast<uint64_t>(k)) {
          s_kbin = b;
          s_n = static_cast<int>(acc);   // candidates: every key in bins >= b
          break;
        }
      }
    }
    __syncthreads();
    use_fast = s_kbin >= 0 && s_n <= CAND_CAP;
  }
  if (!use_fast) {
    select_radix(x, vocab, invT, smx, k, p, seeds[row], amx, hist, hcount, ured, ired, &s_tok,
                 &s_lp);
    if (threadIdx.x == 0) {
      out_tokens[row] = s_tok;
      if (out_logprob) out_logprob[row] = s_lp;
    }
    return;
  }
  const int kbin = s_kbin;
  const int n = s_n;
  __syncthreads();                       // every thread has read s_n before it is reset
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();
  // ---- pass 2: gather (key, index) of every candidate; sort by key desc, index asc ----
  auto take = [&](float v, int i) {
    const uint32_t kk = f2key(v * invT);
    if (static_cast<int>(kk >> 20) >= kbin) {
      const int pos = atomicAdd(&s_n, 1);
      s_cand[pos] = (static_cast<unsigned long long>(kk) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
    }
  };
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int j = threadIdx.x; j < vocab / 4; j += NT) {
      const float4 q = x4[j];
      take(q.x, 4 * j);
      take(q.y, 4 * j + 1);
      take(q.z, 4 * j + 2);
      take(q.w, 4 * j + 3);
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += NT) take(x[i], i);
  }
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int i = n + threadIdx.x; i < n2; i += NT) s_cand[i] = 0ull;  // pads sort last
  __syncthreads();
  bitonic_sort(s_cand, n2);                       // ascending; the order used below is reversed
  auto key_at = [&](int r) { return static_cast<uint32_t>(s_cand[n2 - 1 - r] >> 32); };
  auto idx_at = [&](int r) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(s_cand[n2 - 1 - r]));
  };
  // top-k: keep ranks [0, kept) = every key >= the k-th largest
  const uint32_t kth = key_at(k - 1);
  if (threadIdx.x == 0) s_tok = n;
  __syncthreads();
  for (int r = threadIdx.x; r < n; r += NT)
    if (key_at(r) < kth && (r == 0 || key_at(r - 1) >= kth)) s_tok = r;
  __syncthreads();
  int kept = s_tok;
  // top-p: smallest descending prefix whose mass reaches p * total (whole key groups)
  if (p > 0.f && p < 1.f) {
    // thread t: ranks [t * per, (t + 1) * per)
    const int per = (kept + NT - 1) / NT;
    const int r0 = threadIdx.x * per, r1 = min(kept, r0 + per);
    uint64_t mine = 0;
    for (int r = r0; r < r1; ++r) mine += mass_fx(key2f(key_at(r)), smx);
    uint64_t total = 0;
    const uint64_t excl = block_excl_scan(mine, ured, &total);
    const uint64_t target = static_cast<uint64_t>(static_cast<double>(p) * static_cast<double>(total));
    if (threadIdx.x == 0) s_kbin = kept;   // reused: boundary rank
    __syncthreads();
    uint64_t acc = excl;
    for (int r = r0; r < r1; ++r) {
      const uint64_t before = acc;
      acc += mass_fx(key2f(key_at(r)), smx);
      if (before < target && acc >= target) s_kbin = r;   // unique crossing rank
      if (before >= target && r == 0 && target == 0) s_kbin = 0;
    }
    __syncthreads();
    const int jb = s_kbin;
    if (jb < kept) {
      const uint32_t bkey = key_at(jb);
      if (threadIdx.x == 0) s_tok = kept;
      __syncthreads();
      for (int r = threadIdx.x; r < kept; r += NT)
        if (key_at(r) < bkey && (r == 0 || key_at(r - 1) >= bkey)) s_tok = r;
      __syncthreads();
      kept = s_tok;
    }
  }
  // ---- draw: the kept set in index order ----
  __syncthreads();
  unsigned long long* s_kept = s_cand;   // rebuilt in place: (index << 32) | key, ascending
  {
    // read all kept entries before overwriting (kept <= n <= CAND_CAP: two steps via registers)
    constexpr int MAXPER = CAND_CAP / SThreads;
    unsigned long long tmp[MAXPER];
    int cnt = 0;
    for (int r = threadIdx.x; r < kept; r += NT)
      tmp[cnt++] = (static_cast<unsigned long long>(idx_at(r)) << 32) | key_at(r);
    __syncthreads();
    cnt = 0;
    for (int r = threadIdx.x; r < kept; r += NT) s_kept[r] = tmp[cnt++];
  }
  int m2 = 1;
  while (m2 < kept) m2 <<= 1;
  for (int i = kept + threadIdx.x; i < m2; i += NT) s_kept[i] = ~0ull;   // pads sort last
  __syncthreads();
  bitonic_sort(s_kept, m2);
  {
    const int per = (kept + NT - 1) / NT;
    const int r0 = threadIdx.x * per, r1 = min(kept, r0 + per);
    uint64_t mine = 0;
    for (int r = r0; r < r1; ++r) mine += mass_fx(key2f(static_cast<uint32_t>(s_kept[r])), smx);
    uint64_t kept_total = 0;
    const uint64_t excl = block_excl_scan(mine, ured, &kept_total);
    const uint64_t rr = splitmix64(static_cast<uint64_t>(seeds[row]));
    const double u = static_cast<double>(rr >> 11) * (1.0 / 9007199254740992.0);
    const uint64_t target = static_cast<uint64_t>(u * static_cast<double>(kept_total));
    if (threadIdx.x == 0) s_tok = amx;
    __syncthreads();
    if (mine > 0 && target >= excl && target < excl + mine) {
      uint64_t acc = excl;
      for (int r = r0; r < r1; ++r) {
        acc += mass_fx(key2f(static_cast<uint32_t>(s_kept[r])), smx);
        if (acc > target) {
          s_tok = static_cast<int>(s_kept[r] >> 32);
          break;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      out_tokens[row] = s_tok;
      if (out_logprob)
        out_logprob[row] = (x[s_tok] * invT - smx) - logf(static_cast<float>(kept_total) / 4294967296.0f);
    }
  }
  (void)n;
}

void sample_tokens(const at::Tensor& logits, const at::Tensor& temperature,
                   const at::Tensor& top_k, const at::Tensor& top_p, const at::Tensor& seeds,
                   at::Tensor& out_tokens, const c10::optional<at::Tensor>& out_logprob) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "sample: f32 logits");
  const int B = logits.size(0);
  if (B == 0) return;
  float* lp = nullptr;
  if (out_logprob.has_value() && out_logprob->defined()) lp = out_logprob->data_ptr<float>();
  constexpr size_t smem = CAND_CAP * sizeof(unsigned long long) + NBIN * sizeof(unsigned int);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
    attr = true;
  }
  C10_CUDA_CHECK(launch_k(sample_kernel, dim3(B), dim3(SThreads), smem,
                          at::cuda::getCurrentCUDAStream(), nullptr, 0,
                          logits.data_ptr<float>(), static_cast<int>(logits.stride(0)),
                          static_cast<int>(logits.size(1)), temperature.data_ptr<float>(),
                          top_k.data_ptr<int>(), top_p.data_ptr<float>(),
                          seeds.data_ptr<int64_t>(), out_tokens.data_ptr<int>(), lp));
}

}  // namespace lb
