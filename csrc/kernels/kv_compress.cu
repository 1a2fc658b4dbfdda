// KV-cache compression kernels: H2O attention-mass accumulation and paged KV compaction.
//
// Reference: H2O policy (src/cache/h2o_policy.rs:73-230: cumulative decayed attention per slot,
// decay 0.95, updated from the last layer's attention probabilities copied to the host every
// step, src/model/custom_transformer.rs:546-594) and token eviction by masking
// (src/cache/parallel_cache_builder.rs:1451-1840).  Here both stay on the device:
//
//  * h2o_accumulate: one CTA per sequence recomputes the last layer's attention probabilities
//    of every query head over the cached keys (two passes: row max / sum, then probabilities)
//    and updates score[pos] = decay * score[pos] + sum over heads of p(head, pos).  Scores live
//    in a pool parallel to the KV blocks ([num_blocks * block_size] fp32), so they move with
//    their blocks.
//  * kv_compact: copies selected token slots (all layers, K and V, every KV head) to new slots,
//    used after the host picks the tokens to keep (sinks + recent + heavy hitters).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

constexpr int HD = 128;

// q: [B, Hq, 128] (row stride q_stride), k_cache: [NB, Hkv, BS, 128]
__global__ void __launch_bounds__(256) h2o_accumulate_kernel(
    const bf16* q, int q_stride, const bf16* k_cache, const int* block_tables, int bt_stride,
    const int* seq_lens, float* score, int hq, int hkv, int bs, float scale, float decay) {
  const int seq = blockIdx.x;
  const int L = seq_lens[seq];
  const int* bt = block_tables + static_cast<size_t>(seq) * bt_stride;
  const int group = hq / hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float s_qf[HD];
  __shared__ float red_m[8], red_s[8];
  // decay every cached position once
  for (int p = threadIdx.x; p < L; p += blockDim.x) {
    const size_t slot = static_cast<size_t>(bt[p / bs]) * bs + p % bs;
    score[slot] *= decay;
  }
  __syncthreads();
  for (int h = 0; h < hq; ++h) {
    const int kvh = h / group;
    for (int d = threadIdx.x; d < HD; d += blockDim.x)
      s_qf[d] = __bfloat162float(q[static_cast<size_t>(seq) * q_stride + h * HD + d]) * scale;
    __syncthreads();
    // pass 1: max and sum of exp over keys (each warp takes keys w, w+8, ...)
    float m = -INFINITY, ssum = 0.f;
    for (int p = warp; p < L; p += 8) {
      const size_t slot = static_cast<size_t>(bt[p / bs]) * bs + p % bs;
      const bf16* kr = k_cache + (slot / bs * hkv + kvh) * bs * HD + (slot % bs) * HD;
      float dot = 0.f;
      for (int d = lane; d < HD; d += 32) dot += s_qf[d] * __bfloat162float(kr[d]);
      dot = warp_sum(dot);
      const float mn = fmaxf(m, dot);
      ssum = ssum * __expf(m - mn) + __expf(dot - mn);
      m = mn;
    }
    if (lane == 0) {
      red_m[warp] = m;
      red_s[warp] = ssum;
    }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < 8; ++w) M = fmaxf(M, red_m[w]);
    float S = 0.f;
    for (int w = 0; w < 8; ++w) S += red_m[w] == -INFINITY ? 0.f : red_s[w] * __expf(red_m[w] - M);
    const float inv = S > 0.f ? 1.f / S : 0.f;
    // pass 2: accumulate probabilities (one lane per key after the warp dot product)
    for (int p = warp; p < L; p += 8) {
      const size_t slot = static_cast<size_t>(bt[p / bs]) * bs + p % bs;
      const bf16* kr = k_cache + (slot / bs * hkv + kvh) * bs * HD + (slot % bs) * HD;
      float dot = 0.f;
      for (int d = lane; d < HD; d += 32) dot += s_qf[d] * __bfloat162float(kr[d]);
      dot = warp_sum(dot);
      if (lane == 0) score[slot] += __expf(dot - M) * inv;
    }
    __syncthreads();
  }
}

// storage: [layers, 2, NB, Hkv, BS, 128]; copy token slot src[i] -> dst[i] for every layer/head.
__global__ void kv_compact_kernel(bf16* storage, const int* src, const int* dst, int n,
                                  int layers, int nb, int hkv, int bs, float* score) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int s = src[i], t = dst[i];
  const int sb = s / bs, so = s % bs, tb = t / bs, to = t % bs;
  const size_t layer_stride = static_cast<size_t>(2) * nb * hkv * bs * HD;
  const size_t kv_stride = static_cast<size_t>(nb) * hkv * bs * HD;
  const int per = 2 * hkv * (HD / 8);  // uint4 per (layer) for K and V over all heads
  for (int l = 0; l < layers; ++l) {
    bf16* base = storage + l * layer_stride;
    for (int j = threadIdx.x; j < per; j += blockDim.x) {
      const int kv = j / (hkv * (HD / 8));
      const int rem = j % (hkv * (HD / 8));
      const int h = rem / (HD / 8), c = rem % (HD / 8);
      const uint4* srcp = reinterpret_cast<const uint4*>(
          base + kv * kv_stride + ((static_cast<size_t>(sb) * hkv + h) * bs + so) * HD) + c;
      uint4* dstp = reinterpret_cast<uint4*>(
          base + kv * kv_stride + ((static_cast<size_t>(tb) * hkv + h) * bs + to) * HD) + c;
      *dstp = *srcp;
    }
  }
  if (score != nullptr && threadIdx.x == 0) score[t] = score[s];
}

void h2o_accumulate(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& block_tables,
                    const at::Tensor& seq_lens, at::Tensor& score, double decay, double scale) {
  const int B = seq_lens.size(0);
  if (B == 0) return;
  TORCH_CHECK(q.size(-1) == HD && k_cache.size(3) == HD, "h2o: head dim 128");
  h2o_accumulate_kernel<<<B, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<const bf16*>(k_cache.data_ptr()), block_tables.data_ptr<int>(),
      block_tables.stride(0), seq_lens.data_ptr<int>(), score.data_ptr<float>(), q.size(1),
      k_cache.size(1), k_cache.size(2), static_cast<float>(scale), static_cast<float>(decay));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_compact(at::Tensor& storage, const at::Tensor& src, const at::Tensor& dst,
                const c10::optional<at::Tensor>& score) {
  const int n = src.size(0);
  if (n == 0) return;
  TORCH_CHECK(storage.dim() == 6 && storage.size(5) == HD && storage.is_contiguous(), "storage");
  float* sp = score.has_value() && score->defined() ? score->data_ptr<float>() : nullptr;
  kv_compact_kernel<<<n, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<bf16*>(storage.data_ptr()), src.data_ptr<int>(), dst.data_ptr<int>(), n,
      storage.size(0), storage.size(2), storage.size(3), storage.size(4), sp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lb
