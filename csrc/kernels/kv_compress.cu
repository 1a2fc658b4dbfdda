// KV-cache compression kernels: H2O attention-mass accumulation and paged KV compaction.
//
// Reference: H2O policy (src/cache/h2o_policy.rs:73-230: cumulative decayed attention per slot,
// decay 0.95, updated from the last layer's attention probabilities copied to the host every
// step, src/model/custom_transformer.rs:546-594) and token eviction by masking
// (src/cache/parallel_cache_builder.rs:1451-1840).  Here both stay on the device:
//
//  * h2o_accumulate: recomputes the last layer's attention probabilities of every query head
//    over the cached keys (logits + per-tile softmax partials, then the combination) and
//    updates score[pos] = decay * score[pos] + sum over heads of p(head, pos).  Scores live in a
//    pool parallel to the KV blocks ([num_blocks * block_size] fp32), so they move with their
//    blocks.
//  * kv_compact: copies selected token slots (all layers, K and V, every KV head) to new slots,
//    used after the host picks the tokens to keep (sinks + recent + heavy hitters).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

constexpr int HD = 128;

// ---------------------------------------------------------------------------------------
// H2O accumulation in two launches, both sized by the workspace (max sequences x max model
// length), reading the live lengths from the device -- so they can be captured in the decode
// CUDA graphs -- and deterministic (fixed reduction orders, no atomics).
//
//  h2o_logits_kernel  grid (key tiles, Hkv, B), 256 threads, one key per thread: the logits of
//                     the G query heads of this KV head (q pre-scaled in shared memory) go to
//                     ws_logits[b][h][key]; the tile's per-head max and sum of exp go to
//                     ws_part[b][h][tile] = (m, l).
//  h2o_accum_kernel   grid (key tiles, B): per head, M = max of the tiles' m and L = sum of
//                     l * exp(m - M); then for every key p < len:
//                     score[slot(p)] = decay * score[slot(p)] + sum_h exp(s_h(p) - M_h) / L_h.
// ---------------------------------------------------------------------------------------
constexpr int H2O_TILE = 256;
constexpr int H2O_MAXG = 16;

__global__ void __launch_bounds__(H2O_TILE) h2o_logits_kernel(
    const bf16* q, int q_stride, const bf16* k_cache, const int* block_tables, int bt_stride,
    const int* seq_lens, float* ws_logits, float2* ws_part, int hq, int hkv, int bs, int lmax,
    int tmax, float scale) {
  const int tile = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = hq / hkv;
  const int L = seq_lens[b];
  const int p0 = tile * H2O_TILE;
  float2* part = ws_part + (static_cast<size_t>(b) * hq + kvh * G) * tmax + tile;
  if (p0 >= L) {
    if (threadIdx.x < G) part[static_cast<size_t>(threadIdx.x) * tmax] = make_float2(-INFINITY, 0.f);
    return;
  }
  __shared__ float sq[H2O_MAXG][HD];
  __shared__ float red[8][H2O_MAXG];
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int g = i / HD, d = i % HD;
    sq[g][d] = __bfloat162float(q[static_cast<size_t>(b) * q_stride + (kvh * G + g) * HD + d]) *
               scale;
  }
  __syncthreads();
  const int p = p0 + threadIdx.x;
  const bool valid = p < L;
  float acc[H2O_MAXG];
#pragma unroll
  for (int g = 0; g < H2O_MAXG; ++g) acc[g] = 0.f;
  if (valid) {
    const int* bt = block_tables + static_cast<size_t>(b) * bt_stride;
    const int blk = bt[p / bs];
    const uint4* kr = reinterpret_cast<const uint4*>(
        k_cache + ((static_cast<size_t>(blk) * hkv + kvh) * bs + p % bs) * HD);
#pragma unroll 4
    for (int c = 0; c < HD / 8; ++c) {
      const uint4 v = __ldg(kr + c);
      const bf16* kv8 = reinterpret_cast<const bf16*>(&v);
      float kf[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) kf[j] = __bfloat162float(kv8[j]);
#pragma unroll
      for (int g = 0; g < H2O_MAXG; ++g) {
        if (g < G) {
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[g] = fmaf(sq[g][c * 8 + j], kf[j], acc[g]);
        }
      }
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* lrow = ws_logits + (static_cast<size_t>(b) * hq + kvh * G) * lmax;
  for (int g = 0; g < G; ++g) {
    if (valid) lrow[static_cast<size_t>(g) * lmax + p] = acc[g];
    const float m = warp_max(valid ? acc[g] : -INFINITY);
    if (lane == 0) red[warp][g] = m;
  }
  __syncthreads();
  float M[H2O_MAXG];
  for (int g = 0; g < G; ++g) {
    float m = -INFINITY;
    for (int w = 0; w < 8; ++w) m = fmaxf(m, red[w][g]);
    M[g] = m;
  }
  __syncthreads();
  for (int g = 0; g < G; ++g) {
    const float e = warp_sum(valid ? __expf(acc[g] - M[g]) : 0.f);
    if (lane == 0) red[warp][g] = e;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float l = 0.f;
    for (int w = 0; w < 8; ++w) l += red[w][g];
    part[static_cast<size_t>(g) * tmax] = make_float2(M[g], l);
  }
}

__global__ void __launch_bounds__(H2O_TILE) h2o_accum_kernel(
    const float* ws_logits, const float2* ws_part, const int* block_tables, int bt_stride,
    const int* seq_lens, float* score, int hq, int bs, int lmax, int tmax, float decay) {
  const int tile = blockIdx.x, b = blockIdx.y;
  const int L = seq_lens[b];
  const int p0 = tile * H2O_TILE;
  if (p0 >= L) return;
  extern __shared__ float s_ml[];  // [hq] max, [hq] 1 / sum
  const int ntiles = (L + H2O_TILE - 1) / H2O_TILE;
  for (int h = threadIdx.x; h < hq; h += blockDim.x) {
    const float2* part = ws_part + (static_cast<size_t>(b) * hq + h) * tmax;
    float M = -INFINITY;
    for (int t = 0; t < ntiles; ++t) M = fmaxf(M, part[t].x);
    float S = 0.f;
    for (int t = 0; t < ntiles; ++t) {
      const float2 v = part[t];
      if (v.y > 0.f) S += v.y * __expf(v.x - M);
    }
    s_ml[h] = M;
    s_ml[hq + h] = S > 0.f ? 1.f / S : 0.f;
  }
  __syncthreads();
  const int p = p0 + threadIdx.x;
  if (p >= L) return;
  const float* lcol = ws_logits + static_cast<size_t>(b) * hq * lmax + p;
  float sum = 0.f;
  for (int h = 0; h < hq; ++h) sum += __expf(lcol[static_cast<size_t>(h) * lmax] - s_ml[h]) * s_ml[hq + h];
  const int* bt = block_tables + static_cast<size_t>(b) * bt_stride;
  const size_t slot = static_cast<size_t>(bt[p / bs]) * bs + p % bs;
  score[slot] = score[slot] * decay + sum;
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

// q: [B, Hq, 128] (row stride q.stride(0)); k_cache: [NB, Hkv, BS, 128]; ws_logits: fp32
// [>= B, Hq, Lmax]; ws_part: fp32 [>= B, Hq, ceil(Lmax / 256), 2].  Every seq_len <= Lmax.
void h2o_accumulate(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& block_tables,
                    const at::Tensor& seq_lens, at::Tensor& score, double decay, double scale,
                    at::Tensor& ws_logits, at::Tensor& ws_part) {
  const int B = seq_lens.size(0);
  if (B == 0) return;
  TORCH_CHECK(q.size(-1) == HD && k_cache.size(3) == HD, "h2o: head dim 128");
  const int hq = q.size(1), hkv = k_cache.size(1);
  TORCH_CHECK(hq % hkv == 0 && hq / hkv <= H2O_MAXG, "h2o: group size <= 16");
  TORCH_CHECK(ws_logits.dim() == 3 && ws_logits.size(0) >= B && ws_logits.size(1) == hq &&
                  ws_logits.is_contiguous() && ws_logits.scalar_type() == at::kFloat,
              "h2o: logits workspace [>= B, Hq, Lmax] fp32");
  const int lmax = ws_logits.size(2);
  const int tmax = (lmax + H2O_TILE - 1) / H2O_TILE;
  TORCH_CHECK(ws_part.numel() >= static_cast<int64_t>(B) * hq * tmax * 2 &&
                  ws_part.is_contiguous() && ws_part.scalar_type() == at::kFloat,
              "h2o: partials workspace");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  float2* part = reinterpret_cast<float2*>(ws_part.data_ptr<float>());
  h2o_logits_kernel<<<dim3(tmax, hkv, B), H2O_TILE, 0, st>>>(
      reinterpret_cast<const bf16*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<const bf16*>(k_cache.data_ptr()), block_tables.data_ptr<int>(),
      block_tables.stride(0), seq_lens.data_ptr<int>(), ws_logits.data_ptr<float>(), part, hq,
      hkv, k_cache.size(2), lmax, tmax, static_cast<float>(scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  h2o_accum_kernel<<<dim3(tmax, B), H2O_TILE, 2 * hq * sizeof(float), st>>>(
      ws_logits.data_ptr<float>(), part, block_tables.data_ptr<int>(), block_tables.stride(0),
      seq_lens.data_ptr<int>(), score.data_ptr<float>(), hq, k_cache.size(2), lmax, tmax,
      static_cast<float>(decay));
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
