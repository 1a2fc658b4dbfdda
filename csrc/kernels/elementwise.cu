// Row-wise kernels: token embedding gather, RMSNorm (optionally fused with the residual
// add), and fused rotate-half RoPE + paged KV append.
//
// Reference sites: embedding (src/model/custom_transformer.rs:461), RMSNorm and fused
// add+RMSNorm via candle-layer-norm (src/model/fused_rmsnorm.rs:47-110, block usage
// src/model/custom_transformer_block.rs:329,348), RoPE (src/model/custom_attention.rs:687-728,
// tables src/model/custom_transformer.rs:403-438) and the KV append gather/where/scatter
// (src/cache/parallel_cache_builder.rs:128-185).  Here RoPE uses per-row positions (the
// reference shares one index_pos across a decode batch, custom_transformer.rs:512-520) and
// the rotated K / V are written straight into their paged slots in the same pass.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace lb {

// ---------------------------------------------------------------------------------------
// Token forwarding for overlapped decode: ids[i] = last[src[i]] where src[i] >= 0 (the
// input token of row i is the previous step's sampled token of row src[i], still on the
// device); rows with src[i] < 0 keep the host-provided id.
// ---------------------------------------------------------------------------------------
__global__ void forward_tokens_kernel(int* ids, const int* src, const int* last, int n,
                                      int last_n, int* err) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int s = src[i];
  if (s < 0) return;
  if (s >= last_n) {
    record_error(err, kErrBounds);
    return;
  }
  ids[i] = last[s];
}

// ---------------------------------------------------------------------------------------
// Embedding: out[t, :] = table[ids[t], :]
// ---------------------------------------------------------------------------------------
__global__ void embed_kernel(const int* ids, const bf16* table, bf16* out, int hidden,
                             int vocab, int* err) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) record_error(err, kErrBounds);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

// ---------------------------------------------------------------------------------------
// RMSNorm.  If `residual` is given: residual <- residual + x (rounded to bf16 once), and
// y = norm(residual) * w.  Otherwise y = norm(x) * w.  One CTA per row, 16-byte vectors.
// ---------------------------------------------------------------------------------------
template <int VPT>
__global__ void rmsnorm_kernel(const bf16* x, int ldx, bf16* residual, int ldr, const bf16* w,
                               bf16* y, int ldy, int hidden, float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int nvec = hidden / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      uint4 raw = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * ldx)[vi];
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
      if (residual != nullptr) {
        uint4 rr = reinterpret_cast<const uint4*>(residual + static_cast<size_t>(row) * ldr)[vi];
        const bf16* re = reinterpret_cast<const bf16*>(&rr);
        uint4 outv;
        bf16* oe = reinterpret_cast<bf16*>(&outv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bf16 s = __float2bfloat16(__bfloat162float(e[j]) + __bfloat162float(re[j]));
          oe[j] = s;
          v[i][j] = __bfloat162float(s);
        }
        reinterpret_cast<uint4*>(residual + static_cast<size_t>(row) * ldr)[vi] = outv;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(e[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / hidden + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      uint4 wr = reinterpret_cast<const uint4*>(w)[vi];
      const bf16* we = reinterpret_cast<const bf16*>(&wr);
      uint4 outv;
      bf16* oe = reinterpret_cast<bf16*>(&outv);
#pragma unroll
      for (int j = 0; j < 8; ++j) oe[j] = __float2bfloat16(v[i][j] * inv * __bfloat162float(we[j]));
      reinterpret_cast<uint4*>(y + static_cast<size_t>(row) * ldy)[vi] = outv;
    }
  }
}

// ---------------------------------------------------------------------------------------
// RoPE + KV append.  qkv: [T, (Hq + 2 Hkv) * D] (q rotated in place).  cos_sin: [P, R]
// fp32 (first R/2 = cos, next R/2 = sin), R <= D the rotary width (the true head_dim when
// heads are zero-padded to D; lanes >= R are copied unrotated).  slot[t] = block * BS +
// offset (int32, < 0: skip).  Cache: [num_blocks, Hkv, BS, D].
// ---------------------------------------------------------------------------------------
__global__ void rope_kv_kernel(bf16* qkv, int ld, const int* positions, const int* slots,
                               const float* cos_sin, int max_pos, bf16* k_cache, bf16* v_cache,
                               int hq, int hkv, int head_dim, int rot_dim, int block_size,
                               int* err) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  int pos = positions[t];
  if (pos < 0 || pos >= max_pos) {
    if (threadIdx.x == 0) record_error(err, kErrBounds);
    pos = 0;
  }
  const int half = rot_dim / 2;
  const float* cs = cos_sin + static_cast<size_t>(pos) * rot_dim;
  bf16* row = qkv + static_cast<size_t>(t) * ld;
  const int64_t slot = slots != nullptr ? static_cast<int64_t>(slots[t]) : -1;
  const int64_t blk = slot >= 0 ? slot / block_size : 0;
  const int off = slot >= 0 ? static_cast<int>(slot % block_size) : 0;
  // rotate q and k heads: each thread handles one (head, i) pair for i < half.
  const int nrot = (hq + hkv) * half;
  for (int idx = threadIdx.x; idx < nrot; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    bf16* base = row + h * head_dim;
    const float x1 = __bfloat162float(base[i]);
    const float x2 = __bfloat162float(base[i + half]);
    const float c = cs[i], s = cs[half + i];
    const bf16 r1 = __float2bfloat16(x1 * c - x2 * s);
    const bf16 r2 = __float2bfloat16(x1 * s + x2 * c);
    if (h < hq) {
      base[i] = r1;
      base[i + half] = r2;
    } else if (slot >= 0) {
      const int kh = h - hq;
      bf16* dst = k_cache + ((blk * hkv + kh) * block_size + off) * head_dim;
      dst[i] = r1;
      dst[i + half] = r2;
    }
  }
  // k lanes beyond the rotary width (zero padding) are copied as they are
  if (slot >= 0 && rot_dim < head_dim) {
    const int extra = head_dim - rot_dim;
    for (int idx = threadIdx.x; idx < hkv * extra; idx += blockDim.x) {
      const int kh = idx / extra, dd = rot_dim + idx % extra;
      k_cache[((blk * hkv + kh) * block_size + off) * head_dim + dd] =
          row[(hq + kh) * head_dim + dd];
    }
  }
  if (slot >= 0) {
    const bf16* vsrc = row + (hq + hkv) * head_dim;
    const int nv = hkv * head_dim / 8;
    for (int idx = threadIdx.x; idx < nv; idx += blockDim.x) {
      const int kh = (idx * 8) / head_dim, d = (idx * 8) % head_dim;
      bf16* dst = v_cache + ((blk * hkv + kh) * block_size + off) * head_dim + d;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(vsrc + idx * 8);
    }
  }
}

// ---------------------------------------------------------------------------------------
// RoPE + KV append for 128-wide heads, one warp per (token, head): q heads [0, Hq) are rotated
// in place, k heads [Hq, Hq + Hkv) rotated into their paged K slot, v heads copied into the V
// slot.  Lane l holds elements 4 l .. 4 l + 3; the rotate-half partner of element i < R / 2 is
// i + R / 2, i.e. lane l + R / 8, fetched with one shuffle.  Optional per-head RMSNorm of q and
// k before RoPE (Qwen3: q_norm / k_norm weights of width D, RMS over the true head_dim, result
// rounded to bf16 as a separate norm op would), reference src/model/awq_qwen3.rs:259-267.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    rope_kv_warp_kernel(bf16* qkv, int ld, const int* positions, const int* slots,
                        const float* cos_sin, int max_pos, bf16* k_cache, bf16* v_cache, int T,
                        int hq, int hkv, int rot_dim, int block_size, const bf16* q_norm,
                        const bf16* k_norm, int norm_dim, float eps, int* err) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = 128;
  const int heads = hq + 2 * hkv;
  const long long gw = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (gw >= static_cast<long long>(T) * heads) return;       // warp-uniform
  const int t = static_cast<int>(gw / heads), h = static_cast<int>(gw % heads);
  const int lane = threadIdx.x & 31;
  bf16* src = qkv + static_cast<size_t>(t) * ld + static_cast<size_t>(h) * D;
  const int64_t slot = slots != nullptr ? static_cast<int64_t>(slots[t]) : -1;
  const int64_t blk = slot >= 0 ? slot / block_size : 0;
  const int off = slot >= 0 ? static_cast<int>(slot % block_size) : 0;
  if (h >= hq + hkv) {                                        // v head: 16 lanes x 16 bytes
    if (slot >= 0 && lane < 16) {
      const int kh = h - hq - hkv;
      bf16* dst = v_cache + ((blk * hkv + kh) * block_size + off) * D + lane * 8;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src + lane * 8);
    }
    return;
  }
  int pos = positions[t];
  if (pos < 0 || pos >= max_pos) {
    if (lane == 0) record_error(err, kErrBounds);
    pos = 0;
  }
  const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
  float v[4];
  {
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 a = __bfloat1622float2(p2[0]), b = __bfloat1622float2(p2[1]);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
  const bf16* nw = h < hq ? q_norm : k_norm;
  if (nw != nullptr) {                                        // per-head RMSNorm
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / norm_dim + eps);
    const uint2 wr = *reinterpret_cast<const uint2*>(nw + lane * 4);
    const bf16* we = reinterpret_cast<const bf16*>(&wr);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      v[i] = __bfloat162float(__float2bfloat16(v[i] * inv * __bfloat162float(we[i])));
  }
  const int half = rot_dim >> 1;
  const int e0 = lane * 4;
  const bool rot = e0 < rot_dim;
  const bool first = e0 < half;
  const int plane = !rot ? lane : (first ? lane + (half >> 2) : lane - (half >> 2));
  float pv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) pv[i] = __shfl_sync(0xffffffffu, v[i], plane);
  float o[4] = {v[0], v[1], v[2], v[3]};
  if (rot) {
    const float* cs = cos_sin + static_cast<size_t>(pos) * rot_dim;
    const int j0 = first ? e0 : e0 - half;                     // pair index of element 0
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float c = cs[j0 + i], sn = cs[half + j0 + i];
      // rotate-half: (x1, x2) -> (x1 c - x2 s, x1 s + x2 c)
      o[i] = first ? v[i] * c - pv[i] * sn : pv[i] * sn + v[i] * c;
    }
  }
  uint2 out;
  out.x = pack_bf16x2(o[0], o[1]);
  out.y = pack_bf16x2(o[2], o[3]);
  if (h < hq) {
    *reinterpret_cast<uint2*>(src + lane * 4) = out;
  } else if (slot >= 0) {
    const int kh = h - hq;
    bf16* dst = k_cache + ((blk * hkv + kh) * block_size + off) * D + lane * 4;
    *reinterpret_cast<uint2*>(dst) = out;
  }
}

// ---------------------------------------------------------------------------------------
// Host wrappers
// ---------------------------------------------------------------------------------------
void forward_tokens(at::Tensor& ids, const at::Tensor& src, const at::Tensor& last,
                    at::Tensor& err) {
  const int n = ids.size(0);
  if (n == 0) return;
  TORCH_CHECK(ids.scalar_type() == at::kInt && src.scalar_type() == at::kInt &&
                  last.scalar_type() == at::kInt && src.size(0) >= n && ids.is_contiguous() &&
                  src.is_contiguous() && last.is_contiguous(),
              "forward_tokens: contiguous int32 tensors");
  C10_CUDA_CHECK(launch_k(forward_tokens_kernel, dim3((n + 127) / 128), dim3(128), 0,
                          at::cuda::getCurrentCUDAStream(), nullptr, 0, ids.data_ptr<int>(),
                          src.data_ptr<int>(), last.data_ptr<int>(), n,
                          static_cast<int>(last.size(0)), err.data_ptr<int>()));
}

void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, at::Tensor& err) {
  const int T = ids.size(0);
  if (T == 0) return;
  const int hidden = table.size(1);
  TORCH_CHECK(hidden % 8 == 0 && table.is_contiguous() && out.is_contiguous(), "embedding");
  C10_CUDA_CHECK(launch_k(embed_kernel, dim3(T), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
                          nullptr, 0, ids.data_ptr<int>(),
                          reinterpret_cast<const bf16*>(table.data_ptr()),
                          reinterpret_cast<bf16*>(out.data_ptr()), hidden,
                          static_cast<int>(table.size(0)), err.data_ptr<int>()));
}

void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w,
             at::Tensor& y, double eps) {
  const int T = x.size(0), H = x.size(1);
  if (T == 0) return;
  TORCH_CHECK(H % 8 == 0 && x.stride(1) == 1 && y.stride(1) == 1, "rmsnorm layout");
  bf16* res = nullptr;
  int ldr = 0;
  if (residual.has_value() && residual->defined()) {
    res = reinterpret_cast<bf16*>(residual->data_ptr());
    ldr = residual->stride(0);
  }
  const int threads = 128;
  const int vpt = (H / 8 + threads - 1) / threads;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto wp = reinterpret_cast<const bf16*>(w.data_ptr());
  auto yp = reinterpret_cast<bf16*>(y.data_ptr());
#define LB_RMS(V)                                                                          \
  C10_CUDA_CHECK(launch_k(rmsnorm_kernel<V>, dim3(T), dim3(threads), 0, st, nullptr, 0, xp,    \
                          static_cast<int>(x.stride(0)), res, ldr, wp, yp,                   \
                          static_cast<int>(y.stride(0)), H, static_cast<float>(eps)))
  if (vpt <= 1) LB_RMS(1);
  else if (vpt <= 2) LB_RMS(2);
  else if (vpt <= 4) LB_RMS(4);
  else if (vpt <= 8) LB_RMS(8);
  else TORCH_CHECK(false, "rmsnorm: hidden too large");
#undef LB_RMS
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_kv(at::Tensor& qkv, const at::Tensor& positions, const c10::optional<at::Tensor>& slots,
             const at::Tensor& cos_sin, at::Tensor& k_cache, at::Tensor& v_cache, int64_t hq,
             int64_t hkv, at::Tensor& err, const c10::optional<at::Tensor>& q_norm,
             const c10::optional<at::Tensor>& k_norm, int64_t norm_dim, double eps) {
  const int T = qkv.size(0);
  if (T == 0) return;
  const int D = k_cache.size(3);      // head width (padded)
  const int R = cos_sin.size(1);      // rotary width
  TORCH_CHECK(R <= D && R % 2 == 0 && D % 8 == 0, "rope_kv: rotary width");
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.size(1) >= (hq + 2 * hkv) * D, "rope_kv: qkv layout");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin f32");
  const int* sp = nullptr;
  if (slots.has_value() && slots->defined()) sp = slots->data_ptr<int>();
  const bool has_qn = q_norm.has_value() && q_norm->defined();
  const bool has_kn = k_norm.has_value() && k_norm->defined();
  const bool aligned = reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0 && qkv.stride(0) % 8 == 0;
  if (D == 128 && R % 16 == 0 && aligned) {
    const bf16* qn = nullptr;
    const bf16* kn = nullptr;
    for (int i = 0; i < 2; ++i) {
      const bool has = i == 0 ? has_qn : has_kn;
      if (!has) continue;
      const at::Tensor& t = i == 0 ? *q_norm : *k_norm;
      TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.numel() == D,
                  "rope_kv: q/k norm weights are bf16 [head width]");
      (i == 0 ? qn : kn) = reinterpret_cast<const bf16*>(t.data_ptr());
    }
    const long long warps = static_cast<long long>(T) * (hq + 2 * hkv);
    const int blocks = static_cast<int>((warps + 7) / 8);
    C10_CUDA_CHECK(launch_k(
        rope_kv_warp_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
        nullptr, 0, reinterpret_cast<bf16*>(qkv.data_ptr()), static_cast<int>(qkv.stride(0)),
        positions.data_ptr<int>(), sp, cos_sin.data_ptr<float>(),
        static_cast<int>(cos_sin.size(0)), reinterpret_cast<bf16*>(k_cache.data_ptr()),
        reinterpret_cast<bf16*>(v_cache.data_ptr()), T, static_cast<int>(hq),
        static_cast<int>(hkv), R, static_cast<int>(k_cache.size(2)), qn, kn,
        norm_dim > 0 ? static_cast<int>(norm_dim) : R, static_cast<float>(eps),
        err.data_ptr<int>()));
    return;
  }
  TORCH_CHECK(!has_qn && !has_kn, "rope_kv: q/k norm needs 128-wide heads");
  C10_CUDA_CHECK(launch_k(
      rope_kv_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(), nullptr, 0,
      reinterpret_cast<bf16*>(qkv.data_ptr()), static_cast<int>(qkv.stride(0)),
      positions.data_ptr<int>(), sp, cos_sin.data_ptr<float>(),
      static_cast<int>(cos_sin.size(0)), reinterpret_cast<bf16*>(k_cache.data_ptr()),
      reinterpret_cast<bf16*>(v_cache.data_ptr()), static_cast<int>(hq), static_cast<int>(hkv),
      D, R, static_cast<int>(k_cache.size(2)), err.data_ptr<int>()));
}

}  // namespace lb
