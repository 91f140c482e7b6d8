// Column attention (sequence = vertical levels of one atmospheric column).
//
// The towers of this model family attend over the levels of each column
// separately: tens of thousands of independent (column, head) problems with a
// sequence of ~32 levels and a head dimension of 8-64.  One (column, head)
// problem is a few kB of Q/K/V, far below one 128-row tensor-core tile, and
// the whole op is bound by reading Q, K, V and writing O once (a few hundred
// FLOP per byte are never reached).  So the kernel gives every (column, head)
// one warp: K and V go to shared memory with coalesced loads, lane i owns
// query row i (rows i + 32, … for longer sequences), and the softmax runs
// online in fp32 registers (running max and sum), so nothing of size
// Sq x Skv is ever stored.  The log-sum-exp of every row is kept for the
// backward pass, which recomputes the probabilities (two passes: lane = query
// row for dQ, lane = key row for dK and dV), again without an Sq x Skv buffer.
//
// Layouts: q (G, Sq, D), k and v (G, Skv, D), o (G, Sq, D), lse (G, Sq) fp32;
// G = batch x heads; bf16 or fp32 storage, fp32 arithmetic.

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/library.h>

#include <cmath>

namespace tgcm {
namespace {

constexpr int kAttWarps = 4;    // (column, head) problems per block
constexpr int kAttMaxSeq = 128;
constexpr int kAttMaxDim = 64;

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void stf(T* p, float v) {
  *p = static_cast<T>(v);
}
template <>
__device__ __forceinline__ void stf<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16(v);
}

// Copy rows [0, n) x D of a (n, D) matrix into shared fp32 (warp-cooperative).
template <typename T, int D>
__device__ __forceinline__ void stage(float* s, const T* g, int n, int lane) {
  for (int e = lane; e < n * D; e += 32) s[e] = ldf(g + e);
}

template <typename T, int D>
__global__ void __launch_bounds__(32 * kAttWarps) attn_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                 const T* __restrict__ v, T* __restrict__ o,
                                                                 float* __restrict__ lse, int G, int Sq, int Skv,
                                                                 float scale) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * kAttWarps + warp;
  if (g >= G) return;
  float* ks = sm + warp * 2 * Skv * D;
  float* vs = ks + Skv * D;
  stage<T, D>(ks, k + static_cast<long long>(g) * Skv * D, Skv, lane);
  stage<T, D>(vs, v + static_cast<long long>(g) * Skv * D, Skv, lane);
  __syncwarp();
  for (int i = lane; i < Sq; i += 32) {
    const T* qi = q + (static_cast<long long>(g) * Sq + i) * D;
    float qr[D], acc[D];
#pragma unroll
    for (int d = 0; d < D; ++d) {
      qr[d] = ldf(qi + d) * scale;
      acc[d] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < Skv; ++j) {
      const float* kj = ks + j * D;
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) s = fmaf(qr[d], kj[d], s);
      const float mn = fmaxf(m, s);
      const float corr = __expf(m - mn);  // 0 on the first key (m = -inf)
      const float p = __expf(s - mn);
      l = l * corr + p;
      const float* vj = vs + j * D;
#pragma unroll
      for (int d = 0; d < D; ++d) acc[d] = fmaf(p, vj[d], acc[d] * corr);
      m = mn;
    }
    const float inv = 1.f / l;
    T* oi = o + (static_cast<long long>(g) * Sq + i) * D;
#pragma unroll
    for (int d = 0; d < D; ++d) stf(oi + d, acc[d] * inv);
    lse[static_cast<long long>(g) * Sq + i] = m + __logf(l);
  }
}

// Backward.  Pass 1 (lane = query row i): dQ_i = scale * sum_j ds_ij k_j with
// ds_ij = p_ij (dO_i . v_j - delta_i), delta_i = dO_i . O_i.
// Pass 2 (lane = key row j): dK_j = scale * sum_i ds_ij q_i, dV_j = sum_i p_ij dO_i.
template <typename T, int D>
__global__ void __launch_bounds__(32 * kAttWarps) attn_bwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                 const T* __restrict__ v, const T* __restrict__ o,
                                                                 const T* __restrict__ dout,
                                                                 const float* __restrict__ lse, T* __restrict__ dq,
                                                                 T* __restrict__ dk, T* __restrict__ dv, int G,
                                                                 int Sq, int Skv, float scale) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * kAttWarps + warp;
  if (g >= G) return;
  const int per = 2 * Skv * D + 2 * Sq * D + 2 * Sq;
  float* ks = sm + warp * per;
  float* vs = ks + Skv * D;
  float* qs = vs + Skv * D;      // q * scale
  float* dos = qs + Sq * D;      // dO
  float* ls = dos + Sq * D;      // lse
  float* dl = ls + Sq;           // delta
  const long long qo = static_cast<long long>(g) * Sq * D, ko = static_cast<long long>(g) * Skv * D;
  stage<T, D>(ks, k + ko, Skv, lane);
  stage<T, D>(vs, v + ko, Skv, lane);
  stage<T, D>(qs, q + qo, Sq, lane);
  stage<T, D>(dos, dout + qo, Sq, lane);
  for (int e = lane; e < Sq * D; e += 32) qs[e] *= scale;
  __syncwarp();  // dO rows staged by other lanes are read below
  for (int i = lane; i < Sq; i += 32) {
    ls[i] = lse[static_cast<long long>(g) * Sq + i];
    float dd = 0.f;
    const T* oi = o + qo + i * D;
#pragma unroll
    for (int d = 0; d < D; ++d) dd = fmaf(dos[i * D + d], ldf(oi + d), dd);
    dl[i] = dd;
  }
  __syncwarp();
  // pass 1: dQ
  for (int i = lane; i < Sq; i += 32) {
    float acc[D];
#pragma unroll
    for (int d = 0; d < D; ++d) acc[d] = 0.f;
    const float* qi = qs + i * D;
    const float* doi = dos + i * D;
    for (int j = 0; j < Skv; ++j) {
      const float* kj = ks + j * D;
      const float* vj = vs + j * D;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) {
        s = fmaf(qi[d], kj[d], s);
        dp = fmaf(doi[d], vj[d], dp);
      }
      const float ds = __expf(s - ls[i]) * (dp - dl[i]);
#pragma unroll
      for (int d = 0; d < D; ++d) acc[d] = fmaf(ds, kj[d], acc[d]);
    }
    T* dqi = dq + qo + i * D;
#pragma unroll
    for (int d = 0; d < D; ++d) stf(dqi + d, acc[d] * scale);
  }
  // pass 2: dK, dV
  for (int j = lane; j < Skv; j += 32) {
    float ak[D], av[D];
#pragma unroll
    for (int d = 0; d < D; ++d) ak[d] = av[d] = 0.f;
    const float* kj = ks + j * D;
    const float* vj = vs + j * D;
    for (int i = 0; i < Sq; ++i) {
      const float* qi = qs + i * D;
      const float* doi = dos + i * D;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) {
        s = fmaf(qi[d], kj[d], s);
        dp = fmaf(doi[d], vj[d], dp);
      }
      const float p = __expf(s - ls[i]);
      const float ds = p * (dp - dl[i]);
#pragma unroll
      for (int d = 0; d < D; ++d) {
        ak[d] = fmaf(ds, qi[d], ak[d]);  // q already carries the scale
        av[d] = fmaf(p, doi[d], av[d]);
      }
    }
    T* dkj = dk + ko + j * D;
    T* dvj = dv + ko + j * D;
#pragma unroll
    for (int d = 0; d < D; ++d) {
      stf(dkj + d, ak[d]);
      stf(dvj + d, av[d]);
    }
  }
}

void check_qkv(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "column attention: CUDA tensors expected");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "column attention: (G, S, D) tensors expected");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "column attention: contiguous inputs");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type() &&
                  (q.scalar_type() == at::kBFloat16 || q.scalar_type() == at::kFloat),
              "column attention: q, k, v share one dtype (bf16 or fp32)");
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(2) == k.size(2), "q/k/v shape mismatch");
  TORCH_CHECK(q.size(1) >= 1 && q.size(1) <= kAttMaxSeq && k.size(1) >= 1 && k.size(1) <= kAttMaxSeq,
              "column attention: sequence lengths 1..128");
  const int64_t D = q.size(2);
  TORCH_CHECK(D == 8 || D == 16 || D == 32 || D == 64, "column attention: head dim 8, 16, 32 or 64");
}

template <typename F>
void dispatch_dim(int64_t D, F&& f) {
  switch (D) {
    case 8: f(std::integral_constant<int, 8>()); break;
    case 16: f(std::integral_constant<int, 16>()); break;
    case 32: f(std::integral_constant<int, 32>()); break;
    default: f(std::integral_constant<int, 64>()); break;
  }
}

}  // namespace

std::vector<at::Tensor> column_attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                             double scale) {
  check_qkv(q, k, v);
  c10::cuda::CUDAGuard guard(q.device());
  const int64_t G = q.size(0), Sq = q.size(1), Skv = k.size(1), D = q.size(2);
  auto o = at::empty_like(q);
  auto lse = at::empty({G, Sq}, q.options().dtype(at::kFloat));
  if (G == 0) return {o, lse};
  const size_t smem = static_cast<size_t>(kAttWarps) * 2 * Skv * D * sizeof(float);
  TORCH_CHECK(smem <= 227 * 1024, "column attention: key length x head dim too large for shared memory");
  dim3 grid(static_cast<unsigned>((G + kAttWarps - 1) / kAttWarps));
  auto st = at::cuda::getCurrentCUDAStream();
  dispatch_dim(D, [&](auto dc) {
    constexpr int DD = decltype(dc)::value;
    if (q.scalar_type() == at::kBFloat16) {
      auto kern = attn_fwd_kernel<__nv_bfloat16, DD>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      kern<<<grid, 32 * kAttWarps, smem, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
          reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), reinterpret_cast<__nv_bfloat16*>(o.data_ptr()),
          lse.data_ptr<float>(), static_cast<int>(G), static_cast<int>(Sq), static_cast<int>(Skv),
          static_cast<float>(scale));
    } else {
      auto kern = attn_fwd_kernel<float, DD>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      kern<<<grid, 32 * kAttWarps, smem, st>>>(q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(),
                                               o.data_ptr<float>(), lse.data_ptr<float>(), static_cast<int>(G),
                                               static_cast<int>(Sq), static_cast<int>(Skv),
                                               static_cast<float>(scale));
    }
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

std::vector<at::Tensor> column_attention_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                             const at::Tensor& o, const at::Tensor& dout, const at::Tensor& lse,
                                             double scale) {
  check_qkv(q, k, v);
  TORCH_CHECK(o.sizes() == q.sizes() && dout.sizes() == q.sizes() && o.is_contiguous() && dout.is_contiguous() &&
                  o.scalar_type() == q.scalar_type() && dout.scalar_type() == q.scalar_type(),
              "column attention backward: o / dout must match q");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == q.size(0) * q.size(1),
              "column attention backward: lse (G, Sq) fp32");
  c10::cuda::CUDAGuard guard(q.device());
  const int64_t G = q.size(0), Sq = q.size(1), Skv = k.size(1), D = q.size(2);
  auto dq = at::empty_like(q), dk = at::empty_like(k), dv = at::empty_like(v);
  if (G == 0) return {dq, dk, dv};
  const size_t smem = static_cast<size_t>(kAttWarps) * (2 * Skv * D + 2 * Sq * D + 2 * Sq) * sizeof(float);
  TORCH_CHECK(smem <= 227 * 1024, "column attention backward: sequence x head dim too large for shared memory");
  dim3 grid(static_cast<unsigned>((G + kAttWarps - 1) / kAttWarps));
  auto st = at::cuda::getCurrentCUDAStream();
  dispatch_dim(D, [&](auto dc) {
    constexpr int DD = decltype(dc)::value;
    if (q.scalar_type() == at::kBFloat16) {
      using B16 = __nv_bfloat16;
      auto kern = attn_bwd_kernel<B16, DD>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      kern<<<grid, 32 * kAttWarps, smem, st>>>(
          reinterpret_cast<const B16*>(q.data_ptr()), reinterpret_cast<const B16*>(k.data_ptr()),
          reinterpret_cast<const B16*>(v.data_ptr()), reinterpret_cast<const B16*>(o.data_ptr()),
          reinterpret_cast<const B16*>(dout.data_ptr()), lse.data_ptr<float>(), reinterpret_cast<B16*>(dq.data_ptr()),
          reinterpret_cast<B16*>(dk.data_ptr()), reinterpret_cast<B16*>(dv.data_ptr()), static_cast<int>(G),
          static_cast<int>(Sq), static_cast<int>(Skv), static_cast<float>(scale));
    } else {
      auto kern = attn_bwd_kernel<float, DD>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      kern<<<grid, 32 * kAttWarps, smem, st>>>(q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(),
                                               o.data_ptr<float>(), dout.data_ptr<float>(), lse.data_ptr<float>(),
                                               dq.data_ptr<float>(), dk.data_ptr<float>(), dv.data_ptr<float>(),
                                               static_cast<int>(G), static_cast<int>(Sq), static_cast<int>(Skv),
                                               static_cast<float>(scale));
    }
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dk, dv};
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("column_attention_fwd(Tensor q, Tensor k, Tensor v, float scale) -> Tensor[]");
  m.def("column_attention_bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor dout, Tensor lse, float scale) "
        "-> Tensor[]");
}

TORCH_LIBRARY_IMPL(tgcm, CUDA, m) {
  m.impl("column_attention_fwd", &tgcm::column_attention_fwd);
  m.impl("column_attention_bwd", &tgcm::column_attention_bwd);
}
