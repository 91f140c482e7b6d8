// Layout changes between latitude-major nodal fields and the token rows of
// the column networks, with the per-(channel, latitude) factors applied.
//
//   nodal  (B, C, P)  fp32, P = J·I positions, channel-major (what the
//                     spherical-harmonic synthesis writes and the analysis
//                     reads);
//   tokens (B·P, ld)  one row per column (b, j, i), channels contiguous (what
//                     the tcgen05 linear layers read and write).
//
// to_tokens:   tok[b·P + p, c] = nod[b, c, p] · scale[c, p / I]   for c < C,
//              extra[b·P + p, c - C]                               for C ≤ c < C + F,
//              0                                                   up to ld  (BF16 out);
// from_tokens: nod[b, c, p] = tok[b·P + p, c] · scale[c, p / I]    (fp32 out; tok fp32 or BF16).
//
// Each is the other's adjoint up to the extra columns (which carry no
// gradient), so the forward and backward of the column network use the same
// two kernels.  One 32 x 32 (channel x position) tile per block goes through
// shared memory, so both the channel-major and the token-major side are read
// and written in whole 32-value runs.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/library.h>

#include "alloc.h"

namespace tgcm {
namespace {

constexpr int kTile = 32;
constexpr int kRows = 8;  // block = 32 x 8 threads

__global__ void __launch_bounds__(kTile * kRows) to_tokens_kernel(const float* __restrict__ nod,
                                                                 const float* __restrict__ scale, int C, int P,
                                                                 int I, const __nv_bfloat16* __restrict__ extra,
                                                                 int F, __nv_bfloat16* __restrict__ tok, int ld) {
  __shared__ float tile[kTile][kTile + 1];  // [channel][position]
  const int b = blockIdx.z;
  const int p0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const long long tok0 = static_cast<long long>(b) * P;
  // load: lanes walk positions of one channel row
#pragma unroll
  for (int k = 0; k < kTile / kRows; ++k) {
    const int c = c0 + ty + kRows * k, p = p0 + tx;
    float v = 0.f;
    if (p < P) {
      if (c < C)
        v = nod[(static_cast<long long>(b) * C + c) * P + p] * __ldg(scale + static_cast<long long>(c) * (P / I) + p / I);
      else if (c < C + F)
        v = __bfloat162float(extra[(tok0 + p) * F + (c - C)]);
    }
    tile[ty + kRows * k][tx] = v;
  }
  __syncthreads();
  // store: lanes walk channels of one token row
#pragma unroll
  for (int k = 0; k < kTile / kRows; ++k) {
    const int p = p0 + ty + kRows * k, c = c0 + tx;
    if (p < P && c < ld) tok[(tok0 + p) * ld + c] = __float2bfloat16(tile[tx][ty + kRows * k]);
  }
}

template <typename Tin>
__device__ __forceinline__ float to_f(Tin v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename Tin>
__global__ void __launch_bounds__(kTile * kRows) from_tokens_kernel(const Tin* __restrict__ tok, int ld,
                                                                   const float* __restrict__ scale, int C, int P,
                                                                   int I, float* __restrict__ nod) {
  __shared__ float tile[kTile][kTile + 1];  // [position][channel]
  const int b = blockIdx.z;
  const int p0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const long long tok0 = static_cast<long long>(b) * P;
#pragma unroll
  for (int k = 0; k < kTile / kRows; ++k) {
    const int p = p0 + ty + kRows * k, c = c0 + tx;
    tile[ty + kRows * k][tx] = (p < P && c < C) ? to_f<Tin>(tok[(tok0 + p) * ld + c]) : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kTile / kRows; ++k) {
    const int c = c0 + ty + kRows * k, p = p0 + tx;
    if (p < P && c < C)
      nod[(static_cast<long long>(b) * C + c) * P + p] =
          tile[tx][ty + kRows * k] * __ldg(scale + static_cast<long long>(c) * (P / I) + p / I);
  }
}

}  // namespace

// nod: (B, C, J, I) fp32 contiguous; scale: (C, J) fp32; extra: (B·J·I, F) bf16 or None.
// Returns (B·J·I, ld) bf16 with ld >= C + F.
at::Tensor nodal_to_tokens(const at::Tensor& nod, const at::Tensor& scale, const c10::optional<at::Tensor>& extra,
                           int64_t ld) {
  TORCH_CHECK(nod.is_cuda() && nod.scalar_type() == at::kFloat && nod.dim() == 4 && nod.is_contiguous(),
              "nodal_to_tokens: nod must be a contiguous (B, C, J, I) fp32 CUDA tensor");
  const int64_t B = nod.size(0), C = nod.size(1), J = nod.size(2), I = nod.size(3), P = J * I;
  TORCH_CHECK(scale.is_contiguous() && scale.scalar_type() == at::kFloat && scale.numel() == C * J,
              "nodal_to_tokens: scale must be (C, J) fp32");
  int64_t F = 0;
  const __nv_bfloat16* ex = nullptr;
  if (extra.has_value() && extra->defined()) {
    TORCH_CHECK(extra->is_contiguous() && extra->scalar_type() == at::kBFloat16 && extra->dim() == 2 &&
                    extra->size(0) == B * P,
                "nodal_to_tokens: extra must be (B·J·I, F) bf16");
    F = extra->size(1);
    ex = reinterpret_cast<const __nv_bfloat16*>(extra->data_ptr());
  }
  TORCH_CHECK(ld >= C + F && B <= 65535 && P < (1LL << 31), "nodal_to_tokens: bad sizes");
  c10::cuda::CUDAGuard guard(nod.device());
  auto tok = out_empty({B * P, ld}, nod.options().dtype(at::kBFloat16));
  dim3 grid(static_cast<unsigned>((P + kTile - 1) / kTile), static_cast<unsigned>((ld + kTile - 1) / kTile),
            static_cast<unsigned>(B));
  to_tokens_kernel<<<grid, dim3(kTile, kRows), 0, at::cuda::getCurrentCUDAStream()>>>(
      nod.data_ptr<float>(), scale.data_ptr<float>(), static_cast<int>(C), static_cast<int>(P), static_cast<int>(I),
      ex, static_cast<int>(F), reinterpret_cast<__nv_bfloat16*>(tok.data_ptr()), static_cast<int>(ld));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return tok;
}

// tok: (B·J·I, >= C) fp32 or bf16 with unit column stride; returns (B, C, J, I) fp32.
at::Tensor tokens_to_nodal(const at::Tensor& tok, int64_t C, const at::Tensor& scale, int64_t B, int64_t J,
                           int64_t I) {
  TORCH_CHECK(tok.is_cuda() && tok.dim() == 2 && tok.stride(1) == 1 && tok.size(1) >= C,
              "tokens_to_nodal: tok must be (T, >= C) with unit column stride");
  TORCH_CHECK(tok.scalar_type() == at::kFloat || tok.scalar_type() == at::kBFloat16, "tokens_to_nodal: dtype");
  const int64_t P = J * I;
  TORCH_CHECK(tok.size(0) == B * P && scale.is_contiguous() && scale.scalar_type() == at::kFloat &&
                  scale.numel() == C * J && B <= 65535,
              "tokens_to_nodal: bad sizes");
  c10::cuda::CUDAGuard guard(tok.device());
  auto nod = out_empty({B, C, J, I}, tok.options().dtype(at::kFloat));
  dim3 grid(static_cast<unsigned>((P + kTile - 1) / kTile), static_cast<unsigned>((C + kTile - 1) / kTile),
            static_cast<unsigned>(B));
  auto st = at::cuda::getCurrentCUDAStream();
  const int ld = static_cast<int>(tok.stride(0));
  if (tok.scalar_type() == at::kFloat)
    from_tokens_kernel<float><<<grid, dim3(kTile, kRows), 0, st>>>(tok.data_ptr<float>(), ld, scale.data_ptr<float>(),
                                                                  static_cast<int>(C), static_cast<int>(P),
                                                                  static_cast<int>(I), nod.data_ptr<float>());
  else
    from_tokens_kernel<__nv_bfloat16><<<grid, dim3(kTile, kRows), 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(tok.data_ptr()), ld, scale.data_ptr<float>(), static_cast<int>(C),
        static_cast<int>(P), static_cast<int>(I), nod.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nod;
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("nodal_to_tokens(Tensor nod, Tensor scale, Tensor? extra, int ld) -> Tensor");
  m.def("tokens_to_nodal(Tensor tok, int C, Tensor scale, int B, int J, int I) -> Tensor");
}

TORCH_LIBRARY_IMPL(tgcm, CUDA, m) {
  m.impl("nodal_to_tokens", &tgcm::nodal_to_tokens);
  m.impl("tokens_to_nodal", &tgcm::tokens_to_nodal);
}
