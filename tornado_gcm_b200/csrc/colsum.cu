// Column sums of a row-major BF16 matrix in FP32 (the bias gradient of a
// linear layer: db[o] = sum_t dY[t, o]).
//
// Pass 1: block b sums its slice of rows; each thread owns one 16-byte
// vector (8 columns) and a row lane, so every warp load is a run of full
// sectors; the row lanes are folded in shared memory and the block writes
// one row of partial sums.  Pass 2: 8 row groups per 32-column block add the
// block partials in a fixed order — the result does not depend on scheduling
// (no atomics).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/library.h>

#include "alloc.h"

namespace tgcm {
namespace {

constexpr int kColsumThreads = 256;
constexpr int kColsumBlocks = 296;  // 2 per SM on a 148-SM part

__global__ void __launch_bounds__(kColsumThreads) colsum_partial_kernel(const __nv_bfloat16* __restrict__ x,
                                                                      long long T, int ld, int ncols,
                                                                      float* __restrict__ part) {
  __shared__ float red[kColsumThreads][9];
  const int nvec = (ncols + 7) / 8;
  const int lanes = kColsumThreads / nvec;  // row lanes per block (>= 1: ncols <= 2048)
  const int v = threadIdx.x % nvec, r = threadIdx.x / nvec;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  const long long per = (T + gridDim.x - 1) / gridDim.x;
  const long long t0 = per * blockIdx.x;
  long long t1 = t0 + per;
  if (t1 > T) t1 = T;
  if (r < lanes) {
    const int c0 = v * 8;
    const bool full = c0 + 8 <= ncols && (ld % 8 == 0);
    for (long long t = t0 + r; t < t1; t += lanes) {
      const __nv_bfloat16* row = x + t * ld + c0;
      if (full) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(row));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      } else {
        for (int e = 0; e < 8 && c0 + e < ncols; ++e) acc[e] += __bfloat162float(row[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[threadIdx.x][e] = acc[e];
  __syncthreads();
  if (threadIdx.x < nvec) {
    float s[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] = 0.f;
    for (int rr = 0; rr < lanes; ++rr)
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] += red[rr * nvec + threadIdx.x][e];
    for (int e = 0; e < 8 && threadIdx.x * 8 + e < ncols; ++e)
      part[static_cast<long long>(blockIdx.x) * ncols + threadIdx.x * 8 + e] = s[e];
  }
}

// 32 columns per block, 8 row groups folding the block partials in a fixed order.
__global__ void __launch_bounds__(256) colsum_final_kernel(const float* __restrict__ part, int nblocks, int ncols,
                                                           float* __restrict__ out, int accumulate) {
  __shared__ float red[8][33];
  const int cl = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  float s = 0.f;
  if (c < ncols)
    for (int b = grp; b < nblocks; b += 8) s += part[static_cast<long long>(b) * ncols + c];
  red[grp][cl] = s;
  __syncthreads();
  if (grp == 0 && c < ncols) {
    float t = 0.f;
#pragma unroll
    for (int g2 = 0; g2 < 8; ++g2) t += red[g2][cl];
    out[c] = accumulate ? out[c] + t : t;
  }
}

}  // namespace

namespace {

void colsum_launch(const at::Tensor& x, int64_t ncols, at::Tensor& out, int accumulate) {
  const long long T = x.size(0);
  if (T == 0) {
    if (!accumulate) out.zero_();
    return;
  }
  const int nb = static_cast<int>(T < kColsumBlocks ? T : kColsumBlocks);
  auto part = out_empty({nb, ncols}, x.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  colsum_partial_kernel<<<nb, kColsumThreads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), T,
                                                      static_cast<int>(x.stride(0)), static_cast<int>(ncols),
                                                      part.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  colsum_final_kernel<<<static_cast<unsigned>((ncols + 31) / 32), 256, 0, st>>>(part.data_ptr<float>(), nb,
                                                                                  static_cast<int>(ncols),
                                                                                  out.data_ptr<float>(), accumulate);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void check_x(const at::Tensor& x, int64_t ncols) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "colsum_bf16 expects a (T, ld) bf16 CUDA matrix with unit column stride");
  TORCH_CHECK(ncols >= 1 && ncols <= x.size(1) && ncols <= 2048, "ncols out of range");
}

}  // namespace

// x: (T, ld) bf16 row-major; returns fp32 (ncols) sums of the first ncols columns.
at::Tensor colsum_bf16(const at::Tensor& x, int64_t ncols) {
  check_x(x, ncols);
  c10::cuda::CUDAGuard guard(x.device());
  auto out = out_empty({ncols}, x.options().dtype(at::kFloat));
  colsum_launch(x, ncols, out, 0);
  return out;
}

// out[c] += sum_t x[t, c] for c < ncols (the bias gradient accumulated in place).
void colsum_bf16_acc(const at::Tensor& x, int64_t ncols, at::Tensor& out) {
  check_x(x, ncols);
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() >= ncols &&
                  out.device() == x.device(),
              "colsum_bf16_acc expects a contiguous fp32 output on the same device with >= ncols elements");
  c10::cuda::CUDAGuard guard(x.device());
  colsum_launch(x, ncols, out, 1);
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("colsum_bf16(Tensor x, int ncols) -> Tensor");
  m.def("colsum_bf16_acc(Tensor x, int ncols, Tensor(a!) out) -> ()");
}

TORCH_LIBRARY_IMPL(tgcm, CUDA, m) {
  m.impl("colsum_bf16", &tgcm::colsum_bf16);
  m.impl("colsum_bf16_acc", &tgcm::colsum_bf16_acc);
}
