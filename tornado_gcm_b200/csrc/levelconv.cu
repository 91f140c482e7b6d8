// Data movement of the convolution towers: vertical (level-axis) and
// horizontal (longitude-latitude) convolutions lowered onto GEMMs.
//
// A level convolution with kernel k and 'same' padding is a GEMM over the
// token rows (column, level): row (n, l) of the lowered operand holds the k
// level-neighbours x[n, l + t - pad, :] (t = 0..k-1, zero outside the column)
// side by side, and out = A . W2^T with W2[co, t*C + ci] = W[co, ci, t] runs on
// the tcgen05 BF16 linear kernels (bias and activation fused in their
// epilogue).  These two kernels build A (BF16, row stride padded to a multiple
// of 8) and fold its gradient back onto the levels, applying the previous
// layer's activation derivative on the way:
//   dx[n, l, c] = act'(pre[n, l, c]) * sum_t dA[(n, l - t + pad), t*C + c].
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/library.h>

namespace tgcm {
namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  return static_cast<float>(v);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// one thread per element of A (row-major, ld columns)
template <typename T>
__global__ void level_im2col_kernel(const T* __restrict__ x, __nv_bfloat16* __restrict__ A, long long rows, int L,
                                    int C, int k, int ld, long long x_ld) {
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= rows * ld) return;
  const long long row = idx / ld;
  const int col = static_cast<int>(idx - row * ld);
  float v = 0.f;
  if (col < k * C) {
    const int t = col / C, c = col - t * C;
    const long long n = row / L;
    const int l = static_cast<int>(row - n * L) + t - k / 2;
    if (l >= 0 && l < L) v = to_f(x[(n * L + l) * x_ld + c]);
  }
  A[idx] = __float2bfloat16(v);
}

// one thread per element of dx (rows x C); act: 0 none, 1 relu (derivative from pre > 0)
__global__ void level_col2im_kernel(const __nv_bfloat16* __restrict__ dA, float* __restrict__ dx,
                                    const __nv_bfloat16* __restrict__ pre, long long rows, int L, int C, int k,
                                    int ld, int pre_ld, int act) {
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= rows * C) return;
  const long long row = idx / C;
  const int c = static_cast<int>(idx - row * C);
  const long long n = row / L;
  const int l = static_cast<int>(row - n * L);
  float s = 0.f;
  for (int t = 0; t < k; ++t) {
    const int src = l - t + k / 2;  // output level whose window holds level l at tap t
    if (src >= 0 && src < L) s += __bfloat162float(dA[(n * L + src) * ld + t * C + c]);
  }
  if (pre != nullptr && act == 1 && !(__bfloat162float(pre[row * pre_ld + c]) > 0.f)) s = 0.f;
  dx[idx] = s;
}

// 2-D (lon, lat) lowering: token row (b, i, j) holds x[b, i + (a - pa)*d mod I, j + (t - pt)*d, :]
// for a < kl, t < kt (lat taps outside [0, J) are zero): circular in longitude, zero-padded in latitude.
template <typename T>
__global__ void lonlat_im2col_kernel(const T* __restrict__ x, __nv_bfloat16* __restrict__ A, long long rows, int I,
                                     int J, int C, int kl, int kt, int dil, int ld, long long x_ld) {
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= rows * ld) return;
  const long long row = idx / ld;
  const int col = static_cast<int>(idx - row * ld);
  float v = 0.f;
  if (col < kl * kt * C) {
    const int tap = col / C, c = col - tap * C;
    const int a = tap / kt, t = tap - a * kt;
    const long long b = row / (static_cast<long long>(I) * J);
    const int rem = static_cast<int>(row - b * I * J);
    const int i = rem / J, j = rem - i * J;
    int ii = (i + (a - kl / 2) * dil) % I;
    if (ii < 0) ii += I;
    const int jj = j + (t - kt / 2) * dil;
    if (jj >= 0 && jj < J) v = to_f(x[((b * I + ii) * J + jj) * x_ld + c]);
  }
  A[idx] = __float2bfloat16(v);
}

// adjoint of the lowering, with the previous layer's ReLU derivative (act 1)
__global__ void lonlat_col2im_kernel(const __nv_bfloat16* __restrict__ dA, float* __restrict__ dx,
                                     const __nv_bfloat16* __restrict__ pre, long long rows, int I, int J, int C,
                                     int kl, int kt, int dil, int ld, int pre_ld, int act) {
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= rows * C) return;
  const long long row = idx / C;
  const int c = static_cast<int>(idx - row * C);
  const long long b = row / (static_cast<long long>(I) * J);
  const int rem = static_cast<int>(row - b * I * J);
  const int i = rem / J, j = rem - i * J;
  float s = 0.f;
  for (int a = 0; a < kl; ++a) {
    int io = (i - (a - kl / 2) * dil) % I;  // output column whose tap a reads longitude i
    if (io < 0) io += I;
    for (int t = 0; t < kt; ++t) {
      const int jo = j - (t - kt / 2) * dil;
      if (jo < 0 || jo >= J) continue;
      s += __bfloat162float(dA[((b * I + io) * J + jo) * ld + (a * kt + t) * C + c]);
    }
  }
  if (pre != nullptr && act == 1 && !(__bfloat162float(pre[row * pre_ld + c]) > 0.f)) s = 0.f;
  dx[idx] = s;
}

}  // namespace

// x: (B*I*J, >=C) token rows (fp32/bf16, unit column stride) -> A (B*I*J, ld) bf16.
at::Tensor lonlat_im2col(const at::Tensor& x, int64_t I, int64_t J, int64_t C, int64_t kl, int64_t kt, int64_t dil,
                         int64_t ld) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1 && x.size(1) >= C, "lonlat_im2col: token rows");
  TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16, "fp32 or bf16 input");
  TORCH_CHECK(kl % 2 == 1 && kt % 2 == 1 && dil >= 1 && ld >= kl * kt * C && ld % 8 == 0 && x.size(0) % (I * J) == 0,
              "lonlat_im2col: bad sizes");
  c10::cuda::CUDAGuard guard(x.device());
  const long long rows = x.size(0);
  auto A = at::empty({rows, ld}, x.options().dtype(at::kBFloat16));
  const long long n = rows * ld;
  if (n == 0) return A;
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  auto st = at::cuda::getCurrentCUDAStream();
  auto Ap = reinterpret_cast<__nv_bfloat16*>(A.data_ptr());
  if (x.scalar_type() == at::kFloat)
    lonlat_im2col_kernel<float><<<blocks, 256, 0, st>>>(x.data_ptr<float>(), Ap, rows, I, J, C, kl, kt, dil, ld,
                                                         x.stride(0));
  else
    lonlat_im2col_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), Ap, rows, I, J, C, kl, kt, dil, ld, x.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return A;
}

at::Tensor lonlat_col2im(const at::Tensor& dA, int64_t I, int64_t J, int64_t C, int64_t kl, int64_t kt, int64_t dil,
                         const c10::optional<at::Tensor>& pre, int64_t act) {
  TORCH_CHECK(dA.is_cuda() && dA.dim() == 2 && dA.is_contiguous() && dA.scalar_type() == at::kBFloat16 &&
                  dA.size(1) >= kl * kt * C && dA.size(0) % (I * J) == 0,
              "lonlat_col2im: contiguous bf16 lowered gradient expected");
  c10::cuda::CUDAGuard guard(dA.device());
  const long long rows = dA.size(0);
  auto dx = at::empty({rows, C}, dA.options().dtype(at::kFloat));
  const __nv_bfloat16* pp = nullptr;
  int pre_ld = 0;
  if (pre.has_value() && pre->defined()) {
    TORCH_CHECK(pre->scalar_type() == at::kBFloat16 && pre->dim() == 2 && pre->size(0) == rows &&
                    pre->size(1) >= C && pre->stride(1) == 1,
                "lonlat_col2im: pre must be bf16 token rows");
    pp = reinterpret_cast<const __nv_bfloat16*>(pre->data_ptr());
    pre_ld = static_cast<int>(pre->stride(0));
  }
  const long long n = rows * C;
  if (n == 0) return dx;
  lonlat_col2im_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dA.data_ptr()), dx.data_ptr<float>(), pp, rows, I, J, C, kl, kt, dil,
      static_cast<int>(dA.size(1)), pre_ld, static_cast<int>(act));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

// x: (N, L, C) rows with row stride x_ld (fp32 or bf16) -> A (N*L, ld) bf16, ld >= k*C, ld % 8 == 0.
at::Tensor level_im2col(const at::Tensor& x, int64_t L, int64_t C, int64_t k, int64_t ld) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "level_im2col: (N*L, >=C) CUDA rows expected");
  TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16, "fp32 or bf16 input");
  TORCH_CHECK(k >= 1 && k % 2 == 1 && ld >= k * C && ld % 8 == 0 && x.size(0) % L == 0 && x.size(1) >= C,
              "level_im2col: bad sizes");
  c10::cuda::CUDAGuard guard(x.device());
  const long long rows = x.size(0);
  auto A = at::empty({rows, ld}, x.options().dtype(at::kBFloat16));
  const long long n = rows * ld;
  if (n == 0) return A;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((n + threads - 1) / threads);
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kFloat)
    level_im2col_kernel<float><<<blocks, threads, 0, st>>>(x.data_ptr<float>(),
                                                           reinterpret_cast<__nv_bfloat16*>(A.data_ptr()), rows,
                                                           static_cast<int>(L), static_cast<int>(C),
                                                           static_cast<int>(k), static_cast<int>(ld), x.stride(0));
  else
    level_im2col_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(A.data_ptr()), rows,
        static_cast<int>(L), static_cast<int>(C), static_cast<int>(k), static_cast<int>(ld), x.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return A;
}

// dA: (N*L, ld) bf16 -> dx (N*L, C) fp32; pre: optional (N*L, >=C) bf16 pre-activation, act 1 = relu.
at::Tensor level_col2im(const at::Tensor& dA, int64_t L, int64_t C, int64_t k, const c10::optional<at::Tensor>& pre,
                        int64_t act) {
  TORCH_CHECK(dA.is_cuda() && dA.dim() == 2 && dA.is_contiguous() && dA.scalar_type() == at::kBFloat16,
              "level_col2im: contiguous bf16 (N*L, ld) gradient expected");
  TORCH_CHECK(k >= 1 && k % 2 == 1 && dA.size(1) >= k * C && dA.size(0) % L == 0, "level_col2im: bad sizes");
  c10::cuda::CUDAGuard guard(dA.device());
  const long long rows = dA.size(0);
  auto dx = at::empty({rows, C}, dA.options().dtype(at::kFloat));
  const __nv_bfloat16* pp = nullptr;
  int pre_ld = 0;
  if (pre.has_value() && pre->defined()) {
    TORCH_CHECK(pre->scalar_type() == at::kBFloat16 && pre->dim() == 2 && pre->size(0) == rows &&
                    pre->size(1) >= C && pre->stride(1) == 1,
                "level_col2im: pre must be bf16 (N*L, >=C) rows");
    pp = reinterpret_cast<const __nv_bfloat16*>(pre->data_ptr());
    pre_ld = static_cast<int>(pre->stride(0));
  }
  const long long n = rows * C;
  if (n == 0) return dx;
  const int threads = 256;
  level_col2im_kernel<<<static_cast<unsigned>((n + threads - 1) / threads), threads, 0,
                        at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const __nv_bfloat16*>(dA.data_ptr()),
                                                            dx.data_ptr<float>(), pp, rows, static_cast<int>(L),
                                                            static_cast<int>(C), static_cast<int>(k),
                                                            static_cast<int>(dA.size(1)), pre_ld,
                                                            static_cast<int>(act));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("level_im2col(Tensor x, int L, int C, int k, int ld) -> Tensor");
  m.def("level_col2im(Tensor dA, int L, int C, int k, Tensor? pre, int act) -> Tensor");
  m.def("lonlat_im2col(Tensor x, int I, int J, int C, int kl, int kt, int dil, int ld) -> Tensor");
  m.def("lonlat_col2im(Tensor dA, int I, int J, int C, int kl, int kt, int dil, Tensor? pre, int act) -> Tensor");
}

TORCH_LIBRARY_IMPL(tgcm, CUDA, m) {
  m.impl("level_im2col", &tgcm::level_im2col);
  m.impl("level_col2im", &tgcm::level_col2im);
  m.impl("lonlat_im2col", &tgcm::lonlat_im2col);
  m.impl("lonlat_col2im", &tgcm::lonlat_col2im);
}
