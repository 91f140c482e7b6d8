// FP64 batched GEMM on the FP64 tensor cores (DMMA, mma.sync m8n8k4) for the
// Z0 / "highest"-precision spherical-harmonic transforms.
//
//   C[g][m][n] = alpha * colscale[n] * sum_k A[g][m][k] * B[g][n][k]   (+ beta * C)
//
// Every operand is addressed through element strides (row, k and batch), so
// the four steps of the FP64 transforms (Legendre per zonal row, DFT per
// slice, either direction) are one kernel without transposed copies.  The
// 8-byte elements are staged with cp.async (any stride, zero fill outside the
// matrix) into a two-stage shared-memory ring; four warps each own a 32 x 32
// block of the 64 x 64 tile as 4 x 4 DMMA 8 x 8 accumulators.
//
// Shared layout: As[k][m], Bs[k][n] with a row pitch of 68 doubles, so a
// fragment load (8 rows x 4 k per warp: lanes (m, k) = (lane / 4, lane % 4))
// touches 16 distinct bank pairs per half-warp (pair = (4k + m) mod 16).
//
// FP64 tensor-core throughput on B200 equals its FP64 FMA throughput; the
// kernel's point is FP64 accuracy at GEMM efficiency for the transforms, on
// this repository's own code path.

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdint>

namespace tgcm {
namespace {

constexpr int kDBM = 64, kDBN = 64, kDBK = 16, kDPitch = 68, kDThreads = 128;

struct DgemmArgs {
  const double* A;
  const double* B;
  double* C;
  const double* col_scale;  // [N] or null
  long long a_rs, a_ks, a_gs;
  long long b_rs, b_ks, b_gs;
  long long c_rs, c_cs, c_gs;
  int M, N, K, G;
  double alpha, beta;
};

__device__ __forceinline__ void cp_async8(double* smem, const double* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int src_size = valid ? 8 : 0;  // 0: zero fill, nothing read
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(s), "l"(gmem), "r"(src_size) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(d[0]), "+d"(d[1])
               : "d"(a), "d"(b));
}

// Stage one 64 x 16 operand tile (rows r0.., k k0..) into S[k][row].
// KC: the operand's k stride is 1 (threads walk along k for coalescing).
template <bool KC>
__device__ __forceinline__ void load_tile(double* S, const double* base, long long rs, long long ks, int r0, int k0,
                                          int rows, int K) {
#pragma unroll
  for (int i = 0; i < (kDBM * kDBK) / kDThreads; ++i) {
    const int e = threadIdx.x + i * kDThreads;
    const int r = KC ? e / kDBK : e % kDBM;
    const int k = KC ? e % kDBK : e / kDBM;
    const int gr = r0 + r, gk = k0 + k;
    const bool ok = gr < rows && gk < K;
    const double* src = ok ? base + gr * rs + gk * ks : base;
    cp_async8(S + k * kDPitch + r, src, ok);
  }
}

template <bool AKC, bool BKC>
__global__ void __launch_bounds__(kDThreads) dgemm_dmma_kernel(DgemmArgs p) {
  __shared__ __align__(16) double As[2][kDBK * kDPitch];
  __shared__ __align__(16) double Bs[2][kDBK * kDPitch];
  const int g = blockIdx.z;
  const int m0 = blockIdx.y * kDBM, n0 = blockIdx.x * kDBN;
  const double* A = p.A + g * p.a_gs;
  const double* B = p.B + g * p.b_gs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wm = (warp & 1) * 32, wn = (warp >> 1) * 32;
  double acc[4][4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;

  const int nk = (p.K + kDBK - 1) / kDBK;
  load_tile<AKC>(As[0], A, p.a_rs, p.a_ks, m0, 0, p.M, p.K);
  load_tile<BKC>(Bs[0], B, p.b_rs, p.b_ks, n0, 0, p.N, p.K);
  cp_async_commit();
  for (int t = 0; t < nk; ++t) {
    const int cur = t & 1;
    if (t + 1 < nk) {
      load_tile<AKC>(As[cur ^ 1], A, p.a_rs, p.a_ks, m0, (t + 1) * kDBK, p.M, p.K);
      load_tile<BKC>(Bs[cur ^ 1], B, p.b_rs, p.b_ks, n0, (t + 1) * kDBK, p.N, p.K);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const double* as = As[cur];
    const double* bs = Bs[cur];
#pragma unroll
    for (int kk = 0; kk < kDBK; kk += 4) {
      double a[4], b[4];
      const int kr = kk + (lane & 3);
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = as[kr * kDPitch + wm + i * 8 + (lane >> 2)];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = bs[kr * kDPitch + wn + j * 8 + (lane >> 2)];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) dmma_8x8x4(acc[i][j], a[i], b[j]);
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  double* C = p.C + g * p.c_gs;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = m0 + wm + i * 8 + (lane >> 2);
    if (row >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = n0 + wn + j * 8 + (lane & 3) * 2 + h;
        if (col >= p.N) continue;
        double v = p.alpha * acc[i][j][h];
        if (p.col_scale) v *= p.col_scale[col];
        double* c = C + row * p.c_rs + col * p.c_cs;
        if (p.beta != 0.0) v += p.beta * *c;
        *c = v;
      }
    }
  }
}

}  // namespace

// Batched strided FP64 GEMM.  A, B, C are fp64 CUDA tensors holding the
// operands at the given element strides (the tensors' own shapes are not
// used beyond bounds checks of the largest offset).
void dgemm_strided(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, int64_t M, int64_t N, int64_t K,
                   int64_t G, at::IntArrayRef a_str, at::IntArrayRef b_str, at::IntArrayRef c_str,
                   double alpha, double beta, const c10::optional<at::Tensor>& col_scale) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "dgemm_strided: CUDA tensors expected");
  TORCH_CHECK(A.scalar_type() == at::kDouble && B.scalar_type() == at::kDouble && C.scalar_type() == at::kDouble,
              "dgemm_strided: fp64 operands expected");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && C.is_contiguous(),
              "dgemm_strided: operands are addressed through explicit strides of contiguous storage");
  TORCH_CHECK(a_str.size() == 3 && b_str.size() == 3 && c_str.size() == 3, "strides: (row, k|col, batch)");
  TORCH_CHECK(M > 0 && N > 0 && K > 0 && G > 0 && G <= 65535 && (M + kDBM - 1) / kDBM <= 65535,
              "dgemm_strided: sizes out of range");
  auto last = [](at::IntArrayRef s, int64_t r, int64_t c, int64_t g) {
    return (r - 1) * s[0] + (c - 1) * s[1] + (g - 1) * s[2];
  };
  TORCH_CHECK(last(a_str, M, K, G) < A.numel() && last(b_str, N, K, G) < B.numel() &&
                  last(c_str, M, N, G) < C.numel(),
              "dgemm_strided: operand strides reach beyond the tensors");
  for (at::IntArrayRef v : {a_str, b_str, c_str})
    for (int64_t x : v) TORCH_CHECK(x >= 0, "dgemm_strided: negative strides are not supported");
  c10::cuda::CUDAGuard guard(A.device());
  DgemmArgs p;
  p.A = A.data_ptr<double>();
  p.B = B.data_ptr<double>();
  p.C = C.data_ptr<double>();
  p.col_scale = nullptr;
  if (col_scale.has_value() && col_scale->defined()) {
    TORCH_CHECK(col_scale->is_cuda() && col_scale->scalar_type() == at::kDouble && col_scale->numel() >= N &&
                    col_scale->is_contiguous(),
                "col_scale must be a contiguous fp64 CUDA vector of length >= N");
    p.col_scale = col_scale->data_ptr<double>();
  }
  p.a_rs = a_str[0]; p.a_ks = a_str[1]; p.a_gs = a_str[2];
  p.b_rs = b_str[0]; p.b_ks = b_str[1]; p.b_gs = b_str[2];
  p.c_rs = c_str[0]; p.c_cs = c_str[1]; p.c_gs = c_str[2];
  p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K); p.G = static_cast<int>(G);
  p.alpha = alpha; p.beta = beta;
  dim3 grid(static_cast<unsigned>((N + kDBN - 1) / kDBN), static_cast<unsigned>((M + kDBM - 1) / kDBM),
            static_cast<unsigned>(G));
  auto st = at::cuda::getCurrentCUDAStream();
  const bool akc = p.a_ks == 1, bkc = p.b_ks == 1;
  if (akc && bkc)
    dgemm_dmma_kernel<true, true><<<grid, kDThreads, 0, st>>>(p);
  else if (akc)
    dgemm_dmma_kernel<true, false><<<grid, kDThreads, 0, st>>>(p);
  else if (bkc)
    dgemm_dmma_kernel<false, true><<<grid, kDThreads, 0, st>>>(p);
  else
    dgemm_dmma_kernel<false, false><<<grid, kDThreads, 0, st>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("dgemm_strided(Tensor A, Tensor B, Tensor(a!) C, int M, int N, int K, int G, int[] a_str, int[] b_str, "
        "int[] c_str, float alpha, float beta, Tensor? col_scale) -> ()");
}

TORCH_LIBRARY_IMPL(tgcm, CUDA, m) { m.impl("dgemm_strided", &tgcm::dgemm_strided); }
