// Spectral-space kernels for sm_100a (with CPU twins sharing the same code):
//
//  * spectral_linear: a table-driven linear map between stacked modal
//    fields, y[b, s, m, l] = Σ_terms coef · post[l] · D( pre[l'] · x[b, src, ., .] )(m, l),
//    where D is one of the spherical-harmonic stencils (identity, ∂/∂λ,
//    cosθ ∂/∂θ, secθ ∂/∂θ cos², and the transposes of the latitudinal
//    ones) or a vertical matrix row.  The spectral pre/post-processing of
//    the explicit tendency, of the neural parameterization and of the
//    encoders are all instances of this op, and an op's adjoint is the
//    same kernel with the transposed term table.
//  * sil3_stage: one IMEX-SIL3 stage on a packed prognostic state
//    (channels [ζ | δ | T' | ln ps | tracers]) — explicit combination, the
//    implicit terms of the stage's z-combination, the per-wavenumber
//    implicit solve, and on the last stage the spectral filter and the
//    inner-state sanitiser — plus its adjoint.
#include "alloc.h"
#include <cstdlib>
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <type_traits>
#include <vector>

#ifndef __CUDACC__
#define __host__
#define __device__
#endif

namespace tgcm {

// Term table rows (int32): dst, src, stencil, pre_diag, post_diag, mat, row; coefficient in a float array.
enum Stencil : int {
  kStId = 0,
  kStDlon = 1,
  kStCdlat = 2,     // cosθ ∂/∂θ
  kStHdlat = 3,     // secθ ∂/∂θ (cos²θ ·)
  kStCdlatT = 4,    // transpose of kStCdlat
  kStHdlatT = 5,    // transpose of kStHdlat
  kStVert = 6,      // Σ_k' M[row, k'] x[src + k']
  kStVertT = 7,     // Σ_k' M[k', row] x[src + k']
};

struct LinearArgs {
  const float* x;
  float* y;
  long long xs_b, xs_c, xs_m;  // input strides (batch, channel, m); l stride 1
  long long ys_b, ys_c, ys_m;  // output strides
  const int* row_ptr;          // (C_out + 1) CSR offsets into terms
  const int* terms;            // (n_terms, 7)
  const float* coef;           // (n_terms)
  const float* diag;           // (n_diag, L)
  const float* rec_a;          // (M2, L) recurrence weights a
  const float* rec_b;          // (M2, L) recurrence weights b
  const float* mats;           // (n_mats, n, n)
  int nlev;                    // matrix size n
  int B, C_out, M2, L;
  // zonal wavenumber of each row, or null for the full layout (row r carries
  // |m| = (r + 1) / 2).  A wavenumber-sharded layout keeps the (cos, sin) rows
  // of one m adjacent at odd/even positions, so only |m| needs the table.
  const int* row_m;
  // Bounds-checked mode (ops.set_bounds_check): every term's channel, stencil,
  // diagonal and matrix indices are checked before use; a bad term records
  // kErrBounds in *err and is skipped instead of being dereferenced.
  int check;
  int* err;
  int C_in, n_diag, n_mats;
};

__host__ __device__ __forceinline__ bool term_in_bounds(const LinearArgs& a, int src, int st, int pre, int post,
                                                        int mat, int row) {
  if (st < 0 || st > 7 || pre < -1 || pre >= a.n_diag || post < -1 || post >= a.n_diag) return false;
  if (st == 6 || st == 7)  // vertical terms read an n-level block and one matrix row
    return mat >= 0 && mat < a.n_mats && row >= 0 && row < a.nlev && src >= 0 && src + a.nlev <= a.C_in;
  return src >= 0 && src < a.C_in;
}

__host__ __device__ __forceinline__ bool term_rejected(const LinearArgs& a, int src, int st, int pre, int post,
                                                       int mat, int row) {
  if (!a.check || term_in_bounds(a, src, st, pre, post, mat, row)) return false;
#ifdef __CUDA_ARCH__
  if (a.err != nullptr) atomicCAS(a.err, 0, 5 /* kErrBounds */);
#endif
  return true;
}

__host__ __device__ __forceinline__ int row_wavenumber(const LinearArgs& a, int mr) {
  return a.row_m ? a.row_m[mr] : (mr + 1) >> 1;
}

__host__ __device__ inline float xval(const LinearArgs& a, int b, int c, int mr, int l, int pre) {
  if (l < 0 || l >= a.L) return 0.f;
  const float v = a.x[b * a.xs_b + c * a.xs_c + mr * a.xs_m + l];
  return pre >= 0 ? v * a.diag[pre * a.L + l] : v;
}

__host__ __device__ inline float stencil_val(const LinearArgs& a, int b, int src, int st, int pre, int mr, int l,
                                             int mat, int row) {
  switch (st) {
    case kStId:
      return xval(a, b, src, mr, l, pre);
    case kStDlon: {
      if (mr == 0) return 0.f;
      const int j = row_wavenumber(a, mr);
      return (mr & 1) ? j * xval(a, b, src, mr + 1, l, pre) : -j * xval(a, b, src, mr - 1, l, pre);
    }
    case kStCdlat: {
      float r = 0.f;
      if (l + 1 < a.L) r += (l + 2) * a.rec_a[mr * a.L + l + 1] * xval(a, b, src, mr, l + 1, pre);
      if (l - 1 >= 0) r -= (l - 1) * a.rec_b[mr * a.L + l - 1] * xval(a, b, src, mr, l - 1, pre);
      return r;
    }
    case kStHdlat: {
      float r = 0.f;
      if (l + 1 < a.L) r += l * a.rec_a[mr * a.L + l + 1] * xval(a, b, src, mr, l + 1, pre);
      if (l - 1 >= 0) r -= (l + 1) * a.rec_b[mr * a.L + l - 1] * xval(a, b, src, mr, l - 1, pre);
      return r;
    }
    case kStCdlatT: {
      float r = 0.f;
      if (l - 1 >= 0) r += (l + 1) * a.rec_a[mr * a.L + l] * xval(a, b, src, mr, l - 1, pre);
      if (l + 1 < a.L) r -= l * a.rec_b[mr * a.L + l] * xval(a, b, src, mr, l + 1, pre);
      return r;
    }
    case kStHdlatT: {
      float r = 0.f;
      if (l - 1 >= 0) r += (l - 1) * a.rec_a[mr * a.L + l] * xval(a, b, src, mr, l - 1, pre);
      if (l + 1 < a.L) r -= (l + 2) * a.rec_b[mr * a.L + l] * xval(a, b, src, mr, l + 1, pre);
      return r;
    }
    case kStVert: {
      const float* M = a.mats + static_cast<long long>(mat) * a.nlev * a.nlev;
      float r = 0.f;
      for (int k = 0; k < a.nlev; ++k) r += M[row * a.nlev + k] * xval(a, b, src + k, mr, l, pre);
      return r;
    }
    case kStVertT: {
      const float* M = a.mats + static_cast<long long>(mat) * a.nlev * a.nlev;
      float r = 0.f;
      for (int k = 0; k < a.nlev; ++k) r += M[k * a.nlev + row] * xval(a, b, src + k, mr, l, pre);
      return r;
    }
    default:
      return 0.f;
  }
}

__host__ __device__ inline void linear_point(const LinearArgs& a, int b, int s, int mr, int l) {
  float acc = 0.f;
  for (int t = a.row_ptr[s]; t < a.row_ptr[s + 1]; ++t) {
    const int* T = a.terms + 7 * t;
    if (term_rejected(a, T[1], T[2], T[3], T[4], T[5], T[6])) continue;
    float v = stencil_val(a, b, T[1], T[2], T[3], mr, l, T[5], T[6]);
    if (T[4] >= 0) v *= a.diag[T[4] * a.L + l];
    acc += a.coef[t] * v;
  }
  a.y[b * a.ys_b + s * a.ys_c + mr * a.ys_m + l] = acc;
}

// grid: x over the (m, l) plane of one output channel (one point per thread),
// y over (b, channel); the channel's terms are warp-uniform read-only loads
// and addressing inside one batch sample uses 32-bit offsets.
constexpr int kLinThreads = 256;

struct LinSample {  // one batch sample's input with 32-bit strides
  const float* x;
  int sc, sm, L;
  __device__ __forceinline__ float at(int c, int mr, int l, const float* diag, int pre) const {
    if (l < 0 || l >= L) return 0.f;
    const float v = __ldg(x + c * sc + mr * sm + l);
    return pre >= 0 ? v * __ldg(diag + pre * L + l) : v;
  }
};

__device__ __forceinline__ float stencil_fast(const LinearArgs& a, const LinSample& xs, int src, int st, int pre,
                                              int mr, int l, int mat, int row) {
  const int L = a.L;
  switch (st) {
    case kStId:
      return xs.at(src, mr, l, a.diag, pre);
    case kStDlon: {
      if (mr == 0) return 0.f;
      const int j = row_wavenumber(a, mr);
      return (mr & 1) ? j * xs.at(src, mr + 1, l, a.diag, pre) : -j * xs.at(src, mr - 1, l, a.diag, pre);
    }
    case kStCdlat:
      return (l + 1 < L ? (l + 2) * __ldg(a.rec_a + mr * L + l + 1) * xs.at(src, mr, l + 1, a.diag, pre) : 0.f) -
             (l >= 1 ? (l - 1) * __ldg(a.rec_b + mr * L + l - 1) * xs.at(src, mr, l - 1, a.diag, pre) : 0.f);
    case kStHdlat:
      return (l + 1 < L ? l * __ldg(a.rec_a + mr * L + l + 1) * xs.at(src, mr, l + 1, a.diag, pre) : 0.f) -
             (l >= 1 ? (l + 1) * __ldg(a.rec_b + mr * L + l - 1) * xs.at(src, mr, l - 1, a.diag, pre) : 0.f);
    case kStCdlatT:
      return (l >= 1 ? (l + 1) * __ldg(a.rec_a + mr * L + l) * xs.at(src, mr, l - 1, a.diag, pre) : 0.f) -
             (l + 1 < L ? l * __ldg(a.rec_b + mr * L + l) * xs.at(src, mr, l + 1, a.diag, pre) : 0.f);
    case kStHdlatT:
      return (l >= 1 ? (l - 1) * __ldg(a.rec_a + mr * L + l) * xs.at(src, mr, l - 1, a.diag, pre) : 0.f) -
             (l + 1 < L ? (l + 2) * __ldg(a.rec_b + mr * L + l) * xs.at(src, mr, l + 1, a.diag, pre) : 0.f);
    default:
      return stencil_val(a, 0, src, st, pre, mr, l, mat, row);  // vertical terms: generic path
  }
}

__global__ void __launch_bounds__(kLinThreads) spectral_linear_kernel(LinearArgs a) {
  const int plane = a.M2 * a.L;
  const int idx = blockIdx.x * kLinThreads + threadIdx.x;
  if (idx >= plane) return;
  const int s = blockIdx.y % a.C_out;
  const int b = blockIdx.y / a.C_out;
  const int mr = idx / a.L;
  const int l = idx - mr * a.L;
  LinearArgs ab = a;  // vertical stencils use the generic path on the shifted sample
  ab.x = a.x + b * a.xs_b;
  const LinSample xs{ab.x, static_cast<int>(a.xs_c), static_cast<int>(a.xs_m), a.L};
  const int t0 = __ldg(a.row_ptr + s), t1 = __ldg(a.row_ptr + s + 1);
  float acc = 0.f;
  for (int t = t0; t < t1; ++t) {
    const int* T = a.terms + 7 * t;
    if (term_rejected(a, __ldg(T + 1), __ldg(T + 2), __ldg(T + 3), __ldg(T + 4), __ldg(T + 5), __ldg(T + 6)))
      continue;
    float v = stencil_fast(ab, xs, __ldg(T + 1), __ldg(T + 2), __ldg(T + 3), mr, l, __ldg(T + 5), __ldg(T + 6));
    const int post = __ldg(T + 4);
    if (post >= 0) v *= __ldg(a.diag + post * a.L + l);
    acc = fmaf(__ldg(a.coef + t), v, acc);
  }
  float* yrow = a.y + b * a.ys_b + s * a.ys_c + mr * a.ys_m;
  yrow[l] = acc;
  if (l == a.L - 1)
    for (long long z = a.L; z < a.ys_m; ++z) yrow[z] = 0.f;  // zero the 16-byte row padding
}

// Row kernel: one warp per (b, output channel, m-row); lane handles
// l = lane + 32 j (j < NL).  For each term the warp reads the source row once
// (coalesced, pre-diagonal applied) into a per-warp shared buffer, from which
// the ±1-in-l neighbours of the latitudinal stencils are taken; ∂/∂λ switches
// the source row to the paired ±m row.  Vertical terms use the per-point path.
constexpr int kRowWarps = 8;

// NB batch samples per warp: the recipe tables are identical for every sample,
// so each term's metadata, coefficient, diagonal and recurrence weights are
// read once and applied to NB rows (the kernel is instruction-bound on that
// per-term work).  grid = (m-row blocks, C_out, ceil(B / NB)).
// Up to three 32-wide l chunks fit in 64 registers, which allows four blocks
// (32 warps) per SM: the kernel is latency-bound, so occupancy is what counts.
template <int NL, int NB>
__global__ void __launch_bounds__(32 * kRowWarps, (NL <= 3 ? 4 : 2)) spectral_linear_rows_kernel(LinearArgs a) {
  __shared__ float sbuf[kRowWarps][NB][32 * NL + 2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mr = blockIdx.x * kRowWarps + warp;
  if (mr >= a.M2) return;
  const int s = blockIdx.y;
  const int b0 = blockIdx.z * NB;
  const int nb = min(NB, a.B - b0);
  const int L = a.L;
  float acc[NB][NL];
#pragma unroll
  for (int q = 0; q < NB; ++q)
#pragma unroll
    for (int j = 0; j < NL; ++j) acc[q][j] = 0.f;
  const int t0 = __ldg(a.row_ptr + s), t1 = __ldg(a.row_ptr + s + 1);
  for (int t = t0; t < t1; ++t) {
    const int* T = a.terms + 7 * t;
    const int src = __ldg(T + 1), st = __ldg(T + 2), pre = __ldg(T + 3), post = __ldg(T + 4);
    const float cf = __ldg(a.coef + t);
    if (term_rejected(a, src, st, pre, post, __ldg(T + 5), __ldg(T + 6))) continue;
    if (st == kStVert || st == kStVertT) {
      const int mat = __ldg(T + 5), row = __ldg(T + 6);
#pragma unroll
      for (int q = 0; q < NB; ++q) {
        if (q >= nb) break;
        LinearArgs ab = a;
        ab.x = a.x + (b0 + q) * a.xs_b;
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          const int l = lane + 32 * j;
          if (l < L) {
            float v = stencil_val(ab, 0, src, st, pre, mr, l, mat, row);
            if (post >= 0) v *= __ldg(a.diag + post * L + l);
            acc[q][j] = fmaf(cf, v, acc[q][j]);
          }
        }
      }
      continue;
    }
    int srow = mr;
    float fac = 1.f;
    if (st == kStDlon) {
      if (mr == 0) continue;
      const int jm = row_wavenumber(a, mr);
      srow = (mr & 1) ? mr + 1 : mr - 1;
      fac = (mr & 1) ? static_cast<float>(jm) : -static_cast<float>(jm);
    }
    // per-l factors shared by all samples
    float pdiag[NL], qdiag[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int l = lane + 32 * j;
      pdiag[j] = (pre >= 0 && l < L) ? __ldg(a.diag + pre * L + l) : 1.f;
      qdiag[j] = (post >= 0 && l < L) ? cf * __ldg(a.diag + post * L + l) : cf;
    }
    const float* xr0 = a.x + src * a.xs_c + srow * a.xs_m;
    float xv[NB][NL];
#pragma unroll
    for (int q = 0; q < NB; ++q)
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const int l = lane + 32 * j;
        xv[q][j] = (q < nb && l < L) ? __ldg(xr0 + (b0 + q) * a.xs_b + l) * pdiag[j] : 0.f;
      }
    const bool lat = st == kStCdlat || st == kStHdlat || st == kStCdlatT || st == kStHdlatT;
    if (!lat) {
#pragma unroll
      for (int q = 0; q < NB; ++q)
#pragma unroll
        for (int j = 0; j < NL; ++j) acc[q][j] = fmaf(qdiag[j] * fac, xv[q][j], acc[q][j]);
      continue;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < NB; ++q) {
      float* buf = sbuf[warp][q] + 1;  // buf[l] for l in [-1, 32*NL]
#pragma unroll
      for (int j = 0; j < NL; ++j) buf[lane + 32 * j] = xv[q][j];
      if (lane == 0) {
        buf[-1] = 0.f;
        buf[32 * NL] = 0.f;
      }
    }
    __syncwarp();
    const float* ra = a.rec_a + mr * L;
    const float* rb = a.rec_b + mr * L;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int l = lane + 32 * j;
      if (l >= L) continue;
      // v = cp * x[l+1] + cm * x[l-1]
      float cp, cm;
      if (st == kStCdlat) {
        cp = (l + 1 < L) ? (l + 2) * __ldg(ra + l + 1) : 0.f;
        cm = (l >= 1) ? -(l - 1) * __ldg(rb + l - 1) : 0.f;
      } else if (st == kStHdlat) {
        cp = (l + 1 < L) ? l * __ldg(ra + l + 1) : 0.f;
        cm = (l >= 1) ? -(l + 1) * __ldg(rb + l - 1) : 0.f;
      } else if (st == kStCdlatT) {
        cm = (l >= 1) ? (l + 1) * __ldg(ra + l) : 0.f;
        cp = (l + 1 < L) ? -l * __ldg(rb + l) : 0.f;
      } else {
        cm = (l >= 1) ? (l - 1) * __ldg(ra + l) : 0.f;
        cp = (l + 1 < L) ? -(l + 2) * __ldg(rb + l) : 0.f;
      }
      cp *= qdiag[j];
      cm *= qdiag[j];
#pragma unroll
      for (int q = 0; q < NB; ++q) {
        const float* buf = sbuf[warp][q] + 1;
        const float xp = (l + 1 < L) ? buf[l + 1] : 0.f;
        const float xm = (l >= 1) ? buf[l - 1] : 0.f;
        acc[q][j] = fmaf(cp, xp, fmaf(cm, xm, acc[q][j]));
      }
    }
  }
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    if (q >= nb) break;
    float* yrow = a.y + (b0 + q) * a.ys_b + s * a.ys_c + mr * a.ys_m;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int l = lane + 32 * j;
      if (l < L)
        yrow[l] = acc[q][j];
      else if (l < a.ys_m)
        yrow[l] = 0.f;  // 16-byte row padding
    }
    for (long long z = 32 * NL + lane; z < a.ys_m; z += 32) yrow[z] = 0.f;
  }
}

// Pipelined row kernel.  The warps of a block share one output channel, so
// the channel's term table (up to kPfTerms entries) is staged once in shared
// memory; each warp then issues the source-row loads of term t + 1 before it
// works on term t, so the latency of one term's loads overlaps the previous
// term's arithmetic instead of adding to it.  Arithmetic is that of
// spectral_linear_rows_kernel.
constexpr int kPfTerms = 64;

struct PfTerm {
  int src, st, pre, post, mat, row;
  float cf;
};

// Blocks per SM: the pipeline keeps three NB x NL register arrays (sums, the
// current and the next source rows) live.
template <int NL, int NB>
struct PfOcc {
  static constexpr int value = NB * NL <= 8 ? 4 : (NB * NL <= 12 ? 3 : 2);
};

template <int NL, int NB>
__global__ void __launch_bounds__(32 * kRowWarps, (PfOcc<NL, NB>::value)) spectral_linear_rows_pf_kernel(LinearArgs a) {
  __shared__ float sbuf[kRowWarps][NB][32 * NL + 2];
  __shared__ PfTerm sterm[kPfTerms];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.y;
  const int t0 = __ldg(a.row_ptr + s), t1 = __ldg(a.row_ptr + s + 1);
  const int nt = t1 - t0;
  for (int i = threadIdx.x; i < nt && i < kPfTerms; i += blockDim.x) {
    const int* T = a.terms + 7 * (t0 + i);
    sterm[i] = PfTerm{__ldg(T + 1), __ldg(T + 2), __ldg(T + 3), __ldg(T + 4), __ldg(T + 5), __ldg(T + 6),
                      __ldg(a.coef + t0 + i)};
  }
  __syncthreads();
  const int mr = blockIdx.x * kRowWarps + warp;
  if (mr >= a.M2) return;
  const int b0 = blockIdx.z * NB;
  const int nb = min(NB, a.B - b0);
  const int L = a.L;
  auto term = [&](int i) -> PfTerm {
    if (i < kPfTerms) return sterm[i];
    const int* T = a.terms + 7 * (t0 + i);
    return PfTerm{__ldg(T + 1), __ldg(T + 2), __ldg(T + 3), __ldg(T + 4), __ldg(T + 5), __ldg(T + 6),
                  __ldg(a.coef + t0 + i)};
  };
  // source row of a non-vertical term (the paired ±m row for ∂/∂λ); -1: term contributes nothing
  auto source_row = [&](const PfTerm& m) -> int {
    if (a.check && !term_in_bounds(a, m.src, m.st, m.pre, m.post, m.mat, m.row)) return -1;
    if (m.st == kStVert || m.st == kStVertT) return -1;
    if (m.st == kStDlon) return mr == 0 ? -1 : ((mr & 1) ? mr + 1 : mr - 1);
    return mr;
  };
  auto issue = [&](int i, float (&xo)[NB][NL]) {
    const PfTerm m = term(i);
    const int srow = source_row(m);
    const float* xr0 = a.x + m.src * a.xs_c + (srow < 0 ? 0 : srow) * a.xs_m;
#pragma unroll
    for (int q = 0; q < NB; ++q)
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const int l = lane + 32 * j;
        xo[q][j] = (srow >= 0 && q < nb && l < L) ? __ldg(xr0 + (b0 + q) * a.xs_b + l) : 0.f;
      }
  };
  float acc[NB][NL];
#pragma unroll
  for (int q = 0; q < NB; ++q)
#pragma unroll
    for (int j = 0; j < NL; ++j) acc[q][j] = 0.f;
  float xn[NB][NL];
  if (nt > 0) issue(0, xn);
  for (int i = 0; i < nt; ++i) {
    float xv[NB][NL];
#pragma unroll
    for (int q = 0; q < NB; ++q)
#pragma unroll
      for (int j = 0; j < NL; ++j) xv[q][j] = xn[q][j];
    if (i + 1 < nt) issue(i + 1, xn);
    const PfTerm m = term(i);
    if (term_rejected(a, m.src, m.st, m.pre, m.post, m.mat, m.row)) continue;
    if (m.st == kStVert || m.st == kStVertT) {
#pragma unroll
      for (int q = 0; q < NB; ++q) {
        if (q >= nb) break;
        LinearArgs ab = a;
        ab.x = a.x + (b0 + q) * a.xs_b;
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          const int l = lane + 32 * j;
          if (l < L) {
            float v = stencil_val(ab, 0, m.src, m.st, m.pre, mr, l, m.mat, m.row);
            if (m.post >= 0) v *= __ldg(a.diag + m.post * L + l);
            acc[q][j] = fmaf(m.cf, v, acc[q][j]);
          }
        }
      }
      continue;
    }
    if (source_row(m) < 0) continue;
    float fac = 1.f;
    if (m.st == kStDlon) {
      const int jm = row_wavenumber(a, mr);
      fac = (mr & 1) ? static_cast<float>(jm) : -static_cast<float>(jm);
    }
    float qdiag[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int l = lane + 32 * j;
      const float pd = (m.pre >= 0 && l < L) ? __ldg(a.diag + m.pre * L + l) : 1.f;
#pragma unroll
      for (int q = 0; q < NB; ++q) xv[q][j] *= pd;
      qdiag[j] = (m.post >= 0 && l < L) ? m.cf * __ldg(a.diag + m.post * L + l) : m.cf;
    }
    const bool lat = m.st == kStCdlat || m.st == kStHdlat || m.st == kStCdlatT || m.st == kStHdlatT;
    if (!lat) {
#pragma unroll
      for (int q = 0; q < NB; ++q)
#pragma unroll
        for (int j = 0; j < NL; ++j) acc[q][j] = fmaf(qdiag[j] * fac, xv[q][j], acc[q][j]);
      continue;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < NB; ++q) {
      float* buf = sbuf[warp][q] + 1;  // buf[l] for l in [-1, 32*NL]
#pragma unroll
      for (int j = 0; j < NL; ++j) buf[lane + 32 * j] = xv[q][j];
      if (lane == 0) {
        buf[-1] = 0.f;
        buf[32 * NL] = 0.f;
      }
    }
    __syncwarp();
    const float* ra = a.rec_a + mr * L;
    const float* rb = a.rec_b + mr * L;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int l = lane + 32 * j;
      if (l >= L) continue;
      float cp, cm;
      if (m.st == kStCdlat) {
        cp = (l + 1 < L) ? (l + 2) * __ldg(ra + l + 1) : 0.f;
        cm = (l >= 1) ? -(l - 1) * __ldg(rb + l - 1) : 0.f;
      } else if (m.st == kStHdlat) {
        cp = (l + 1 < L) ? l * __ldg(ra + l + 1) : 0.f;
        cm = (l >= 1) ? -(l + 1) * __ldg(rb + l - 1) : 0.f;
      } else if (m.st == kStCdlatT) {
        cm = (l >= 1) ? (l + 1) * __ldg(ra + l) : 0.f;
        cp = (l + 1 < L) ? -l * __ldg(rb + l) : 0.f;
      } else {
        cm = (l >= 1) ? (l - 1) * __ldg(ra + l) : 0.f;
        cp = (l + 1 < L) ? -(l + 2) * __ldg(rb + l) : 0.f;
      }
      cp *= qdiag[j];
      cm *= qdiag[j];
#pragma unroll
      for (int q = 0; q < NB; ++q) {
        const float* buf = sbuf[warp][q] + 1;
        const float xp = (l + 1 < L) ? buf[l + 1] : 0.f;
        const float xm = (l >= 1) ? buf[l - 1] : 0.f;
        acc[q][j] = fmaf(cp, xp, fmaf(cm, xm, acc[q][j]));
      }
    }
  }
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    if (q >= nb) break;
    float* yrow = a.y + (b0 + q) * a.ys_b + s * a.ys_c + mr * a.ys_m;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int l = lane + 32 * j;
      if (l < L)
        yrow[l] = acc[q][j];
      else if (l < a.ys_m)
        yrow[l] = 0.f;  // 16-byte row padding
    }
    for (long long z = 32 * NL + lane; z < a.ys_m; z += 32) yrow[z] = 0.f;
  }
}

// Row-kernel variant: the pipelined kernel up to five 32-wide l chunks (measured
// at TL63, post recipe and its adjoint: 0.142 -> 0.130 ms and 0.119 -> 0.101 ms;
// whole training step 389 -> 379 ms); beyond that its three register arrays
// spill and the unpipelined kernel runs.  TGCM_RECIPE_PIPELINE=0 / 1 forces
// one variant (for comparisons).
static bool recipe_pipelined(int nl) {
  static int v = -2;
  if (v == -2) {
    const char* e = std::getenv("TGCM_RECIPE_PIPELINE");
    v = (e == nullptr || e[0] == '\0') ? -1 : (e[0] == '0' ? 0 : 1);
  }
  return v < 0 ? nl <= 5 : v == 1;
}

template <int NL, int NB>
static void launch_rows_nb(const LinearArgs& a, cudaStream_t st) {
  dim3 grid(static_cast<unsigned>((a.M2 + kRowWarps - 1) / kRowWarps), static_cast<unsigned>(a.C_out),
            static_cast<unsigned>((a.B + NB - 1) / NB));
  if (recipe_pipelined(NL))
    spectral_linear_rows_pf_kernel<NL, NB><<<grid, 32 * kRowWarps, 0, st>>>(a);
  else
    spectral_linear_rows_kernel<NL, NB><<<grid, 32 * kRowWarps, 0, st>>>(a);
}

template <int NL>
static void launch_rows(const LinearArgs& a, cudaStream_t st) {
  if (a.B >= 4 && NL <= 5)
    launch_rows_nb<NL, 4>(a, st);
  else if (a.B >= 2)
    launch_rows_nb<NL, 2>(a, st);
  else
    launch_rows_nb<NL, 1>(a, st);
}

// Bounds-checked mode of the table-driven kernels (debug; off by default).
static bool g_bounds_check = false;

void set_bounds_check(bool on) { g_bounds_check = on; }

bool bounds_check_enabled() { return g_bounds_check; }

// x: (B, C_in, M2, Lx) ; returns y: (B, C_out, M2, Ly) with Ly = out_lpad (>= L), pad zero.
at::Tensor spectral_linear(const at::Tensor& x, int64_t L, int64_t C_out, int64_t out_lpad, const at::Tensor& row_ptr,
                           const at::Tensor& terms, const at::Tensor& coef, const at::Tensor& diag,
                           const at::Tensor& rec_a, const at::Tensor& rec_b, const at::Tensor& mats, int64_t nlev,
                           const c10::optional<at::Tensor>& row_m, const c10::optional<at::Tensor>& err) {
  TORCH_CHECK(x.dim() == 4 && x.scalar_type() == at::kFloat && x.stride(3) == 1, "x must be (B, C, M2, L) fp32");
  const int64_t B = x.size(0), M2 = x.size(2);
  // the CUDA kernel writes the padding columns itself; the CPU loop does not
  auto y = (out_lpad > L && !x.is_cuda()) ? at::zeros({B, C_out, M2, out_lpad}, x.options())
                                          : out_empty({B, C_out, M2, out_lpad}, x.options());
  LinearArgs a;
  a.x = x.data_ptr<float>();
  a.y = y.data_ptr<float>();
  a.xs_b = x.stride(0); a.xs_c = x.stride(1); a.xs_m = x.stride(2);
  a.ys_b = y.stride(0); a.ys_c = y.stride(1); a.ys_m = y.stride(2);
  a.row_ptr = row_ptr.data_ptr<int>();
  a.terms = terms.data_ptr<int>();
  a.coef = coef.data_ptr<float>();
  a.diag = diag.data_ptr<float>();
  a.rec_a = rec_a.data_ptr<float>();
  a.rec_b = rec_b.data_ptr<float>();
  a.mats = mats.data_ptr<float>();
  a.nlev = static_cast<int>(nlev);
  a.B = static_cast<int>(B); a.C_out = static_cast<int>(C_out); a.M2 = static_cast<int>(M2); a.L = static_cast<int>(L);
  a.check = g_bounds_check ? 1 : 0;
  a.err = (err.has_value() && err->defined() && err->is_cuda() == x.is_cuda()) ? err->data_ptr<int>() : nullptr;
  a.C_in = static_cast<int>(x.size(1));
  a.n_diag = static_cast<int>(diag.size(0));
  a.n_mats = static_cast<int>(mats.size(0));
  a.row_m = nullptr;
  if (row_m.has_value() && row_m->defined()) {
    TORCH_CHECK(row_m->scalar_type() == at::kInt && row_m->numel() == M2 && row_m->is_contiguous() &&
                    row_m->device() == x.device(),
                "row_m must be a contiguous int32 (M2) tensor on x's device");
    a.row_m = row_m->data_ptr<int>();
  }
  if (x.is_cuda()) {
    c10::cuda::CUDAGuard guard(x.device());
    TORCH_CHECK(C_out <= 65535 && B <= 65535 && M2 * L < (1LL << 31), "spectral_linear: launch grid too large");
    TORCH_CHECK(x.stride(1) < (1LL << 31) && x.size(1) * x.stride(1) < (1LL << 31),
                "spectral_linear: one batch sample must fit 32-bit offsets");
    auto st = at::cuda::getCurrentCUDAStream();
    if (L <= 32) launch_rows<1>(a, st);
    else if (L <= 64) launch_rows<2>(a, st);
    else if (L <= 96) launch_rows<3>(a, st);
    else if (L <= 160) launch_rows<5>(a, st);
    else if (L <= 288) launch_rows<9>(a, st);
    else {
      dim3 grid(static_cast<unsigned>((M2 * L + kLinThreads - 1) / kLinThreads), static_cast<unsigned>(B * C_out));
      spectral_linear_kernel<<<grid, kLinThreads, 0, st>>>(a);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    for (int b = 0; b < B; ++b)
      for (int s = 0; s < C_out; ++s)
        for (int mr = 0; mr < M2; ++mr)
          for (int l = 0; l < L; ++l) linear_point(a, b, s, mr, l);
  }
  return y;
}

// ── SIL3 stage on a packed state ───────────────────────────────────────────
constexpr int kStageMaxLev = 64;
constexpr int kStageMaxE = 3;

struct StageArgs {
  // packed tensors (B, C, M2, L) contiguous
  const float* y0;
  const float* E[kStageMaxE];
  const float* P;
  const float* y2;    // extra implicit-combination input (stage 3) or null
  float* out;
  const float* gin;   // adjoint: cotangent of the stage output
  float* g_y0;
  float* g_E[kStageMaxE];
  float* g_P;
  float* g_y2;
  float ce[kStageMaxE];
  int nE;
  float cp, cg, eta;
  const float* G; const float* H; const float* Minv; const float* lam; const float* tref; const float* dsig;
  const float* MinvT;  // (n*n, L): MinvT[(i*n + j)*L + l] = Minv[l][i][j], or null
  const float* filt;  // (L) or null
  float clamp_abs;
  float R;
  int final_stage;
  int B, C, n, M2, L;
};

template <typename Mat>
__host__ __device__ void stage_column_fwd(const StageArgs& a, int b, int mr, int l, Mat mat) {
  const int n = a.n;
  const long long cs = static_cast<long long>(a.M2) * a.L;
  const long long base = static_cast<long long>(b) * a.C * cs + static_cast<long long>(mr) * a.L + l;
  auto at_ = [&](const float* p, int c) -> float { return p[base + c * cs]; };
  const float f = a.filt ? a.filt[l] : 1.f;
  auto finish = [&](float v) -> float {
    if (!a.final_stage) return v;
    v *= f;
    if (v != v) v = 0.f;
    if (v > a.clamp_abs) v = a.clamp_abs;
    if (v < -a.clamp_abs) v = -a.clamp_abs;
    return v;
  };
  auto expl = [&](int c) -> float {
    float v = at_(a.y0, c) + a.cp * at_(a.P, c);
    for (int j = 0; j < a.nE; ++j) v += a.ce[j] * at_(a.E[j], c);
    return v;
  };
  // vorticity (channels [0, n)) and tracers (channels [3n+1, C)): explicit only
  for (int c = 0; c < n; ++c) a.out[base + c * cs] = finish(expl(c));
  for (int c = 3 * n + 1; c < a.C; ++c) a.out[base + c * cs] = finish(expl(c));
  // implicit channels
  float zd[kStageMaxLev], zt[kStageMaxLev], rd[kStageMaxLev], rt[kStageMaxLev], od[kStageMaxLev];
  for (int k = 0; k < n; ++k) {
    zd[k] = at_(a.y0, n + k) + (a.y2 ? at_(a.y2, n + k) : 0.f);
    zt[k] = at_(a.y0, 2 * n + k) + (a.y2 ? at_(a.y2, 2 * n + k) : 0.f);
  }
  const float zp = at_(a.y0, 3 * n) + (a.y2 ? at_(a.y2, 3 * n) : 0.f);
  const float lam = a.lam[l];
  float zp_g = 0.f;
  for (int i = 0; i < n; ++i) {
    float gt = 0.f, hd = 0.f;
    for (int j = 0; j < n; ++j) {
      gt += mat(0, i, j) * zt[j];
      hd += mat(1, i, j) * zd[j];
    }
    // rhs = explicit + cg * G(z)
    rd[i] = expl(n + i) + a.cg * (-lam * (gt + a.R * a.tref[i] * zp));
    rt[i] = expl(2 * n + i) + a.cg * (-hd);
    zp_g += a.dsig[i] * zd[i];
  }
  const float rp = expl(3 * n) + a.cg * (-zp_g);
  // solve: r = rd - eta*lam*(G rt + R Tr rp); δ = Minv r; T = rt - eta H δ; p = rp - eta Δσ·δ
  const float el = a.eta * lam;
  float tmp[kStageMaxLev];
  for (int i = 0; i < n; ++i) {
    float gt = 0.f;
    for (int j = 0; j < n; ++j) gt += mat(0, i, j) * rt[j];
    tmp[i] = rd[i] - el * (gt + a.R * a.tref[i] * rp);
  }
  float sp = 0.f;
  for (int i = 0; i < n; ++i) {
    float s = 0.f;
    for (int j = 0; j < n; ++j) s += mat(2, i, j) * tmp[j];
    od[i] = s;
    sp += a.dsig[i] * s;
  }
  for (int i = 0; i < n; ++i) {
    float hd = 0.f;
    for (int j = 0; j < n; ++j) hd += mat(1, i, j) * od[j];
    a.out[base + (n + i) * cs] = finish(od[i]);
    a.out[base + (2 * n + i) * cs] = finish(rt[i] - a.eta * hd);
  }
  a.out[base + 3 * n * cs] = finish(rp - a.eta * sp);
}

template <typename Mat>
__host__ __device__ void stage_column_adj(const StageArgs& a, int b, int mr, int l, Mat mat) {
  const int n = a.n;
  const long long cs = static_cast<long long>(a.M2) * a.L;
  const long long base = static_cast<long long>(b) * a.C * cs + static_cast<long long>(mr) * a.L + l;
  const float f = a.filt ? a.filt[l] : 1.f;
  // cotangent of the pre-filter value: g * f * [not clamped]
  auto gpre = [&](int c) -> float {
    float g = a.gin[base + c * cs];
    if (!a.final_stage) return g;
    const float o = a.out[base + c * cs];  // saved forward output
    if (o >= a.clamp_abs || o <= -a.clamp_abs) return 0.f;
    return g * f;
  };
  auto scatter = [&](int c, float r) {
    a.g_y0[base + c * cs] = r;
    a.g_P[base + c * cs] = a.cp * r;
    for (int j = 0; j < a.nE; ++j) a.g_E[j][base + c * cs] = a.ce[j] * r;
  };
  for (int c = 0; c < n; ++c) scatter(c, gpre(c));
  for (int c = 3 * n + 1; c < a.C; ++c) scatter(c, gpre(c));
  if (a.g_y2) {
    for (int c = 0; c < n; ++c) a.g_y2[base + c * cs] = 0.f;
    for (int c = 3 * n + 1; c < a.C; ++c) a.g_y2[base + c * cs] = 0.f;
  }
  // transpose of the solve: inputs (d̄, t̄, p̄) = cotangents of (δ, T, p)
  float dd[kStageMaxLev], tt[kStageMaxLev], r[kStageMaxLev], od[kStageMaxLev], ot[kStageMaxLev];
  for (int k = 0; k < n; ++k) {
    dd[k] = gpre(n + k);
    tt[k] = gpre(2 * n + k);
  }
  const float pp = gpre(3 * n);
  const float lam = a.lam[l];
  const float el = a.eta * lam;
  for (int i = 0; i < n; ++i) {
    float htt = 0.f;
    for (int j = 0; j < n; ++j) htt += mat(1, j, i) * tt[j];
    r[i] = dd[i] - a.eta * htt - a.eta * a.dsig[i] * pp;
  }
  float trd = 0.f;
  for (int i = 0; i < n; ++i) {
    float s = 0.f;
    for (int j = 0; j < n; ++j) s += mat(2, j, i) * r[j];
    od[i] = s;  // cotangent of rd (δ* side)
    trd += a.tref[i] * s;
  }
  for (int i = 0; i < n; ++i) {
    float gtr = 0.f;
    for (int j = 0; j < n; ++j) gtr += mat(0, j, i) * od[j];
    ot[i] = tt[i] - el * gtr;  // cotangent of rt
  }
  const float op = pp - el * a.R * trd;  // cotangent of rp
  // rhs = explicit + cg * G(z): explicit part
  for (int i = 0; i < n; ++i) {
    scatter(n + i, od[i]);
    scatter(2 * n + i, ot[i]);
  }
  scatter(3 * n, op);
  // z-part: z̄ = cg Gᵀ(ō) with Gᵀ: δ̄z = −Hᵀ t̄ − Δσ p̄ ; T̄z = −λ Gᵀ d̄ ; p̄z = −λ R Tr·d̄
  float trdot = 0.f;
  for (int i = 0; i < n; ++i) trdot += a.tref[i] * od[i];
  for (int i = 0; i < n; ++i) {
    float htb = 0.f, gta = 0.f;
    for (int j = 0; j < n; ++j) {
      htb += mat(1, j, i) * ot[j];
      gta += mat(0, j, i) * od[j];
    }
    const float zd = a.cg * (-htb - a.dsig[i] * op);
    const float zt = a.cg * (-lam * gta);
    a.g_y0[base + (n + i) * cs] += zd;
    a.g_y0[base + (2 * n + i) * cs] += zt;
    if (a.g_y2) {
      a.g_y2[base + (n + i) * cs] = zd;
      a.g_y2[base + (2 * n + i) * cs] = zt;
    }
  }
  const float zp = a.cg * (-lam * a.R * trdot);
  a.g_y0[base + 3 * n * cs] += zp;
  if (a.g_y2) a.g_y2[base + 3 * n * cs] = zp;
}

constexpr int kStageL = 4;
constexpr int kStageM = 32;

__global__ void sil3_stage_kernel(StageArgs a, int adjoint) {
  extern __shared__ float sm[];
  const int n = a.n;
  float* sG = sm;
  float* sH = sG + n * n;
  float* sMi = sH + n * n;
  const int l0 = blockIdx.x * kStageL;
  const int b = blockIdx.y;
  for (int i = threadIdx.x; i < n * n; i += blockDim.x) {
    sG[i] = a.G[i];
    sH[i] = a.H[i];
  }
  for (int i = threadIdx.x; i < kStageL * n * n; i += blockDim.x) {
    const int ll = l0 + i / (n * n);
    sMi[i] = ll < a.L ? a.Minv[static_cast<long long>(ll) * n * n + i % (n * n)] : 0.f;
  }
  __syncthreads();
  const int tl = threadIdx.x % kStageL;
  const int tm = threadIdx.x / kStageL;
  const int l = l0 + tl;
  if (l >= a.L) return;
  const float* mi = sMi + tl * n * n;
  auto mat = [sG, sH, mi, n](int kind, int i, int j) -> float {
    return kind == 0 ? sG[i * n + j] : (kind == 1 ? sH[i * n + j] : mi[i * n + j]);
  };
  for (int m = tm; m < a.M2; m += kStageM) {
    if (adjoint)
      stage_column_adj(a, b, m, l, mat);
    else
      stage_column_fwd(a, b, m, l, mat);
  }
}

template <bool TRANS>
struct SMat {  // n x n matrix in shared memory with padded row stride
  const float* m;
  int ld;
  __device__ __forceinline__ float operator()(int i, int j) const { return TRANS ? m[j * ld + i] : m[i * ld + j]; }
};

template <bool TRANS>
struct GMat {  // per-l matrix from its l-fastest global copy
  const float* m;
  long long ms;
  int n;
  __device__ __forceinline__ float operator()(int i, int j) const {
    return TRANS ? m[(j * n + i) * ms] : m[(i * n + j) * ms];
  }
};

// yo[kk] = Σ_j M(q*P + kk, j) x_j; x is spread over the Q lanes of the group
// (lane gl + qq owns x[qq*P .. qq*P + P-1]) and gathered with shuffles.
template <int P, int Q, typename Mat>
__device__ __forceinline__ void mv_group(const Mat& M, const float (&xo)[P], float (&yo)[P], int q, int gl) {
#pragma unroll
  for (int kk = 0; kk < P; ++kk) yo[kk] = 0.f;
#pragma unroll 1
  for (int qq = 0; qq < Q; ++qq) {
#pragma unroll
    for (int jj = 0; jj < P; ++jj) {
      const float xv = __shfl_sync(0xffffffffu, xo[jj], gl + qq);
#pragma unroll
      for (int kk = 0; kk < P; ++kk) yo[kk] = fmaf(M(q * P + kk, qq * P + jj), xv, yo[kk]);
    }
  }
}

// Quarter-split stage kernel: Q = 4 threads share one (b, m, l) column, each
// owning N / 4 consecutive levels; vectors are exchanged with warp shuffles
// inside the 4-lane group, so a thread keeps 3 x N/4 values in registers
// instead of 3 x N (occupancy) while the arithmetic is that of
// stage_column_fwd / stage_column_adj.  A warp covers 8 consecutive l of one
// (b, m) row: every channel access is a 32-byte run per quarter.
// Four blocks per SM (64 registers, a 104-byte spill): at batch 4 on TL63 the
// 516 blocks of a launch then run in one wave instead of 1.16 waves of three
// blocks per SM (80 registers); the latency-bound kernel went from 53.8 to
// 38.0 ms per training step.
//
// SMI (shared-memory inverse): a block covers kStageLT consecutive l of eight
// (b, m) rows (warp w: row w, lane group g: l = tile + g), so the per-l
// inverses of its columns are the kStageLT matrices of one tile, staged once in
// shared memory (row stride N + 1, matrix stride ≡ 1 mod 32 banks: the 32 lanes
// of a matvec step hit 32 distinct banks) instead of being read per column
// from the l-fastest global copy.
constexpr int kStageLT = 8;

template <bool SMI, bool TR>
__device__ __forceinline__ typename std::conditional<SMI, SMat<TR>, GMat<TR>>::type stage_minv(
    const float* smi, int ld, const float* gmi, long long ms, int n) {
  if constexpr (SMI)
    return SMat<TR>{smi, ld};
  else
    return GMat<TR>{gmi, ms, n};
}

template <int N, bool SMI>
__global__ void __launch_bounds__(256, 4) sil3_stage_q4_kernel(StageArgs a, int adjoint) {
  constexpr int Q = 4;
  constexpr int P = N / Q;
  constexpr int LD = N + 1;  // padded row stride of G, H in shared memory (conflict-free)
  constexpr int MS = N * LD + 1;  // stride of the per-l inverses in the shared tile
  __shared__ float sG[N * LD], sH[N * LD], sTr[N], sDs[N];
  __shared__ float sMi[SMI ? kStageLT * MS : 1];
  for (int i = threadIdx.x; i < N * N; i += blockDim.x) {
    sG[(i / N) * LD + i % N] = a.G[i];
    sH[(i / N) * LD + i % N] = a.H[i];
  }
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    sTr[i] = a.tref[i];
    sDs[i] = a.dsig[i];
  }
  const int n_lt = (a.L + kStageLT - 1) / kStageLT;
  if constexpr (SMI) {
    const int l0 = (blockIdx.x % n_lt) * kStageLT;
    for (int i = threadIdx.x; i < kStageLT * N * N; i += blockDim.x) {
      const int ll = i % kStageLT, ij = i / kStageLT;
      const int lg = l0 + ll;
      sMi[ll * MS + (ij / N) * LD + ij % N] = lg < a.L ? a.MinvT[static_cast<long long>(ij) * a.L + lg] : 0.f;
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int q = lane & (Q - 1);
  const int gl = lane & ~(Q - 1);
  bool valid;
  int b, mr, l;
  if constexpr (SMI) {
    const int lloc = lane >> 2;
    l = (blockIdx.x % n_lt) * kStageLT + lloc;
    const int bm = (blockIdx.x / n_lt) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    valid = l < a.L && bm < a.B * a.M2;
    const int bmv = valid ? bm : 0;
    if (!valid) l = 0;
    b = bmv / a.M2;
    mr = bmv - b * a.M2;
  } else {
    const int total = a.B * a.M2 * a.L;
    const int t = blockIdx.x * (blockDim.x / Q) + threadIdx.x / Q;
    valid = t < total;
    const int tt = valid ? t : 0;
    const int bm = tt / a.L;
    l = tt - bm * a.L;
    b = bm / a.M2;
    mr = bm - b * a.M2;
  }
  const long long cs = static_cast<long long>(a.M2) * a.L;
  const long long base = static_cast<long long>(b) * a.C * cs + static_cast<long long>(mr) * a.L + l;
  const float* mi = a.MinvT + l;
  const float* smi = sMi + (SMI ? (lane >> 2) * MS : 0);
  const long long ms = a.L;
  const float f = a.filt ? a.filt[l] : 1.f;
  const float lam = a.lam[l];
  const float el = a.eta * lam;
  const unsigned full = 0xffffffffu;

  auto group_sum = [&](float v) -> float {
    v += __shfl_xor_sync(full, v, 1);
    v += __shfl_xor_sync(full, v, 2);
    return v;
  };
  const SMat<false> G_{sG, LD};
  const SMat<false> H_{sH, LD};
  const SMat<true> Gt{sG, LD};
  const SMat<true> Ht{sH, LD};
  const auto Mi = stage_minv<SMI, false>(smi, LD, mi, ms, N);
  const auto Mit = stage_minv<SMI, true>(smi, LD, mi, ms, N);

  if (!adjoint) {
    auto finish = [&](float v) -> float {
      if (!a.final_stage) return v;
      v *= f;
      if (v != v) v = 0.f;
      return fminf(fmaxf(v, -a.clamp_abs), a.clamp_abs);
    };
    auto expl = [&](int c) -> float {
      float v = a.y0[base + c * cs] + a.cp * a.P[base + c * cs];
#pragma unroll
      for (int j = 0; j < kStageMaxE; ++j)
        if (j < a.nE) v += a.ce[j] * a.E[j][base + c * cs];
      return v;
    };
    if (valid) {
      for (int c = q; c < N; c += Q) a.out[base + c * cs] = finish(expl(c));
      for (int c = 3 * N + 1 + q; c < a.C; c += Q) a.out[base + c * cs] = finish(expl(c));
    }
    float x[P], y[P], z[P], tmp[P];
    const float zp = valid ? a.y0[base + 3 * N * cs] + (a.y2 ? a.y2[base + 3 * N * cs] : 0.f) : 0.f;
    float zpg = 0.f;
#pragma unroll
    for (int kk = 0; kk < P; ++kk) {
      const int k = q * P + kk;
      x[kk] = valid ? a.y0[base + (N + k) * cs] + (a.y2 ? a.y2[base + (N + k) * cs] : 0.f) : 0.f;
      y[kk] = valid ? a.y0[base + (2 * N + k) * cs] + (a.y2 ? a.y2[base + (2 * N + k) * cs] : 0.f) : 0.f;
      zpg += sDs[k] * x[kk];
    }
    zpg = group_sum(zpg);
    mv_group<P, Q>(G_, y, tmp, q, gl);  // G z_T
#pragma unroll
    for (int kk = 0; kk < P; ++kk) {
      const int i = q * P + kk;
      z[kk] = (valid ? expl(N + i) : 0.f) + a.cg * (-lam * (tmp[kk] + a.R * sTr[i] * zp));
    }
    mv_group<P, Q>(H_, x, tmp, q, gl);  // H z_δ
#pragma unroll
    for (int kk = 0; kk < P; ++kk) y[kk] = (valid ? expl(2 * N + q * P + kk) : 0.f) - a.cg * tmp[kk];
    const float rp = (valid ? expl(3 * N) : 0.f) - a.cg * zpg;
    mv_group<P, Q>(G_, y, tmp, q, gl);  // G rt
#pragma unroll
    for (int kk = 0; kk < P; ++kk) z[kk] -= el * (tmp[kk] + a.R * sTr[q * P + kk] * rp);
    mv_group<P, Q>(Mi, z, x, q, gl);  // δ = Minv z
    float sp = 0.f;
#pragma unroll
    for (int kk = 0; kk < P; ++kk) sp += sDs[q * P + kk] * x[kk];
    sp = group_sum(sp);
    mv_group<P, Q>(H_, x, tmp, q, gl);  // H δ
    if (valid) {
#pragma unroll
      for (int kk = 0; kk < P; ++kk) {
        const int i = q * P + kk;
        a.out[base + (N + i) * cs] = finish(x[kk]);
        a.out[base + (2 * N + i) * cs] = finish(y[kk] - a.eta * tmp[kk]);
      }
      if (q == 0) a.out[base + 3 * N * cs] = finish(rp - a.eta * sp);
    }
    return;
  }
  // adjoint (one kernel for both directions: measured faster than two
  // specialised instances, 53.4 vs 63.9 ms per training step)
  auto gpre = [&](int c) -> float {
    const float g = a.gin[base + c * cs];
    if (!a.final_stage) return g;
    const float o = a.out[base + c * cs];
    if (o >= a.clamp_abs || o <= -a.clamp_abs) return 0.f;
    return g * f;
  };
  auto scatter = [&](int c, float r, float zextra, bool has_z) {
    a.g_y0[base + c * cs] = r + zextra;
    a.g_P[base + c * cs] = a.cp * r;
#pragma unroll
    for (int j = 0; j < kStageMaxE; ++j)
      if (j < a.nE) a.g_E[j][base + c * cs] = a.ce[j] * r;
    if (a.g_y2) a.g_y2[base + c * cs] = has_z ? zextra : 0.f;
  };
  if (valid) {
    for (int c = q; c < N; c += Q) scatter(c, gpre(c), 0.f, false);
    for (int c = 3 * N + 1 + q; c < a.C; c += Q) scatter(c, gpre(c), 0.f, false);
  }
  float x[P], y[P], r[P], tmp[P];
  const float pp = valid ? gpre(3 * N) : 0.f;
#pragma unroll
  for (int kk = 0; kk < P; ++kk) y[kk] = valid ? gpre(2 * N + q * P + kk) : 0.f;  // t̄
  mv_group<P, Q>(Ht, y, tmp, q, gl);  // Hᵀ t̄
#pragma unroll
  for (int kk = 0; kk < P; ++kk) {
    const int i = q * P + kk;
    r[kk] = (valid ? gpre(N + i) : 0.f) - a.eta * tmp[kk] - a.eta * sDs[i] * pp;
  }
  mv_group<P, Q>(Mit, r, x, q, gl);  // od = Minvᵀ r
  float trd = 0.f;
#pragma unroll
  for (int kk = 0; kk < P; ++kk) trd += sTr[q * P + kk] * x[kk];
  trd = group_sum(trd);
  mv_group<P, Q>(Gt, x, tmp, q, gl);  // Gᵀ od
#pragma unroll
  for (int kk = 0; kk < P; ++kk) y[kk] -= el * tmp[kk];  // ot
  const float op = pp - el * a.R * trd;
  mv_group<P, Q>(Ht, y, tmp, q, gl);  // Hᵀ ot
  float gta[P];
  mv_group<P, Q>(Gt, x, gta, q, gl);  // Gᵀ od
  if (valid) {
#pragma unroll
    for (int kk = 0; kk < P; ++kk) {
      const int i = q * P + kk;
      scatter(N + i, x[kk], a.cg * (-tmp[kk] - sDs[i] * op), true);
      scatter(2 * N + i, y[kk], a.cg * (-lam * gta[kk]), true);
    }
    if (q == 0) scatter(3 * N, op, a.cg * (-lam * a.R * trd), true);
  }
}

static const float* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<float>() : nullptr;
}

// Stage kernel variant: 1 (default) = per-l inverses staged in shared memory per
// l tile, 0 = read per column from the l-fastest global copy; TGCM_STAGE_SMEM_MINV
// selects one (for comparisons).
static bool stage_smem_minv() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("TGCM_STAGE_SMEM_MINV");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

static void run_stage(StageArgs& a, const at::Tensor& like, int adjoint) {
  if (like.is_cuda() && a.n == 32 && a.MinvT != nullptr) {
    c10::cuda::CUDAGuard guard(like.device());
    if (stage_smem_minv()) {
      const long long n_lt = (a.L + kStageLT - 1) / kStageLT;
      const long long n_bm = (static_cast<long long>(a.B) * a.M2 + 7) / 8;
      sil3_stage_q4_kernel<32, true><<<static_cast<unsigned>(n_lt * n_bm), 256, 0,
                                       at::cuda::getCurrentCUDAStream()>>>(a, adjoint);
    } else {
      const long long total = static_cast<long long>(a.B) * a.M2 * a.L;
      sil3_stage_q4_kernel<32, false><<<static_cast<unsigned>((total + 63) / 64), 256, 0,
                                        at::cuda::getCurrentCUDAStream()>>>(a, adjoint);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else if (like.is_cuda()) {
    c10::cuda::CUDAGuard guard(like.device());
    dim3 grid((a.L + kStageL - 1) / kStageL, a.B);
    const size_t smem = (2 * a.n * a.n + kStageL * a.n * a.n) * sizeof(float);
    sil3_stage_kernel<<<grid, kStageL * kStageM, smem, at::cuda::getCurrentCUDAStream()>>>(a, adjoint);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    const int n = a.n;
    for (int b = 0; b < a.B; ++b)
      for (int l = 0; l < a.L; ++l) {
        const float* mi = a.Minv + static_cast<long long>(l) * n * n;
        const float* g = a.G;
        const float* h = a.H;
        auto mat = [g, h, mi, n](int kind, int i, int j) -> float {
          return kind == 0 ? g[i * n + j] : (kind == 1 ? h[i * n + j] : mi[i * n + j]);
        };
        for (int m = 0; m < a.M2; ++m) {
          if (adjoint)
            stage_column_adj(a, b, m, l, mat);
          else
            stage_column_fwd(a, b, m, l, mat);
        }
      }
  }
}

static void fill_common(StageArgs& a, const at::Tensor& y0, const std::vector<double>& ce, double cp, double cg,
                        double eta, const at::Tensor& G, const at::Tensor& H, const at::Tensor& Minv,
                        const at::Tensor& lam, const at::Tensor& tref, const at::Tensor& dsig,
                        const c10::optional<at::Tensor>& filt, double clamp_abs, double R, int64_t final_stage,
                        int64_t n) {
  TORCH_CHECK(y0.dim() == 4 && y0.is_contiguous() && y0.scalar_type() == at::kFloat, "packed state must be contiguous fp32");
  TORCH_CHECK(n <= kStageMaxLev && static_cast<int>(ce.size()) <= kStageMaxE, "stage limits exceeded");
  a.nE = static_cast<int>(ce.size());
  for (int j = 0; j < a.nE; ++j) a.ce[j] = static_cast<float>(ce[j]);
  a.cp = static_cast<float>(cp); a.cg = static_cast<float>(cg); a.eta = static_cast<float>(eta);
  a.G = G.data_ptr<float>(); a.H = H.data_ptr<float>(); a.Minv = Minv.data_ptr<float>();
  a.lam = lam.data_ptr<float>(); a.tref = tref.data_ptr<float>(); a.dsig = dsig.data_ptr<float>();
  a.filt = ptr_or_null(filt);
  a.clamp_abs = static_cast<float>(clamp_abs);
  a.R = static_cast<float>(R);
  a.final_stage = static_cast<int>(final_stage);
  a.B = static_cast<int>(y0.size(0)); a.C = static_cast<int>(y0.size(1)); a.n = static_cast<int>(n);
  a.M2 = static_cast<int>(y0.size(2)); a.L = static_cast<int>(y0.size(3));
}

at::Tensor sil3_stage(const at::Tensor& y0, std::vector<at::Tensor> E, const at::Tensor& P,
                      const c10::optional<at::Tensor>& y2, std::vector<double> ce, double cp, double cg, double eta,
                      const at::Tensor& G, const at::Tensor& H, const at::Tensor& Minv, const at::Tensor& lam,
                      const at::Tensor& tref, const at::Tensor& dsig, const c10::optional<at::Tensor>& filt,
                      double clamp_abs, double R, int64_t final_stage, int64_t n,
                      const c10::optional<at::Tensor>& minv_t) {
  StageArgs a;
  memset(&a, 0, sizeof(a));
  fill_common(a, y0, ce, cp, cg, eta, G, H, Minv, lam, tref, dsig, filt, clamp_abs, R, final_stage, n);
  a.MinvT = ptr_or_null(minv_t);
  TORCH_CHECK(E.size() == ce.size(), "one coefficient per explicit tendency");
  auto out = out_empty_like(y0);
  a.y0 = y0.data_ptr<float>();
  for (size_t j = 0; j < E.size(); ++j) {
    TORCH_CHECK(E[j].is_contiguous() && E[j].sizes() == y0.sizes(), "E shape");
    a.E[j] = E[j].data_ptr<float>();
  }
  TORCH_CHECK(P.is_contiguous() && P.sizes() == y0.sizes(), "P shape");
  a.P = P.data_ptr<float>();
  a.y2 = ptr_or_null(y2);
  a.out = out.data_ptr<float>();
  run_stage(a, y0, 0);
  return out;
}

std::vector<at::Tensor> sil3_stage_adjoint(const at::Tensor& gout, const at::Tensor& out, int64_t nE, int64_t has_y2,
                                           std::vector<double> ce, double cp, double cg, double eta,
                                           const at::Tensor& G, const at::Tensor& H, const at::Tensor& Minv,
                                           const at::Tensor& lam, const at::Tensor& tref, const at::Tensor& dsig,
                                           const c10::optional<at::Tensor>& filt, double clamp_abs, double R,
                                           int64_t final_stage, int64_t n, const c10::optional<at::Tensor>& minv_t) {
  StageArgs a;
  memset(&a, 0, sizeof(a));
  fill_common(a, gout, ce, cp, cg, eta, G, H, Minv, lam, tref, dsig, filt, clamp_abs, R, final_stage, n);
  a.MinvT = ptr_or_null(minv_t);
  auto g_y0 = out_empty_like(gout);
  auto g_P = out_empty_like(gout);
  std::vector<at::Tensor> res{g_y0};
  std::vector<at::Tensor> gE;
  for (int64_t j = 0; j < nE; ++j) {
    gE.push_back(out_empty_like(gout));
    a.g_E[j] = gE.back().data_ptr<float>();
  }
  at::Tensor g_y2;
  if (has_y2) {
    g_y2 = out_empty_like(gout);
    a.g_y2 = g_y2.data_ptr<float>();
  }
  a.gin = gout.data_ptr<float>();
  a.out = const_cast<float*>(out.data_ptr<float>());
  a.g_y0 = g_y0.data_ptr<float>();
  a.g_P = g_P.data_ptr<float>();
  run_stage(a, gout, 1);
  for (auto& t : gE) res.push_back(t);
  res.push_back(g_P);
  if (has_y2) res.push_back(g_y2);
  return res;
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("spectral_linear(Tensor x, int L, int C_out, int out_lpad, Tensor row_ptr, Tensor terms, Tensor coef, "
        "Tensor diag, Tensor rec_a, Tensor rec_b, Tensor mats, int nlev, Tensor? row_m=None, Tensor? err=None) -> Tensor");
  m.def("set_bounds_check(bool on) -> ()", &tgcm::set_bounds_check);
  m.def("bounds_check_enabled() -> bool", &tgcm::bounds_check_enabled);
  m.def("sil3_stage(Tensor y0, Tensor[] E, Tensor P, Tensor? y2, float[] ce, float cp, float cg, float eta, "
        "Tensor G, Tensor H, Tensor Minv, Tensor lam, Tensor tref, Tensor dsig, Tensor? filt, float clamp_abs, "
        "float R, int final_stage, int n, Tensor? minv_t=None) -> Tensor");
  m.def("sil3_stage_adjoint(Tensor gout, Tensor out, int nE, int has_y2, float[] ce, float cp, float cg, float eta, "
        "Tensor G, Tensor H, Tensor Minv, Tensor lam, Tensor tref, Tensor dsig, Tensor? filt, float clamp_abs, "
        "float R, int final_stage, int n, Tensor? minv_t=None) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(tgcm, CompositeExplicitAutograd, m) {
  m.impl("spectral_linear", &tgcm::spectral_linear);
  m.impl("sil3_stage", &tgcm::sil3_stage);
  m.impl("sil3_stage_adjoint", &tgcm::sil3_stage_adjoint);
}
