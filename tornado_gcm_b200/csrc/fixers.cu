// Z2 conservation fixer on a packed state, FP64 accumulation (sm_100a + CPU twin).
//
// Packed state y (B, C, M2, L) with channels [ζ (n) | δ (n) | T' (n) | ln ps | …].
// Per sample b:
//   E(y)   = Σ over the first 3n channels of y²      (FP64)
//   D      = E(y_before) − E(y)                      (energy deficit)
//   mass   : ln ps(0,0) ← ln ps_before(0,0)
//   energy : T'_k(0,0) ← sign(T'_k(0,0)) · sqrt(T'_k(0,0)² + s·D)  for every level k,
//            applied only when T'_k(0,0)² + s·D > 0 for all k (else unchanged).
//   s = 1/n (mode 2, the default of the Python classes) spreads the deficit
//   over the n levels, so E(out) = E(y_before) exactly; s = 1 (mode 1) is the
//   reference's formula, which adds the whole deficit at every level and so
//   injects (n - 1)·D of spurious energy per step (the global-mean
//   temperature modes grow until the state blows up in long rollouts with
//   strong dissipation: at 1.4° with 32 levels, after about 21 hours).
// This is the lite fixer of reference neural/fixers.py:228-326 (mass fix of
// :113-143 followed by the energy fix of :146-190); squares are formed in
// FP64, which is at least as accurate as the reference's input-precision
// squares.
//
// Launches: forward = partial sums (grid (kBlocks, B)) + apply (grid
// (kBlocks, B)); backward = one elementwise launch.  The partial sums are
// reduced in a fixed order inside every consumer block, so results are
// deterministic (no atomics).

#include "alloc.h"
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cmath>
#include <vector>

namespace tgcm {
namespace {

constexpr int kFixBlocks = 64;   // partial sums per sample
constexpr int kFixThreads = 256;
constexpr int kFixMaxLev = 256;

struct FixArgs {
  const float* y;
  const float* yb;
  const float* gout;
  const double* part;  // (B, kFixBlocks, 2): Σ y², Σ yb²
  double* part_out;
  float* out;
  float* g_y;
  float* g_yb;
  long long sample;    // C * M2 * L
  long long chan;      // M2 * L
  long long energy_n;  // 3n * M2 * L
  int n, B, fix_mass, fix_energy;
  double dscale;       // share of the deficit added at each level (1/n or 1)
  const double* gd;    // (B) deficit cotangents supplied by the caller, or null
};

// Deficit and admissibility of sample b from the partial sums (fixed order).
__host__ __device__ inline void deficit_of(const FixArgs& a, int b, double* D, int* ok) {
  double e = 0.0, eb = 0.0;
  for (int i = 0; i < kFixBlocks; ++i) {
    e += a.part[(static_cast<long long>(b) * kFixBlocks + i) * 2 + 0];
    eb += a.part[(static_cast<long long>(b) * kFixBlocks + i) * 2 + 1];
  }
  *D = (eb - e) * a.dscale;  // increment of T'_k(0,0)^2 at each level
  int good = 1;
  const float* t00 = a.y + b * a.sample + 2LL * a.n * a.chan;
  for (int k = 0; k < a.n; ++k) {
    const double t = t00[k * a.chan];
    if (!(t * t + *D > 0.0)) good = 0;
  }
  *ok = good;
}

__host__ __device__ inline double sgn(double t) { return t > 0.0 ? 1.0 : (t < 0.0 ? -1.0 : 0.0); }

__host__ __device__ inline float apply_point(const FixArgs& a, int b, long long off, double D, int ok) {
  const float v = a.y[b * a.sample + off];
  const long long c = off / a.chan, r = off - c * a.chan;
  if (r == 0) {
    if (a.fix_mass && c == 3LL * a.n) return a.yb[b * a.sample + off];
    if (a.fix_energy && ok && c >= 2LL * a.n && c < 3LL * a.n) {
      const double t = v;
      return static_cast<float>(sgn(t) * sqrt(t * t + D));
    }
  }
  return v;
}

// Backward of apply for one element; g_D is the per-sample deficit cotangent.
__host__ __device__ inline void adjoint_point(const FixArgs& a, int b, long long off, double D, int ok, double gD) {
  const long long i = b * a.sample + off;
  const long long c = off / a.chan, r = off - c * a.chan;
  double g = a.gout[i];
  double gb = 0.0;
  if (r == 0 && a.fix_mass && c == 3LL * a.n) {
    gb = g;
    g = 0.0;
  } else if (r == 0 && a.fix_energy && ok && c >= 2LL * a.n && c < 3LL * a.n) {
    const double t = a.y[i];
    const double s = sqrt(t * t + D);
    g = s > 0.0 ? g * fabs(t) / s : 0.0;
  }
  if (a.fix_energy && off < a.energy_n) {
    g -= 2.0 * static_cast<double>(a.y[i]) * gD;
    gb += 2.0 * static_cast<double>(a.yb[i]) * gD;
  }
  a.g_y[i] = static_cast<float>(g);
  if (a.g_yb) a.g_yb[i] = static_cast<float>(gb);
}

__host__ __device__ inline double deficit_cotangent(const FixArgs& a, int b, double D, int ok) {
  if (!a.fix_energy || !ok) return 0.0;
  double gD = 0.0;
  for (int k = 0; k < a.n; ++k) {
    const long long i = b * a.sample + (2LL * a.n + k) * a.chan;
    const double t = a.y[i];
    const double s = sqrt(t * t + D);
    if (s > 0.0) gD += static_cast<double>(a.gout[i]) * sgn(t) / (2.0 * s);
  }
  return gD * a.dscale;  // cotangent of the raw deficit E(y_before) - E(y)
}

__device__ inline double block_sum(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  double r = 0.0;
  if (threadIdx.x == 0)
    for (int i = 0; i < kFixThreads / 32; ++i) r += sh[i];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kFixThreads) fix_partial_kernel(FixArgs a) {
  __shared__ double sh[kFixThreads / 32];
  const int b = blockIdx.y;
  double s = 0.0, sb = 0.0;
  const float* y = a.y + b * a.sample;
  const float* yb = a.yb + b * a.sample;
  for (long long i = blockIdx.x * static_cast<long long>(kFixThreads) + threadIdx.x; i < a.energy_n;
       i += static_cast<long long>(kFixBlocks) * kFixThreads) {
    const double v = y[i], vb = yb[i];
    s += v * v;
    sb += vb * vb;
  }
  const double ts = block_sum(s, sh);
  const double tsb = block_sum(sb, sh);
  if (threadIdx.x == 0) {
    a.part_out[(static_cast<long long>(b) * kFixBlocks + blockIdx.x) * 2 + 0] = ts;
    a.part_out[(static_cast<long long>(b) * kFixBlocks + blockIdx.x) * 2 + 1] = tsb;
  }
}

__global__ void __launch_bounds__(kFixThreads) fix_apply_kernel(FixArgs a) {
  __shared__ double sD;
  __shared__ int sOk;
  const int b = blockIdx.y;
  if (threadIdx.x == 0) {
    double D = 0.0;
    int ok = 0;
    if (a.fix_energy) deficit_of(a, b, &D, &ok);
    sD = D;
    sOk = ok;
  }
  __syncthreads();
  const double D = sD;
  const int ok = sOk;
  for (long long off = blockIdx.x * static_cast<long long>(kFixThreads) + threadIdx.x; off < a.sample;
       off += static_cast<long long>(gridDim.x) * kFixThreads)
    a.out[b * a.sample + off] = apply_point(a, b, off, D, ok);
}

__global__ void __launch_bounds__(kFixThreads) fix_adjoint_kernel(FixArgs a) {
  __shared__ double sD, sG;
  __shared__ int sOk;
  const int b = blockIdx.y;
  if (threadIdx.x == 0) {
    double D = 0.0;
    int ok = 0;
    if (a.fix_energy) deficit_of(a, b, &D, &ok);
    sD = D;
    sOk = ok;
    sG = a.gd ? a.gd[b] : deficit_cotangent(a, b, D, ok);
  }
  __syncthreads();
  const double D = sD, gD = sG;
  const int ok = sOk;
  for (long long off = blockIdx.x * static_cast<long long>(kFixThreads) + threadIdx.x; off < a.sample;
       off += static_cast<long long>(gridDim.x) * kFixThreads)
    adjoint_point(a, b, off, D, ok, gD);
}

// fix_energy: 0 off, 1 whole deficit at every level (reference formula), 2 deficit split over the levels.
FixArgs make_args(const at::Tensor& y, const at::Tensor& yb, int64_t n, bool fix_mass, int64_t fix_energy) {
  TORCH_CHECK(y.dim() == 4 && y.is_contiguous() && y.scalar_type() == at::kFloat, "packed state must be contiguous fp32 (B, C, M2, L)");
  TORCH_CHECK(yb.sizes() == y.sizes() && yb.is_contiguous() && yb.scalar_type() == at::kFloat, "before-state shape");
  TORCH_CHECK(n >= 1 && n <= kFixMaxLev && 3 * n + 1 <= y.size(1), "level count does not fit the packed channels");
  FixArgs a;
  memset(&a, 0, sizeof(a));
  a.y = y.data_ptr<float>();
  a.yb = yb.data_ptr<float>();
  a.B = static_cast<int>(y.size(0));
  a.chan = y.size(2) * y.size(3);
  a.sample = y.size(1) * a.chan;
  a.energy_n = 3 * n * a.chan;
  a.n = static_cast<int>(n);
  a.fix_mass = fix_mass ? 1 : 0;
  TORCH_CHECK(fix_energy >= 0 && fix_energy <= 2, "fix_energy: 0 off, 1 reference formula, 2 split over levels");
  a.fix_energy = fix_energy ? 1 : 0;
  a.dscale = fix_energy == 2 ? 1.0 / static_cast<double>(n) : 1.0;
  return a;
}

void partial_sums(FixArgs& a, at::Tensor& part, const at::Tensor& like) {
  a.part_out = part.data_ptr<double>();
  a.part = part.data_ptr<double>();
  if (like.is_cuda()) {
    fix_partial_kernel<<<dim3(kFixBlocks, a.B), kFixThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  // CPU twin: same partition and per-block order of the partial sums is not
  // needed for correctness; one partial per sample, the rest zero.
  for (int b = 0; b < a.B; ++b) {
    double s = 0.0, sb = 0.0;
    for (long long i = 0; i < a.energy_n; ++i) {
      const double v = a.y[b * a.sample + i], vb = a.yb[b * a.sample + i];
      s += v * v;
      sb += vb * vb;
    }
    for (int i = 0; i < kFixBlocks; ++i) {
      a.part_out[(static_cast<long long>(b) * kFixBlocks + i) * 2 + 0] = i == 0 ? s : 0.0;
      a.part_out[(static_cast<long long>(b) * kFixBlocks + i) * 2 + 1] = i == 0 ? sb : 0.0;
    }
  }
}

int apply_blocks(const FixArgs& a) {
  const long long need = (a.sample + kFixThreads - 1) / kFixThreads;
  return static_cast<int>(need < 256 ? need : 256);
}

}  // namespace

namespace {

void check_part(const at::Tensor& part, const FixArgs& a, const at::Tensor& y) {
  TORCH_CHECK(part.scalar_type() == at::kDouble && part.is_contiguous() &&
                  part.numel() == static_cast<int64_t>(a.B) * kFixBlocks * 2 && part.device() == y.device(),
              "partial sums must be a contiguous fp64 (B, 64, 2) tensor on the state's device");
}

}  // namespace

// Partial energy sums alone: (B, 64, 2) fp64 (sum of y^2, sum of y_before^2 per block).
// A caller whose modal rows are spread over several GPUs adds the ranks'
// partial sums (an all-reduce) and passes the total to packed_fix_apply.
at::Tensor packed_fix_partial(const at::Tensor& y, const at::Tensor& yb, int64_t n, bool fix_mass,
                              int64_t fix_energy) {
  c10::OptionalDeviceGuard guard(y.device());
  FixArgs a = make_args(y, yb, n, fix_mass, fix_energy);
  auto part = out_empty({a.B, kFixBlocks, 2}, y.options().dtype(at::kDouble));
  partial_sums(a, part, y);
  return part;
}

// Returns (fixed state, partial sums); the partial sums feed the backward.
// part_in: partial sums computed (and possibly reduced over ranks) by the caller.
std::vector<at::Tensor> packed_fix(const at::Tensor& y, const at::Tensor& yb, int64_t n, bool fix_mass,
                                   int64_t fix_energy, const c10::optional<at::Tensor>& part_in) {
  c10::OptionalDeviceGuard guard(y.device());
  FixArgs a = make_args(y, yb, n, fix_mass, fix_energy);
  at::Tensor part;
  if (part_in.has_value() && part_in->defined()) {
    check_part(*part_in, a, y);
    part = *part_in;
    a.part = part.data_ptr<double>();
  } else {
    part = out_empty({a.B, kFixBlocks, 2}, y.options().dtype(at::kDouble));
    partial_sums(a, part, y);
  }
  auto out = out_empty_like(y);
  a.out = out.data_ptr<float>();
  if (y.is_cuda()) {
    fix_apply_kernel<<<dim3(apply_blocks(a), a.B), kFixThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    for (int b = 0; b < a.B; ++b) {
      double D = 0.0;
      int ok = 0;
      if (a.fix_energy) deficit_of(a, b, &D, &ok);
      for (long long off = 0; off < a.sample; ++off) out.data_ptr<float>()[b * a.sample + off] = apply_point(a, b, off, D, ok);
    }
  }
  return {out, part};
}

// gd (optional, (B) fp64): the deficit cotangents, computed by the caller when
// the (0,0) modes live on another rank; otherwise they come from y's own rows.
std::vector<at::Tensor> packed_fix_adjoint(const at::Tensor& gout, const at::Tensor& y, const at::Tensor& yb,
                                           const at::Tensor& part, int64_t n, bool fix_mass, int64_t fix_energy,
                                           bool need_before, const c10::optional<at::Tensor>& gd) {
  c10::OptionalDeviceGuard guard(y.device());
  FixArgs a = make_args(y, yb, n, fix_mass, fix_energy);
  TORCH_CHECK(gout.sizes() == y.sizes() && gout.is_contiguous() && gout.scalar_type() == at::kFloat, "gradient shape");
  check_part(part, a, y);
  a.part = part.data_ptr<double>();
  if (gd.has_value() && gd->defined()) {
    TORCH_CHECK(gd->scalar_type() == at::kDouble && gd->is_contiguous() && gd->numel() == a.B &&
                    gd->device() == y.device(),
                "gd must be a contiguous fp64 (B) tensor on the state's device");
    a.gd = gd->data_ptr<double>();
  }
  a.gout = gout.data_ptr<float>();
  auto g_y = out_empty_like(y);
  at::Tensor g_yb = need_before ? out_empty_like(y) : at::Tensor();
  a.g_y = g_y.data_ptr<float>();
  a.g_yb = need_before ? g_yb.data_ptr<float>() : nullptr;
  if (y.is_cuda()) {
    fix_adjoint_kernel<<<dim3(apply_blocks(a), a.B), kFixThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    for (int b = 0; b < a.B; ++b) {
      double D = 0.0;
      int ok = 0;
      if (a.fix_energy) deficit_of(a, b, &D, &ok);
      const double gD = a.gd ? a.gd[b] : deficit_cotangent(a, b, D, ok);
      for (long long off = 0; off < a.sample; ++off) adjoint_point(a, b, off, D, ok, gD);
    }
  }
  if (!need_before) return {g_y};
  return {g_y, g_yb};
}

// ── FP64 reductions (one block per row, fixed order: deterministic) ─────────
// sphere_integrate: out[b] = Σ_{i,j} w[j] · z[b, i, j]   (z (B, I, J), w (J))
// sum_squares:      out[b] = Σ_k x[b, k]²                 (x (B, N))
namespace {

constexpr int kRedThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kRedThreads) row_reduce_kernel(const T* __restrict__ x, const double* __restrict__ w,
                                                               long long n, long long inner, double* out) {
  __shared__ double sh[kRedThreads / 32];
  const int b = blockIdx.x;
  const T* row = x + b * n;
  double s = 0.0;
  for (long long i = threadIdx.x; i < n; i += kRedThreads) {
    const double v = static_cast<double>(row[i]);
    s += w ? w[i % inner] * v : v * v;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double r = 0.0;
    for (int i = 0; i < kRedThreads / 32; ++i) r += sh[i];
    out[b] = r;
  }
}

at::Tensor row_reduce(const at::Tensor& x2, const c10::optional<at::Tensor>& w, int64_t inner) {
  TORCH_CHECK(x2.dim() == 2 && x2.is_contiguous(), "row_reduce: contiguous (B, N) input");
  TORCH_CHECK(x2.scalar_type() == at::kFloat || x2.scalar_type() == at::kDouble, "row_reduce: fp32/fp64 input");
  const int64_t B = x2.size(0), N = x2.size(1);
  auto out = out_empty({B}, x2.options().dtype(at::kDouble));
  at::Tensor wd;
  if (w.has_value() && w->defined()) {
    wd = w->to(x2.device(), at::kDouble).contiguous();
    TORCH_CHECK(wd.numel() == inner && N % inner == 0, "row_reduce: weight length must divide the row");
  }
  if (B == 0) return out;
  if (x2.is_cuda()) {
    c10::cuda::CUDAGuard guard(x2.device());
    auto st = at::cuda::getCurrentCUDAStream();
    const double* wp = wd.defined() ? wd.data_ptr<double>() : nullptr;
    if (x2.scalar_type() == at::kFloat)
      row_reduce_kernel<float><<<B, kRedThreads, 0, st>>>(x2.data_ptr<float>(), wp, N, inner, out.data_ptr<double>());
    else
      row_reduce_kernel<double><<<B, kRedThreads, 0, st>>>(x2.data_ptr<double>(), wp, N, inner, out.data_ptr<double>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    auto xd = x2.to(at::kDouble);
    const double* xp = xd.data_ptr<double>();
    const double* wp = wd.defined() ? wd.data_ptr<double>() : nullptr;
    for (int64_t b = 0; b < B; ++b) {
      double s = 0.0;
      for (int64_t i = 0; i < N; ++i) {
        const double v = xp[b * N + i];
        s += wp ? wp[i % inner] * v : v * v;
      }
      out.data_ptr<double>()[b] = s;
    }
  }
  return out;
}

}  // namespace

at::Tensor sphere_integrate(const at::Tensor& z, const at::Tensor& w) {
  TORCH_CHECK(z.dim() >= 2 && w.dim() == 1 && w.size(0) == z.size(-1), "sphere_integrate: z (..., I, J), w (J)");
  auto lead = z.sizes().slice(0, z.dim() - 2).vec();
  auto x2 = z.reshape({-1, z.size(-2) * z.size(-1)}).contiguous();
  return row_reduce(x2, w, z.size(-1)).reshape(lead);
}

at::Tensor sum_squares(const at::Tensor& x, int64_t n_trailing) {
  TORCH_CHECK(n_trailing >= 1 && n_trailing <= x.dim(), "sum_squares: bad trailing dim count");
  auto lead = x.sizes().slice(0, x.dim() - n_trailing).vec();
  int64_t n = 1;
  for (int64_t d = x.dim() - n_trailing; d < x.dim(); ++d) n *= x.size(d);
  auto x2 = x.reshape({-1, n}).contiguous();
  return row_reduce(x2, c10::nullopt, 1).reshape(lead);
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("sphere_integrate(Tensor z, Tensor w) -> Tensor");
  m.def("sum_squares(Tensor x, int n_trailing) -> Tensor");
  m.def("packed_fix(Tensor y, Tensor y_before, int n, bool fix_mass, int fix_energy, Tensor? part=None) -> Tensor[]");
  m.def("packed_fix_partial(Tensor y, Tensor y_before, int n, bool fix_mass, int fix_energy) -> Tensor");
  m.def("packed_fix_adjoint(Tensor gout, Tensor y, Tensor y_before, Tensor part, int n, bool fix_mass, "
        "int fix_energy, bool need_before, Tensor? gd=None) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(tgcm, CompositeExplicitAutograd, m) {
  m.impl("packed_fix", &tgcm::packed_fix);
  m.impl("packed_fix_partial", &tgcm::packed_fix_partial);
  m.impl("packed_fix_adjoint", &tgcm::packed_fix_adjoint);
  m.impl("sphere_integrate", &tgcm::sphere_integrate);
  m.impl("sum_squares", &tgcm::sum_squares);
}
