// Dycore kernels for sm_100a (and their CPU twins, same per-column code):
//
//  * column_fwd / column_vjp: the nonlinear nodal explicit tendency of the
//    primitive equations and its reverse-mode derivative, one thread per
//    (sample, lon, lat) column (dycore_column.h).
//  * implicit_apply: the per-wavenumber vertical operators of the IMEX
//    scheme on (δ, T', ln ps) spectral columns — the implicit terms G and
//    the implicit solve (I − ηG)⁻¹ by block elimination with a cached
//    per-l Schur-complement inverse — plus their transposes (adjoints).
//    One thread per (sample, m, l) column; matrices staged in shared memory.
#include "alloc.h"
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <stdexcept>
#include <vector>

#include "dycore_column.h"
#include "dycore_column_warp.cuh"

namespace tgcm {

static ColumnConsts consts_from(const at::Tensor& level_consts, int64_t n, int64_t nt, int64_t hum,
                                int64_t hum_terms, const std::vector<int64_t>& clouds, int64_t vadv, double R,
                                double kappa, double rv, double cpv) {
  TORCH_CHECK(n >= 2 && n <= kMaxLevels, "levels must be in [2, 64]");
  TORCH_CHECK(nt >= 0 && nt <= kMaxTracers, "at most 8 tracers");
  auto lc = level_consts.to(at::kCPU, at::kFloat).contiguous();
  TORCH_CHECK(lc.dim() == 2 && lc.size(0) == 5 && lc.size(1) == n, "level_consts must be (5, n)");
  ColumnConsts c;
  memset(&c, 0, sizeof(c));
  c.n = static_cast<int>(n);
  c.nt = static_cast<int>(nt);
  c.hum = static_cast<int>(hum);
  c.hum_terms = static_cast<int>(hum_terms);
  c.n_clouds = static_cast<int>(clouds.size());
  for (size_t i = 0; i < clouds.size() && i < kMaxTracers; ++i) c.clouds[i] = static_cast<int>(clouds[i]);
  c.vadv = static_cast<int>(vadv);
  c.R = static_cast<float>(R);
  c.kappa = static_cast<float>(kappa);
  c.rv = static_cast<float>(rv);
  c.cpv = static_cast<float>(cpv);
  const float* p = lc.data_ptr<float>();
  for (int k = 0; k < n; ++k) {
    c.dsig[k] = p[0 * n + k];
    c.alpha[k] = p[1 * n + k];
    c.tref[k] = p[2 * n + k];
    c.idc[k] = p[3 * n + k];
    c.cs[k] = p[4 * n + k];
  }
  return c;
}

// Optional fused geopotential matrix: a (n, n) fp32 copy on the data's device;
// the returned tensor keeps it alive for the duration of the call.
static at::Tensor attach_gmat(ColumnConsts& c, const c10::optional<at::Tensor>& gmat, const at::Tensor& like,
                              int64_t n) {
  c.gmat = nullptr;
  if (!gmat.has_value() || !gmat->defined()) return at::Tensor();
  TORCH_CHECK(gmat->dim() == 2 && gmat->size(0) == n && gmat->size(1) == n, "gmat must be (n, n)");
  at::Tensor g = gmat->to(like.device(), at::kFloat).contiguous();
  c.gmat = g.data_ptr<float>();
  return g;
}

// Raise a column kernel's dynamic shared-memory limit once per (kernel, device).
static void set_col_smem(const void* fn, size_t bytes) {
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  for (auto& d : done)
    if (d.first == fn && d.second == dev) return;
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  done.emplace_back(fn, dev);
  TORCH_CHECK(bytes <= 64 * 1024, "column kernel staging exceeds 64 KB");
}

// ── column kernels ──────────────────────────────────────────────────────────
template <int MAXL>
__global__ void column_fwd_kernel(ColumnConsts c, SliceIndex ix, const float* __restrict__ in,
                                  float* __restrict__ out, const float* __restrict__ sec2,
                                  const float* __restrict__ cor, int B, int I, int J, int lat_major) {
  const long long plane = static_cast<long long>(I) * J;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(B) * plane) return;
  const int b = static_cast<int>(idx / plane);
  const long long ij = idx - static_cast<long long>(b) * plane;
  const int j = lat_major ? static_cast<int>(ij / I) : static_cast<int>(ij % J);
  const float* ib = in + static_cast<long long>(b) * ix.n_in * plane + ij;
  float* ob = out + static_cast<long long>(b) * ix.n_out * plane + ij;
  auto rd = [ib, plane](int q) -> float { return __ldg(ib + q * plane); };
  auto wr = [ob, plane](int q, float v) { ob[q * plane] = v; };
  column_forward<MAXL>(c, ix, rd, wr, sec2[j], cor[j]);
}

template <int MAXL, int MAXT>
__global__ void column_vjp_kernel(ColumnConsts c, SliceIndex ix, const float* __restrict__ in,
                                  const float* __restrict__ gout, float* __restrict__ gin,
                                  const float* __restrict__ sec2, const float* __restrict__ cor, int B, int I,
                                  int J, int lat_major) {
  const long long plane = static_cast<long long>(I) * J;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(B) * plane) return;
  const int b = static_cast<int>(idx / plane);
  const long long ij = idx - static_cast<long long>(b) * plane;
  const int j = lat_major ? static_cast<int>(ij / I) : static_cast<int>(ij % J);
  const float* ib = in + static_cast<long long>(b) * ix.n_in * plane + ij;
  const float* gb = gout + static_cast<long long>(b) * ix.n_out * plane + ij;
  float* gib = gin + static_cast<long long>(b) * ix.n_in * plane + ij;
  auto rd = [ib, plane](int q) -> float { return __ldg(ib + q * plane); };
  auto rg = [gb, plane](int q) -> float { return __ldg(gb + q * plane); };
  auto wg = [gib, plane](int q, float v) { gib[q * plane] = v; };
  column_vjp<MAXL, MAXT>(c, ix, rd, rg, wg, sec2[j], cor[j]);
}

static void check_nodal(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() && t.dim() == 3, name,
              " must be a contiguous fp32 (slices, lon, lat) tensor");
}

at::Tensor column_fwd(const at::Tensor& nin, const at::Tensor& sec2, const at::Tensor& cor,
                      const at::Tensor& level_consts, int64_t batch, int64_t n, int64_t nt, int64_t hum,
                      int64_t hum_terms, std::vector<int64_t> clouds, int64_t vadv, double R, double kappa,
                      double rv, double cpv, bool lat_major, const c10::optional<at::Tensor>& gmat) {
  check_nodal(nin, "nin");
  ColumnConsts c = consts_from(level_consts, n, nt, hum, hum_terms, clouds, vadv, R, kappa, rv, cpv);
  at::Tensor gm = attach_gmat(c, gmat, nin, n);
  SliceIndex ix = make_slice_index(c);
  const int64_t I = lat_major ? nin.size(2) : nin.size(1), J = lat_major ? nin.size(1) : nin.size(2);
  TORCH_CHECK(nin.size(0) == batch * ix.n_in, "nin slice count mismatch: expected ", batch * ix.n_in);
  auto out = out_empty({batch * ix.n_out, nin.size(1), nin.size(2)}, nin.options());
  auto s2 = sec2.to(nin.device(), at::kFloat).contiguous();
  auto co = cor.to(nin.device(), at::kFloat).contiguous();
  if (nin.is_cuda()) {
    c10::cuda::CUDAGuard guard(nin.device());
    const long long total = batch * I * J;
    const int threads = 128;
    const unsigned blocks = static_cast<unsigned>((total + threads - 1) / threads);
    auto st = at::cuda::getCurrentCUDAStream();
    if (n <= 32) {
      const unsigned wblocks = static_cast<unsigned>((total + kColWarps - 1) / kColWarps);
      const int h = hum_terms ? 1 : 0;
      const int slots = std::max(col_in_fields(static_cast<int>(nt), h), col_out_fields(static_cast<int>(nt), h));
      const size_t smem = static_cast<size_t>(slots) * kSlotFloats * sizeof(float);
      set_col_smem(reinterpret_cast<const void*>(column_fwd_warp_kernel), smem);
      column_fwd_warp_kernel<<<wblocks, 32 * kColWarps, smem, st>>>(
          c, ix, nin.data_ptr<float>(), out.data_ptr<float>(), s2.data_ptr<float>(), co.data_ptr<float>(),
          static_cast<int>(batch), static_cast<int>(I), static_cast<int>(J), lat_major ? 1 : 0);
    } else if (n <= 32)
      column_fwd_kernel<32><<<blocks, threads, 0, st>>>(c, ix, nin.data_ptr<float>(), out.data_ptr<float>(),
                                                        s2.data_ptr<float>(), co.data_ptr<float>(),
                                                        static_cast<int>(batch), static_cast<int>(I),
                                                        static_cast<int>(J), lat_major ? 1 : 0);
    else
      column_fwd_kernel<kMaxLevels><<<blocks, threads, 0, st>>>(c, ix, nin.data_ptr<float>(), out.data_ptr<float>(),
                                                                s2.data_ptr<float>(), co.data_ptr<float>(),
                                                                static_cast<int>(batch), static_cast<int>(I),
                                                                static_cast<int>(J), lat_major ? 1 : 0);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    const float* in = nin.data_ptr<float>();
    float* o = out.data_ptr<float>();
    const long long plane = I * J;
    for (int64_t b = 0; b < batch; ++b)
      for (long long ij = 0; ij < plane; ++ij) {
        const float* ib = in + b * ix.n_in * plane + ij;
        float* ob = o + b * ix.n_out * plane + ij;
        auto rd = [ib, plane](int q) -> float { return ib[q * plane]; };
        auto wr = [ob, plane](int q, float v) { ob[q * plane] = v; };
        const int j = lat_major ? static_cast<int>(ij / I) : static_cast<int>(ij % J);
        column_forward(c, ix, rd, wr, s2.data_ptr<float>()[j], co.data_ptr<float>()[j]);
      }
  }
  return out;
}

at::Tensor column_vjp_op(const at::Tensor& nin, const at::Tensor& gout, const at::Tensor& sec2,
                         const at::Tensor& cor, const at::Tensor& level_consts, int64_t batch, int64_t n, int64_t nt,
                         int64_t hum, int64_t hum_terms, std::vector<int64_t> clouds, int64_t vadv, double R,
                         double kappa, double rv, double cpv, bool lat_major, const c10::optional<at::Tensor>& gmat) {
  check_nodal(nin, "nin");
  check_nodal(gout, "gout");
  ColumnConsts c = consts_from(level_consts, n, nt, hum, hum_terms, clouds, vadv, R, kappa, rv, cpv);
  at::Tensor gm = attach_gmat(c, gmat, nin, n);
  SliceIndex ix = make_slice_index(c);
  const int64_t I = lat_major ? nin.size(2) : nin.size(1), J = lat_major ? nin.size(1) : nin.size(2);
  TORCH_CHECK(gout.size(0) == batch * ix.n_out, "gout slice count mismatch");
  auto gin = out_empty_like(nin);
  auto s2 = sec2.to(nin.device(), at::kFloat).contiguous();
  auto co = cor.to(nin.device(), at::kFloat).contiguous();
  if (nin.is_cuda()) {
    c10::cuda::CUDAGuard guard(nin.device());
    const long long total = batch * I * J;
    const int threads = 64;
    const unsigned blocks = static_cast<unsigned>((total + threads - 1) / threads);
    auto st = at::cuda::getCurrentCUDAStream();
    const int bi = static_cast<int>(batch), ii = static_cast<int>(I), jj = static_cast<int>(J), lm = lat_major ? 1 : 0;
    if (n <= 32) {
      const unsigned wblocks = static_cast<unsigned>((total + kColWarps - 1) / kColWarps);
      const int h = hum_terms ? 1 : 0;
      const int slots = col_in_fields(static_cast<int>(nt), h) + col_out_fields(static_cast<int>(nt), h);
      const size_t smem = static_cast<size_t>(slots) * kSlotFloats * sizeof(float);
      set_col_smem(reinterpret_cast<const void*>(column_vjp_warp_kernel), smem);
      column_vjp_warp_kernel<<<wblocks, 32 * kColWarps, smem, st>>>(c, ix, nin.data_ptr<float>(), gout.data_ptr<float>(),
                                                                gin.data_ptr<float>(), s2.data_ptr<float>(),
                                                                co.data_ptr<float>(), bi, ii, jj, lm);
    } else if (n <= 32 && nt <= 4)
      column_vjp_kernel<32, 4><<<blocks, threads, 0, st>>>(c, ix, nin.data_ptr<float>(), gout.data_ptr<float>(),
                                                             gin.data_ptr<float>(), s2.data_ptr<float>(),
                                                             co.data_ptr<float>(), bi, ii, jj, lm);
    else
      column_vjp_kernel<kMaxLevels, kMaxTracers><<<blocks, threads, 0, st>>>(
          c, ix, nin.data_ptr<float>(), gout.data_ptr<float>(), gin.data_ptr<float>(), s2.data_ptr<float>(),
          co.data_ptr<float>(), bi, ii, jj, lm);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    const float* in = nin.data_ptr<float>();
    const float* go = gout.data_ptr<float>();
    float* gi = gin.data_ptr<float>();
    const long long plane = I * J;
    for (int64_t b = 0; b < batch; ++b)
      for (long long ij = 0; ij < plane; ++ij) {
        const float* ib = in + b * ix.n_in * plane + ij;
        const float* gb = go + b * ix.n_out * plane + ij;
        float* gib = gi + b * ix.n_in * plane + ij;
        auto rd = [ib, plane](int q) -> float { return ib[q * plane]; };
        auto rg = [gb, plane](int q) -> float { return gb[q * plane]; };
        auto wg = [gib, plane](int q, float v) { gib[q * plane] = v; };
        const int j = lat_major ? static_cast<int>(ij / I) : static_cast<int>(ij % J);
        column_vjp(c, ix, rd, rg, wg, s2.data_ptr<float>()[j], co.data_ptr<float>()[j]);
      }
  }
  return gin;
}

// ── implicit vertical operators ─────────────────────────────────────────────
// Modes: 0 solve (I − ηG)x = rhs; 1 transpose of the solve; 2 implicit terms G x; 3 transpose of G.
// Solve by elimination: r = δ* − ηλ(G T* + R Tr p*); δ = Minv_l r; T = T* − ηHδ; p = p* − ηΔσ·δ.
struct ImplicitArgs {
  const float* d_in;  const float* t_in;  const float* p_in;
  float* d_out;       float* t_out;       float* p_out;
  long long sb_d, sk_d, sb_t, sk_t, sb_p;   // input strides (batch, level); (m, l) plane contiguous
  long long ob_d, ok_d, ob_t, ok_t, ob_p;   // output strides
  const float* G;     // (n, n)
  const float* H;     // (n, n)
  const float* Minv;  // (L, n, n)  (mode 0/1)
  const float* lam;   // (L)
  const float* tref;  // (n)
  const float* dsig;  // (n)
  float R, eta;
  int B, n, M2, L, mode;
};

template <typename Ld>
__host__ __device__ __forceinline__ void implicit_column(const ImplicitArgs& a, int b, int m, int l, Ld mat) {
  const int n = a.n;
  const long long pl = static_cast<long long>(m) * a.L + l;
  float d[kMaxLevels], t[kMaxLevels], r[kMaxLevels];
  for (int k = 0; k < n; ++k) {
    d[k] = a.d_in[b * a.sb_d + k * a.sk_d + pl];
    t[k] = a.t_in[b * a.sb_t + k * a.sk_t + pl];
  }
  float p = a.p_in[b * a.sb_p + pl];
  const float lam = a.lam[l];
  const float el = a.eta * lam;
  float od[kMaxLevels], ot[kMaxLevels], op = 0.f;
  // mat(kind, i, j): kind 0 = G, 1 = H, 2 = Minv_l
  if (a.mode == 0) {
    for (int i = 0; i < n; ++i) {
      float gt = 0.f;
      for (int j = 0; j < n; ++j) gt += mat(0, i, j) * t[j];
      r[i] = d[i] - el * (gt + a.R * a.tref[i] * p);
    }
    for (int i = 0; i < n; ++i) {
      float s = 0.f;
      for (int j = 0; j < n; ++j) s += mat(2, i, j) * r[j];
      od[i] = s;
    }
    float sp = 0.f;
    for (int i = 0; i < n; ++i) {
      float hd = 0.f;
      for (int j = 0; j < n; ++j) hd += mat(1, i, j) * od[j];
      ot[i] = t[i] - a.eta * hd;
      sp += a.dsig[i] * od[i];
    }
    op = p - a.eta * sp;
  } else if (a.mode == 1) {
    // inputs are cotangents (d̄, t̄, p̄) of (δ, T, p); outputs cotangents of (δ*, T*, p*)
    for (int i = 0; i < n; ++i) {
      float htt = 0.f;
      for (int j = 0; j < n; ++j) htt += mat(1, j, i) * t[j];
      r[i] = d[i] - a.eta * htt - a.eta * a.dsig[i] * p;  // total cotangent of δ
    }
    for (int i = 0; i < n; ++i) {
      float s = 0.f;
      for (int j = 0; j < n; ++j) s += mat(2, j, i) * r[j];
      od[i] = s;  // r̄ = Minvᵀ δ̄_total  -> cotangent of δ*
    }
    float tr_dot = 0.f;
    for (int i = 0; i < n; ++i) {
      float gtr = 0.f;
      for (int j = 0; j < n; ++j) gtr += mat(0, j, i) * od[j];
      ot[i] = t[i] - el * gtr;
      tr_dot += a.tref[i] * od[i];
    }
    op = p - el * a.R * tr_dot;
  } else if (a.mode == 2) {
    float sp = 0.f;
    for (int i = 0; i < n; ++i) {
      float gt = 0.f, hd = 0.f;
      for (int j = 0; j < n; ++j) {
        gt += mat(0, i, j) * t[j];
        hd += mat(1, i, j) * d[j];
      }
      od[i] = -lam * (gt + a.R * a.tref[i] * p);
      ot[i] = -hd;
      sp += a.dsig[i] * d[i];
    }
    op = -sp;
  } else {
    // transpose of G: inputs (ā, b̄, c̄) -> δ̄ = −Hᵀ b̄ − Δσ c̄ ; T̄ = −λ Gᵀ ā ; p̄ = −λ R Tr·ā
    float tr_dot = 0.f;
    for (int i = 0; i < n; ++i) {
      float htb = 0.f, gta = 0.f;
      for (int j = 0; j < n; ++j) {
        htb += mat(1, j, i) * t[j];
        gta += mat(0, j, i) * d[j];
      }
      od[i] = -htb - a.dsig[i] * p;
      ot[i] = -lam * gta;
      tr_dot += a.tref[i] * d[i];
    }
    op = -lam * a.R * tr_dot;
  }
  for (int k = 0; k < n; ++k) {
    a.d_out[b * a.ob_d + k * a.ok_d + pl] = od[k];
    a.t_out[b * a.ob_t + k * a.ok_t + pl] = ot[k];
  }
  a.p_out[b * a.ob_p + pl] = op;
}

constexpr int kImplicitL = 4;   // wavenumbers per block
constexpr int kImplicitM = 32;  // zonal rows per block pass

__global__ void implicit_kernel(ImplicitArgs a) {
  extern __shared__ float sm[];
  const int n = a.n;
  float* sG = sm;
  float* sH = sG + n * n;
  float* sMi = sH + n * n;  // kImplicitL * n * n
  const int l0 = blockIdx.x * kImplicitL;
  const int b = blockIdx.y;
  const bool need_minv = a.mode <= 1;
  for (int i = threadIdx.x; i < n * n; i += blockDim.x) {
    sG[i] = a.G[i];
    sH[i] = a.H[i];
  }
  if (need_minv) {
    for (int i = threadIdx.x; i < kImplicitL * n * n; i += blockDim.x) {
      const int ll = l0 + i / (n * n);
      sMi[i] = ll < a.L ? a.Minv[static_cast<long long>(ll) * n * n + i % (n * n)] : 0.f;
    }
  }
  __syncthreads();
  const int tl = threadIdx.x % kImplicitL;
  const int tm = threadIdx.x / kImplicitL;
  const int l = l0 + tl;
  if (l >= a.L) return;
  const float* mi = sMi + tl * n * n;
  auto mat = [sG, sH, mi, n](int kind, int i, int j) -> float {
    return kind == 0 ? sG[i * n + j] : (kind == 1 ? sH[i * n + j] : mi[i * n + j]);
  };
  for (int m = tm; m < a.M2; m += kImplicitM) implicit_column(a, b, m, l, mat);
}

static long long bstride(const at::Tensor& t) { return t.dim() >= 4 ? t.stride(0) : 0; }

std::vector<at::Tensor> implicit_apply(const at::Tensor& d, const at::Tensor& t, const at::Tensor& p,
                                       const at::Tensor& G, const at::Tensor& H, const c10::optional<at::Tensor>& Minv,
                                       const at::Tensor& lam, const at::Tensor& tref, const at::Tensor& dsig,
                                       double R, double eta, int64_t mode) {
  TORCH_CHECK(d.scalar_type() == at::kFloat && t.scalar_type() == at::kFloat && p.scalar_type() == at::kFloat,
              "fp32 spectral fields expected");
  TORCH_CHECK(d.dim() == 4 && t.dim() == 4 && p.dim() == 4, "fields must be (B, levels, 2M-1, L)");
  for (const auto* x : {&d, &t, &p})
    TORCH_CHECK(x->stride(3) == 1 && x->stride(2) == x->size(3), "(m, l) planes must be contiguous");
  const int64_t B = d.size(0), n = d.size(1), M2 = d.size(2), L = d.size(3);
  TORCH_CHECK(n <= kMaxLevels, "too many levels");
  auto od = out_empty({B, n, M2, L}, d.options());
  auto ot = out_empty({B, n, M2, L}, d.options());
  auto opp = out_empty({B, 1, M2, L}, d.options());
  auto dev = d.device();
  auto Gc = G.to(dev, at::kFloat).contiguous(), Hc = H.to(dev, at::kFloat).contiguous();
  auto lc = lam.to(dev, at::kFloat).contiguous(), trc = tref.to(dev, at::kFloat).contiguous();
  auto dsc = dsig.to(dev, at::kFloat).contiguous();
  at::Tensor Mc;
  if (mode <= 1) {
    TORCH_CHECK(Minv.has_value(), "solve modes need the per-l inverse");
    Mc = Minv->to(dev, at::kFloat).contiguous();
  }
  ImplicitArgs a;
  a.d_in = d.data_ptr<float>(); a.t_in = t.data_ptr<float>(); a.p_in = p.data_ptr<float>();
  a.d_out = od.data_ptr<float>(); a.t_out = ot.data_ptr<float>(); a.p_out = opp.data_ptr<float>();
  a.sb_d = d.stride(0); a.sk_d = d.stride(1); a.sb_t = t.stride(0); a.sk_t = t.stride(1); a.sb_p = p.stride(0);
  a.ob_d = od.stride(0); a.ok_d = od.stride(1); a.ob_t = ot.stride(0); a.ok_t = ot.stride(1); a.ob_p = opp.stride(0);
  a.G = Gc.data_ptr<float>(); a.H = Hc.data_ptr<float>(); a.Minv = mode <= 1 ? Mc.data_ptr<float>() : nullptr;
  a.lam = lc.data_ptr<float>(); a.tref = trc.data_ptr<float>(); a.dsig = dsc.data_ptr<float>();
  a.R = static_cast<float>(R); a.eta = static_cast<float>(eta);
  a.B = static_cast<int>(B); a.n = static_cast<int>(n); a.M2 = static_cast<int>(M2); a.L = static_cast<int>(L);
  a.mode = static_cast<int>(mode);
  if (d.is_cuda()) {
    c10::cuda::CUDAGuard guard(dev);
    dim3 grid((L + kImplicitL - 1) / kImplicitL, B);
    const size_t smem = (2 * n * n + kImplicitL * n * n) * sizeof(float);
    implicit_kernel<<<grid, kImplicitL * kImplicitM, smem, at::cuda::getCurrentCUDAStream()>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    const float* g = a.G;
    const float* h = a.H;
    for (int b = 0; b < B; ++b)
      for (int l = 0; l < L; ++l) {
        const float* mi = a.Minv ? a.Minv + static_cast<long long>(l) * n * n : nullptr;
        const int nn = static_cast<int>(n);
        auto mat = [g, h, mi, nn](int kind, int i, int j) -> float {
          return kind == 0 ? g[i * nn + j] : (kind == 1 ? h[i * nn + j] : mi[i * nn + j]);
        };
        for (int m = 0; m < M2; ++m) implicit_column(a, b, m, l, mat);
      }
  }
  return {od, ot, opp};
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("column_fwd(Tensor nin, Tensor sec2, Tensor cor, Tensor level_consts, int batch, int n, int nt, int hum, "
        "int hum_terms, int[] clouds, int vadv, float R, float kappa, float rv, float cpv, bool lat_major=False, "
        "Tensor? gmat=None) -> Tensor");
  m.def("column_vjp(Tensor nin, Tensor gout, Tensor sec2, Tensor cor, Tensor level_consts, int batch, int n, "
        "int nt, int hum, int hum_terms, int[] clouds, int vadv, float R, float kappa, float rv, float cpv, bool lat_major=False, "
        "Tensor? gmat=None) -> Tensor");
  m.def("implicit_apply(Tensor d, Tensor t, Tensor p, Tensor G, Tensor H, Tensor? Minv, Tensor lam, Tensor tref, "
        "Tensor dsig, float R, float eta, int mode) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(tgcm, CompositeExplicitAutograd, m) {
  m.impl("column_fwd", &tgcm::column_fwd);
  m.impl("column_vjp", &tgcm::column_vjp_op);
  m.impl("implicit_apply", &tgcm::implicit_apply);
}
