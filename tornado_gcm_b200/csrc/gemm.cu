// Host side of the tcgen05 GEMM engine: tensor-map encoding (cached), the
// template dispatch table, and the two users built on it:
//   * spherical-harmonic transforms (TF32): Legendre synthesis/analysis as
//     per-wavenumber grouped GEMMs in "pair" addressing, real DFT synthesis/
//     analysis as batched GEMMs against a resident Fourier basis;
//   * BF16 linear layers: forward with fused bias + activation (+ saved
//     pre-activation), data-gradient with the activation derivative fused,
//     weight-gradient with split-K fp32 accumulation.
#include "alloc.h"
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <unordered_map>

#include "gemm_sm100.cuh"

namespace tgcm {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn get_encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("tgcm: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

struct TmapKey {
  uint64_t ptr;
  int dtype;
  uint64_t d0, d1, d2, s1, s2;
  uint32_t b0, b1, b2;
  int swz;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && dtype == o.dtype && d0 == o.d0 && d1 == o.d1 && d2 == o.d2 && s1 == o.s1 &&
           s2 == o.s2 && b0 == o.b0 && b1 == o.b1 && b2 == o.b2 && swz == o.swz;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    size_t h = std::hash<uint64_t>()(k.ptr);
    auto mix = [&h](uint64_t v) { h ^= std::hash<uint64_t>()(v) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2); };
    mix(k.dtype); mix(k.d0); mix(k.d1); mix(k.d2); mix(k.s1); mix(k.s2); mix(k.b0); mix(k.b1); mix(k.b2); mix(k.swz);
    return h;
  }
};

// dtype: 1 = bf16, 2 = fp32.  dims innermost first; strides in bytes for dims 1, 2.
// swz: 0 = 128-byte swizzle of 16-byte chunks (K-major operands, MN-major BF16),
//      1 = 128-byte swizzle of 32-byte chunks (MN-major TF32 operands).
static CUtensorMap make_tmap(const void* ptr, int dtype, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                             uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2, int swz = 0) {
  static std::mutex mu;
  static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  TmapKey key{reinterpret_cast<uint64_t>(ptr), dtype, d0, d1, d2, s1, s2, b0, b1, b2, swz};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int esize = dtype == 1 ? 2 : 4;
  if (reinterpret_cast<uint64_t>(ptr) % 16 != 0) throw std::runtime_error("tgcm: TMA base address not 16B aligned");
  if (s1 % 16 != 0 || s2 % 16 != 0) throw std::runtime_error("tgcm: TMA strides must be multiples of 16 bytes");
  if (b0 * esize != 128) throw std::runtime_error("tgcm: TMA box inner extent must be 128 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {d0, d1, d2 == 0 ? 1 : d2};
  cuuint64_t strides[2] = {s1, s2 == 0 ? s1 * d1 : s2};
  if (strides[1] % 16 != 0) strides[1] = ((strides[1] + 15) / 16) * 16;
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_fn()(&map, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                               3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swz == 1 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("tgcm: cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, map);
  return map;
}

template <int BN>
struct StagesFor {
  static constexpr int value = BN <= 80 ? 4 : 3;
};

// Optional per-CTA cycle-counter buffer (diagnostics; see GemmParams::prof).
static unsigned long long* g_prof_buf = nullptr;
static int64_t g_prof_ctas = 0;
static int64_t g_prof_target = -1;  // record only this launch index (-1: every launch)
static int64_t g_prof_count = 0;

template <int FMT, int BN, bool A_MN, bool B_MN>
static void launch_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t stream) {
  constexpr int ST = StagesFor<BN>::value;
  using S = GemmSmem<FMT, BN, ST>;
  auto kern = gemm_sm100_kernel<FMT, BN, ST, A_MN, B_MN>;
  static bool attr_set[64] = {false};
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur >= 64 || !attr_set[cur]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    if (cur < 64) attr_set[cur] = true;
  }
  // persistent launch: at most one CTA per SM, each walking tiles with stride gridDim.x
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int n_sm = (dev < 64 && sms[dev] > 0) ? sms[dev] : 148;
  const int tiles = gemm_total_tiles(p);
  if (tiles == 0) return;
  dim3 grid(tiles < n_sm ? tiles : n_sm);
  GemmParams q = p;
  q.prof = nullptr;
  if (g_prof_buf != nullptr && grid.x <= g_prof_ctas) {
    if (g_prof_target < 0 || g_prof_count == g_prof_target) q.prof = g_prof_buf;
    ++g_prof_count;
  }
  kern<<<grid, kGemmThreads, S::kTotal, stream>>>(ta, tb, q);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("tgcm gemm launch: ") + cudaGetErrorString(e));
}

// Gathered-B launch (fused weight all-gather): BF16, K-major A and B, BN in {64, 128}.
template <int BN>
static void launch_gather(const CUtensorMap& ta, const BMapSet& bm, const GemmParams& p, cudaStream_t stream) {
  constexpr int ST = 3;  // leaves room for a resident 64-row B block up to K = 768
  using S = GemmSmem<1, BN, ST>;
  auto kern = gemm_sm100_gather_kernel<1, BN, ST>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    if (dev < 64) attr_set[dev] = true;
  }
  int n_sm = 148;
  cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = gemm_total_tiles(p);
  if (tiles == 0) return;
  GemmParams q = p;
  size_t smem = S::kTotal;
  dim3 grid(tiles < n_sm ? tiles : n_sm);
  // resident B when the whole (BN x K) block fits next to the ring: every CTA keeps one column block
  const int nkb = (p.K + 63) / 64;
  const size_t res_bytes = static_cast<size_t>(nkb) * BN * 128;
  const size_t res_off = (static_cast<size_t>(S::kTotal) + 1023) / 1024 * 1024;
  if (res_off + res_bytes <= 227 * 1024 && p.tiles_n <= n_sm) {
    q.b_res_kb = nkb;
    q.b_res_off = static_cast<int>(res_off - 1024);  // offsets are taken from the 1024-aligned base
    smem = res_off + res_bytes;
    const int per = n_sm / p.tiles_n;
    grid.x = static_cast<unsigned>(per * p.tiles_n);
    if (static_cast<int>(grid.x) > tiles) grid.x = static_cast<unsigned>(tiles);
    grid.x = grid.x / p.tiles_n * p.tiles_n;
    if (grid.x == 0) grid.x = static_cast<unsigned>(p.tiles_n);
  }
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  kern<<<grid, kGemmThreads, smem, stream>>>(ta, bm, q);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("tgcm gather gemm launch: ") + cudaGetErrorString(e));
}

// Runtime dispatch over the instantiated configurations.
static void gemm_dispatch(int fmt, int bn, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmParams& p, cudaStream_t st) {
#define TGCM_CASE(F, B, AM, BM)                                  \
  if (fmt == F && bn == B && a_mn == AM && b_mn == BM) {         \
    launch_cfg<F, B, AM, BM>(ta, tb, p, st);                     \
    return;                                                      \
  }
  TGCM_CASE(2, 16, false, false)
  TGCM_CASE(2, 32, false, false)
  TGCM_CASE(2, 64, false, false)
  TGCM_CASE(2, 128, false, false)
  TGCM_CASE(2, 256, false, false)
  TGCM_CASE(2, 80, false, false)
  TGCM_CASE(2, 144, false, false)
  TGCM_CASE(2, 64, false, true)
  TGCM_CASE(2, 128, false, true)
  TGCM_CASE(2, 192, false, true)
  TGCM_CASE(2, 256, false, true)
  TGCM_CASE(2, 192, false, false)
  TGCM_CASE(1, 64, false, false)
  TGCM_CASE(1, 128, false, false)
  TGCM_CASE(1, 64, false, true)
  TGCM_CASE(1, 128, false, true)
  TGCM_CASE(1, 64, true, true)
  TGCM_CASE(1, 128, true, true)
#undef TGCM_CASE
  throw std::runtime_error("tgcm: no GEMM configuration for fmt=" + std::to_string(fmt) + " bn=" + std::to_string(bn));
}

// Row-major epilogue of the plain GEMMs: 0 = staged through shared memory,
// 1 = direct 16-byte row stores for the data-gradient GEMMs (default), 2 = direct
// stores for every output type.  TGCM_GEMM_EPI selects one (for comparisons).
static int g_epi_mode = -1;

static int epi_direct_mode() {
  if (g_epi_mode < 0) {
    const char* e = std::getenv("TGCM_GEMM_EPI");
    g_epi_mode = (e == nullptr || e[0] < '0' || e[0] > '2') ? 1 : e[0] - '0';
  }
  return g_epi_mode;
}

// Select the row-major epilogue variant for later launches; returns the previous one.
int64_t gemm_set_epilogue(int64_t mode) {
  TORCH_CHECK(mode >= 0 && mode <= 2, "epilogue mode must be 0, 1 or 2");
  const int64_t prev = epi_direct_mode();
  g_epi_mode = static_cast<int>(mode);
  return prev;
}

static GemmParams default_params() {
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.route_slot = -1;
  p.k_splits = 1;
  p.alpha = 1.f;
  p.a_group_div = 1;
  p.b_group_div = 1;
  p.epi_direct = epi_direct_mode();
  return p;
}

static int* err_ptr(const c10::optional<at::Tensor>& err) {
  if (err.has_value() && err->defined()) return err->data_ptr<int>();
  return nullptr;
}

static int pick_bn_j(int64_t j) { return j <= 64 ? 64 : (j <= 128 ? 128 : 256); }

static int sm_count() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return 148;
  if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev] > 0 ? sms[dev] : 148;
}

// Tile width for the one-GEMM Fourier transforms (N = S·J columns): the
// persistent grid runs ceil(tiles / SMs) rounds, so the width that minimises
// rounds x width wastes least of the last round (S·J = 82 688 on 148 SMs:
// 256 -> 2.18 rounds run as 3; 192 -> 2.91 rounds).
static int pick_bn_wide(int64_t n_cols, int64_t tiles_m) {
  const int64_t sms = sm_count();
  int best = 256;
  int64_t best_cost = -1;
  for (int bn : {256, 192, 128}) {
    const int64_t tiles = tiles_m * ((n_cols + bn - 1) / bn);
    const int64_t cost = ((tiles + sms - 1) / sms) * bn;
    if (best_cost < 0 || cost < best_cost) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}
static int pick_bn_l(int64_t l) { return l <= 80 ? 80 : 144; }
static int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ── spherical-harmonic transforms ───────────────────────────────────────────
// Nodal layouts: "lon-major" (S, I, J) = the public (…, lon, lat) layout, and
// "lat-major" (S, J, I) used inside the fused dycore.  The synthesis keeps its
// intermediate m-major, W (M2, S·J): the per-m Legendre GEMM then writes whole
// rows of J values (16-byte stores) and the DFT GEMM reads W as an MN-major
// TF32 operand (32-byte-atom swizzle).  The analysis GEMMs take K-major
// operands, so a lon-major analysis input is transposed first.
//
// x: (S, M2, L) fp32 modal view (last-dim stride 1, row stride 16B-aligned), logical L;
// P: (Mw, J, Lp);  F: (I, M2p).  Returns nodal (S, I, J) or (S, J, I).  ws: >= M2·S·J floats.
at::Tensor sht_synth(const at::Tensor& x, int64_t L, const at::Tensor& P, const at::Tensor& F, const at::Tensor& ws,
                     const c10::optional<at::Tensor>& col_scale, const c10::optional<at::Tensor>& err,
                     bool lat_major) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.dim() == 3, "x must be a (S, M2, L) fp32 CUDA tensor");
  TORCH_CHECK(x.stride(2) == 1 && (x.stride(1) * 4) % 16 == 0 && (x.stride(0) * 4) % 16 == 0,
              "x rows must be contiguous with 16-byte aligned strides");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t S = x.size(0), M2 = x.size(1);
  const int64_t Mw = P.size(0), J = P.size(1), Lp = P.size(2);
  const int64_t I = F.size(0), M2p = F.size(1);
  TORCH_CHECK(M2 == 2 * Mw - 1 && M2p % 4 == 0 && M2p >= M2 && Lp >= L, "basis shape mismatch");
  TORCH_CHECK(ws.numel() >= S * J * M2, "workspace too small");
  auto out = lat_major ? out_empty({S, J, I}, x.options()) : out_empty({S, I, J}, x.options());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int bnj = pick_bn_j(J);
  {
    CUtensorMap ta = make_tmap(x.data_ptr(), 2, L, M2, S, x.stride(1) * 4, x.stride(0) * 4, 32, 2, 64);
    CUtensorMap tb = make_tmap(P.data_ptr(), 2, L, J, Mw, Lp * 4, J * Lp * 4, 32, bnj, 1);
    GemmParams p = default_params();
    p.M = 2 * S; p.N = J; p.K = L; p.groups = Mw;
    p.tiles_m = cdiv(S, 64); p.tiles_n = cdiv(J, bnj);
    p.a_pair = 1; p.k_tri = 1;
    p.C = ws.data_ptr(); p.c_pair = 1; p.c_ps = J; p.c_pmr = S * J; p.c_sc = 1;  // W[mrow][s·J + j]
    p.err = err_ptr(err);
    gemm_dispatch(2, bnj, false, false, ta, tb, p, st);
  }
  const bool one_gemm = lat_major && !(col_scale.has_value() && col_scale->defined());
  if (one_gemm) {
    // lat-major output: out[s, j, i] = Σ_k F[i, k] W[k, (s, j)] is ONE GEMM with
    // N = S·J (MN-major B: the (s, j) columns of W are contiguous) and a linear
    // output map n·I + i.
    CUtensorMap ta = make_tmap(F.data_ptr(), 2, M2, I, 1, M2p * 4, I * M2p * 4, 32, 128, 1);
    CUtensorMap tb = make_tmap(ws.data_ptr(), 2, S * J, M2, 1, S * J * 4, M2 * S * J * 4, 32, 32, 1, 1);
    GemmParams p = default_params();
    p.M = I; p.N = S * J; p.K = M2; p.groups = 1;
    p.tiles_m = cdiv(I, 128);
    const int bnw = pick_bn_wide(S * J, p.tiles_m);
    p.tiles_n = cdiv(S * J, bnw);
    p.C = out.data_ptr(); p.c_sg = 0; p.c_sr = 1; p.c_sc = I;
    p.err = err_ptr(err);
    gemm_dispatch(2, bnw, false, true, ta, tb, p, st);
  } else {
    // one GEMM per slice s: B[j][k] = W[k][s·J + j] (MN-major, batch coordinate s)
    CUtensorMap ta = make_tmap(F.data_ptr(), 2, M2, I, 1, M2p * 4, I * M2p * 4, 32, 128, 1);
    CUtensorMap tb = make_tmap(ws.data_ptr(), 2, J, M2, S, S * J * 4, J * 4, 32, 32, 1, 1);
    GemmParams p = default_params();
    p.M = I; p.N = J; p.K = M2; p.groups = S;
    p.tiles_m = cdiv(I, 128); p.tiles_n = cdiv(J, bnj);
    p.a_group_div = 0; p.b_group_div = 1;
    p.C = out.data_ptr(); p.c_sg = I * J;
    if (lat_major) { p.c_sr = 1; p.c_sc = I; } else { p.c_sr = J; p.c_sc = 1; }
    if (col_scale.has_value() && col_scale->defined()) p.col_scale = col_scale->data_ptr<float>();
    p.err = err_ptr(err);
    gemm_dispatch(2, bnj, false, true, ta, tb, p, st);
  }
  return out;
}

// N: nodal (S, J, I) if lat_major else (S, I, J);  Ft: (M2, I);  Pt: (Mw, L, J);  returns (S, M2, Lo).
// peer_ptrs (optional, int64 CPU): the Legendre step adds its (S, M2, Lo) result
// into every listed fp32 buffer (the ranks' symmetric output buffers, this one
// included) with system-scope reductions instead of writing `out`; the caller
// zeroes those buffers beforehand and synchronises the ranks afterwards.
at::Tensor sht_anal(const at::Tensor& N_in, const at::Tensor& Ft, const at::Tensor& Pt, int64_t Lo,
                    const at::Tensor& ws, const c10::optional<at::Tensor>& col_scale,
                    const c10::optional<at::Tensor>& err, bool lat_major,
                    const c10::optional<at::Tensor>& peer_ptrs) {
  TORCH_CHECK(N_in.is_cuda() && N_in.scalar_type() == at::kFloat && N_in.dim() == 3, "N must be fp32 CUDA (S, ., .)");
  c10::cuda::CUDAGuard guard(N_in.device());
  at::Tensor N = lat_major ? N_in.contiguous() : N_in.transpose(1, 2).contiguous();  // -> (S, J, I)
  const int64_t S = N.size(0), J = N.size(1), I = N.size(2);
  const int64_t M2 = Ft.size(0);
  const int64_t Mw = Pt.size(0), L = Pt.size(1);
  TORCH_CHECK(Ft.size(1) == I && Pt.size(2) == J && J % 4 == 0 && I % 4 == 0, "basis shape mismatch");
  TORCH_CHECK(ws.numel() >= S * M2 * J, "workspace too small");
  TORCH_CHECK(Lo >= L, "output row length too small");
  // Columns L..Lo-1 of a padded row are never written or read (consumers take
  // the [..., :L] view; TMA maps of the modal rows stop at L).  With peer
  // reductions the result lands in the peers' buffers and `out` stays empty.
  const bool to_peers = peer_ptrs.has_value() && peer_ptrs->defined();
  auto out = to_peers ? out_empty({0}, N.options()) : out_empty({S, M2, Lo}, N.options());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int bnj = pick_bn_j(J);
  // 1) real DFT analysis.  Without a column scale it is ONE GEMM over all (s, j):
  //    Z (M2 x S·J) = Ft (M2 x I) . N^T, stored m-major (M2, S, J); with a column
  //    scale (w_j) it is S grouped GEMMs storing (S, M2, J).
  const bool one_gemm = !(col_scale.has_value() && col_scale->defined());
  if (one_gemm) {
    const int64_t tm_a = cdiv(M2, 128);
    const int bnw = pick_bn_wide(S * J, tm_a);
    CUtensorMap ta = make_tmap(Ft.data_ptr(), 2, I, M2, 1, I * 4, M2 * I * 4, 32, 128, 1);
    CUtensorMap tb = make_tmap(N.data_ptr(), 2, I, S * J, 1, I * 4, S * J * I * 4, 32, bnw, 1);
    GemmParams p = default_params();
    p.M = M2; p.N = S * J; p.K = I; p.groups = 1;
    p.tiles_m = tm_a; p.tiles_n = cdiv(S * J, bnw);
    p.C = ws.data_ptr(); p.c_sg = 0; p.c_sr = S * J; p.c_sc = 1;
    p.err = err_ptr(err);
    gemm_dispatch(2, bnw, false, false, ta, tb, p, st);
  } else {
    CUtensorMap ta = make_tmap(Ft.data_ptr(), 2, I, M2, 1, I * 4, M2 * I * 4, 32, 128, 1);
    CUtensorMap tb = make_tmap(N.data_ptr(), 2, I, J, S, I * 4, J * I * 4, 32, bnj, 1);
    GemmParams p = default_params();
    p.M = M2; p.N = J; p.K = I; p.groups = S;
    p.tiles_m = cdiv(M2, 128); p.tiles_n = cdiv(J, bnj);
    p.a_group_div = 0; p.b_group_div = 1;
    p.C = ws.data_ptr(); p.c_sg = M2 * J; p.c_sr = J; p.c_sc = 1;
    if (col_scale.has_value() && col_scale->defined()) p.col_scale = col_scale->data_ptr<float>();
    p.err = err_ptr(err);
    gemm_dispatch(2, bnj, false, false, ta, tb, p, st);
  }
  // 2) Legendre analysis per zonal wavenumber: out rows (slice, cos/sin), cols l
  {
    const int bnl = pick_bn_l(L);
    // A rows (m-row, slice): ws is (M2, S, J) after the one-GEMM DFT, else (S, M2, J)
    CUtensorMap ta = one_gemm ? make_tmap(ws.data_ptr(), 2, J, M2, S, S * J * 4, J * 4, 32, 2, 64)
                              : make_tmap(ws.data_ptr(), 2, J, M2, S, J * 4, M2 * J * 4, 32, 2, 64);
    CUtensorMap tb = make_tmap(Pt.data_ptr(), 2, J, L, Mw, J * 4, L * J * 4, 32, bnl, 1);
    GemmParams p = default_params();
    p.M = 2 * S; p.N = L; p.K = J; p.groups = Mw;
    p.tiles_m = cdiv(S, 64); p.tiles_n = cdiv(L, bnl);
    p.a_pair = 1;
    p.C = out.data_ptr(); p.c_pair = 1; p.c_ps = M2 * Lo; p.c_pmr = Lo; p.c_sc = 1;
    p.err = err_ptr(err);
    if (to_peers) {
      TORCH_CHECK(!peer_ptrs->is_cuda() && peer_ptrs->scalar_type() == at::kLong && peer_ptrs->numel() >= 1 &&
                      peer_ptrs->numel() <= 8,
                  "peer_ptrs must be 1..8 int64 addresses on the CPU");
      p.n_peers = static_cast<int>(peer_ptrs->numel());
      for (int i = 0; i < p.n_peers; ++i) p.peer_C[i] = reinterpret_cast<float*>(peer_ptrs->data_ptr<int64_t>()[i]);
    }
    gemm_dispatch(2, bnl, false, false, ta, tb, p, st);
  }
  return out;
}

// ── transforms sharded over zonal wavenumbers and latitude blocks ──────────
// Modal fields live on the rank that owns their zonal wavenumber (local rows
// [m=0 slot | (cos, sin) pairs of the owned m]); nodal fields are split into W
// latitude blocks of Jr rows.  The grid <-> spectral transpose between the two
// layouts is done by the Legendre GEMMs themselves: their epilogue writes each
// output element straight into the buffer of the rank that needs it (plain
// peer stores for synthesis, system-scope reductions for analysis; no TMA and
// no multicast on peer memory).  The caller synchronises the ranks with a
// peer barrier after the routed GEMM and double-buffers the destinations.
static void check_peer_table(const at::Tensor& ptrs, int64_t world) {
  TORCH_CHECK(!ptrs.is_cuda() && ptrs.scalar_type() == at::kLong && ptrs.numel() == world && world >= 1 && world <= 8,
              "peer pointer table must hold one int64 address per rank (1..8) on the CPU");
  for (int64_t i = 0; i < world; ++i)
    TORCH_CHECK(ptrs.data_ptr<int64_t>()[i] % 16 == 0, "peer buffers must be 16-byte aligned");
}

// Synthesis, Legendre step.  x: local modal (S, M2_loc, Lx) fp32 view;
// P_loc: (G, J, Lp) Legendre table of the local groups (zero slots where
// group_m < 0); group_m: (G) int32 on the device (zonal wavenumber per local
// group).  Writes W_d[row(m)][s*Jr + (j - d*Jr)] on rank d = j / Jr, where W_d
// is the (M2, S*Jr) buffer at w_ptrs[d].
void sht_synth_routed(const at::Tensor& x, int64_t L, const at::Tensor& P_loc, const at::Tensor& group_m,
                      const at::Tensor& w_ptrs, int64_t Jr, int64_t M2_full, const c10::optional<at::Tensor>& err) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.dim() == 3, "x must be a (S, M2, L) fp32 CUDA tensor");
  TORCH_CHECK(x.stride(2) == 1 && (x.stride(1) * 4) % 16 == 0 && (x.stride(0) * 4) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x rows must be contiguous with 16-byte aligned strides");
  TORCH_CHECK(P_loc.is_contiguous() && P_loc.scalar_type() == at::kFloat && P_loc.dim() == 3, "P_loc (G, J, Lp)");
  TORCH_CHECK(group_m.is_cuda() && group_m.scalar_type() == at::kInt && group_m.numel() == P_loc.size(0),
              "group_m must be int32 (G) on the device");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t S = x.size(0), M2l = x.size(1);
  const int64_t G = P_loc.size(0), J = P_loc.size(1), Lp = P_loc.size(2);
  TORCH_CHECK(M2l <= 2 * G - 1 + 1 && Lp >= L && L <= x.size(2), "layout mismatch");
  TORCH_CHECK(Jr > 0 && Jr % 4 == 0 && J % Jr == 0, "latitude blocks must be multiples of 4 rows");
  check_peer_table(w_ptrs, J / Jr);
  // tile width: a divisor of the latitude block where one exists, so that every
  // tile has one destination rank (staged, coalesced peer stores)
  int bnj = pick_bn_j(J);
  for (int cand : {256, 128, 64, 32, 16})
    if (cand <= bnj && Jr % cand == 0) {
      bnj = cand;
      break;
    }
  CUtensorMap ta = make_tmap(x.data_ptr(), 2, L, M2l, S, x.stride(1) * 4, x.stride(0) * 4, 32, 2, 64);
  CUtensorMap tb = make_tmap(P_loc.data_ptr(), 2, L, J, G, Lp * 4, J * Lp * 4, 32, bnj, 1);
  GemmParams p = default_params();
  p.M = 2 * S; p.N = J; p.K = L; p.groups = G;
  p.tiles_m = cdiv(S, 64); p.tiles_n = cdiv(J, bnj);
  p.a_pair = 1; p.k_tri = 1;
  p.c_pair = 1; p.c_ps = Jr; p.c_pmr = S * Jr; p.c_sc = 1;
  p.route_mode = 1; p.route_cols = static_cast<int>(Jr); p.group_map = group_m.data_ptr<int>();
  p.route_rows = static_cast<int>(M2_full);
  p.n_peers = static_cast<int>(J / Jr);
  for (int i = 0; i < p.n_peers; ++i) p.peer_C[i] = reinterpret_cast<float*>(w_ptrs.data_ptr<int64_t>()[i]);
  p.err = err_ptr(err);
  gemm_dispatch(2, bnj, false, false, ta, tb, p, at::cuda::getCurrentCUDAStream());
}

// Synthesis, Fourier step on this rank's block: out (S, Jr, I) lat-major =
// sum_k F[i, k] W[k, s*Jr + j] for the (M2, S*Jr) m-major buffer W (one GEMM).
at::Tensor sht_synth_dft(const at::Tensor& W, int64_t S, int64_t Jr, const at::Tensor& F,
                         const c10::optional<at::Tensor>& err) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kFloat && W.is_contiguous(), "W must be contiguous fp32");
  c10::cuda::CUDAGuard guard(W.device());
  const int64_t I = F.size(0), M2p = F.size(1);
  const int64_t M2 = W.numel() / (S * Jr);
  TORCH_CHECK(W.numel() == M2 * S * Jr && M2 <= M2p && Jr % 4 == 0, "W must be (M2, S*Jr)");
  auto out = out_empty({S, Jr, I}, W.options());
  CUtensorMap ta = make_tmap(F.data_ptr(), 2, M2, I, 1, M2p * 4, I * M2p * 4, 32, 128, 1);
  CUtensorMap tb = make_tmap(W.data_ptr(), 2, S * Jr, M2, 1, S * Jr * 4, M2 * S * Jr * 4, 32, 32, 1, 1);
  GemmParams p = default_params();
  p.M = I; p.N = S * Jr; p.K = M2; p.groups = 1;
  p.tiles_m = cdiv(I, 128);
  const int bnw = pick_bn_wide(S * Jr, p.tiles_m);
  p.tiles_n = cdiv(S * Jr, bnw);
  p.C = out.data_ptr(); p.c_sg = 0; p.c_sr = 1; p.c_sc = I;
  p.err = err_ptr(err);
  gemm_dispatch(2, bnw, false, true, ta, tb, p, at::cuda::getCurrentCUDAStream());
  return out;
}

// Analysis of this rank's latitude block: N (S, Jr, I) lat-major -> Z (M2, S*Jr)
// (one-GEMM DFT into ws) -> per zonal wavenumber m the partial Legendre sums over
// the block's latitudes, added into the (S, M2_loc, Lo) buffer of m's owner
// (out_ptrs[group_dest[m] >> 16], local group group_dest[m] & 0xffff).
// Pt_loc: (Mw, L, Jr) — the (weighted) Legendre table restricted to the block.
void sht_anal_routed(const at::Tensor& N_in, const at::Tensor& Ft, const at::Tensor& Pt_loc, int64_t Lo,
                     int64_t M2_loc, const at::Tensor& ws, const at::Tensor& group_dest, const at::Tensor& out_ptrs,
                     const c10::optional<at::Tensor>& err, int64_t slot) {
  TORCH_CHECK(N_in.is_cuda() && N_in.scalar_type() == at::kFloat && N_in.dim() == 3, "N must be fp32 CUDA (S, Jr, I)");
  c10::cuda::CUDAGuard guard(N_in.device());
  at::Tensor N = N_in.contiguous();
  const int64_t S = N.size(0), Jr = N.size(1), I = N.size(2);
  const int64_t M2 = Ft.size(0);
  const int64_t Mw = Pt_loc.size(0), L = Pt_loc.size(1);
  TORCH_CHECK(Ft.size(1) == I && Pt_loc.size(2) == Jr && Jr % 4 == 0 && I % 4 == 0 && M2 == 2 * Mw - 1,
              "basis shape mismatch");
  TORCH_CHECK(Pt_loc.is_contiguous() && group_dest.is_cuda() && group_dest.scalar_type() == at::kInt &&
                  group_dest.numel() == Mw,
              "Pt_loc contiguous, group_dest int32 (Mw) on the device");
  TORCH_CHECK(ws.numel() >= S * M2 * Jr, "workspace too small");
  TORCH_CHECK(Lo >= L && Lo % 4 == 0 && M2_loc >= 1, "output rows must be padded to a multiple of 4");
  const int64_t world = out_ptrs.numel();
  check_peer_table(out_ptrs, world);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  {
    const int64_t tm_a = cdiv(M2, 128);
    const int bnw = pick_bn_wide(S * Jr, tm_a);
    CUtensorMap ta = make_tmap(Ft.data_ptr(), 2, I, M2, 1, I * 4, M2 * I * 4, 32, 128, 1);
    CUtensorMap tb = make_tmap(N.data_ptr(), 2, I, S * Jr, 1, I * 4, S * Jr * I * 4, 32, bnw, 1);
    GemmParams p = default_params();
    p.M = M2; p.N = S * Jr; p.K = I; p.groups = 1;
    p.tiles_m = tm_a; p.tiles_n = cdiv(S * Jr, bnw);
    p.C = ws.data_ptr(); p.c_sg = 0; p.c_sr = S * Jr; p.c_sc = 1;
    p.err = err_ptr(err);
    gemm_dispatch(2, bnw, false, false, ta, tb, p, st);
  }
  {
    const int bnl = pick_bn_l(L);
    CUtensorMap ta = make_tmap(ws.data_ptr(), 2, Jr, M2, S, S * Jr * 4, Jr * 4, 32, 2, 64);
    CUtensorMap tb = make_tmap(Pt_loc.data_ptr(), 2, Jr, L, Mw, Jr * 4, L * Jr * 4, 32, bnl, 1);
    GemmParams p = default_params();
    p.M = 2 * S; p.N = L; p.K = Jr; p.groups = Mw;
    p.tiles_m = cdiv(S, 64); p.tiles_n = cdiv(L, bnl);
    p.a_pair = 1;
    p.c_pair = 1; p.c_ps = M2_loc * Lo; p.c_pmr = Lo; p.c_sc = 1;
    p.route_mode = 2; p.group_map = group_dest.data_ptr<int>(); p.route_rows = static_cast<int>(M2_loc);
    p.route_slot = slot;  // >= 0: this rank's slot of the owners' buffers (plain stores)
    p.n_peers = static_cast<int>(world);
    for (int i = 0; i < p.n_peers; ++i) p.peer_C[i] = reinterpret_cast<float*>(out_ptrs.data_ptr<int64_t>()[i]);
    p.err = err_ptr(err);
    gemm_dispatch(2, bnl, false, false, ta, tb, p, st);
  }
}

// ── BF16 linear layers ──────────────────────────────────────────────────────
// X: (T, Kp) bf16;  W: (O, Kp) bf16;  bias (O) fp32.  out (T, O) bf16 or fp32.
void linear_fwd(const at::Tensor& X, const at::Tensor& W, const c10::optional<at::Tensor>& bias, int64_t act,
                at::Tensor& out, const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& err) {
  TORCH_CHECK(X.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16, "bf16 operands expected");
  TORCH_CHECK(X.is_contiguous() && W.is_contiguous() && out.is_contiguous(), "contiguous operands expected");
  c10::cuda::CUDAGuard guard(X.device());
  const int64_t T = X.size(0), Kp = X.size(1), O = W.size(0);
  TORCH_CHECK(W.size(1) == Kp && Kp % 8 == 0, "feature dim must be padded to a multiple of 8");
  const int bn = O <= 64 ? 64 : 128;
  CUtensorMap ta = make_tmap(X.data_ptr(), 1, Kp, T, 1, Kp * 2, T * Kp * 2, 64, 128, 1);
  CUtensorMap tb = make_tmap(W.data_ptr(), 1, Kp, O, 1, Kp * 2, O * Kp * 2, 64, bn, 1);
  GemmParams p = default_params();
  p.M = T; p.N = O; p.K = Kp; p.groups = 1;
  p.tiles_m = cdiv(T, 128); p.tiles_n = cdiv(O, bn);
  p.C = out.data_ptr(); p.c_sr = O; p.c_sc = 1; p.c_sg = 0;
  p.out_bf16 = out.scalar_type() == at::kBFloat16 ? 1 : 0;
  if (bias.has_value() && bias->defined()) p.bias = bias->data_ptr<float>();
  p.act = static_cast<int>(act);
  if (aux.has_value() && aux->defined()) p.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
  p.err = err_ptr(err);
  gemm_dispatch(1, bn, false, false, ta, tb, p, at::cuda::getCurrentCUDAStream());
}

// Fused all-gather + linear: out (T, O) = act(X . W^T + bias) where the
// weight W (O, Kp) is row-sharded over the ranks: shard r holds rows
// [r * rows, (r + 1) * rows) in symmetric memory and w_ptrs lists the
// shards' addresses (int64, CPU).  The producer warp reads every B tile
// straight from its owner's shard with plain TMA loads over NVLink, so the
// gathered weight is never materialised.  rows must be a multiple of 16.
void linear_fwd_gathered(const at::Tensor& X, const at::Tensor& w_ptrs, int64_t rows, int64_t O,
                         const c10::optional<at::Tensor>& bias, int64_t act, at::Tensor& out,
                         const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& err) {
  TORCH_CHECK(X.scalar_type() == at::kBFloat16 && X.is_contiguous() && out.is_contiguous(), "bf16 X expected");
  TORCH_CHECK(!w_ptrs.is_cuda() && w_ptrs.scalar_type() == at::kLong && w_ptrs.numel() >= 1 && w_ptrs.numel() <= 8,
              "w_ptrs must hold 1..8 int64 addresses on the CPU");
  TORCH_CHECK(rows > 0 && rows % 16 == 0, "shard rows must be a positive multiple of 16");
  const int64_t nmaps = w_ptrs.numel();
  // shards of `rows` rows each in rank order; trailing ranks may hold no row of W
  TORCH_CHECK(O <= rows * nmaps, "O inconsistent with the shard layout");
  c10::cuda::CUDAGuard guard(X.device());
  const int64_t T = X.size(0), Kp = X.size(1);
  TORCH_CHECK(Kp % 8 == 0, "feature dim must be padded to a multiple of 8");
  TORCH_CHECK(out.size(0) == T && out.size(1) == O, "out shape mismatch");
  const int bn = 64;  // resident B blocks of 64 rows
  CUtensorMap ta = make_tmap(X.data_ptr(), 1, Kp, T, 1, Kp * 2, T * Kp * 2, 64, 128, 1);
  BMapSet bm;
  memset(&bm, 0, sizeof(bm));
  for (int64_t i = 0; i < nmaps; ++i) {
    const void* ptr = reinterpret_cast<const void*>(w_ptrs.data_ptr<int64_t>()[i]);
    bm.m[i] = make_tmap(ptr, 1, Kp, rows, 1, Kp * 2, rows * Kp * 2, 64, 16, 1);
  }
  GemmParams p = default_params();
  p.M = T; p.N = O; p.K = Kp; p.groups = 1;
  p.tiles_m = cdiv(T, 128); p.tiles_n = cdiv(O, bn);
  p.C = out.data_ptr(); p.c_sr = O; p.c_sc = 1; p.c_sg = 0;
  p.out_bf16 = out.scalar_type() == at::kBFloat16 ? 1 : 0;
  if (bias.has_value() && bias->defined()) p.bias = bias->data_ptr<float>();
  p.act = static_cast<int>(act);
  if (aux.has_value() && aux->defined()) p.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
  p.err = err_ptr(err);
  p.n_bmaps = static_cast<int>(nmaps);
  p.b_rows_per_map = static_cast<int>(rows);
  launch_gather<64>(ta, bm, p, at::cuda::getCurrentCUDAStream());
}

// dX (T, Kp) = dY (T, O) . W (O, Kp), optionally times act'(pre) of the layer input.
void linear_dgrad(const at::Tensor& dY, const at::Tensor& W, at::Tensor& dX,
                  const c10::optional<at::Tensor>& pre, int64_t pre_act, const c10::optional<at::Tensor>& err) {
  c10::cuda::CUDAGuard guard(dY.device());
  const int64_t T = dY.size(0), O = dY.size(1), Kp = W.size(1);
  TORCH_CHECK(O % 8 == 0, "output features must be a multiple of 8");
  const int bn = Kp <= 64 ? 64 : 128;
  CUtensorMap ta = make_tmap(dY.data_ptr(), 1, O, T, 1, O * 2, T * O * 2, 64, 128, 1);
  CUtensorMap tb = make_tmap(W.data_ptr(), 1, Kp, O, 1, Kp * 2, O * Kp * 2, 64, 64, 1);
  GemmParams p = default_params();
  p.M = T; p.N = Kp; p.K = O; p.groups = 1;
  p.tiles_m = cdiv(T, 128); p.tiles_n = cdiv(Kp, bn);
  p.C = dX.data_ptr(); p.c_sr = Kp; p.c_sc = 1;
  p.out_bf16 = dX.scalar_type() == at::kBFloat16 ? 1 : 0;
  if (pre.has_value() && pre->defined()) {
    p.grad_pre = reinterpret_cast<const __nv_bfloat16*>(pre->data_ptr());
    p.grad_act = static_cast<int>(pre_act);
  }
  p.err = err_ptr(err);
  gemm_dispatch(1, bn, false, true, ta, tb, p, at::cuda::getCurrentCUDAStream());
}

// dW (O, Kp) fp32 += dY^T (O x T) . X (T x Kp)   [split-K, atomics]
void linear_wgrad(const at::Tensor& dY, const at::Tensor& X, at::Tensor& dW, int64_t splits,
                  const c10::optional<at::Tensor>& err) {
  c10::cuda::CUDAGuard guard(dY.device());
  const int64_t T = dY.size(0), O = dY.size(1), Kp = X.size(1);
  TORCH_CHECK(dW.scalar_type() == at::kFloat && dW.size(0) == O && dW.size(1) == Kp, "dW shape");
  const int bn = Kp <= 64 ? 64 : 128;
  CUtensorMap ta = make_tmap(dY.data_ptr(), 1, O, T, 1, O * 2, T * O * 2, 64, 64, 1);
  CUtensorMap tb = make_tmap(X.data_ptr(), 1, Kp, T, 1, Kp * 2, T * Kp * 2, 64, 64, 1);
  GemmParams p = default_params();
  p.M = O; p.N = Kp; p.K = T; p.groups = 1;
  p.tiles_m = cdiv(O, 128); p.tiles_n = cdiv(Kp, bn);
  const int64_t kblocks = cdiv(T, 64);
  // one wave of tiles: every split adds its partial tile into dW once, so fewer
  // splits mean fewer reductions into the same addresses
  int64_t sp = splits > 0 ? splits : std::max<int64_t>(1, 148 / (p.tiles_m * p.tiles_n));
  sp = std::min<int64_t>(sp, kblocks);
  p.k_splits = static_cast<int>(sp);
  p.beta = 1.f;
  p.C = dW.data_ptr(); p.c_sr = Kp; p.c_sc = 1;
  p.err = err_ptr(err);
  gemm_dispatch(1, bn, true, true, ta, tb, p, at::cuda::getCurrentCUDAStream());
}

// ── batched TF32 GEMM ───────────────────────────────────────────────────────
// C[g] (M x N) = alpha * A[g] (M x K) . B[g] (N x K)^T, fp32 data read as TF32.
// A (G, M, K) and B (G, N, K) may be strided views: last dim contiguous, the
// other two strides multiples of 4 elements, base 16-byte aligned.  C is any
// (G, M, N) fp32 view (the epilogue stores through its strides).
void bgemm_tf32(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, double alpha,
                const c10::optional<at::Tensor>& err) {
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3 && C.dim() == 3, "bgemm_tf32 expects 3-D operands");
  TORCH_CHECK(A.scalar_type() == at::kFloat && B.scalar_type() == at::kFloat && C.scalar_type() == at::kFloat,
              "bgemm_tf32 expects fp32 operands");
  const int64_t G = A.size(0), M = A.size(1), K = A.size(2), N = B.size(1);
  TORCH_CHECK(B.size(0) == G && B.size(2) == K && C.size(0) == G && C.size(1) == M && C.size(2) == N,
              "bgemm_tf32 shape mismatch");
  TORCH_CHECK(A.stride(2) == 1 && B.stride(2) == 1, "bgemm_tf32: K must be the contiguous dim");
  TORCH_CHECK(A.stride(1) % 4 == 0 && A.stride(0) % 4 == 0 && B.stride(1) % 4 == 0 && B.stride(0) % 4 == 0,
              "bgemm_tf32: operand strides must be multiples of 4 elements");
  c10::cuda::CUDAGuard guard(A.device());
  const int bn = N <= 64 ? 64 : (N <= 128 ? 128 : 256);
  CUtensorMap ta = make_tmap(A.data_ptr(), 2, K, M, G, A.stride(1) * 4, A.stride(0) * 4, 32, 128, 1);
  CUtensorMap tb = make_tmap(B.data_ptr(), 2, K, N, G, B.stride(1) * 4, B.stride(0) * 4, 32, bn, 1);
  GemmParams p = default_params();
  p.M = static_cast<int>(M); p.N = static_cast<int>(N); p.K = static_cast<int>(K);
  p.groups = static_cast<int>(G);
  p.tiles_m = static_cast<int>(cdiv(M, 128)); p.tiles_n = static_cast<int>(cdiv(N, bn));
  p.alpha = static_cast<float>(alpha);
  p.C = C.data_ptr(); p.c_sg = C.stride(0); p.c_sr = C.stride(1); p.c_sc = C.stride(2);
  p.err = err_ptr(err);
  gemm_dispatch(2, bn, false, false, ta, tb, p, at::cuda::getCurrentCUDAStream());
}

// Route the GEMM kernels' per-CTA cycle counters into `buf` ((ctas, 8) int64 on
// the device), or stop recording when `buf` is absent.
void gemm_profile_buffer(const c10::optional<at::Tensor>& buf, int64_t launch_index) {
  g_prof_target = launch_index;
  g_prof_count = 0;
  if (buf.has_value() && buf->defined()) {
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong && buf->dim() == 2 && buf->size(1) == 8 &&
                    buf->is_contiguous(),
                "profile buffer must be a contiguous (ctas, 8) int64 CUDA tensor");
    g_prof_buf = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    g_prof_ctas = buf->size(0);
  } else {
    g_prof_buf = nullptr;
    g_prof_ctas = 0;
  }
}

}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("gemm_profile_buffer(Tensor? buf, int launch_index=-1) -> ()");
  m.def("gemm_set_epilogue(int mode) -> int");
  m.def("bgemm_tf32(Tensor A, Tensor B, Tensor(a!) C, float alpha, Tensor? err) -> ()");
  m.def("sht_synth(Tensor x, int L, Tensor P, Tensor F, Tensor ws, Tensor? col_scale, Tensor? err, bool lat_major) -> Tensor");
  m.def("sht_anal(Tensor N, Tensor Ft, Tensor Pt, int Lo, Tensor ws, Tensor? col_scale, Tensor? err, bool lat_major, "
        "Tensor? peer_ptrs=None) -> Tensor");
  m.def("sht_synth_routed(Tensor x, int L, Tensor P_loc, Tensor group_m, Tensor w_ptrs, int Jr, int M2_full, "
        "Tensor? err) -> ()");
  m.def("sht_synth_dft(Tensor W, int S, int Jr, Tensor F, Tensor? err) -> Tensor");
  m.def("sht_anal_routed(Tensor N, Tensor Ft, Tensor Pt_loc, int Lo, int M2_loc, Tensor ws, Tensor group_dest, "
        "Tensor out_ptrs, Tensor? err, int slot=-1) -> ()");
  m.def("linear_fwd(Tensor X, Tensor W, Tensor? bias, int act, Tensor(a!) out, Tensor? aux, Tensor? err) -> ()");
  m.def("linear_fwd_gathered(Tensor X, Tensor w_ptrs, int rows, int O, Tensor? bias, int act, Tensor(a!) out, "
        "Tensor? aux, Tensor? err) -> ()");
  m.def("linear_dgrad(Tensor dY, Tensor W, Tensor(a!) dX, Tensor? pre, int pre_act, Tensor? err) -> ()");
  m.def("linear_wgrad(Tensor dY, Tensor X, Tensor(a!) dW, int splits, Tensor? err) -> ()");
}

TORCH_LIBRARY_IMPL(tgcm, CUDA, m) {
  m.impl("sht_synth", &tgcm::sht_synth);
  m.impl("sht_anal", &tgcm::sht_anal);
  m.impl("sht_synth_routed", &tgcm::sht_synth_routed);
  m.impl("sht_synth_dft", &tgcm::sht_synth_dft);
  m.impl("sht_anal_routed", &tgcm::sht_anal_routed);
  m.impl("linear_fwd", &tgcm::linear_fwd);
  m.impl("linear_fwd_gathered", &tgcm::linear_fwd_gathered);
  m.impl("linear_dgrad", &tgcm::linear_dgrad);
  m.impl("linear_wgrad", &tgcm::linear_wgrad);
  m.impl("bgemm_tf32", &tgcm::bgemm_tf32);
}

TORCH_LIBRARY_IMPL(tgcm, CompositeExplicitAutograd, m) {
  m.impl("gemm_profile_buffer", &tgcm::gemm_profile_buffer);
  m.impl("gemm_set_epilogue", &tgcm::gemm_set_epilogue);
}
