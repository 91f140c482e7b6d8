// Allocation-free spherical-harmonic synthesis: the C entry point declared in
// sht_noalloc.h.  See that header for who needs it, the size limit and the
// sharing rules of the static intermediate buffer.
//
// The computation is the two-GEMM synthesis of the regular op in gemm.cu:
//   1. Legendre, one group per zonal wavenumber m (pair addressing: the cos
//      and sin rows of 64 slices form one 128-row tile), triangular in l:
//        W[s, j, 2m-1 / 2m] = sum_l x[s, 2m-1 / 2m, l] * P[m, j, l]
//   2. real Fourier, one group per slice:
//        out[s, i, j] = sum_k F[i, k] * W[s, j, k]
// W lives in the file-scope array below instead of a PyTorch buffer.  The
// kernels are the same tcgen05 TF32 GEMM template; they are instantiated here
// with their own pipeline depths so this file's kernels are distinct symbols
// from the ones gemm.cu launches.

#include "sht_noalloc.h"

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "gemm_sm100.cuh"

// The intermediate W of every call, on every device that loads this code.
static __device__ __align__(256) float tgcm_sht_noalloc_scratch[TGCM_SHT_NOALLOC_SCRATCH_FLOATS];

namespace {

constexpr int kMaxDevices = 64;

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_setup_mu;
EncodeFn g_encode = nullptr;
// Device address of the scratch array per device ordinal; null until set up.
float* g_scratch_addr[kMaxDevices] = {};
// Multiprocessor count per device ordinal (persistent grid size).
int g_num_sms[kMaxDevices] = {};

template <int BN>
struct Stages {  // pipeline depths chosen to differ from the regular op's instantiations
  static constexpr int value = BN == 64 ? 3 : 2;
};

template <int BN>
using Kernel = void (*)(const CUtensorMap, const CUtensorMap, const tgcm::GemmParams);

template <int BN>
constexpr Kernel<BN> kernel_for() {
  return tgcm::gemm_sm100_kernel<2, BN, Stages<BN>::value, false, false>;
}

template <int BN>
constexpr int smem_bytes() {
  return tgcm::GemmSmem<2, BN, Stages<BN>::value>::kTotal;
}

int cuda_fail(const char* what, cudaError_t e) {
  fprintf(stderr, "tgcm_sht_synth_noalloc: %s failed: %s\n", what, cudaGetErrorString(e));
  return TGCM_SHT_NOALLOC_ERR_CUDA;
}

// One-time set-up of device `dev` (the current device): the scratch address
// and the dynamic shared-memory limit of the three kernel configurations.
int setup_device(int dev, float** scratch) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_addr[dev] != nullptr) {
    *scratch = g_scratch_addr[dev];
    return TGCM_SHT_NOALLOC_OK;
  }
  if (g_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return cuda_fail("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)", e);
    if (q != cudaDriverEntryPointSuccess || fn == nullptr) {
      fprintf(stderr, "tgcm_sht_synth_noalloc: driver has no cuTensorMapEncodeTiled\n");
      return TGCM_SHT_NOALLOC_ERR_CUDA;
    }
    g_encode = reinterpret_cast<EncodeFn>(fn);
  }
  void* addr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&addr, tgcm_sht_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail("cudaGetSymbolAddress(scratch)", e);
  if (addr == nullptr || reinterpret_cast<uintptr_t>(addr) % 256 != 0) {
    fprintf(stderr, "tgcm_sht_synth_noalloc: scratch array address is not 256-byte aligned\n");
    return TGCM_SHT_NOALLOC_ERR_CUDA;
  }
  if ((e = cudaFuncSetAttribute(kernel_for<64>(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem_bytes<64>())) != cudaSuccess ||
      (e = cudaFuncSetAttribute(kernel_for<128>(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem_bytes<128>())) != cudaSuccess ||
      (e = cudaFuncSetAttribute(kernel_for<256>(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem_bytes<256>())) != cudaSuccess)
    return cuda_fail("cudaFuncSetAttribute(max dynamic shared memory)", e);
  int sms = 0;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return cuda_fail("cudaDeviceGetAttribute(multiprocessor count)", e);
  g_num_sms[dev] = sms > 0 ? sms : 1;
  g_scratch_addr[dev] = static_cast<float*>(addr);
  *scratch = g_scratch_addr[dev];
  return TGCM_SHT_NOALLOC_OK;
}

// fp32 3-D tiled tensor map, 128-byte swizzle; dims innermost first, strides
// in bytes for dims 1 and 2.  Built on the caller's stack, never cached.
bool encode(CUtensorMap* map, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
            uint32_t b0, uint32_t b1, uint32_t b2) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0 || s1 % 16 != 0 || s2 % 16 != 0) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

tgcm::GemmParams base_params(int* err) {
  tgcm::GemmParams p;
  memset(&p, 0, sizeof(p));
  p.k_splits = 1;
  p.alpha = 1.f;
  p.a_group_div = 1;
  p.b_group_div = 1;
  p.err = err;
  return p;
}

// Persistent launch: at most one CTA per SM (the kernels walk their tiles).
template <int BN>
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const tgcm::GemmParams& p, int n_sm,
                   cudaStream_t st) {
  const int tiles = tgcm::gemm_total_tiles(p);
  if (tiles == 0) return cudaSuccess;
  dim3 grid(tiles < n_sm ? tiles : n_sm);
  kernel_for<BN>()<<<grid, tgcm::kGemmThreads, smem_bytes<BN>(), st>>>(ta, tb, p);
  return cudaGetLastError();
}

cudaError_t launch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const tgcm::GemmParams& p, int n_sm,
                      cudaStream_t st) {
  if (bn == 64) return launch<64>(ta, tb, p, n_sm, st);
  if (bn == 128) return launch<128>(ta, tb, p, n_sm, st);
  return launch<256>(ta, tb, p, n_sm, st);
}

long long cdiv(long long a, long long b) { return (a + b - 1) / b; }

bool aligned16(const void* p) { return p != nullptr && reinterpret_cast<uintptr_t>(p) % 16 == 0; }

int reject(const char* why) {
  fprintf(stderr, "tgcm_sht_synth_noalloc: %s\n", why);
  return TGCM_SHT_NOALLOC_ERR_ARGS;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int tgcm_sht_synth_noalloc(
    const float* x, long long S, long long M2, long long L, long long x_row_stride, long long x_slice_stride,
    const float* P, long long Mw, long long J, long long Lp, const float* F, long long I, long long M2p, float* out,
    int lat_major, int* err, cudaStream_t stream) {
  if (!aligned16(x) || !aligned16(P) || !aligned16(F) || !aligned16(out))
    return reject("x, P, F and out must be non-null and 16-byte aligned");
  if (S < 1 || L < 1 || Mw < 1 || J < 1 || I < 1) return reject("all sizes must be positive");
  if (M2 != 2 * Mw - 1) return reject("M2 must equal 2 * Mw - 1");
  // The triangular Legendre GEMM starts group m at K = floor(m / 32) * 32;
  // a group whose start is at or beyond L would write none of its W rows,
  // and the Fourier GEMM would then read stale scratch.
  if (((Mw - 1) / 32) * 32 >= L) return reject("floor((Mw - 1) / 32) * 32 must be below L (use Mw <= L)");
  if (Lp < L || Lp % 4 != 0) return reject("Lp must be >= L and a multiple of 4");
  if (M2p < M2 || M2p % 4 != 0) return reject("M2p must be >= M2 and a multiple of 4");
  if (x_row_stride < L || x_row_stride % 4 != 0 || x_slice_stride % 4 != 0 ||
      x_slice_stride < (M2 - 1) * x_row_stride + L)
    return reject("x strides must be multiples of 4 floats and cover the (M2, L) rows");
  const long long need = S * J * M2p;
  if (need > static_cast<long long>(TGCM_SHT_NOALLOC_SCRATCH_FLOATS)) {
    fprintf(stderr,
            "tgcm_sht_synth_noalloc: S * J * M2p = %lld floats of scratch requested, the static limit is %u "
            "floats (16 MiB); split the slices over several calls\n",
            need, TGCM_SHT_NOALLOC_SCRATCH_FLOATS);
    return TGCM_SHT_NOALLOC_ERR_TOO_LARGE;
  }
  const int bnj = J <= 64 ? 64 : (J <= 128 ? 128 : 256);
  if (cdiv(J, bnj) > 65535 || cdiv(S, 64) * Mw > 65535 || cdiv(I, 128) * S > 65535)
    return reject("launch grid too large for these sizes");

  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return reject("device ordinal out of range");
  float* ws = nullptr;
  int rc = setup_device(dev, &ws);
  if (rc != TGCM_SHT_NOALLOC_OK) return rc;

  CUtensorMap ta1, tb1, ta2, tb2;
  if (!encode(&ta1, x, L, M2, S, x_row_stride * 4, x_slice_stride * 4, 32, 2, 64) ||
      !encode(&tb1, P, L, J, Mw, Lp * 4, J * Lp * 4, 32, bnj, 1) ||
      !encode(&ta2, F, M2, I, 1, M2p * 4, I * M2p * 4, 32, 128, 1) ||
      !encode(&tb2, ws, M2, J, S, M2p * 4, J * M2p * 4, 32, bnj, 1)) {
    fprintf(stderr, "tgcm_sht_synth_noalloc: cuTensorMapEncodeTiled rejected an operand\n");
    return TGCM_SHT_NOALLOC_ERR_ARGS;
  }

  // 1) Legendre: W (pair layout, row stride M2p) from x and P.
  tgcm::GemmParams p1 = base_params(err);
  p1.M = static_cast<int>(2 * S);
  p1.N = static_cast<int>(J);
  p1.K = static_cast<int>(L);
  p1.groups = static_cast<int>(Mw);
  p1.tiles_m = static_cast<int>(cdiv(S, 64));
  p1.tiles_n = static_cast<int>(cdiv(J, bnj));
  p1.a_pair = 1;
  p1.k_tri = 1;
  p1.C = ws;
  p1.c_pair = 1;
  p1.c_ps = J * M2p;
  p1.c_pmr = 1;
  p1.c_sc = M2p;
  const int n_sm = g_num_sms[dev];
  if ((e = launch_bn(bnj, ta1, tb1, p1, n_sm, stream)) != cudaSuccess) return cuda_fail("Legendre GEMM launch", e);

  // 2) Fourier: out from F and W, one group per slice.
  tgcm::GemmParams p2 = base_params(err);
  p2.M = static_cast<int>(I);
  p2.N = static_cast<int>(J);
  p2.K = static_cast<int>(M2);
  p2.groups = static_cast<int>(S);
  p2.tiles_m = static_cast<int>(cdiv(I, 128));
  p2.tiles_n = static_cast<int>(cdiv(J, bnj));
  p2.a_group_div = 0;
  p2.b_group_div = 1;
  p2.C = out;
  p2.c_sg = I * J;
  if (lat_major) {
    p2.c_sr = 1;
    p2.c_sc = I;
  } else {
    p2.c_sr = J;
    p2.c_sc = 1;
  }
  if ((e = launch_bn(bnj, ta2, tb2, p2, n_sm, stream)) != cudaSuccess) return cuda_fail("Fourier GEMM launch", e);
  return TGCM_SHT_NOALLOC_OK;
}
