// tcgen05 GEMM engine for sm_100a.
//
//   C[g][m][n] = epi( alpha * sum_k A[g][m][k] * B[g][n][k] )
//
// * Operands are staged by TMA (3-D tensor maps, 128-byte swizzle, no
//   multicast) into a STAGES-deep shared-memory ring; one elected thread
//   issues tcgen05.mma (kind::tf32 for fp32 data, kind::f16 for BF16) with
//   the fp32 accumulator in TMEM; four epilogue warps read TMEM with
//   tcgen05.ld and apply the fused epilogue.
// * Tile: 128 (M) x BN (N) x BK (K = 128 bytes of operand per stage).
// * A and B may each be K-major or MN-major (compile-time).
// * "Pair" addressing serves the per-wavenumber Legendre GEMMs: the 128
//   A-rows of a tile are 64 slices x {cos, sin} rows of one zonal
//   wavenumber m (group g = m), loaded as one 3-D box (BK, 2, 64).
// * Split-K over gridDim.z accumulates with fp32 atomics.
// * Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
//   issuer, warps 2-5 epilogue (warp % 4 selects the TMEM lane quarter).
// * All mbarrier waits are bounded (common.cuh); on a timeout the kernel
//   records an error code and drains instead of hanging.
#pragma once

#include "common.cuh"

namespace tgcm {

struct GemmParams {
  int M, N, K;       // per-group problem (M = rows of C; in pair mode M = 2*S)
  int groups;        // gridDim.y covers tiles_m * groups
  int tiles_m, tiles_n;
  int k_splits;      // gridDim.z
  int a_pair;        // A rows = (slice, cos/sin) pairs of group g
  int a_group_div;   // plain A: batch coordinate = g / a_group_div
  int b_group_div;   // B: batch coordinate = g / b_group_div
  int k_tri;         // start K at floor(g / BK) * BK (triangular Legendre synthesis)
  // epilogue addressing (element strides)
  void* C;
  long long c_sg, c_sr, c_sc;  // plain
  int c_pair;
  long long c_ps, c_pmr;       // pair: slice stride, zonal-row stride (col stride = c_sc)
  int out_bf16;
  float alpha, beta;
  const float* bias;       // [N] or null
  const float* col_scale;  // [N] or null
  int act;
  __nv_bfloat16* aux;            // pre-activation copy (plain layout of C) or null
  const __nv_bfloat16* grad_pre; // multiply by act'(grad_pre) (plain layout) or null
  int grad_act;
  int* err;
};

template <int FMT>
struct FmtTraits;
template <>
struct FmtTraits<1> {  // BF16, kind::f16
  static constexpr int kElem = 2;
  static constexpr int kBK = 64;
  static constexpr int kUK = 16;
};
template <>
struct FmtTraits<2> {  // fp32 data read as TF32, kind::tf32
  static constexpr int kElem = 4;
  static constexpr int kBK = 32;
  static constexpr int kUK = 8;
};

template <int BN>
struct TmemCols {
  static constexpr uint32_t value = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

template <int FMT, int BN, int STAGES>
struct GemmSmem {
  static constexpr int kA = 128 * 128;        // bytes per A stage
  static constexpr int kB = BN * 128;         // bytes per B stage
  static constexpr int kStage = kA + kB;
  static constexpr int kBars = 1024;          // barrier / bookkeeping area
  static constexpr int kTotal = STAGES * kStage + kBars + 1024;  // + alignment slack
};

__device__ __forceinline__ void store_out(const GemmParams& p, long long off, float v) {
  if (p.out_bf16) {
    __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + off;
    if (p.beta != 0.f) v += p.beta * __bfloat162float(*c);
    *c = __float2bfloat16(v);
  } else {
    float* c = reinterpret_cast<float*>(p.C) + off;
    if (p.k_splits > 1) {
      atomicAdd(c, v);
    } else {
      if (p.beta != 0.f) v += p.beta * (*c);
      *c = v;
    }
  }
}

template <int FMT, int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(192, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const GemmParams p) {
  using T = FmtTraits<FMT>;
  using S = GemmSmem<FMT, BN, STAGES>;
  constexpr int BK = T::kBK;
  constexpr int CH = 128 / T::kElem;  // elements per 128-byte MN chunk
  constexpr uint32_t kTmemCols = TmemCols<BN>::value;
  constexpr uint32_t kIdesc = make_idesc(FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, 128, BN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bar_area = smem + STAGES * S::kStage;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tmem_full_bar = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // tile coordinates
  const int tn = blockIdx.x;
  const int tm = blockIdx.y % p.tiles_m;
  const int g = blockIdx.y / p.tiles_m;
  const int split = blockIdx.z;

  int k_begin = p.k_tri ? (g / BK) * BK : 0;
  int k_total_blocks = (p.K - k_begin + BK - 1) / BK;
  if (k_total_blocks < 0) k_total_blocks = 0;
  const int kb_per_split = (k_total_blocks + p.k_splits - 1) / p.k_splits;
  const int kb0 = split * kb_per_split;
  int kb1 = kb0 + kb_per_split;
  if (kb1 > k_total_blocks) kb1 = k_total_blocks;
  const int num_kb = kb1 > kb0 ? kb1 - kb0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tmem_full_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (num_kb == 0) {
    // nothing to accumulate for this split: leave C untouched
  } else if (warp == 0) {
    if (lane == 0) {
      const int a_batch = p.a_group_div > 0 ? g / p.a_group_div : 0;
      const int b_batch = p.b_group_div > 0 ? g / p.b_group_div : 0;
      const int a_mr = (g == 0) ? 0 : 2 * g - 1;
      int issued = 0;
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* sa = smem + s * S::kStage;
        uint8_t* sb = sa + S::kA;
        const int k0 = k_begin + (kb0 + i) * BK;
        mbar_arrive_expect_tx(&full_bar[s], S::kStage);
        if (!A_MN) {
          if (p.a_pair)
            tma_load_3d(sa, &tmap_a, &full_bar[s], k0, a_mr, tm * 64);
          else
            tma_load_3d(sa, &tmap_a, &full_bar[s], k0, tm * 128, a_batch);
        } else {
#pragma unroll
          for (int q = 0; q < 128 / CH; ++q)
            tma_load_3d(sa + q * BK * 128, &tmap_a, &full_bar[s], tm * 128 + q * CH, k0, a_batch);
        }
        if (!B_MN) {
          tma_load_3d(sb, &tmap_b, &full_bar[s], k0, tn * BN, b_batch);
        } else {
#pragma unroll
          for (int q = 0; q < BN / CH; ++q)
            tma_load_3d(sb + q * BK * 128, &tmap_b, &full_bar[s], tn * BN + q * CH, k0, b_batch);
        }
        ++issued;
      }
      // drain: make sure every TMA this thread issued has landed before exit
      for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i) {
        mbar_wait(&full_bar[i % STAGES], (i / STAGES) & 1, p.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&full_bar[s], ph, p.err, kErrTimeoutFull)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * S::kStage);
        const uint32_t sb = sa + S::kA;
#pragma unroll
        for (int k = 0; k < BK / T::kUK; ++k) {
          uint64_t adesc, bdesc;
          if (!A_MN)
            adesc = make_sw128_desc(sa + k * 32, 16, 1024);
          else
            adesc = make_sw128_desc(sa + k * T::kUK * 128, BK * 128, 1024);
          if (!B_MN)
            bdesc = make_sw128_desc(sb + k * 32, 16, 1024);
          else
            bdesc = make_sw128_desc(sb + k * T::kUK * 128, BK * 128, 1024);
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          if (FMT == 2)
            umma_tf32(tmem_base, adesc, bdesc, kIdesc, acc);
          else
            umma_bf16(tmem_base, adesc, bdesc, kIdesc, acc);
        }
        tc_commit(&empty_bar[s]);
      }
      // signal the epilogue (also on abort, so it does not wait forever)
      tc_commit(tmem_full_bar);
      (void)ok;
    }
  } else {
    // epilogue warps 2..5
    const int q = warp & 3;
    const bool have = mbar_wait(tmem_full_bar, 0, p.err, kErrTimeoutTmemFull);
    tc_fence_after();
    if (have && !*abort_flag) {
      const int r = q * 32 + lane;
      const uint32_t taddr_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      long long row_off = 0;
      bool row_ok;
      if (p.c_pair) {
        const int s_idx = tm * 64 + (r >> 1);
        const int pm = r & 1;
        const int mr = (g == 0) ? 0 : 2 * g - 1 + pm;
        row_ok = (s_idx < p.M / 2) && !(g == 0 && pm == 1);
        row_off = static_cast<long long>(s_idx) * p.c_ps + static_cast<long long>(mr) * p.c_pmr;
      } else {
        const int row = tm * 128 + r;
        row_ok = row < p.M;
        row_off = static_cast<long long>(g) * p.c_sg + static_cast<long long>(row) * p.c_sr;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(taddr_row + c0, v);
        tmem_ld_wait();
        if (!row_ok) continue;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int col = tn * BN + c0 + j;
          if (col >= p.N) break;
          float x = __uint_as_float(v[j]) * p.alpha;
          if (p.col_scale) x *= p.col_scale[col];
          if (p.bias && split == 0) x += p.bias[col];
          const long long off = row_off + static_cast<long long>(col) * p.c_sc;
          if (p.aux) p.aux[off] = __float2bfloat16(x);
          if (p.grad_pre) x *= act_grad(p.grad_act, __bfloat162float(p.grad_pre[off]));
          x = apply_act(p.act, x);
          store_out(p, off, x);
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace tgcm
