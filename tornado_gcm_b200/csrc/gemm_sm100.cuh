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
  // Peer reduction (fused cross-GPU sum): when n_peers > 0 every output value
  // is added with a system-scope reduction into the same offset of each
  // peer's fp32 buffer peer_C[i] (this GPU's own buffer included) instead of
  // being stored to C.  Plain red.add over NVLink, no TMA, no multicast.
  int n_peers;
  float* peer_C[8];
  // Gathered B (fused all-gather): when n_bmaps > 0 the B rows are spread over
  // n_bmaps tensor maps of b_rows_per_map rows each (the ranks' weight shards,
  // read in place from peer memory with plain, non-multicast TMA loads); a
  // B tile is fetched as BN/16 boxes of 16 rows, each from the map owning it.
  int n_bmaps;
  int b_rows_per_map;
  // Resident B (gathered mode only): every CTA owns one column block tn
  // (gridDim.x is a multiple of tiles_n) and loads its whole B block
  // (b_res_kb k-blocks) once into shared memory at byte offset b_res_off of
  // the aligned dynamic smem; the ring then carries A only.  Each remote
  // weight row then crosses NVLink once per CTA instead of once per tile.
  int b_res_kb;
  int b_res_off;
  // optional per-CTA cycle counters (diagnostics): [cta][0..7] =
  // producer wait, producer issue, mma wait-empty-acc, mma wait-full, mma issue,
  // epilogue wait, epilogue work, tiles
  unsigned long long* prof;
  // Transforms sharded over zonal wavenumbers (modal side) and latitude blocks
  // (nodal side); pair addressing, output routed to the ranks' buffers
  // peer_C[rank] with plain peer stores / reductions (no TMA, no multicast).
  //  route_mode 1 (synthesis Legendre): local group g is zonal wavenumber
  //    m = group_map[g] (-1: empty slot, nothing stored); output column j goes
  //    to rank j / route_cols at column j % route_cols and row 2m-1+pm (0 for
  //    m = 0) of that rank's m-major buffer; k_tri starts K at floor(m/BK)·BK.
  //  route_mode 2 (analysis Legendre): group g is zonal wavenumber g; it goes
  //    to rank group_map[g] >> 16 as local group group_map[g] & 0xffff (row
  //    2·gl-1+pm, 0 for gl = 0), added with system-scope reductions.
  int route_mode;
  int route_cols;
  int route_rows;    // rows of each destination buffer (entries beyond it: kErrBounds, skipped)
  const int* group_map;
  // route_mode 2 with route_slot >= 0: plain stores into this rank's slot of the
  // owner's buffer (element offset route_slot) instead of reductions; the owner
  // adds the ranks' slots after the barrier.
  long long route_slot;
  // row-major epilogue variant (see epilogue_rowmajor_dispatch)
  int epi_direct;
};

__device__ __forceinline__ void st_global_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

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
  static constexpr int kStaging = 8 * 32 * 144;  // epilogue staging tiles (8 warps x 32 rows x 144 B)
  static constexpr int kBars = 1024;          // barrier / bookkeeping area
  static constexpr int kTotal = STAGES * kStage + kStaging + kBars + 1024;  // + alignment slack
};

__device__ __forceinline__ void red_add_sys(float* addr, float v) {
  asm volatile("red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void red_add_sys_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ void store_out(const GemmParams& p, long long off, float v) {
  if (p.n_peers > 0) {
    for (int i = 0; i < p.n_peers; ++i) red_add_sys(p.peer_C[i] + off, v);
    return;
  }
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

// 2 control warps (TMA producer, MMA issuer) + 8 epilogue warps.
constexpr int kGemmThreads = 320;
constexpr int kEpiWarps = 8;

// Tile t of the launch → (tn, tm, g, split); tn fastest.
struct TileCoord {
  int tn, tm, g, split;
};

__device__ __forceinline__ TileCoord tile_coord(const GemmParams& p, int t) {
  TileCoord c;
  c.tn = t % p.tiles_n;
  int r = t / p.tiles_n;
  const int mg = p.tiles_m * p.groups;
  const int y = r % mg;
  c.split = r / mg;
  c.tm = y % p.tiles_m;
  c.g = y / p.tiles_m;
  return c;
}

template <int BK>
__device__ __forceinline__ int tile_kblocks(const GemmParams& p, int g, int split, int* kb0_out, int* kbegin_out) {
  int k_m = g;
  if (p.k_tri && p.route_mode == 1) {
    k_m = __ldg(p.group_map + g);
    if (k_m < 0) k_m = 0;
  }
  const int k_begin = p.k_tri ? (k_m / BK) * BK : 0;
  int total = (p.K - k_begin + BK - 1) / BK;
  if (total < 0) total = 0;
  const int per = (total + p.k_splits - 1) / p.k_splits;
  const int kb0 = split * per;
  int kb1 = kb0 + per;
  if (kb1 > total) kb1 = total;
  *kb0_out = kb0;
  *kbegin_out = k_begin;
  return kb1 > kb0 ? kb1 - kb0 : 0;
}

__host__ __device__ inline int gemm_total_tiles(const GemmParams& p) {
  return p.tiles_n * p.tiles_m * p.groups * p.k_splits;
}

// ── vectorised row-major epilogue ──────────────────────────────────────────
// One warp handles 32 rows (its TMEM lane quarter) x 32 columns per chunk.
// Lane r holds row r's 32 accumulator values (tcgen05.ld); bias, column
// scale, activation and its derivative are applied in registers; the chunk
// goes through a padded shared-memory tile and leaves (or, for the
// pre-activation operand of dgrad, arrives) as 16-byte vectors, so every
// global access of the warp is a run of whole 16-byte sectors.
constexpr int kStageRowBf16 = 80;   // 32 bf16 + 16 B pad (conflict-free v4 accesses)
constexpr int kStageRowF32 = 144;   // 32 fp32 + 16 B pad

// Copy a 32 x 32 bf16 chunk between the staging tile and global memory.
// dir = 0: staging → global, dir = 1: global → staging.  Rows ≥ nrows and
// columns ≥ ncols are skipped; partial 8-column vectors fall back to scalars.
__device__ __forceinline__ void chunk_copy_bf16(uint8_t* stage, __nv_bfloat16* g, long long ld, int nrows, int ncols,
                                                int lane, int dir) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = lane + 32 * i;
    const int row = v >> 2, seg = v & 3;
    if (row >= nrows) continue;
    uint8_t* sp = stage + row * kStageRowBf16 + seg * 16;
    __nv_bfloat16* gp = g + row * ld + seg * 8;
    if (seg * 8 + 8 <= ncols) {
      if (dir == 0)
        *reinterpret_cast<uint4*>(gp) = *reinterpret_cast<const uint4*>(sp);
      else
        *reinterpret_cast<uint4*>(sp) = __ldg(reinterpret_cast<const uint4*>(gp));
    } else {
      __nv_bfloat16* se = reinterpret_cast<__nv_bfloat16*>(sp);
      for (int e = 0; e < 8 && seg * 8 + e < ncols; ++e) {
        if (dir == 0)
          gp[e] = se[e];
        else
          se[e] = gp[e];
      }
    }
  }
}

__device__ __forceinline__ void chunk_store_f32(const uint8_t* stage, float* g, long long ld, int nrows, int ncols,
                                                int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int v = lane + 32 * i;
    const int row = v >> 3, seg = v & 7;
    if (row >= nrows) continue;
    const uint8_t* sp = stage + row * kStageRowF32 + seg * 16;
    float* gp = g + row * ld + seg * 4;
    if (seg * 4 + 4 <= ncols) {
      *reinterpret_cast<float4*>(gp) = *reinterpret_cast<const float4*>(sp);
    } else {
      const float* se = reinterpret_cast<const float*>(sp);
      for (int e = 0; e < 4 && seg * 4 + e < ncols; ++e) gp[e] = se[e];
    }
  }
}

__device__ __forceinline__ void red_add_gpu_v4(float* addr, float4 v) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// Split-K partial sums of a 32 x 32 fp32 chunk added into global memory with
// 16-byte reductions (eight lanes per row), from the staging tile.
__device__ __forceinline__ void chunk_red_f32(const uint8_t* stage, float* g, long long ld, int nrows, int ncols,
                                              int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int v = lane + 32 * i;
    const int row = v >> 3, seg = v & 7;
    if (row >= nrows) continue;
    const uint8_t* sp = stage + row * kStageRowF32 + seg * 16;
    float* gp = g + row * ld + seg * 4;
    if (seg * 4 + 4 <= ncols) {
      red_add_gpu_v4(gp, *reinterpret_cast<const float4*>(sp));
    } else {
      const float* se = reinterpret_cast<const float*>(sp);
      for (int e = 0; e < 4 && seg * 4 + e < ncols; ++e) atomicAdd(gp + e, se[e]);
    }
  }
}

// Epilogue of one 32-row x BN tile slice for split-K fp32 row-major C with
// 16-byte aligned rows: alpha-scaled partial sums added with vector reductions
// (the scalar atomics of the generic path made the weight-gradient GEMM bound
// by the L2 atomic units: 16 384 atomics per tile, 32 partial tiles per output).
template <int BN>
__device__ __noinline__ void epilogue_splitk_red(const GemmParams& p, uint32_t taddr_row, uint8_t* stage, int tm,
                                                    int tn, int g, int q, int half, int lane) {
  // parameters in registers (see epilogue_pair_rows)
  const int N = p.N;
  const float alpha = p.alpha;
  const long long c_sr = p.c_sr;
  const int row0 = tm * 128 + q * 32;
  const int nrows = p.M - row0 < 32 ? p.M - row0 : 32;
  float* __restrict__ Cb = reinterpret_cast<float*>(p.C) + static_cast<long long>(g) * p.c_sg +
                           static_cast<long long>(row0) * c_sr;
  uint8_t* my = stage + lane * kStageRowF32;
#pragma unroll 1
  for (int c0 = half * 32; c0 < BN; c0 += 64) {
    const int ncolc = (BN - c0) >= 32 ? 32 : (BN - c0);
    const int col0 = tn * BN + c0;
    int ncols = N - col0;
    if (ncols > ncolc) ncols = ncolc;
#pragma unroll 1
    for (int h = 0; h < ncolc; h += 16) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(taddr_row + c0 + h, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(my + 4 * (h + j)) =
            make_float4(__uint_as_float(v[j]) * alpha, __uint_as_float(v[j + 1]) * alpha,
                        __uint_as_float(v[j + 2]) * alpha, __uint_as_float(v[j + 3]) * alpha);
    }
    if (ncols <= 0 || nrows <= 0) continue;
    __syncwarp();
    chunk_red_f32(stage, Cb + col0, c_sr, nrows, ncols, lane);
    __syncwarp();
  }
}

// act(x) / act'(pre) on a 32-value chunk; the switch is warp-uniform and sits
// outside the element loops, so one epilogue instance serves every activation
// (six inlined instances of the whole epilogue made the kernel spill).
__device__ __forceinline__ void act_chunk(int act, float (&x)[32]) {
  switch (act) {
#define TGCM_ACT_CASE(A)                                    \
  case A:                                                  \
    _Pragma("unroll") for (int j = 0; j < 32; ++j) x[j] = act_fast<A>(x[j]); \
    break;
    TGCM_ACT_CASE(kActRelu)
    TGCM_ACT_CASE(kActGelu)
    TGCM_ACT_CASE(kActGeluTanh)
    TGCM_ACT_CASE(kActSilu)
    TGCM_ACT_CASE(kActTanh)
#undef TGCM_ACT_CASE
    default: break;
  }
}

// x[j] *= act'(pre[j]) with the bf16 pre-activations of the chunk at `pre`.
__device__ __forceinline__ void act_grad_chunk(int act, float (&x)[32], const uint8_t* pre) {
  switch (act) {
#define TGCM_ACTG_CASE(A)                                                                        \
  case A:                                                                                        \
    _Pragma("unroll") for (int j = 0; j < 32; j += 2) {                                          \
      const float2 pr = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(pre + 2 * j)); \
      x[j] *= act_grad_fast<A>(pr.x);                                                           \
      x[j + 1] *= act_grad_fast<A>(pr.y);                                                       \
    }                                                                                            \
    break;
    TGCM_ACTG_CASE(kActRelu)
    TGCM_ACTG_CASE(kActGelu)
    TGCM_ACTG_CASE(kActGeluTanh)
    TGCM_ACTG_CASE(kActSilu)
    TGCM_ACTG_CASE(kActTanh)
#undef TGCM_ACTG_CASE
    default: break;
  }
}

// Epilogue of one 32-row x BN tile slice for row-major C with 16-byte aligned
// rows.  ACT is the forward activation (or, with grad_pre, the activation
// whose derivative multiplies the result).
template <int BN>
__device__ __forceinline__ void epilogue_rowmajor_vec(const GemmParams& p, int ACT, uint32_t taddr_row,
                                                      uint8_t* stage, int tm, int tn, int g, int q, int half,
                                                      int lane) {
  const int row0 = tm * 128 + q * 32;
  const int nrows = p.M - row0 < 32 ? p.M - row0 : 32;
#pragma unroll 1
  for (int c0 = half * 32; c0 < BN; c0 += 64) {
    const int ncolc = (BN - c0) >= 32 ? 32 : (BN - c0);
    const int col0 = tn * BN + c0;
    int ncols = p.N - col0;
    if (ncols > ncolc) ncols = ncolc;
    uint32_t v0[16], v1[16];
    tmem_ld_32x32b_x16(taddr_row + c0, v0);
    if (ncolc == 32) tmem_ld_32x32b_x16(taddr_row + c0 + 16, v1);
    tmem_ld_wait();
    if (ncols <= 0 || nrows <= 0) continue;
    const long long base = static_cast<long long>(g) * p.c_sg + static_cast<long long>(row0) * p.c_sr + col0;
    float x[32];
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = __uint_as_float(v0[j]) * p.alpha;
#pragma unroll
    for (int j = 0; j < 16; ++j) x[16 + j] = (ncolc == 32) ? __uint_as_float(v1[j]) * p.alpha : 0.f;
    if (p.col_scale) {
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] *= (j < ncols) ? __ldg(p.col_scale + col0 + j) : 0.f;
    }
    if (p.bias) {
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] += (j < ncols) ? __ldg(p.bias + col0 + j) : 0.f;
    }
    uint8_t* my = stage + lane * kStageRowBf16;
    if (p.aux) {  // pre-activation copy (bf16)
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        *reinterpret_cast<__nv_bfloat162*>(my + 2 * j) = __floats2bfloat162_rn(x[j], x[j + 1]);
      __syncwarp();
      chunk_copy_bf16(stage, p.aux + base, p.c_sr, nrows, ncols, lane, 0);
      __syncwarp();
    }
    if (p.grad_pre) {  // x *= act'(pre)
      chunk_copy_bf16(stage, const_cast<__nv_bfloat16*>(p.grad_pre) + base, p.c_sr, nrows, ncols, lane, 1);
      __syncwarp();
      act_grad_chunk(ACT, x, my);
      __syncwarp();
    } else {
      act_chunk(ACT, x);
    }
    if (p.out_bf16) {
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        *reinterpret_cast<__nv_bfloat162*>(my + 2 * j) = __floats2bfloat162_rn(x[j], x[j + 1]);
      __syncwarp();
      chunk_copy_bf16(stage, reinterpret_cast<__nv_bfloat16*>(p.C) + base, p.c_sr, nrows, ncols, lane, 0);
    } else {
      uint8_t* myf = stage + lane * kStageRowF32;
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(myf + 4 * j) = make_float4(x[j], x[j + 1], x[j + 2], x[j + 3]);
      __syncwarp();
      chunk_store_f32(stage, reinterpret_cast<float*>(p.C) + base, p.c_sr, nrows, ncols, lane);
    }
    __syncwarp();
  }
}

// Routed pair epilogue of the sharded transforms (route_mode 1 / 2, see
// GemmParams).  One lane per output row r of the tile (slice tm*64 + r/2,
// cos/sin row r%2); 16 accumulator columns per TMEM load, moved as 4-wide
// vectors (the routed column blocks and the destination rows are multiples of
// 4 floats, checked by the host).
template <int BN>
__device__ __noinline__ void epilogue_routed(const GemmParams& p, uint32_t taddr_row, int tm, int tn, int g, int half,
                                             int r) {
  const int S = p.M / 2, N = p.N, mode = p.route_mode, rc = p.route_cols;
  const float alpha = p.alpha;
  const long long c_ps = p.c_ps, c_pmr = p.c_pmr;
  const int s_idx = tm * 64 + (r >> 1);
  const int pm = r & 1;
  const int gm = __ldg(p.group_map + g);
  int dst = 0, row = 0;
  bool ok = s_idx < S;
  if (mode == 1) {
    ok = ok && gm >= 0 && !(gm == 0 && pm == 1) && !(g == 0 && pm == 1);
    row = gm == 0 ? 0 : 2 * gm - 1 + pm;
  } else {
    dst = gm >> 16;
    const int gl = gm & 0xffff;
    ok = ok && !(g == 0 && pm == 1) && !(gl == 0 && pm == 1);
    row = gl == 0 ? 0 : 2 * gl - 1 + pm;
  }
  if (ok && (row >= p.route_rows || dst < 0 || dst >= p.n_peers)) {  // a corrupt routing table
    record_error(p.err, kErrBounds);
    ok = false;
  }
  const long long row_off = static_cast<long long>(s_idx) * c_ps + static_cast<long long>(row) * c_pmr;
#pragma unroll 1
  for (int c0 = half * 16; c0 < BN; c0 += 32) {
    uint32_t v[16];
    tmem_ld_32x32b_x16(taddr_row + c0, v);
    tmem_ld_wait();
    if (!ok) continue;
    const int colb = tn * BN + c0;
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const int col = colb + j;
      if (col >= N) break;
      const float a0 = __uint_as_float(v[j]) * alpha, a1 = __uint_as_float(v[j + 1]) * alpha;
      const float a2 = __uint_as_float(v[j + 2]) * alpha, a3 = __uint_as_float(v[j + 3]) * alpha;
      if (mode == 1) {
        const int d = col / rc;
        float* out = p.peer_C[d] + row_off + (col - d * rc);
        if (col + 4 <= N) {
          st_global_v4(out, a0, a1, a2, a3);
        } else {
          const float t[4] = {a0, a1, a2, a3};
          for (int e = 0; col + e < N; ++e) out[e] = t[e];
        }
      } else {
        float* out = p.peer_C[dst] + row_off + col;
        if (col + 4 <= N) {
          red_add_sys_v4(out, a0, a1, a2, a3);
        } else {
          const float t[4] = {a0, a1, a2, a3};
          for (int e = 0; col + e < N; ++e) red_add_sys(out + e, t[e]);
        }
      }
    }
  }
}

// Epilogue of a pair-addressed tile (per-wavenumber Legendre GEMMs) whose
// output rows are contiguous (c_sc == 1): tile row r = 2·s + {cos, sin} of
// slice tm·64 + s goes to C + s·c_ps + mrow·c_pmr.  Plain fp32 stores scaled
// by alpha.  The 32 x 32 chunk is staged in shared memory; with 16-byte
// aligned rows eight lanes cover one row with 16-byte stores, otherwise the
// 32 lanes write 32 consecutive values of one row per instruction.
//
// The routed (sharded-transform) tiles use the same path with a per-tile
// destination: Cdst = the owning rank's buffer, g the wavenumber index of the
// destination rows, col_shift subtracted from the column index, and `reduce`
// turning the 16-byte stores into system-scope 16-byte reductions.
template <int BN>
__device__ __noinline__ void epilogue_pair_rows(const GemmParams& p, uint32_t taddr_row, uint8_t* stage, int tm,
                                                   int tn, int g, int q, int half, int lane, float* Cdst = nullptr,
                                                   int col_shift = 0, int reduce = 0) {
  // Parameters are read once into registers: `p` is reached through a generic
  // pointer here, so every global store below would otherwise force the
  // compiler to load the fields again.
  const int S = p.M / 2, N = p.N;
  const long long c_ps = p.c_ps, c_pmr = p.c_pmr;
  const float alpha = p.alpha;
  float* __restrict__ C = (Cdst != nullptr ? Cdst : reinterpret_cast<float*>(p.C)) - col_shift;
  const bool vec = (reinterpret_cast<uintptr_t>(C) % 16 == 0) && (c_ps % 4 == 0) && (c_pmr % 4 == 0);
  auto row_off = [&](int r, bool* ok) -> long long {
    const int s_idx = tm * 64 + (r >> 1);
    const int pm = r & 1;
    const int mr = (g == 0) ? 0 : 2 * g - 1 + pm;
    *ok = (s_idx < S) && !(g == 0 && pm == 1);
    return static_cast<long long>(s_idx) * c_ps + static_cast<long long>(mr) * c_pmr;
  };
#pragma unroll 1
  for (int c0 = half * 32; c0 < BN; c0 += 64) {
    const int ncolc = (BN - c0) >= 32 ? 32 : (BN - c0);
    const int col0 = tn * BN + c0;
    int ncols = N - col0;
    if (ncols > ncolc) ncols = ncolc;
    uint8_t* my = stage + lane * kStageRowF32;
    // 16 columns at a time: load, scale, stage (keeps 16 accumulator registers live)
#pragma unroll 1
    for (int h = 0; h < ncolc; h += 16) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(taddr_row + c0 + h, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(my + 4 * (h + j)) =
            make_float4(__uint_as_float(v[j]) * alpha, __uint_as_float(v[j + 1]) * alpha,
                        __uint_as_float(v[j + 2]) * alpha, __uint_as_float(v[j + 3]) * alpha);
    }
    if (ncols <= 0) continue;
    __syncwarp();
    if (vec) {
      const int seg = lane & 7;
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int rr = (lane + 32 * i) >> 3;
        bool ok;
        const long long off = row_off(q * 32 + rr, &ok);
        if (!ok || seg * 4 >= ncols) continue;
        const uint8_t* sp = stage + rr * kStageRowF32 + seg * 16;
        float* gp = C + off + col0 + seg * 4;
        if (seg * 4 + 4 <= ncols) {
          const float4 v4 = *reinterpret_cast<const float4*>(sp);
          if (reduce)
            red_add_sys_v4(gp, v4.x, v4.y, v4.z, v4.w);
          else
            *reinterpret_cast<float4*>(gp) = v4;
        } else {
          const float* se = reinterpret_cast<const float*>(sp);
          for (int e = 0; seg * 4 + e < ncols; ++e) {
            if (reduce)
              red_add_sys(gp + e, se[e]);
            else
              gp[e] = se[e];
          }
        }
      }
    } else {
      const float* sf = reinterpret_cast<const float*>(stage);
#pragma unroll 4
      for (int rr = 0; rr < 32; ++rr) {
        bool ok;
        const long long off = row_off(q * 32 + rr, &ok);
        if (ok && lane < ncols) {
          if (reduce)
            red_add_sys(C + off + col0 + lane, sf[rr * (kStageRowF32 / 4) + lane]);
          else
            C[off + col0 + lane] = sf[rr * (kStageRowF32 / 4) + lane];
        }
      }
    }
    __syncwarp();
  }
}

__device__ __forceinline__ uint32_t u4_word(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ void u4_set(uint4& v, int i, uint32_t w) {
  if (i == 0) v.x = w; else if (i == 1) v.y = w; else if (i == 2) v.z = w; else v.w = w;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// x[j] *= act'(pre[j]) with the chunk's 32 bf16 pre-activations held in registers
// (word w of pre4 carries columns 2w (low half) and 2w + 1 (high half)).
__device__ __forceinline__ void act_grad_regs(int act, float (&x)[32], const uint4 (&pre4)[4]) {
  switch (act) {
#define TGCM_ACTR_CASE(A)                                                         \
  case A:                                                                         \
    _Pragma("unroll") for (int w = 0; w < 16; ++w) {                              \
      const uint32_t u = u4_word(pre4[w >> 2], w & 3);                            \
      x[2 * w] *= act_grad_fast<A>(__uint_as_float(u << 16));                     \
      x[2 * w + 1] *= act_grad_fast<A>(__uint_as_float(u & 0xffff0000u));         \
    }                                                                             \
    break;
    TGCM_ACTR_CASE(kActRelu)
    TGCM_ACTR_CASE(kActGelu)
    TGCM_ACTR_CASE(kActGeluTanh)
    TGCM_ACTR_CASE(kActSilu)
    TGCM_ACTR_CASE(kActTanh)
#undef TGCM_ACTR_CASE
    default: break;
  }
}

// Row-major epilogue without a staging tile.  Lane r of the warp owns row r of
// its 32-row slice: the pre-activations of a chunk (dgrad) and the bias (one
// value per lane, broadcast by shuffles) are requested before the accumulator
// is read, so their latency overlaps tcgen05.ld, and the lane's 32 results
// leave as 16-byte vectors along its own row (four per bf16 chunk, eight per
// fp32 chunk).  No shared memory and no warp barriers sit on the path; the
// staged epilogue above trades those for fully covered 128-byte lines.
template <int BN>
__device__ __noinline__ void epilogue_rowmajor_direct(const GemmParams& p, int ACT, uint32_t taddr_row, int tm, int tn,
                                                      int g, int q, int half, int lane) {
  const int row = tm * 128 + q * 32 + lane;
  const bool row_ok = row < p.M;
  const long long rbase = static_cast<long long>(g) * p.c_sg + static_cast<long long>(row) * p.c_sr;
  const float alpha = p.alpha;
  const float* bias = p.bias;
  const __nv_bfloat16* gpre = p.grad_pre;
  __nv_bfloat16* aux = p.aux;
  const int out_bf16 = p.out_bf16;
  const int N = p.N;
#pragma unroll 1
  for (int c0 = half * 32; c0 < BN; c0 += 64) {
    const int ncolc = (BN - c0) >= 32 ? 32 : (BN - c0);
    const int col0 = tn * BN + c0;
    int ncols = N - col0;
    if (ncols > ncolc) ncols = ncolc;
    const bool full = ncols == 32;
    uint4 pre4[4];
    if (gpre != nullptr && row_ok && full) {
      const uint4* src = reinterpret_cast<const uint4*>(gpre + rbase + col0);
#pragma unroll
      for (int i = 0; i < 4; ++i) pre4[i] = __ldg(src + i);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) pre4[i] = make_uint4(0u, 0u, 0u, 0u);
      if (gpre != nullptr && row_ok) {  // ragged chunk: scalar loads of the valid columns
        const __nv_bfloat16* src = gpre + rbase + col0;
#pragma unroll
        for (int w = 0; w < 16; ++w) {
          const uint32_t lo = (2 * w < ncols) ? static_cast<uint32_t>(__bfloat16_as_ushort(src[2 * w])) : 0u;
          const uint32_t hi = (2 * w + 1 < ncols) ? static_cast<uint32_t>(__bfloat16_as_ushort(src[2 * w + 1])) : 0u;
          u4_set(pre4[w >> 2], w & 3, lo | (hi << 16));
        }
      }
    }
    const float bl = (bias != nullptr && lane < ncols) ? __ldg(bias + col0 + lane) : 0.f;
    uint32_t v0[16], v1[16];
    tmem_ld_32x32b_x16(taddr_row + c0, v0);
    if (ncolc == 32) tmem_ld_32x32b_x16(taddr_row + c0 + 16, v1);
    tmem_ld_wait();
    float x[32];
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = __uint_as_float(v0[j]) * alpha;
#pragma unroll
    for (int j = 0; j < 16; ++j) x[16 + j] = (ncolc == 32) ? __uint_as_float(v1[j]) * alpha : 0.f;
    if (ncols <= 0) continue;
    if (bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] += __shfl_sync(0xffffffffu, bl, j);
    }
    if (aux != nullptr && row_ok) {
      __nv_bfloat16* ap = aux + rbase + col0;
      if (full) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<uint4*>(ap)[i] =
              make_uint4(pack_bf16x2(x[8 * i], x[8 * i + 1]), pack_bf16x2(x[8 * i + 2], x[8 * i + 3]),
                         pack_bf16x2(x[8 * i + 4], x[8 * i + 5]), pack_bf16x2(x[8 * i + 6], x[8 * i + 7]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) ap[j] = __float2bfloat16(x[j]);
      }
    }
    if (gpre != nullptr)
      act_grad_regs(ACT, x, pre4);
    else
      act_chunk(ACT, x);
    if (row_ok && out_bf16) {
      __nv_bfloat16* cp = reinterpret_cast<__nv_bfloat16*>(p.C) + rbase + col0;
      if (full) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<uint4*>(cp)[i] =
              make_uint4(pack_bf16x2(x[8 * i], x[8 * i + 1]), pack_bf16x2(x[8 * i + 2], x[8 * i + 3]),
                         pack_bf16x2(x[8 * i + 4], x[8 * i + 5]), pack_bf16x2(x[8 * i + 6], x[8 * i + 7]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) cp[j] = __float2bfloat16(x[j]);
      }
    } else if (row_ok) {
      float* cp = reinterpret_cast<float*>(p.C) + rbase + col0;
      if (full) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          reinterpret_cast<float4*>(cp)[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) cp[j] = x[j];
      }
    }
    __syncwarp();  // reconverge before the next chunk's tcgen05.ld
  }
}

template <int FMT, int BN>
__device__ __forceinline__ void epilogue_rowmajor_dispatch(const GemmParams& p, int act, uint32_t taddr_row,
                                                           uint8_t* stage, int tm, int tn, int g, int q, int half,
                                                           int lane) {
  // epi_direct: 1 = direct stores where the pre-activation prefetch pays (data
  // gradients; measured at T = 32768, 384 x 384: dgrad 0.069 -> 0.055 ms, while
  // the forward with its two outputs stayed at 0.055 ms staged, 0.056 direct),
  // 2 = direct stores for every output type
  // (BF16 GEMMs with 128-wide tiles only: the TF32 transforms and the 64-wide tiles keep
  // the staged path and their register budget)
  if (FMT == 1 && BN >= 128 && !p.col_scale && (p.epi_direct >= 2 || (p.epi_direct == 1 && p.grad_pre != nullptr)))
    epilogue_rowmajor_direct<BN>(p, act, taddr_row, tm, tn, g, q, half, lane);
  else
    epilogue_rowmajor_vec<BN>(p, act, taddr_row, stage, tm, tn, g, q, half, lane);
}

// Persistent kernel: each CTA walks tiles t = blockIdx.x, +gridDim.x, ….
//   warp 0     TMA producer; runs ahead across tiles through the STAGES ring
//   warp 1     TMEM owner + MMA issuer; accumulates tile i into TMEM buffer i % 2
//   warps 2-9  epilogue; drains buffer i % 2 while the MMA fills the other one
//              (warp % 4 selects the TMEM lane quarter, (warp - 2) / 4 the
//              half of the column chunks it handles)
// Barriers: full/empty per ring stage (phase from a CTA-wide k-block
// counter), tmem_full/tmem_empty per accumulator buffer (phase from the
// CTA's count of non-empty tiles).
struct BMapSet {
  CUtensorMap m[8];
};

template <int FMT, int BN, int STAGES, bool A_MN, bool B_MN>
__device__ __forceinline__ void gemm_sm100_body(const CUtensorMap& tmap_a, const CUtensorMap* tmaps_b,
                                                const GemmParams& p) {
  const CUtensorMap& tmap_b = tmaps_b[0];
  using T = FmtTraits<FMT>;
  using S = GemmSmem<FMT, BN, STAGES>;
  constexpr int BK = T::kBK;
  constexpr int CH = 128 / T::kElem;  // elements per 128-byte MN chunk
  constexpr uint32_t kAccCols = TmemCols<BN>::value;
  constexpr uint32_t kTmemCols = 2 * kAccCols;
  constexpr uint32_t kIdesc = make_idesc(FMT, A_MN ? 1 : 0, B_MN ? 1 : 0, 128, BN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* staging = reinterpret_cast<float*>(smem + STAGES * S::kStage);
  uint8_t* bar_area = smem + STAGES * S::kStage + S::kStaging;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tmem_full_bar = empty_bar + STAGES;   // [2]
  uint64_t* tmem_empty_bar = tmem_full_bar + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* bres_bar = reinterpret_cast<uint64_t*>(bar_area + 512);  // resident-B arrival
  uint8_t* bres = smem + p.b_res_off;
  const bool b_resident = p.b_res_kb > 0;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles = gemm_total_tiles(p);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full_bar[b], 1);
      mbar_init(&tmem_empty_bar[b], kEpiWarps * 32);
    }
    *abort_flag = 0;
    mbar_init(bres_bar, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      int kb_global = 0;
      unsigned long long t_wait = 0, t_issue = 0;
      if (b_resident) {  // this CTA's B block, once: BN/16 boxes of 16 rows per k-block
        const int tn = blockIdx.x % p.tiles_n;
        mbar_arrive_expect_tx(bres_bar, static_cast<uint32_t>(p.b_res_kb) * BN * 128);
        for (int kb = 0; kb < p.b_res_kb; ++kb)
          for (int q = 0; q < BN / 16; ++q) {
            const int row = tn * BN + q * 16;
            int owner = row / p.b_rows_per_map;
            if (owner >= p.n_bmaps) owner = p.n_bmaps - 1;
            tma_load_3d(bres + (kb * BN + q * 16) * 128, &tmaps_b[owner], bres_bar, kb * BK,
                        row - owner * p.b_rows_per_map, 0);
          }
      }
      for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
        const TileCoord tc = tile_coord(p, t);
        int kb0, k_begin;
        const int num_kb = tile_kblocks<BK>(p, tc.g, tc.split, &kb0, &k_begin);
        const int a_batch = p.a_group_div > 0 ? tc.g / p.a_group_div : 0;
        const int b_batch = p.b_group_div > 0 ? tc.g / p.b_group_div : 0;
        const int a_mr = (tc.g == 0) ? 0 : 2 * tc.g - 1;
        for (int i = 0; i < num_kb; ++i, ++kb_global) {
          const int s = kb_global % STAGES;
          const uint32_t ph = (kb_global / STAGES) & 1;
          const unsigned long long c0 = p.prof ? clock64() : 0ull;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) {
            *abort_flag = 1;
            break;
          }
          if (p.prof) t_wait += clock64() - c0;
          if (*abort_flag) break;
          uint8_t* sa = smem + s * S::kStage;
          uint8_t* sb = sa + S::kA;
          const int k0 = k_begin + (kb0 + i) * BK;
          mbar_arrive_expect_tx(&full_bar[s], b_resident ? S::kA : S::kStage);
          if (!A_MN) {
            if (p.a_pair)
              tma_load_3d(sa, &tmap_a, &full_bar[s], k0, a_mr, tc.tm * 64);
            else
              tma_load_3d(sa, &tmap_a, &full_bar[s], k0, tc.tm * 128, a_batch);
          } else {
#pragma unroll
            for (int q = 0; q < 128 / CH; ++q)
              tma_load_3d(sa + q * BK * 128, &tmap_a, &full_bar[s], tc.tm * 128 + q * CH, k0, a_batch);
          }
          if (b_resident) {
            // B is resident
          } else if (p.n_bmaps > 0) {
#pragma unroll
            for (int q = 0; q < BN / 16; ++q) {
              const int row = tc.tn * BN + q * 16;
              int owner = row / p.b_rows_per_map;
              if (owner >= p.n_bmaps) owner = p.n_bmaps - 1;  // tail rows: out of bounds, zero fill
              tma_load_3d(sb + q * 16 * 128, &tmaps_b[owner], &full_bar[s], k0, row - owner * p.b_rows_per_map,
                          b_batch);
            }
          } else if (!B_MN) {
            tma_load_3d(sb, &tmap_b, &full_bar[s], k0, tc.tn * BN, b_batch);
          } else {
#pragma unroll
            for (int q = 0; q < BN / CH; ++q)
              tma_load_3d(sb + q * BK * 128, &tmap_b, &full_bar[s], tc.tn * BN + q * CH, k0, b_batch);
          }
        }
      }
      // drain: every load this thread issued has landed before the CTA exits
      for (int i = (kb_global > STAGES ? kb_global - STAGES : 0); i < kb_global; ++i)
        mbar_wait(&full_bar[i % STAGES], (i / STAGES) & 1, p.err, kErrTimeoutDrain);
      if (b_resident) mbar_wait(bres_bar, 0, p.err, kErrTimeoutDrain);
      if (p.prof) {
        p.prof[blockIdx.x * 8 + 0] = t_wait;
        p.prof[blockIdx.x * 8 + 1] = t_issue;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int kb_global = 0, tile_i = 0;
      unsigned long long t_acc = 0, t_full = 0;
      if (b_resident && !mbar_wait(bres_bar, 0, p.err, kErrTimeoutFull)) *abort_flag = 1;
      for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
        const TileCoord tc = tile_coord(p, t);
        int kb0, k_begin;
        const int num_kb = tile_kblocks<BK>(p, tc.g, tc.split, &kb0, &k_begin);
        if (num_kb == 0) continue;
        const int acc = tile_i & 1;
        const uint32_t use = static_cast<uint32_t>(tile_i >> 1);
        unsigned long long c0 = p.prof ? clock64() : 0ull;
        if (!mbar_wait(&tmem_empty_bar[acc], (use & 1) ^ 1, p.err, kErrTimeoutEmpty)) {
          *abort_flag = 1;
          break;
        }
        if (p.prof) t_acc += clock64() - c0;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc) * kAccCols;
        for (int i = 0; i < num_kb; ++i, ++kb_global) {
          const int s = kb_global % STAGES;
          const uint32_t ph = (kb_global / STAGES) & 1;
          c0 = p.prof ? clock64() : 0ull;
          if (!mbar_wait(&full_bar[s], ph, p.err, kErrTimeoutFull)) {
            *abort_flag = 1;
            break;
          }
          if (p.prof) t_full += clock64() - c0;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * S::kStage);
          const uint32_t sb = b_resident ? smem_u32(bres + (kb0 + i) * BN * 128) : sa + S::kA;
#pragma unroll
          for (int k = 0; k < BK / T::kUK; ++k) {
            uint64_t adesc, bdesc;
            // MN-major operands: BF16 uses the 16-byte-atom 128-byte swizzle
            // (8-row K groups, sbo 1024); TF32 needs the 32-byte-atom swizzle
            // (4-row K groups, sbo 512).
            if (!A_MN)
              adesc = make_sw128_desc(sa + k * 32, 16, 1024);
            else if (FMT == 2)
              adesc = make_sw128b32_desc(sa + k * T::kUK * 128, BK * 128, 512);
            else
              adesc = make_sw128_desc(sa + k * T::kUK * 128, BK * 128, 1024);
            if (!B_MN)
              bdesc = make_sw128_desc(sb + k * 32, 16, 1024);
            else if (FMT == 2)
              bdesc = make_sw128b32_desc(sb + k * T::kUK * 128, BK * 128, 512);
            else
              bdesc = make_sw128_desc(sb + k * T::kUK * 128, BK * 128, 1024);
            const uint32_t accum = (i > 0 || k > 0) ? 1u : 0u;
            if (FMT == 2)
              umma_tf32(d_tmem, adesc, bdesc, kIdesc, accum);
            else
              umma_bf16(d_tmem, adesc, bdesc, kIdesc, accum);
          }
          tc_commit(&empty_bar[s]);
        }
        // signal the epilogue (also on abort, so it does not wait for nothing)
        tc_commit(&tmem_full_bar[acc]);
        ++tile_i;
      }
      if (p.prof) {
        p.prof[blockIdx.x * 8 + 2] = t_acc;
        p.prof[blockIdx.x * 8 + 3] = t_full;
        p.prof[blockIdx.x * 8 + 7] = tile_i;
      }
    }
  } else {
    // epilogue warps 2..9
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    int tile_i = 0;
    unsigned long long t_ew = 0, t_work = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
      const TileCoord tc = tile_coord(p, t);
      int kb0, k_begin;
      if (tile_kblocks<BK>(p, tc.g, tc.split, &kb0, &k_begin) == 0) continue;
      const int acc = tile_i & 1;
      const uint32_t use = static_cast<uint32_t>(tile_i >> 1);
      ++tile_i;
      const unsigned long long c0 = p.prof ? clock64() : 0ull;
      const bool have = mbar_wait(&tmem_full_bar[acc], use & 1, p.err, kErrTimeoutTmemFull);
      tc_fence_after();
      const unsigned long long c1 = p.prof ? clock64() : 0ull;
      if (p.prof) t_ew += c1 - c0;
      if (!have || *abort_flag) break;
      const int tm = tc.tm, tn = tc.tn, g = tc.g, split = tc.split;
      const uint32_t taddr_row = tmem_base + static_cast<uint32_t>(acc) * kAccCols +
                                 (static_cast<uint32_t>(q * 32) << 16);
      const bool plain = !p.bias && !p.col_scale && !p.aux && !p.grad_pre && p.act == 0 && !p.out_bf16 &&
                         p.k_splits == 1 && p.beta == 0.f && p.n_peers == 0;
      const int esz = p.out_bf16 ? 2 : 4;
      const bool vec_ok = !p.c_pair && p.c_sc == 1 && p.c_sr != 1 && p.k_splits == 1 && p.beta == 0.f &&
                          p.n_peers == 0 &&
                          (reinterpret_cast<uintptr_t>(p.C) % 16 == 0) && ((p.c_sr * esz) % 16 == 0) &&
                          ((p.c_sg * esz) % 16 == 0) && (BN % 8 == 0) &&
                          (!p.aux || (reinterpret_cast<uintptr_t>(p.aux) % 16 == 0 && (p.c_sr * 2) % 16 == 0 &&
                                      (p.c_sg * 2) % 16 == 0)) &&
                          (!p.grad_pre || (reinterpret_cast<uintptr_t>(p.grad_pre) % 16 == 0 &&
                                           (p.c_sr * 2) % 16 == 0 && (p.c_sg * 2) % 16 == 0));
      const bool red_ok = p.k_splits > 1 && !p.c_pair && p.c_sc == 1 && p.c_sr != 1 && !p.bias && !p.col_scale &&
                          !p.aux && !p.grad_pre && p.act == 0 && !p.out_bf16 && p.n_peers == 0 &&
                          (reinterpret_cast<uintptr_t>(p.C) % 16 == 0) && ((p.c_sr * 4) % 16 == 0) &&
                          ((p.c_sg * 4) % 16 == 0);
      // Routed tiles of the sharded transforms: every tile has one destination rank
      // (analysis: the owner of wavenumber g; synthesis: the owner of the tile's
      // latitude block when the block width is a multiple of BN) and goes through
      // the staged, coalesced pair-row path; other synthesis tiles use the per-lane
      // routed path.
      int r_dst = -1, r_g = 0, r_shift = 0;
      if (p.route_mode == 2) {
        const int gm = __ldg(p.group_map + g);
        r_dst = gm >> 16;
        r_g = gm & 0xffff;
        if (r_dst >= p.n_peers || 2 * r_g >= p.route_rows) {
          record_error(p.err, kErrBounds);
          r_dst = -2;
        }
      } else if (p.route_mode == 1 && p.route_cols % BN == 0) {
        r_g = __ldg(p.group_map + g);
        r_dst = (tn * BN) / p.route_cols;
        r_shift = r_dst * p.route_cols;
        if (r_g < 0) {
          r_dst = -2;  // empty wavenumber slot: nothing to store
        } else if (r_dst >= p.n_peers || 2 * r_g >= p.route_rows) {
          record_error(p.err, kErrBounds);
          r_dst = -2;
        }
      }
      if (r_dst == -2) {
        // nothing to write for this tile; fall through to release the accumulator
      } else if (r_dst >= 0) {
        uint8_t* stage = reinterpret_cast<uint8_t*>(staging) + (warp - 2) * (32 * kStageRowF32);
        const bool slot = p.route_mode == 2 && p.route_slot >= 0;
        epilogue_pair_rows<BN>(p, taddr_row, stage, tm, tn, r_g, q, half, lane,
                               p.peer_C[r_dst] + (slot ? p.route_slot : 0), r_shift,
                               p.route_mode == 2 && !slot);
      } else if (red_ok) {
        uint8_t* stage = reinterpret_cast<uint8_t*>(staging) + (warp - 2) * (32 * kStageRowF32);
        epilogue_splitk_red<BN>(p, taddr_row, stage, tm, tn, g, q, half, lane);
      } else if (p.c_pair && p.c_sc == 1 && plain) {
        uint8_t* stage = reinterpret_cast<uint8_t*>(staging) + (warp - 2) * (32 * kStageRowF32);
        epilogue_pair_rows<BN>(p, taddr_row, stage, tm, tn, g, q, half, lane);
      } else if (vec_ok) {
        uint8_t* stage = reinterpret_cast<uint8_t*>(staging) + (warp - 2) * (32 * kStageRowF32);
        epilogue_rowmajor_dispatch<FMT, BN>(p, p.grad_pre ? p.grad_act : p.act, taddr_row, stage, tm, tn, g, q, half,
                                       lane);
      } else if (!p.c_pair && p.c_sc == 1 && p.c_sr != 1) {
        // Row-major C: stage each 32-row x 32-column block through shared
        // memory so that lanes walk along a row and every store instruction
        // writes one contiguous row segment.
        float* stage = staging + (warp - 2) * (32 * 33);
#pragma unroll 1
        for (int c0 = half * 32; c0 < BN; c0 += 64) {
          const int ncol = (BN - c0) >= 32 ? 32 : (BN - c0);
          uint32_t v0[16], v1[16];
          tmem_ld_32x32b_x16(taddr_row + c0, v0);
          if (ncol == 32) tmem_ld_32x32b_x16(taddr_row + c0 + 16, v1);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) stage[lane * 33 + j] = __uint_as_float(v0[j]);
          if (ncol == 32) {
#pragma unroll
            for (int j = 0; j < 16; ++j) stage[lane * 33 + 16 + j] = __uint_as_float(v1[j]);
          }
          __syncwarp();
          const int col = tn * BN + c0 + lane;
          const bool col_ok = lane < ncol && col < p.N;
          const int row0 = tm * 128 + q * 32;
          if (plain) {
            float* cbase = reinterpret_cast<float*>(p.C) + static_cast<long long>(g) * p.c_sg + col;
#pragma unroll 8
            for (int rr = 0; rr < 32; ++rr)
              if (col_ok && row0 + rr < p.M)
                cbase[static_cast<long long>(row0 + rr) * p.c_sr] = stage[rr * 33 + lane] * p.alpha;
          } else {
            const float cs = (col_ok && p.col_scale) ? p.col_scale[col] : 1.f;
            const float bs = (col_ok && p.bias && split == 0) ? p.bias[col] : 0.f;
#pragma unroll 4
            for (int rr = 0; rr < 32; ++rr) {
              const int row = row0 + rr;
              if (!col_ok || row >= p.M) continue;
              float x = stage[rr * 33 + lane] * p.alpha * cs + bs;
              const long long off =
                  static_cast<long long>(g) * p.c_sg + static_cast<long long>(row) * p.c_sr + col;
              if (p.aux) p.aux[off] = __float2bfloat16(x);
              if (p.grad_pre) x *= act_grad(p.grad_act, __bfloat162float(p.grad_pre[off]));
              x = apply_act(p.act, x);
              store_out(p, off, x);
            }
          }
          __syncwarp();
        }
      } else {
        // Column-strided C (lat-major transforms, pair layout): one lane per
        // row keeps consecutive lanes on consecutive addresses where the
        // layout allows it.
        const int r = q * 32 + lane;
        long long row_off = 0;
        bool row_ok;
        if (p.route_mode) {
          epilogue_routed<BN>(p, taddr_row, tm, tn, g, half, r);
          row_ok = false;
        } else if (p.c_pair) {
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
        for (int c0 = half * 16; c0 < BN && !p.route_mode; c0 += 32) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(taddr_row + c0, v);
          tmem_ld_wait();
          if (!row_ok) continue;
          const int colb = tn * BN + c0;
          if (p.n_peers > 0 && p.c_sc == 1 && colb + 16 <= p.N && !p.bias && !p.col_scale && p.act == 0 &&
              ((row_off + colb) & 3) == 0) {
            // peer reduction of 16 consecutive outputs: four 16-byte reductions per peer
            for (int i = 0; i < p.n_peers; ++i) {
              float* dst = p.peer_C[i] + row_off + colb;
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                red_add_sys_v4(dst + j, __uint_as_float(v[j]) * p.alpha, __uint_as_float(v[j + 1]) * p.alpha,
                               __uint_as_float(v[j + 2]) * p.alpha, __uint_as_float(v[j + 3]) * p.alpha);
            }
            continue;
          }
          if (plain && colb + 16 <= p.N) {
            float* cp = reinterpret_cast<float*>(p.C) + row_off + static_cast<long long>(colb) * p.c_sc;
#pragma unroll
            for (int j = 0; j < 16; ++j) cp[j * p.c_sc] = __uint_as_float(v[j]) * p.alpha;
            continue;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = colb + j;
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
      // this thread has finished reading the accumulator: release the buffer
      tc_fence_before();
      mbar_arrive(&tmem_empty_bar[acc]);
      if (p.prof) t_work += clock64() - c1;
    }
    if (p.n_peers > 0) __threadfence_system();  // peer reductions performed before the kernel ends
    if (p.prof && warp == 2 && lane == 0) {
      p.prof[blockIdx.x * 8 + 5] = t_ew;
      p.prof[blockIdx.x * 8 + 6] = t_work;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int FMT, int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const GemmParams p) {
  gemm_sm100_body<FMT, BN, STAGES, A_MN, B_MN>(tmap_a, &tmap_b, p);
}

// B gathered from up to 8 tensor maps (peer weight shards), K-major B only.
template <int FMT, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_gather_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ BMapSet bmaps,
                             const GemmParams p) {
  gemm_sm100_body<FMT, BN, STAGES, false, false>(tmap_a, bmaps.m, p);
}

}  // namespace tgcm
