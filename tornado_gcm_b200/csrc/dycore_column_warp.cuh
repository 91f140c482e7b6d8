// Warp-per-column versions of column_forward / column_vjp (dycore_column.h)
// for n <= 32 levels: lane k holds level k, so every per-level array of the
// thread-per-column code is one register, the column integrals are warp
// scans / reductions, vertical neighbours are one shuffle away and the fused
// geopotential matrix is a broadcast matvec.  (The thread-per-column VJP kept
// ~21 arrays of n floats per thread in local memory.)
//
// A block is 8 warps = 8 consecutive columns of the flattened (sample,
// lon·lat) index.  Fields are staged through a [32 levels][8 columns] shared
// tile: the global loads/stores of a tile are 32-byte sector aligned runs of
// 8 consecutive columns, and each warp then reads its column's 32 levels
// from shared memory.  Every thread of the block takes part in every tile
// (tail columns load zeros and store nothing), so the block-wide barriers
// are uniform.
//
// Semantics are those of column_forward / column_vjp; only the order of the
// floating-point sums differs (tree scans instead of sequential sweeps).
#pragma once

#include "dycore_column.h"

namespace tgcm {

constexpr int kColWarps = 8;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float wscan_incl(float v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__device__ __forceinline__ float wscan_suffix(float v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_down_sync(kFull, v, o);
    if (lane + o < 32) v += t;
  }
  return v;
}

// value of lane-1 (0 on lane 0) and of lane+1 (0 on lanes >= n-1)
__device__ __forceinline__ float from_below_lane(float v, int lane) {
  const float t = __shfl_up_sync(kFull, v, 1);
  return lane > 0 ? t : 0.f;
}
__device__ __forceinline__ float from_above_lane(float v, int lane, int n) {
  const float t = __shfl_down_sync(kFull, v, 1);
  return lane + 1 < n ? t : 0.f;
}

// Shared-memory staging of whole fields: slot s is a [32 levels][8 columns]
// tile (row pitch 9).  fetch() issues the global load of this thread's
// (level, column) element of a field and parks it in its slot without a
// barrier, so all fields of a phase are in flight at once; after one
// __syncthreads each warp reads its column's levels with get().  Outputs go
// the other way (put → barrier → flush).
constexpr int kSlotPitch = kColWarps + 1;
constexpr int kSlotFloats = 32 * kSlotPitch;

struct ColBlock {
  long long plane;
  long long off_in_c, off_out_c;  // this thread's staging column: sample offsets into in / out
  long long off_in_w, off_out_w;  // this warp's column
  bool valid_c, valid_w;
  int k_c, c_c, lane, warp;
  float* sm;

  __device__ void init(float* smem) {
    sm = smem;
    lane = threadIdx.x & 31;
    warp = threadIdx.x >> 5;
    k_c = threadIdx.x >> 3;
    c_c = threadIdx.x & 7;
  }

  __device__ void fetch(const float* __restrict__ src, bool out_side, int q0, int nlev, int slot) {
    const long long off = out_side ? off_out_c : off_in_c;
    float v = 0.f;
    if (valid_c && k_c < nlev) v = __ldg(src + off + static_cast<long long>(q0 + k_c) * plane);
    sm[slot * kSlotFloats + k_c * kSlotPitch + c_c] = v;
  }

  // fields f = 0..nf-1 (slices f * nlev ...) into slots slot0 + f; eight loads in flight per batch
  __device__ void fetch_fields(const float* __restrict__ src, bool out_side, int nf, int nlev, int slot0) {
    const long long off = out_side ? off_out_c : off_in_c;
    const bool ok = valid_c && k_c < nlev;
    for (int f0 = 0; f0 < nf; f0 += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = (ok && f0 + j < nf) ? __ldg(src + off + static_cast<long long>((f0 + j) * nlev + k_c) * plane) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (f0 + j < nf) sm[(slot0 + f0 + j) * kSlotFloats + k_c * kSlotPitch + c_c] = v[j];
    }
  }

  __device__ float get(int slot) const { return sm[slot * kSlotFloats + lane * kSlotPitch + warp]; }

  __device__ void put(int slot, float v) { sm[slot * kSlotFloats + lane * kSlotPitch + warp] = v; }

  __device__ void flush(float* __restrict__ dst, bool out_side, int q0, int nlev, int slot) const {
    if (valid_c && k_c < nlev)
      dst[(out_side ? off_out_c : off_in_c) + static_cast<long long>(q0 + k_c) * plane] =
          sm[slot * kSlotFloats + k_c * kSlotPitch + c_c];
  }

  __device__ float scalar(const float* __restrict__ src, bool out_side, int q) const {
    if (!valid_w) return 0.f;
    return __ldg(src + (out_side ? off_out_w : off_in_w) + static_cast<long long>(q) * plane);
  }
};

__device__ __forceinline__ void col_block_setup(ColBlock& cb, long long plane, long long total, int n_in, int n_out,
                                                int I, int J, int lat_major, int* j_w) {
  cb.plane = plane;
  const long long g0 = static_cast<long long>(blockIdx.x) * kColWarps;
  {
    const long long g = g0 + cb.c_c;
    cb.valid_c = g < total;
    const long long b = cb.valid_c ? g / plane : 0, ij = cb.valid_c ? g - b * plane : 0;
    cb.off_in_c = b * n_in * plane + ij;
    cb.off_out_c = b * n_out * plane + ij;
  }
  {
    const long long g = g0 + cb.warp;
    cb.valid_w = g < total;
    const long long b = cb.valid_w ? g / plane : 0, ij = cb.valid_w ? g - b * plane : 0;
    cb.off_in_w = b * n_in * plane + ij;
    cb.off_out_w = b * n_out * plane + ij;
    *j_w = lat_major ? static_cast<int>(ij / I) : static_cast<int>(ij % J);
  }
}

// Every n-level field of the column is a run of n slices starting at f * n
// (inputs: vort div temp u v tracers... qx qy; outputs: fu fv ke tn tu tv,
// (tr tr_u tr_v) per tracer, tdiff hdiv hvort), see make_slice_index.
__host__ __device__ inline int col_in_fields(int nt, int h) { return 5 + nt + 2 * h; }
__host__ __device__ inline int col_out_fields(int nt, int h) { return 6 + 3 * nt + 3 * h; }

// trv[idx] for a runtime idx without spilling the register array to local memory
__device__ __forceinline__ float pick(const float (&a)[kMaxTracers], int idx) {
  float r = 0.f;
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t) r = (t == idx) ? a[t] : r;
  return r;
}

// Per-block copies of the level constants and of the fused geopotential
// matrix.  The kernel parameters hold them, but a lane-dependent index into
// parameter space is serialised by the constant cache, and a row of G read
// across lanes is a 32-line strided global access; both are staged once per
// block instead (rows padded to 33 floats: conflict-free row and column reads).
struct ColShared {
  float dsig[32], alpha[32], tref[32], idc[32], cs[32];
  float g[32][33];
};

__device__ __forceinline__ void col_shared_fill(ColShared& sh, const ColumnConsts& c) {
  const int t = threadIdx.x, n = c.n;
  if (t < n) {
    sh.dsig[t] = c.dsig[t];
    sh.alpha[t] = c.alpha[t];
    sh.tref[t] = c.tref[t];
    sh.idc[t] = c.idc[t];
    sh.cs[t] = c.cs[t];
  }
  if (c.gmat != nullptr)
    for (int i = t; i < n * n; i += blockDim.x) sh.g[i / n][i % n] = __ldg(c.gmat + i);
}

// per-level constants of lane k (zeros beyond n)
struct LevelConsts {
  float dsig, alpha, alpha_m, tref, tref_p, tref_m, idc, idc_m, cs;
  __device__ void load(const ColShared& sh, int n, int k) {
    const bool in = k < n;
    dsig = in ? sh.dsig[k] : 1.f;
    alpha = in ? sh.alpha[k] : 0.f;
    alpha_m = (in && k > 0) ? sh.alpha[k - 1] : 0.f;
    tref = in ? sh.tref[k] : 0.f;
    tref_p = (k + 1 < n) ? sh.tref[k + 1] : 0.f;
    tref_m = (in && k > 0) ? sh.tref[k - 1] : 0.f;
    idc = (k + 1 < n) ? sh.idc[k] : 0.f;
    idc_m = (in && k > 0) ? sh.idc[k - 1] : 0.f;
    cs = (k + 1 < n) ? sh.cs[k] : 0.f;
  }
};

// ── forward ─────────────────────────────────────────────────────────────────
// dynamic shared memory: max(in_fields, out_fields) slots
__global__ void __launch_bounds__(32 * kColWarps) column_fwd_warp_kernel(
    ColumnConsts c, SliceIndex ix, const float* __restrict__ in, float* __restrict__ out,
    const float* __restrict__ sec2, const float* __restrict__ cor, int B, int I, int J, int lat_major) {
  extern __shared__ float smem_cols[];
  __shared__ ColShared csh;
  col_shared_fill(csh, c);
  const long long plane = static_cast<long long>(I) * J, total = static_cast<long long>(B) * plane;
  ColBlock cb;
  cb.init(smem_cols);
  int j_w = 0;
  col_block_setup(cb, plane, total, ix.n_in, ix.n_out, I, J, lat_major, &j_w);
  const int n = c.n, k = cb.lane, h = c.hum_terms ? 1 : 0;
  const int nin_f = col_in_fields(c.nt, h), nout_f = col_out_fields(c.nt, h);
  cb.fetch_fields(in, false, nin_f, n, 0);
  const float gx = cb.scalar(in, false, ix.gx), gy = cb.scalar(in, false, ix.gy);
  const float lap = c.hum_terms ? cb.scalar(in, false, ix.lap) : 0.f;
  const float s2 = cb.valid_w ? sec2[j_w] : 0.f, fcor = cb.valid_w ? cor[j_w] : 0.f;
  const bool lv = k < n;
  __syncthreads();
  LevelConsts L;
  L.load(csh, n, k);
  const float vort = cb.get(0), dv = cb.get(1), T = cb.get(2), u = cb.get(3), v = cb.get(4);
  float trv[kMaxTracers];
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t) trv[t] = (t < c.nt) ? cb.get(5 + t) : 0.f;
  float qx = 0.f, qy = 0.f;
  if (c.hum_terms) {
    qx = cb.get(5 + c.nt);
    qy = cb.get(6 + c.nt);
  }

  const float A = (u * gx + v * gy) * s2;
  const float ea = lv ? A * L.dsig : 0.f, fa = lv ? (dv + A) * L.dsig : 0.f;
  const float fe = wscan_incl(ea, k), ff = wscan_incl(fa, k);
  const float FE = wsum(ea), FF = wsum(fa);
  const bool last = k >= n - 1;
  const float sf = last ? 0.f : L.cs * FF - ff, se = last ? 0.f : L.cs * FE - fe;
  const float sf_m = from_below_lane(sf, k), se_m = from_below_lane(se, k);
  const float fe_m = from_below_lane(fe, k), ff_m = from_below_lane(ff, k);
  // -1/2 (w_k (x_{k+1}-x_k) idc_k + w_{k-1} (x_k - x_{k-1}) idc_{k-1})
  auto vadv = [&](float x) -> float {
    const float xp = from_above_lane(x, k, n), xm = from_below_lane(x, k);
    if (!c.vadv) return 0.f;
    const float dxp = last ? 0.f : (xp - x) * L.idc;
    const float dxm = k == 0 ? 0.f : (x - xm) * L.idc_m;
    return -0.5f * (sf * dxp + sf_m * dxm);
  };
  float q_hum = 0.f, adjf = 1.f;
  if (c.hum_terms) {
    q_hum = c.hum >= 0 ? pick(trv, c.hum) : 0.f;
    adjf = 1.f + (c.rv - 1.f) * q_hum;
    for (int t = 0; t < c.n_clouds; ++t) adjf -= pick(trv, c.clouds[t]);
  }
  const float rt = c.R * T * adjf;
  const float tv = vort + fcor;
  const float o_fu = (-v * tv - vadv(u) + rt * gx) * s2;
  const float o_fv = (u * tv - vadv(v) + rt * gy) * s2;
  float tvert = vadv(T);
  if (c.vadv) {
    const float dtp = last ? 0.f : (L.tref_p - L.tref) * L.idc;
    const float dtm = k == 0 ? 0.f : (L.tref - L.tref_m) * L.idc_m;
    tvert += -0.5f * (se * dtp + se_m * dtm);
  }
  const float he = (L.alpha * fe + L.alpha_m * fe_m) / L.dsig;
  const float hf = (L.alpha * ff + L.alpha_m * ff_m) / L.dsig;
  float vin = T;
  if (c.hum_terms) {
    const float D = 1.f + (c.cpv - 1.f) * q_hum;
    vin = T * ((1.f + (c.rv - 1.f) * q_hum) / D) + L.tref * (((c.rv - c.cpv) * q_hum) / D);
  }
  const float o_tn = T * dv + tvert + c.kappa * (L.tref * (A - he) + vin * (A - hf));
  float tr_out[kMaxTracers];
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t) tr_out[t] = (t < c.nt) ? trv[t] * dv + vadv(trv[t]) : 0.f;
  float o_td = 0.f, o_hd = 0.f, o_hv = 0.f;
  if (c.hum_terms) {
    const float rd = c.R * (c.rv - 1.f);
    const float tdk = lv ? q_hum * (T + L.tref) * (c.rv - 1.f) : 0.f;
    o_td = tdk;
    if (c.gmat) {  // (G td)_k = sum_j G[k][j] td_j
      float acc = 0.f;
      for (int jj = 0; jj < n; ++jj) {
        const float tj = __shfl_sync(kFull, tdk, jj);
        if (lv) acc = fmaf(csh.g[k][jj], tj, acc);
      }
      o_td = acc;
    }
    o_hd = rd * L.tref * s2 * (qx * gx + qy * gy) + q_hum * lap * L.tref * rd;
    o_hv = rd * L.tref * s2 * (gx * qy - gy * qx);
  }
  __syncthreads();  // all warps have read their inputs: the slots are reused for outputs
  cb.put(0, o_fu);
  cb.put(1, o_fv);
  cb.put(2, 0.5f * (u * u + v * v) * s2);
  cb.put(3, o_tn);
  cb.put(4, u * T * s2);
  cb.put(5, v * T * s2);
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t) {
    if (t < c.nt) {
      cb.put(6 + 3 * t, tr_out[t]);
      cb.put(7 + 3 * t, u * trv[t] * s2);
      cb.put(8 + 3 * t, v * trv[t] * s2);
    }
  }
  if (c.hum_terms) {
    cb.put(6 + 3 * c.nt, o_td);
    cb.put(7 + 3 * c.nt, o_hd);
    cb.put(8 + 3 * c.nt, o_hv);
  }
  __syncthreads();
  for (int f = 0; f < nout_f; ++f) cb.flush(out, true, f * n, n, f);
  if (cb.valid_w && k == 0) out[cb.off_out_w + static_cast<long long>(ix.lnps) * plane] = -FE;
}

// ── reverse mode ────────────────────────────────────────────────────────────
// dynamic shared memory: in_fields + out_fields slots (inputs, then output cotangents)
__global__ void __launch_bounds__(32 * kColWarps, 4) column_vjp_warp_kernel(
    ColumnConsts c, SliceIndex ix, const float* __restrict__ in, const float* __restrict__ gout,
    float* __restrict__ gin, const float* __restrict__ sec2, const float* __restrict__ cor, int B, int I, int J,
    int lat_major) {
  extern __shared__ float smem_cols[];
  __shared__ ColShared csh;
  col_shared_fill(csh, c);
  const long long plane = static_cast<long long>(I) * J, total = static_cast<long long>(B) * plane;
  ColBlock cb;
  cb.init(smem_cols);
  int j_w = 0;
  col_block_setup(cb, plane, total, ix.n_in, ix.n_out, I, J, lat_major, &j_w);
  const int n = c.n, k = cb.lane, h = c.hum_terms ? 1 : 0, nt = c.nt;
  const int NI = col_in_fields(nt, h), NO = col_out_fields(nt, h);
  cb.fetch_fields(in, false, NI, n, 0);
  cb.fetch_fields(gout, true, NO, n, NI);
  const float gx = cb.scalar(in, false, ix.gx), gy = cb.scalar(in, false, ix.gy);
  const float lap = c.hum_terms ? cb.scalar(in, false, ix.lap) : 0.f;
  const float g_lnps = cb.scalar(gout, true, ix.lnps);
  const float s2 = cb.valid_w ? sec2[j_w] : 0.f, fcor = cb.valid_w ? cor[j_w] : 0.f;
  const bool lv = k < n;
  const bool last = k >= n - 1;
  __syncthreads();
  LevelConsts L;
  L.load(csh, n, k);
  const float vort = cb.get(0), dv = cb.get(1), T = cb.get(2), u = cb.get(3), v = cb.get(4);
  float trv[kMaxTracers];
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t) trv[t] = (t < nt) ? cb.get(5 + t) : 0.f;

  // forward-sweep quantities
  const float A = (u * gx + v * gy) * s2;
  const float ea = lv ? A * L.dsig : 0.f, fa = lv ? (dv + A) * L.dsig : 0.f;
  const float fe = wscan_incl(ea, k), ff = wscan_incl(fa, k);
  const float FE = wsum(ea), FF = wsum(fa);
  (void)FE;
  const float sf = last ? 0.f : L.cs * FF - ff;
  const float sf_m = from_below_lane(sf, k);
  const float ff_m = from_below_lane(ff, k);
  (void)fe;

  float q_hum = 0.f, adjf = 1.f;
  if (c.hum_terms) {
    q_hum = c.hum >= 0 ? pick(trv, c.hum) : 0.f;
    adjf = 1.f + (c.rv - 1.f) * q_hum;
    for (int t = 0; t < c.n_clouds; ++t) adjf -= pick(trv, c.clouds[t]);
  }
  const float rt = c.R * T * adjf;
  const float tv = vort + fcor;

  // cotangent accumulators of lane k (level k)
  float g_u = 0.f, g_v = 0.f, g_T = 0.f, g_div = 0.f, g_vort = 0.f, g_A = 0.f;
  float g_fe = 0.f, g_ff = 0.f, g_sf = 0.f, g_se = 0.f, g_qx = 0.f, g_qy = 0.f, g_q = 0.f;
  float g_tr[kMaxTracers];
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t) g_tr[t] = 0.f;
  float g_gx = 0.f, g_gy = 0.f, g_lap = 0.f;  // per-lane partials, reduced at the end

  // vertical-advection adjoint of out_k = -1/2 (w_k dx_k + w_{k-1} dx_{k-1}) with cotangent V_k:
  // own level gets the w_k and x_k parts, lane k-1 the w_{k-1} and x_{k-1} parts, lane k+1 the x_{k+1} part.
  auto vadv_adj = [&](float x, float V, float& gw_acc, float& gx_acc) {
    const float xp = from_above_lane(x, k, n), xm = from_below_lane(x, k);
    const float gP = lv ? -0.5f * V : 0.f;
    const float dxp = last ? 0.f : (xp - x) * L.idc;
    const float dxm = k == 0 ? 0.f : (x - xm) * L.idc_m;
    const float gd = last ? 0.f : gP * sf * L.idc;          // +gx[k+1], -gx[k]
    const float gd2 = k == 0 ? 0.f : gP * sf_m * L.idc_m;   // +gx[k], -gx[k-1]
    gw_acc += gP * dxp + from_above_lane(gP * dxm, k, n);
    gx_acc += -gd + gd2 + from_below_lane(gd, k) - from_above_lane(gd2, k, n);
  };

  {  // momentum fluxes and kinetic energy
    const float Gfu = cb.get(NI + 0) * s2, Gfv = cb.get(NI + 1) * s2;
    g_v += -Gfu * tv;
    g_vort += -Gfu * v + Gfv * u;
    g_u += Gfv * tv;
    const float g_rt = Gfu * gx + Gfv * gy;
    g_gx += Gfu * rt;
    g_gy += Gfv * rt;
    g_T += g_rt * c.R * adjf;
    const float g_adj = g_rt * c.R * T;
    if (c.hum_terms) {
      g_q += g_adj * (c.rv - 1.f);
      for (int t = 0; t < c.n_clouds; ++t) {
#pragma unroll
        for (int tt = 0; tt < kMaxTracers; ++tt)
          if (tt == c.clouds[t]) g_tr[tt] -= g_adj;
      }
    }
    if (c.vadv) {
      vadv_adj(u, -Gfu, g_sf, g_u);
      vadv_adj(v, -Gfv, g_sf, g_v);
    }
    const float Gke = cb.get(NI + 2) * s2;
    g_u += Gke * u;
    g_v += Gke * v;
  }
  {  // temperature tendency
    const float Gt = cb.get(NI + 3);
    g_T += Gt * dv;
    g_div += Gt * T;
    const float Gk = Gt * c.kappa;
    const float hf = (L.alpha * ff + L.alpha_m * ff_m) / L.dsig;
    float vin = T, dvin_dT = 1.f, dvin_dq = 0.f;
    if (c.hum_terms) {
      const float D = 1.f + (c.cpv - 1.f) * q_hum;
      const float num1 = 1.f + (c.rv - 1.f) * q_hum;
      const float num2 = (c.rv - c.cpv) * q_hum;
      vin = T * (num1 / D) + L.tref * (num2 / D);
      dvin_dT = num1 / D;
      dvin_dq = (T * ((c.rv - 1.f) * D - num1 * (c.cpv - 1.f)) + L.tref * ((c.rv - c.cpv) * D - num2 * (c.cpv - 1.f))) /
                (D * D);
    }
    g_A += lv ? Gk * (L.tref + vin) : 0.f;
    const float g_vin = Gk * (A - hf);
    g_T += g_vin * dvin_dT;
    g_q += g_vin * dvin_dq;
    const float g_he = lv ? -Gk * L.tref : 0.f;
    const float g_hf = lv ? -Gk * vin : 0.f;
    // he_k = (alpha_k fe_k + alpha_{k-1} fe_{k-1}) / dsig_k (same for hf / ff)
    g_fe += g_he * L.alpha / L.dsig + from_above_lane(g_he * L.alpha_m / L.dsig, k, n);
    g_ff += g_hf * L.alpha / L.dsig + from_above_lane(g_hf * L.alpha_m / L.dsig, k, n);
    if (c.vadv) {
      vadv_adj(T, Gt, g_sf, g_T);
      // T_ref part: w = se, x = tref (constant): only the w cotangents
      const float gP = lv ? -0.5f * Gt : 0.f;
      const float dtp = last ? 0.f : (L.tref_p - L.tref) * L.idc;
      const float dtm = k == 0 ? 0.f : (L.tref - L.tref_m) * L.idc_m;
      g_se += gP * dtp + from_above_lane(gP * dtm, k, n);
    }
    const float Gtu = cb.get(NI + 4) * s2, Gtv = cb.get(NI + 5) * s2;
    g_u += Gtu * T;
    g_T += Gtu * u + Gtv * v;
    g_v += Gtv * T;
  }
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t) {  // tracers
    if (t < nt) {
      const float tr = trv[t];
      const float Gtr = cb.get(NI + 6 + 3 * t);
      const float Gu = cb.get(NI + 7 + 3 * t) * s2;
      const float Gv = cb.get(NI + 8 + 3 * t) * s2;
      g_tr[t] += Gtr * dv + Gu * u + Gv * v;
      g_div += Gtr * tr;
      g_u += Gu * tr;
      g_v += Gv * tr;
      if (c.vadv) vadv_adj(tr, Gtr, g_sf, g_tr[t]);
    }
  }
  if (c.hum_terms) {
    const float rd = c.R * (c.rv - 1.f);
    const float qx = cb.get(5 + nt), qy = cb.get(6 + nt);
    const float Gtd_raw = cb.get(NI + 6 + 3 * nt);
    float Gtd = Gtd_raw;
    if (c.gmat) {  // (G^T g)_k = sum_j G[j][k] g_j
      float acc = 0.f;
      for (int jj = 0; jj < n; ++jj) {
        const float gj = __shfl_sync(kFull, Gtd_raw, jj);
        if (lv) acc = fmaf(csh.g[jj][k], gj, acc);
      }
      Gtd = acc;
    }
    if (lv) {
      g_q += Gtd * (T + L.tref) * (c.rv - 1.f);
      g_T += Gtd * q_hum * (c.rv - 1.f);
    }
    const float Ghd = cb.get(NI + 7 + 3 * nt);
    const float cd = rd * L.tref * s2;
    g_qx += Ghd * cd * gx;
    g_qy += Ghd * cd * gy;
    g_gx += Ghd * cd * qx;
    g_gy += Ghd * cd * qy;
    g_q += Ghd * lap * L.tref * rd;
    g_lap += Ghd * q_hum * L.tref * rd;
    const float Ghv = cb.get(NI + 8 + 3 * nt);
    g_gx += Ghv * cd * qy;
    g_qy += Ghv * cd * gx;
    g_gy -= Ghv * cd * qx;
    g_qx -= Ghv * cd * gy;
#pragma unroll
    for (int tt = 0; tt < kMaxTracers; ++tt)
      if (tt == c.hum) g_tr[tt] += g_q;
  }
  // sigma-dot: sf_k = cs_k FF - ff_k ; se_k = cs_k FE - fe_k (k < n-1)
  const float g_FF = wsum(last ? 0.f : L.cs * g_sf);
  const float g_FE = wsum(last ? 0.f : L.cs * g_se) - g_lnps;
  if (!last) {
    g_ff -= g_sf;
    g_fe -= g_se;
  }
  if (k == n - 1) {  // FE = fe_{n-1}, FF = ff_{n-1}
    g_fe += g_FE;
    g_ff += g_FF;
  }
  if (!lv) {
    g_fe = 0.f;
    g_ff = 0.f;
  }
  // prefix sums -> suffix sums of the cotangents
  const float sa = wscan_suffix(g_fe, k), sb = wscan_suffix(g_ff, k);
  if (lv) {
    g_A += (sa + sb) * L.dsig;
    g_div += sb * L.dsig;
  }
  // A_k = (u gx + v gy) s2
  g_u += g_A * gx * s2;
  g_v += g_A * gy * s2;
  g_gx += g_A * u * s2;
  g_gy += g_A * v * s2;

  const float sgx = wsum(lv ? g_gx : 0.f), sgy = wsum(lv ? g_gy : 0.f), slap = wsum(lv ? g_lap : 0.f);
  __syncthreads();  // every warp is done reading the slots
  cb.put(0, g_vort);
  cb.put(1, g_div);
  cb.put(2, g_T);
  cb.put(3, g_u);
  cb.put(4, g_v);
#pragma unroll
  for (int t = 0; t < kMaxTracers; ++t)
    if (t < nt) cb.put(5 + t, g_tr[t]);
  if (c.hum_terms) {
    cb.put(5 + nt, g_qx);
    cb.put(6 + nt, g_qy);
  }
  __syncthreads();
  for (int f = 0; f < NI; ++f) cb.flush(gin, false, f * n, n, f);
  if (cb.valid_w && k == 0) {
    gin[cb.off_in_w + static_cast<long long>(ix.gx) * plane] = sgx;
    gin[cb.off_in_w + static_cast<long long>(ix.gy) * plane] = sgy;
    if (c.hum_terms) gin[cb.off_in_w + static_cast<long long>(ix.lap) * plane] = slap;
  }
}

}  // namespace tgcm
