// Per-column nonlinear explicit tendency of the sigma-coordinate primitive
// equations and its hand-written reverse-mode derivative (VJP).
//
// One column = one (sample, lon, lat) point with `n` sigma levels.  Inputs
// and outputs are "slices" of a stacked nodal buffer: value of slice q for
// this column sits at  base[q * slice_stride].  The functions are
// __host__ __device__ so the CUDA kernel and the CPU oracle run the very
// same code.
//
// Slice layout (per sample), n levels, NT tracers, h = humidity ? 1 : 0:
//   IN : vort[n] div[n] temp[n] u[n] v[n] tracer_t[n]... (qx[n] qy[n])^h gx gy (lap)^h
//   OUT: flux_u[n] flux_v[n] ke[n] temp[n] temp_u[n] temp_v[n]
//        (tr[n] tr_u[n] tr_v[n]) per tracer, (tdiff[n] hum_div[n] hum_vort[n])^h, lnps
//
// Semantics follow nodal_explicit_tendencies() in core/primitive_equations.py
// (the reference's explicit_terms, core/primitive_equations.py:612-1025).
#pragma once

#ifndef __CUDACC__
#define __host__
#define __device__
#define __forceinline__ inline
#endif

namespace tgcm {

constexpr int kMaxLevels = 64;
constexpr int kMaxTracers = 8;

struct ColumnConsts {
  int n;            // levels
  int nt;           // tracers
  int hum;          // humidity tracer index in [0, nt) or -1 (humidity terms off)
  int hum_terms;    // 1 when the humidity-key is configured (moist terms on)
  int n_clouds;
  int clouds[kMaxTracers];
  int vadv;         // vertical advection on/off
  float R, kappa, rv, cpv;
  float dsig[kMaxLevels];
  float alpha[kMaxLevels];
  float tref[kMaxLevels];
  float idc[kMaxLevels];
  float cs[kMaxLevels];
  // When set (n x n, row-major): the humidity temperature-difference output
  // tdiff_k is replaced by Σ_k' gmat[k][k'] tdiff_k' (the geopotential
  // operator applied in the column instead of on the spectral side).
  const float* gmat;
};

struct SliceIndex {
  int vort, div, temp, u, v, tr, qx, qy, gx, gy, lap;                // IN
  int fu, fv, ke, tn, tu, tv, otr, tdiff, hdiv, hvort, lnps;         // OUT
  int n_in, n_out;
};

__host__ __device__ __forceinline__ SliceIndex make_slice_index(const ColumnConsts& c) {
  SliceIndex s;
  const int n = c.n, h = c.hum_terms ? 1 : 0;
  s.vort = 0; s.div = n; s.temp = 2 * n; s.u = 3 * n; s.v = 4 * n; s.tr = 5 * n;
  s.qx = (5 + c.nt) * n; s.qy = s.qx + n;
  s.gx = (5 + c.nt + 2 * h) * n; s.gy = s.gx + 1; s.lap = s.gx + 2;
  s.n_in = s.gx + 2 + h;
  s.fu = 0; s.fv = n; s.ke = 2 * n; s.tn = 3 * n; s.tu = 4 * n; s.tv = 5 * n; s.otr = 6 * n;
  s.tdiff = (6 + 3 * c.nt) * n; s.hdiv = s.tdiff + n; s.hvort = s.hdiv + n;
  s.lnps = (6 + 3 * c.nt + 3 * h) * n;
  s.n_out = s.lnps + 1;
  return s;
}

// ── forward ─────────────────────────────────────────────────────────────────
template <int MAXL = kMaxLevels, typename In, typename Out>
__host__ __device__ void column_forward(const ColumnConsts& c, const SliceIndex& ix, In in, Out out, float s2,
                                        float fcor) {
  const int n = c.n;
  float td[MAXL];
  const float gx = in(ix.gx), gy = in(ix.gy);
  const float lap = c.hum_terms ? in(ix.lap) : 0.f;
  // pass 1: column totals of the two sigma-flux integrands
  float FE = 0.f, FF = 0.f;
  for (int k = 0; k < n; ++k) {
    const float A = (in(ix.u + k) * gx + in(ix.v + k) * gy) * s2;
    FE += A * c.dsig[k];
    FF += (in(ix.div + k) + A) * c.dsig[k];
  }
  out(ix.lnps, -FE);
  // pass 2: sweep down the column
  float fe = 0.f, ff = 0.f;            // inclusive prefix sums at level k
  float fe_prev = 0.f, ff_prev = 0.f;  // at level k-1
  float sf_prev = 0.f, se_prev = 0.f;  // sigma-dot at boundary k-1/2
  // x(k+1) lookahead values for vertical differences
  for (int k = 0; k < n; ++k) {
    const float u = in(ix.u + k), v = in(ix.v + k), T = in(ix.temp + k), dv = in(ix.div + k);
    const float A = (u * gx + v * gy) * s2;
    fe += A * c.dsig[k];
    ff += (dv + A) * c.dsig[k];
    const bool last = (k == n - 1);
    const float sf = last ? 0.f : c.cs[k] * FF - ff;  // boundary k+1/2
    const float se = last ? 0.f : c.cs[k] * FE - fe;
    // vertical differences at k+1/2 and k-1/2
    auto dxp = [&](int q) -> float { return last ? 0.f : (in(q + k + 1) - in(q + k)) * c.idc[k]; };
    auto dxm = [&](int q) -> float { return k == 0 ? 0.f : (in(q + k) - in(q + k - 1)) * c.idc[k - 1]; };
    auto vadv = [&](int q, float wp, float wm) -> float {
      if (!c.vadv) return 0.f;
      return -0.5f * (wp * dxp(q) + wm * dxm(q));
    };
    float q_hum = 0.f, adjf = 1.f;
    if (c.hum_terms) {
      q_hum = c.hum >= 0 ? in(ix.tr + c.hum * n + k) : 0.f;
      adjf = 1.f + (c.rv - 1.f) * q_hum;
      for (int t = 0; t < c.n_clouds; ++t) adjf -= in(ix.tr + c.clouds[t] * n + k);
    }
    const float rt = c.R * T * adjf;
    const float tv = in(ix.vort + k) + fcor;
    const float au = -vadv(ix.u, sf, sf_prev);
    const float av = -vadv(ix.v, sf, sf_prev);
    out(ix.fu + k, (-v * tv + au + rt * gx) * s2);
    out(ix.fv + k, (u * tv + av + rt * gy) * s2);
    out(ix.ke + k, 0.5f * (u * u + v * v) * s2);
    // temperature
    float tvert = 0.f;
    if (c.vadv) {
      tvert = vadv(ix.temp, sf, sf_prev);
      const float dtp = last ? 0.f : (c.tref[k + 1] - c.tref[k]) * c.idc[k];
      const float dtm = k == 0 ? 0.f : (c.tref[k] - c.tref[k - 1]) * c.idc[k - 1];
      tvert += -0.5f * (se * dtp + se_prev * dtm);
    }
    const float he = (c.alpha[k] * fe + (k > 0 ? c.alpha[k - 1] * fe_prev : 0.f)) / c.dsig[k];
    const float hf = (c.alpha[k] * ff + (k > 0 ? c.alpha[k - 1] * ff_prev : 0.f)) / c.dsig[k];
    const float mean_part = c.tref[k] * (A - he);
    float vin = T;
    if (c.hum_terms) {
      const float D = 1.f + (c.cpv - 1.f) * q_hum;
      vin = T * ((1.f + (c.rv - 1.f) * q_hum) / D) + c.tref[k] * (((c.rv - c.cpv) * q_hum) / D);
    }
    const float var_part = vin * (A - hf);
    out(ix.tn + k, T * dv + tvert + c.kappa * (mean_part + var_part));
    out(ix.tu + k, u * T * s2);
    out(ix.tv + k, v * T * s2);
    for (int t = 0; t < c.nt; ++t) {
      const int q = ix.tr + t * n;
      const float tr = in(q + k);
      out(ix.otr + 3 * t * n + k, tr * dv + vadv(q, sf, sf_prev));
      out(ix.otr + 3 * t * n + n + k, u * tr * s2);
      out(ix.otr + 3 * t * n + 2 * n + k, v * tr * s2);
    }
    if (c.hum_terms) {
      const float rd = c.R * (c.rv - 1.f);
      const float qx = in(ix.qx + k), qy = in(ix.qy + k);
      const float tdk = q_hum * (T + c.tref[k]) * (c.rv - 1.f);
      if (c.gmat)
        td[k] = tdk;
      else
        out(ix.tdiff + k, tdk);
      out(ix.hdiv + k, rd * c.tref[k] * s2 * (qx * gx + qy * gy) + q_hum * lap * c.tref[k] * rd);
      out(ix.hvort + k, rd * c.tref[k] * s2 * (gx * qy - gy * qx));
    }
    fe_prev = fe;
    ff_prev = ff;
    sf_prev = sf;
    se_prev = se;
  }
  if (c.hum_terms && c.gmat) {
    for (int k = 0; k < n; ++k) {
      float acc = 0.f;
      for (int j = 0; j < n; ++j) acc += c.gmat[k * n + j] * td[j];
      out(ix.tdiff + k, acc);
    }
  }
}

// ── reverse mode ────────────────────────────────────────────────────────────
// `gin(q, v)` accumulates v into the cotangent of input slice q (each input
// slice of the column is written exactly once at the end: the function
// keeps the accumulators in local arrays and calls gin once per slice).
// MAXL / MAXT bound the per-column scratch arrays (levels / tracers); the GPU
// launches the smallest instantiation that fits, which keeps the thread's
// local-memory footprint proportional to the actual column.
template <int MAXL = kMaxLevels, int MAXT = kMaxTracers, typename In, typename GOut, typename GIn>
__host__ __device__ void column_vjp(const ColumnConsts& c, const SliceIndex& ix, In in, GOut gout, GIn gin,
                                    float s2, float fcor) {
  const int n = c.n;
  const float gx = in(ix.gx), gy = in(ix.gy);
  const float lap = c.hum_terms ? in(ix.lap) : 0.f;
  float FE = 0.f, FF = 0.f;
  for (int k = 0; k < n; ++k) {
    const float A = (in(ix.u + k) * gx + in(ix.v + k) * gy) * s2;
    FE += A * c.dsig[k];
    FF += (in(ix.div + k) + A) * c.dsig[k];
  }
  // forward-sweep quantities needed in reverse: prefix sums and sigma-dot
  float fe[MAXL], ff[MAXL], sf[MAXL], se[MAXL];
  {
    float a = 0.f, b = 0.f;
    for (int k = 0; k < n; ++k) {
      const float A = (in(ix.u + k) * gx + in(ix.v + k) * gy) * s2;
      a += A * c.dsig[k];
      b += (in(ix.div + k) + A) * c.dsig[k];
      fe[k] = a;
      ff[k] = b;
      sf[k] = (k == n - 1) ? 0.f : c.cs[k] * FF - b;
      se[k] = (k == n - 1) ? 0.f : c.cs[k] * FE - a;
    }
  }
  // cotangent accumulators
  float g_u[MAXL], g_v[MAXL], g_T[MAXL], g_div[MAXL], g_vort[MAXL];
  float g_A[MAXL], g_fe[MAXL], g_ff[MAXL], g_sf[MAXL], g_se[MAXL];
  float g_tr[MAXT][MAXL];
  float g_qx[MAXL], g_qy[MAXL];
  for (int k = 0; k < n; ++k) {
    g_u[k] = g_v[k] = g_T[k] = g_div[k] = g_vort[k] = 0.f;
    g_A[k] = g_fe[k] = g_ff[k] = g_sf[k] = g_se[k] = 0.f;
    g_qx[k] = g_qy[k] = 0.f;
    for (int t = 0; t < c.nt; ++t) g_tr[t][k] = 0.f;
  }
  float g_gx = 0.f, g_gy = 0.f, g_lap = 0.f, g_FE = 0.f, g_FF = 0.f;
  // cotangent of the per-level tdiff values (through gmat when it is fused)
  float g_td[MAXL];
  if (c.hum_terms) {
    for (int k = 0; k < n; ++k) {
      if (c.gmat) {
        float acc = 0.f;
        for (int j = 0; j < n; ++j) acc += c.gmat[j * n + k] * gout(ix.tdiff + j);
        g_td[k] = acc;
      } else {
        g_td[k] = gout(ix.tdiff + k);
      }
    }
  }
  g_FE -= gout(ix.lnps);

  // vertical-advection adjoint: out_k = -1/2 (w_k dx_k + w_{k-1} dx_{k-1});
  // adds to cotangents of w (boundary values) and of x slices.
  // Implemented per level inside the main loop via the products P_k = w_k dx_k.
  for (int k = 0; k < n; ++k) {
    const float u = in(ix.u + k), v = in(ix.v + k), T = in(ix.temp + k), dv = in(ix.div + k);
    const float A = (u * gx + v * gy) * s2;
    float q_hum = 0.f, adjf = 1.f;
    if (c.hum_terms) {
      q_hum = c.hum >= 0 ? in(ix.tr + c.hum * n + k) : 0.f;
      adjf = 1.f + (c.rv - 1.f) * q_hum;
      for (int t = 0; t < c.n_clouds; ++t) adjf -= in(ix.tr + c.clouds[t] * n + k);
    }
    const float rt = c.R * T * adjf;
    const float tv = in(ix.vort + k) + fcor;
    // flux_u = (-v tv + au + rt gx) s2 ; flux_v = (u tv + av + rt gy) s2
    const float Gfu = gout(ix.fu + k) * s2, Gfv = gout(ix.fv + k) * s2;
    g_v[k] += -Gfu * tv;
    g_vort[k] += -Gfu * v + Gfv * u;
    g_u[k] += Gfv * tv;
    float g_rt = Gfu * gx + Gfv * gy;
    g_gx += Gfu * rt;
    g_gy += Gfv * rt;
    // au = -vadv(sf, u) -> d/d(vadv) = -Gfu ; av likewise
    const float Vu = -Gfu, Vv = -Gfv;  // cotangents of vadv(sf,u)_k, vadv(sf,v)_k
    // rt = R T adjf
    g_T[k] += g_rt * c.R * adjf;
    const float g_adj = g_rt * c.R * T;
    // ke
    const float Gke = gout(ix.ke + k) * s2;
    g_u[k] += Gke * u;
    g_v[k] += Gke * v;
    // temperature tendency
    const float Gt = gout(ix.tn + k);
    g_T[k] += Gt * dv;
    g_div[k] += Gt * T;
    // vertical advection of T (cotangent Gt on vadv(sf,T)_k) and of T_ref (Gt on vadv(se,Tref)_k)
    float VT = c.vadv ? Gt : 0.f;
    float VTr = c.vadv ? Gt : 0.f;
    // adiabatic: kappa * (Tref (A - he) + vin (A - hf))
    const float Gk = Gt * c.kappa;
    const float he = (c.alpha[k] * fe[k] + (k > 0 ? c.alpha[k - 1] * fe[k - 1] : 0.f)) / c.dsig[k];
    const float hf = (c.alpha[k] * ff[k] + (k > 0 ? c.alpha[k - 1] * ff[k - 1] : 0.f)) / c.dsig[k];
    float vin = T, dvin_dT = 1.f, dvin_dq = 0.f;
    if (c.hum_terms) {
      const float D = 1.f + (c.cpv - 1.f) * q_hum;
      const float num1 = 1.f + (c.rv - 1.f) * q_hum;
      const float num2 = (c.rv - c.cpv) * q_hum;
      vin = T * (num1 / D) + c.tref[k] * (num2 / D);
      dvin_dT = num1 / D;
      // d/dq [T num1/D + Tr num2/D] = T((rv-1) D - num1 (cpv-1))/D^2 + Tr((rv-cpv) D - num2 (cpv-1))/D^2
      dvin_dq = (T * ((c.rv - 1.f) * D - num1 * (c.cpv - 1.f)) +
                 c.tref[k] * ((c.rv - c.cpv) * D - num2 * (c.cpv - 1.f))) / (D * D);
    }
    g_A[k] += Gk * (c.tref[k] + vin);
    const float g_vin = Gk * (A - hf);
    g_T[k] += g_vin * dvin_dT;
    float g_q = g_vin * dvin_dq;
    // he, hf adjoints -> prefix sums
    const float g_he = -Gk * c.tref[k];
    const float g_hf = -Gk * vin;
    g_fe[k] += g_he * c.alpha[k] / c.dsig[k];
    g_ff[k] += g_hf * c.alpha[k] / c.dsig[k];
    if (k > 0) {
      g_fe[k - 1] += g_he * c.alpha[k - 1] / c.dsig[k];
      g_ff[k - 1] += g_hf * c.alpha[k - 1] / c.dsig[k];
    }
    // temp_u, temp_v
    const float Gtu = gout(ix.tu + k) * s2, Gtv = gout(ix.tv + k) * s2;
    g_u[k] += Gtu * T;
    g_T[k] += Gtu * u + Gtv * v;
    g_v[k] += Gtv * T;
    // vertical advection adjoints for u, v, T, Tref (sf / se)
    if (c.vadv) {
      // out_k gets -1/2 (P_k + P_{k-1}) with P_k = w_k dx_k (k < n-1)
      auto vadv_adj = [&](int q, float V, float* gw, const float* w, float* gx_arr, bool const_x) {
        // contribution to P_k and P_{k-1}
        const float gP = -0.5f * V;
        if (k < n - 1) {
          const float dx = (const_x ? (c.tref[k + 1] - c.tref[k]) : (in(q + k + 1) - in(q + k))) * c.idc[k];
          gw[k] += gP * dx;
          if (!const_x) {
            const float gd = gP * w[k] * c.idc[k];
            gx_arr[k + 1] += gd;
            gx_arr[k] -= gd;
          }
        }
        if (k > 0) {
          const float dx = (const_x ? (c.tref[k] - c.tref[k - 1]) : (in(q + k) - in(q + k - 1))) * c.idc[k - 1];
          gw[k - 1] += gP * dx;
          if (!const_x) {
            const float gd = gP * w[k - 1] * c.idc[k - 1];
            gx_arr[k] += gd;
            gx_arr[k - 1] -= gd;
          }
        }
      };
      vadv_adj(ix.u, Vu, g_sf, sf, g_u, false);
      vadv_adj(ix.v, Vv, g_sf, sf, g_v, false);
      vadv_adj(ix.temp, VT, g_sf, sf, g_T, false);
      vadv_adj(0, VTr, g_se, se, nullptr, true);
      for (int t = 0; t < c.nt; ++t) {
        const int q = ix.tr + t * n;
        const float Gtr = gout(ix.otr + 3 * t * n + k);
        vadv_adj(q, Gtr, g_sf, sf, g_tr[t], false);
      }
    }
    // tracers
    for (int t = 0; t < c.nt; ++t) {
      const int q = ix.tr + t * n;
      const float tr = in(q + k);
      const float Gtr = gout(ix.otr + 3 * t * n + k);
      const float Gu = gout(ix.otr + 3 * t * n + n + k) * s2;
      const float Gv = gout(ix.otr + 3 * t * n + 2 * n + k) * s2;
      g_tr[t][k] += Gtr * dv + Gu * u + Gv * v;
      g_div[k] += Gtr * tr;
      g_u[k] += Gu * tr;
      g_v[k] += Gv * tr;
    }
    if (c.hum_terms) {
      const float rd = c.R * (c.rv - 1.f);
      const float qx = in(ix.qx + k), qy = in(ix.qy + k);
      const float Gtd = g_td[k];
      g_q += Gtd * (T + c.tref[k]) * (c.rv - 1.f);
      g_T[k] += Gtd * q_hum * (c.rv - 1.f);
      const float Ghd = gout(ix.hdiv + k);
      const float cd = rd * c.tref[k] * s2;
      g_qx[k] += Ghd * cd * gx;
      g_qy[k] += Ghd * cd * gy;
      g_gx += Ghd * cd * qx;
      g_gy += Ghd * cd * qy;
      g_q += Ghd * lap * c.tref[k] * rd;
      g_lap += Ghd * q_hum * c.tref[k] * rd;
      const float Ghv = gout(ix.hvort + k);
      g_gx += Ghv * cd * qy;
      g_qy[k] += Ghv * cd * gx;
      g_gy -= Ghv * cd * qx;
      g_qx[k] -= Ghv * cd * gy;
      // adjustment factor: adjf = 1 + (rv-1) q - sum clouds
      g_q += g_adj * (c.rv - 1.f);
      for (int t = 0; t < c.n_clouds; ++t) g_tr[c.clouds[t]][k] -= g_adj;
      if (c.hum >= 0) g_tr[c.hum][k] += g_q;
    }
  }
  // sigma-dot: sf_k = cs_k FF - ff_k ; se_k = cs_k FE - fe_k  (k < n-1)
  for (int k = 0; k < n - 1; ++k) {
    g_FF += c.cs[k] * g_sf[k];
    g_ff[k] -= g_sf[k];
    g_FE += c.cs[k] * g_se[k];
    g_fe[k] -= g_se[k];
  }
  // FE = fe_{n-1}, FF = ff_{n-1}
  g_fe[n - 1] += g_FE;
  g_ff[n - 1] += g_FF;
  // prefix sums -> suffix sums of cotangents
  float sa = 0.f, sb = 0.f;
  for (int k = n - 1; k >= 0; --k) {
    sa += g_fe[k];
    sb += g_ff[k];
    // fe_k = sum_{k'<=k} A_k' dsig_k' ; ff_k = sum (div + A) dsig
    g_A[k] += (sa + sb) * c.dsig[k];
    g_div[k] += sb * c.dsig[k];
  }
  // A_k = (u gx + v gy) s2
  for (int k = 0; k < n; ++k) {
    const float u = in(ix.u + k), v = in(ix.v + k);
    g_u[k] += g_A[k] * gx * s2;
    g_v[k] += g_A[k] * gy * s2;
    g_gx += g_A[k] * u * s2;
    g_gy += g_A[k] * v * s2;
  }
  for (int k = 0; k < n; ++k) {
    gin(ix.vort + k, g_vort[k]);
    gin(ix.div + k, g_div[k]);
    gin(ix.temp + k, g_T[k]);
    gin(ix.u + k, g_u[k]);
    gin(ix.v + k, g_v[k]);
    for (int t = 0; t < c.nt; ++t) gin(ix.tr + t * n + k, g_tr[t][k]);
    if (c.hum_terms) {
      gin(ix.qx + k, g_qx[k]);
      gin(ix.qy + k, g_qy[k]);
    }
  }
  gin(ix.gx, g_gx);
  gin(ix.gy, g_gy);
  if (c.hum_terms) gin(ix.lap, g_lap);
}

}  // namespace tgcm
