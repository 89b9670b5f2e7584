// fdm_device.cuh -- device-side F-16 6-DoF + FCS frame for sm_100a (fp64, one thread per aircraft).
//
// Physics: JSBSim v1.0.0 F-16 as restated by the reference (cuda_fdm/gen/fdm.cuh:609-649 and
// the functions it calls).  The frame order, integrators, FCS, engine, atmosphere, air data and
// the 40 aerodynamic coefficient terms are the reference's; the implementation is organised for
// the GPU:
//   * the coefficient data (F16_TAB, 11.9 KB) is staged once per block in shared memory,
//     together with per-segment reciprocal spans and per-layer atmosphere constants computed
//     by the block at start-up, so no table lookup divides;
//   * the 25 lookups that share the 12-point angle-of-attack grid use ONE segment search per
//     frame; the 3 elevator-column, 2 beta13 and 4 beta7 tables share one column search each;
//   * kinematics run in the ECI frame: the local NED frame in ECI (Tl2i) is built from the
//     inertial longitude atan2(py,px) directly and J2 gravity is evaluated in ECI, so the
//     earth-position angle never needs a sin/cos (it only advances, as the reference does);
//   * euler angles (3 transcendentals) are produced only for the frame whose obs17 is written;
//     the FCS only needs cos(theta)cos(phi), which is the (3,3) element of Tl2b;
//   * sin/cos of alpha and beta come from the body velocity components, pow() is exp(b*log a).
// These are exact identities; they change results only at the rounding level (parity
// tolerance 1e-9 relative, one frame, against the oracle).
#pragma once
#include <stdint.h>
#include "f16_tables.h"

namespace f16 {

// ---------------- shared-memory table image ----------------
// [0, F16_TAB_LEN)                 : coefficient data (F16_TAB)
// [F16_TAB_LEN, 2*F16_TAB_LEN)     : reciprocal of the span that starts at the same index
//                                    (valid for every abscissa/grid array)
// then ATM_K_* per-layer constants
constexpr int TAB_RSPAN = F16_TAB_LEN;
constexpr int ATM_TB = 2 * F16_TAB_LEN;          // base temperature of layer b (8)
constexpr int ATM_EXPP = ATM_TB + 8;             // g0*Mair/(Rstar*L_b)           (8)
constexpr int ATM_KISO = ATM_EXPP + 8;           // -g0*Mair/(Rstar*Tb_b)         (8)
constexpr int ATM_EXPD = ATM_KISO + 8;           // -1/(1+g0*Mair/(Rstar*L_b))    (8)
constexpr int ATM_KDISO = ATM_EXPD + 8;          // -(Rstar*T_b)/(g0*Mair)        (8)
constexpr int ATM_TOL = ATM_KDISO + 8;           // T_b / L_b                      (8)
constexpr int ATM_RDB = ATM_TOL + 8;             // 1/rho_b                        (9)
constexpr int ATM_LTB = ATM_RDB + 9;             // log(T_b)                       (8)
constexpr int SMEM_DOUBLES = ATM_LTB + 8;

// Threads per block of the FDM kernels (one aircraft per thread).
#ifndef F16_FDM_THREADS
#define F16_FDM_THREADS 256
#endif
constexpr int FDM_THREADS = F16_FDM_THREADS;


__device__ const double g_tab[F16_TAB_LEN] = {F16_TAB_VALUES};

constexpr double DT = 1.0 / 60.0;
constexpr double ROT = F16C_ROTATION_RATE;

// Reference table1d (fdm.cuh:50-60) with the span division replaced by the staged reciprocal.
// Out-of-line calls of the library's fp64 exp and log: the frame body is instantiated twice
// (with and without its outputs) and each inline expansion carries the whole function; one body
// each shortens the code the warps fetch (-0.7% per step, same results bit for bit).  atan2 stays
// inline: out of line it measured slower (+1.6%).
static __device__ __noinline__ double exp_ool(double x) { return exp(x); }
static __device__ __noinline__ double log_ool(double x) { return log(x); }

__device__ __forceinline__ double lut1(const double* __restrict__ T, int xo, int yo, int n, double k) {
  const double* x = T + xo;
  const double* y = T + yo;
  if (k <= x[0]) return y[0];
  if (k >= x[n - 1]) return y[n - 1];
  int r = 1;
  while (r < n - 1 && x[r] < k) r++;
  double f = (k - x[r - 1]) * T[TAB_RSPAN + xo + r - 1];
  f = f > 1.0 ? 1.0 : f;
  return f * (y[r] - y[r - 1]) + y[r - 1];
}

// Segment on a grid: index r in [1, n-1] and fraction (reference table2d row/col search,
// fdm.cuh:61-79).  edge = -1 below the grid, +1 above, 0 inside (for table1d's end clamps).
struct Seg {
  int r;
  double f;      // clamped to [0,1] (table2d semantics)
  int edge;
};
__device__ __forceinline__ Seg seg_find(const double* __restrict__ T, int xo, int n, double k) {
  const double* x = T + xo;
  int r = 1;
  while (r < n - 1 && x[r] < k) r++;
  Seg s;
  s.r = r;
  double f = (k - x[r - 1]) * T[TAB_RSPAN + xo + r - 1];
  s.f = f < 0.0 ? 0.0 : (f > 1.0 ? 1.0 : f);
  s.edge = (k <= x[0]) ? -1 : ((k >= x[n - 1]) ? 1 : 0);
  return s;
}
// table1d on a pre-searched grid (exact end clamps)
__device__ __forceinline__ double lut1s(const double* __restrict__ T, int yo, int n, const Seg& s) {
  const double* y = T + yo;
  if (s.edge < 0) return y[0];
  if (s.edge > 0) return y[n - 1];
  return s.f * (y[s.r] - y[s.r - 1]) + y[s.r - 1];
}
// table2d on pre-searched row and column segments
__device__ __forceinline__ double lut2s(const double* __restrict__ T, int dofs, int nc, const Seg& rs, const Seg& cs) {
  const double* d = T + dofs;
  int r = rs.r, c = cs.r;
  double a00 = d[(r - 1) * nc + c - 1], a10 = d[r * nc + c - 1];
  double a01 = d[(r - 1) * nc + c], a11 = d[r * nc + c];
  double c1 = rs.f * (a10 - a00) + a00;
  double c2 = rs.f * (a11 - a01) + a01;
  return c1 + cs.f * (c2 - c1);
}

__device__ __forceinline__ double clampd(double x, double lo, double hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Block start-up: stage the table image in shared memory (all threads participate).
__device__ __forceinline__ void stage_tables(double* __restrict__ S) {
  for (int i = threadIdx.x; i < F16_TAB_LEN; i += blockDim.x) S[i] = g_tab[i];
  __syncthreads();
  for (int i = threadIdx.x; i < F16_TAB_LEN - 1; i += blockDim.x) {
    double d = S[i + 1] - S[i];
    S[TAB_RSPAN + i] = (d != 0.0) ? 1.0 / d : 0.0;
  }
  // per-layer atmosphere constants: thread b computes layer b (the block waits at the barrier
  // below for the slowest layer only)
  if (threadIdx.x < 8) {
    const double* AL = S + F16T_ATM_ALT;
    const double* LA = S + F16T_ATM_LAPSE;
    const double gm = F16C_g0 * F16C_Mair;
    {
      const int b = threadIdx.x;
      // base temperature as the reference evaluates it: T(geometric(base altitude)) (fdm.cuh:190)
      double gp_b = AL[b];
      double h = (gp_b * F16C_EarthRadius) / (F16C_EarthRadius - gp_b);
      double gp = (h * F16C_EarthRadius) / (F16C_EarthRadius + h);
      double Tb;
      if (gp >= 0.0) {
        const double* X = S + F16T_ATM_ALT;
        const double* Y = S + F16T_ATM_TMP;
        if (gp <= X[0]) Tb = Y[0];
        else if (gp >= X[8]) Tb = Y[8];
        else {
          int r = 1;
          while (r < 8 && X[r] < gp) r++;
          double f = (gp - X[r - 1]) / (X[r] - X[r - 1]);
          if (f > 1.0) f = 1.0;
          Tb = f * (Y[r] - Y[r - 1]) + Y[r - 1];
        }
      } else {
        Tb = S[F16T_ATM_TMP] + gp * LA[0];
      }
      S[ATM_TB + b] = Tb;
      double L = LA[b];
      S[ATM_EXPP + b] = (L != 0.0) ? gm / (F16C_Rstar * L) : 0.0;
      S[ATM_KISO + b] = -gm / (F16C_Rstar * Tb);
      S[ATM_EXPD + b] = (L != 0.0) ? -1.0 / (1.0 + gm / (F16C_Rstar * L)) : 0.0;
      double Tt = S[F16T_ATM_TMP + b];
      S[ATM_KDISO + b] = -(F16C_Rstar * Tt) / gm;
      S[ATM_TOL + b] = (L != 0.0) ? Tt / L : 0.0;
      S[ATM_LTB + b] = log(Tb);
    }
  }
  if (threadIdx.x < 9) S[ATM_RDB + threadIdx.x] = 1.0 / S[F16T_ATM_DBRK + threadIdx.x];
  __syncthreads();
}

// ---------------- ISA atmosphere (fdm.cuh:174-224) ----------------
struct Air {
  double T, P, rho, ia, sigma, densalt;   // ia: 1 / speed of sound
};
__device__ __forceinline__ double geopot(double h) { return (h * F16C_EarthRadius) / (F16C_EarthRadius + h); }
__device__ __forceinline__ double geomet(double g) { return (g * F16C_EarthRadius) / (F16C_EarthRadius - g); }
__device__ __forceinline__ void isa(const double* __restrict__ S, double h, Air& o) {
  const double* AL = S + F16T_ATM_ALT;
  double gp = geopot(h);
  double T = (gp >= 0.0) ? lut1(S, F16T_ATM_ALT, F16T_ATM_TMP, 9, gp) : S[F16T_ATM_TMP] + gp * S[F16T_ATM_LAPSE];
  // pressure layer (fdm.cuh:181-194)
  int b = 7;
  double base = AL[7];
  for (int k = 0; k < 7; k++) {
    if (gp < AL[k + 1]) { b = k; base = AL[k]; break; }
  }
  double Tb = S[ATM_TB + b];
  double dh = gp - base;
  double L = S[F16T_ATM_LAPSE + b];
  double P;
  if (L != 0.0) {
    // (Tb / (Tb + L dh))^e as exp(e (log Tb - log(Tb + L dh))), log Tb staged per layer
    P = S[F16T_ATM_PBRK + b] * exp_ool(S[ATM_EXPP + b] * (S[ATM_LTB + b] - log_ool(Tb + L * dh)));
  } else {
    P = S[F16T_ATM_PBRK + b] * exp_ool(dh * S[ATM_KISO + b]);
  }
  const double ia = rsqrt(F16C_SHRatio * F16C_Reng * T);
  double rho = P * (F16C_SHRatio * ia * ia);          // P / (R T), with 1 / (R T) = gamma ia^2
  o.T = T;
  o.P = P;
  o.rho = rho;
  o.ia = ia;
  o.sigma = rho * (1.0 / (F16C_StdDaySLpressure / (F16C_Reng * F16C_StdDaySLtemperature)));
  // density altitude (fdm.cuh:195-206)
  int d = 7;
  for (int k = 0; k < 7; k++) {
    if (rho >= S[F16T_ATM_DBRK + k + 1]) { d = k; break; }
  }
  double Hb = AL[d], Ld = S[F16T_ATM_LAPSE + d];
  double da;
  double ratio = rho * S[ATM_RDB + d];
  if (Ld != 0.0) da = Hb + S[ATM_TOL + d] * (exp_ool(S[ATM_EXPD + d] * log_ool(ratio)) - 1.0);
  else da = Hb + S[ATM_KDISO + d] * log_ool(ratio);
  o.densalt = geomet(da);
}

// ---------------- mass properties (fdm.cuh:226-262), fuel split evenly over the two tanks ----------------
struct Mass {
  double cgx, cgz, mass, inv_mass;
  double Ixx, Iyy, Izz, Ixz;           // J = [[Ixx,0,-Ixz],[0,Iyy,0],[-Ixz,0,Izz]]
  double k1, k3, k4, k6;               // Jinv = [[k1,0,k3],[0,k4,0],[k3,0,k6]]
  double rpx, rpz;                     // aero reference point in body ft (y = 0)
};
// point-mass inertia contribution (reference mb_pm_inertia), diagonal + xz term only:
// the F-16 points lie in the symmetry plane except the two tanks at +-65 in (equal fuel), whose
// xy/yz products cancel exactly; the cg stays on the plane (cg_y == 0 exactly).
__device__ __forceinline__ void pm_add(double m, double rx, double ry, double rz, double cgx, double cgz,
                                       double& Jxx, double& Jyy, double& Jzz, double& Jxz) {
  const double k = F16C_INCHTOFT;
  double vx = k * (cgx - rx), vy = k * ry, vz = k * (cgz - rz);
  double sx = m * vx, sy = m * vy, sz = m * vz;
  double xx = sx * vx, yy = sy * vy, zz = sz * vz, xz = -sx * vz;
  Jxx += yy + zz;
  Jyy += xx + zz;
  Jzz += xx + yy;
  Jxz += xz;
}
__device__ __forceinline__ void mass_props(double fuel, Mass& o) {
  const double empty = 17400.0, pw = 230.0;
  double f0 = fuel * 0.5;
  double w = empty + (f0 + f0) + pw;
  double iw = 1.0 / w;
  o.cgx = (empty * -193.0 + pw * -336.2 + f0 * -174.4 + f0 * -174.4) * iw;
  o.cgz = (empty * -5.1 + pw * 0.0 + f0 * 5.0 + f0 * 5.0) * iw;
  double Jxx = 9496.0, Jyy = 55814.0, Jzz = 63100.0, Jxz = -982.0;
  const double ls = F16C_LBTOSLUG;
  pm_add(ls * empty, -193.0, 0.0, -5.1, o.cgx, o.cgz, Jxx, Jyy, Jzz, Jxz);
  pm_add(ls * pw, -336.2, 0.0, 0.0, o.cgx, o.cgz, Jxx, Jyy, Jzz, Jxz);
  pm_add(ls * f0, -174.4, 65.0, 5.0, o.cgx, o.cgz, Jxx, Jyy, Jzz, Jxz);
  pm_add(ls * f0, -174.4, -65.0, 5.0, o.cgx, o.cgz, Jxx, Jyy, Jzz, Jxz);
  double Ixx = Jxx, Iyy = Jyy, Izz = Jzz, Ixz = -Jxz;
  // reference inverse (fdm.cuh:245-252) with Ixy = Iyz = 0
  double k1 = Iyy * Izz, k3 = Iyy * Ixz;
  double den = 1.0 / (Ixx * k1 - Ixz * k3);
  o.k1 = k1 * den;
  o.k3 = k3 * den;
  o.k4 = (Izz * Ixx - Ixz * Ixz) * den;
  o.k6 = (Ixx * Iyy) * den;
  o.Ixx = Ixx; o.Iyy = Iyy; o.Izz = Izz; o.Ixz = Ixz;
  o.mass = ls * w;
  o.inv_mass = iw * (1.0 / ls);
  o.rpx = F16C_INCHTOFT * (o.cgx - -189.5);
  o.rpz = F16C_INCHTOFT * (o.cgz - 3.9);
}

// ---------------- FCS (fdm.cuh:264-418) ----------------
__device__ __forceinline__ bool near_eq(double a, double b) {
  return fabs(a - b) <= 1e-9 * fmax(fmax(1.0, fabs(a)), fabs(b));
}
constexpr int ACT_MAX_PASSES = 16;   // hard bound on actuator passes per FCS step

// two-detent actuator [-d, d] with equal times (aileron/elevator/rudder/lef); rate = 2d/t.
// The reference's pass loop (fdm.cuh:264-290 with two detents) moves at most once: a pass either
// reaches the target (y = x, after which the loop test finds them equal, or for a NaN target
// finds the remaining time NaN) or spends all of dt.  So it is one conditional step here,
// straight-line code the compiler can interleave across the three control channels.
__device__ __forceinline__ double act2(double& out, double in, double dlo, double dhi, double t, double inv_rate,
                                       double dt, bool seeded, double seed) {
  const double x = clampd(in * dhi, dlo, dhi);
  double y = seeded ? seed : out;
  const double rate = (dhi - dlo) / t;
  if (dt > 0.0 && !near_eq(x, y)) {
    if (t <= 0.0) {
      y = x;
    } else {
      const double need = fabs((x - y) * inv_rate);
      if (dt < need) y = (y < x) ? y + dt * rate : y - dt * rate;
      else y = x;
    }
  }
  out = y;
  return y;
}
// general multi-detent actuator (reference kinemat_run, fdm.cuh:264-290)
template <int N>
__device__ __forceinline__ double actn(double& out, double in, const double (&det)[N], const double (&tim)[N],
                                       double dt, bool seeded, double seed) {
  double rem = dt, x = in * det[N - 1];
  double y = seeded ? seed : out;
  x = clampd(x, det[0], det[N - 1]);
  for (int it = 0; it < ACT_MAX_PASSES && rem > 0.0 && !near_eq(x, y); it++) {
    int k = 1;
    for (;;) {
      bool go = (x < y) ? (det[k] < y) : (det[k] <= y);
      if (!go) break;
      k++;
      if (k >= N) break;
    }
    if (k >= N) k = N - 1;
    if (tim[k] <= 0.0) { y = x; break; }
    double rate = (det[k] - det[k - 1]) / tim[k];
    double tgt = clampd(x, det[k - 1], det[k]);
    double need = fabs((tgt - y) / rate);
    if (rem < need) {
      need = rem;
      if (y < x) y += need * rate; else y -= need * rate;
    } else {
      y = tgt;
    }
    rem -= need;
  }
  out = y;
  return y;
}
// PID (fdm.cuh:292-305); s = (input_prev, input_prev2, i_out_total)
__device__ __forceinline__ double pid(double kp, double ki, double kd, double& ip, double& ip2, double& iout,
                                      double in, double trig, bool clip, double lo, double hi, double dt,
                                      double inv_dt) {
  double dv = (in - ip) * inv_dt;
  double dI = 0.0;
  if (fabs(trig) < 0.000001) dI = 1.5 * in - 0.5 * ip;
  if (trig < 0.0) iout = 0.0;
  iout += ki * dt * dI;
  double out = kp * in + iout + kd * dv;
  ip2 = (trig < 0.0) ? 0.0 : ip;
  ip = in;
  if (clip) out = clampd(out, lo, hi);
  return out;
}
__device__ __forceinline__ double surface(double in, double lim) {
  // reference aerosurface_zc with symmetric limits (+-1 -> +-lim)
  return (in == 0.0) ? 0.0 : in * lim;
}

struct Surf {
  double ail, ele, rud, lef, flap, gear;
};
// kin: tef, aileron, elevator, rudder, gear, lef; pids: roll(3), gload(3), yaw(3); pa: prev aux
__device__ __forceinline__ void fcs(const double* __restrict__ S, double* kin, double* pd, double c_ail,
                                    double c_ele, double c_rud, const double* pa, double cthcph, double dt,
                                    double inv_dt, double gear_pos, Surf& o) {
  double alpha = pa[0], mach = pa[1], vc = pa[2], vg = pa[3], npy = pa[4], npz = pa[5];
  double p = pa[6], q = pa[7], r = pa[8];
  // flaps
  double tef = (vc < 250.0) ? 0.349 : ((mach > 0.9) ? -0.0349 : 0.0);
  const double d_tef[3] = {-1.0, 0.0, 1.0}, t_tef[3] = {3.0, 0.0, 3.0};
  double tef_c = actn<3>(kin[0], 2.864789 * tef, d_tef, t_tef, dt, false, 0.0);
  // roll
  double roll_err = c_ail - 0.31821 * p;
  double roll_pid = pid(3.0, 0.0005, -0.00125, pd[0], pd[1], pd[2], roll_err, (vc < 20.0) ? 0.0 : 1.0, false, 0,
                        0, dt, inv_dt);
  double roll_cmd = clampd(roll_pid + c_ail, -1.0, 1.0);
  double ail_n = act2(kin[1], roll_cmd, -1.0, 1.0, 0.3, 0.3 / 2.0, dt, false, 0.0);
  double ail_comp = lut1(S, F16T_FCS_AIL_SPEED_X, F16T_FCS_AIL_SPEED_Y, 2, mach) * ail_n;
  double fl = clampd(-tef_c - ail_comp, -1.0, 1.0);
  double fr = clampd(tef_c - ail_comp, -1.0, 1.0);
  o.flap = 1.4324 * (fl + fr);
  o.ail = surface(roll_cmd, 0.375);
  // pitch
  double gcorr = npz - cthcph;
  double ele_lim = clampd(c_ele + 0.0, -1.0, 0.44);
  double ele_sched = lut1(S, F16T_FCS_ELEV_SCHED_X, F16T_FCS_ELEV_SCHED_Y, 5, alpha) * ele_lim;
  double pitch_err = ele_sched + 6.2 * q - 0.020 * gcorr;
  double g_pid = pid(0.3, 0.025, 0.0, pd[3], pd[4], pd[5], pitch_err, (vc < 5.0) ? 0.0 : 1.0, true, -1.0, 1.0, dt,
                     inv_dt);
  double pitch_cmd = clampd(ele_sched + 1.0472 * alpha + g_pid, -1.0, 1.0);
  double ele_n = act2(kin[2], pitch_cmd, -1.0, 1.0, 0.3, 0.3 / 2.0, dt, false, 0.0);
  o.ele = surface(ele_n, 0.436);
  // yaw
  double yaw_err = c_rud + lut1(S, F16T_FCS_YAW_RATE_X, F16T_FCS_YAW_RATE_Y, 3, vg) * r + 0.25 * npy;
  double y_pid = pid(0.1055, 0.00001, 0.00005, pd[6], pd[7], pd[8], yaw_err, (vc < 10.0) ? 0.0 : 1.0, true, -1.0,
                     1.0, dt, inv_dt);
  double yaw_cmd = clampd(c_rud + 0.0 + y_pid, -1.0, 1.0);
  double rud_n = act2(kin[3], yaw_cmd, -1.0, 1.0, 0.4, 0.4 / 2.0, dt, true, y_pid);
  o.rud = surface(rud_n, 0.524);
  // landing gear: the actuator is re-seeded to 0.30 every frame with command 0, so its output
  // is the same every frame (gear_actuator() below); the reference evaluates it in place.
  double gear = gear_pos;
  kin[4] = gear;
  o.gear = gear;
  // leading-edge flaps (weight on wheels is always 0)
  double lef;
  if (gear == 0.0 && alpha > 0.2618) lef = 0.436;
  else if (alpha > 0.0873) lef = 0.262;
  else if (mach > 0.9) lef = -0.0349;
  else lef = 0.0;
  o.lef = lef;
  act2(kin[5], 2.293578 * lef, -1.0, 1.0, 3.0, 3.0 / 2.0, dt, false, 0.0);
}

// Landing-gear actuator output for one FCS step (fdm.cuh:392-394): command 0, seeded 0.30.
__device__ __forceinline__ double gear_actuator(double fcs_dt) {
  const double d_gear[2] = {0.0, 1.0}, t_gear[2] = {0.0, 5.0};
  double out = 0.0;
  return actn<2>(out, 0.0, d_gear, t_gear, fcs_dt, true, 0.30);
}

// ---------------- turbine (fdm.cuh:420-455) ----------------
__device__ __forceinline__ double approach(double v, double tgt, double up, double dn, double dt) {
  if (v > tgt) { v -= dt * dn; if (v < tgt) v = tgt; }
  else if (v < tgt) { v += dt * up; if (v > tgt) v = tgt; }
  return v;
}
// eng: N1, N2, N2norm, FF.  Returns thrust; fuel burn and pitching-moment arm via refs.
__device__ __forceinline__ double turbine(const double* __restrict__ S, double* eng, double thr, double mach,
                                          double densalt, double Tk, double sigma, double& burn) {
  const double dt = DT;
  double tp = thr, aug;
  if (tp > 1.0) { aug = tp - 1.0; tp -= aug; } else aug = 0.0;
  const double n1f = F16C_MAXN1 - F16C_IDLEN1, n2f = F16C_MAXN2 - F16C_IDLEN2;
  const double base = 90.0 / (F16C_BYPASSRATIO + 3.0);
  double n = eng[2] + 0.1;
  if (n > 1.0) n = 1.0;
  double om = 1.0 - n;
  double iden = 1.0 / (1.0 + 3.0 * om * om * om + (1.0 - sigma));
  double up = base * iden;                 // delay 1.0*base (N1 and N2 spool-up)
  double n2dn = (3.0 * base) * iden, n1dn = (2.4 * base) * iden;
  eng[1] = approach(eng[1], F16C_IDLEN2 + tp * n2f, up, n2dn, dt);
  eng[0] = approach(eng[0], F16C_IDLEN1 + tp * n1f, up, n1dn, dt);
  eng[2] = (eng[1] - F16C_IDLEN2) * (1.0 / n2f);
  Seg rs = seg_find(S, F16T_GRID_DENSALT, 8, densalt);
  // The idle (0..1.0) and military (0..1.4) Mach grids are the first 6 / 8 points of the
  // afterburner grid (0..2.6, same values): one search on it gives all three segments exactly
  // (past a shorter grid's end the segment is its last with fraction 1, as table2d clamps).
  Seg ma = seg_find(S, F16T_ENG_AUG_MACH, 14, mach);
  Seg mi = ma, mm = ma;
  if (ma.r > 5) { mi.r = 5; mi.f = 1.0; }
  if (ma.r > 7) { mm.r = 7; mm.f = 1.0; }
  double idle = F16C_MILTHRUST * lut2s(S, F16T_ENG_IDLE, 8, mi, rs);
  double mil = (F16C_MILTHRUST - idle) * lut2s(S, F16T_ENG_MIL, 8, mm, rs);
  double thrust = idle + mil * eng[2] * eng[2];
  double o2 = 1.0 - eng[2];
  double tsfc = F16C_TSFC * sqrt(Tk * (1.0 / 389.7)) * (0.84 + o2 * o2);
  eng[3] = approach(eng[3], thrust * tsfc, 1000.0, 10000.0, dt);
  if (eng[3] < F16C_IdleFF) eng[3] = F16C_IdleFF;
  if (aug > 0.0) {
    double td = (F16C_MAXTHRUST * lut2s(S, F16T_ENG_AUG, 8, ma, rs)) - thrust;
    thrust += td * aug;
    eng[3] = approach(eng[3], thrust * F16C_ATSFC, 5000.0, 10000.0, dt);
  }
  burn = eng[3] * (dt / 3600.0);
  return thrust;
}

// ---------------- calibrated airspeed (fdm.cuh:457-470) ----------------
__device__ __forceinline__ double mach_from_qc(double qc) {
  double A = qc * (1.0 / F16C_StdDaySLpressure) + 1.0;
  double m = sqrt(5.0 * (exp_ool(log_ool(A) * (1.0 / 3.5)) - 1.0));
  if (m > 1.0) {
    for (int i = 0; i < 10; i++) {
      double t = 1.0 - 1.0 / (7.0 * m * m);
      m = 0.8812848543473311 * sqrt(A * (t * t * sqrt(t)));
    }
  }
  return m;
}
__device__ __forceinline__ double vcas_kts(double mach, double P) {
  if (!(fabs(mach) > 0.0)) return 0.0;
  double pt;
  if (mach < 0.0) pt = P;
  else if (mach < 1.0) {
    double k = 1.0 + 0.2 * mach * mach;
    pt = P * k * k * k * sqrt(k);
  } else {
    double m2 = mach * mach;
    double d = 7.0 * m2 - 1.0;
    pt = P * 166.92158009316827 * (m2 * m2 * m2 * mach) / (d * d * sqrt(d));
  }
  return F16C_STD_SL_SOUNDSPEED * mach_from_qc(pt - P) * F16C_FPSTOKTS;
}

// ---------------- live aircraft state ----------------
struct Ac {
  double pos[3], vel[3], q[4], pqri[3], epa, fuel;
  double uvwidot[3], pqridot[3], qdot[4];
  double ivel1[3], ivel2[3];       // integrator history of eci_vel: deq_ivel[0], deq_ivel[1]
  double uvd1[3];                  // integrator history of the ECI acceleration: deq_uvwidot[0]
  double pbacc[3], ppqridot[3], ppqri[3];   // previous-frame accelerations: state fields, set
                                            // only by the frame whose state is stored
  double nld[2];                            // pilot load factor (y, z) of the coming frame
  double pa[9], eng[4], kin[6], pid[9];
};

// Pilot-station load factor (y, z) a frame computes from the previous frame's body
// accelerations (reference air data, fdm.cuh:471-497), with the eye point of the cg at `fuel`
// (mass_props' own expressions).  Evaluated when the accelerations are produced, for the frame
// that uses them, so the nine values need not stay live across the frame boundary.
__device__ __forceinline__ void load_factor(double fuel, const double* ba, const double* pd, const double* pr,
                                            double* nld) {
  const double empty = 17400.0, pw = 230.0;
  const double f0 = fuel * 0.5;
  const double iw = 1.0 / (empty + (f0 + f0) + pw);
  const double cgx = (empty * -193.0 + pw * -336.2 + f0 * -174.4 + f0 * -174.4) * iw;
  const double cgz = (empty * -5.1 + pw * 0.0 + f0 * 5.0 + f0 * 5.0) * iw;
  const double ex = F16C_INCHTOFT * (cgx - -336.2), ez = F16C_INCHTOFT * (cgz - 29.5);   // eye point (y = 0)
  const double c1y = pd[2] * ex - pd[0] * ez, c1z = -pd[1] * ex;
  const double c2x = pr[1] * ez, c2y = pr[2] * ex - pr[0] * ez, c2z = -pr[1] * ex;
  const double c3y = pr[2] * c2x - pr[0] * c2z, c3z = pr[0] * c2y - pr[1] * c2x;
  nld[0] = (ba[1] + c1y + c3y) * (1.0 / F16C_SLGRAVITY);
  nld[1] = (ba[2] + c1z + c3z) * (1.0 / F16C_SLGRAVITY);
}

struct FrameOut {
  double euler[3], uvw[3], alpha, beta, mach, vt, alt;
};

// Propagation half of the reference fdm_step (fdm.cuh:611-627): rect-Euler q (+ normalize) and
// body rates, AB3 position, AB2 velocity, earth position angle.  The values pushed into the
// integrator histories this frame are s.qdot, s.pqridot, s.vel and s.uvwidot as they are on entry.
__device__ __forceinline__ void propagate(Ac& s) {
  const double dt = DT;
  // ---- propagate (rect-Euler q and pqri, AB3 position, AB2 velocity) ----
  #pragma unroll
  for (int i = 0; i < 4; i++) s.q[i] = s.q[i] + dt * s.qdot[i];
  {
    const double qq = s.q[0] * s.q[0] + s.q[1] * s.q[1] + s.q[2] * s.q[2] + s.q[3] * s.q[3];
    if (qq != 0.0) {
      const double k = rsqrt(qq);                 // 1 / |q|
      s.q[0] *= k; s.q[1] *= k; s.q[2] *= k; s.q[3] *= k;
    }
  }
  #pragma unroll
  for (int i = 0; i < 3; i++) s.pqri[i] = s.pqri[i] + dt * s.pqridot[i];
  #pragma unroll
  for (int i = 0; i < 3; i++) {
    double v0 = s.vel[i];
    s.pos[i] = s.pos[i] + (dt / 12.0) * (23.0 * v0 - 16.0 * s.ivel1[i] + 5.0 * s.ivel2[i]);
    s.ivel2[i] = s.ivel1[i];
    s.ivel1[i] = v0;
    double u0 = s.uvwidot[i];
    s.vel[i] = s.vel[i] + dt * (1.5 * u0 - 0.5 * s.uvd1[i]);
    s.uvd1[i] = u0;
  }
  s.epa += ROT * dt;
}

// Kinematics + force path + derivative update of the reference fdm_step (fdm.cuh:629-648).
// gear_pos: landing-gear actuator output, constant per launch (seeded to 0.30 every frame).
// want_out: this frame's air data / euler angles go to `out` and the accelerations to the state's
// previous-frame fields (a literal at the call site folds the branches away)
__device__ __forceinline__ void dynamics(const double* __restrict__ S, Ac& s, double c_ail, double c_ele,
                                         double c_rud, double c_thr, double fcs_dt, double inv_fcs_dt,
                                         double gear_pos, FrameOut& out, const bool WANT_OUT) {
  // ---- kinematics (fdm.cuh:544-563) in ECI ----
  const double px = s.pos[0], py = s.pos[1], pz = s.pos[2];
  // reciprocal square roots, the lengths as products (rounding-level differences from
  // sqrt and a division)
  double rxy2 = px * px + py * py, rad2 = rxy2 + pz * pz;
  double irxy = rsqrt(rxy2), irad = rsqrt(rad2);
  double rxy = rxy2 * irxy, rad = rad2 * irad;
  double slo = py * irxy, clo = px * irxy;     // inertial longitude
  double sla = pz * irad, cla = rxy * irad;    // geocentric latitude
  // Tl2i columns = local N, E, D axes in ECI
  double N0 = -clo * sla, N1 = -slo * sla, N2 = cla;
  double E0 = -slo, E1 = clo;
  double D0 = -clo * cla, D1 = -slo * cla, D2 = -sla;
  // Ti2b from the quaternion (fdm.cuh:85-92)
  double a = s.q[0], b = s.q[1], c = s.q[2], d = s.q[3];
  double aa = a * a, bb = b * b, cc = c * c, dd = d * d;
  double ab = a * b, ac = a * c, ad = a * d, bc = b * c, bd = b * d, cd = c * d;
  double T00 = aa + bb - cc - dd, T01 = 2.0 * (bc + ad), T02 = 2.0 * (bd - ac);
  double T10 = 2.0 * (bc - ad), T11 = aa - bb + cc - dd, T12 = 2.0 * (cd + ab);
  double T20 = 2.0 * (bd + ac), T21 = 2.0 * (cd - ab), T22 = aa - bb - cc + dd;
  // inertial velocity relative to the rotating earth
  double dv0 = s.vel[0] + ROT * py, dv1 = s.vel[1] - ROT * px, dv2 = s.vel[2];
  double u = T00 * dv0 + T01 * dv1 + T02 * dv2;
  double v = T10 * dv0 + T11 * dv1 + T12 * dv2;
  double w = T20 * dv0 + T21 * dv1 + T22 * dv2;
  double p = s.pqri[0] - T02 * ROT, q = s.pqri[1] - T12 * ROT, r = s.pqri[2] - T22 * ROT;
  // NED ground-velocity components: Tl2i^T * dv
  double vn = N0 * dv0 + N1 * dv1 + N2 * dv2;
  double ve = E0 * dv0 + E1 * dv1;
  // Tl2b third column: cos(theta)cos(phi) = Tl2b[2][2] (body z . local D) -- FCS input
  double L22 = T20 * D0 + T21 * D1 + T22 * D2;
  if (WANT_OUT) {
    double L02 = T00 * D0 + T01 * D1 + T02 * D2;
    double L12 = T10 * D0 + T11 * D1 + T12 * D2;
    double L00 = T00 * N0 + T01 * N1 + T02 * N2;
    double L01 = T00 * E0 + T01 * E1;
    double L21 = T20 * E0 + T21 * E1;
    double L11 = T10 * E0 + T11 * E1;
    // reference mat_to_euler (fdm.cuh:123-131)
    if (L02 <= -1.0 || 1.0 <= L02) {
      out.euler[1] = (L02 <= -1.0) ? 0.5 * M_PI : -0.5 * M_PI;
      out.euler[0] = atan2(-L21, L11);
      out.euler[2] = 0.0;
    } else {
      out.euler[1] = asin(-L02);
      out.euler[0] = atan2(L12, L22);
      double psi = atan2(L01, L00);
      out.euler[2] = (psi < 0.0) ? psi + 2.0 * M_PI : psi;
    }
    out.uvw[0] = u; out.uvw[1] = v; out.uvw[2] = w;
  }
  // next quaternion rate (fdm.cuh:99-105), from the propagated q and pqri
  s.qdot[0] = -0.5 * (s.q[1] * s.pqri[0] + s.q[2] * s.pqri[1] + s.q[3] * s.pqri[2]);
  s.qdot[1] = 0.5 * (s.q[0] * s.pqri[0] - s.q[3] * s.pqri[1] + s.q[2] * s.pqri[2]);
  s.qdot[2] = 0.5 * (s.q[3] * s.pqri[0] + s.q[0] * s.pqri[1] - s.q[1] * s.pqri[2]);
  s.qdot[3] = 0.5 * (-s.q[2] * s.pqri[0] + s.q[1] * s.pqri[1] + s.q[0] * s.pqri[2]);

  // ---- force path (fdm.cuh:566-607) ----
  double alt = rad - F16C_SEA_LEVEL_RADIUS;
  Air at;
  isa(S, alt, at);
  Mass mp;
  mass_props(s.fuel, mp);
  Surf sf;
  fcs(S, s.kin, s.pid, c_ail, c_ele, c_rud, s.pa, L22, fcs_dt, inv_fcs_dt, gear_pos, sf);
  // air data (fdm.cuh:471-497)
  double uw = u * u + w * w, vt2 = uw + v * v;
  const double ivt = vt2 > 0.0 ? rsqrt(vt2) : 0.0, isuw = uw > 0.0 ? rsqrt(uw) : 0.0;
  const double vt = vt2 * ivt, suw = uw * isuw;
  double al = 0.0, be = 0.0;
  if (vt > 0.001) {
    be = atan2(v, suw);
    if (uw >= 1e-6) al = atan2(w, u);
  }
  double qbar = 0.5 * at.rho * vt2;
  double mach = vt * at.ia;
  double vg = sqrt(vn * vn + ve * ve);
  // pilot-station load factor from the previous frame's accelerations (load_factor)
  const double npy = s.nld[0], npz = s.nld[1];
  double vc = vcas_kts(mach, at.P);
  // engine (thr_pos = 2*cmd, fdm.cuh:586-587)
  double burn;
  double thrust = turbine(S, s.eng, 2.0 * c_thr, mach, at.densalt, at.T, at.sigma, burn);
  // aerodynamics: one segment search per shared grid
  double i2v = 0.5 * ivt;                       // 1 / (2 vt), 0 at rest
  double b2v = 30.0 * i2v, c2v = 11.32 * i2v;
  Seg sa = seg_find(S, F16T_ALPHA, 12, al);
  Seg se = seg_find(S, F16T_GRID_ELEV, F16N_GRID_ELEV, sf.ele);
  Seg sb13 = seg_find(S, F16T_GRID_BETA13, F16N_GRID_BETA13, be);
  Seg sb7 = seg_find(S, F16T_GRID_BETA7, F16N_GRID_BETA7, be);
  const double kge = S[F16T_KCLGE_Y + F16N_KCLGE_Y - 1];      // KCLGE(765 ft) is past the table end
  // the nine Mach tables share one search on the union of their grids (resampled copies,
  // F16T_MU_*: the same piecewise-linear functions)
  Seg sm = seg_find(S, F16T_MACHU, F16N_MACHU, mach);
#define A1(nm) lut1s(S, F16T_##nm, 12, sa)
#define M1(nm, n) lut1s(S, F16T_MU_##nm, F16N_MACHU, sm)
  double k = qbar * 300.0;
  double ssum;
  ssum = 0.0;
  ssum += k * lut2s(S, F16T_CDDH, F16N_GRID_ELEV, sa, se);
  ssum += k * M1(CDMACH, 4);
  ssum += k * sf.lef * A1(CDDLEF);
  ssum += k * sf.flap * 0.08;
  ssum += k * sf.gear * 0.027;
  ssum += k * q * c2v * A1(CDQ);
  ssum += k * q * c2v * sf.lef * A1(CDQ_DLEF);
  double DR = ssum;
  ssum = 0.0;
  ssum += k * be * -1.146;
  ssum += k * be * M1(CYB_M, 3);
  ssum += k * sf.ail * -0.0226;
  ssum += k * sf.rud * 0.086;
  ssum += k * b2v * p * A1(CYP);
  ssum += k * b2v * r * A1(CYR);
  double SI = ssum;
  ssum = 0.0;
  ssum += k * kge * lut2s(S, F16T_CLDH, F16N_GRID_ELEV, sa, se);
  ssum += k * sf.lef * kge * A1(CLDLEF);
  ssum += k * sf.flap * kge * 0.35;
  ssum += k * q * kge * c2v * A1(CLQ);
  double LI = ssum;
  double kb = k * 30.0, kc = k * 11.32;
  ssum = 0.0;
  ssum += kb * lut2s(S, F16T_CLB, F16N_GRID_BETA13, sa, sb13);
  ssum += kb * be * M1(CLB_M, 6);
  ssum += kb * b2v * p * A1(CLP);
  ssum += kb * b2v * r * A1(CLR);
  ssum += kb * sf.ail * lut2s(S, F16T_CLDA, F16N_GRID_BETA7, sa, sb7);
  ssum += kb * al * sf.ail * M1(CLDA_M, 3);
  ssum += kb * al * sf.rud * M1(CLDR_M, 2);
  ssum += kb * sf.rud * lut2s(S, F16T_CLDR, F16N_GRID_BETA7, sa, sb7);
  double RO = ssum;
  ssum = 0.0;
  ssum += kc * lut2s(S, F16T_CMDH, F16N_GRID_ELEV, sa, se);
  ssum += kc * al * M1(CMA_M, 6);
  ssum += kc * c2v * q * A1(CMQ);
  double PI_ = ssum;
  ssum = 0.0;
  ssum += kb * lut2s(S, F16T_CNB, F16N_GRID_BETA13, sa, sb13);
  ssum += kb * be * M1(CNB_M, 8);
  ssum += kb * b2v * p * A1(CNP);
  ssum += kb * b2v * r * A1(CNR);
  ssum += kb * sf.ail * M1(CNDA_M, 6);
  ssum += kb * sf.ail * lut2s(S, F16T_CNDA, F16N_GRID_BETA7, sa, sb7);
  ssum += kb * sf.rud * lut2s(S, F16T_CNDR, F16N_GRID_BETA7, sa, sb7);
  ssum += kb * al * sf.rud * M1(CNDR_M, 3);
  double YA = ssum;
#undef A1
#undef M1
  // wind -> body (fdm.cuh:592-598); sin/cos of alpha and beta from the body velocity
  double ca, sa_, cb, sb;
  if (al == 0.0) { ca = 1.0; sa_ = 0.0; } else { ca = u * isuw; sa_ = w * isuw; }
  if (be == 0.0) { cb = 1.0; sb = 0.0; } else { cb = suw * ivt; sb = v * ivt; }
  double drag = -DR, side = SI, lift = -LI;
  double Fx = ca * cb * drag + (-ca * sb) * side + (-sa_) * lift;
  double Fy = sb * drag + cb * side;
  double Fz = sa_ * cb * drag + (-sa_ * sb) * side + ca * lift;
  // moments about the cg: r x F with r = (rpx, 0, rpz); engine moment (0, rz*thrust, 0)
  double rz_e = F16C_INCHTOFT * mp.cgz;
  double Mx = RO + (0.0 * Fz - mp.rpz * Fy);
  double My = PI_ + (mp.rpz * Fx - mp.rpx * Fz) + rz_e * thrust;
  double Mz = YA + (mp.rpx * Fy - 0.0 * Fx);
  double F0 = Fx + thrust;
  // J2 gravity directly in ECI (fdm.cuh:155-171 rotated back by Tec2i)
  double ar = F16C_SEMI_MAJOR * irad;
  double pc = 1.5 * F16C_J2const * ar * ar;
  double kxy = 1.0 - 5.0 * (sla * sla), kz = 3.0 - 5.0 * (sla * sla);
  double g = F16C_GM * irad * irad;
  double gx = -g * ((1.0 + pc * kxy) * px * irad);
  double gy = -g * ((1.0 + pc * kxy) * py * irad);
  double gz = -g * ((1.0 + pc * kz) * pz * irad);
  // accelerations (fdm.cuh:499-517)
  double wi0 = p + T02 * ROT, wi1 = q + T12 * ROT, wi2 = r + T22 * ROT;      // body rates incl. earth
  double Jw0 = mp.Ixx * wi0 - mp.Ixz * wi2, Jw1 = mp.Iyy * wi1, Jw2 = -mp.Ixz * wi0 + mp.Izz * wi2;
  double m0 = Mx - (wi1 * Jw2 - wi2 * Jw1);
  double m1 = My - (wi2 * Jw0 - wi0 * Jw2);
  double m2 = Mz - (wi0 * Jw1 - wi1 * Jw0);
  double pdd0 = mp.k1 * m0 + mp.k3 * m2;
  double pdd1 = mp.k4 * m1;
  double pdd2 = mp.k3 * m0 + mp.k6 * m2;
  double ba0 = F0 * mp.inv_mass, ba1 = Fy * mp.inv_mass, ba2 = Fz * mp.inv_mass;
  s.uvwidot[0] = T00 * ba0 + T10 * ba1 + T20 * ba2 + gx;
  s.uvwidot[1] = T01 * ba0 + T11 * ba1 + T21 * ba2 + gy;
  s.uvwidot[2] = T02 * ba0 + T12 * ba1 + T22 * ba2 + gz;
  s.pqridot[0] = pdd0; s.pqridot[1] = pdd1; s.pqridot[2] = pdd2;
  s.fuel -= burn;
  {
    const double ba[3] = {ba0, ba1, ba2}, pdd[3] = {pdd0, pdd1, pdd2}, wi[3] = {wi0, wi1, wi2};
    load_factor(s.fuel, ba, pdd, wi, s.nld);
    if (WANT_OUT) {
#pragma unroll
      for (int i = 0; i < 3; i++) { s.pbacc[i] = ba[i]; s.ppqridot[i] = pdd[i]; s.ppqri[i] = wi[i]; }
    }
  }
  s.pa[0] = al; s.pa[1] = mach; s.pa[2] = vc; s.pa[3] = vg;
  s.pa[4] = npy; s.pa[5] = npz; s.pa[6] = p; s.pa[7] = q; s.pa[8] = r;
  if (WANT_OUT) {
    out.alpha = al; out.beta = be; out.mach = mach; out.vt = vt; out.alt = alt;
  }
}

}  // namespace f16
