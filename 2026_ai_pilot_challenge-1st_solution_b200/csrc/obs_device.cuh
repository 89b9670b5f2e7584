// obs_device.cuh -- fused 184-D observation / final-safe reward / termination, device side.
//
// Semantics: the reference's fused kernels research/competition_36500/runtime/cuda_fdm/gen/
// obs_kernel.cu (kin9 :96-145, geometry :148-330, build_obs_one :336-482, init_reward_kernel
// :485-501, advance_kernel :504-626, build_obs_kernel :628-649).  Organisation for B200: one
// thread per ENVIRONMENT handles both aircraft, so the two 9-DoF states are built once and
// everything the two perspectives share is computed once:
//   * body matrices R_o, R_p (ned2body of each aircraft) -- 2 instead of 8+ evaluations;
//   * the line of sight u = (p - o)/|p - o| and its body projections v_o = R_o u,
//     v_p = R_p (-u): ATA, LOS azimuth/elevation of one side and aspect of the other side are
//     all read from these two vectors;
//   * NED velocities, their direction frames (also the bank-angle frames) and the LOS frames.
// Arithmetic is fp64 throughout (observations are rounded to fp32 at the store, as STORE does).
#pragma once
#include <stdint.h>
#include "../../include/f16env.h"

namespace f16 {
namespace obs {

constexpr double D2R = 0.017453292519943295;
constexpr double R2D = 57.29577951308232;
constexpr double PI2 = 6.283185307179586;
constexpr double FT2M = 0.3048;
constexpr double M2FT = 3.28084;
constexpr double SLR_FT = 20925646.32546;
constexpr double ROT = 7.292115e-5;
constexpr double WA = 6378137.0;
constexpr double WE2 = 0.0066943799901411;
// observation constants (R/claude_code/my_observation.py:97-149)
constexpr double MAX_SPEED = 600.0, MAX_RANGE_M = 2500.0, MAX_CLOSURE = 1000.0, VSPEED_SCALE = 100.0;
constexpr double PQR_SCALE = 4.0, AOA_SCALE = 30.0, SSLIP_SCALE = 15.0, MIN_ALT_M = 304.8, ALT_DANGER = 300.0;
constexpr double MAX_ALT_M = 15000.0, ENERGY_ADV = 5000.0, PURSUIT_ATA = 30.0, PURSUIT_RANGE = 3000.0;
constexpr double FUEL_BURN = 8.0e-5, FUEL_REF = 300.0, REL_VEL = 600.0, GACC = 9.80665, EPISODE_MAX = 200.0;
constexpr double TLIM_TOL = 1.0e-8;
// damage cones (my_observation.py damage tiers)
constexpr double MIN_DMG_R_FT = 500.0, T1_MAX = 3000.0, T2_MAX = 3500.0, T3_MAX = 4000.0;
constexpr double T1_CONE = 1.0, T2_CONE = 2.0, T3_CONE = 3.0, T2_START = 100.0, T3_START = 150.0;
// final-safe reward (obs_kernel.cu:48-52)
constexpr double GEOM_BUDGET = 5.0, GEOM_REF_SEC = 200.0, SHAPING_BASE = 0.0001;
constexpr double ALT_LOG_SCALE_M = 304.8, ALT_LOG_FLOOR = 1.0e-4;

struct M3 {
  double m[3][3];
};
struct V3 {
  double x, y, z;
};

__device__ __forceinline__ double clampd(double x, double a, double b) { return x < a ? a : (x > b ? b : x); }
__device__ __forceinline__ double nrm(const V3& v) { return sqrt(v.x * v.x + v.y * v.y + v.z * v.z); }
__device__ __forceinline__ V3 mv(const M3& A, const V3& v) {
  return {A.m[0][0] * v.x + A.m[0][1] * v.y + A.m[0][2] * v.z, A.m[1][0] * v.x + A.m[1][1] * v.y + A.m[1][2] * v.z,
          A.m[2][0] * v.x + A.m[2][1] * v.y + A.m[2][2] * v.z};
}
__device__ __forceinline__ V3 mvT(const M3& A, const V3& v) {
  return {A.m[0][0] * v.x + A.m[1][0] * v.y + A.m[2][0] * v.z, A.m[0][1] * v.x + A.m[1][1] * v.y + A.m[2][1] * v.z,
          A.m[0][2] * v.x + A.m[1][2] * v.y + A.m[2][2] * v.z};
}


// Out-of-line calls of the library's fp64 sincos / atan2 / acos / asin / exp / log and fp32
// tanhf.  Inlined, each call site carries the function's whole body, rarely taken branches
// included; the row builder has dozens of sites, and with one body per function its code
// shrinks enough to cut the instruction-fetch stalls that dominated it (k_obs_step -15%, same
// results bit for bit).  The values are the library functions' own.
static __device__ __noinline__ double2 sincos_ool(double x) {
  double s, c;
  sincos(x, &s, &c);
  return make_double2(s, c);
}
static __device__ __noinline__ double atan2_ool(double y, double x) { return atan2(y, x); }
static __device__ __noinline__ double acos_ool(double x) { return acos(x); }
static __device__ __noinline__ double asin_ool(double x) { return asin(x); }
static __device__ __noinline__ double exp_ool(double x) { return exp(x); }
static __device__ __noinline__ double log_ool(double x) { return log(x); }
static __device__ __noinline__ float tanhf_ool(float x) { return tanhf(x); }

// R_ned_to_body = Tx(roll) Ty(pitch) Tz(yaw), angles in degrees (obs_kernel.cu:75-84)
// sc (optional) receives sin/cos of roll, pitch, yaw -- the attitude observation features.
__device__ __forceinline__ M3 ned2body(double roll, double pitch, double yaw, double* sc = nullptr) {
  double sr, cr, sp, cp, sy, cy;
  { const double2 t = sincos_ool(roll * D2R); sr = t.x; cr = t.y; }
  { const double2 t = sincos_ool(pitch * D2R); sp = t.x; cp = t.y; }
  { const double2 t = sincos_ool(yaw * D2R); sy = t.x; cy = t.y; }
  if (sc) {
    sc[0] = sr; sc[1] = cr; sc[2] = sp; sc[3] = cp; sc[4] = sy; sc[5] = cy;
  }
  M3 R;
  R.m[0][0] = cp * cy; R.m[0][1] = cp * sy; R.m[0][2] = -sp;
  R.m[1][0] = sr * sp * cy - cr * sy; R.m[1][1] = sr * sp * sy + cr * cy; R.m[1][2] = sr * cp;
  R.m[2][0] = cr * sp * cy + sr * sy; R.m[2][1] = cr * sp * sy - sr * cy; R.m[2][2] = cr * cp;
  return R;
}

// ned2body from the sin/cos of roll, pitch, yaw (sc as ned2body writes them)
__device__ __forceinline__ M3 ned2body_sc(const double* sc) {
  const double sr = sc[0], cr = sc[1], sp = sc[2], cp = sc[3], sy = sc[4], cy = sc[5];
  M3 R;
  R.m[0][0] = cp * cy; R.m[0][1] = cp * sy; R.m[0][2] = -sp;
  R.m[1][0] = sr * sp * cy - cr * sy; R.m[1][1] = sr * sp * sy + cr * cy; R.m[1][2] = sr * cp;
  R.m[2][0] = cr * sp * cy + sr * sy; R.m[2][1] = cr * sp * sy - sr * cy; R.m[2][2] = cr * cp;
  return R;
}

struct Origin {
  double ox, oy, oz, sl, cl, so, co;
};

// FDM state row -> official 9-DoF: N, E (tangent plane about the official origin, from the
// geodetic position at MSL altitude), D = -MSL; roll/pitch/yaw deg; body u, v, w m/s.
// sin/cos of atan2(y, x) without the angle: (y, x) / hypot(x, y); at the origin the angle is
// atan2's signed-zero result, taken the long way (never on a real state).
__device__ __forceinline__ void sincos_atan2(double y, double x, double* s, double* c) {
  const double h = sqrt(x * x + y * y);
  if (h > 0.0) {
    const double ih = 1.0 / h;
    *s = y * ih;
    *c = x * ih;
  } else {
    const double2 t = sincos_ool(atan2_ool(y, x));
    *s = t.x;
    *c = t.y;
  }
}

// sc (optional) receives sin/cos of roll, pitch, yaw (the attitude features and the inputs of
// ned2body_sc), from the same matrix elements the angles come from: sin/cos(atan2(y, x)) =
// (y, x) / hypot and cos(asin(-z)) = sqrt(1 - z^2) -- identities, rounding-level differences
// from the reference's sin/cos of the degree values.
template <typename Row>
__device__ __forceinline__ void kin9(const Row& st, const Origin& O, double s9[9], double* sc = nullptr) {
  double px = st(0), py = st(1), pz = st(2), vx = st(3), vy = st(4), vz = st(5);
  double q0 = st(6), q1 = st(7), q2 = st(8), q3 = st(9), epa = st(13);
  double se, ce;
  sincos(epa, &se, &ce);
  double ex = ce * px + se * py, ey = -se * px + ce * py, ez = pz;
  double rxy = sqrt(ex * ex + ey * ey);
  double radius = sqrt(ex * ex + ey * ey + ez * ez);
  double sLa = ez / radius, cLa = rxy / radius, sLo = ey / rxy, cLo = ex / rxy;
  // local NED axes in ECI: Tl2i = Tec2i * Tl2ec
  double N0 = -cLo * sLa, N1 = -sLo * sLa, N2 = cLa;
  double E0 = -sLo, E1 = cLo;
  double D0 = -cLo * cLa, D1 = -sLo * cLa, D2 = -sLa;
  double Ni0 = ce * N0 - se * N1, Ni1 = se * N0 + ce * N1;
  double Ei0 = ce * E0 - se * E1, Ei1 = se * E0 + ce * E1;
  double Di0 = ce * D0 - se * D1, Di1 = se * D0 + ce * D1;
  double a0 = q0 * q0, a1 = q1 * q1, a2 = q2 * q2, a3 = q3 * q3;
  double b01 = q0 * q1, b02 = q0 * q2, b03 = q0 * q3, b12 = q1 * q2, b13 = q1 * q3, b23 = q2 * q3;
  double T00 = a0 + a1 - a2 - a3, T01 = 2.0 * (b12 + b03), T02 = 2.0 * (b13 - b02);
  double T10 = 2.0 * (b12 - b03), T11 = a0 - a1 + a2 - a3, T12 = 2.0 * (b23 + b01);
  double T20 = 2.0 * (b13 + b02), T21 = 2.0 * (b23 - b01), T22 = a0 - a1 - a2 + a3;
  double L00 = T00 * Ni0 + T01 * Ni1 + T02 * N2;
  double L01 = T00 * Ei0 + T01 * Ei1;
  double L02 = T00 * Di0 + T01 * Di1 + T02 * D2;
  double L12 = T10 * Di0 + T11 * Di1 + T12 * D2;
  double L22 = T20 * Di0 + T21 * Di1 + T22 * D2;
  double theta = asin_ool(-clampd(L02, -1.0, 1.0));
  double phi = atan2_ool(L12, L22);
  double psi = atan2_ool(L01, L00);
  if (sc) {
    sincos_atan2(L12, L22, &sc[0], &sc[1]);
    const double sp = -clampd(L02, -1.0, 1.0);
    sc[2] = sp;
    sc[3] = sqrt(fmax(0.0, (1.0 - sp) * (1.0 + sp)));
    sincos_atan2(L01, L00, &sc[4], &sc[5]);
  }
  if (psi < 0.0) psi += PI2;
  double dv0 = vx + ROT * py, dv1 = vy - ROT * px, dv2 = vz;
  double u = T00 * dv0 + T01 * dv1 + T02 * dv2;
  double v = T10 * dv0 + T11 * dv1 + T12 * dv2;
  double w = T20 * dv0 + T21 * dv1 + T22 * dv2;
  double alt_m = (radius - SLR_FT) * FT2M;
  // closed-form geodetic latitude (obs_kernel.cu:127-133), then back to ECEF at MSL altitude
  double exm = ex * FT2M, eym = ey * FT2M, ezm = ez * FT2M;
  const double b = WA * 0.99664718933525254;        // WA * sqrt(1 - WE2)
  const double ep2 = (WA * WA - b * b) / (b * b);
  double pxy = sqrt(exm * exm + eym * eym);
  double sth, cth;
  sincos_atan2(ezm * WA, pxy * b, &sth, &cth);
  double slat, clat;                                // of lat = atan2(num, den)
  sincos_atan2(ezm + ep2 * b * (sth * sth * sth), pxy - WE2 * WA * (cth * cth * cth), &slat, &clat);
  double ir = 1.0 / pxy;
  double slon = eym * ir, clon = exm * ir;          // sin/cos of atan2(eym, exm)
  double Nr = WA / sqrt(1.0 - WE2 * slat * slat);
  double hx = (Nr + alt_m) * clat * clon, hy = (Nr + alt_m) * clat * slon, hz = (Nr * (1.0 - WE2) + alt_m) * slat;
  double dx = hx - O.ox, dy = hy - O.oy, dz = hz - O.oz;
  s9[0] = -O.sl * O.co * dx - O.sl * O.so * dy + O.cl * dz;
  s9[1] = -O.so * dx + O.co * dy;
  s9[2] = -alt_m;
  s9[3] = phi * R2D;
  s9[4] = theta * R2D;
  s9[5] = psi * R2D;
  s9[6] = u * FT2M;
  s9[7] = v * FT2M;
  s9[8] = w * FT2M;
}

// frame whose x axis is along x with roll fixed by gravity (obs_kernel.cu:179-203)
__device__ __forceinline__ M3 dir_frame(const V3& x) {
  M3 R;
  double nx = nrm(x);
  if (nx < 1e-8) {
    R.m[0][0] = 1; R.m[0][1] = 0; R.m[0][2] = 0;
    R.m[1][0] = 0; R.m[1][1] = 1; R.m[1][2] = 0;
    R.m[2][0] = 0; R.m[2][1] = 0; R.m[2][2] = 1;
    return R;
  }
  const double ix = 1.0 / nx;
  V3 xn = {x.x * ix, x.y * ix, x.z * ix};
  // reference order: down (0,0,1), then north (1,0,0), then east (0,1,0)
  V3 z = {-xn.z * xn.x, -xn.z * xn.y, 1.0 - xn.z * xn.z};
  if (nrm(z) < 1e-6) {
    z = {1.0 - xn.x * xn.x, -xn.x * xn.y, -xn.x * xn.z};
    if (nrm(z) < 1e-6) z = {-xn.y * xn.x, 1.0 - xn.y * xn.y, -xn.y * xn.z};
  }
  const double iz = 1.0 / nrm(z);
  z = {z.x * iz, z.y * iz, z.z * iz};
  V3 y = {z.y * xn.z - z.z * xn.y, z.z * xn.x - z.x * xn.z, z.x * xn.y - z.y * xn.x};
  const double iy = 1.0 / nrm(y);
  y = {y.x * iy, y.y * iy, y.z * iy};
  z = {xn.y * y.z - xn.z * y.y, xn.z * y.x - xn.x * y.z, xn.x * y.y - xn.y * y.x};
  R.m[0][0] = xn.x; R.m[0][1] = xn.y; R.m[0][2] = xn.z;
  R.m[1][0] = y.x; R.m[1][1] = y.y; R.m[1][2] = y.z;
  R.m[2][0] = z.x; R.m[2][1] = z.y; R.m[2][2] = z.z;
  return R;
}

__device__ __forceinline__ double normz(double x, double lo, double hi) {
  double mid = (hi + lo) * 0.5, half = (hi - lo) * 0.5;
  return (clampd(x, lo, hi) - mid) / half;
}
__device__ __forceinline__ double damage(double r_ft, double ata_abs, double t) {
  double a = fabs(ata_abs);
  if (r_ft >= MIN_DMG_R_FT && r_ft <= T1_MAX && a < T1_CONE) return 1.0 * (T1_MAX - r_ft) / (T1_MAX - MIN_DMG_R_FT);
  if (t >= T2_START && r_ft >= MIN_DMG_R_FT && r_ft <= T2_MAX && a < T2_CONE)
    return 0.3 * (T2_MAX - r_ft) / (T2_MAX - MIN_DMG_R_FT);
  if (t >= T3_START && r_ft >= MIN_DMG_R_FT && r_ft <= T3_MAX && a < T3_CONE)
    return 0.1 * (T3_MAX - r_ft) / (T3_MAX - MIN_DMG_R_FT);
  return 0.0;
}
__device__ __forceinline__ double smooth3(double x, double a, double b) {
  double z = clampd((x - a) / (b - a), 0.0, 1.0);
  return z * z * (3.0 - 2.0 * z);
}
__device__ __forceinline__ V3 unit_or(const V3& v, const V3& fb) {
  double n = nrm(v);
  V3 s = v;
  if (!(n >= 1e-9) || !isfinite(n)) {
    s = fb;
    n = nrm(fb);
  }
  if (!(n >= 1e-9) || !isfinite(n)) return {1.0, 0.0, 0.0};
  const double in = 1.0 / n;
  return {s.x * in, s.y * in, s.z * in};
}
__device__ __forceinline__ double align3(const V3& a, const V3& b) {
  V3 au = unit_or(a, {1.0, 0.0, 0.0});
  V3 bu = unit_or(b, au);
  double q = 0.5 * (1.0 + clampd(au.x * bu.x + au.y * bu.y + au.z * bu.z, -1.0, 1.0));
  return clampd(q * q * q, 0.0, 1.0);
}
__device__ __forceinline__ double safe_lead(const V3& rel, const V3& ov, const V3& tv, const V3& fwd, double dist_m,
                                            double dist_ft, double ata) {
  V3 los = unit_or(rel, fwd);
  V3 path = unit_or(ov, fwd);
  double spd = nrm(ov);
  if (spd < 30.0) spd = 30.0;
  double tau = clampd(dist_m / spd, 0.30, 1.50);
  V3 lv = {rel.x + tv.x * tau, rel.y + tv.y * tau, rel.z + tv.z * tau};
  V3 lead = unit_or(lv, los);
  double intercept = 0.40 * align3(fwd, lead) + 0.60 * align3(path, lead);
  double direct = align3(fwd, los);
  double w = smooth3(dist_ft, 1000.0, 2500.0) * smooth3(fabs(ata), 3.0, 8.0);
  return clampd(w * intercept + (1.0 - w) * direct, 0.0, 1.0);
}
__device__ __forceinline__ double broad(double ata) {
  ata = clampd(fabs(ata), 0.0, 180.0);
  return (ata <= 30.0) ? 1.0 : clampd((180.0 - ata) / 150.0, 0.0, 1.0);
}
__device__ __forceinline__ double side_score(const V3& rel, const V3& ov, const V3& tv, const V3& fwd, double dist_m,
                                             double dist_ft, double ata, double t, double rg, double cq) {
  double lead = safe_lead(rel, ov, tv, fwd, dist_m, dist_ft, ata);
  double gate = 1.0 - smooth3(fabs(ata), 3.0, 8.0);
  double control = clampd(gate * rg * cq, 0.0, 1.0);
  double fine = damage(dist_ft, fabs(ata), t);
  return clampd(0.50 * broad(ata) + 0.20 * lead + 0.20 * control + 0.10 * fine, 0.0, 1.0);
}
__device__ __forceinline__ double alt_log(double alt_m) {
  double s = alt_m / ALT_LOG_SCALE_M;
  return log_ool(s < ALT_LOG_FLOOR ? ALT_LOG_FLOOR : s);
}
__device__ __forceinline__ void log_so3(const M3& R, double inv_dt, double out[3]) {
  double tr = R.m[0][0] + R.m[1][1] + R.m[2][2];
  const double c = clampd((tr - 1.0) * 0.5, -1.0, 1.0);
  double theta = acos_ool(c);
  double den = 2.0 * sqrt((1.0 - c) * (1.0 + c)), sc = 0.0;     // 2 sin(acos c)
  if (theta >= 1e-8 && fabs(den) >= 1e-8) sc = theta / den;
  out[0] = (R.m[2][1] - R.m[1][2]) * sc * inv_dt;
  out[1] = (R.m[0][2] - R.m[2][0]) * sc * inv_dt;
  out[2] = (R.m[1][0] - R.m[0][1]) * sc * inv_dt;
}
// The reference's STORE (obs_kernel.cu:331-333): a non-finite double becomes +-10 / 0, then the
// value is rounded to fp32 (a finite double past the float range stays infinite).  The rounded
// value is tested first, so the double is only inspected on the rare non-finite path.
__device__ __forceinline__ float store_val(double v) {
  float f = (float)v;
  if (!isfinite(f) && !isfinite(v)) f = (v > 0.0) ? 10.0f : ((v < 0.0) ? -10.0f : 0.0f);
  return f;
}
__device__ __forceinline__ float store_f(float f) {
  return isfinite(f) ? f : ((f > 0.0f) ? 10.0f : ((f < 0.0f) ? -10.0f : 0.0f));
}

// ---------------- lane-pair organisation ----------------
// One thread per AIRCRAFT: the two aircraft of environment e are the adjacent lanes a = 2e and
// a = 2e + 1 (k = a & 1) of one warp.  Each lane builds its own aircraft's geometry once and
// stages it in shared memory, field-major [field][thread], where the partner lane reads it (a
// warp reads 32 consecutive doubles of one field: no bank conflicts); the per-lane register
// set is then one aircraft's working values, not an engagement's.  Values the reference
// computes once per environment from side 0's view (LOS delta, range, geometry-advantage
// quality terms) are computed by both lanes from the same operands in the same order, and side
// 1 takes the exact negations the reference takes (md = -delta, mu = -u), so both lanes hold
// the reference's bits.  Partner values that are read before they are overwritten (old HP,
// tracker validity, previous altitude log) travel by shuffle, never through memory.
enum StageField : int {
  F_S = 0,       // 9-DoF: N, E, D (m), roll, pitch, yaw (deg), u, v, w (m/s)
  F_R = 9,       // ned2body, row-major
  F_ATT = 18,    // sin/cos of roll, pitch, yaw
  F_VN = 24,     // NED velocity
  F_SPD = 27,    // |body velocity|
  F_FV = 28,     // dir_frame(NED velocity), row-major
  F_FL = 37,     // dir_frame(line of sight from this aircraft to the other)
  F_PROJ = 46,   // body-frame unit line of sight to the other aircraft
  F_ATA = 49,    // ATA at the other aircraft (deg)
  F_HP = 50,     // reconstruction values of the row: HP, fuel (the damage rates, read by the
                 // own lane only, are passed to obs_row as arguments)
  F_FUEL = 51,
  F_PQR = 52,    // body rates from the attitude change
  NFIELD = 55
};

template <int T>
struct Lanes {
  double* sm;     // the block's staging array, NFIELD x T
  int i;          // threadIdx.x
  unsigned pm;    // the pair's lane mask
  __device__ __forceinline__ double& own(int f) const { return sm[f * T + i]; }
  __device__ __forceinline__ double par(int f) const { return sm[f * T + (i ^ 1)]; }
  // aircraft c (0: even, 1: odd) of the pair
  __device__ __forceinline__ double col(int f, int c) const { return sm[f * T + ((i & ~1) | c)]; }
  __device__ __forceinline__ V3 vec(int f, int c) const { return {col(f, c), col(f + 1, c), col(f + 2, c)}; }
  __device__ __forceinline__ M3 mat(int f, int c) const {
    M3 M;
#pragma unroll
    for (int r = 0; r < 3; r++)
#pragma unroll
      for (int q = 0; q < 3; q++) M.m[r][q] = col(f + 3 * r + q, c);
    return M;
  }
  __device__ __forceinline__ void put_vec(int f, const V3& v) const { own(f) = v.x; own(f + 1) = v.y; own(f + 2) = v.z; }
  __device__ __forceinline__ void put_mat(int f, const M3& M) const {
#pragma unroll
    for (int r = 0; r < 3; r++)
#pragma unroll
      for (int q = 0; q < 3; q++) own(f + 3 * r + q) = M.m[r][q];
  }
  __device__ __forceinline__ void sync() const { __syncwarp(pm); }
  __device__ __forceinline__ double xchg(double v) const { return __shfl_xor_sync(pm, v, 1); }
  __device__ __forceinline__ int xchg(int v) const { return __shfl_xor_sync(pm, v, 1); }
};

// Own aircraft: 9-DoF, body matrix and attitude sin/cos, NED velocity, speed, velocity frame.
// The current body matrix is built from the attitude sin/cos kin9 derives from the matrix
// elements (no sincos); the previous one (ned2body of the stored degrees, as the reference)
// only when prev is given: the aircraft's previous attitude when its history is valid, else
// NULL; with it the body rates log_SO3(R_prev R^T) / dt of advance_kernel are staged in F_PQR
// (zero without).
template <int T, typename Row>
__device__ __forceinline__ void stage_aircraft(const Lanes<T>& L, const Row& row, const Origin& O,
                                               const double* prev = nullptr, double inv_dt = 0.0) {
  double s[9], att[6];
  kin9(row, O, s, att);
#pragma unroll
  for (int j = 0; j < 9; j++) L.own(F_S + j) = s[j];
#pragma unroll
  for (int j = 0; j < 6; j++) L.own(F_ATT + j) = att[j];
  const M3 R = ned2body_sc(att);
  L.put_mat(F_R, R);
  const V3 vb = {s[6], s[7], s[8]};
  const V3 vn = mvT(R, vb);
  L.put_vec(F_VN, vn);
  L.own(F_SPD) = nrm(vb);
  L.put_mat(F_FV, dir_frame(vn));
  double lg[3] = {0.0, 0.0, 0.0};
  if (prev) {
    const M3 Np = ned2body(prev[0], prev[1], prev[2]);
    M3 rd;
    for (int i = 0; i < 3; i++)
      for (int j = 0; j < 3; j++)
        rd.m[i][j] = Np.m[i][0] * R.m[j][0] + Np.m[i][1] * R.m[j][1] + Np.m[i][2] * R.m[j][2];
    log_so3(rd, inv_dt, lg);
  }
  L.put_vec(F_PQR, V3{lg[0], lg[1], lg[2]});
}

// The pair's line of sight from side 0 (reference P.delta, P.dist, P.u): identical on both lanes.
struct Los {
  V3 d0;          // aircraft 1 - aircraft 0 (m)
  double dist;
  V3 u0;          // d0 / dist, zero when dist == 0
};

// After stage_aircraft on both lanes: the pair's LOS, and this aircraft's body-frame LOS, ATA
// and LOS frame staged (reference make_pair and the Fl frames of build_obs).
template <int T>
__device__ __forceinline__ Los stage_los(const Lanes<T>& L, int k) {
  Los g;
  g.d0 = {L.col(F_S, 1) - L.col(F_S, 0), L.col(F_S + 1, 1) - L.col(F_S + 1, 0), L.col(F_S + 2, 1) - L.col(F_S + 2, 0)};
  g.dist = nrm(g.d0);
  if (g.dist > 0.0) g.u0 = {g.d0.x / g.dist, g.d0.y / g.dist, g.d0.z / g.dist};
  else g.u0 = {0.0, 0.0, 0.0};
  const V3 d = k ? V3{-g.d0.x, -g.d0.y, -g.d0.z} : g.d0;
  const V3 u = k ? V3{-g.u0.x, -g.u0.y, -g.u0.z} : g.u0;
  const V3 pj = mv(L.mat(F_R, k), u);
  L.put_vec(F_PROJ, pj);
  L.own(F_ATA) = acos_ool(clampd(pj.x, -1.0, 1.0)) * R2D;
  L.put_mat(F_FL, dir_frame(d));
  return g;
}

// Symmetric geometry advantage (obs_kernel.cu:305-324) from this lane's side: G for side 0,
// -G for side 1.  Each lane scores its own side; the two scores meet by shuffle.
template <int T>
__device__ __forceinline__ double geometry_advantage(const Lanes<T>& L, int k, const Los& g, double t) {
  const double dm = g.dist, df = dm / FT2M;
  const V3 los = unit_or(g.d0, {1.0, 0.0, 0.0});
  const V3 vo = L.vec(F_VN, 0), vp = L.vec(F_VN, 1);
  const double closing = (vo.x - vp.x) * los.x + (vo.y - vp.y) * los.y + (vo.z - vp.z) * los.z;
  double ms = 0.5 * (nrm(vo) + nrm(vp));
  if (ms < 100.0) ms = 100.0;
  const double ratio = closing / ms;
  const double desired = 0.20 * smooth3(df, 2000.0, 4500.0) - 0.12 * (1.0 - smooth3(df, 650.0, 900.0));
  const double dq = (ratio - desired) / 0.15;
  const double cq = exp_ool(-0.5 * dq * dq);
  const double rg = smooth3(df, 600.0, 900.0) * (1.0 - smooth3(df, 3200.0, 4300.0));
  const V3 rel = k ? V3{-g.d0.x, -g.d0.y, -g.d0.z} : g.d0;
  const V3 fwd = {L.col(F_R + 0, k), L.col(F_R + 1, k), L.col(F_R + 2, k)};
  const double S = side_score(rel, k ? vp : vo, k ? vo : vp, fwd, dm, df, L.own(F_ATA), t, rg, cq);
  const double Sp = L.xchg(S);
  const double go = clampd((k ? Sp : S) - (k ? S : Sp), -1.0, 1.0);
  return k ? -go : go;
}

// 16-byte staged writer of one fp32 observation row
struct RowWriter {
  float* out;
  float buf[4];
  int n;
  __device__ __forceinline__ void push(float f) {
    buf[n & 3] = f;
    n++;
    if ((n & 3) == 0) reinterpret_cast<float4*>(out)[(n >> 2) - 1] = make_float4(buf[0], buf[1], buf[2], buf[3]);
  }
  // a feature computed in fp32: NaN -> 0, +-inf -> +-10
  __device__ __forceinline__ void putf(float f) {
    if (!isfinite(f)) f = (f > 0.0f) ? 10.0f : ((f < 0.0f) ? -10.0f : 0.0f);
    push(f);
  }
  // a feature computed in fp64, stored as the reference's STORE does
  __device__ __forceinline__ void put(double v) { push(store_val(v)); }
};

// normz with the constant half-range folded into a reciprocal: (clamp(x) - mid) / half as one
// multiply (1 ulp of fp64 at most; every feature is stored as fp32)
__device__ __forceinline__ double normz_k(double x, double lo, double hi) {
  return (clampd(x, lo, hi) - (hi + lo) * 0.5) * (2.0 / (hi - lo));
}

// The last 20 features (the action history, newest first): read from `hist`, zeros (a fresh
// episode), or already written by the history push.
enum HistMode : int { HIST_READ = 0, HIST_ZERO = 1, HIST_DONE = 2 };

// This lane's 184 features (obs_kernel.cu:336-482) after stage_aircraft, stage_los and the
// reconstruction fields are staged on both lanes; aux: the 21 future-position features or NULL.
template <int T>
__device__ __forceinline__ void obs_row(const Lanes<T>& L, int k, const Los& g, double t, int hist_mode,
                                       const double* hist, float* __restrict__ out, double* __restrict__ aux,
                                       double dealt, double taken) {
  const int o = k, p = 1 - k;
  const M3 Ro = L.mat(F_R, o);
  const V3 ovn = L.vec(F_VN, o), tvn = L.vec(F_VN, p);
  if (aux) {
    aux[0] = L.col(F_S, o); aux[1] = L.col(F_S + 1, o); aux[2] = L.col(F_S + 2, o);
    aux[3] = ovn.x; aux[4] = ovn.y; aux[5] = ovn.z;
    aux[6] = L.col(F_S, p); aux[7] = L.col(F_S + 1, p); aux[8] = L.col(F_S + 2, p);
    aux[9] = tvn.x; aux[10] = tvn.y; aux[11] = tvn.z;
    for (int i = 0; i < 3; i++)
      for (int j = 0; j < 3; j++) aux[12 + 3 * i + j] = Ro.m[i][j];
  }
  const double sg = (k == 0) ? 1.0 : -1.0;
  const V3 pl = (g.dist > 1e-6) ? g.u0 : V3{0.0, 0.0, 0.0};
  const V3 los = {sg * pl.x, sg * pl.y, sg * pl.z};
  const V3 rvn = {tvn.x - ovn.x, tvn.y - ovn.y, tvn.z - ovn.z};
  const double os = L.col(F_SPD, o), ts = L.col(F_SPD, p), oalt = -L.col(F_S + 2, o), talt = -L.col(F_S + 2, p);
  const double dist = g.dist;
  double clos = 0.0;
  if (dist > 1e-6) clos = (ovn.x - tvn.x) * los.x + (ovn.y - tvn.y) * los.y + (ovn.z - tvn.z) * los.z;
  const double ata = L.col(F_ATA, o), eata = L.col(F_ATA, p);
  // sin/cos of ATA, aspect, LOS azimuth and elevation straight from the body-frame LOS
  // projections (the reference takes acos/atan2/asin and then sin/cos of the result):
  //   ATA = acos(x)            -> cos = x, sin = sqrt(1 - x^2)        (ATA in [0,180])
  //   aspect = s*acos(-x')     -> cos = -x', sin = s*sqrt(1 - x'^2)   (s: sign rule below)
  //   az = atan2(y, x)         -> (y, x) / hypot(x, y)
  //   el = -asin(z)            -> sin = -z, cos = sqrt(1 - z^2)
  const V3 db = L.vec(F_PROJ, o);
  const double cx = clampd(db.x, -1.0, 1.0);
  const double s_ata = sqrt(fmax(0.0, (1.0 - cx) * (1.0 + cx))), c_ata = cx;
  const V3 bt = L.vec(F_PROJ, p);
  const double t0 = clampd(-bt.x, -1.0, 1.0), t1 = -bt.y, t2 = bt.z;
  const double asg = (t1 > 0.0) ? 1.0 : ((t1 < 0.0) ? -1.0 : ((t2 >= 0.0) ? 1.0 : -1.0));
  const double c_aa = t0, s_aa = asg * sqrt(fmax(0.0, (1.0 - t0) * (1.0 + t0)));
  const double hxy = sqrt(db.x * db.x + db.y * db.y);
  double c_az = 1.0, s_az = 0.0;
  if (hxy > 0.0) { c_az = db.x / hxy; s_az = db.y / hxy; }
  else if (db.x < 0.0 || (db.x == 0.0 && signbit(db.x))) { c_az = -1.0; }
  const double cz = clampd(db.z, -1.0, 1.0);
  const double s_el = -cz, c_el = sqrt(fmax(0.0, (1.0 - cz) * (1.0 + cz)));
  const double u = L.col(F_S + 6, o), v = L.col(F_S + 7, o), w = L.col(F_S + 8, o);
  float aoa = 0.0f, ss = 0.0f;
  if (os >= 1.0) {
    aoa = atan2f((float)w, (float)u) * (float)R2D;
    ss = atan2f((float)v, (float)sqrt(u * u + w * w)) * (float)R2D;
  }
  const double vs = -ovn.z;
  const double ea = (oalt + os * os / (2.0 * GACC)) - (talt + ts * ts / (2.0 * GACC));
  const double cone = (t >= T3_START) ? T3_CONE : ((t >= T2_START) ? T2_CONE : T1_CONE);
  const double mr = (t >= T3_START) ? T3_MAX : ((t >= T2_START) ? T2_MAX : T1_MAX);
  // bounded output nonlinearities in fp32 (each feature is stored as fp32)
  const float fa = (float)(ata * (1.0 / 3.0)), fe = (float)(eata * (1.0 / 3.0));
  const float ash = 2.0f * expf(-(fa * fa)) - 1.0f;
  const float amg = tanhf_ool((float)((cone - fabs(ata)) / cone));
  const float eash = 2.0f * expf(-(fe * fe)) - 1.0f;
  const float eamg = tanhf_ool((float)((cone - fabs(eata)) / cone));
  const double rmin = MIN_DMG_R_FT * FT2M, rmax = mr * FT2M, ispan = 1.0 / (rmax - rmin);
  const float rn = tanhf_ool((float)((dist - rmin) * ispan)), rf = tanhf_ool((float)((rmax - dist) * ispan));
  double pa = 1.0 - fabs(ata) / PURSUIT_ATA, pr = 1.0 - dist / PURSUIT_RANGE;
  if (pa < 0.0) pa = 0.0;
  if (pr < 0.0) pr = 0.0;
  const double me_hp = L.col(F_HP, o), th_hp = L.col(F_HP, p);
  RowWriter wr{out, {0, 0, 0, 0}, 0};
  wr.put(normz_k(os, 0.0, MAX_SPEED));
  wr.put(normz_k(ts, 0.0, MAX_SPEED));
  wr.putf(tanhf_ool(aoa * (float)(1.0 / AOA_SCALE)));
  wr.putf(tanhf_ool(ss * (float)(1.0 / SSLIP_SCALE)));
  wr.putf(tanhf_ool((float)((oalt - MIN_ALT_M) * (1.0 / ALT_DANGER))));
  wr.put(normz_k(vs, -VSPEED_SCALE, VSPEED_SCALE));
  wr.put(normz_k(me_hp, 0.0, 1.0));
  wr.put(normz_k(th_hp, 0.0, 1.0));
  wr.put(me_hp - th_hp);
  wr.put(ea / (fabs(ea) + ENERGY_ADV));
  wr.put(normz_k(dist, 0.0, MAX_RANGE_M));
  wr.put(normz_k(clos, -MAX_CLOSURE, MAX_CLOSURE));
  wr.put(s_ata); wr.put(c_ata);
  wr.put(s_aa); wr.put(c_aa);
  wr.put(s_az); wr.put(c_az);
  wr.put(s_el); wr.put(c_el);
  wr.putf(ash);
  wr.putf(amg);
  wr.putf(eash);
  wr.putf(eamg);
  wr.putf(rn);
  wr.putf(rf);
  wr.put(normz_k(t, 0.0, EPISODE_MAX));
  for (int i = 0; i < 6; i++) wr.put(L.col(F_ATT + i, o));     // sin/cos roll, pitch, yaw (own)
  for (int i = 0; i < 6; i++) wr.put(L.col(F_ATT + i, p));     // (target)
  // bank about the velocity vector: mu = atan2(y.z, y.y) of the body y axis (row 1 of R) in
  // the velocity frame; sin/cos(mu) = (y.z, y.y) / hypot
  for (int q = 0; q < 2; q++) {
    const int c = q == 0 ? o : p;
    const V3 by = {L.col(F_R + 3, c), L.col(F_R + 4, c), L.col(F_R + 5, c)};
    const V3 yv = mv(L.mat(F_FV, c), by);
    const double h = sqrt(yv.y * yv.y + yv.z * yv.z);
    if (h > 0.0) { wr.put(yv.z / h); wr.put(yv.y / h); }
    else { wr.put(yv.z); wr.put(signbit(yv.y) ? -1.0 : 1.0); }
  }
  wr.put(normz_k(L.col(F_FUEL, o), 0.0, 1.0));
  wr.put(normz_k(L.col(F_FUEL, p), 0.0, 1.0));
  wr.put(clampd(2.0 * dealt - 1.0, -1.0, 1.0));
  wr.put(clampd(2.0 * taken - 1.0, -1.0, 1.0));
  wr.put(2.0 * (pa * pr) - 1.0);
  wr.put(normz_k(oalt, 0.0, MAX_ALT_M));
  wr.put(normz_k(talt, 0.0, MAX_ALT_M));
  // 38 frame-projected vectors in VEC_LAYOUT order (obs_kernel.cu:457-464); frames by index:
  // 0 own body, 1 target body, 2 own velocity, 3 target velocity, 4 LOS
  const int cols = o | (p << 1) | (o << 2) | (p << 3) | (o << 4);      // staging column of frame f
  auto frame = [&](int f) -> M3 {
    const int base = f < 2 ? F_R : (f < 4 ? F_FV : F_FL);
    return L.mat(base, (cols >> f) & 1);
  };
  // gravity (0,0,1) in frames mybody, oppbody, myvel, oppvel, los  -> unit
#pragma unroll
  for (int f = 0; f < 5; f++) { V3 c = mv(frame(f), V3{0.0, 0.0, 1.0}); wr.put(c.x); wr.put(c.y); wr.put(c.z); }
  // los in frames world, mybody, oppbody, myvel, oppvel -> unit
  wr.put(los.x); wr.put(los.y); wr.put(los.z);
#pragma unroll
  for (int f = 0; f < 4; f++) { V3 c = mv(frame(f), los); wr.put(c.x); wr.put(c.y); wr.put(c.z); }
  // The remaining 84 features (80..163) start on a 16-byte boundary and come in items of one
  // vector in one frame (3 features); four items are 12 features = three float4 stores, so the
  // items run as a rolled loop over groups of four (compact code: this kernel is otherwise
  // bound by instruction fetch), with the source vector and frame of each item decoded from
  // its index.
  //   velocity items (features 80-127): own_vel in world, mybody, oppbody, oppvel, los;
  //   tgt_vel in world, mybody, oppbody, myvel, los; rel_vel in world and all five frames.
  //   Frame code 0 = world, f + 1 = frame f; 3 bits per item.
  //   omega items (features 128-163): own_omega then tgt_omega, each in world and frames 0-4.
  const V3 oom = mvT(Ro, L.vec(F_PQR, o)), tom = mvT(L.mat(F_R, p), L.vec(F_PQR, p));
  constexpr unsigned long long VEL_FRAMES =
      (0ull << 0) | (1ull << 3) | (2ull << 6) | (4ull << 9) | (5ull << 12) |
      (0ull << 15) | (1ull << 18) | (2ull << 21) | (3ull << 24) | (5ull << 27) |
      (0ull << 30) | (1ull << 33) | (2ull << 36) | (3ull << 39) | (4ull << 42) | (5ull << 45);
  float4* out4 = reinterpret_cast<float4*>(out);
  const double kv = 1.0 / REL_VEL;
  const float ip = (float)(1.0 / PQR_SCALE);
#pragma unroll 1
  for (int it = 0; it < 28; it += 4) {
    float v[12];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int item = it + j;
      const bool omega = item >= 16;
      int fc;
      V3 x;
      if (!omega) {
        fc = (int)((VEL_FRAMES >> (3 * item)) & 7);
        x = item < 5 ? ovn : (item < 10 ? tvn : rvn);
      } else {
        fc = (item - 16) % 6;
        x = item < 22 ? oom : tom;
      }
      const V3 c = fc == 0 ? x : mv(frame(fc - 1), x);
      if (!omega) {
        v[3 * j + 0] = store_val(clampd(c.x, -REL_VEL, REL_VEL) * kv);
        v[3 * j + 1] = store_val(clampd(c.y, -REL_VEL, REL_VEL) * kv);
        v[3 * j + 2] = store_val(clampd(c.z, -REL_VEL, REL_VEL) * kv);
      } else {
        v[3 * j + 0] = store_f(tanhf_ool((float)c.x * ip));
        v[3 * j + 1] = store_f(tanhf_ool((float)c.y * ip));
        v[3 * j + 2] = store_f(tanhf_ool((float)c.z * ip));
      }
    }
    const int q = (80 + 3 * it) >> 2;
#pragma unroll
    for (int j = 0; j < 3; j++) out4[q + j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  wr.n = 164;
  if (hist_mode == HIST_READ) {
    for (int j = 0; j < 20; j++) wr.put(hist[j]);
  } else if (hist_mode == HIST_ZERO) {
    for (int j = 0; j < 20; j++) wr.put(0.0);
  }
}

}  // namespace obs
}  // namespace f16
