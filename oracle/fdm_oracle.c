/*
 * fdm_oracle.c -- TEST INFRASTRUCTURE ONLY (the parity checker; never shipped or measured).
 *
 * Plain-C CPU restatement of the reference's JSBSim-v1.0.0 F-16 frame step and of its IC
 * seeding, written from the reference sources:
 *   frame step      cuda_fdm/gen/fdm.cuh:609-649 (fdm_step) and the functions it calls
 *   batch contract  cuda_fdm/gen/fdm_kernel.cu:32-47 (fdm_step_batch, obs17 columns)
 *   IC -> seed      cuda_fdm/ic.py:18-138 and cuda_fdm/ref/jsb_fdm.py:142-210 (FDM.seed)
 * The arithmetic keeps the reference's operation order, so compiled with the same flags
 * (-O2 -ffp-contract=off) it reproduces oracle/_ref (the reference header compiled as-is)
 * bit for bit; tests/test_oracle_fdm.py pins that.
 *
 * State rows are the reference's (nac,101) AoS layout (include/f16env.h F16_S_*).
 */
#include <math.h>
#include <string.h>
#include "../include/f16env.h"
#include "../2026_ai_pilot_challenge-1st_solution_b200/csrc/f16_tables.h"

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

static const double TAB[F16_TAB_LEN] = {F16_TAB_VALUES};
#define T(name) (TAB + F16T_##name)
#define DT_FRAME (1.0 / 60.0)           /* fdm.cuh:22 */
#define HB_MAC 765.0                    /* fdm.cuh:24 */
#define GEAR_FORCE 0.30                 /* fdm.cuh:25 */

/* ---------------- small helpers (fdm.cuh:28-47) ---------------- */
static double clampd(double x, double lo, double hi) { return x < lo ? lo : (x > hi ? hi : x); }
static double mx(double a, double b) { return a > b ? a : b; }
static void cross3(const double a[3], const double b[3], double o[3]) {
  o[0] = a[1] * b[2] - a[2] * b[1];
  o[1] = a[2] * b[0] - a[0] * b[2];
  o[2] = a[0] * b[1] - a[1] * b[0];
}
static void matvec(const double A[3][3], const double v[3], double o[3]) {
  for (int i = 0; i < 3; i++) o[i] = A[i][0] * v[0] + A[i][1] * v[1] + A[i][2] * v[2];
}
static void matmul(const double A[3][3], const double B[3][3], double O[3][3]) {
  for (int i = 0; i < 3; i++)
    for (int j = 0; j < 3; j++) O[i][j] = A[i][0] * B[0][j] + A[i][1] * B[1][j] + A[i][2] * B[2][j];
}
static void transp(const double A[3][3], double O[3][3]) {
  for (int i = 0; i < 3; i++)
    for (int j = 0; j < 3; j++) O[i][j] = A[j][i];
}

/* ---------------- FGTable lookups (fdm.cuh:50-79) ---------------- */
static double lookup1(const double* x, const double* y, int n, double key) {
  if (key <= x[0]) return y[0];
  if (key >= x[n - 1]) return y[n - 1];
  int r = 1;
  while (r < n - 1 && x[r] < key) r++;
  double span = x[r] - x[r - 1], f;
  if (span != 0.0) {
    f = (key - x[r - 1]) / span;
    if (f > 1.0) f = 1.0;
  } else {
    f = 1.0;
  }
  return f * (y[r] - y[r - 1]) + y[r - 1];
}
static double lookup2(const double* rx, int nr, const double* cx, int nc, const double* d,
                      double rk, double ck) {
  int r = 1, c = 1;
  while (r < nr - 1 && rx[r] < rk) r++;
  while (r > 1 && rx[r - 1] > rk) r--;
  while (c < nc - 1 && cx[c] < ck) c++;
  while (c > 1 && cx[c - 1] > ck) c--;
  double fr = clampd((rk - rx[r - 1]) / (rx[r] - rx[r - 1]), 0.0, 1.0);
  double fc = clampd((ck - cx[c - 1]) / (cx[c] - cx[c - 1]), 0.0, 1.0);
  double a0 = fr * (d[r * nc + c - 1] - d[(r - 1) * nc + c - 1]) + d[(r - 1) * nc + c - 1];
  double a1 = fr * (d[r * nc + c] - d[(r - 1) * nc + c]) + d[(r - 1) * nc + c];
  return a0 + fc * (a1 - a0);
}
#define TAB1_A(name, key) lookup1(T(ALPHA), T(name), 12, key)
#define TAB1(name, key) lookup1(T(name##_X), T(name##_Y), F16N_##name##_X, key)
#define TAB2_A(name, grid, rk, ck) lookup2(T(ALPHA), 12, T(GRID_##grid), F16N_GRID_##grid, T(name), rk, ck)
#define TAB2_E(name, rk, ck) lookup2(T(name##_MACH), F16N_##name##_MACH, T(GRID_DENSALT), F16N_GRID_DENSALT, T(name), rk, ck)

/* ---------------- frames (fdm.cuh:85-171) ---------------- */
static void q2dcm(const double q[4], double M[3][3]) {
  double a = q[0], b = q[1], c = q[2], d = q[3];
  double aa = a * a, bb = b * b, cc = c * c, dd = d * d;
  double ab = a * b, ac = a * c, ad = a * d, bc = b * c, bd = b * d, cd = c * d;
  M[0][0] = aa + bb - cc - dd; M[0][1] = 2.0 * (bc + ad); M[0][2] = 2.0 * (bd - ac);
  M[1][0] = 2.0 * (bc - ad); M[1][1] = aa - bb + cc - dd; M[1][2] = 2.0 * (cd + ab);
  M[2][0] = 2.0 * (bd + ac); M[2][1] = 2.0 * (cd - ab); M[2][2] = aa - bb - cc + dd;
}
static void qnormalize(double q[4]) {
  double m = sqrt(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
  if (m == 0.0) return;
  double k = 1.0 / m;
  q[0] *= k; q[1] *= k; q[2] *= k; q[3] *= k;
}
static void qrate(const double q[4], const double w[3], double o[4]) {
  o[0] = -0.5 * (q[1] * w[0] + q[2] * w[1] + q[3] * w[2]);
  o[1] = 0.5 * (q[0] * w[0] - q[3] * w[1] + q[2] * w[2]);
  o[2] = 0.5 * (q[3] * w[0] + q[0] * w[1] - q[1] * w[2]);
  o[3] = 0.5 * (-q[2] * w[0] + q[1] * w[1] + q[0] * w[2]);
}
static void euler2q(double phi, double tht, double psi, double q[4]) {
  double st = sin(0.5 * tht), sp = sin(0.5 * psi), sf = sin(0.5 * phi);
  double ct = cos(0.5 * tht), cp = cos(0.5 * psi), cf = cos(0.5 * phi);
  double cfct = cf * ct, cfst = cf * st, sfst = sf * st, sfct = sf * ct;
  q[0] = cfct * cp + sfst * sp;
  q[1] = sfct * cp - cfst * sp;
  q[2] = cfst * cp + sfct * sp;
  q[3] = cfct * sp - sfst * cp;
  qnormalize(q);
}
static void dcm2q(const double m[3][3], double Q[4]) {
  /* column-major walk of the matrix as JSBSim's FGMatrix33::GetQuaternion (fdm.cuh:113-121) */
  double c[9] = {m[0][0], m[1][0], m[2][0], m[0][1], m[1][1], m[2][1], m[0][2], m[1][2], m[2][2]};
  double tr[4] = {1.0 + c[0] + c[4] + c[8], 1.0 + c[0] - c[4] - c[8], 1.0 - c[0] + c[4] - c[8],
                  1.0 - c[0] - c[4] + c[8]};
  int k = 0;
  for (int i = 1; i < 4; i++)
    if (tr[i] > tr[k]) k = i;
  if (k == 0) {
    Q[0] = 0.5 * sqrt(tr[0]);
    Q[1] = 0.25 * (c[7] - c[5]) / Q[0]; Q[2] = 0.25 * (c[2] - c[6]) / Q[0]; Q[3] = 0.25 * (c[3] - c[1]) / Q[0];
  } else if (k == 1) {
    Q[1] = 0.5 * sqrt(tr[1]);
    Q[0] = 0.25 * (c[7] - c[5]) / Q[1]; Q[2] = 0.25 * (c[3] + c[1]) / Q[1]; Q[3] = 0.25 * (c[2] + c[6]) / Q[1];
  } else if (k == 2) {
    Q[2] = 0.5 * sqrt(tr[2]);
    Q[0] = 0.25 * (c[2] - c[6]) / Q[2]; Q[1] = 0.25 * (c[3] + c[1]) / Q[2]; Q[3] = 0.25 * (c[7] + c[5]) / Q[2];
  } else {
    Q[3] = 0.5 * sqrt(tr[3]);
    Q[0] = 0.25 * (c[3] - c[1]) / Q[3]; Q[1] = 0.25 * (c[6] + c[2]) / Q[3]; Q[2] = 0.25 * (c[7] + c[5]) / Q[3];
  }
}
static void dcm2euler(const double m[3][3], double e[3]) {
  double s = m[0][2], th;
  int lock = 0;
  if (s <= -1.0) { th = 0.5 * M_PI; lock = 1; }
  else if (1.0 <= s) { th = -0.5 * M_PI; lock = 1; }
  else th = asin(-s);
  if (lock) {
    e[0] = atan2(-m[2][1], m[1][1]);
    e[2] = 0.0;
  } else {
    e[0] = atan2(m[1][2], m[2][2]);
    e[2] = atan2(m[0][1], m[0][0]);
    if (e[2] < 0.0) e[2] += 2.0 * M_PI;
  }
  e[1] = th;
}
static void epa_rot(double epa, double M[3][3]) {
  double c = cos(epa), s = sin(epa);
  M[0][0] = c; M[0][1] = s; M[0][2] = 0.0;
  M[1][0] = -s; M[1][1] = c; M[1][2] = 0.0;
  M[2][0] = 0.0; M[2][1] = 0.0; M[2][2] = 1.0;
}
static void local_frame(const double p[3], double* rad, double* lat, double Tl2ec[3][3]) {
  double x = p[0], y = p[1], z = p[2];
  double r = sqrt(x * x + y * y + z * z), rxy = sqrt(x * x + y * y);
  double slon, clon, slat, clat;
  if (rxy == 0.0) { slon = 0.0; clon = 1.0; } else { slon = y / rxy; clon = x / rxy; }
  if (r == 0.0) { slat = 0.0; clat = 1.0; } else { slat = z / r; clat = rxy / r; }
  *lat = (rxy == 0.0 && z == 0.0) ? 0.0 : atan2(z, rxy);
  double Tec2l[3][3] = {{-clon * slat, -slon * slat, clat}, {-slon, clon, 0.0}, {-clon * clat, -slon * clat, -slat}};
  transp(Tec2l, Tl2ec);
  *rad = r;
}
static void j2_gravity(const double p[3], double lat, double o[3]) {
  double x = p[0], y = p[1], z = p[2];
  double r = sqrt(x * x + y * y + z * z);
  double sl = sin(lat);
  double ar = F16C_SEMI_MAJOR / r;
  double pc = 1.5 * F16C_J2const * ar * ar;
  double kxy = 1.0 - 5.0 * (sl * sl), kz = 3.0 - 5.0 * (sl * sl);
  double g = F16C_GM / (r * r);
  o[0] = -g * ((1.0 + (pc * kxy)) * x / r);
  o[1] = -g * ((1.0 + (pc * kxy)) * y / r);
  o[2] = -g * ((1.0 + (pc * kz)) * z / r);
}

/* ---------------- ISA atmosphere (fdm.cuh:174-224) ---------------- */
static double geopot(double h) { return (h * F16C_EarthRadius) / (F16C_EarthRadius + h); }
static double geomet(double gp) { return (gp * F16C_EarthRadius) / (F16C_EarthRadius - gp); }
static double isa_temp(double h) {
  double gp = geopot(h);
  if (gp >= 0.0) return lookup1(T(ATM_ALT), T(ATM_TMP), 9, gp);
  return lookup1(T(ATM_ALT), T(ATM_TMP), 9, 0.0) + gp * T(ATM_LAPSE)[0];
}
static double isa_press(double h) {
  double gp = geopot(h);
  double base = T(ATM_ALT)[0];
  int b = 0;
  for (int k = 0; k < 9 - 2; k++) {
    double nxt = T(ATM_ALT)[k + 1];
    if (gp < nxt) { b = k; break; }
    base = nxt;
    b = k + 1;
  }
  double Tb = isa_temp(geomet(base));
  double dh = gp - base, L = T(ATM_LAPSE)[b];
  if (L != 0.0) {
    double ex = F16C_g0 * F16C_Mair / (F16C_Rstar * L);
    double fac = Tb / (Tb + L * dh);
    return T(ATM_PBRK)[b] * pow(fac, ex);
  }
  return T(ATM_PBRK)[b] * exp(-F16C_g0 * F16C_Mair * dh / (F16C_Rstar * Tb));
}
static double isa_densalt(double rho) {
  int b = 0;
  for (int k = 0; k < 9 - 2; k++) {
    if (rho >= T(ATM_DBRK)[k + 1]) { b = k; break; }
    b = k + 1;
  }
  double Tb = T(ATM_TMP)[b], Hb = T(ATM_ALT)[b], L = T(ATM_LAPSE)[b], rb = T(ATM_DBRK)[b], h;
  if (L != 0.0) {
    double ex = -1.0 / (1.0 + (F16C_g0 * F16C_Mair) / (F16C_Rstar * L));
    h = Hb + (Tb / L) * (pow(rho / rb, ex) - 1.0);
  } else {
    double k = -(F16C_Rstar * Tb) / (F16C_g0 * F16C_Mair);
    h = Hb + k * log(rho / rb);
  }
  return geomet(h);
}
typedef struct { double T, P, rho, a, sigma, densalt; } Air;
static void isa(double h, Air* o) {
  o->T = isa_temp(h);
  o->P = isa_press(h);
  o->rho = o->P / (F16C_Reng * o->T);
  o->a = sqrt(F16C_SHRatio * F16C_Reng * o->T);
  double rho0 = F16C_StdDaySLpressure / (F16C_Reng * F16C_StdDaySLtemperature);
  o->sigma = o->rho / rho0;
  o->densalt = isa_densalt(o->rho);
}

/* ---------------- mass & inertia (fdm.cuh:226-262) ---------------- */
typedef struct { double cg[3], mass, J[3][3], Jinv[3][3], rp[3]; } MassProps;
static void to_body_ft(const double r[3], const double cg[3], double o[3]) {
  o[0] = F16C_INCHTOFT * (cg[0] - r[0]);
  o[1] = F16C_INCHTOFT * (r[1] - cg[1]);
  o[2] = F16C_INCHTOFT * (cg[2] - r[2]);
}
static void point_mass_J(double m, const double r[3], const double cg[3], double M[3][3]) {
  double v0 = F16C_INCHTOFT * (cg[0] - r[0]), v1 = F16C_INCHTOFT * (r[1] - cg[1]), v2 = F16C_INCHTOFT * (cg[2] - r[2]);
  double s0 = m * v0, s1 = m * v1, s2 = m * v2;
  double xx = s0 * v0, yy = s1 * v1, zz = s2 * v2, xy = -s0 * v1, xz = -s0 * v2, yz = -s1 * v2;
  M[0][0] = yy + zz; M[0][1] = xy; M[0][2] = xz;
  M[1][0] = xy; M[1][1] = xx + zz; M[1][2] = yz;
  M[2][0] = xz; M[2][1] = yz; M[2][2] = xx + yy;
}
static void mass_props(double fuel, MassProps* o) {
  static const double cg0[3] = {-193.0, 0.0, -5.1}, pilot[3] = {-336.2, 0.0, 0.0};
  static const double tk0[3] = {-174.4, 65.0, 5.0}, tk1[3] = {-174.4, -65.0, 5.0};
  static const double arp[3] = {-189.5, 0.0, 3.9};
  static const double J0[3][3] = {{9496.0, 0.0, -982.0}, {0.0, 55814.0, 0.0}, {-982.0, 0.0, 63100.0}};
  const double empty = 17400.0, pw = 230.0;
  double f0 = fuel / 2.0, f1 = f0;
  double w = empty + (f0 + f1) + pw;
  for (int i = 0; i < 3; i++) o->cg[i] = (empty * cg0[i] + pw * pilot[i] + f0 * tk0[i] + f1 * tk1[i]) / w;
  double J[3][3], t[3][3];
  memcpy(J, J0, sizeof J);
  const double* pts[4] = {cg0, pilot, tk0, tk1};
  double ms[4] = {F16C_LBTOSLUG * empty, F16C_LBTOSLUG * pw, F16C_LBTOSLUG * f0, F16C_LBTOSLUG * f1};
  for (int k = 0; k < 4; k++) {
    point_mass_J(ms[k], pts[k], o->cg, t);
    for (int i = 0; i < 3; i++)
      for (int j = 0; j < 3; j++) J[i][j] += t[i][j];
  }
  double Ixx = J[0][0], Iyy = J[1][1], Izz = J[2][2], Ixy = -J[0][1], Ixz = -J[0][2], Iyz = -J[1][2];
  double k1 = (Iyy * Izz - Iyz * Iyz), k2 = (Iyz * Ixz + Ixy * Izz), k3 = (Ixy * Iyz + Iyy * Ixz);
  double den = 1.0 / (Ixx * k1 - Ixy * k2 - Ixz * k3);
  k1 *= den; k2 *= den; k3 *= den;
  double k4 = (Izz * Ixx - Ixz * Ixz) * den, k5 = (Ixy * Ixz + Iyz * Ixx) * den, k6 = (Ixx * Iyy - Ixy * Ixy) * den;
  double Ji[3][3] = {{k1, k2, k3}, {k2, k4, k5}, {k3, k5, k6}};
  memcpy(o->Jinv, Ji, sizeof Ji);
  double Jm[3][3] = {{Ixx, -Ixy, -Ixz}, {-Ixy, Iyy, -Iyz}, {-Ixz, -Iyz, Izz}};
  memcpy(o->J, Jm, sizeof Jm);
  o->mass = F16C_LBTOSLUG * w;
  to_body_ft(arp, o->cg, o->rp);
}

/* ---------------- FCS (fdm.cuh:264-418; component dt is a parameter) ---------------- */
static int near_equal(double a, double b) { return fabs(a - b) <= 1e-9 * mx(mx(1.0, fabs(a)), fabs(b)); }
static double actuator(const double* det, const double* tim, int n, double* out, double in, int scale,
                       int seeded, double seedv, double dt) {
  double rem = dt, x = in;
  if (scale) x *= det[n - 1];
  double y = seeded ? seedv : *out;
  x = clampd(x, det[0], det[n - 1]);
  while (rem > 0.0 && !near_equal(x, y)) {
    int k = 1;
    for (;;) {
      int go = (x < y) ? (det[k] < y) : (det[k] <= y);
      if (!go) break;
      k++;
      if (k >= n) break;
    }
    if (k >= n) k = n - 1;
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
  *out = y;
  return y;
}
static double pid(double kp, double ki, double kd, double* s /* ip, ip2, iout */, double in,
                  double trig, int clip, double lo, double hi, double dt) {
  double dv = (in - s[0]) / dt;
  double dI = 0.0;
  if (fabs(trig) < 0.000001) dI = 1.5 * in - 0.5 * s[0];
  if (trig < 0.0) s[2] = 0.0;
  s[2] += ki * dt * dI;
  double out = kp * in + s[2] + kd * dv;
  s[1] = (trig < 0.0) ? 0.0 : s[0];
  s[0] = in;
  if (clip) out = clampd(out, lo, hi);
  return out;
}
static double surface(double in, double inmin, double inmax, double outmin, double outmax) {
  if (in == 0.0) return 0.0;
  if (in > 0.0) return (in / inmax) * outmax;
  return (in / inmin) * outmin;
}
typedef struct { double ail, ele, rud, lef, flap, sb, gear; } Surfaces;
static void fcs(double* kin /*6*/, double* pids /*9*/, double c_ail, double c_ele, double c_rud,
                const double* pa /* prev aux 9 */, double pitch, double roll, double dt, Surfaces* o) {
  static const double d_tef[3] = {-1.0, 0.0, 1.0}, t_tef[3] = {3.0, 0.0, 3.0};
  static const double d_pm1[2] = {-1.0, 1.0}, t_ail[2] = {0.3, 0.3}, t_rud[2] = {0.4, 0.4}, t_lef[2] = {3.0, 3.0};
  static const double d_gear[2] = {0.0, 1.0}, t_gear[2] = {0.0, 5.0};
  double alpha = pa[0], mach = pa[1], vc = pa[2], vg = pa[3], npy = pa[4], npz = pa[5];
  double p = pa[6], q = pa[7], r = pa[8];
  /* flaps */
  double tef = (vc < 250.0) ? 0.349 : ((mach > 0.9) ? -0.0349 : 0.0);
  double tef_c = actuator(d_tef, t_tef, 3, &kin[0], 2.864789 * tef, 1, 0, 0.0, dt);
  /* roll channel */
  double roll_err = c_ail - 0.31821 * p;
  double roll_pid = pid(3.0, 0.0005, -0.00125, &pids[0], roll_err, (vc < 20.0) ? 0.0 : 1.0, 0, 0, 0, dt);
  double roll_cmd = clampd(roll_pid + c_ail, -1.0, 1.0);
  double ail_n = actuator(d_pm1, t_ail, 2, &kin[1], roll_cmd, 1, 0, 0.0, dt);
  double ail_comp = TAB1(FCS_AIL_SPEED, mach) * ail_n;
  double flap_l = clampd(-tef_c - ail_comp, -1.0, 1.0);
  double flap_r = clampd(tef_c - ail_comp, -1.0, 1.0);
  o->flap = 1.4324 * (flap_l + flap_r);
  o->ail = surface(roll_cmd, -1.0, 1.0, -0.375, 0.375);
  /* pitch channel */
  double gcorr = npz - cos(pitch) * cos(roll);
  double ele_lim = clampd(c_ele + 0.0, -1.0, 0.44);
  double ele_sched = TAB1(FCS_ELEV_SCHED, alpha) * ele_lim;
  double pitch_err = ele_sched + 6.2 * q - 0.020 * gcorr;
  double g_pid = pid(0.3, 0.025, 0.0, &pids[3], pitch_err, (vc < 5.0) ? 0.0 : 1.0, 1, -1.0, 1.0, dt);
  double pitch_cmd = clampd(ele_sched + 1.0472 * alpha + g_pid, -1.0, 1.0);
  double ele_n = actuator(d_pm1, t_ail, 2, &kin[2], pitch_cmd, 1, 0, 0.0, dt);
  o->ele = surface(ele_n, -1.0, 1.0, -0.436, 0.436);
  /* yaw channel */
  double yaw_err = c_rud + TAB1(FCS_YAW_RATE, vg) * r + 0.25 * npy;
  double y_pid = pid(0.1055, 0.00001, 0.00005, &pids[6], yaw_err, (vc < 10.0) ? 0.0 : 1.0, 1, -1.0, 1.0, dt);
  double yaw_cmd = clampd(c_rud + 0.0 + y_pid, -1.0, 1.0);
  double rud_n = actuator(d_pm1, t_rud, 2, &kin[3], yaw_cmd, 1, 1, y_pid, dt);
  o->rud = surface(rud_n, -1.0, 1.0, -0.524, 0.524);
  /* landing gear held by the external force, weight-on-wheels 0 */
  double gear = actuator(d_gear, t_gear, 2, &kin[4], 0.0, 1, 1, GEAR_FORCE, dt);
  o->gear = gear;
  /* leading-edge flaps (gear_wow == 0 always) */
  double lef;
  if (gear == 0.0 && alpha > 0.2618) lef = 0.436;
  else if (alpha > 0.0873) lef = 0.262;
  else if (mach > 0.9) lef = -0.0349;
  else lef = 0.0;
  o->lef = lef;
  actuator(d_pm1, t_lef, 2, &kin[5], 2.293578 * lef, 1, 0, 0.0, dt);
  o->sb = 0.0;
}

/* ---------------- turbine (fdm.cuh:420-455) ---------------- */
static double approach(double v, double tgt, double up, double dn, double dt) {
  if (v > tgt) { v -= dt * dn; if (v < tgt) v = tgt; }
  else if (v < tgt) { v += dt * up; if (v > tgt) v = tgt; }
  return v;
}
static double spool_rate(double delay, double sigma, double n2n) {
  double n = n2n + 0.1;
  if (n > 1.0) n = 1.0;
  double om = 1.0 - n;
  return delay / (1.0 + 3.0 * om * om * om + (1.0 - sigma));
}
static void turbine(double* e /* N1, N2, N2norm, FF */, double thr, double mach, double densalt, double Tk,
                    double sigma, const double cg[3], double* thrust_o, double* burn_o, double F[3], double M[3]) {
  const double dt = DT_FRAME;
  double tp = thr, aug;
  if (tp > 1.0) { aug = tp - 1.0; tp -= aug; } else aug = 0.0;
  double n1f = F16C_MAXN1 - F16C_IDLEN1, n2f = F16C_MAXN2 - F16C_IDLEN2;
  double base = 90.0 / (F16C_BYPASSRATIO + 3.0);
  double n2up = spool_rate(1.0 * base, sigma, e[2]), n2dn = spool_rate(3.0 * base, sigma, e[2]);
  double n1up = spool_rate(1.0 * base, sigma, e[2]), n1dn = spool_rate(2.4 * base, sigma, e[2]);
  e[1] = approach(e[1], F16C_IDLEN2 + tp * n2f, n2up, n2dn, dt);
  e[0] = approach(e[0], F16C_IDLEN1 + tp * n1f, n1up, n1dn, dt);
  e[2] = (e[1] - F16C_IDLEN2) / n2f;
  double idle = F16C_MILTHRUST * TAB2_E(ENG_IDLE, mach, densalt);
  double mil = (F16C_MILTHRUST - idle) * TAB2_E(ENG_MIL, mach, densalt);
  double thrust = idle + mil * e[2] * e[2];
  double om = 1.0 - e[2];
  double tsfc = F16C_TSFC * sqrt(Tk / 389.7) * (0.84 + om * om);
  e[3] = approach(e[3], thrust * tsfc, 1000.0, 10000.0, dt);
  if (e[3] < F16C_IdleFF) e[3] = F16C_IdleFF;
  thrust = thrust * (1.0 - F16C_BLEEDDEMAND);
  if (aug > 0.0) {
    double td = (F16C_MAXTHRUST * TAB2_E(ENG_AUG, mach, densalt)) - thrust;
    thrust += td * aug;
    e[3] = approach(e[3], thrust * F16C_ATSFC, 5000.0, 10000.0, dt);
  }
  double rz = F16C_INCHTOFT * (cg[2] - 0.0), ry = F16C_INCHTOFT * (0.0 - cg[1]);
  *thrust_o = thrust;
  F[0] = thrust; F[1] = 0.0; F[2] = 0.0;
  M[0] = 0.0; M[1] = rz * thrust; M[2] = -ry * thrust;
  *burn_o = e[3] / 3600.0 * dt;
}

/* ---------------- air data (fdm.cuh:457-497) ---------------- */
static double total_pressure(double m, double p) {
  if (m < 0.0) return p;
  if (m < 1.0) { double k = 1.0 + 0.2 * m * m; return p * k * k * k * sqrt(k); }
  return p * 166.92158009316827 * pow(m, 7.0) / pow(7.0 * m * m - 1.0, 2.5);
}
static double mach_from_qc(double qc, double p) {
  double A = qc / p + 1.0;
  double m = sqrt(5.0 * (pow(A, 1.0 / 3.5) - 1.0));
  if (m > 1.0)
    for (int i = 0; i < 10; i++) { double t = 1.0 - 1.0 / (7.0 * m * m); m = 0.8812848543473311 * sqrt(A * pow(t, 2.5)); }
  return m;
}
static double cas_from_mach(double m, double p) {
  double qc = total_pressure(m, p) - p;
  return F16C_STD_SL_SOUNDSPEED * mach_from_qc(qc, F16C_StdDaySLpressure);
}
typedef struct { double alpha, beta, vt, qbar, mach, p, q, r, vg, npy, npz, vc; } AirData;
static void air_data(const double uvw[3], const double pqr[3], const double vned[3], double rho, double a,
                     double P, const double cg[3], const double pbacc[3], const double ppqridot[3],
                     const double ppqri[3], AirData* o) {
  double u = uvw[0], v = uvw[1], w = uvw[2];
  double uw = u * u + w * w, vt2 = uw + v * v, vt = sqrt(vt2);
  double al = 0.0, be = 0.0;
  if (vt > 0.001) { be = atan2(v, sqrt(uw)); if (uw >= 1e-6) al = atan2(w, u); }
  o->alpha = al; o->beta = be; o->vt = vt;
  o->qbar = 0.5 * rho * vt2;
  o->mach = vt / a;
  o->vg = sqrt(vned[0] * vned[0] + vned[1] * vned[1]);
  static const double eye[3] = {-336.2, 0.0, 29.5};
  double r_eye[3], c1[3], c2[3], c3[3];
  to_body_ft(eye, cg, r_eye);
  cross3(ppqridot, r_eye, c1);
  cross3(ppqri, r_eye, c2);
  cross3(ppqri, c2, c3);
  double ay = pbacc[1] + c1[1] + c3[1], az = pbacc[2] + c1[2] + c3[2];
  o->npy = ay / F16C_SLGRAVITY; o->npz = az / F16C_SLGRAVITY;
  double vcas = (fabs(o->mach) > 0.0) ? cas_from_mach(o->mach, P) : 0.0;
  o->vc = vcas * F16C_FPSTOKTS;
  o->p = pqr[0]; o->q = pqr[1]; o->r = pqr[2];
}

/* ---------------- aerodynamics (f16_gen.cuh:170-238; 40 coefficient terms) ---------------- */
static void aero(double qb, double al, double be, double mach, double b2v, double c2v, double kge, double p,
                 double q, double r, double ail, double ele, double rud, double lef, double flap, double sb,
                 double gear, double o[6]) {
  double s, k = qb * 300.0;
  s = 0.0;                                   /* drag */
  s += k * TAB2_A(CDDH, ELEV, al, ele);
  s += k * TAB1(CDMACH, mach);
  s += k * lef * TAB1_A(CDDLEF, al);
  s += k * flap * 0.08;
  s += k * gear * 0.027;
  s += k * sb * TAB1_A(CDDSB, al);
  s += k * q * c2v * TAB1_A(CDQ, al);
  s += k * q * c2v * lef * TAB1_A(CDQ_DLEF, al);
  o[0] = s;
  s = 0.0;                                   /* side force */
  s += k * be * -1.146;
  s += k * be * TAB1(CYB_M, mach);
  s += k * ail * -0.0226;
  s += k * rud * 0.086;
  s += k * b2v * p * TAB1_A(CYP, al);
  s += k * b2v * r * TAB1_A(CYR, al);
  o[1] = s;
  s = 0.0;                                   /* lift */
  s += k * kge * TAB2_A(CLDH, ELEV, al, ele);
  s += k * lef * kge * TAB1_A(CLDLEF, al);
  s += k * flap * kge * 0.35;
  s += k * kge * sb * TAB1_A(CLDSB, al);
  s += k * q * kge * c2v * TAB1_A(CLQ, al);
  s += k * q * c2v * sb * TAB1_A(CLQ_DSB, al);
  o[2] = s;
  double kb = k * 30.0, kc = k * 11.32;
  s = 0.0;                                   /* roll */
  s += kb * TAB2_A(CLB, BETA13, al, be);
  s += kb * be * TAB1(CLB_M, mach);
  s += kb * b2v * p * TAB1_A(CLP, al);
  s += kb * b2v * r * TAB1_A(CLR, al);
  s += kb * ail * TAB2_A(CLDA, BETA7, al, be);
  s += kb * al * ail * TAB1(CLDA_M, mach);
  s += kb * al * rud * TAB1(CLDR_M, mach);
  s += kb * rud * TAB2_A(CLDR, BETA7, al, be);
  o[3] = s;
  s = 0.0;                                   /* pitch */
  s += kc * TAB2_A(CMDH, ELEV, al, ele);
  s += kc * al * TAB1(CMA_M, mach);
  s += kc * sb * TAB1_A(CMDSB, al);
  s += kc * c2v * q * TAB1_A(CMQ, al);
  o[4] = s;
  s = 0.0;                                   /* yaw */
  s += kb * TAB2_A(CNB, BETA13, al, be);
  s += kb * be * TAB1(CNB_M, mach);
  s += kb * b2v * p * TAB1_A(CNP, al);
  s += kb * b2v * r * TAB1_A(CNR, al);
  s += kb * ail * TAB1(CNDA_M, mach);
  s += kb * ail * TAB2_A(CNDA, BETA7, al, be);
  s += kb * rud * TAB2_A(CNDR, BETA7, al, be);
  s += kb * al * rud * TAB1(CNDR_M, mach);
  o[5] = s;
}

/* ---------------- kinematics + force path (fdm.cuh:544-607) ---------------- */
typedef struct {
  double uvw[3], pqr[3], vned[3], ecef[3], Ti2b[3][3], Tec2i[3][3], radius, lat, euler[3];
} Kin;
static void kinematics(const double* s, Kin* k) {
  double Ti2ec[3][3], Tl2ec[3][3], Tl2i[3][3], Tl2b[3][3], Tb2l[3][3];
  epa_rot(s[F16_S_EPA], Ti2ec);
  transp(Ti2ec, k->Tec2i);
  matvec(Ti2ec, s + F16_S_POS, k->ecef);
  local_frame(k->ecef, &k->radius, &k->lat, Tl2ec);
  matmul(k->Tec2i, Tl2ec, Tl2i);
  q2dcm(s + F16_S_Q, k->Ti2b);
  matmul(k->Ti2b, Tl2i, Tl2b);
  transp(Tl2b, Tb2l);
  const double w[3] = {0.0, 0.0, F16C_ROTATION_RATE};
  double wr[3], dv[3], wb[3];
  cross3(w, s + F16_S_POS, wr);
  for (int i = 0; i < 3; i++) dv[i] = s[F16_S_VEL + i] - wr[i];
  matvec(k->Ti2b, dv, k->uvw);
  matvec(k->Ti2b, w, wb);
  for (int i = 0; i < 3; i++) k->pqr[i] = s[F16_S_PQRI + i] - wb[i];
  matvec(Tb2l, k->uvw, k->vned);
  dcm2euler(Tl2b, k->euler);
}
typedef struct { double uvwidot[3], pqridot[3], bacc[3], pqri[3]; AirData ad; double thrust, burn, alt; } Forces;
static void force_path(const double* s, double* kin6, double* pid9, double* eng4, double fuel,
                       double c_ail, double c_ele, double c_rud, double c_thr, const double* pa,
                       const double* pbacc, const double* ppqridot, const double* ppqri, const Kin* k,
                       double fcs_dt, Forces* f) {
  f->alt = k->radius - F16C_SEA_LEVEL_RADIUS;
  Air at;
  isa(f->alt, &at);
  MassProps mp;
  mass_props(fuel, &mp);
  Surfaces sf;
  fcs(kin6, pid9, c_ail, c_ele, c_rud, pa, k->euler[1], k->euler[0], fcs_dt, &sf);
  air_data(k->uvw, k->pqr, k->vned, at.rho, at.a, at.P, mp.cg, pbacc, ppqridot, ppqri, &f->ad);
  double Fe[3], Me[3];
  turbine(eng4, 2.0 * c_thr, f->ad.mach, at.densalt, at.T, at.sigma, mp.cg, &f->thrust, &f->burn, Fe, Me);
  double vt = f->ad.vt, two = 2.0 * vt;
  double b2v = (two != 0.0) ? 30.0 / two : 0.0, c2v = (two != 0.0) ? 11.32 / two : 0.0;
  double kge = TAB1(KCLGE, HB_MAC);
  double A[6];
  aero(f->ad.qbar, f->ad.alpha, f->ad.beta, f->ad.mach, b2v, c2v, kge, f->ad.p, f->ad.q, f->ad.r, sf.ail,
       sf.ele, sf.rud, sf.lef, sf.flap, sf.sb, sf.gear, A);
  double drag = -A[0], side = A[1], lift = -A[2];
  double ca = cos(f->ad.alpha), sa = sin(f->ad.alpha), cb = cos(f->ad.beta), sb = sin(f->ad.beta);
  double Fx = ca * cb * drag + (-ca * sb) * side + (-sa) * lift;
  double Fy = sb * drag + cb * side;
  double Fz = sa * cb * drag + (-sa * sb) * side + ca * lift;
  double rx = mp.rp[0], ry = mp.rp[1], rz = mp.rp[2];
  double mr[3] = {ry * Fz - rz * Fy, rz * Fx - rx * Fz, rx * Fy - ry * Fx};
  double F[3] = {Fx + Fe[0], Fy + Fe[1], Fz + Fe[2]};
  double M[3] = {A[3] + mr[0] + Me[0], A[4] + mr[1] + Me[1], A[5] + mr[2] + Me[2]};
  double ge[3], g[3];
  j2_gravity(k->ecef, k->lat, ge);
  matvec(k->Tec2i, ge, g);
  /* accelerations (fdm.cuh:499-517) */
  const double w[3] = {0.0, 0.0, F16C_ROTATION_RATE};
  double wb[3], Jw[3], gyro[3], mm[3], Tb2i[3][3], tmp[3];
  matvec(k->Ti2b, w, wb);
  double pqri[3] = {k->pqr[0] + wb[0], k->pqr[1] + wb[1], k->pqr[2] + wb[2]};
  matvec(mp.J, pqri, Jw);
  cross3(pqri, Jw, gyro);
  for (int i = 0; i < 3; i++) mm[i] = M[i] - gyro[i];
  matvec(mp.Jinv, mm, f->pqridot);
  double ba[3] = {F[0] / mp.mass, F[1] / mp.mass, F[2] / mp.mass};
  for (int i = 0; i < 3; i++) { f->bacc[i] = ba[i]; f->pqri[i] = pqri[i]; }
  transp(k->Ti2b, Tb2i);
  matvec(Tb2i, ba, tmp);
  for (int i = 0; i < 3; i++) f->uvwidot[i] = tmp[i] + g[i];
}

/* ---------------- one frame (fdm.cuh:609-649) ---------------- */
static void shift_in(double* deq, int w, const double* v) {
  for (int i = 0; i < w; i++) { deq[2 * w + i] = deq[w + i]; deq[w + i] = deq[i]; deq[i] = v[i]; }
}
static void frame(double* s, double ail, double ele, double rud, double thr, double fcs_dt, double* obs17) {
  const double dt = DT_FRAME;
  shift_in(s + F16_S_DEQ_Q, 4, s + F16_S_QDOT);
  for (int i = 0; i < 4; i++) s[F16_S_Q + i] = s[F16_S_Q + i] + dt * s[F16_S_DEQ_Q + i];
  qnormalize(s + F16_S_Q);
  shift_in(s + F16_S_DEQ_PQRI, 3, s + F16_S_PQRIDOT);
  for (int i = 0; i < 3; i++) s[F16_S_PQRI + i] = s[F16_S_PQRI + i] + dt * s[F16_S_DEQ_PQRI + i];
  shift_in(s + F16_S_DEQ_IVEL, 3, s + F16_S_VEL);
  const double* h = s + F16_S_DEQ_IVEL;
  for (int i = 0; i < 3; i++)
    s[F16_S_POS + i] = s[F16_S_POS + i] + (dt / 12.0) * (23.0 * h[i] - 16.0 * h[3 + i] + 5.0 * h[6 + i]);
  shift_in(s + F16_S_DEQ_UVWIDOT, 3, s + F16_S_UVWIDOT);
  const double* g = s + F16_S_DEQ_UVWIDOT;
  for (int i = 0; i < 3; i++) s[F16_S_VEL + i] = s[F16_S_VEL + i] + dt * (1.5 * g[i] - 0.5 * g[3 + i]);
  s[F16_S_EPA] += F16C_ROTATION_RATE * dt;

  Kin k;
  kinematics(s, &k);
  qrate(s + F16_S_Q, s + F16_S_PQRI, s + F16_S_QDOT);
  Forces f;
  force_path(s, s + F16_S_KIN, s + F16_S_PID, s + F16_S_ENG, s[F16_S_FUEL], ail, ele, rud, thr,
             s + F16_S_PREV_AUX, s + F16_S_PREV_BACC, s + F16_S_PREV_PQRIDOT, s + F16_S_PREV_PQRI, &k,
             fcs_dt, &f);
  s[F16_S_FUEL] -= f.burn;
  for (int i = 0; i < 3; i++) {
    s[F16_S_UVWIDOT + i] = f.uvwidot[i];
    s[F16_S_PQRIDOT + i] = f.pqridot[i];
    s[F16_S_PREV_BACC + i] = f.bacc[i];
    s[F16_S_PREV_PQRIDOT + i] = f.pqridot[i];
    s[F16_S_PREV_PQRI + i] = f.pqri[i];
  }
  double* pa = s + F16_S_PREV_AUX;
  pa[0] = f.ad.alpha; pa[1] = f.ad.mach; pa[2] = f.ad.vc; pa[3] = f.ad.vg;
  pa[4] = f.ad.npy; pa[5] = f.ad.npz; pa[6] = f.ad.p; pa[7] = f.ad.q; pa[8] = f.ad.r;
  if (obs17) {
    for (int i = 0; i < 3; i++) {
      obs17[i] = s[F16_S_POS + i]; obs17[3 + i] = s[F16_S_VEL + i];
      obs17[6 + i] = k.euler[i]; obs17[9 + i] = k.uvw[i];
    }
    obs17[12] = f.ad.alpha; obs17[13] = f.ad.beta; obs17[14] = f.ad.mach; obs17[15] = f.ad.vt;
    obs17[16] = f.alt;
  }
}

/* Batch step: states (nac,101) AoS in place; cmd (nac,4); obs17 (nac,17) or NULL. */
int oracle_fdm_step(double* states, const double* cmd, long nac, int substeps, double fcs_dt, double* obs17) {
  if (!states || !cmd || nac < 0 || substeps < 1) return 1;
  for (long a = 0; a < nac; a++) {
    double* s = states + a * F16_STATE_N;
    const double* c = cmd + a * 4;
    for (int k = 0; k < substeps; k++)
      frame(s, c[0], c[1], c[2], c[3], fcs_dt, (obs17 && k == substeps - 1) ? obs17 + a * 17 : 0);
  }
  return 0;
}

/* ---------------- IC -> seed row (ic.py:18-138, jsb_fdm.py:142-210) ---------------- */
static void geodetic_ecef(double lat, double lon, double alt, double o[3]) {
  /* WGS84 normal through (lat,lon), point chosen so that |ecef| = a + alt (ic.py:18-39) */
  double a = F16C_SEMI_MAJOR, e2 = F16C_E2;
  double sp = sin(lat), cp = cos(lat), sl = sin(lon), cl = cos(lon);
  double N = a / sqrt(1.0 - e2 * sp * sp);
  double A = cp * cp, B = sp * sp, P = N, Q = N * (1.0 - e2);
  double b = A * P + B * Q, c = A * P * P + B * Q * Q, R = a + alt;
  double t = -b + sqrt(b * b - c + R * R);
  o[0] = (N + t) * cp * cl;
  o[1] = (N + t) * cp * sl;
  o[2] = (N * (1.0 - e2) + t) * sp;
}
int oracle_seed_ic(const double* ic /* F16_IC_N */, double fcs_dt, double* s /* 101 */) {
  const double d2r = M_PI / 180.0;
  double lat = ic[F16_IC_LAT_DEG] * d2r, lon = ic[F16_IC_LON_DEG] * d2r, alt = ic[F16_IC_ALT_FT];
  double vt = ic[F16_IC_VT_FPS];
  double phi = ic[F16_IC_PHI_DEG] * d2r, psi = ic[F16_IC_PSI_DEG] * d2r, tht = ic[F16_IC_THETA_DEG] * d2r;
  double al = ic[F16_IC_ALPHA_DEG] * d2r, be = ic[F16_IC_BETA_DEG] * d2r;
  double fuel = ic[F16_IC_FUEL_LBS], ff = ic[F16_IC_FUELFLOW_PPH];
  double ecef[3];
  if (ic[F16_IC_GEOCENTRIC] != 0.0) {
    double r = F16C_SEMI_MAJOR + alt;
    ecef[0] = r * cos(lat) * cos(lon); ecef[1] = r * cos(lat) * sin(lon); ecef[2] = r * sin(lat);
  } else {
    geodetic_ecef(lat, lon, alt, ecef);
  }
  memset(s, 0, sizeof(double) * F16_STATE_N);
  /* epa = 0: ECI == ECEF (ic.py:63-65) */
  double Ti2ec[3][3], Tec2i[3][3], Tl2ec[3][3], Tl2i[3][3], Ti2l[3][3], Tl2b[3][3], Ti2b[3][3], Tb2i[3][3];
  double rad, glat, ql[4];
  epa_rot(0.0, Ti2ec);
  transp(Ti2ec, Tec2i);
  double pos[3];
  matvec(Tec2i, ecef, pos);
  local_frame(ecef, &rad, &glat, Tl2ec);
  matmul(Tec2i, Tl2ec, Tl2i);
  transp(Tl2i, Ti2l);
  euler2q(phi, tht, psi, ql);
  q2dcm(ql, Tl2b);
  matmul(Tl2b, Ti2l, Ti2b);
  transp(Ti2b, Tb2i);
  double uvw[3] = {vt * cos(al) * cos(be), vt * sin(be), vt * sin(al) * cos(be)};
  const double w[3] = {0.0, 0.0, F16C_ROTATION_RATE};
  double vb[3], wr[3];
  matvec(Tb2i, uvw, vb);
  cross3(w, pos, wr);
  for (int i = 0; i < 3; i++) { s[F16_S_POS + i] = pos[i]; s[F16_S_VEL + i] = vb[i] + wr[i]; }
  /* FDM.seed (jsb_fdm.py:142-210): the attitude chain is rebuilt from the ECI position. */
  s[F16_S_EPA] = 0.0;
  s[F16_S_FUEL] = fuel;
  double ecef2[3], rad2, lat2, Tl2ec2[3][3], Tl2i2[3][3], Ti2l2[3][3], Ti2b2[3][3];
  matvec(Ti2ec, s + F16_S_POS, ecef2);
  local_frame(ecef2, &rad2, &lat2, Tl2ec2);
  matmul(Tec2i, Tl2ec2, Tl2i2);
  transp(Tl2i2, Ti2l2);
  matmul(Tl2b, Ti2l2, Ti2b2);
  dcm2q(Ti2b2, s + F16_S_Q);
  double wb[3];
  matvec(Ti2b2, w, wb);
  for (int i = 0; i < 3; i++) s[F16_S_PQRI + i] = 0.0 + wb[i];
  /* prev_aux from the IC (ic.py:127-132) */
  Air at;
  isa(alt, &at);
  double mach = vt / at.a;
  double vcas = (fabs(mach) > 0.0) ? cas_from_mach(mach, at.P) : 0.0;
  double* pa = s + F16_S_PREV_AUX;
  pa[0] = al; pa[1] = mach; pa[2] = vcas * F16C_FPSTOKTS; pa[3] = vt; pa[4] = 0.0; pa[5] = -1.0;
  pa[6] = 0.0; pa[7] = 0.0; pa[8] = 0.0;
  /* one throwaway force path with a fresh FCS / engine and commands (0,0,0,0.8) */
  Kin k;
  kinematics(s, &k);
  double tmp_kin[6] = {0}, tmp_pid[9] = {0}, tmp_eng[4] = {100.0, 100.0, (100.0 - F16C_IDLEN2) / (F16C_MAXN2 - F16C_IDLEN2), ff};
  const double zero3[3] = {0.0, 0.0, 0.0};
  double ppqri[3] = {s[F16_S_PQRI], s[F16_S_PQRI + 1], s[F16_S_PQRI + 2]};
  Forces f;
  force_path(s, tmp_kin, tmp_pid, tmp_eng, fuel, 0.0, 0.0, 0.0, 0.8, pa, zero3, zero3, ppqri, &k, fcs_dt, &f);
  for (int i = 0; i < 3; i++) {
    s[F16_S_UVWIDOT + i] = f.uvwidot[i];
    s[F16_S_PQRIDOT + i] = f.pqridot[i];
    s[F16_S_PREV_BACC + i] = f.bacc[i];
    s[F16_S_PREV_PQRIDOT + i] = f.pqridot[i];
    s[F16_S_PREV_PQRI + i] = f.pqri[i];
  }
  qrate(s + F16_S_Q, s + F16_S_PQRI, s + F16_S_QDOT);
  for (int k2 = 0; k2 < 3; k2++) {
    for (int i = 0; i < 4; i++) s[F16_S_DEQ_Q + 4 * k2 + i] = s[F16_S_QDOT + i];
    for (int i = 0; i < 3; i++) {
      s[F16_S_DEQ_PQRI + 3 * k2 + i] = s[F16_S_PQRIDOT + i];
      s[F16_S_DEQ_IVEL + 3 * k2 + i] = s[F16_S_VEL + i];
      s[F16_S_DEQ_UVWIDOT + 3 * k2 + i] = s[F16_S_UVWIDOT + i];
    }
  }
  /* fresh engine (N1 = N2 = 100) with the IC fuel flow, fresh FCS (all zero) */
  s[F16_S_ENG + 0] = 100.0; s[F16_S_ENG + 1] = 100.0;
  s[F16_S_ENG + 2] = (100.0 - F16C_IDLEN2) / (F16C_MAXN2 - F16C_IDLEN2);
  s[F16_S_ENG + 3] = ff;
  return 0;
}
