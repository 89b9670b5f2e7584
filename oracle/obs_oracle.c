/*
 * obs_oracle.c -- TEST INFRASTRUCTURE ONLY (the parity checker; never shipped or measured).
 *
 * Plain-C CPU restatement of the reference's fused 184-D observation / final-safe reward /
 * termination kernels, research/competition_36500/runtime/cuda_fdm/gen/obs_kernel.cu:
 *   kin9 :96-145, geometry helpers :148-330, build_obs_one :336-482,
 *   init_reward_kernel :485-501, advance_kernel :504-626, build_obs_kernel :628-649.
 * Loops over environments / aircraft replace the one-thread-per-item launches.  States are
 * the reference's (nac,101) AoS rows.  Pinned against the reference's torch path
 * (R/cuda_fdm/obs_reward.py BatchObsReward, enable_kernel=False) by tests/golden/obs_*.npz.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define D2R 0.017453292519943295
#define R2D 57.29577951308232
#define PI2 6.283185307179586
#define FT2M 0.3048
#define M2FT 3.28084
#define SLR_FT 20925646.32546
#define ROT 7.292115e-5
#define WA 6378137.0
#define WE2 0.0066943799901411
/* observation constants (claude_code/my_observation.py:97-149) */
#define MAX_SPEED 600.0
#define MAX_RANGE_M 2500.0
#define MAX_CLOSURE 1000.0
#define VSPEED_SCALE 100.0
#define PQR_SCALE 4.0
#define AOA_SCALE 30.0
#define SSLIP_SCALE 15.0
#define MIN_ALT_M 304.8
#define ALT_DANGER 300.0
#define MAX_ALT_M 15000.0
#define ENERGY_ADV 5000.0
#define PURSUIT_ATA 30.0
#define PURSUIT_RANGE 3000.0
#define FUEL_BURN 8.0e-5
#define FUEL_REF 300.0
#define REL_VEL 600.0
#define GACC 9.80665
#define EPISODE_MAX 200.0
#define TLIM_TOL 1.0e-8
#define MIN_DMG_R_FT 500.0
#define T1_MAX 3000.0
#define T2_MAX 3500.0
#define T3_MAX 4000.0
#define T1_CONE 1.0
#define T2_CONE 2.0
#define T3_CONE 3.0
#define T2_START 100.0
#define T3_START 150.0
#define GEOM_BUDGET 5.0
#define GEOM_REF_SEC 200.0
#define SHAPING_BASE 0.0001
#define ALT_LOG_SCALE_M 304.8
#define ALT_LOG_FLOOR 1.0e-4

typedef struct { double ox, oy, oz, sl, cl, so, co; } Origin;

static double clampd(double x, double a, double b) { return x < a ? a : (x > b ? b : x); }
static double norm3(const double v[3]) { return sqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]); }
static void mat_mul(const double A[3][3], const double B[3][3], double C[3][3]) {
  for (int i = 0; i < 3; i++)
    for (int j = 0; j < 3; j++) {
      double s = 0.0;
      for (int k = 0; k < 3; k++) s += A[i][k] * B[k][j];
      C[i][j] = s;
    }
}
static void mv(const double A[3][3], const double v[3], double o[3]) {
  for (int i = 0; i < 3; i++) o[i] = A[i][0] * v[0] + A[i][1] * v[1] + A[i][2] * v[2];
}
static void mvT(const double A[3][3], const double v[3], double o[3]) {
  for (int i = 0; i < 3; i++) o[i] = A[0][i] * v[0] + A[1][i] * v[1] + A[2][i] * v[2];
}
/* roll/pitch/yaw (deg) -> R_ned_to_body = Tx Ty Tz (obs_kernel.cu:75-84) */
static void ned2body(double roll, double pitch, double yaw, double R[3][3]) {
  double r = roll * D2R, p = pitch * D2R, y = yaw * D2R;
  double cr = cos(r), sr = sin(r), cp = cos(p), sp = sin(p), cy = cos(y), sy = sin(y);
  double Tx[3][3] = {{1, 0, 0}, {0, cr, sr}, {0, -sr, cr}};
  double Ty[3][3] = {{cp, 0, -sp}, {0, 1, 0}, {sp, 0, cp}};
  double Tz[3][3] = {{cy, sy, 0}, {-sy, cy, 0}, {0, 0, 1}};
  double TyTz[3][3];
  mat_mul(Ty, Tz, TyTz);
  mat_mul(Tx, TyTz, R);
}

/* FDM state row -> official 9-DoF N/E/D m, roll/pitch/yaw deg, body u/v/w m/s (:96-145) */
static void kin9(const double* st, const Origin* O, double s9[9]) {
  double px = st[0], py = st[1], pz = st[2], vx = st[3], vy = st[4], vz = st[5];
  double q0 = st[6], q1 = st[7], q2 = st[8], q3 = st[9], epa = st[13];
  double ce = cos(epa), se = sin(epa);
  double ex = ce * px + se * py, ey = -se * px + ce * py, ez = pz;
  double radius = sqrt(ex * ex + ey * ey + ez * ez), rxy = sqrt(ex * ex + ey * ey);
  double sLa = ez / radius, cLa = rxy / radius, sLo = ey / rxy, cLo = ex / rxy;
  double Tec2l[3][3] = {{-cLo * sLa, -sLo * sLa, cLa}, {-sLo, cLo, 0.0}, {-cLo * cLa, -sLo * cLa, -sLa}};
  double Tl2ec[3][3];
  for (int i = 0; i < 3; i++)
    for (int j = 0; j < 3; j++) Tl2ec[i][j] = Tec2l[j][i];
  double Tec2i[3][3] = {{ce, -se, 0}, {se, ce, 0}, {0, 0, 1}};
  double Tl2i[3][3], Ti2b[3][3], Tl2b[3][3];
  mat_mul(Tec2i, Tl2ec, Tl2i);
  double a0 = q0 * q0, a1 = q1 * q1, a2 = q2 * q2, a3 = q3 * q3;
  double b01 = q0 * q1, b02 = q0 * q2, b03 = q0 * q3, b12 = q1 * q2, b13 = q1 * q3, b23 = q2 * q3;
  Ti2b[0][0] = a0 + a1 - a2 - a3; Ti2b[0][1] = 2.0 * (b12 + b03); Ti2b[0][2] = 2.0 * (b13 - b02);
  Ti2b[1][0] = 2.0 * (b12 - b03); Ti2b[1][1] = a0 - a1 + a2 - a3; Ti2b[1][2] = 2.0 * (b23 + b01);
  Ti2b[2][0] = 2.0 * (b13 + b02); Ti2b[2][1] = 2.0 * (b23 - b01); Ti2b[2][2] = a0 - a1 - a2 + a3;
  mat_mul(Ti2b, Tl2i, Tl2b);
  double d02 = clampd(Tl2b[0][2], -1.0, 1.0);
  double theta = asin(-d02);
  double phi = atan2(Tl2b[1][2], Tl2b[2][2]);
  double psi = atan2(Tl2b[0][1], Tl2b[0][0]);
  if (psi < 0.0) psi += PI2;
  double dv[3] = {vx - (-ROT * py), vy - (ROT * px), vz}, vb[3];
  mv(Ti2b, dv, vb);
  double alt_m = (radius - SLR_FT) * FT2M;
  /* official bridge: tangent-origin N/E from the geodetic position at MSL altitude; D = -MSL */
  double exm = ex * FT2M, eym = ey * FT2M, ezm = ez * FT2M;
  double b = WA * sqrt(1.0 - WE2);
  double ep2 = (WA * WA - b * b) / (b * b);
  double pxy = sqrt(exm * exm + eym * eym);
  double lon = atan2(eym, exm);
  double th = atan2(ezm * WA, pxy * b);
  double s3 = sin(th) * sin(th) * sin(th), c3 = cos(th) * cos(th) * cos(th);
  double lat = atan2(ezm + ep2 * b * s3, pxy - WE2 * WA * c3);
  double slat = sin(lat), clat = cos(lat), slon = sin(lon), clon = cos(lon);
  double Nr = WA / sqrt(1.0 - WE2 * slat * slat);
  double hx = (Nr + alt_m) * clat * clon, hy = (Nr + alt_m) * clat * slon, hz = (Nr * (1.0 - WE2) + alt_m) * slat;
  double dx = hx - O->ox, dy = hy - O->oy, dz = hz - O->oz;
  s9[0] = -O->sl * O->co * dx - O->sl * O->so * dy + O->cl * dz;
  s9[1] = -O->so * dx + O->co * dy;
  s9[2] = -alt_m;
  s9[3] = phi * R2D; s9[4] = theta * R2D; s9[5] = psi * R2D;
  s9[6] = vb[0] * FT2M; s9[7] = vb[1] * FT2M; s9[8] = vb[2] * FT2M;
}

static double ata_deg(const double so[9], const double st[9]) {
  double p[3] = {st[0] - so[0], st[1] - so[1], st[2] - so[2]};
  double n = norm3(p);
  if (n > 0.0) { p[0] /= n; p[1] /= n; p[2] /= n; }
  double R[3][3], pt[3];
  ned2body(so[3], so[4], so[5], R);
  mv(R, p, pt);
  return acos(clampd(pt[0], -1.0, 1.0)) * R2D;
}
static double aspect_deg(const double so[9], const double st[9]) {
  double R[3][3], b[3];
  ned2body(st[3], st[4], st[5], R);
  double p[3] = {so[0] - st[0], so[1] - st[1], so[2] - st[2]};
  double n = norm3(p);
  if (n > 0.0) { p[0] /= n; p[1] /= n; p[2] /= n; }
  mv(R, p, b);
  double t0 = -b[0], t1 = -b[1], t2 = b[2];
  double sg = (t1 > 0.0) ? 1.0 : ((t1 < 0.0) ? -1.0 : ((t2 >= 0.0) ? 1.0 : -1.0));
  return sg * acos(clampd(t0, -1.0, 1.0)) * R2D;
}
static void los_az_el(const double so[9], const double st[9], double* az, double* el) {
  double d[3] = {st[0] - so[0], st[1] - so[1], st[2] - so[2]};
  double n = norm3(d);
  if (n > 0.0) { d[0] /= n; d[1] /= n; d[2] /= n; }
  double R[3][3], db[3];
  ned2body(so[3], so[4], so[5], R);
  mv(R, d, db);
  *az = atan2(db[1], db[0]) * R2D;
  *el = -asin(clampd(db[2], -1.0, 1.0)) * R2D;
}
/* frame whose x axis is along x, roll fixed by gravity (down, then north, then east) */
static void dir_frame(const double x[3], double R[3][3]) {
  double nx = norm3(x);
  if (nx < 1e-8) {
    memset(R, 0, sizeof(double) * 9);
    R[0][0] = R[1][1] = R[2][2] = 1.0;
    return;
  }
  double xn[3] = {x[0] / nx, x[1] / nx, x[2] / nx};
  static const double refs[3][3] = {{0, 0, 1}, {1, 0, 0}, {0, 1, 0}};
  double z[3] = {0, 0, 0};
  for (int r = 0; r < 3; r++) {
    double d = refs[r][0] * xn[0] + refs[r][1] * xn[1] + refs[r][2] * xn[2];
    double zz[3] = {refs[r][0] - d * xn[0], refs[r][1] - d * xn[1], refs[r][2] - d * xn[2]};
    double nn = norm3(zz);
    if (r < 2 && nn < 1e-6) continue;
    z[0] = zz[0]; z[1] = zz[1]; z[2] = zz[2];
    break;
  }
  double nz = norm3(z);
  z[0] /= nz; z[1] /= nz; z[2] /= nz;
  double y[3] = {z[1] * xn[2] - z[2] * xn[1], z[2] * xn[0] - z[0] * xn[2], z[0] * xn[1] - z[1] * xn[0]};
  double ny = norm3(y);
  y[0] /= ny; y[1] /= ny; y[2] /= ny;
  z[0] = xn[1] * y[2] - xn[2] * y[1]; z[1] = xn[2] * y[0] - xn[0] * y[2]; z[2] = xn[0] * y[1] - xn[1] * y[0];
  for (int j = 0; j < 3; j++) { R[0][j] = xn[j]; R[1][j] = y[j]; R[2][j] = z[j]; }
}
static void bank_sincos(const double Rb2n[3][3], const double dir[3], double* s, double* c) {
  double Rf[3][3], yv[3];
  dir_frame(dir, Rf);
  double by[3] = {Rb2n[0][1], Rb2n[1][1], Rb2n[2][1]};
  mv(Rf, by, yv);
  double mu = atan2(yv[2], yv[1]);
  *s = sin(mu);
  *c = cos(mu);
}
static void log_so3(const double R[3][3], double dt, double out[3]) {
  double tr = R[0][0] + R[1][1] + R[2][2];
  double theta = acos(clampd((tr - 1.0) * 0.5, -1.0, 1.0));
  double ax[3] = {R[2][1] - R[1][2], R[0][2] - R[2][0], R[1][0] - R[0][1]};
  double den = 2.0 * sin(theta), sc = 0.0;
  if (theta >= 1e-8 && fabs(den) >= 1e-8) sc = theta / den;
  double inv = 1.0 / (dt > 1e-8 ? dt : 1e-8);
  for (int i = 0; i < 3; i++) out[i] = ax[i] * sc * inv;
}
static double normz(double x, double lo, double hi) {
  if (hi <= lo) return 0.0;
  double mid = (hi + lo) * 0.5, half = (hi - lo) * 0.5;
  return (clampd(x, lo, hi) - mid) / half;
}
static double damage(double r_ft, double ata_abs, double t) {
  double a = fabs(ata_abs);
  if (r_ft >= MIN_DMG_R_FT && r_ft <= T1_MAX && a < T1_CONE) return 1.0 * (T1_MAX - r_ft) / (T1_MAX - MIN_DMG_R_FT);
  if (t >= T2_START && r_ft >= MIN_DMG_R_FT && r_ft <= T2_MAX && a < T2_CONE)
    return 0.3 * (T2_MAX - r_ft) / (T2_MAX - MIN_DMG_R_FT);
  if (t >= T3_START && r_ft >= MIN_DMG_R_FT && r_ft <= T3_MAX && a < T3_CONE)
    return 0.1 * (T3_MAX - r_ft) / (T3_MAX - MIN_DMG_R_FT);
  return 0.0;
}
static double smooth3(double x, double a, double b) {
  double z = clampd((x - a) / (b - a), 0.0, 1.0);
  return z * z * (3.0 - 2.0 * z);
}
static void unit_or(const double v[3], const double fb[3], double out[3]) {
  double n = norm3(v);
  const double* src = v;
  if (!(n >= 1e-9) || !isfinite(n)) { src = fb; n = norm3(fb); }
  if (!(n >= 1e-9) || !isfinite(n)) { out[0] = 1.0; out[1] = 0.0; out[2] = 0.0; return; }
  out[0] = src[0] / n; out[1] = src[1] / n; out[2] = src[2] / n;
}
static double align3(const double a[3], const double b[3]) {
  static const double ex[3] = {1.0, 0.0, 0.0};
  double au[3], bu[3];
  unit_or(a, ex, au);
  unit_or(b, au, bu);
  double q = 0.5 * (1.0 + clampd(au[0] * bu[0] + au[1] * bu[1] + au[2] * bu[2], -1.0, 1.0));
  return clampd(q * q * q, 0.0, 1.0);
}
static void velocity_ned(const double s[9], double vn[3], double fwd[3]) {
  double R[3][3];
  ned2body(s[3], s[4], s[5], R);
  double vb[3] = {s[6], s[7], s[8]};
  mvT(R, vb, vn);
  fwd[0] = R[0][0]; fwd[1] = R[0][1]; fwd[2] = R[0][2];
}
static double safe_lead(const double so[9], const double st[9], const double ov[3], const double tv[3],
                        const double fwd[3], double dist_m, double dist_ft, double ata) {
  double rel[3] = {st[0] - so[0], st[1] - so[1], st[2] - so[2]}, los[3], path[3], lead[3];
  unit_or(rel, fwd, los);
  unit_or(ov, fwd, path);
  double spd = norm3(ov);
  if (spd < 30.0) spd = 30.0;
  double tau = clampd(dist_m / spd, 0.30, 1.50);
  double lv[3] = {rel[0] + tv[0] * tau, rel[1] + tv[1] * tau, rel[2] + tv[2] * tau};
  unit_or(lv, los, lead);
  double intercept = 0.40 * align3(fwd, lead) + 0.60 * align3(path, lead);
  double direct = align3(fwd, los);
  double w = smooth3(dist_ft, 1000.0, 2500.0) * smooth3(fabs(ata), 3.0, 8.0);
  return clampd(w * intercept + (1.0 - w) * direct, 0.0, 1.0);
}
static double broad(double ata) {
  ata = clampd(fabs(ata), 0.0, 180.0);
  return (ata <= 30.0) ? 1.0 : clampd((180.0 - ata) / 150.0, 0.0, 1.0);
}
static double side_score(const double so[9], const double st[9], const double ov[3], const double tv[3],
                         const double fwd[3], double dist_m, double dist_ft, double ata, double t, double rg,
                         double cq) {
  double lead = safe_lead(so, st, ov, tv, fwd, dist_m, dist_ft, ata);
  double gate = 1.0 - smooth3(fabs(ata), 3.0, 8.0);
  double control = clampd(gate * rg * cq, 0.0, 1.0);
  double fine = damage(dist_ft, fabs(ata), t);
  return clampd(0.50 * broad(ata) + 0.20 * lead + 0.20 * control + 0.10 * fine, 0.0, 1.0);
}
static double geometry_advantage(const double so[9], const double st[9], double t) {
  double rel[3] = {st[0] - so[0], st[1] - so[1], st[2] - so[2]};
  double dm = norm3(rel), df = dm / FT2M;
  static const double ex[3] = {1.0, 0.0, 0.0};
  double los[3], vo[3], vp[3], fo[3], fp[3];
  unit_or(rel, ex, los);
  velocity_ned(so, vo, fo);
  velocity_ned(st, vp, fp);
  double closing = (vo[0] - vp[0]) * los[0] + (vo[1] - vp[1]) * los[1] + (vo[2] - vp[2]) * los[2];
  double ms = 0.5 * (norm3(vo) + norm3(vp));
  if (ms < 100.0) ms = 100.0;
  double ratio = closing / ms;
  double desired = 0.20 * smooth3(df, 2000.0, 4500.0) - 0.12 * (1.0 - smooth3(df, 650.0, 900.0));
  double dq = (ratio - desired) / 0.15;
  double cq = exp(-0.5 * dq * dq);
  double rg = smooth3(df, 600.0, 900.0) * (1.0 - smooth3(df, 3200.0, 4300.0));
  double a1 = ata_deg(so, st), a2 = ata_deg(st, so);
  double S1 = side_score(so, st, vo, vp, fo, dm, df, a1, t, rg, cq);
  double S2 = side_score(st, so, vp, vo, fp, dm, df, a2, t, rg, cq);
  return clampd(S1 - S2, -1.0, 1.0);
}
static double alt_log(double alt_m) {
  double s = alt_m / ALT_LOG_SCALE_M;
  return log(s < ALT_LOG_FLOOR ? ALT_LOG_FLOOR : s);
}
static float store(double v) {
  if (!isfinite(v)) v = (v > 0.0) ? 10.0 : ((v < 0.0) ? -10.0 : 0.0);
  return (float)v;
}

/* one perspective's 184 features (:336-482) */
static void obs_one(const double so[9], const double st[9], double hp_o, double hp_t, double fu_o, double fu_t,
                    const double pqr_o[3], const double pqr_t[3], double dealt, double taken, double t,
                    const double* acth, float* out, double* aux) {
  double Ro[3][3], Rt[3][3];
  ned2body(so[3], so[4], so[5], Ro);
  ned2body(st[3], st[4], st[5], Rt);
  double ovb[3] = {so[6], so[7], so[8]}, tvb[3] = {st[6], st[7], st[8]}, ovn[3], tvn[3];
  mvT(Ro, ovb, ovn);
  mvT(Rt, tvb, tvn);
  if (aux) {
    for (int i = 0; i < 3; i++) {
      aux[i] = so[i]; aux[3 + i] = ovn[i]; aux[6 + i] = st[i]; aux[9 + i] = tvn[i];
      for (int j = 0; j < 3; j++) aux[12 + 3 * i + j] = Ro[i][j];
    }
  }
  double rvn[3] = {tvn[0] - ovn[0], tvn[1] - ovn[1], tvn[2] - ovn[2]};
  double os = norm3(ovb), ts = norm3(tvb), oalt = -so[2], talt = -st[2];
  double del[3] = {st[0] - so[0], st[1] - so[1], st[2] - so[2]};
  double dist = norm3(del), los[3] = {0, 0, 0}, clos = 0.0;
  if (dist > 1e-6) {
    los[0] = del[0] / dist; los[1] = del[1] / dist; los[2] = del[2] / dist;
    clos = (ovn[0] - tvn[0]) * los[0] + (ovn[1] - tvn[1]) * los[1] + (ovn[2] - tvn[2]) * los[2];
  }
  double ata = ata_deg(so, st), eata = ata_deg(st, so), aa = aspect_deg(so, st), az, el;
  los_az_el(so, st, &az, &el);
  double u = ovb[0], v = ovb[1], w = ovb[2], aoa = 0.0, ss = 0.0;
  if (os >= 1.0) { aoa = atan2(w, u) * R2D; ss = atan2(v, sqrt(u * u + w * w)) * R2D; }
  double vs = -ovn[2];
  double eo = oalt + os * os / (2.0 * GACC), et = talt + ts * ts / (2.0 * GACC), ea = eo - et;
  double cone = (t >= T3_START) ? T3_CONE : ((t >= T2_START) ? T2_CONE : T1_CONE);
  double mr = (t >= T3_START) ? T3_MAX : ((t >= T2_START) ? T2_MAX : T1_MAX);
  double csafe = cone > 1e-6 ? cone : 1e-6;
  double ash = 2.0 * exp(-((ata / 3.0) * (ata / 3.0))) - 1.0;
  double amg = tanh((cone - fabs(ata)) / csafe);
  double eash = 2.0 * exp(-((eata / 3.0) * (eata / 3.0))) - 1.0;
  double eamg = tanh((cone - fabs(eata)) / csafe);
  double rmin = MIN_DMG_R_FT * FT2M, rmax = mr * FT2M, span = rmax - rmin;
  if (span < 1e-6) span = 1e-6;
  double rn = tanh((dist - rmin) / span), rf = tanh((rmax - dist) / span);
  double Rbo[3][3], Rbt[3][3], obs_, obc, tbs, tbc;
  for (int i = 0; i < 3; i++)
    for (int j = 0; j < 3; j++) { Rbo[i][j] = Ro[j][i]; Rbt[i][j] = Rt[j][i]; }
  bank_sincos(Rbo, ovn, &obs_, &obc);
  bank_sincos(Rbt, tvn, &tbs, &tbc);
  double pa = 1.0 - fabs(ata) / PURSUIT_ATA, pr = 1.0 - dist / PURSUIT_RANGE;
  if (pa < 0.0) pa = 0.0;
  if (pr < 0.0) pr = 0.0;
  double pursuit = 2.0 * (pa * pr) - 1.0;
  double sc[50] = {
      normz(os, 0.0, MAX_SPEED), normz(ts, 0.0, MAX_SPEED), tanh(aoa / AOA_SCALE), tanh(ss / SSLIP_SCALE),
      tanh((oalt - MIN_ALT_M) / ALT_DANGER), normz(vs, -VSPEED_SCALE, VSPEED_SCALE), normz(hp_o, 0.0, 1.0),
      normz(hp_t, 0.0, 1.0), hp_o - hp_t, ea / (fabs(ea) + ENERGY_ADV), normz(dist, 0.0, MAX_RANGE_M),
      normz(clos, -MAX_CLOSURE, MAX_CLOSURE), sin(ata * D2R), cos(ata * D2R), sin(aa * D2R), cos(aa * D2R),
      sin(az * D2R), cos(az * D2R), sin(el * D2R), cos(el * D2R), ash, amg, eash, eamg, rn, rf,
      normz(t, 0.0, EPISODE_MAX), sin(so[3] * D2R), cos(so[3] * D2R), sin(so[4] * D2R), cos(so[4] * D2R),
      sin(so[5] * D2R), cos(so[5] * D2R), sin(st[3] * D2R), cos(st[3] * D2R), sin(st[4] * D2R),
      cos(st[4] * D2R), sin(st[5] * D2R), cos(st[5] * D2R), obs_, obc, tbs, tbc, normz(fu_o, 0.0, 1.0),
      normz(fu_t, 0.0, 1.0), clampd(2.0 * dealt - 1.0, -1.0, 1.0), clampd(2.0 * taken - 1.0, -1.0, 1.0),
      pursuit, normz(oalt, 0.0, MAX_ALT_M), normz(talt, 0.0, MAX_ALT_M)};
  for (int i = 0; i < 50; i++) out[i] = store(sc[i]);
  /* 38 frame-projected vectors (:447-479): frames world, mybody, oppbody, myvel, oppvel, los;
     vectors gravity, los, own_vel, tgt_vel, rel_vel, own_omega, tgt_omega; kinds unit/vel/omega */
  double oom[3], tom[3];
  mvT(Ro, pqr_o, oom);
  mvT(Rt, pqr_t, tom);
  double I3[3][3] = {{1, 0, 0}, {0, 1, 0}, {0, 0, 1}}, Fm[3][3], Fo[3][3], Fl[3][3];
  dir_frame(ovn, Fm);
  dir_frame(tvn, Fo);
  dir_frame(del, Fl);
  const double (*F[6])[3] = {I3, Ro, Rt, Fm, Fo, Fl};
  double grav[3] = {0, 0, 1};
  const double* V[7] = {grav, los, ovn, tvn, rvn, oom, tom};
  static const int LAY[38][3] = {
      {0, 1, 0}, {0, 2, 0}, {0, 3, 0}, {0, 4, 0}, {0, 5, 0}, {1, 0, 0}, {1, 1, 0}, {1, 2, 0}, {1, 3, 0}, {1, 4, 0},
      {2, 0, 1}, {2, 1, 1}, {2, 2, 1}, {2, 4, 1}, {2, 5, 1}, {3, 0, 1}, {3, 1, 1}, {3, 2, 1}, {3, 3, 1}, {3, 5, 1},
      {4, 0, 1}, {4, 1, 1}, {4, 2, 1}, {4, 3, 1}, {4, 4, 1}, {4, 5, 1}, {5, 0, 2}, {5, 1, 2}, {5, 2, 2}, {5, 3, 2},
      {5, 4, 2}, {5, 5, 2}, {6, 0, 2}, {6, 1, 2}, {6, 2, 2}, {6, 3, 2}, {6, 4, 2}, {6, 5, 2}};
  for (int i = 0; i < 38; i++) {
    const double (*M)[3] = F[LAY[i][1]];
    const double* vv = V[LAY[i][0]];
    for (int r = 0; r < 3; r++) {
      double c = M[r][0] * vv[0] + M[r][1] * vv[1] + M[r][2] * vv[2];
      double val = LAY[i][2] == 0 ? c : (LAY[i][2] == 1 ? normz(c, -REL_VEL, REL_VEL) : tanh(c / PQR_SCALE));
      out[50 + 3 * i + r] = store(val);
    }
  }
  for (int j = 0; j < 20; j++) out[164 + j] = store(acth[j]);
}

static Origin origin(const double* o7) {
  Origin O = {o7[0], o7[1], o7[2], o7[3], o7[4], o7[5], o7[6]};
  return O;
}

/* init_reward_kernel (:485-501) */
void oracle_obs_init_reward(const double* states, const uint8_t* env_mask, double* prev_x, uint8_t* prev_x_valid,
                            double* prev_alt_log, const double* t_sec, long nenv, const double* origin7) {
  Origin O = origin(origin7);
  for (long e = 0; e < nenv; e++) {
    if (env_mask && !env_mask[e]) continue;
    long o = 2 * e, p = o + 1;
    double so[9], sp[9];
    kin9(states + o * 101, &O, so);
    kin9(states + p * 101, &O, sp);
    double g = geometry_advantage(so, sp, t_sec[e]);
    prev_x[o] = g; prev_x[p] = -g;
    prev_x_valid[o] = 1; prev_x_valid[p] = 1;
    prev_alt_log[o] = alt_log(-so[2]); prev_alt_log[p] = alt_log(-sp[2]);
  }
}

/* advance_kernel (:504-626); rp = {dt, min_alt, max_time, own_w, dmg_scale, shap_scale, win, loss,
   timeout_win, timeout_loss, timeout_draw, alt_hunt_coef} */
void oracle_obs_advance(const double* states, const double* actions, double* hp, double* fuel, double* t_sec,
                        double* prev_att, uint8_t* prev_valid, double* pqr, double* dealt, double* taken,
                        double* hp_loss, double* act_hist, double* prev_x, uint8_t* prev_x_valid,
                        double* prev_alt_log, double* reward, uint8_t* term, uint8_t* trunc_, long nenv,
                        const double* origin7, const double* rp, int mode) {
  Origin O = origin(origin7);
  double dt = rp[0], min_alt = rp[1], max_time = rp[2], own_w = rp[3], dsc = rp[4], shs = rp[5];
  double win_r = rp[6], loss_r = rp[7], tw = rp[8], tl = rp[9], td = rp[10], coef = rp[11];
  for (long e = 0; e < nenv; e++) {
    long o = 2 * e, p = o + 1;
    for (int k = 0; k < 2; k++) {
      long a = k == 0 ? o : p;
      double* ah = act_hist + a * 20;
      memmove(ah + 4, ah, 16 * sizeof(double));
      for (int c = 0; c < 4; c++) ah[c] = actions[a * 4 + c];
    }
    double so[9], sp[9];
    kin9(states + o * 101, &O, so);
    kin9(states + p * 101, &O, sp);
    double dpos[3] = {sp[0] - so[0], sp[1] - so[1], sp[2] - so[2]};
    double r_ft = norm3(dpos) * M2FT;
    double ata_op = ata_deg(so, sp), ata_po = ata_deg(sp, so);
    double t0 = t_sec[e];
    double ro = damage(r_ft, ata_op, t0), rpd = damage(r_ft, ata_po, t0);
    double ho0 = hp[o], hp0 = hp[p];
    double ho = ho0 - rpd * dt, hpn = hp0 - ro * dt;
    if (ho < 0.0) ho = 0.0;
    if (hpn < 0.0) hpn = 0.0;
    double lo = ho0 - ho, lp = hp0 - hpn;
    hp[o] = ho; hp[p] = hpn;
    hp_loss[o] = lo; hp_loss[p] = lp;
    dealt[o] = ro; taken[o] = rpd; dealt[p] = rpd; taken[p] = ro;
    double vo = sqrt(so[6] * so[6] + so[7] * so[7] + so[8] * so[8]);
    double vpp = sqrt(sp[6] * sp[6] + sp[7] * sp[7] + sp[8] * sp[8]);
    double fo = fuel[o] - FUEL_BURN * (vo / FUEL_REF) * dt, fp = fuel[p] - FUEL_BURN * (vpp / FUEL_REF) * dt;
    fuel[o] = fo < 0.0 ? 0.0 : fo;
    fuel[p] = fp < 0.0 ? 0.0 : fp;
    for (int k = 0; k < 2; k++) {
      long a = k == 0 ? o : p;
      const double* s = k == 0 ? so : sp;
      double Np[3][3], Nc[3][3], rd[3][3], lg[3] = {0, 0, 0};
      ned2body(prev_att[a * 3], prev_att[a * 3 + 1], prev_att[a * 3 + 2], Np);
      ned2body(s[3], s[4], s[5], Nc);
      for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) {
          double acc = 0;
          for (int m = 0; m < 3; m++) acc += Np[i][m] * Nc[j][m];
          rd[i][j] = acc;
        }
      if (prev_valid[a]) log_so3(rd, dt, lg);
      for (int i = 0; i < 3; i++) { pqr[a * 3 + i] = lg[i]; prev_att[a * 3 + i] = s[3 + i]; }
      prev_valid[a] = 1;
    }
    double t1 = t0 + dt;
    t_sec[e] = t1;
    double ao = -so[2], ap = -sp[2];
    int fin = 1;
    for (int k = 0; k < 9; k++)
      if (!isfinite(so[k]) || !isfinite(sp[k])) fin = 0;
    uint8_t te = (ao < min_alt) || (ap < min_alt) || (ho <= 0.0) || (hpn <= 0.0) || (!fin);
    uint8_t tr = (!te) && (t1 >= max_time - TLIM_TOL);
    term[e] = te;
    trunc_[e] = tr;
    double go = geometry_advantage(so, sp, t1), gp = -go;
    double lgo = alt_log(ao), lgp = alt_log(ap);
    double pgo = prev_x_valid[o] ? prev_x[o] : go, pgp = prev_x_valid[p] ? prev_x[p] : gp;
    double gm = shs / SHAPING_BASE;
    double rgo = gm * (GEOM_BUDGET / GEOM_REF_SEC) * 0.5 * (pgo + go) * dt;
    double rgp = gm * (GEOM_BUDGET / GEOM_REF_SEC) * 0.5 * (pgp + gp) * dt;
    if (mode == 1) {
      rgo = prev_x_valid[p] ? coef * (prev_alt_log[p] - lgp) : 0.0;
      rgp = prev_x_valid[o] ? coef * (prev_alt_log[o] - lgo) : 0.0;
    }
    prev_x[o] = go; prev_x[p] = gp; prev_x_valid[o] = 1; prev_x_valid[p] = 1;
    prev_alt_log[o] = lgo; prev_alt_log[p] = lgp;
    double rdo = (lp - lo * own_w) * dsc, rdp = (lo - lp * own_w) * dsc;
    if (mode == 2) { rdo = lp * dsc; rdp = lo * dsc; }
    else if (mode == 3) { rdo = -(lo * own_w) * dsc; rdp = -(lp * own_w) * dsc; }
    double rto = 0.0, rtp = 0.0;
    if (te) {
      if (ao < min_alt) rto = -ho * dsc;
      else if (ap < min_alt) rto = hpn * dsc;
      else { if (hpn <= 0.0) rto += win_r; if (ho <= 0.0) rto += loss_r; }
      if (ap < min_alt) rtp = -hpn * dsc;
      else if (ao < min_alt) rtp = ho * dsc;
      else { if (ho <= 0.0) rtp += win_r; if (hpn <= 0.0) rtp += loss_r; }
    } else if (tr) {
      rto = (ho > hpn) ? tw : ((ho < hpn) ? tl : td);
      rtp = (hpn > ho) ? tw : ((hpn < ho) ? tl : td);
    }
    reward[o] = rdo + rgo + rto;
    reward[p] = rdp + rgp + rtp;
  }
}

/* build_obs_kernel (:628-649) */
void oracle_obs_build(const double* states, const uint8_t* env_mask, const double* hp, const double* fuel,
                      const double* t_sec, const double* pqr, const double* dealt, const double* taken,
                      const double* act_hist, float* obs, long nac, const double* origin7, double* aux) {
  Origin O = origin(origin7);
  for (long a = 0; a < nac; a++) {
    long e = a >> 1, par = a ^ 1;
    if (env_mask && !env_mask[e]) continue;
    double so[9], st[9];
    kin9(states + a * 101, &O, so);
    kin9(states + par * 101, &O, st);
    obs_one(so, st, hp[a], hp[par], fuel[a], fuel[par], pqr + a * 3, pqr + par * 3, dealt[a], taken[a], t_sec[e],
            act_hist + a * 20, obs + a * 184, (aux && !(a & 1)) ? aux + e * 21 : 0);
  }
}

/* kin9 of every aircraft, for tests */
void oracle_kin9(const double* states, long nac, const double* origin7, double* s9) {
  Origin O = origin(origin7);
  for (long a = 0; a < nac; a++) kin9(states + a * 101, &O, s9 + a * 9);
}

/* ---------------------------------------------------------------------------------------------
 * External 214-D observation for frozen external opponents
 * (research/competition_36500/runtime/cuda_fdm/external_observation.cu, run by
 * BatchObsReward.kernel_advance / build_external_obs, obs_reward.py:417-420, 487-496).
 * ------------------------------------------------------------------------------------------- */

/* external_acceleration (:2-9): NED velocity of each aircraft from its 9-DoF state; the
   finite-difference acceleration against the stored previous velocity where the aircraft's
   attitude history is valid (0 otherwise); the velocity becomes the stored previous one. */
void oracle_external_accel(const double* states, const uint8_t* valid, double* previous, double* accel, long nac,
                           const double* origin7, double dt) {
  Origin O = origin(origin7);
  for (long a = 0; a < nac; a++) {
    double s[9], R[3][3], v[3];
    kin9(states + a * 101, &O, s);
    ned2body(s[3], s[4], s[5], R);
    mvT(R, s + 6, v);
    for (int i = 0; i < 3; i++) {
      accel[a * 3 + i] = valid[a] ? (v[i] - previous[a * 3 + i]) / dt : 0.0;
      previous[a * 3 + i] = v[i];
    }
  }
}

/* external_observation (:10-28): the 184-D row with 30 acceleration features inserted before
   the 20-value action history: own acceleration in the world, own-body, target-body,
   target-velocity and line-of-sight frames, then the target's in the world, own-body,
   target-body, own-velocity and line-of-sight frames, each clamped to +-150 m/s^2 and scaled
   to [-1, 1]. */
void oracle_external_obs(const double* states, const double* accel, const float* original, float* out, long nac,
                         const double* origin7) {
  Origin O = origin(origin7);
  for (long a = 0; a < nac; a++) {
    long b = a ^ 1;
    double s[9], t[9], Ro[3][3], Rt[3][3], vo[3], vt[3], delta[3];
    kin9(states + a * 101, &O, s);
    kin9(states + b * 101, &O, t);
    ned2body(s[3], s[4], s[5], Ro);
    ned2body(t[3], t[4], t[5], Rt);
    mvT(Ro, s + 6, vo);
    mvT(Rt, t + 6, vt);
    for (int i = 0; i < 3; i++) delta[i] = t[i] - s[i];
    double I[3][3] = {{1, 0, 0}, {0, 1, 0}, {0, 0, 1}}, Fo[3][3], Ft[3][3], Fl[3][3];
    dir_frame(vo, Fo);
    dir_frame(vt, Ft);
    dir_frame(delta, Fl);
    const double (*F[6])[3] = {I, Ro, Rt, Fo, Ft, Fl};
    static const int order[10] = {0, 1, 2, 4, 5, 0, 1, 2, 3, 5};
    float* row = out + a * 214;
    for (int i = 0; i < 164; i++) row[i] = original[a * 184 + i];
    for (int i = 0; i < 10; i++) {
      double v[3];
      mv(F[order[i]], accel + (i < 5 ? a : b) * 3, v);
      for (int j = 0; j < 3; j++) row[164 + i * 3 + j] = store(normz(v[j], -150.0, 150.0));
    }
    for (int i = 0; i < 20; i++) row[194 + i] = original[a * 184 + 164 + i];
  }
}
