// obs_kernels.cu -- observation / reward / termination kernels and their C-ABI entry points.
//
// All kernels run one thread per environment (both aircraft): the two 9-DoF states are built
// from the FDM rows once (14 state columns each, coalesced in the SoA layout), the shared
// geometry once (obs_device.cuh Pair), and each aircraft's 184-float row is written with 16-byte
// vector stores.  Reconstruction buffers keep the reference's per-aircraft layout
// (R/cuda_fdm/obs_reward.py:338-353) so the reference's tensors can be passed as they are.
#include "common.cuh"
#include "obs_device.cuh"

namespace f16 {
namespace obs {

constexpr int OBS_THREADS = 128;
// Resident blocks per SM the step kernels are compiled for (64 registers per thread): the row
// builder's live set does not fit in registers at any occupancy, and trading register spills
// (to L1, which these kernels do not otherwise use) for 32 resident warps measured fastest on a
// B200 (sweep 1..16: post-step 0.58 -> 0.44 ms, obs step 1.00 -> 0.84 ms).
#ifndef F16_OBS_MIN_BLOCKS
#define F16_OBS_MIN_BLOCKS 8
#endif

template <int LAYOUT>
struct RowRef {
  const double* __restrict__ p;
  int64_t ld, a;
  __device__ __forceinline__ double operator()(int c) const {
    return LAYOUT == F16_LAYOUT_SOA ? p[(int64_t)c * ld + a] : p[a * F16_STATE_N + c];
  }
};

__device__ __forceinline__ Origin origin_of(const f16_origin& o) { return {o.ox, o.oy, o.oz, o.slat, o.clat, o.slon, o.clon}; }

template <int LAYOUT>
__device__ __forceinline__ void load_pair(const double* st, int64_t ld, int64_t e, const Origin& O, Pair& P) {
  kin9(RowRef<LAYOUT>{st, ld, 2 * e}, O, P.s[0]);
  kin9(RowRef<LAYOUT>{st, ld, 2 * e + 1}, O, P.s[1]);
  make_pair(P);
}

// action-history push of one aircraft (roll by one, newest first): hist[0..19] <- (a, hist[0..15])
__device__ __forceinline__ void push_hist(double* __restrict__ h, const double* __restrict__ act, double out[20]) {
  const double2* h2 = reinterpret_cast<const double2*>(h);
  double2 o[8];
#pragma unroll
  for (int i = 0; i < 8; i++) o[i] = h2[i];
  const double2* a2 = reinterpret_cast<const double2*>(act);
  double2 x = a2[0], y = a2[1];
  out[0] = x.x; out[1] = x.y; out[2] = y.x; out[3] = y.y;
#pragma unroll
  for (int i = 0; i < 8; i++) { out[4 + 2 * i] = o[i].x; out[5 + 2 * i] = o[i].y; }
  double2* w = reinterpret_cast<double2*>(h);
#pragma unroll
  for (int i = 0; i < 10; i++) w[i] = make_double2(out[2 * i], out[2 * i + 1]);
}

struct AdvanceOut {
  double hp[2], fuel[2], dealt[2], taken[2], t;
  V3 pqr[2];
  double hist[2][20];
};

// advance_kernel semantics (obs_kernel.cu:504-626) for environment e on a built Pair.
__device__ __forceinline__ void advance_env(const Pair& P, int64_t e, const f16_recon& rc, const f16_reward_cfg& cfg,
                                            const double* __restrict__ actions, double* __restrict__ reward,
                                            uint8_t* __restrict__ term, uint8_t* __restrict__ trunc_,
                                            AdvanceOut& A) {
  const int64_t o = 2 * e, p = o + 1;
  const double dt = cfg.dt;
  push_hist(rc.act_hist + o * 20, actions + o * 4, A.hist[0]);
  push_hist(rc.act_hist + p * 20, actions + p * 4, A.hist[1]);
  double r_ft = P.dist * M2FT;
  double t_old = rc.t_sec[e];
  double rate_o = damage(r_ft, P.ata[0], t_old), rate_p = damage(r_ft, P.ata[1], t_old);
  double ho0 = rc.hp[o], hp0 = rc.hp[p];
  double ho = ho0 - rate_p * dt, hpn = hp0 - rate_o * dt;
  if (ho < 0.0) ho = 0.0;
  if (hpn < 0.0) hpn = 0.0;
  double lo = ho0 - ho, lp = hp0 - hpn;
  rc.hp[o] = ho; rc.hp[p] = hpn;
  rc.hp_loss[o] = lo; rc.hp_loss[p] = lp;
  rc.dmg_dealt[o] = rate_o; rc.dmg_taken[o] = rate_p;
  rc.dmg_dealt[p] = rate_p; rc.dmg_taken[p] = rate_o;
  A.hp[0] = ho; A.hp[1] = hpn;
  A.dealt[0] = rate_o; A.taken[0] = rate_p; A.dealt[1] = rate_p; A.taken[1] = rate_o;
  double fo = rc.fuel[o] - FUEL_BURN * (P.spd[0] / FUEL_REF) * dt;
  double fp = rc.fuel[p] - FUEL_BURN * (P.spd[1] / FUEL_REF) * dt;
  A.fuel[0] = fo < 0.0 ? 0.0 : fo;
  A.fuel[1] = fp < 0.0 ? 0.0 : fp;
  rc.fuel[o] = A.fuel[0]; rc.fuel[p] = A.fuel[1];
  // body rates from the attitude change: log_SO3(R_prev R_curr^T) / dt
  const double inv_dt = 1.0 / (dt > 1e-8 ? dt : 1e-8);
  for (int k = 0; k < 2; k++) {
    int64_t a = o + k;
    double lg[3] = {0.0, 0.0, 0.0};
    if (rc.prev_valid[a]) {
      M3 Np = ned2body(rc.prev_att[a * 3], rc.prev_att[a * 3 + 1], rc.prev_att[a * 3 + 2]);
      const M3& Nc = P.R[k];
      M3 rd;
      for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++)
          rd.m[i][j] = Np.m[i][0] * Nc.m[j][0] + Np.m[i][1] * Nc.m[j][1] + Np.m[i][2] * Nc.m[j][2];
      log_so3(rd, inv_dt, lg);
    }
    rc.pqr[a * 3] = lg[0]; rc.pqr[a * 3 + 1] = lg[1]; rc.pqr[a * 3 + 2] = lg[2];
    A.pqr[k] = {lg[0], lg[1], lg[2]};
    rc.prev_att[a * 3] = P.s[k][3]; rc.prev_att[a * 3 + 1] = P.s[k][4]; rc.prev_att[a * 3 + 2] = P.s[k][5];
    rc.prev_valid[a] = 1;
  }
  double t_new = t_old + dt;
  rc.t_sec[e] = t_new;
  A.t = t_new;
  double ao = -P.s[0][2], ap = -P.s[1][2];
  bool fin = true;
  for (int k = 0; k < 9; k++)
    if (!isfinite(P.s[0][k]) || !isfinite(P.s[1][k])) fin = false;
  uint8_t te = (ao < cfg.min_alt) || (ap < cfg.min_alt) || (ho <= 0.0) || (hpn <= 0.0) || (!fin);
  uint8_t tr = (!te) && (t_new >= cfg.max_time - TLIM_TOL);
  term[e] = te;
  trunc_[e] = tr;
  double go = geometry_advantage(P, t_new), gp = -go;
  double lgo = alt_log(ao), lgp = alt_log(ap);
  uint8_t vo = rc.prev_x_valid[o], vp = rc.prev_x_valid[p];
  double pgo = vo ? rc.prev_x[o] : go, pgp = vp ? rc.prev_x[p] : gp;
  double gm = cfg.shaping_reward_scale / SHAPING_BASE;
  double rgo = gm * (GEOM_BUDGET / GEOM_REF_SEC) * 0.5 * (pgo + go) * dt;
  double rgp = gm * (GEOM_BUDGET / GEOM_REF_SEC) * 0.5 * (pgp + gp) * dt;
  if (cfg.reward_mode == 1) {
    rgo = vp ? cfg.alt_hunt_coef * (rc.prev_alt_log[p] - lgp) : 0.0;
    rgp = vo ? cfg.alt_hunt_coef * (rc.prev_alt_log[o] - lgo) : 0.0;
  }
  rc.prev_x[o] = go; rc.prev_x[p] = gp;
  rc.prev_x_valid[o] = 1; rc.prev_x_valid[p] = 1;
  rc.prev_alt_log[o] = lgo; rc.prev_alt_log[p] = lgp;
  const double dsc = cfg.damage_scale, ow = cfg.own_damage_weight;
  double rdo = (lp - lo * ow) * dsc, rdp = (lo - lp * ow) * dsc;
  if (cfg.reward_mode == 2) { rdo = lp * dsc; rdp = lo * dsc; }
  else if (cfg.reward_mode == 3) { rdo = -(lo * ow) * dsc; rdp = -(lp * ow) * dsc; }
  double rto = 0.0, rtp = 0.0;
  if (te) {
    if (ao < cfg.min_alt) rto = -ho * dsc;
    else if (ap < cfg.min_alt) rto = hpn * dsc;
    else { if (hpn <= 0.0) rto += cfg.win_reward; if (ho <= 0.0) rto += cfg.loss_reward; }
    if (ap < cfg.min_alt) rtp = -hpn * dsc;
    else if (ao < cfg.min_alt) rtp = ho * dsc;
    else { if (ho <= 0.0) rtp += cfg.win_reward; if (hpn <= 0.0) rtp += cfg.loss_reward; }
  } else if (tr) {
    rto = (ho > hpn) ? cfg.timeout_win_reward : ((ho < hpn) ? cfg.timeout_loss_reward : cfg.timeout_draw_reward);
    rtp = (hpn > ho) ? cfg.timeout_win_reward : ((hpn < ho) ? cfg.timeout_loss_reward : cfg.timeout_draw_reward);
  }
  reward[o] = rdo + rgo + rto;
  reward[p] = rdp + rgp + rtp;
}

// Both observation rows of environment e from a built Pair and the two aircraft's recon values.
__device__ __forceinline__ void obs_env(const Pair& P, int64_t e, const Side* sd, double t, float* __restrict__ obs,
                                        double* __restrict__ aux) {
  M3 Fv[2] = {dir_frame(P.vn[0]), dir_frame(P.vn[1])};
  V3 md = {-P.delta.x, -P.delta.y, -P.delta.z};
  M3 Fl0 = dir_frame(P.delta);
  obs_row(P, 0, sd[0], sd[1], t, Fv, Fl0, obs + (2 * e) * 184, aux ? aux + e * 21 : nullptr);
  M3 Fl1 = dir_frame(md);
  obs_row(P, 1, sd[1], sd[0], t, Fv, Fl1, obs + (2 * e + 1) * 184, nullptr);
}

template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS) k_obs_build(const double* __restrict__ st, int64_t ld, int64_t nenv,
                                                           const uint8_t* __restrict__ mask, const f16_recon rc,
                                                           const f16_origin og, float* __restrict__ obs,
                                                           double* __restrict__ aux) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nenv || (mask && !mask[e])) return;
  Origin O = origin_of(og);
  Pair P;
  load_pair<LAYOUT>(st, ld, e, O, P);
  Side sd[2];
  for (int k = 0; k < 2; k++) {
    int64_t a = 2 * e + k;
    sd[k] = {rc.hp[a], rc.fuel[a], rc.dmg_dealt[a], rc.dmg_taken[a],
             {rc.pqr[a * 3], rc.pqr[a * 3 + 1], rc.pqr[a * 3 + 2]}, rc.act_hist + a * 20};
  }
  obs_env(P, e, sd, rc.t_sec[e], obs, aux);
}

template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS) k_obs_advance(const double* __restrict__ st, int64_t ld, int64_t nenv,
                                                             const double* __restrict__ actions, const f16_recon rc,
                                                             const f16_reward_cfg cfg, const f16_origin og,
                                                             double* __restrict__ reward, uint8_t* __restrict__ term,
                                                             uint8_t* __restrict__ trunc_) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nenv) return;
  Origin O = origin_of(og);
  Pair P;
  load_pair<LAYOUT>(st, ld, e, O, P);
  AdvanceOut A;
  advance_env(P, e, rc, cfg, actions, reward, term, trunc_, A);
}

// Fused: advance (reward, termination, reconstruction update) then both observation rows,
// reading each FDM row once (the reference launches advance_kernel then build_obs_kernel).
template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS, F16_OBS_MIN_BLOCKS) k_obs_step(const double* __restrict__ st, int64_t ld, int64_t nenv,
                                                          const double* __restrict__ actions, const f16_recon rc,
                                                          const f16_reward_cfg cfg, const f16_origin og,
                                                          double* __restrict__ reward, uint8_t* __restrict__ term,
                                                          uint8_t* __restrict__ trunc_, float* __restrict__ obs,
                                                          double* __restrict__ aux) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nenv) return;
  Origin O = origin_of(og);
  Pair P;
  load_pair<LAYOUT>(st, ld, e, O, P);
  AdvanceOut A;
  advance_env(P, e, rc, cfg, actions, reward, term, trunc_, A);
  Side sd[2];
  for (int k = 0; k < 2; k++) sd[k] = {A.hp[k], A.fuel[k], A.dealt[k], A.taken[k], A.pqr[k], A.hist[k]};
  obs_env(P, e, sd, A.t, obs, aux);
}

template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS) k_obs_init_reward(const double* __restrict__ st, int64_t ld,
                                                                 int64_t nenv, const uint8_t* __restrict__ mask,
                                                                 const f16_recon rc, const f16_origin og) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nenv || (mask && !mask[e])) return;
  Origin O = origin_of(og);
  Pair P;
  load_pair<LAYOUT>(st, ld, e, O, P);
  double g = geometry_advantage(P, rc.t_sec[e]);
  int64_t o = 2 * e, p = o + 1;
  rc.prev_x[o] = g; rc.prev_x[p] = -g;
  rc.prev_x_valid[o] = 1; rc.prev_x_valid[p] = 1;
  rc.prev_alt_log[o] = alt_log(-P.s[0][2]);
  rc.prev_alt_log[p] = alt_log(-P.s[1][2]);
}

// Everything GpuDogfightVecEnv.step does after the physics step (R/cuda_fdm/rl_env.py:514-551),
// in one launch: advance, terminal observations, terminal HP / MSL altitude, and for finished
// environments the autoreset from the IC pool (state rows, reconstruction reset, reward-tracker
// anchoring, fresh observations).  pool: (pool_size, 2, 101) AoS rows; pick: pool row per env.
template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS, F16_OBS_MIN_BLOCKS) k_env_post(double* __restrict__ st, int64_t ld, int64_t nenv,
                                                          const double* __restrict__ actions, const f16_recon rc,
                                                          const f16_reward_cfg cfg, const f16_origin og,
                                                          const double* __restrict__ pool, int64_t pool_size,
                                                          const int64_t* __restrict__ pick,
                                                          double* __restrict__ reward, uint8_t* __restrict__ term,
                                                          uint8_t* __restrict__ trunc_, uint8_t* __restrict__ done,
                                                          float* __restrict__ obs, float* __restrict__ terminal_obs,
                                                          double* __restrict__ terminal_hp,
                                                          double* __restrict__ terminal_alt, double* __restrict__ aux) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nenv) return;
  Origin O = origin_of(og);
  Pair P;
  load_pair<LAYOUT>(st, ld, e, O, P);
  AdvanceOut A;
  advance_env(P, e, rc, cfg, actions, reward, term, trunc_, A);
  const int64_t o = 2 * e, p = o + 1;
  bool fin = term[e] || trunc_[e];
  done[e] = fin;
  for (int k = 0; k < 2; k++) {
    int64_t a = o + k;
    terminal_hp[a] = A.hp[k];
    RowRef<LAYOUT> R{st, ld, a};
    double x = R(0), y = R(1), z = R(2);
    terminal_alt[a] = (sqrt(x * x + y * y + z * z) - SLR_FT) * FT2M;
  }
  Side sd[2];
  for (int k = 0; k < 2; k++) sd[k] = {A.hp[k], A.fuel[k], A.dealt[k], A.taken[k], A.pqr[k], A.hist[k]};
  if (terminal_obs) obs_env(P, e, sd, A.t, terminal_obs, nullptr);
  if (!fin) {
    obs_env(P, e, sd, A.t, obs, aux);
    return;
  }
  // autoreset: new rows from the pool, fresh reconstruction state, anchored trackers
  int64_t row = pick[e];
  row = row < 0 ? 0 : (row >= pool_size ? pool_size - 1 : row);
  const double* src = pool + row * 2 * F16_STATE_N;
  for (int k = 0; k < 2; k++) {
    int64_t a = o + k;
    for (int c = 0; c < F16_STATE_N; c++) {
      double v = src[k * F16_STATE_N + c];
      if (LAYOUT == F16_LAYOUT_SOA) st[(int64_t)c * ld + a] = v;
      else st[a * F16_STATE_N + c] = v;
    }
    rc.hp[a] = 1.0; rc.fuel[a] = 1.0;
    rc.prev_att[a * 3] = 0.0; rc.prev_att[a * 3 + 1] = 0.0; rc.prev_att[a * 3 + 2] = 0.0;
    rc.prev_valid[a] = 0;
    rc.pqr[a * 3] = 0.0; rc.pqr[a * 3 + 1] = 0.0; rc.pqr[a * 3 + 2] = 0.0;
    rc.dmg_dealt[a] = 0.0; rc.dmg_taken[a] = 0.0; rc.hp_loss[a] = 0.0;
    double2* h = reinterpret_cast<double2*>(rc.act_hist + a * 20);
    for (int i = 0; i < 10; i++) h[i] = make_double2(0.0, 0.0);
    A.hist[k][0] = 0.0;
    for (int i = 0; i < 20; i++) A.hist[k][i] = 0.0;
  }
  rc.t_sec[e] = 0.0;
  Pair Q;
  load_pair<LAYOUT>(st, ld, e, O, Q);
  double g = geometry_advantage(Q, 0.0);
  rc.prev_x[o] = g; rc.prev_x[p] = -g;
  rc.prev_x_valid[o] = 1; rc.prev_x_valid[p] = 1;
  rc.prev_alt_log[o] = alt_log(-Q.s[0][2]);
  rc.prev_alt_log[p] = alt_log(-Q.s[1][2]);
  Side zs[2];
  for (int k = 0; k < 2; k++) zs[k] = {1.0, 1.0, 0.0, 0.0, {0.0, 0.0, 0.0}, A.hist[k]};
  obs_env(Q, e, zs, 0.0, obs, aux);
}

// 9-DoF export (R/cuda_fdm/rl_env.py:558-566 state9_flat): one thread per aircraft
template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS) k_state9(const double* __restrict__ st, int64_t ld, int64_t nac,
                                                        const f16_origin og, double* __restrict__ s9) {
  int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= nac) return;
  Origin O = origin_of(og);
  double v[9];
  kin9(RowRef<LAYOUT>{st, ld, a}, O, v);
  for (int i = 0; i < 9; i++) s9[a * 9 + i] = v[i];
}

// ---------------- external 214-D observation (R/cuda_fdm/external_observation.cu) ----------------
// Per aircraft: NED velocity from the 9-DoF state; acceleration = (v - v_prev) / dt where the
// aircraft's attitude history is valid (0 otherwise); v becomes v_prev.  Launched before the
// advance (which sets prev_valid), as BatchObsReward.kernel_advance does (obs_reward.py:417-420).
template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS) k_external_accel(const double* __restrict__ st, int64_t ld, int64_t nac,
                                                                const uint8_t* __restrict__ valid,
                                                                double* __restrict__ previous,
                                                                double* __restrict__ accel, const f16_origin og,
                                                                double dt) {
  int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= nac) return;
  Origin O = origin_of(og);
  double s[9];
  kin9(RowRef<LAYOUT>{st, ld, a}, O, s);
  M3 R = ned2body(s[3], s[4], s[5]);
  V3 v = mvT(R, V3{s[6], s[7], s[8]});
  const double vv[3] = {v.x, v.y, v.z};
  const bool ok = valid[a] != 0;
  for (int i = 0; i < 3; i++) {
    accel[a * 3 + i] = ok ? (vv[i] - previous[a * 3 + i]) / dt : 0.0;
    previous[a * 3 + i] = vv[i];
  }
}

// The 214-D row of aircraft a: columns 0-163 of its 184-D row, then 30 acceleration features
// (own acceleration in the world, own-body, target-body, target-velocity and line-of-sight
// frames; the target's in the world, own-body, target-body, own-velocity and line-of-sight
// frames; each clamped to +-150 m/s^2 and scaled to [-1, 1]), then the 20 action-history values.
template <int LAYOUT>
__global__ void __launch_bounds__(OBS_THREADS) k_external_obs(const double* __restrict__ st, int64_t ld, int64_t nac,
                                                              const double* __restrict__ accel,
                                                              const float* __restrict__ obs184,
                                                              float* __restrict__ out, const f16_origin og) {
  int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= nac) return;
  const int64_t b = a ^ 1;
  Origin O = origin_of(og);
  double s[9], t[9];
  kin9(RowRef<LAYOUT>{st, ld, a}, O, s);
  kin9(RowRef<LAYOUT>{st, ld, b}, O, t);
  const M3 Ro = ned2body(s[3], s[4], s[5]), Rt = ned2body(t[3], t[4], t[5]);
  const V3 vo = mvT(Ro, V3{s[6], s[7], s[8]}), vt = mvT(Rt, V3{t[6], t[7], t[8]});
  const M3 Fo = dir_frame(vo), Ft = dir_frame(vt), Fl = dir_frame(V3{t[0] - s[0], t[1] - s[1], t[2] - s[2]});
  M3 I;
  for (int i = 0; i < 3; i++)
    for (int j = 0; j < 3; j++) I.m[i][j] = i == j ? 1.0 : 0.0;
  const float* src = obs184 + a * 184;
  float* row = out + a * 214;
  for (int i = 0; i < 164; i++) row[i] = src[i];
  const V3 acc_a = {accel[a * 3], accel[a * 3 + 1], accel[a * 3 + 2]};
  const V3 acc_b = {accel[b * 3], accel[b * 3 + 1], accel[b * 3 + 2]};
  // frame order of the ten vectors: I, own body, target body, target velocity, LOS (own
  // acceleration); I, own body, target body, own velocity, LOS (target acceleration)
  const M3* frames[10] = {&I, &Ro, &Rt, &Ft, &Fl, &I, &Ro, &Rt, &Fo, &Fl};
#pragma unroll
  for (int i = 0; i < 10; i++) {
    const V3 v = mv(*frames[i], i < 5 ? acc_a : acc_b);
    row[164 + 3 * i + 0] = store_val(normz(v.x, -150.0, 150.0));
    row[164 + 3 * i + 1] = store_val(normz(v.y, -150.0, 150.0));
    row[164 + 3 * i + 2] = store_val(normz(v.z, -150.0, 150.0));
  }
  for (int i = 0; i < 20; i++) row[194 + i] = src[164 + i];
}

inline int grid_for(int64_t n) { return (int)((n + OBS_THREADS - 1) / OBS_THREADS); }

inline int check_recon(const f16_recon* rc, bool need_all) {
  if (!rc) return F16_ERR_ARG;
  if (!rc->hp || !rc->fuel || !rc->t_sec || !rc->pqr || !rc->dmg_dealt || !rc->dmg_taken || !rc->act_hist)
    return F16_ERR_ARG;
  if (need_all && (!rc->prev_att || !rc->prev_valid || !rc->hp_loss || !rc->prev_x || !rc->prev_x_valid ||
                   !rc->prev_alt_log))
    return F16_ERR_ARG;
  if (!aligned(rc->act_hist, 16)) return F16_ERR_ALIGN;
  return F16_OK;
}

inline int check_common(const double* st, int layout, int64_t ld, int64_t nenv, const f16_origin* og) {
  if (!st || nenv <= 0 || !og) return F16_ERR_ARG;
  if (layout != F16_LAYOUT_SOA && layout != F16_LAYOUT_AOS) return F16_ERR_ARG;
  if (layout == F16_LAYOUT_SOA && ld < 2 * nenv) return F16_ERR_ARG;
  return F16_OK;
}

}  // namespace obs
}  // namespace f16

using namespace f16;
using namespace f16::obs;

#define F16_DISPATCH_LAYOUT(layout, KERNEL, GRID, ...)                                      \
  do {                                                                                      \
    if ((layout) == F16_LAYOUT_SOA)                                                         \
      KERNEL<F16_LAYOUT_SOA><<<(GRID), OBS_THREADS, 0, s>>>(__VA_ARGS__);                   \
    else                                                                                    \
      KERNEL<F16_LAYOUT_AOS><<<(GRID), OBS_THREADS, 0, s>>>(__VA_ARGS__);                   \
  } while (0)

extern "C" int f16_obs_build(const double* state, int layout, int64_t ld, int64_t nenv, const uint8_t* env_mask,
                             const f16_recon* recon, const f16_origin* origin, float* obs, double* aux,
                             f16_stream_t stream) {
  int rc = check_common(state, layout, ld, nenv, origin);
  if (rc) return rc;
  if ((rc = check_recon(recon, false))) return rc;
  if (!obs) return F16_ERR_ARG;
  if (!aligned(obs, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  F16_DISPATCH_LAYOUT(layout, k_obs_build, grid_for(nenv), state, ld, nenv, env_mask, *recon, *origin, obs, aux);
  return launch_status();
}

extern "C" int f16_obs_advance(const double* state, int layout, int64_t ld, int64_t nenv, const double* actions,
                               const f16_recon* recon, const f16_reward_cfg* cfg, const f16_origin* origin,
                               double* reward, uint8_t* term, uint8_t* trunc_, f16_stream_t stream) {
  int rc = check_common(state, layout, ld, nenv, origin);
  if (rc) return rc;
  if ((rc = check_recon(recon, true))) return rc;
  if (!cfg || !actions || !reward || !term || !trunc_) return F16_ERR_ARG;
  if (cfg->reward_mode < 0 || cfg->reward_mode > 3) return F16_ERR_ARG;
  if (!aligned(actions, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  F16_DISPATCH_LAYOUT(layout, k_obs_advance, grid_for(nenv), state, ld, nenv, actions, *recon, *cfg, *origin, reward,
                      term, trunc_);
  return launch_status();
}

extern "C" int f16_obs_step(const double* state, int layout, int64_t ld, int64_t nenv, const double* actions,
                            const f16_recon* recon, const f16_reward_cfg* cfg, const f16_origin* origin,
                            double* reward, uint8_t* term, uint8_t* trunc_, float* obs, double* aux,
                            f16_stream_t stream) {
  int rc = check_common(state, layout, ld, nenv, origin);
  if (rc) return rc;
  if ((rc = check_recon(recon, true))) return rc;
  if (!cfg || !actions || !reward || !term || !trunc_ || !obs) return F16_ERR_ARG;
  if (cfg->reward_mode < 0 || cfg->reward_mode > 3) return F16_ERR_ARG;
  if (!aligned(actions, 16) || !aligned(obs, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  F16_DISPATCH_LAYOUT(layout, k_obs_step, grid_for(nenv), state, ld, nenv, actions, *recon, *cfg, *origin, reward,
                      term, trunc_, obs, aux);
  return launch_status();
}

extern "C" int f16_obs_init_reward(const double* state, int layout, int64_t ld, int64_t nenv,
                                   const uint8_t* env_mask, const f16_recon* recon, const f16_origin* origin,
                                   f16_stream_t stream) {
  int rc = check_common(state, layout, ld, nenv, origin);
  if (rc) return rc;
  if (!recon || !recon->t_sec || !recon->prev_x || !recon->prev_x_valid || !recon->prev_alt_log) return F16_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  F16_DISPATCH_LAYOUT(layout, k_obs_init_reward, grid_for(nenv), state, ld, nenv, env_mask, *recon, *origin);
  return launch_status();
}

extern "C" int f16_env_post_step(double* state, int layout, int64_t ld, int64_t nenv, const double* actions,
                                 const f16_recon* recon, const f16_reward_cfg* cfg, const f16_origin* origin,
                                 const double* ic_pool, int64_t pool_size, const int64_t* pick, double* reward,
                                 uint8_t* term, uint8_t* trunc_, uint8_t* done, float* obs, float* terminal_obs,
                                 double* terminal_hp, double* terminal_alt_m, double* aux, f16_stream_t stream) {
  int rc = check_common(state, layout, ld, nenv, origin);
  if (rc) return rc;
  if ((rc = check_recon(recon, true))) return rc;
  if (!cfg || !actions || !ic_pool || pool_size <= 0 || !pick || !reward || !term || !trunc_ || !done || !obs ||
      !terminal_hp || !terminal_alt_m)
    return F16_ERR_ARG;
  if (cfg->reward_mode < 0 || cfg->reward_mode > 3) return F16_ERR_ARG;
  if (!aligned(actions, 16) || !aligned(obs, 16) || (terminal_obs && !aligned(terminal_obs, 16))) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  F16_DISPATCH_LAYOUT(layout, k_env_post, grid_for(nenv), state, ld, nenv, actions, *recon, *cfg, *origin, ic_pool,
                      pool_size, pick, reward, term, trunc_, done, obs, terminal_obs, terminal_hp, terminal_alt_m,
                      aux);
  return launch_status();
}

extern "C" int f16_state9(const double* state, int layout, int64_t ld, int64_t nac, const f16_origin* origin,
                          double* s9, f16_stream_t stream) {
  if (!state || nac <= 0 || !origin || !s9) return F16_ERR_ARG;
  if (layout != F16_LAYOUT_SOA && layout != F16_LAYOUT_AOS) return F16_ERR_ARG;
  if (layout == F16_LAYOUT_SOA && ld < nac) return F16_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  F16_DISPATCH_LAYOUT(layout, k_state9, grid_for(nac), state, ld, nac, *origin, s9);
  return launch_status();
}

extern "C" int f16_external_accel(const double* state, int layout, int64_t ld, int64_t nac, const uint8_t* valid,
                                  double* previous, double* accel, const f16_origin* origin, double dt,
                                  f16_stream_t stream) {
  if (!state || !valid || !previous || !accel || !origin || nac <= 0 || !(dt > 0.0)) return F16_ERR_ARG;
  if (layout != F16_LAYOUT_SOA && layout != F16_LAYOUT_AOS) return F16_ERR_ARG;
  if (layout == F16_LAYOUT_SOA && ld < nac) return F16_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (layout == F16_LAYOUT_SOA)
    obs::k_external_accel<F16_LAYOUT_SOA><<<obs::grid_for(nac), obs::OBS_THREADS, 0, s>>>(state, ld, nac, valid,
                                                                                          previous, accel, *origin, dt);
  else
    obs::k_external_accel<F16_LAYOUT_AOS><<<obs::grid_for(nac), obs::OBS_THREADS, 0, s>>>(state, ld, nac, valid,
                                                                                          previous, accel, *origin, dt);
  return launch_status();
}

extern "C" int f16_external_obs(const double* state, int layout, int64_t ld, int64_t nac, const double* accel,
                                const float* obs184, float* out214, const f16_origin* origin, f16_stream_t stream) {
  if (!state || !accel || !obs184 || !out214 || !origin || nac <= 0 || (nac & 1)) return F16_ERR_ARG;
  if (layout != F16_LAYOUT_SOA && layout != F16_LAYOUT_AOS) return F16_ERR_ARG;
  if (layout == F16_LAYOUT_SOA && ld < nac) return F16_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (layout == F16_LAYOUT_SOA)
    obs::k_external_obs<F16_LAYOUT_SOA><<<obs::grid_for(nac), obs::OBS_THREADS, 0, s>>>(state, ld, nac, accel, obs184,
                                                                                        out214, *origin);
  else
    obs::k_external_obs<F16_LAYOUT_AOS><<<obs::grid_for(nac), obs::OBS_THREADS, 0, s>>>(state, ld, nac, accel, obs184,
                                                                                        out214, *origin);
  return launch_status();
}
