// obs_kernels.cu -- observation / reward / termination kernels and their C-ABI entry points.
//
// The per-environment kernels run one thread per AIRCRAFT, the two aircraft of an environment
// on adjacent lanes (obs_device.cuh, lane-pair organisation): each lane reads its own FDM row
// (14 state columns, consecutive lanes on consecutive addresses in the SoA layout), stages its
// aircraft's geometry in shared memory for the partner, updates its own reconstruction values
// and writes its own 184-float row with 16-byte vector stores.  Reconstruction buffers keep
// the reference's per-aircraft layout (R/cuda_fdm/obs_reward.py:338-353) so the reference's
// tensors can be passed as they are.
#include "common.cuh"
#include "obs_device.cuh"

namespace f16 {
namespace obs {

constexpr int OBS_THREADS = 128;        // per-aircraft kernels without staging (state9, external)
// Lane-pair kernels: 64 threads (32 environments) per block and 27.5 KB of staging, so 8 blocks
// (16 warps) fit per SM with up to 128 registers per thread -- the row builder's working set then
// stays in registers (one thread per environment needed more than 255 and spilled at every
// occupancy).  With the out-of-line library calls 8 blocks measured 3.9% faster than 7 for
// k_obs_step (about 1% slower for k_env_post, whose autoreset path spills a little at 128).
#ifndef F16_OBS_PAIR_THREADS
#define F16_OBS_PAIR_THREADS 64
#endif
#ifndef F16_OBS_PAIR_MIN_BLOCKS
#define F16_OBS_PAIR_MIN_BLOCKS 8
#endif
constexpr int PT = F16_OBS_PAIR_THREADS;
static_assert(PT % 32 == 0, "pairs must not straddle warps");

template <int LAYOUT>
struct RowRef {
  const double* __restrict__ p;
  int64_t ld, a;
  __device__ __forceinline__ double operator()(int c) const {
    return LAYOUT == F16_LAYOUT_SOA ? p[(int64_t)c * ld + a] : p[a * F16_STATE_N + c];
  }
};

__device__ __forceinline__ Origin origin_of(const f16_origin& o) { return {o.ox, o.oy, o.oz, o.slat, o.clat, o.slon, o.clon}; }

// Lane setup of a lane-pair kernel; false for lanes past the last aircraft (whole pairs, since
// the aircraft count is even).
struct PairLane {
  int64_t a, e;
  int k;
};
__device__ __forceinline__ bool pair_lane(int64_t nenv, PairLane& pl) {
  pl.a = (int64_t)blockIdx.x * PT + threadIdx.x;
  pl.e = pl.a >> 1;
  pl.k = (int)(pl.a & 1);
  return pl.a < 2 * nenv;
}
__device__ __forceinline__ Lanes<PT> lanes_of(double* sm) {
  return {sm, (int)threadIdx.x, 3u << (threadIdx.x & 30)};
}

// Both staging passes for the pair (stage_aircraft, then stage_los once both are staged);
// prev / inv_dt as in stage_aircraft.
template <int LAYOUT>
__device__ __forceinline__ Los stage_pair(const Lanes<PT>& L, const double* st, int64_t ld, int64_t a, int k,
                                          const Origin& O, const double* prev = nullptr, double inv_dt = 0.0) {
  stage_aircraft(L, RowRef<LAYOUT>{st, ld, a}, O, prev, inv_dt);
  L.sync();
  Los g = stage_los(L, k);
  L.sync();
  return g;
}

// action-history push of one aircraft (roll by one, newest first): hist[0..19] <- (a, hist[0..15]).
// The new history is also the last 20 features of the aircraft's observation row (columns
// 164-183, stored as the reference's STORE does): written here into each row given (rows may
// be NULL), while the values are in registers, instead of being read back for the row.
__device__ __forceinline__ void push_hist(double* h, const double* __restrict__ act, float* row_a, float* row_b) {
  const double2* h2 = reinterpret_cast<const double2*>(h);
  double2 o[10];
#pragma unroll
  for (int i = 0; i < 8; i++) o[2 + i] = h2[i];
  const double2* a2 = reinterpret_cast<const double2*>(act);
  o[0] = a2[0];
  o[1] = a2[1];
  double2* w = reinterpret_cast<double2*>(h);
#pragma unroll
  for (int i = 0; i < 10; i++) w[i] = o[i];
  float* rows[2] = {row_a, row_b};
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if (!rows[r]) continue;
    float4* d = reinterpret_cast<float4*>(rows[r] + 164);
#pragma unroll
    for (int i = 0; i < 5; i++)
      d[i] = make_float4(store_val(o[2 * i].x), store_val(o[2 * i].y), store_val(o[2 * i + 1].x),
                         store_val(o[2 * i + 1].y));
  }
}

// Reconstruction values of a fresh episode staged for the observation row.
template <int T>
__device__ __forceinline__ void stage_fresh(const Lanes<T>& L) {
  L.own(F_HP) = 1.0; L.own(F_FUEL) = 1.0;
  L.own(F_PQR) = 0.0; L.own(F_PQR + 1) = 0.0; L.own(F_PQR + 2) = 0.0;
}

// The aircraft's previous attitude when its history is valid (body rates), else NULL.
__device__ __forceinline__ const double* prev_attitude(const f16_recon& rc, int64_t a) {
  return rc.prev_valid[a] ? rc.prev_att + a * 3 : nullptr;
}
__device__ __forceinline__ double inv_dt_of(const f16_reward_cfg& cfg) { return 1.0 / (cfg.dt > 1e-8 ? cfg.dt : 1e-8); }

struct Advanced {
  double hp, t;        // this aircraft's HP after the step; the environment's new clock
  double dealt, taken; // this step's damage rates dealt / taken (row features of the own lane only,
                       // so they travel in registers, not through the staging array)
  bool te, tr;         // the environment's termination / truncation
};

// advance_kernel semantics (obs_kernel.cu:504-626) for this lane's aircraft after stage_pair:
// damage / HP / fuel / body rates / attitude history of the aircraft, the environment's clock
// and flags (written by the even lane), the aircraft's final-safe reward and reward trackers;
// the row's reconstruction values are staged.
template <int T>
__device__ __forceinline__ Advanced advance_lane(const Lanes<T>& L, const PairLane& pl, const Los& g,
                                                 const f16_recon& rc, const f16_reward_cfg& cfg,
                                                 const double* __restrict__ actions, double* __restrict__ reward,
                                                 uint8_t* __restrict__ term, uint8_t* __restrict__ trunc_,
                                                 float* hist_row_a = nullptr, float* hist_row_b = nullptr) {
  const int64_t a = pl.a, e = pl.e;
  const int k = pl.k;
  const double dt = cfg.dt;
  push_hist(rc.act_hist + a * 20, actions + a * 4, hist_row_a, hist_row_b);
  const double r_ft = g.dist * M2FT;
  const double t_old = rc.t_sec[e];
  const double ata = L.own(F_ATA), ata_p = L.par(F_ATA);
  const double rate = damage(r_ft, ata, t_old), rate_p = damage(r_ft, ata_p, t_old);
  const double h0 = rc.hp[a];
  const double h0_p = L.xchg(h0);
  double h = h0 - rate_p * dt, h_p = h0_p - rate * dt;
  if (h < 0.0) h = 0.0;
  if (h_p < 0.0) h_p = 0.0;
  const double lo = h0 - h, lp = h0_p - h_p;
  rc.hp[a] = h;
  rc.hp_loss[a] = lo;
  rc.dmg_dealt[a] = rate;
  rc.dmg_taken[a] = rate_p;
  double f = rc.fuel[a] - FUEL_BURN * (L.own(F_SPD) / FUEL_REF) * dt;
  if (f < 0.0) f = 0.0;
  rc.fuel[a] = f;
  // body rates from the attitude change (staged by stage_aircraft from the previous attitude)
  rc.pqr[a * 3] = L.own(F_PQR); rc.pqr[a * 3 + 1] = L.own(F_PQR + 1); rc.pqr[a * 3 + 2] = L.own(F_PQR + 2);
  rc.prev_att[a * 3] = L.own(F_S + 3); rc.prev_att[a * 3 + 1] = L.own(F_S + 4); rc.prev_att[a * 3 + 2] = L.own(F_S + 5);
  rc.prev_valid[a] = 1;
  const double t_new = t_old + dt;
  const double alt = -L.own(F_S + 2), alt_p = -L.par(F_S + 2);
  bool fin = true;
  for (int j = 0; j < 9; j++)
    if (!isfinite(L.col(F_S + j, 0)) || !isfinite(L.col(F_S + j, 1))) fin = false;
  const bool te = (alt < cfg.min_alt) || (alt_p < cfg.min_alt) || (h <= 0.0) || (h_p <= 0.0) || (!fin);
  const bool tr = (!te) && (t_new >= cfg.max_time - TLIM_TOL);
  if (k == 0) {
    rc.t_sec[e] = t_new;
    term[e] = te;
    trunc_[e] = tr;
  }
  const double gx = geometry_advantage(L, k, g, t_new);
  const double lga = alt_log(alt), lga_p = alt_log(alt_p);
  const int valid = rc.prev_x_valid[a];
  const int valid_p = L.xchg(valid);
  const double alt_log_prev_p = L.xchg(rc.prev_alt_log[a]);
  const double pg = valid ? rc.prev_x[a] : gx;
  const double gm = cfg.shaping_reward_scale / SHAPING_BASE;
  double rgx = gm * (GEOM_BUDGET / GEOM_REF_SEC) * 0.5 * (pg + gx) * dt;
  if (cfg.reward_mode == 1) rgx = valid_p ? cfg.alt_hunt_coef * (alt_log_prev_p - lga_p) : 0.0;
  rc.prev_x[a] = gx;
  rc.prev_x_valid[a] = 1;
  rc.prev_alt_log[a] = lga;
  const double dsc = cfg.damage_scale, ow = cfg.own_damage_weight;
  double rd = (lp - lo * ow) * dsc;
  if (cfg.reward_mode == 2) rd = lp * dsc;
  else if (cfg.reward_mode == 3) rd = -(lo * ow) * dsc;
  double rt = 0.0;
  if (te) {
    if (alt < cfg.min_alt) rt = -h * dsc;
    else if (alt_p < cfg.min_alt) rt = h_p * dsc;
    else { if (h_p <= 0.0) rt += cfg.win_reward; if (h <= 0.0) rt += cfg.loss_reward; }
  } else if (tr) {
    rt = (h > h_p) ? cfg.timeout_win_reward : ((h < h_p) ? cfg.timeout_loss_reward : cfg.timeout_draw_reward);
  }
  reward[a] = rd + rgx + rt;
  L.own(F_HP) = h; L.own(F_FUEL) = f;
  return {h, t_new, rate, rate_p, te, tr};
}

template <int LAYOUT>
__global__ void __launch_bounds__(PT, F16_OBS_PAIR_MIN_BLOCKS) k_obs_build(const double* __restrict__ st, int64_t ld,
                                                                           int64_t nenv, const uint8_t* __restrict__ mask,
                                                                           const f16_recon rc, const f16_origin og,
                                                                           float* __restrict__ obs,
                                                                           double* __restrict__ aux) {
  __shared__ double sm[NFIELD * PT];
  PairLane pl;
  if (!pair_lane(nenv, pl) || (mask && !mask[pl.e])) return;
  const Lanes<PT> L = lanes_of(sm);
  const Los g = stage_pair<LAYOUT>(L, st, ld, pl.a, pl.k, origin_of(og));
  const int64_t a = pl.a;
  L.own(F_HP) = rc.hp[a]; L.own(F_FUEL) = rc.fuel[a];
  L.own(F_PQR) = rc.pqr[a * 3]; L.own(F_PQR + 1) = rc.pqr[a * 3 + 1]; L.own(F_PQR + 2) = rc.pqr[a * 3 + 2];
  L.sync();
  obs_row(L, pl.k, g, rc.t_sec[pl.e], HIST_READ, rc.act_hist + a * 20, obs + a * 184,
          (aux && pl.k == 0) ? aux + pl.e * 21 : nullptr, rc.dmg_dealt[a], rc.dmg_taken[a]);
}

template <int LAYOUT>
__global__ void __launch_bounds__(PT, F16_OBS_PAIR_MIN_BLOCKS) k_obs_advance(const double* __restrict__ st, int64_t ld,
                                                                             int64_t nenv,
                                                                             const double* __restrict__ actions,
                                                                             const f16_recon rc, const f16_reward_cfg cfg,
                                                                             const f16_origin og,
                                                                             double* __restrict__ reward,
                                                                             uint8_t* __restrict__ term,
                                                                             uint8_t* __restrict__ trunc_) {
  __shared__ double sm[NFIELD * PT];
  PairLane pl;
  if (!pair_lane(nenv, pl)) return;
  const Lanes<PT> L = lanes_of(sm);
  const Los g = stage_pair<LAYOUT>(L, st, ld, pl.a, pl.k, origin_of(og), prev_attitude(rc, pl.a), inv_dt_of(cfg));
  advance_lane(L, pl, g, rc, cfg, actions, reward, term, trunc_);
}

// Fused: advance (reward, termination, reconstruction update) then the observation rows,
// reading each FDM row once (the reference launches advance_kernel then build_obs_kernel).
template <int LAYOUT>
__global__ void __launch_bounds__(PT, F16_OBS_PAIR_MIN_BLOCKS) k_obs_step(const double* __restrict__ st, int64_t ld,
                                                                          int64_t nenv,
                                                                          const double* __restrict__ actions,
                                                                          const f16_recon rc, const f16_reward_cfg cfg,
                                                                          const f16_origin og,
                                                                          double* __restrict__ reward,
                                                                          uint8_t* __restrict__ term,
                                                                          uint8_t* __restrict__ trunc_,
                                                                          float* __restrict__ obs,
                                                                          double* __restrict__ aux) {
  __shared__ double sm[NFIELD * PT];
  PairLane pl;
  if (!pair_lane(nenv, pl)) return;
  const Lanes<PT> L = lanes_of(sm);
  const Los g = stage_pair<LAYOUT>(L, st, ld, pl.a, pl.k, origin_of(og), prev_attitude(rc, pl.a), inv_dt_of(cfg));
  const Advanced A = advance_lane(L, pl, g, rc, cfg, actions, reward, term, trunc_, obs + pl.a * 184);
  L.sync();
  obs_row(L, pl.k, g, A.t, HIST_DONE, nullptr, obs + pl.a * 184, (aux && pl.k == 0) ? aux + pl.e * 21 : nullptr,
          A.dealt, A.taken);
}

template <int LAYOUT>
__global__ void __launch_bounds__(PT, F16_OBS_PAIR_MIN_BLOCKS) k_obs_init_reward(const double* __restrict__ st,
                                                                                 int64_t ld, int64_t nenv,
                                                                                 const uint8_t* __restrict__ mask,
                                                                                 const f16_recon rc,
                                                                                 const f16_origin og) {
  __shared__ double sm[NFIELD * PT];
  PairLane pl;
  if (!pair_lane(nenv, pl) || (mask && !mask[pl.e])) return;
  const Lanes<PT> L = lanes_of(sm);
  const Los g = stage_pair<LAYOUT>(L, st, ld, pl.a, pl.k, origin_of(og));
  const double gx = geometry_advantage(L, pl.k, g, rc.t_sec[pl.e]);
  rc.prev_x[pl.a] = gx;
  rc.prev_x_valid[pl.a] = 1;
  rc.prev_alt_log[pl.a] = alt_log(-L.own(F_S + 2));
}

// k_env_post's autoreset of one aircraft (both lanes of the environment run it): the pool row,
// fresh reconstruction state, anchored reward trackers, restaged geometry.
template <int LAYOUT>
__device__ __forceinline__ void env_reset_row(const Lanes<PT>& L, const PairLane& pl, double* __restrict__ st,
                                              int64_t ld, const double* __restrict__ pool, int64_t pool_size,
                                              const int64_t* __restrict__ pick, const f16_recon& rc, const Origin& O,
                                              Los& g) {
  const int64_t a = pl.a, e = pl.e;
  // autoreset: this aircraft's row from the pool, fresh reconstruction state, anchored trackers
  int64_t row = pick[e];
  row = row < 0 ? 0 : (row >= pool_size ? pool_size - 1 : row);
  const double* src = pool + (row * 2 + pl.k) * F16_STATE_N;
  for (int c = 0; c < F16_STATE_N; c++) {
    const double v = src[c];
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
  if (pl.k == 0) rc.t_sec[e] = 0.0;
  L.sync();                                     // the partner's rows are written: restage
  g = stage_pair<LAYOUT>(L, st, ld, a, pl.k, O);
  const double gx = geometry_advantage(L, pl.k, g, 0.0);
  rc.prev_x[a] = gx;
  rc.prev_x_valid[a] = 1;
  rc.prev_alt_log[a] = alt_log(-L.own(F_S + 2));
  stage_fresh(L);
  L.sync();
}

// Everything GpuDogfightVecEnv.step does after the physics step (R/cuda_fdm/rl_env.py:514-551),
// in one launch: advance, terminal observations, terminal HP / MSL altitude, and for finished
// environments the autoreset from the IC pool (state rows, reconstruction reset, reward-tracker
// anchoring, fresh observations).  pool: (pool_size, 2, 101) AoS rows; pick: pool row per env.
template <int LAYOUT>
__global__ void __launch_bounds__(PT, F16_OBS_PAIR_MIN_BLOCKS) k_env_post(double* __restrict__ st, int64_t ld,
                                                                          int64_t nenv,
                                                                          const double* __restrict__ actions,
                                                                          const f16_recon rc, const f16_reward_cfg cfg,
                                                                          const f16_origin og,
                                                                          const double* __restrict__ pool,
                                                                          int64_t pool_size,
                                                                          const int64_t* __restrict__ pick,
                                                                          double* __restrict__ reward,
                                                                          uint8_t* __restrict__ term,
                                                                          uint8_t* __restrict__ trunc_,
                                                                          uint8_t* __restrict__ done,
                                                                          float* __restrict__ obs,
                                                                          float* __restrict__ terminal_obs,
                                                                          double* __restrict__ terminal_hp,
                                                                          double* __restrict__ terminal_alt,
                                                                          double* __restrict__ aux) {
  __shared__ double sm[NFIELD * PT];
  PairLane pl;
  if (!pair_lane(nenv, pl)) return;
  const Lanes<PT> L = lanes_of(sm);
  const Origin O = origin_of(og);
  const int64_t a = pl.a, e = pl.e;
  Los g = stage_pair<LAYOUT>(L, st, ld, a, pl.k, O, prev_attitude(rc, a), inv_dt_of(cfg));
  const Advanced A = advance_lane(L, pl, g, rc, cfg, actions, reward, term, trunc_, obs + a * 184,
                                  terminal_obs ? terminal_obs + a * 184 : nullptr);
  const bool fin = A.te || A.tr;
  if (pl.k == 0) done[e] = fin;
  terminal_hp[a] = A.hp;
  {
    RowRef<LAYOUT> R{st, ld, a};
    const double x = R(0), y = R(1), z = R(2);
    terminal_alt[a] = (sqrt(x * x + y * y + z * z) - SLR_FT) * FT2M;
  }
  L.sync();
  double* ax = (aux && pl.k == 0) ? aux + e * 21 : nullptr;
  if (terminal_obs) obs_row(L, pl.k, g, A.t, HIST_DONE, nullptr, terminal_obs + a * 184, nullptr, A.dealt, A.taken);
  if (fin) env_reset_row<LAYOUT>(L, pl, st, ld, pool, pool_size, pick, rc, O, g);
  // one row-builder call for both outcomes (a finished environment's row after its reset)
  obs_row(L, pl.k, g, fin ? 0.0 : A.t, fin ? HIST_ZERO : HIST_DONE, nullptr, obs + a * 184, ax,
          fin ? 0.0 : A.dealt, fin ? 0.0 : A.taken);
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
// lane-pair kernels: one thread per aircraft
inline int pair_grid(int64_t nenv) { return (int)((2 * nenv + PT - 1) / PT); }

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

#define F16_DISPATCH_LAYOUT(layout, KERNEL, GRID, BLOCK, ...)                               \
  do {                                                                                      \
    if ((layout) == F16_LAYOUT_SOA)                                                         \
      KERNEL<F16_LAYOUT_SOA><<<(GRID), (BLOCK), 0, s>>>(__VA_ARGS__);                       \
    else                                                                                    \
      KERNEL<F16_LAYOUT_AOS><<<(GRID), (BLOCK), 0, s>>>(__VA_ARGS__);                       \
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
  F16_DISPATCH_LAYOUT(layout, k_obs_build, pair_grid(nenv), PT, state, ld, nenv, env_mask, *recon, *origin, obs, aux);
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
  F16_DISPATCH_LAYOUT(layout, k_obs_advance, pair_grid(nenv), PT, state, ld, nenv, actions, *recon, *cfg, *origin, reward,
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
  F16_DISPATCH_LAYOUT(layout, k_obs_step, pair_grid(nenv), PT, state, ld, nenv, actions, *recon, *cfg, *origin, reward,
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
  F16_DISPATCH_LAYOUT(layout, k_obs_init_reward, pair_grid(nenv), PT, state, ld, nenv, env_mask, *recon, *origin);
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
  F16_DISPATCH_LAYOUT(layout, k_env_post, pair_grid(nenv), PT, state, ld, nenv, actions, *recon, *cfg, *origin, ic_pool,
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
  F16_DISPATCH_LAYOUT(layout, k_state9, grid_for(nac), OBS_THREADS, state, ld, nac, *origin, s9);
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
