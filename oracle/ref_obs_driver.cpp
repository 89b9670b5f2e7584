// ref_obs_driver.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Host-compiled run of the reference's own observation / reward kernels: its NVRTC source
// research/competition_36500/runtime/cuda_fdm/gen/obs_kernel.cu, with
// research/competition_36500/runtime/cuda_fdm/external_observation.cu appended the way
// BatchObsReward.enable_external_observations does (R/cuda_fdm/obs_reward.py:471-481), is
// #included from its original location; a small shim maps the CUDA qualifiers to host C++ and
// each entry point below runs the kernel body once per thread index, as a launch would.  Built
// by oracle/build.py with g++ -O2 -ffp-contract=off (the reference compiles the source with
// --fmad=false).  The output (oracle/_ref/libobsref.so) pins oracle/obs_oracle.c.
#include <cmath>
#include <cstdint>
#include <cstdio>

using std::isfinite;

// ---- CUDA-to-host shim
#define __device__
#define __forceinline__ inline
#define __global__
struct ShimDim { unsigned x, y, z; };
static ShimDim blockIdx = {0, 0, 0}, blockDim = {1, 1, 1}, threadIdx = {0, 0, 0};
static inline void shim_thread(long i) { blockIdx.x = (unsigned)i; blockDim.x = 1; threadIdx.x = 0; }

#include "obs_kernel.cu"
#include "external_observation.cu"

extern "C" {

void ref_obs_init_reward(const double* states, const unsigned char* env_mask, double* prev_geometry,
                         unsigned char* prev_geometry_valid, double* prev_alt_log, const double* t_sec, int nenv,
                         const double* o7) {
  for (long e = 0; e < nenv; e++) {
    shim_thread(e);
    init_reward_kernel(states, env_mask, prev_geometry, prev_geometry_valid, prev_alt_log, t_sec, nenv, o7[0], o7[1],
                       o7[2], o7[3], o7[4], o7[5], o7[6]);
  }
}

// cfg: dt, min_alt, max_time, own_w, dmg_scale, shap_scale, win_r, loss_r, timeout_win_r,
// timeout_loss_r, timeout_draw_r, alt_hunt_coef
void ref_obs_advance(const double* states, const double* actions, double* hp, double* fuel, double* t_sec,
                     double* prev_att, unsigned char* prev_valid, double* pqr, double* last_dmg_dealt,
                     double* last_dmg_taken, double* hp_loss, double* act_hist, double* prev_x,
                     unsigned char* prev_x_valid, double* prev_alt_log, double* reward, unsigned char* term,
                     unsigned char* trunc_, int nenv, const double* o7, const double* cfg, int reward_mode) {
  for (long e = 0; e < nenv; e++) {
    shim_thread(e);
    advance_kernel(states, actions, hp, fuel, t_sec, prev_att, prev_valid, pqr, last_dmg_dealt, last_dmg_taken,
                   hp_loss, act_hist, prev_x, prev_x_valid, prev_alt_log, reward, term, trunc_, nenv, o7[0], o7[1],
                   o7[2], o7[3], o7[4], o7[5], o7[6], cfg[0], cfg[1], cfg[2], cfg[3], cfg[4], cfg[5], cfg[6], cfg[7],
                   cfg[8], cfg[9], cfg[10], reward_mode, cfg[11]);
  }
}

void ref_obs_build(const double* states, const unsigned char* env_mask, const double* hp, const double* fuel,
                   const double* t_sec, const double* pqr, const double* last_dmg_dealt,
                   const double* last_dmg_taken, const double* act_hist, float* obs, int nac, const double* o7,
                   double* aux) {
  for (long a = 0; a < nac; a++) {
    shim_thread(a);
    build_obs_kernel(states, env_mask, hp, fuel, t_sec, pqr, last_dmg_dealt, last_dmg_taken, act_hist, obs, nac,
                     o7[0], o7[1], o7[2], o7[3], o7[4], o7[5], o7[6], aux);
  }
}

void ref_external_accel(const double* states, const unsigned char* valid, double* previous, double* accel, int nac,
                        const double* o7, double dt) {
  for (long a = 0; a < nac; a++) {
    shim_thread(a);
    external_acceleration(states, valid, previous, accel, nac, o7[0], o7[1], o7[2], o7[3], o7[4], o7[5], o7[6], dt);
  }
}

void ref_external_obs(const double* states, const double* accel, const float* original, float* out, int nac,
                      const double* o7) {
  for (long a = 0; a < nac; a++) {
    shim_thread(a);
    external_observation(states, accel, original, out, nac, o7[0], o7[1], o7[2], o7[3], o7[4], o7[5], o7[6]);
  }
}

}  // extern "C"
