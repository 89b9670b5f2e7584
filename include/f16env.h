/*
 * f16env.h -- C ABI of the B200-native F-16 parallel-environment hot path.
 *
 * One shared library (libf16env.so, built for sm_100a) exports these entry points.  Every
 * pointer is a DEVICE pointer unless the name says "host"; the caller owns all buffers.
 * Every entry point returns an f16_status (0 = OK) and never throws.  Kernels are enqueued on
 * the given stream (NULL = legacy default stream); no entry point synchronises the host,
 * except where stated.
 *
 * Aircraft / environment numbering follows the reference (cuda_fdm/gpu_env.py:1-7 and
 * cuda_fdm/obs_reward.py:10-11): nac = 2*nenv aircraft, aircraft a = 2e (ownship) and 2e+1
 * (opponent) belong to environment e, partner(a) = a^1.
 */
#ifndef F16ENV_H
#define F16ENV_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* f16_stream_t;   /* == cudaStream_t */

typedef enum {
  F16_OK = 0,
  F16_ERR_ARG = 1,         /* null pointer, negative/zero size, bad enum value */
  F16_ERR_ALIGN = 2,       /* pointer not aligned as the entry point requires */
  F16_ERR_LAUNCH = 3,      /* CUDA launch/configuration error (cudaGetLastError) */
  F16_ERR_NONFINITE = 4,   /* a checked output was non-finite (only when checks are on) */
  F16_ERR_CUDA = 5,        /* other CUDA runtime error */
  F16_ERR_TOO_LARGE = 6    /* size above a documented maximum */
} f16_status;

/* ------------------------------------------------------------------------------------------
 * FDM state layout: 101 fp64 per aircraft, in the reference's FdmState order
 * (cuda_fdm/gen/fdm.cuh:519-528; flattening in cuda_fdm/ic.py:92-114).
 * ---------------------------------------------------------------------------------------- */
#define F16_STATE_N 101
#define F16_S_POS 0          /* eci_pos[3] ft */
#define F16_S_VEL 3          /* eci_vel[3] ft/s */
#define F16_S_Q 6            /* attitude quaternion ECI->body [4] */
#define F16_S_PQRI 10        /* inertial body rates [3] rad/s */
#define F16_S_EPA 13         /* earth position angle rad */
#define F16_S_FUEL 14        /* total fuel lb */
#define F16_S_UVWIDOT 15     /* carried ECI acceleration [3] */
#define F16_S_PQRIDOT 18     /* carried angular acceleration [3] */
#define F16_S_QDOT 21        /* carried quaternion rate [4] */
#define F16_S_DEQ_Q 25       /* integrator history, 3 x 4 (newest first) */
#define F16_S_DEQ_PQRI 37    /* 3 x 3 */
#define F16_S_DEQ_IVEL 46    /* 3 x 3 */
#define F16_S_DEQ_UVWIDOT 55 /* 3 x 3 */
#define F16_S_PREV_BACC 64   /* previous body acceleration [3] */
#define F16_S_PREV_PQRIDOT 67
#define F16_S_PREV_PQRI 70
#define F16_S_PREV_AUX 73    /* alpha, mach, vc_kts, vg_fps, n_pilot_y, n_pilot_z, p, q, r */
#define F16_S_ENG 82         /* N1, N2, N2norm, FuelFlow_pph */
#define F16_S_KIN 86         /* kinematic actuators tef, aileron, elevator, rudder, gear, lef */
#define F16_S_PID 92         /* roll, g-load, yaw PIDs: (input_prev, input_prev2, i_out_total) */

/* obs17 columns of the reference fdm_step_batch (cuda_fdm/gen/fdm_kernel.cu:28-46) */
#define F16_OBS17_N 17

/* State storage: element (aircraft a, column c) lives at state[c*ld + a] ("SoA", ld >= nac,
 * coalesced on the GPU) when layout == F16_LAYOUT_SOA, or at state[a*101 + c] ("AoS", the
 * reference's (nac,101) row-major tensor) when layout == F16_LAYOUT_AOS. */
#define F16_LAYOUT_SOA 0
#define F16_LAYOUT_AOS 1

/* ------------------------------------------------------------------------------------------
 * (1) FDM + FCS integration.
 * Replaces the NVRTC kernel fdm_step_batch (cuda_fdm/gen/fdm_kernel.cu:32-47) launched by
 * GpuDogfight.step (cuda_fdm/gpu_env.py:95-106).  Runs `substeps` frames of 1/60 s per
 * aircraft with the commands held (aileron, elevator, rudder in [-1,1], throttle in [0,1]).
 *   state   : 101 x nac fp64, layout as above, updated in place
 *   cmd     : nac x 4 fp64 row-major (the reference's (nac,4) actions tensor)
 *   fcs_dt  : FCS component dt; 1/120 = cuda_fdm/gen/fdm.cuh:23, 1/60 = the 184-D lineage
 *   obs17   : nac x 17 fp64 row-major, or NULL
 * ---------------------------------------------------------------------------------------- */
int f16_fdm_step(double* state, int layout, int64_t ld, int64_t nac,
                 const double* cmd, int substeps, double fcs_dt,
                 double* obs17, f16_stream_t stream);

/* Same, with the commands given as action-bin indices (nac x 4 uint8, bins 0..num_bins-1)
 * mapped in-kernel as the reference's action_to_env does (R/cuda_fdm/ppo_gpu.py:361-369):
 * channel value = grid_host[idx] (the caller's float32 torch.linspace(-1,1,num_bins), a HOST
 * pointer, 2 <= num_bins <= 64), throttle = 0.5f*v + 0.5f in float32. */
int f16_fdm_step_bins(double* state, int layout, int64_t ld, int64_t nac,
                      const uint8_t* bins, const float* grid_host, int num_bins, int substeps,
                      double fcs_dt, double* obs17, f16_stream_t stream);

/* Both forms in one entry point, plus the per-aircraft finite flag the reference's env step
 * computes after physics (R/cuda_fdm/rl_env.py:517, torch.isfinite(states).all(1)) produced by
 * the same launch: finite[a] = 1 when every one of the 101 state values of aircraft a is finite
 * after the step.  Exactly one of cmd / bins is non-NULL; obs17 and finite may be NULL. */
typedef struct {
  const double* cmd;        /* nac x 4 fp64, or NULL */
  const uint8_t* bins;      /* nac x 4 uint8 bins, or NULL */
  const float* grid_host;   /* with bins: host fp32 grid of num_bins values */
  int num_bins;
  double* obs17;            /* nac x 17 fp64, or NULL */
  uint8_t* finite;          /* nac uint8, or NULL */
} f16_fdm_io;
int f16_fdm_step_ex(double* state, int layout, int64_t ld, int64_t nac, const f16_fdm_io* io,
                    int substeps, double fcs_dt, f16_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * (1b) Initial-condition seeder (replaces the CPU path cuda_fdm/ic.py:117-138 ->
 * cuda_fdm/ref/jsb_fdm.py:142-210): builds the 101-double seed row of each aircraft from
 * its IC, including the one throwaway force-path evaluation that seeds the integrators.
 *   ic : nac x F16_IC_N fp64 row-major, columns below.
 * ---------------------------------------------------------------------------------------- */
#define F16_IC_N 12
#define F16_IC_LAT_DEG 0
#define F16_IC_LON_DEG 1
#define F16_IC_ALT_FT 2
#define F16_IC_VT_FPS 3
#define F16_IC_PHI_DEG 4
#define F16_IC_THETA_DEG 5
#define F16_IC_PSI_DEG 6
#define F16_IC_ALPHA_DEG 7
#define F16_IC_BETA_DEG 8
#define F16_IC_FUEL_LBS 9
#define F16_IC_FUELFLOW_PPH 10
#define F16_IC_GEOCENTRIC 11     /* 0 = geodetic latitude (default), 1 = geocentric */
int f16_seed_ic(const double* ic, int64_t nac, double* state, int layout, int64_t ld,
                double fcs_dt, f16_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * (2) Fused 184-D observation / final-safe reward / termination.
 * Replaces the reference's NVRTC kernels init_reward_kernel, advance_kernel and
 * build_obs_kernel (research/competition_36500/runtime/cuda_fdm/gen/obs_kernel.cu:485,504,628)
 * launched by BatchObsReward.kernel_init_reward_state / kernel_advance / kernel_build_obs
 * (R/cuda_fdm/obs_reward.py:410-468).  One GPU thread per environment handles both aircraft.
 *
 * f16_recon holds DEVICE pointers to the reference's reconstruction buffers, in its layout
 * (obs_reward.py:338-353): per aircraft (nac = 2*nenv) hp, fuel, dmg_dealt, dmg_taken, hp_loss,
 * prev_x, prev_alt_log [nac] fp64; prev_att, pqr [nac][3] fp64; act_hist [nac][5][4] fp64
 * (newest first, 16-byte aligned); prev_valid, prev_x_valid [nac] uint8 (torch.bool);
 * per environment t_sec [nenv] fp64.
 * ---------------------------------------------------------------------------------------- */
typedef struct {
  double* hp;
  double* fuel;
  double* t_sec;
  double* prev_att;
  uint8_t* prev_valid;
  double* pqr;
  double* dmg_dealt;
  double* dmg_taken;
  double* hp_loss;
  double* act_hist;
  double* prev_x;
  uint8_t* prev_x_valid;
  double* prev_alt_log;
} f16_recon;

/* kernel_advance arguments (obs_reward.py:410-438; MY_REWARD_CONFIG, my_reward.py:45-104) */
typedef struct {
  double dt;                    /* RL step, 0.1 s */
  double min_alt;               /* hard deck, m (304.8) */
  double max_time;              /* episode limit, s (200) */
  double own_damage_weight;
  double damage_scale;
  double shaping_reward_scale;
  double win_reward, loss_reward;
  double timeout_win_reward, timeout_loss_reward, timeout_draw_reward;
  double alt_hunt_coef;
  int32_t reward_mode;          /* 0 standard, 1 altitude hunt, 2 attack, 3 defense */
  int32_t reserved;
} f16_reward_cfg;

/* official N/E origin (ECEF m of BaseLat/BaseLon and its sin/cos; obs_reward.py:376-383) */
typedef struct {
  double ox, oy, oz, slat, clat, slon, clon;
} f16_origin;

/* init_reward_kernel: geometry / log-altitude trackers of the masked environments (mask NULL =
 * all). */
int f16_obs_init_reward(const double* state, int layout, int64_t ld, int64_t nenv,
                        const uint8_t* env_mask, const f16_recon* recon, const f16_origin* origin,
                        f16_stream_t stream);

/* advance_kernel: action-history push, damage/HP, fuel, SO(3) body rates, time, termination
 * (term/trunc [nenv] uint8) and reward [nac] fp64. actions [nac][4] fp64, 16-byte aligned. */
int f16_obs_advance(const double* state, int layout, int64_t ld, int64_t nenv, const double* actions,
                    const f16_recon* recon, const f16_reward_cfg* cfg, const f16_origin* origin,
                    double* reward, uint8_t* term, uint8_t* trunc_, f16_stream_t stream);

/* build_obs_kernel: obs [nac][184] fp32 (16-byte aligned) of the masked environments (NULL =
 * all; unmasked rows are left untouched), aux [nenv][21] fp64 future-position features or NULL. */
int f16_obs_build(const double* state, int layout, int64_t ld, int64_t nenv, const uint8_t* env_mask,
                  const f16_recon* recon, const f16_origin* origin, float* obs, double* aux,
                  f16_stream_t stream);

/* advance + build_obs of every environment in one launch (each FDM row read once). */
int f16_obs_step(const double* state, int layout, int64_t ld, int64_t nenv, const double* actions,
                 const f16_recon* recon, const f16_reward_cfg* cfg, const f16_origin* origin,
                 double* reward, uint8_t* term, uint8_t* trunc_, float* obs, double* aux,
                 f16_stream_t stream);

/* Everything GpuDogfightVecEnv.step does after the physics step (R/cuda_fdm/rl_env.py:514-551)
 * in one launch: advance (reward [nac], term/trunc/done [nenv] uint8), terminal observations
 * (terminal_obs [nac][184] fp32, or NULL to skip), terminal_hp / terminal_alt_m [nac] fp64
 * (radial MSL altitude of the pre-reset state), then for every finished environment the
 * autoreset: its two state rows are replaced by ic_pool[pick[e]] (ic_pool: [pool_size][2][101]
 * fp64 AoS, pick: [nenv] int64), its reconstruction buffers are reset as reset_envs does, the
 * reward trackers are re-anchored (init_reward_kernel) and obs [nac][184] receives the fresh
 * observation; live environments get their terminal observation in obs. */
int f16_env_post_step(double* state, int layout, int64_t ld, int64_t nenv, const double* actions,
                      const f16_recon* recon, const f16_reward_cfg* cfg, const f16_origin* origin,
                      const double* ic_pool, int64_t pool_size, const int64_t* pick,
                      double* reward, uint8_t* term, uint8_t* trunc_, uint8_t* done, float* obs,
                      float* terminal_obs, double* terminal_hp, double* terminal_alt_m, double* aux,
                      f16_stream_t stream);

/* Official 9-DoF export of every aircraft (R/cuda_fdm/rl_env.py:558-566 state9_flat):
 * s9 [nac][9] fp64 = N, E, D m; roll, pitch, yaw deg; body u, v, w m/s. */
int f16_state9(const double* state, int layout, int64_t ld, int64_t nac, const f16_origin* origin,
               double* s9, f16_stream_t stream);

/* External 214-D observation for frozen external opponents (no counterpart kernel on the main
 * path; replaces R/cuda_fdm/external_observation.cu external_acceleration / external_observation
 * launched by BatchObsReward.kernel_advance / build_external_obs, obs_reward.py:417-420, 487-496).
 * f16_external_accel: per aircraft NED velocity -> accel = (v - previous) / dt where valid[a]
 *   (the recon prev_valid BEFORE the advance updates it; 0 otherwise), previous = v.
 *   previous, accel: [nac][3] fp64.
 * f16_external_obs: out214 [nac][214] fp32 from the 184-D rows obs184 [nac][184] and accel. */
int f16_external_accel(const double* state, int layout, int64_t ld, int64_t nac, const uint8_t* valid,
                       double* previous, double* accel, const f16_origin* origin, double dt,
                       f16_stream_t stream);
int f16_external_obs(const double* state, int layout, int64_t ld, int64_t nac, const double* accel,
                     const float* obs184, float* out214, const f16_origin* origin, f16_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * (3) Policy / value MLP forward on the tcgen05 tensor cores (bf16 in, fp32 accumulate).
 * Replaces the rollout forwards of R/claude_code/model.py MLPDiscreteActorCritic (actor_logits,
 * critic; :162-241) driven by R/cuda_fdm/ppo_gpu.py actor_step / value_step (:273-291) and the
 * frozen-opponent pools OpponentPool.act / ActiveLeaguePool.act (:536-592, :877-898), with the
 * per-channel Categorical sample (Gumbel-max, counter-based RNG) and its summed log-probability
 * fused into the last layer.
 *
 * A network: n_layers <= 4 Linear layers (nn.Linear layout: weight [out][in] bf16 or fp16
 * row-major (the descriptor's operand type),
 * device, 16-byte aligned, in a multiple of 8), hidden widths multiples of 64 up to 512, ReLU
 * (activation 0) or tanh (1) after every hidden layer; head 1 = categorical with
 * width[last] = act_dim * num_bins <= 96, head 2 = value with width[last] = 1.
 * ---------------------------------------------------------------------------------------- */
typedef struct {
  int in_dim;
  int n_layers;
  int width[4];
  int activation;
  int head;
  int act_dim, num_bins;
  const void* weight[4];
  const float* bias[4];
  int operand;              /* F16_OPERAND_BF16 (0, a zero-initialised descriptor) or
                               F16_OPERAND_FP16: the type of the weights, of the policy input x
                               and of the hidden activations; one type for every network of a set */
  const float* head_weight_f32;  /* optional, value head (head 2) with n_layers >= 2: the head's
                               weight row in fp32, device, 16-byte aligned [width[n_layers-2]].
                               Such a head is computed in fp32 from the last hidden layer's fp32
                               activations (bias + activation, then the dot product with this row);
                               NULL: the same with weight[n_layers-1] converted to fp32 */
} f16_mlp_desc;

#define F16_OPERAND_BF16 0
#define F16_OPERAND_FP16 1

typedef struct f16_mlp_set_s f16_mlp_set;   /* opaque: up to 20 networks with their TMA maps */

/* Build the weight tensor maps of n networks (the weight / bias buffers must outlive the set). */
int f16_mlp_set_create(const f16_mlp_desc* descs, int n, f16_mlp_set** out);
int f16_mlp_set_destroy(f16_mlp_set* set);

typedef struct {
  const void* x;            /* [rows][ldx] policy input (normalised observations) in the set's operand
                               type (bf16 or fp16), device */
  int64_t rows, ldx;
  int n_groups;             /* row groups; group g owns rows [group_end[g-1], group_end[g]), every
                               group starting at a multiple of 128 rows */
  const int64_t* group_end; /* host [n_groups] */
  const int* group_net;     /* host [n_groups][nets_per_group]: network index in the set, -1 none */
  int nets_per_group;       /* 1 or 2 (e.g. actor + critic on the same rows) */
  uint8_t* bins;            /* categorical: sampled bins, row r at bins[r*bins_stride + bins_offset + c] */
  int64_t bins_stride;
  int bins_offset;
  int32_t* act_idx;         /* optional [rows][act_dim] int32 */
  float* logp;              /* [rows] summed log-probability of the sampled bins */
  float* value;             /* [rows] value head */
  float* logits;            /* optional [rows][logits_ld] raw head output (tests) */
  int64_t logits_ld;
  uint64_t seed, step;      /* RNG key of this call */
  int deterministic;        /* 1: argmax (the reference's deterministic=True / sample=False) */
  int* err;                 /* optional device int: set non-zero if a bounded wait timed out */
  /* optional env commands of the sampled bins, action_to_env (ppo_gpu.py:361-369) fused:
   * cmd[r*cmd_stride + cmd_offset + c] = (double)grid[bin] for c < 3 and
   * (double)(0.5f*grid[bin] + 0.5f) for the throttle channel c = 3 (fp32 arithmetic, as the
   * reference's float32 action tensor).  grid: device fp32 [num_bins] (torch.linspace). */
  double* cmd;
  int64_t cmd_stride;
  int cmd_offset;
  const float* grid;
  /* optional device counter added to `step` when the kernel runs (NULL: none), so one captured
   * CUDA graph can be replayed with a fresh RNG step each time */
  const uint64_t* step_dev;
  /* optional device int64 [n_groups]: the groups' cumulative row ends read by the kernel instead
   * of group_end (which is then ignored), for a grouping computed on the device without a host
   * round trip (the frozen-opponent pool, ppo_gpu.py:877-898).  Ends past `rows` are clamped;
   * group_net stays a host array. */
  const int64_t* group_end_dev;
} f16_policy_args;

int f16_policy_forward(const f16_mlp_set* set, const f16_policy_args* args, f16_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * (4) Rollout arithmetic (R/cuda_fdm/ppo_gpu.py).
 * f16_gae replaces the GAE loop of PPOGPUTrainer.collect_rollout (:1983-1995), bit for bit:
 * rew, val, done, adv, ret are [T][ld] fp32 (done = the episode-start flags b_done), last_val
 * and next_done [n] fp32; gamma and lam are the Python floats of the config.
 * ---------------------------------------------------------------------------------------- */
int f16_gae(const float* rew, const float* val, const float* done, const float* last_val,
            const float* next_done, int T, int64_t n, int64_t ld, double gamma, double lam,
            float* adv, float* ret, f16_stream_t stream);

/* RunningNorm.update (:195-207) over x [B][ldx] fp32 (D features): batch mean / population
 * variance merged into mean, var [D] and count [1] (fp32, device).  scratch: device buffer of
 * f16_norm_scratch_doubles(B, D) doubles, 16-byte aligned. */
int f16_norm_update(const float* x, int64_t B, int D, int64_t ldx, float* mean, float* var, float* count,
                    double* scratch, int64_t scratch_doubles, f16_stream_t stream);
int64_t f16_norm_scratch_doubles(int64_t B, int D);

/* The same update split in two around a cross-rank reduction (no counterpart in the reference,
 * which is single-GPU): f16_norm_sums writes sums [D][2] fp64 (sum, sum of squares of each
 * feature over this rank's B rows, 16-byte aligned); after an allreduce-sum of sums over the
 * ranks, f16_norm_merge_sums merges the global batch of B_total rows into mean / var / count,
 * so every rank holds the same normaliser.  On one rank the pair equals f16_norm_update bit
 * for bit. */
int f16_norm_sums(const float* x, int64_t B, int D, int64_t ldx, double* sums, double* scratch,
                  int64_t scratch_doubles, f16_stream_t stream);
int f16_norm_merge_sums(const double* sums, int64_t B_total, int D, float* mean, float* var,
                        float* count, f16_stream_t stream);

/* f16_norm_update without a caller scratch buffer (no counterpart in the reference).  For hosts
 * that may not allocate device memory inside their step loop (a sealed memory pool or arena):
 * the fp64 partial sums go to a library-owned device array of F16_NORM_STATIC_SCRATCH_PAIRS
 * (sum, sum of squares) pairs, so ceil(B / 512) * D must not exceed it (else
 * F16_ERR_TOO_LARGE, nothing launched).  No allocation happens in any call.  Every call made
 * outside a stream capture looks that array's address up (cudaGetSymbolAddress, with the device
 * current), so a device reset between calls is harmless; a call inside a capture uses the address
 * the last uncaptured call found, so make one call on the device before any stream capture.  Nothing needs to be zeroed beforehand.  The
 * array is shared per device: calls that may run at the same time on one device (different
 * streams or host threads) race; calls on one stream are ordered. */
#define F16_NORM_STATIC_SCRATCH_PAIRS 131072
int f16_norm_update_static(const float* x, int64_t B, int D, int64_t ldx, float* mean, float* var,
                           float* count, f16_stream_t stream);

/* RunningNorm.normalize (:209-212): clamp((x - mean) / sqrt(var + eps), +-clip) into y [B][ldy]
 * fp32 and/or y_bf16 [B][ldb] bf16 (columns D..ldb-1 zero-filled; either output may be NULL). */
int f16_norm_apply(const float* x, int64_t B, int D, int64_t ldx, const float* mean, const float* var,
                   double eps, double clip, float* y, int64_t ldy, void* y_bf16, int64_t ldb,
                   f16_stream_t stream);

/* The same, plus: mean == var == NULL passes the values through unchanged (the un-normalised
 * opponent input, ppo_gpu.py:583, cast into the bf16 layout), and `nonfinite` (device uint32,
 * optional) is incremented when an output value is NaN or infinite, so the rollout's final
 * isfinite check of the observation buffer (ppo_gpu.py:2003-2008) needs no extra pass. */
int f16_norm_apply_checked(const float* x, int64_t B, int D, int64_t ldx, const float* mean,
                           const float* var, double eps, double clip, float* y, int64_t ldy,
                           void* y_bf16, int64_t ldb, uint32_t* nonfinite, f16_stream_t stream);

/* f16_norm_apply_checked with the 16-bit output in either policy operand type: operand
 * F16_OPERAND_BF16 writes what f16_norm_apply_checked writes; F16_OPERAND_FP16 writes fp16
 * (round to nearest, saturated at +-65504, NaN kept) into y_half [B][ldh], the input of an
 * fp16 network set. */
int f16_norm_apply_half(const float* x, int64_t B, int D, int64_t ldx, const float* mean,
                        const float* var, double eps, double clip, float* y, int64_t ldy,
                        void* y_half, int64_t ldh, int operand, uint32_t* nonfinite, f16_stream_t stream);

/* Per-row-group normalise + scatter into a 16-bit policy input (no counterpart in the
 * reference, which runs one torch normalise per pool entry after a host-synchronised split,
 * ppo_gpu.py:877-898): row r of x [B][ldx] fp32 (D features) is normalised with the statistics
 * of group g = group_of_row[r] (mean_ptrs[g] / var_ptrs[g], device arrays of n_groups device
 * pointers to fp32 [D]; a NULL pair passes the row through unchanged) and written to row
 * dst_row[r] of y_half [*][ldh] (columns D..ldh-1 zero).  group_of_row and dst_row: device int64
 * [B]; a group index outside [0, n_groups) is an error recorded in *nonfinite's bit 31 (the row
 * is skipped), so nothing is read from a bad pointer. */
int f16_norm_apply_scatter(const float* x, int64_t B, int D, int64_t ldx, const int64_t* group_of_row,
                           const int64_t* dst_row, const float* const* mean_ptrs, const float* const* var_ptrs,
                           int n_groups, double eps, double clip, void* y_half, int64_t ldh, int operand,
                           uint32_t* nonfinite, f16_stream_t stream);

/* Per-step bookkeeping of collect_rollout (ppo_gpu.py:1914-1960) in one launch, after the env
 * step: b_rew[e] = (float)reward[2e]; next_done[e] = done[e]; ep_ret / ep_len updated and
 * reset on done exactly as the reference's fp32 expressions; and the rollout statistics
 * accumulated into stats (fp64, zeroed by the caller at rollout start):
 *   stats[0] ret_sum, [1] len_sum, [2] ep_count, [3] win_sum, [4] loss_sum, [5] alt_loss_sum,
 *   [6] opponent_alt_loss_sum, [7] set to 1 if any environment's finite flag is 0 (the
 *   reference's trajectory_finite, negated), [8 + g] win_by_opp[g],
 *   [8 + n_opp + g] loss_by_opp[g], [8 + 2 n_opp + g] ep_by_opp[g]   (n_opp <= 32).
 * Win / loss follow the reference (terminal HP and altitude vs min_alt, 1e-9 HP margin). */
typedef struct {
  const double* reward;        /* [nac] env reward; the learner is aircraft 2e */
  const uint8_t* done;         /* [nenv] */
  const double* terminal_hp;   /* [nac] */
  const double* terminal_alt;  /* [nac] m */
  const int64_t* opp_row;      /* [nenv] opponent index of each environment, or NULL */
  int n_opp;
  double min_alt;              /* m */
  const uint8_t* finite;       /* [nenv] terminal_state_finite of this step, or NULL */
  float* b_rew;                /* [nenv] rollout reward row t */
  float* next_done;            /* [nenv] */
  float* ep_ret;               /* [nenv] */
  float* ep_len;               /* [nenv] */
  double* stats;               /* [8 + 3 n_opp] */
} f16_record_args;
int f16_rollout_record(int64_t nenv, const f16_record_args* args, f16_stream_t stream);

/* Per-step scoring of batched payoff evaluation (R/cuda_fdm/batched_payoff.py:131-156; the
 * single-matchup form ppo_gpu.py:1467-1500), after the env step.  Environments still playing
 * their first game (finished[e] == 0) are active: an active environment whose terminal state
 * flag, terminal HP, terminal altitude or reward is not finite increments nonfinite.  An active
 * environment that is done is scored for the left policy, which flies aircraft left_slot[e]:
 * dead = HP <= 0 or altitude below min_alt; win = only the other side dead, or both alive and
 * left HP > right HP + 1e-9; loss symmetric; score 1 / 0.5 / 0 (win / draw / loss, fp32);
 * own_crash / opp_crash = the left / right aircraft's altitude below min_alt; finished[e] = 1;
 * and the finish count of its matchup (lanes consecutive environments per matchup) is
 * incremented -- the increment that completes the matchup writes final_step = step. */
typedef struct {
  const uint8_t* done;          /* [nenv] */
  const double* terminal_hp;    /* [nac] */
  const double* terminal_alt;   /* [nac] m */
  const uint8_t* finite;        /* [nenv] the step's terminal_state_finite */
  const double* reward;         /* [nac] */
  const uint8_t* left_slot;     /* [nenv] aircraft (0 / 1) flown by the left policy */
  int64_t lanes;                /* environments per matchup (> 0) */
  double min_alt;               /* m */
  int32_t step;                 /* 1-based step index */
  uint8_t* finished;            /* [nenv] */
  float* scores;                /* [nenv] */
  uint8_t* own_crash;           /* [nenv] */
  uint8_t* opp_crash;           /* [nenv] */
  int32_t* finished_count;      /* [nenv / lanes], zeroed by the caller */
  int32_t* final_step;          /* [nenv / lanes] */
  int32_t* nonfinite;           /* [1], zeroed by the caller */
  const int64_t* step_dev;      /* optional device counter added to `step` (graph replays), or NULL */
} f16_payoff_args;
int f16_payoff_record(int64_t nenv, const f16_payoff_args* args, f16_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * PPO update: fp32-accurate products on the bf16 tensor cores (no counterpart kernels in the
 * reference, whose update R/cuda_fdm/ppo_gpu.py:2020-2144 multiplies in fp32 with cuBLAS
 * SGEMM).  An fp32 value v is carried as three bf16 terms, hi = bf16(v), lo = bf16(v - hi),
 * mid = bf16(v - hi - lo) (round to nearest; both differences are exact in fp32), so
 * mid + lo + hi carries v's 24 significant bits.  A split row of `cols` values is three parts of
 * p = cols rounded up to 8 columns, [mid | lo | hi] (out[r][0..p) = mid, [p..2p) = lo,
 * [2p..3p) = hi), each part's columns cols..p zero, so every part starts 16-byte aligned; with
 * parts = 6 the row continues [lo | hi | hi], the A operand of one GEMM over all six term
 * products (B = [hi; hi; mid; lo; lo; hi]: hi*hi last in K).  Row strides >= parts * p.  cols
 * is a multiple of 4 everywhere; fp32 pointers are 16-byte aligned with row strides a multiple
 * of 4 elements, split pointers 8-byte aligned with row strides a multiple of 4. */
#define F16_ACT_NONE 0
#define F16_ACT_RELU 1   /* torch.relu: clamp_min(v, 0); backward threshold_backward(g, h, 0) */
#define F16_ACT_TANH 2   /* torch.tanh; backward g (1 - h h) */

/* Split of x [rows][cols] (row stride ldx) into out (row stride ldo). */
int f16_split3_bf16(const float* x, int64_t rows, int cols, int64_t ldx, void* out, int64_t ldo,
                    int parts, f16_stream_t stream);

/* A layer's epilogue (the bias add of torch's F.linear and the activation module that follows
 * it, R/claude_code/model.py:34-44): y [rows][cols] := act(y + bias) in place; if hs is
 * non-null also its split (row stride ldhs), the next layer's operand. */
int f16_bias_act_split(float* y, int64_t rows, int cols, int64_t ldy, const float* bias, int act,
                       void* hs, int64_t ldhs, int parts, f16_stream_t stream);

/* A layer's backward prologue: g_y = act'(g_h; h) (h = the layer's activated output, unread for
 * F16_ACT_NONE), written as its split gys (row stride ldgs), and col_part [nblk][cols]: block b's
 * column sums of g_y over rows [b rpb, (b + 1) rpb), rpb = ceil(rows / nblk), summed in a fixed
 * order (the bias gradient is the sum of the nblk rows).  cols <= 1024. */
int f16_act_grad_split(const float* gh, int64_t ldg, const float* h, int64_t ldh, int64_t rows, int cols,
                       int act, void* gys, int64_t ldgs, int parts, float* col_part, int nblk,
                       f16_stream_t stream);

/* A hidden layer followed by a width-1 Linear (the critic's value head, model.py:34-44 with
 * out_dim 1): y := act(y + bias) in place as f16_bias_act_split, and v[r] = sum_c y[r][c] wv[c]
 * + bv[0] (wv [cols], bv a device scalar). */
int f16_bias_act_value(float* y, int64_t rows, int cols, int64_t ldy, const float* bias, int act,
                       const float* wv, const float* bv, float* v, f16_stream_t stream);

/* Its backward: f16_act_grad_split with g_h[r][c] = gv[r] wv[c] formed in the kernel, plus
 * v_part [nblk][cols], block b's column sums of gv[r] h[r][c] (the head weight's gradient is
 * the sum of the nblk rows). */
int f16_act_grad_split_value(const float* gv, const float* wv, const float* h, int64_t ldh, int64_t rows,
                             int cols, int act, void* gys, int64_t ldgs, int parts, float* col_part,
                             float* v_part, int nblk, f16_stream_t stream);

/* The update's categorical head: torch.distributions.Categorical(logits=z.view(-1, A, B)) with
 * log_prob(action).sum(-1) and entropy().sum(-1) (MLPDiscreteActorCritic.evaluate_actions,
 * R/claude_code/model.py:198-215).  logits [M][A*B] (row stride ldz), action [M][A] as uint8
 * (act_bytes 1) or int64 (8), B <= 32, A*B <= 128.  Per group l = z - logsumexp(z),
 * p = softmax(l), log_prob = l[action], entropy = -sum(max(l, -FLT_MAX) p).  Forward writes
 * logp[M], ent[M] and ORs into *flags (zeroed by the caller) 1 for a NaN logit and 2 for an
 * action outside [0, B) -- the argument checks torch's distribution makes (the host raises). */
int f16_categorical_fwd(const float* logits, int64_t ldz, int64_t M, int A, int B, const void* action,
                        int act_bytes, float* logp, float* ent, int* flags, f16_stream_t stream);

/* Its gradient: gz [M][A*B] (row stride ldg) = g_lp (onehot(action) - p) - g_ent p (max(l, -FLT_MAX) + H)
 * per group, H the group's entropy; g_lp / g_ent [M] may be null (zero). */
int f16_categorical_bwd(const float* logits, int64_t ldz, int64_t M, int A, int B, const void* action,
                        int act_bytes, const float* g_lp, const float* g_ent, float* gz, int64_t ldg,
                        f16_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Diagnostics (no counterpart in the reference): FP64 FMA-pipe probe, the measured roofline
 * denominator of the FDM kernel.  Launches `blocks` x 256 threads running 8 independent FMA
 * chains for `iters` iterations; *flops receives the FP64 flop count (host pointer).
 * `scratch` must hold blocks*256 doubles (never written in practice).
 * ---------------------------------------------------------------------------------------- */
int f16_probe_fp64(double* scratch, int64_t iters, int blocks, double* flops, f16_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Library information.
 * ---------------------------------------------------------------------------------------- */
const char* f16_version(void);
const char* f16_status_string(int status);

#ifdef __cplusplus
}
#endif
#endif /* F16ENV_H */
