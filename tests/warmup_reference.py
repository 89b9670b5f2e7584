"""Host-checked staggered warm-up -- TEST INFRASTRUCTURE ONLY (the comparator of the device loop).

Restates the reference's loop (research/competition_36500/runtime/cuda_fdm/rl_env.py:386-441,
``GpuDogfightVecEnv._staggered_warmup``): every step the host tests the departure and capture
masks, re-seeds departed envs with boolean indexing, captures envs at their target phase with
boolean-indexed copies and stops once every env is captured; envs never captured are re-seeded
and captured at the end.  The physics / advance / reset calls are the env's own (the same
kernels the device loop launches), so a comparison pins the loop's bookkeeping: ages, targets,
departures, captures and the reconstruction buffers.

One deliberate difference from the reference, shared with the device loop so the two can be
compared bit for bit: departed envs are re-seeded from the env's IC pool at caller-given rows
(``pool_picks``) instead of with freshly sampled ICs (both come from the same official IC
distribution).
"""
import torch

STATE_N = 101


def host_checked_warmup(env, max_steps, actions, targ, pool_picks):
    """Run the reference loop on ``env`` from its current state.  ``actions[i]`` is the (nac, 4)
    command of step i; ``targ`` the per-env target phases; ``pool_picks`` as for
    ``GpuDogfightVecEnv._warmup_loop_device``.  Returns (captured states, captured
    reconstruction buffers, finite flag, steps run, departure events)."""
    dev = env.device
    age = torch.zeros(env.nenv, dtype=torch.long, device=dev)
    captured_mask = torch.zeros(env.nenv, dtype=torch.bool, device=dev)
    captured = env.sim.states.clone()
    obr_buf = env.obr.clone_state()
    captured_mask |= targ == 0
    warm_finite = torch.ones((), dtype=torch.bool, device=dev)

    def reseed(mask, i):
        rows = mask.repeat_interleave(2)
        picked = env.ic_pool[pool_picks[i]].reshape(env.nac, STATE_N)
        env.sim.states[rows] = picked[rows]
        env.obr.reset_envs(mask)
        env.obr.kernel_init_reward_state(env.sim.states, mask)

    steps = departures = 0
    for i in range(max_steps):
        a = actions[i]
        env.sim.step(a, substeps=env.substeps)
        steps += 1
        finite_env = torch.isfinite(env.sim.states).reshape(env.nenv, -1).all(dim=1)
        warm_finite.logical_and_((finite_env | captured_mask).all())
        env.obr.kernel_advance(env.sim.states, a.contiguous(), cfg=env.reward_cfg, min_alt=env.min_altitude_m,
                               max_time=env.max_engage_time_s)
        s9 = env.state9_flat().view(env.nenv, 2, 9)
        alt = -s9[:, :, 2]
        dep = ((alt < 100.0) | (~torch.isfinite(s9).all(dim=2))).any(dim=1) & (~captured_mask)
        if bool(dep.any()):
            departures += int(dep.sum())
            reseed(dep, i)
            age[dep] = 0
        age = age + (~captured_mask).long()
        hit = (~captured_mask) & (age == targ)
        if bool(hit.any()):
            rows = hit.repeat_interleave(2)
            captured[rows] = env.sim.states[rows]
            env.obr.capture_into(obr_buf, hit)
            captured_mask |= hit
        if bool(captured_mask.all()):
            break
    if not bool(captured_mask.all()):
        rest = ~captured_mask
        reseed(rest, max_steps)
        rows = rest.repeat_interleave(2)
        captured[rows] = env.sim.states[rows]
        env.obr.capture_into(obr_buf, rest)
    return captured, obr_buf, bool(warm_finite), steps, departures
