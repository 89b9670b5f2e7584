"""GAE and RunningNorm restatements -- TEST INFRASTRUCTURE ONLY.

``gae`` restates the rollout GAE of R/cuda_fdm/ppo_gpu.py:1983-1995 in numpy float32 with the
reference's operation order (each torch elementwise op rounds to fp32; Python scalars enter as
float32, and gamma * gae_lambda is a Python double product), so it matches the torch loop bit
for bit.  ``running_norm_update`` / ``running_norm_apply`` restate RunningNorm
(ppo_gpu.py:184-212) in float32.
"""
import numpy as np

F = np.float32


def gae(rew, val, done, last_val, next_done, gamma, lam):
    rew, val, done = (np.asarray(a, F) for a in (rew, val, done))
    last_val, next_done = np.asarray(last_val, F), np.asarray(next_done, F)
    T = rew.shape[0]
    g = F(gamma)
    gl = F(gamma * lam)
    adv = np.zeros_like(rew)
    lastgae = np.zeros(rew.shape[1], F)
    for t in reversed(range(T)):
        if t == T - 1:
            nnt = F(1.0) - next_done
            nv = last_val
        else:
            nnt = F(1.0) - done[t + 1]
            nv = val[t + 1]
        delta = (rew[t] + (g * nv) * nnt) - val[t]
        lastgae = delta + (gl * nnt) * lastgae
        adv[t] = lastgae
    return adv, adv + val


def running_norm_update(mean, var, count, x):
    """Chan merge of a batch into (mean, var, count) in float32 (ppo_gpu.py:195-207)."""
    x = np.asarray(x, np.float64)
    bm = x.mean(0).astype(F)
    bv = x.var(0).astype(F)
    bc = F(x.shape[0])
    mean, var, count = np.asarray(mean, F), np.asarray(var, F), F(count)
    delta = bm - mean
    tot = count + bc
    mean = mean + delta * (bc / tot)
    M2 = (var * count + bv * bc) + (delta * delta) * ((count * bc) / tot)
    return mean, M2 / tot, tot


def running_norm_apply(x, mean, var, eps=1e-8, clip=10.0):
    x = np.asarray(x, F)
    n = (x - mean) / np.sqrt(var + F(eps))
    return np.clip(n, -clip, clip)
