"""The seeded PPO-update case of ppo_update.npz, shared by make_golden.py (which runs the
reference's update on it) and tests/test_ppo_update.py (which runs this package's)."""
import torch

PPO_CFG = dict(update_epochs=3, num_minibatches=4, target_kl=0.03, ent_coef=0.01, clip_coef=0.2, vf_coef=0.5,
               max_grad_norm=0.5, lr=3e-4, norm_adv=True)
PPO_HIDDEN = (32, 32)


def ppo_inputs(model, seed, T=4, n=48):
    """Deterministic rollout of ppo_update.npz: observations, actions, old log-probs near the
    initial policy's (so ratios straddle the clip range), values, advantages, returns."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    obs = torch.randn(T, n, 184, generator=g)
    act = torch.randint(0, 21, (T, n, 4), generator=g)
    with torch.no_grad():
        lp, _ = model.evaluate_actions(obs.flatten(0, 1), act.flatten(0, 1))
    old_logp = lp.view(T, n) + 0.2 * torch.randn(T, n, generator=g)
    b_val = torch.randn(T, n, generator=g)
    adv = torch.randn(T, n, generator=g) * 2.0
    ret = adv + b_val
    return obs, act, old_logp, b_val, adv, ret
