"""PPO update (trainer.ppo_update) on CPU: parity with the reference's own update, and the
data-parallel path on two gloo ranks.

1. tests/golden/ppo_update.npz holds the parameters and statistics after the reference's
   PPOGPUTrainer.update (R/cuda_fdm/ppo_gpu.py:2020-2144) on a seeded rollout; this package's
   update on the same rollout, model initialisation and RNG seed must reproduce them (parameters
   within 1e-6 absolute + 1e-5 relative; epoch count, early stop and optimiser steps exact).
2. Two gloo ranks each holding half of a rollout, one epoch of one minibatch: gradients are
   averaged over the ranks and advantages normalised over the union, so the parameters after
   the step equal a single-rank update on the concatenated rollout within 2e-6 (summation order
   differs) and are identical on both ranks.
"""
import os
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import GOLDEN, pkg_module

sys.path.insert(0, str(GOLDEN))
from ppo_case import PPO_CFG, PPO_HIDDEN, ppo_inputs  # noqa: E402


def _flat(model):
    return torch.cat([p.detach().reshape(-1) for p in model.parameters()])


def test_update_matches_reference_golden():
    tr = pkg_module("trainer")
    g = np.load(GOLDEN / "ppo_update.npz")
    seed = int(g["seed"])
    torch.manual_seed(seed)
    model = tr.MLPActorCritic(184, 4, 21, hidden=PPO_HIDDEN, activation="tanh")
    init = _flat(model).double()
    np.testing.assert_allclose([float(init.sum()), float(init.abs().sum())], g["init_sum"], rtol=1e-12)
    obs, act, old_logp, b_val, adv, ret = ppo_inputs(model, seed)
    cfg = tr.PPOConfig(hidden=PPO_HIDDEN, activation="tanh", **PPO_CFG)
    a_opt = torch.optim.Adam(model.actor_parameters(), lr=cfg.lr, eps=1e-5)
    c_opt = torch.optim.Adam(model.critic_parameters(), lr=cfg.lr, eps=1e-5)
    torch.manual_seed(seed + 1)
    res = tr.ppo_update(model, a_opt, c_opt, cfg, obs, act.to(torch.uint8), old_logp, b_val, adv, ret)
    got = _flat(model).numpy()
    np.testing.assert_allclose(got, g["params"], atol=1e-6, rtol=1e-5)
    assert res["epochs"] == int(g["epochs"]) and res["early"] == bool(g["early"])
    assert res["optimizer_steps"] == int(g["optimizer_steps"])
    for k in ("pl", "vl", "ent", "kl", "cf", "ev", "actor_grad_norm", "critic_grad_norm"):
        np.testing.assert_allclose(float(res[k]), float(g[k]), rtol=1e-5, atol=1e-7, err_msg=k)


def _dp_rank(rank, world, port, path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tr = pkg_module("trainer")
        torch.manual_seed(7)
        model = tr.MLPActorCritic(184, 4, 21, hidden=PPO_HIDDEN, activation="tanh")
        obs, act, old_logp, b_val, adv, ret = ppo_inputs(model, 11, T=4, n=64)
        half = slice(rank * 32, (rank + 1) * 32)           # this rank's environments
        cfg = tr.PPOConfig(hidden=PPO_HIDDEN, activation="tanh", update_epochs=1, num_minibatches=1,
                           target_kl=None, ent_coef=0.01)
        a_opt = torch.optim.Adam(model.actor_parameters(), lr=cfg.lr, eps=1e-5)
        c_opt = torch.optim.Adam(model.critic_parameters(), lr=cfg.lr, eps=1e-5)
        tr.ppo_update(model, a_opt, c_opt, cfg, obs[:, half], act[:, half], old_logp[:, half], b_val[:, half],
                      adv[:, half], ret[:, half], group=dist.group.WORLD)
        torch.save(_flat(model), f"{path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_data_parallel_update_equals_single_rank_on_concatenation(tmp_path):
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "params")
    mp.start_processes(_dp_rank, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    p0, p1 = torch.load(f"{path}.0"), torch.load(f"{path}.1")
    assert torch.equal(p0, p1), "ranks diverged"

    tr = pkg_module("trainer")
    torch.manual_seed(7)
    model = tr.MLPActorCritic(184, 4, 21, hidden=PPO_HIDDEN, activation="tanh")
    start = _flat(model).clone()
    obs, act, old_logp, b_val, adv, ret = ppo_inputs(model, 11, T=4, n=64)
    cfg = tr.PPOConfig(hidden=PPO_HIDDEN, activation="tanh", update_epochs=1, num_minibatches=1, target_kl=None,
                       ent_coef=0.01)
    a_opt = torch.optim.Adam(model.actor_parameters(), lr=cfg.lr, eps=1e-5)
    c_opt = torch.optim.Adam(model.critic_parameters(), lr=cfg.lr, eps=1e-5)
    tr.ppo_update(model, a_opt, c_opt, cfg, obs, act, old_logp, b_val, adv, ret)
    single = _flat(model)
    assert float((single - start).abs().max()) > 1e-5          # the step moved the parameters
    torch.testing.assert_close(p0, single, atol=2e-6, rtol=0.0)
