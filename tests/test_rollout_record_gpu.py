"""Step-level fusions of the rollout -- needs a B200.

* f16_fdm_step_ex: same state as f16_fdm_step bit for bit, and its per-aircraft finite flag
  equals torch.isfinite(state).all() after the step (the reference's terminal_state_finite,
  R/cuda_fdm/rl_env.py:517), including aircraft whose seeds carry a NaN / inf (every table
  index in the kernel comes from bounded comparisons, so non-finite inputs stay in bounds).
* f16_rollout_record: against the reference's torch bookkeeping of collect_rollout
  (ppo_gpu.py:1914-1960) over two consecutive steps: reward row, next-done, episode return and
  length bit for bit; counts exactly; return / length sums within 1e-4 relative + 1e-2 (the
  kernel sums in fp64, torch in fp32 with cancellation).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import GOLDEN, pkg_module

pytestmark = pytest.mark.gpu


def test_fdm_step_ex_finite_flags(cuda):
    _lib = pkg_module("_lib")
    ge = pkg_module("gpu_env")
    ic = pkg_module("ic")
    L = _lib.load()
    g = np.load(GOLDEN / "fdm_cfg1.npz")
    seeds = torch.as_tensor(g["seeds"]).clone()
    seeds[5, 6] = float("nan")                 # quaternion component
    seeds[9, 3] = float("inf")                 # ECI velocity
    seeds[11, 40] = float("inf")               # a history slot the step overwrites unread
    nac = seeds.shape[0]
    fcs_dt = float(g["fcs_dt"])
    cmd = ic.bins_to_commands(torch.as_tensor(g["bins"][0])).double().to(cuda).contiguous()
    a = ge.GpuDogfight(nac // 2, substeps=6, fcs_dt=fcs_dt, device=cuda)
    b = ge.GpuDogfight(nac // 2, substeps=6, fcs_dt=fcs_dt, device=cuda)
    a.load_seed(seeds); b.load_seed(seeds)
    s = _lib.stream_of(a.states_soa)
    _lib.check(L.f16_fdm_step(_lib.ptr(a.states_soa), 0, nac, nac, _lib.ptr(cmd), 6, fcs_dt, None, s), "step")
    finite = torch.full((nac,), 7, dtype=torch.uint8, device=cuda)
    io = _lib.FdmIO(cmd=cmd.data_ptr(), finite=finite.data_ptr())
    _lib.check(L.f16_fdm_step_ex(_lib.ptr(b.states_soa), 0, nac, nac, C.byref(io), 6, fcs_dt, s), "step_ex")
    torch.cuda.synchronize()
    sa, sb = a.states_soa, b.states_soa
    assert torch.equal(torch.isnan(sa), torch.isnan(sb))
    assert torch.equal(torch.nan_to_num(sa, 0.0, 1.0, -1.0), torch.nan_to_num(sb, 0.0, 1.0, -1.0))
    exp = torch.isfinite(sb).all(dim=0).to(torch.uint8)
    assert torch.equal(finite, exp)
    assert int(exp[5]) == 0 and int(exp[9]) == 0 and int(exp.sum()) >= nac - 3


def torch_record(st, reward, done, th, ta, rows, n_opp, min_alt, finite):
    """The reference's per-step expressions (ppo_gpu.py:1914-1960) on the same buffers."""
    raw_reward = reward[:, 0].float()
    done_env = done.float()
    st["b_rew"] = raw_reward
    st["next_done"] = done_env
    st["traj"] = st["traj"] & finite.all()
    st["ep_ret"] += raw_reward
    st["ep_len"] += 1.0
    st["ret_sum"] += (st["ep_ret"] * done_env).sum()
    st["len_sum"] += (st["ep_len"] * done_env).sum()
    st["ep_count"] += done_env.sum()
    keep = 1.0 - done_env
    st["ep_ret"] = st["ep_ret"] * keep
    st["ep_len"] = st["ep_len"] * keep
    own_alt_dead = ta[:, 0] < min_alt
    own_dead = (th[:, 0] <= 0.0) | own_alt_dead
    opp_dead = (th[:, 1] <= 0.0) | (ta[:, 1] < min_alt)
    both_alive = (~own_dead) & (~opp_dead)
    win = (opp_dead & ~own_dead) | (both_alive & (th[:, 0] > th[:, 1] + 1e-9))
    loss = (own_dead & ~opp_dead) | (both_alive & (th[:, 0] < th[:, 1] - 1e-9))
    done_b = done.bool()
    dwin = (win & done_b).float()
    dloss = (loss & done_b).float()
    st["win_sum"] += dwin.sum(); st["loss_sum"] += dloss.sum()
    st["alt_loss_sum"] += (loss & own_alt_dead & done_b).float().sum()
    st["opponent_alt_loss_sum"] += (win & (ta[:, 1] < min_alt) & done_b).float().sum()
    st["win_by_opp"].scatter_add_(0, rows, dwin)
    st["loss_by_opp"].scatter_add_(0, rows, dloss)
    st["ep_by_opp"].scatter_add_(0, rows, done_b.float())


def test_rollout_record_matches_reference_bookkeeping(cuda):
    _lib = pkg_module("_lib")
    L = _lib.load()
    n, P, min_alt = 50_000, 5, 304.8
    gen = torch.Generator(device=cuda).manual_seed(3)
    dev = cuda
    ep_ret = torch.randn(n, device=dev, generator=gen) * 3
    ep_len = torch.randint(0, 100, (n,), device=dev, generator=gen).float()
    stats = torch.zeros(8 + 3 * P, dtype=torch.float64, device=dev)
    next_done = torch.zeros(n, device=dev)
    b_rew = torch.zeros(n, device=dev)
    ref = {"ep_ret": ep_ret.clone(), "ep_len": ep_len.clone(), "traj": torch.ones((), dtype=torch.bool, device=dev)}
    for k in ("ret_sum", "len_sum", "ep_count", "win_sum", "loss_sum", "alt_loss_sum", "opponent_alt_loss_sum"):
        ref[k] = torch.zeros((), device=dev)
    for k in ("win_by_opp", "loss_by_opp", "ep_by_opp"):
        ref[k] = torch.zeros(P, device=dev)
    rows = torch.randint(0, P, (n,), device=dev, generator=gen)
    for step in range(2):
        reward = torch.randn(n, 2, dtype=torch.float64, device=dev, generator=gen)
        done = torch.rand(n, device=dev, generator=gen) < 0.3
        th = torch.rand(n, 2, dtype=torch.float64, device=dev, generator=gen) * 1.2 - 0.2
        th[:100, 1] = th[:100, 0] + 5e-10               # HP ties inside the 1e-9 margin
        ta = torch.rand(n, 2, dtype=torch.float64, device=dev, generator=gen) * 2000.0
        finite = torch.rand(n, device=dev, generator=gen) > (1e-4 if step == 1 else 0.0)
        a = _lib.RecordArgs(reward=reward.data_ptr(), done=done.data_ptr(), terminal_hp=th.data_ptr(),
                            terminal_alt=ta.data_ptr(), opp_row=rows.data_ptr(), n_opp=P, min_alt=min_alt,
                            finite=finite.data_ptr(), b_rew=b_rew.data_ptr(), next_done=next_done.data_ptr(),
                            ep_ret=ep_ret.data_ptr(), ep_len=ep_len.data_ptr(), stats=stats.data_ptr())
        _lib.check(L.f16_rollout_record(n, C.byref(a), _lib.stream_of(stats)), "f16_rollout_record")
        torch_record(ref, reward, done, th, ta, rows, P, min_alt, finite)
        torch.cuda.synchronize()
        assert torch.equal(b_rew, ref["b_rew"]) and torch.equal(next_done, ref["next_done"])
        assert torch.equal(ep_ret, ref["ep_ret"]) and torch.equal(ep_len, ref["ep_len"])
        st = stats.cpu()
        for i, k in enumerate(("ret_sum", "len_sum")):
            np.testing.assert_allclose(float(st[i]), float(ref[k]), rtol=1e-4, atol=1e-2, err_msg=k)
        for i, k in enumerate(("ep_count", "win_sum", "loss_sum", "alt_loss_sum", "opponent_alt_loss_sum")):
            assert float(st[2 + i]) == float(ref[k]), k
        assert (float(st[7]) == 0.0) == bool(ref["traj"])
        for j, k in enumerate(("win_by_opp", "loss_by_opp", "ep_by_opp")):
            assert torch.equal(st[8 + j * P:8 + (j + 1) * P].float(), ref[k].cpu()), k
