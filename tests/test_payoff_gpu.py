"""Batched payoff evaluation on a B200.

* f16_payoff_record against oracle/payoff.py over twelve random steps: scores, crash flags,
  finished lanes, matchup completion step and the non-finite count, bit for bit; and over the
  steps of tests/golden/payoff.npz against what the reference's own evaluate_chunk loop scored.
* BatchedPayoff with argmax policies: a matchup's result does not depend on the other
  matchups in the batch (rights [B, C, B] give matchups 0 and 2 identical results, equal to a
  run of [B] alone), with a normaliser on one policy and a 214-D external-observation policy.
* Sampled policies: the same evaluation seed replays exactly; every lane scores 0 / 0.5 / 1.
"""
import numpy as np
import pytest
import torch

from conftest import pkg_module
from oracle import payoff as OP

pytestmark = pytest.mark.gpu


def test_payoff_record_kernel_matches_oracle(cuda):
    _lib = pkg_module("_lib")
    L = _lib.load()
    rng = np.random.default_rng(11)
    nenv, lanes, min_alt = 96, 16, 304.8
    nm = nenv // lanes
    left_slot = (np.arange(nenv) % lanes >= lanes // 2).astype(np.uint8)
    o = dict(fin=np.zeros(nenv, np.uint8), sc=np.full(nenv, np.nan, np.float32), oc=np.zeros(nenv, np.uint8),
             pc=np.zeros(nenv, np.uint8), cnt=np.zeros(nm, np.int64), fs=np.zeros(nm, np.int64))
    dv = dict(fin=torch.zeros(nenv, dtype=torch.uint8, device=cuda),
              sc=torch.full((nenv,), float("nan"), device=cuda),
              oc=torch.zeros(nenv, dtype=torch.uint8, device=cuda), pc=torch.zeros(nenv, dtype=torch.uint8, device=cuda),
              cnt=torch.zeros(nm, dtype=torch.int32, device=cuda), fs=torch.zeros(nm, dtype=torch.int32, device=cuda),
              bad=torch.zeros(1, dtype=torch.int32, device=cuda))
    ls_d = torch.as_tensor(left_slot, device=cuda)
    for step in range(1, 13):
        hp = rng.choice([0.0, 0.25, 0.5, 0.5 + 5e-10, 0.5 + 2e-9, 1.0], size=(nenv, 2))
        alt = rng.choice([200.0, 304.8, 304.9, 5000.0], size=(nenv, 2))
        done = (rng.random(nenv) < (1.0 if step == 12 else 0.3)).astype(np.uint8)
        finite = (rng.random(nenv) > (0.05 if step == 4 else 0.0)).astype(np.uint8)
        reward = rng.normal(size=(nenv, 2))
        if step == 7:
            reward[rng.random(nenv) < 0.05, 1] = np.inf
        bad = OP.payoff_record(done, hp.ravel(), alt.ravel(), finite, reward.ravel(), left_slot, lanes, min_alt,
                               step, o["fin"], o["sc"], o["oc"], o["pc"], o["cnt"], o["fs"])
        t = {k: torch.as_tensor(np.ascontiguousarray(v), device=cuda)
             for k, v in dict(done=done, hp=hp.ravel(), alt=alt.ravel(), finite=finite, reward=reward.ravel()).items()}
        dv["bad"].zero_()
        a = _lib.PayoffArgs(done=t["done"].data_ptr(), terminal_hp=t["hp"].data_ptr(), terminal_alt=t["alt"].data_ptr(),
                            finite=t["finite"].data_ptr(), reward=t["reward"].data_ptr(), left_slot=ls_d.data_ptr(),
                            lanes=lanes, min_alt=min_alt, step=step, finished=dv["fin"].data_ptr(),
                            scores=dv["sc"].data_ptr(), own_crash=dv["oc"].data_ptr(), opp_crash=dv["pc"].data_ptr(),
                            finished_count=dv["cnt"].data_ptr(), final_step=dv["fs"].data_ptr(),
                            nonfinite=dv["bad"].data_ptr())
        _lib.check(L.f16_payoff_record(nenv, a, _lib.stream_of(dv["sc"])), "f16_payoff_record")
        torch.cuda.synchronize()
        assert int(dv["bad"].item()) == bad
        assert np.array_equal(dv["fin"].cpu().numpy(), o["fin"])
        np.testing.assert_array_equal(dv["sc"].cpu().numpy(), o["sc"])
        assert np.array_equal(dv["oc"].cpu().numpy(), o["oc"])
        assert np.array_equal(dv["pc"].cpu().numpy(), o["pc"])
        assert dv["cnt"].cpu().numpy().tolist() == o["cnt"].tolist()
        assert dv["fs"].cpu().numpy().tolist() == o["fs"].tolist()
    assert o["fin"].all()



def test_payoff_record_kernel_matches_reference_run(cuda):
    """The kernel over payoff.npz's scripted steps gives the reference loop's scores, crash
    flags and completion steps (batched_payoff.py:131-156 run on CPU when the fixture was made)."""
    from test_payoff import check_against_reference, replay_payoff_fixture
    _lib = pkg_module("_lib")
    L = _lib.load()
    dv = {}

    def kernel_record(step, d, left_slot, lanes, min_alt, st):
        nenv = d["done"].shape[0]
        if not dv:
            dv.update(fin=torch.zeros(nenv, dtype=torch.uint8, device=cuda),
                      sc=torch.full((nenv,), float("nan"), device=cuda),
                      oc=torch.zeros(nenv, dtype=torch.uint8, device=cuda),
                      pc=torch.zeros(nenv, dtype=torch.uint8, device=cuda),
                      cnt=torch.zeros(len(st["cnt"]), dtype=torch.int32, device=cuda),
                      fs=torch.zeros(len(st["fs"]), dtype=torch.int32, device=cuda),
                      bad=torch.zeros(1, dtype=torch.int32, device=cuda),
                      ls=torch.as_tensor(left_slot, device=cuda))
        t = {k: torch.as_tensor(np.ascontiguousarray(v), device=cuda)
             for k, v in dict(done=d["done"].astype(np.uint8), hp=d["hp"].ravel(), alt=d["alt"].ravel(),
                              finite=d["finite"].astype(np.uint8), reward=d["reward"].ravel()).items()}
        dv["bad"].zero_()
        a = _lib.PayoffArgs(done=t["done"].data_ptr(), terminal_hp=t["hp"].data_ptr(), terminal_alt=t["alt"].data_ptr(),
                            finite=t["finite"].data_ptr(), reward=t["reward"].data_ptr(),
                            left_slot=dv["ls"].data_ptr(), lanes=lanes, min_alt=min_alt, step=step,
                            finished=dv["fin"].data_ptr(), scores=dv["sc"].data_ptr(), own_crash=dv["oc"].data_ptr(),
                            opp_crash=dv["pc"].data_ptr(), finished_count=dv["cnt"].data_ptr(),
                            final_step=dv["fs"].data_ptr(), nonfinite=dv["bad"].data_ptr())
        _lib.check(L.f16_payoff_record(nenv, a, _lib.stream_of(dv["sc"])), "f16_payoff_record")
        torch.cuda.synchronize()
        st["bad"].append(int(dv["bad"].item()))
        for k in ("fin", "sc", "oc", "pc", "cnt", "fs"):
            st[k][:] = dv[k].cpu().numpy()

    g, st = replay_payoff_fixture(kernel_record)
    check_against_reference(g, st)

def _policies(cuda):
    tr = pkg_module("trainer")
    ro = pkg_module("rollout")
    payoff = pkg_module("payoff")
    mk = lambda s, d=184: (torch.manual_seed(s), tr.MLPActorCritic(obs_dim=d, hidden=(128, 128),
                                                                   activation="relu").to(cuda))[1]
    A, B, C, E = mk(1), mk(2), mk(3), mk(4, 214)
    norm = ro.RunningNorm(184, cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    norm.update(torch.randn(4096, 184, device=cuda, generator=g) * 3.0 + 1.0)
    return (payoff.EvalPolicy(A), payoff.EvalPolicy(B, norm), payoff.EvalPolicy(C), payoff.EvalPolicy(E))


def _key(s):
    return (s["paired_scores"], s["steps"], s["wins"], s["losses"], s["own_alt_loss_count"],
            s["opponent_alt_loss_count"])


def test_batched_matchups_are_independent(cuda):
    payoff = pkg_module("payoff")
    A, B, C, E = _policies(cuda)
    bp = payoff.BatchedPayoff(per_order=8, capacity=4, seed=3, device=cuda)
    res = bp.evaluate(A, [B, C, B, E], seed_block=1, sample=False)
    assert _key(res[0]) == _key(res[2])
    alone_b = bp.evaluate(A, [B], seed_block=1, sample=False)[0]
    alone_e = bp.evaluate(A, [E], seed_block=1, sample=False)[0]
    assert _key(alone_b) == _key(res[0])
    assert _key(alone_e) == _key(res[3])
    for r in res:
        assert r["games"] == 16 and r["wins"] + r["draws"] + r["losses"] == 16 and r["steps"] > 0


def test_sampled_evaluation_replays(cuda):
    payoff = pkg_module("payoff")
    A, B, C, _ = _policies(cuda)
    bp = payoff.BatchedPayoff(per_order=8, capacity=2, seed=9, device=cuda)
    r1 = bp.evaluate(A, [B, C], seed_block=2)
    r2 = bp.evaluate(A, [B, C], seed_block=2)
    assert [_key(x) for x in r1] == [_key(x) for x in r2]
    for r in r1:
        assert set(np.unique(np.asarray(r["paired_scores"]) * 2).tolist()) <= {0.0, 0.5, 1.0, 1.5, 2.0}
        assert r["stochastic"] and r["policy_rng_seed"] == r2[0]["policy_rng_seed"]


def test_graph_replay_equals_eager(cuda):
    """The captured decision graph (device step counter) reproduces the eager loop exactly."""
    payoff = pkg_module("payoff")
    A, B, C, _ = _policies(cuda)
    bp = payoff.BatchedPayoff(per_order=4, capacity=2, seed=21, device=cuda)
    g = bp.evaluate(A, [B, C], seed_block=3, use_graph=True)
    e = bp.evaluate(A, [B, C], seed_block=3, use_graph=False, check_every=1)
    assert [_key(x) for x in g] == [_key(x) for x in e]
