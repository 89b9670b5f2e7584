"""Batched payoff scoring oracle (CPU).

oracle/payoff.py restates the per-lane scoring of R/cuda_fdm/batched_payoff.py:131-156.  Here
it is pinned against a line-by-line torch transcription of those expressions (the reference
computes them inline in evaluate_chunk, which needs its trainer and a CUDA env) over random
multi-step inputs with ties, altitude losses, double kills and non-finite values, and against
hand-scored cases.  summarize_pair's counts are checked against the oracle's outcome_summary.
"""
import numpy as np
import torch

from conftest import pkg_module
from oracle import payoff as OP


def torch_reference_step(st, done, hp, alt, finite, reward, left_slot, min_alt, lanes, step):
    """batched_payoff.py:131-156 as written (torch, nenv lanes, the reference's names)."""
    nenv = done.shape[0]
    all_rows = torch.arange(nenv)
    active = ~st["finished"]
    fin = (finite & torch.isfinite(hp).all(dim=1) & torch.isfinite(alt).all(dim=1)
           & torch.isfinite(reward).all(dim=1))
    finite_ok = bool((fin | ~active).all())
    newly = done.bool() & active
    lhp, rhp = hp[all_rows, left_slot], hp[all_rows, 1 - left_slot]
    lalt, ralt = alt[all_rows, left_slot], alt[all_rows, 1 - left_slot]
    ld = (lhp <= 0) | (lalt < min_alt)
    rd = (rhp <= 0) | (ralt < min_alt)
    alive = ~ld & ~rd
    win = (rd & ~ld) | (alive & (lhp > rhp + 1e-9))
    loss = (ld & ~rd) | (alive & (lhp < rhp - 1e-9))
    st["scores"] = torch.where(newly, win.float() + .5 * (~win & ~loss).float(), st["scores"])
    st["own"] = torch.where(newly, lalt < min_alt, st["own"])
    st["opp"] = torch.where(newly, ralt < min_alt, st["opp"])
    st["finished"] |= newly
    done_m = st["finished"].view(-1, lanes).all(dim=1).tolist()
    for i, d in enumerate(done_m):
        if d and not st["steps"][i]:
            st["steps"][i] = step
    return finite_ok


def random_step(rng, nenv, p_done=0.3, p_bad=0.0):
    hp = rng.choice([0.0, 0.25, 0.5, 0.5 + 5e-10, 0.5 + 2e-9, 1.0], size=(nenv, 2))
    alt = rng.choice([200.0, 304.8, 304.9, 5000.0], size=(nenv, 2))
    done = (rng.random(nenv) < p_done).astype(np.uint8)
    finite = np.ones(nenv, np.uint8)
    reward = rng.normal(size=(nenv, 2))
    if p_bad:
        bad = rng.random(nenv) < p_bad
        hp[bad, 0] = np.nan
    return done, hp, alt, finite, reward


def test_oracle_matches_reference_expressions():
    rng = np.random.default_rng(7)
    nenv, lanes, min_alt = 48, 8, 304.8
    left_slot = (np.arange(nenv) % lanes >= lanes // 2).astype(np.uint8)
    st = {"finished": torch.zeros(nenv, dtype=torch.bool), "scores": torch.full((nenv,), float("nan")),
          "own": torch.zeros(nenv, dtype=torch.bool), "opp": torch.zeros(nenv, dtype=torch.bool),
          "steps": [0] * (nenv // lanes)}
    fin = np.zeros(nenv, np.uint8)
    sc = np.full(nenv, np.nan, np.float32)
    oc = np.zeros(nenv, np.uint8)
    pc = np.zeros(nenv, np.uint8)
    cnt = np.zeros(nenv // lanes, np.int64)
    fs = np.zeros(nenv // lanes, np.int64)
    for step in range(1, 13):
        done, hp, alt, finite, reward = random_step(rng, nenv, p_bad=0.05 if step == 6 else 0.0)
        if step == 12:
            done[:] = 1
        ok_ref = torch_reference_step(st, torch.as_tensor(done), torch.as_tensor(hp), torch.as_tensor(alt),
                                      torch.as_tensor(finite.astype(bool)), torch.as_tensor(reward),
                                      torch.as_tensor(left_slot.astype(np.int64)), min_alt, lanes, step)
        bad = OP.payoff_record(done, hp.ravel(), alt.ravel(), finite, reward.ravel(), left_slot, lanes, min_alt,
                               step, fin, sc, oc, pc, cnt, fs)
        assert (bad == 0) == ok_ref
        assert np.array_equal(fin.astype(bool), st["finished"].numpy())
        np.testing.assert_array_equal(sc, st["scores"].numpy())
        assert np.array_equal(oc.astype(bool), st["own"].numpy())
        assert np.array_equal(pc.astype(bool), st["opp"].numpy())
        assert fs.tolist() == st["steps"]
    assert fin.all() and set(np.unique(sc).tolist()) <= {0.0, 0.5, 1.0}


def test_hand_scored_cases():
    # lane: (hp_left, hp_right, alt_left, alt_right) with left flying aircraft 0 or 1
    cases = [((1.0, 0.0, 5000, 5000), 1.0), ((0.0, 1.0, 5000, 5000), 0.0), ((0.0, 0.0, 5000, 5000), 0.5),
             ((0.6, 0.5, 5000, 5000), 1.0), ((0.5, 0.5 + 5e-10, 5000, 5000), 0.5),
             ((0.5, 0.5 + 2e-9, 5000, 5000), 0.0), ((1.0, 1.0, 100, 5000), 0.0), ((1.0, 0.2, 5000, 100), 1.0),
             ((1.0, 1.0, 100, 100), 0.5)]
    for slot in (0, 1):
        n = len(cases)
        hp = np.zeros((n, 2)); alt = np.zeros((n, 2))
        for i, ((hl, hr, al, ar), _) in enumerate(cases):
            hp[i, slot], hp[i, 1 - slot] = hl, hr
            alt[i, slot], alt[i, 1 - slot] = al, ar
        fin = np.zeros(n, np.uint8); sc = np.full(n, np.nan, np.float32)
        oc = np.zeros(n, np.uint8); pc = np.zeros(n, np.uint8)
        cnt = np.zeros(n, np.int64); fs = np.zeros(n, np.int64)
        OP.payoff_record(np.ones(n, np.uint8), hp.ravel(), alt.ravel(), np.ones(n, np.uint8), np.zeros(2 * n),
                         np.full(n, slot, np.uint8), 1, 304.8, 3, fin, sc, oc, pc, cnt, fs)
        assert sc.tolist() == [c[1] for c in cases]
        assert oc.tolist() == [int(c[0][2] < 304.8) for c in cases]
        assert pc.tolist() == [int(c[0][3] < 304.8) for c in cases]
        assert fs.tolist() == [3] * n


def test_summarize_pair_counts():
    payoff = pkg_module("payoff")
    rng = np.random.default_rng(3)
    per_order = 8
    scores = rng.choice([0.0, 0.5, 1.0], size=2 * per_order)
    la = rng.random(2 * per_order) < 0.3
    ra = rng.random(2 * per_order) < 0.3
    s = payoff.summarize_pair(scores, la, ra, per_order, final_step=321, seed_block=2, eval_seed=99)
    agg = OP.outcome_summary(scores, la)
    for k in ("score", "games", "wins", "draws", "losses", "alt_loss_rate"):
        assert s[k] == agg[k]
    assert s["forward"] == OP.outcome_summary(scores[:per_order], la[:per_order])
    assert s["reverse"] == OP.outcome_summary(1.0 - scores[per_order:], ra[per_order:])
    assert s["paired_scores"] == (0.5 * (scores[:per_order] + scores[per_order:])).tolist()
    assert s["steps"] == 321 and s["opponent_alt_loss_count"] == int(ra.sum())
    assert s["wins_by_opponent_altitude"] == int(((scores == 1.0) & ra).sum())
    assert s["losses_by_own_altitude"] == int(((scores == 0.0) & la).sum())
