"""Batched payoff scoring oracle (CPU).

oracle/payoff.py restates the per-lane scoring of R/cuda_fdm/batched_payoff.py:131-156.  It is
pinned to the reference itself: tests/golden/payoff.npz holds what the reference's own
``evaluate_chunk`` loop (scoring inline at :131-156, summaries from
PPOGPUTrainer._summarize_clean_pair, ppo_gpu.py:1517-1575) produced on CPU for a scripted
sequence of terminal values (tests/golden/payoff_case.py; ties, 1e-9 HP margins, altitude losses,
non-finite values on finished lanes).  Replaying the same steps through the oracle must give the
reference's scores, crash flags and completion steps, and ``payoff.summarize_pair`` its summary
fields.  Hand-scored cases cover both seat orders.
"""
import json
import sys

import numpy as np

from conftest import GOLDEN, pkg_module
from oracle import payoff as OP

if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))


def replay_payoff_fixture(record):
    """Replay payoff.npz's steps through ``record(step, d, left_slot, lanes, min_alt, state)`` (the
    oracle or the kernel); returns (fixture, state) with state's arrays after the last step."""
    from payoff_case import payoff_steps
    g = np.load(GOLDEN / "payoff.npz")
    per_order, capacity, nsteps = int(g["per_order"]), int(g["capacity"]), int(g["nsteps"])
    lanes = 2 * per_order
    nenv = lanes * capacity
    left_slot = np.tile(np.repeat(np.array([0, 1], np.uint8), per_order), capacity)
    state = dict(fin=np.zeros(nenv, np.uint8), sc=np.full(nenv, np.nan, np.float32), oc=np.zeros(nenv, np.uint8),
                 pc=np.zeros(nenv, np.uint8), cnt=np.zeros(capacity, np.int64), fs=np.zeros(capacity, np.int64),
                 bad=[])
    for k, d in enumerate(payoff_steps(g["seed"], nenv, nsteps)):
        record(k + 1, d, left_slot, lanes, float(g["min_alt"]), state)
        if state["fs"].all():
            break
    return g, state


def oracle_record(step, d, left_slot, lanes, min_alt, st):
    st["bad"].append(OP.payoff_record(d["done"].astype(np.uint8), d["hp"].ravel(), d["alt"].ravel(),
                                      d["finite"].astype(np.uint8), d["reward"].ravel(), left_slot, lanes, min_alt,
                                      step, st["fin"], st["sc"], st["oc"], st["pc"], st["cnt"], st["fs"]))


def check_against_reference(g, st):
    lanes = 2 * int(g["per_order"])
    for i in range(int(g["nright"])):
        r = slice(i * lanes, (i + 1) * lanes)
        np.testing.assert_array_equal(st["sc"][r], g[f"scores{i}"])
        assert st["oc"][r].tolist() == g[f"own{i}"].tolist()
        assert st["pc"][r].tolist() == g[f"opp{i}"].tolist()
        assert int(st["fs"][i]) == int(g[f"final_step{i}"])
    assert not any(st["bad"]), "non-finite values fell only on finished lanes"


def test_oracle_matches_reference_run():
    g, st = replay_payoff_fixture(oracle_record)
    check_against_reference(g, st)


def test_summarize_pair_matches_reference_summary():
    payoff = pkg_module("payoff")
    g = np.load(GOLDEN / "payoff.npz")
    po = int(g["per_order"])
    for i in range(int(g["nright"])):
        ref = json.loads(str(g[f"summary{i}"]))
        got = payoff.summarize_pair(g[f"scores{i}"], g[f"own{i}"].astype(bool), g[f"opp{i}"].astype(bool), po,
                                    int(g[f"final_step{i}"]), seed_block=ref["seed_block"],
                                    eval_seed=ref["policy_rng_seed"])
        assert set(got) == set(ref), set(got) ^ set(ref)
        for k in ref:
            assert got[k] == ref[k], (k, got[k], ref[k])


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
