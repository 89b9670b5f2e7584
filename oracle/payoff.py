"""Batched payoff scoring restated in numpy -- TEST INFRASTRUCTURE ONLY.

``payoff_record`` restates one step of the per-lane scoring of the reference's batched payoff
evaluation (R/cuda_fdm/batched_payoff.py:131-156; the single-matchup loop
R/cuda_fdm/ppo_gpu.py:1467-1500 computes the same outcome): lanes still playing their first
game are active; a non-finite terminal flag / HP / altitude / reward on an active lane is an
error; a done active lane is scored for the left policy from the terminal HP and MSL altitude
of the aircraft it flies and of its opponent (1 win, 0.5 draw, 0 loss, 1e-9 HP margin) and
stops being active.  ``outcome_summary`` restates PPOGPUTrainer._outcome_summary
(ppo_gpu.py:1410-1418).  It updates its arrays in place like the kernel it checks.
"""
import numpy as np


def payoff_record(done, terminal_hp, terminal_alt, finite, reward, left_slot, lanes, min_alt, step,
                  finished, scores, own_crash, opp_crash, finished_count, final_step):
    """Returns the number of active lanes with a non-finite value (the kernel's counter)."""
    nenv = done.shape[0]
    hp = np.asarray(terminal_hp, np.float64).reshape(nenv, 2)
    alt = np.asarray(terminal_alt, np.float64).reshape(nenv, 2)
    rew = np.asarray(reward, np.float64).reshape(nenv, 2)
    rows = np.arange(nenv)
    ls = np.asarray(left_slot).astype(np.int64)
    active = ~finished.astype(bool)
    finite_lanes = (finite.astype(bool) & np.isfinite(hp).all(1) & np.isfinite(alt).all(1)
                    & np.isfinite(rew).all(1))
    bad = int(np.count_nonzero(active & ~finite_lanes))
    newly = done.astype(bool) & active
    lhp, rhp = hp[rows, ls], hp[rows, 1 - ls]
    lalt, ralt = alt[rows, ls], alt[rows, 1 - ls]
    ld = (lhp <= 0.0) | (lalt < min_alt)
    rd = (rhp <= 0.0) | (ralt < min_alt)
    alive = ~ld & ~rd
    win = (rd & ~ld) | (alive & (lhp > rhp + 1e-9))
    loss = (ld & ~rd) | (alive & (lhp < rhp - 1e-9))
    outcome = win.astype(np.float32) + np.float32(0.5) * (~win & ~loss).astype(np.float32)
    scores[newly] = outcome[newly]
    own_crash[newly] = (lalt < min_alt)[newly]
    opp_crash[newly] = (ralt < min_alt)[newly]
    finished[newly] = 1
    for m in np.unique(rows[newly] // lanes):
        before = finished_count[m]
        finished_count[m] += int(np.count_nonzero(newly[m * lanes:(m + 1) * lanes]))
        if before < lanes and finished_count[m] == lanes:
            final_step[m] = step
    return bad


def outcome_summary(scores, altitude_losses):
    scores = np.asarray(scores, dtype=np.float64)
    altitude_losses = np.asarray(altitude_losses, dtype=np.bool_)
    wins = int(np.count_nonzero(scores == 1.0))
    losses = int(np.count_nonzero(scores == 0.0))
    return {"score": float(scores.mean()), "games": int(scores.size), "wins": wins,
            "draws": int(scores.size - wins - losses), "losses": losses,
            "alt_loss_rate": float(altitude_losses.mean())}
