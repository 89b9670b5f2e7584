"""Inputs of tests/golden/payoff.npz (shared by make_golden.py and the tests, which regenerate
them from the seed stored in the fixture instead of storing every step)."""
import numpy as np


def payoff_steps(seed, nenv, nsteps):
    """Per-step terminal values of the scripted payoff run: HP with exact ties and 1e-9 margins,
    altitudes on both sides of the 304.8 m floor, random done flags (all done on the last step),
    a few non-finite values that fall only on lanes already finished (which the reference must
    ignore)."""
    rng = np.random.default_rng(int(seed))
    out = []
    finished = np.zeros(nenv, bool)
    for k in range(nsteps):
        hp = rng.choice([0.0, 0.25, 0.5, 0.5 + 5e-10, 0.5 + 2e-9, 1.0], size=(nenv, 2))
        alt = rng.choice([200.0, 304.8, 304.9, 5000.0], size=(nenv, 2))
        done = (rng.random(nenv) < (1.0 if k == nsteps - 1 else 0.25))
        finite = np.ones(nenv, bool)
        reward = rng.normal(size=(nenv, 2))
        if k >= 2 and finished.any():                      # garbage on lanes that already finished
            idx = np.flatnonzero(finished)[: 3]
            hp[idx, 0] = np.nan
            finite[idx] = False
        out.append(dict(hp=hp, alt=alt, done=done, finite=finite, reward=reward))
        finished |= done
    return out
