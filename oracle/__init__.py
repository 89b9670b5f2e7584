"""CPU parity checkers for the F-16 environment hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may
import this package.  The shipped package never imports it and has no CPU fallback.

* ``oracle.fdm``  -- ctypes front end of fdm_oracle.c (our C restatement of the reference
  FDM) and of oracle/_ref (the reference's own fdm.cuh, host-compiled).
* ``oracle.obs``  -- numpy restatement of the fused observation / reward / termination path.
* ``oracle.gae``  -- numpy restatement of the rollout GAE.
"""
