"""Host logic of PPOTrainer that needs no GPU: the rollout statistics summed over data-parallel
ranks (``reduce_stats``, the league EMA inputs of the reference's multi-process trainer), on two
gloo ranks, and its single-rank no-op."""
import os
import socket
import types

import torch
import torch.multiprocessing as mp

from conftest import pkg_module

NAMES = ("ret_sum", "len_sum", "ep_count", "win_sum", "loss_sum", "alt_loss_sum", "opponent_alt_loss_sum")


def _stats(rank, n_opp=3):
    g = torch.Generator().manual_seed(100 + rank)
    st = {k: torch.rand((), generator=g, dtype=torch.float64) * 10 for k in NAMES}
    for k in ("win_by_opp", "loss_by_opp", "ep_by_opp"):
        st[k] = torch.randint(0, 9, (n_opp,), generator=g).to(torch.float64)
    return st


def _rank(rank, world, port, path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tr = pkg_module("trainer")
        me = types.SimpleNamespace(world=world, group=dist.group.WORLD)
        out = tr.PPOTrainer.reduce_stats(me, _stats(rank))
        torch.save({k: v.clone() for k, v in out.items()}, f"{path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_reduce_stats_sums_over_two_ranks(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "stats")
    mp.start_processes(_rank, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    r0, r1 = torch.load(f"{path}.0"), torch.load(f"{path}.1")
    a, b = _stats(0), _stats(1)
    assert set(r0) == set(a)
    for k in a:
        assert torch.equal(r0[k], r1[k]), f"{k} differs between the ranks"
        assert r0[k].shape == a[k].shape
        torch.testing.assert_close(r0[k].double(), a[k] + b[k], rtol=1e-6, atol=0.0)


def test_reduce_stats_single_rank_is_identity():
    tr = pkg_module("trainer")
    st = _stats(0)
    out = tr.PPOTrainer.reduce_stats(types.SimpleNamespace(world=1, group=None), st)
    assert out is st
