"""Hot-expert replication (EPLB): the placement algorithm on the host, and the
dispatch's replica choice in the CPU restatement (the CUDA kernels are checked
against the same restatement in tests/test_gpu_ep.py)."""
import numpy as np
import pytest
import torch

from oracle import ep_oracle
from trials_b200 import ep


def _rank_loads(pl, load):
    reps = np.bincount(pl.phys_to_logical, minlength=pl.num_experts)
    per_slot = load[pl.phys_to_logical] / reps[pl.phys_to_logical]
    return per_slot.reshape(pl.G, pl.slots).sum(axis=1)


def test_placement_replicates_hot_experts_and_balances_ranks():
    E, G, S = 16, 4, 6  # 24 slots: 8 spare
    load = np.ones(E)
    load[[3, 7, 11]] = [40.0, 20.0, 10.0]
    pl = ep.eplb_placement(load, G, S)
    reps = np.bincount(pl.phys_to_logical, minlength=E)
    assert reps.min() >= 1 and reps.sum() == G * S and reps.max() <= G
    assert reps[3] >= reps[7] >= reps[11] > 1
    assert (reps[[e for e in range(E) if e not in (3, 7, 11)]] == 1).all()
    ident = load.reshape(G, E // G).sum(axis=1)
    loads = _rank_loads(pl, load)
    assert loads.max() < 0.5 * ident.max()
    assert loads.max() / loads.mean() < 1.25
    for r in range(G):  # no rank holds two replicas of one expert; slots in expert order
        le = pl.local_experts(r)
        assert len(set(le.tolist())) == S and (np.diff(le) > 0).all()
    t = pl.table()
    for e in range(E):
        n = t[e, 0]
        assert n == reps[e] and (pl.phys_to_logical[t[e, 1:1 + n]] == e).all() and (t[e, 1 + n:] == -1).all()


def test_placement_without_spare_slots_and_identity():
    load = np.arange(8, dtype=float)
    pl = ep.eplb_placement(load, 2, 4)
    assert sorted(pl.phys_to_logical.tolist()) == list(range(8))
    ident = ep.Placement.identity(8, 2)
    assert ident.is_identity() and not ep.Placement(8, 2, 4, np.array([1, 0, 2, 3, 4, 5, 6, 7])).is_identity()
    with pytest.raises(ValueError):
        ep.eplb_placement(load, 2, 3)  # fewer slots than experts
    with pytest.raises(ValueError):
        ep.Placement(8, 2, 4, np.array([0, 0, 1, 2, 3, 4, 5, 6]))  # expert 7 has no slot


def test_replica_choice_prefers_the_local_replica_then_rotates():
    E, G, S = 4, 2, 3
    pl = ep.Placement(E, G, S, np.array([0, 1, 2, 0, 3, 1]))  # expert 0 in slots 0, 3; expert 1 in 1, 5
    table = pl.table()
    # on rank 1 expert 0 stays local (slot 3); on rank 0 too (slot 0)
    assert ep_oracle.target(table, S, E, 1, 0, 5, 1, 2) == 3
    assert ep_oracle.target(table, S, E, 0, 0, 5, 1, 2) == 0
    # expert 2 has one replica (rank 0)
    assert ep_oracle.target(table, S, E, 1, 2, 0, 0, 2) == 2
    # invalid ids are dropped
    assert ep_oracle.target(table, S, E, 0, -1, 0, 0, 2) == -1 and ep_oracle.target(table, S, E, 0, 4, 0, 0, 2) == -1
    # a replica table whose expert has no local replica rotates by t*topk + j
    pl2 = ep.Placement(E, 3, 2, np.array([0, 1, 0, 2, 0, 3]))
    t2 = pl2.table()
    got = [ep_oracle.target(t2, 2, E, 5, 0, t, j, 2) for t in range(3) for j in range(2)]
    assert got == [0, 2, 4, 0, 2, 4]


def test_place_experts_gathers_the_rank_slots():
    w = torch.arange(6 * 2).view(6, 2)
    pl = ep.Placement(6, 2, 4, np.array([5, 0, 1, 5, 2, 3, 4, 0]))
    assert torch.equal(ep.place_experts(w, pl, 1), w[[2, 3, 4, 0]])
