"""Expert-parallel load rebalancing.

Reference behaviour: core/optimization/gollek-plugin-elastic-ep/…/elasticep/
ElasticExpertParallelismRunner.java:312-346 (a background loop reads per-expert token counters,
asks ``ep_rebalance`` for a new expert → GPU assignment and remaps every expert that moved).

Here a placement is a permutation ``perm`` of the experts: physical slot p holds logical expert
``perm[p]``, and rank r owns the physical slots [r * E_loc, (r + 1) * E_loc). Routing always runs
over the logical experts (router rows never move, so group-limited routing and tie-breaking are
untouched); the router kernel maps each chosen expert to its physical slot through the layer's
logical -> physical table. Rebalancing rewrites that table and moves the weights of the experts
that change rank; the MoE kernels and the model output do not change. The new placement is
  1) balanced: experts in decreasing load go to the least-loaded rank that still has a free slot
     (longest-processing-time-first under a per-rank capacity of E_loc);
  2) cheap to reach: the balanced groups are matched to ranks so that as many experts as possible
     stay where they are (a linear assignment on "experts already there").
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np


def balanced_groups(loads: np.ndarray, world: int) -> List[List[int]]:
    """Split experts into ``world`` groups of E / world experts with near-equal total load."""
    E = len(loads)
    cap = E // world
    order = np.lexsort((np.arange(E), -np.asarray(loads, dtype=np.float64)))  # by load, ties to lower id
    groups: List[List[int]] = [[] for _ in range(world)]
    tot = np.zeros(world)
    for e in order:
        free = [r for r in range(world) if len(groups[r]) < cap]
        r = min(free, key=lambda q: (tot[q], q))
        groups[r].append(int(e))
        tot[r] += loads[e]
    return groups


def imbalance(loads: np.ndarray, perm: np.ndarray, world: int) -> float:
    """max over ranks of the rank's load / the mean rank load (1.0 = perfectly balanced)."""
    per_rank = np.asarray(loads, dtype=np.float64)[np.asarray(perm)].reshape(world, -1).sum(1)
    mean = per_rank.mean()
    return float(per_rank.max() / mean) if mean > 0 else 1.0


def plan_placement(loads: np.ndarray, perm: np.ndarray, world: int) -> np.ndarray:
    """New placement for logical-expert ``loads`` given the current placement ``perm``."""
    from scipy.optimize import linear_sum_assignment
    E = len(loads)
    if E % world:
        raise ValueError("the expert count must be divisible by the expert-parallel size")
    cap = E // world
    perm = np.asarray(perm)
    cur_rank = np.empty(E, dtype=np.int64)
    cur_rank[perm] = np.arange(E) // cap
    groups = balanced_groups(loads, world)
    stay = np.array([[sum(cur_rank[e] == r for e in g) for r in range(world)] for g in groups])
    gi, ri = linear_sum_assignment(-stay)
    new = np.empty(E, dtype=np.int64)
    for g, r in zip(gi, ri):
        # experts already on rank r keep their slot order, newcomers follow
        here = [int(e) for e in perm[r * cap:(r + 1) * cap] if e in set(groups[g])]
        rest = sorted(e for e in groups[g] if e not in set(here))
        new[r * cap:(r + 1) * cap] = here + rest
    if imbalance(loads, perm, world) <= imbalance(loads, new, world) + 1e-12:
        return perm.copy()  # nothing to gain: stay
    return new


def moves(old: np.ndarray, new: np.ndarray, world: int) -> List[Tuple[int, int, int, int]]:
    """(logical expert, source rank, source slot, destination slot) of every expert that changes
    rank between placements ``old`` and ``new`` (slots are physical)."""
    E = len(old)
    cap = E // world
    where = np.empty(E, dtype=np.int64)
    where[np.asarray(old)] = np.arange(E)
    out = []
    for p_new, e in enumerate(np.asarray(new)):
        p_old = int(where[e])
        if p_old // cap != p_new // cap:
            out.append((int(e), p_old // cap, p_old, p_new))
    return out
