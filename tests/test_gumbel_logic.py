"""CPU tests: the Gumbel root driver's host-side decisions against the
reference's OWN functions, called on the same CPU tensors.

The reference's orchestrator is built with ``__new__`` (as the reference's
tests/test_gpu_training_logic.py does); both sides get the same
queen-surround qualifying masks, priors, logits, allowed masks and Gumbel
draws, and must return identical tensors:

* ``_root_candidate_slots`` (fnn_mcts_orchestrator.py:384-444): the reserve
  for queen-surround moves ranked by prior, filled by prior top-k; and,
  with the reserve off, Gumbel top-k;
* ``_build_policy_target`` (:144-191): adaptive temperature bisection with
  the top-1 cap, and the fixed-temperature form.
Runs where the reference tree exists."""
import numpy as np
import pytest
import torch

from tests.reference_cpu import reference_available, reference_module, torch_on_cpu

pytestmark = pytest.mark.skipif(not reference_available(), reason="needs the reference tree")


@pytest.fixture(scope="module")
def R():
    return reference_module("hive_fnn.fnn_mcts_orchestrator")


def _pair(R, **cfg):
    from hive_neuralnet_b200.orchestrator import FNNMCTSConfig, FNNMCTSOrchestrator
    ref = R.FNNMCTSOrchestrator.__new__(R.FNNMCTSOrchestrator)
    ref.config = R.FNNMCTSConfig(**cfg)
    ref._max_legal = 256
    ref._row_idx_cache, ref._keep_rank_cache = {}, {}
    mine = FNNMCTSOrchestrator.__new__(FNNMCTSOrchestrator)
    mine.config = FNNMCTSConfig(**cfg)
    mine._max_legal = 256
    mine.device = torch.device("cpu")
    mine._slot_idx = torch.arange(256, dtype=torch.int64).unsqueeze(0)
    return ref, mine


def _inputs(rng, B, tie_frac=0.0):
    nl = rng.integers(0, 257, B).astype(np.int32)
    nl[: B // 8] = rng.integers(0, 20, B // 8)  # short lists: fewer legal moves than k
    valid = np.arange(256)[None, :] < nl[:, None]
    logits = rng.normal(size=(B, 256)).astype(np.float32)
    if tie_frac:
        logits = np.where(rng.uniform(size=(B, 256)) < tie_frac, 0.5, logits).astype(np.float32)
    e = np.where(valid, np.exp(logits), 0).astype(np.float32)
    priors = (e / np.maximum(e.sum(1, keepdims=True), 1e-30)).astype(np.float32)
    allowed = valid & (rng.uniform(size=(B, 256)) < 0.85)
    qual = valid & (rng.uniform(size=(B, 256)) < rng.uniform(0, 0.1, (B, 1)))
    t = torch.from_numpy
    legal_logits = torch.where(t(allowed), t(priors).clamp(min=1e-20).log(), torch.full((B, 256), -1e30))
    return t(nl), t(priors), legal_logits, t(allowed), t(qual)


@pytest.mark.parametrize("reserve,k,ties", [(6, 16, 0.0), (6, 16, 0.3), (2, 4, 0.0), (16, 16, 0.0), (0, 16, 0.0),
                                            (0, 3, 0.2)])
def test_root_candidate_slots_match_reference(R, reserve, k, ties):
    rng = np.random.default_rng(100 * reserve + k)
    B = 96
    nl, priors, logits, allowed, qual = _inputs(rng, B, ties)
    ref, mine = _pair(R, queen_surround_reserve_slots=reserve, max_num_considered_actions=k)
    states = torch.zeros((B, 3424), dtype=torch.uint8)
    legal = torch.zeros((B, 256, 6), dtype=torch.uint8)
    ref._queen_surround_qualifying_mask = lambda *a: qual
    mine._queen_surround_qualifying_mask = lambda *a: qual
    draws = []
    torch.manual_seed(7)
    with torch_on_cpu(draws):
        want = ref._root_candidate_slots(states, legal, nl, priors, logits, B, allowed_slot_mask=allowed.clone())
    it = iter(draws)
    mine._uniform = lambda *shape: torch.from_numpy(next(it))
    got = mine._root_candidate_slots(states, legal, nl, priors, logits, B, allowed.clone())
    assert got.dtype == torch.int32
    assert torch.equal(got, want.to(torch.int32))


@pytest.mark.parametrize("adaptive,cap,tmax", [(True, 0.7, 7.0), (True, 0.3, 3.0), (True, 0.99, 7.0),
                                               (False, 0.7, 7.0)])
def test_policy_target_matches_reference(R, adaptive, cap, tmax):
    rng = np.random.default_rng(int(cap * 100) + int(adaptive))
    B = 128
    valid = torch.from_numpy(np.arange(256)[None, :] < rng.integers(1, 257, B)[:, None])
    visited = valid & torch.from_numpy(rng.uniform(size=(B, 256)) < 0.3)
    visited[:, 0] |= valid[:, 0]
    raw = torch.from_numpy((rng.normal(size=(B, 256)) * rng.uniform(0.5, 30, (B, 1))).astype(np.float32))
    logits = torch.where(visited, raw, torch.full_like(raw, -1e30))
    cfg = dict(adaptive_policy_target_temperature=adaptive, policy_target_top1_cap=cap,
               policy_target_max_temperature=tmax, policy_target_temperature=1.7)
    ref, mine = _pair(R, **cfg)
    with torch_on_cpu():
        wp, wt = ref._build_policy_target(logits, valid)
    gp, gt = mine._build_policy_target(logits, valid)
    assert torch.equal(gp, wp) and torch.equal(gt, wt)
