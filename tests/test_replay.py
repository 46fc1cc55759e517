"""Replay-sample exchange: pack/unpack round trip and the all-gather across
two gloo ranks on CPU (the code path NCCL runs on the GPUs), plus a rank that
never joins: the other rank's collective ends with an error, not a hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from hive_neuralnet_b200.orchestrator import FNNTrainingExample
from hive_neuralnet_b200.replay import gather_examples, pack_examples, unpack_examples


def _examples(rank, n):
    rng = np.random.default_rng(100 + rank)
    out = []
    for i in range(n):
        k = int(rng.integers(1, 257))
        out.append(FNNTrainingExample(rng.integers(0, 256, 3424, dtype=np.uint8),
                                      rng.random(k, dtype=np.float32), float(rng.choice([-1.0, 0.0, 1.0])),
                                      bool(i % 3), bool(i % 2 == 0), float(1 + i % 2), 1.0))
    return out


def _same(a, b):
    assert len(a) == len(b)
    for x, y in zip(a, b):
        assert np.array_equal(x.state_bytes, y.state_bytes)
        assert np.array_equal(x.policy_target, y.policy_target)
        assert (x.value_target, x.use_for_policy, x.use_for_value, x.value_weight, x.surprise_weight) == \
               (y.value_target, y.use_for_policy, y.use_for_value, y.value_weight, y.surprise_weight)


def test_pack_unpack_round_trip():
    ex = _examples(0, 17)
    buf = pack_examples(ex)
    assert buf.dtype == np.uint8 and buf.size == sum(16 + 3424 + 4 * len(e.policy_target) for e in ex)
    _same(unpack_examples(buf), ex)
    assert unpack_examples(pack_examples([])) == []
    with pytest.raises(ValueError):
        unpack_examples(buf[:-3])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, counts, mode, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if mode == "leave" and rank == 1:
        dist.destroy_process_group()
        return  # leaves between steps, before the gather
    try:
        got = gather_examples(_examples(rank, counts[rank]))
        np.save(os.path.join(out_dir, f"r{rank}.npy"), pack_examples(got))
    except Exception as e:  # the peer left: the collective reports an error
        with open(os.path.join(out_dir, f"r{rank}.err"), "w") as f:
            f.write(type(e).__name__)
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_gather_examples_two_gloo_ranks(tmp_path):
    counts = [5, 9]
    mp.spawn(_worker, args=(2, _free_port(), counts, "ok", str(tmp_path)), nprocs=2, join=True)
    want = _examples(0, counts[0]) + _examples(1, counts[1])
    for r in range(2):
        _same(unpack_examples(np.load(tmp_path / f"r{r}.npy")), want)


def test_gather_reports_a_rank_that_left(tmp_path):
    mp.spawn(_worker, args=(2, _free_port(), [3, 3], "leave", str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "r0.err").exists() and not (tmp_path / "r0.npy").exists()
