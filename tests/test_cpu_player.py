"""CPU tests: oracle/cpu_player.py (the restated FNN CPU player timed as the
Gumbel search's CPU baseline) against the reference's own
FNNNativeCPUPlayer (hive_fnn/fnn_native_cpu_player.py), both over the
reference's cpu_native backend compiled into oracle/_ref: same chosen move
and same visit counts under every root child, with and without Gumbel noise.
Runs where the reference tree and the backend build exist."""
import os
import sys
import types

import numpy as np
import pytest
import torch

from oracle import cpu_player as CP
from oracle import oracle as O

pytestmark = pytest.mark.skipif(CP.backend_path() is None or not O.reference_available(),
                                reason="needs the reference tree and oracle/_ref's cpu_native build")


@pytest.fixture(scope="module")
def reference_player_module():
    backend = CP.load_backend()
    sys.modules["hive_cpu_native"] = types.SimpleNamespace(load_extension=lambda: backend)
    # the reference tree goes on the path only for this import: it has a
    # `tests` package of its own that would shadow this repository's
    saved = list(sys.path)
    sys.path.append(O.reference_dir())
    try:
        import hive_fnn.fnn_native_cpu_player as R  # the reference module
        from hive_fnn.fnn_network import HiveFNN
    finally:
        sys.path[:] = saved
    return R, HiveFNN


@pytest.mark.parametrize("noise", [0.0, 1.0])
def test_port_matches_reference_player(reference_player_module, noise):
    R, RefFNN = reference_player_module
    threads = torch.get_num_threads()
    torch.manual_seed(0)
    net = RefFNN().eval()
    orc = O.oracle()
    st = np.concatenate([orc.generate_positions(41, 0, 4, 30, 0), orc.generate_positions(42, 0, 4, 80, 7)])
    try:
        for i, s in enumerate(st):
            if int(s[3415]) != 0:
                continue
            cfg = R.FNNNativeCPUConfig(num_simulations=48, gumbel_noise_scale=noise)
            ref = R.FNNNativeCPUPlayer(net, cfg)
            root = R._NativeNode(s.tobytes(), result=0)
            np.random.seed(100 + i)
            want = ref._gumbel_search(root)
            mine = CP.CPUPlayer(net, CP.PlayerConfig(num_simulations=48, gumbel_noise_scale=noise))
            node = CP.Node(s.tobytes(), result=0)
            np.random.seed(100 + i)
            got = mine.gumbel_search(node)
            assert got == want
            assert [k.n for k in node.kids] == [c.visit_count for c in root.children]
            assert [k.w for k in node.kids] == [c.total_value for c in root.children]
            assert mine.sims == sum(c.visit_count for c in root.children)
    finally:
        torch.set_num_threads(threads)
