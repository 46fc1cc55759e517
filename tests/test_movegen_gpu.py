"""GPU parity: the sm_100a kernels against the CPU oracle, bit-exact.

Inputs are seeded random-playout positions (BASELINE configs 1 and 2
recipe); the oracle is pinned to the reference by tests/test_oracle.py.
Every comparison is bit-exact: move lists (order, duplicates, zero padding),
num_legal, the 122 features compared as raw float bits.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ext():
    from hive_neuralnet_b200.hive_gpu import load_extension
    return load_extension()


@pytest.fixture(scope="module")
def orc():
    return O.oracle()


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


CASES = [(0, 60, 4096), (7, 120, 16384), (7, 200, 4096), (1, 90, 2048), (4, 90, 2048), (2, 90, 2048)]


@pytest.mark.parametrize("mask,max_ply,count", CASES)
def test_legal_moves_and_features_bit_exact(ext, orc, mask, max_ply, count):
    st = orc.generate_positions(4242 + mask * 7 + max_ply, 0, count, max_ply, mask)
    mo, no, fo = orc.legal_moves_features(st)
    mg, ng, fg = ext.generate_legal_moves_and_fnn_features_batch(_cuda(st), count)
    ng, mg, fg = ng.cpu().numpy(), mg.cpu().numpy(), fg.cpu().numpy()
    bad = np.where(ng != no)[0]
    assert len(bad) == 0, f"num_legal differs at {bad[:10]}"
    bad = np.where((mg != mo).reshape(count, -1).any(1))[0]
    assert len(bad) == 0, f"move lists differ at {bad[:10]}"
    bad = np.where((_bits(fg) != _bits(fo)).any(1))[0]
    assert len(bad) == 0, f"features differ at {bad[:10]}: cols {np.where(fg[bad[0]] != fo[bad[0]])}"


def test_moves_only_and_extract_features(ext, orc):
    st = orc.generate_positions(99, 0, 4096, 120, 7)
    mo, no, fo = orc.legal_moves_features(st)
    mg, ng = ext.generate_legal_moves_batch(_cuda(st), 4096)
    assert np.array_equal(mg.cpu().numpy(), mo) and np.array_equal(ng.cpu().numpy(), no)
    # features of a supplied list: the full list, and the compact list
    fg = ext.extract_fnn_features_batch(_cuda(st), _cuda(mo), _cuda(no), 4096).cpu().numpy()
    assert np.array_equal(_bits(fg), _bits(fo))
    cm, cn = orc.compact_moves(st)
    fc = orc.features(st, cm, cn)
    fgc = ext.extract_fnn_features_batch(_cuda(st), _cuda(cm), _cuda(cn), 4096).cpu().numpy()
    assert np.array_equal(_bits(fgc), _bits(fc))


def test_golden_small_through_gpu(ext):
    g = np.load(os.path.join(GOLD, "golden_small.npz"))
    st = g["states"]
    mg, ng, fg = ext.generate_legal_moves_and_fnn_features_batch(_cuda(st), len(st))
    assert np.array_equal(mg.cpu().numpy(), g["moves"])
    assert np.array_equal(ng.cpu().numpy(), g["num_legal"])
    assert np.array_equal(_bits(fg.cpu().numpy()), _bits(g["features"]))
    sf = ext.fnn_successor_features_batch(_cuda(st), _cuda(g["moves"]), _cuda(g["succ_roots"]),
                                          _cuda(g["succ_moves"]), len(g["succ_roots"]))
    assert np.array_equal(_bits(sf.cpu().numpy()), _bits(g["succ_features"]))
    act = ext.legal_moves_to_actions_batch(_cuda(st), mg, ng, len(st)).cpu().numpy()
    assert np.array_equal(act, g["actions"])
    cen = ext.compute_centroids_batch(_cuda(st), len(st)).cpu().numpy()
    assert np.array_equal(cen, g["centroids"])


@pytest.mark.parametrize("mask,max_ply,count", [(0, 60, 2048), (7, 120, 4096)])
def test_successor_features_bit_exact(ext, orc, mask, max_ply, count):
    st = orc.generate_positions(555 + mask, 0, count, max_ply, mask)
    mo, no, _ = orc.legal_moves_features(st)
    roots = np.repeat(np.arange(count, dtype=np.int64), no)
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in no])
    fo = orc.successor_features(st, mo, roots, idx)
    fg = ext.fnn_successor_features_batch(_cuda(st), _cuda(mo), _cuda(roots), _cuda(idx), len(roots))
    fg = fg.cpu().numpy()
    bad = np.where((_bits(fg) != _bits(fo)).any(1))[0]
    assert len(bad) == 0, f"{len(bad)} successor rows differ, first {bad[:5]}"


@pytest.mark.parametrize("mask,max_ply", [(0, 60), (7, 120)])
def test_gpu_playout_generator_matches_oracle(ext, orc, mask, max_ply):
    with open(os.path.join(GOLD, "golden_digests.json")) as f:
        dig = json.load(f)
    count = 4096
    g = ext.generate_positions(31337 + mask, 0, count, max_ply, mask).cpu().numpy()
    o = orc.generate_positions(31337 + mask, 0, count, max_ply, mask)
    bad = np.where((g != o).any(1))[0]
    assert len(bad) == 0, f"playouts differ at {bad[:10]}"
    # the config-1 parity set itself, generated on the GPU, against the reference digest
    p = dig["config1_base_4096"]["params"]
    g1 = ext.generate_positions(p["seed"], p["first_game"], p["count"], p["max_ply"], p["expansion_mask"])
    import hashlib
    assert hashlib.sha256(g1.cpu().numpy().tobytes()).hexdigest() == dig["config1_base_4096"]["states"]


def test_state_ops(ext, orc):
    st = ext.create_initial_states(64, 7)
    o = orc.generate_positions(0, 0, 1, 0, 7)
    assert np.array_equal(st.cpu().numpy(), np.repeat(o, 64, 0))
    assert (ext.check_results_batch(st, 64) == 0).all()
    pos = orc.generate_positions(2024, 0, 2048, 150, 7)
    mo, no, _ = orc.legal_moves_features(pos)
    pick = np.array([mo[i, (i * 13) % no[i]] if no[i] else np.zeros(6, np.uint8) for i in range(len(pos))],
                    np.uint8)
    t = _cuda(pos)
    ext.apply_moves_batch(t, _cuda(pick), len(pos))
    want = orc.apply_moves(pos, pick)
    assert np.array_equal(t.cpu().numpy(), want)
    res = ext.check_results_batch(t, len(pos)).cpu().numpy()
    assert np.array_equal(res, want[:, 3415].astype(np.int32))


def test_device_error_word_clean(ext):
    assert ext.device_error_word(clear=True) == 0


def test_queen_escape_and_child_probe(ext, orc):
    st = np.concatenate([orc.generate_positions(808, 0, 1024, 120, 7), orc.generate_positions(809, 0, 1024, 60, 0)])
    qe = ext.queen_escape_flags_batch(_cuda(st), len(st)).cpu().numpy()
    assert np.array_equal(qe, orc.queen_escape(st))
    mo, no, _ = orc.legal_moves_features(st)
    sub = st[:256]
    res, sur, esc = (x.cpu().numpy() for x in ext.child_probe_batch(_cuda(sub), _cuda(mo[:256]), _cuda(no[:256]),
                                                                     256, True))
    for i in range(0, 256, 5):
        n = no[i]
        kids = orc.apply_moves(np.repeat(sub[i:i + 1], n, 0), mo[i, :n])
        assert np.array_equal(res[i, :n], kids[:, 3415].astype(np.int32))
        assert np.array_equal(esc[i, :n], orc.queen_escape(kids))
        assert (res[i, n:] == 0).all() and (sur[i, n:] == 0).all()
        for j in range(n):
            k = kids[j]
            color = int(k[3412]) & 1
            qc = int(k[3392 + 2 * color]) | (int(k[3393 + 2 * color]) << 8)
            want = 0
            if qc != 0xFFFF:
                r, c = divmod(qc, 23)
                for dr, dc in ((0, 1), (-1, 1), (-1, 0), (0, -1), (1, -1), (1, 0)):
                    if 0 <= r + dr < 23 and 0 <= c + dc < 23 and k[2645 + (r + dr) * 23 + c + dc] > 0:
                        want += 1
            assert sur[i, j] == want


def test_host_buffer_pipeline_matches_device_call(ext, orc):
    """The chunked host-buffer form gives the same bytes as the device call (ragged last chunk)."""
    st = orc.generate_positions(4711, 0, 5000, 120, 7)
    tall = st[:, 2645:2645 + 529].max(1) >= 3
    assert 0 < tall.sum() < len(st)  # both sides of the staged upload's level test
    # the staged upload leaves level bytes above each cell's height as they
    # were: poison the staging slots so that a byte it should have sent shows
    slots, _ = ext._staging(torch.device("cuda", torch.cuda.current_device()), 1024)
    for slot in slots:
        slot[0].fill_(0xA7)
    mg, ng, fg = (x.cpu().numpy() for x in ext.generate_legal_moves_and_fnn_features_batch(_cuda(st), 5000))
    raw = torch.empty(5000 * 3424 + 8, dtype=torch.uint8).pin_memory()
    odd = raw[8:].view(5000, 3424)  # pinned but off a 16-byte boundary: full copy
    odd.copy_(torch.from_numpy(st))
    for host in (torch.from_numpy(st).pin_memory(), torch.from_numpy(st), odd):
        mh, nh, fh = ext.generate_legal_moves_and_fnn_features_host(host, 5000, chunk=1024)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(mh.numpy(), mg)
        assert np.array_equal(nh.numpy(), ng)
        assert np.array_equal(_bits(fh.numpy()), _bits(fg))


@pytest.mark.parametrize("prefix", [0, 8, 96, 248, 256])
def test_host_pipeline_prefix_download_into_poisoned_buffers(ext, orc, prefix):
    """Pinned output buffers full of 0xAB: the prefix download (hv_download_moves)
    plus the host-cleared row tails give the device call's bytes, for any prefix
    (lists shorter and longer than it, a ragged last chunk); a pageable moves
    buffer takes the full copy."""
    st = orc.generate_positions(5150 + prefix, 0, 3000, 200, 7)
    mg, ng, fg = (x.cpu().numpy() for x in ext.generate_legal_moves_and_fnn_features_batch(_cuda(st), 3000))
    if prefix in (8, 96):
        assert (ng > prefix).any() and (ng < prefix).any()
    host = torch.from_numpy(st).pin_memory()
    for pinned in (True, False):
        out = (torch.full((3000, 256, 6), 0xAB, dtype=torch.uint8, pin_memory=pinned),
               torch.full((3000,), -7, dtype=torch.int32, pin_memory=pinned),
               torch.full((3000, 122), float("nan"), dtype=torch.float32, pin_memory=pinned))
        mh, nh, fh = ext.generate_legal_moves_and_fnn_features_host(host, 3000, out=out, chunk=1024,
                                                                    move_prefix=prefix)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(mh.numpy(), mg)
        assert np.array_equal(nh.numpy(), ng)
        assert np.array_equal(_bits(fh.numpy()), _bits(fg))


def test_download_moves_rejects_bad_prefix(ext):
    lib = ext._lib
    d = torch.zeros((4, 256, 6), dtype=torch.uint8, device="cuda")
    n = torch.zeros((4,), dtype=torch.int32, device="cuda")
    h = torch.zeros((4, 256, 6), dtype=torch.uint8).pin_memory()
    s = torch.cuda.current_stream().cuda_stream
    for bad in (-8, 12, 264):
        assert lib.hv_download_moves(d.data_ptr(), n.data_ptr(), 4, h.data_ptr(), bad, s) != 0
    assert lib.hv_download_moves(d.data_ptr(), n.data_ptr(), -1, h.data_ptr(), 96, s) != 0
    assert lib.hv_download_moves(d.data_ptr(), n.data_ptr(), 4, h.data_ptr(), 96, s) == 0
    torch.cuda.current_stream().synchronize()


@pytest.mark.parametrize("mask,max_ply", [(0, 60), (7, 120), (7, 200)])
def test_hybrid_transformer_inputs_bit_exact(ext, orc, mask, max_ply):
    """Piece tokens, global and move features (state_encoder.cuh:372-550) against the oracle,
    standalone and fused with move generation."""
    st = orc.generate_positions(9090 + mask + max_ply, 0, 4096, max_ply, mask)
    mo, no, fo = orc.legal_moves_features(st)
    want = orc.hybrid_encode(st, mo, no)
    d = _cuda(st)
    tok = ext.hybrid_transformer_encode_with_moves_batch(d, _cuda(mo), _cuda(no), 4096)
    mf = ext.hybrid_transformer_move_features_batch(d, _cuda(mo), _cuda(no), 4096)
    fused = ext.generate_legal_moves_and_hybrid_root_features_batch(d, 4096)
    assert tok[4].dtype == torch.bool
    got = [t.cpu().numpy() for t in tok]
    got[4] = got[4].astype(np.uint8)
    for name, g, o in zip(("tf", "tq", "tr", "tz", "tm", "gf", "nt"), got, want[:7]):
        assert np.array_equal(np.ascontiguousarray(g).view(np.uint8), np.ascontiguousarray(o).view(np.uint8)), name
    assert np.array_equal(_bits(mf.cpu().numpy()), _bits(want[7]))
    m, n, f = (x.cpu().numpy() for x in fused[:3])
    assert np.array_equal(m, mo) and np.array_equal(n, no) and np.array_equal(_bits(f), _bits(fo))
    assert np.array_equal(_bits(fused[3].cpu().numpy()), _bits(want[0]))
    assert np.array_equal(fused[7].cpu().numpy().astype(np.uint8), want[4])
    assert np.array_equal(_bits(fused[8].cpu().numpy()), _bits(want[5]))
    assert np.array_equal(_bits(fused[9].cpu().numpy()), _bits(want[7]))


def test_legal_mask_matches_action_indices(ext, orc):
    """legal_mask_kernel (state_encoder.cuh:908-976): ones exactly at the oracle's action indices."""
    st = np.concatenate([orc.generate_positions(515, 0, 256, 60, 0), orc.generate_positions(516, 0, 256, 150, 7)])
    mo, no, _ = orc.legal_moves_features(st)
    act, _ = orc.actions(st, mo, no)
    masks, nl = ext.generate_legal_mask_batch(_cuda(st), len(st))
    mv2, nl2, masks2 = ext.generate_legal_moves_and_mask_batch(_cuda(st), len(st))
    want = np.zeros((len(st), 85834), np.float32)
    for i in range(len(st)):
        a = act[i, :no[i]]
        want[i, a[a >= 0]] = 1.0
    assert np.array_equal(nl.cpu().numpy(), no) and np.array_equal(nl2.cpu().numpy(), no)
    assert np.array_equal(mv2.cpu().numpy(), mo)
    assert np.array_equal(masks.cpu().numpy(), want) and np.array_equal(masks2.cpu().numpy(), want)


def test_linked_halves_match_fused_entry(ext, orc):
    """hv_generate_legal_moves_linked + hv_fnn_features_linked give the fused entry's bytes."""
    st = _cuda(orc.generate_positions(5150, 0, 3000, 120, 7))
    mg, ng, fg = ext.generate_legal_moves_and_fnn_features_batch(st, 3000)
    lib = ext._lib
    mv = torch.zeros_like(mg)
    nl = torch.zeros_like(ng)
    ft = torch.zeros_like(fg)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.hv_generate_legal_moves_linked(st.data_ptr(), 3000, mv.data_ptr(), nl.data_ptr(), ft.data_ptr(), s) == 0
    assert lib.hv_fnn_features_linked(st.data_ptr(), mv.data_ptr(), nl.data_ptr(), 3000, ft.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert torch.equal(mv, mg) and torch.equal(nl, ng)
    assert np.array_equal(_bits(ft.cpu().numpy()), _bits(fg.cpu().numpy()))


@pytest.mark.parametrize("count", [1, 2, 3, 33, 4145])
def test_fused_entry_small_and_ragged_batches(ext, orc, count):
    """The fused entry's position counters: one position (no claiming
    launch), two (one claimed position plus position 0), and counts around
    the number of resident warps."""
    st = orc.generate_positions(7000 + count, 0, count, 120, 7)
    mo, no, fo = orc.legal_moves_features(st)
    mg, ng, fg = (x.cpu().numpy() for x in ext.generate_legal_moves_and_fnn_features_batch(_cuda(st), count))
    assert np.array_equal(ng, no) and np.array_equal(mg, mo)
    assert np.array_equal(_bits(fg), _bits(fo))
