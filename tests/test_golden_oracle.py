"""The CPU oracle reproduces the committed golden fixtures (regression pin of the
checker itself; the fixtures are made by tests/golden/make_golden.py)."""
import glob
import os

import numpy as np
import pytest

from tests.golden.make_golden import load

FIXTURES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p)[:-4] for p in FIXTURES])
def test_oracle_matches_golden(oracle_mod, path):
    O = oracle_mod
    art, z = load(path)
    idx = O.OracleIndex(art)
    ids, dists, _, probes = idx.search(z["queries"], z["k"], z["nprobe"], want_probes=True)
    assert np.array_equal(ids, z["exp_ids"])
    assert np.array_equal(dists.view(np.uint32), z["exp_dists"].view(np.uint32))
    assert np.array_equal(probes, z["exp_probes"])
    f_ids, f_d, _ = idx.search(z["queries"], z["k"], z["nprobe"], filter_mode=O.FILTER_FUSED,
                               bitsets=z["bitsets"], bitset_len=int(z["bitset_len"][0]),
                               query_bitset=z["query_bitset"])
    assert np.array_equal(f_ids, z["exp_fused_ids"])
    p_ids, p_d, p_c = idx.search(z["queries"], z["k"], z["nprobe"], filter_mode=O.FILTER_POST,
                                 bitsets=z["bitsets"], bitset_len=int(z["bitset_len"][0]),
                                 query_bitset=z["query_bitset"])
    assert np.array_equal(p_c, z["exp_post_counts"])
    assert np.array_equal(p_ids, z["exp_post_ids"])


def test_post_filter_semantics(oracle_mod):
    """Post mode drops exactly the filtered ids of the unfiltered result, in order
    (src/faiss/ivf_usq.rs:688-715)."""
    O = oracle_mod
    art, z = load(FIXTURES[0])
    blen = int(z["bitset_len"][0])
    for q in range(z["queries"].shape[0]):
        b = int(z["query_bitset"][q])
        row = z["exp_ids"][q]
        if b < 0:
            keep = row
        else:
            w = z["bitsets"][b]
            keep = [int(i) for i in row
                    if not (0 <= int(i) < blen and (int(w[int(i) >> 6]) >> (int(i) & 63)) & 1)]
        c = int(z["exp_post_counts"][q])
        assert list(z["exp_post_ids"][q][:c]) == list(keep)
