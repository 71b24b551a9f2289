"""The Python mirror carries the reference's IvfUsqIndex / IvfUsqConfig names.

Reference: src/faiss/ivf_usq.rs (IvfUsqConfig builders :36-72, IvfUsqIndex :175-411).
No GPU call is made: this checks names and the config builders only.
"""
from hanns_b200.ivf_usq import IvfUsqConfig, IvfUsqIndex, METRIC_IP


def test_index_methods_named_like_the_reference():
    for name in ("train", "add", "search", "save", "load", "count", "ntotal", "size",
                 "set_nprobe", "has_raw_data"):
        assert callable(getattr(IvfUsqIndex, name)), name


def test_config_builders_chain():
    c = (IvfUsqConfig(768, 4096, 4).with_nprobe(32).with_metric(METRIC_IP).with_rotation_seed(7)
         .with_high_accuracy_scan(True).with_rerank_k(100))
    assert (c.dim, c.nlist, c.bits_per_dim, c.nprobe, c.metric_type, c.rotation_seed) == \
        (768, 4096, 4, 32, METRIC_IP, 7)
    assert c.use_high_accuracy_scan and c.rerank_k == 100
