"""Failure paths on the GPU, without faulting the GPU.

* A bounded wait inside the tensor-core list scan is made to run out (a wait limit of
  1 ns, set through the C ABI): the scan records an error code, lets the MMAs it issued
  finish, frees its tensor memory and returns; the search fails with an error message,
  and the next search on the same index and context equals the oracle again.
* Host-side fault injection: device allocations or host-to-device copies made to fail as
  if CUDA had returned an error.  The C ABI returns an error code with a message; after
  the injection is switched off the same calls succeed.
No kernel is given a bad address and nothing traps: the faults exist only on the host.
"""
import os

import numpy as np
import pytest

from tests.golden.make_golden import load

pytestmark = pytest.mark.gpu

FIXTURE = os.path.join(os.path.dirname(__file__), "golden", "l2_4bit_d128.npz")


@pytest.fixture(scope="module")
def lib():
    from hanns_b200 import _lib
    L = _lib.lib()
    if L.hanns_gpu_device_count() < 1:
        pytest.fail("no CUDA device visible to libhanns_gpu")
    return L


def _search(idx, z):
    from hanns_b200.ivf_usq import SearchRequest
    return idx.search(z["queries"], SearchRequest(top_k=int(z["k"]), nprobe=int(z["nprobe"])))


def _equal_oracle(r, z):
    ids = r.ids.reshape(z["exp_ids"].shape)
    d = r.distances.reshape(z["exp_ids"].shape)
    return np.array_equal(ids, z["exp_ids"]) and np.array_equal(d.view(np.uint32), z["exp_dists"].view(np.uint32))


def test_expired_scan_wait_reports_and_recovers(lib):
    from hanns_b200.ivf_usq import IvfUsqIndex
    art, z = load(FIXTURE)
    assert (np.diff(art["list_offsets"]) > 150).any()  # FastScan GEMMs run
    idx = IvfUsqIndex.from_artifact(art)
    assert _equal_oracle(_search(idx, z), z)
    assert lib.hanns_gpu_ivf_usq_set_scan_wait_ns(idx._h, 1) == 0
    with pytest.raises(RuntimeError, match="bounded wait expired"):
        _search(idx, z)
    assert lib.hanns_gpu_ivf_usq_set_scan_wait_ns(idx._h, 2_000_000_000) == 0
    assert _equal_oracle(_search(idx, z), z)
    assert lib.hanns_gpu_ivf_usq_set_scan_wait_ns(idx._h, 0) == 2  # HANNS_INVALID_ARG


@pytest.mark.parametrize("what", ["alloc", "h2d"])
def test_injected_host_faults(lib, what):
    from hanns_b200.ivf_usq import IvfUsqIndex
    art, z = load(FIXTURE)
    try:
        assert lib.hanns_gpu_debug_inject_fault(what.encode()) == 0
        with pytest.raises((ValueError, RuntimeError)) as ei:
            idx = IvfUsqIndex.from_artifact(art)  # uploads the artifact (allocations + copies)
            _search(idx, z)
        msg = str(ei.value).lower()
        assert ("injected" in msg) if what == "h2d" else ("memory" in msg)
    finally:
        assert lib.hanns_gpu_debug_inject_fault(b"none") == 0
    idx = IvfUsqIndex.from_artifact(art)
    assert _equal_oracle(_search(idx, z), z)
    assert lib.hanns_gpu_debug_inject_fault(b"bogus") != 0
