"""hanns_gpu_coarse_probes_static: the coarse-probe step for callers that cannot allocate.

Processes that hand all device memory to their own pool, and latency-critical paths
that must not call cudaMalloc/cudaFree, use this entry point; it runs on a fixed
scratch array compiled into the library.  This test calls it through the C ABI twice
in a row (different query sets, so the second call overwrites the shared scratch) and
checks that each call's probes equal the probes of the regular search path
(hanns_gpu_ivf_usq_debug_query) exactly -- probes are integers, so the tolerance is 0.
It also checks that an oversize request is refused without running.  The file name
makes pytest collect it last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_static_scratch_coarse_probes_match_search_path():
    import torch

    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqIndex
    from tests.golden.make_golden import load
    import glob
    import os

    L = _lib.lib()
    assert L.hanns_gpu_device_count() >= 1
    path = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "ip_4bit_k100.npz")))[0]
    art, z = load(path)
    idx = IvfUsqIndex.from_artifact(art, device=0)
    rng = np.random.default_rng(123)
    d, nlist = int(art["dim"]), int(art["nlist"])
    cent = torch.from_numpy(np.ascontiguousarray(art["centroids"], np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call, nq in enumerate([300, 77]):
        qn = (z["queries"][rng.integers(0, z["queries"].shape[0], nq)]
              + 0.05 * rng.normal(size=(nq, d))).astype(np.float32)
        nprobe = 5 if call == 0 else 8
        expected = idx.debug_query(qn, nprobe)["probes"]
        q = torch.from_numpy(qn).cuda()
        out = torch.full((nq, nprobe), -7, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        rc = L.hanns_gpu_coarse_probes_static(q.data_ptr(), nq, cent.data_ptr(), nlist, d, nprobe,
                                              out.data_ptr(), stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), expected)
    # beyond the fixed scratch: refused with a clear message, output untouched
    big_nq = (16 << 20) // (4 * nlist) + 1
    q = torch.zeros(big_nq, d, dtype=torch.float32, device="cuda")
    out = torch.full((big_nq, 1), -7, dtype=torch.int32, device="cuda")
    rc = L.hanns_gpu_coarse_probes_static(q.data_ptr(), big_nq, cent.data_ptr(), nlist, d, 1,
                                          out.data_ptr(), stream)
    torch.cuda.synchronize()
    assert rc == 2
    assert "scratch" in _lib.last_error()
    assert int(out.min()) == -7 and int(out.max()) == -7
    # every device that loads the library has its own copy of the scratch array: with a
    # second GPU, one call with that device current (its own queries and centroids) equals
    # the search path of an index living on that device
    if L.hanns_gpu_device_count() >= 2:
        idx1 = IvfUsqIndex.from_artifact(art, device=1)
        qn = z["queries"][:64].astype(np.float32)
        expected = idx1.debug_query(qn, 6)["probes"]
        with torch.cuda.device(1):
            q1 = torch.from_numpy(qn).cuda(1)
            c1 = torch.from_numpy(np.ascontiguousarray(art["centroids"], np.float32)).cuda(1)
            o1 = torch.full((64, 6), -7, dtype=torch.int32, device="cuda:1")
            rc = L.hanns_gpu_coarse_probes_static(q1.data_ptr(), 64, c1.data_ptr(), nlist, d, 6,
                                                  o1.data_ptr(), torch.cuda.current_stream(1).cuda_stream)
            assert rc == 0, _lib.last_error()
            torch.cuda.synchronize(1)
        assert np.array_equal(o1.cpu().numpy(), expected)
