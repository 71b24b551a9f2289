"""Multi-rank host logic on CPU (gloo, world size 2): list ownership and the exact
cross-shard merge.

Each rank owns the lists that hanns_gpu_shard_owners assigns to it (the same map
IvfUsqGpu::shard uses), keeps the oracle's candidates of its own lists, reduces them to
a per-rank top-k keyed by (distance, probe rank, FastScan key, list position) -- the
key the GPU shard search emits -- all-gathers, and merges by that key.  The merged
rows must equal the single-index result of the golden fixtures bit for bit, which is
what the NCCL path (all_gather + hanns_gpu_merge_shards_device) relies on.
"""
import glob
import os
import socket

import numpy as np
import pytest

FIXTURES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _key(f):
    b = int(np.float32(f).view(np.uint32))
    return (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)


def _worker(rank, world, port, path, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    from hanns_b200 import _lib
    from oracle import oracle as O
    from tests.golden.make_golden import load

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        art, z = load(path)
        nlist = int(art["nlist"])
        sizes = np.ascontiguousarray(np.diff(art["list_offsets"]), np.int64)
        owner = np.zeros(nlist, np.int32)
        L = _lib.lib()
        assert L.hanns_gpu_shard_owners(sizes.ctypes.data_as(_lib.i64p), nlist, world,
                                        owner.ctypes.data_as(_lib.i32p)) == 0
        owners = [None] * world
        dist.all_gather_object(owners, owner.tolist())
        assert all(o == owners[0] for o in owners)
        k, nprobe = int(z["k"]), int(z["nprobe"])
        oi = O.OracleIndex(art)
        rows = []
        for qi in range(z["queries"].shape[0]):
            c = oi.candidates(z["queries"][qi], k, nprobe)
            rank_of = {int(l): r for r, l in enumerate(z["exp_probes"][qi])}
            mine = []
            for lst, loc, fs, dd in zip(c["list"], c["local"], c["fs"], c["dist"]):
                if owner[lst] != rank:
                    continue
                fkey = 0 if fs == np.iinfo(np.int32).min else 32767 - int(fs)
                key = (_key(dd), rank_of[int(lst)], fkey, int(loc))
                mine.append((key, int(art["ids"][art["list_offsets"][lst] + loc]), float(dd)))
            mine.sort(key=lambda t: t[0])
            rows.append(mine[:k])
        gathered = [None] * world
        dist.all_gather_object(gathered, rows)
        ok = True
        for qi in range(z["queries"].shape[0]):
            merged = sorted((t for g in gathered for t in g[qi]), key=lambda t: t[0])[:k]
            ids = [t[1] for t in merged] + [-1] * (k - len(merged))
            ds = np.array([t[2] for t in merged] + [np.inf] * (k - len(merged)), np.float32)
            ok &= ids == z["exp_ids"][qi].tolist()
            ok &= bool(np.array_equal(ds.view(np.uint32), z["exp_dists"][qi].view(np.uint32)))
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("path", FIXTURES[:3], ids=[os.path.basename(p)[:-4] for p in FIXTURES[:3]])
def test_two_rank_shard_merge_equals_single_index(path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    assert out[0] and out[1]


def test_shard_owners_balanced():
    from hanns_b200 import _lib
    L = _lib.lib()
    rng = np.random.default_rng(0)
    sizes = rng.integers(0, 1000, 4096).astype(np.int64)
    for world in (1, 2, 4, 8):
        owner = np.zeros(4096, np.int32)
        assert L.hanns_gpu_shard_owners(sizes.ctypes.data_as(_lib.i64p), 4096, world,
                                        owner.ctypes.data_as(_lib.i32p)) == 0
        w = sizes.astype(np.float64) ** 2
        loads = np.bincount(owner, weights=w, minlength=world)
        assert owner.min() >= 0 and owner.max() < world
        assert loads.max() - loads.min() <= w.max()


def _rank_loss_worker(rank, world, port, mode, out):
    import datetime
    import sys
    import time
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    from hanns_b200.sharded import gather_query_state

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # a short group timeout is what ends a collective whose peer never arrives
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    full = [torch.zeros(8 * world, dtype=torch.uint8)]
    local = [torch.full((8,), rank, dtype=torch.uint8)]
    gather_query_state(full, local)  # one healthy exchange step
    ok = full[0].view(world, 8).tolist() == [[r] * 8 for r in range(world)]
    if rank == world - 1:
        if mode == "exit":
            os._exit(0)  # the rank dies between steps, no collective in flight
        time.sleep(15)   # the rank stalls: it never joins the next step
        os._exit(0)
    t0 = time.time()
    try:
        gather_query_state(full, local)
        out[rank] = ("no error", time.time() - t0, ok)
    except Exception as e:  # the survivor learns of the loss on the host
        out[rank] = (type(e).__name__, time.time() - t0, ok)
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_rank_loss_ends_the_next_exchange(mode):
    """Failure detection of the multi-GPU protocol, on CPU ranks (gloo): after one good
    all-gather of query state, the last rank exits (or stalls) between steps.  The other
    rank's next all-gather ends with an error -- at once when the peer's connection closes,
    within the group's 4 s timeout when it stalls -- instead of waiting for ever."""
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    out = mgr.dict()
    port = _free_port()
    ctx = mp.start_processes(_rank_loss_worker, args=(2, port, mode, out), nprocs=2,
                             start_method="spawn", join=False)
    import time
    deadline = time.time() + 60
    while not ctx.join(timeout=2) and time.time() < deadline:
        pass
    err, waited, ok = out[0]
    assert ok
    assert err != "no error"
    assert waited < 12.0
