"""hanns_b200.sharded: list-sharded search with one batch per rank.

CPU (gloo, world size 2): the two exchange steps of the module -- gather_query_state and
return_partials -- carry real tensors between ranks; each rank's shard rows come from the
oracle's candidates of the lists it owns (hanns_gpu_shard_owners), keyed as the GPU shard
search keys them, and the merge of what return_partials delivered must equal the golden
rows of the rank's own queries bit for bit.

GPU (gloo, world size 2 on one device): ShardedIvfUsq end to end -- prepare, all-gather,
shard scan, all-to-all, merge -- against a single-GPU search of the whole index, for
the device and the host entry points and several pipelined batches.
"""
import glob
import os
import socket

import numpy as np
import pytest

FIXTURES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _total_order(f):
    b = np.asarray(f, np.float32).view(np.uint32).astype(np.uint64)
    return np.where(b & 0x80000000, ~b & 0xFFFFFFFF, b | 0x80000000)


def _exchange_worker(rank, world, port, path, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from hanns_b200 import _lib
    from hanns_b200.sharded import gather_query_state, return_partials
    from oracle import oracle as O
    from tests.golden.make_golden import load

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        art, z = load(path)
        nlist = int(art["nlist"])
        k, nprobe = int(z["k"]), int(z["nprobe"])
        sizes = np.ascontiguousarray(np.diff(art["list_offsets"]), np.int64)
        owner = np.zeros(nlist, np.int32)
        assert _lib.lib().hanns_gpu_shard_owners(sizes.ctypes.data_as(_lib.i64p), nlist, world,
                                                 owner.ctypes.data_as(_lib.i32p)) == 0
        n = z["queries"].shape[0] // world
        mine = slice(rank * n, (rank + 1) * n)
        # the "query state" here is the raw query plus its expected probes, as bytes
        q_local = torch.from_numpy(np.ascontiguousarray(z["queries"][mine], np.float32))
        p_local = torch.from_numpy(np.ascontiguousarray(z["exp_probes"][mine], np.int32))
        local = [q_local.view(torch.uint8).reshape(-1), p_local.view(torch.uint8).reshape(-1)]
        full = [torch.empty(world * t.numel(), dtype=torch.uint8) for t in local]
        gather_query_state(full, local)
        qs = full[0].view(torch.float32).reshape(world * n, -1).numpy()
        ps = full[1].view(torch.int32).reshape(world * n, -1).numpy()
        assert np.array_equal(qs, np.asarray(z["queries"][:world * n], np.float32))
        oi = O.OracleIndex(art)
        sh_d = np.full((world * n, k), np.inf, np.float32)
        sh_k = np.full((world * n, k), -1, np.int64)  # ~0 as int64: an empty slot
        sh_i = np.full((world * n, k), -1, np.int64)
        for qi in range(world * n):
            c = oi.candidates(qs[qi], k, nprobe)
            rank_of = {int(l): r for r, l in enumerate(ps[qi])}
            rows = []
            for lst, loc, fs, dd in zip(c["list"], c["local"], c["fs"], c["dist"]):
                if owner[lst] != rank:
                    continue
                fkey = 0 if fs == np.iinfo(np.int32).min else 32767 - int(fs)
                key = (rank_of[int(lst)] << 48) | (fkey << 32) | int(loc)
                rows.append((int(_total_order(dd)), key, float(dd),
                             int(art["ids"][art["list_offsets"][lst] + loc])))
            rows.sort()
            for j, (_, key, dd, gid) in enumerate(rows[:k]):
                sh_d[qi, j], sh_k[qi, j], sh_i[qi, j] = dd, key, gid
        send = [torch.from_numpy(a) for a in (sh_d, sh_k, sh_i)]
        recv = [torch.empty(world, n, k, dtype=t.dtype) for t in send]
        return_partials(recv, send)
        rd, rk, ri = (t.numpy() for t in recv)
        ok = True
        for j in range(n):
            cand = [(int(_total_order(rd[s, j, c])), int(rk[s, j, c]) & 0xFFFFFFFFFFFFFFFF,
                     float(rd[s, j, c]), int(ri[s, j, c]))
                    for s in range(world) for c in range(k) if rk[s, j, c] != -1]
            cand.sort()
            ids = [t[3] for t in cand[:k]] + [-1] * (k - min(k, len(cand)))
            ds = np.array([t[2] for t in cand[:k]] + [np.inf] * (k - min(k, len(cand))), np.float32)
            ok &= ids == z["exp_ids"][rank * n + j].tolist()
            ok &= bool(np.array_equal(ds.view(np.uint32), z["exp_dists"][rank * n + j].view(np.uint32)))
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def _spawn(target, world, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (out,)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    return [out.get(r) for r in range(world)]


@pytest.mark.parametrize("path", FIXTURES[:3], ids=[os.path.basename(p)[:-4] for p in FIXTURES[:3]])
def test_exchange_one_batch_per_rank(path):
    res = _spawn(_exchange_worker, 2, path)
    assert res == [True, True]


def _gpu_worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from hanns_b200.ivf_usq import IvfUsqIndex
    from hanns_b200.sharded import ShardedIvfUsq
    from oracle import oracle as O
    from tests.golden.make_golden import mixture

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(0)
        rng = np.random.default_rng(31)
        d, k, nprobe, n, nb = 128, 10, 6, 300, 3
        x, _ = mixture(rng, 20000, d, 32, 0.4, False)
        q, _ = mixture(rng, world * n * nb, d, 32, 0.4, False)
        art = O.build_artifact(x, 24, 4, O.METRIC_L2, rotation_seed=3, kmeans_iters=5, kmeans_seed=2)
        full = IvfUsqIndex.from_artifact(art)
        # rank r's batches: rows [(b * world + r) * n, ... + n)
        mine = [q[(b * world + rank) * n:(b * world + rank + 1) * n] for b in range(nb)]
        exp = []
        for m in mine:
            e_ids = torch.empty(n, k, dtype=torch.int64, device="cuda")
            e_d = torch.empty(n, k, dtype=torch.float32, device="cuda")
            dq = torch.from_numpy(m).cuda()
            full.search_device(dq.data_ptr(), n, k, nprobe, e_ids.data_ptr(), e_d.data_ptr())
            exp.append((e_ids.cpu().numpy(), e_d.cpu().numpy()))
        full.close()
        sh = ShardedIvfUsq(IvfUsqIndex.from_artifact(art), k, nprobe, n)
        dqs = [torch.from_numpy(m).cuda() for m in mine]
        outs = [(torch.empty(n, k, dtype=torch.int64, device="cuda"),
                 torch.empty(n, k, dtype=torch.float32, device="cuda")) for _ in range(nb)]
        sh.search_device([t.data_ptr() for t in dqs], outs)
        torch.cuda.synchronize()
        ok = all(np.array_equal(o[0].cpu().numpy(), e[0]) and
                 np.array_equal(o[1].cpu().numpy().view(np.uint32), e[1].view(np.uint32))
                 for o, e in zip(outs, exp))
        hq = [torch.from_numpy(m).pin_memory() for m in mine]
        hi = [torch.empty(n, k, dtype=torch.int64).pin_memory() for _ in range(nb)]
        hd = [torch.empty(n, k, dtype=torch.float32).pin_memory() for _ in range(nb)]
        sh.search_host(hq, hi, hd)
        ok &= all(np.array_equal(i.numpy(), e[0]) and
                  np.array_equal(dd.numpy().view(np.uint32), e[1].view(np.uint32))
                  for i, dd, e in zip(hi, hd, exp))
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_two_ranks_equal_single_gpu():
    res = _spawn(_gpu_worker, 2)
    assert res == [True, True]
