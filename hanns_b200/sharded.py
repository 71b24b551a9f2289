"""List-sharded IVF-USQ search over a process group, one rank per GPU.

The reference searches on one host (src/faiss/ivf_usq.rs:322-352); this module spreads one
index over the ranks of a torch.distributed group.  Every rank holds the whole inverted
lists that hanns_gpu_shard_owners assigns to it; the centroids and the rotation are
replicated.  A step on rank r, for the batch of queries that the caller gave rank r:

  1. prepare the batch (coarse probes, rotation, the per-query state arrays of
     hanns_gpu_ivf_usq_query_state_bytes: probes, scalars, FastScan LUT, q_i8),
  2. all-gather the state, so that every rank holds the state of every rank's batch,
  3. scan the rank's own lists for all of them (hanns_gpu_ivf_usq_search_prepared_shard_device:
     per query the shard's top-k with its tie key),
  4. send each query's shard top-k to the rank whose batch it belongs to (all-to-all), and
  5. merge the world shard lists of the rank's own queries (hanns_gpu_merge_shards_device).

The tie key (probe rank, FastScan key, list position) orders exactly as the single-index
stable sort of src/faiss/ivf_usq.rs:590-593, so the merged rows equal a search of the whole
index on one GPU bit for bit.  Consecutive batches are pipelined (the library's device calls
return once enqueued): the all-gather of batch i+1's state runs while batch i is scanned,
and batch i's all-to-all and merge (on a second stream) while batch i+1 is prepared.

`split_search_device` is the other layout: one batch shared by all ranks, each rank
prepares 1/world of it, and every rank ends with the merged rows of the whole batch.
"""
from __future__ import annotations

import numpy as np

from . import _lib as L


def gather_query_state(full, local, group=None, async_op=False):
    """All-gathers per-query state arrays: full[i] (world * n rows) <- local[i] (n rows) of
    every rank, rank-major, so that query j of rank s lands at row s * n + j."""
    import torch.distributed as dist
    works = [dist.all_gather_into_tensor(f, l, group=group, async_op=async_op)
             for f, l in zip(full, local)]
    return works if async_op else None


def return_partials(recv, send, group=None, async_op=False):
    """All-to-all of shard top-k rows: send[i] holds world * n query rows (rank-major, as
    gathered); afterwards recv[i][s] holds rank s's rows for this rank's n queries, the
    [world][n][k] layout hanns_gpu_merge_shards_device reads."""
    import torch.distributed as dist
    works = [dist.all_to_all_single(r, s, group=group, async_op=async_op)
             for r, s in zip(recv, send)]
    return works if async_op else None


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {L.last_error()}")


class ShardedIvfUsq:
    """One rank's part of a list-sharded index.

    `index` is this rank's IvfUsqIndex holding the whole index; the constructor keeps only
    the lists this rank owns.  `batch` is the number of queries each rank brings to a step
    (equal on all ranks), `k` and `nprobe` those of the search.  Every rank of the group
    must call the same methods with the same arguments in the same order.
    """

    def __init__(self, index, k: int, nprobe: int, batch: int, group=None):
        import torch
        import torch.distributed as dist
        self.idx, self.k, self.group = index, int(k), group
        self.nprobe = max(1, min(int(nprobe), index.config.nlist))
        self.batch = int(batch)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.dev = torch.device("cuda", index.device)
        index.shard(self.rank, self.world)
        lib = L.lib()
        parts = np.zeros(5, np.int64)
        _check(lib.hanns_gpu_ivf_usq_query_state_bytes(index._h, self.nprobe, _i64(parts)),
               "query_state_bytes")
        # probes, scalars, FastScan LUT, q_i8 (dp4a layout): both list scans read these four
        self.n_state = 4
        self.parts = [int(b) for b in parts[:self.n_state]]
        u8 = dict(dtype=torch.uint8, device=self.dev)
        W, n, kk = self.world, self.batch, self.k
        # double-buffered state: batch i+1 is prepared while batch i's state is in flight
        self.st_local = [[torch.empty(n * b, **u8) for b in self.parts] for _ in range(2)]
        self.st_full = [[torch.empty(W * n * b, **u8) for b in self.parts] for _ in range(2)]
        # shard rows (sent) and received rows, double-buffered: batch i's all-to-all and merge
        # run beside batch i+1's preparation and scan
        self.sh = [[torch.empty(W * n, kk, dtype=torch.float32, device=self.dev),
                    torch.empty(W * n, kk, dtype=torch.int64, device=self.dev),
                    torch.empty(W * n, kk, dtype=torch.int64, device=self.dev)] for _ in range(2)]
        self.recv = [[torch.empty(W, n, kk, dtype=t.dtype, device=self.dev) for t in self.sh[0]]
                     for _ in range(2)]
        self.launches = 0
        self._stream = None
        self._mstream = None
        # per-batch CUDA events of search_device when True (stage_times() reads them)
        self.timing = False
        self._ev = []

    def _work_stream(self, stream):
        """The stream the library calls run on: `stream`, or one of the module's own (the
        library runs calls on the legacy default stream synchronously), ordered after the
        caller's current stream."""
        import torch
        cur = torch.cuda.current_stream(self.dev)
        if stream is None:
            if self._stream is None:
                self._stream = torch.cuda.Stream(self.dev)
            stream = self._stream
        if stream.cuda_stream == 0:
            raise ValueError("pass a created stream, not the legacy default stream")
        stream.wait_stream(cur)
        return stream, cur

    # ------------------------------------------------------------ steps
    def _ptrs(self, tensors):
        return [t.data_ptr() for t in tensors] + [None] * (5 - len(tensors))

    def _prepare(self, d_queries: int, slot: int, stream: int):
        _check(L.lib().hanns_gpu_ivf_usq_prepare_device(
            self.idx._h, d_queries, self.batch, self.nprobe, *self._ptrs(self.st_local[slot]),
            stream), "prepare_device")
        self.launches += self.idx.last_launches()

    def _scan(self, slot: int, stream: int, out_slot: int = 0):
        d, key, ids = self.sh[out_slot]
        _check(L.lib().hanns_gpu_ivf_usq_search_prepared_shard_device(
            self.idx._h, self.world * self.batch, self.k, self.nprobe,
            *self._ptrs(self.st_full[slot]), d.data_ptr(), key.data_ptr(), ids.data_ptr(), stream),
            "search_prepared_shard_device")
        self.launches += self.idx.last_launches()

    def _merge(self, out_ids, out_d, stream: int, slot: int = 0):
        d, key, ids = self.recv[slot]
        _check(L.lib().hanns_gpu_merge_shards_device(d.data_ptr(), key.data_ptr(), ids.data_ptr(),
                                                     self.world, self.batch, self.k,
                                                     out_ids.data_ptr(), out_d.data_ptr(), stream),
               "merge_shards_device")
        self.launches += 1

    def search_device(self, batches, outs, stream=None, before=None, prepared=None, after=None):
        """Searches a sequence of this rank's batches.

        batches: device pointers (ints) to `batch` x dim f32 queries each; outs: one
        (ids int64 [batch, k], distances f32 [batch, k]) pair of device tensors per batch.
        Stream-ordered on `stream` (a created torch stream; default: one of the module's own,
        which the caller's current stream then waits for).  Host hooks for copies: before(i)
        runs right before batch i is prepared, prepared(i) right after, after(i) right after
        its merge is enqueued.  Returns with the last merge enqueued.
        """
        import torch
        st, cur = self._work_stream(stream)
        sp = st.cuda_stream
        if self._mstream is None:
            self._mstream = torch.cuda.Stream(self.dev)
        ms = self._mstream
        ms.wait_stream(st)
        merged = [None, None]   # event: the merge that last read recv[b] is done
        a2a = [None, None]      # works of the all-to-all that last read sh[b]
        pending = None  # (index, slot, gather works) of the batch whose state is in flight
        n = len(batches)
        # timing: per batch six events -- prepare begin / end, scan begin (state gathered) /
        # end on the work stream, all-to-all done / merge done on the merge stream
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(n)] if self.timing else None
        with torch.cuda.stream(st):
            for i in range(n + 1):
                nxt = None
                if i < n:
                    slot = i % 2
                    if before:
                        before(i)
                    if ev:
                        ev[i][0].record(st)
                    self._prepare(batches[i], slot, sp)
                    if ev:
                        ev[i][1].record(st)
                    if prepared:
                        prepared(i)
                    nxt = (i, slot, gather_query_state(self.st_full[slot], self.st_local[slot],
                                                       self.group, async_op=True))
                if pending is not None:
                    j, b, works = pending
                    for w in works:
                        w.wait()
                    for w in a2a[b] or ():
                        w.wait()  # batch j-2's all-to-all has read sh[b]
                    if ev:
                        ev[j][2].record(st)
                    self._scan(b, sp, b)
                    if ev:
                        ev[j][3].record(st)
                    if merged[b] is not None:
                        st.wait_event(merged[b])  # batch j-2's merge has read recv[b]
                    a2a[b] = return_partials(self.recv[b], self.sh[b], self.group, async_op=True)
                    with torch.cuda.stream(ms):
                        for w in a2a[b]:
                            w.wait()
                        if ev:
                            ev[j][4].record(ms)
                        ids, dist_ = outs[j]
                        self._merge(ids, dist_, ms.cuda_stream, b)
                        if ev:
                            ev[j][5].record(ms)
                        merged[b] = torch.cuda.Event()
                        merged[b].record(ms)
                        if after:
                            after(j)
                pending = nxt
        if ev:
            self._ev.extend(ev)
        st.wait_stream(ms)
        if cur != st:
            cur.wait_stream(st)

    def stage_times(self, last: int = 0):
        """Median ms per batch of each stage over the batches timed so far (the last `last`
        when > 0): prepare; state wait (from the end of the next batch's preparation to the
        start of the scan: the all-gather not hidden behind that preparation); scan;
        all-to-all (scan end to shard rows received); merge; step (prepare begin to the
        next batch's prepare begin).  Waits for the events; clears them."""
        import statistics
        ev = self._ev[-last:] if last else self._ev
        self._ev = []
        if not ev:
            return {}
        for e in ev:
            e[5].synchronize()
        rows = {"prepare": [], "state_wait": [], "scan": [], "all_to_all": [], "merge": [], "step": []}
        for i, e in enumerate(ev):
            rows["prepare"].append(e[0].elapsed_time(e[1]))
            rows["scan"].append(e[2].elapsed_time(e[3]))
            rows["all_to_all"].append(e[3].elapsed_time(e[4]))
            rows["merge"].append(e[4].elapsed_time(e[5]))
            if i + 1 < len(ev):
                rows["state_wait"].append(ev[i + 1][1].elapsed_time(e[2]))
                rows["step"].append(e[0].elapsed_time(ev[i + 1][0]))
        return {k: statistics.median(v) for k, v in rows.items() if v}

    def search_host(self, queries, out_ids, out_dists):
        """Searches this rank's batches from host memory.

        queries: list of host tensors (batch x dim f32, pinned for overlap); out_ids /
        out_dists: lists of host tensors [batch, k] (int64 / f32) of the same length.
        Batch i+1 is copied in on a copy stream while batch i is prepared; each batch's
        rows are copied out after its merge.  Returns when every copy has finished.
        """
        import torch
        st, _ = self._work_stream(None)
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(self.dev)
        cp = self._copy_stream
        d = int(queries[0].shape[1])
        if getattr(self, "_dq", None) is None or self._dq[0].shape[1] != d:
            self._dq = [torch.empty(self.batch, d, dtype=torch.float32, device=self.dev)
                        for _ in range(2)]
            self._res = (torch.empty(self.batch, self.k, dtype=torch.int64, device=self.dev),
                         torch.empty(self.batch, self.k, dtype=torch.float32, device=self.dev))
        n = len(queries)
        up = [torch.cuda.Event() for _ in range(2)]
        read = [torch.cuda.Event() for _ in range(2)]

        def upload(i):
            with torch.cuda.stream(cp):
                if i >= 2:
                    cp.wait_event(read[i % 2])  # batch i-2 was prepared from this buffer
                self._dq[i % 2].copy_(queries[i], non_blocking=True)
                up[i % 2].record(cp)

        def before(i):
            if i + 1 < n:
                upload(i + 1)
            st.wait_event(up[i % 2])

        def prepared(i):
            read[i % 2].record(st)

        def after(j):
            out_ids[j].copy_(self._res[0], non_blocking=True)
            out_dists[j].copy_(self._res[1], non_blocking=True)

        upload(0)
        self.search_device([self._dq[i % 2].data_ptr() for i in range(n)], [self._res] * n, st,
                           before, prepared, after)
        st.synchronize()

    def search(self, queries: np.ndarray):
        """Host convenience: one batch (batch x dim f32) in, (ids, distances) out."""
        import torch
        q = torch.from_numpy(np.ascontiguousarray(queries, np.float32).reshape(self.batch, -1))
        ids = torch.empty(self.batch, self.k, dtype=torch.int64)
        ds = torch.empty(self.batch, self.k, dtype=torch.float32)
        self.search_host([q], [ids], [ds])
        return ids.numpy(), ds.numpy()


class SplitShardedIvfUsq(ShardedIvfUsq):
    """One batch shared by all ranks: rank r prepares rows [r*n, (r+1)*n) of it (n = batch
    / world), every rank scans its lists for the whole batch, the shard rows are
    all-gathered and every rank merges the whole batch."""

    def __init__(self, index, k: int, nprobe: int, batch: int, group=None):
        import torch
        import torch.distributed as dist
        world = dist.get_world_size(group)
        if batch % world:
            raise ValueError("the batch must split evenly over the ranks")
        super().__init__(index, k, nprobe, batch // world, group)
        self.total = batch
        self.gath = [torch.empty(self.world, batch, self.k, dtype=t.dtype, device=self.dev)
                     for t in self.sh[0]]

    def split_search_device(self, d_queries: int, out_ids, out_d, stream=None):
        """d_queries: device pointer to the whole batch (batch x dim f32, the same batch
        on every rank); out_ids / out_d: [batch, k] device tensors, filled on every rank."""
        import torch
        import torch.distributed as dist
        st, cur = self._work_stream(stream)
        sp = st.cuda_stream
        row = self.idx.config.dim * 4
        with torch.cuda.stream(st):
            self._prepare(d_queries + self.rank * self.batch * row, 0, sp)
            gather_query_state(self.st_full[0], self.st_local[0], self.group)
            self._scan(0, sp)
            for g, s in zip(self.gath, self.sh[0]):
                dist.all_gather_into_tensor(g, s, group=self.group)
            d, key, ids = self.gath
            _check(L.lib().hanns_gpu_merge_shards_device(d.data_ptr(), key.data_ptr(),
                                                         ids.data_ptr(), self.world, self.total,
                                                         self.k, out_ids.data_ptr(),
                                                         out_d.data_ptr(), sp),
                   "merge_shards_device")
            self.launches += 1
        if cur != st:
            cur.wait_stream(st)


def _i64(a):
    return a.ctypes.data_as(L.i64p)
