"""IVF-USQ batched search benchmark (B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload B]

Workload B (default): 1,000,000 x 768 fp32 base from a 1,024-component Gaussian mixture
(centres ~ N(0,1), sigma 0.5), every vector L2-normalised; 10,000 normalised queries
from the same mixture; IVF-USQ 4-bit, inner product, nlist 4,096, nprobe 32, k 10,
seed 7.  Seeded synthetic data stands in for the reference's Cohere-Wiki-1M set.

A step is one batched search of the 10,000 queries.  `value` = queries/s with the
queries and the index already in HBM (CUDA events on the launching stream); `e2e` =
the same through the host-pointer C ABI call (pinned host queries in, ids and
distances out, copies inside the timed region).  With N > 1 (torchrun, one rank per
GPU) the inverted lists are sharded over the ranks (LPT on |L|^2) and every rank brings
its own batch of 10,000 queries (rank 0's is the single-GPU batch, the others are further
draws from the same mixture): it prepares its batch (coarse probes, rotation, query
state), the query state is all-gathered over NCCL, every rank scans its lists for all
ranks' batches, the shard top-k go back to the batch's rank in an NCCL all-to-all and
each rank merges its own rows (per-rank work fixed: weak scaling; `value` counts all
ranks' queries).  Batches are pipelined: a batch's all-gather runs while the next batch is
prepared.  --split keeps one 10,000-query batch for the whole job instead (each rank
prepares 1/N of it; strong scaling).

--impl reference times the CPU restatement of the reference's search path (the
oracle; the Rust reference cannot be built here) on the host cores, on the same
frozen index, one bounded sample of queries per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: n, d, comps, sigma, nq, nlist, nprobe, k, nbits, metric(0 L2/1 IP), seed, normalise
    "B": dict(n=1_000_000, d=768, comps=1024, sigma=0.5, nq=10_000, nlist=4096, nprobe=32, k=10,
              nbits=4, metric=1, seed=7, normalise=True),
    "C": dict(n=1_000_000, d=768, comps=1024, sigma=0.5, nq=10_000, nlist=4096, nprobe=32, k=100,
              nbits=8, metric=1, seed=11, normalise=True),
    "A": dict(n=100_000, d=128, comps=64, sigma=0.3, nq=1_000, nlist=256, nprobe=16, k=10,
              nbits=4, metric=0, seed=42, normalise=False),
    "D": dict(n=260_000, d=3072, comps=256, sigma=0.4, nq=5_000, nlist=1024, nprobe=24, k=10,
              nbits=8, metric=1, seed=3, normalise=True),
    # the 8x-compression variant of D: 4-bit codes, FastScan runs on lists above 150 rows
    "D4": dict(n=260_000, d=3072, comps=256, sigma=0.4, nq=5_000, nlist=1024, nprobe=24, k=10,
               nbits=4, metric=1, seed=3, normalise=True),
    # scale-out shape: a step is one query batch of 16,384 (the configuration's batch size
    # for its 100,000-query set); lists average ~305 rows, below n_cand = 1,500, so
    # FastScan never runs and the rerank is the whole scan.  k-means on 16 rows per list
    # (1 Mi rows), 10 iterations: the build is not timed.
    "E": dict(n=20_000_000, d=768, comps=16384, sigma=0.5, nq=16_384, nlist=65536, nprobe=64,
              k=100, nbits=4, metric=1, seed=19, normalise=True, train_per_list=16,
              kmeans_iters=10),
}
TRAIN_ROWS_PER_LIST = 64
KMEANS_ITERS = 25  # KMeans::new max_iter (src/quantization/kmeans.rs:44-56), early stop at shift < 1e-2
CACHE_DIR = os.environ.get("HANNS_BENCH_CACHE", "/tmp/hanns_b200_bench_cache")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def int8_peak():
    """Dense int8 tensor rate: the B200 runs int8 (like fp8) at twice its dense bf16 rate
    (4.5 vs 2.25 P nominal), so the peak is 2 x the measured cuBLAS bf16 burst figure."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return 2.0 * float(json.load(f)["bf16_tflops"]), "derived: 2 x measured bf16 burst"
    except Exception:
        return 2.0 * 1590.0, "derived: 2 x fallback bf16 burst"


def scan_tc_ops(art, probes, k, nbits, tc_max_rows=2048):
    """int8 MMA operations (2 per multiply-add) the tensor-core list scan issues for one
    batch: per item (one list, up to tc_queries_per_item queries, N rounded up to 16) the
    FastScan GEMM (K = 4 D, lists above n_cand) and the rerank GEMM (K = D) over all T
    tiles of 128 rows."""
    from oracle.oracle import n_candidates
    D = int(art["padded_dim"])
    ncand = n_candidates(nbits, k)
    sizes = np.diff(np.asarray(art["list_offsets"], dtype=np.int64))
    pr = probes.reshape(-1)
    q_per_list = np.bincount(pr[(pr >= 0) & (pr < sizes.shape[0])], minlength=sizes.shape[0])
    ops = 0
    for l in np.nonzero((q_per_list > 0) & (sizes > 0) & (sizes <= tc_max_rows))[0]:
        n, q = int(sizes[l]), int(q_per_list[l])
        t = (n + 127) // 128
        qpi = min(128, (256 // t) & ~15)  # tc_queries_per_item: N * T <= 256
        kk = D + (4 * D if n > ncand else 0)
        full, rest = divmod(q, qpi)
        nsum = full * qpi + ((rest + 15) // 16) * 16
        ops += 2 * 128 * t * nsum * kk
    return ops


# ------------------------------------------------------------------ data
def _mixture_draw(w, centres, g, n):
    import torch
    lab = torch.randint(0, w["comps"], (n,), generator=g, device=centres.device)
    x = centres[lab] + w["sigma"] * torch.randn(n, w["d"], generator=g, device=centres.device)
    if w["normalise"]:
        x = x / x.norm(dim=1, keepdim=True)
    return x.contiguous()


def _centres(w, g, device):
    import torch
    return torch.randn(w["comps"], w["d"], generator=g, device=device)


def _mixture_draw_chunked(w, centres, g, n, chunk=1 << 21):
    """The same mixture drawn 2 Mi rows at a time into one preallocated tensor (a base of
    tens of GB leaves no room for the single-shot draw's temporaries)."""
    import torch
    x = torch.empty(n, w["d"], dtype=torch.float32, device=centres.device)
    for s in range(0, n, chunk):
        x[s:s + chunk] = _mixture_draw(w, centres, g, min(chunk, n - s))
    return x


def make_data(w, device="cuda"):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(w["seed"])
    centres = _centres(w, g, device)
    draw = _mixture_draw_chunked if w["n"] > (1 << 22) else _mixture_draw
    base = draw(w, centres, g, w["n"])
    queries = _mixture_draw(w, centres, g, w["nq"])
    return base, queries


def extra_queries(w, device, r):
    """Batch r >= 1 of queries from the same mixture (batch 0 is make_data's)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(w["seed"])
    centres = _centres(w, g, device)
    g2 = torch.Generator(device=device)
    g2.manual_seed(w["seed"] * 1_000_003 + r)
    return _mixture_draw(w, centres, g2, w["nq"])


def exact_topk(base, queries, k, metric, base_chunk=1 << 20):
    """Exact fp32 top-k ids (no TF32), base rows taken 1 Mi at a time."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    out = []
    for s in range(0, queries.shape[0], 1024):
        q = queries[s:s + 1024]
        best_v = best_i = None
        for b0 in range(0, base.shape[0], base_chunk):
            xb = base[b0:b0 + base_chunk]
            ip = q @ xb.T
            score = ip if metric == 1 else -((xb * xb).sum(1)[None, :] - 2 * ip)
            v, i = score.topk(min(k, xb.shape[0]), dim=1)
            i = i + b0
            if best_v is None:
                best_v, best_i = v, i
            else:
                v = torch.cat([best_v, v], 1)
                i = torch.cat([best_i, i], 1)
                best_v, j = v.topk(k, dim=1)
                best_i = i.gather(1, j)
        out.append(best_i)
    return torch.cat(out).cpu().numpy()


def build_index(w, base_np, device):
    """Trains on a seeded subsample and adds every row (GPU build path, C ABI)."""
    from hanns_b200.ivf_usq import IvfUsqConfig, IvfUsqIndex
    cfg = IvfUsqConfig(w["d"], w["nlist"], w["nbits"], nprobe=w["nprobe"], metric_type=w["metric"],
                       rotation_seed=42)
    idx = IvfUsqIndex(cfg, device=device)
    rng = np.random.default_rng(w["seed"])
    ntrain = train_rows(w)
    tr = base_np[np.sort(rng.choice(base_np.shape[0], ntrain, replace=False))]
    iters = w.get("kmeans_iters", KMEANS_ITERS)
    t0 = time.time()
    idx.train(tr, kmeans_iters=iters, kmeans_seed=w["seed"])
    t1 = time.time()
    idx.add(base_np)
    log(f"[build] train {t1 - t0:.1f}s ({ntrain} rows, {iters} iters) add {time.time() - t1:.1f}s")
    return idx


def train_rows(w):
    return min(w["n"], w.get("train_per_list", TRAIN_ROWS_PER_LIST) * w["nlist"])


def cache_path(name):
    return os.path.join(CACHE_DIR, f"workload_{name}_kpp_artifact.npz")


def load_artifact(name):
    z = np.load(cache_path(name))
    return {k: (z[k].item() if z[k].ndim == 0 else z[k]) for k in z.files}


def get_artifact(name, w, base, device, cache=None):
    """Frozen index of the workload: built with the GPU build path once, cached on disk
    (by default only indexes of at most 4 Mi rows: the 20 M-row one is ~12 GB)."""
    p = cache_path(name)
    if os.path.exists(p):
        return load_artifact(name)
    idx = build_index(w, base.cpu().numpy(), device)
    art = idx.export_artifact()
    idx.close()
    if cache is None:
        cache = w["n"] <= (1 << 22)
    if not cache:
        return art
    os.makedirs(CACHE_DIR, exist_ok=True)
    tmp = p + f".tmp{os.getpid()}.npz"
    np.savez(tmp, **art)
    os.replace(tmp, p)
    return art


def scan_bytes(art, probes, k, nbits):
    """Algorithmic bytes of the list-scan kernel for one batch: per (query, probe),
    |L|*D/8 sign bytes when FastScan runs, plus (code bytes + 16 B meta + 8 B id) per
    reranked candidate."""
    from oracle.oracle import n_candidates
    D = int(art["padded_dim"])
    cb = (D * nbits + 7) // 8
    ncand = n_candidates(nbits, k)
    sizes = np.diff(art["list_offsets"])[probes.reshape(-1)]
    fs = sizes > ncand
    return int((sizes * (D // 8) * fs).sum() + (np.minimum(sizes, ncand) * (cb + 24)).sum())


def measured_traffic(name, kernel):
    """(DRAM bytes per launch, kernel ms under ncu, file) from the committed ncu summary of
    this kernel on this workload, or (None, None, None)."""
    import re
    path = os.path.join("profiles", f"{kernel}_workload_{name}.md")
    try:
        with open(os.path.join(ROOT, path)) as f:
            txt = f.read()
    except OSError:
        return None, None, None
    m = re.search(r"dram_bytes_per_launch \| (\d+)", txt)
    t = re.search(r"gpu__time_duration_ms \| ([0-9.]+)", txt)
    return (int(m.group(1)) if m else None), (float(t.group(1)) if t else None), path


def index_stats(art, probes, k, nbits):
    """List-size and list-grouping figures of one batch: what the scan's work depends on."""
    from oracle.oracle import n_candidates
    sizes = np.diff(np.asarray(art["list_offsets"], dtype=np.int64))
    nlist = sizes.shape[0]
    ncand = n_candidates(nbits, k)
    pr = probes.reshape(-1)
    pr = pr[(pr >= 0) & (pr < nlist)]
    q_per_list = np.bincount(pr, minlength=nlist)
    probed = q_per_list > 0
    psz = sizes[pr]
    return {"list_rows": {"min": int(sizes.min()), "median": float(np.median(sizes)),
                          "mean": float(sizes.mean()), "p99": float(np.percentile(sizes, 99)),
                          "max": int(sizes.max()), "empty": int((sizes == 0).sum())},
            "probed_list_rows_mean": float(psz.mean()) if psz.size else 0.0,
            "queries_per_probed_list": {"mean": float(q_per_list[probed].mean()) if probed.any() else 0.0,
                                        "max": int(q_per_list.max())},
            "n_cand": int(ncand),
            "pairs_with_fastscan": float((psz > ncand).mean()) if psz.size else 0.0,
            "reranked_rows_per_query": float(np.minimum(psz, ncand).sum() / max(probes.shape[0], 1))}


def scan_roofline_tc(workload, alg_bytes, ops, scan_s, world):
    """Roofline of the tensor-core list scan kernel (the dominant kernel): executed int8 MMA
    ops per launch over its live CUDA-event launch time against the dense int8 rate; beside
    it the per-(query, probe) stream bytes of the reference's loop (algorithmic_*) and the
    DRAM bytes ncu measured for one launch (dram_*).  Neither the tensor pipe nor DRAM is
    the limit: `limiter` names what is."""
    peak, src = int8_peak()
    hbm, hbm_kind = peaks()
    kernel = "scan_tc_kernel"
    traffic, ncu_ms, path = measured_traffic(workload, kernel) if world == 1 else (None, None, None)
    achieved = ops / scan_s / 1e12
    roof = {"kernel": kernel, "bound": "tensor", "unit": "TOPS", "achieved": achieved, "peak": peak,
            "frac": achieved / peak, "peak_source": src, "launch_ms": scan_s * 1e3,
            "mma_ops_per_launch": ops, "traffic": traffic,
            "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch ({path}, "
                               f"{ncu_ms} ms under ncu)") if traffic else "no ncu capture for this workload",
            "algorithmic_bytes_per_launch": alg_bytes, "algorithmic_gbs": alg_bytes / scan_s / 1e9,
            "algorithmic_frac_of_hbm": alg_bytes / scan_s / 1e9 / hbm, "hbm_peak_gbs": hbm,
            "hbm_peak_source": hbm_kind,
            "limiter": "operand staging: the A builder warps' global loads of sign words and codes "
                       "(long-scoreboard stalls) before they expand one-hot rows / unpack codes into "
                       "a 32 KiB ring stage, and the mbarrier hand-off of each stage to the MMA "
                       "warp; tensor activity also varies by SM with the list sizes of its items"}
    if traffic:
        roof["dram_gbs"] = traffic / scan_s / 1e9
        roof["dram_frac_of_hbm"] = roof["dram_gbs"] / hbm
    return roof


def scan_roofline(workload, alg_bytes, scan_s, world):
    """Roofline of the list scan (the dominant stage).

    achieved / frac use the DRAM bytes ncu measured for one launch on this workload (the
    committed summary under profiles/) over the live CUDA-event launch time; the
    per-(query, probe) stream bytes of the reference's loop (sign bytes of every FastScan
    list plus code + meta + id bytes of every reranked row) are reported beside it as
    algorithmic_* -- list grouping reads each list once per batch, so those bytes mostly
    come from L2 and the scan is limited by instruction issue, not by HBM."""
    peak, peak_kind = peaks()
    kernel = "scan_lists_kernel"
    traffic, ncu_ms, path = measured_traffic(workload, kernel) if world == 1 else (None, None, None)
    alg_gbs = alg_bytes / scan_s / 1e9
    roof = {"kernel": kernel, "bound": "hbm", "unit": "GB/s", "peak": peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
            "launch_ms": scan_s * 1e3, "traffic": traffic,
            "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch ({path}, "
                               f"{ncu_ms} ms under ncu)") if traffic else "no ncu capture for this workload",
            "limiter": "integer instruction issue (FastScan LUT lookups, dp4a rerank, kept-set selection)",
            "algorithmic_bytes_per_launch": alg_bytes, "algorithmic_gbs": alg_gbs,
            "algorithmic_frac_of_hbm": alg_gbs / peak}
    if traffic:
        roof["achieved"] = traffic / scan_s / 1e9
        roof["achieved_basis"] = "measured DRAM bytes per launch / CUDA-event launch time"
    else:
        roof["achieved"] = alg_gbs
        roof["achieved_basis"] = "algorithmic stream bytes (no DRAM capture for this workload)"
    roof["frac"] = roof["achieved"] / peak
    return roof


class ClockSampler:
    """SM clock and clock-event (throttle) reasons polled through NVML every 2 ms while the
    timed region runs (read-only queries; no setting is changed)."""

    REASONS = [("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown")]

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.stop = threading.Event()
        self.nv = None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
        except Exception:
            self.nv = None
        return self

    def _poll(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((sm, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def __exit__(self, *a):
        self.stop.set()
        if self.nv:
            self.t.join(timeout=2)
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return None
        reasons = set()
        for _, rs in self.samples:
            for name, attr in self.REASONS:
                if rs & getattr(self.nv, attr, 0):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "NVML, 2 ms poll"}


# ------------------------------------------------------------------ reference arm
def run_reference(args, w, rank, world):
    """CPU restatement of the reference search path (oracle), all host threads."""
    if rank != 0:
        return
    import torch
    from oracle import oracle as O
    if not os.path.exists(cache_path(args.workload)):
        # the frozen index is built by the GPU build path in a process of its own: the timed
        # process maps no library of this repository
        subprocess.run([sys.executable, os.path.abspath(__file__), "--prepare-artifact",
                        "--workload", args.workload], check=True)
    art = load_artifact(args.workload)
    base, queries = make_data(w, "cuda" if torch.cuda.is_available() else "cpu")
    q = queries.cpu().numpy()
    del base
    oi = O.OracleIndex(art)
    cores = os.cpu_count() or 1
    # sample size: ~8 s of host work per step, measured on a first probe
    t0 = time.perf_counter()
    oi.search(q[:64], w["k"], w["nprobe"], nthreads=cores)
    per_q = (time.perf_counter() - t0) / 64
    sample = int(min(w["nq"], max(64, 8.0 / max(per_q, 1e-9))))
    for _ in range(args.warmup):
        oi.search(q[:min(sample, 64)], w["k"], w["nprobe"], nthreads=cores)
    times = []
    for s in range(args.steps):
        off = (s * sample) % max(w["nq"] - sample + 1, 1)
        t0 = time.perf_counter()
        oi.search(q[off:off + sample], w["k"], w["nprobe"], nthreads=cores)
        times.append(time.perf_counter() - t0)
    qps = sample * len(times) / sum(times)
    line = {
        "impl": "reference", "metric": "ivf_usq_search_qps", "value": qps, "unit": "queries/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "strong" if args.split else "weak",
        "vs_baseline": None, "dtype": "u8*i8->i32, f32 epilogue", "data": "synthetic",
        "config": config_block(args.workload, w, world, args.split),
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": cores, "kind": "port",
                         "sample": f"{sample} queries per step of the {w['nq']}-query batch, "
                                   "oracle restatement (AVX-512BW/VNNI semantics), OpenMP over queries"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(name, w, world, split=False):
    if world == 1:
        par = "1 GPU"
    elif split:
        par = (f"lists sharded over {world} GPUs; one batch split over the ranks for preparation, "
               "NCCL all-gather of the query state and of the shard top-k")
    else:
        par = (f"lists sharded over {world} GPUs; one batch per rank, NCCL all-gather of the "
               "query state, NCCL all-to-all of the shard top-k")
    return {"workload": f"IVF-USQ {w['nbits']}-bit {'IP' if w['metric'] else 'L2'}, "
                        f"base {w['n']}x{w['d']} Gaussian mixture ({w['comps']} comps, sigma {w['sigma']}"
                        f"{', normalised' if w['normalise'] else ''}), {w['nq']} queries, "
                        f"nlist {w['nlist']}, nprobe {w['nprobe']}, k {w['k']}, seed {w['seed']}",
            "name": name, "n": w["n"], "dim": w["d"], "nlist": w["nlist"], "nprobe": w["nprobe"],
            "k": w["k"], "nbits": w["nbits"], "query_batch": w["nq"],
            "global_batch": w["nq"] if (world == 1 or split) else w["nq"] * world,
            "parallelism": par,
            "l2_policy": "index larger than L2 (no flush needed)",
            "build": f"train on {train_rows(w)} sampled rows ({w.get('train_per_list', TRAIN_ROWS_PER_LIST)} "
                     f"per list): seeded k-means++ seeding, empty lists restarted, at most "
                     f"{w.get('kmeans_iters', KMEANS_ITERS)} iterations (shift < 1e-2 stops); "
                     f"every base row added"}


# ------------------------------------------------------------------ our arm
def run_ours(args, w, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqIndex

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    base, queries = make_data(w, dev)
    # rank 0 builds the index with the GPU build path (or loads the cached artifact);
    # the other ranks load what rank 0 wrote
    # (an index too large for the disk cache is built by every rank at once: the GPU build
    # is deterministic, so all ranks hold the same index)
    shared_cache = w["n"] <= (1 << 22)
    if rank == 0 or not shared_cache:
        art = get_artifact(args.workload, w, base, local_rank)
    if world > 1:
        dist.barrier()
        if rank != 0 and shared_cache:
            art = get_artifact(args.workload, w, base, local_rank)
    idx = IvfUsqIndex.from_artifact(art, device=local_rank)
    if args.no_recall:
        del base
        base = None
        torch.cuda.empty_cache()
    nq, k, nprobe = w["nq"], w["k"], w["nprobe"]
    # a stream of our own: device calls on it are stream-ordered (they return once enqueued)
    stream = torch.cuda.Stream(dev)
    out_ids = torch.empty(nq, k, dtype=torch.int64, device=dev)
    out_d = torch.empty(nq, k, dtype=torch.float32, device=dev)
    L = _lib.lib()
    launches = [0]
    split = world > 1 and args.split
    if world > 1:
        from hanns_b200.sharded import ShardedIvfUsq, SplitShardedIvfUsq
        # rank r searches its own batch (rank 0's is the single-GPU batch); with --split one
        # batch is shared by all ranks
        mine = queries if (split or rank == 0) else extra_queries(w, dev, rank)
        if split:
            sh = SplitShardedIvfUsq(idx, k, nprobe, nq)
        else:
            sh = ShardedIvfUsq(idx, k, nprobe, nq)
            sh.timing = True
        sh.scan_ms = []

    def run_steps(n):
        with torch.cuda.stream(stream):
            if world == 1:
                for _ in range(n):
                    idx.search_device(queries.data_ptr(), nq, k, nprobe, out_ids.data_ptr(),
                                      out_d.data_ptr(), 0, stream.cuda_stream)
                    launches[0] += idx.last_launches()
            elif split:
                for _ in range(n):
                    sh.split_search_device(mine.data_ptr(), out_ids, out_d, stream)
            else:
                sh.search_device([mine.data_ptr()] * n, [(out_ids, out_d)] * n, stream)

    run_steps(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        sh.launches = 0
    launches[0] = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0.record(stream)
        run_steps(args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = ev0.elapsed_time(ev1)
    # list-scan kernel time of the timed steps, from the library's stage events (each step is
    # one search call, or a prepare call and a scan call)
    calls = args.steps if world == 1 else 2 * args.steps
    st_sum, st_cnt, _ = idx.stage_ms_recent(calls)
    scan_ms = [float(st_sum[5]) / max(int(st_cnt[5]), 1)]
    # the list scan's kernels, each timed by CUDA events on the launching stream
    kt_sum, kt_cnt = idx.scan_kernel_ms_recent(calls)
    scan_kernels_ms = {name: float(kt_sum[i]) / max(int(kt_cnt[i]), 1)
                       for i, name in enumerate(IvfUsqIndex.SCAN_KERNELS)}
    rank_stages = None
    if world > 1:
        launches[0] = sh.launches
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        if not split:
            # per-rank stage medians of the timed batches (CUDA events), max and min over ranks
            mine_st = sh.stage_times(args.steps)
            every = [None] * world
            dist.all_gather_object(every, mine_st)
            rank_stages = {kk: {"max": max(e[kk] for e in every), "min": min(e[kk] for e in every),
                                "rank_of_max": int(np.argmax([e[kk] for e in every]))}
                           for kk in mine_st}
    job_nq = nq if (world == 1 or split) else nq * world
    value = job_nq * args.steps / (ms / 1e3)
    stages = idx.stage_ms().tolist()
    res_ids = out_ids.cpu().numpy()
    shard_parity = None
    if world > 1:
        # every rank's merged rows must equal a single-GPU search of the whole index
        full = IvfUsqIndex.from_artifact(art, device=local_rank)
        f_ids = torch.empty(nq, k, dtype=torch.int64, device=dev)
        f_d = torch.empty(nq, k, dtype=torch.float32, device=dev)
        full.search_device(mine.data_ptr(), nq, k, nprobe, f_ids.data_ptr(), f_d.data_ptr(), 0,
                           stream.cuda_stream)
        torch.cuda.synchronize()
        cnt = torch.tensor([nq, int((f_ids == out_ids).all(1).sum()),
                            int((f_d.view(torch.int32) == out_d.view(torch.int32)).all(1).sum())],
                           device=dev)
        if not split:
            dist.all_reduce(cnt)
        shard_parity = {"queries_checked": int(cnt[0]), "ids_equal_rows": int(cnt[1]),
                        "dists_bit_equal_rows": int(cnt[2])}
        full.close()

    # ---- e2e through the host-pointer API (pinned buffers)
    e2e = None
    if world == 1:
        hq = torch.empty(nq, w["d"], dtype=torch.float32).pin_memory()
        hq.copy_(queries.cpu())
        h_ids = torch.empty(nq, k, dtype=torch.int64).pin_memory()
        h_d = torch.empty(nq, k, dtype=torch.float32).pin_memory()
        f32p, i64p = _lib.f32p, _lib.i64p
        import ctypes as C

        def e2e_step():
            rc = L.hanns_gpu_ivf_usq_search(idx._h, C.cast(hq.data_ptr(), f32p), nq, k, nprobe, 0, None,
                                            0, 0, None, C.cast(h_ids.data_ptr(), i64p),
                                            C.cast(h_d.data_ptr(), f32p), None)
            assert rc == 0, _lib.last_error()

        for _ in range(max(1, args.warmup)):
            e2e_step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        el = time.perf_counter() - t0
        e2e = {"value": nq * args.steps / el, "unit": "queries/s",
               "h2d_bytes_per_step": nq * w["d"] * 4, "d2h_bytes_per_step": nq * k * 12,
               "path": "hanns_gpu_ivf_usq_search (host pointers, pinned)"}
        assert np.array_equal(h_ids.numpy(), res_ids), "e2e and device paths disagree"
    elif split:
        # every rank holds the batch in pinned host memory and copies its share in; rank 0
        # copies the merged rows out
        per = nq // world
        hq = torch.empty(nq, w["d"], dtype=torch.float32).pin_memory()
        hq.copy_(queries.cpu())
        h_ids = torch.empty(nq, k, dtype=torch.int64).pin_memory()
        h_d = torch.empty(nq, k, dtype=torch.float32).pin_memory()
        qdev = torch.empty(nq, w["d"], dtype=torch.float32, device=dev)

        def e2e_step():
            qdev[rank * per:(rank + 1) * per].copy_(hq[rank * per:(rank + 1) * per], non_blocking=True)
            sh.split_search_device(qdev.data_ptr(), out_ids, out_d, stream)
            if rank == 0:
                h_ids.copy_(out_ids, non_blocking=True)
                h_d.copy_(out_d, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

        for _ in range(max(1, args.warmup)):
            e2e_step()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        el = torch.tensor([time.perf_counter() - t0], device=dev)
        dist.all_reduce(el, op=dist.ReduceOp.MAX)
        e2e = {"value": nq * args.steps / float(el.item()), "unit": "queries/s",
               "h2d_bytes_per_step": nq * w["d"] * 4, "d2h_bytes_per_step": nq * k * 12,
               "path": "per rank: pinned H2D of its 1/N of the batch, query preparation, NCCL "
                       "all-gather of the query state, scan of its lists, NCCL all-gather of the "
                       "shard top-k, merge; rank 0 D2H (max over ranks)"}
        if rank == 0:
            assert np.array_equal(h_ids.numpy(), res_ids), "e2e and device paths disagree"
    else:
        # every rank's batch from pinned host memory through ShardedIvfUsq.search_host
        hq = torch.empty(nq, w["d"], dtype=torch.float32).pin_memory()
        hq.copy_(mine.cpu())
        h_ids = torch.empty(nq, k, dtype=torch.int64).pin_memory()
        h_d = torch.empty(nq, k, dtype=torch.float32).pin_memory()
        sh.search_host([hq] * max(1, args.warmup), [h_ids] * max(1, args.warmup),
                       [h_d] * max(1, args.warmup))
        dist.barrier()
        t0 = time.perf_counter()
        sh.search_host([hq] * args.steps, [h_ids] * args.steps, [h_d] * args.steps)
        el = torch.tensor([time.perf_counter() - t0], device=dev)
        dist.all_reduce(el, op=dist.ReduceOp.MAX)
        e2e = {"value": nq * world * args.steps / float(el.item()), "unit": "queries/s",
               "h2d_bytes_per_step": nq * world * w["d"] * 4,
               "d2h_bytes_per_step": nq * world * k * 12,
               "path": "ShardedIvfUsq.search_host on every rank: pinned H2D of its batch (copy "
                       "stream, one batch ahead), preparation, NCCL all-gather of the query state, "
                       "scan of its lists, NCCL all-to-all of the shard top-k, merge, D2H of its "
                       "rows (max over ranks)"}
        assert np.array_equal(h_ids.numpy(), res_ids), "e2e and device paths disagree"

    if rank != 0:
        return
    # ---- roofline of the list-scan kernel (rank 0's launch)
    if world > 1 and not split:
        allq = torch.cat([queries] + [extra_queries(w, dev, r) for r in range(1, world)])
    else:
        allq = queries
    probes = idx.debug_query(allq.cpu().numpy(), nprobe)["probes"]
    del allq
    stats = index_stats(art, probes, k, w["nbits"])
    art_local = art if world == 1 else idx.export_artifact()
    if world > 1:
        # the shard's lists: lists it does not own are empty in its export
        own = np.diff(art_local["list_offsets"]) > 0
        probes = probes[own[probes]]
    alg = scan_bytes(art_local, probes, k, w["nbits"])
    if os.environ.get("HANNS_GPU_SCAN") == "simt":
        roof = scan_roofline(args.workload, alg, scan_kernels_ms["scan_simt"] / 1e3, world)
    else:
        roof = scan_roofline_tc(args.workload, alg, scan_tc_ops(art_local, probes, k, w["nbits"]),
                                scan_kernels_ms["scan_tc"] / 1e3, world)
    roof["scan_stage_ms"] = statistics.median(scan_ms)
    roof["scan_kernels_ms"] = scan_kernels_ms

    # ---- recall and parity sample
    rec = None
    if base is not None:
        gt = exact_topk(base, queries, k, w["metric"])
        rec = float(np.mean([len(set(gt[i]) & set(res_ids[i])) / k for i in range(nq)]))
        del base
    cpu = None
    parity = None
    if world == 1 and not args.no_cpu:
        from oracle import oracle as O
        oi = O.OracleIndex(art)
        cores = os.cpu_count() or 1
        qn = queries.cpu().numpy()
        t0 = time.perf_counter()
        oi.search(qn[:64], k, nprobe, nthreads=cores)
        per_q = (time.perf_counter() - t0) / 64
        sample = int(min(nq, max(64, 8.0 / max(per_q, 1e-9))))
        t0 = time.perf_counter()
        o_ids, o_d, _ = oi.search(qn[:sample], k, nprobe, nthreads=cores)
        el = time.perf_counter() - t0
        cpu = {"value": sample / el, "unit": "queries/s", "cores": cores, "kind": "port",
               "sample": f"first {sample} of the {nq} queries, oracle restatement, OpenMP over queries"}
        gd = out_d.cpu().numpy()[:sample]
        parity = {"queries_checked": sample,
                  "ids_equal_rows": int((o_ids == res_ids[:sample]).all(1).sum()),
                  "dists_bit_equal_rows": int((o_d.view(np.uint32) == gd.view(np.uint32)).all(1).sum())}
    line = {
        "metric": "ivf_usq_search_qps", "value": value, "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "strong" if split else "weak", "vs_baseline": None,
        "dtype": "u8*i8->i32, f32 epilogue", "data": "synthetic",
        "config": config_block(args.workload, w, world, split),
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": launches[0], "clocks": clk.summary(),
        "recall_at_k": rec,
        "recall_note": f"exact fp32 ground truth over all {w['n']} rows; the index's k-means saw "
                       f"{train_rows(w)} sampled rows (the reference trains on every row)",
        "index_stats": stats,
        "parity_vs_oracle": parity, "parity_vs_single_gpu": shard_parity,
        "stage_ms_last_step": dict(zip(IvfUsqIndex.STAGES, stages)),
        "rank_stage_ms": rank_stages,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="B", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline / parity sample")
    ap.add_argument("--no-recall", action="store_true", help="skip exact ground truth (frees the base early)")
    ap.add_argument("--prepare-artifact", action="store_true",
                    help="build and cache the workload's frozen index, then exit")
    ap.add_argument("--scale", type=int, default=1,
                    help="divide the workload's rows, lists and queries by this factor (list sizes "
                         "and queries per list unchanged): the small case of the same kernels for "
                         "ncu captures; not a bench line")
    ap.add_argument("--split", action="store_true",
                    help="N > 1: one batch split over the ranks (strong scaling) instead of one "
                         "batch per rank (weak scaling)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = dict(WORKLOADS[args.workload])
    if args.scale > 1:
        for key in ("n", "nlist", "nq"):
            w[key] //= args.scale
        args.workload = f"{args.workload}_scale{args.scale}"
        WORKLOADS[args.workload] = w
    if args.prepare_artifact:
        base, _ = make_data(w, "cuda")
        get_artifact(args.workload, w, base, 0, cache=True)
        return
    if args.impl == "reference":
        run_reference(args, w, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, w, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
