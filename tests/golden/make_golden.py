"""Generates the committed golden fixtures under tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

Each fixture holds a frozen IVF-USQ artifact (list order), a query batch and the
oracle's outputs for it (reference semantics, AVX-512 mode): per-query ids and
distances, coarse probes, query state (q_rot, q_i8, LUT) and, for bitset cases,
the filtered outputs.  The GPU tests compare the CUDA path against these bit for
bit, without needing the oracle at run time.

Inputs are seeded synthetic Gaussian mixtures (the reference's datasets are not
available); the generator is numpy's PCG64 with the seed stored in the file.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402


def mixture(rng, n, d, comps, sigma, normalise):
    centres = rng.normal(size=(comps, d)).astype(np.float32)
    lab = rng.integers(0, comps, n)
    x = (centres[lab] + sigma * rng.normal(size=(n, d))).astype(np.float32)
    if normalise:
        x /= np.linalg.norm(x, axis=1, keepdims=True).astype(np.float32)
    return x.astype(np.float32), centres


CASES = [
    # name, n, d, comps, sigma, normalise, nlist, nbits, metric, k, nprobe, nq, seed, dup
    ("l2_4bit_d128", 3000, 128, 16, 0.3, False, 8, 4, O.METRIC_L2, 10, 3, 48, 42, 0),
    ("ip_8bit_d96", 2400, 96, 16, 0.5, True, 4, 8, O.METRIC_IP, 10, 2, 48, 7, 0),
    ("ip_4bit_k100", 2000, 192, 8, 0.5, True, 8, 4, O.METRIC_IP, 100, 4, 24, 11, 0),
    ("l2_4bit_dups_d64", 3000, 64, 6, 0.3, False, 6, 4, O.METRIC_L2, 20, 3, 40, 5, 1),
    ("l2_8bit_small_lists", 300, 65, 4, 0.4, False, 24, 8, O.METRIC_L2, 7, 24, 16, 3, 0),
]


def make_case(name, n, d, comps, sigma, normalise, nlist, nbits, metric, k, nprobe, nq, seed, dup):
    rng = np.random.default_rng(seed)
    x, _ = mixture(rng, n, d, comps, sigma, normalise)
    if dup:  # exact duplicates -> equal codes -> equal distances (tie order matters)
        x[1::3] = x[0::3][: x[1::3].shape[0]]
    q, _ = mixture(rng, nq, d, comps, sigma, normalise)
    q[:4] = x[:4]  # self queries
    art = O.build_artifact(x, nlist, nbits, metric, rotation_seed=seed, kmeans_iters=8,
                           kmeans_seed=seed)
    idx = O.OracleIndex(art)
    ids, dists, counts, probes = idx.search(q, k, nprobe, want_probes=True)
    # per-query bitsets: 3 bitsets, 20% density, queries cycle through -1, 0, 1, 2
    blen = n + 5
    words = (blen + 63) // 64
    bits = np.zeros((3, words), np.uint64)
    for b in range(3):
        m = rng.random(blen) < 0.2
        for i in np.nonzero(m)[0]:
            bits[b, i >> 6] |= np.uint64(1) << np.uint64(i & 63)
    qb = (np.arange(nq) % 4 - 1).astype(np.int32)
    f_ids, f_dists, f_counts = idx.search(q, k, nprobe, filter_mode=O.FILTER_FUSED, bitsets=bits,
                                          bitset_len=blen, query_bitset=qb)
    p_ids, p_dists, p_counts = idx.search(q, k, nprobe, filter_mode=O.FILTER_POST, bitsets=bits,
                                          bitset_len=blen, query_bitset=qb)
    st = [O.query_state(art, q[i]) for i in range(nq)]
    out = {key: art[key] for key in ("centroids", "rotation", "rotated_centroid", "list_offsets",
                                     "ids", "norms", "norms_sq", "vmaxs", "quant_qualities", "codes",
                                     "sign_bits")}
    out.update(
        meta=np.array([d, art["padded_dim"], nbits, nlist, metric, k, nprobe, seed], np.int64),
        queries=q, exp_ids=ids, exp_dists=dists, exp_probes=probes,
        exp_q_rot=np.stack([s["q_rot"] for s in st]), exp_q_i8=np.stack([s["q_i8"] for s in st]),
        exp_lut=np.stack([s["lut"] for s in st]),
        exp_scalars=np.array([[s["q_scale"], s["centroid_score"], s["q_norm_sq"], s["lut_scale"]]
                              for s in st], np.float32),
        exp_q_i8_sum=np.array([s["q_i8_sum"] for s in st], np.int32),
        bitsets=bits, bitset_len=np.array([blen], np.int64), query_bitset=qb,
        exp_fused_ids=f_ids, exp_fused_dists=f_dists,
        exp_post_ids=p_ids, exp_post_dists=p_dists, exp_post_counts=p_counts,
    )
    idx.close()
    return out


def load(path: str) -> tuple[dict, dict]:
    """Returns (artifact dict, fixture dict)."""
    z = dict(np.load(path))
    d, D, nbits, nlist, metric, k, nprobe, seed = (int(v) for v in z["meta"])
    art = dict(dim=d, padded_dim=D, nbits=nbits, nlist=nlist, metric=metric)
    for key in ("centroids", "rotation", "rotated_centroid", "list_offsets", "ids", "norms",
                "norms_sq", "vmaxs", "quant_qualities", "codes", "sign_bits"):
        art[key] = z[key]
    z.update(k=k, nprobe=nprobe, seed=seed)
    return art, z


def main():
    for c in CASES:
        out = make_case(*c)
        path = os.path.join(HERE, f"{c[0]}.npz")
        np.savez_compressed(path, **out)
        print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
