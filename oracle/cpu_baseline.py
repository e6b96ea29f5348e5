"""The oracle run on all host cores -- the CPU baseline `bench.py` reports
(TEST / MEASUREMENT INFRASTRUCTURE ONLY; never part of the product path).

The reference cannot run here (MLX is absent and its VQ runtime is not in
the repository), so the baseline is this CPU restatement of the reference
semantics (`moe_ref`): router, per-expert dequantise-then-matmul, combine
and shared expert, with the experts spread over a thread pool (numpy
releases the GIL in the dequantisation and the matmuls). Every timed call is
a whole block call: all routed experts, the combine and the shared expert.

Threads: one pool worker per host core, and the BLAS library held to one
thread while the pool runs (`threadpoolctl`), so that the workers do not
each start a BLAS thread per core (cores x cores threads).
"""
from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor
from contextlib import contextmanager

import numpy as np

from . import moe_ref as R


def threads() -> int:
    return max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity")
               else (os.cpu_count() or 1))


@contextmanager
def pool_of(n: int):
    """A pool of n workers with BLAS held to one thread each."""
    from threadpoolctl import threadpool_limits
    with threadpool_limits(limits=1), ThreadPoolExecutor(n) as pool:
        yield pool


def _expert_rows(x, inds, p, vq, e):
    """SwitchGLU rows of expert e: (pair ids, [n, H] bf16 outputs)."""
    T, k = inds.shape
    pairs = np.nonzero(inds.reshape(-1) == e)[0]
    rows = x[pairs // k]
    xin = R.f16_sat(rows) if vq else rows
    g = R.linear(xin, p["gate"][e])
    u = R.linear(xin, p["up"][e])
    a = R.swiglu(u, g)
    ain = R.f16_sat(a) if vq else a
    return pairs, R.linear(ain, p["down"][e])


def _shared(x, p):
    return R.shared_expert(x, p["shared_expert_gate"], p["shared_up"], p["shared_gate"],
                           p["shared_down"])


def block(x, p, k, vq, pool: ThreadPoolExecutor):
    """`moe_ref.sparse_moe_block` with the routed experts (and the shared
    expert, as one more task) on `pool`."""
    inds, scores, _ = R.router(x, p["router"], k)
    routed = np.unique(inds)
    shared = pool.submit(_shared, x, p) if "shared_gate" in p else None
    parts = list(pool.map(lambda e: _expert_rows(x, inds, p, vq, int(e)), routed))
    T = x.shape[0]
    y = np.zeros((T * k, p["down"].shape[1]), np.float32)
    for pairs, rows in parts:
        y[pairs] = rows
    out = R.combine(y.reshape(T, k, -1), scores)
    if shared is not None:
        out = R.bf16(out.astype(np.float64) + shared.result())
    return out


def time_block(x, p, k, vq, n_threads=None, repeats=1):
    """(seconds per full block call, threads) on the host cores."""
    n = n_threads or threads()
    with pool_of(n) as pool:
        t0 = time.perf_counter()
        for _ in range(repeats):
            block(x, p, k, vq, pool)
        return (time.perf_counter() - t0) / repeats, n
