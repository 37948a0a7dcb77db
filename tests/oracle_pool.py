"""Run the CPU oracle over many sequences at once (test helper).

The oracle's work per sequence is numpy matrix products and element-wise ops,
which release the GIL, so a thread pool with single-threaded BLAS runs one
sequence per host core. No process is forked (nothing here touches the GPU).
"""
import os
from concurrent.futures import ThreadPoolExecutor

from threadpoolctl import threadpool_limits


def oracle_map(fn, items, workers=None):
    """[fn(x) for x in items], computed in parallel, in order."""
    items = list(items)
    workers = workers or max(1, min(len(items), os.cpu_count() or 1))
    with threadpool_limits(limits=1):
        with ThreadPoolExecutor(max_workers=workers) as ex:
            return list(ex.map(fn, items))
