"""Host-side multi-GPU logic: item partitions and the gather of per-rank results.

The data path has no exchange step (items are independent), so what needs
testing is the partition (every item exactly once, balanced by attention cost)
and the host gather, here over world-size-2 ``gloo`` process groups on the CPU,
including a rank that fails before the gather.
"""

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from tests.conftest import ROOT  # noqa: E402


def _sharding():
    import importlib.util

    spec = importlib.util.spec_from_file_location("omni_sharding", ROOT / "omni-tokenizer_b200" / "sharding.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


S = _sharding()


@pytest.mark.parametrize("n,world", [(0, 1), (7, 1), (7, 2), (512, 8), (3, 4), (1536, 3)])
def test_even_split_covers_every_item_once(n, world):
    parts = S.even_split(n, world)
    assert len(parts) == world
    flat = [i for p in parts for i in p]
    assert flat == list(range(n))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_balanced_bins_for_varlen_batch(world):
    # 64 segments with lengths U{100..1500}.
    lengths = np.random.default_rng(1003).integers(100, 1501, size=64)
    bins = S.balanced_bins(lengths, world)
    assert sorted(i for b in bins for i in b) == list(range(64))
    assert all(b == sorted(b) for b in bins)
    loads = S.bin_loads(lengths, bins)
    total, biggest = sum(loads), max(float(n) ** 2 for n in lengths)
    # Greedy LPT: no bin exceeds the mean by more than one item.
    assert max(loads) <= total / world + biggest
    if world > 1:
        assert max(loads) / (total / world) < 1.10
    assert S.balanced_bins(lengths, world) == bins  # deterministic


def test_balanced_bins_rejects_bad_world():
    with pytest.raises(ValueError):
        S.balanced_bins([1, 2], 0)
    with pytest.raises(ValueError):
        S.even_split(3, 0)


def test_gather_single_process():
    out = S.gather_results([2, 0, 1], ["c", "a", "b"], 3)
    assert out == ["a", "b", "c"]
    with pytest.raises(ValueError):
        S.gather_results([0, 1], ["a"], 2)
    with pytest.raises(ValueError):
        S.gather_results([0], ["a"], 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, queue):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        lengths = np.random.default_rng(7).integers(100, 1501, size=37)
        bins = S.balanced_bins(lengths, world)
        mine = bins[rank]
        # Stand-in for the per-item GPU result: a value only that item determines.
        results = [int(lengths[i]) * 3 + i for i in mine]
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the gather")
        out = S.gather_results(mine, results, len(lengths))
        queue.put((rank, "ok", out == [int(n) * 3 + i for i, n in enumerate(lengths)]))
    except Exception as exc:  # reported to the parent, never swallowed
        queue.put((rank, "error", type(exc).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=120)
        got[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return got


def test_gather_over_gloo_world_size_2():
    got = _run("ok")
    assert got == {0: ("ok", True), 1: ("ok", True)}


def test_rank_failure_surfaces_as_error_on_the_other_rank():
    got = _run("fail")
    assert got[1] == ("error", "RuntimeError")
    assert got[0][0] == "error"  # the surviving rank's gather fails (peer gone / timeout)
