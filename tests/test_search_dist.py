"""Distributed host logic of the template search on CPU ranks (gloo, world
size 2): sharding, global template indices, the single packed-key MAX
all-reduce, tie-breaking across ranks, and a rank failure that must end the
other rank with an error instead of a hang."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
from zipfft_b200.search import shard_range  # noqa: E402


def test_shard_range_partitions():
    for n in (0, 1, 7, 8, 8192, 8193):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(n=6, h=5, w=4, H=32, W=32, dup=None):
    g = torch.Generator().manual_seed(0)
    img = torch.randn((H, W), generator=g)
    tm = torch.randn((n, h, w), generator=g)
    if dup is not None:  # an identical template in each shard: a tie everywhere
        tm[dup[1]] = tm[dup[0]]
    from oracle import xcorr_oracle as O

    spec = torch.from_numpy(O.image_spectrum_T(img.numpy()))
    return tm, spec


def _worker(rank, world, port, dup, fail_rank, out_dir):
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    from tests.search_cpu_ops import CPU_OPS
    from zipfft_b200.search import template_search

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the reduction")
        tm, spec = _inputs(dup=dup)
        mx, am, sm, sq = template_search(tm, spec, 32, 32, batch_size=2, full=True,
                                         device=torch.device("cpu"), ops=CPU_OPS, stats=True)
        np.save(os.path.join(out_dir, f"max{rank}.npy"), mx.numpy())
        np.save(os.path.join(out_dir, f"arg{rank}.npy"), am.numpy())
        np.save(os.path.join(out_dir, f"sum{rank}.npy"), sm.numpy())
        np.save(os.path.join(out_dir, f"sumsq{rank}.npy"), sq.numpy())
    finally:
        dist.destroy_process_group()


def _reference(dup=None):
    from oracle import xcorr_oracle as O

    tm, spec = _inputs(dup=dup)
    res = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), 32, 32, True, True).astype(np.float32)
    return res.max(axis=0), res.argmax(axis=0)


@pytest.mark.parametrize("dup", [None, (1, 4)])
def test_two_rank_search_matches_single_process(tmp_path, dup):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, dup, -1, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ref_max, ref_arg = _reference(dup)
    from oracle import xcorr_oracle as O

    tm, spec = _inputs(dup=dup)
    res = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), 32, 32, True, True)
    for r in range(2):
        mx = np.load(tmp_path / f"max{r}.npy")
        am = np.load(tmp_path / f"arg{r}.npy")
        assert np.array_equal(mx, ref_max)
        assert np.array_equal(am, ref_arg)  # ties (dup) keep the lower index, 1 not 4
        # per-batch float32 partial sums added in float64, then the SUM all-reduce
        assert O.rel_l2(res.sum(axis=0), np.load(tmp_path / f"sum{r}.npy")) < 1e-6
        assert O.rel_l2((res ** 2).sum(axis=0), np.load(tmp_path / f"sumsq{r}.npy")) < 1e-6
    assert np.array_equal(np.load(tmp_path / "sum0.npy"), np.load(tmp_path / "sum1.npy"))
    if dup is not None:
        assert not np.any(np.load(tmp_path / "arg0.npy") == dup[1])


def test_rank_failure_ends_the_other_rank_with_an_error(tmp_path):
    """Rank 1 fails before the collective; rank 0 must not hang: its
    all-reduce ends with an error within the process-group timeout."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, None, 1, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert procs[1].exitcode != 0
    assert procs[0].exitcode != 0
    assert not (tmp_path / "max0.npy").exists()


def _shard_worker(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    from tests.search_cpu_ops import CPU_OPS
    from zipfft_b200.search import shard_range, template_search

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        tm, spec = _inputs(n=7)
        lo, hi = (0, 4) if rank == 0 else (4, 7)  # uneven shards, each rank holds only its own
        mx, am = template_search(tm[lo:hi].clone(), spec, 32, 32, batch_size=2, full=True,
                                 device=torch.device("cpu"), ops=CPU_OPS, shard_base=lo)
        np.save(os.path.join(out_dir, f"max{rank}.npy"), mx.numpy())
        np.save(os.path.join(out_dir, f"arg{rank}.npy"), am.numpy())
    finally:
        dist.destroy_process_group()


def test_two_rank_search_with_local_shards(tmp_path):
    """Each rank passes only its own templates (shard_base = their first
    global index); the combined maps equal the single-process search."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    from oracle import xcorr_oracle as O

    tm, spec = _inputs(n=7)
    res = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), 32, 32, True, True).astype(np.float32)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"max{r}.npy"), res.max(axis=0))
        assert np.array_equal(np.load(tmp_path / f"arg{r}.npy"), res.argmax(axis=0))
