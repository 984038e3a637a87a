"""Per-batch checkpoint and resume of the template search (host logic, CPU
stand-in ops): a search stopped after any checkpoint and resumed from it gives
exactly the uninterrupted result, on one process and on two gloo ranks whose
job is preempted mid-shard."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
from tests.search_cpu_ops import CPU_OPS  # noqa: E402
from zipfft_b200.search import SearchCheckpoint, template_search  # noqa: E402

H = W = 32


def _inputs(n=9, h=5, w=4):
    from oracle import xcorr_oracle as O

    g = torch.Generator().manual_seed(7)
    img = torch.randn((H, W), generator=g)
    tm = torch.randn((n, h, w), generator=g)
    return tm, torch.from_numpy(O.image_spectrum_T(img.numpy()))


class Preempted(Exception):
    pass


def _search(tm, spec, **kw):
    return template_search(tm, spec, H, W, batch_size=2, full=True, device=torch.device("cpu"),
                           ops=CPU_OPS, **kw)


@pytest.mark.parametrize("stop_after", [1, 2, 4])
def test_resume_after_preemption_matches_uninterrupted(tmp_path, stop_after):
    tm, spec = _inputs()
    ref_max, ref_arg = _search(tm, spec)
    seen = []

    def save_then_stop(cp):
        path = str(tmp_path / f"cp{len(seen)}.pt")
        cp.save(path)
        seen.append(path)
        if len(seen) == stop_after:
            raise Preempted

    with pytest.raises(Preempted):
        _search(tm, spec, checkpoint_every=1, on_checkpoint=save_then_stop)
    cp = SearchCheckpoint.load(seen[-1])
    assert cp.next_index == 2 * stop_after and cp.n_templates == 9
    mx, am = _search(tm, spec, resume=cp)
    assert torch.equal(mx, ref_max) and torch.equal(am, ref_arg)


def test_checkpoint_cadence_and_last_batch():
    tm, spec = _inputs()
    got = []
    _search(tm, spec, checkpoint_every=2, on_checkpoint=got.append)
    # batches end at 2, 4, 6, 8, 9: every second one that leaves work
    assert [c.next_index for c in got] == [4, 8]
    # a snapshot is a copy, not a view of the live maps
    assert not torch.equal(got[0].max_map, got[1].max_map)


def test_resume_rejects_another_search():
    tm, spec = _inputs()
    got = []
    _search(tm, spec, checkpoint_every=1, on_checkpoint=got.append)
    cp = got[0]
    with pytest.raises(ValueError, match="different search"):
        _search(tm[:8], spec, resume=cp)
    bad = SearchCheckpoint(cp.n_templates, 0, 1, 12, cp.max_map, cp.arg_map)
    with pytest.raises(ValueError, match="outside"):
        _search(tm, spec, resume=bad)
    small = SearchCheckpoint(cp.n_templates, 0, 1, 2, cp.max_map[:4], cp.arg_map[:4])
    with pytest.raises(ValueError, match="maps are"):
        _search(tm, spec, resume=small)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir, phase):
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        tm, spec = _inputs()
        path = os.path.join(out_dir, f"rank{rank}.pt")
        if phase == 0:
            def save_then_stop(cp):
                cp.save(path)
                raise Preempted  # the whole job stops before its reduction

            _search(tm, spec, checkpoint_every=1, on_checkpoint=save_then_stop)
        else:
            mx, am = _search(tm, spec, resume=SearchCheckpoint.load(path))
            np.save(os.path.join(out_dir, f"max{rank}.npy"), mx.numpy())
            np.save(os.path.join(out_dir, f"arg{rank}.npy"), am.numpy())
    finally:
        dist.destroy_process_group()


def test_two_rank_search_resumes_from_per_rank_checkpoints(tmp_path):
    ctx = mp.get_context("spawn")
    for phase in (0, 1):
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), phase))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        assert all(p.exitcode is not None for p in procs), "a rank hung"
        codes = [p.exitcode for p in procs]
        assert (all(c != 0 for c in codes) if phase == 0 else all(c == 0 for c in codes)), codes
    tm, spec = _inputs()
    ref_max, ref_arg = _search(tm, spec)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"max{r}.npy"), ref_max.numpy())
        assert np.array_equal(np.load(tmp_path / f"arg{r}.npy"), ref_arg.numpy())


def test_stats_search_resumes_with_its_sums(tmp_path):
    """stats=True: checkpoints carry the sum maps; a resumed search equals the
    uninterrupted one, and a checkpoint without sums is refused."""
    tm, spec = _inputs()
    ref = _search(tm, spec, stats=True)
    got = []

    def save_then_stop(cp):
        got.append(cp)
        raise Preempted

    with pytest.raises(Preempted):
        _search(tm, spec, stats=True, checkpoint_every=2, on_checkpoint=save_then_stop)
    path = str(tmp_path / "cp.pt")
    got[0].save(path)
    cp = SearchCheckpoint.load(path)
    assert cp.sum_map is not None and cp.next_index == 4
    out = _search(tm, spec, stats=True, resume=cp)
    for a, b in zip(out, ref):
        assert torch.equal(a, b)
    plain = []
    _search(tm, spec, checkpoint_every=2, on_checkpoint=plain.append)
    with pytest.raises(ValueError, match="no sum maps"):
        _search(tm, spec, stats=True, resume=plain[0])


def test_batch_bounds_ramp_covers_the_shard_in_order():
    """Host-resident templates: the first batches ramp up from the launch
    group size, doubling up to the batch size; the ranges tile the shard."""
    from zipfft_b200.search import SEARCH_GROUP, batch_bounds

    for start, stop, nb in [(0, 1024, 256), (5, 1000, 256), (0, 7, 256), (3, 40, 8), (0, 0, 4)]:
        plain = list(batch_bounds(start, stop, nb))
        ramp = list(batch_bounds(start, stop, nb, ramp=True))
        for bounds in (plain, ramp):
            if not bounds:
                assert start == stop
                continue
            assert [b[0] for b in bounds] == [start] + [b[1] for b in bounds[:-1]]
            assert bounds[-1][1] == stop
            assert all(0 < b1 - b0 <= nb for b0, b1 in bounds)
        assert all(b1 - b0 == nb for b0, b1 in plain[:-1])
        if ramp:
            sizes = [b1 - b0 for b0, b1 in ramp]
            assert sizes[0] == min(nb, SEARCH_GROUP, stop - start)
            assert all(b <= min(2 * a, nb) for a, b in zip(sizes, sizes[1:]))
    assert [b1 - b0 for b0, b1 in batch_bounds(0, 1024, 256, ramp=True)] == \
        [16, 32, 64, 128, 256, 256, 256, 16]
