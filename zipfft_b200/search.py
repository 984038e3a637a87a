"""Multi-GPU 2D template matching: per-pixel maximum and argmax of the
cross-correlation over a large template set.

One process per GPU (torch.distributed, NCCL).  The image spectrum is
replicated; the templates are split into contiguous shards, one per rank;
every rank streams its shard through `padded_rconv2d.corr_max` in batches
(templates copied from host memory on a side stream, double-buffered), and
the per-rank maps are combined with a single all-reduce (MAX) of packed
64-bit keys (order-preserving float bits high, inverted template index low,
so ties keep the lowest index).  No data moves between GPUs before that one
reduction.  The reference has no multi-GPU code; this is the search its
README motivates (2DTM), with the template set as the sharded dimension.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import torch

from . import _lib


def shard_range(n_templates: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous shard [lo, hi) of template indices for `rank`."""
    base, extra = divmod(n_templates, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


@dataclass
class SearchOps:
    """The per-GPU operations of the search (the CUDA library by default).

    corr_max(batch (n, h, w), workspace, conv_data, max_map, arg_map, H, W,
             template_index_base, reset, sum_map=None, sumsq_map=None) folds n
    templates into the maps (and into the float32 sum / sum-of-squares maps if
    given).  reset: 0 folds into every map, RESET_ALL lets the batch's first
    template overwrite every map, RESET_SUMS only the sum maps (the maximum
    keeps running: each batch then yields float32 partial sums)."""

    corr_max: Callable
    pack: Callable       # (max_map, arg_map) -> int64 keys
    unpack: Callable     # (keys, max_map, arg_map) -> None (in place)
    workspace: Callable  # (H, W, h, device) -> workspace tensor


RESET_ALL = 1   # the batch's first template overwrites every map
RESET_SUMS = 2  # ... overwrites the sum maps only


# Templates per launch of the search's kernels: the workspace holds this many
# intermediate slices (1.07 GB at 4096^2), so the inverse row pass folds 16
# templates into each row group of the maps while those map rows stay in L2,
# and the column pass reads each spectrum column from DRAM once per 16.
SEARCH_GROUP = 16


def search_workspace_elems(H: int, W: int, h: int, group: int = SEARCH_GROUP) -> int:
    """complex64 elements of a workspace of `group` intermediate slices (the
    library then runs `group` templates through each kernel per launch)."""
    del h  # the slices hold each template's row spectra too
    return group * (_lib.load().zfft_workspace_bytes(H, W) // 8)


def batch_bounds(start: int, stop: int, nb: int, ramp: bool = False):
    """The [b0, b1) template ranges of a shard, batches of nb.  ramp: the
    first batches grow from SEARCH_GROUP templates, doubling up to nb, so
    that the first copy from host memory is small and each later copy
    overlaps the computation of the batch before it (with eight ranks
    sharing the host's copy bandwidth, a first batch of 256 templates of
    384^2 took 6.6 ms to arrive, against 0.4 ms for 16)."""
    size = min(nb, SEARCH_GROUP) if ramp else nb
    b0 = start
    while b0 < stop:
        b1 = min(b0 + size, stop)
        yield b0, b1
        b0 = b1
        size = min(2 * size, nb)


def _cuda_workspace(H: int, W: int, h: int, device) -> torch.Tensor:
    return torch.empty(search_workspace_elems(H, W, h), dtype=torch.complex64, device=device)


def _cuda_corr_max(batch, workspace, conv_data, max_map, arg_map, H, W, template_index_base,
                   reset, sum_map=None, sumsq_map=None) -> None:
    n, h, w = batch.shape
    oy, ox = max_map.shape
    dev = batch.device.index
    stream = torch.cuda.current_stream(dev).cuda_stream
    lib = _lib.load()
    if sum_map is not None:
        # Maximum, argmax and sum of squares per template; the batch's sum map
        # is the correlation map of its summed template (correlation is
        # linear): one more correlation per batch instead of a sum map read
        # and written per template.
        st = lib.zfft_padded_real_corr_2d_max_stats(
            batch.data_ptr(), n, h, w, workspace.data_ptr(), workspace.numel() * 8,
            conv_data.data_ptr(), max_map.data_ptr(), arg_map.data_ptr(), None,
            sumsq_map.data_ptr(), oy, ox, H, W, int(template_index_base), int(reset), dev,
            stream)
        _lib.check(st)
        summed = batch.sum(dim=0, keepdim=True, dtype=torch.float64).to(torch.float32)
        fresh = int(reset) in (RESET_ALL, RESET_SUMS)
        dst = sum_map if fresh else torch.empty_like(sum_map)
        st = lib.zfft_padded_real_corr_2d(
            summed.data_ptr(), 1, h, w, workspace.data_ptr(), workspace.numel() * 8,
            conv_data.data_ptr(), dst.data_ptr(), oy, ox, H, W, dev, stream)
        _lib.check(st)
        if not fresh:
            sum_map += dst
        return
    else:
        st = lib.zfft_padded_real_corr_2d_max(
            batch.data_ptr(), n, h, w, workspace.data_ptr(), workspace.numel() * 8,
            conv_data.data_ptr(), max_map.data_ptr(), arg_map.data_ptr(), oy, ox, H, W,
            int(template_index_base), 1 if int(reset) == RESET_ALL else 0, dev, stream)
    _lib.check(st)


def _cuda_pack(max_map: torch.Tensor, arg_map: torch.Tensor) -> torch.Tensor:
    keys = torch.empty(max_map.shape, dtype=torch.int64, device=max_map.device)
    dev = max_map.device.index
    _lib.check(_lib.load().zfft_pack_max_arg(max_map.data_ptr(), arg_map.data_ptr(),
                                             keys.data_ptr(), max_map.numel(), dev,
                                             torch.cuda.current_stream(dev).cuda_stream))
    return keys


def _cuda_unpack(keys: torch.Tensor, max_map: torch.Tensor, arg_map: torch.Tensor) -> None:
    dev = keys.device.index
    _lib.check(_lib.load().zfft_unpack_max_arg(keys.data_ptr(), max_map.data_ptr(),
                                               arg_map.data_ptr(), keys.numel(), dev,
                                               torch.cuda.current_stream(dev).cuda_stream))


CUDA_OPS = SearchOps(_cuda_corr_max, _cuda_pack, _cuda_unpack, _cuda_workspace)


@dataclass
class SearchCheckpoint:
    """One rank's progress through its shard: the running maps (host tensors)
    after the templates of the shard before global index `next_index`.  A
    search restarted with `resume=` continues from there; every rank resumes
    from its own checkpoint (the maps are per rank until the final
    reduction)."""

    n_templates: int
    rank: int
    world: int
    next_index: int
    max_map: torch.Tensor
    arg_map: torch.Tensor
    sum_map: Optional[torch.Tensor] = None    # with stats=True (float64)
    sumsq_map: Optional[torch.Tensor] = None

    def save(self, path: str) -> None:
        torch.save({"n_templates": self.n_templates, "rank": self.rank, "world": self.world,
                    "next_index": self.next_index, "max_map": self.max_map,
                    "arg_map": self.arg_map, "sum_map": self.sum_map,
                    "sumsq_map": self.sumsq_map}, path)

    @staticmethod
    def load(path: str) -> "SearchCheckpoint":
        d = torch.load(path, map_location="cpu", weights_only=True)
        return SearchCheckpoint(int(d["n_templates"]), int(d["rank"]), int(d["world"]),
                                int(d["next_index"]), d["max_map"], d["arg_map"],
                                d.get("sum_map"), d.get("sumsq_map"))


def template_search(templates: torch.Tensor, conv_data: torch.Tensor, fft_size_y: int,
                    fft_size_x: int, *, batch_size: int = 256, full: bool = True,
                    group=None, device: Optional[torch.device] = None,
                    ops: SearchOps = CUDA_OPS, checkpoint_every: int = 0,
                    on_checkpoint: Optional[Callable[[SearchCheckpoint], None]] = None,
                    resume: Optional[SearchCheckpoint] = None, stats: bool = False,
                    shard_base: Optional[int] = None,
                    phase_events: Optional[dict] = None) -> Tuple[torch.Tensor, ...]:
    """Maximum and argmax (global template index) of the correlation per pixel.

    templates: (N, h, w) float32 -- the whole set (every rank passes the same
    tensor, on the host (pinned memory is fastest) or on its device); each rank
    correlates its contiguous shard.  conv_data: (W/2+1, H) complex64
    spectrum on this rank's device.  Returns (max_map float32, arg_map int32),
    (H, W) if `full` else the valid crop, identical on every rank.

    Checkpoints: with checkpoint_every = k > 0, `on_checkpoint` receives a
    SearchCheckpoint (maps copied to the host, which synchronises the device)
    after every k-th batch of this rank's shard that leaves templates to do.
    resume: a checkpoint of this rank from an earlier run of the same search
    (same template count, rank and world size); the shard continues at its
    next_index with its maps.  The result equals the uninterrupted search's.

    stats=True: also the per-pixel sum and sum of squares of the correlations
    over all templates, for z-score normalisation; returns (max_map, arg_map,
    sum_map, sumsq_map).  Per batch, the kernels sum the squares in float32
    and the batch's sum map is the correlation map of its summed template
    (correlation is linear); the batches (and the ranks, with one all-reduce)
    are added in float64, so the sums are float64 and their rounding grows
    with the batch size, not with the number of templates.

    shard_base: `templates` is then only this rank's shard (each rank loads
    its own templates), its first template having global index shard_base;
    nothing is split further.  The ranks' shards must not overlap.

    Device memory: the maps, two template batches (from host memory), and a
    workspace of SEARCH_GROUP intermediate slices (16 x H x W/2 complex64,
    1.07 GB at 4096^2), so that 16 templates share each kernel launch.

    phase_events: a dict that receives timing events recorded on the compute
    stream at each phase boundary ("start", "first_copy" (the first batch is
    on the device), "batches", "pack", "reduce", "unpack", "end"; the last
    four only with more than one rank), for
    per-phase device times once the stream has been synchronised."""
    import torch.distributed as dist

    distributed = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if distributed else 1
    rank = dist.get_rank(group) if distributed else 0
    dev = device or conv_data.device
    N, h, w = templates.shape
    H, W = int(fft_size_y), int(fft_size_x)
    oy, ox = (H, W) if full else (H - h + 1, W - w + 1)
    if shard_base is None:
        lo, hi = shard_range(N, rank, world)
        off = 0
    else:
        if shard_base < 0:
            raise ValueError(f"shard_base must be >= 0, got {shard_base}")
        lo, hi, off = shard_base, shard_base + N, shard_base

    start = lo
    if resume is not None:
        if (resume.n_templates, resume.rank, resume.world) != (N, rank, world):
            raise ValueError(
                f"checkpoint of a different search: {resume.n_templates} templates, rank "
                f"{resume.rank} of {resume.world}; this is {N} templates, rank {rank} of {world}")
        if not lo <= resume.next_index <= hi:
            raise ValueError(f"checkpoint index {resume.next_index} outside this rank's shard "
                             f"[{lo}, {hi})")
        if tuple(resume.max_map.shape) != (oy, ox) or tuple(resume.arg_map.shape) != (oy, ox):
            raise ValueError(f"checkpoint maps are {tuple(resume.max_map.shape)}, the search's "
                             f"are {(oy, ox)}")
        if stats and (resume.sum_map is None or resume.sumsq_map is None):
            raise ValueError("checkpoint has no sum maps; it comes from a search without stats")
        start = resume.next_index
        max_map = resume.max_map.to(device=dev, dtype=torch.float32, copy=True).contiguous()
        arg_map = resume.arg_map.to(device=dev, dtype=torch.int32, copy=True).contiguous()
    else:
        max_map = torch.full((oy, ox), float("-inf"), dtype=torch.float32, device=dev)
        arg_map = torch.full((oy, ox), -1, dtype=torch.int32, device=dev)
    sum_map = sumsq_map = part_sum = part_sumsq = None
    if stats:
        if resume is not None:
            sum_map = resume.sum_map.to(device=dev, dtype=torch.float64, copy=True).contiguous()
            sumsq_map = resume.sumsq_map.to(device=dev, dtype=torch.float64,
                                            copy=True).contiguous()
        else:  # an empty shard contributes zeros
            sum_map = torch.zeros((oy, ox), dtype=torch.float64, device=dev)
            sumsq_map = torch.zeros((oy, ox), dtype=torch.float64, device=dev)
        # one batch's float32 partial sums (written afresh by every batch)
        part_sum = torch.empty((oy, ox), dtype=torch.float32, device=dev)
        part_sumsq = torch.empty((oy, ox), dtype=torch.float32, device=dev)
    nb = min(batch_size, max(hi - lo, 1))
    workspace = ops.workspace(H, W, h, dev)

    on_host = templates.device.type == "cpu"
    compute = torch.cuda.current_stream(dev) if dev.type == "cuda" else None
    copy = torch.cuda.Stream(dev) if (on_host and dev.type == "cuda") else None
    bufs = [torch.empty((nb, h, w), dtype=torch.float32, device=dev) for _ in range(2)] \
        if on_host else None
    events = [None, None]

    def stage(i: int, b0: int, b1: int) -> torch.Tensor:
        if not on_host:
            return templates[b0 - off:b1 - off]
        buf = bufs[i][: b1 - b0]
        if copy is not None:
            copy.wait_stream(compute) if events[i] is None else copy.wait_event(events[i])
            with torch.cuda.stream(copy):
                buf.copy_(templates[b0 - off:b1 - off], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy)
            compute.wait_event(ev)
        else:
            buf.copy_(templates[b0 - off:b1 - off])
        return buf

    def mark(name: str) -> None:
        if phase_events is not None and compute is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(compute)
            phase_events[name] = ev

    mark("start")
    # A resumed shard has maps to fold into; a fresh one starts by overwriting.
    first = start == lo
    for j, (b0, b1) in enumerate(batch_bounds(start, hi, nb, ramp=on_host)):
        batch = stage(j % 2, b0, b1)
        if j == 0:
            mark("first_copy")
        if stats:
            ops.corr_max(batch, workspace, conv_data, max_map, arg_map, H, W, b0,
                         RESET_ALL if first else RESET_SUMS, part_sum, part_sumsq)
            sum_map += part_sum
            sumsq_map += part_sumsq
        else:
            ops.corr_max(batch, workspace, conv_data, max_map, arg_map, H, W, b0,
                         RESET_ALL if first else 0)
        first = False
        if copy is not None:  # the buffer may be refilled once this batch's kernels ran
            ev = torch.cuda.Event()
            ev.record(compute)
            events[j % 2] = ev
        if checkpoint_every > 0 and on_checkpoint is not None and (j + 1) % checkpoint_every == 0 \
                and b1 < hi:
            snap = (lambda m: None if m is None else m.to("cpu", copy=True))
            on_checkpoint(SearchCheckpoint(N, rank, world, b1, snap(max_map), snap(arg_map),
                                           snap(sum_map), snap(sumsq_map)))

    mark("batches")
    if world > 1:
        keys = ops.pack(max_map, arg_map)
        mark("pack")
        dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
        mark("reduce")
        ops.unpack(keys, max_map, arg_map)
        mark("unpack")
        if stats:
            both = torch.stack([sum_map, sumsq_map])
            dist.all_reduce(both, op=dist.ReduceOp.SUM, group=group)
            sum_map, sumsq_map = both[0], both[1]
        mark("end")
    if stats:
        return max_map, arg_map, sum_map, sumsq_map
    return max_map, arg_map
