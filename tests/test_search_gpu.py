"""The fused running max / argmax (corr_max), the packed keys, and the
template search on the GPU, against the oracle."""
import numpy as np
import pytest
import torch

from oracle import xcorr_oracle as O
from tests.gpu_helpers import make_inputs
from zipfft_b200 import _lib

pytestmark = pytest.mark.gpu


def maps(ref):
    """Oracle max / argmax over templates and the pixels whose winner is
    unambiguous (lead over the runner-up above the tolerance)."""
    order = np.sort(ref, axis=0)
    sure = (order[-1] - order[-2]) > 1e-4 * np.abs(ref).max()
    return ref.max(axis=0), ref.argmax(axis=0), sure


def run_corr_max(tm, spec, H, W, full, base=0, reset=True, mx=None, am=None, ws=None):
    import zipfft

    dev = torch.device("cuda", 0)
    B, h, w = tm.shape
    oy, ox = O.out_shape(h, w, H, W, full)
    if mx is None:
        mx = torch.full((oy, ox), float("nan"), device=dev)
        am = torch.full((oy, ox), -7, dtype=torch.int32, device=dev)
    if ws is None:
        ws = torch.empty((B, H, W // 2 + 1), dtype=torch.complex64, device=dev)
    zipfft.padded_rconv2d.corr_max(tm.to(dev), ws, spec.to(dev), mx, am, H, W,
                                   template_index_base=base, reset=reset)
    torch.cuda.synchronize()
    return mx, am


@pytest.mark.parametrize("B,h,w,H,W,full", [(6, 16, 16, 64, 64, True), (5, 40, 30, 256, 512, False),
                                            (9, 100, 100, 1024, 1024, True),
                                            (4, 384, 384, 3840, 3840, True)])
def test_corr_max_matches_oracle(B, h, w, H, W, full):
    _, tm, spec = make_inputs(B, h, w, H, W, seed=B + h)
    mx, am = run_corr_max(tm, spec, H, W, full)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, True, full)
    rmax, rarg, sure = maps(ref)
    got_max, got_arg = mx.cpu().numpy(), am.cpu().numpy()
    assert O.rel_l2(rmax, got_max) < 5e-6
    assert O.max_abs_over_peak(rmax, got_max) < 1e-4
    assert sure.mean() > 0.99
    assert np.array_equal(got_arg[sure], rarg[sure])  # bit-exact where the margin is clear


def test_corr_max_in_batches_equals_one_call():
    _, tm, spec = make_inputs(7, 64, 64, 512, 512, seed=4)
    mx1, am1 = run_corr_max(tm, spec, 512, 512, True)
    mx2, am2 = run_corr_max(tm[:3], spec, 512, 512, True, base=0, reset=True)
    run_corr_max(tm[3:], spec, 512, 512, True, base=3, reset=False, mx=mx2, am=am2)
    assert torch.equal(mx1, mx2) and torch.equal(am1, am2)


@pytest.mark.parametrize("B,h,w,H,W,full", [(6, 96, 96, 1024, 1024, True),
                                            (5, 40, 30, 256, 512, False),
                                            (3, 256, 256, 4096, 4096, True)])
def test_corr_max_stats_match_oracle(B, h, w, H, W, full):
    """Per-pixel sum and sum of squares over the templates, accumulated over
    two calls (the first resets), next to the running max / argmax."""
    import zipfft

    _, tm, spec = make_inputs(B, h, w, H, W, seed=B + h + 1)
    dev = torch.device("cuda", 0)
    oy, ox = O.out_shape(h, w, H, W, full)
    mx = torch.full((oy, ox), float("nan"), device=dev)
    am = torch.full((oy, ox), -7, dtype=torch.int32, device=dev)
    sm = torch.full((oy, ox), float("nan"), device=dev)
    sq = torch.full((oy, ox), float("nan"), device=dev)
    ws = torch.empty((B, H, W // 2 + 1), dtype=torch.complex64, device=dev)
    tm_d, sp_d = tm.to(dev), spec.to(dev)
    k = B // 2
    zipfft.padded_rconv2d.corr_max(tm_d[:k], ws[:k], sp_d, mx, am, H, W, 0, True, sm, sq)
    zipfft.padded_rconv2d.corr_max(tm_d[k:], ws[k:], sp_d, mx, am, H, W, k, False, sm, sq)
    torch.cuda.synchronize()
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, True, full)
    rmax, rarg, sure = maps(ref)
    assert O.rel_l2(rmax, mx.cpu().numpy()) < 5e-6
    assert np.array_equal(am.cpu().numpy()[sure], rarg[sure])
    assert O.rel_l2(ref.sum(axis=0), sm.cpu().numpy()) < 5e-6
    assert O.rel_l2((ref ** 2).sum(axis=0), sq.cpu().numpy()) < 5e-6
    # the max / argmax maps are the same with and without the statistics
    mx2, am2 = run_corr_max(tm, spec, H, W, full)
    assert torch.equal(mx, mx2) and torch.equal(am, am2)


def test_search_stats_over_1024_templates_match_float64_sums():
    """stats=True over 1024 templates from host memory in batches of up to
    256 (the first ones ramped up from 16): the kernels sum each batch in
    float32 and the search adds the batches in float64, so the per-pixel sums
    stay within the batch's rounding of the oracle's float64 sums (naive
    float32 accumulation over all 1024 would not)."""
    from zipfft_b200.search import template_search

    H = W = 256
    N, h = 1024, 16
    _, tm, spec = make_inputs(N, h, h, H, W, seed=31)
    dev = torch.device("cuda", 0)
    mx, am, sm, sq = template_search(tm, spec.to(dev), H, W, batch_size=256, full=True,
                                     stats=True)
    torch.cuda.synchronize()
    assert sm.dtype == torch.float64 and sq.dtype == torch.float64
    ref_s = np.zeros((H, W))
    ref_q = np.zeros((H, W))
    ref_m = np.full((H, W), -np.inf)
    for b0 in range(0, N, 128):
        ref = O.padded_corr2d_f64(tm[b0:b0 + 128].numpy(), spec.numpy(), H, W, True, True)
        ref_s += ref.sum(axis=0)
        ref_q += (ref ** 2).sum(axis=0)
        ref_m = np.maximum(ref_m, ref.max(axis=0))
    scale = np.sqrt(ref_q.max())
    assert np.abs(sm.cpu().numpy() - ref_s).max() / scale < 1e-5
    assert O.rel_l2(ref_q, sq.cpu().numpy()) < 5e-6
    assert O.rel_l2(ref_m, mx.cpu().numpy()) < 5e-6


def test_corr_max_stats_argument_errors():
    import zipfft

    _, tm, spec = make_inputs(2, 16, 16, 64, 64, seed=2)
    dev = torch.device("cuda", 0)
    mx = torch.empty((64, 64), device=dev)
    am = torch.empty((64, 64), dtype=torch.int32, device=dev)
    ws = torch.empty((2, 64, 33), dtype=torch.complex64, device=dev)
    with pytest.raises(RuntimeError, match="given together"):
        zipfft.padded_rconv2d.corr_max(tm.to(dev), ws, spec.to(dev), mx, am, 64, 64,
                                       sum_map=torch.empty_like(mx))
    with pytest.raises(RuntimeError, match="shape"):
        zipfft.padded_rconv2d.corr_max(tm.to(dev), ws, spec.to(dev), mx, am, 64, 64,
                                       sum_map=torch.empty((64, 63), device=dev),
                                       sumsq_map=torch.empty_like(mx))


def test_tie_keeps_lowest_index():
    _, tm, spec = make_inputs(4, 32, 32, 256, 256, seed=8)
    tm[3] = tm[1]  # identical templates: every pixel ties between 1 and 3
    mx, am = run_corr_max(tm, spec, 256, 256, True)
    assert not torch.any(am == 3)


def test_pack_unpack_round_trip_and_order():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    vals = torch.tensor([-3.5, -0.0, 0.0, 1e-30, 2.0, 2.0, float("inf"), -float("inf")], device=dev)
    idx = torch.tensor([5, 1, 2, 3, 9, 4, 0, 7], dtype=torch.int32, device=dev)
    keys = torch.empty(8, dtype=torch.int64, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.zfft_pack_max_arg(vals.data_ptr(), idx.data_ptr(), keys.data_ptr(), 8, 0, s))
    v2 = torch.empty_like(vals)
    i2 = torch.empty_like(idx)
    _lib.check(lib.zfft_unpack_max_arg(keys.data_ptr(), v2.data_ptr(), i2.data_ptr(), 8, 0, s))
    torch.cuda.synchronize()
    assert torch.equal(vals.view(torch.int32), v2.view(torch.int32))  # bit-exact, incl. -0.0
    assert torch.equal(idx, i2)
    k = keys.cpu().tolist()
    # larger value wins; equal values: lower index wins
    assert k[4] < k[5] and max(k) == k[6] and min(k) == k[7] and k[0] < k[1] < k[2] < k[3]


def test_search_planted_templates_known_answer():
    """A reduced version of the full search: 256 templates of 384^2, copies of
    template 77 planted at 20 positions with amplitude 0.5; the search finds
    template 77 at exactly those positions."""
    from zipfft_b200.search import template_search

    H = 4096
    rng = np.random.default_rng(50)
    img = rng.standard_normal((H, H)).astype(np.float32)
    g = torch.Generator().manual_seed(5)
    tm = torch.randn((256, 384, 384), generator=g)
    tm = (tm - tm.mean(dim=(1, 2), keepdim=True)) / tm.std(dim=(1, 2), keepdim=True)
    k = 77
    pos = set()
    while len(pos) < 20:
        y, x = (int(v) for v in rng.integers(0, H - 384, size=2))
        if all(abs(y - a) > 400 or abs(x - b) > 400 for a, b in pos):
            pos.add((y, x))
    for (y, x) in pos:
        img[y:y + 384, x:x + 384] += 0.5 * tm[k].numpy()
    spec = torch.from_numpy(O.image_spectrum_T(img)).cuda()
    marks = {}
    mx, am = template_search(tm.pin_memory(), spec, H, H, batch_size=64, full=True,
                             phase_events=marks)
    torch.cuda.synchronize()
    assert list(marks) == ["start", "first_copy", "batches"]  # one rank: no reduction phases
    assert 0 <= marks["start"].elapsed_time(marks["first_copy"]) \
        <= marks["start"].elapsed_time(marks["batches"])
    mx, am = mx.cpu().numpy(), am.cpu().numpy()
    for (y, x) in pos:
        assert am[y, x] == k
        assert mx[y, x] > 0.4 * 384 * 384
    top = np.argsort(mx.ravel())[::-1][:20]
    assert sorted((int(i // H), int(i % H)) for i in top) == sorted(pos)


def test_search_resume_on_gpu_matches_uninterrupted(tmp_path):
    """A search stopped at a checkpoint (maps copied to the host and saved)
    and resumed from the file equals the uninterrupted search bit for bit."""
    from zipfft_b200.search import SearchCheckpoint, template_search

    H = 1024
    _, tm, spec = make_inputs(40, 96, 96, H, H, seed=11)
    spec = spec.cuda()
    ref_mx, ref_am = template_search(tm.pin_memory(), spec, H, H, batch_size=8)
    path = str(tmp_path / "cp.pt")

    class Stop(Exception):
        pass

    def save_and_stop(cp):
        cp.save(path)
        raise Stop

    with pytest.raises(Stop):
        template_search(tm.pin_memory(), spec, H, H, batch_size=8, checkpoint_every=3,
                        on_checkpoint=save_and_stop)
    cp = SearchCheckpoint.load(path)
    assert cp.next_index == 24
    mx, am = template_search(tm.pin_memory(), spec, H, H, batch_size=8, resume=cp)
    torch.cuda.synchronize()
    assert torch.equal(mx, ref_mx) and torch.equal(am, ref_am)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_search_two_gpus_nccl(tmp_path):
    import subprocess
    import sys

    script = tmp_path / "run.py"
    script.write_text(
        "import os, sys, datetime, numpy as np, torch, torch.distributed as dist\n"
        f"sys.path.insert(0, {repr(str(__import__('pathlib').Path(__file__).resolve().parents[1]))})\n"
        "from oracle import xcorr_oracle as O\n"
        "from zipfft_b200.search import template_search\n"
        "r = int(os.environ['RANK']); torch.cuda.set_device(r)\n"
        "dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),"
        " device_id=torch.device('cuda', r))\n"
        "g = torch.Generator().manual_seed(3)\n"
        "img = torch.randn((512, 512), generator=g); tm = torch.randn((10, 40, 40), generator=g)\n"
        "spec = torch.from_numpy(O.image_spectrum_T(img.numpy())).cuda()\n"
        "mx, am, sm, sq = template_search(tm, spec, 512, 512, batch_size=3, stats=True)\n"
        "ref = O.padded_corr2d_f64(tm.numpy(), spec.cpu().numpy(), 512, 512, True, True)\n"
        "order = np.sort(ref, 0); sure = (order[-1] - order[-2]) > 1e-4 * np.abs(ref).max()\n"
        "ok = np.array_equal(am.cpu().numpy()[sure], ref.argmax(0)[sure]) and "
        "O.rel_l2(ref.max(0), mx.cpu().numpy()) < 5e-6 and "
        "O.rel_l2(ref.sum(0), sm.cpu().numpy()) < 5e-6 and "
        "O.rel_l2((ref ** 2).sum(0), sq.cpu().numpy()) < 5e-6\n"
        "dist.destroy_process_group(); sys.exit(0 if ok else 1)\n")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29517", str(script)]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300,
                         env={**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"})
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]


@pytest.mark.parametrize("B,h,w,H,W,full,stats", [(5, 256, 256, 2048, 2048, True, False),
                                                  (7, 40, 30, 1024, 512, False, True),
                                                  (4, 384, 384, 3840, 3840, True, True)])
def test_grouped_running_maps_equal_per_template_launches(B, h, w, H, W, full, stats):
    """The running-map call with a workspace of B slices runs the templates as
    one batched group (each block folds a row group's templates in order);
    the maps, argmax and sums equal the one-slice workspace's per-template
    launches bit for bit."""
    from zipfft_b200 import _lib
    from zipfft_b200.search import RESET_ALL, _cuda_corr_max

    _, tm, spec = make_inputs(B, h, w, H, W, seed=B + h)
    dev = torch.device("cuda", 0)
    oy, ox = O.out_shape(h, w, H, W, full)
    res = []
    slice_elems = _lib.load().zfft_workspace_bytes(H, W) // 8
    for slices in (1, B):  # through the C ABI, which takes any workspace size
        ws = torch.empty(slices * slice_elems, dtype=torch.complex64, device=dev)
        mx = torch.empty((oy, ox), device=dev)
        am = torch.empty((oy, ox), dtype=torch.int32, device=dev)
        sm = torch.empty((oy, ox), device=dev) if stats else None
        sq = torch.empty((oy, ox), device=dev) if stats else None
        _cuda_corr_max(tm.to(dev), ws, spec.to(dev), mx, am, H, W, 3, RESET_ALL, sm, sq)
        torch.cuda.synchronize()
        res.append([t.cpu() for t in (mx, am, sm, sq) if t is not None])
    for a, b in zip(*res):
        assert torch.equal(a, b)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, True, full)
    assert O.rel_l2(ref.max(axis=0), res[1][0].numpy()) < 5e-6
    assert int(res[1][1].min()) >= 3 and int(res[1][1].max()) < 3 + B


def test_max_stats_without_sum_map_matches_with_it():
    """zfft_padded_real_corr_2d_max_stats with sum_map NULL accumulates the
    maximum, argmax and sum of squares exactly as with a sum map (bit for
    bit); the search's sum map, taken as the correlation map of each batch's
    summed template, matches the oracle's float64 sums."""
    from zipfft_b200 import _lib

    B, h, w, H, W = 6, 40, 30, 512, 256
    _, tm, spec = make_inputs(B, h, w, H, W, seed=77)
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    ws = torch.empty(B * lib.zfft_workspace_bytes(H, W) // 8, dtype=torch.complex64, device=dev)
    stream = torch.cuda.current_stream(0).cuda_stream
    tm_d, spec_d = tm.to(dev), spec.to(dev)  # held: the calls below are asynchronous
    out = []
    for with_sum in (True, False):
        mx = torch.empty((H, W), device=dev)
        am = torch.empty((H, W), dtype=torch.int32, device=dev)
        sm = torch.zeros((H, W), device=dev)
        sq = torch.empty((H, W), device=dev)
        _lib.check(lib.zfft_padded_real_corr_2d_max_stats(
            tm_d.data_ptr(), B, h, w, ws.data_ptr(), ws.numel() * 8, spec_d.data_ptr(),
            mx.data_ptr(), am.data_ptr(), sm.data_ptr() if with_sum else None, sq.data_ptr(),
            H, W, H, W, 0, 1, 0, stream))
        torch.cuda.synchronize()
        out.append((mx.cpu(), am.cpu(), sq.cpu(), sm.cpu()))
    for a, b in zip(out[0][:3], out[1][:3]):
        assert torch.equal(a, b)
    assert not out[1][3].any()  # no sum map: nothing written to the untouched buffer

    from zipfft_b200.search import template_search

    mx, am, sm, sq = template_search(tm, spec_d, H, W, batch_size=4, full=True, stats=True)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, True, True)
    scale = np.sqrt((ref ** 2).sum(axis=0).max())
    assert np.abs(sm.cpu().numpy() - ref.sum(axis=0)).max() / scale < 1e-5
    assert O.rel_l2((ref ** 2).sum(axis=0), sq.cpu().numpy()) < 5e-6
