"""CPU stand-ins for the per-GPU operations of zipfft_b200.search, used only
to exercise the distributed host logic (sharding, index bases, the packed-key
MAX reduction, tie-breaking) on gloo ranks without a GPU.  The correlations
come from the oracle; the key format restates the library's packing
(high 32 bits: float bits in unsigned order, low 32 bits: 0xFFFFFFFF - index,
sign bit flipped for signed comparison)."""
import numpy as np
import torch

from oracle import xcorr_oracle as O
from zipfft_b200.search import SearchOps


def corr_max(batch, workspace, conv_data, max_map, arg_map, H, W, base, reset, sum_map=None,
             sumsq_map=None):
    full = tuple(max_map.shape) == (H, W)
    res = O.padded_corr2d_f64(batch.numpy(), conv_data.numpy(), H, W, True, full)
    mx = max_map.numpy()
    am = arg_map.numpy()
    for t in range(res.shape[0]):
        v = res[t].astype(np.float32)
        first = reset == 1 and t == 0        # RESET_ALL: every map
        first_sums = reset in (1, 2) and t == 0  # RESET_SUMS: the sum maps only
        upd = np.ones_like(mx, bool) if first else (v > mx)
        mx[upd] = v[upd]
        am[upd] = base + t
        if sum_map is not None:  # float32 accumulation within the call, as on the GPU
            s, q = sum_map.numpy(), sumsq_map.numpy()
            s[...] = v if first_sums else s + v
            q[...] = v * v if first_sums else q + v * v


def pack(max_map, arg_map):
    u = max_map.numpy().view(np.uint32).astype(np.uint64)
    u = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    low = (0xFFFFFFFF - arg_map.numpy().astype(np.int64).astype(np.uint64)) & 0xFFFFFFFF
    k = (u << np.uint64(32)) | low
    k = k ^ np.uint64(0x8000000000000000)
    return torch.from_numpy(k.view(np.int64).copy())


def unpack(keys, max_map, arg_map):
    k = keys.numpy().view(np.uint64) ^ np.uint64(0x8000000000000000)
    u = (k >> np.uint64(32)) & np.uint64(0xFFFFFFFF)
    u = np.where(u & 0x80000000, u & 0x7FFFFFFF, (~u) & 0xFFFFFFFF).astype(np.uint32)
    max_map.numpy()[...] = u.view(np.float32)
    arg_map.numpy()[...] = (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64)


def workspace(H, W, h, device):
    return torch.empty(1)


CPU_OPS = SearchOps(corr_max, pack, unpack, workspace)
