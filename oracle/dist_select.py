"""Distributed k-smallest selection, restated in numpy.

TEST INFRASTRUCTURE ONLY.  Mirrors the multi-rank path of the product's
selector (three histogram passes over 32-bit keys — bits 31..20, 19..8, 7..0
— each summed across ranks, then the boundary ties split in (rank, index)
order from a gather of per-rank tie counts) so the algorithm can be checked
on CPU ranks (gloo) against the single-rank oracle.  `allreduce(arr)` must
return the element-wise sum over ranks; `allgather(x)` the list of every
rank's value in rank order.
"""
import numpy as np

INVALID = 0xFFFFFFFF


def select_local(keys, k_global, allreduce, allgather, rank):
    """keys: uint32 array of this rank (INVALID = ineligible).  Returns the
    indices this rank contributes to the global k smallest (ascending)."""
    keys = np.asarray(keys, np.uint32)
    valid = keys != INVALID
    vk = keys[valid]
    # pass 0: top 12 bits + eligible count
    h = np.bincount(vk >> 20, minlength=4096).astype(np.int64)
    h = np.concatenate([h, [valid.sum()]])
    h = allreduce(h)
    n_el = int(h[4096])
    k = min(k_global, n_el)
    if k == 0:
        return np.zeros(0, np.uint32)
    rem = k
    cum = np.cumsum(h[:4096])
    b0 = int(np.searchsorted(cum, rem))        # first bin with cum >= rem
    rem -= int(cum[b0 - 1]) if b0 > 0 else 0
    prefix = b0 << 20
    # pass 1: bits 19..8 inside bin b0
    m1 = (vk >> 20) == b0
    h1 = allreduce(np.bincount((vk[m1] >> 8) & 0xFFF, minlength=4096).astype(np.int64))
    cum = np.cumsum(h1)
    b1 = int(np.searchsorted(cum, rem))
    rem -= int(cum[b1 - 1]) if b1 > 0 else 0
    prefix |= b1 << 8
    # pass 2: bits 7..0
    m2 = (vk >> 8) == (prefix >> 8)
    local2 = np.bincount(vk[m2] & 0xFF, minlength=256).astype(np.int64)
    h2 = allreduce(local2)
    cum = np.cumsum(h2)
    b2 = int(np.searchsorted(cum, rem))
    rem -= int(cum[b2 - 1]) if b2 > 0 else 0
    kth = prefix | b2
    # tie split: ranks before this one take their ties first
    ties = allgather(int(local2[b2]))
    before = sum(ties[:rank])
    take = max(0, min(rem - before, ties[rank]))
    idx = np.nonzero(valid & (keys < kth))[0]
    tie_idx = np.nonzero(keys == kth)[0][:take]
    return np.sort(np.concatenate([idx, tie_idx]).astype(np.uint32))
