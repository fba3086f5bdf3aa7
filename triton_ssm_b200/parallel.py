"""Partitioning the hot path over the GPUs of one node.

* Batch x head (and stream) sharding: the units of configs 1, 2, 3 and 5 are
  independent, so each rank owns a contiguous range of them and no data-path
  collective exists (``shard_range``).
* Sequence sharding of the multi-head scan (config 4): rank r owns the r-th
  contiguous slice of L.  Each rank scans its slice from a zero state, the
  ranks exchange (final state, whole-slice decay) with one all-gather (about
  Bt*H*P*N*4 bytes per rank), and each rank chains its outputs to the slices
  before it with ``ssd_carry_fixup``.  The arithmetic is the reference's
  block carry scan (ssm_scan.py:53-98) lifted from blocks to slices.
"""
import math

import torch
import torch.distributed as dist

from . import ops


def shard_range(n, rank, world):
    """Contiguous [start, stop) share of n units for `rank` of `world`."""
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def _all_gather_packed(S, d, group):
    """One all-gather of every rank's (S, d), packed into a single f32 buffer."""
    world = dist.get_world_size(group)
    flat = torch.cat([S.reshape(-1), d.reshape(-1)])
    bufs = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(bufs, flat, group=group)
    n = S.numel()
    S_all = torch.stack([b[:n].view_as(S) for b in bufs]).contiguous()
    d_all = torch.stack([b[n:].view_as(d) for b in bufs]).contiguous()
    return S_all, d_all


def ssd_local_pieces(Bt, H, L, sms):
    """In-device pieces per sequence for a long slice: the power of two up to 8
    whose Bt*H*pieces CTAs (one per SM at a time) fill the last wave best,
    keeping pieces of at least 16384 tokens so that the carry fix-up (which
    stops once the decay underflows, typically within a few thousand tokens)
    stays a small fraction of the work."""
    best, best_eff = 1, 0.0
    for K in (1, 2, 4, 8):
        if L % (64 * K) or (K > 1 and L // K < 16384):
            continue
        n = Bt * H * K
        eff = n / (math.ceil(n / sms) * sms)
        if eff > best_eff + 1e-9:
            best, best_eff = K, eff
    return best


def ssd_sequence_parallel(x, dt, A_log, B, C, D, group=None, bdisc="euler", y=None,
                          local_scan=None, fixup=None):
    """Multi-head scan of a sequence sharded over the ranks of `group`.

    x [Bt,Ls,H*P], dt [Bt,Ls,H], B, C [Bt,Ls,H,N] are this rank's slice of the
    sequence (rank order = sequence order); A_log [H], D [H*P] are replicated.
    Returns this rank's outputs y [Bt,Ls,H*P] — the same values as a scan of
    the whole sequence on one device.

    ``local_scan(x, dt, A_log, B, C, D) -> (y, S, d)`` and
    ``fixup(S_all, d_all, rank, C, dt, A_log, y)`` default to the CUDA
    operators; the multi-process CPU tests substitute the CPU oracle for both
    to exercise this orchestration over gloo.
    """
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if local_scan is None:
        def local_scan(x, dt, A_log, B, C, D):
            sms = torch.cuda.get_device_properties(x.device).multi_processor_count
            K = ssd_local_pieces(x.shape[0], B.shape[2], x.shape[1], sms)
            return ops.multihead_ssm(x, A_log, B, C, dt, D, bdisc=bdisc, y=y, return_state=True,
                                     return_decay=True, pieces=K)
    if fixup is None:
        fixup = ops.ssd_carry_fixup
    yl, S, d = local_scan(x, dt, A_log, B, C, D)
    if world == 1:
        return yl
    S_all, d_all = _all_gather_packed(S, d, group)
    fixup(S_all, d_all, rank, C, dt, A_log, yl)
    return yl
