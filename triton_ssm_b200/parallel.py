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


class _ExchangeBuffers:
    """Preallocated send and receive buffers of the carry exchange, kept per
    (device, shape, world): send = this rank's [final state | log2 decay],
    recv = every rank's, [world, n + m] f32, filled by one all-gather."""

    _cache = {}

    @classmethod
    def get(cls, device, Bt, H, P, N, world):
        key = (str(device), Bt, H, P, N, world)
        buf = cls._cache.get(key)
        if buf is None:
            n, m = Bt * H * P * N, Bt * H
            send = torch.empty(n + m, device=device, dtype=torch.float32)
            recv = torch.empty(world * (n + m), device=device, dtype=torch.float32)
            buf = (send, recv, n)
            cls._cache[key] = buf
        return buf


def exchange_carries(send, recv, group=None):
    """One all-gather of every rank's packed [state | decay] into ``recv``
    (flat [world * len(send)] f32); returns the [world, len(send)] view."""
    dist.all_gather_into_tensor(recv, send, group=group)
    return recv.view(-1, send.numel())


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
                          local_scan=None, fixup=None, marks=None):
    """Multi-head scan of a sequence sharded over the ranks of `group`.

    x [Bt,Ls,H*P], dt [Bt,Ls,H], B, C [Bt,Ls,H,N] are this rank's slice of the
    sequence (rank order = sequence order); A_log [H], D [H*P] are replicated.
    Returns this rank's outputs y [Bt,Ls,H*P] — the same values as a scan of
    the whole sequence on one device.

    Steps: the local scan writes the slice's final state and log2 decay
    straight into a preallocated send buffer; one all-gather
    (``all_gather_into_tensor``) fills a preallocated [world, n + m] receive
    buffer; ``ssd_carry_fixup_packed`` reads the carries from it in place.

    ``local_scan(x, dt, A_log, B, C, D) -> (y, S, d)`` and
    ``fixup(S_all, d_all, rank, C, dt, A_log, y)`` default to the CUDA
    operators; the multi-process CPU tests substitute the CPU oracle for both
    to exercise this orchestration over gloo.  ``marks``: a list to which a
    CUDA event recorded after the local scan is appended (the caller times
    the exchange and fix-up from it).
    """
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    Bt, Ls, HP = x.shape
    H, N = B.shape[2], B.shape[3]
    P = HP // H
    if local_scan is None and fixup is None:
        sms = torch.cuda.get_device_properties(x.device).multi_processor_count
        K = ssd_local_pieces(Bt, H, Ls, sms)
        if world == 1:
            yl = ops.multihead_ssm(x, A_log, B, C, dt, D, bdisc=bdisc, y=y, pieces=K)
            if marks is not None:
                marks.append(_event())
            return yl
        send, recv, n = _ExchangeBuffers.get(x.device, Bt, H, P, N, world)
        yl, _, _ = ops.multihead_ssm(x, A_log, B, C, dt, D, bdisc=bdisc, y=y, return_state=True,
                                     return_decay=True, pieces=K, state_out=send[:n].view(Bt, H, P, N),
                                     decay_out=send[n:].view(Bt, H))
        if marks is not None:
            marks.append(_event())
        packed = exchange_carries(send, recv, group)
        ops.ssd_carry_fixup_packed(packed, rank, C, dt, A_log, yl, P=P)
        return yl
    if local_scan is None or fixup is None:
        raise ValueError("ssd_sequence_parallel: give both local_scan and fixup, or neither")
    yl, S, d = local_scan(x, dt, A_log, B, C, D)
    if world == 1:
        return yl
    n = S.numel()
    send = torch.cat([S.reshape(-1), d.reshape(-1)]).float()
    recv = torch.empty(world * send.numel(), dtype=send.dtype, device=send.device)
    packed = exchange_carries(send, recv, group)
    S_all = packed[:, :n].reshape((world,) + tuple(S.shape))
    d_all = packed[:, n:].reshape((world,) + tuple(d.shape))
    fixup(S_all, d_all, rank, C, dt, A_log, yl)
    return yl


def _event():
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    return ev
