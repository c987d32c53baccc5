"""The sequence-split decode (config 4's multi-GPU path) on 2 GPUs: NCCL ranks,
each with a contiguous token range, partials all-gathered and merged on
device; every rank's merged output must match a single-GPU decode of the whole
context within the attention tolerance.  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, result_dir):
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    from tailorquantkernel_b200 import shard, tqk
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        nq, nkv, hd = 64, 8, 128
        g = torch.Generator(device="cuda").manual_seed(77)  # the same full context on every rank
        kp = tqk.quantize_rows(torch.randn(nkv, n, hd, device="cuda", generator=g))
        vp = tqk.quantize_rows(torch.randn(nkv, n, hd, device="cuda", generator=g))
        q = torch.randn(nq * hd, device="cuda", generator=g)
        s, ln = shard.seq_range(n, rank, world)
        kl, vl = kp[:, s:s + ln].contiguous(), vp[:, s:s + ln].contiguous()
        out = torch.empty(nq * hd, device="cuda")
        partial = torch.empty(nq * (hd + 2), device="cuda")
        for _ in range(2):  # twice: the buffers are reusable
            shard.seqsplit_attend(dist, tqk, kl, vl, nq, nkv, hd, ln, q, out, partial)
        full = torch.empty(nq * hd, device="cuda")
        tqk.attend(kp, vp, nq, nkv, hd, n, n - 1, q, full)
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.stack([out.cpu().numpy(), full.cpu().numpy()]))
        assert tqk.device_status() == 0
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [20000, 100])
def test_sequence_split_two_gpus(cuda, tmp_path, n):
    import torch
    import torch.multiprocessing as mp
    from _cases import tolerance_ok
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_rank_main, args=(2, _free_port(), n, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        got, ref = np.load(tmp_path / f"rank{r}.npy")
        ok, max_abs, rel = tolerance_ok(got, ref)
        assert ok, f"rank {r}: max abs {max_abs:.3g} rel {rel:.3g}"


def _rank_main_p2p(rank, world, port, n, steps, result_dir):
    """Sequence split with the exchange over peer memory (shard.PeerExchange):
    a different q every step, so a step that read a stale mailbox slot of an
    earlier epoch would not match."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    from tailorquantkernel_b200 import shard, tqk
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        nq, nkv, hd = 64, 8, 128
        g = torch.Generator(device="cuda").manual_seed(78)
        kp = tqk.quantize_rows(torch.randn(nkv, n, hd, device="cuda", generator=g))
        vp = tqk.quantize_rows(torch.randn(nkv, n, hd, device="cuda", generator=g))
        qs = torch.randn(steps, nq * hd, device="cuda", generator=g)
        s, ln = shard.seq_range(n, rank, world)
        kl, vl = kp[:, s:s + ln].contiguous(), vp[:, s:s + ln].contiguous()
        ex = shard.PeerExchange(dist, tqk, nq, hd)
        outs = torch.empty(steps, nq * hd, device="cuda")
        for i in range(steps):
            shard.seqsplit_attend_p2p(ex, tqk, kl, vl, nq, nkv, hd, ln, qs[i], outs[i])
        refs = torch.empty(steps, nq * hd, device="cuda")
        for i in range(steps):
            tqk.attend(kp, vp, nq, nkv, hd, n, n - 1, qs[i], refs[i])
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"p2p_rank{rank}.npy"), np.stack([outs.cpu().numpy(), refs.cpu().numpy()]))
        assert tqk.device_status() == 0
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("n,steps", [(20000, 5), (100, 3)])
def test_sequence_split_peer_exchange_two_gpus(cuda, tmp_path, n, steps):
    """tqk_exchange_merge on 2 GPUs: every step's merged output on every rank
    matches a single-GPU decode of the whole context for that step's q."""
    import torch
    import torch.multiprocessing as mp
    from _cases import tolerance_ok
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_rank_main_p2p, args=(2, _free_port(), n, steps, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        got, ref = np.load(tmp_path / f"p2p_rank{r}.npy")
        for i in range(steps):
            ok, max_abs, rel = tolerance_ok(got[i], ref[i])
            assert ok, f"rank {r} step {i}: max abs {max_abs:.3g} rel {rel:.3g}"


def test_exchange_merge_single_rank(cuda):
    """tqk_exchange_merge with a world of one (no peer traffic, the mailbox's tickets and
    parity slots still cycle): three epochs in a row equal tqk_merge_partials of the
    same one-part records, and mailboxes that are not whole peer buffers are refused."""
    import torch
    from tailorquantkernel_b200 import tqk
    nq, nkv, hd, n = 64, 8, 128, 3000
    g = torch.Generator(device="cuda").manual_seed(79)
    kp = tqk.quantize_rows(torch.randn(nkv, n, hd, device="cuda", generator=g))
    vp = tqk.quantize_rows(torch.randn(nkv, n, hd, device="cuda", generator=g))
    box = tqk.peer_buffer_alloc(tqk.tqk_exchange_mailbox_bytes(1, nq, hd))
    try:
        for epoch in (1, 2, 3):
            q = torch.randn(nq * hd, device="cuda", generator=g)
            slot = tqk.exchange_slot(box, nq, hd, epoch)
            tqk.decode(tqk.decode_args(kp, vp, nq, nkv, hd, n, q, slot, len0=n, out_mode=tqk.OUT_PARTIAL))
            got = torch.full((nq * hd,), float("nan"), device="cuda")
            tqk.exchange_merge(nq, hd, 1, 0, [box], epoch, got)
            ref = torch.empty(nq * hd, device="cuda")
            tqk.merge_partials(slot, 1, nq * (hd + 2), nq, hd, ref)
            torch.cuda.synchronize()
            assert torch.equal(got, ref), epoch
        with pytest.raises(tqk.TQKError):
            tqk.exchange_merge(nq, hd, 1, 0, [box + 4], 4, got)
        assert tqk.device_status() == 0
    finally:
        tqk.peer_buffer_free(box)


def test_exchange_wait_times_out_without_peer(cuda):
    """Failure detection without a fault: a two-rank exchange whose peer never
    raises its flag (the "peer" mailbox is a second local buffer nobody writes).
    The kernel's bounded wait gives up after about a second, records the timeout
    in the device error word, leaves the output unwritten and returns; the
    context stays usable and the next exchange succeeds."""
    import time

    import torch
    from tailorquantkernel_b200 import tqk
    nq, hd = 64, 128
    nbytes = tqk.tqk_exchange_mailbox_bytes(2, nq, hd)
    boxes = [tqk.peer_buffer_alloc(nbytes), tqk.peer_buffer_alloc(nbytes)]
    solo = tqk.peer_buffer_alloc(tqk.tqk_exchange_mailbox_bytes(1, nq, hd))
    try:
        assert tqk.device_status(clear=True) == 0
        out = torch.full((nq * hd,), float("nan"), device="cuda")
        t0 = time.time()
        tqk.exchange_merge(nq, hd, 2, 0, boxes, 1, out)
        torch.cuda.synchronize()
        waited = time.time() - t0
        assert 0.5 < waited < 30, waited
        assert tqk.device_status(clear=True) == 1  # the timeout code of the device error word
        assert torch.isnan(out).all()  # nothing merged
        # recovery: a one-rank exchange over a zeroed mailbox (l = 0 everywhere) writes zeros
        tqk.exchange_merge(nq, hd, 1, 0, [solo], 1, out)
        torch.cuda.synchronize()
        assert torch.count_nonzero(out).item() == 0
        assert tqk.device_status() == 0
    finally:
        for b in boxes + [solo]:
            tqk.peer_buffer_free(b)
