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


def _rank_main_heads(rank, world, port, result_dir):
    """kv-head-group split of a 3-layer decode (bench config 2's multi-GPU path) on `world` GPUs:
    each rank appends and attends for its kv heads of every layer, tqk_exchange_gather assembles
    the output; two steps at consecutive positions with different q / k / v."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle
    from tailorquantkernel_b200 import shard, tqk
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    pg = None
    try:
        port_ = oracle.Oracle("port")
        layers, nq, nkv, hd, pos, steps = 3, 32, 8, 128, 700, 2
        mt, per, group = pos + steps, nkv // world, nq // nkv
        rng = np.random.default_rng(90)  # the same full problem on every rank
        kf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
        vf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
        kf[:, :, pos:] = 0.0
        vf[:, :, pos:] = 0.0
        kp_full, vp_full = port_.quantize_rows(kf), port_.quantize_rows(vf)  # [L][nkv][mt][row]
        qs = rng.standard_normal((steps, layers, nq * hd), dtype=np.float32)
        ks = rng.standard_normal((steps, layers, nkv * hd), dtype=np.float32)
        vs = rng.standard_normal((steps, layers, nkv * hd), dtype=np.float32)
        lo = rank * per
        kl = torch.from_numpy(np.ascontiguousarray(kp_full[:, lo:lo + per])).cuda()
        vl = torch.from_numpy(np.ascontiguousarray(vp_full[:, lo:lo + per])).cuda()
        pg = shard.PeerGather(dist, tqk, layers, per * group * hd)
        outs = []
        for s in range(steps):
            q = torch.from_numpy(shard.head_split_slice(qs[s], layers, nq, hd, rank, world)).cuda()
            k = torch.from_numpy(shard.head_split_slice(ks[s], layers, nkv, hd, rank, world)).cuda()
            v = torch.from_numpy(shard.head_split_slice(vs[s], layers, nkv, hd, rank, world)).cuda()
            out = torch.full((layers, nq * hd), float("nan"), device="cuda")
            slot = pg.begin()
            tqk.decode(shard.head_split_args(tqk, kl, vl, layers, nq, nkv, hd, mt, world, q, slot, len0=pos + s + 1,
                                             k_new=k, v_new=v))
            pg.end(out)
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
        refs = []
        for s in range(steps):
            ref = np.empty((layers, nq * hd), np.float32)
            for layer in range(layers):
                assert port_.store_kv(kp_full[layer], vp_full[layer], nkv, hd, mt, pos + s, ks[s, layer],
                                      vs[s, layer]) == 0
                ref[layer] = port_.attend(kp_full[layer], vp_full[layer], nq, nkv, hd, mt, pos + s, qs[s, layer])
            refs.append(ref)
        rows_ok = np.array_equal(kl.cpu().numpy(), kp_full[:, lo:lo + per]) and \
            np.array_equal(vl.cpu().numpy(), vp_full[:, lo:lo + per])
        np.save(os.path.join(result_dir, f"heads_rank{rank}.npy"), np.stack([np.stack(outs), np.stack(refs)]))
        with open(os.path.join(result_dir, f"heads_rank{rank}.txt"), "w") as f:
            f.write(f"{int(rows_ok)} {tqk.device_status()}")
    finally:
        if pg is not None:
            pg.close()
        dist.destroy_process_group()


def test_head_split_gather_two_gpus(cuda, tmp_path):
    """The kv-head-group split over 2 GPUs against the oracle: every rank's gathered output of
    every layer and step within the attention tolerance of the oracle's store_kv + attend_q8,
    and each rank's appended cache rows bit-exact."""
    import torch
    import torch.multiprocessing as mp
    from _cases import tolerance_ok
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_rank_main_heads, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        rows_ok, status = (int(x) for x in open(tmp_path / f"heads_rank{r}.txt").read().split())
        assert rows_ok == 1 and status == 0, (r, rows_ok, status)
        got, ref = np.load(tmp_path / f"heads_rank{r}.npy")
        for s in range(got.shape[0]):
            ok, max_abs, rel = tolerance_ok(got[s], ref[s])
            assert ok, f"rank {r} step {s}: max abs {max_abs:.3g} rel {rel:.3g}"


def test_head_split_single_gpu_matches_oracle(cuda):
    """The head-split item layout (two kv heads per item, spanning layers when a rank holds one
    kv head per layer) on one GPU, for the shares of 2, 4 and 8 ranks emulated one after the
    other, with a world-1 gather: each share's output equals the oracle's heads of it."""
    import torch

    import oracle
    from _cases import tolerance_ok
    from tailorquantkernel_b200 import shard, tqk
    port_ = oracle.Oracle("port")
    layers, nq, nkv, hd, pos = 4, 32, 8, 128, 300
    mt = pos + 1
    rng = np.random.default_rng(91)
    kf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
    vf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
    kf[:, :, pos:] = 0.0
    vf[:, :, pos:] = 0.0
    kp_full, vp_full = port_.quantize_rows(kf), port_.quantize_rows(vf)
    q = rng.standard_normal((layers, nq * hd), dtype=np.float32)
    k = rng.standard_normal((layers, nkv * hd), dtype=np.float32)
    v = rng.standard_normal((layers, nkv * hd), dtype=np.float32)
    ref = np.empty((layers, nq * hd), np.float32)
    kp_ref, vp_ref = kp_full.copy(), vp_full.copy()
    for layer in range(layers):
        assert port_.store_kv(kp_ref[layer], vp_ref[layer], nkv, hd, mt, pos, k[layer], v[layer]) == 0
        ref[layer] = port_.attend(kp_ref[layer], vp_ref[layer], nq, nkv, hd, mt, pos, q[layer])
    for world in (2, 4, 8):
        per, group = nkv // world, nq // nkv
        for rank in range(world):
            lo = rank * per
            kl = torch.from_numpy(np.ascontiguousarray(kp_full[:, lo:lo + per])).cuda()
            vl = torch.from_numpy(np.ascontiguousarray(vp_full[:, lo:lo + per])).cuda()
            ql = torch.from_numpy(shard.head_split_slice(q, layers, nq, hd, rank, world)).cuda()
            kn = torch.from_numpy(shard.head_split_slice(k, layers, nkv, hd, rank, world)).cuda()
            vn = torch.from_numpy(shard.head_split_slice(v, layers, nkv, hd, rank, world)).cuda()
            chunk = per * group * hd
            box = tqk.peer_buffer_alloc(tqk.tqk_gather_mailbox_bytes(1, layers, chunk))
            try:
                out = torch.full((layers, chunk), float("nan"), device="cuda")
                slot = tqk.gather_slot(box, layers, chunk, 1)
                tqk.decode(shard.head_split_args(tqk, kl, vl, layers, nq, nkv, hd, mt, world, ql, slot, len0=pos + 1,
                                                 k_new=kn, v_new=vn))
                tqk.exchange_gather(layers, chunk, 1, 0, [box], 1, out)
                torch.cuda.synchronize()
            finally:
                tqk.peer_buffer_free(box)
            want = shard.head_split_slice(ref, layers, nq, hd, rank, world)
            ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), want)
            assert ok, f"world {world} rank {rank}: max abs {max_abs:.3g} rel {rel:.3g}"
            assert np.array_equal(kl.cpu().numpy(), kp_ref[:, lo:lo + per])
            assert np.array_equal(vl.cpu().numpy(), vp_ref[:, lo:lo + per])
    assert tqk.device_status() == 0


def test_gather_wait_times_out_without_peer(cuda):
    """tqk_exchange_gather's bounded wait, as the exchange's: a two-rank gather whose peer
    mailbox nobody writes gives up after about a second, records the timeout and returns;
    a one-rank gather afterwards works."""
    import time

    import torch
    from tailorquantkernel_b200 import tqk
    groups, chunk = 4, 256
    boxes = [tqk.peer_buffer_alloc(tqk.tqk_gather_mailbox_bytes(2, groups, chunk)) for _ in range(2)]
    solo = tqk.peer_buffer_alloc(tqk.tqk_gather_mailbox_bytes(1, groups, chunk))
    try:
        assert tqk.device_status(clear=True) == 0
        out = torch.full((groups, 2 * chunk), float("nan"), device="cuda")
        t0 = time.time()
        tqk.exchange_gather(groups, chunk, 2, 0, boxes, 1, out)
        torch.cuda.synchronize()
        assert 0.5 < time.time() - t0 < 30
        assert tqk.device_status(clear=True) == 1
        assert torch.isnan(out).all()
        out1 = torch.full((groups, chunk), float("nan"), device="cuda")
        tqk.exchange_gather(groups, chunk, 1, 0, [solo], 1, out1)  # a zeroed slot gathers zeros
        torch.cuda.synchronize()
        assert torch.count_nonzero(out1).item() == 0
        with pytest.raises(tqk.TQKError):
            tqk.exchange_gather(groups, 3, 1, 0, [solo], 1, out1)  # chunk not a multiple of 4
        assert tqk.device_status() == 0
    finally:
        for b in boxes + [solo]:
            tqk.peer_buffer_free(b)


def test_fused_gather_two_ranks_emulated_on_one_gpu(cuda):
    """tqk_decode_q8_gather with two ranks emulated one after the other on one GPU (both
    ranks' pair buffers are local, so nothing waits on another kernel): each rank's decode of
    its kv heads writes its units' outputs into both buffers as {value, epoch} pairs; then
    tqk_gather_collect of each buffer passes at once and gives the whole output, within the
    attention tolerance of the oracle; then a second step of the other parity with different
    q, k and v."""
    import torch

    import oracle
    from _cases import tolerance_ok
    from tailorquantkernel_b200 import shard, tqk
    port_ = oracle.Oracle("port")
    layers, nq, nkv, hd, pos, world = 4, 32, 8, 128, 500, 2
    mt, per, group = pos + 2, nkv // world, nq // nkv
    rng = np.random.default_rng(92)
    kf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
    vf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
    kf[:, :, pos:] = 0.0
    vf[:, :, pos:] = 0.0
    kp_full, vp_full = port_.quantize_rows(kf), port_.quantize_rows(vf)
    chunk = per * group
    n = layers * world * chunk * hd
    pair_bytes = (n * 8 + 255) // 256 * 256
    boxes = [tqk.peer_buffer_alloc(2 * pair_bytes) for _ in range(world)]
    try:
        planes = []
        for r in range(world):
            lo = r * per
            planes.append((torch.from_numpy(np.ascontiguousarray(kp_full[:, lo:lo + per])).cuda(),
                           torch.from_numpy(np.ascontiguousarray(vp_full[:, lo:lo + per])).cuda()))
        kout = torch.empty(layers, chunk * hd, device="cuda")
        for step in range(2):
            epoch = step + 1
            off = (epoch & 1) * pair_bytes
            q = rng.standard_normal((layers, nq * hd), dtype=np.float32)
            k = rng.standard_normal((layers, nkv * hd), dtype=np.float32)
            v = rng.standard_normal((layers, nkv * hd), dtype=np.float32)
            for r in range(world):
                ql = torch.from_numpy(shard.head_split_slice(q, layers, nq, hd, r, world)).cuda()
                kn = torch.from_numpy(shard.head_split_slice(k, layers, nkv, hd, r, world)).cuda()
                vn = torch.from_numpy(shard.head_split_slice(v, layers, nkv, hd, r, world)).cuda()
                args = shard.head_split_args(tqk, planes[r][0], planes[r][1], layers, nq, nkv, hd, mt, world, ql, kout,
                                             len0=pos + step + 1, k_new=kn, v_new=vn)
                tqk.decode_gather(args, tqk.gather_dst(world, r, [b + off for b in boxes], chunk, epoch))
                torch.cuda.synchronize()
            ref = np.empty((layers, nq * hd), np.float32)
            for layer in range(layers):
                assert port_.store_kv(kp_full[layer], vp_full[layer], nkv, hd, mt, pos + step, k[layer], v[layer]) == 0
                ref[layer] = port_.attend(kp_full[layer], vp_full[layer], nq, nkv, hd, mt, pos + step, q[layer])
            for r in range(world):
                out = torch.full((layers, nq * hd), float("nan"), device="cuda")
                tqk.gather_collect(boxes[r] + off, n, epoch, out)
                torch.cuda.synchronize()
                ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), ref)
                assert ok, f"step {step} buffer {r}: max abs {max_abs:.3g} rel {rel:.3g}"
                ep = tqk.device_array(boxes[r] + off, (n, 2), "int32")[:, 1].cpu().numpy()
                assert (ep == epoch).all()
            for r in range(world):
                lo = r * per
                assert np.array_equal(planes[r][0].cpu().numpy(), kp_full[:, lo:lo + per])
                assert np.array_equal(planes[r][1].cpu().numpy(), vp_full[:, lo:lo + per])
        assert tqk.device_status() == 0
    finally:
        for b in boxes:
            tqk.peer_buffer_free(b)


def test_gather_collect_times_out_and_recovers(cuda):
    """tqk_gather_collect on pairs that never show the epoch gives up after about a second,
    records the timeout in the device error word and returns; on pairs that show it, it
    writes their values."""
    import time

    import torch
    from tailorquantkernel_b200 import tqk
    n = 3000
    box = tqk.peer_buffer_alloc(n * 8)
    try:
        assert tqk.device_status(clear=True) == 0
        out = torch.empty(n, device="cuda")
        t0 = time.time()
        tqk.gather_collect(box, n, 1, out)  # zeroed pairs: epoch 1 never arrives
        torch.cuda.synchronize()
        assert 0.5 < time.time() - t0 < 30
        assert tqk.device_status(clear=True) == 1
        pairs = tqk.device_array(box, (n, 2), "int32")
        vals = torch.arange(n, device="cuda", dtype=torch.float32) * 0.5
        pairs[:, 0] = vals.view(torch.int32)
        pairs[:, 1] = 7
        tqk.gather_collect(box, n, 7, out)
        torch.cuda.synchronize()
        assert torch.equal(out, vals)
        assert tqk.device_status() == 0
        with pytest.raises(tqk.TQKError):
            tqk.gather_collect(box + 4, n - 1, 7, out)  # not 8-byte aligned
    finally:
        tqk.peer_buffer_free(box)


def _rank_main_fused(rank, world, port, result_dir):
    """The fused kv-head-group split (shard.PeerHeadSplit) on `world` GPUs: three steps at
    consecutive positions, so both parity buffers are used and one is reused."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle
    from tailorquantkernel_b200 import shard, tqk
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    hs = None
    try:
        port_ = oracle.Oracle("port")
        layers, nq, nkv, hd, pos, steps = 3, 32, 8, 128, 700, 3
        mt, per, group = pos + steps, nkv // world, nq // nkv
        rng = np.random.default_rng(93)
        kf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
        vf = rng.standard_normal((layers, nkv, mt, hd), dtype=np.float32)
        kf[:, :, pos:] = 0.0
        vf[:, :, pos:] = 0.0
        kp_full, vp_full = port_.quantize_rows(kf), port_.quantize_rows(vf)
        qs = rng.standard_normal((steps, layers, nq * hd), dtype=np.float32)
        ks = rng.standard_normal((steps, layers, nkv * hd), dtype=np.float32)
        vs = rng.standard_normal((steps, layers, nkv * hd), dtype=np.float32)
        lo = rank * per
        kl = torch.from_numpy(np.ascontiguousarray(kp_full[:, lo:lo + per])).cuda()
        vl = torch.from_numpy(np.ascontiguousarray(vp_full[:, lo:lo + per])).cuda()
        kout = torch.empty(layers, per * group * hd, device="cuda")
        outs = []
        for s in range(steps):
            q = torch.from_numpy(shard.head_split_slice(qs[s], layers, nq, hd, rank, world)).cuda()
            k = torch.from_numpy(shard.head_split_slice(ks[s], layers, nkv, hd, rank, world)).cuda()
            v = torch.from_numpy(shard.head_split_slice(vs[s], layers, nkv, hd, rank, world)).cuda()
            args = shard.head_split_args(tqk, kl, vl, layers, nq, nkv, hd, mt, world, q, kout, len0=pos + s + 1,
                                         k_new=k, v_new=v)
            if hs is None:
                hs = shard.PeerHeadSplit(dist, tqk, layers, per * group, hd)
            outs.append(hs.step(args).clone())
        torch.cuda.synchronize()
        refs = []
        for s in range(steps):
            ref = np.empty((layers, nq * hd), np.float32)
            for layer in range(layers):
                assert port_.store_kv(kp_full[layer], vp_full[layer], nkv, hd, mt, pos + s, ks[s, layer],
                                      vs[s, layer]) == 0
                ref[layer] = port_.attend(kp_full[layer], vp_full[layer], nq, nkv, hd, mt, pos + s, qs[s, layer])
            refs.append(ref)
        rows_ok = np.array_equal(kl.cpu().numpy(), kp_full[:, lo:lo + per]) and \
            np.array_equal(vl.cpu().numpy(), vp_full[:, lo:lo + per])
        np.save(os.path.join(result_dir, f"fused_rank{rank}.npy"),
                np.stack([np.stack([o.cpu().numpy() for o in outs]), np.stack(refs)]))
        with open(os.path.join(result_dir, f"fused_rank{rank}.txt"), "w") as f:
            f.write(f"{int(rows_ok)} {tqk.device_status()}")
    finally:
        if hs is not None:
            hs.close()
        dist.destroy_process_group()


def test_fused_head_split_all_gpus(cuda, tmp_path):
    """The fused kv-head-group split over every GPU of the box (2, 4 or 8 ranks; the 8 kv heads
    must divide) against the oracle (three steps, both parities)."""
    import torch
    import torch.multiprocessing as mp
    from _cases import tolerance_ok
    n = torch.cuda.device_count()
    world = 8 if n >= 8 else 4 if n >= 4 else 2
    if n < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_rank_main_fused, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        rows_ok, status = (int(x) for x in open(tmp_path / f"fused_rank{r}.txt").read().split())
        assert rows_ok == 1 and status == 0, (r, rows_ok, status)
        got, ref = np.load(tmp_path / f"fused_rank{r}.npy")
        for s in range(got.shape[0]):
            ok, max_abs, rel = tolerance_ok(got[s], ref[s])
            assert ok, f"rank {r} step {s}: max abs {max_abs:.3g} rel {rel:.3g}"
