"""Host logic of the multi-GPU paths (tailorquantkernel_b200.shard), on CPU.

The partitions (sequence ranges, kv-head groups, length-balanced batches) are
checked directly; the sequence split's exchange runs as two gloo ranks on
127.0.0.1 with the ranks' partial records computed in float64 by the test
itself (standing in for the device's TQK_OUT_PARTIAL output, same layout
{acc[head_dim], m (natural log), l}).  The merged result must equal attention
over the whole context.
"""
import os
import socket

import numpy as np
import pytest

from tailorquantkernel_b200 import shard


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("n", [0, 1, 63, 64, 65, 4097, 131072])
def test_seq_range_partitions_the_context(n, world):
    covered = []
    for r in range(world):
        s, ln = shard.seq_range(n, r, world)
        assert ln >= 0 and (ln == 0 or s % shard.TILE_TOKENS == 0)
        covered.extend(range(s, s + ln))
    assert covered == list(range(n))


def test_seq_range_balance_and_errors():
    lens = [shard.seq_range(131072, r, 8)[1] for r in range(8)]
    assert lens == [16384] * 8
    with pytest.raises(ValueError):
        shard.seq_range(10, 2, 2)


def test_head_range():
    assert [shard.head_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 2), (4, 2), (6, 2)]
    with pytest.raises(ValueError):
        shard.head_range(8, 0, 3)


def test_batch_shard_is_a_balanced_partition():
    rng = np.random.default_rng(3)
    lens = rng.integers(512, 8193, 64)
    for world in (1, 2, 4, 8):
        owned = shard.batch_shard(lens, world)
        assert sorted(i for o in owned for i in o) == list(range(64))
        loads = [int(lens[o].sum()) for o in owned]
        assert max(loads) - min(loads) <= int(lens.max())


def _attention_partial(q, k, v, lo, hi, scale):
    """float64 {acc, m, l} per q head over tokens [lo, hi) (empty -> m = -inf, l = 0)."""
    nq, hd = q.shape
    group = nq // k.shape[0]
    rec = np.zeros((nq, hd + 2))
    for h in range(nq):
        kh, vh = k[h // group, lo:hi], v[h // group, lo:hi]
        if hi <= lo:
            rec[h, hd] = -np.inf
            continue
        s = kh @ q[h] * scale
        m = s.max()
        p = np.exp(s - m)
        rec[h, :hd] = p @ vh
        rec[h, hd], rec[h, hd + 1] = m, p.sum()
    return rec


def _merge(parts):
    """Log-sum-exp merge of [world][nq][hd+2] records (what tqk_merge_partials computes)."""
    hd = parts.shape[2] - 2
    m = parts[:, :, hd].max(axis=0)
    w = np.where(parts[:, :, hd + 1] > 0, np.exp(parts[:, :, hd] - m), 0.0)
    l = (w * parts[:, :, hd + 1]).sum(axis=0)
    return (w[:, :, None] * parts[:, :, :hd]).sum(axis=0) / l[:, None]


def _problem(n):
    rng = np.random.default_rng(11)
    return (rng.standard_normal((8, 128)), rng.standard_normal((2, n, 128)), rng.standard_normal((2, n, 128)))


def _rank_main(rank, world, port, n, result_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = _problem(n)
        s, ln = shard.seq_range(n, rank, world)
        local = torch.from_numpy(_attention_partial(q, k, v, s, s + ln, 128 ** -0.5).reshape(-1))
        gathered = shard.gather_partials(dist, local)
        assert tuple(gathered.shape) == (world, local.numel())
        merged = _merge(gathered.numpy().reshape(world, 8, 130))
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), merged)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n", [1000, 40])  # 40 < 2 tiles: rank 1 gets an empty range
def test_two_gloo_ranks_sequence_split(tmp_path, n):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), n, str(tmp_path)), nprocs=world, join=True)
    q, k, v = _problem(n)
    full = _attention_partial(q, k, v, 0, n, 128 ** -0.5)
    ref = full[:, :128] / full[:, 129:130]
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


# ---------------------------------------------------------------------------
# kv-head-group split (bench config 2 on N GPUs): layout and gather
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_split_items_keep_the_gqa_mapping(world):
    """shard.head_split_args hands a rank's kv heads of every layer to the kernel as items of two
    kv heads.  Walking the items the way the kernel does (item i, kv head j of the item, q head h of
    the item -> kv head h // group) must visit every (layer, q head) of the rank exactly once, each
    paired with its own layer's kv head h_global // group, at the offsets the planes, q, out and the
    appended rows really have."""
    from tailorquantkernel_b200 import tqk
    layers, nq, nkv, hd, mt = 32, 32, 8, 128, 4097
    group, nb, per = nq // nkv, hd // 32, nkv // world
    a = shard.head_split_args(tqk, 1 << 20, 1 << 21, layers, nq, nkv, hd, mt, world, 1 << 22, 1 << 23, len0=mt,
                              k_new=1 << 24, v_new=1 << 25)
    assert a.n_kv_heads * a.n_items == layers * per and a.n_q_heads == a.n_kv_heads * group
    assert a.max_tokens == mt and a.len0 == mt and a.head_dim == hd
    seen = set()
    for rank in range(world):
        for i in range(a.n_items):
            for h in range(a.n_q_heads):
                kvh = h // group  # the kernel's GQA rule inside an item
                plane_row = (i * a.item_stride) // (mt * nb) + kvh          # kv-head row of the rank's planes
                q_row = (i * a.q_item_stride) // hd + h                     # q-head row of the rank's q / out
                assert a.q_item_stride == a.out_item_stride
                assert (i * a.kv_new_item_stride) // hd + kvh == plane_row  # appended row of that kv head
                layer, local_kv = divmod(plane_row, per)
                q_layer, local_q = divmod(q_row, per * group)
                assert q_layer == layer and local_q // group == local_kv
                seen.add((rank, layer, rank * per * group + local_q))
    assert len(seen) == world * layers * per * group == layers * nq  # every (layer, q head) of the job once


def _rank_main_heads(rank, world, port, result_dir):
    """float64 attention of this rank's kv heads (every layer), gathered with gloo into the
    [layers][world][chunk] layout tqk_exchange_gather writes."""
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers, nq, nkv, hd, n = 3, 8, 4, 16, 50
        rng = np.random.default_rng(12)
        q = rng.standard_normal((layers, nq * hd))
        k = rng.standard_normal((layers, nkv, n, hd))
        v = rng.standard_normal((layers, nkv, n, hd))
        per, group = nkv // world, nq // nkv
        ql = shard.head_split_slice(q, layers, nq, hd, rank, world).reshape(layers, per * group, hd)
        lo = rank * per
        local = np.empty((layers, per * group * hd))
        for layer in range(layers):
            rec = _attention_partial(ql[layer], k[layer, lo:lo + per], v[layer, lo:lo + per], 0, n, hd ** -0.5)
            local[layer] = (rec[:, :hd] / rec[:, hd + 1:hd + 2]).reshape(-1)
        parts = [torch.empty(layers, per * group * hd, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(local))
        out = torch.stack(parts, 1).reshape(layers, nq * hd)  # out[g][r][:] = rank r's group g
        np.save(os.path.join(result_dir, f"heads{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_head_split(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank_main_heads, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    layers, nq, nkv, hd, n = 3, 8, 4, 16, 50
    rng = np.random.default_rng(12)
    q = rng.standard_normal((layers, nq * hd))
    k = rng.standard_normal((layers, nkv, n, hd))
    v = rng.standard_normal((layers, nkv, n, hd))
    ref = np.empty((layers, nq * hd))
    for layer in range(layers):
        rec = _attention_partial(q[layer].reshape(nq, hd), k[layer], v[layer], 0, n, hd ** -0.5)
        ref[layer] = (rec[:, :hd] / rec[:, hd + 1:hd + 2]).reshape(-1)
    for r in range(world):
        np.testing.assert_allclose(np.load(tmp_path / f"heads{r}.npy"), ref, rtol=1e-12, atol=1e-12)


# ---------------------------------------------------------------------------
# failure detection on the host: a rank that leaves between steps
# ---------------------------------------------------------------------------
def _rank_main_leaver(rank, world, port, result_dir):
    """Rank 1 runs one step and then leaves (returns without taking part in the next step's
    collective, as a crashed or killed rank would); rank 0's next exchange must end with an
    error within the process group's short timeout instead of waiting for good."""
    import time
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    q, k, v = _problem(200)
    s, ln = shard.seq_range(200, rank, world)
    local = torch.from_numpy(_attention_partial(q, k, v, s, s + ln, 128 ** -0.5).reshape(-1))
    shard.gather_partials(dist, local)  # step 1: every rank
    if rank == 1:
        return  # leaves between steps, with nothing in flight
    t0 = time.time()
    try:
        shard.gather_partials(dist, local)  # step 2: the peer never joins
        outcome = "completed"
    except Exception as e:  # noqa: BLE001  (gloo raises RuntimeError / DistBackendError)
        outcome = f"error {type(e).__name__}"
    with open(os.path.join(result_dir, "leaver.txt"), "w") as f:
        f.write(f"{outcome}\n{time.time() - t0:.2f}\n")


def test_rank_leaving_between_steps_errors_instead_of_hanging(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main_leaver, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    outcome, waited = open(tmp_path / "leaver.txt").read().split("\n")[:2]
    assert outcome.startswith("error"), outcome
    assert float(waited) < 60.0
