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
