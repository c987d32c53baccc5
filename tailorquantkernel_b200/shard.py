"""Multi-GPU partitioning of the Q8 decode attention (one process per GPU).

The reference runs on one CPU; its decode attention has no cross-device
dimension.  On a box of B200s the work splits three ways, only one of which
needs a collective:

* by kv-head group (one sequence, the kv heads and their q-head groups divided
  over the ranks): every rank writes a disjoint slice of the output heads;
* by batch (many sequences, divided over the ranks, balanced by length):
  every rank owns whole sequences;
* by sequence (one very long context, contiguous token ranges per rank): each
  rank computes log-sum-exp partials {acc, m, l} of its range
  (TQK_OUT_PARTIAL) and the ranks exchange and merge them -- the only
  exchange step.  PeerExchange does it in one kernel over peer memory
  (tqk_exchange_merge: the decode writes into the rank's own mailbox, a flag
  per epoch in every peer, the peers' records read over NVLink and merged);
  seqsplit_attend does it with an NCCL all-gather and tqk_merge_partials.

The functions here are pure host logic plus torch.distributed calls; the GPU
work goes through libtqk's C ABI (tailorquantkernel_b200.tqk).
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

TILE_TOKENS = 64  # the decode kernels' tile: ranges start on tile boundaries


def seq_range(n_tokens: int, rank: int, world: int, align: int = TILE_TOKENS) -> Tuple[int, int]:
    """Token range [start, start + length) of `rank` when a context of n_tokens is
    split into `world` contiguous ranges.  Range starts fall on multiples of
    `align` (whole decode tiles); the last rank takes the remainder.  Ranges
    are disjoint and cover [0, n_tokens); a rank may get an empty range when
    n_tokens is smaller than world * align."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_tokens < 0:
        raise ValueError("n_tokens must be >= 0")
    tiles = (n_tokens + align - 1) // align
    start_tile = tiles * rank // world
    end_tile = tiles * (rank + 1) // world
    start = min(start_tile * align, n_tokens)
    end = min(end_tile * align, n_tokens) if rank + 1 < world else n_tokens
    return start, end - start


def head_range(n_kv: int, rank: int, world: int) -> Tuple[int, int]:
    """kv heads [start, start + count) of `rank` for the kv-head-group split; the
    q heads of a kv head travel with it.  n_kv must divide evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_kv % world:
        raise ValueError(f"{n_kv} kv heads do not divide over {world} ranks")
    per = n_kv // world
    return rank * per, per


def head_split_args(tqk, k_local, v_local, n_layers: int, n_q: int, n_kv: int, head_dim: int, max_tokens: int,
                    world: int, q_local, out_local, *, len0: int, k_new=None, v_new=None):
    """Decode arguments of one rank's share of the kv-head-group split of n_layers
    layers (the reference's per-kv-head loop of attend_q8,
    model/attention_layer.c:134-149, divided over GPUs).

    The rank holds per = n_kv / world kv heads of every layer, with their
    per * group q heads (group = n_q / n_kv):
      k_local / v_local: Q8 planes [n_layers * per][max_tokens][head_dim/32];
      q_local, out_local: [n_layers][per * group][head_dim] floats;
      k_new / v_new (optional fused append at len0 - 1): [n_layers][per][head_dim].
    The share is handed to the kernel as items of two kv heads -- one kv head of
    two consecutive layers when per == 1 -- so that the kernel that packs two kv
    heads per CTA runs at every world size; the output layout does not change."""
    if n_kv % world or n_q % n_kv:
        raise ValueError(f"{n_q} q / {n_kv} kv heads do not split over {world} ranks")
    per, group = n_kv // world, n_q // n_kv
    heads = n_layers * per
    kv_item = 2 if heads % 2 == 0 else 1
    nb = head_dim // 32
    return tqk.decode_args(k_local, v_local, kv_item * group, kv_item, head_dim, max_tokens, q_local, out_local,
                           n_items=heads // kv_item, item_stride_blocks=kv_item * max_tokens * nb, len0=len0,
                           q_item_stride=kv_item * group * head_dim, out_item_stride=kv_item * group * head_dim,
                           k_new=k_new, v_new=v_new, kv_new_item_stride=kv_item * head_dim)


def head_split_slice(x, n_layers: int, n_heads: int, head_dim: int, rank: int, world: int):
    """Rank `rank`'s heads of a per-layer head-major array x [n_layers][n_heads * head_dim] (numpy
    or torch): [n_layers][n_heads/world * head_dim], contiguous.  For q (n_heads = n_q) this is the
    q heads of the rank's kv heads; for k_new / v_new (n_heads = n_kv) its kv heads."""
    per = n_heads // world
    y = x.reshape(n_layers, n_heads, head_dim)[:, rank * per:(rank + 1) * per]
    y = y.reshape(n_layers, per * head_dim)
    return y.contiguous() if hasattr(y, "contiguous") else y.copy()


def batch_shard(lens: Sequence[int], world: int) -> List[List[int]]:
    """Sequences of a ragged batch per rank, balanced by total length: longest
    first, each to the currently lightest rank (ties to the lower rank).  Every
    sequence index appears exactly once; each rank's list is in ascending order."""
    if world <= 0:
        raise ValueError("world must be positive")
    loads = [0] * world
    owned: List[List[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda j: (-int(lens[j]), j)):
        r = min(range(world), key=lambda w: (loads[w], w))
        owned[r].append(i)
        loads[r] += int(lens[i])
    return [sorted(o) for o in owned]


def gather_partials(dist, local, group=None):
    """All-gathers each rank's partial records (a contiguous tensor of the same
    shape on every rank) into one [world, *local.shape] tensor, rank order."""
    import torch
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "gloo":  # host ranks (tests): list form
        dist.all_gather(list(out.unbind(0)), local.contiguous(), group=group)
    else:
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def seqsplit_attend(dist, tqk, k_local, v_local, n_q: int, n_kv: int, head_dim: int, n_local: int, q, out,
                    partial, gathered=None, stream=None):
    """One decode step of a context split by sequence: attention of q over this
    rank's n_local tokens as partials, all-gather, log-sum-exp merge into out.

    k_local / v_local: this rank's Q8 planes [n_kv][n_local][head_dim/32];
    partial: device float tensor [n_q * (head_dim + 2)] for this rank's record;
    gathered: optional preallocated [world, n_q * (head_dim + 2)] tensor.
    Every rank ends with the full output."""
    args = tqk.decode_args(k_local, v_local, n_q, n_kv, head_dim, max(n_local, 1), q, partial, len0=n_local,
                           out_mode=tqk.OUT_PARTIAL)
    tqk.decode(args, stream=stream)
    world = dist.get_world_size()
    if gathered is None:
        gathered = gather_partials(dist, partial)
    else:
        dist.all_gather_into_tensor(gathered, partial)
    tqk.merge_partials(gathered, world, n_q * (head_dim + 2), n_q, head_dim, out, stream=stream)
    return out


class _PeerMailboxes:
    """One mailbox per rank (tqk_peer_buffer_alloc, `nbytes` bytes), mapped in every
    other rank through CUDA IPC handles swapped once with torch.distributed, and
    the epoch counter of the flag protocol that tqk_exchange_merge and
    tqk_exchange_gather share.  close() frees everything once every rank has
    finished its last step."""

    def __init__(self, dist, tqk, nbytes: int, group=None):
        import torch
        self.tqk, self.dist, self.group = tqk, dist, group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.local = tqk.peer_buffer_alloc(nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, tqk.ipc_get_handle(self.local), group=group)
        self.opened = []
        self.mailboxes = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.mailboxes.append(self.local)
            else:
                ptr = tqk.ipc_open_handle(h)
                self.opened.append(ptr)
                self.mailboxes.append(ptr)
        self.epoch = 0
        torch.cuda.synchronize()
        dist.barrier(group=group)  # every mailbox is zeroed and mapped before the first step

    def close(self):
        """Unmaps the peers' mailboxes and frees this rank's.  A peer's last step
        reads this rank's mailbox over NVLink after it has seen this rank's flag,
        which can be after this rank has finished its own step: so every rank
        first waits for its own work and then for every other rank (a barrier)
        before anything is unmapped or freed.  Every rank must call close()."""
        import torch
        if self.local is None:
            return
        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)
        for ptr in self.opened:
            self.tqk.ipc_close_handle(ptr)
        self.opened = []
        self.tqk.peer_buffer_free(self.local)
        self.local = None


class PeerExchange(_PeerMailboxes):
    """The sequence split's exchange step over peer memory for ranks on the GPUs of
    one box.  Per step: begin() gives the slot this rank's partial records go to,
    end() launches tqk_exchange_merge.  Every rank must run the same steps in the
    same order, and close() on every rank at the end."""

    def __init__(self, dist, tqk, n_heads: int, head_dim: int, group=None):
        self.n_heads, self.head_dim = n_heads, head_dim
        world = dist.get_world_size(group)
        nbytes = tqk.tqk_exchange_mailbox_bytes(world, n_heads, head_dim)
        if nbytes == 0:
            raise ValueError(f"no mailbox layout for world {world}, {n_heads} heads of {head_dim}")
        super().__init__(dist, tqk, nbytes, group)

    def begin(self) -> int:
        """Starts the next step: the device address its partial records must be written to."""
        self.epoch += 1
        return self.tqk.exchange_slot(self.local, self.n_heads, self.head_dim, self.epoch)

    def end(self, out, stream=None):
        """Merges every rank's records of the step into out (all ranks get the same)."""
        self.tqk.exchange_merge(self.n_heads, self.head_dim, self.world, self.rank, self.mailboxes, self.epoch, out,
                                stream=stream)
        return out


class PeerGather(_PeerMailboxes):
    """The kv-head-group split's gather over peer memory: each rank attends to its
    kv heads (and their q heads) of every layer and writes its output slice,
    [n_groups][chunk_floats] floats, to the slot begin() returns; end() launches
    tqk_exchange_gather, after which out is [n_groups][world][chunk_floats] on
    every rank (for the decode: [layers][n_q_heads][head_dim])."""

    def __init__(self, dist, tqk, n_groups: int, chunk_floats: int, group=None):
        self.n_groups, self.chunk = n_groups, chunk_floats
        world = dist.get_world_size(group)
        nbytes = tqk.tqk_gather_mailbox_bytes(world, n_groups, chunk_floats)
        if nbytes == 0:
            raise ValueError(f"no gather mailbox for world {world}, {n_groups} groups of {chunk_floats} floats")
        super().__init__(dist, tqk, nbytes, group)

    def begin(self) -> int:
        self.epoch += 1
        return self.tqk.gather_slot(self.local, self.n_groups, self.chunk, self.epoch)

    def end(self, out, stream=None):
        self.tqk.exchange_gather(self.n_groups, self.chunk, self.world, self.rank, self.mailboxes, self.epoch, out,
                                 stream=stream)
        return out


class PeerHeadSplit(_PeerMailboxes):
    """The kv-head-group split with the gather fused into the decode
    (tqk_decode_q8_gather).  Every rank's peer buffer holds two pair buffers
    by step parity, [n_groups][world][chunk_heads][head_dim] {value, epoch}
    pairs each.  A step decodes this rank's heads, the decode writing every
    unit's output into every rank's pair buffer of the step's parity, then
    tqk_gather_collect waits until every local pair shows the step's epoch and
    writes the plain output [n_groups][world * chunk_heads * head_dim] floats.
    Parity buffers make the reuse safe: a rank's step e + 2 writes a buffer
    only after it has collected its step e + 1, which needs every rank's pairs
    of e + 1, which each rank writes only after it has collected step e."""

    def __init__(self, dist, tqk, n_groups: int, chunk_heads: int, head_dim: int, group=None):
        import torch
        world = dist.get_world_size(group)
        self.n_groups, self.chunk_heads, self.head_dim = n_groups, chunk_heads, head_dim
        self.n = n_groups * world * chunk_heads * head_dim
        self.pair_bytes = (self.n * 8 + 255) // 256 * 256
        super().__init__(dist, tqk, 2 * self.pair_bytes, group)
        self.out = torch.empty(n_groups, world * chunk_heads * head_dim, device="cuda")

    def step(self, args, workspace=None, stream=None):
        """One step: returns the output tensor (ready once the stream reaches this point)."""
        self.epoch += 1
        off = (self.epoch & 1) * self.pair_bytes
        dst = self.tqk.gather_dst(self.world, self.rank, [m + off for m in self.mailboxes], self.chunk_heads,
                                  self.epoch)
        self.tqk.decode_gather(args, dst, workspace=workspace, stream=stream)
        self.tqk.gather_collect(self.local + off, self.n, self.epoch, self.out, stream=stream)
        return self.out


def seqsplit_attend_p2p(exchange: PeerExchange, tqk, k_local, v_local, n_q: int, n_kv: int, head_dim: int,
                        n_local: int, q, out, stream=None):
    """seqsplit_attend with the exchange over peer memory: decode of this rank's
    range straight into its mailbox slot, then one tqk_exchange_merge launch."""
    slot = exchange.begin()
    args = tqk.decode_args(k_local, v_local, n_q, n_kv, head_dim, max(n_local, 1), q, slot, len0=n_local,
                           out_mode=tqk.OUT_PARTIAL)
    tqk.decode(args, stream=stream)
    return exchange.end(out, stream=stream)
