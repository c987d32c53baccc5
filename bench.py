"""Benchmark of the B200 Q8 GQA decode attention (the reference's attend_q8 +
store_kv hot path) on BASELINE.json's headline configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

Default workload (config 2, Llama-3-8B-shaped decode): 32 layers, 32 q / 8 kv
heads, head_dim 128, Q8 KV cache of 4096 positions plus the token appended each
step (n = 4097), q ~ N(0,1) rotated by RoPE (theta 500000) at position 4096.
One step = one token: for every layer the fused kernel appends the new K/V row
(bit-exact Q8) and attends -- a single multi-layer launch of libtqk.so's
tqk_decode_q8.  K/V per step is 302 MB, larger than the 126 MB L2, so no flush
is needed between steps.

For N > 1 (torchrun, one process per GPU) the same token is divided by kv-head
group: rank r attends to kv heads [r*8/N, (r+1)*8/N) of every layer (with
their q heads); the decode itself pushes every finished unit's output heads into
every rank's buffer over NVLink as value+epoch pairs (tqk_decode_q8_gather), and
tqk_gather_collect closes the step once every pair has arrived: strong scaling, value = tokens / the slowest rank's time.
Each rank then rotates over N copies of its cache slice, so that its working
set stays 302 MB (larger than L2).  The timed region is about 2 s by default so
that the clock sampler sees it several times.

Rank 0 prints one JSON line.  --impl reference times the reference's own CPU
code for the same workload (oracle/_ref/libtqref_avx2.so: the reference's AVX2
attention composed as its attend_q8, all host threads) and prints the same line
with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q8 GQA decode attention tokens/s and HBM GB/s (% peak) at 1/2/4/8 B200"
QK, BB = 32, 36


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (bf16 dense, burst)"
    except Exception:
        return 1590.0, "fallback"


def _traffic_from_profile(name: str):
    """dram bytes per launch recorded from an ncu capture (profiles/<name>.txt)."""
    path = os.path.join(ROOT, "profiles", name + ".txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip().split()[0])
    except OSError:
        pass
    return None


class Clocks:
    """Samples nvidia-smi about every 200 ms on a thread while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        import threading
        self.index = index
        self.rows = []
        self.stop = threading.Event()
        self.first = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        try:
            out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                  "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10).stdout
        except (OSError, subprocess.TimeoutExpired):
            return
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def _run(self):
        while not self.stop.is_set():
            self._sample()
            self.first.set()
            self.stop.wait(0.2)

    def __enter__(self):
        # the first nvidia-smi query (its start-up holds the driver for a while) completes before the
        # timed region starts, so that a short region is not stalled by it; later samples, every
        # 200 ms, fall inside the region
        self.thread.start()
        self.first.wait(15)
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=15)
        if not self.rows:
            self._sample()
        return False

    def summary(self):
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [x for x in (num(r[1]) for r in self.rows) if x is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(self.rows[0][2]),
                "reasons": reasons, "samples": len(self.rows)}


class HostBuffer:
    """Page-locked host memory from cudaHostAlloc (mapped into the device's address space: a kernel
    may read or write it over PCIe) with raw cudaMemcpyAsync copies.  torch's pinned-tensor copy_
    costs tens of microseconds of host time per call, which a synchronised step exposes in full."""

    def __init__(self, nbytes: int):
        from cuda.bindings import runtime as rt
        self.rt, self.nbytes = rt, nbytes
        err, self.ptr = rt.cudaHostAlloc(nbytes, 0)
        if int(err) != 0:
            raise RuntimeError(f"cudaHostAlloc({nbytes}): {err}")

    def fill_from(self, t) -> None:
        """Copies a CUDA tensor's bytes in (set-up, synchronous)."""
        self._check(self.rt.cudaMemcpy(self.ptr, t.data_ptr(), t.numel() * t.element_size(),
                                       self.rt.cudaMemcpyKind.cudaMemcpyDeviceToHost))

    def to_device(self, dev_ptr: int, nbytes: int, stream: int, offset: int = 0) -> None:
        self._check(self.rt.cudaMemcpyAsync(dev_ptr, self.ptr + offset, nbytes,
                                            self.rt.cudaMemcpyKind.cudaMemcpyHostToDevice, stream))

    def from_device(self, dev_ptr: int, nbytes: int, stream: int) -> None:
        self._check(self.rt.cudaMemcpyAsync(self.ptr, dev_ptr, nbytes, self.rt.cudaMemcpyKind.cudaMemcpyDeviceToHost,
                                            stream))

    def _check(self, r):
        err = r[0] if isinstance(r, tuple) else r
        if int(err) != 0:
            raise RuntimeError(f"CUDA runtime: {err}")

    def __del__(self):
        try:
            self.rt.cudaFreeHost(self.ptr)
        except Exception:  # noqa: BLE001  (interpreter shutdown)
            pass


# ---------------------------------------------------------------------------
# synthetic inputs: the reference benches' own generator
# ---------------------------------------------------------------------------
# Every config draws its K/V, q and appended rows (and norm weights, sequence lengths and outlier
# picks) from the stream of the reference's benches: one xorshift64 generator from the seed
# 88172645463325252 read through normal_sample / uniform_open (tools/bench_forward.c:82,199-210).
# A config lays its inputs out as consecutive windows of that stream in a fixed order that does
# not depend on the number of GPUs, so a rank fills its own share of the same global inputs.
# Uniforms come from the same generator from step 2^62 on, which no normal sample reaches.
UNIFORM_BASE = 1 << 62


class LibGen:
    """Our arm: tqk_fill_normal / tqk_fill_uniform (host threads, each jumping ahead to its
    window; the same floats as the reference's sequential generator)."""
    kind = "tqk_fill_normal"

    def normal(self, first: int, n: int, scale: float = 1.0) -> np.ndarray:
        from tailorquantkernel_b200 import tqk
        return tqk.fill_normal(first, n, scale)

    def uniform(self, first: int, n: int) -> np.ndarray:
        from tailorquantkernel_b200 import tqk
        return tqk.fill_uniform(UNIFORM_BASE + first, n)


_XS_MASK = (1 << 64) - 1


def _xs_step(x: int) -> int:
    x ^= (x << 13) & _XS_MASK
    x ^= x >> 7
    return x ^ ((x << 17) & _XS_MASK)


class RefGen:
    """The reference arm: the reference's own normal_sample / uniform_open (oracle/_ref/libtqref_rng.so,
    tools/bench_forward.c compiled in place; sequential), started at any window by jumping the
    xorshift64 state: the step is linear over GF(2), so T^k is applied from its powers of two."""
    kind = "reference normal_sample"
    SEED = 88172645463325252

    def __init__(self, path: str):
        import ctypes
        self._ct = ctypes
        self.lib = ctypes.CDLL(path)
        cols = [_xs_step(1 << i) for i in range(64)]
        self.pows = [cols]
        for _ in range(63):
            m = self.pows[-1]
            self.pows.append([self._apply(m, c) for c in m])

    @staticmethod
    def _apply(m, v: int) -> int:
        r, i = 0, 0
        while v:
            if v & 1:
                r ^= m[i]
            v >>= 1
            i += 1
        return r

    def _state(self, steps: int) -> int:
        x, k = self.SEED, 0
        while steps:
            if steps & 1:
                x = self._apply(self.pows[k], x)
            steps >>= 1
            k += 1
        return x

    def _fill(self, fn, steps: int, n: int) -> np.ndarray:
        ct = self._ct
        out = np.empty(n, np.float32)
        st = ct.c_uint64(self._state(steps))
        fn(ct.byref(st), ct.c_void_p(out.ctypes.data), ct.c_size_t(n))
        return out

    def normal(self, first: int, n: int, scale: float = 1.0) -> np.ndarray:
        out = self._fill(self.lib.tqref_normal_fill, 2 * first, n)
        return out if scale == 1.0 else out * np.float32(scale)

    def uniform(self, first: int, n: int) -> np.ndarray:
        return self._fill(self.lib.tqref_uniform_fill, UNIFORM_BASE + first, n)


def reference_generator():
    """The reference's own generator for the reference arm, else (no reference build here) the
    library's, which gives the same floats."""
    path = os.path.join(ROOT, "oracle", "_ref", "libtqref_rng.so")
    return RefGen(path) if os.path.exists(path) else LibGen()


def outliers(gen, first_u: int, x: np.ndarray) -> np.ndarray:
    """1% of the entries times 8 (config 3): entry i is picked when uniform #(first_u + i) < 0.01."""
    u = gen.uniform(first_u, x.size).reshape(x.shape)
    return np.where(u < np.float32(0.01), x * np.float32(8), x)


def ragged_lengths(gen, count: int, lo: int, hi: int) -> np.ndarray:
    """count lengths uniform on [lo, hi] from uniforms #0.. (u in (0, 1] -> lo + floor(u * (hi - lo + 1)),
    u = 1 clamped to hi)."""
    u = gen.uniform(0, count).astype(np.float64)
    return np.minimum(lo + np.floor(u * (hi - lo + 1)), hi).astype(np.int32)


def device_q8_rows(gen, first: int, rows: int, hd: int, out=None):
    """rows x hd normal samples from `first`, quantised on the device into Q8 rows (the bit-exact
    quantiser): written into `out` ([rows, hd/32*36] uint8, contiguous) or returned."""
    import torch
    from tailorquantkernel_b200 import tqk
    x = torch.from_numpy(gen.normal(first, rows * hd)).cuda().view(rows, hd)
    return tqk.quantize_rows(x, out=out)


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_init(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if n_gpus > 1 and world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} needs torchrun with {n_gpus} processes (WORLD_SIZE={world})")
    return rank, local, world


def pg_init(world, local):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def max_over_ranks(dist, value: float) -> float:
    import torch
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    import torch
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def config2_stream(layers, n_q, n_kv, hd, mt):
    """Config 2's inputs in the reference stream, in this order: for every layer, K then V, every kv
    head's mt rows of hd values; then for every layer that step's q [n_q*hd], k [n_kv*hd] and
    v [n_kv*hd]; then the q and k RMSNorm weights [layers][hd] each (as 1 + 0.1 x, --prologue)."""
    rows = mt * hd
    step = layers * 2 * n_kv * rows
    return {"kv": lambda layer, p, h: ((layer * 2 + p) * n_kv + h) * rows, "step": step,
            "norms": step + layers * (n_q + 2 * n_kv) * hd}


def describe_config2(layers, n_q, n_kv, hd, pos, prologue=False):
    """config entry of config 2 (shared by our arm and the reference arm)."""
    row = hd // QK * BB
    kv_bytes = 2 * layers * n_kv * (pos + 1) * row
    pro = (", q/k RMSNorm + RoPE(500000) fused into the launch (Qwen3-style prologue)" if prologue
           else ", RoPE(500000) q")
    return {"workload": f"config2: Llama-3-8B-shaped Q8 GQA decode, all {layers} layers, {n_q} q / {n_kv} kv heads, "
                        f"head_dim {hd}, context {pos} + 1 appended token (n={pos + 1})" + pro,
            "layers": layers, "seq_len": pos + 1, "kv_bytes_per_token": kv_bytes,
            "l2": f"no flush: inputs larger than L2 ({kv_bytes / 1e6:.0f} MB of K/V per step vs 126 MB L2)"
                  if kv_bytes > 126e6 else f"{kv_bytes / 1e6:.1f} MB of K/V per step (smaller than L2)"}


class Config2:
    """Llama-3-8B-shaped decode: L layers of one sequence, fused append + attention.

    One GPU: one tqk_decode_q8 launch over all layers (32 items of 8 kv heads).
    N GPUs: the kv-head-group split.  Rank r holds kv heads head_range(8, r, N)
    of every layer (its slice of each layer's cache, with their q heads): its
    own launch over those heads, then tqk_exchange_gather, which gives every
    rank the whole output [layers][32 q heads][head_dim] over peer memory.
    The rank's slice is laid out [layers * per][max_tokens][nb], viewed as
    items of two kv heads, so the packed two-heads-per-CTA kernel runs at
    every N (at N = 8 an item is one kv head of two consecutive layers)."""
    name = "config2"
    scaling = "strong"  # one token of one sequence; N GPUs divide its kv heads

    def __init__(self, seed: int, layers=32, n_q=32, n_kv=8, hd=128, pos=4096, prologue=False, rank=0, world=1,
                 dist=None):
        import torch
        from tailorquantkernel_b200 import shard, tqk
        self.tqk, self.world, self.rank = tqk, world, rank
        self.L, self.nq, self.nkv, self.hd, self.pos = layers, n_q, n_kv, hd, pos
        self.prologue = prologue
        self.mt = pos + 1
        self.nb = hd // QK
        group = n_q // n_kv
        kvh0, per = shard.head_range(n_kv, rank, world)
        if prologue and world > 1:
            raise SystemExit("--prologue runs on one GPU only")
        self.per = per
        # on N GPUs each rank holds 1/N of the cache, less than L2 for N >= 4: it rotates over N
        # copies of its slice, one per step, so that its working set stays the whole cache's size
        self.copies = world
        gen = LibGen()
        off = config2_stream(layers, n_q, n_kv, hd, self.mt)
        row = self.nb * BB
        # setup (untimed): this rank's kv heads of the global N(0,1) K/V, quantised on the device
        self.kp = torch.empty(self.copies, layers, per, self.mt, row, dtype=torch.uint8, device="cuda")
        self.vp = torch.empty_like(self.kp)
        for layer in range(layers):
            for p, plane in enumerate((self.kp, self.vp)):
                device_q8_rows(gen, off["kv"](layer, p, kvh0), per * self.mt, hd,
                               out=plane[0, layer].view(per * self.mt, row))
        for c in range(1, self.copies):
            self.kp[c].copy_(self.kp[0])
            self.vp[c].copy_(self.vp[0])
        qkv = gen.normal(off["step"], layers * (n_q + 2 * n_kv) * hd).reshape(layers, n_q + 2 * n_kv, hd)
        q = np.ascontiguousarray(qkv[:, :n_q]).reshape(layers, n_q * hd)  # the same q at every N
        pro = {}
        if prologue:
            # Qwen3-style layer: per-layer q/k RMSNorm weights and the RoPE table of position pos,
            # applied inside the decode launch (q and the appended k arrive un-normalised)
            inv = np.float32(500000.0) ** (-2.0 * np.arange(hd // 2, dtype=np.float32) / np.float32(hd))
            ang = np.float32(pos) * inv.astype(np.float32)
            self.rope_cos = torch.from_numpy(np.tile(np.cos(ang).astype(np.float32), (layers, 1))).cuda()
            self.rope_sin = torch.from_numpy(np.tile(np.sin(ang).astype(np.float32), (layers, 1))).cuda()
            norms = 1 + np.float32(0.1) * gen.normal(off["norms"], 2 * layers * hd).reshape(2, layers, hd)
            self.q_norm = torch.from_numpy(np.ascontiguousarray(norms[0])).cuda()
            self.k_norm = torch.from_numpy(np.ascontiguousarray(norms[1])).cuda()
            pro = dict(q_norm=self.q_norm, k_norm=self.k_norm, norm_item_stride=hd, norm_eps=1e-6,
                       rope_cos=self.rope_cos, rope_sin=self.rope_sin, rope_item_stride=hd // 2)
        else:
            q = rope_np(q, hd, pos, 500000.0)
        q = q.reshape(layers, n_q, hd)[:, kvh0 * group:(kvh0 + per) * group].reshape(layers, per * group * hd)
        k_new = np.ascontiguousarray(qkv[:, n_q + kvh0:n_q + kvh0 + per]).reshape(layers, per * hd)
        v_new = np.ascontiguousarray(qkv[:, n_q + n_kv + kvh0:n_q + n_kv + kvh0 + per]).reshape(layers, per * hd)
        # q, k_new and v_new live in one device buffer, so the end-to-end leg moves a step's inputs
        # with one host-to-device copy (per chunk of layers on one GPU: [layer][q | k_new | v_new])
        lq, lkv = per * group * hd, per * hd
        nq_f, nkv_f = layers * lq, layers * lkv
        self.lrow = lq + 2 * lkv
        self.inbuf = torch.empty(layers, self.lrow, device="cuda")
        self.inbuf[:, :lq].copy_(torch.from_numpy(np.ascontiguousarray(q)))
        self.inbuf[:, lq:lq + lkv].copy_(torch.from_numpy(k_new))
        self.inbuf[:, lq + lkv:].copy_(torch.from_numpy(v_new))
        self.lq, self.lkv = lq, lkv
        self.out = torch.empty(layers, n_q * hd, device="cuda")  # the whole output, on every rank
        if world == 1:
            self.gather = None
            self.pro = pro
            self.args = self._layer_args(0, layers)
        else:
            # q, k_new, v_new of this rank's heads as three packed arrays of one buffer
            flat = torch.empty(nq_f + 2 * nkv_f, device="cuda")
            self.q = flat[:nq_f].view(layers, lq)
            self.k_new = flat[nq_f:nq_f + nkv_f].view(layers, lkv)
            self.v_new = flat[nq_f + nkv_f:].view(layers, lkv)
            self.q.copy_(self.inbuf[:, :lq])
            self.k_new.copy_(self.inbuf[:, lq:lq + lkv])
            self.v_new.copy_(self.inbuf[:, lq + lkv:])
            self.inbuf = flat
            # the decode of this rank's heads pushes every unit's output into every rank's buffer
            # (tqk_decode_q8_gather); kout is the plain decode's output for the kernel-only timing
            self.kout = torch.empty(layers, lq, device="cuda")
            self.args_by = [shard.head_split_args(tqk, self.kp[c], self.vp[c], layers, n_q, n_kv, hd, self.mt, world,
                                                  self.q, self.kout, len0=pos + 1, k_new=self.k_new, v_new=self.v_new)
                            for c in range(self.copies)]
            self.gather = shard.PeerHeadSplit(dist, tqk, layers, per * group, hd)
            self.out = self.gather.out  # the whole output, [layers][n_q * head_dim], on every rank
            self.kernel_count = 0
        # algorithmic bytes of one step on this rank: K/V rows read + the appended Q8 rows written
        self.kv_bytes = 2 * layers * n_kv * (pos + 1) * self.nb * BB   # the whole job
        self.bytes_per_step = 2 * layers * per * (pos + 1) * self.nb * BB + 2 * layers * per * self.nb * BB
        self.tokens_per_step = 1
        self.launches_per_step = 1 if world == 1 else 2  # decode (+ the gather)
        # page-locked host buffers of the end-to-end leg: every rank copies its inputs in, rank 0
        # receives the whole output (the job's bytes are the sums over ranks)
        self.in_bytes = (nq_f + 2 * nkv_f) * 4
        self.h_in = HostBuffer(self.in_bytes)
        self.h_in.fill_from(self.inbuf)
        self.h_out = HostBuffer(self.out.numel() * 4)
        self.h2d = self.in_bytes * world
        self.d2h = self.out.numel() * 4
        self.e2e_api = ("per step: q, k and v (786 KB) in from page-locked host memory with one cudaMemcpyAsync, "
                        "then tqk_decode_q8 (C ABI) with its out in page-locked host memory (the kernel writes the "
                        "512 KB output over PCIe), then a stream synchronisation" if world == 1 else
                        "per rank: its q/k/v slice in from pinned host memory, tqk_decode_q8_gather over its kv "
                        "heads + tqk_gather_collect; rank 0 copies the whole output out; stream-synchronised every step")

    def _layer_args(self, first: int, count: int, out=None):
        """One-GPU decode arguments of layers [first, first + count): raw addresses into the cache,
        the interleaved input buffer and the output."""
        base = self.inbuf.data_ptr() + first * self.lrow * 4
        plane = self.nkv * self.mt * self.nb * BB  # bytes of one layer's plane
        out = self.out[first:first + count] if out is None else out
        return self.tqk.decode_args(self.kp.data_ptr() + first * plane, self.vp.data_ptr() + first * plane, self.nq,
                                    self.nkv, self.hd, self.mt, base, out, n_items=count,
                                    item_stride_blocks=self.nkv * self.mt * self.nb, len0=self.pos + 1,
                                    q_item_stride=self.lrow, out_item_stride=self.nq * self.hd,
                                    k_new=base + self.lq * 4, v_new=base + (self.lq + self.lkv) * 4,
                                    kv_new_item_stride=self.lrow,
                                    **{k: (v[first:first + count] if hasattr(v, "shape") else v)
                                       for k, v in self.pro.items()})

    def step(self):
        if self.gather is None:
            self.tqk.decode(self.args)
            return
        self.gather.step(self.args_by[(self.gather.epoch + 1) % self.copies])

    def kernel_step(self):
        """The decode launch of a step alone (its bytes are this rank's share), for the roofline."""
        self.kernel_count += 1
        self.tqk.decode(self.args_by[self.kernel_count % self.copies])

    def prepare_e2e(self):
        """The end-to-end step: the inputs copied in from page-locked host memory with one
        cudaMemcpyAsync, then the decode; on one GPU the decode writes its output straight into
        page-locked host memory (the kernel's final stores cross PCIe while other units still
        run), on several GPUs rank 0 copies the gathered output out."""
        import torch
        self.stream_handle = torch.cuda.current_stream().cuda_stream
        if self.world == 1:
            self.e2e_args = self._layer_args(0, self.L, out=self.h_out.ptr)

    def step_e2e(self):
        import torch
        st = self.stream_handle
        self.h_in.to_device(self.inbuf.data_ptr(), self.in_bytes, st)
        if self.world == 1:
            self.tqk.decode(self.e2e_args, stream=st)
        else:
            self.step()
            if self.rank == 0:
                self.h_out.from_device(self.out.data_ptr(), self.d2h, st)
        torch.cuda.current_stream().synchronize()

    def describe(self):
        return describe_config2(self.L, self.nq, self.nkv, self.hd, self.pos, self.prologue)

    def per_rank(self):
        return {"kv_heads_per_layer": self.per, "cache_copies_rotated": self.copies}

    def parallelism(self, world):
        if world == 1:
            return "single GPU"
        group = self.nq // self.nkv
        return (f"kv-head-group split over {world} GPUs: {self.per} kv head(s) and their {self.per * group} q heads "
                f"of every layer per GPU; the decode pushes each unit's output to every GPU over NVLink as "
                f"value+epoch pairs (tqk_decode_q8_gather + tqk_gather_collect)")

    def close(self):
        if self.gather is not None:
            self.gather.close()
            self.gather = None

    # the reference's CPU path on the same workload (host planes)
    def host_planes(self):
        if self.world != 1:
            raise RuntimeError("the CPU baseline runs at N = 1")
        x = self.inbuf.cpu().numpy()
        return self.kp[0].cpu().numpy(), self.vp[0].cpu().numpy(), np.ascontiguousarray(x[:, :self.lq]), \
            np.ascontiguousarray(x[:, self.lq:self.lq + self.lkv]), np.ascontiguousarray(x[:, self.lq + self.lkv:])


def config4_stream(n_kv, n, hd, p, h):
    """Config 4's inputs in the reference stream: K then V (p = 0, 1), every kv head's n rows of hd
    values, then q (p = 2)."""
    return (p * n_kv + h) * n * hd


def describe_config4(n_q, n_kv, hd, n):
    kv_bytes = 2 * n_kv * n * (hd // QK) * BB
    return {"workload": f"config4: Llama-3-70B-shaped Q8 GQA long-context decode, 1 layer, {n_q} q / {n_kv} kv "
                        f"heads, head_dim {hd}, context {n}",
            "layers": 1, "seq_len": n, "kv_bytes_per_token": kv_bytes,
            "l2": f"no flush: inputs larger than L2 ({kv_bytes / 1e6:.0f} MB of K/V per step vs 126 MB L2)"
                  if kv_bytes > 126e6 else f"{kv_bytes / 1e6:.1f} MB of K/V per step (smaller than L2)"}


class Config4:
    """Llama-3-70B-shaped long-context decode: one layer, 64 q / 8 kv heads,
    head_dim 128, context 131072.  With N ranks the context is split into N
    contiguous token ranges; each rank computes log-sum-exp partials of its
    range, and the ranks exchange and merge them: by default in one
    tqk_exchange_merge launch over peer memory (the decode writes into the
    rank's mailbox, the peers' records are read over NVLink), with
    exchange="nccl" by an NCCL all-gather and
    tqk_merge_partials.  One step is one token for the whole job."""
    name = "config4"
    scaling = "strong"  # the context is fixed; each rank gets 1/N of it

    def __init__(self, seed: int, rank: int = 0, world: int = 1, dist=None, n=131072, n_q=64, n_kv=8, hd=128,
                 exchange: str = "p2p"):
        import torch
        from tailorquantkernel_b200 import shard, tqk
        self.tqk, self.shard, self.dist, self.world = tqk, shard, dist, world
        self.L, self.nq, self.nkv, self.hd, self.n = 1, n_q, n_kv, hd, n
        self.mt, self.pos = n, n - 1
        self.nb = hd // QK
        self.start, self.n_local = shard.seq_range(n, rank, world)
        # on N GPUs a rank's range is 1/N of the cache: it rotates over N copies of it, one per step, so
        # that its working set stays the whole cache's size (larger than L2)
        self.copies = world
        self.count = 0
        gen = LibGen()
        rows = max(self.n_local, 1)
        self.kp = torch.zeros(self.copies, n_kv, rows, self.nb * BB, dtype=torch.uint8, device="cuda")
        self.vp = torch.zeros_like(self.kp)
        for p, plane in enumerate((self.kp, self.vp)):  # this rank's positions of the global K/V
            for h in range(n_kv):
                if self.n_local:
                    device_q8_rows(gen, config4_stream(n_kv, n, hd, p, h) + self.start * hd, self.n_local, hd,
                                   out=plane[0, h])
        for c in range(1, self.copies):
            self.kp[c].copy_(self.kp[0])
            self.vp[c].copy_(self.vp[0])
        self.q = torch.from_numpy(gen.normal(config4_stream(n_kv, n, hd, 2, 0), n_q * hd)).cuda()  # on every rank
        self.out = torch.empty(n_q * hd, device="cuda")
        self.partial = torch.empty(n_q * (hd + 2), device="cuda")
        self.gathered = torch.empty(world, n_q * (hd + 2), device="cuda")
        self.args = tqk.decode_args(self.kp, self.vp, n_q, n_kv, hd, max(self.n_local, 1), self.q, self.out,
                                    len0=self.n_local)
        self.kv_bytes = 2 * n_kv * n * self.nb * BB            # the whole context, all ranks
        self.bytes_per_step = 2 * n_kv * self.n_local * self.nb * BB  # this rank's decode kernel
        self.tokens_per_step = 1
        self.launches_per_step = 1 if world == 1 else 2  # decode (+ exchange-merge, or merge after NCCL)
        self.exchange = exchange
        self.peer = shard.PeerExchange(dist, tqk, n_q, hd) if world > 1 and exchange == "p2p" else None
        self.e2e_api = ("tqk_decode_q8 (C ABI, log-sum-exp partials of this rank's range) + tqk_exchange_merge "
                        if self.peer is not None else "tqk_decode_q8 (C ABI) ") + \
            "with pinned host q in and the attention output out, stream-synchronised every step"
        self.h_q = HostBuffer(self.q.numel() * 4)
        self.h_q.fill_from(self.q)
        self.h_out = HostBuffer(self.out.numel() * 4)
        self.h2d = self.q.numel() * 4
        self.d2h = self.out.numel() * 4

    def step(self):
        if self.world == 1:
            self.tqk.decode(self.args)
            return
        self.count += 1
        kp, vp = self.kp[self.count % self.copies], self.vp[self.count % self.copies]
        if self.peer is not None:
            self.shard.seqsplit_attend_p2p(self.peer, self.tqk, kp, vp, self.nq, self.nkv, self.hd, self.n_local,
                                           self.q, self.out)
        else:
            self.shard.seqsplit_attend(self.dist, self.tqk, kp, vp, self.nq, self.nkv, self.hd, self.n_local, self.q,
                                       self.out, self.partial, gathered=self.gathered)

    def kernel_step(self):
        """This rank's decode launch alone (partials of its range), for the roofline."""
        self.count += 1
        c = self.count % self.copies
        args = self.tqk.decode_args(self.kp[c], self.vp[c], self.nq, self.nkv, self.hd, max(self.n_local, 1), self.q,
                                    self.partial, len0=self.n_local, out_mode=self.tqk.OUT_PARTIAL)
        self.tqk.decode(args)

    def step_e2e(self):
        import torch
        s = torch.cuda.current_stream()
        self.h_q.to_device(self.q.data_ptr(), self.h2d, s.cuda_stream)
        self.step()
        self.h_out.from_device(self.out.data_ptr(), self.d2h, s.cuda_stream)
        s.synchronize()

    def describe(self):
        return describe_config4(self.nq, self.nkv, self.hd, self.n)

    def per_rank(self):
        return {"tokens_per_rank": self.n_local, "cache_copies_rotated": self.copies}

    def parallelism(self, world):
        if world == 1:
            return "single GPU"
        if self.peer is not None:
            return (f"sequence-split over {world} GPUs: log-sum-exp partials exchanged over peer memory and "
                    "merged in one kernel (tqk_exchange_merge)")
        return f"sequence-split over {world} GPUs: log-sum-exp partials all-gathered with NCCL, merged on device"

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def host_planes(self):
        return self.kp.cpu().numpy(), self.vp.cpu().numpy(), self.q.cpu().numpy(), None, None


def rope_np(x, hd, pos, theta):
    """Half-split RoPE of the reference (model/rope.c:4-22) on every head of x [..., heads*hd]."""
    i = np.arange(hd // 2, dtype=np.float64)
    a = pos * np.power(theta, -2.0 * i / hd)
    c, s = np.cos(a), np.sin(a)
    h = x.reshape(-1, hd).astype(np.float64)
    x0, x1 = h[:, : hd // 2].copy(), h[:, hd // 2:].copy()
    h[:, : hd // 2] = x0 * c - x1 * s
    h[:, hd // 2:] = x0 * s + x1 * c
    return h.astype(np.float32).reshape(x.shape)


def config3_stream(all_lens, n_q, n_kv, hd):
    """Config 3's inputs in the reference stream: the 64 lengths are uniforms #0..63; then for every
    sequence b, K then V, every kv head's len_b rows of hd values; then every sequence's q [n_q*hd].
    The outlier pick of normal sample i is uniform #(64 + i)."""
    starts = np.concatenate([[0], np.cumsum(all_lens.astype(np.int64))]) * (2 * n_kv * hd)
    q0 = int(starts[-1])
    return {"kv": lambda b, p: int(starts[b]) + p * n_kv * int(all_lens[b]) * hd,
            "q": lambda b: q0 + b * n_q * hd, "u": lambda i: len(all_lens) + i}


def describe_config3(all_lens, lo, mt, n_q, n_kv, hd):
    kv_bytes = 2 * n_kv * int(np.sum(all_lens)) * (hd // QK) * BB
    return {"workload": f"config3: ragged batched Q8 GQA decode, {len(all_lens)} sequences, lengths U[{lo}, {mt}] "
                        f"(sum {int(np.sum(all_lens))}), {n_q} q / {n_kv} kv heads, head_dim {hd}, 1% x8 outliers",
            "layers": 1, "batch": len(all_lens), "kv_bytes_per_step": kv_bytes,
            "l2": f"no flush: inputs larger than L2 ({kv_bytes / 1e6:.0f} MB of K/V per step vs 126 MB L2)"
                  if kv_bytes > 126e6 else f"{kv_bytes / 1e6:.1f} MB of K/V per step (smaller than L2)"}


class Config3:
    """Ragged batched decode: 64 sequences, lengths uniform
    in [512, 8192], 32 q / 8 kv heads, head_dim 128, K/V ~ N(0,1) with 1% of
    the entries x8 (outlier blocks).  One launch attends every sequence of
    the rank's share (ragged device lengths).  With N ranks the 64 sequences
    are divided by total length (shard.batch_shard); one step = one token
    for each of the 64 sequences."""
    name = "config3"
    scaling = "strong"  # the batch of 64 is fixed; each rank takes a share
    B = 64

    def __init__(self, seed: int, rank: int = 0, world: int = 1, n_q=32, n_kv=8, hd=128, mt=8192, lo=512):
        import torch
        from tailorquantkernel_b200 import shard, tqk
        self.tqk = tqk
        self.L, self.nq, self.nkv, self.hd, self.mt, self.lo = 1, n_q, n_kv, hd, mt, lo
        self.nb = hd // QK
        gen = LibGen()
        self.all_lens = ragged_lengths(gen, self.B, lo, mt)
        off = config3_stream(self.all_lens, n_q, n_kv, hd)
        self.mine = shard.batch_shard(self.all_lens, world)[rank]
        lens = self.all_lens[self.mine]
        nloc = len(self.mine)
        self.kp = torch.zeros(nloc, n_kv, mt, self.nb * BB, dtype=torch.uint8, device="cuda")
        self.vp = torch.zeros_like(self.kp)
        for i, b in enumerate(self.mine):  # one sequence at a time: bounded fp32 scratch
            n = int(self.all_lens[b])
            for p, plane in enumerate((self.kp, self.vp)):
                x = outliers(gen, off["u"](off["kv"](b, p)), gen.normal(off["kv"](b, p), n_kv * n * hd))
                x = torch.from_numpy(x).cuda().view(n_kv, n, hd)
                for h in range(n_kv):
                    tqk.quantize_rows(x[h], out=plane[i, h, :n])
        self.lens = torch.from_numpy(lens).cuda()
        self.q = torch.from_numpy(np.stack([gen.normal(off["q"](b), n_q * hd) for b in self.mine])).cuda()
        self.out = torch.empty(nloc, n_q * hd, device="cuda")
        self.kv_bytes = 2 * n_kv * int(self.all_lens.sum()) * self.nb * BB  # the whole batch
        self.bytes_per_step = 2 * n_kv * int(lens.sum()) * self.nb * BB   # this rank's decode kernel
        # a rank's share of the batch can be smaller than L2: it then rotates over copies of its planes,
        # one per step, so that at least twice L2's 126 MB is read between two reads of the same bytes
        self.copies = 1 if world == 1 else max(1, -(-252_000_000 // max(self.bytes_per_step, 1)))
        kps, vps = [self.kp], [self.vp]
        for _ in range(self.copies - 1):
            kps.append(self.kp.clone())
            vps.append(self.vp.clone())
        self.kps, self.vps = kps, vps
        self.all_args = [tqk.decode_args(kps[c], vps[c], n_q, n_kv, hd, mt, self.q, self.out, n_items=nloc,
                                         item_stride_blocks=n_kv * mt * self.nb, lens=self.lens,
                                         max_len=int(lens.max()), q_item_stride=n_q * hd, out_item_stride=n_q * hd)
                         for c in range(self.copies)]
        self.args = self.all_args[0]
        self.count = 0
        self.tokens_per_step = self.B  # for the whole job: each step is one token of every sequence
        self.launches_per_step = 1
        self.e2e_api = ("tqk_decode_q8 (C ABI, ragged device lengths) with the rank's sequences' pinned host q in "
                        "and their attention outputs out, stream-synchronised every step")
        self.h_q = HostBuffer(self.q.numel() * 4)
        self.h_q.fill_from(self.q)
        self.h_out = HostBuffer(self.out.numel() * 4)
        self.h2d = self.q.numel() * 4
        self.d2h = self.out.numel() * 4

    def step(self):
        self.count += 1
        self.tqk.decode(self.all_args[self.count % self.copies])

    def step_e2e(self):
        import torch
        s = torch.cuda.current_stream()
        self.h_q.to_device(self.q.data_ptr(), self.h2d, s.cuda_stream)
        self.step()
        self.h_out.from_device(self.out.data_ptr(), self.d2h, s.cuda_stream)
        s.synchronize()

    def describe(self):
        return describe_config3(self.all_lens, self.lo, self.mt, self.nq, self.nkv, self.hd)

    def per_rank(self):
        return {"sequences_per_rank": len(self.mine), "cache_copies_rotated": self.copies}

    @staticmethod
    def parallelism(world):
        return (f"batch-sharded over {world} GPUs by total length, no collective" if world > 1 else "single GPU")

    def host_planes(self):
        raise NotImplementedError("the CPU baseline of config 3 uses HostConfig3")


def prefill_flops(n_q, hd, pos0, n):
    """2*2*head_dim FLOPs (QK^T and PV) per (query head, visible key) of a causal chunk."""
    pairs = n * pos0 + n * (n + 1) // 2
    return n_q * pairs * 2 * 2 * hd


def config5_stream(n_q, n_kv, hd, pos0, n):
    """Config 5's inputs in the reference stream: K then V of the cached prefix, every kv head's pos0
    rows of hd values; then the chunk's q [n][n_q*hd], k [n][n_kv*hd] and v [n][n_kv*hd]."""
    kv = 2 * n_kv * pos0 * hd
    return {"kv": lambda p, h: (p * n_kv + h) * pos0 * hd, "q": kv, "k": kv + n * n_q * hd,
            "v": kv + n * (n_q + n_kv) * hd}


def describe_config5(n_q, n_kv, hd, pos0, n):
    return {"workload": f"config5: chunked causal prefill, {n} new tokens at positions {pos0}..{pos0 + n - 1} over a "
                        f"{pos0}-position Q8 cache, {n_q} q / {n_kv} kv heads, head_dim {hd}",
            "tokens_per_step": n, "flops_per_step": prefill_flops(n_q, hd, pos0, n),
            "l2": "the Q8 K/V of a kv head is L2-resident by design; timed back to back"}


class Config5:
    """Chunked causal prefill: 2048 new tokens at positions
    2048..4095 appended to a Q8 cache holding 2048 prior positions, each
    attending causally to everything before it; 32 q / 8 kv heads, head_dim
    128.  One step = one tqk_prefill_q8 call (bit-exact Q8 append of the 2048
    K/V rows + the tcgen05 attention kernel), i.e. 2048 tokens."""
    name = "config5"
    scaling = "weak"  # replicas: every rank prefills its own sequence
    bound = "tensor"
    e2e_steps = 50        # each end-to-end step moves 82 MB over PCIe

    def __init__(self, seed: int, n_q=32, n_kv=8, hd=128, pos0=2048, n=2048):
        import torch
        from tailorquantkernel_b200 import tqk
        self.tqk = tqk
        self.L, self.nq, self.nkv, self.hd, self.pos0, self.n = 1, n_q, n_kv, hd, pos0, n
        self.FLOPS = prefill_flops(n_q, hd, pos0, n)  # 103,095,992,320 at the default shape
        self.mt = pos0 + n
        self.nb = hd // QK
        gen = LibGen()
        off = config5_stream(n_q, n_kv, hd, pos0, n)
        self.kp = torch.zeros(n_kv, self.mt, self.nb * BB, dtype=torch.uint8, device="cuda")
        self.vp = torch.zeros_like(self.kp)
        for p, plane in enumerate((self.kp, self.vp)):
            for h in range(n_kv):
                device_q8_rows(gen, off["kv"](p, h), pos0, hd, out=plane[h, :pos0])
        dev = lambda key, w: torch.from_numpy(gen.normal(off[key], n * w * hd)).cuda().view(n, w * hd)  # noqa: E731
        self.q, self.k_new, self.v_new = dev("q", n_q), dev("k", n_kv), dev("v", n_kv)
        self.out = torch.empty(n, n_q * hd, device="cuda")
        self.tokens_per_step = n
        self.launches_per_step = 3  # the append, the K/V tile staging and the attention
        self.bytes_per_step = 2 * n_kv * self.mt * self.nb * BB
        self.e2e_api = ("tqk_prefill_q8 (C ABI) with the chunk's pinned host q, k and v in and the attention "
                        "output out, stream-synchronised every step")
        self.h_q = self.q.cpu().pin_memory()
        self.h_k = self.k_new.cpu().pin_memory()
        self.h_v = self.v_new.cpu().pin_memory()
        self.h_out = torch.empty_like(self.out, device="cpu").pin_memory()
        self.h2d = (self.h_q.numel() + self.h_k.numel() + self.h_v.numel()) * 4
        self.d2h = self.h_out.numel() * 4

    def step(self):
        self.tqk.prefill(self.kp, self.vp, self.nq, self.nkv, self.hd, self.mt, self.pos0, self.n, self.q,
                         self.k_new, self.v_new, self.out)

    def step_e2e(self):
        import torch
        s = torch.cuda.current_stream()
        self.q.copy_(self.h_q, non_blocking=True)
        self.k_new.copy_(self.h_k, non_blocking=True)
        self.v_new.copy_(self.h_v, non_blocking=True)
        self.step()
        self.h_out.copy_(self.out, non_blocking=True)
        s.synchronize()

    def describe(self):
        return describe_config5(self.nq, self.nkv, self.hd, self.pos0, self.n)

    @staticmethod
    def parallelism(world):
        return "replicas: one sequence per GPU, no collective" if world > 1 else "single GPU"

    def host_planes(self):
        return (self.kp.cpu().numpy(), self.vp.cpu().numpy(), self.q.cpu().numpy(), self.k_new.cpu().numpy(),
                self.v_new.cpu().numpy())


def q8_weight_rows_np(rng, rows: int, cols: int) -> np.ndarray:
    """Random packed Q8 weight rows (packer/packer.h layout: per 32 columns a float scale and 32
    int8): int8 uniform in [-127, 127], scales uniform in [0.002, 0.02)."""
    nb = cols // QK
    w = np.empty((rows, nb, BB), np.uint8)
    w[:, :, 4:] = rng.integers(-127, 128, (rows, nb, QK), dtype=np.int8).view(np.uint8)
    w[:, :, :4] = rng.uniform(0.002, 0.02, (rows, nb)).astype(np.float32).view(np.uint8).reshape(rows, nb, 4)
    return w.reshape(rows, nb * BB)


def config6_stream(layers, n_kv, hd, mt, hidden):
    """Config 6's inputs in the reference stream: K/V as config 2's (every layer, K then V, every kv
    head's mt rows), then the input activation [hidden], then the q and k RMSNorm weights
    [layers][hd] each (as 1 + 0.1 x).  The weight matrices are random packed Q8 rows (numpy, the
    same bytes in both arms)."""
    x = layers * 2 * n_kv * mt * hd
    return {"kv": lambda layer, p, h: ((layer * 2 + p) * n_kv + h) * mt * hd, "x": x, "norms": x + hidden}


def describe_config6(layers, n_q, n_kv, hd, hidden, pos):
    row = hd // QK * BB
    q_dim, kv_dim = n_q * hd, n_kv * hd
    wbytes = layers * (q_dim * hidden + 2 * kv_dim * hidden + hidden * q_dim) // QK * BB
    kv_bytes = 2 * layers * n_kv * (pos + 1) * row
    return {"workload": f"config6: Llama-3-8B-shaped attention stack, one token through {layers} attention layers "
                        f"(Q8 wq/wk/wv/wo, q/k RMSNorm + RoPE(500000), Q8 cache append at {pos} and attention "
                        f"over {pos + 1} positions, output projection), each layer's output feeding the next",
            "layers": layers, "seq_len": pos + 1, "hidden": hidden,
            "weight_bytes_per_token": wbytes, "kv_bytes_per_token": kv_bytes,
            "l2": f"no flush: inputs larger than L2 ({(wbytes + kv_bytes) / 1e9:.2f} GB per step vs 126 MB L2)"
                  if wbytes + kv_bytes > 126e6 else "smaller than L2"}


class Config6:
    """A Llama-3-8B-shaped attention stack on the device: one token through 32 attention layers
    (tqk_attention_layer: q/k/v projection with the activation quantisation, decode with the fused
    q/k RMSNorm + RoPE + append at position 4096, output projection), each layer's output feeding
    the next layer's input, the 96 launches captured once in a CUDA graph and replayed per step.
    Q8 weights (1.51 GB for the 32 layers) and the Q8 cache (302 MB) stay in HBM."""
    name = "config6"
    scaling = "weak"
    e2e_steps = 2000
    data = ("synthetic: K/V, input and norm weights from the reference benches' generator (xorshift64 + "
            "Box-Muller, seed 88172645463325252), K/V quantised to Q8 on the device; seeded random packed Q8 "
            "weights (int8 uniform, scales uniform in [0.002, 0.02))")

    def __init__(self, seed: int, layers=32, n_q=32, n_kv=8, hd=128, hidden=4096, pos=4096):
        import torch
        from tailorquantkernel_b200 import tqk
        self.tqk = tqk
        self.L, self.nq, self.nkv, self.hd, self.hidden, self.pos = layers, n_q, n_kv, hd, hidden, pos
        self.mt = pos + 1
        self.nb = hd // QK
        rng = np.random.default_rng(seed)
        q_dim, kv_dim = n_q * hd, n_kv * hd
        shapes = {"wq": (q_dim, hidden), "wk": (kv_dim, hidden), "wv": (kv_dim, hidden), "wo": (hidden, q_dim)}
        self.w = [{n: torch.from_numpy(q8_weight_rows_np(rng, *sh)).cuda() for n, sh in shapes.items()}
                  for _ in range(layers)]
        gen = LibGen()
        off = config6_stream(layers, n_kv, hd, self.mt, hidden)
        norms = 1 + np.float32(0.1) * gen.normal(off["norms"], 2 * layers * hd).reshape(2, layers, hd)
        self.qn = [torch.from_numpy(norms[0, l].copy()).cuda() for l in range(layers)]
        self.kn = [torch.from_numpy(norms[1, l].copy()).cuda() for l in range(layers)]
        self.kp = [device_q8_rows(gen, off["kv"](l, 0, 0), n_kv * self.mt, hd).view(n_kv, self.mt, -1)
                   for l in range(layers)]
        self.vp = [device_q8_rows(gen, off["kv"](l, 1, 0), n_kv * self.mt, hd).view(n_kv, self.mt, -1)
                   for l in range(layers)]
        inv = np.float32(500000.0) ** (-2.0 * np.arange(hd // 2, dtype=np.float32) / np.float32(hd))
        ang = np.float32(pos) * inv.astype(np.float32)
        self.cos = torch.from_numpy(np.cos(ang).astype(np.float32)).cuda()
        self.sin = torch.from_numpy(np.sin(ang).astype(np.float32)).cuda()
        self.acts = [torch.from_numpy(gen.normal(off["x"], hidden)).cuda()]
        self.acts += [torch.empty(hidden, device="cuda") for _ in range(layers)]
        self.scratch = torch.empty(tqk.layer_scratch_floats(n_q, n_kv, hd), device="cuda")
        self.ws = torch.zeros(1 << 22, dtype=torch.uint8, device="cuda")
        self.args = [tqk.attention_layer_args(self.w[l], tqk.FMT_Q8, self.qn[l], self.kn[l], n_q, n_kv, hd, hidden,
                                              1e-6, self.kp[l], self.vp[l], self.mt, pos, self.cos, self.sin,
                                              self.acts[l], self.acts[l + 1], self.scratch)
                     for l in range(layers)]
        # captured on a side stream (CUDA requires it), replayed on the current one
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            tqk.workspace_init(self.ws, cap)
            for l in range(layers):  # eager once: sets the kernels up outside capture
                tqk.attention_layer(self.args[l], self.ws, cap)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=cap):
                for l in range(layers):
                    tqk.attention_layer(self.args[l], self.ws, cap)
        cap.synchronize()
        self.stream = torch.cuda.current_stream()
        wbytes = sum(t.numel() for t in self.w[0].values()) * layers
        self.weight_bytes = wbytes
        self.kv_bytes = 2 * layers * n_kv * (pos + 1) * self.nb * BB
        self.bytes_per_step = wbytes + self.kv_bytes + 2 * layers * n_kv * self.nb * BB
        self.tokens_per_step = 1
        self.launches_per_step = 3 * layers
        self.h_x = HostBuffer(hidden * 4)
        self.h_x.fill_from(self.acts[0])
        self.h_out = HostBuffer(hidden * 4)
        self.h2d = hidden * 4
        self.d2h = hidden * 4
        self.e2e_api = ("tqk_attention_layer x 32 (C ABI) replayed as one CUDA graph, with the token's input "
                        "copied in from pinned host memory and the last layer's output copied out, "
                        "stream-synchronised every step")

    def step(self):
        self.graph.replay()

    def step_e2e(self):
        st = self.stream.cuda_stream
        self.h_x.to_device(self.acts[0].data_ptr(), self.h2d, st)
        self.graph.replay()
        self.h_out.from_device(self.acts[-1].data_ptr(), self.d2h, st)
        self.stream.synchronize()

    def describe(self):
        return describe_config6(self.L, self.nq, self.nkv, self.hd, self.hidden, self.pos)

    @staticmethod
    def parallelism(world):
        return "replicas: every GPU runs its own token" if world > 1 else "single GPU"


def config7_stream(layers, n_kv, hd, mt, hidden):
    """Config 7's cache and norm weights in the reference stream: K/V as config 2's, then for every
    layer its input and post-attention RMSNorm weights [hidden] and q / k norm weights [hd] (as
    1 + 0.1 x), then the final norm [hidden].  The weight matrices are random packed Q8 rows."""
    kv = layers * 2 * n_kv * mt * hd
    per = 2 * hidden + 2 * hd
    return {"kv": lambda layer, p, h: ((layer * 2 + p) * n_kv + h) * mt * hd,
            "norms": lambda layer: kv + layer * per, "final_norm": kv + layers * per}


def describe_config7(layers, n_q, n_kv, hd, hidden, inter, vocab, pos):
    row = hd // QK * BB
    q_dim, kv_dim = n_q * hd, n_kv * hd
    per_layer = (q_dim * hidden + 2 * kv_dim * hidden + hidden * q_dim + 3 * inter * hidden) // QK * BB
    wbytes = layers * per_layer + vocab * hidden // QK * BB
    kv_bytes = 2 * layers * n_kv * (pos + 1) * row
    return {"workload": f"config7: Llama-3-8B-shaped whole-token decode on the device (tq_forward_token): embedding, "
                        f"{layers} layers of RMSNorm + attention (Q8 wq/wk/wv/wo, q/k RMSNorm + RoPE(500000), Q8 "
                        f"cache append at {pos}, attention over {pos + 1} positions) + RMSNorm + Q8 MLP "
                        f"({inter} wide, SiLU), final RMSNorm, tied Q8 lm_head over {vocab} tokens, greedy choice",
            "layers": layers, "seq_len": pos + 1, "hidden": hidden, "intermediate": inter, "vocab": vocab,
            "weight_bytes_per_token": wbytes, "kv_bytes_per_token": kv_bytes,
            "l2": f"no flush: inputs larger than L2 ({(wbytes + kv_bytes) / 1e9:.2f} GB per step vs 126 MB L2)"}


def random_q8_rows(rows: int, cols: int, g):
    """Random packed Q8 rows made on the device (int8 uniform, scales uniform in [0.002, 0.02))."""
    import torch
    nb = cols // QK
    w = torch.randint(0, 256, (rows, nb, BB), dtype=torch.uint8, device="cuda", generator=g)
    d = torch.empty(rows, nb, device="cuda").uniform_(0.002, 0.02, generator=g)
    w[:, :, :4] = d.view(torch.uint8).view(rows, nb, 4)
    return w.view(rows, nb * BB)


class Config7:
    """A Llama-3-8B-shaped token through the whole decoder stack on the device (tqk_forward_token,
    the reference's tq_forward_token of model/context.c:104-122): 8.7 GB of Q8 weights and 302 MB
    of Q8 cache per token, the 260 launches captured once in a CUDA graph and replayed per step
    (the position stays at 4096, so each step rewrites the same cache row)."""
    name = "config7"
    scaling = "weak"
    e2e_steps = 200
    data = ("synthetic: K/V and norm weights from the reference benches' generator (xorshift64 + Box-Muller, "
            "seed 88172645463325252), K/V quantised to Q8 on the device; seeded random packed Q8 weights made "
            "on the device (int8 uniform, scales uniform in [0.002, 0.02)); RoPE tables of float32 numpy")

    def __init__(self, seed: int, layers=32, n_q=32, n_kv=8, hd=128, hidden=4096, inter=14336, vocab=128256,
                 pos=4096):
        import torch
        from tailorquantkernel_b200 import tqk
        self.tqk = tqk
        self.L, self.nq, self.nkv, self.hd, self.hidden, self.inter, self.vocab, self.pos = \
            layers, n_q, n_kv, hd, hidden, inter, vocab, pos
        self.mt = pos + 1
        g = torch.Generator(device="cuda").manual_seed(seed)
        gen = LibGen()
        q_dim, kv_dim = n_q * hd, n_kv * hd
        off = config7_stream(layers, n_kv, hd, self.mt, hidden)
        norm = lambda first, n: torch.from_numpy(1 + np.float32(0.1) * gen.normal(first, n)).cuda()  # noqa: E731
        self.layers = []
        for layer in range(layers):
            nrm = off["norms"](layer)
            d = {"input_norm": norm(nrm, hidden), "post_norm": norm(nrm + hidden, hidden),
                 "q_norm": norm(nrm + 2 * hidden, hd), "k_norm": norm(nrm + 2 * hidden + hd, hd),
                 "wq": random_q8_rows(q_dim, hidden, g), "wk": random_q8_rows(kv_dim, hidden, g),
                 "wv": random_q8_rows(kv_dim, hidden, g), "wo": random_q8_rows(hidden, q_dim, g),
                 "wgate": random_q8_rows(inter, hidden, g), "wup": random_q8_rows(inter, hidden, g),
                 "wdown": random_q8_rows(hidden, inter, g)}
            for p, key in enumerate(("k_cache", "v_cache")):
                d[key] = device_q8_rows(gen, off["kv"](layer, p, 0), n_kv * self.mt, hd).view(n_kv, self.mt, -1)
            self.layers.append(d)
        self.embed = random_q8_rows(vocab, hidden, g)
        self.final_norm = norm(off["final_norm"], hidden)
        inv = np.float32(500000.0) ** (-2.0 * np.arange(hd // 2, dtype=np.float32) / np.float32(hd))
        ang = np.arange(self.mt, dtype=np.float32)[:, None] * inv[None, :].astype(np.float32)
        self.cos = torch.from_numpy(np.cos(ang).astype(np.float32)).cuda()
        self.sin = torch.from_numpy(np.sin(ang).astype(np.float32)).cuda()
        cfg = {"n_layers": layers, "n_q_heads": n_q, "n_kv_heads": n_kv, "head_dim": hd, "hidden_size": hidden,
               "intermediate_size": inter, "vocab_size": vocab, "max_tokens": self.mt, "rms_eps": 1e-5}
        self.model = tqk.model_struct(cfg, self.layers, self.embed, self.final_norm, self.cos, self.sin, fmt=0)
        self.scratch = torch.empty(tqk.forward_scratch_bytes(self.model) // 4, device="cuda")
        self.logits = torch.empty(vocab, device="cuda")
        self.next = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.ws = torch.zeros(1 << 22, dtype=torch.uint8, device="cuda")
        self.token = 17
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            tqk.workspace_init(self.ws, cap)
            tqk.forward_token(self.model, self.token, pos, self.scratch, self.logits, self.next, self.ws, cap)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=cap):
                tqk.forward_token(self.model, self.token, pos, self.scratch, self.logits, self.next, self.ws, cap)
        cap.synchronize()
        self.stream = torch.cuda.current_stream()
        d = describe_config7(layers, n_q, n_kv, hd, hidden, inter, vocab, pos)
        self.weight_bytes, self.kv_bytes = d["weight_bytes_per_token"], d["kv_bytes_per_token"]
        self.bytes_per_step = self.weight_bytes + self.kv_bytes + 2 * layers * n_kv * (hd // QK) * BB
        self.tokens_per_step = 1
        self.launches_per_step = 2 + 8 * layers + 2
        self.h_out = HostBuffer(vocab * 4)
        self.h2d = 0  # the token id is a host argument of the call
        self.d2h = vocab * 4
        self.e2e_api = ("tqk_forward_token x 1 (C ABI) replayed as one CUDA graph per token, the logits copied out to "
                        "page-locked host memory, stream-synchronised every step")

    def step(self):
        self.graph.replay()

    def step_e2e(self):
        self.graph.replay()
        self.h_out.from_device(self.logits.data_ptr(), self.d2h, self.stream.cuda_stream)
        self.stream.synchronize()

    def describe(self):
        return describe_config7(self.L, self.nq, self.nkv, self.hd, self.hidden, self.inter, self.vocab, self.pos)

    @staticmethod
    def parallelism(world):
        return "replicas: every GPU runs its own token" if world > 1 else "single GPU"


class HostConfig6:
    """Config 6 on the host only, for the reference's attention_layer (CPU): the same shapes, random
    packed Q8 weights and a cache quantised by the reference's own quantiser."""
    name = "config6"

    def __init__(self, orc, seed: int, layers=32, n_q=32, n_kv=8, hd=128, hidden=4096, pos=4096):
        self.L, self.nq, self.nkv, self.hd, self.hidden, self.pos = layers, n_q, n_kv, hd, hidden, pos
        self.mt = pos + 1
        self.nb = hd // QK
        rng = np.random.default_rng(seed)
        q_dim, kv_dim = n_q * hd, n_kv * hd
        shapes = {"wq": (q_dim, hidden), "wk": (kv_dim, hidden), "wv": (kv_dim, hidden), "wo": (hidden, q_dim)}
        self.w = [{n: q8_weight_rows_np(rng, *sh) for n, sh in shapes.items()} for _ in range(layers)]
        gen = reference_generator()
        off = config6_stream(layers, n_kv, hd, self.mt, hidden)
        norms = 1 + np.float32(0.1) * gen.normal(off["norms"], 2 * layers * hd).reshape(2, layers, hd)
        self.qn = [norms[0, l].copy() for l in range(layers)]
        self.kn = [norms[1, l].copy() for l in range(layers)]
        row = self.nb * BB
        self.kp, self.vp = ([orc.quantize_rows_bulk(gen.normal(off["kv"](l, p, 0), n_kv * self.mt * hd)
                                                    .reshape(n_kv, self.mt, hd)) for l in range(layers)]
                            for p in (0, 1))
        self.x = gen.normal(off["x"], hidden)
        wbytes = sum(a.size for a in self.w[0].values()) * layers
        self.kv_bytes = 2 * layers * n_kv * (pos + 1) * row
        self.bytes_per_step = wbytes + self.kv_bytes + 2 * layers * n_kv * row

    def describe(self):
        return describe_config6(self.L, self.nq, self.nkv, self.hd, self.hidden, self.pos)


class HostConfig7:
    """Config 7 on the host for the reference's own tq_forward_token (model/context.c:104-122): the
    same shapes, random packed Q8 weights (int8 uniform, scales uniform in [0.002, 0.02)) and a Q8
    cache of pos positions, quantised by the reference's quantiser, that the context starts from."""
    name = "config7"

    def __init__(self, orc, seed: int, layers=32, n_q=32, n_kv=8, hd=128, hidden=4096, inter=14336, vocab=128256,
                 pos=4096):
        self.L, self.nq, self.nkv, self.hd, self.hidden, self.inter, self.vocab, self.pos = \
            layers, n_q, n_kv, hd, hidden, inter, vocab, pos
        self.mt = pos + 1
        rng = np.random.default_rng(seed)
        gen = reference_generator()
        off = config7_stream(layers, n_kv, hd, self.mt, hidden)
        q_dim, kv_dim = n_q * hd, n_kv * hd
        norm = lambda first, n: 1 + np.float32(0.1) * gen.normal(first, n)  # noqa: E731
        lay = []
        self.planes = []
        for layer in range(layers):
            nrm = off["norms"](layer)
            lay.append({"input_norm": norm(nrm, hidden), "post_norm": norm(nrm + hidden, hidden),
                        "q_norm": norm(nrm + 2 * hidden, hd), "k_norm": norm(nrm + 2 * hidden + hd, hd),
                        "wq": q8_weight_rows_np(rng, q_dim, hidden), "wk": q8_weight_rows_np(rng, kv_dim, hidden),
                        "wv": q8_weight_rows_np(rng, kv_dim, hidden), "wo": q8_weight_rows_np(rng, hidden, q_dim),
                        "wgate": q8_weight_rows_np(rng, inter, hidden), "wup": q8_weight_rows_np(rng, inter, hidden),
                        "wdown": q8_weight_rows_np(rng, hidden, inter)})
            self.planes.append(tuple(orc.quantize_rows_bulk(gen.normal(off["kv"](layer, p, 0), n_kv * self.mt * hd)
                                                            .reshape(n_kv, self.mt, hd)) for p in (0, 1)))
        self.model = {"cfg": {"n_q_heads": n_q, "n_kv_heads": n_kv, "head_dim": hd, "hidden_size": hidden,
                              "rope_theta": 500000.0, "rms_eps": 1e-5, "n_layers": layers,
                              "intermediate_size": inter, "vocab_size": vocab},
                      "fmt": "8", "embed": q8_weight_rows_np(rng, vocab, hidden),
                      "final_norm": norm(off["final_norm"], hidden), "layers": lay}
        d = describe_config7(layers, n_q, n_kv, hd, hidden, inter, vocab, pos)
        self.bytes_per_step = d["weight_bytes_per_token"] + d["kv_bytes_per_token"]

    def describe(self):
        return describe_config7(self.L, self.nq, self.nkv, self.hd, self.hidden, self.inter, self.vocab, self.pos)


def reference_forward_seconds(orc, wl, tokens: int):
    """Times the reference's tq_forward_token (all host threads: its matmuls and attention use
    OpenMP) from position pos - tokens + 1 on: one context runs 1 token, another 1 + tokens, and the
    difference over `tokens` is the per-token time (the context set-up and cache fill cancel).  When
    that difference is under a tenth of the longer run (shapes so small that set-up noise dominates),
    the longer run's time per token is returned instead.  Returns (seconds per token, tokens, threads)."""
    threads = os.cpu_count() or 1
    start = (wl.pos - tokens, wl.planes)
    t0 = time.perf_counter()
    _, rc1, _ = orc.forward_tokens(wl.model, [17], wl.mt, start_planes=start)
    t1 = time.perf_counter()
    _, rc2, _ = orc.forward_tokens(wl.model, [17] * (1 + tokens), wl.mt, start_planes=start)
    t2 = time.perf_counter()
    if rc1 != [0] or rc2 != [0] * (1 + tokens):
        raise RuntimeError(f"the reference's tq_forward_token returned {rc1} / {rc2}")
    diff = (t2 - t1) - (t1 - t0)
    if diff < 0.1 * (t2 - t1):  # set-up noise swamps the tokens (tiny shapes): the whole second run per token
        return (t2 - t1) / (1 + tokens), tokens, threads
    return diff / tokens, tokens, threads


def reference_layers_seconds(orc, wl, budget_s: float, max_tokens: int | None = None, min_tokens: int = 2):
    """Times the reference's attention_layer (model/attention_layer.c:169-194) through all layers for
    whole tokens on the host's cores, until budget_s passes.  Returns (median seconds per token,
    tokens, threads)."""
    threads = os.cpu_count() or 1
    times = []
    t_end = time.perf_counter() + budget_s
    while (time.perf_counter() < t_end or len(times) < min_tokens) and (max_tokens is None or len(times) < max_tokens):
        t0 = time.perf_counter()
        x = wl.x
        for layer in range(wl.L):
            x = orc.attention_layer(wl.w[layer], "8", wl.qn[layer], wl.kn[layer], wl.nq, wl.nkv, wl.hd, wl.hidden,
                                    500000.0, 1e-6, wl.kp[layer], wl.vp[layer], wl.mt, wl.pos, x)
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times), threads


class HostConfig2:
    """Config 2 built on the host only, for the reference arm: K/V ~ N(0,1) per
    layer quantised by the reference's own quantize_row_q8."""
    name = "config2"

    def __init__(self, orc, seed: int, layers=32, n_q=32, n_kv=8, hd=128, pos=4096):
        self.L, self.nq, self.nkv, self.hd, self.pos = layers, n_q, n_kv, hd, pos
        self.mt = pos + 1
        self.nb = hd // QK
        gen = reference_generator()
        off = config2_stream(layers, n_q, n_kv, hd, self.mt)
        row = self.nb * BB
        self.kp = np.empty((layers, n_kv, self.mt, row), np.uint8)
        self.vp = np.empty((layers, n_kv, self.mt, row), np.uint8)
        for layer in range(layers):
            for p, plane in enumerate((self.kp, self.vp)):
                x = gen.normal(off["kv"](layer, p, 0), n_kv * self.mt * hd).reshape(n_kv, self.mt, hd)
                plane[layer] = orc.quantize_rows_bulk(x)
        qkv = gen.normal(off["step"], layers * (n_q + 2 * n_kv) * hd).reshape(layers, n_q + 2 * n_kv, hd)
        self.q = rope_np(np.ascontiguousarray(qkv[:, :n_q]).reshape(layers, n_q * hd), hd, pos, 500000.0)
        self.k_new = np.ascontiguousarray(qkv[:, n_q:n_q + n_kv]).reshape(layers, n_kv * hd)
        self.v_new = np.ascontiguousarray(qkv[:, n_q + n_kv:]).reshape(layers, n_kv * hd)
        self.kv_bytes = 2 * layers * n_kv * (pos + 1) * row
        self.bytes_per_step = self.kv_bytes + 2 * layers * n_kv * row

    def host_planes(self):
        return self.kp, self.vp, self.q, self.k_new, self.v_new

    def describe(self):
        return describe_config2(self.L, self.nq, self.nkv, self.hd, self.pos)


class HostConfig3:
    """Config 3 on the host for the reference CPU path: the batch's lengths, with
    planes built (reference quantiser) for the first 4 sequences only -- the
    bounded sample the CPU baseline times."""
    name = "config3"

    def __init__(self, orc, seed: int, n_q=32, n_kv=8, hd=128, mt=8192, lo=512, sample=4):
        self.L, self.nq, self.nkv, self.hd, self.mt, self.lo = 1, n_q, n_kv, hd, mt, lo
        gen = reference_generator()
        self.all_lens = ragged_lengths(gen, Config3.B, lo, mt)
        off = config3_stream(self.all_lens, n_q, n_kv, hd)
        self.sample = list(range(sample))
        self.sample_lens = self.all_lens[:sample]
        row = hd // QK * BB
        self.kp, self.vp = [], []
        for b in self.sample:
            n = int(self.sample_lens[b])
            for p, planes in enumerate((self.kp, self.vp)):
                x = np.zeros((n_kv, mt, hd), np.float32)
                x[:, :n] = outliers(gen, off["u"](off["kv"](b, p)),
                                    gen.normal(off["kv"](b, p), n_kv * n * hd)).reshape(n_kv, n, hd)
                planes.append(orc.quantize_rows_bulk(x).reshape(n_kv, mt, row))
        self.q = np.stack([gen.normal(off["q"](b), n_q * hd) for b in self.sample])
        self.bytes_per_step = 2 * n_kv * int(self.all_lens.sum()) * row
        self.n = 1

    def describe(self):
        return describe_config3(self.all_lens, self.lo, self.mt, self.nq, self.nkv, self.hd)


class HostConfig4:
    """Config 4 built on the host only, for the reference arm (one layer, 64 q /
    8 kv heads, context 131072, no append)."""
    name = "config4"

    def __init__(self, orc, seed: int, n=131072, n_q=64, n_kv=8, hd=128):
        self.L, self.nq, self.nkv, self.hd, self.n = 1, n_q, n_kv, hd, n
        self.mt, self.pos = n, n - 1
        self.nb = hd // QK
        gen = reference_generator()
        row = self.nb * BB
        self.kp, self.vp = (orc.quantize_rows_bulk(gen.normal(config4_stream(n_kv, n, hd, p, 0), n_kv * n * hd)
                                                   .reshape(n_kv, n, hd)).reshape(1, n_kv, n, row) for p in (0, 1))
        self.q = gen.normal(config4_stream(n_kv, n, hd, 2, 0), n_q * hd).reshape(1, n_q * hd)
        self.kv_bytes = 2 * n_kv * n * row
        self.bytes_per_step = self.kv_bytes

    def host_planes(self):
        return self.kp, self.vp, self.q, None, None

    def describe(self):
        return describe_config4(self.nq, self.nkv, self.hd, self.n)


class HostConfig5:
    """Config 5 built on the host only, for the reference arm."""
    name = "config5"

    def __init__(self, orc, seed: int, n_q=32, n_kv=8, hd=128, pos0=2048, n=2048):
        self.L, self.nq, self.nkv, self.hd, self.pos0, self.n = 1, n_q, n_kv, hd, pos0, n
        self.FLOPS = prefill_flops(n_q, hd, pos0, n)
        self.mt = pos0 + n
        gen = reference_generator()
        off = config5_stream(n_q, n_kv, hd, pos0, n)
        row = hd // QK * BB
        planes = []
        for p in (0, 1):
            x = np.zeros((n_kv, self.mt, hd), np.float32)
            x[:, :pos0] = gen.normal(off["kv"](p, 0), n_kv * pos0 * hd).reshape(n_kv, pos0, hd)
            planes.append(orc.quantize_rows_bulk(x).reshape(n_kv, self.mt, row))
        self.kp, self.vp = planes
        self.q = gen.normal(off["q"], n * n_q * hd).reshape(n, n_q * hd)
        self.k_new = gen.normal(off["k"], n * n_kv * hd).reshape(n, n_kv * hd)
        self.v_new = gen.normal(off["v"], n * n_kv * hd).reshape(n, n_kv * hd)
        self.bytes_per_step = 2 * n_kv * self.mt * row

    def host_planes(self):
        return self.kp, self.vp, self.q, self.k_new, self.v_new

    def describe(self):
        return describe_config5(self.nq, self.nkv, self.hd, self.pos0, self.n)


# ---------------------------------------------------------------------------
# reference CPU path (oracle/_ref: the reference's AVX2 build) -- baseline only
# ---------------------------------------------------------------------------
def reference_oracle():
    """The reference's AVX2 build when it was compiled here, else the restatement."""
    import oracle
    kind = "reference" if oracle.available("ref_avx2") else "port"
    return oracle.Oracle("ref_avx2" if kind == "reference" else "port"), kind


def reference_token_seconds(orc, wl, budget_s: float, max_tokens: int | None = None, min_tokens: int = 2):
    """Times the reference's CPU store_kv + attend_q8 for whole tokens (all
    layers), with all host threads, until `budget_s` passes (at least
    min_tokens).  Returns (median seconds per token, tokens, threads)."""
    threads = os.cpu_count() or 1
    kp, vp, q, kn, vn = wl.host_planes()
    times = []
    t_end = time.perf_counter() + budget_s
    while (time.perf_counter() < t_end or len(times) < min_tokens) and (max_tokens is None or len(times) < max_tokens):
        t0 = time.perf_counter()
        for layer in range(wl.L):
            if kn is not None:
                orc.store_kv(kp[layer], vp[layer], wl.nkv, wl.hd, wl.mt, wl.pos, kn[layer], vn[layer])
            orc.attend(kp[layer], vp[layer], wl.nq, wl.nkv, wl.hd, wl.mt, wl.pos, q[layer], threads=threads)
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times), threads


def reference_ragged_seconds(orc, wl, budget_s: float, min_reps: int = 2):
    """Times the reference's CPU attend_q8 (all host threads) on the sampled
    sequences of config 3; returns (median seconds per batch token at the
    batch's mean length, sequence-tokens timed, threads)."""
    threads = os.cpu_count() or 1
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < min_reps:
        t0 = time.perf_counter()
        for i in range(len(wl.sample)):
            n = int(wl.sample_lens[i])
            orc.attend(wl.kp[i], wl.vp[i], wl.nq, wl.nkv, wl.hd, wl.mt, n - 1, wl.q[i], threads=threads)
        per_key = (time.perf_counter() - t0) / float(wl.sample_lens.sum())  # seconds per cached position
        times.append(per_key * float(wl.all_lens.mean()))
    return statistics.median(times), len(times) * len(wl.sample), threads


def reference_prefill_token_seconds(orc, wl, budget_s: float, sample: int = 32, min_reps: int = 2):
    """Times the reference's CPU attention_layer_batch path (append + causal
    attention, all host threads) on the first `sample` tokens of the chunk,
    repeated until `budget_s` passes.  Returns (median seconds per token,
    tokens timed, threads)."""
    threads = os.cpu_count() or 1
    kp, vp, q, kn, vn = wl.host_planes()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < min_reps:
        t0 = time.perf_counter()
        orc.prefill(kp, vp, wl.nq, wl.nkv, wl.hd, wl.mt, wl.pos0, sample, q[:sample], kn[:sample], vn[:sample],
                    threads=threads)
        times.append((time.perf_counter() - t0) / sample)
    return statistics.median(times), len(times) * sample, threads


# --tiny: shapes small enough for the CPU test of the reference arm (tests/test_bench_cpu.py);
# never a benchmark line
TINY = {2: dict(layers=2, pos=255), 3: dict(mt=256, lo=64), 4: dict(n=2048), 5: dict(pos0=64, n=64),
        7: dict(layers=2, hidden=512, inter=1024, vocab=1000, pos=255),
        6: dict(layers=2, hidden=512, pos=255)}
SCALING = {2: "strong", 3: "strong", 4: "strong", 5: "weak", 6: "weak", 7: "weak"}


def global_batch(config: int, world: int) -> int:
    """Sequences in flight in one step of the whole job: config 3 is a batch of 64, configs 2 and 4 one
    sequence divided over the GPUs, configs 5 and 6 one sequence per GPU (replicas)."""
    return {2: 1, 3: Config3.B, 4: 1}.get(config, world)


def run_reference(args):
    rank, local, world = dist_init(args.gpus)
    if rank != 0:
        return 0  # the reference is a single-process CPU library: rank 0 alone runs it
    orc, kind = reference_oracle()
    gen_kind = reference_generator().kind
    shape = TINY[args.config] if args.tiny else {}
    if args.config == 7:
        wl = HostConfig7(orc, seed=7000, **shape)
        sec, n, threads = reference_forward_seconds(orc, wl, max(1, min(args.steps, 3)))
        sample = (f"{n} tokens through the reference's tq_forward_token ending at position {wl.pos} (a context "
                  f"of 1 + {n} tokens minus one of 1 token, so set-up and cache fill cancel)")
    elif args.config == 6:
        wl = HostConfig6(orc, seed=6000, **shape)
        reference_layers_seconds(orc, wl, 0.0, max_tokens=1, min_tokens=1)
        sec, n, threads = reference_layers_seconds(orc, wl, args.ref_seconds, max_tokens=args.steps,
                                                   min_tokens=min(args.steps, 3))
        sample = f"{n} whole tokens through the reference's attention_layer x {wl.L}, median per token"
    elif args.config == 5:
        wl = HostConfig5(orc, seed=5000, **shape)
        sec, n, threads = reference_prefill_token_seconds(orc, wl, args.ref_seconds)
        sample = (f"{n} tokens: the first 32 tokens of the chunk through the reference's append + causal "
                  f"attention, repeated, median per token")
    elif args.config == 3:
        wl = HostConfig3(orc, seed=3000, **shape)
        sec, n, threads = reference_ragged_seconds(orc, wl, args.ref_seconds)
        sample = (f"{n} sequence-tokens of config 3 (the first 4 sequences through the reference's attend_q8), "
                  f"median, scaled to the batch's mean length")
    else:
        wl = HostConfig2(orc, seed=1000, **shape) if args.config == 2 else HostConfig4(orc, seed=4000, **shape)
        # bounded: at most --steps whole tokens, stopping after --ref-seconds of CPU work
        reference_token_seconds(orc, wl, 0.0, max_tokens=args.warmup, min_tokens=args.warmup)
        sec, n, threads = reference_token_seconds(orc, wl, args.ref_seconds, max_tokens=args.steps,
                                                  min_tokens=min(args.steps, 3))
        sample = (f"{n} whole tokens of {wl.name} ({wl.L} layer(s) of "
                  f"{'store_kv + ' if args.config == 2 else ''}attend_q8), median per token")
    # sec is the CPU time of one token: of one sequence at the batch's mean length for config 3 (whose
    # step is one token of each of its 64 sequences), of one chunk token for config 5 (whose step is
    # the whole chunk), of the whole step otherwise
    value = 1.0 / sec
    per_step = sec * (Config3.B if args.config == 3 else wl.n if args.config == 5 else 1)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": n,
            "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
            "scaling": SCALING[args.config], "vs_baseline": None, "dtype": "int8+fp32",
            "data": f"synthetic, from the reference benches' generator ({gen_kind})",
            "impl": "reference",
            "config": {**wl.describe(), "global_batch": global_batch(args.config, 1),
                       "parallelism": "reference CPU (its OpenMP over kv heads, all host threads)"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                             "sample": sample + f", ~{args.ref_seconds:.0f} s budget"},
            "hbm_gbs_equivalent": (wl.bytes_per_step / Config3.B if args.config == 3 else wl.bytes_per_step)
                                  / sec / 1e9 * (wl.n if args.config == 5 else 1),
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    rank, local, world = dist_init(args.gpus)
    torch.cuda.set_device(local)
    dist = pg_init(world, local)
    from tailorquantkernel_b200 import tqk
    peak, peak_kind = _peaks()

    shape = TINY[args.config] if args.tiny else {}
    if args.config == 2:
        wl = Config2(seed=1000, prologue=args.prologue, rank=rank, world=world, dist=dist, **shape)
    elif args.config == 3:
        wl = Config3(seed=3000, rank=rank, world=world, **shape)
    elif args.config == 4:
        wl = Config4(seed=4000, rank=rank, world=world, dist=dist, exchange=args.exchange, **shape)
    elif args.config == 6:
        wl = Config6(seed=6000 + rank, **shape)
    elif args.config == 7:
        wl = Config7(seed=7000 + rank, **shape)
    else:
        wl = Config5(seed=5000 + rank, **shape)
    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        wl.step()
    barrier(dist)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        barrier(dist)
        ev0.record(stream)
        for _ in range(args.steps):
            wl.step()
        ev1.record(stream)
        barrier(dist)
    t_local = ev0.elapsed_time(ev1) / 1e3
    t = max_over_ranks(dist, t_local)
    status = tqk.device_status()

    # the dominant kernel's own launch time: the step itself on one GPU; on several GPUs (where a
    # step adds the gather or the exchange) the same decode launches timed alone, after the
    # timed region, on the stream they run on
    if world > 1 and hasattr(wl, "kernel_step"):
        for _ in range(3):
            wl.kernel_step()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(args.steps):
            wl.kernel_step()
        k1.record(stream)
        k1.synchronize()
        kernel_s = k0.elapsed_time(k1) / 1e3 / args.steps
    else:
        kernel_s = t_local / args.steps
    kernel_s = max_over_ranks(dist, kernel_s)

    # end to end through the C ABI with host buffers (pinned H2D of q/k/v, D2H of out)
    e2e_steps = min(args.steps, getattr(wl, "e2e_steps", args.steps))
    if hasattr(wl, "prepare_e2e"):
        wl.prepare_e2e()
    for _ in range(10):
        wl.step_e2e()
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        wl.step_e2e()
    t_e2e = max_over_ranks(dist, time.perf_counter() - t0)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and wl.name == "config3":
        orc, kind = reference_oracle()
        sec, n, threads = reference_ragged_seconds(orc, HostConfig3(orc, seed=3000), args.cpu_seconds)
        cpu = {"value": 1.0 / sec, "unit": "tokens/s", "cores": threads, "kind": kind,
               "sample": f"{n} sequence-tokens of config 3 (the first 4 sequences through the reference's "
                         f"attend_q8), ~{args.cpu_seconds:.0f} s budget, median per token, scaled to the batch's "
                         f"mean length"}
    elif rank == 0 and world == 1 and not args.no_cpu_baseline and wl.name == "config5":
        orc, kind = reference_oracle()
        sec, n, threads = reference_prefill_token_seconds(orc, wl, args.cpu_seconds)
        cpu = {"value": 1.0 / sec, "unit": "tokens/s", "cores": threads, "kind": kind,
               "sample": f"{n} tokens: the first 32 tokens of the chunk through the reference's append + causal "
                         f"attention, repeated for ~{args.cpu_seconds:.0f} s, median per token"}
    elif wl.name == "config7":
        cpu = None  # the reference arm (--impl reference --config 7) times the reference's forward
    elif rank == 0 and world == 1 and not args.no_cpu_baseline and wl.name == "config6":
        orc, kind = reference_oracle()
        sec, n, threads = reference_layers_seconds(orc, HostConfig6(orc, seed=6000), args.cpu_seconds)
        cpu = {"value": 1.0 / sec, "unit": "tokens/s", "cores": threads, "kind": kind,
               "sample": f"{n} whole tokens through the reference's attention_layer x 32 (its AVX2 matmuls, "
                         f"Q8 cache at 4096), ~{args.cpu_seconds:.0f} s budget, median per token"}
    elif rank == 0 and world == 1 and not args.no_cpu_baseline:
        orc, kind = reference_oracle()
        sec, n, threads = reference_token_seconds(orc, wl, args.cpu_seconds)
        cpu = {"value": 1.0 / sec, "unit": "tokens/s", "cores": threads, "kind": kind,
               "sample": f"{n} whole tokens of {wl.name} ({wl.L} layer(s) of "
                         f"{'store_kv + ' if wl.name == 'config2' else ''}attend_q8), "
                         f"~{args.cpu_seconds:.0f} s budget, median per token"}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        per_launch = kernel_s
        if getattr(wl, "bound", "hbm") == "tensor":
            tpeak, tpeak_kind = _tensor_peak()
            achieved = wl.FLOPS / per_launch / 1e12
            roofline = {"bound": "tensor", "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
                        "frac": achieved / tpeak, "peak_kind": tpeak_kind,
                        "algorithmic_flops_per_step": wl.FLOPS,
                        "note": "step time includes the 2048-row Q8 append (a separate small kernel)",
                        "traffic": _traffic_from_profile("prefill_q8_" + wl.name)}
        else:
            achieved = wl.bytes_per_step / per_launch / 1e9
            roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                        "frac": achieved / peak, "peak_kind": peak_kind,
                        "algorithmic_bytes_per_launch": wl.bytes_per_step,
                        "traffic": _traffic_from_profile(("layers_" if wl.name in ("config6", "config7")
                                                          else "decode_q8_")
                                                         + wl.name)}
        jobs = world if wl.scaling == "weak" else 1  # weak: every rank runs its own sequence
        if world > 1:
            roofline["note"] = ("the slowest rank's decode launch timed alone (without the step's gather or "
                                "exchange); bytes are that rank's share")
        line = {
            "metric": METRIC,
            "value": jobs * args.steps * wl.tokens_per_step / t,
            "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3,
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
            "dtype": "int8+fp32",
            "data": getattr(wl, "data", "synthetic: N(0,1) from the reference benches' generator (xorshift64 + "
                                        "Box-Muller, seed 88172645463325252; tqk_fill_normal), K/V quantised to Q8 "
                                        "on the device, q RoPE'd"),
            "config": {**wl.describe(), "global_batch": global_batch(args.config, world),
                       "parallelism": wl.parallelism(world)},
            **({"per_gpu": wl.per_rank()} if hasattr(wl, "per_rank") else {}),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": jobs * e2e_steps * wl.tokens_per_step / t_e2e, "unit": "tokens/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h,
                    "api": wl.e2e_api},
            "gpu_launches": args.steps * wl.launches_per_step,
            **({"hbm_gbs": achieved} if roofline["bound"] == "hbm" else {}),
            "clocks": clk.summary(),
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if hasattr(wl, "close"):
        wl.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5, 6, 7])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0, help="CPU budget of the --impl reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="config 4 on several GPUs: the partials' exchange over peer memory or by NCCL")
    ap.add_argument("--tiny", action="store_true",
                    help="shrunken shapes for the CPU test of the reference arm and quick GPU checks; not a "
                         "benchmark of the configs")
    ap.add_argument("--prologue", action="store_true",
                    help="config 2 with the q/k RMSNorm + RoPE prologue fused into the decode launch")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    return run_reference(args) if args.impl == "reference" else run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
