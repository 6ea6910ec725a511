"""Full-array reductions sharded over the GPUs of one node.

One process per GPU.  Each rank holds a contiguous shard [offset, offset +
n_local) of the logical array, reduces it with one kernel launch into a
small partial, and the partials are combined by one collective:

    sum f32   -> f64 partial,                      all_reduce SUM
    sum i32   -> i32 partial (two's-complement),   all_reduce SUM (wraps: bit-exact)
    argmax    -> packed i64 key (signed totalOrder key << 32 | 0xFFFFFFFF - global index),
                                                    all_reduce MAX
    sum of any other ReduceSum input type (f16, bf16, f64, e4m3, e5m2: f64
    partial; u32: its 32 bits carried as i32, which wrap identically)

The partial kernels are the hot-path reductions; the collective is
torch.distributed (NCCL over NVLink on GPUs; gloo in the CPU tests, where
`partial_fn` supplies the per-rank partial instead of a kernel).
"""
from __future__ import annotations

import contextlib
from typing import Any, Callable, Optional

import numpy as np
import torch
import torch.distributed as dist

from .hotpath import (ARGMAX_TYPE_BYTES, ORDERED_GROUP_BYTES, ORDERED_TYPES, POLICIES, REDUCE_ARGMAX_F32, REDUCE_SUM_F32,
                      REDUCE_SUM_I32, SUM_TYPE_BYTES, SUM_TYPE_CODES, argmax_value, unpack_argmax_key)

MAX_PACKED_INDEX = 0xFFFFFFFF  # packed argmax keys carry 32-bit global indices


# Shard granule (elements) for order-fixed sums: a multiple of every input
# type's 256 KiB group, so each GPU holds whole groups.
ORDERED_GRANULE = 1 << 18


def shard_bounds(n_total: int, world: int, rank: int, granule: int = 1) -> tuple[int, int]:
    """Contiguous shard of rank `rank`: [offset, offset + count).  With
    granule 1 the first n_total % world ranks take one extra element; with a
    larger granule every shard but the last non-empty one is a whole number
    of granules (ceil(units / world) each), so only trailing ranks are short."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if granule < 1:
        raise ValueError("granule must be >= 1")
    if granule == 1:
        base, extra = divmod(n_total, world)
        offset = rank * base + min(rank, extra)
        return offset, base + (1 if rank < extra else 0)
    units = -(-n_total // granule)
    per = -(-units // world)
    lo = min(rank * per * granule, n_total)
    hi = min((rank + 1) * per * granule, n_total)
    return lo, hi - lo


def combine_sum_f64(partial: torch.Tensor, group: Any = None) -> torch.Tensor:
    dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial


def combine_sum_i32(partial: torch.Tensor, group: Any = None) -> torch.Tensor:
    dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial


def sum_partial_dtype(dtype: str) -> torch.dtype:
    """Partial (and collective) type of a typed sum: i32 for the 32-bit
    integer inputs, f64 for the floating-point ones."""
    if dtype not in SUM_TYPE_CODES:
        raise ValueError(f"no ReduceSum accumulator for {dtype!r}")
    return torch.int32 if dtype in ("i32", "u32") else torch.float64


def sum_partial_value(dtype: str, partial: torch.Tensor) -> float | int:
    v = partial.item()
    return int(v) % (1 << 32) if dtype == "u32" else v


def combine_argmax(packed: torch.Tensor, group: Any = None) -> torch.Tensor:
    dist.all_reduce(packed, op=dist.ReduceOp.MAX, group=group)
    return packed


_I64_MIN, _I64_MAX = -(1 << 63), (1 << 63) - 1


def combine_argmax_records(rec: torch.Tensor, key_bits: int, group: Any = None) -> torch.Tensor:
    """Replace this rank's argmax record `rec` = [word0, index] (int64[2],
    index -1 when the shard was empty) by the global one: the records are
    all-gathered and every rank picks the largest order key, lowest global
    index on ties.  word0 is the key itself for 64-bit keys (f64) and the
    packed form (key << 32 | 0xFFFFFFFF - index) for 32-bit keys; the
    result keeps that form (low word 0 when the index needs more than 32
    bits) and carries the full index in rec[1].  For 64-bit keys, and for
    arrays whose indices exceed the 32 bits a packed key can carry."""
    if key_bits not in (32, 64):
        raise ValueError("order keys are 32 or 64 bits")
    world = dist.get_world_size(group)
    parts = [torch.empty_like(rec) for _ in range(world)]
    dist.all_gather(parts, rec, group=group)
    g = torch.stack(parts)
    valid = g[:, 1] >= 0
    keys = g[:, 0] if key_bits == 64 else torch.div(g[:, 0], 1 << 32, rounding_mode="floor")
    keys = torch.where(valid, keys, torch.full_like(keys, _I64_MIN))
    best = keys.max()
    idx = torch.where(valid & (keys == best), g[:, 1], torch.full_like(g[:, 1], _I64_MAX)).min()
    if key_bits == 64:
        word0 = best
    else:
        low = torch.where(idx <= MAX_PACKED_INDEX, MAX_PACKED_INDEX - idx, torch.zeros_like(idx))
        word0 = best * (1 << 32) + low
    any_valid = valid.any()
    rec[0] = torch.where(any_valid, word0, torch.full_like(word0, _I64_MIN))
    rec[1] = torch.where(any_valid, idx, torch.full_like(idx, -1))
    return rec


class ShardedReducer:
    """Per-rank reduction + one all_reduce per op.

    `*_async` methods enqueue the kernel on `stream` and start the
    all_reduce asynchronously, so the collective of one op overlaps the
    kernel of the next (the three reductions are independent).  Each op has
    its own partial buffer; before a kernel overwrites it, the stream waits
    for that buffer's previous all_reduce.  Call `wait()` (device-side) before
    reading results on `stream`; the `*_result` helpers do so."""

    def __init__(self, hotpath: Any, device: torch.device, n_total: int, group: Any = None, granule: int = 1):
        self.hp = hotpath
        self.device = device
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_total = n_total
        self.granule = granule
        self.offset, self.count = shard_bounds(n_total, self.world, self.rank, granule)
        self.counts = [shard_bounds(n_total, self.world, r, granule)[1] for r in range(self.world)]
        self.f64 = torch.zeros(1, dtype=torch.float64, device=device)
        self.i32 = torch.zeros(1, dtype=torch.int32, device=device)
        self.arg = torch.zeros(2, dtype=torch.int64, device=device)
        self.workspace = torch.zeros(hotpath.workspace_bytes, dtype=torch.uint8, device=device)
        self.typed: dict[str, torch.Tensor] = {}  # partial of each typed sum
        self.typed_arg: dict[Any, torch.Tensor] = {}  # record of each typed argmax
        self._ordered: dict[str, dict[str, torch.Tensor]] = {}  # per-type buffers of order-fixed sums
        self._ordered_groups: dict[str, int] = {}  # this rank's group count per type
        self._pending: dict[Any, Any] = {}

    @staticmethod
    def _on(stream: Optional[torch.cuda.Stream]):
        """Make `stream` torch's current stream: torch orders collectives and
        Work.wait() against the current stream."""
        return torch.cuda.stream(stream) if isinstance(stream, torch.cuda.Stream) else contextlib.nullcontext()

    def _release(self, key: Any, shard: torch.Tensor, stream: Optional[torch.cuda.Stream]) -> None:
        if shard.numel() != self.count:
            raise ValueError(f"rank {self.rank} shard holds {shard.numel()} elements, expected {self.count}")
        prior = self._pending.pop(key, None)
        if prior is not None:
            with self._on(stream):
                prior.wait()  # the stream waits until that all_reduce has released the partial

    def _reduce(self, op: int, shard: torch.Tensor, out: torch.Tensor, stream: Optional[torch.cuda.Stream]):
        self._release(op, shard, stream)
        self.hp.reduce_into(op, shard, out, n=self.count,
                            stream=stream if stream is not None else torch.cuda.current_stream(),
                            index_base=self.offset, workspace=self.workspace)

    def _combine(self, op: Any, tensor: torch.Tensor, reduce_op, stream: Optional[torch.cuda.Stream]) -> None:
        if self.world > 1:
            with self._on(stream):
                self._pending[op] = dist.all_reduce(tensor, op=reduce_op, group=self.group, async_op=True)

    def wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Make `stream` (default: the current stream) wait for every
        outstanding all_reduce."""
        with self._on(stream):
            for work in self._pending.values():
                work.wait()
        self._pending.clear()

    def sum_f32_async(self, shard: torch.Tensor, stream=None) -> torch.Tensor:
        self._reduce(REDUCE_SUM_F32, shard, self.f64, stream)
        self._combine(REDUCE_SUM_F32, self.f64, dist.ReduceOp.SUM, stream)
        return self.f64

    def sum_i32_async(self, shard: torch.Tensor, stream=None) -> torch.Tensor:
        self._reduce(REDUCE_SUM_I32, shard, self.i32, stream)
        self._combine(REDUCE_SUM_I32, self.i32, dist.ReduceOp.SUM, stream)
        return self.i32

    @property
    def packed_argmax(self) -> bool:
        """Global indices fit the packed key's 32 bits: argmax partials
        combine with one all_reduce MAX; otherwise records are gathered."""
        return self.n_total - 1 <= MAX_PACKED_INDEX

    def argmax_f32_async(self, shard: torch.Tensor, stream=None) -> torch.Tensor:
        self._reduce(REDUCE_ARGMAX_F32, shard, self.arg, stream)
        if self.packed_argmax:
            self._combine(REDUCE_ARGMAX_F32, self.arg[:1], dist.ReduceOp.MAX, stream)
        elif self.world > 1:
            with self._on(stream):
                combine_argmax_records(self.arg, 32, self.group)
        return self.arg

    def argmax_async(self, dtype: str, shard: torch.Tensor, stream=None) -> torch.Tensor:
        """max / argmax of any OrderedType over the sharded array.  32-bit
        order keys travel packed with the index (one all_reduce MAX, as for
        f32); f64 records are all-gathered and the (max key, lowest index)
        winner picked on the device.  Returns the combined 16-byte record."""
        if dtype == "f32":
            return self.argmax_f32_async(shard, stream)
        if dtype not in ARGMAX_TYPE_BYTES:
            raise ValueError(f"no max/argmax order for {dtype!r}")
        key = ("argmax", dtype)
        if key not in self.typed_arg:
            self.typed_arg[key] = torch.zeros(2, dtype=torch.int64, device=self.device)
        rec = self.typed_arg[key]
        self._release(key, shard, stream)
        s = stream if stream is not None else torch.cuda.current_stream()
        self.hp.reduce_argmax_into(dtype, shard, rec, n=self.count, stream=s, index_base=self.offset,
                                   workspace=self.workspace)
        if self.world == 1:
            return rec
        if dtype != "f64" and self.packed_argmax:
            self._combine(key, rec[:1], dist.ReduceOp.MAX, stream)
            return rec
        with self._on(stream):
            combine_argmax_records(rec, 64 if dtype == "f64" else 32, self.group)
        return rec

    def argmax(self, dtype: str, shard: torch.Tensor, stream=None) -> tuple[float | int, int]:
        rec = self.argmax_async(dtype, shard, stream)
        self.wait(stream)
        if dtype == "f32":
            return self.argmax_result(rec)
        r = rec.cpu().numpy()
        if dtype != "f64" and self.world > 1 and self.packed_argmax:
            # after the all_reduce MAX only the packed word is global
            packed = int(r[0])
            if packed == _I64_MIN:
                return float("nan"), -1
            r = np.array([packed, MAX_PACKED_INDEX - (packed & MAX_PACKED_INDEX)], np.int64)
        return argmax_value(dtype, r)

    def _ordered_buffers(self, dtype: str) -> dict[str, torch.Tensor]:
        """Workspace, local / gathered group partials and result of an
        order-fixed sum of `dtype` (allocated on first use)."""
        if dtype not in self._ordered:
            itemsize = SUM_TYPE_BYTES[dtype]
            per_group = ORDERED_GROUP_BYTES // itemsize
            groups = [-(-c // per_group) for c in self.counts]
            m = max(max(groups), 1)
            ws_bytes = self.hp.policy_workspace_bytes(dtype, self.count, "deterministic")
            self._ordered[dtype] = {
                "ws": torch.zeros(ws_bytes, dtype=torch.uint8, device=self.device),
                "local": torch.zeros(m, dtype=torch.float64, device=self.device),
                "gathered": torch.zeros(m * self.world, dtype=torch.float64, device=self.device),
                "out": torch.zeros(1, dtype=torch.float64, device=self.device),
            }
            self._ordered_groups[dtype] = groups[self.rank]
        return self._ordered[dtype]

    def _sum_ordered_async(self, dtype: str, shard: torch.Tensor, policy: str, stream) -> torch.Tensor:
        """Order-fixed sum over the GPUs: each rank writes its shard's group
        partials, one all_gather concatenates them in array order, and every
        rank runs the same final tree -- the same bits as one GPU."""
        itemsize = SUM_TYPE_BYTES[dtype]
        if self.count and ((self.offset * itemsize) % ORDERED_GROUP_BYTES or shard.data_ptr() % 16):
            raise ValueError("order-fixed sharded sums need 16-byte-aligned shards of whole 256 KiB groups "
                             f"(construct the reducer with granule={ORDERED_GRANULE})")
        b = self._ordered_buffers(dtype)
        key = ("ordered", dtype)
        self._release(key, shard, stream)
        s = stream if stream is not None else torch.cuda.current_stream()
        with self._on(stream):
            self.hp.reduce_sum_into(dtype, shard, b["out"], n=self.count, stream=s, workspace=b["ws"], policy=policy)
            ng = self._ordered_groups[dtype]
            b["local"].zero_()
            b["local"][:ng].copy_(b["ws"][256:256 + 8 * ng].view(torch.float64))
            dist.all_gather_into_tensor(b["gathered"], b["local"], group=self.group)
            self.hp.reduce_ordered_final_into(b["gathered"], b["gathered"].numel(), b["out"], stream=s)
        return b["out"]

    def sum_async(self, dtype: str, shard: torch.Tensor, stream=None, policy: str = "fast") -> torch.Tensor:
        """ReduceSum of any accumulator input type over the sharded array:
        one kernel on this rank's shard, one all_reduce SUM of the partial.
        policy "deterministic" / "strict" (floating-point inputs): the
        order-fixed sum, bit-identical to one GPU's (needs granule-aligned
        shards)."""
        if policy not in POLICIES:
            raise ValueError(f"unknown reduction policy {policy!r}")
        if policy != "fast" and dtype in ORDERED_TYPES and self.world > 1:
            return self._sum_ordered_async(dtype, shard, policy, stream)
        if policy != "fast" and dtype in ORDERED_TYPES:
            b = self._ordered_buffers(dtype)
            self._release(("ordered", dtype), shard, stream)
            self.hp.reduce_sum_into(dtype, shard, b["out"], n=self.count,
                                    stream=stream if stream is not None else torch.cuda.current_stream(),
                                    workspace=b["ws"], policy=policy)
            return b["out"]
        if dtype not in self.typed:
            self.typed[dtype] = torch.zeros(1, dtype=sum_partial_dtype(dtype), device=self.device)
        out = self.typed[dtype]
        key = ("sum", dtype)
        self._release(key, shard, stream)
        self.hp.reduce_sum_into(dtype, shard, out, n=self.count,
                                stream=stream if stream is not None else torch.cuda.current_stream(),
                                workspace=self.workspace)
        self._combine(key, out, dist.ReduceOp.SUM, stream)
        return out

    def sum(self, dtype: str, shard: torch.Tensor, stream=None, policy: str = "fast") -> float | int:
        out = self.sum_async(dtype, shard, stream, policy)
        self.wait(stream)
        return sum_partial_value(dtype, out)

    def sum_f32(self, shard: torch.Tensor, stream=None) -> float:
        self.sum_f32_async(shard, stream)
        self.wait(stream)
        return float(self.f64.item())

    def sum_i32(self, shard: torch.Tensor, stream=None) -> int:
        self.sum_i32_async(shard, stream)
        self.wait(stream)
        return int(self.i32.item())

    def argmax_f32(self, shard: torch.Tensor, stream=None) -> tuple[float, int]:
        self.argmax_f32_async(shard, stream)
        self.wait(stream)
        return self.argmax_result(self.arg)

    @staticmethod
    def argmax_result(arg: torch.Tensor) -> tuple[float, int]:
        """(value, global index) of a combined f32 record: the packed word
        carries both while the index fits 32 bits; beyond that the gathered
        record's second word holds the index."""
        packed, index = (int(v) for v in arg.tolist())
        if packed == _I64_MIN:
            return float("nan"), -1
        value, packed_index = unpack_argmax_key(packed)
        return value, index if index > MAX_PACKED_INDEX else packed_index


def cpu_sharded_combine(partial_fn: Callable[[int, int, int], tuple[float, int, int]], n_total: int) -> tuple:
    """The combine steps of ShardedReducer on CPU tensors (gloo): `partial_fn
    (rank, offset, count)` returns this rank's (f64 sum, i32 sum, packed
    argmax key); returns the combined triple.  Used by the multi-process CPU
    tests of the collective logic."""
    world, rank = dist.get_world_size(), dist.get_rank()
    offset, count = shard_bounds(n_total, world, rank)
    s, i, k = partial_fn(rank, offset, count)
    ts = combine_sum_f64(torch.tensor([s], dtype=torch.float64))
    ti = combine_sum_i32(torch.tensor([i], dtype=torch.int32))
    tk = combine_argmax(torch.tensor([k], dtype=torch.int64))
    return float(ts.item()), int(ti.item()), int(tk.item())
