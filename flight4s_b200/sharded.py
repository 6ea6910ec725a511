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

Failure handling (the reference has one GPU per context and no collective,
so this follows its host-side failure model: errors surface as exceptions
on the host, nothing hangs):
  * `RankMonitor` -- liveness through the process group's store: each rank
    announces the step it is about to run, and before launching anything a
    rank checks that every peer has announced that step.  A peer that left
    (`leave()`) or fell silent raises `RankFailure` on the survivors, on
    the host, before any kernel or collective of that step is queued.
  * `PendingCollectives.wait_checked(timeout_s)` -- a bounded host wait on
    the in-flight collectives: a collective that fails (a peer's
    connection closed) or does not finish in time aborts the communicator
    (`ProcessGroup.abort`, which for NCCL is ncclCommAbort) and raises
    `CollectiveFailure` / `CollectiveTimeout`.  The NCCL backend's own
    watchdog polls ncclCommGetAsyncError and enforces the process group's
    timeout behind this.
"""
from __future__ import annotations

import contextlib
import time
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


class CollectiveFailure(RuntimeError):
    """A collective of the sharded combine failed; its communicator has
    been aborted and the process group must be destroyed and recreated."""


class CollectiveTimeout(CollectiveFailure):
    """A collective did not complete within its bound (a peer stopped
    answering); the communicator has been aborted."""


class RankFailure(RuntimeError):
    """A peer rank left the job or stopped announcing steps; raised on the
    host before this rank queues any work of the step."""


def abort_group(group: Any = None) -> None:
    """Abort the communicator of `group` (default: the world group) so no
    rank blocks in it any longer.  For NCCL this is ncclCommAbort."""
    pg = group if group is not None else dist.group.WORLD
    try:
        pg.abort()
    except Exception:  # already aborted or torn down: nothing left to unblock
        pass


class PendingCollectives:
    """The in-flight asynchronous all_reduces of a reducer, one per key.

    `release(key)` orders the current stream after the key's previous
    collective (its buffer is about to be rewritten), `wait()` orders the
    current stream after all of them without blocking the host, and
    `wait_checked(timeout_s)` blocks the host for at most `timeout_s`: a
    collective that failed or is still running then aborts the
    communicator and raises."""

    def __init__(self, group: Any = None):
        self.group = group
        self._pending: dict[Any, Any] = {}

    def __contains__(self, key: Any) -> bool:
        return key in self._pending

    def __len__(self) -> int:
        return len(self._pending)

    def start(self, key: Any, tensor: torch.Tensor, op: Any) -> None:
        self._pending[key] = dist.all_reduce(tensor, op=op, group=self.group, async_op=True)

    def release(self, key: Any) -> None:
        prior = self._pending.pop(key, None)
        if prior is not None:
            prior.wait()

    def wait(self) -> None:
        for work in self._pending.values():
            work.wait()
        self._pending.clear()

    def wait_checked(self, timeout_s: float, poll_s: float = 2e-4) -> None:
        deadline = time.monotonic() + timeout_s
        for key, work in list(self._pending.items()):
            while not work.is_completed():
                if time.monotonic() > deadline:
                    self._pending.clear()
                    abort_group(self.group)
                    raise CollectiveTimeout(f"collective {key!r} did not complete within {timeout_s:g} s; "
                                            "communicator aborted")
                time.sleep(poll_s)
            try:
                work.wait()  # raises the collective's error, if it had one
            except Exception as exc:
                self._pending.clear()
                abort_group(self.group)
                raise CollectiveFailure(f"collective {key!r} failed: {exc}; communicator aborted") from exc
        self._pending.clear()


class RankMonitor:
    """Host-side liveness of the ranks of a process group, through the
    group's store (a TCP key-value store every rank reaches without the
    communicator).  Each rank calls `enter_step(s)` before queuing the work
    of step s: it announces s and returns once every peer has announced s,
    or raises `RankFailure` if a peer has left (`leave()`) or has not
    announced s within `timeout_s`.  A rank that stops between steps is
    therefore noticed before anything of the next step is launched."""

    def __init__(self, group: Any = None, timeout_s: float = 10.0, poll_s: float = 1e-3, prefix: str = "f4s/ranks",
                 store: Any = None):
        self.group = group
        pg = group if group is not None else dist.group.WORLD
        self.store = store if store is not None else pg.get_group_store()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = timeout_s
        self.poll_s = poll_s
        self.prefix = prefix
        self.step = 0

    def _key(self, what: str, rank: int) -> str:
        return f"{self.prefix}/{what}/{rank}"

    def enter_step(self, step: Optional[int] = None) -> int:
        step = self.step + 1 if step is None else step
        if step <= self.step:
            raise ValueError(f"steps must increase: {step} after {self.step}")
        try:
            self.store.add(self._key("step", self.rank), step - self.step)
        except Exception as exc:
            raise RankFailure(f"rank liveness store unreachable before step {step}: {exc}") from exc
        self.step = step
        deadline = time.monotonic() + self.timeout_s
        waiting = [r for r in range(self.world) if r != self.rank]
        while waiting:
            still = []
            for r in waiting:
                try:
                    left = self.store.add(self._key("left", r), 0)
                    reached = self.store.add(self._key("step", r), 0)
                except Exception as exc:  # the store went away with the rank hosting it
                    raise RankFailure(f"rank liveness store unreachable before step {step}: {exc}") from exc
                if left:
                    raise RankFailure(f"rank {r} left the job before step {step}")
                if reached < step:
                    still.append(r)
            waiting = still
            if waiting:
                if time.monotonic() > deadline:
                    raise RankFailure(f"rank(s) {waiting} did not reach step {step} within {self.timeout_s:g} s")
                time.sleep(self.poll_s)
        return step

    def leave(self) -> None:
        """Announce that this rank leaves between steps; peers raise
        RankFailure at their next `enter_step`."""
        self.store.add(self._key("left", self.rank), 1)


class ShardedReducer:
    """Per-rank reduction + one all_reduce per op.

    `*_async` methods enqueue the kernel on `stream` and start the
    all_reduce asynchronously, so the collective of one op overlaps the
    kernel of the next (the three reductions are independent).  Each op has
    its own partial buffer; before a kernel overwrites it, the stream waits
    for that buffer's previous all_reduce.  Call `wait()` (device-side) before
    reading results on `stream`; the `*_result` helpers do so.

    Inside `batch()` the kernels of several ops are queued back to back and
    their all_reduces start together when the block ends; the f32 sum, i32
    sum and f32 argmax then alternate between two partial buffers, so the
    next batch's kernels never wait for this batch's collectives.  With the
    hot path's launch overlap on, consecutive kernels of a batch also
    overlap each other's start and finish (nothing is recorded between them).

    Failure handling: `wait_checked(timeout_s)` bounds the host's wait for
    the in-flight collectives (a failed or overdue one aborts the
    communicator and raises `CollectiveFailure` / `CollectiveTimeout`), and
    with a `monitor` (a `RankMonitor`) `begin_step()` raises `RankFailure`
    before a step's first launch when a peer has left."""

    def __init__(self, hotpath: Any, device: torch.device, n_total: int, group: Any = None, granule: int = 1,
                 monitor: Optional[RankMonitor] = None):
        self.hp = hotpath
        self.device = device
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_total = n_total
        self.granule = granule
        self.offset, self.count = shard_bounds(n_total, self.world, self.rank, granule)
        self.counts = [shard_bounds(n_total, self.world, r, granule)[1] for r in range(self.world)]
        # two partial buffers per op; `_cur` is the one written last
        self._partials = {REDUCE_SUM_F32: [torch.zeros(1, dtype=torch.float64, device=device) for _ in range(2)],
                          REDUCE_SUM_I32: [torch.zeros(1, dtype=torch.int32, device=device) for _ in range(2)],
                          REDUCE_ARGMAX_F32: [torch.zeros(2, dtype=torch.int64, device=device) for _ in range(2)]}
        self._cur = {op: 0 for op in self._partials}
        self._deferred: Optional[list] = None  # collectives queued inside batch()
        self.workspace = torch.zeros(hotpath.workspace_bytes, dtype=torch.uint8, device=device)
        self.typed: dict[str, torch.Tensor] = {}  # partial of each typed sum
        self.typed_arg: dict[Any, torch.Tensor] = {}  # record of each typed argmax
        self._ordered: dict[str, dict[str, torch.Tensor]] = {}  # per-type buffers of order-fixed sums
        self._ordered_groups: dict[str, int] = {}  # this rank's group count per type
        self._pending = PendingCollectives(group)
        self.monitor = monitor

    @property
    def f64(self) -> torch.Tensor:
        """The f32 sum's partial (after wait(): the combined sum) of the last launch."""
        return self._partials[REDUCE_SUM_F32][self._cur[REDUCE_SUM_F32]]

    @property
    def i32(self) -> torch.Tensor:
        return self._partials[REDUCE_SUM_I32][self._cur[REDUCE_SUM_I32]]

    @property
    def arg(self) -> torch.Tensor:
        return self._partials[REDUCE_ARGMAX_F32][self._cur[REDUCE_ARGMAX_F32]]

    def _target(self, op: int) -> tuple[Any, torch.Tensor]:
        """(pending key, buffer) the next launch of `op` writes.  In a batch
        it is the buffer not written last time, whose collective (two
        batches back) has long finished; otherwise the same buffer."""
        idx = self._cur[op] ^ 1 if self._deferred is not None else self._cur[op]
        self._cur[op] = idx
        return (op, idx), self._partials[op][idx]

    @contextlib.contextmanager
    def batch(self, stream: Optional[torch.cuda.Stream] = None):
        """Queue several reductions on `stream` back to back and start their
        all_reduces together when the block ends (see the class notes)."""
        if self._deferred is not None:
            raise RuntimeError("batches do not nest")
        # The buffers this batch writes were last combined two batches ago:
        # order the stream after those collectives here, before the first
        # kernel, so nothing is queued between the batch's kernels.
        with self._on(stream):
            for op, idx in self._cur.items():
                if (op, idx ^ 1) in self._pending:
                    self._pending.release((op, idx ^ 1))
        self._deferred = []
        try:
            yield self
        finally:
            deferred, self._deferred = self._deferred, None
            if self.world > 1:
                with self._on(stream):
                    for key, tensor, reduce_op in deferred:
                        self._pending.start(key, tensor, reduce_op)

    @staticmethod
    def _on(stream: Optional[torch.cuda.Stream]):
        """Make `stream` torch's current stream: torch orders collectives and
        Work.wait() against the current stream."""
        return torch.cuda.stream(stream) if isinstance(stream, torch.cuda.Stream) else contextlib.nullcontext()

    def _release(self, key: Any, shard: torch.Tensor, stream: Optional[torch.cuda.Stream]) -> None:
        if shard.numel() != self.count:
            raise ValueError(f"rank {self.rank} shard holds {shard.numel()} elements, expected {self.count}")
        if key in self._pending:
            with self._on(stream):
                self._pending.release(key)  # the stream waits until that all_reduce has released the partial

    def _combine(self, op: Any, tensor: torch.Tensor, reduce_op, stream: Optional[torch.cuda.Stream]) -> None:
        if self.world > 1:
            if self._deferred is not None:
                self._deferred.append((op, tensor, reduce_op))
                return
            with self._on(stream):
                self._pending.start(op, tensor, reduce_op)

    def wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Make `stream` (default: the current stream) wait for every
        outstanding all_reduce."""
        with self._on(stream):
            self._pending.wait()

    def wait_checked(self, timeout_s: float, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Block the host until every outstanding all_reduce has completed,
        for at most `timeout_s`; a failed or overdue collective aborts the
        communicator and raises CollectiveFailure / CollectiveTimeout."""
        with self._on(stream):
            self._pending.wait_checked(timeout_s)

    def begin_step(self, step: Optional[int] = None) -> int:
        """With a monitor: announce the next step and raise RankFailure if a
        peer has left or not reached it (nothing of the step is queued yet).
        Without one: a no-op returning 0."""
        return self.monitor.enter_step(step) if self.monitor is not None else 0

    def abort(self) -> None:
        """Abort the communicator: in-flight collectives end with an error
        on every rank instead of waiting for a peer that is gone."""
        abort_group(self.group)

    def _reduce_partial(self, op: int, shard: torch.Tensor, stream) -> tuple[Any, torch.Tensor]:
        key, out = self._target(op)
        self._release(key, shard, stream)
        self.hp.reduce_into(op, shard, out, n=self.count,
                            stream=stream if stream is not None else torch.cuda.current_stream(),
                            index_base=self.offset, workspace=self.workspace)
        return key, out

    def sum_f32_async(self, shard: torch.Tensor, stream=None) -> torch.Tensor:
        key, out = self._reduce_partial(REDUCE_SUM_F32, shard, stream)
        self._combine(key, out, dist.ReduceOp.SUM, stream)
        return out

    def sum_i32_async(self, shard: torch.Tensor, stream=None) -> torch.Tensor:
        key, out = self._reduce_partial(REDUCE_SUM_I32, shard, stream)
        self._combine(key, out, dist.ReduceOp.SUM, stream)
        return out

    @property
    def packed_argmax(self) -> bool:
        """Global indices fit the packed key's 32 bits: argmax partials
        combine with one all_reduce MAX; otherwise records are gathered."""
        return self.n_total - 1 <= MAX_PACKED_INDEX

    def argmax_f32_async(self, shard: torch.Tensor, stream=None) -> torch.Tensor:
        key, out = self._reduce_partial(REDUCE_ARGMAX_F32, shard, stream)
        if self.packed_argmax:
            self._combine(key, out[:1], dist.ReduceOp.MAX, stream)
        elif self.world > 1:
            with self._on(stream):
                combine_argmax_records(out, 32, self.group)
        return out

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
