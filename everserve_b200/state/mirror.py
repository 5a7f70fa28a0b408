"""Committed KV mirrored into the per-node store (everserve-store, C++), over mirror.proto.

Per step, on a side stream behind the forward, one kernel launch (``kv_gather``) copies the
step's rows of every layer and every held kv head into a staging file the store can map: a
shared-memory file in the rank's store directory, pinned and mapped into the device, laid out
``[layers, heads, capacity, 2, d]`` (capacities are powers of two from 8, pooled and reused). A
sender thread waits for the copy's event and sends one ``Commit`` naming the file and the step's
slots; the store copies the rows into its tables and acknowledges. ``fence(s)`` waits for step
s's acknowledgement; the engine fences two steps back, so the copy and the send overlap two
decode steps and the step thread never reads device memory. On the CPU engine the rows are copied
synchronously into the staging file.

A spare restores a lost rank from its own node's store: ``Restore`` names each table's file and
written slot ranges, the rows are read from the mapped files and scattered into the cache
(``kv_scatter`` on the device).

Reference parity: MirrorClient / MirrorCommittedKV of core/everserve/state/mirror.py:71-945 (the
same store protocol; the B200 path gathers all layers in one kernel launch into mapped memory).
"""

from __future__ import annotations

import queue
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Mapping

import numpy as np
import torch

from .. import wire
from ..proto import mirror as pb
from ..proto import signals as spb
from .kvcopy import PagedKV

TABLE_STRIDE = 1000  # table id = layer * 1000 + head slot
DEPTH = 2  # steps a rank may run ahead of its acknowledged commits


class MirrorError(RuntimeError):
    pass


_DTYPES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32", torch.uint8: "uint8",
           torch.float8_e4m3fn: "float8_e4m3fn"}
_FROM = {v: k for k, v in _DTYPES.items()}


class MirrorClient:
    """One request/reply connection to the node's store (thread-safe)."""

    def __init__(self, address: str, timeout: float = 30.0):
        self.address = address
        self._sock = wire.connect(address, timeout)
        self._lock = threading.Lock()

    def call(self, req) -> object:
        with self._lock:
            wire.send(self._sock, req.SerializeToString())
            rep = pb.MirrorReply()
            rep.ParseFromString(wire.recv(self._sock))
        if rep.error:
            raise MirrorError(rep.error)
        return rep

    def open(self, engine: str, rank: int):
        return self.call(pb.MirrorRequest(open=pb.Open(engine=engine, rank=rank, protocol=spb.PROTOCOL_VERSION,
                                                       protocol_oldest=spb.PROTOCOL_OLDEST))).opened

    def prepare(self, engine: str, rank: int, tables, dtype: str, shape, slots: int) -> None:
        self.call(pb.MirrorRequest(prepare=pb.Prepare(engine=engine, rank=rank, tables=list(tables), dtype=dtype,
                                                      shape=list(shape), slots=slots)))

    def commit(self, engine: str, rank: int, epoch: int, step: int, staged, counts: Mapping[str, int]) -> int:
        ids = list(counts)
        rep = self.call(pb.MirrorRequest(commit=pb.Commit(
            engine=engine, rank=rank, epoch=epoch, step=step, staged=staged, request_ids=ids,
            committed_tokens=[int(counts[i]) for i in ids])))
        return rep.commit_ack.step

    def restore(self, engine: str, rank: int, since_step: int = 0):
        return self.call(pb.MirrorRequest(restore=pb.RestoreRequest(engine=engine, rank=rank,
                                                                    since_step=since_step))).restore

    def committed(self, engine: str, request_ids) -> dict[str, int]:
        rep = self.call(pb.MirrorRequest(committed=pb.CommittedQuery(engine=engine, request_ids=list(request_ids))))
        return dict(zip(rep.committed.request_ids, rep.committed.committed_tokens))

    def evicted(self, engine: str, request_id: str, kept_tokens: int) -> None:
        self.call(pb.MirrorRequest(evicted=pb.Evicted(engine=engine, request_id=request_id, kept_tokens=kept_tokens)))

    def finished(self, engine: str, request_ids) -> None:
        self.call(pb.MirrorRequest(finished=pb.Finished(engine=engine, request_ids=list(request_ids))))

    def replicate(self, engine: str, rank: int, targets) -> None:
        self.call(pb.MirrorRequest(replicate=pb.Replicate(engine=engine, rank=rank, targets=list(targets))))

    def close(self) -> None:
        try:
            self._sock.close()
        except OSError:
            pass


def pinnable(path: str, mounts: str | None = None) -> bool:
    """Whether pages of files under `path` can be pinned for the device: files on tmpfs (the
    node's /dev/shm). Pinning a mapping of a file on a disk-backed filesystem fails, and has
    crashed the process inside the registration, so it is never attempted there. `mounts`: the
    text of /proc/mounts (read when not given)."""
    if mounts is None:
        try:
            with open("/proc/mounts") as f:
                mounts = f.read()
        except OSError:
            return False
    real = os.path.realpath(path)
    best, fstype = "", ""
    for line in mounts.splitlines():
        parts = line.split()
        if len(parts) < 3:
            continue
        mnt = parts[1].replace("\\040", " ")
        if (real == mnt or real.startswith(mnt.rstrip("/") + "/")) and len(mnt) > len(best):
            best, fstype = mnt, parts[2]
    return fstype == "tmpfs"


@dataclass
class _Stage:
    name: str
    path: str
    tensor: torch.Tensor  # [layers, heads, cap, 2, d] over the shared file
    dev_ptr: int = 0
    # where the file's pages cannot be pinned (a data directory on a disk-backed filesystem, not
    # tmpfs), the gather writes this pinned copy and the sender thread copies it into the file
    bounce: torch.Tensor | None = None

    @property
    def capacity(self) -> int:
        return self.tensor.shape[2]


@dataclass
class _Job:
    epoch: int
    step: int
    counts: dict
    stage: _Stage
    slots: list[int]
    event: object = None
    times: dict = field(default_factory=dict)
    keep: object = None


class MirrorCommittedKV:
    """CommittedKV over everserve-store (see module doc)."""

    def __init__(self, client: MirrorClient, engine: str, rank: int, caches: list[torch.Tensor], kv: PagedKV,
                 heads: list[int] | None = None, depth: int = DEPTH, store_slots: int | None = None):
        self.client, self.engine, self.rank = client, engine, rank
        self.caches, self.kv = caches, kv
        self.heads = list(range(kv.heads)) if heads is None else list(heads)
        self.device = caches[0].device
        self.dtype = caches[0].dtype
        self.depth = depth
        opened = client.open(engine, rank)
        self.rank_dir, self.stage_prefix = opened.rank_dir, opened.stage_prefix
        self._seq = 0
        self._pool: list[_Stage] = []
        self._pool_lock = threading.Lock()
        self._jobs: queue.Queue = queue.Queue()
        self._acked = -1
        self._ack_cond = threading.Condition()
        self._error: BaseException | None = None
        self._committed: dict[str, int] = {}
        self.restored_step = -1  # the last step a restore covered
        self._pinnable: bool | None = None  # staging files pinnable in place (see pinnable)
        self._pending_slots: list[int] = []
        self._history: list[dict] = []
        self.stats_record = {"commits": 0, "fence_waits": 0, "fence_wait_s": 0.0, "bytes": 0}
        self._side = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self._C = None
        if self.device.type == "cuda":
            from .. import _ext

            self._C = _ext.load()
            self._layer_ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64, device=self.device)
            self._heads_dev = torch.tensor(self.heads, dtype=torch.int64, device=self.device)
        self._sender = threading.Thread(target=self._send_loop, name=f"mirror-sender-{rank}", daemon=True)
        self._sender.start()
        if store_slots:
            client.prepare(engine, rank, self.tables(), _DTYPES[self.dtype], [2, kv.head_dim], store_slots)

    def tables(self) -> list[int]:
        return [l * TABLE_STRIDE + h for l in range(len(self.caches)) for h in self.heads]

    # ---- staging files -------------------------------------------------------------------------
    def _staging(self, n: int) -> _Stage:
        cap = max(8, 1 << max(0, (n - 1).bit_length()))
        shape = (len(self.caches), len(self.heads), cap, 2, self.kv.head_dim)
        with self._pool_lock:
            for i, st in enumerate(self._pool):
                if tuple(st.tensor.shape) == shape:
                    return self._pool.pop(i)
        self._seq += 1
        name = f"{self.stage_prefix}{self._seq}.rows"
        path = f"{self.rank_dir}/{name}"
        numel = int(np.prod(shape))
        nbytes = numel * torch.empty((), dtype=self.dtype).element_size()
        with open(path, "wb") as f:
            f.truncate(nbytes)
        t = torch.from_file(path, shared=True, size=numel, dtype=self.dtype).view(shape)
        st = _Stage(name, path, t)
        if self._C is not None:
            if self._pinnable is None:
                self._pinnable = pinnable(self.rank_dir)
            if self._pinnable:
                st.dev_ptr = int(self._C.host_register_mapped(t.data_ptr(), nbytes))
            else:
                # runtime-allocated pinned memory the gather writes through its device address
                st.bounce = torch.empty(shape, dtype=self.dtype, pin_memory=True)
                st.dev_ptr = int(self._C.host_device_pointer(st.bounce.data_ptr()))
        return st

    def _release(self, st: _Stage) -> None:
        with self._pool_lock:
            if len(self._pool) <= self.depth + 1:
                self._pool.append(st)
                return
        if self._C is not None and st.dev_ptr and st.bounce is None:
            self._C.host_unregister(st.tensor.data_ptr())

    # ---- the pipeline --------------------------------------------------------------------------
    def save(self, layer: int, kv: torch.Tensor | None = None, slots: torch.Tensor | None = None) -> None:
        """Layers write their rows in the forward; the commit gathers every layer in one launch."""

    def commit(self, epoch: int, step: int, counts: Mapping[str, int], slots=None) -> None:
        if self._error is not None:
            raise MirrorError(f"the store link failed: {self._error}")
        slot_list = [int(s) for s in (slots.tolist() if isinstance(slots, torch.Tensor) else (slots or []))]
        st = self._staging(max(1, len(slot_list)))
        job = _Job(epoch, step, dict(counts), st, slot_list)
        job.times["commit"] = time.perf_counter()
        if slot_list:
            if self._C is not None:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(self.device))
                # the slots go up from pinned memory without blocking the host: a pageable copy
                # would wait for the side stream, i.e. for the step, before the next step launches
                host_sl = torch.tensor(slot_list, dtype=torch.int64).pin_memory()
                with torch.cuda.stream(self._side):
                    self._side.wait_event(ev)
                    sl = host_sl.to(self.device, non_blocking=True)
                    self._C.kv_gather(self._layer_ptrs, sl, self._heads_dev, st.dev_ptr, st.capacity, self.kv.head_dim,
                                      self.kv.block_size, self.kv.strides(), st.tensor.element_size())
                    done = torch.cuda.Event()
                    done.record(self._side)
                job.event = done
                job.keep = (host_sl, sl)  # alive until the gather has run (the sender waits on `done`)
                self._last_gather = done
            else:
                sl = torch.tensor(slot_list, dtype=torch.int64)
                heads = torch.tensor(self.heads, dtype=torch.int64)
                for l, cache in enumerate(self.caches):
                    st.tensor[l, :, : len(slot_list)] = self.kv.rows_of_heads(cache, sl, heads)
        self._committed.update({k: int(v) for k, v in counts.items()})
        self._jobs.put(job)
        self.stats_record["commits"] += 1

    def _describe(self, job: _Job):
        st = job.stage
        row_bytes = 2 * self.kv.head_dim * st.tensor.element_size()
        return pb.StagedStep(
            stage=st.name, base_offset=0, layer_stride=len(self.heads) * st.capacity * row_bytes,
            head_stride=st.capacity * row_bytes, layers=list(range(len(self.caches))), heads=self.heads,
            table_stride=TABLE_STRIDE, slots=job.slots, dtype=_DTYPES[self.dtype], shape=[2, self.kv.head_dim])

    def _send_loop(self) -> None:
        while True:
            job = self._jobs.get()
            if job is None:
                return
            try:
                if job.event is not None:
                    job.event.synchronize()
                if job.stage.bounce is not None and job.slots:
                    n = len(job.slots)
                    job.stage.tensor[:, :, :n].copy_(job.stage.bounce[:, :, :n])
                job.times["gathered"] = time.perf_counter()
                staged = self._describe(job) if job.slots else None
                self.client.commit(self.engine, self.rank, job.epoch, job.step, staged, job.counts)
                job.times["acked"] = time.perf_counter()
                self.stats_record["bytes"] += len(job.slots) * len(self.caches) * len(self.heads) * 2 * \
                    self.kv.head_dim * job.stage.tensor.element_size()
                self._history.append(job.times)
                del self._history[:-256]
                with self._ack_cond:
                    self._acked = max(self._acked, job.step)
                    self._ack_cond.notify_all()
            except BaseException as e:  # noqa: BLE001 - surfaced by fence/commit
                with self._ack_cond:
                    self._error = e
                    self._ack_cond.notify_all()
            finally:
                self._release(job.stage)

    def fence(self, step: int, timeout_s: float = 30.0) -> None:
        if step < 0:
            return
        t0 = time.perf_counter()
        with self._ack_cond:
            while self._acked < step and self._error is None:
                if not self._ack_cond.wait(timeout=max(0.0, timeout_s - (time.perf_counter() - t0))):
                    if time.perf_counter() - t0 >= timeout_s:
                        raise MirrorError(f"step {step} was not acknowledged within {timeout_s} s")
        waited = time.perf_counter() - t0
        if waited > 1e-4:
            self.stats_record["fence_waits"] += 1
            self.stats_record["fence_wait_s"] += waited
        if self._error is not None:
            raise MirrorError(f"the store link failed: {self._error}")

    def join_stream(self, stream=None) -> None:
        """Make `stream` (default: the current one) wait for the last gather launched, so work
        recorded after it on that stream also covers the commits' device copies."""
        ev = getattr(self, "_last_gather", None)
        if ev is not None:
            (stream or torch.cuda.current_stream(self.device)).wait_event(ev)

    def flush(self, timeout_s: float = 30.0) -> None:
        """Wait for every commit issued so far."""
        deadline = time.perf_counter() + timeout_s
        while not self._jobs.empty() and time.perf_counter() < deadline:
            time.sleep(0.001)
        with self._ack_cond:
            pass

    def committed(self, request_id: str) -> int:
        return self._committed.get(request_id, 0)

    def stats(self):
        return dict(self.stats_record)

    def timeline(self):
        return list(self._history)

    def evicted(self, request_id: str, kept_tokens: int) -> None:
        self._committed[request_id] = kept_tokens
        self.client.evicted(self.engine, request_id, kept_tokens)

    def finished(self, request_id: str) -> None:
        self._committed.pop(request_id, None)
        self.client.finished(self.engine, [request_id])

    def clear(self) -> None:
        self._committed.clear()

    def close(self) -> None:
        self._jobs.put(None)
        self._sender.join(timeout=5)
        with self._pool_lock:
            pool, self._pool = self._pool, []
        for st in pool:
            if self._C is not None and st.dev_ptr and st.bounce is None:
                self._C.host_unregister(st.tensor.data_ptr())

    # ---- restore -------------------------------------------------------------------------------
    def restore(self, dead_rank: int, moves=None, since_step: int = 0) -> dict[str, int]:
        """Write `dead_rank`'s committed rows into this rank's caches; returns committed counts."""
        rep = self.client.restore(self.engine, dead_rank, since_step)
        self.restored_step = int(rep.step)
        for ref in rep.tables:
            layer, head = divmod(ref.layer, TABLE_STRIDE)
            if layer >= len(self.caches) or head not in self.heads:
                continue
            slots = [s for r in ref.written for s in range(r.start, r.start + r.count)]
            if not slots:
                continue
            num = int(np.prod(list(ref.shape)))
            table = torch.from_file(ref.path, shared=False, size=num, dtype=_FROM[ref.dtype]).view(*ref.shape)
            sl = torch.tensor(slots, dtype=torch.int64)
            rows = table.index_select(0, sl).unsqueeze(0)  # [1 head, n, 2, d]
            hi = torch.tensor([head], dtype=torch.int64)
            cache = self.caches[layer]
            if self._C is not None:
                host = rows.contiguous().pin_memory()
                dev_rows = host.to(self.device, non_blocking=True)
                ptr = torch.tensor([cache.data_ptr()], dtype=torch.int64, device=self.device)
                self._C.kv_scatter(ptr, sl.to(self.device), hi.to(self.device), dev_rows.data_ptr(), len(slots),
                                   self.kv.head_dim, self.kv.block_size, self.kv.strides(), cache.element_size())
            else:
                self.kv.write_rows(cache, sl, hi, rows)
        if self._C is not None:
            torch.cuda.synchronize(self.device)
        counts = dict(zip(rep.request_ids, rep.committed_tokens))
        self._committed.update(counts)
        return counts
