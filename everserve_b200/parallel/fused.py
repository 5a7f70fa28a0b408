"""The tensor-parallel collective on peer memory: fused GEMM + all-reduce and a failure-detecting
all-reduce, with NCCL for what the kernels do not take.

One instance per rank. It owns the rank's symmetric buffer (a driver VMM allocation outside
torch's allocator, shared by file descriptor: ``parallel.symm``; its memory outlives a member that
dies, so survivors' bounded waits end cleanly), maps every member's buffer, and keeps small device tables
the kernels read on every launch (so captured CUDA graphs follow membership changes): the member
buffers' addresses, the member order, and the call counter. Its control words live in the slot
region (``parallel.slot``), mapped into the device.

Implements the reference's slot-collective protocol (core/everserve/comm/slot.py:22-48):
``can_take``, ``all_reduce_into``, ``set_members``, ``abort``, ``resume``, ``variant``.
"""

from __future__ import annotations

import atexit
import os
import threading
import uuid

import torch
import torch.distributed as dist

from .. import _ext
from ..ops import prefetch_target, weight_args
from .nccl import GroupCollective
from .slot import HANDLE_BYTES, MAX_ROWS, SlotRegion
from .symm import PeerMapping, SymmetricBuffer


BEAT_PERIOD_US = 500  # how often a member's heartbeat thread advances its beat word


class FusedTPCollective:
    """``nvls=True`` pushes through an NVSwitch multicast mapping of the members' buffers (one copy
    leaves each GPU); the buffers then come from torch's symmetric-memory rendezvous and the
    members are fixed (rows = ranks). The default P2P variant pushes with stores into each
    member's IPC-mapped buffer and supports membership changes; it is the one used wherever a
    member may die (a dead process bound to a multicast object is not survivable on this pool)."""

    def __init__(self, device: torch.device, group=None, region: SlotRegion | None = None, row: int | None = None,
                 members: list[int] | None = None, region_name: str | None = None, nvls: bool = False,
                 barrier=None):
        """With `group` (a torch.distributed group) the members are its ranks and NCCL carries what
        the kernels do not take. Detached (no group: `region`, `row`, `members` and a `barrier`
        callable given) the members are rows of an existing region and every collective runs on
        the peer-memory kernels (large all-reduces in chunks, all-gathers as sums of disjoint
        slices), so a membership change needs no communicator at all."""
        self.C = _ext.load()
        self.device = torch.device(device)
        self.group = group
        self.detached = group is None and region is not None
        if self.detached:
            if members is None or row is None or barrier is None:
                raise ValueError("a detached collective needs its region row, members and a barrier")
            self.nccl = None
            self.size = len(members)
            self.rank = members.index(row) if row in members else -1
            self._barrier = barrier
        else:
            self.nccl = GroupCollective(group)
            self.size = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
            self._barrier = lambda: dist.barrier(group)
        self.row = self.rank if row is None else row
        self._own_region = region is None
        if region is None:
            name = region_name or self._agree_name()
            if self.rank == 0:
                region = SlotRegion.create(name)
            dist.barrier(group)
            if self.rank != 0:
                region = SlotRegion.open(name)
        self.region = region
        self.max_elems = int(self.C.comm_max_elems(len(members) if members is not None else self.size))
        self.two_shot = 1 if os.environ.get("ES_AR_TWO_SHOT", "0") == "1" else 0
        self.nvls = bool(nvls)
        self.mc = 0
        self._symm = None
        self._addrs = [0] * MAX_ROWS
        self._opened: dict[int, PeerMapping] = {}
        self._map_lock = threading.RLock()
        nbytes = int(self.C.comm_buffer_bytes())
        with torch.cuda.device(self.device):
            self.region.map_device(self.C)
            self.ctrl = self.region.ctrl_device(self.row)
            self.peers = torch.zeros(MAX_ROWS, dtype=torch.int64, device=self.device)
            self.order = torch.zeros(1 + MAX_ROWS, dtype=torch.int32, device=self.device)
            self.call = torch.zeros(2, dtype=torch.int32, device=self.device)
            self.seqs = torch.zeros(8192, dtype=torch.int32, device=self.device)
            if self.nvls:
                import torch.distributed._symmetric_memory as symm_mem

                self._symm = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
                self._symm.zero_()
                torch.cuda.synchronize(self.device)
                name = (group or dist.group.WORLD).group_name
                h = symm_mem.rendezvous(self._symm, name)
                self.mc = int(getattr(h, "multicast_ptr", 0) or 0)
                if not self.mc:
                    raise RuntimeError("no NVLS multicast mapping for this group")
                for r, ptr in enumerate(h.buffer_ptrs):
                    self._addrs[r] = int(ptr)
                self.own = self._addrs[self.row]
            else:
                self._buf = SymmetricBuffer(self.C, nbytes, self._sock_path(self.row))
                self.own = self._buf.ptr
                self._addrs[self.row] = self.own
        self.region.set_pid(self.row, os.getpid())
        # this member's heartbeat (a native thread): peers' kernels name it dead when it stops. It
        # writes into the slot region's mapping, so it stops before the process unmaps it, also when
        # the owner never calls close()
        self._beat = int(self.C.heartbeat_start(self.region.beat_address(self.row), BEAT_PERIOD_US))
        atexit.register(self._stop_beat)
        if not self.nvls:
            name = os.path.basename(self._sock_path(self.row)).encode()
            self.region.publish(self.row, name + bytes(HANDLE_BYTES - len(name)))
        self.members = list(members) if members is not None else list(range(self.size))
        self._barrier()
        if self.nvls:
            with torch.cuda.device(self.device):
                self.peers.copy_(torch.tensor(self._addrs, dtype=torch.int64))
        else:
            self._open(self.members)
        self._write_order()
        self._counting = None
        # objects on this group's members and control words (the routed experts' all-to-all) that
        # follow its membership changes: set_members(rows), resume(), close()
        self.attached: list = []
        if self.nvls:
            self.variant = "nvls"
        else:
            self.variant = "p2p"

    def _agree_name(self) -> str:
        obj = [f"es_slot_{os.getpid()}_{uuid.uuid4().hex[:8]}"]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(self.group, 0) if self.group else 0, group=self.group)
        return obj[0]

    # ---- tables --------------------------------------------------------------------------------
    def _sock_path(self, row: int) -> str:
        return f"{self.region.path}.r{row}.fd"

    def _open(self, rows) -> None:
        with self._map_lock:
            self._open_locked(rows)

    def _open_locked(self, rows) -> None:
        for r in rows:
            if r == self.row or r in self._opened:
                continue
            name = self.region.handle(r).rstrip(b"\0").decode()
            with torch.cuda.device(self.device):
                self._opened[r] = PeerMapping(self.C, os.path.join(os.path.dirname(self.region.path), name))
            self._addrs[r] = self._opened[r].ptr
        with torch.cuda.device(self.device):
            self.peers.copy_(torch.tensor(self._addrs, dtype=torch.int64))

    def premap(self, rows) -> None:
        """Map buffers of rows that may become members (a standing spare's) ahead of time."""
        with self._map_lock:
            self._open(rows)

    def release_rows(self, rows) -> None:
        """Unmap rows that are no longer members (call with this member quiescent)."""
        torch.cuda.synchronize(self.device)
        for r in rows:
            m = self._opened.pop(r, None)
            if m is not None:
                m.close()
                self._addrs[r] = 0
        with torch.cuda.device(self.device):
            self.peers.copy_(torch.tensor(self._addrs, dtype=torch.int64))

    def _write_order(self) -> None:
        rows = [len(self.members), *self.members] + [0] * (MAX_ROWS - len(self.members))
        self.region.set_order(self.row, self.members)
        with torch.cuda.device(self.device):
            self.order.copy_(torch.tensor(rows, dtype=torch.int32))

    def _comm(self):
        return self.peers, self.order, self.call, self.ctrl, self.row, self.mc, self.seqs

    # ---- slot-collective protocol --------------------------------------------------------------
    def can_take(self, t: torch.Tensor) -> bool:
        return (t.dtype == torch.bfloat16 and t.is_contiguous() and t.device == self.device
                and t.numel() <= self.max_elems and t.data_ptr() % 16 == 0)

    def all_reduce_into(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if self.can_take(inp) and out.is_contiguous() and out.data_ptr() % 16 == 0:
            self.C.fdar(inp, out, *self._comm())
            return out
        if self.nccl is None or inp.dtype == torch.bfloat16:
            # above one call's size: several calls of the same failure-detecting kernels
            return self._chunked_all_reduce(inp, out)
        if out.data_ptr() != inp.data_ptr():
            out.copy_(inp)
        return self.nccl.all_reduce(out)

    def _chunked_all_reduce(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """A tensor above one call's size (or not bf16) in calls the kernels take (in place when
        both are contiguous bf16: a call reads each chunk of its input before it writes it)."""
        step = self.max_elems - self.max_elems % 8
        if (inp.dtype == out.dtype == torch.bfloat16 and inp.is_contiguous() and out.is_contiguous()
                and inp.data_ptr() % 16 == 0 and out.data_ptr() % 16 == 0):
            src, dst = inp.reshape(-1), out.reshape(-1)
            for i in range(0, src.numel(), step):
                self.C.fdar(src[i : i + step], dst[i : i + step], *self._comm())
            return out
        src = inp.reshape(-1).to(torch.bfloat16).contiguous()
        dst = torch.empty_like(src)
        for i in range(0, src.numel(), step):
            self.C.fdar(src[i : i + step], dst[i : i + step], *self._comm())
        out.copy_(dst.view(out.shape).to(out.dtype))
        return out

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        return self.all_reduce_into(t, t)

    def linear_allreduce(self, ops, x: torch.Tensor, w: torch.Tensor, residual=None, scale=None,
                         pre=None, prefetch=None) -> torch.Tensor:
        """Row-parallel linear (x . w^T * scale + pre) summed over the members, then the residual;
        one fused kernel at decode sizes. ES_AR_TWO_SHOT=1 makes the fused sum a reduce-scatter to
        each tile's owner and an all-gather (a quarter of the one-shot push's NVLink bytes at 8)."""
        if x.shape[0] <= 64 and x.dtype == torch.bfloat16:
            out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
            wt, wp = weight_args(w)
            self.C.gemm_allreduce(x, wt, out, residual, ops.status, ops.num_sms, *self._comm(), scale, pre,
                                  self.two_shot, 0, wp, prefetch_target(prefetch))
            return out
        if x.dtype == torch.bfloat16 and not torch.cuda.is_current_stream_capturing():
            return self._linear_allreduce_overlapped(ops, x, w, residual, scale, pre)
        y = self.all_reduce(ops.linear(x, w, scale=scale, pre=pre))
        if residual is not None:
            y = (y.float() + residual.float()).to(y.dtype)
        return y

    def linear_reduce_scatter(self, ops, x: torch.Tensor, w: torch.Tensor, residual=None) -> torch.Tensor:
        """Row-parallel linear whose sum over the members is reduce-scattered by tokens: the member at
        position j keeps tokens [j * per, (j + 1) * per), per = ceil(M / members), as [per, N] (rows
        past M are padding), plus `residual` (its own [per, N] slice). One fused kernel at decode
        sizes (the sum's words go to the member keeping the token only)."""
        M, n = x.shape[0], len(self.members)
        per = -(-M // n)
        pos = self.members.index(self.row)
        out = torch.empty(per, w.shape[0], dtype=x.dtype, device=x.device)
        if M <= 64 and x.dtype == torch.bfloat16 and not self.nvls:
            wt, wp = weight_args(w)
            self.C.gemm_allreduce(x, wt, out, residual, ops.status, ops.num_sms, *self._comm(), None, None, 0, per,
                                  wp)
            return out
        full = self.linear_allreduce(ops, x, w)
        out.zero_()
        lo, hi = min(M, pos * per), min(M, (pos + 1) * per)
        out[: hi - lo] = full[lo:hi]
        if residual is not None:
            out = (out.float() + residual.float()).to(out.dtype)
        return out

    def gather_linear(self, ops, x: torch.Tensor, w: torch.Tensor, residual=None) -> torch.Tensor:
        """Column-parallel linear over the member-order concatenation of every member's token rows
        ([per, K] here, the same per on every member): [per * members, N]. One fused kernel at
        decode sizes (the rows reach every member's own buffer by peer stores inside the GEMM, whose
        activation tiles then come from local memory)."""
        per, n = x.shape[0], len(self.members)
        out = torch.empty(per * n, w.shape[0], dtype=x.dtype, device=x.device)
        # the fused kernel's CTAs all wait for every member's pushers, so its grid must be resident
        # at once: at most one 128-row weight tile per SM (the lm_head's vocabulary slice is not)
        fits = (w.shape[0] + 127) // 128 <= ops.num_sms
        if per * n <= 64 and fits and x.dtype == torch.bfloat16 and not self.nvls and x.stride(1) == 1:
            wt, wp = weight_args(w)
            self.C.gemm_allgather(x, wt, out, residual, ops.status, ops.num_sms, *self._comm(), n, self.own, wp)
            return out
        rows = torch.zeros(per * n, x.shape[1], dtype=x.dtype, device=x.device)
        pos = self.members.index(self.row)
        rows[pos * per : (pos + 1) * per] = x
        self.all_reduce_into(rows, rows)  # disjoint rows: the sum is the gather, exactly
        return ops.linear(rows, w, residual=residual)

    ROW_BLOCK = 512  # rows per GEMM block of an overlapped row-parallel linear

    def _linear_allreduce_overlapped(self, ops, x, w, residual, scale, pre) -> torch.Tensor:
        """Prefill sizes: the GEMM in blocks of rows, each block's all-reduce on a second stream
        while the next block's GEMM runs (the same failure-detecting kernels; every member runs
        the blocks in the same order), then the residual."""
        M = x.shape[0]
        y = torch.empty(M, w.shape[0], dtype=x.dtype, device=x.device)
        main = torch.cuda.current_stream(self.device)
        if getattr(self, "_comm_stream", None) is None:
            self._comm_stream = torch.cuda.Stream(self.device)
        side = self._comm_stream
        side.wait_stream(main)
        for r0 in range(0, M, self.ROW_BLOCK):
            r1 = min(M, r0 + self.ROW_BLOCK)
            ops.linear(x[r0:r1], w, out=y[r0:r1], scale=None if scale is None else scale[r0:r1],
                       pre=None if pre is None else pre[r0:r1])
            ev = torch.cuda.Event()
            ev.record(main)
            side.wait_event(ev)
            with torch.cuda.stream(side):
                blk = y[r0:r1]
                self.all_reduce_into(blk, blk)
        main.wait_stream(side)
        y.record_stream(side)
        if residual is not None:
            y = (y.float() + residual.float()).to(y.dtype)
        return y

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """Every member's tensor concatenated along the last dim, in member (rank) order."""
        if self.nccl is not None:
            return self.nccl.all_gather(t)
        if self.size == 1:
            return t
        n = t.shape[-1]
        if t.dtype == torch.bfloat16:
            full = torch.zeros(*t.shape[:-1], n * self.size, dtype=torch.bfloat16, device=t.device)
            full[..., self.rank * n : (self.rank + 1) * n] = t
            flat = full.reshape(-1)
            self.all_reduce_into(flat, flat)  # x + 0 is exact: disjoint slices sum to the gather
            return full
        # other dtypes travel as their bytes, one byte per bf16 element (0..255 are exact in bf16)
        raw = t.contiguous().view(torch.uint8).reshape(*t.shape[:-1], -1)
        nb = raw.shape[-1]
        full = torch.zeros(*raw.shape[:-1], nb * self.size, dtype=torch.bfloat16, device=t.device)
        full[..., self.rank * nb : (self.rank + 1) * nb] = raw.to(torch.bfloat16)
        flat = full.reshape(-1)
        self.all_reduce_into(flat, flat)
        got = full.to(torch.uint8).reshape(*raw.shape[:-1], self.size, nb)
        return got.view(t.dtype).reshape(*t.shape[:-1], n * self.size)

    def set_members(self, members, epoch: int = 0) -> None:
        """Program the member order (rows in rank position); call with this member quiescent."""
        del epoch
        if self.nvls and list(members) != self.members:
            raise RuntimeError("the NVLS variant has fixed members; use the P2P variant for membership changes")
        self.members = [int(m) for m in members]
        self.size = len(self.members)
        if self.row in self.members:
            self.rank = self.members.index(self.row)
        self._open(self.members)
        self._write_order()
        for a in self.attached:
            a.set_members(self.members)

    def abort(self) -> None:
        self.region.set_abort([self.row], 1)

    def resume(self) -> None:
        """Zero the call counter and this member's own buffer once the stream is idle."""
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            self.call.zero_()
            self.seqs.zero_()
            if self._symm is not None:
                self._symm.zero_()
            else:
                self.C.memset_async(self.own, int(self.C.comm_buffer_bytes()))
            torch.cuda.synchronize(self.device)
        for a in self.attached:
            a.resume()
        self.region.clear_late(self.row)
        self.region.set_u32(self.row, 16, 0)  # status
        self.region.set_abort([self.row], 0)

    def status(self) -> int:
        return self.region.status(self.row)

    def late_rows(self) -> list[int]:
        m = self.region.late(self.row)
        return [r for r in range(MAX_ROWS) if m >> r & 1]

    def set_bound_ns(self, ns: int) -> None:
        self.region.set_bound_ns([self.row], ns)

    def count_launches(self, counts) -> None:
        """Bench hook: count this collective's kernel launches into counts['n'] (None stops)."""
        if counts is None:
            if self._counting is not None:
                self.C = self._counting
                self._counting = None
            return
        real = self.C
        self._counting = real

        class Counting:
            def __getattr__(self, name):
                fn = getattr(real, name)
                if name in ("fdar", "gemm_allreduce", "gemm_allgather"):
                    def wrapped(*a, **k):
                        counts["n"] += 1
                        return fn(*a, **k)
                    return wrapped
                return fn

        self.C = Counting()

    def set_beat_limit_us(self, us: int) -> None:
        """Kernels of this member name a peer dead once its beat stands still `us` microseconds
        (0: off; the bound and the host's checks still apply)."""
        self.region.set_beat_limit_us([self.row], int(us))

    def _stop_beat(self) -> None:
        if getattr(self, "_beat", 0):
            self.C.heartbeat_stop(self._beat)
            self._beat = 0

    def close(self) -> None:
        self._stop_beat()
        for a in self.attached:
            a.close()
        self.attached = []
        for m in self._opened.values():
            try:
                m.close()
            except RuntimeError:
                pass
        self._opened.clear()
        if self.own and not self.nvls:
            self._buf.close()
        self.own = 0
        self._symm = None
        self.region.close(self.C, unlink=self._own_region and self.rank == 0)
