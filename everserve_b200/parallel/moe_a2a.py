"""Expert parallelism with routed tokens: the all-to-all dispatch and combine over NVLink peer memory.

Each member of the expert-parallel group owns ``el = E / W`` experts (position p owns experts
``p*el .. p*el + el - 1``) and holds its own tokens. One call:

1. ``dispatch``: every member pushes each of its tokens' rows to the members owning the token's k
   experts (peer stores into the owner's symmetric buffer, one segment per sender and expert), then
   waits (bounded) until every sender's rows for its own experts have arrived;
2. the experts: for each local expert, the gate/up GEMM, SiLU-mul and the down GEMM over the rows it
   received. The GEMMs are grouped by sender segments: token tiles holding no received row are
   skipped whole, so an expert no token chose reads no weights, and prefill does the routed FLOPs;
3. ``ready``: this member's outputs are written (a flag in every member's buffer);
4. ``combine``: every member reads its tokens' k expert outputs from the owners' buffers (peer loads)
   and sums them, weighted, in slot order in fp32.

Every wait is bounded and reports through the member's control words (the abort word, the late
mask and the status word of the tensor-parallel collective's slot region), so a dead owner makes
the call end with a status instead of a hang. Buffers are driver VMM allocations that outlive a
member that dies. Member positions map to buffer rows through a device table, so the members'
traffic follows a membership change inside captured graphs; which experts a member runs is fixed
when its graph is captured, so a spare captures its graphs after it has taken its position.

``ExpertAllToAll.emulated`` plays the whole group on one GPU: one kernel launch carries every
member's traffic between local buffers (the single-GPU numerics test).

Reference parity: the reference carries expert traffic only through the tensor-parallel
all-reduce of the engines it wraps (adapters/vllm/everserve_vllm/identity.py:255 maps the expert
rank to the TP rank); the routed all-to-all is this framework's addition.
"""

from __future__ import annotations

import torch

from .. import _ext

MAX_ROWS = 8
CTRL_BYTES = 32  # one member's control words: abort, late, bound_ns, status, padding


class ExpertAllToAll:
    def __init__(self, C, device, *, experts: int, top_k: int, hidden: int, cap: int, addrs: list[int],
                 members: list[int], own_rows: list[int], pos: int, ctrl: int, splits: int | None = None):
        self.C = C
        self.device = torch.device(device)
        self.E, self.k, self.H, self.cap = int(experts), int(top_k), int(hidden), int(cap)
        self.W = len(members)
        if self.E % self.W:
            raise ValueError(f"{self.E} experts do not divide over {self.W} members")
        if self.H % 8:
            raise ValueError("the hidden size must be a multiple of 8 (16-byte rows)")
        self.el = self.E // self.W
        self.own_rows = [int(r) for r in own_rows]  # the buffers this process owns, one per member played
        self.pos, self.nz = int(pos), len(self.own_rows)
        self.members = [int(r) for r in members]
        self.splits = int(splits or max(1, min(32, 148 // max(1, self.E))))
        self.bytes = int(C.moe_buffer_bytes(self.el, self.W, self.cap, self.H))
        self._addrs = list(addrs) + [0] * (MAX_ROWS - len(addrs))
        self.ctrl = int(ctrl)
        with torch.cuda.device(self.device):
            self.peers = torch.tensor(self._addrs, dtype=torch.int64, device=self.device)
            # count, the row of each position, then the first position this process plays (the
            # kernels read it here, so captured graphs follow a spare's take)
            self.members_t = torch.tensor(self._member_rows(), dtype=torch.int32, device=self.device)
            self.call = torch.zeros(2 * self.nz, dtype=torch.int32, device=self.device)
        self._views: dict[int, torch.Tensor] = {}

    # ---- construction --------------------------------------------------------------------------
    @classmethod
    def emulated(cls, device, members: int, *, experts: int, top_k: int, hidden: int, cap: int, splits=None):
        """All `members` positions in this process, buffers in this GPU's memory."""
        C = _ext.load()
        device = torch.device(device)
        el = experts // members
        nbytes = int(C.moe_buffer_bytes(el, members, cap, hidden))
        bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=device) for _ in range(members)]
        ctrl = torch.zeros(members * CTRL_BYTES, dtype=torch.uint8, device=device)
        self = cls(C, device, experts=experts, top_k=top_k, hidden=hidden, cap=cap,
                   addrs=[b.data_ptr() for b in bufs], members=list(range(members)),
                   own_rows=list(range(members)), pos=0, ctrl=ctrl.data_ptr(), splits=splits)
        self._keep = (bufs, ctrl)
        return self

    @classmethod
    def over(cls, tp, *, experts: int, top_k: int, hidden: int, cap: int, splits=None):
        """One position per process: the group, control words and descriptor exchange of a
        peer-memory tensor-parallel collective (``FusedTPCollective``, P2P variant)."""
        from .symm import PeerMapping, SymmetricBuffer

        if getattr(tp, "nvls", False):
            raise ValueError("the expert all-to-all maps members' buffers itself; use the P2P collective")
        C = tp.C
        el = experts // len(tp.members)
        nbytes = int(C.moe_buffer_bytes(el, len(tp.members), cap, hidden))
        # one descriptor socket per row and instance (every member attaches its instances in the
        # same order, so the n-th names agree)
        n = sum(isinstance(a, ExpertAllToAll) for a in getattr(tp, "attached", []))
        path = lambda r: f"{tp.region.path}.r{r}.moe{n}.fd"  # noqa: E731
        with torch.cuda.device(tp.device):
            buf = SymmetricBuffer(C, nbytes, path(tp.row))
            C.memset_async(buf.ptr, buf.size)
            torch.cuda.synchronize(tp.device)
        tp._barrier()
        addrs = [0] * MAX_ROWS
        addrs[tp.row] = buf.ptr
        opened = {}
        member = tp.row in tp.members  # a spare holds no position until it takes one
        with torch.cuda.device(tp.device):
            for r in tp.members if member else ():
                if r != tp.row:
                    opened[r] = PeerMapping(C, path(r))
                    addrs[r] = opened[r].ptr
        self = cls(C, tp.device, experts=experts, top_k=top_k, hidden=hidden, cap=cap, addrs=addrs,
                   members=tp.members, own_rows=[tp.row], pos=tp.members.index(tp.row) if member else -1,
                   ctrl=int(tp.ctrl), splits=splits)
        self._buf, self._opened, self._path, self._tp = buf, opened, path, tp
        if hasattr(tp, "attached"):
            tp.attached.append(self)  # membership changes and resumes of the group reach this too
        return self

    def _member_rows(self) -> list[int]:
        return [self.W, *self.members] + [0] * (MAX_ROWS - self.W) + [self.pos]

    # ---- views of a member's own buffer --------------------------------------------------------
    def _own(self, z: int) -> torch.Tensor:
        row = self.own_rows[z]
        if row not in self._views:
            keep = getattr(self, "_keep", None)
            if keep is not None:
                self._views[row] = keep[0][row]
            else:
                self._views[row] = self.C.device_view(self._addrs[row], self.bytes, self.device.index or 0)
        return self._views[row]

    def _rows(self, z: int, region: int, el: int) -> torch.Tensor:
        seg = self.W * self.cap * self.H * 2
        off = int(self.C.moe_header_bytes()) + (region * self.el + el) * seg
        return self._own(z)[off : off + seg].view(torch.bfloat16).view(self.W * self.cap, self.H)

    def expert_rows(self, el: int, z: int = 0) -> torch.Tensor:
        """Local expert `el`'s received rows [W * cap, H]: sender p's at rows [p * cap, ...)."""
        return self._rows(z, 0, el)

    def expert_out(self, el: int, z: int = 0) -> torch.Tensor:
        """Where local expert `el`'s outputs go, row for row."""
        return self._rows(z, 1, el)

    def counts(self, el: int, z: int = 0) -> torch.Tensor:
        """Rows each sender position sent to local expert `el` (int32 [W])."""
        off = int(self.C.moe_counts_offset()) + el * int(self.C.moe_counts_stride()) * 4
        return self._own(z)[off : off + 4 * self.W].view(torch.int32)

    # ---- one call ------------------------------------------------------------------------------
    def _args(self):
        return self.peers, self.members_t, self.call, self.ctrl, self.pos

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """x [nz, T, H] bf16 and ids [nz, T, k] int32 of the members played; returns each row's
        place in its expert's segment ([nz, T, k] int32)."""
        if x.shape[1] > self.cap:
            raise ValueError(f"{x.shape[1]} tokens exceed the segment capacity {self.cap}")
        place = torch.empty_like(ids)
        self.C.moe_dispatch(x, ids, place, *self._args(), self.E, self.el, self.cap, self.splits)
        return place

    def ready(self) -> None:
        self.C.moe_ready(*self._args(), self.nz, self.E, self.el, self.k, self.H, self.cap)

    def combine(self, ids: torch.Tensor, weights: torch.Tensor, place: torch.Tensor, num_sms: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(ids.shape[0], ids.shape[1], self.H, dtype=torch.bfloat16, device=self.device)
        self.C.moe_combine(ids, weights, place, out, *self._args(), self.E, self.el, self.cap, num_sms)
        return out

    def run_experts(self, ops, gate_up, down) -> None:
        """Each local expert of each member played over what it received: `gate_up(e)` [2I, H] and
        `down(e)` [H, I] give global expert e's weights."""
        if self.pos < 0:
            # no position: no experts; a graph captured now would keep running none after a take
            assert not torch.cuda.is_current_stream_capturing(), "capture the expert graph after the take"
            return
        for z in range(self.nz):
            for el in range(self.el):
                e = (self.pos + z) * self.el + el
                valid = self.counts(el, z)
                gu = ops.linear(self.expert_rows(el, z), gate_up(e), valid=valid, valid_cap=self.cap)
                ops.linear(ops.silu_mul(gu), down(e), out=self.expert_out(el, z), valid=valid, valid_cap=self.cap)

    def __call__(self, ops, x, ids, weights, gate_up, down) -> torch.Tensor:
        """The whole mixture layer for the members played: [nz, T, H] in, [nz, T, H] out."""
        place = self.dispatch(x, ids)
        self.run_experts(ops, gate_up, down)
        self.ready()
        return self.combine(ids, weights, place, ops.num_sms)

    # ---- membership and failure ------------------------------------------------------------------
    def status(self, z: int = 0) -> int:
        keep = getattr(self, "_keep", None)
        if keep is not None:
            return int(keep[1].view(torch.int32)[z * CTRL_BYTES // 4 + 4].item())
        return self._tp.status()

    def set_members(self, members: list[int]) -> None:
        """A spare took a position: map its buffer and point the position at it (call quiescent)."""
        from .symm import PeerMapping

        if getattr(self, "_path", None) is None:
            raise RuntimeError("an emulated group has fixed members")
        if len(members) != self.W:
            raise ValueError("the group keeps its size; a spare takes a position")
        me = self.own_rows[0]
        with torch.cuda.device(self.device):
            for r in members:
                if r != me and r not in self._opened:
                    self._opened[r] = PeerMapping(self.C, self._path(r))
                    self._addrs[r] = self._opened[r].ptr
            self.members = [int(r) for r in members]
            self.pos = self.members.index(me) if me in self.members else -1
            self.peers.copy_(torch.tensor(self._addrs, dtype=torch.int64))
            self.members_t.copy_(torch.tensor(self._member_rows(), dtype=torch.int32))

    def resume(self) -> None:
        """Zero the call counter and this member's flags once the stream is idle (every member
        does, at the same boundary)."""
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            self.call.zero_()
            for z in range(self.nz):
                self._own(z)[: int(self.C.moe_header_bytes())].zero_()
            torch.cuda.synchronize(self.device)

    def close(self) -> None:
        for m in getattr(self, "_opened", {}).values():
            try:
                m.close()
            except RuntimeError:
                pass
        self._opened = {}
        self._views.clear()
        if getattr(self, "_buf", None) is not None:
            self._buf.close()
            self._buf = None


def default_cap(tokens: int) -> int:
    """Segment rows for `tokens` tokens per member: every token fits (a sender sends an expert at
    most one row per token), rounded up to a multiple of 64 so the token tiles line up."""
    return max(64, (tokens + 63) // 64 * 64)


__all__ = ["ExpertAllToAll", "default_cap"]
