"""Ulysses sequence parallelism: sequence <-> head exchange around attention.

Mirrors ec-jt/vdn src/inference/utils/ulysses_runtime.py (sequence_splits,
balanced_splits, UlyssesRuntime.configure / sequence_to_heads /
heads_to_sequence / gather_sequence / video_frame_mean_async, init_ulysses)
for the standard (head-sharded) exchange, and its branch-parallel layout
(enable_branch_parallel, dispatch_fields_to_branches_overlapped,
branches_to_sequence: n softmax ranks + P - n VDA ranks, uneven all-to-alls on
two dispatch communicators).  One process per GPU.  Two standard exchange
modes with identical routing (every row / head arrives where the reference
sends it):

  "alltoall"  the reference's form: one torch.distributed all_to_all_single per
              direction on the NCCL process group;
  "peer"      (default for the block) the producers store into the consumers'
              memory over NVLink: see vdn_b200.peer.

Timeouts are short by default so that a rank that never joins ends the others'
next collective with an error.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from datetime import timedelta

import torch
import torch.distributed as dist

__all__ = ["sequence_splits", "balanced_splits", "UlyssesRuntime", "init_ulysses"]


def sequence_splits(sequence_length: int, world_size: int) -> tuple[int, ...]:
    """Contiguous shards: ceil(S/P) rows on ranks 0..P-2, the remainder last (ulysses_runtime.py:26-46)."""
    if sequence_length <= 0 or world_size <= 0:
        raise ValueError("sequence_length and world_size must be positive")
    if world_size == 1:
        return (sequence_length,)
    chunk = math.ceil(sequence_length / world_size)
    last = sequence_length - chunk * (world_size - 1)
    if last <= 0:
        base, extra = divmod(sequence_length, world_size)
        return tuple(base + (rank < extra) for rank in range(world_size))
    return (chunk,) * (world_size - 1) + (last,)


def balanced_splits(total: int, parts: int) -> tuple[int, ...]:
    """Contiguous split with imbalance at most one (ulysses_runtime.py:49-59)."""
    if total <= 0 or parts <= 0 or parts > total:
        raise ValueError(f"need 0 < parts <= total; got total={total}, parts={parts}")
    base, extra = divmod(total, parts)
    return tuple(base + (rank < extra) for rank in range(parts))


@dataclass
class UlyssesRuntime:
    rank: int
    world_size: int
    local_rank: int
    device: torch.device
    backend: str
    group: object | None = None
    sequence_length: int = 0
    splits: tuple[int, ...] = ()
    local_start: int = 0
    local_end: int = 0
    heads_per_rank: int = 0
    num_heads: int = 0
    # Branch-parallel layout (ulysses_runtime.py:176-217): ranks [0, softmax_ranks)
    # run the window softmax for their share of ALL heads, the remaining ranks the
    # VDA branch for theirs; 0 = the standard layout (every rank owns H/P heads of
    # both branches).
    softmax_ranks: int = 0
    softmax_head_splits: tuple[int, ...] = ()
    linear_head_splits: tuple[int, ...] = ()
    softmax_dispatch_group: object | None = None
    linear_dispatch_group: object | None = None
    timeout_seconds: int = 120
    profile_enabled: bool = False
    profile_events: dict = field(default_factory=dict)
    # "peer": producers store into peer memory (vdn_b200.peer); "alltoall": the
    # reference's NCCL all-to-all exchange (sequence_to_heads / heads_to_sequence).
    exchange_mode: str = "peer"
    _exchanges: dict = field(default_factory=dict)

    @property
    def is_main(self) -> bool:
        return self.rank == 0

    def barrier(self) -> None:
        dist.barrier(group=self.group)

    # ------------------------------------------------------- branch-parallel layout
    @property
    def branch_parallel(self) -> bool:
        return self.softmax_ranks > 0

    @property
    def branch_kind(self) -> str:
        if not self.branch_parallel:
            raise RuntimeError("branch_kind is only defined for branch-parallel Ulysses")
        return "softmax" if self.rank < self.softmax_ranks else "linear"

    @property
    def branch_head_splits(self) -> tuple[int, ...]:
        """Heads per rank in rank order: the softmax ranks' shares, then the linear ranks'."""
        if not self.branch_parallel:
            raise RuntimeError("branch_head_splits requires branch-parallel Ulysses")
        return self.softmax_head_splits + self.linear_head_splits

    @property
    def branch_heads(self) -> int:
        return self.branch_head_splits[self.rank]

    @property
    def branch_first_head(self) -> int:
        """First original head of this rank's contiguous head range inside its branch."""
        if self.branch_kind == "softmax":
            return sum(self.softmax_head_splits[:self.rank])
        return sum(self.linear_head_splits[:self.rank - self.softmax_ranks])

    def enable_branch_parallel(self, softmax_ranks: int) -> None:
        """Split the ranks into `softmax_ranks` softmax ranks and world_size - softmax_ranks
        VDA ranks (ulysses_runtime.py:208-217).  Collective when a process group is up:
        every rank calls it, and the two dispatch communicators are created here."""
        if isinstance(softmax_ranks, bool) or not isinstance(softmax_ranks, int) or \
                not 0 < softmax_ranks < self.world_size:
            raise ValueError(f"softmax_ranks must lie in [1, {self.world_size - 1}], got {softmax_ranks}")
        if self.sequence_length:
            raise RuntimeError("enable branch parallelism before the first forward")
        self.softmax_ranks = softmax_ranks
        if self.softmax_dispatch_group is None and dist.is_available() and dist.is_initialized():
            ranks = list(range(self.world_size)) if self.group is None else \
                dist.get_process_group_ranks(self.group)
            timeout = timedelta(seconds=self.timeout_seconds)
            self.softmax_dispatch_group = dist.new_group(ranks=ranks, timeout=timeout)
            self.linear_dispatch_group = dist.new_group(ranks=ranks, timeout=timeout)

    def configure(self, sequence_length: int, num_heads: int) -> None:
        if not self.branch_parallel and num_heads % self.world_size:
            raise ValueError(f"Ulysses needs num_heads divisible by world_size; got "
                             f"{num_heads} heads on {self.world_size} ranks")
        splits = sequence_splits(sequence_length, self.world_size)
        if any(size <= 0 for size in splits):
            raise ValueError(f"Ulysses requires at least one row per rank; S={sequence_length}, "
                             f"P={self.world_size}")
        if self.sequence_length and self.sequence_length != sequence_length:
            raise RuntimeError("one Ulysses process supports one packed sequence geometry; "
                               f"already configured for {self.sequence_length}, got {sequence_length}")
        self.sequence_length = sequence_length
        self.splits = splits
        self.local_start = sum(splits[: self.rank])
        self.local_end = self.local_start + splits[self.rank]
        self.num_heads = num_heads
        if self.branch_parallel:
            self.softmax_head_splits = balanced_splits(num_heads, self.softmax_ranks)
            self.linear_head_splits = balanced_splits(num_heads, self.world_size - self.softmax_ranks)
            self.heads_per_rank = self.branch_heads
        else:
            self.heads_per_rank = num_heads // self.world_size

    def _pack_branch_targets(self, q, k, v, scalar, shared, head_splits, first_target):
        """Send buffer and per-target sizes of one branch's dispatch.

        Target `first_target + i` receives, for every local row, its `head_splits[i]`
        heads as [q (d) | k (d) | v (d) | scalar (1)] followed by the `shared` row
        (the wire layout of ulysses_runtime.py:63-117, written here with strided
        copies straight from the source fields: no intermediate full-width pack).
        """
        rows = self.splits[self.rank]
        d = v.shape[-1]
        per_head = 3 * d + 1
        sw = 0 if shared is None else shared.shape[-1]
        scalar = scalar.reshape(rows, -1)
        sizes = [0] * self.world_size
        for i, heads in enumerate(head_splits):
            sizes[first_target + i] = rows * (heads * per_head + sw)
        send = v.new_empty(sum(sizes))
        offset = h0 = 0
        for i, heads in enumerate(head_splits):
            width = heads * per_head + sw
            seg = send[offset:offset + rows * width].view(rows, width)
            body = seg[:, :heads * per_head].view(rows, heads, per_head)
            hs = slice(h0, h0 + heads)
            body[:, :, 0:d].copy_(q[:, hs])
            body[:, :, d:2 * d].copy_(k[:, hs])
            body[:, :, 2 * d:3 * d].copy_(v[:, hs])
            body[:, :, 3 * d].copy_(scalar[:, hs])
            if sw:
                seg[:, heads * per_head:].copy_(shared)
            offset += rows * width
            h0 += heads
        return send, sizes

    def dispatch_fields_to_branches_overlapped(self, softmax_q, softmax_k, value, softmax_gate,
                                               linear_q, linear_k, linear_beta, linear_shared):
        """Sequence shard -> branch heads, one uneven all-to-all per branch on its own
        communicator (ulysses_runtime.py:254-398).

        Inputs are this rank's rows: q / k / v [S_rank, H, d], softmax gate and beta
        [S_rank, H] (or [S_rank, H, 1]), the shared per-token row [S_rank, W] that only
        the linear ranks receive (the output gate's low-rank hidden).  Returns
        (packed [S, branch_heads, 3d + 1], shared [S, W] on linear ranks else None,
        pending) after waiting for this rank's own branch only; `pending` holds the
        other branch's work handle and buffers -- wait on pending[0] before reusing them.
        """
        if self.softmax_dispatch_group is None or self.linear_dispatch_group is None:
            raise RuntimeError("overlapped dispatch communicators were not initialized")
        rows = self.splits[self.rank]
        for name, t in (("softmax_q", softmax_q), ("softmax_k", softmax_k), ("value", value),
                        ("linear_q", linear_q), ("linear_k", linear_k)):
            if t.ndim != 3 or t.shape[0] != rows or t.shape[1] != self.num_heads:
                raise ValueError(f"{name} has {tuple(t.shape)}, expected ({rows}, {self.num_heads}, d)")
        d = value.shape[-1]
        per_head = 3 * d + 1
        sw = linear_shared.shape[-1]
        if linear_shared.shape[0] != rows:
            raise ValueError("linear_shared must hold this rank's rows")

        soft_send, soft_in = self._pack_branch_targets(softmax_q, softmax_k, value, softmax_gate, None,
                                                       self.softmax_head_splits, 0)
        soft_width = self.branch_heads * per_head if self.branch_kind == "softmax" else 0
        soft_out = [r * soft_width for r in self.splits]
        soft_recv = value.new_empty(sum(soft_out))
        soft_work = dist.all_to_all_single(soft_recv, soft_send, output_split_sizes=soft_out,
                                           input_split_sizes=soft_in, group=self.softmax_dispatch_group,
                                           async_op=True)

        lin_send, lin_in = self._pack_branch_targets(linear_q, linear_k, value, linear_beta, linear_shared,
                                                     self.linear_head_splits, self.softmax_ranks)
        lin_width = self.branch_heads * per_head + sw if self.branch_kind == "linear" else 0
        lin_out = [r * lin_width for r in self.splits]
        lin_recv = value.new_empty(sum(lin_out))
        lin_work = dist.all_to_all_single(lin_recv, lin_send, output_split_sizes=lin_out,
                                          input_split_sizes=lin_in, group=self.linear_dispatch_group,
                                          async_op=True)

        S, hb = self.sequence_length, self.branch_heads
        if self.branch_kind == "softmax":
            soft_work.wait()
            packed = soft_recv.view(S, hb, per_head)
            return packed, None, (lin_work, lin_send, lin_recv)
        lin_work.wait()
        recv = lin_recv.view(S, lin_width)
        packed = recv[:, :hb * per_head].view(S, hb, per_head)
        return packed, recv[:, hb * per_head:], (soft_work, soft_send, soft_recv)

    def branches_to_sequence(self, branch_tensor: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """[S, branch_heads, D] -> (softmax [S_rank, H, D], linear [S_rank, H, D]) in ONE
        uneven all-to-all: the reverse exchange is also the branch merge
        (ulysses_runtime.py:401-448)."""
        if not self.branch_parallel:
            raise RuntimeError("branches_to_sequence requires branch-parallel Ulysses")
        if branch_tensor.ndim != 3 or tuple(branch_tensor.shape[:2]) != (self.sequence_length,
                                                                          self.branch_heads):
            raise ValueError(f"branch output has {tuple(branch_tensor.shape)}, expected "
                             f"({self.sequence_length}, {self.branch_heads}, D)")
        width = branch_tensor.shape[-1]
        rows = self.splits[self.rank]
        in_splits = [r * self.branch_heads * width for r in self.splits]
        out_splits = [rows * h * width for h in self.branch_head_splits]
        recv = branch_tensor.new_empty(sum(out_splits))
        dist.all_to_all_single(recv, branch_tensor.contiguous().view(-1), output_split_sizes=out_splits,
                               input_split_sizes=in_splits, group=self.group)
        chunks, offset = [], 0
        for size, heads in zip(out_splits, self.branch_head_splits):
            chunks.append(recv[offset:offset + size].view(rows, heads, width))
            offset += size
        return (torch.cat(chunks[:self.softmax_ranks], dim=1),
                torch.cat(chunks[self.softmax_ranks:], dim=1))

    def exchange(self, num_heads: int, head_dim: int, frames: int = 0, row_width: int = 0):
        """The peer-memory exchange of the configured geometry (built once, cached)."""
        from .peer import PeerExchange
        key = (self.sequence_length, num_heads, head_dim, frames, row_width)
        ex = self._exchanges.get(key)
        if ex is None:
            if not self.sequence_length:
                raise RuntimeError("configure() the runtime before building an exchange")
            ex = self._exchanges[key] = PeerExchange(self, self.sequence_length, num_heads, head_dim,
                                                     frames, row_width)
        return ex

    def close(self) -> None:
        """Release peer mappings (collective: every rank calls it before destroy_process_group)."""
        for ex in self._exchanges.values():
            ex.close()
        self._exchanges.clear()

    def profile_start(self):
        if not self.profile_enabled:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def profile_end(self, name, start):
        if start is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.profile_events.setdefault(name, []).append((start, e))

    def profile_milliseconds(self):
        torch.cuda.synchronize(self.device)
        return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in self.profile_events.items()}

    def sequence_to_heads(self, tensor: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[S_rank, H, W] -> [S, H/P, W] (ulysses_runtime.py:451-519)."""
        local_rows, heads, width = tensor.shape
        if local_rows != self.splits[self.rank]:
            raise ValueError(f"local rows {local_rows} != configured {self.splits[self.rank]}")
        if heads != self.heads_per_rank * self.world_size:
            raise ValueError(f"heads {heads} != {self.heads_per_rank * self.world_size}")
        send = (tensor.view(local_rows, self.world_size, self.heads_per_rank, width)
                .permute(1, 0, 2, 3).contiguous().view(-1))
        unit = self.heads_per_rank * width
        recv = out if out is not None else tensor.new_empty(self.sequence_length * unit)
        dist.all_to_all_single(recv.view(-1), send,
                               output_split_sizes=[rows * unit for rows in self.splits],
                               input_split_sizes=[local_rows * unit] * self.world_size,
                               group=self.group)
        return recv.view(self.sequence_length, self.heads_per_rank, width)

    def heads_to_sequence(self, tensor: torch.Tensor) -> torch.Tensor:
        """[S, H/P, W] -> [S_rank, H, W] (ulysses_runtime.py:522-582)."""
        sequence_length, local_heads, width = tensor.shape
        if sequence_length != self.sequence_length or local_heads != self.heads_per_rank:
            raise ValueError(f"head shard has {tuple(tensor.shape[:2])}, expected "
                             f"({self.sequence_length}, {self.heads_per_rank})")
        unit = self.heads_per_rank * width
        local_rows = self.splits[self.rank]
        recv = tensor.new_empty(local_rows * unit * self.world_size)
        dist.all_to_all_single(recv, tensor.contiguous().view(-1),
                               output_split_sizes=[local_rows * unit] * self.world_size,
                               input_split_sizes=[rows * unit for rows in self.splits],
                               group=self.group)
        return (recv.view(self.world_size, local_rows, self.heads_per_rank, width)
                .permute(1, 0, 2, 3).contiguous()
                .view(local_rows, self.heads_per_rank * self.world_size, width))

    def gather_sequence(self, tensor: torch.Tensor) -> torch.Tensor:
        """All-gather a sequence shard, padding confined to the last rank (ulysses_runtime.py:585-603)."""
        local_rows = tensor.shape[0]
        max_rows = max(self.splits)
        padded = tensor
        if local_rows < max_rows:
            padded = tensor.new_zeros((max_rows, *tensor.shape[1:]))
            padded[:local_rows].copy_(tensor)
        gathered = tensor.new_empty((self.world_size * max_rows, *tensor.shape[1:]))
        dist.all_gather_into_tensor(gathered, padded.contiguous(), group=self.group)
        if self.splits[:-1] == (max_rows,) * (self.world_size - 1):
            return gathered[: self.sequence_length]
        chunks = gathered.view(self.world_size, max_rows, *tensor.shape[1:])
        return torch.cat([chunks[r, :n] for r, n in enumerate(self.splits)], dim=0)

    def local_frame_sums(self, local_x: torch.Tensor, num_frames: int, tokens_per_frame: int,
                         video_start: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        """Per-frame fp32 sums of this rank's rows, one contiguous slice per frame
        (deterministic; ulysses_runtime.py:606-635).  `out` [num_frames, W] fp32."""
        if out is None:
            sums = torch.zeros(num_frames, local_x.shape[-1], device=local_x.device, dtype=torch.float32)
        else:
            sums = out
            sums.zero_()
        v0, v1 = video_start, video_start + num_frames * tokens_per_frame
        lo, hi = max(self.local_start, v0), min(self.local_end, v1)
        if hi <= lo:
            return sums
        first = (lo - v0) // tokens_per_frame
        last = (hi - 1 - v0) // tokens_per_frame
        for frame in range(first, last + 1):
            a = max(lo, v0 + frame * tokens_per_frame)
            b = min(hi, v0 + (frame + 1) * tokens_per_frame)
            torch.sum(local_x[a - self.local_start:b - self.local_start], 0, dtype=torch.float32,
                      out=sums[frame])
        return sums

    def video_frame_mean_async(self, local_x, num_frames, tokens_per_frame, video_start=0):
        """Launch the frame-sum all-reduce; returns (sums, work) (ulysses_runtime.py:638-643)."""
        sums = self.local_frame_sums(local_x, num_frames, tokens_per_frame, video_start)
        work = dist.all_reduce(sums, async_op=True, group=self.group)
        return sums, work


def init_ulysses(backend: str = "nccl", *, profile_enabled: bool = False,
                 timeout_seconds: int = 120) -> UlyssesRuntime:
    """Initialise the process group from torchrun's environment and bind LOCAL_RANK."""
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
        device = torch.device("cuda", local_rank)
    else:
        device = torch.device("cpu")
    if not dist.is_initialized():
        kwargs = dict(backend=backend, timeout=timedelta(seconds=timeout_seconds))
        if backend == "nccl":
            kwargs["device_id"] = device
        dist.init_process_group(**kwargs)
    rank = dist.get_rank()
    actual = dist.get_world_size()
    if actual != world_size and "WORLD_SIZE" in os.environ:
        raise RuntimeError(f"WORLD_SIZE={world_size}, process group has {actual}")
    return UlyssesRuntime(rank=rank, world_size=actual, local_rank=local_rank, device=device,
                          backend=backend, profile_enabled=profile_enabled,
                          timeout_seconds=timeout_seconds)
