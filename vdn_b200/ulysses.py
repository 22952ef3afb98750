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
import types
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist

from .linear_attention import frame_sums

__all__ = ["sequence_splits", "balanced_splits", "ShardPlan", "UlyssesRuntime", "init_ulysses",
           "install_ulysses"]


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


@dataclass(frozen=True)
class ShardPlan:
    """Where the rows and the heads of one packed-sequence geometry live.

    Rows: contiguous shards by `sequence_splits`.  Heads: the standard layout gives
    every rank H/P heads of both branches (`head_splits` = (H/P,) * P); the
    branch-parallel layout gives ranks [0, softmax_ranks) the window softmax and the
    other ranks the VDA branch, each group dividing ALL heads with `balanced_splits`
    (`head_splits` = the softmax ranks' shares, then the linear ranks').  The checks
    and their messages are the reference runtime's (ulysses_runtime.py:219-251).
    """
    sequence_length: int
    num_heads: int
    splits: tuple
    head_splits: tuple
    softmax_ranks: int = 0

    @classmethod
    def build(cls, sequence_length: int, num_heads: int, world_size: int, softmax_ranks: int = 0):
        if not softmax_ranks and num_heads % world_size:
            raise ValueError(f"Ulysses needs num_heads divisible by world_size; got "
                             f"{num_heads} heads on {world_size} ranks")
        splits = sequence_splits(sequence_length, world_size)
        if min(splits) <= 0:
            raise ValueError(f"Ulysses requires at least one row per rank; S={sequence_length}, "
                             f"P={world_size}")
        if softmax_ranks:
            heads = (balanced_splits(num_heads, softmax_ranks)
                     + balanced_splits(num_heads, world_size - softmax_ranks))
        else:
            heads = (num_heads // world_size,) * world_size
        return cls(sequence_length, num_heads, splits, heads, softmax_ranks)

    def rows(self, rank: int) -> tuple[int, int]:
        """[start, end) of rank's sequence shard."""
        start = sum(self.splits[:rank])
        return start, start + self.splits[rank]

    def branch_of(self, rank: int) -> str:
        return "softmax" if rank < self.softmax_ranks else "linear"

    def first_head(self, rank: int) -> int:
        """First head of rank's contiguous range, counted inside its own branch."""
        group0 = 0 if rank < self.softmax_ranks else self.softmax_ranks
        return sum(self.head_splits[group0:rank])


class UlyssesRuntime:
    """One rank's view of Ulysses sequence parallelism (the reference's UlyssesRuntime,
    ulysses_runtime.py:120-643): the shard plan, the sequence <-> head exchanges and the
    frame-sum reduction.  `exchange_mode` picks the standard exchange: "peer" (the
    producers store over NVLink, vdn_b200.peer) or "alltoall" (NCCL all-to-all, the
    reference's form); the branch-parallel layout always uses uneven all-to-alls."""

    def __init__(self, rank: int, world_size: int, local_rank: int, device, backend: str, *,
                 group=None, timeout_seconds: int = 120, profile_enabled: bool = False,
                 exchange_mode: str = "peer"):
        self.rank, self.world_size, self.local_rank = rank, world_size, local_rank
        self.device, self.backend, self.group = torch.device(device), backend, group
        self.timeout_seconds, self.profile_enabled = timeout_seconds, profile_enabled
        self.exchange_mode = exchange_mode
        self.plan: ShardPlan | None = None
        self.softmax_ranks = 0
        self.softmax_dispatch_group = None
        self.linear_dispatch_group = None
        self.profile_events: dict = {}
        self._exchanges: dict = {}

    # ------------------------------------------------------------ the shard plan
    def _need_plan(self) -> ShardPlan:
        if self.plan is None:
            raise RuntimeError("configure() the Ulysses runtime first")
        return self.plan

    @property
    def sequence_length(self) -> int:
        return 0 if self.plan is None else self.plan.sequence_length

    @property
    def num_heads(self) -> int:
        return 0 if self.plan is None else self.plan.num_heads

    @property
    def splits(self) -> tuple:
        return () if self.plan is None else self.plan.splits

    @property
    def local_start(self) -> int:
        return 0 if self.plan is None else self.plan.rows(self.rank)[0]

    @property
    def local_end(self) -> int:
        return 0 if self.plan is None else self.plan.rows(self.rank)[1]

    @property
    def heads_per_rank(self) -> int:
        return 0 if self.plan is None else self.plan.head_splits[self.rank]

    @property
    def softmax_head_splits(self) -> tuple:
        return () if self.plan is None else self.plan.head_splits[:self.softmax_ranks]

    @property
    def linear_head_splits(self) -> tuple:
        return () if self.plan is None else self.plan.head_splits[self.softmax_ranks:]

    @property
    def is_main(self) -> bool:
        return self.rank == 0

    @property
    def branch_parallel(self) -> bool:
        return self.softmax_ranks > 0

    @property
    def branch_kind(self) -> str:
        if not self.branch_parallel:
            raise RuntimeError("branch_kind is only defined for branch-parallel Ulysses")
        return "softmax" if self.rank < self.softmax_ranks else "linear"

    @property
    def branch_head_splits(self) -> tuple:
        """Heads per rank in rank order: the softmax ranks' shares, then the linear ranks'."""
        if not self.branch_parallel:
            raise RuntimeError("branch_head_splits requires branch-parallel Ulysses")
        return self._need_plan().head_splits

    @property
    def branch_heads(self) -> int:
        return self.branch_head_splits[self.rank]

    @property
    def branch_first_head(self) -> int:
        """First original head of this rank's contiguous head range inside its branch."""
        self.branch_kind  # raises outside the branch-parallel layout
        return self._need_plan().first_head(self.rank)

    def barrier(self) -> None:
        dist.barrier(group=self.group)

    def enable_branch_parallel(self, softmax_ranks: int) -> None:
        """Split the ranks into `softmax_ranks` softmax ranks and world_size - softmax_ranks
        VDA ranks (ulysses_runtime.py:208-217).  Collective when a process group is up:
        every rank calls it, and the two dispatch communicators are created here."""
        valid = isinstance(softmax_ranks, int) and not isinstance(softmax_ranks, bool)
        if not (valid and 0 < softmax_ranks < self.world_size):
            raise ValueError(f"softmax_ranks must lie in [1, {self.world_size - 1}], got {softmax_ranks}")
        if self.plan is not None:
            raise RuntimeError("enable branch parallelism before the first forward")
        self.softmax_ranks = softmax_ranks
        if self.softmax_dispatch_group is None and dist.is_available() and dist.is_initialized():
            members = (list(range(self.world_size)) if self.group is None
                       else dist.get_process_group_ranks(self.group))
            limit = timedelta(seconds=self.timeout_seconds)
            self.softmax_dispatch_group, self.linear_dispatch_group = (
                dist.new_group(ranks=members, timeout=limit) for _ in range(2))

    def configure(self, sequence_length: int, num_heads: int) -> None:
        """Fix the packed-sequence geometry (one per process, as in the reference)."""
        plan = ShardPlan.build(sequence_length, num_heads, self.world_size, self.softmax_ranks)
        if self.plan is not None and self.plan.sequence_length != sequence_length:
            raise RuntimeError("one Ulysses process supports one packed sequence geometry; "
                               f"already configured for {self.plan.sequence_length}, got {sequence_length}")
        self.plan = plan

    def reset(self) -> None:
        """Drop the geometry (and its peer exchanges) so that configure() can set another;
        collective under the peer exchange."""
        self.close()
        self.plan = None

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
        soft_work = _all_to_all(soft_recv, soft_send, soft_out, soft_in, self.softmax_dispatch_group,
                                async_op=True)

        lin_send, lin_in = self._pack_branch_targets(linear_q, linear_k, value, linear_beta, linear_shared,
                                                     self.linear_head_splits, self.softmax_ranks)
        lin_width = self.branch_heads * per_head + sw if self.branch_kind == "linear" else 0
        lin_out = [r * lin_width for r in self.splits]
        lin_recv = value.new_empty(sum(lin_out))
        lin_work = _all_to_all(lin_recv, lin_send, lin_out, lin_in, self.linear_dispatch_group,
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
        _all_to_all(recv, branch_tensor.contiguous().view(-1), out_splits, in_splits, self.group)
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

    def reset_profile(self) -> None:
        self.profile_events.clear()

    def profile_milliseconds(self):
        torch.cuda.synchronize(self.device)
        return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in self.profile_events.items()}

    def sequence_to_heads(self, tensor: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[S_rank, H, W] (this rank's rows, every head) -> [S, H/P, W] (every row, this
        rank's heads): one all-to-all whose send buffer holds, per destination rank, its
        head group of our rows (ulysses_runtime.py:451-519)."""
        plan = self._need_plan()
        rows, heads, width = tensor.shape
        if rows != plan.splits[self.rank]:
            raise ValueError(f"local rows {rows} != configured {plan.splits[self.rank]}")
        hl = self.heads_per_rank
        if heads != hl * self.world_size:
            raise ValueError(f"heads {heads} != {hl * self.world_size}")
        send = torch.stack(tensor.split(hl, dim=1))             # [P, rows, hl, W] contiguous
        unit = hl * width
        recv = out if out is not None else tensor.new_empty(plan.sequence_length * unit)
        _all_to_all(recv.view(-1), send.view(-1), [n * unit for n in plan.splits],
                    [rows * unit] * self.world_size, self.group)
        return recv.view(plan.sequence_length, hl, width)

    def heads_to_sequence(self, tensor: torch.Tensor) -> torch.Tensor:
        """[S, H/P, W] -> [S_rank, H, W]: the inverse routing (ulysses_runtime.py:522-582)."""
        plan = self._need_plan()
        seq, hl, width = tensor.shape
        if seq != plan.sequence_length or hl != self.heads_per_rank:
            raise ValueError(f"head shard has {(seq, hl)}, expected "
                             f"({plan.sequence_length}, {self.heads_per_rank})")
        rows = plan.splits[self.rank]
        unit = hl * width
        recv = tensor.new_empty(self.world_size * rows * unit)
        _all_to_all(recv, tensor.contiguous().view(-1), [rows * unit] * self.world_size,
                    [n * unit for n in plan.splits], self.group)
        # recv holds one [rows, hl, W] block per source rank, in head order.
        return torch.cat(recv.view(self.world_size, rows, hl, width).unbind(0), dim=1)

    def gather_sequence(self, tensor: torch.Tensor) -> torch.Tensor:
        """Every rank's shard, concatenated in rank order: [S, ...] (ulysses_runtime.py:585-603).
        Shards are padded to the longest for the all-gather; when only the last shard is
        short, the valid rows are the gathered buffer's prefix (no extra copy)."""
        plan = self._need_plan()
        if self.world_size == 1:
            return tensor
        longest = max(plan.splits)
        tail = tuple(tensor.shape[1:])
        shard = tensor.contiguous()
        if shard.shape[0] < longest:
            shard = torch.cat([shard, tensor.new_zeros((longest - shard.shape[0], *tail))])
        gathered = tensor.new_empty((self.world_size * longest, *tail))
        dist.all_gather_into_tensor(gathered, shard, group=self.group)
        if all(n == longest for n in plan.splits[:-1]):
            return gathered[:plan.sequence_length]
        blocks = gathered.view(self.world_size, longest, *tail)
        return torch.cat([blocks[r, :n] for r, n in enumerate(plan.splits)])

    def local_frame_sums(self, local_x: torch.Tensor, num_frames: int, tokens_per_frame: int,
                         video_start: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        """Per-frame fp32 sums of this rank's rows, one contiguous slice per frame
        (deterministic; ulysses_runtime.py:606-635).  `out` [num_frames, W] fp32."""
        v0 = video_start
        lo, hi = self.local_start, self.local_end
        # Frame f's rows clipped to this rank's shard, as offsets into local_x; frames
        # outside the shard get empty ranges (zero sums).
        bounds = [min(max(v0 + f * tokens_per_frame, lo), hi) - lo for f in range(num_frames + 1)]
        if local_x.is_cuda:
            return frame_sums(local_x, bounds, 1.0, out=out)
        # Host tensors (gloo process groups): one torch sum per frame slice.
        sums = out if out is not None else torch.empty(num_frames, local_x.shape[-1], dtype=torch.float32)
        for f in range(num_frames):
            torch.sum(local_x[bounds[f]:bounds[f + 1]], 0, dtype=torch.float32, out=sums[f])
        return sums

    def video_frame_mean_async(self, local_x, num_frames, tokens_per_frame, video_start=0):
        """Launch the frame-sum all-reduce; returns (sums, work) (ulysses_runtime.py:638-643)."""
        sums = self.local_frame_sums(local_x, num_frames, tokens_per_frame, video_start)
        work = dist.all_reduce(sums, async_op=True, group=self.group)
        return sums, work


def _all_to_all(recv, send, out_sizes, in_sizes, group, async_op=False):
    return dist.all_to_all_single(recv, send, output_split_sizes=out_sizes, input_split_sizes=in_sizes,
                                  group=group, async_op=async_op)


def init_ulysses(backend: str = "nccl", *, profile_enabled: bool = False,
                 timeout_seconds: int = 120) -> UlyssesRuntime:
    """Runtime for this process from torchrun's environment (RANK, WORLD_SIZE, LOCAL_RANK,
    MASTER_*), the reference's entry point (ulysses_runtime.py:646-682).  "nccl" binds
    LOCAL_RANK's GPU (and passes it to the process group so NCCL connects eagerly); the
    process group is created unless one exists.  The short default timeout makes a rank
    that never joins end the others' next collective with an error."""
    env_world = os.environ.get("WORLD_SIZE")
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cpu")
    if backend == "nccl":
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
    if not dist.is_initialized():
        extra = {"device_id": device} if backend == "nccl" else {}
        dist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_seconds), **extra)
    world = dist.get_world_size()
    if env_world is not None and int(env_world) != world:
        raise RuntimeError(f"WORLD_SIZE={env_world}, process group has {world}")
    return UlyssesRuntime(dist.get_rank(), world, local_rank, device, backend,
                          profile_enabled=profile_enabled, timeout_seconds=timeout_seconds)


# ---------------------------------------------------------------- model install
def _hybrid_blocks(model):
    blocks = getattr(model, "transformer_blocks", None)
    if blocks is None:
        return []
    from .block import HybridBlock
    return [b for b in blocks if isinstance(b, HybridBlock)]


def _ulysses_block_forward(self, x, temb, frames, tokens, runtime=None, text_rows=0):
    """An installed block: this rank's rows in and out, attention head-sharded through the
    runtime bound by install_ulysses (the reference swaps attn.forward for
    _ulysses_attention_forward / _branch_parallel_attention_forward, ulysses.py:271-598)."""
    from .block import HybridBlock
    rt = self._ulysses_runtime if runtime is None else runtime
    if rt is not None and rt.world_size == 1:
        rt = None                         # one rank: the unsharded block, no collectives
    return HybridBlock.forward(self, x, temb, frames, tokens, rt, text_rows=text_rows)


def _ulysses_transformer_forward(self, x, temb, frames, tokens, text_rows=0):
    """The installed model forward (ulysses.py:601-714 without the checkpoint's embedders):
    x is the whole packed sequence [text_rows + frames * tokens, hidden]; the runtime is
    configured for it, this rank keeps its contiguous row shard through every block, and
    the shards are all-gathered at the end, so every rank returns the whole output."""
    if torch.is_grad_enabled():
        raise RuntimeError("Ulysses forward is inference-only; use torch.no_grad()")
    rt = self._ulysses_runtime
    blocks = self.transformer_blocks
    if x.shape[0] != text_rows + frames * tokens:
        raise ValueError("x must hold text_rows + frames * tokens rows")
    rt.configure(x.shape[0], blocks[0].cfg.heads)
    local = x[rt.local_start:rt.local_end].contiguous()
    for block in blocks:
        local = block(local, temb, frames, tokens, text_rows=text_rows)
    return local if rt.world_size == 1 else rt.gather_sequence(local)


def install_ulysses(model, runtime: UlyssesRuntime, *, softmax_ranks: int | None = None) -> None:
    """Install Ulysses on this already-built inference model instance (ulysses.py:717-764).

    `model.transformer_blocks` holds the HybridBlocks (HybridStack).  softmax_ranks
    None / 0 keeps the standard layout (every rank owns H/P heads of both branches);
    n > 0 makes n softmax ranks and world - n VDA ranks.  The checks and messages are
    the reference's.  Each block's forward is bound to the runtime and the model's
    forward becomes the sharded transformer forward.  The reference's VDA-overlap
    restriction (standard eight-way only) does not apply: every layout here runs the
    VDA branch on its side stream."""
    blocks = _hybrid_blocks(model)
    if not blocks:
        raise ValueError("Ulysses path currently requires a HybridAttention checkpoint")
    heads = blocks[0].cfg.heads
    if softmax_ranks:
        runtime.enable_branch_parallel(softmax_ranks)
    if heads % runtime.world_size:
        raise ValueError(f"{heads} attention heads are not divisible by {runtime.world_size} ranks")
    for block in blocks:
        if block.cfg.heads != heads:
            raise ValueError("all H3 blocks must have the same attention head count")
        if block.cfg.hidden != block.cfg.heads * block.cfg.head_dim:
            raise ValueError(
                "the inference Ulysses pack currently requires linear_head_dim == attention head_dim")
    for block in blocks:
        block._ulysses_runtime = runtime
        block.forward = types.MethodType(_ulysses_block_forward, block)
    model._ulysses_runtime = runtime
    model.forward = types.MethodType(_ulysses_transformer_forward, model)
