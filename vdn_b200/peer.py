"""Peer memory for the Ulysses exchange (CUDA IPC over NVLink / NVSwitch).

The reference exchanges q / k / v and the attention outputs with NCCL
all-to-all (src/inference/utils/ulysses_runtime.py:451-582).  Here every rank
maps the other ranks' receive buffers into its own address space once per
sequence geometry, and the producing kernels store into them directly:

  * the QKV GEMM (vdn_mxfp8_gemm_scatter) writes each head's q / k / v slice of
    its rows into the head owner's buffer [T, H/P, 3d], so the transfer runs
    inside the GEMM's epilogue, tile by tile;
  * vdn_mxfp8_quantize_scatter writes the head-sharded softmax and VDA outputs
    as MXFP8 codes and scales into the row owner's padded GEMM operands, so the
    output projection starts from its usual [rows, hidden] MXFP8 input.

A stream-ordered NCCL all-reduce of one element (`fence`) separates a producer
from its consumers on every rank.  No multicast objects are used.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["PeerBuffer", "PeerExchange"]

_ALIGN = 256


def _up(n: int, a: int = _ALIGN) -> int:
    return (n + a - 1) // a * a


class _Interface:
    """Minimal __cuda_array_interface__ (v3) over a raw byte range."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self.owner = owner
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


class PeerBuffer:
    """A zero-filled device buffer of this rank, mapped into every rank of the group.

    `ptrs[p]` is rank p's buffer as seen from this process (this rank's own
    allocation at p == rank).  Sizes may differ across ranks.
    """

    def __init__(self, nbytes: int, rank: int, world: int, device: torch.device, group=None):
        self.nbytes, self.rank, self.world, self.device = int(nbytes), rank, world, device
        ptr = C.c_void_p()
        _lib.call("vdn_peer_alloc", C.c_size_t(self.nbytes), C.byref(ptr))
        self.local = ptr.value
        self.ptrs = [0] * world
        self.ptrs[rank] = self.local
        self._opened = []
        if world > 1:
            handle = (C.c_uint8 * 64)()
            _lib.call("vdn_ipc_handle", C.c_void_p(self.local), handle)
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
            every = torch.empty(world * 64, dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = every.view(world, 64).cpu()
            for p in range(world):
                if p == rank:
                    continue
                raw = (C.c_uint8 * 64)(*every[p].tolist())
                out = C.c_void_p()
                _lib.call("vdn_ipc_open", raw, C.byref(out))
                self.ptrs[p] = out.value
                self._opened.append(out.value)

    def view(self, dtype: torch.dtype, shape, offset: int = 0) -> torch.Tensor:
        """A torch view of this rank's own buffer (no copy)."""
        numel = 1
        for s in shape:
            numel *= int(s)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        if offset < 0 or offset + nbytes > self.nbytes:
            raise ValueError("view exceeds the peer buffer")
        raw = torch.as_tensor(_Interface(self.local + offset, nbytes, self), device=self.device)
        return raw.view(dtype).view(*shape)

    def close(self) -> None:
        for ptr in self._opened:
            _lib.call("vdn_ipc_close", C.c_void_p(ptr))
        self._opened = []
        if self.local:
            _lib.call("vdn_peer_free", C.c_void_p(self.local))
            self.local = 0


class PeerExchange:
    """Peer buffers of one Ulysses geometry: T rows, H heads of d, hidden = H * d.

    heads side (per rank, all T rows, its H/P heads): qkv [T, H/P, 3d] bf16
    sequence side (per rank, its rows, padded to 128): MXFP8 codes [rp, hidden]
    and swizzled scales of the softmax output and of the VDA output.
    """

    def __init__(self, runtime, T: int, H: int, d: int, frames: int = 0, row_width: int = 0):
        rt = runtime
        if H % rt.world_size:
            raise ValueError("heads must divide over the ranks")
        if rt.world_size > 8:
            raise ValueError("the peer exchange supports at most 8 ranks (one node)")
        if d % 128:
            raise ValueError("the peer exchange needs head_dim % 128 == 0")
        self.rt, self.T, self.H, self.d = rt, T, H, d
        self.P, self.hl = rt.world_size, H // rt.world_size
        self.hidden = H * d
        self.head0 = rt.rank * self.hl
        self.row_starts = [0]
        for n in rt.splits:
            self.row_starts.append(self.row_starts[-1] + n)
        rows = rt.splits[rt.rank]

        self.rp = (rows + 127) // 128 * 128
        dev = rt.device
        # heads side
        self.heads = PeerBuffer(T * self.hl * 3 * d * 2, rt.rank, self.P, dev, rt.group)
        # sequence side: [att codes | att scales | lin codes | lin scales]
        codes, scales = self.rp * self.hidden, self.rp * self.hidden // 32
        self.off = [0, _up(codes), _up(codes) + _up(scales), 2 * _up(codes) + _up(scales)]
        self.seq = PeerBuffer(2 * _up(codes) + 2 * _up(scales), rt.rank, self.P, dev, rt.group)
        # QKV scatter table: 128-column chunk of the [q | k | v] GEMM output -> the
        # owner's address of that chunk in row 0 (a head of d % 128 == 0 columns
        # spans whole chunks, so every chunk has exactly one owner).
        table = []
        for col in range(0, 3 * self.hidden, 128):
            part, rem = divmod(col, self.hidden)
            h, e = divmod(rem, d)
            p, j = divmod(h, self.hl)
            table.append(self.heads.ptrs[p] + ((j * 3 + part) * d + e) * 2)
        self.chunk_dst = torch.tensor(table, dtype=torch.int64, device=dev)
        self.dst_ld = self.hl * 3 * d
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)
        # Per-token side inputs gathered on every rank ([T, row_width] bf16) and the
        # per-rank frame sums ([P, frames, hidden] fp32), published by copy-engine
        # copies into every peer (no SM time taken from the overlapping GEMM).
        self.frames, self.row_width = frames, row_width
        rows_bytes = _up(max(1, T * row_width * 2))
        sums_bytes = _up(max(1, self.P * frames * self.hidden * 4))
        self.side = PeerBuffer(rows_bytes + sums_bytes + _ALIGN, rt.rank, self.P, dev, rt.group)
        self._sums_off = rows_bytes
        # device fence: one uint64 flag per rank in every rank's buffer (bytes 0-63)
        # and this rank's epoch counter (bytes 128-135), zero-initialised
        self._flags_off = rows_bytes + sums_bytes
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fence_mode = "device"
        # sequence-side destinations of every rank, for the scatter quantiser
        seq_ptrs = self.seq.ptrs
        self.att_dst = [(p + self.off[0], p + self.off[1]) for p in seq_ptrs]
        self.lin_dst = [(p + self.off[2], p + self.off[3]) for p in seq_ptrs]

    # ----------------------------------------------------------------- views
    def qkv(self) -> torch.Tensor:
        return self.heads.view(torch.bfloat16, (self.T, self.hl, 3 * self.d))

    def operands(self):
        """This rank's ((att codes, att scales), (lin codes, lin scales)) GEMM inputs."""
        c, s = self.rp * self.hidden, self.rp * self.hidden // 32
        att = (self.seq.view(torch.uint8, (self.rp, self.hidden), self.off[0]),
               self.seq.view(torch.uint8, (s,), self.off[1]))
        lin = (self.seq.view(torch.uint8, (self.rp, self.hidden), self.off[2]),
               self.seq.view(torch.uint8, (s,), self.off[3]))
        return att, lin

    def rows(self) -> torch.Tensor:
        """[T, row_width] bf16: every rank's published side rows (valid after a fence)."""
        return self.side.view(torch.bfloat16, (self.T, self.row_width))

    def local_rows(self) -> torch.Tensor:
        """This rank's slot [rows, row_width] of rows(); write it, then publish_rows()."""
        lo = self.row_starts[self.rt.rank]
        return self.rows()[lo:lo + self.rows_local]

    @property
    def rows_local(self) -> int:
        return self.rt.splits[self.rt.rank]

    def sums(self) -> torch.Tensor:
        """[P, frames, hidden] fp32: every rank's published frame sums (valid after a fence)."""
        return self.side.view(torch.float32, (self.P, self.frames, self.hidden), self._sums_off)

    def publish_rows(self) -> None:
        lo = self.row_starts[self.rt.rank]
        off = lo * self.row_width * 2
        self._publish(off, self.rows_local * self.row_width * 2)

    def publish_sums(self) -> None:
        slot = self.frames * self.hidden * 4
        self._publish(self._sums_off + self.rt.rank * slot, slot)

    def _publish(self, offset: int, nbytes: int) -> None:
        """This rank's bytes [offset, offset + nbytes) of `side` into every peer, one launch."""
        peers = [self.side.ptrs[p] + offset for p in range(self.P) if p != self.rt.rank]
        stream = _lib.stream_of(self.rt.device)
        src = self.side.local + offset
        body = nbytes // 16 * 16
        if body:
            _lib.call("vdn_peer_broadcast", C.c_void_p(src), C.c_size_t(body), len(peers),
                      (C.c_void_p * len(peers))(*peers), stream)
        if nbytes > body:  # a ragged tail (odd row widths): copy engines
            for dst in peers:
                _lib.call("vdn_copy_async", C.c_void_p(dst + body), C.c_void_p(src + body),
                          C.c_size_t(nbytes - body), stream)

    # ------------------------------------------------------------ operations
    def gather_rows_async(self, x: torch.Tensor):
        """All-gather this rank's [rows, W] into [P * max_rows, W]; returns (buffer, work)."""
        mx = max(self.rt.splits)
        src = x
        if x.shape[0] < mx:
            src = x.new_zeros((mx, *x.shape[1:]))
            src[: x.shape[0]].copy_(x)
        out = x.new_empty((self.P * mx, *x.shape[1:]))
        work = dist.all_gather_into_tensor(out, src.contiguous(), group=self.rt.group, async_op=True)
        return out, work

    def finish_rows(self, gathered: torch.Tensor) -> torch.Tensor:
        """The [T, W] rows of a gather_rows_async buffer, in sequence order."""
        splits = self.rt.splits
        mx = max(splits)
        if all(n == mx for n in splits[:-1]):
            return gathered[: self.T]
        chunks = gathered.view(self.P, mx, *gathered.shape[1:])
        return torch.cat([chunks[p, :n] for p, n in enumerate(splits)], dim=0)

    def fence(self) -> None:
        """Stream-ordered rendezvous: every rank's earlier kernels (and their peer
        stores) complete before any rank's later kernels run.  "device": one
        vdn_peer_fence launch (flags in peer memory, bounded waits); "nccl": a
        one-element NCCL all-reduce."""
        if self.fence_mode == "nccl":
            dist.all_reduce(self._flag, group=self.rt.group)
            return
        flags = (C.c_void_p * self.P)(*[p + self._flags_off for p in self.side.ptrs])
        _lib.call("vdn_peer_fence", self.P, flags, C.c_void_p(self.side.local + self._flags_off),
                  self.rt.rank, C.c_void_p(self.side.local + self._flags_off + 128), _lib.ptr(self.status),
                  _lib.stream_of(self.rt.device))

    def check(self) -> None:
        """Raise RuntimeError if a device fence timed out (reads a device flag: syncs)."""
        if int(self.status.item()):
            self.status.zero_()
            raise RuntimeError("Ulysses peer fence timed out waiting for another rank")

    def scatter_quantize(self, src: torch.Tensor, dst) -> None:
        """src [T, H/P, d] bf16 view (last dim contiguous) -> owners' MXFP8 operands."""
        t, hl, d = src.shape
        if (t, hl, d) != (self.T, self.hl, self.d) or src.dtype != torch.bfloat16 or src.stride(-1) != 1:
            raise ValueError("scatter source must be a bf16 [T, H/P, d] view")
        n = self.P
        starts = (C.c_int64 * (n + 1))(*self.row_starts)
        codes = (C.c_void_p * n)(*[c for c, _ in dst])
        scales = (C.c_void_p * n)(*[s for _, s in dst])
        _lib.call("vdn_mxfp8_quantize_scatter", _lib.ptr(src), t, hl, d, src.stride(0), src.stride(1),
                  self.head0, self.hidden, n, starts, codes, scales, None, _lib.stream_of(src.device))

    def close(self) -> None:
        torch.cuda.synchronize(self.rt.device)
        if self.P > 1:
            dist.barrier(group=self.rt.group)
        self.heads.close()
        self.seq.close()
        self.side.close()
