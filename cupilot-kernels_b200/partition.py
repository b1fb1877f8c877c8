"""Single-box partitioner: one process per GPU, torch.distributed for plumbing.

Two ways to spread one operator call over the GPUs of a node:

* Batch / M sharding (batched, 3-D and 4-D products, any plain GEMM along M):
  rank r owns a contiguous, balanced slice of the batch (or of M) and
  computes it with the local kernel.  No communication: outputs stay sharded
  (`gather_rows` brings them together when a caller wants one tensor).
* K splitting (large-K, reference kernels/6_Matmul_with_large_K_dimension_best_kernel.cu,
  whose 8 streams + 7 `C.add_` on one GPU at K6:147-200 become ranks +
  a reduction): rank r multiplies A[:, K_r] by B[K_r, :] locally, then the
  partial products are summed on the root over NVLink.  On GPUs the sum
  is the library's own peer-memory reduction (b2g_splitk_peer_reduce: each
  rank pushes its partial into the root's mailbox right behind its GEMM, the
  root adds them; no NCCL call, no host synchronisation); otherwise, or when
  every rank needs C, one NCCL (gloo on CPU) reduce / all-reduce.

The local product is the package's own GEMM (`ops`); callers may inject a
different `local_matmul` (the host-side tests run the orchestration on CPU
ranks with gloo).  Every collective runs under the process group's timeout,
so a rank that dies or stalls surfaces as an error on the others instead of
a hang.
"""
from __future__ import annotations

import datetime
from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of `total` items owned by `rank`; the first
    total % world ranks get one extra item."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request total={total} world={world} rank={rank}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def shard_plan(total: int, world: int) -> List[Tuple[int, int]]:
    return [shard_range(total, world, r) for r in range(world)]


def k_split_plan(k: int, world: int, align: int = 32) -> List[Tuple[int, int]]:
    """K ranges per rank, rounded to `align` (the kernel's K block) so no
    rank's slice straddles a K block except the last; every range may be
    empty only when k < world * align."""
    blocks = (k + align - 1) // align
    out = []
    for r in range(world):
        b0, b1 = shard_range(blocks, world, r)
        out.append((min(b0 * align, k), min(b1 * align, k)))
    return out


def _default_matmul():
    import importlib

    ops = importlib.import_module(__package__ + ".ops")
    return lambda A, B: ops.gemm(A, B, False, False, 0)


@dataclass
class Partitioner:
    """Per-rank view of the node: rank, world size and the process group."""

    rank: int
    world: int
    group: Optional[dist.ProcessGroup] = None
    local_matmul: Optional[Callable] = None

    @classmethod
    def from_env(cls, local_matmul: Optional[Callable] = None, group=None) -> "Partitioner":
        if dist.is_available() and dist.is_initialized():
            return cls(dist.get_rank(group), dist.get_world_size(group), group, local_matmul)
        return cls(0, 1, None, local_matmul)

    def _mm(self):
        if self.local_matmul is None:
            self.local_matmul = _default_matmul()
        return self.local_matmul

    # ------------------------------------------------------------ sharding
    def batch_range(self, batch: int) -> Tuple[int, int]:
        return shard_range(batch, self.world, self.rank)

    def batched_matmul_shard(self, A_shard: torch.Tensor, B_shard: torch.Tensor,
                             bmm: Optional[Callable] = None) -> torch.Tensor:
        """C[b] = A[b] B[b] for this rank's batch slice (no communication)."""
        if bmm is None:
            import importlib

            bmm = importlib.import_module(__package__ + ".ops").p3.forward
        return bmm(A_shard, B_shard)

    def gather_rows(self, local: torch.Tensor, total_rows: int) -> torch.Tensor:
        """All-gather row shards (of shard_plan sizes) into one tensor on every rank."""
        if self.world == 1:
            return local
        plan = shard_plan(total_rows, self.world)
        width = max(b - a for a, b in plan)
        pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        pad[: local.shape[0]] = local
        bufs = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(bufs, pad, group=self.group)
        return torch.cat([bufs[r][: b - a] for r, (a, b) in enumerate(plan)], dim=0)

    # ------------------------------------------------------------ K splitting
    def k_range(self, k: int) -> Tuple[int, int]:
        return k_split_plan(k, self.world)[self.rank]

    def split_k_matmul(self, A_k: torch.Tensor, B_k: torch.Tensor, root: int = 0,
                       all_ranks: bool = False, method: str = "auto") -> Optional[torch.Tensor]:
        """Given this rank's K slice (A[:, K_r], B[K_r, :]), return C = A B on
        the root (None elsewhere), or on every rank when all_ranks.

        method: "fused" runs this rank's product and the peer-memory sum in one
        kernel (b2g_gemm_splitk_peer; CUDA tensors, one node), "peer" runs the
        product and then the stand-alone peer-memory reduction, "collective"
        one NCCL / gloo reduce; "auto" picks "fused" for CUDA tensors on more
        than one rank unless all_ranks.
        """
        if method == "auto" and A_k.is_cuda and self.world > 1 and not all_ranks:
            method = "fused"
        if method == "fused":
            if all_ranks:
                raise ValueError("the peer reduction delivers C to the root only")
            red = self.peer_reducer(A_k.shape[0] * B_k.shape[1])
            C = red.matmul(A_k, B_k, root)
            return C if self.rank == root else None
        if A_k.shape[1] == 0:
            part = torch.zeros(A_k.shape[0], B_k.shape[1], dtype=A_k.dtype, device=A_k.device)
        else:
            part = self._mm()(A_k, B_k)
        if self.world == 1:
            return part
        if method == "auto":
            method = "peer" if (A_k.is_cuda and not all_ranks) else "collective"
        if method == "peer":
            if all_ranks:
                raise ValueError("the peer reduction delivers C to the root only")
            red = self.peer_reducer(part.numel())
            red.reduce(part, part if self.rank == root else None, root)
            return part if self.rank == root else None
        if all_ranks:
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            return part
        dist.reduce(part, dst=root, op=dist.ReduceOp.SUM, group=self.group)
        return part if self.rank == root else None

    def split_k_matmul_async(self, A_k: torch.Tensor, B_k: torch.Tensor,
                             root: int = 0) -> Optional[torch.Tensor]:
        """split_k_matmul with the cross-GPU sum taken off the caller's
        stream: the GEMM runs on the current stream, the peer reduction on a
        side stream behind it, so the next call's GEMM does not wait for this
        call's sum.  The returned C (root) is complete only after `join()`,
        which makes the current stream wait for every sum issued so far."""
        if self.world == 1 or not A_k.is_cuda:
            return self.split_k_matmul(A_k, B_k, root=root)
        part = self._mm()(A_k, B_k)
        red = self.peer_reducer(part.numel())
        cur = torch.cuda.current_stream(part.device)
        side = self.__dict__.get("_side")
        if side is None:
            side = torch.cuda.Stream(part.device)
            self.__dict__["_side"] = side
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            red.reduce(part, part if self.rank == root else None, root)
        part.record_stream(side)      # the allocator keeps it until the side stream is done
        return part if self.rank == root else None

    def join(self) -> None:
        """Make the current stream wait for the sums split_k_matmul_async issued."""
        side = self.__dict__.get("_side")
        if side is not None:
            torch.cuda.current_stream(side.device).wait_stream(side)

    def peer_reducer(self, elems: int, backend=None) -> "PeerReducer":
        """The mailbox set for partials of `elems` floats, created on first use
        (a collective call: every rank must reach it)."""
        cache = self.__dict__.setdefault("_peer", {})
        if elems not in cache:
            cache[elems] = PeerReducer(self, elems, backend)
        return cache[elems]


class PeerReducer:
    """Mailboxes of the peer-memory K-split reduction for one partial size.

    Every rank creates its mailbox (device memory, b2g_peer_mailbox_create),
    the IPC handles are exchanged with one all_gather_object over the
    process group, and every rank opens the others'.  `reduce` then runs one
    epoch of the protocol on the current stream: the root adds the other
    ranks' partials into `out` (which holds its own); the others push theirs.
    All ranks must call `reduce` in the same order.  `backend` is the C-ABI
    binding (capi); tests inject a stand-in.
    """

    def __init__(self, part: "Partitioner", elems: int, backend=None):
        if backend is None:
            import importlib

            backend = importlib.import_module(__package__ + ".capi")
        self.backend = backend
        self.part = part
        self.elems = int(elems)
        self.epoch = 0
        own, handle = backend.peer_mailbox_create(self.elems, part.world)
        handles = [None] * part.world
        dist.all_gather_object(handles, handle, group=part.group)
        self.own = own
        self.mailboxes = [own if r == part.rank else backend.peer_mailbox_open(handles[r])
                          for r in range(part.world)]
        # Every rank has opened every mailbox before any rank writes into one.
        dist.barrier(group=part.group)

    def reduce(self, partial: Optional[torch.Tensor], out: Optional[torch.Tensor],
               root: int = 0) -> None:
        """Root: out += the other ranks' partials.  Others: push `partial`."""
        self.epoch += 1
        is_root = self.part.rank == root
        t = out if is_root else partial
        if t is None or t.numel() != self.elems or not t.is_contiguous():
            raise ValueError("peer reduce needs a contiguous tensor of the mailbox's size")
        fast = getattr(self.backend, "torch_splitk_peer_reduce", None)
        if fast is not None and t.is_cuda:
            fast(t, self.mailboxes, self.part.rank, root, self.epoch)   # raises on failure
            return
        stream = torch.cuda.current_stream(t.device).cuda_stream if t.is_cuda else 0
        rc = self.backend.splitk_peer_reduce(0 if is_root else t.data_ptr(),
                                             t.data_ptr() if is_root else 0, self.elems,
                                             self.mailboxes, self.part.rank, root, self.epoch,
                                             stream)
        if rc != 0:
            raise RuntimeError(f"b2g_splitk_peer_reduce failed (status {rc})")

    def matmul(self, A_k: torch.Tensor, B_k: torch.Tensor, root: int = 0) -> torch.Tensor:
        """One epoch as a single kernel: this rank's slice product A_k B_k and
        the cross-GPU sum (b2g_gemm_splitk_peer).  Returns the product tensor:
        the full sum on the root, this rank's partial elsewhere."""
        if A_k.shape[0] * B_k.shape[1] != self.elems:
            raise ValueError("the product's size differs from the mailbox's")
        self.epoch += 1
        fused = getattr(self.backend, "torch_gemm_splitk_peer", None)
        if fused is None:
            raise RuntimeError("the fused K-split needs the Torch extension's binding")
        return fused(A_k, B_k, self.mailboxes, self.part.rank, root, self.epoch)

    def close(self) -> None:
        for r, ptr in enumerate(self.mailboxes):
            if r != self.part.rank:
                self.backend.peer_mailbox_close(ptr)
        self.backend.peer_mailbox_destroy(self.own)
        self.mailboxes = []


def init_node(backend: str = "nccl", timeout_s: float = 60.0) -> Partitioner:
    """Join the node's process group from torchrun's environment (RANK,
    WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT) with a bounded timeout."""
    import os

    if not dist.is_initialized():
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    return Partitioner.from_env()
