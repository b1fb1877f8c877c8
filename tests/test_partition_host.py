"""Single-box partitioner, host side: shard math, and the K-split / gather
orchestration on world-size-2 gloo CPU ranks (the local product is injected
as a CPU matmul; no GPU).  Failure detection: a rank that dies before the
reduction surfaces as an error on its peer within the group timeout."""
import datetime
import multiprocessing as mp
import os
import socket
import time

import pytest
import torch

from conftest import import_pkg

part = import_pkg("partition")


@pytest.mark.parametrize("total,world", [(0, 1), (1, 1), (7, 3), (128, 8), (16, 8), (5, 8),
                                         (262144, 8), (129, 2)])
def test_shard_plan_covers_exactly_and_balances(total, world):
    plan = part.shard_plan(total, world)
    assert plan[0][0] == 0 and plan[-1][1] == total
    for (a, b), (c, d) in zip(plan, plan[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in plan]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_requests():
    for args in [(10, 0, 0), (10, 2, 2), (-1, 2, 0)]:
        with pytest.raises(ValueError):
            part.shard_range(*args)


@pytest.mark.parametrize("k,world", [(262144, 8), (262144, 3), (100, 4), (31, 2), (4096, 1)])
def test_k_split_plan_aligned_and_complete(k, world):
    plan = part.k_split_plan(k, world)
    assert plan[0][0] == 0 and plan[-1][1] == k
    for (a, b), (c, d) in zip(plan, plan[1:]):
        assert b == c
    for a, b in plan[:-1]:
        assert a % 32 == 0 and (b % 32 == 0 or b == k)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, scenario, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    timeout = datetime.timedelta(seconds=4)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
    p = part.Partitioner(rank, world, None, local_matmul=lambda A, B: A @ B)
    g = torch.Generator().manual_seed(0)
    M, K, N = 24, 200, 17
    A = torch.randn(M, K, generator=g, dtype=torch.float64)
    B = torch.randn(K, N, generator=g, dtype=torch.float64)
    try:
        if scenario == "split_k":
            k0, k1 = p.k_range(K)
            C = p.split_k_matmul(A[:, k0:k1], B[k0:k1], root=0)
            if rank == 0:
                q.put(("ok", float((C - A @ B).abs().max())))
            C2 = p.split_k_matmul(A[:, k0:k1], B[k0:k1], all_ranks=True)
            q.put(("all", rank, float((C2 - A @ B).abs().max())))
        elif scenario == "gather":
            r0, r1 = p.batch_range(M)
            full = p.gather_rows(A[r0:r1] * 2, M)
            q.put(("gather", rank, float((full - 2 * A).abs().max())))
        elif scenario == "peer_orchestration":
            fake = FakePeerBackend(rank)
            red = p.peer_reducer(M * N, backend=fake)
            assert p.peer_reducer(M * N, backend=fake) is red      # one mailbox set per size
            part_t = torch.zeros(M, N)
            for _ in range(2):
                red.reduce(None, part_t, root=0) if rank == 0 else \
                    red.reduce(part_t, None, root=0)
            red.close()
            q.put(("peer", rank, red.epoch, fake.calls, fake.closed, fake.destroyed))
        elif scenario == "fused_orchestration":
            fake = FakePeerBackend(rank)
            red = p.peer_reducer(M * N, backend=fake)
            k0, k1 = p.k_range(K)
            part_t = torch.zeros(M, N)
            outs = []
            for step in range(4):            # epochs alternate: fused, two-kernel, ...
                if step % 2 == 0:
                    C = red.matmul(A[:, k0:k1], B[k0:k1], root=0)
                    outs.append(float((C - A[:, k0:k1] @ B[k0:k1]).abs().max()))
                else:
                    red.reduce(None, part_t, root=0) if rank == 0 else \
                        red.reduce(part_t, None, root=0)
            try:
                red.matmul(A[:, :3], B[:3, :5], root=0)
                bad = "accepted"
            except ValueError:
                bad = "rejected"
            red.close()
            q.put(("fused", rank, red.epoch, fake.fused, [c[6] for c in fake.calls], max(outs),
                   bad))
        elif scenario == "dead_peer":
            if rank == 1:
                os._exit(3)          # leaves between steps, nothing in flight
            t0 = time.time()
            try:
                k0, k1 = p.k_range(K)
                p.split_k_matmul(A[:, k0:k1], B[k0:k1], root=0)
                q.put(("no_error", time.time() - t0))
            except Exception as e:    # the reduce cannot complete without rank 1
                q.put(("error", time.time() - t0, type(e).__name__))
    finally:
        if scenario != "dead_peer":
            dist.destroy_process_group()


class FakePeerBackend:
    """Stand-in for the C-ABI mailbox calls: pointers 1000 + rank for a rank's
    own mailbox, 2000 + rank for a peer's opened from its handle."""

    def __init__(self, rank):
        self.rank = rank
        self.calls = []
        self.closed = []
        self.destroyed = []

    def peer_mailbox_create(self, elems, world):
        return 1000 + self.rank, f"mailbox-of-{self.rank}".encode().ljust(64, b"\0")

    def peer_mailbox_open(self, handle):
        return 2000 + int(handle.rstrip(b"\0").decode().split("-")[-1])

    def peer_mailbox_close(self, ptr):
        self.closed.append(ptr)

    def peer_mailbox_destroy(self, ptr):
        self.destroyed.append(ptr)

    def splitk_peer_reduce(self, partial, out, elems, mailboxes, rank, root, epoch, stream):
        self.calls.append((bool(partial), bool(out), elems, list(mailboxes), rank, root, epoch))
        return 0

    def torch_gemm_splitk_peer(self, A, B, mailboxes, rank, root, epoch):
        self.__dict__.setdefault("fused", []).append((list(mailboxes), rank, root, epoch))
        return A @ B


def _run(scenario, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return out, [pr.exitcode for pr in procs]


def test_split_k_reduce_matches_full_product_on_gloo_ranks():
    out, codes = _run("split_k")
    assert codes == [0, 0]
    ok = [o for o in out if o[0] == "ok"]
    assert ok and ok[0][1] < 1e-9
    alls = [o for o in out if o[0] == "all"]
    assert len(alls) == 2 and all(o[2] < 1e-9 for o in alls)


def test_gather_rows_reassembles_shards():
    out, codes = _run("gather")
    assert codes == [0, 0]
    assert len(out) == 2 and all(o[2] == 0.0 for o in out)


def test_dead_peer_surfaces_as_error_not_hang():
    out, codes = _run("dead_peer", timeout=90)
    assert codes[1] == 3
    res = [o for o in out if o[0] in ("error", "no_error")]
    assert res and res[0][0] == "error", res
    assert res[0][1] < 60


def test_peer_reducer_exchanges_handles_and_counts_epochs():
    """The peer-memory reduction's host side on gloo ranks: IPC handles go
    round with all_gather_object, each rank's table lists every mailbox in
    rank order (its own pointer, the others opened from their handles), all
    ranks call with the same epochs, the root passes `out` and the others
    `partial`, and close() unmaps the peers' mailboxes and frees its own."""
    out, codes = _run("peer_orchestration")
    assert codes == [0, 0]
    res = {o[1]: o for o in out if o[0] == "peer"}
    assert set(res) == {0, 1}
    M, N = 24, 17
    for rank, (_, _, epoch, calls, closed, destroyed) in res.items():
        assert epoch == 2
        table = [1000, 2001] if rank == 0 else [2000, 1001]
        assert [c[6] for c in calls] == [1, 2]
        for partial, outp, elems, mbs, r, root, _ in calls:
            assert elems == M * N and mbs == table and r == rank and root == 0
            assert (partial, outp) == ((False, True) if rank == 0 else (True, False))
        assert closed == [t for i, t in enumerate(table) if i != rank]
        assert destroyed == [1000 + rank]


def test_fused_split_k_shares_the_epoch_sequence_with_the_two_kernel_path():
    """PeerReducer.matmul (the one-kernel K split, b2g_gemm_splitk_peer) on
    gloo ranks with a stand-in binding: it passes this rank's slices, the
    mailbox table, the rank and the root, and draws its epochs from the same
    counter as reduce(), so the two paths alternate epoch by epoch (1, 3 fused;
    2, 4 two-kernel); a product of another size than the mailbox's is
    rejected."""
    out, codes = _run("fused_orchestration")
    assert codes == [0, 0]
    res = {o[1]: o for o in out if o[0] == "fused"}
    assert set(res) == {0, 1}
    for rank, (_, _, epoch, fused, reduce_epochs, err, bad) in res.items():
        table = [1000, 2001] if rank == 0 else [2000, 1001]
        assert epoch == 4
        assert [f[3] for f in fused] == [1, 3] and reduce_epochs == [2, 4]
        assert all(f[0] == table and f[1] == rank and f[2] == 0 for f in fused)
        assert err < 1e-12 and bad == "rejected"
