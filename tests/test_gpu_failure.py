"""Failure paths, made to fire without faulting or hanging a GPU.

1. The bounded mbarrier wait of the staged kernels (tma.cuh): a one-warp
   kernel (tb_b200_selftest_wait) waits for 16 bytes that no copy brings,
   with a 2 ms limit.  The wait must give up, raise
   TB_B200_FLAG_WAIT_TIMEOUT in the status word, and return: the context
   stays usable and the next kernels give correct results.  The same wait
   with the copy supplied must end without a flag.

2. The communicator's bounded wait (tb_b200_comm_wait, 2 GPUs, one process
   each, NVLS off).  Both ranks run one sharded gather; rank 1 then leaves
   the job between steps, with nothing of its own in flight.  Rank 0 learns
   nothing on the host and queues its next gather, whose NCCL exchange
   waits for a peer that is gone.  With TB_B200_COMM_TIMEOUT_S=3 the wait
   must end in TB_ERR_DEVICE after the communicator is aborted, within a
   few seconds, and rank 0's context must still run kernels.
"""
import os
import time

import numpy as np
import pytest

import tb_b200 as T
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_returns(cuda):
    import torch
    torch.cuda.set_device(cuda)
    assert T.check_status() == (0, 0)
    # supplied: the copy completes the wait
    T.check(T.lib().tb_b200_selftest_wait(1, 2000, None), "selftest_wait")
    assert T.check_status() == (0, 0)
    # never supplied: the wait gives up after 2 ms and raises the flag
    t0 = time.perf_counter()
    T.check(T.lib().tb_b200_selftest_wait(0, 2000, None), "selftest_wait")
    rc, flags = T.check_status()
    assert rc == 8 and flags == T.FLAG_WAIT_TIMEOUT
    assert time.perf_counter() - t0 < 5.0
    assert T.check_status() == (0, 0)  # cleared
    # the context still works: a staged softmax and a gather agree with the oracle
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((8, 32000)) * 3).astype(np.float32)
    y = T.softmax(torch.from_numpy(x).to(cuda)).cpu().numpy().astype(np.float64)
    want = O.softmax(x)
    assert (np.abs(y - want).max(axis=1) / np.abs(want).max(axis=1)).max() <= 1e-5
    table = rng.standard_normal((100, 64)).astype(np.float32)
    ids = rng.integers(0, 100, 50).astype(np.int32)
    e = T.embedding(torch.from_numpy(ids).to(cuda), torch.from_numpy(table).to(cuda))
    assert np.array_equal(e.cpu().numpy(), table[ids])
    assert T.check_status() == (0, 0)
    # arguments: the limit is bounded
    assert T.lib().tb_b200_selftest_wait(0, 0, None) == 8
    assert T.lib().tb_b200_selftest_wait(0, 1000001, None) == 8


def _proc_exited(pid):
    """True once `pid` has exited (gone, or a zombie not yet reaped)."""
    try:
        with open(f"/proc/{pid}/stat") as f:
            return f.read().rsplit(")", 1)[1].split()[0] in ("Z", "X")
    except OSError:
        return True


def _leaving_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        os.environ["TB_B200_COMM_TIMEOUT_S"] = "3"
        torch.cuda.set_device(rank)
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                              timeout=__import__("datetime").timedelta(seconds=60))
        if rank == 0:
            store.set("uid", T.comm_unique_id())
        T.comm_init(world, rank, store.get("uid"), rank)
        rng = np.random.default_rng(5)
        n, vocab, dim = 2048, 4000, 1024
        ids = rng.integers(0, vocab, n).astype(np.int32)
        table = rng.standard_normal((vocab, dim)).astype(np.float32)
        vlo, vhi = T.partition(vocab, world, rank)
        tlo, thi = T.partition(n, world, rank)
        shard = torch.from_numpy(np.ascontiguousarray(table[vlo:vhi])).cuda()
        y = T.embedding_sharded(ids, shard, vocab)
        rc1 = T.comm_wait()
        ok1 = rc1 == 0 and np.array_equal(y.cpu().numpy(), table[ids[tlo:thi]])
        torch.cuda.synchronize()
        store.set(f"done{rank}", "1")
        store.wait(["done0", "done1"])
        if rank == 1:
            # leave between steps: nothing of this rank is in flight
            store.set("pid1", str(os.getpid()))
            q.put((rank, ok1, "" if ok1 else f"first gather rc {rc1}"))
            q.close()
            q.join_thread()
            os._exit(0)
        pid1 = int(store.get("pid1"))
        t0 = time.time()
        while not _proc_exited(pid1) and time.time() - t0 < 60:
            time.sleep(0.05)
        t0 = time.perf_counter()
        rc_q = T.lib().tb_b200_embedding_sharded(T.F32, n, dim, vocab, ids.ctypes.data,
                                                 T.ptr(shard), T.ptr(y), T.cur_stream())
        rc2 = T.comm_wait() if rc_q == 0 else rc_q
        waited = time.perf_counter() - t0
        rank_after, n_after = T.comm_info()
        # the context still runs kernels: a local gather from the shard
        local = torch.arange(64, dtype=torch.int32, device="cuda")
        e = T.embedding(local, shard)
        ok_ctx = (np.array_equal(e.cpu().numpy(), table[vlo:vlo + 64])
                  and T.check_status() == (0, 0))
        ok = ok1 and rc2 == 16 and waited < 30 and (rank_after, n_after) == (0, 0) and ok_ctx
        q.put((rank, ok, f"first {ok1} rc2 {rc2} waited {waited:.1f}s comm {n_after} "
                         f"ctx {ok_ctx}"))
    except Exception as e:
        q.put((rank, False, repr(e)))


def test_comm_wait_times_out_when_a_rank_leaves():
    import multiprocessing as mp
    import torch
    from test_multiproc import free_port
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_leaving_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in range(2):
            res.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    res.sort()
    assert len(res) == 2
    for rank, ok, msg in res:
        assert ok, f"rank {rank}: {msg}"
