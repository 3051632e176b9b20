"""Multi-process paths of the vocab-sharded embedding
(tb_b200_embedding_sharded, include/tb_b200.h), one process per rank.

CPU (gloo, world sizes 2 and 3): every rank builds only its own exchange
plan with tb_b200_shard_plan and moves its rows with torch.distributed
send/recv in the order the NCCL path groups them; the assembled token part
must equal the full-table gather (tb_cpu_embedding_f32,
src/ops/embedding.c:4-14) -- the plan is consistent across processes.

GPU (2 GPUs, skipped on fewer): the library's NCCL exchange itself, and
the one-kernel gather over peer memory (tb_b200_embedding_sharded_p2p,
shards mapped through CUDA IPC), both bit-exact against the oracle for f32
and bf16 tables.
"""
import ctypes as C
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "tensorbit-run_b200"))
sys.path.insert(0, ROOT)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def problem(n, vocab, dim, seed):
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, vocab, n).astype(np.int32)
    table = rng.standard_normal((vocab, dim), dtype=np.float32)
    return ids, table


def _gloo_rank(rank, world, port, n, vocab, dim, q):
    import torch
    import torch.distributed as dist
    import tb_b200 as T
    from oracle import oracle as O
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        ids, table = problem(n, vocab, dim, 1234)
        vlo, vhi = T.partition(vocab, world, rank)
        tlo, thi = T.partition(n, world, rank)
        shard = table[vlo:vhi]
        sc, rc, send, recv, ld, ls = T.shard_plan(ids, vocab, world, rank)
        out = np.full((thi - tlo, dim), np.nan, np.float32)
        out[ld] = shard[ls]
        sendbuf = torch.from_numpy(np.ascontiguousarray(shard[send]))
        recvbuf = torch.empty((int(rc.sum()), dim), dtype=torch.float32)
        reqs, so, ro = [], 0, 0
        for p in range(world):
            if p == rank:
                continue
            if sc[p]:
                reqs.append(dist.isend(sendbuf[so:so + sc[p]].contiguous(), p))
            if rc[p]:
                reqs.append(dist.irecv(recvbuf[ro:ro + rc[p]], p))
            so += int(sc[p])
            ro += int(rc[p])
        for r in reqs:
            r.wait()
        out[recv] = recvbuf.numpy()
        ok = np.array_equal(out, O.embedding(ids[tlo:thi], table))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))


def run_ranks(target, world, *args, timeout=180):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=timeout))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return sorted(results)


@pytest.mark.parametrize("world,n,vocab,dim", [(2, 1000, 32000, 16), (3, 257, 1000, 8)])
def test_sharded_embedding_exchange_gloo(world, n, vocab, dim):
    res = run_ranks(_gloo_rank, world, n, vocab, dim)
    assert len(res) == world
    for rank, ok, err in res:
        assert ok, f"rank {rank}: {err or 'token part differs from the full-table gather'}"


def _nccl_rank(rank, world, port, n, vocab, dim, q):
    import torch
    import torch.distributed as dist
    import tb_b200 as T
    from oracle import oracle as O
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        uid = [T.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        T.comm_init(world, rank, uid[0], rank)
        ids, table = problem(n, vocab, dim, 99)
        vlo, vhi = T.partition(vocab, world, rank)
        tlo, thi = T.partition(n, world, rank)
        oks = []
        for host in (table, O.f32_to_bf16(table)):  # f32, then bf16 bits
            ref = O.embedding(ids[tlo:thi], host)
            shard = torch.from_numpy(np.ascontiguousarray(host[vlo:vhi]))
            if host.dtype == np.uint16:
                shard = shard.view(torch.int16).view(torch.bfloat16)
            y = T.embedding_sharded(ids, shard.cuda(), vocab)
            torch.cuda.synchronize()
            got = y.cpu()
            if host.dtype == np.uint16:
                got = got.view(torch.int16)
            oks.append(np.array_equal(got.numpy().view(host.dtype), ref))
        T.comm_destroy()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, all(oks), ""))
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.gpu
def test_sharded_embedding_nccl_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_ranks(_nccl_rank, 2, 4096, 32000, 4096)
    assert len(res) == 2
    for rank, ok, err in res:
        assert ok, f"rank {rank}: {err or 'sharded gather differs from the full-table gather'}"


def _p2p_rank(rank, world, port, n, vocab, dim, q):
    """One kernel, no collective: this rank's rows read straight from the
    owners' shards through CUDA IPC mappings (peer loads over NVLink)."""
    import torch
    import torch.distributed as dist
    import tb_b200 as T
    from oracle import oracle as O
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        ids, table = problem(n, vocab, dim, 98)
        vlo, vhi = T.partition(vocab, world, rank)
        tlo, thi = T.partition(n, world, rank)
        oks = []
        for host in (table, O.f32_to_bf16(table)):  # f32, then bf16 bits
            shard = torch.from_numpy(np.ascontiguousarray(host[vlo:vhi]))
            if host.dtype == np.uint16:
                shard = shard.view(torch.int16).view(torch.bfloat16)
            shard = shard.cuda()
            handles = [None] * world
            dist.all_gather_object(handles, T.p2p_export(shard))
            addrs = [shard.data_ptr() if r == rank else T.p2p_import(*handles[r])
                     for r in range(world)]
            my_ids = torch.from_numpy(ids[tlo:thi].astype(np.int32)).cuda()
            for _ in range(2):  # twice: the mappings stay valid
                y = T.embedding_sharded_p2p(my_ids, addrs, vocab, dim, shard.dtype)
                torch.cuda.synchronize()
                got = y.cpu()
                if host.dtype == np.uint16:
                    got = got.view(torch.int16)
                oks.append(np.array_equal(got.numpy().view(host.dtype),
                                          O.embedding(ids[tlo:thi], host)))
            oks.append(T.check_status() == (0, 0))
            # ids outside [0, vocab): zero rows and the token-range flag, no read
            bad = torch.tensor([-1, vocab, 0], dtype=torch.int32, device="cuda")
            y = T.embedding_sharded_p2p(bad, addrs, vocab, dim, shard.dtype)
            rc, flags = T.check_status()
            got = y.cpu().view(torch.int16 if host.dtype == np.uint16 else torch.int32).numpy()
            oks.append(rc != 0 and flags == 1 and not got[:2].any()
                       and np.array_equal(got[2].view(host.dtype), host[0]))
            for r in range(world):
                if r != rank:
                    T.p2p_close(addrs[r], handles[r][1])
            dist.barrier()  # every importer closed before the owner frees its shard
            del shard
        dist.destroy_process_group()
        q.put((rank, all(oks), "" if all(oks) else f"checks {oks}"))
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("n,vocab,dim", [(4096, 32003, 4096), (333, 1001, 1000), (333, 1001, 100)])
def test_sharded_embedding_p2p_two_gpus(n, vocab, dim):
    """Odd vocabularies (rank 0 holds one row more: the uneven partition
    rule); rows of 16 KB, of 4000 / 2000 bytes (16-byte words, a ragged last
    batch) and of 400 / 200 bytes (the bf16 rows move as 4-byte words)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_ranks(_p2p_rank, 2, n, vocab, dim)
    assert len(res) == 2
    for rank, ok, err in res:
        assert ok, f"rank {rank}: {err or 'p2p gather differs from the full-table gather'}"


def _window_rank(rank, world, port, n, vocab, dim, q):
    """One kernel over NCCL symmetric memory: each rank's table part sits in
    a window every rank can load from (tb_b200_embedding_sharded_window)."""
    import torch
    import torch.distributed as dist
    import tb_b200 as T
    from oracle import oracle as O
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        uid = [T.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        T.comm_init(world, rank, uid[0], rank)
        ids, table = problem(n, vocab, dim, 97)
        vlo, vhi = T.partition(vocab, world, rank)
        tlo, thi = T.partition(n, world, rank)
        oks = []
        for host in (table, O.f32_to_bf16(table)):  # f32, then bf16 bits
            esz = host.dtype.itemsize
            cap = -(-vocab // world) * dim * esz  # the largest part: same size everywhere
            addr = T.comm_window_alloc(cap)
            part = torch.from_numpy(np.ascontiguousarray(host[vlo:vhi])).cuda()
            T.check(T.lib().tb_b200_memcpy_d2d(C.c_void_p(addr), T.ptr(part), part.numel() * esz,
                                               None), "d2d")
            torch.cuda.synchronize()
            dist.barrier()  # every shard written before any rank gathers
            tdt = torch.bfloat16 if host.dtype == np.uint16 else torch.float32
            my_ids = torch.from_numpy(ids[tlo:thi].astype(np.int32)).cuda()
            for _ in range(2):
                y = T.embedding_sharded_window(my_ids, addr, vocab, dim, tdt)
                torch.cuda.synchronize()
                got = y.cpu().view(torch.int16 if tdt == torch.bfloat16 else torch.int32).numpy()
                oks.append(np.array_equal(got.view(host.dtype), O.embedding(ids[tlo:thi], host)))
            oks.append(T.check_status() == (0, 0))
            bad = torch.tensor([-1, vocab, 0], dtype=torch.int32, device="cuda")
            y = T.embedding_sharded_window(bad, addr, vocab, dim, tdt)
            rc, flags = T.check_status()
            got = y.cpu().view(torch.int16 if tdt == torch.bfloat16 else torch.int32).numpy()
            oks.append(rc != 0 and flags == 1 and not got[:2].any()
                       and np.array_equal(got[2].view(host.dtype), host[0]))
            dist.barrier()  # every rank done reading before the windows go
            T.comm_window_free(addr)
        T.comm_destroy()
        dist.destroy_process_group()
        q.put((rank, all(oks), "" if all(oks) else f"checks {oks}"))
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("n,vocab,dim", [(4096, 32003, 4096), (333, 1001, 1000)])
def test_sharded_embedding_window_two_gpus(n, vocab, dim):
    """Odd vocabularies (uneven parts); 16 KB rows and 4000 / 2000-byte rows."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_ranks(_window_rank, 2, n, vocab, dim)
    assert len(res) == 2
    for rank, ok, err in res:
        assert ok, f"rank {rank}: {err or 'window gather differs from the full-table gather'}"
