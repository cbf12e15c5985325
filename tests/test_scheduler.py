"""Window scheduler host logic: sharding and gathering over gloo ranks on CPU."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from parakeet_cuda_b200.scheduler import WindowScheduler, shard


def test_shard_is_a_balanced_partition():
    for n in (0, 1, 7, 8, 64, 65):
        for world in (1, 2, 3, 4, 8):
            parts = [shard(n, world, r) for r in range(world)]
            flat = [i for p in parts for i in p]
            assert flat == list(range(n))
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update({'RANK': str(rank), 'WORLD_SIZE': str(world), 'LOCAL_RANK': str(rank),
                       'MASTER_ADDR': '127.0.0.1', 'MASTER_PORT': str(port)})
    sched = WindowScheduler(backend='gloo', timeout_s=60)
    windows = [f'w{i}' for i in range(9)]
    mine = sched.assign(windows)
    results = [(w, sched.rank, len(w)) for w in mine]
    gathered = sched.gather(results)
    worst = sched.max_over_ranks(float(sched.rank + 1))
    sched.barrier()
    q.put((sched.rank, mine, gathered, worst))
    sched.close()


def test_gloo_two_ranks_assign_and_gather():
    world, port = 2, _free_port()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, mine, gathered, worst = q.get(timeout=120)
        out[rank] = (mine, gathered, worst)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][0] == [f'w{i}' for i in range(5)]
    assert out[1][0] == [f'w{i}' for i in range(5, 9)]
    assert [g[0] for g in out[0][1]] == [f'w{i}' for i in range(9)]
    assert out[1][1] is None
    assert out[0][2] == out[1][2] == 2.0


def _failing_worker(rank, world, port, q):
    os.environ.update({'RANK': str(rank), 'WORLD_SIZE': str(world), 'LOCAL_RANK': str(rank),
                       'MASTER_ADDR': '127.0.0.1', 'MASTER_PORT': str(port)})
    sched = WindowScheduler(backend='gloo', timeout_s=5)
    if rank == 1:
        q.put((rank, 'left'))
        q.close()
        q.join_thread()
        os._exit(3)  # a worker that dies between steps, before the gather
    try:
        sched.gather(['x'])
        q.put((rank, 'no error'))
    except Exception as e:  # the surviving rank sees an error instead of hanging
        q.put((rank, type(e).__name__))


def test_gloo_dead_rank_surfaces_as_error():
    world, port = 2, _free_port()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msgs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert msgs[1] == 'left'
    assert msgs[0] != 'no error'
