"""Multi-process (world size 2, gloo, CPU) tests of the sequence-sharding
host logic: shard ranges, the max/sum counter reduction used for whole-job
throughput, the response gather, and a failing rank surfacing as an error on
the other rank instead of a hang."""
import datetime
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from flash_dllm_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        if mode == "ok":
            start, end = shard.shard_range(5, rank, world)
            times, counts = shard.reduce_counters([1.0 + rank, 3.0 - rank], [10.0 * (rank + 1), 1.0])
            local = [[start + i] * (start + i + 1) for i in range(end - start)]
            allr = shard.gather_responses(local, start, 5)
            q.put((rank, (start, end), times, counts, allr))
        else:
            if rank == 1:
                os._exit(3)  # dies between steps, before the result gather
            try:
                shard.reduce_counters([1.0], [1.0])
                q.put((rank, "no error"))
            except Exception as e:  # the peer's death must surface as an error
                q.put((rank, "error", type(e).__name__))
    finally:
        if mode == "ok":
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = []
    for p in ps:
        p.join(timeout=120)
    while not q.empty():
        out.append(q.get())
    for p in ps:
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0]), [p.exitcode for p in ps]


def test_shard_reduce_gather_world2():
    out, codes = _run("ok")
    assert codes == [0, 0] and len(out) == 2
    (r0, s0, t0, c0, a0), (r1, s1, t1, c1, a1) = out
    assert s0 == (0, 3) and s1 == (3, 5)
    assert t0 == t1 == [2.0, 3.0]          # max over ranks
    assert c0 == c1 == [30.0, 2.0]         # sum over ranks
    want = [[i] * (i + 1) for i in range(5)]
    assert a0 == a1 == want


def test_dead_rank_raises_on_peer():
    out, codes = _run("dead")
    assert codes[1] == 3
    assert out and out[0][0] == 0 and out[0][1] == "error"


def test_shard_range_covers_all():
    from flash_dllm_b200.shard import shard_range
    for n in range(0, 20):
        for w in range(1, 9):
            spans = [shard_range(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)
