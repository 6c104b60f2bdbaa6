"""Multi-process (batch-split) plumbing on CPU with the gloo backend, world size 2:
shard arithmetic, barrier, max over ranks, the checksum gather, and a rank that
dies before a collective (the survivor must get an error, not hang)."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

import ranks

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shards_cover_batch_exactly_once():
    for n in (1, 7, 64, 256, 1000):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                first, cnt = ranks.shard(n, ranks.Rank(r, world, r))
                seen.extend(range(first, first + cnt))
            assert seen == list(range(n)), (n, world)


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "cache-aware-wino-implementation_b200"))
    import ranks as rk_mod

    r = rk_mod.from_env()
    try:
        rk_mod.init(r, "gloo", timeout_s=5.0)
        if mode == "die" and rank == 1:
            raise SystemExit(3)  # leaves between steps, before the next collective
        rk_mod.barrier(r)
        t = rk_mod.max_over_ranks(10.0 + rank, r)
        sums = rk_mod.gather_floats(100.0 * rank, r)
        first, cnt = rk_mod.shard(64 * world, r)
        q.put((rank, "ok", t, sums, first, cnt))
        rk_mod.finish(r)
    except SystemExit:
        raise
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
    alive = [p for p in ps if p.is_alive()]
    for p in alive:
        p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out), [p.exitcode for p in ps], alive


def test_two_ranks_gloo():
    out, codes, alive = _run(2, "ok")
    assert not alive and codes == [0, 0]
    assert [o[1] for o in out] == ["ok", "ok"]
    for rank, _, t, sums, first, cnt in out:
        assert t == 11.0
        assert sums == [0.0, 100.0]
        assert (first, cnt) == (64 * rank, 64)


def test_dead_rank_is_detected_not_hung():
    out, codes, alive = _run(2, "die")
    assert not alive, "a surviving rank hung instead of failing"
    assert codes[1] == 3
    assert out and out[0][0] == 0 and out[0][1] == "error"
