"""Multi-process (batch-split) plumbing on CPU with the gloo backend, world size 2:
shard arithmetic, barrier, max over ranks, the checksum gather, the split ->
gather -> check path that bench.py runs after its timed region (each rank's
output of its shard stands in for the GPU's; a mistake planted in one rank's
output must be caught for that rank only), and a rank that dies before a
collective (the survivor must get an error, not hang)."""
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


def _split_worker(rank, world, port, plant, q):
    """One rank of a split run: convolve this rank's shard of a small layer (the CPU
    oracle stands in for the GPU kernel), gather the sampled outputs to rank 0 and check
    them there with bench.py's own helpers."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    root = os.path.dirname(HERE)
    for p in (os.path.join(root, "cache-aware-wino-implementation_b200"),
              os.path.join(root, "oracle"), root):
        sys.path.insert(0, p)
    import torch

    import bench
    import oracle
    import ranks as rk_mod
    import workloads

    r = rk_mod.from_env()
    try:
        rk_mod.init(r, "gloo", timeout_s=20.0)
        layer = workloads.Layer(1, 0, 6, 8, 12, 10, 9, 2, True, "uniform")
        first, cnt = rk_mod.shard(layer.n, r)
        g, bias = workloads.make_weights(layer)
        x = workloads.make_input(layer, cnt, first_image=first)
        y = oracle.conv_layer(x, oracle.weight_transform(g, 4), bias, 4, True)
        if plant and rank == 1:
            y[-1, 3, 4, 5] += 1e-2  # the last image of rank 1's shard is wrong
        samples = bench.gather_samples(torch.from_numpy(y), first, cnt, r, None)
        res = None
        if rank == 0:
            res = bench.check_samples(
                layer, samples, lambda i: workloads.make_input(layer, 1, first_image=i)[0], g,
                bias)
        q.put((rank, "ok", first, cnt, res))
        rk_mod.finish(r)
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None, None))


def _run_split(world, plant):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_split_worker, args=(r, world, port, plant, q))
          for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    alive = [p for p in ps if p.is_alive()]
    for p in alive:
        p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda o: o[0]), [p.exitcode for p in ps], alive


@pytest.mark.parametrize("plant", [False, True])
def test_split_gather_check(plant):
    out, codes, alive = _run_split(2, plant)
    assert not alive and codes == [0, 0], out
    assert [o[1] for o in out] == ["ok", "ok"], out
    assert [(o[2], o[3]) for o in out] == [(0, 3), (3, 3)]
    res = out[0][4]
    rows = res["per_rank"]
    assert [d["rank"] for d in rows] == [0, 1]
    assert [d["images"] for d in rows] == [[0, 2], [3, 5]]
    assert rows[0]["max_abs_err"] == 0.0
    if plant:
        assert not res["ok"]
        assert abs(rows[1]["max_abs_err"] - 1e-2) < 1e-6
    else:
        assert res["ok"] and rows[1]["max_abs_err"] == 0.0


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
