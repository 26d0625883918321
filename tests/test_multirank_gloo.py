"""Sharded decode across ranks (host logic on CPU, gloo backend, 2 ranks).

Each rank restricts the pool and the queries to its KV-head shard
(kvx.shard.head_ranges), decodes its heads with the oracle, all-gathers the
outputs and reassembles them (kvx.shard.gathered_to_heads); the result must
equal the unsharded decode bit for bit (the oracle is deterministic per
head).  A rank that fails before the collective makes the others time out
with an error instead of hanging.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, result_q, fail_rank):
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests"),
                    os.path.join(ROOT, "adaptive-hierarchical-llm-inference-engine_b200")]
    import datetime

    import torch
    import torch.distributed as dist

    import kvgen
    from kvx.shard import gathered_to_heads, head_ranges
    from oracle import Oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        o = Oracle()
        lens = np.array([3, 40, 17], np.int32)
        bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=9)
        pool = kvgen.normal(10, (num_pages, 2, 8, 16, 128)).astype(np.float16)
        q = kvgen.normal(11, (3, 24, 128))
        (k0, k1), (q0, q1) = head_ranges(8, 24, world, rank)
        local = o.paged_decode(np.ascontiguousarray(pool[:, :, k0:k1]), bt, lens, q[:, q0:q1])
        t = torch.from_numpy(local)
        out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype)
        dist.all_gather_into_tensor(out, t)
        full = gathered_to_heads(out.view((world,) + tuple(t.shape))).numpy()
        ref = o.paged_decode(pool, bt, lens, q)
        result_q.put((rank, bool(np.array_equal(full, ref)), None))
    except Exception as e:  # reported to the parent, never hangs
        result_q.put((rank, False, type(e).__name__ + ": " + str(e)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return sorted(res)


def test_two_rank_sharded_decode_equals_unsharded():
    res = _run(2)
    assert all(ok for _, ok, _ in res), res


def test_rank_failure_is_reported_not_hung():
    res = _run(2, fail_rank=1)
    assert res[1][1] is False and "injected" in res[1][2]
    assert res[0][1] is False  # the surviving rank's collective errors out (timeout)


def test_head_ranges_cover_all_heads():
    from kvx.shard import head_ranges
    for world in (1, 2, 4, 8):
        kv, qh = set(), set()
        for r in range(world):
            (a, b), (c, d) = head_ranges(8, 64, world, r)
            kv |= set(range(a, b))
            qh |= set(range(c, d))
            assert all(h // 8 in range(a, b) for h in range(c, d))  # GQA group stays local
        assert kv == set(range(8)) and qh == set(range(64))
    with pytest.raises(ValueError):
        head_ranges(8, 24, 3, 0)
