"""Sharded decode on two GPUs over NCCL (one process per GPU).

Rank r owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and the q-heads that map to them
(kvx.shard.head_ranges).  Two paths are checked against the oracle's
unsharded append + paged GQA decode (oracle/kvx_oracle.c, restating
cache/kv_cache.cpp and runtime/cpu_ops.cpp), within the attention tolerance:

- kvx.decode on each rank's shard of the pool, outputs all-gathered with
  torch.distributed (NCCL) and reassembled with kvx.shard.gathered_to_heads;
- adaptive_engine_decode_step on each rank's shard through the C ABI with
  host buffers, the engine all-gathering each layer's output over its own
  NCCL communicator (adaptive_engine_set_comm), rank 0 reading the gathered
  rows back.

A third case makes rank 1's step fail on the host (the layer it must bring
to the device cannot evict a victim: both device slabs hold pinned layers):
rank 1 returns KVX_EBUSY and rank 0, whose own work succeeded, returns
KVX_EPEER; neither waits in NCCL, because the failing rank still takes every
collective step.  No GPU fault is involved, NVLS is off, and the process
group has a short timeout, so a rank that fails otherwise makes the other
one end with an error rather than wait.
"""
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RTOL, ATOL = 1e-3, 1e-2
HKV, HQ, DIM, PT = 8, 24, 128, 16


def _worker(rank, world, port, tmpdir, result_q, mode):
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests"),
                    os.path.join(ROOT, "adaptive-hierarchical-llm-inference-engine_b200")]
    import datetime

    import torch
    import torch.distributed as dist

    import kvgen
    import kvx
    import kvx.engine as E
    from kvx.shard import gathered_to_heads, head_ranges
    from oracle import Oracle

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    report = {}
    api = None
    try:
        o = Oracle()
        (k0, k1), (q0, q1) = head_ranges(HKV, HQ, world, rank)

        if mode == "fail":
            report.update(_failing_step(rank, world, tmpdir, dist, E))
            dist.barrier()
            result_q.put((rank, report, None))
            return
        # kvx.decode per shard + torch NCCL all-gather
        lens = np.array([1, 17, 300, 1000, 64], np.int32)
        bt, num_pages = kvgen.paged_layout(lens, PT, 0, seed=21)
        pool = kvgen.normal(22, (num_pages, 2, HKV, PT, DIM)).astype(np.float16)
        q = kvgen.normal(23, (lens.size, HQ, DIM)).astype(np.float16)
        dev = torch.device("cuda", rank)
        shard = torch.from_numpy(np.ascontiguousarray(pool[:, :, k0:k1])).to(dev)
        local = kvx.decode(shard, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev),
                           torch.from_numpy(np.ascontiguousarray(q[:, q0:q1])).to(dev))
        gathered = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=dev)
        dist.all_gather_into_tensor(gathered, local)
        full = gathered_to_heads(gathered).float().cpu().numpy()
        ref = o.paged_decode(pool, bt, lens, q.astype(np.float32))
        report["kvx_excess"] = float((np.abs(full - ref) - (ATOL + RTOL * np.abs(ref))).max())

        # the engine's decode step, NCCL inside the engine
        layers, pages, batch = 3, 48, 3
        api = E.api()
        api.stop()
        E.configure(layers=layers, pages_per_layer=pages, max_batch=batch, gpu_layer_slots=layers,
                    kv_heads=HKV // world, q_heads=HQ // world, device=rank,
                    offload_dir=os.path.join(tmpdir, f"rank{rank}"))
        api.start()
        uid = [E.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        E.set_comm(rank, world, uid[0])
        elens = np.array([5, 130, 255], np.int32)
        E.set_sequences(elens, reserve_tokens=4, seed=3)
        ebt = E.block_table(batch)
        pools = [kvgen.normal(40 + l, (pages, 2, HKV, PT, DIM)).astype(np.float16)
                 for l in range(layers)]
        for l in range(layers):
            E.load_layer(l, np.ascontiguousarray(pools[l][:, :, k0:k1]))
        eq = kvgen.normal(50, (layers, batch, HQ, DIM)).astype(np.float16)
        ek = kvgen.normal(51, (layers, batch, HKV, DIM)).astype(np.float16)
        ev = kvgen.normal(52, (layers, batch, HKV, DIM)).astype(np.float16)
        out = np.zeros((layers, world, batch, HQ // world, DIM), np.float16) if rank == 0 else None
        E.decode_step(np.ascontiguousarray(eq[:, :, q0:q1]), np.ascontiguousarray(ek[:, :, k0:k1]),
                      np.ascontiguousarray(ev[:, :, k0:k1]), out)
        if rank == 0:
            worst = -np.inf
            for l in range(layers):
                o.append(pools[l], ebt, elens, ek[l], ev[l], PT)
                eref = o.paged_decode(pools[l], ebt, elens + 1, eq[l].astype(np.float32))
                got = gathered_to_heads(out[l]).astype(np.float32)
                worst = max(worst, float((np.abs(got - eref) - (ATOL + RTOL * np.abs(eref))).max()))
            report["engine_excess"] = worst
        dist.barrier()
        result_q.put((rank, report, None))
    except Exception as e:  # reported to the parent, never hangs
        result_q.put((rank, report, type(e).__name__ + ": " + str(e)[:300]))
    finally:
        try:
            if api is not None:
                api.stop()
            dist.destroy_process_group()
        except Exception:
            pass


def _failing_step(rank, world, tmpdir, dist, E):
    """Rank 1 keeps 2 of its 3 layers on the device, both pinned, so bringing
    layer 2 back fails (KVX_EBUSY) in the middle of the step."""
    layers, pages, batch = 3, 16, 2
    api = E.api()
    api.stop()
    E.configure(layers=layers, pages_per_layer=pages, max_batch=batch,
                gpu_layer_slots=layers if rank == 0 else 2, kv_heads=HKV // world,
                q_heads=HQ // world, device=rank, offload_dir=os.path.join(tmpdir, f"f{rank}"))
    api.start()
    try:
        uid = [E.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        E.set_comm(rank, world, uid[0])
        E.set_sequences(np.array([20, 7], np.int32), reserve_tokens=2, seed=1)
        if rank == 1:
            assert api.keepLayer(0) >= 1 and api.keepLayer(1) >= 1
        hq, hkv = HQ // world, HKV // world
        q = np.zeros((layers, batch, hq, DIM), np.float16)
        kv = np.zeros((layers, batch, hkv, DIM), np.float16)
        out = np.zeros((layers, world, batch, hq, DIM), np.float16) if rank == 0 else None
        status = 0
        try:
            E.decode_step(q, kv, kv, out)
        except E.KvxError as e:
            status = e.status
        if rank == 1:
            for l in (0, 1):
                E.lib.adaptive_engine_test_release_layer(l)
        return {"status": status}
    finally:
        api.stop()


def _spawn(tmp_path, mode):
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), q, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    return res


def _need_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")


def test_two_gpu_sharded_decode_matches_oracle(tmp_path):
    _need_two_gpus()
    res = _spawn(tmp_path, "parity")
    for rank, report, err in res:
        assert err is None, (rank, err)
        assert report["kvx_excess"] <= 0, (rank, report)
    assert res[0][1]["engine_excess"] <= 0, res[0][1]


def test_failing_rank_does_not_hang_its_peer(tmp_path):
    _need_two_gpus()
    res = _spawn(tmp_path, "fail")
    for rank, report, err in res:
        assert err is None, (rank, err)
    assert res[1][1]["status"] == -2, res   # KVX_EBUSY: victims pinned
    assert res[0][1]["status"] == -9, res   # KVX_EPEER
