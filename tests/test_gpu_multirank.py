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

A third case runs the engine at 28 layers (grouped all-gathers, contexts
split over several CTAs) with the read-back first on rank 0, then shared
between the ranks.  A fourth makes rank 1's step fail on the host (the layer it must bring
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
        if mode == "engine28":
            report.update(_engine_28_layers(rank, world, tmpdir, dist, E, o, (k0, k1), (q0, q1)))
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


def _engine_28_layers(rank, world, tmpdir, dist, E, o, kr, qr):
    """adaptive_engine_decode_step at 28 layers on two GPUs: layer groups of
    2, 7, 7, 7, 3 and 2, one all-gather per group, contexts up to 5,000
    tokens (several splits).  Step 0: rank 0 reads every layer back; step 1:
    the read-back shared (rank r copies layers l % 2 == r).  Each rank checks
    what it read against the oracle's unsharded append + decode."""
    import kvgen
    from kvx.shard import gathered_to_heads
    (k0, k1), (q0, q1) = kr, qr
    L, B = 28, 3
    lens = np.array([5000, 2100, 777], np.int32)
    pages = int(((lens + 2 + PT - 1) // PT).sum())
    api = E.api()
    api.stop()
    E.configure(layers=L, pages_per_layer=pages, max_batch=B, gpu_layer_slots=L, kv_heads=HKV // world,
                q_heads=HQ // world, device=rank, offload_dir=os.path.join(tmpdir, f"e28_{rank}"))
    api.start()
    try:
        uid = [E.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        E.set_comm(rank, world, uid[0])
        E.set_sequences(lens, reserve_tokens=2, seed=7)
        bt = E.block_table(B)
        keep = {}
        for l in range(L):
            pool = kvgen.normal(300 + l, (pages, 2, HKV, PT, DIM)).astype(np.float16)
            E.load_layer(l, np.ascontiguousarray(pool[:, :, k0:k1]))
            if rank == 0 or l % world == rank:
                keep[l] = pool
        q = kvgen.normal(330, (2, L, B, HQ, DIM)).astype(np.float16)
        k = kvgen.normal(331, (2, L, B, HKV, DIM)).astype(np.float16)
        v = kvgen.normal(332, (2, L, B, HKV, DIM)).astype(np.float16)
        shape = (L, world, B, HQ // world, DIM)
        out = [np.zeros(shape, np.float16) if rank == 0 else None, np.zeros(shape, np.float16)]
        for step in range(2):
            if step == 1:
                E.set_readback_share(True)
            E.decode_step(np.ascontiguousarray(q[step][:, :, q0:q1]), np.ascontiguousarray(k[step][:, :, k0:k1]),
                          np.ascontiguousarray(v[step][:, :, k0:k1]), out[step])
        E.set_readback_share(False)
        worst, checked = -np.inf, 0
        for l, pool in sorted(keep.items()):
            for step in range(2):
                pos = (lens + step).astype(np.int32)
                o.append(pool, bt, pos, k[step][l], v[step][l], PT)
                mine = (rank == 0) if step == 0 else (l % world == rank)
                if not mine:
                    continue
                ref = o.paged_decode(pool, bt, pos + 1, q[step][l].astype(np.float32))
                got = gathered_to_heads(out[step][l]).astype(np.float32)
                worst = max(worst, float((np.abs(got - ref) - (ATOL + RTOL * np.abs(ref))).max()))
                checked += 1
        if rank != 0:  # layers rank 1 does not read stay untouched
            assert not out[1][[l for l in range(L) if l % world != rank]].any()
        return {"engine28_excess": worst, "engine28_checked": checked}
    finally:
        api.stop()


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


def test_two_gpu_engine_28_layers_grouped_gathers_and_shared_read_back(tmp_path):
    _need_two_gpus()
    res = _spawn(tmp_path, "engine28")
    for rank, report, err in res:
        assert err is None, (rank, err)
        assert report["engine28_excess"] <= 0, (rank, report)
    assert res[0][1]["engine28_checked"] == 28 + 14 and res[1][1]["engine28_checked"] == 14, res


def test_failing_rank_does_not_hang_its_peer(tmp_path):
    _need_two_gpus()
    res = _spawn(tmp_path, "fail")
    for rank, report, err in res:
        assert err is None, (rank, err)
    assert res[1][1]["status"] == -2, res   # KVX_EBUSY: victims pinned
    assert res[0][1]["status"] == -9, res   # KVX_EPEER


def test_one_process_decodes_on_two_devices(oracle):
    """The kernels that need more than 48 KB of shared memory (fp16 and int8
    tensor-core decode, dense attention) set that attribute per device: a
    process that decodes on device 0 and then on device 1 gets the oracle's
    result on both."""
    _need_two_gpus()
    sys.path[:0] = [os.path.join(ROOT, "tests"), os.path.join(ROOT, "adaptive-hierarchical-llm-inference-engine_b200")]
    import kvgen
    import kvx
    lens = np.array([900, 4096, 33], np.int32)
    bt, num_pages = kvgen.paged_layout(lens, PT, 0, seed=401)
    pool = kvgen.normal(402, (num_pages, 2, HKV, PT, DIM)).astype(np.float16)
    q = kvgen.normal(403, (lens.size, HQ, DIM)).astype(np.float16)
    ref = oracle.paged_decode(pool, bt, lens, q.astype(np.float32))
    qd_, kd_ = kvgen.normal(404, (300, DIM)), kvgen.normal(405, (700, DIM))
    vd_ = kvgen.normal(406, (700, DIM))
    for dev in (0, 1):
        with torch.cuda.device(dev):
            d = torch.device("cuda", dev)
            got = kvx.decode(torch.from_numpy(pool).to(d), torch.from_numpy(bt).to(d), torch.from_numpy(lens).to(d),
                             torch.from_numpy(q).to(d)).float().cpu().numpy()
            assert (np.abs(got - ref) - (ATOL + RTOL * np.abs(ref))).max() <= 0, dev
            codes, stats = kvx.compress_int8(torch.from_numpy(pool).to(d))
            cpool = codes.view(num_pages, 2, HKV, PT, DIM)
            got8 = kvx.decode(cpool, torch.from_numpy(bt).to(d), torch.from_numpy(lens).to(d),
                              torch.from_numpy(q).to(d), stats=stats).float().cpu().numpy()
            ref8 = oracle.paged_decode(codes.cpu().numpy().reshape(cpool.shape), bt, lens, q.astype(np.float32),
                                       stats=stats.cpu().numpy().reshape(num_pages, 2, HKV, 4))
            assert (np.abs(got8 - ref8) - (ATOL + RTOL * np.abs(ref8))).max() <= 0, dev
            att = kvx.attention_dense(torch.from_numpy(qd_).float().to(d), torch.from_numpy(kd_).float().to(d),
                                      torch.from_numpy(vd_).float().to(d)).cpu().numpy()
            s = qd_ @ kd_.T / np.sqrt(DIM)
            p = np.exp(s - s.max(1, keepdims=True))
            want = (p / p.sum(1, keepdims=True)) @ vd_
            assert np.abs(att - want).max() <= 1e-4 * max(1.0, np.abs(want).max()), dev
