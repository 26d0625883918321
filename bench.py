"""Benchmark: batched fragmented paged decode (the KV-cache hot path).

Workload (one step): for each of 28 layers of Llama-3.2-3B KV geometry
(8 KV heads x 128, fp16, 24 q-heads, GQA group 3) and batch 32 with context
lengths U[512, 8192] (seeded) and randomly permuted physical pages, append
one token per sequence into its page, then run paged GQA decode attention
over the whole context.  Metric: KV bytes read by decode per second (GB/s),
whole job.  With --gpus N the KV heads are sharded over N ranks (each rank
owns 8/N heads and the matching q-heads, for all sequences) and the
attention outputs are all-gathered over NCCL each layer; the batch grows to
32*N sequences so every GPU reads the same bytes per step (weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "adaptive-hierarchical-llm-inference-engine_b200")
for _p in (PKG, os.path.join(ROOT, "tests"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import kvgen  # noqa: E402

METRIC = "paged-decode KV GB/s"
LAYERS, HKV, HQ, DIM, PT, BATCH = 28, 8, 24, 128, 16, 32
CTX_LO, CTX_HI, SEED = 512, 8192, 20241201
WORKLOAD = "batched fragmented decode: Llama-3.2-3B KV (28L, 8kv x128, 24q), fp16, B32, ctx U[512,8192], permuted pages"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check after the timed region")
    ap.add_argument("--no-append-compress", action="store_true", help="skip the append / compressKv measurement")
    ap.add_argument("--no-config5", action="store_true", help="skip the 70B-geometry workload")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers per step (profiling of a smaller case; the metric is defined at 28)")
    ap.add_argument("--pages", type=int, default=1 << 20,
                    help="config 3: pages compressed (1,048,576 defines the configuration; fewer for profiling)")
    ap.add_argument("--tier-context", type=int, default=65536,
                    help="config 4: tokens per sequence (65,536 defines the configuration)")
    ap.add_argument("--tier-device-gb", type=float, default=40.0, help="config 4: device pool cap")
    ap.add_argument("--tier-ram-gb", type=float, default=0.0,
                    help="config 4: RAM tier size (0: every non-resident frame in pinned RAM; "
                         "else the rest go to a spill file, the disk tier)")
    ap.add_argument("--tier-host-policy", action="store_true",
                    help="config 4: the LRU bookkeeping on the host (kvx_tier_step) instead of as kernels on the "
                         "device (kvx_tier_step_device, the default: the step's ids go up, the block tables come "
                         "out of the policy, no host planning)")
    ap.add_argument("--tier-prefetch", action="store_true",
                    help="config 4: plan and load per layer, the Scheduler's prefetch depth (kvx_scheduler_depth, "
                         "fed each plan's load latency) deciding how many layers ahead of the decode")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5],
                    help="2: the headline workload; 1, 3, 5: the other configurations of the path")
    ap.add_argument("--kernels", action="store_true",
                    help="time every kernel the headline line does not (one JSON line each; ncu target)")
    ap.add_argument("--kernel-iters", type=int, default=10, help="with --kernels: timed launches per kernel")
    ap.add_argument("--shapes", action="store_true",
                    help="decode across batch x context shapes (fp16, int8 and fp32 pools, GQA 3 and 8), "
                         "one JSON line per shape")
    ap.add_argument("--shape-pools", default="fp16,int8,fp32",
                    help="with --shapes: which pool kinds to run (comma-separated)")
    ap.add_argument("--shape-chunks", default="",
                    help="with --shapes: comma-separated chunk sizes (pages per CTA) to time beside "
                         "the library's own choice, forced through KVX_DECODE_CHUNK")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def workload_lens(batch=BATCH):
    # the first 32 values of the stream are the same for every batch size
    return kvgen.randint(SEED, batch, CTX_LO, CTX_HI).astype(np.int64)


# --------------------------------------------------------------------------
GROUP = 7      # layers per all-gather group (N > 1)
OUT_RING = 8   # output buffers an N > 1 run rotates through


def make_decode_step(kvx, views, bt, positions, nk, nv, q, ws, err, outs, world=1, comm=None, dist=None,
                     group=GROUP):
    """The timed step.  step(k) appends, for every layer l, the token at
    positions[k] (rows nk[l] / nv[l]) and decodes over positions[k] + 1
    tokens into outs[k % len(outs)][l]: one kvx.append_decode launch per
    layer, all on the current stream with nothing in between, so each launch
    may start while the previous one drains (programmatic dependent launch);
    the layers share one decode workspace.

    With world > 1 the layers' outputs are all-gathered (NCCL) on `comm`,
    one all-gather per group of `group` layers (a group's rows are
    contiguous): step.gathered[g] is [world][layers of g][batch][hq][128],
    step.gathered_rows(l, r) rank r's rows of layer l.  The last launch of a
    group signals its completion (kvx_append_decode_signal: the last CTA
    stores the step's epoch) and `comm` waits for that word
    (kvx_stream_wait_geq) before the group's all-gather, so no event sits
    between two decode launches.
    Outputs rotate through len(outs) buffers; every len(outs) - 1 steps the
    compute stream waits for the all-gathers of two steps back, the only
    point where it waits for `comm`."""
    import torch
    L = len(views)
    R = len(outs)
    main = torch.cuda.current_stream()
    ngroups = (L + group - 1) // group
    done = torch.zeros((ngroups, 2), dtype=torch.int32, device=bt.device) if world > 1 else None
    gathered = [torch.empty((world, min(L, g0 + group) - g0) + tuple(outs[0].shape[1:]), device=bt.device,
                            dtype=outs[0].dtype) for g0 in range(0, L, group)] if world > 1 else None
    gathers_done = [torch.cuda.Event() for _ in range(R)] if world > 1 else None
    sync = "stream memory wait on the group's completion word"
    if world > 1:
        try:
            kvx.stream_wait_geq(done[0, 1:], 0, stream=comm)  # satisfied at once
        except kvx.KvxError:
            sync = "event per group (no stream memory operations)"
    assert world == 1 or R >= 3, "the output ring needs at least 3 buffers"

    def gather(gi, out):
        l0 = gi * group
        dst = gathered[gi]
        dist.all_gather_into_tensor(dst.view((-1,) + tuple(dst.shape[2:])), out[l0:l0 + dst.shape[1]])

    def step(k):
        out = outs[k % R]
        if world > 1 and k >= 2 and k % (R - 1) == 0:
            # steps k .. k + R - 2 reuse buffers whose all-gathers ran at
            # steps up to k - 2
            main.wait_event(gathers_done[(k - 2) % R])
        for l in range(L):
            last_of_group = world > 1 and (l % group == group - 1 or l == L - 1)
            if last_of_group and sync.startswith("stream"):
                gi = l // group
                kvx.append_decode_signal(views[l], bt, positions[k], nk[l], nv[l], q[l], done[gi], k + 1,
                                         out=out[l], workspace=ws, error_flag=err)
                with torch.cuda.stream(comm):
                    kvx.stream_wait_geq(done[gi, 1:], k + 1, stream=comm)
                    gather(gi, out)
            else:
                kvx.append_decode(views[l], bt, positions[k], nk[l], nv[l], q[l], out=out[l], workspace=ws,
                                  error_flag=err)
                if last_of_group:
                    ev = torch.cuda.Event()
                    ev.record()
                    with torch.cuda.stream(comm):
                        comm.wait_event(ev)
                        gather(l // group, out)
        if world > 1:
            gathers_done[k % R].record(comm)

    step.gather_sync = sync
    step.gathered = gathered
    step.gathered_rows = (lambda l, r: gathered[l // group][r, l % group]) if world > 1 else None
    return step


class ParitySample:
    """An oracle check of the timed run, outside the timed region: for a
    seeded sample of layers and sequences, the pages as they were before the
    first step are copied to the host; afterwards the oracle appends every
    step's rows to them (KVManager::save_page semantics,
    cache/kv_cache.cpp:111-127), the result must equal the device pages bit
    for bit, and the oracle's decode over the final context
    (TensorOps::attention, runtime/tensor_ops.cpp:179-219) must match this
    rank's rows of the last step within 1e-3 relative / 1e-2 absolute.
    With several ranks every rank checks its own KV heads, and the gathered
    buffer's slot of each rank must equal that rank's local rows bit for bit
    (compared through per-rank checksums); the figures are reduced over the
    ranks."""
    RTOL, ATOL = 1e-3, 1e-2

    def __init__(self, bt_np, lens0, hkv, hq, world, rank, views, layers=None, seqs=4):
        import torch
        self.bt, self.lens0, self.hkv, self.hq, self.world, self.rank = bt_np, lens0, hkv, hq, world, rank
        L = len(views)
        self.layers = sorted({0, L // 2, L - 1} if layers is None else set(layers))
        rng = np.random.default_rng(SEED + 99)
        self.seqs = np.sort(rng.choice(len(lens0), size=min(seqs, len(lens0)), replace=False))
        self.views = views
        self.before = {}
        for l in self.layers:
            pool = self._pool(views[l])
            for s in self.seqs:
                pages = self.bt[s][self.bt[s] >= 0]
                self.before[(l, s)] = pool[torch.from_numpy(pages.astype(np.int64)).cuda()].cpu().numpy()

    @staticmethod
    def _pool(view):
        if not hasattr(view, "num_pages"):  # already a tensor
            return view
        from kvx import pool_tensor
        return pool_tensor(view)

    def verify(self, q, nk, nv, positions, last_out, gathered_rows, dist):
        """positions: [steps][batch] (host or device) -- every step's append
        position per sequence, in order; last_out: this rank's rows of the
        last step; gathered_rows(l, r): rank r's rows of layer l in the
        gathered buffer (several ranks)."""
        import torch
        from oracle import Oracle
        o = Oracle()
        positions = positions.cpu().numpy() if hasattr(positions, "cpu") else np.asarray(positions)
        total_steps = positions.shape[0]
        rows = 0
        excess = -np.inf
        pool_ok = True
        for l in self.layers:
            pool = self._pool(self.views[l])
            k_l, v_l, q_l = nk[l].cpu().numpy(), nv[l].cpu().numpy(), q[l].float().cpu().numpy()
            for s in self.seqs:
                pages = self.bt[s][self.bt[s] >= 0]
                host = self.before[(l, s)].copy()
                bt1 = np.arange(pages.size, dtype=np.int32)[None, :]
                for k in range(total_steps):
                    pos = positions[k, s:s + 1].astype(np.int32)
                    o.append(host, bt1, pos, k_l[s:s + 1], v_l[s:s + 1], 16)
                dev = pool[torch.from_numpy(pages.astype(np.int64)).cuda()].cpu().numpy()
                pool_ok = pool_ok and np.array_equal(dev.view(np.uint16), host.view(np.uint16))
                T = positions[-1, s:s + 1].astype(np.int32) + 1
                ref = o.paged_decode(host, bt1, T, q_l[s:s + 1])
                got = last_out[l, s:s + 1].float().cpu().numpy()
                excess = max(excess, float((np.abs(got - ref) - (self.ATOL + self.RTOL * np.abs(ref))).max()))
                rows += self.hq
        gather_mismatch = 0
        if dist is not None:
            # this rank's local rows of the last step and every rank's slot of
            # the gathered buffer, compared as checksums of the raw bits
            def csum(t):
                return int(t.contiguous().view(torch.int16).to(torch.int64).sum().item())
            nl, B = last_out.shape[0], last_out.shape[1]
            mine = torch.tensor([csum(last_out[l]) for l in range(nl)], dtype=torch.int64, device="cuda")
            every = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(every, mine)
            for l in range(nl):
                for r in range(self.world):
                    if csum(gathered_rows(l, r)) != every[r][l].item():
                        gather_mismatch += 1
            t = torch.tensor([excess, float(rows), 0.0 if pool_ok else 1.0, float(gather_mismatch)],
                             dtype=torch.float64, device="cuda")
            mx, sm = t.clone(), t.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            dist.all_reduce(sm, op=dist.ReduceOp.SUM)
            excess, rows, pool_ok = mx[0].item(), int(sm[1].item()), mx[2].item() == 0
            gather_mismatch = int(sm[3].item())
        return {"ok": bool(pool_ok and excess <= 0 and gather_mismatch == 0), "rows_checked": rows,
                "max_excess": round(excess, 6), "tolerance": "|gpu - oracle| <= 1e-2 + 1e-3 |oracle|",
                "pool_pages_bitexact": bool(pool_ok), "gather_slot_mismatches": gather_mismatch,
                "sample": f"layers {list(self.layers)} x sequences {list(map(int, self.seqs))} per rank "
                          f"(all {self.hq} local q-heads), {total_steps} appends each",
                "oracle": "C restatement of the reference's save_page + TensorOps::attention"}


# --------------------------------------------------------------------------
APPEND_CHUNK = 256      # tokens each sequence appends per layer in the append measurement
COMPRESS_PAGES = 1 << 20  # the compressKv sweep's pages (16 tokens x 8 KV heads x 128, fp16)


def _max_over_ranks(ms, dist):
    import torch
    if dist is None:
        return ms
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def _timed_events(fn, iters, warm=3):
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def run_append_compress(world, rank, hkv, dist=None, compress_pages=COMPRESS_PAGES, layers=None, check=True):
    """The metric's second half: append tokens/s and compressKv tokens/s.

    Append (KVManager::save_page per token, cache/kv_cache.cpp:111-127): each
    of 32 x N sequences appends a chunk of 256 tokens, starting at a seeded
    offset inside a page, into every one of the 28 layers' pools (this rank's
    KV heads, randomly permuted pages); one kvx_append_chunk launch per layer.
    A token is one sequence position of one layer (its K and V rows of every
    KV head, split over the ranks), so the job's tokens grow with N (weak
    scaling, as the decode).  Bytes per token and rank: 2 x hkv x 256 B read
    and the same written.

    Compress (KVCompressionEngine::compressToINT8, native-engine/cpp/
    KVCompressionEngine.cpp:83-113, one call per (page, head) block of 2048
    elements): the 1,048,576 pages x 16 tokens x 8 KV heads x 128 fp16 of the
    compressKv sweep (N(0,1), 1% of elements x20), each rank compressing its
    8/N heads of every page (strong scaling: the job is fixed).  A token is
    one of the 16 rows of a page.  Bytes per (page, head) block: 4 KiB read,
    2 KiB + 16 B written.

    Both are timed with CUDA events over several launches (max over ranks)
    and checked against the oracle on a sample: appended pages bit for bit,
    codes and QuantizationStats bit for bit."""
    import torch
    import kvx
    L = LAYERS if layers is None else layers
    peak, peak_kind = peaks()
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 31 + rank)
    res = {}
    # ---- append
    B, n = BATCH * world, APPEND_CHUNK
    slices = n // PT + 1
    starts_np = kvgen.randint(SEED + 32, B, 0, PT - 1).astype(np.int32)
    pages = B * slices
    perm = kvgen.permutation(SEED + 33, pages).astype(np.int32)
    bt_np = perm.reshape(B, slices)
    bt = torch.from_numpy(bt_np).cuda()
    starts = torch.from_numpy(starts_np).cuda()
    pools = [torch.zeros((pages, 2, hkv, PT, DIM), device="cuda", dtype=torch.float16) for _ in range(L)]
    rows_k = [torch.randn((B, n, hkv, DIM), generator=g, device="cuda", dtype=torch.float16) for _ in range(L)]
    rows_v = [torch.randn((B, n, hkv, DIM), generator=g, device="cuda", dtype=torch.float16) for _ in range(L)]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")

    def append_all():
        for l in range(L):
            kvx.append_chunk(pools[l], bt, starts, rows_k[l], rows_v[l], error_flag=err)

    if dist is not None:
        dist.barrier()
    ms = _max_over_ranks(_timed_events(append_all, 10), dist)
    tok_rank_bytes = 2 * hkv * DIM * 2 * 2  # K and V rows read + written
    launch_ms = ms / L
    per_launch_bytes = B * n * tok_rank_bytes
    app = {"tokens_per_s": round(B * n * L / (ms / 1e3), 1), "unit": "tokens/s",
           "token": "one sequence position of one layer (K and V rows of all 8 KV heads, over the ranks)",
           "sequences": B, "chunk_tokens": n, "layers": L, "ms_per_step": round(ms, 4),
           "scaling": "weak (32 sequences per GPU)",
           "roofline": {"bound": "hbm", "achieved": round(per_launch_bytes / (launch_ms / 1e3) / 1e9, 1),
                        "peak": peak, "unit": "GB/s", "peak_kind": peak_kind,
                        "frac": round(per_launch_bytes / (launch_ms / 1e3) / 1e9 / peak, 4),
                        "kernel": "append_chunk_kernel", "mean_launch_us": round(launch_ms * 1e3, 2),
                        "bytes_per_launch": per_launch_bytes}}
    assert err.item() == 0, f"append error flag {err.item()}"
    if check:
        from oracle import Oracle
        o = Oracle()
        host = np.zeros((pages, 2, hkv, PT, DIM), np.float16)
        rk, rv = rows_k[0].cpu().numpy(), rows_v[0].cpu().numpy()
        for t in range(n):
            o.append(host, bt_np, starts_np + t, rk[:, t], rv[:, t], 16)
        app["parity"] = {"layer0_pool_bitexact": bool(np.array_equal(pools[0].cpu().numpy().view(np.uint16),
                                                                     host.view(np.uint16))),
                         "oracle": "KVManager::save_page per token (C restatement)"}
    del pools, rows_k, rows_v
    torch.cuda.empty_cache()
    res["append"] = app
    # ---- compress: this rank's KV heads of every page, [pages][hkv] blocks
    blocks = compress_pages * hkv
    x = torch.empty((blocks, PT * DIM), device="cuda", dtype=torch.float16)
    for c in range(0, blocks, 1 << 20):
        part = torch.randn((min(1 << 20, blocks - c), PT * DIM), generator=g, device="cuda")
        part[torch.rand(part.shape, generator=g, device="cuda") < 0.01] *= 20.0
        x[c:c + part.shape[0]] = part.half()
        del part
    codes = torch.empty((blocks, PT * DIM), device="cuda", dtype=torch.int8)
    stats = torch.empty((blocks, 4), device="cuda", dtype=torch.float32)
    if dist is not None:
        dist.barrier()
    ms = _max_over_ranks(_timed_events(lambda: kvx.compress_int8(x, codes=codes, stats=stats), 5), dist)
    nbytes = blocks * (PT * DIM * 3 + 16)
    comp = {"tokens_per_s": round(compress_pages * PT / (ms / 1e3), 1), "unit": "tokens/s",
            "token": "one of a page's 16 rows (8 KV heads x 128 fp16, over the ranks)",
            "pages": compress_pages, "blocks_per_gpu": blocks, "ms": round(ms, 4),
            "scaling": "strong (the 1,048,576 pages split by KV head)",
            "roofline": {"bound": "hbm", "achieved": round(nbytes / (ms / 1e3) / 1e9, 1), "peak": peak,
                         "unit": "GB/s", "peak_kind": peak_kind,
                         "frac": round(nbytes / (ms / 1e3) / 1e9 / peak, 4), "kernel": "compress_2048_kernel",
                         "bytes_per_launch": nbytes}}
    if check:
        from oracle import Oracle
        o = Oracle()
        pick = np.sort(np.random.default_rng(SEED + 34).choice(blocks, size=64, replace=False))
        idx = torch.from_numpy(pick).cuda()
        rc, rs = o.compress_int8_blocks(x[idx].cpu().numpy(), PT * DIM)
        comp["parity"] = {"blocks_checked": int(pick.size),
                          "codes_bitexact": bool(np.array_equal(codes[idx].cpu().numpy().ravel(), rc.ravel())),
                          "stats_bitexact": bool(np.array_equal(stats[idx].cpu().numpy().view(np.uint32).ravel(),
                                                                rs.view(np.uint32).ravel())),
                          "oracle": "KVCompressionEngine::compressToINT8 per block (C restatement)"}
    del x, codes, stats
    torch.cuda.empty_cache()
    res["compress"] = comp
    return res


# --------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    import kvx
    import kvx.engine as E

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    assert HKV % world == 0, "KV heads must divide evenly over the GPUs"
    hkv, hq = HKV // world, HQ // world
    B = BATCH * world
    steps, warm = args.steps, args.warmup
    total_steps = steps + warm

    # the engine owns the paged KV cache: one fp16 pool per layer, this
    # rank's KV heads, sequences with seeded lengths and permuted pages
    lens0 = workload_lens(B)
    reserve = max(total_steps, E2E_WARM + E2E_MAX_STEPS + 1)  # the e2e pass appends after the timed steps
    need_pages = int(((lens0 + reserve + PT - 1) // PT).sum())
    # the RAM and int8 tiers' slabs are made by start(): four of each (the
    # layer moves below use layer 0)
    E.configure(layers=LAYERS, kv_heads=hkv, q_heads=hq, max_batch=B, pages_per_layer=need_pages,
                gpu_layer_slots=LAYERS, device=local, ram_layer_slots=4, int8_layer_slots=4)
    api = E.api()
    api.start()
    E.set_sequences(lens0.astype(np.int32), reserve_tokens=reserve, seed=SEED + 1)
    bt_np = E.block_table(B)
    max_pages = bt_np.shape[1]
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 17 * rank)
    for l in range(LAYERS):  # N(0,1) fp16 context, generated on the device
        E.load_layer(l, torch.randn((need_pages, 2, hkv, PT, DIM), generator=g, device="cuda",
                                    dtype=torch.float16))
    views = [E.layer_view(l) for l in range(LAYERS)]
    bt = torch.from_numpy(bt_np).cuda()
    q = torch.randn((LAYERS, B, hq, DIM), generator=g, device="cuda", dtype=torch.float16)
    nk = torch.randn((LAYERS, B, hkv, DIM), generator=g, device="cuda", dtype=torch.float16)
    nv = torch.randn((LAYERS, B, hkv, DIM), generator=g, device="cuda", dtype=torch.float16)
    ring = OUT_RING if world > 1 else 1
    outs = [torch.empty((LAYERS, B, hq, DIM), device="cuda", dtype=torch.float16) for _ in range(ring)]
    ws = kvx.decode_workspace(B, hq, max_pages)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # every step's positions up front: no kernel between two steps' launches
    positions = torch.from_numpy(np.stack([lens0 + k for k in range(total_steps)]).astype(np.int32)).cuda()
    comm = torch.cuda.Stream() if world > 1 else None
    main = torch.cuda.current_stream()
    # the parity sample: its pages as they are before the first step
    check = ParitySample(bt_np, lens0, hkv, hq, world, rank, views) if not args.no_parity else None
    step = make_decode_step(kvx, views, bt, positions, nk, nv, q, ws, err, outs, world=world,
                            comm=comm, dist=dist if world > 1 else None)

    def kv_bytes(lens_after):  # algorithmic K+V bytes decode reads for one layer
        return int(lens_after.sum()) * 2 * hkv * DIM * 2

    for k in range(warm):
        step(k)
    if world > 1:
        main.wait_stream(comm)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    t0.record()
    for k in range(warm, warm + steps):
        step(k)
    if world > 1:  # the last group's all-gathers belong to the timed work
        main.wait_stream(comm)
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    assert err.item() == 0, f"device error flag {err.item()}"
    parity = None
    if check is not None:  # outside the timed region, before anything else writes the pools
        last = outs[(total_steps - 1) % ring]
        parity = check.verify(q, nk, nv, positions, last, step.gathered_rows, dist if world > 1 else None)

    lens_timed = [lens0 + warm + k + 1 for k in range(steps)]
    rank_bytes = sum(kv_bytes(L) * LAYERS for L in lens_timed)
    t_max = ms
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_max = t.item()
    total_bytes = rank_bytes * world
    value = total_bytes / (t_max / 1e3) / 1e9

    # roofline of the decode kernel: algorithmic bytes per launch / mean launch time
    mean_layer_bytes = rank_bytes / (steps * LAYERS)
    qo_bytes = 2 * B * hq * DIM * 2 + B * max_pages * 4 + B * 4 + 2 * B * hkv * DIM * 2
    # launches overlap by design (each starts while the previous drains), so
    # a launch's duration is the timed region (CUDA events on the launching
    # stream) divided by the launches in it
    mean_dec_ms = ms / (steps * LAYERS)
    achieved = (mean_layer_bytes + qo_bytes) / (mean_dec_ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    traffic = None
    tp = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get("bytes_per_launch")
        except Exception:
            traffic = None

    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": round(t_max / steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded N(0,1) K/V/Q, seeded context lengths and page permutation)",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "batch": B, "batch_per_gpu_equiv": BATCH,
                   "kv_heads": HKV,
                   "q_heads": HQ, "head_dim": DIM, "page_tokens": PT,
                   "parallelism": f"kv-head shard x{world}" + (" + NCCL all-gather" if world > 1 else ""),
                   "l2": "inputs larger than L2 (KV pool ~17 GB)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_kind": peak_kind, "kernel": "tc_decode_kernel (append + decode + split combine fused)",
                     "mean_launch_us": round(mean_dec_ms * 1e3, 2),
                     "launch_duration": "timed region / launches (consecutive launches overlap)"},
        "gpu_launches": steps * LAYERS,
        "clocks": clk,
        "parity": parity,
    }
    if world > 1:
        result["config"]["gather_sync"] = step.gather_sync
    del outs, ws, check, step
    if not args.no_append_compress:
        result["append_compress"] = run_append_compress(world, rank, hkv, dist if world > 1 else None)
    if not args.no_e2e:
        result["e2e"], bufs = run_e2e(args, E, lens0, hq, hkv, world, rank, B)
        torch.cuda.synchronize()
        if world == 1:  # after everything timed: it rewrites layer 0
            result["engine_ops"] = run_engine_ops(api, need_pages * 2 * hkv * PT * DIM * 2, E, bufs)
    if world > 1:
        dist.barrier()
    api.stop()
    del views
    torch.cuda.empty_cache()
    if not args.no_config5:
        result["config5_70b"] = run_config5_sharded(args, world, rank, dist if world > 1 else None)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(sample_layers=LAYERS, min_seconds=10.0)
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_engine_ops(api, slab_bytes, E=None, bufs=None):
    """The NativeEngineApi layer moves (native-engine/llama_wrapper/
    llama_wrapper.cpp:220-433 in the reference, simulations there) on layer
    0 of the bench's engine: wall time of each blocking call, and its bytes
    per second for the moves that carry the whole layer.  The RAM and int8
    slabs were made by start(), so the first move to RAM costs what the
    later ones do.  Then a move during a decode step: compressKv(0) issued
    while a whole 28-layer step runs (the step waits for its kernels with the
    engine lock released; the move waits only for layer 0's group)."""
    import threading
    out = {"layer_bytes": int(slab_bytes)}
    if E is not None and bufs is not None:
        t0 = time.perf_counter()
        E.decode_step(*bufs)
        step_ms = (time.perf_counter() - t0) * 1e3
        done = {}
        th = threading.Thread(target=lambda: (E.decode_step(*bufs), done.setdefault("t", time.perf_counter())))
        th.start()
        while not E.lib.adaptive_engine_step_in_flight() and th.is_alive():
            pass
        t1 = time.perf_counter()
        rc = api.compressKv(0)
        t2 = time.perf_counter()
        th.join()
        out["compressKv_during_step"] = {
            "ms": round((t2 - t1) * 1e3, 3), "returned": int(rc), "step_alone_ms": round(step_ms, 3),
            "returned_before_step_end": bool(t2 < done.get("t", 0.0)),
            "step_end_after_move_ms": round((done.get("t", t2) - t2) * 1e3, 3)}
        assert api.moveKvToGpu(0) > 0
    for name, fn, moved in (("moveKvToRam_first", api.moveKvToRam, True), ("moveKvToGpu", api.moveKvToGpu, True),
                            ("moveKvToRam", api.moveKvToRam, True), ("moveKvToGpu_again", api.moveKvToGpu, True),
                            ("compressKv", api.compressKv, True), ("moveKvToGpu_from_int8", api.moveKvToGpu, True),
                            ("offloadKv", api.offloadKv, True), ("moveKvToGpu_from_file", api.moveKvToGpu, True)):
        t0 = time.perf_counter()
        rc = fn(0)
        ms = (time.perf_counter() - t0) * 1e3
        out[name] = {"ms": round(ms, 2), "returned": int(rc)}
        if moved and rc > 0:
            out[name]["GBps"] = round(slab_bytes / (ms / 1e3) / 1e9, 1)
    return out


E2E_WARM, E2E_MAX_STEPS = 3, 64


def run_e2e(args, E, lens0, hq, hkv, world, rank, B):
    """The same step through the engine's public C ABI with host buffers:
    adaptive_engine_decode_step copies every layer's q / new K / new V from
    pinned host memory, runs append + decode per layer, all-gathers the
    layer's attention output over NCCL when there are several GPUs, and
    copies the (gathered) outputs back, all inside the timed region (wall
    clock around the blocking call, max over ranks)."""
    import torch
    if world > 1:
        import torch.distributed as dist
        uid = [E.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        E.set_comm(rank, world, uid[0])
    steps = max(8, min(args.steps, E2E_MAX_STEPS))
    h_q = torch.randn((LAYERS, B, hq, DIM), dtype=torch.float16).pin_memory()
    h_k = torch.randn((LAYERS, B, hkv, DIM), dtype=torch.float16).pin_memory()
    h_v = torch.randn((LAYERS, B, hkv, DIM), dtype=torch.float16).pin_memory()
    # the gathered result comes back to the host once per step: with several
    # GPUs each rank reads back its share of the layers (l % N == rank) over
    # its own host link
    h_o = torch.empty((LAYERS, world, B, hq, DIM), dtype=torch.float16).pin_memory()
    if world > 1:
        E.set_readback_share(True)
    for _ in range(E2E_WARM):  # warm-up: the engine's sequences start at lens0
        E.decode_step(h_q, h_k, h_v, h_o)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    nbytes = 0
    t0 = time.perf_counter()
    for k in range(steps):
        E.decode_step(h_q, h_k, h_v, h_o)
        nbytes += int((lens0 + E2E_WARM + 1 + k).sum()) * 2 * hkv * DIM * 2 * LAYERS
    secs = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([secs], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = t.item()
    return ({"value": round(nbytes * world / secs / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": int(h_q.numel() * 2 + h_k.numel() * 2 + h_v.numel() * 2),
            "d2h_bytes_per_step": LAYERS * world * B * hq * DIM * 2, "steps": steps,
            "path": "adaptive_engine_decode_step (C ABI) with pinned host buffers" +
                    (", NCCL all-gather of outputs in the engine, each rank reading back its share of the "
                     "gathered layers (d2h bytes summed over ranks)" if world > 1 else "")},
            (h_q, h_k, h_v, h_o))


# --------------------------------------------------------------------------
def cpu_baseline(sample_layers=1, min_seconds=0.0, max_layers=4 * LAYERS):
    """The reference's own CPU code (oracle/_ref/libkvref.so, built from the
    reference sources) on this host's cores: layers of the step (append one
    token per sequence with KVManager::save_page, then single-query attention
    per (sequence, q-head) composed from TensorOps matmul/softmax), fanned
    over all host threads.  Runs sample_layers layers, then more until
    min_seconds of CPU work have passed (at most max_layers).  Falls back to
    the C restatement (port)."""
    threads = os.cpu_count() or 1
    lens = workload_lens() + 1
    kind = "reference"
    try:
        from oracle import Reference
        R = Reference()
    except Exception:
        R, kind = None, "port"
    total_s = 0.0
    total_bytes = 0
    rng = np.random.default_rng(SEED)
    tmax = int(lens.max())
    Kall = rng.standard_normal((HKV, tmax, DIM), dtype=np.float32)
    Vall = rng.standard_normal((HKV, tmax, DIM), dtype=np.float32)
    layers = 0
    while layers < sample_layers or (total_s < min_seconds and layers < max_layers):
        layers += 1
        for s in range(BATCH):
            T = int(lens[s])
            K = np.ascontiguousarray(Kall[:, :T])
            V = np.ascontiguousarray(Vall[:, :T])
            q = rng.standard_normal((HQ, DIM), dtype=np.float32)
            out = np.empty((HQ, DIM), np.float32)
            if R is not None:
                # one call per sequence: HQ units over HKV kv-heads (unit u -> kv u % HKV
                # is the helper's mapping; reorder q so unit u reads kv-head u // G)
                qq = np.ascontiguousarray(q.reshape(HKV, HQ // HKV, DIM).transpose(1, 0, 2).reshape(HQ, DIM))
                dt = R.L.kvref_time_decode(qq, np.ascontiguousarray(K), np.ascontiguousarray(V), HKV, HQ, T, DIM,
                                           threads, out)
            else:
                from oracle import Oracle
                o = Oracle()
                t0 = time.perf_counter()
                for h in range(HQ):
                    o.attention_row(q[h], K[h // (HQ // HKV)], V[h // (HQ // HKV)])
                dt = time.perf_counter() - t0
            total_s += dt
            total_bytes += T * 2 * HKV * DIM * 2
    append_s = 0.0
    if R is not None:
        with tempfile.TemporaryDirectory(dir="/dev/shm" if os.path.isdir("/dev/shm") else None) as d:
            cwd = os.getcwd()
            os.chdir(d)
            try:
                rows = kvgen.normal(77, (BATCH, HKV * DIM))
                append_s = R.L.kvref_time_append(rows, BATCH, HKV, DIM, PT, b"pages")
            finally:
                os.chdir(cwd)
    # one layer's appends, timed once, stand for every pass's
    value = total_bytes / (total_s + layers * append_s) / 1e9
    return {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{layers} layer passes ({LAYERS} make one step), each {BATCH}x{HQ} single-query "
                      f"attentions (TensorOps matmul/softmax) and {BATCH} appends via KVManager::save_page "
                      f"(timed once per call), {threads} threads",
            "seconds": round(total_s + layers * append_s, 3)}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup):
        cpu_baseline(1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        vals.append(cpu_baseline(1))
    wall = time.perf_counter() - t0
    v = statistics.median([x["value"] for x in vals])
    base = vals[-1]
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "sample": base["sample"]},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": base["cores"], "kind": base["kind"],
                         "sample": base["sample"]},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# --------------------------------------------------------------------------
def _events_time(fn, iters, warm=3):
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters  # ms


def run_config1(args):
    """One layer of Llama-3.2-3B attention geometry (24 q / 8 kv heads x 128),
    fp32, batch 1: 1024 tokens appended one at a time into 16-token pages
    (sequential physical pages), then one decode for a fresh query."""
    import torch
    import kvx
    T = 1024
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED)
    pool = torch.zeros((T // PT, 2, HKV, PT, DIM), device="cuda", dtype=torch.float32)
    bt = torch.arange(T // PT, dtype=torch.int32, device="cuda").view(1, -1)
    rows = torch.randn((T, 2, 1, HKV, DIM), generator=g, device="cuda", dtype=torch.float32)
    pos = [torch.tensor([t], dtype=torch.int32, device="cuda") for t in range(T)]
    q = torch.randn((1, HQ, DIM), generator=g, device="cuda", dtype=torch.float32)
    lens = torch.tensor([T], dtype=torch.int32, device="cuda")
    ws = kvx.decode_workspace(1, HQ, T // PT)

    def appends():
        for t in range(T):
            kvx.append(pool, bt, pos[t], rows[t, 0], rows[t, 1])
    ms_app = _events_time(appends, 5, 1)
    # the same 1024 single-token launches captured once in a CUDA graph and
    # replayed: what a token costs on the device without the host's launches
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        appends()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        appends()
    ms_graph = _events_time(graph.replay, 5, 1)
    ms_dec = _events_time(lambda: kvx.decode(pool, bt, lens, q, workspace=ws), 200)
    # 20 decodes captured once and replayed: the device time of one, without
    # the host's per-call cost (which the loop above measures)
    dout = torch.empty_like(q)
    with torch.cuda.stream(side):
        for _ in range(3):
            kvx.decode(pool, bt, lens, q, out=dout, workspace=ws)
    torch.cuda.current_stream().wait_stream(side)
    dgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dgraph):
        for _ in range(20):
            kvx.decode(pool, bt, lens, q, out=dout, workspace=ws)
    ms_dec_graph = _events_time(dgraph.replay, 10, 2) / 20
    kv_bytes = T * 2 * HKV * DIM * 4
    # TensorOps::attention over the whole sequence for one head (the
    # cuda_attention drop-in): [1024][128] fp32 queries, keys and values
    qd, kd, vd = (torch.randn((T, DIM), generator=g, device="cuda") for _ in range(3))
    od = torch.empty_like(qd)
    ms_att = _events_time(lambda: kvx.attention_dense(qd, kd, vd, out=od), 20)
    # 20 calls captured once and replayed: the kernel's device time
    with torch.cuda.stream(side):
        for _ in range(3):
            kvx.attention_dense(qd, kd, vd, out=od)
    torch.cuda.current_stream().wait_stream(side)
    agraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(agraph):
        for _ in range(20):
            kvx.attention_dense(qd, kd, vd, out=od)
    ms_att_graph = _events_time(agraph.replay, 10, 2) / 20
    print(json.dumps({"config": 1, "workload": "1 layer, 24q/8kv x128, fp32, B1, 1024 tokens appended one by one, then decode",
                      "append_tokens_per_s": round(T / (ms_app / 1e3), 1),
                      "append_us_per_token": round(ms_app * 1e3 / T, 2),
                      "append_us_per_token_graph": round(ms_graph * 1e3 / T, 2),
                      "dense_attention": {"us": round(ms_att * 1e3, 1),
                                          "GFLOPs": round(4 * T * T * DIM / (ms_att / 1e3) / 1e9, 1),
                                          "us_graph": round(ms_att_graph * 1e3, 2),
                                          "GFLOPs_graph": round(4 * T * T * DIM / (ms_att_graph / 1e3) / 1e9, 1),
                                          "kernel": "attention_umma_kernel + combine_splits_kernel (tcgen05 kind::tf32, 3xTF32 products)"},
                      "decode_us": round(ms_dec * 1e3, 2),
                      "decode_GBps": round(kv_bytes / (ms_dec / 1e3) / 1e9, 1),
                      "decode_us_graph": round(ms_dec_graph * 1e3, 2),
                      "decode_GBps_graph": round(kv_bytes / (ms_dec_graph / 1e3) / 1e9, 1),
                      "note": "latency-bound: one launch per token (from Python, or replayed from a CUDA graph), "
                              "8 MiB of K/V per decode"}), flush=True)


def run_config3(args):
    """compressKv round trip: 1,048,576 pages of 16 tokens x 8 KV heads x 128
    fp16 (N(0,1), 1% of elements x20), quantised per (page, head) block with
    the reference's int8 scheme, dequantised, then decode (batch 32, context
    4096, 24 q-heads) reading the int8 pages with fused dequantisation."""
    import torch
    import kvx
    peak, peak_kind = peaks()
    pages = args.pages
    blocks = pages * HKV  # one (page, head) block of 2048 elements
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 3)
    x = torch.empty((blocks, PT * DIM), device="cuda", dtype=torch.float16)
    for c in range(0, blocks, 1 << 20):  # fill in chunks (bounded temporaries)
        part = torch.randn((min(1 << 20, blocks - c), PT * DIM), generator=g, device="cuda")
        mask = torch.rand(part.shape, generator=g, device="cuda") < 0.01
        part[mask] *= 20.0
        x[c:c + part.shape[0]] = part.half()
        del part, mask
    codes = torch.empty((blocks, PT * DIM), device="cuda", dtype=torch.int8)
    stats = torch.empty((blocks, 4), device="cuda", dtype=torch.float32)
    back = torch.empty_like(x)
    ms_c = _events_time(lambda: kvx.compress_int8(x, codes=codes, stats=stats), 5)
    ms_d = _events_time(lambda: kvx.decompress_int8(codes, stats, dtype=torch.float16, out=back), 5)
    err = True  # |x - dequant(quant(x))| <= scale/2 per block (fp32 dequant), in chunks
    for c in range(0, blocks, 1 << 20):
        part = kvx.decompress_int8(codes[c:c + (1 << 20)], stats[c:c + (1 << 20)]).view(-1, PT * DIM)
        e = (part - x[c:c + (1 << 20)].float()).abs().amax(dim=1)
        err = err and bool((e <= stats[c:c + (1 << 20), 2] * 0.5001 + 1e-6).all().item())
        del part, e
    n = x.numel()
    c_bytes = n * 2 + n + blocks * 16
    d_bytes = n + blocks * 16 + n * 2
    # the engine's other codecs on the same pages: NF4 (uniform 4-bit) ...
    nf4_codes = torch.empty(n // 2, device="cuda", dtype=torch.uint8)
    nf4_stats = torch.empty((blocks, 4), device="cuda", dtype=torch.float32)
    ms_nc = _events_time(lambda: kvx.compress_nf4(x, codes=nf4_codes, stats=nf4_stats), 5)
    ms_nd = _events_time(lambda: kvx.decompress_nf4(nf4_codes, nf4_stats, dtype=torch.float16, out=back), 5)
    nc_bytes = n * 2 + n // 2 + blocks * 16
    del nf4_codes, nf4_stats, back
    # ... and the exponent-wrapping FP16 of fp32 data (4 GiB in)
    x32 = torch.randn(1 << 30, generator=g, device="cuda", dtype=torch.float32)
    h16 = torch.empty(1 << 30, device="cuda", dtype=torch.int16)
    ms_we = _events_time(lambda: kvx.fp16_wrap_encode(x32, out=h16), 5)
    ms_wd = _events_time(lambda: kvx.fp16_wrap_decode(h16, out=x32), 5)
    # the disk tier's truncating codec (compression/kv_compress.cpp:6-60) on the same arrays
    ms_te = _events_time(lambda: kvx.f32_to_f16_trunc(x32, out=h16), 5)
    ms_td = _events_time(lambda: kvx.f16_trunc_to_f32(h16, out=x32), 5)
    w_bytes = (1 << 30) * 6
    del x32, h16
    # decode over int8 pages: batch 32, context 4096, one layer, 24 q-heads
    B, T = 32, 4096
    npg = T // PT
    lens = torch.full((B,), T, dtype=torch.int32, device="cuda")
    # the 1,048,576 K-or-V pages pair up into 524,288 (K, V) pages of the pool layout
    kv_pages = pages // 2
    pool = codes.view(kv_pages, 2, HKV, PT, DIM)
    pstats = stats.view(kv_pages, 2, HKV, 4)
    bt = torch.randperm(kv_pages, generator=g, device="cuda")[: B * npg].to(torch.int32).view(B, npg).contiguous()
    q = torch.randn((B, HQ, DIM), generator=g, device="cuda", dtype=torch.float16)
    ws = kvx.decode_workspace(B, HQ, npg)
    ms_q = _events_time(lambda: kvx.decode(pool, bt, lens, q, stats=pstats, workspace=ws), 20)
    q_bytes = B * T * 2 * HKV * DIM * 1 + B * npg * 2 * HKV * 16
    cpu = cpu_compress_baseline() if not args.no_cpu_baseline else None
    print(json.dumps({
        "config": 3, "workload": f"{pages:,} pages x 16 tok x 8 heads x 128 fp16, 1% outliers x20; int8 per (page, head)",
        "compress": {"GBps": round(c_bytes / (ms_c / 1e3) / 1e9, 1), "ms": round(ms_c, 3),
                     "frac_of_peak": round(c_bytes / (ms_c / 1e3) / 1e9 / peak, 3)},
        "decompress": {"GBps": round(d_bytes / (ms_d / 1e3) / 1e9, 1), "ms": round(ms_d, 3),
                       "frac_of_peak": round(d_bytes / (ms_d / 1e3) / 1e9 / peak, 3)},
        "roundtrip_error_within_scale_half": bool(err),
        "nf4": {"compress_GBps": round(nc_bytes / (ms_nc / 1e3) / 1e9, 1),
                "compress_frac_of_peak": round(nc_bytes / (ms_nc / 1e3) / 1e9 / peak, 3),
                "decompress_GBps": round(nc_bytes / (ms_nd / 1e3) / 1e9, 1),
                "decompress_frac_of_peak": round(nc_bytes / (ms_nd / 1e3) / 1e9 / peak, 3)},
        "fp16_wrap": {"encode_GBps": round(w_bytes / (ms_we / 1e3) / 1e9, 1),
                      "decode_GBps": round(w_bytes / (ms_wd / 1e3) / 1e9, 1),
                      "encode_frac_of_peak": round(w_bytes / (ms_we / 1e3) / 1e9 / peak, 3),
                      "decode_frac_of_peak": round(w_bytes / (ms_wd / 1e3) / 1e9 / peak, 3)},
        "fp16_trunc": {"encode_GBps": round(w_bytes / (ms_te / 1e3) / 1e9, 1),
                       "decode_GBps": round(w_bytes / (ms_td / 1e3) / 1e9, 1),
                       "encode_frac_of_peak": round(w_bytes / (ms_te / 1e3) / 1e9 / peak, 3),
                       "decode_frac_of_peak": round(w_bytes / (ms_td / 1e3) / 1e9 / peak, 3)},
        "int8_decode": {"GBps": round(q_bytes / (ms_q / 1e3) / 1e9, 1), "us": round(ms_q * 1e3, 1),
                        "batch": B, "context": T, "frac_of_peak": round(q_bytes / (ms_q / 1e3) / 1e9 / peak, 3)},
        "peak": peak, "peak_kind": peak_kind, "cpu_baseline": cpu}), flush=True)


def cpu_compress_baseline(blocks=16384):
    """KVCompressionEngine INT8 (oracle/_ref, the reference's code) per
    2048-element block over all host threads, on a sample of blocks."""
    try:
        from oracle import Reference
        R = Reference()
    except Exception as e:
        return {"unavailable": str(e)[:120]}
    threads = os.cpu_count() or 1
    x = np.random.default_rng(SEED).standard_normal((blocks, 2048), dtype=np.float32)
    codes = np.empty((blocks, 2048), np.int8)
    stats = np.empty((blocks, 4), np.float32)
    secs = R.L.kvref_time_compress(x, codes, stats, blocks, 2048, threads)
    # same byte accounting as the GPU (fp16 in: the reference takes fp32)
    gbps = blocks * (2048 * 2 + 2048 + 16) / secs / 1e9
    return {"value": round(gbps, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"{blocks} blocks of 2048 through KVCompressionEngine::compress(INT8)"}


def pinned_peaks(nbytes=2 << 30):
    """cudaMemcpyAsync over the host link with pinned memory: H2D, D2H and
    both at once on two streams (GB/s)."""
    import torch
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    h2 = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    d2 = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()

    def timed(fn, reps=4):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / reps

    def h2d():
        with torch.cuda.stream(s1):
            d.copy_(h, non_blocking=True)

    def d2h():
        with torch.cuda.stream(s2):
            h2.copy_(d2, non_blocking=True)

    def both():
        h2d()
        d2h()

    th, td, tb = timed(h2d), timed(d2h), timed(both)
    res = {"h2d": round(nbytes / th / 1e9, 1), "d2h": round(nbytes / td / 1e9, 1),
           "bidir_sum": round(2 * nbytes / tb / 1e9, 1)}
    del h, h2, d, d2
    return res


def cpu_tier_baseline(universe=4096, accesses=20000):
    """The reference's page tier on the host: KVManager (cache/kv_cache.cpp)
    with a third of the pages in memory and the rest as fp16 page files,
    serving load_page over a Zipf(1.1) stream; bytes = misses x 64 KiB."""
    try:
        from oracle import Reference
        ref = Reference()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference library not loadable: {e}"}
    ids = kvgen.permutation(SEED + 41, universe)[kvgen.zipf_pages(SEED + 42, accesses, universe, 1.1)]
    with tempfile.TemporaryDirectory() as d:
        sec, misses = ref.time_tier(ids.astype(np.int32), universe, universe // 3, PT * HKV * DIM, d)
    return {"value": round(misses * 65536 / sec / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "reference",
            "sample": f"KVManager capacity {universe // 3} of {universe} pages (64 KiB fp16 page files), "
                      f"{accesses} Zipf(1.1) load_page calls, {misses} misses"}


def select_timing(n):
    """Victim selection on the device over n frames: kvx_lru_select over
    access stamps (LRUEvictionPolicy / KVCacheGPU::findLRUPage) and
    kvx_evict_select over EvictionMetrics records for LRU, TokenWeighted and
    AttentionBased (AdvancedEvictionPolicy::selectPageToEvict); seeded
    synthetic stamps and attention values."""
    import torch
    import kvx
    # kvx_evict_metrics (include/kvx.h): the reference's EvictionMetrics layout
    rec = np.dtype([("last_access_token", "<u8"), ("total_attention", "<f4"), ("average_attention", "<f4"),
                    ("access_frequency", "<f4"), ("_pad0", "<u4"), ("creation_time", "<u8"),
                    ("page_size", "<u8"), ("page_id", "<i4"), ("_pad1", "<u4")])
    assert rec.itemsize == 48
    rng = np.random.default_rng(SEED + 9)
    m = np.zeros(n, rec)
    m["last_access_token"] = rng.integers(0, 1 << 40, n, dtype=np.uint64)
    m["average_attention"] = rng.random(n, dtype=np.float32)
    m["total_attention"] = m["average_attention"] * 4
    m["page_id"] = np.arange(n, dtype=np.int32)
    pages = torch.from_numpy(m.view(np.uint8).copy()).cuda()
    stamps = torch.from_numpy(m["last_access_token"].copy().view(np.int64)).cuda()
    out = {"frames": n}
    ms = _events_time(lambda: kvx.lru_select(stamps), 20)
    out["lru_stamps"] = {"us": round(ms * 1e3, 1), "GBps": round(n * 8 / (ms / 1e3) / 1e9, 1)}
    for name, pol in (("lru", 0), ("token_weighted", 1), ("attention_based", 2)):
        ms = _events_time(lambda: kvx.evict_select(pol, pages), 10)
        out[name] = {"us": round(ms * 1e3, 1), "GBps": round(n * 48 / (ms / 1e3) / 1e9, 1)}
    return out


SCHED_MAX_DEPTH = 4  # the reference Scheduler's default max_depth


def _config4_prefetch_loop(tier, kvx, pool, stream_ids, q, lens, out, ws, L, B, ACC, C, dpol):
    """Config 4 planned and loaded per layer, as the reference's
    InferenceController::schedulePrefetch (runtime/inference.cpp:61-84)
    prefetches per layer: before the decode of layer unit g (step k, layer l)
    the loop asks the Scheduler (scheduler/scheduler.cpp:15-37, through
    kvx_scheduler_depth) for a depth d and plans units up to g + d, each
    plan one kvx_tier step of that layer's B x ACC page accesses (the same
    access order as a whole step, so KVManager's decisions are unchanged).
    The latency of each unit's load (plan issued -> frames resident, CUDA
    events) goes to observeLoadLatency; the cache pressure is the store's
    (resident frames / capacity).  The store runs with lookahead
    SCHED_MAX_DEPTH - 1, so any depth the Scheduler can answer is legal."""
    import collections
    import torch
    from kvx.scheduler import Scheduler
    steps = len(stream_ids)
    G, n = steps * L, B * ACC
    NB = SCHED_MAX_DEPTH + 3  # block-table / id buffers in flight
    sched = Scheduler(SCHED_MAX_DEPTH)
    btl = [torch.empty((B, ACC), dtype=torch.int32, device="cuda") for _ in range(NB)]
    used = [torch.cuda.Event() for _ in range(NB)]
    e_issue = [torch.cuda.Event(enable_timing=True) for _ in range(G)]
    e_ready = [torch.cuda.Event(enable_timing=True) for _ in range(G)]
    if dpol:
        ids_pinned = torch.from_numpy(np.stack(stream_ids)).pin_memory()
        ids_dev = [torch.empty(n, dtype=torch.int32, device="cuda") for _ in range(NB)]
        planst = torch.cuda.Stream()
    else:
        bt_host = [torch.empty(n, dtype=torch.int32, pin_memory=True) for _ in range(NB)]
        up = [torch.cuda.Event() for _ in range(NB)]
    plan_s, planned, observed = 0.0, 0, []
    depths = collections.Counter()

    def plan(u):
        nonlocal plan_s
        i, (k, l) = u % NB, divmod(u, L)
        h0 = time.perf_counter()
        if dpol:
            with torch.cuda.stream(planst):
                if u >= NB:  # unit u-NB's decode read btl[i] (after its plan read ids_dev[i])
                    planst.wait_event(used[i])
                ids_dev[i].copy_(ids_pinned[k, l * n:(l + 1) * n], non_blocking=True)
                e_issue[u].record(planst)
            tier.step_device(ids_dev[i], btl[i].view(-1), stream=planst)
        else:
            if u >= NB:
                up[i].synchronize()  # the upload of unit u-NB read bt_host[i]
            e_issue[u].record()
            tier.step(stream_ids[k][l * n:(l + 1) * n], dev_slot=bt_host[i].numpy(), evicted=False, hit=False)
            btl[i].view(-1).copy_(bt_host[i], non_blocking=True)  # after unit u-NB's decode (same stream)
            up[i].record()
        plan_s += time.perf_counter() - h0

    for u in range(G):
        d = sched.depth(u, C, C)  # the store is full: resident == capacity
        depths[d] += 1
        while planned < G and planned <= u + d:
            plan(planned)
            planned += 1
        tier.wait_resident()
        e_ready[u].record()
        kvx.decode(pool, btl[u % NB], lens, q[u % L], out=out[u % L], workspace=ws)
        used[u % NB].record()
        tier.mark_read()
        if u >= 2 and e_ready[u - 2].query():
            ms = e_issue[u - 2].elapsed_time(e_ready[u - 2])
            sched.observe(ms)
            observed.append(ms)
    sched.close()
    return {"driver": "Scheduler::getPrefetchDepth per layer (kvx_scheduler_depth), max_depth "
                      f"{SCHED_MAX_DEPTH}, store lookahead {SCHED_MAX_DEPTH - 1}",
            "units_per_step": L, "accesses_per_unit": n,
            "depths": {str(k): v for k, v in sorted(depths.items())},
            "observed_load_ms": {"mean": round(float(np.mean(observed)), 3) if observed else None,
                                 "count": len(observed)},
            "plan_s": plan_s,
            # the last NB units' block tables (resident frames), for timing the decode alone
            "tables": [btl[(G - NB + (l % NB)) % NB] for l in range(L)]}


def device_plan_timing(U, C, S, n, step_ids, warm, steps=8):
    """Device time of one step's plan (the policy kernels of
    kvx_tier_step_device) at config 4's geometry: CUDA events on the store's
    plan stream around the plan, every earlier copy finished (16-byte frames
    keep the store small)."""
    import torch
    from kvx.tier import Tier
    t = Tier(16, U, C, S, device=0, device_policy=True, max_step=n)
    for k in range(warm):
        ids = step_ids(k)
        for o in range(0, ids.size, 16384):
            t.step(ids[o:o + 16384], evicted=False, hit=False)
    t.sync()
    ids_d = [torch.from_numpy(step_ids(warm + k)).cuda() for k in range(steps)]
    slots = torch.empty(n, dtype=torch.int32, device="cuda")
    plan = t.plan_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    for k in range(steps):
        ev[k][0].record(plan)
        t.step_device(ids_d[k], slots, stream=plan)
        ev[k][1].record(plan)
        t.sync()
    us = sorted(a.elapsed_time(b) * 1e3 for a, b in ev)
    t.close()
    return {"median_us": round(us[len(us) // 2], 1), "min_us": round(us[0], 1), "steps": steps,
            "accesses": n, "how": "CUDA events on the plan stream around kvx_tier_step_device"}


def run_config4(args):
    """Tiered eviction under memory pressure.  Llama-3.2-3B KV (28 layers, 8
    kv heads x 128, fp16) at batch 16 with 65,536-token contexts: 1,835,008
    page frames of 64 KiB (one 16-token page of all 8 heads, K and V), 120 GB,
    against a device pool capped at 40 GB (610,351 frames); the rest lives in
    a pinned host arena.  Each decode step every (layer, sequence) reads 256 of
    its 4096 pages, drawn Zipf(1.1) over a seeded per-(layer, sequence)
    ranking.  The store (kvx_tier) applies KVManager's LRU to the step's
    accesses in order, then loads the misses and writes the victims back over
    the host link on two copy streams while the previous step's decode runs;
    decode (B16, 4096 tokens of pages per sequence, 24 q-heads) reads the
    frames in place.  Reported: frames moved per second per direction against
    the measured pinned-copy peak, decode GB/s, hit rate, step time."""
    import torch
    import kvx
    from kvx.tier import Tier
    L, B, P = 28, 16, args.tier_context // PT
    ACC = P // 16  # pages read per (layer, sequence) per step: 256 at 65,536 tokens
    FB = 2 * HKV * PT * DIM * 2
    U = L * B * P
    C = int(args.tier_device_gb * 1e9) // FB
    S = max(4096, ((L * B * ACC) * 3 // 7) // 4096 * 4096)  # 49152 at full size
    H = int(args.tier_ram_gb * 1e9) // FB if args.tier_ram_gb > 0 else 0
    spill_dir = tempfile.mkdtemp(prefix="kvx_spill_", dir=os.environ.get("KVX_SPILL_DIR")) if H else None
    steps = args.steps
    warm = max(args.warmup, 16)
    link = pinned_peaks()
    # access stream: per (layer, sequence) ranks Zipf(1.1), ranks -> pages by a seeded permutation
    rows = L * B
    perms = np.stack([kvgen.permutation(SEED + 1000 + i, P) for i in range(rows)]).astype(np.int32)
    base = (np.arange(rows, dtype=np.int64) * P)[:, None]

    def step_ids(k):
        r = kvgen.zipf_pages(SEED + 5000 + k, rows * ACC, P, 1.1).reshape(rows, ACC)
        return (base + np.take_along_axis(perms, r, axis=1)).astype(np.int32).ravel()

    t0 = time.perf_counter()
    dpol = not args.tier_host_policy and not H  # the disk tier runs on the host policy
    look = SCHED_MAX_DEPTH - 1 if args.tier_prefetch else 0
    tier = Tier(FB, U, C, S, device=0, load_ctas=int(os.environ.get("KVX_TIER_LOAD_CTAS", "0")),
                store_ctas=int(os.environ.get("KVX_TIER_STORE_CTAS", "0")), host_frames=H,
                spill_path=None if not H else os.path.join(spill_dir, "frames.bin"),
                device_policy=dpol, max_step=rows * ACC if dpol else 0, lookahead=look)
    alloc_s = time.perf_counter() - t0
    dev = tier.device_tensor()
    host = tier.host_array()
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 4)
    chunk = 1 << 30
    for o in range(0, dev.numel(), chunk):  # device frames: random fp16
        n = min(chunk, dev.numel() - o)
        dev[o:o + n] = torch.randn(n // 2, generator=g, device="cuda", dtype=torch.float16).view(torch.uint8)
    src = torch.randn(chunk // 2, generator=g, device="cuda", dtype=torch.float16).view(torch.uint8)
    ht = torch.from_numpy(host)
    for o in range(0, ht.numel(), chunk):  # host frames: copies of one random GiB
        n = min(chunk, ht.numel() - o)
        ht[o:o + n].copy_(src[:n])
    torch.cuda.synchronize()
    if H:  # disk frames (ids C + H ..): the same GiB, written once at their offsets
        blob = src.cpu().numpy().tobytes()
        with open(os.path.join(spill_dir, "frames.bin"), "r+b") as f:
            f.seek((C + H) * FB)
            left = (U - C - H) * FB
            while left:
                n = min(len(blob), left)
                f.write(blob[:n])
                left -= n
        del blob
    del src
    # warm-up: the policy and the copies only, in chunks that fit the spare slots
    for k in range(warm):
        ids = step_ids(k)
        for o in range(0, ids.size, 16384):
            tier.step(ids[o:o + 16384], evicted=False, hit=False)
            if look:
                tier.mark_read()  # nothing reads warm-up frames
    tier.sync()
    q = torch.randn((L, B, HQ, DIM), generator=g, device="cuda", dtype=torch.float16)
    lens = torch.full((B,), ACC * PT, dtype=torch.int32, device="cuda")
    out = torch.empty((L, B, HQ, DIM), device="cuda", dtype=torch.float16)
    ws = kvx.decode_workspace(B, HQ, ACC)
    pool = tier.paged(HKV)
    bt_host = [torch.empty(rows * ACC, dtype=torch.int32, pin_memory=True) for _ in range(2)]
    bt_dev = [torch.empty((L, B, ACC), dtype=torch.int32, device="cuda") for _ in range(2)]
    up = [torch.cuda.Event() for _ in range(2)]
    stream_ids = [step_ids(warm + k) for k in range(steps)]
    if dpol:  # the step's ids go up from pinned memory; the policy writes the block table
        ids_pinned = torch.from_numpy(np.stack(stream_ids)).pin_memory()
        ids_dev = [torch.empty(rows * ACC, dtype=torch.int32, device="cuda") for _ in range(2)]
        plan = torch.cuda.Stream()  # plans run ahead of the decode stream, beside the copies
        dec_done = [torch.cuda.Event() for _ in range(2)]
    before = tier.totals()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    plan_s = 0.0
    e0.record()
    pre = None
    if args.tier_prefetch:
        pre = _config4_prefetch_loop(tier, kvx, pool, stream_ids, q, lens, out, ws, L, B, ACC, C, dpol)
        plan_s = pre.pop("plan_s")
        last_tables = pre.pop("tables")
    for k in range(steps if pre is None else 0):
        p = k & 1
        if dpol:
            with torch.cuda.stream(plan):
                if k >= 2:  # step k-2's decode read bt_dev[p] (and waited for its plan, which read ids_dev[p])
                    plan.wait_event(dec_done[p])
                ids_dev[p].copy_(ids_pinned[k], non_blocking=True)
            h0 = time.perf_counter()
            tier.step_device(ids_dev[p], bt_dev[p].view(-1), stream=plan)
            plan_s += time.perf_counter() - h0
            tier.wait_resident()
        else:
            if k >= 2:
                up[p].synchronize()  # the block-table upload of step k-2 read this buffer
            h0 = time.perf_counter()
            tier.step(stream_ids[k], dev_slot=bt_host[p].numpy(), evicted=False, hit=False)
            plan_s += time.perf_counter() - h0
            tier.wait_resident()
            bt_dev[p].view(-1).copy_(bt_host[p], non_blocking=True)
            up[p].record()
        for l in range(L):
            kvx.decode(pool, bt_dev[p][l], lens, q[l], out=out[l], workspace=ws)
        tier.mark_read()
        if dpol:
            dec_done[p].record()
    e1.record()
    tier.sync()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    after = tier.totals()
    mv = {k2: after[k2] - before[k2] for k2 in after}
    # decode alone, frames resident (last step's tables)
    if pre is None:
        last_tables = [bt_dev[(steps - 1) & 1][l] for l in range(L)]
    dec_ms = _events_time(lambda: [kvx.decode(pool, last_tables[l], lens, q[l], out=out[l],
                                              workspace=ws) for l in range(L)], 3)
    dec_bytes = rows * ACC * FB
    sel = select_timing(C)
    dplan = device_plan_timing(U, C, S, rows * ACC, step_ids, warm) if not H else None
    h2d_gbs = mv["frames_h2d"] * FB / (ms / 1e3) / 1e9
    d2h_gbs = mv["frames_d2h"] * FB / (ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    cpu = cpu_tier_baseline() if not args.no_cpu_baseline else None
    res = {
        "config": 4, "workload": f"tiered eviction: Llama-3.2-3B KV (28L, 8kv x128, fp16), B16, ctx {args.tier_context} = "
                                 f"{U:,} frames x 64 KiB; device pool {args.tier_device_gb:g} GB ({C:,} frames); per step "
                                 f"each (layer, seq) reads {ACC} pages drawn Zipf(1.1); KVManager LRU"
                                 + (f"; RAM tier {args.tier_ram_gb:g} GB, the rest on disk" if H else ""),
        "steps": steps, "warmup_steps": warm, "ms_per_step": round(ms / steps, 3),
        "hit_rate": round(mv["hits"] / max(1, mv["accesses"]), 4),
        "frames_per_step": {"h2d": round(mv["frames_h2d"] / steps, 1), "d2h": round(mv["frames_d2h"] / steps, 1),
                            "reloads": round(mv["reloads"] / steps, 2)},
        "migrate": {"h2d_GBps": round(h2d_gbs, 1), "d2h_GBps": round(d2h_gbs, 1),
                    "h2d_frac_of_pinned_peak": round(h2d_gbs / link["h2d"], 3),
                    "d2h_frac_of_pinned_peak": round(d2h_gbs / link["d2h"], 3),
                    "sum_frac_of_bidir_peak": round((h2d_gbs + d2h_gbs) / link["bidir_sum"], 3)},
        "pinned_peak_GBps": link,
        "decode": {"GBps_overlapped": round(steps * dec_bytes / (ms / 1e3) / 1e9, 1),
                   "ms_alone_per_step": round(dec_ms, 3),
                   "GBps_alone": round(dec_bytes / (dec_ms / 1e3) / 1e9, 1),
                   "frac_of_hbm_peak_alone": round(dec_bytes / (dec_ms / 1e3) / 1e9 / peak, 3)},
        "policy": "device (kvx_tier_step_device)" if dpol else "host (kvx_tier_step)",
        "prefetch": pre,
        "host_plan_ms_per_step": round(plan_s / steps * 1e3, 3),
        "device_plan_latency": dplan,
        "victim_select": sel,
        "disk_tier": None if not H else {
            "ram_tier_GB": round(H * FB / 1e9, 1), "spill_file_GB": round(U * FB / 1e9, 1),
            "frames_per_step": {"read": round(mv["frames_disk_read"] / steps, 1),
                                "written": round(mv["frames_disk_write"] / steps, 1)},
            "GBps": {"read": round(mv["frames_disk_read"] * FB / (ms / 1e3) / 1e9, 2),
                     "write": round(mv["frames_disk_write"] * FB / (ms / 1e3) / 1e9, 2)}},
        "host_arena_GB": round(((H if H else U - C) + S) * FB / 1e9, 1), "device_arena_GB": round((C + S) * FB / 1e9, 1),
        "alloc_s": round(alloc_s, 1), "clocks": clk, "peak": peak, "peak_kind": peak_kind,
        "cpu_baseline": cpu}
    print(json.dumps(res), flush=True)
    tier.close()
    if spill_dir:
        import shutil
        shutil.rmtree(spill_dir, ignore_errors=True)


SHAPES = ((1, 32768), (1, 131072), (4, 16384), (8, 32768), (16, 8192), (32, 4096), (64, 2048),
          (128, 1024), (256, 512))
SHAPES_I8 = ((32, 4096), (8, 32768), (32, 8192))
SHAPES_F32 = ((1, 32768), (32, 4096), (128, 1024))


def run_shapes(args):
    """kvx.decode over uniform-length batches: 8 KV heads x 128, 16-token
    pages in a seeded random permutation, q-heads 24 (GQA 3) and 64 (GQA 8);
    fp16 pools for SHAPES, int8 pools (random codes, one {min, max, scale,
    zero point} per block) for SHAPES_I8, fp32 pools with fp32 queries (the
    SIMT kernel) for SHAPES_F32.  GB/s of K/V (+ stats) read per
    launch: CUDA events around 60 back-to-back launches that rotate over 3
    copies of the pool when one copy is under 1 GiB, so no launch finds its
    pages in L2."""
    import torch
    import kvx
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED)
    forced = [int(c) for c in args.shape_chunks.split(",") if c.strip()]

    def timed(fns, iters=60, warm=6):
        for i in range(warm):
            fns[i % len(fns)]()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(iters):
            fns[i % len(fns)]()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / iters

    def sweep(fns, nbytes):
        res = {}
        for c in [None] + forced:
            if c is None:
                os.environ.pop("KVX_DECODE_CHUNK", None)
            else:
                os.environ["KVX_DECODE_CHUNK"] = str(c)
            try:
                ms = timed(fns)
            finally:
                os.environ.pop("KVX_DECODE_CHUNK", None)
            res["default" if c is None else str(c)] = round(nbytes / (ms / 1e3) / 1e9, 1)
        return res

    kinds = {k.strip() for k in args.shape_pools.split(",")}
    for pool_kind, shapes in (("fp16", SHAPES), ("int8", SHAPES_I8), ("fp32", SHAPES_F32)):
        if pool_kind not in kinds:
            continue
        for B, T in shapes:
            npg = T // PT
            lens = torch.full((B,), T, dtype=torch.int32, device="cuda")
            if pool_kind in ("fp16", "fp32"):
                dt = torch.float16 if pool_kind == "fp16" else torch.float32
                page_bytes = 2 * HKV * PT * DIM * dt.itemsize
                nrot = 3 if B * npg * page_bytes < (1 << 30) else 1
                pools = [torch.randn((B * npg, 2, HKV, PT, DIM), generator=g, device="cuda", dtype=dt)
                         for _ in range(nrot)]
                stats = None
                nbytes = B * npg * page_bytes
            else:
                page_bytes = 2 * HKV * PT * DIM
                nrot = 3 if B * npg * page_bytes < (1 << 30) else 1
                pools = [torch.randint(-128, 127, (B * npg, 2, HKV, PT, DIM), generator=g, device="cuda",
                                       dtype=torch.int8) for _ in range(nrot)]
                stats = torch.zeros((B * npg, 2, HKV, 4), device="cuda")
                stats[..., 2] = 0.01
                stats[..., 3] = -1.0
                nbytes = B * npg * (page_bytes + 2 * HKV * 16)
            bts = [torch.randperm(B * npg, generator=g, device="cuda").to(torch.int32).view(B, npg).contiguous()
                   for _ in range(nrot)]
            for hq in (24, 64):
                q = torch.randn((B, hq, DIM), generator=g, device="cuda",
                                dtype=torch.float32 if pool_kind == "fp32" else torch.float16)
                ws = kvx.decode_workspace(B, hq, npg)
                out = torch.empty_like(q)
                fns = [lambda r=r: kvx.decode(pools[r], bts[r], lens, q, stats=stats, out=out, workspace=ws)
                       for r in range(nrot)]
                print(json.dumps({"shapes": "paged decode", "pool": pool_kind, "batch": B, "context": T,
                                  "q_heads": hq, "kv_heads": HKV, "GBps": sweep(fns, nbytes)}), flush=True)
            del pools, bts, stats
            torch.cuda.empty_cache()


L5_FULL, HQ5, HKV5, B5, T5 = 80, 64, 8, 64, 32768


def run_config5_sharded(args, world, rank, dist=None, budget_bytes=150e9):
    """Llama-3-70B KV geometry (80 layers, 64 q-heads, 8 KV heads x 128,
    GQA group 8, fp16), batch 64, 32,768-token contexts, 16-token pages
    randomly permuted; KV heads sharded over the N GPUs (8/N heads each),
    outputs all-gathered over NCCL per group of layers -- the same step as
    the headline (make_decode_step), each step appending token 32,767 and
    decoding over 32,768.  The whole cache (687 GB) fits only at N = 8 (86 GB
    per GPU, all 80 layers); with fewer GPUs each holds its shard of as many
    layers as fit in ~150 GB and the result is given per layer and projected
    to 80 (the layers are identical, so a step's time is linear in them).
    The same fixed job is split N ways (strong scaling per layer)."""
    import torch
    import kvx
    hkv, hq = HKV5 // world, HQ5 // world
    npg = T5 // PT
    pages = B5 * npg + B5  # one spare page per sequence
    layer_bytes = pages * 2 * hkv * PT * DIM * 2
    free, _ = torch.cuda.mem_get_info()
    L = int(max(1, min(L5_FULL, min(budget_bytes, free - 12e9) // layer_bytes)))
    if dist is not None:  # the same layer count on every rank
        t = torch.tensor([L], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        L = int(t.item())
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 5 + 101 * rank)
    pools = [torch.empty((pages, 2, hkv, PT, DIM), device="cuda", dtype=torch.float16).normal_(generator=g)
             for _ in range(L)]
    perm = kvgen.permutation(SEED + 6, pages).astype(np.int32)
    bt_np = perm[: B5 * (npg + 1)].reshape(B5, npg + 1)
    bt = torch.from_numpy(bt_np).cuda()
    lens0 = np.full(B5, T5 - 1, np.int64)  # each step appends token T-1: context T
    steps = max(3, min(args.steps, 6))
    warm = 2
    positions = torch.full((warm + steps, B5), T5 - 1, dtype=torch.int32, device="cuda")
    q = torch.randn((L, B5, hq, DIM), generator=g, device="cuda", dtype=torch.float16)
    nk = torch.randn((L, B5, hkv, DIM), generator=g, device="cuda", dtype=torch.float16)
    ring = OUT_RING if world > 1 else 1
    outs = [torch.empty((L, B5, hq, DIM), device="cuda", dtype=torch.float16) for _ in range(ring)]
    ws = kvx.decode_workspace(B5, hq, npg + 1)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    comm = torch.cuda.Stream() if world > 1 else None
    main = torch.cuda.current_stream()
    check = ParitySample(bt_np, lens0, hkv, hq, world, rank, pools, layers=(0, L - 1), seqs=2) \
        if not args.no_parity else None
    step = make_decode_step(kvx, pools, bt, positions, nk, nk, q, ws, err, outs, world=world,
                            comm=comm, dist=dist)
    for k in range(warm):
        step(k)
    if world > 1:
        main.wait_stream(comm)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for k in range(warm, warm + steps):
        step(k)
    if world > 1:
        main.wait_stream(comm)
    b.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(a.elapsed_time(b) / steps, dist)
    assert err.item() == 0, f"device error flag {err.item()}"
    parity = None
    if check is not None:
        parity = check.verify(q, nk, nk, positions, outs[(warm + steps - 1) % ring], step.gathered_rows, dist)
    kv_rank = B5 * T5 * 2 * hkv * DIM * 2 * L  # bytes one rank reads per step
    peak, peak_kind = peaks()
    res = {"workload": "Llama-3-70B KV (80L, 64q/8kv x128, G8), fp16, B64, ctx 32768, permuted pages",
           "layers_resident": L, "layers_full": L5_FULL, "kv_heads_per_gpu": hkv,
           "ms_per_step": round(ms, 3), "ms_per_layer": round(ms / L, 4),
           "projected_80_layer_step_ms": round(ms / L * L5_FULL, 2),
           "value": round(kv_rank * world / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
           "per_gpu_frac_of_peak": round(kv_rank / (ms / 1e3) / 1e9 / peak, 4), "peak": peak,
           "peak_kind": peak_kind, "scaling": "strong per layer (the 8 KV heads split over the GPUs)",
           "parallelism": f"kv-head shard x{world}" + (" + NCCL all-gather" if world > 1 else ""),
           "parity": parity}
    del pools, outs, ws, q, nk, step
    torch.cuda.empty_cache()
    return res


def run_config5(args):
    """Config 5 alone (see run_config5_sharded); one JSON line from rank 0."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    res = run_config5_sharded(args, world, rank, dist if world > 1 else None)
    res.update({"config": 5, "n_gpus": world})
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_kernel_profiles(args):
    """One JSON line per kernel that the headline line does not time: a
    stated size (a few GB on the device at most, inputs above L2), the
    algorithmic bytes one launch moves and its mean duration over
    args.kernel_iters launches (CUDA events, after one warm-up), against the
    measured HBM copy peak (the host link's measured pinned copy peak for
    frame migration).  Also the target of the per-kernel ncu captures."""
    import torch
    import kvx
    peak, peak_kind = peaks()
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 77)
    iters = args.kernel_iters
    rows = []

    def emit(name, kernel, size, nbytes, fn, bound="hbm", ref=None):
        ms = _timed_events(fn, iters, warm=1)
        gbps = nbytes / (ms / 1e3) / 1e9
        rows.append({"kernels": name, "kernel": kernel, "size": size, "bytes_per_launch": int(nbytes),
                     "us": round(ms * 1e3, 2), "GBps": round(gbps, 1), "bound": bound,
                     "frac": round(gbps / (ref if ref else peak), 4),
                     "peak": ref if ref else peak, "peak_kind": "measured pinned copy" if ref else peak_kind})
        print(json.dumps(rows[-1]), flush=True)

    # single-token append (kvx_append): 4096 sequences x 8 kv heads, fp16
    B = 4096
    pool = torch.zeros((B, 2, HKV, PT, DIM), device="cuda", dtype=torch.float16)
    bt = torch.randperm(B, generator=g, device="cuda").to(torch.int32).view(B, 1).contiguous()
    pos = torch.randint(0, PT, (B,), generator=g, device="cuda", dtype=torch.int32)
    nk = torch.randn((B, HKV, DIM), generator=g, device="cuda", dtype=torch.float16)
    emit("append", "append_kernel", f"{B} sequences x 8 kv heads x 128, fp16, one token each",
         B * 2 * HKV * DIM * 2 * 2, lambda: kvx.append(pool, bt, pos, nk, nk))
    del pool, bt, pos, nk
    # chunked append: the append measurement's launch (32 sequences x 256 tokens)
    n = APPEND_CHUNK
    pages = BATCH * (n // PT + 1)
    pool = torch.zeros((pages, 2, HKV, PT, DIM), device="cuda", dtype=torch.float16)
    bt = torch.randperm(pages, generator=g, device="cuda").to(torch.int32).view(BATCH, -1).contiguous()
    starts = torch.randint(0, PT, (BATCH,), generator=g, device="cuda", dtype=torch.int32)
    rk = torch.randn((BATCH, n, HKV, DIM), generator=g, device="cuda", dtype=torch.float16)
    emit("append_chunk", "append_chunk_kernel", f"{BATCH} sequences x {n} tokens x 8 kv heads x 128, fp16",
         BATCH * n * HKV * DIM * 2 * 2 * 2, lambda: kvx.append_chunk(pool, bt, starts, rk, rk))
    del pool, bt, starts, rk
    # SIMT decode over an fp32 pool: batch 32 x 4096 tokens, 24 q-heads
    Bd, T = 32, 4096
    npg = T // PT
    pool = torch.randn((Bd * npg, 2, HKV, PT, DIM), generator=g, device="cuda", dtype=torch.float32)
    bt = torch.randperm(Bd * npg, generator=g, device="cuda").to(torch.int32).view(Bd, npg).contiguous()
    lens = torch.full((Bd,), T, dtype=torch.int32, device="cuda")
    q = torch.randn((Bd, HQ, DIM), generator=g, device="cuda", dtype=torch.float32)
    ws = kvx.decode_workspace(Bd, HQ, npg)
    out = torch.empty_like(q)
    emit("decode_fp32_pool", "paged_decode_kernel", "fp32 pool, batch 32 x 4096 tokens, 8 kv / 24 q heads",
         Bd * T * 2 * HKV * DIM * 4, lambda: kvx.decode(pool, bt, lens, q, out=out, workspace=ws))
    del pool, bt, lens, q, ws, out
    # codecs over 256 Mi elements
    N = 1 << 28
    x32 = torch.randn(N, generator=g, device="cuda")
    h16 = torch.empty(N, device="cuda", dtype=torch.int16)
    emit("fp16_trunc_encode", "encode_trunc_kernel", "256 Mi fp32 -> fp16 bits", N * 6,
         lambda: kvx.f32_to_f16_trunc(x32, out=h16))
    emit("fp16_trunc_decode", "f16_decode_tile_kernel", "256 Mi fp16 bits -> fp32", N * 6,
         lambda: kvx.f16_trunc_to_f32(h16, out=x32))
    emit("fp16_wrap_encode", "fp16_wrap_encode_kernel", "256 Mi fp32 -> fp16 bits", N * 6,
         lambda: kvx.fp16_wrap_encode(x32, out=h16))
    emit("fp16_wrap_decode", "f16_decode_tile_kernel", "256 Mi fp16 bits -> fp32", N * 6,
         lambda: kvx.fp16_wrap_decode(h16, out=x32))
    xh = x32[: N // 2].half()
    del h16
    blocks = xh.numel() // 2048
    nf4 = torch.empty(xh.numel() // 2, device="cuda", dtype=torch.uint8)
    st = torch.empty((blocks, 4), device="cuda", dtype=torch.float32)
    back = torch.empty_like(xh)
    emit("nf4_compress", "compress_2048_kernel (15 steps)", "128 Mi fp16 in 2048-element blocks",
         xh.numel() * 2 + nf4.numel() + blocks * 16, lambda: kvx.compress_nf4(xh, codes=nf4, stats=st))
    emit("nf4_decompress", "decompress_nf4_2048_kernel", "128 Mi fp16 out of 2048-element blocks",
         xh.numel() * 2 + nf4.numel() + blocks * 16,
         lambda: kvx.decompress_nf4(nf4, st, dtype=torch.float16, out=back))
    del x32, xh, nf4, st, back
    # victim selection over the tiered-eviction pool's 610,351 frames
    nfr = 610351
    stamps = torch.randint(0, 1 << 40, (nfr,), generator=g, device="cuda", dtype=torch.int64)
    emit("lru_select", "select_kernel", f"{nfr} u64 stamps", nfr * 8, lambda: kvx.lru_select(stamps))
    recs = torch.randint(0, 255, (nfr * 48,), generator=g, device="cuda", dtype=torch.uint8)
    emit("evict_select_lru", "select_kernel", f"{nfr} EvictionMetrics records (48 B)", nfr * 48,
         lambda: kvx.evict_select(0, recs))
    del stamps, recs
    # frame migration: 8192 frames of 64 KiB each way, pinned mapped host arena
    fb, nf = 65536, 8192
    link = pinned_peaks(nbytes=fb * nf)
    host = torch.empty(fb * nf, dtype=torch.uint8).pin_memory()
    dev = torch.empty(fb * nf, device="cuda", dtype=torch.uint8)
    perm_d = torch.randperm(nf, generator=g, device="cuda").to(torch.int32)
    perm_h = torch.randperm(nf, generator=g, device="cuda").to(torch.int32)
    hp = host.data_ptr()
    emit("migrate_h2d", "migrate_kernel", f"{nf} frames x 64 KiB, host -> device (scattered slots, 16 CTAs)",
         fb * nf, lambda: kvx.migrate_frames(dev, nf, hp, nf, perm_d, perm_h, fb, 1, 16), "host link",
         link["h2d"])
    emit("migrate_d2h", "migrate_kernel", f"{nf} frames x 64 KiB, device -> host (scattered slots, 16 CTAs)",
         fb * nf, lambda: kvx.migrate_frames(dev, nf, hp, nf, perm_d, perm_h, fb, 0, 16), "host link",
         link["d2h"])
    del host, dev
    # dense attention (cuda_attention drop-in), fp32: one key tile per CTA
    # (1024 x 1024) and 16 tiles per CTA (4096 x 4096)
    for T in (1024, 4096):
        qd, kd, vd = (torch.randn((T, DIM), generator=g, device="cuda") for _ in range(3))
        od = torch.empty_like(qd)
        ms = _timed_events(lambda: kvx.attention_dense(qd, kd, vd, out=od), iters, warm=1)
        flops = 4 * T * T * DIM
        rows.append({"kernels": "attention_dense", "kernel": "attention_umma_kernel + combine_splits_kernel",
                     "size": f"{T} x {T} x 128 fp32",
                     "us": round(ms * 1e3, 2), "TFLOPs": round(flops / (ms / 1e3) / 1e12, 2),
                     "note": "3 tcgen05 tf32 MMAs per product (3xTF32): the tensor pipe runs 3x the algorithmic flops"})
        print(json.dumps(rows[-1]), flush=True)


def main():
    global LAYERS
    args = parse()
    LAYERS = args.layers
    if args.impl == "reference":
        run_reference(args)
    elif args.shapes:
        run_shapes(args)
    elif args.kernels:
        run_kernel_profiles(args)
    elif args.config == 1:
        run_config1(args)
    elif args.config == 3:
        run_config3(args)
    elif args.config == 4:
        run_config4(args)
    elif args.config == 5:
        run_config5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
