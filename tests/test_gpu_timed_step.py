"""The bench's timed step, checked end to end against the oracle.

bench.make_decode_step is the exact function bench.py times: 28 layers of
kvx.append_decode launched back to back on one stream (programmatic
dependent launch, each CTA releasing the next launch at its start), one
decode workspace shared by all layers, positions for every step prepared up
front.  Here it runs two steps back to back (the second step's first launch
overlaps the first step's last one) at the Llama-3.2-3B KV geometry (8 KV
heads x 128, 24 q-heads, fp16 pools with randomly permuted pages) with
batch 8 and contexts of 2,048-8,192 tokens: contexts above 4,096 tokens
exceed the 256-page chunk cap, so those sequences are split over several
CTAs and their split combine runs under the overlapped launches.

Every layer's output of both steps must match the oracle's append + paged
GQA decode (KVManager::save_page, cache/kv_cache.cpp:111-127, then
TensorOps::attention, runtime/tensor_ops.cpp:179-219) within
|gpu - ref| <= 1e-2 + 1e-3 |ref|, and every layer's pool must equal the
oracle's appends bit for bit.
"""
import os
import sys

import numpy as np
import pytest

import kvgen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

RTOL, ATOL = 1e-3, 1e-2


@pytest.fixture(scope="module")
def kvx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kvx as k
    assert k.lib.kvx_device_check() == 0, "not an sm_100 device"
    return k


def assert_close(got, want, what):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    excess = np.abs(got - want) - (ATOL + RTOL * np.abs(want))
    assert excess.max() <= 0, f"{what}: max excess {excess.max():.3e}, max abs err {np.abs(got - want).max():.3e}"


def test_bench_step_chain_matches_oracle(kvx, oracle):
    import bench
    L, B, HKV, HQ, STEPS = bench.LAYERS, 8, 8, 24, 2
    assert L == 28
    lens0 = kvgen.randint(606, B, 2048, 8192)
    assert lens0.max() > 4096 and lens0.min() >= 2048
    bt, num_pages = kvgen.paged_layout(lens0, 16, STEPS, seed=607)
    g = torch.Generator(device="cuda")
    g.manual_seed(608)
    pools = [torch.randn((num_pages, 2, HKV, 16, 128), generator=g, device="cuda", dtype=torch.float16)
             for _ in range(L)]
    pools0 = [p.clone() for p in pools]
    q = torch.randn((L, B, HQ, 128), generator=g, device="cuda", dtype=torch.float16)
    nk = torch.randn((L, B, HKV, 128), generator=g, device="cuda", dtype=torch.float16)
    nv = torch.randn((L, B, HKV, 128), generator=g, device="cuda", dtype=torch.float16)
    positions = torch.from_numpy(np.stack([lens0 + k for k in range(STEPS)]).astype(np.int32)).cuda()
    outs = [torch.full((L, B, HQ, 128), float("nan"), device="cuda", dtype=torch.float16) for _ in range(STEPS)]
    bt_d = torch.from_numpy(bt).cuda()
    ws = kvx.decode_workspace(B, HQ, bt.shape[1])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    step = bench.make_decode_step(kvx, pools, bt_d, positions, nk, nv, q, ws, err, outs)
    for k in range(STEPS):
        step(k)
    torch.cuda.synchronize()
    assert err.item() == 0
    # every launch left the shared split counters at zero: the workspace is
    # [B][HQ][splits][128] partial sums, [B][HQ][splits][2] (max, sum), then
    # the counters, with splits = ceil(max_pages / 4)
    splits = (bt.shape[1] + 3) // 4
    ctr0 = B * HQ * splits * 130
    counters = ws.view(torch.int32)[ctr0:ctr0 + B * HQ]
    assert int(counters.abs().sum().item()) == 0

    pos_np = positions.cpu().numpy()
    for l in range(L):
        host = pools0[l].cpu().numpy()
        k_l, v_l, q_l = nk[l].cpu().numpy(), nv[l].cpu().numpy(), q[l].float().cpu().numpy()
        for k in range(STEPS):
            oracle.append(host, bt, pos_np[k], k_l, v_l, 16)
            ref = oracle.paged_decode(host, bt, (lens0 + k + 1).astype(np.int32), q_l)
            assert_close(outs[k][l].float().cpu().numpy(), ref, f"layer {l} step {k}")
        assert np.array_equal(pools[l].cpu().numpy().view(np.uint16), host.view(np.uint16)), f"pool of layer {l}"


def test_bench_parity_sample_passes_on_a_correct_run(kvx):
    """bench.ParitySample, the check bench.py prints as "parity", reports
    ok for the chain above (one rank)."""
    import bench
    L, B, HKV, HQ, STEPS = 4, 8, 8, 24, 3
    lens0 = kvgen.randint(646, B, 512, 4096)
    bt, num_pages = kvgen.paged_layout(lens0, 16, STEPS, seed=647)
    g = torch.Generator(device="cuda")
    g.manual_seed(648)
    pools = [torch.randn((num_pages, 2, HKV, 16, 128), generator=g, device="cuda", dtype=torch.float16)
             for _ in range(L)]
    q = torch.randn((L, B, HQ, 128), generator=g, device="cuda", dtype=torch.float16)
    nk = torch.randn((L, B, HKV, 128), generator=g, device="cuda", dtype=torch.float16)
    nv = torch.randn((L, B, HKV, 128), generator=g, device="cuda", dtype=torch.float16)
    positions = torch.from_numpy(np.stack([lens0 + k for k in range(STEPS)]).astype(np.int32)).cuda()
    outs = [torch.empty((L, B, HQ, 128), device="cuda", dtype=torch.float16)]
    bt_d = torch.from_numpy(bt).cuda()
    ws = kvx.decode_workspace(B, HQ, bt.shape[1])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    check = bench.ParitySample(bt, lens0, HKV, HQ, 1, 0, pools)
    step = bench.make_decode_step(kvx, pools, bt_d, positions, nk, nv, q, ws, err, outs)
    for k in range(STEPS):
        step(k)
    torch.cuda.synchronize()
    res = check.verify(q, nk, nv, positions, outs[0], None, None)
    assert res["ok"] and res["pool_pages_bitexact"] and res["rows_checked"] == 3 * 4 * HQ, res


def test_signal_word_and_stream_wait(kvx):
    """The completion word of a signalled launch: after the launch it holds
    the epoch and the counter is back at zero; a stream that waits for the
    word before reading the output reads the finished rows."""
    B, HKV, HQ = 8, 8, 24
    lens0 = kvgen.randint(616, B, 1024, 8192)
    bt, num_pages = kvgen.paged_layout(lens0, 16, 1, seed=617)
    g = torch.Generator(device="cuda")
    g.manual_seed(618)
    pool = torch.randn((num_pages, 2, HKV, 16, 128), generator=g, device="cuda", dtype=torch.float16)
    q = torch.randn((B, HQ, 128), generator=g, device="cuda", dtype=torch.float16)
    nk = torch.randn((B, HKV, 128), generator=g, device="cuda", dtype=torch.float16)
    pos = torch.from_numpy(lens0.astype(np.int32)).cuda()
    bt_d = torch.from_numpy(bt).cuda()
    ws = kvx.decode_workspace(B, HQ, bt.shape[1])
    done = torch.zeros(2, dtype=torch.int32, device="cuda")
    side = torch.cuda.Stream()
    want = kvx.append_decode(pool.clone(), bt_d, pos, nk, nk, q, workspace=kvx.decode_workspace(B, HQ, bt.shape[1]))
    for epoch in (1, 2, 3):
        out = torch.full_like(q, float("nan"))
        kvx.append_decode_signal(pool, bt_d, pos, nk, nk, q, done, epoch, out=out, workspace=ws)
        with torch.cuda.stream(side):
            kvx.stream_wait_geq(done[1:], epoch, stream=side)
            copy = out.clone()
        torch.cuda.synchronize()
        assert done.tolist() == [0, epoch]
        assert torch.equal(copy, out)
        assert torch.equal(out, want)
