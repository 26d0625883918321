"""kvx_decode_noalloc: the decode entry point for callers that cannot allocate
device memory when they decode (a JNI caller holding only the buffers it was
handed, an engine capped at a fixed memory budget, code under another
framework's allocator).  Its split-K scratch is a static device array inside
the library instead of a caller-provided workspace.

The test calls it through the C ABI (ctypes) and checks it against the
allocating entry point kvx_decode on the same inputs, twice in a row (the
shared array keeps the previous call's contents), within the tolerance of the
other decode tests.  This file is collected last so a failure here never
hides another test's result.
"""
import ctypes as C

import numpy as np
import pytest

import kvgen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-2


@pytest.fixture(scope="module")
def kvx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kvx as k
    assert k.lib.kvx_device_check() == 0, "not an sm_100 device"
    return k


def noalloc(kvx, pool, bt, lens, q, out, err, stats=None):
    kv = kvx.paged(pool, stats)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return kvx.lib.kvx_decode_noalloc(
        C.byref(kv), C.c_void_p(bt.data_ptr()), bt.shape[1], C.c_void_p(lens.data_ptr()),
        q.shape[0], q.shape[1], C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()),
        kvx.KVX_F32 if q.dtype == torch.float32 else kvx.KVX_F16, 0.0,
        C.c_void_p(err.data_ptr()), stream)


# (pool dtype, q/out dtype, batch, q-heads, context range, seed)
CASES = {
    # the library's own chunk choice already fits the scratch
    "f16-pool-f16-io": ("f16", torch.float16, 32, 24, (512, 8192), 515),
    "f16-pool-f32-io": ("f16", torch.float32, 32, 24, (512, 8192), 525),
    # 4096 rows of GQA-16 over contexts up to 16K tokens: the scratch holds 3
    # splits per row, so its floor (344 pages) overrides the chunk choice and
    # the CTAs run longer than the block-table slice they stage
    "f16-pool-scratch-bound": ("f16", torch.float16, 32, 128, (12288, 16384), 535),
    # fp32 pools take the SIMT kernel, whose chunks are short: the floor binds
    "f32-pool-scratch-bound": ("f32", torch.float32, 32, 24, (4096, 8192), 545),
    # int8 pools with per-block statistics
    "i8-pool": ("i8", torch.float16, 32, 24, (512, 8192), 555),
}


def make_case(case):
    kind, qdt, batch, hq, (lo, hi), seed = CASES[case]
    lens = kvgen.randint(seed, batch, lo, hi).astype(np.int32)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=seed + 1)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 2)
    shape = (num_pages, 2, 8, 16, 128)
    stats = None
    if kind == "i8":
        pool = torch.randint(-128, 128, shape, generator=g, device="cuda", dtype=torch.int8)
        lo_v = torch.randn((num_pages, 2, 8), generator=g, device="cuda") - 2.0
        scale = torch.rand((num_pages, 2, 8), generator=g, device="cuda") * 0.03 + 1e-3
        stats = torch.stack([lo_v, lo_v + 255 * scale, scale, lo_v], dim=-1).contiguous()
    else:
        pool = torch.randn(shape, generator=g, device="cuda",
                           dtype=torch.float16 if kind == "f16" else torch.float32)
    q = torch.randn((batch, hq, 128), generator=g, device="cuda", dtype=qdt)
    return pool, stats, torch.from_numpy(bt).cuda(), torch.from_numpy(lens).cuda(), q


@pytest.mark.parametrize("case", sorted(CASES))
def test_noalloc_matches_allocating_decode_twice(kvx, case):
    pool, stats, bt_d, lens_d, q = make_case(case)
    want = kvx.decode(pool, bt_d, lens_d, q, stats=stats).float().cpu().numpy()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        assert noalloc(kvx, pool, bt_d, lens_d, q, out, err, stats) == 0
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        excess = np.abs(got - want) - (ATOL + RTOL * np.abs(want))
        assert excess.max() <= 0, f"call {call}: max excess {excess.max():.3e}"
    assert err.item() == 0


def test_noalloc_allocates_nothing(kvx):
    """A warm call changes neither torch's allocator nor the device's free
    memory (cudaMemGetInfo)."""
    pool, stats, bt_d, lens_d, q = make_case("f16-pool-scratch-bound")
    out = torch.empty_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert noalloc(kvx, pool, bt_d, lens_d, q, out, err) == 0  # first call: address lookup
    torch.cuda.synchronize()
    torch_before = torch.cuda.memory_allocated()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert noalloc(kvx, pool, bt_d, lens_d, q, out, err) == 0
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == torch_before
    assert free_after == free_before
    assert err.item() == 0


def test_noalloc_rejects_what_its_scratch_cannot_hold(kvx):
    cap = kvx.lib.kvx_decode_noalloc_scratch_bytes()
    assert cap == 8 << 20
    # one split per (sequence, q-head) row needs 130 floats + a counter
    rows = cap // (130 * 4 + 4) + 1
    pool = torch.zeros((1, 2, 1, 16, 128), dtype=torch.float16, device="cuda")
    bt = torch.zeros((rows, 1), dtype=torch.int32, device="cuda")
    lens = torch.ones(rows, dtype=torch.int32, device="cuda")
    q = torch.zeros((rows, 1, 128), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert noalloc(kvx, pool, bt, lens, q, out, err) == -8
    assert kvx.lib.kvx_status_string(-8).startswith(b"request exceeds")
