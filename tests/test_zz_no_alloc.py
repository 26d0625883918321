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


def noalloc(kvx, pool, bt, lens, q, out, err):
    kv = kvx.paged(pool)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return kvx.lib.kvx_decode_noalloc(
        C.byref(kv), C.c_void_p(bt.data_ptr()), bt.shape[1], C.c_void_p(lens.data_ptr()),
        q.shape[0], q.shape[1], C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()),
        kvx.KVX_F32 if q.dtype == torch.float32 else kvx.KVX_F16, 0.0,
        C.c_void_p(err.data_ptr()), stream)


@pytest.mark.parametrize("io", ["f16", "f32"])
def test_noalloc_matches_allocating_decode_twice(kvx, io):
    lens = kvgen.randint(515, 32, 512, 8192).astype(np.int32)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=516)
    dtype = torch.float16 if io == "f16" else torch.float32
    g = torch.Generator(device="cuda")
    g.manual_seed(517)
    pool = torch.randn((num_pages, 2, 8, 16, 128), generator=g, device="cuda", dtype=torch.float16)
    q = torch.randn((32, 24, 128), generator=g, device="cuda", dtype=dtype)
    bt_d = torch.from_numpy(bt).cuda()
    lens_d = torch.from_numpy(lens).cuda()
    want = kvx.decode(pool, bt_d, lens_d, q).float().cpu().numpy()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        assert noalloc(kvx, pool, bt_d, lens_d, q, out, err) == 0
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        excess = np.abs(got - want) - (ATOL + RTOL * np.abs(want))
        assert excess.max() <= 0, f"call {call}: max excess {excess.max():.3e}"
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
