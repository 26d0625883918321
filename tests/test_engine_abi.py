"""The engine behind the reference's C ABI (NativeEngineApi).

C tests ported from the reference's native-engine/llama_wrapper/tests/*.c
run as separate processes that dlopen libadaptive_engine.so by name, as the
reference's JNI loader does.  The export check needs no GPU; the others
start the engine and so run on the GPU.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "adaptive-hierarchical-llm-inference-engine_b200")
CDIR = os.path.join(ROOT, "tests", "cpp")


@pytest.fixture(scope="module")
def built():
    subprocess.run(["make", "-s", "-C", CDIR], check=True)
    return os.path.join(CDIR, "_build")


def run(built, name, tmp_path, **env):
    e = dict(os.environ)
    e["LD_LIBRARY_PATH"] = PKG + ":" + e.get("LD_LIBRARY_PATH", "")
    e.setdefault("ADAPTIVELLM_KV_LAYERS", "8")
    e.setdefault("ADAPTIVELLM_KV_PAGES", "64")
    e["ADAPTIVELLM_KV_OFFLOAD_DIR"] = str(tmp_path)
    e.update(env)
    r = subprocess.run([os.path.join(built, name)], env=e, capture_output=True, text=True,
                       timeout=120)
    return r.returncode, r.stdout + r.stderr


def test_engine_exports_get_api(built, tmp_path):
    rc, out = run(built, "test_adaptive_engine_exports", tmp_path)
    assert rc == 0, out


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["test_kv_operations", "test_pinned_eviction",
                                  "test_prefetch_evict", "test_concurrent_pin_unpin"])
def test_reference_c_tests(built, tmp_path, name):
    rc, out = run(built, name, tmp_path)
    assert rc == 0, out


@pytest.mark.gpu
def test_kv_operations_under_memory_pressure(built, tmp_path):
    # two device slabs for eight layers: every move to the GPU evicts the LRU layer
    rc, out = run(built, "test_kv_operations", tmp_path, ADAPTIVELLM_KV_GPU_LAYERS="2")
    assert rc == 0, out
