"""The drop-in boundary as floyd's C code would use it: the moonlight_* shim
(floyd_b200/shim/moonlight_cuda.c) and the fm_* offload calls, compiled with
the system C compiler and linked against libfloyd_cuda.so, running floyd's
own Metal-test assertion sets (tests/c/test_moonlight_cuda.c mirrors
tests/test_moonlight_metal_{primitives,mla,moe,runtime}.c; tests/c/
test_fm_cuda.c mirrors tests/test_backend_metal.c) on a tiny Moonlight
container written by tests/golden/make_container.py."""
import os
import shutil
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "floyd_b200")


def cc():
    for c in (os.environ.get("CC_FOR_TESTS"), "/usr/bin/gcc", "gcc", "cc"):
        if c and shutil.which(c):
            return c
    pytest.fail("no C compiler")


def build(tmp, sources, out):
    import floyd_b200
    floyd_b200.lib()  # the library exists (built in-tree)
    cmd = [cc(), "-O2", "-Wall", "-I", os.path.join(ROOT, "include"), "-I",
           os.path.join(ROOT, "floyd_b200", "shim"), "-I", os.path.join(ROOT, "tests", "c")]
    cmd += [os.path.join(ROOT, s) for s in sources]
    cmd += ["-L", LIBDIR, "-lfloyd_cuda", "-Wl,-rpath," + LIBDIR, "-lm", "-o", os.path.join(tmp, out)]
    subprocess.run(cmd, check=True)
    return os.path.join(tmp, out)


@pytest.fixture(scope="module")
def container(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("moonlight_tiny"))
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_container
    make_container.build(d)
    return os.path.join(d, "model"), os.path.join(d, "oracle.safetensors")


def test_moonlight_shim_runs_floyd_metal_assertions(container, tmp_path):
    exe = build(str(tmp_path), ["tests/c/test_moonlight_cuda.c", "floyd_b200/shim/moonlight_cuda.c"],
                "test_moonlight_cuda")
    out = subprocess.run([exe, container[0], container[1]], capture_output=True, text=True, timeout=300)
    print(out.stdout)
    print(out.stderr)
    assert out.returncode == 0 and out.stdout.strip().endswith("OK"), out.stdout + out.stderr


def test_fm_offload_runs_floyd_backend_assertions(tmp_path):
    exe = build(str(tmp_path), ["tests/c/test_fm_cuda.c"], "test_fm_cuda")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(out.stdout)
    assert out.returncode == 0 and out.stdout.strip().endswith("OK"), out.stdout + out.stderr


def test_model_open_rejects_incomplete_containers(container, tmp_path):
    """A container without one of the tensors the model needs is refused
    with the tensor's name (moonlight_model.c reports missing files the same
    way); a missing directory or config fails cleanly."""
    import ctypes

    import floyd_b200
    from safetensors.numpy import load_file, save_file
    lib = floyd_b200.lib()
    err = ctypes.create_string_buffer(512)
    h = ctypes.c_void_p()
    assert not lib.fc_model_open(ctypes.byref(h), str(tmp_path / "none").encode(), 0, err, 512)
    assert b"config.json" in err.value
    bad = tmp_path / "bad"
    bad.mkdir()
    shutil.copy(os.path.join(container[0], "config.json"), bad / "config.json")
    t = load_file(os.path.join(container[0], "model.safetensors"))
    t.pop("model.layers.1.self_attn.o_proj.weight")
    t.pop("model.layers.1.self_attn.o_proj.weight.qs")
    save_file(t, str(bad / "model.safetensors"))
    assert not lib.fc_model_open(ctypes.byref(h), str(bad).encode(), 0, err, 512)
    assert b"model.layers.1.self_attn.o_proj.weight" in err.value
