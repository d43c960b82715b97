"""The C-ABI library loads and exports every function include/*.h declares;
without a GPU every entry point fails cleanly with an error message (no CPU
fallback, no crash)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b((?:fc|fm)_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    # static inline helpers of floyd_synth.h are not exported
    return {n for n in names if not n.startswith("fc_synth") and n not in
            ("fc_tensor_id", "fc_mulhilo32", "fc_philox4x32_10")}


def test_library_exports_every_declared_symbol():
    import floyd_b200
    lib = floyd_b200.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(floyd_b200._lib.SIGNATURES) == declared_functions()


def test_library_is_built_for_sm100a_only():
    import floyd_b200
    from floyd_b200 import build
    text = open(build.__file__).read()
    assert "arch=compute_100a,code=sm_100a" in text
    assert os.path.exists(floyd_b200._lib.LIB_PATH)


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES", None) is None and
                    os.path.exists("/dev/nvidia0"), reason="a GPU is present")
def test_without_gpu_model_creation_fails_cleanly():
    import floyd_b200
    from floyd_b200 import CONFIGS
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(floyd_b200.FloydError) as exc:
        floyd_b200.Model(CONFIGS["c1_tiny"])
    assert "CUDA" in str(exc.value) or "device" in str(exc.value)


def test_invalid_configs_are_rejected_before_allocation():
    import floyd_b200
    from floyd_b200 import CONFIGS, scaled
    bad = scaled(CONFIGS["c1_tiny"], hidden_size=1000)
    with pytest.raises(floyd_b200.FloydError) as exc:
        floyd_b200.Model(bad)
    assert "multiple of 32" in str(exc.value)
    bad = scaled(CONFIGS["c1_tiny"], kv_lora_rank=384)
    with pytest.raises(floyd_b200.FloydError):
        floyd_b200.Model(bad)


def test_host_entry_points_reject_null_arguments():
    import floyd_b200
    lib = floyd_b200.lib()
    err = ctypes.create_string_buffer(128)
    assert lib.fc_model_create(None, None, 0, err, len(err)) == 0
    assert lib.fc_session_create(None, None, None, err, len(err)) == 0
    assert lib.fc_session_position(None) == 0
    assert lib.fc_session_create_batch(None, None, None, err, len(err)) == 0
    assert lib.fc_session_batch_seed(None, 0, 0, 1, 0, err, len(err)) == 0
    assert lib.fc_session_verify_batch(None, None, 3, None, None, None, err, len(err)) == 0
    assert b"invalid" in err.value
    assert lib.fc_session_batch_position(None, 0) == -1
    assert lib.fc_session_batch_rollback(None, 0, 0, err, len(err)) == 0
    assert lib.fc_runtime_argmax(None, 10) == -1
    lib.fc_model_close(None)
    lib.fc_session_destroy(None)


def test_batch_page_table_layout():
    """Host-side page table of batch sessions: the shared prefix pages are the
    same physical pages for every sequence, the other pages are private and
    disjoint, and every entry is a valid physical page."""
    import numpy as np
    import floyd_b200
    lib = floyd_b200.lib()
    ctx, nseq, shared = 16448, 8, 1024
    pps = (ctx + 63) // 64
    table = np.full(nseq * pps, -1, dtype=np.int32)
    ip = ctypes.POINTER(ctypes.c_int)
    pages = lib.fc_test_batch_page_table(ctx, nseq, shared, table.ctypes.data_as(ip), table.size)
    sp = shared // 64
    assert pages == sp + nseq * (pps - sp)
    t = table.reshape(nseq, pps)
    assert (t >= 0).all() and (t < pages).all()
    assert (t[:, :sp] == np.arange(sp)).all()                       # one shared copy
    private = t[:, sp:].ravel()
    assert len(np.unique(private)) == private.size                   # disjoint tails
    assert not np.intersect1d(private, np.arange(sp)).size
    # an ordinary session's table is the identity
    one = np.zeros(pps, dtype=np.int32)
    assert lib.fc_test_batch_page_table(ctx, 1, 0, one.ctypes.data_as(ip), one.size) == pps
    assert (one == np.arange(pps)).all()
    # invalid requests
    assert lib.fc_test_batch_page_table(ctx, nseq, 100, table.ctypes.data_as(ip), table.size) == -1
    assert lib.fc_test_batch_page_table(ctx, nseq, shared, table.ctypes.data_as(ip), 10) == -1
