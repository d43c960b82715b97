"""ctypes bindings of the CPU oracle (liboracle.so) - TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline and
--impl reference legs may import this module.  The CUDA backend never does.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_HARNESS = os.path.join(HERE, "_ref", "libref_harness.so")


def build():
    """Builds liboracle.so (and oracle/_ref when the reference is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        from floyd_b200._lib import FcAcceptConfig, FcModelConfig
        L = ctypes.CDLL(LIB)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        IP, FP = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float)
        sig = {
            "orc_philox4x32_10": (None, [ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32),
                                         ctypes.POINTER(ctypes.c_uint32)]),
            "orc_fp16_to_f32": (F, [ctypes.c_uint16]),
            "orc_f32_to_fp16": (ctypes.c_uint16, [F]),
            "orc_e8m0_to_f32": (F, [ctypes.c_uint8]),
            "orc_e2m1_to_f32": (F, [ctypes.c_uint8]),
            "orc_gemv": (None, [I, P, FP, FP, I, I, FP, I, FP]),
            "orc_rmsnorm": (None, [FP, FP, I, I, F, FP]),
            "orc_rope": (None, [FP, FP, I, I, F]),
            "orc_route": (I, [FP, FP, I, I, I, I, F, IP, IP, FP]),
            "orc_argmax": (I, [FP, I]),
            "orc_accept_greedy": (I, [IP, IP, I]),
            "orc_accept_sample": (I, [FP, I, IP, I, F, ctypes.c_uint64, ctypes.c_uint64, IP]),
            "orc_accept_uniform": (F, [ctypes.c_uint64, ctypes.c_uint64, I]),
            "orc_gumbel": (F, [ctypes.c_uint64, ctypes.c_uint64, I, I]),
            "orc_model_create": (P, [ctypes.POINTER(FcModelConfig), ctypes.c_uint64]),
            "orc_model_free": (None, [P]),
            "orc_model_set_f32": (I, [P, ctypes.c_char_p, FP, ctypes.c_size_t]),
            "orc_model_get_tensor": (ctypes.c_size_t, [P, ctypes.c_char_p, I, P, ctypes.c_size_t]),
            "orc_session_create": (P, [P, I, I]),
            "orc_session_free": (None, [P]),
            "orc_session_position": (I, [P]),
            "orc_session_set_position": (None, [P, I]),
            "orc_session_seed_context": (I, [P, I, ctypes.c_uint64]),
            "orc_session_seed_range": (I, [P, I, I, ctypes.c_uint64]),
            "orc_session_forward": (I, [P, IP, I, FP, FP, IP]),
            "orc_session_copy_kv": (I, [P, I, FP, FP, I]),
            "orc_session_verify": (I, [P, IP, I, ctypes.POINTER(FcAcceptConfig), IP, IP, IP, FP, IP]),
            "orc_session_drafts": (I, [P, IP, I]),
            "orc_dspark_rows": (I, [P, I, I]),
            "orc_dspark_propose": (I, [P, I, I, IP, FP]),
            "orc_part_times": (None, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _ip(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


def philox(counter, key):
    c = (ctypes.c_uint32 * 4)(*counter)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    lib().orc_philox4x32_10(c, k, o)
    return list(o)


def gemv(fmt, values, scales, x, f32=None):
    """y[s][o] for logical values [O][K] (int8) and fp32 scales [O][K/32]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    S, K = x.shape
    if fmt == 0:
        f32 = np.ascontiguousarray(f32, dtype=np.float32)
        O = f32.shape[0]
        vp, sp, fp = None, None, _fp(f32)
    else:
        values = np.ascontiguousarray(values, dtype=np.int8)
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        O = values.shape[0]
        vp, sp, fp = values.ctypes.data_as(ctypes.c_void_p), _fp(scales), None
    y = np.zeros((S, O), dtype=np.float32)
    lib().orc_gemv(fmt, vp, sp, fp, O, K, _fp(x), S, _fp(y))
    return y


def route(logits, bias, top_k, score_fn, normalize, scale, fixed=None):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    E = len(logits)
    idx = np.zeros(top_k, dtype=np.int32)
    w = np.zeros(top_k, dtype=np.float32)
    bp = _fp(np.ascontiguousarray(bias, dtype=np.float32)) if bias is not None else None
    fx = np.ascontiguousarray(fixed, dtype=np.int32) if fixed is not None else None
    n = lib().orc_route(_fp(logits), bp, E, top_k, score_fn, normalize, scale,
                        _ip(fx) if fx is not None else None, _ip(idx), _fp(w))
    return n, idx, w


def part_times():
    """(attention s, ffn s) spent by oracle forwards since the last call."""
    a, f = ctypes.c_double(), ctypes.c_double()
    lib().orc_part_times(ctypes.byref(a), ctypes.byref(f))
    return a.value, f.value


class OracleModel:
    def __init__(self, config, seed):
        from floyd_b200._lib import FcModelConfig
        from floyd_b200.configs import model_fields
        self.config = dict(config)
        self._cfg = FcModelConfig.from_dict(model_fields(config))
        self.handle = lib().orc_model_create(ctypes.byref(self._cfg), ctypes.c_uint64(seed))
        if not self.handle:
            raise RuntimeError("oracle model creation failed")

    def set_f32(self, name, data):
        data = np.ascontiguousarray(data, dtype=np.float32)
        if not lib().orc_model_set_f32(self.handle, name.encode(), _fp(data), data.size):
            raise RuntimeError(f"oracle: cannot set {name}")

    def get_tensor(self, name, nbytes, scales=False):
        out = np.zeros(nbytes, dtype=np.uint8)
        n = lib().orc_model_get_tensor(self.handle, name.encode(), int(scales),
                                       out.ctypes.data_as(ctypes.c_void_p), nbytes)
        if not n:
            raise RuntimeError(f"oracle: no tensor {name}")
        return out[:n]

    def close(self):
        if self.handle:
            lib().orc_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OracleSession:
    def __init__(self, model, context_size, kv_fp16=True):
        self.model = model
        self.handle = lib().orc_session_create(model.handle, context_size, int(kv_fp16))
        if not self.handle:
            raise RuntimeError("oracle session creation failed")

    def seed_context(self, positions, seed):
        if not lib().orc_session_seed_context(self.handle, positions, ctypes.c_uint64(seed)):
            raise RuntimeError("oracle seed failed")

    def seed_range(self, start, end, seed):
        """Synthetic KV for positions [start, end) (position -> max(position, end))."""
        if not lib().orc_session_seed_range(self.handle, start, end, ctypes.c_uint64(seed)):
            raise RuntimeError("oracle seed failed")

    def forward(self, ids, want_layers=False, want_routes=False):
        c = self.model.config
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        rows = len(ids)
        logits = np.zeros((rows, c["vocab_size"]), dtype=np.float32)
        layers = (np.zeros((c["layer_count"], rows, c["hidden_size"]), dtype=np.float32)
                  if want_layers else None)
        routes = (np.zeros((c["layer_count"], rows, c["experts_per_token"]), dtype=np.int32)
                  if want_routes else None)
        ok = lib().orc_session_forward(self.handle, _ip(ids), rows, _fp(logits),
                                       _fp(layers) if layers is not None else None,
                                       _ip(routes) if routes is not None else None)
        if not ok:
            raise RuntimeError("oracle forward failed")
        return logits, layers, routes

    def drafts(self):
        """MTP drafter proposals of the last verify."""
        out = np.zeros(64, dtype=np.int32)
        n = lib().orc_session_drafts(self.handle, _ip(out), 64)
        return out[:n].tolist()

    def verify(self, ids, mode=0, temperature=1.0, seed=0, counter=0):
        from floyd_b200._lib import FcAcceptConfig
        c = self.model.config
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        k = len(ids) - 1
        acc = FcAcceptConfig(mode, temperature, seed, counter)
        emitted = np.zeros(len(ids), dtype=np.int32)
        n = ctypes.c_int()
        nxt = ctypes.c_int()
        logits = np.zeros((len(ids), c["vocab_size"]), dtype=np.float32)
        tops = np.zeros(len(ids), dtype=np.int32)
        if not lib().orc_session_verify(self.handle, _ip(ids), k, ctypes.byref(acc), _ip(emitted),
                                        ctypes.byref(n), ctypes.byref(nxt), _fp(logits), _ip(tops)):
            raise RuntimeError("oracle verify failed")
        return emitted[:n.value].tolist(), nxt.value, logits, tops

    def copy_kv(self, layer):
        c = self.model.config
        P = self.position()
        lat = np.zeros((max(P, 1), c["kv_lora_rank"]), dtype=np.float32)
        rope = np.zeros((max(P, 1), c["qk_rope_dim"]), dtype=np.float32)
        lib().orc_session_copy_kv(self.handle, layer, _fp(lat), _fp(rope), max(P, 1))
        return lat[:P], rope[:P]

    def dspark_rows(self, p0, r):
        if not lib().orc_dspark_rows(self.handle, p0, r):
            raise RuntimeError("oracle dspark rows failed")

    def dspark_propose(self, p, input_id):
        out = np.zeros(5, dtype=np.int32)
        conf = np.zeros(5, dtype=np.float32)
        if not lib().orc_dspark_propose(self.handle, p, input_id, _ip(out), _fp(conf)):
            raise RuntimeError("oracle dspark propose failed")
        return out.tolist(), conf

    def position(self):
        return lib().orc_session_position(self.handle)

    def set_position(self, p):
        lib().orc_session_set_position(self.handle, p)

    def close(self):
        if self.handle:
            lib().orc_session_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
