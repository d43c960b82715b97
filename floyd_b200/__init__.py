"""floyd_b200 - B200-native (sm_100a) backend for floyd's speculative-decode
verify step.

The product is the C ABI in include/floyd_cuda.h (libfloyd_cuda.so).  This
module is a thin host mirror of that ABI for Python callers and tests; its
method names follow floyd's Metal session API (moonlight_metal.h:46-66):
    Model.open_synthetic / Model.close / Model.info / Model.device_name
    Session.prefill / append / decode / verify / rollback / reset /
    position / stats
Every call goes to the CUDA library; there is no CPU path.
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import (ACCEPT_GREEDY, ACCEPT_SAMPLE, FMT_F32, FMT_MXFP4, FMT_Q4, FMT_Q8,
                   SCORE_SIGMOID, SCORE_SOFTMAX, SCORE_SQRT_SOFTPLUS, FcAcceptConfig,
                   FcModelConfig, FcOptions, FcBatchOptions)
from .configs import CONFIGS, model_fields, scaled, step_bytes

__all__ = ["Model", "Session", "BatchSession", "FloydError", "CONFIGS", "blocks_to_logical", "BLOCKS_Q8_0", "BLOCKS_MXFP4", "model_fields", "scaled", "step_bytes",
           "FMT_F32", "FMT_Q8", "FMT_Q4", "FMT_MXFP4", "ACCEPT_GREEDY", "ACCEPT_SAMPLE",
           "SCORE_SOFTMAX", "SCORE_SIGMOID", "SCORE_SQRT_SOFTPLUS", "lib"]


class FloydError(RuntimeError):
    pass


BLOCKS_Q8_0, BLOCKS_MXFP4 = 8, 39  # FcBlockType (ggml type ids)


def blocks_to_logical(block_type, blocks, rows, cols):
    """Host conversion of GGUF blocks to (values, group scales) in the logical
    layout of Model.set_tensor (fc_blocks_to_logical; no GPU needed)."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    if block_type == BLOCKS_Q8_0:
        values = np.zeros((rows, cols), dtype=np.int8)
        scales = np.zeros((rows, cols // 32), dtype=np.uint16)
    else:
        values = np.zeros((rows, cols // 2), dtype=np.uint8)
        scales = np.zeros((rows, cols // 32), dtype=np.uint8)
    err = _err()
    if not lib().fc_blocks_to_logical(int(block_type), blocks.ctypes.data_as(ctypes.c_void_p), blocks.nbytes,
                                      rows, cols, values.ctypes.data_as(ctypes.c_void_p),
                                      scales.ctypes.data_as(ctypes.c_void_p), err, len(err)):
        raise FloydError(err.value.decode())
    return values, scales


def io_bytes():
    """(h2d, d2h) bytes of the parameter and result records every forward
    pass copies (fc_io_bytes)."""
    h, d = ctypes.c_size_t(), ctypes.c_size_t()
    lib().fc_io_bytes(ctypes.byref(h), ctypes.byref(d))
    return int(h.value), int(d.value)


def accept_trials(logits, ids, mode=ACCEPT_SAMPLE, temperature=1.0, seed=0, counter=0, trials=1):
    """The device acceptance kernels on given logits [rows][vocab] for
    `trials` consecutive Philox counters (fc_test_accept); returns
    (commits, next_tokens) arrays."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    commits = np.zeros(trials, dtype=np.int32)
    nxt = np.zeros(trials, dtype=np.int32)
    acc = _lib.FcAcceptConfig(mode, temperature, seed, counter)
    e = _err()
    if not lib().fc_test_accept(logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), rows, vocab,
                                _i32(ids)[1], ctypes.byref(acc), trials, _i32(commits)[1],
                                _i32(nxt)[1], e, len(e)):
        raise FloydError(e.value.decode())
    return commits, nxt


def lib():
    return _lib.load()


def _err():
    return ctypes.create_string_buffer(512)


def _i32(a):
    a = np.ascontiguousarray(a, dtype=np.int32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


def _f32_out(n):
    a = np.zeros(n, dtype=np.float32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class Model:
    """A resident model (fc_model_*)."""

    def __init__(self, config, device=0, seed=None, rank=0, world=1):
        self._lib = lib()
        self.config = dict(config)
        cfg = FcModelConfig.from_dict(model_fields(config))
        handle = ctypes.c_void_p()
        err = _err()
        if world > 1:
            ok = self._lib.fc_model_create_ep(ctypes.byref(handle), ctypes.byref(cfg), device,
                                              rank, world, err, len(err))
        else:
            ok = self._lib.fc_model_create(ctypes.byref(handle), ctypes.byref(cfg), device, err,
                                           len(err))
        if not ok:
            raise FloydError(err.value.decode())
        self.handle = handle
        if seed is not None:
            self.fill_synthetic(seed)

    def fill_synthetic(self, seed):
        err = _err()
        if not self._lib.fc_model_fill_synthetic(self.handle, ctypes.c_uint64(seed), err, len(err)):
            raise FloydError(err.value.decode())

    def set_tensor(self, name, data):
        data = np.ascontiguousarray(data)
        err = _err()
        if not self._lib.fc_model_set_tensor(self.handle, name.encode(), data.ctypes.data_as(ctypes.c_void_p),
                                             data.nbytes, err, len(err)):
            raise FloydError(err.value.decode())

    def set_tensor_blocks(self, name, block_type, blocks):
        """One q8 / MXFP4 matrix from GGUF Q8_0 / MXFP4 blocks (exact)."""
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        err = _err()
        if not self._lib.fc_model_set_tensor_blocks(self.handle, name.encode(), int(block_type),
                                                    blocks.ctypes.data_as(ctypes.c_void_p), blocks.nbytes,
                                                    err, len(err)):
            raise FloydError(err.value.decode())

    def set_tensor_rowscale(self, name, values, row_scales):
        """One int8 / int4 matrix of the Moonlight container (per-row fp32 scales)."""
        values = np.ascontiguousarray(values, dtype=np.uint8)
        row_scales = np.ascontiguousarray(row_scales, dtype=np.float32)
        err = _err()
        if not self._lib.fc_model_set_tensor_rowscale(
                self.handle, name.encode(), values.ctypes.data_as(ctypes.c_void_p), values.nbytes,
                row_scales.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(row_scales), err, len(err)):
            raise FloydError(err.value.decode())

    def get_tensor(self, name, nbytes, dtype=np.uint8):
        out = np.zeros(nbytes, dtype=np.uint8)
        err = _err()
        if not self._lib.fc_model_get_tensor(self.handle, name.encode(), out.ctypes.data_as(ctypes.c_void_p),
                                             nbytes, err, len(err)):
            raise FloydError(err.value.decode())
        return out.view(dtype)

    def info(self):
        return self._lib.fc_model_info(self.handle).to_dict()

    def device_name(self):
        return self._lib.fc_device_name(self.handle).decode()

    def close(self):
        if getattr(self, "handle", None):
            self._lib.fc_model_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """A decoding session (fc_session_*)."""

    def __init__(self, model, context_size, max_batch):
        self._lib = model._lib
        self.model = model
        self.vocab = model.config["vocab_size"]
        opt = FcOptions(context_size, max_batch)
        handle = ctypes.c_void_p()
        err = _err()
        if not self._lib.fc_session_create(ctypes.byref(handle), model.handle, ctypes.byref(opt), err,
                                           len(err)):
            raise FloydError(err.value.decode())
        self.handle = handle

    def _check(self, ok, err):
        if not ok:
            raise FloydError(err.value.decode())

    def prefill(self, ids):
        ids, p = _i32(ids)
        out, op = _f32_out(self.vocab)
        err = _err()
        self._check(self._lib.fc_session_prefill(self.handle, p, len(ids), op, err, len(err)), err)
        return out

    def append(self, ids):
        ids, p = _i32(ids)
        out, op = _f32_out(self.vocab)
        err = _err()
        self._check(self._lib.fc_session_append(self.handle, p, len(ids), op, err, len(err)), err)
        return out

    def decode(self, token):
        out, op = _f32_out(self.vocab)
        err = _err()
        self._check(self._lib.fc_session_decode(self.handle, int(token), op, err, len(err)), err)
        return out

    def verify(self, ids, mode=ACCEPT_GREEDY, temperature=1.0, seed=0, counter=0,
               want_logits=False):
        """Returns (emitted tokens, next_token, last_logits or None)."""
        ids, p = _i32(ids)
        k = len(ids) - 1
        acc = FcAcceptConfig(mode, temperature, seed, counter)
        emitted = np.zeros(len(ids), dtype=np.int32)
        n = ctypes.c_int()
        nxt = ctypes.c_int()
        logits, lp = (_f32_out(self.vocab) if want_logits else (None, None))
        err = _err()
        self._check(self._lib.fc_session_verify(
            self.handle, p, k, ctypes.byref(acc), emitted.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
            ctypes.byref(n), ctypes.byref(nxt), lp, err, len(err)), err)
        return emitted[:n.value].tolist(), nxt.value, logits

    def rollback(self, position):
        err = _err()
        self._check(self._lib.fc_session_rollback(self.handle, int(position), err, len(err)), err)

    def exchange_wait_ms(self):
        """Device time the expert-exchange combines spent waiting for the
        peers since the previous call (fc_session_exchange_wait_ms)."""
        return float(self._lib.fc_session_exchange_wait_ms(self.handle))

    def last_kernel_count(self):
        """Kernels launched by the last forward pass (graph kernel nodes)."""
        return int(self._lib.fc_session_last_kernel_count(self.handle))

    def drafts(self):
        """The on-device drafter's proposals from the last verify."""
        out = np.zeros(8, dtype=np.int32)
        n = self._lib.fc_session_drafts(self.handle, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), 8)
        return out[:max(n, 0)].tolist()

    def ep_handle(self):
        """This rank's expert-parallel receive-region handle (bytes)."""
        buf = ctypes.create_string_buffer(64)
        err = _err()
        self._check(self._lib.fc_session_ep_handle(self.handle, buf, 64, err, len(err)), err)
        return buf.raw

    def ep_connect(self, handles):
        """Connects to every rank's region; `handles` in rank order."""
        blob = b"".join(handles)
        err = _err()
        self._check(self._lib.fc_session_ep_connect(self.handle, blob, len(handles), err, len(err)), err)

    def seed_context(self, positions, seed):
        err = _err()
        self._check(self._lib.fc_session_seed_context(self.handle, int(positions),
                                                      ctypes.c_uint64(seed), err, len(err)), err)

    def row_logits(self, rows):
        out = np.zeros((rows, self.vocab), dtype=np.float32)
        if not self._lib.fc_session_copy_row_logits(
                self.handle, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), rows):
            raise FloydError("row logits unavailable")
        return out

    def copy_kv(self, layer):
        cfg = self.model.config
        P = self.position()
        lat = np.zeros((max(P, 1), cfg["kv_lora_rank"]), dtype=np.float32)
        rope = np.zeros((max(P, 1), cfg["qk_rope_dim"]), dtype=np.float32)
        if not self._lib.fc_test_copy_kv(self.handle, layer,
                                         lat.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                         rope.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), max(P, 1)):
            raise FloydError("copy_kv failed")
        return lat[:P], rope[:P]

    def routes(self, layer, rows):
        out = np.zeros((rows, self.model.config["experts_per_token"]), dtype=np.int32)
        if not self._lib.fc_test_copy_routes(self.handle, layer,
                                             out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), rows):
            raise FloydError("copy_routes failed")
        return out

    def layer_outputs(self, rows):
        cfg = self.model.config
        out = np.zeros((cfg["layer_count"], rows, cfg["hidden_size"]), dtype=np.float32)
        if not self._lib.fc_test_copy_layer_outputs(
                self.handle, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), rows):
            raise FloydError("layer outputs unavailable")
        return out

    def set_layer_trace(self, enabled=True):
        self._lib.fc_session_set_layer_trace(self.handle, int(enabled))

    def set_profiling(self, enabled=True):
        if not self._lib.fc_session_set_profiling(self.handle, int(enabled)):
            raise FloydError("profiling unavailable")

    def profile(self):
        '''{kernel name: (total ms, launches)} of the profiled passes.'''
        out = {}
        i = 0
        name = ctypes.create_string_buffer(64)
        ms = ctypes.c_double()
        n = ctypes.c_uint64()
        while self._lib.fc_session_profile(self.handle, i, name, len(name), ctypes.byref(ms), ctypes.byref(n)):
            out[name.value.decode()] = (ms.value, n.value)
            i += 1
        return out

    def profile_reset(self):
        self._lib.fc_session_profile_reset(self.handle)

    def position(self):
        return self._lib.fc_session_position(self.handle)

    def reset(self):
        self._lib.fc_session_reset(self.handle)

    def stats(self):
        s = self._lib.fc_session_stats(self.handle)
        return {name: getattr(s, name) for name, _ in s._fields_}

    def close(self):
        if getattr(self, "handle", None):
            self._lib.fc_session_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
class BatchSession(Session):
    """Several sequences over one paged latent cache (fc_session_create_batch):
    a shared prefix, private pages per sequence, and one verify of
    rows_per_sequence rows for every sequence per verify_batch call."""

    def __init__(self, model, context_size, sequences, rows_per_sequence, shared_prefix=0):
        self._lib = model._lib
        self.model = model
        self.vocab = model.config["vocab_size"]
        self.sequences = sequences
        self.rows = rows_per_sequence
        opt = FcBatchOptions(context_size, sequences, rows_per_sequence, shared_prefix)
        handle = ctypes.c_void_p()
        err = _err()
        if not self._lib.fc_session_create_batch(ctypes.byref(handle), model.handle, ctypes.byref(opt), err,
                                                 len(err)):
            raise FloydError(err.value.decode())
        self.handle = handle

    def seed(self, sequence, start, end, seed):
        err = _err()
        self._check(self._lib.fc_session_batch_seed(self.handle, sequence, start, end, ctypes.c_uint64(seed),
                                                    err, len(err)), err)

    def verify_batch(self, ids, accept=None):
        """ids: [sequences][rows_per_sequence]; accept: None (greedy) or one
        (mode, temperature, seed, counter) per sequence.  Returns
        (n_emitted list, next_token list)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(self.sequences, self.rows)
        acc = None
        if accept is not None:
            acc = (FcAcceptConfig * self.sequences)(*[FcAcceptConfig(*a) for a in accept])
        n = np.zeros(self.sequences, dtype=np.int32)
        nxt = np.zeros(self.sequences, dtype=np.int32)
        err = _err()
        ip = ctypes.POINTER(ctypes.c_int)
        self._check(self._lib.fc_session_verify_batch(
            self.handle, ids.ctypes.data_as(ip), self.rows - 1, acc, n.ctypes.data_as(ip), nxt.ctypes.data_as(ip),
            err, len(err)), err)
        return n.tolist(), nxt.tolist()

    def position_of(self, sequence):
        return int(self._lib.fc_session_batch_position(self.handle, sequence))

    def rollback_seq(self, sequence, position):
        err = _err()
        self._check(self._lib.fc_session_batch_rollback(self.handle, sequence, int(position), err, len(err)), err)


