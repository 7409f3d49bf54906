"""Python mirror of the llmx C ABI (include/llmx.h) over ctypes.

Mirrors the reference host interfaces of host/host_qwen_8x64.cpp in the
LLM-ACCEL tree: ``Accelerator`` ~ accelerator_t (run_composed_decoder_stack,
execute_bound_resident_task, bind_controller_data_ports), ``Model`` ~
model_data_t, ``Executor`` ~ qwen_executor_t.  Errors raise ``LlmxError``
carrying the controller status code, as the reference host throws on a bad
status (check_status host:3028-3049).

The compute path is the CUDA library libllmx.so built from csrc/; importing
this module never falls back to a CPU implementation -- a missing library or
GPU is an error.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# LLMX_TIMELINE=1 loads the measurement build (build.py --timeline): the same
# kernels, each launch stamping its start and end for llmx_timeline_read.
TIMELINE = os.environ.get("LLMX_TIMELINE") == "1"
LIB_PATH = os.path.join(HERE, "libllmx_timeline.so" if TIMELINE else "libllmx.so")

OK = 0
BAD_OPERATOR, BAD_TOKEN_COUNT, BAD_TILE_LENGTH, BAD_POSITION, BAD_LAYER = 1, 2, 3, 4, 5
ERR_CUDA, ERR_ARG, ERR_STATE, ERR_NCCL, ERR_RANGE, ERR_NOMEM, ERR_IO, ERR_UNSUPPORTED, ERR_TIMEOUT = range(100, 109)
OP_NOP, OP_ATTENTION, OP_FFN, OP_FINAL_NORM = 0, 18, 19, 20
# per-operator modes (operator_kind_t host:69-91)
(OP_Q_PROJECTION, OP_K_PROJECTION, OP_V_PROJECTION, OP_O_PROJECTION, OP_FFN_GATE, OP_FFN_UP, OP_FFN_DOWN,
 OP_RMSNORM, OP_SILU_MUL, OP_RESIDUAL_ADD) = range(1, 11)
OP_DECODER_LAYER, OP_ATTN_PREFILL_BLOCK = 16, 17
FEATURE_OPS = tuple(range(1, 11))
AR_NONE, AR_NCCL, AR_PEER = 0, 1, 2
MAX_ROWS = 8
KERNEL_QKV, KERNEL_ATTN, KERNEL_O, KERNEL_GATE_UP, KERNEL_DOWN, KERNEL_FINAL_NORM = range(6)


class LlmxError(RuntimeError):
    def __init__(self, code, what=""):
        self.code = code
        msg = f"{what}: {strerror(code)} ({code})"
        detail = last_error()
        if detail:
            msg += f" [{detail}]"
        super().__init__(msg)


class Shape(C.Structure):
    _fields_ = [(n, C.c_int32) for n in
                ("vocab", "hidden", "inter", "layers", "heads", "kv_heads", "max_seq")]

    @property
    def head_dim(self):
        return self.hidden // self.heads

    @property
    def kv_channels(self):
        return self.kv_heads * self.head_dim

    def tuple(self):
        return tuple(getattr(self, f) for f, _ in self._fields_)


class Status(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("op", "code", "token_count", "output_waves", "mm_tasks",
                                          "vector_tasks", "completed_packets", "last_task")] + \
               [("reserved", C.c_uint32 * 8)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_ if f != "reserved"}


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python llm-accel_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        i16p = np.ctypeslib.ndpointer(np.int16, flags="C_CONTIGUOUS")
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        vp, sp, stp = C.c_void_p, C.POINTER(Shape), C.POINTER(Status)
        sig = {
            "llmx_profile": (C.c_int, [C.c_char_p, sp]),
            "llmx_shape_validate": (C.c_int, [sp]),
            "llmx_validate_task": (C.c_int, [sp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, stp]),
            "llmx_validate_operator": (C.c_int, [sp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, stp]),
            "llmx_feature_dims": (C.c_int, [sp, C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                            C.POINTER(C.c_int)]),
            "llmx_run_feature": (C.c_int, [vp, C.c_uint32, i16p, C.c_uint32, C.c_uint32, vp, C.c_uint32,
                                           C.c_uint32, C.c_uint32, C.c_uint32, i16p, C.c_uint32, stp]),
            "llmx_run_prefill_attention_block": (C.c_int, [vp, i16p, C.c_uint32, C.c_uint32, C.c_uint32, i16p,
                                                           stp]),
            "llmx_strerror": (C.c_char_p, [C.c_int]),
            "llmx_last_error": (C.c_char_p, []),
            "llmx_exp_tables": (C.c_int, [i16p, i16p]),
            "llmx_rope_table": (C.c_int, [C.c_int, C.c_int, i16p]),
            "llmx_gauss_fill": (C.c_int, [C.c_uint64, C.c_uint64, C.c_double, C.c_uint64, i16p, C.c_size_t]),
            "llmx_model_create": (C.c_int, [sp, C.POINTER(vp)]),
            "llmx_model_destroy": (None, [vp]),
            "llmx_model_init_reference_random": (C.c_int, [vp, C.c_uint32, C.c_int]),
            "llmx_model_init_gaussian": (C.c_int, [vp, C.c_uint64, C.c_double, C.c_int]),
            "llmx_model_load_packed": (C.c_int, [vp, C.c_char_p, C.c_int]),
            "llmx_layer_weight_elems": (C.c_size_t, [sp]),
            "llmx_model_layer": (C.POINTER(C.c_int16), [vp, C.c_uint32]),
            "llmx_model_norms": (C.POINTER(C.c_int16), [vp]),
            "llmx_model_embedding": (C.POINTER(C.c_int16), [vp]),
            "llmx_model_embed": (C.c_int, [vp, u32p, C.c_uint32, i16p]),
            "llmx_model_lm_head_argmax": (C.c_int, [vp, i16p, C.c_int, C.POINTER(C.c_uint32)]),
            "llmx_tp_unique_id": (C.c_int, [vp]),
            "llmx_create": (C.c_int, [sp, C.c_int, C.c_int, C.c_int, vp, C.POINTER(vp)]),
            "llmx_destroy": (C.c_int, [vp]),
            "llmx_upload_model": (C.c_int, [vp, vp]),
            "llmx_upload_layer": (C.c_int, [vp, C.c_uint32, i16p]),
            "llmx_upload_norms": (C.c_int, [vp, i16p]),
            "llmx_reset_kv": (C.c_int, [vp]),
            "llmx_write_kv": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_uint32, i16p, i16p]),
            "llmx_read_kv": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_uint32, i16p, i16p]),
            "llmx_write_hidden": (C.c_int, [vp, C.c_uint32, i16p, C.c_uint32]),
            "llmx_read_hidden": (C.c_int, [vp, C.c_uint32, i16p, C.c_uint32]),
            "llmx_bind": (C.c_int, [vp, C.c_uint32, C.c_uint32]),
            "llmx_task": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, stp]),
            "llmx_stack": (C.c_int, [vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int,
                                     C.c_int, vp, stp]),
            "llmx_stack_async": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int]),
            "llmx_synchronize": (C.c_int, [vp]),
            "llmx_stream": (vp, [vp]),
            "llmx_hidden_device_ptr": (vp, [vp, C.c_uint32]),
            "llmx_kernel_launches": (C.c_uint64, [vp]),
            "llmx_device_bytes": (C.c_uint64, [vp]),
            "llmx_time_kernel": (C.c_int, [vp, C.c_int, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int,
                                           C.POINTER(C.c_double)]),
            "llmx_run_prompt_block": (C.c_int, [vp, vp, u32p, C.c_uint32, C.c_uint32, C.c_int, i16p]),
            "llmx_run_token": (C.c_int, [vp, vp, C.c_uint32, C.c_uint32, i16p]),
            "llmx_lm_head_argmax_device": (C.c_int, [vp, C.c_uint32, C.c_uint32, vp, C.c_uint32, vp, vp]),
            "llmx_upload_vocab": (C.c_int, [vp, vp]),
            "llmx_allreduce_kind": (C.c_int, [vp]),
            "llmx_decode_fuses_o": (C.c_int, [vp]),
            "llmx_selftest_ar_timeout": (C.c_int, [vp, C.c_uint32]),
            "llmx_generate": (C.c_int, [vp, u32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp]),
        }
        if TIMELINE:
            sig.update({
                "llmx_timeline_reset": (C.c_int, [vp]),
                "llmx_timeline_slots": (C.c_int, []),
                "llmx_timeline_name": (C.c_char_p, [C.c_int]),
                "llmx_timeline_read": (C.c_int, [vp, np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS"),
                                                 C.c_int]),
            })
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def strerror(code):
    return lib().llmx_strerror(code).decode()


def last_error():
    return lib().llmx_last_error().decode()


def check(rc, what=""):
    if rc != OK:
        raise LlmxError(rc, what)


def profile(name) -> Shape:
    s = Shape()
    check(lib().llmx_profile(name.encode(), C.byref(s)), f"profile {name}")
    return s


def shape(name_or_tuple, **overrides) -> Shape:
    s = profile(name_or_tuple) if isinstance(name_or_tuple, str) else Shape(*name_or_tuple)
    for k, v in overrides.items():
        setattr(s, k, v)
    return s


def validate_task(s: Shape, op, layer, position, rows):
    st = Status()
    code = lib().llmx_validate_task(C.byref(s), op, layer, position, rows, C.byref(st))
    return code, st


def validate_operator(s: Shape, op, layer, position, rows):
    """Validation of the controller image with the per-operator schedulers."""
    st = Status()
    code = lib().llmx_validate_operator(C.byref(s), op, layer, position, rows, C.byref(st))
    return code, st


def feature_dims(s: Shape, op):
    """(in_dim, out_dim, needs_rhs) of a feature operator (host:2015-2061)."""
    i, o, r = C.c_uint32(), C.c_uint32(), C.c_int()
    check(lib().llmx_feature_dims(C.byref(s), op, C.byref(i), C.byref(o), C.byref(r)),
          f"operator {op} is not a feature operator")
    return i.value, o.value, bool(r.value)


def exp_tables():
    e = np.zeros(2049, np.int16)
    p = np.zeros(2049, np.int16)
    check(lib().llmx_exp_tables(e, p))
    return e, p


def rope_table(head_dim, max_seq):
    t = np.zeros((max_seq, head_dim), np.int16)
    check(lib().llmx_rope_table(head_dim, max_seq, t))
    return t


def gauss_fill(seed, stream, sigma_raw, n, index0=0):
    out = np.zeros(n, np.int16)
    check(lib().llmx_gauss_fill(seed, stream, sigma_raw, index0, out, n))
    return out


class Model:
    """model_data_t host:779-1022: dense per-layer weights, norms, embedding, LM head."""

    def __init__(self, s: Shape):
        self.shape = s
        self.h = C.c_void_p()
        check(lib().llmx_model_create(C.byref(s), C.byref(self.h)), "model_create")

    def close(self):
        if self.h:
            lib().llmx_model_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_reference_random(self, seed, keep_layers=0):
        check(lib().llmx_model_init_reference_random(self.h, seed, keep_layers), "init_reference_random")
        return self

    def init_gaussian(self, seed, w_sigma=0.02, lm_head=False):
        check(lib().llmx_model_init_gaussian(self.h, seed, w_sigma, int(lm_head)), "init_gaussian")
        return self

    def load_packed(self, directory, tie_embeddings=False):
        check(lib().llmx_model_load_packed(self.h, directory.encode(), int(tie_embeddings)), "load_packed")
        return self

    def layer(self, l) -> np.ndarray:
        n = lib().llmx_layer_weight_elems(C.byref(self.shape))
        p = lib().llmx_model_layer(self.h, l)
        if not p:
            raise LlmxError(ERR_STATE, f"layer {l} not resident")
        return np.ctypeslib.as_array(p, shape=(n,))

    def norms(self) -> np.ndarray:
        s = self.shape
        return np.ctypeslib.as_array(lib().llmx_model_norms(self.h), shape=(2 * s.layers + 1, s.hidden))

    def embed(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros((len(t), self.shape.hidden), np.int16)
        check(lib().llmx_model_embed(self.h, t, len(t), out), "embed")
        return out

    def lm_head_argmax(self, hidden_row, threads=0) -> int:
        tok = C.c_uint32()
        check(lib().llmx_model_lm_head_argmax(self.h, np.ascontiguousarray(hidden_row, np.int16).reshape(-1),
                                              threads, C.byref(tok)), "lm_head_argmax")
        return tok.value


def lm_head_argmax_device(hidden_ptr, rows, hidden_size, lm_head_ptr, vocab, tokens_ptr, stream=None):
    """llmx_lm_head_argmax_device on device pointers (ints); allocates nothing.
    Returns the status code without raising."""
    return lib().llmx_lm_head_argmax_device(hidden_ptr, rows, hidden_size, lm_head_ptr, vocab, tokens_ptr,
                                            stream)


def tp_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().llmx_tp_unique_id(C.cast(buf, C.c_void_p)), "tp_unique_id")
    return buf.raw


class Accelerator:
    """accelerator_t host:1024-3087 on one B200 (one tensor-parallel rank)."""

    def __init__(self, s: Shape, device=0, tp_rank=0, tp_size=1, tp_id: bytes | None = None):
        self.shape = s
        self.h = C.c_void_p()
        idbuf = C.create_string_buffer(tp_id, 128) if tp_id else None
        check(lib().llmx_create(C.byref(s), device, tp_rank, tp_size,
                                C.cast(idbuf, C.c_void_p) if idbuf is not None else None,
                                C.byref(self.h)), "create")

    def close(self):
        if self.h:
            lib().llmx_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def upload_model(self, m: Model):
        check(lib().llmx_upload_model(self.h, m.h), "upload_model")

    # measurement build only (LLMX_TIMELINE=1)
    def timeline_reset(self):
        check(lib().llmx_timeline_reset(self.h), "timeline_reset")

    def timeline_read(self):
        """Launches that ran since timeline_reset(), in start order: (slot,
        name, start_ns, end_ns) from %globaltimer on this context's device."""
        n = lib().llmx_timeline_slots()
        out = np.zeros(2 * max(n, 1), np.uint64)
        check(lib().llmx_timeline_read(self.h, out, n), "timeline_read")
        runs = [(s, lib().llmx_timeline_name(s).decode(), int(out[2 * s]), int(out[2 * s + 1]))
                for s in range(n) if int(out[2 * s]) != 0xFFFFFFFFFFFFFFFF]
        return sorted(runs, key=lambda r: r[2])

    def upload_layer(self, layer, dense):
        check(lib().llmx_upload_layer(self.h, layer, np.ascontiguousarray(dense, np.int16).reshape(-1)),
              "upload_layer")

    def upload_norms(self, norms):
        check(lib().llmx_upload_norms(self.h, np.ascontiguousarray(norms, np.int16).reshape(-1)),
              "upload_norms")

    def reset_kv(self):
        check(lib().llmx_reset_kv(self.h), "reset_kv")

    def write_kv(self, layer, position, k, v):
        """k, v: [kv_heads][count][head_dim] Q8.8 rows of positions [position, position+count)."""
        k = np.ascontiguousarray(k, np.int16)
        v = np.ascontiguousarray(v, np.int16)
        check(lib().llmx_write_kv(self.h, layer, position, k.shape[1], k.reshape(-1), v.reshape(-1)),
              "write_kv")

    def read_kv(self, layer, position, count):
        s = self.shape
        k = np.zeros((s.kv_heads, count, s.head_dim), np.int16)
        v = np.zeros_like(k)
        check(lib().llmx_read_kv(self.h, layer, position, count, k.reshape(-1), v.reshape(-1)), "read_kv")
        return k, v

    def write_hidden(self, pair, rows):
        rows = np.ascontiguousarray(rows, np.int16)
        check(lib().llmx_write_hidden(self.h, pair, rows.reshape(-1), rows.shape[0]), "write_hidden")

    def read_hidden(self, pair, nrows):
        out = np.zeros((nrows, self.shape.hidden), np.int16)
        check(lib().llmx_read_hidden(self.h, pair, out.reshape(-1), nrows), "read_hidden")
        return out

    def bind(self, out_pair, in_pair):
        check(lib().llmx_bind(self.h, out_pair, in_pair), "bind")

    def task(self, op, layer, position, rows, raise_on_error=True):
        st = Status()
        rc = lib().llmx_task(self.h, op, layer, position, rows, C.byref(st))
        if raise_on_error:
            check(rc, f"task {op}")
        return rc, st

    def run_feature(self, op, lhs, rhs=None, layer=0, position=0):
        """run_feature host:1088-1130: one feature operator (1-10) on rows of lhs.
        Returns (out [rows][out_dim], status)."""
        lhs = np.ascontiguousarray(lhs, np.int16)
        if lhs.ndim != 2:
            raise ValueError("lhs must be [rows][cols]")
        try:
            out_dim = feature_dims(self.shape, op)[1]
        except LlmxError:
            out_dim = 0
        out = np.zeros((lhs.shape[0], max(out_dim, 1)), np.int16)
        rp, rr, rc_ = None, 0, 0
        if rhs is not None:
            rhs = np.ascontiguousarray(rhs, np.int16)
            if rhs.ndim == 1:
                rhs = rhs.reshape(1, -1)
            rp, rr, rc_ = rhs.ctypes.data, rhs.shape[0], rhs.shape[1]
        st = Status()
        rc = lib().llmx_run_feature(self.h, op, lhs.reshape(-1), lhs.shape[0], lhs.shape[1], rp, rr, rc_, layer,
                                    position, out.reshape(-1), out_dim, C.byref(st))
        check(rc, f"feature operator {op}")
        return out, st

    def run_prefill_attention_block(self, query, position, layer=0):
        """run_prefill_attention_block host:1647-1690: query [kv_heads][rows][G][head_dim]
        (post-RoPE) against the layer's KV cache; returns (out of the same shape, status)."""
        s = self.shape
        q = np.ascontiguousarray(query, np.int16)
        G = s.heads // s.kv_heads
        if q.ndim != 4 or q.shape[0] != s.kv_heads or q.shape[2] != G or q.shape[3] != s.head_dim:
            raise ValueError("prefill attention block shape mismatch")
        out = np.zeros_like(q)
        st = Status()
        rc = lib().llmx_run_prefill_attention_block(self.h, q.reshape(-1), position, q.shape[1], layer,
                                                    out.reshape(-1), C.byref(st))
        check(rc, "prefill attention block")
        return out, st

    def stack(self, hidden, layer_begin=0, layer_count=None, position=0, include_final_norm=True,
              materialize=True):
        s = self.shape
        hidden = np.ascontiguousarray(hidden, np.int16)
        rows = hidden.shape[0]
        layer_count = s.layers - layer_begin if layer_count is None else layer_count
        out = np.zeros((rows, s.hidden), np.int16)
        st = Status()
        check(lib().llmx_stack(self.h, hidden.ctypes.data, rows, layer_begin, layer_count, position,
                               int(include_final_norm), int(materialize), out.ctypes.data, C.byref(st)),
              "stack")
        return out if materialize else None

    def stack_raw(self, in_ptr, rows, layer_begin, layer_count, position, include_final_norm=True,
                  out_ptr=None):
        """llmx_stack on caller-owned host buffers (e.g. pinned memory)."""
        st = Status()
        check(lib().llmx_stack(self.h, in_ptr, rows, layer_begin, layer_count, position,
                               int(include_final_norm), int(out_ptr is not None), out_ptr, C.byref(st)),
              "stack")

    def time_kernel(self, kernel, layer, position, rows, iters):
        ms = C.c_double()
        check(lib().llmx_time_kernel(self.h, kernel, layer, position, rows, iters, C.byref(ms)),
              "time_kernel")
        return ms.value

    def stack_async(self, rows, layer_begin, layer_count, position, include_final_norm=True):
        check(lib().llmx_stack_async(self.h, rows, layer_begin, layer_count, position,
                                     int(include_final_norm)), "stack_async")

    def synchronize(self):
        check(lib().llmx_synchronize(self.h), "synchronize")

    @property
    def stream(self):
        return lib().llmx_stream(self.h)

    def hidden_ptr(self, pair):
        return lib().llmx_hidden_device_ptr(self.h, pair)

    @property
    def kernel_launches(self):
        return lib().llmx_kernel_launches(self.h)

    @property
    def device_bytes(self):
        return lib().llmx_device_bytes(self.h)

    def selftest_ar_timeout(self, poll_limit):
        """Return code of a bounded all-reduce wait that is made to expire (LLMX_ERR_TIMEOUT)."""
        return lib().llmx_selftest_ar_timeout(self.h, poll_limit)

    @property
    def decode_fuses_o(self):
        """Whether one-row stacks run the O projection inside the attention kernel."""
        return bool(lib().llmx_decode_fuses_o(self.h))

    @property
    def allreduce_kind(self):
        """AR_NONE (one GPU), AR_NCCL or AR_PEER: how the ranks add their partial sums."""
        return lib().llmx_allreduce_kind(self.h)

    def upload_vocab(self, m: Model):
        check(lib().llmx_upload_vocab(self.h, m.h), "upload_vocab")

    def generate(self, prompt, max_new, block_rows=8, layer_count=0, last_block=False):
        """Greedy generation on the device (host:9016-9132).  Returns the max_new
        tokens, plus the last prompt block's final-normed rows if last_block."""
        p = np.ascontiguousarray(prompt, np.uint32)
        toks = np.zeros(max(int(max_new), 1), np.uint32)
        nlast = (len(p) - 1) % block_rows + 1 if len(p) else 0
        rows = np.zeros((nlast, self.shape.hidden), np.int16) if last_block else None
        check(lib().llmx_generate(self.h, p, len(p), block_rows, layer_count, max_new,
                                  toks.ctypes.data_as(C.c_void_p),
                                  rows.ctypes.data_as(C.c_void_p) if rows is not None else None), "generate")
        toks = [int(t) for t in toks[:max_new]]
        return (toks, rows) if last_block else toks


class Executor:
    """qwen_executor_t host:7607-8161: embedding + stack + LM head on the host."""

    def __init__(self, acc: Accelerator, model: Model):
        self.acc, self.model = acc, model

    def run_prompt_block(self, tokens, position, materialize=True):
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.zeros((len(t), self.acc.shape.hidden), np.int16)
        check(lib().llmx_run_prompt_block(self.acc.h, self.model.h, t, len(t), position, int(materialize),
                                          out.reshape(-1)), "run_prompt_block")
        return out if materialize else None

    def run_token(self, token, position):
        out = np.zeros((1, self.acc.shape.hidden), np.int16)
        check(lib().llmx_run_token(self.acc.h, self.model.h, token, position, out.reshape(-1)), "run_token")
        return out
