"""ctypes binding of the CPU oracle (test infrastructure only).

Only the pytest suite, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` leg import this module, and only as the checker or the timed
CPU baseline.  The product library never loads ``liboracle.so``.

The oracle restates the reference's ap_fixed golden model
(host/host_qwen_8x64.cpp) with integer arithmetic; see llmx_oracle.c for the
line-by-line citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

EXP_ROUND = 0
EXP_TRUNC = 1


class Shape(C.Structure):
    _fields_ = [(n, C.c_int32) for n in
                ("vocab", "hidden", "inter", "layers", "heads", "kv_heads", "max_seq")]

    @property
    def head_dim(self):
        return self.hidden // self.heads

    @property
    def kv_channels(self):
        return self.kv_heads * self.head_dim

    @property
    def group(self):
        return self.heads // self.kv_heads


# Profiles of parse_profile host:348-379 (vocab, hidden, inter, layers, heads,
# kv_heads, max_seq).
PROFILES = {
    "small": (64, 64, 128, 2, 4, 2, 32),
    "medium": (128, 128, 256, 2, 4, 2, 64),
    "qwen-layer": (128, 2048, 11008, 1, 16, 2, 96),
    "qwen-layer-long": (128, 2048, 11008, 1, 16, 2, 2048),
    "qwen2.5-3b": (151936, 2048, 11008, 36, 16, 2, 2048),
}


def shape(name_or_tuple, **overrides) -> Shape:
    vals = PROFILES[name_or_tuple] if isinstance(name_or_tuple, str) else name_or_tuple
    s = Shape(*vals)
    for k, v in overrides.items():
        setattr(s, k, v)
    return s


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        i16p = np.ctypeslib.ndpointer(np.int16, flags="C_CONTIGUOUS")
        i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
        u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
        sp = C.POINTER(Shape)
        sig = {
            "orc_exp_tables": (None, [C.c_int, i16p, i16p]),
            "orc_set_exp_mode": (None, [C.c_int]),
            "orc_get_exp_mode": (C.c_int, []),
            "orc_set_tables": (None, [i16p, i16p]),
            "orc_set_threads": (None, [C.c_int]),
            "orc_recip": (C.c_int16, [C.c_int16]),
            "orc_rsqrt": (C.c_int16, [C.c_int32]),
            "orc_silu": (C.c_int16, [C.c_int16]),
            "orc_exp_fm": (C.c_int16, [C.c_int16]),
            "orc_prob": (C.c_int16, [C.c_int16]),
            "orc_inv_rms_const": (C.c_int16, [C.c_int32]),
            "orc_projection": (None, [i16p, C.c_int, C.c_int, i16p, C.c_int, i16p]),
            "orc_projection_partial": (None, [i16p, C.c_int, C.c_int, i16p, C.c_int, C.c_int,
                                              C.c_int, C.c_int, i64p]),
            "orc_round_partial": (None, [i64p, C.c_size_t, i16p]),
            "orc_rmsnorm": (None, [i16p, C.c_int, C.c_int, i16p, i16p]),
            "orc_silu_mul": (None, [i16p, i16p, C.c_size_t, i16p]),
            "orc_residual": (None, [i16p, i16p, C.c_size_t, i16p]),
            "orc_rope_table": (None, [C.c_int, C.c_int, i16p]),
            "orc_attention_group": (None, [i16p, C.c_int, i16p, i16p, C.c_int, C.c_int,
                                           C.c_int, i16p]),
            "orc_layer_weight_elems": (C.c_size_t, [sp]),
            "orc_task18": (None, [sp, i16p, i16p, i16p, i16p, i16p, i16p, C.c_int, C.c_int,
                                  C.c_int, i16p]),
            "orc_task19": (None, [sp, i16p, i16p, i16p, C.c_int, i16p]),
            "orc_prefill_sequence_layer": (None, [sp, i16p, i16p, i16p, i16p, i16p, C.c_int,
                                                  C.c_int, C.c_void_p, i16p]),
            "orc_lm_head_argmax": (C.c_int32, [i16p, i16p, C.c_int, C.c_int, C.c_int]),
            "orc_checksum": (C.c_uint64, [i16p, C.c_size_t]),
            "orc_mt_uniform_fill": (None, [C.c_uint32, C.c_int, C.c_int, i16p, C.c_size_t]),
            "orc_ref_random_model": (C.c_int, [sp, C.c_uint32, C.c_int, C.c_void_p, i16p,
                                               C.c_void_p]),
            "orc_gauss_table": (C.c_int, [C.c_double, u64p, C.c_int, C.POINTER(C.c_int)]),
            "orc_gauss_fill": (None, [C.c_uint64, C.c_uint64, C.c_double, C.c_uint64, i16p,
                                      C.c_size_t]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _c16(a):
    return np.ascontiguousarray(a, dtype=np.int16)


# ---------------------------------------------------------------------------
# thin numpy wrappers
# ---------------------------------------------------------------------------
def set_exp_mode(mode: int):
    lib().orc_set_exp_mode(mode)


def set_threads(n: int):
    lib().orc_set_threads(n)


def set_tables(e16, p18):
    lib().orc_set_tables(_c16(e16), _c16(p18))


def exp_tables(mode: int):
    e = np.zeros(2049, np.int16)
    p = np.zeros(2049, np.int16)
    lib().orc_exp_tables(mode, e, p)
    return e, p


def projection(x, w):
    x = _c16(x)
    w = _c16(w)
    rows, k = x.shape
    o = w.shape[0]
    y = np.zeros((rows, o), np.int16)
    lib().orc_projection(x, rows, k, w, o, y)
    return y


def projection_partial(x, w, k_begin, k_end):
    x = _c16(x)
    w = _c16(w)
    rows, k = x.shape
    o = w.shape[0]
    p = np.zeros((rows, o), np.int64)
    lib().orc_projection_partial(x, rows, k, w, w.shape[1], o, k_begin, k_end, p)
    return p


def round_partial(p):
    p = np.ascontiguousarray(p, dtype=np.int64)
    y = np.zeros(p.shape, np.int16)
    lib().orc_round_partial(p, p.size, y)
    return y


def rmsnorm(x, w):
    x = _c16(x)
    rows, n = x.shape
    y = np.zeros_like(x)
    lib().orc_rmsnorm(x, rows, n, _c16(w), y)
    return y


def silu_mul(g, u):
    g = _c16(g)
    y = np.zeros_like(g)
    lib().orc_silu_mul(g, _c16(u), g.size, y)
    return y


def residual(a, b):
    a = _c16(a)
    y = np.zeros_like(a)
    lib().orc_residual(a, _c16(b), a.size, y)
    return y


def rope_table(head_dim, max_seq):
    t = np.zeros((max_seq, head_dim), np.int16)
    lib().orc_rope_table(head_dim, max_seq, t)
    return t


def attention_group(q, k, v, payload=1):
    q = _c16(q)
    g, hd = q.shape
    ctx = k.shape[0]
    out = np.zeros_like(q)
    lib().orc_attention_group(q, g, _c16(k), _c16(v), ctx, hd, payload, out)
    return out


def layer_weight_elems(s: Shape) -> int:
    return lib().orc_layer_weight_elems(C.byref(s))


def layer_views(s: Shape, blob):
    """Split a dense per-layer blob into Q,K,V,O,Gate,Up,Down [out][in] views."""
    H, I, KV = s.hidden, s.inter, s.kv_channels
    dims = [(H, H), (KV, H), (KV, H), (H, H), (I, H), (I, H), (H, I)]
    out, off = [], 0
    for o, i in dims:
        out.append(blob[off:off + o * i].reshape(o, i))
        off += o * i
    return out


def task18(s, layer_w, attn_norm, rope, k_cache, v_cache, hidden, position, payload=1):
    hidden = _c16(hidden)
    rows = hidden.shape[0]
    out = np.zeros_like(hidden)
    lib().orc_task18(C.byref(s), layer_w, _c16(attn_norm), rope, k_cache, v_cache, hidden,
                     rows, position, payload, out)
    return out


def task19(s, layer_w, ffn_norm, hidden):
    hidden = _c16(hidden)
    out = np.zeros_like(hidden)
    lib().orc_task19(C.byref(s), layer_w, _c16(ffn_norm), hidden, hidden.shape[0], out)
    return out


def prefill_sequence_layer(s, layer_w, attn_norm, ffn_norm, rope, hidden, payload=1):
    hidden = _c16(hidden)
    rows = hidden.shape[0]
    post = np.zeros_like(hidden)
    out = np.zeros_like(hidden)
    lib().orc_prefill_sequence_layer(C.byref(s), layer_w, _c16(attn_norm), _c16(ffn_norm),
                                     rope, hidden, rows, payload,
                                     post.ctypes.data_as(C.c_void_p), out)
    return post, out


def lm_head_argmax(h, w, threads=None):
    h = _c16(h).reshape(-1)
    w = _c16(w)
    threads = threads or min(32, os.cpu_count() or 1)
    return int(lib().orc_lm_head_argmax(h, w, w.shape[0], w.shape[1], threads))


def checksum(x) -> int:
    x = _c16(x)
    return int(lib().orc_checksum(x.reshape(-1), x.size))


def mt_uniform(seed, lo, hi, shape_):
    n = int(np.prod(shape_))
    out = np.zeros(n, np.int16)
    lib().orc_mt_uniform_fill(seed & 0xFFFFFFFF, lo, hi, out, n)
    return out.reshape(shape_)


def ref_random_model(s: Shape, seed: int, keep_layers: int, with_embedding=True):
    """initialize_random_model host:842-869 decoded into dense per-layer blobs."""
    emb = np.zeros(s.vocab * s.hidden, np.int16) if with_embedding else None
    norms = np.zeros((2 * s.layers + 1) * s.hidden, np.int16)
    le = layer_weight_elems(s)
    dense = np.zeros(keep_layers * le, np.int16)
    lib().orc_ref_random_model(C.byref(s), seed, keep_layers,
                               emb.ctypes.data_as(C.c_void_p) if emb is not None else None,
                               norms, dense.ctypes.data_as(C.c_void_p))
    return (emb.reshape(s.vocab, s.hidden) if emb is not None else None,
            norms.reshape(2 * s.layers + 1, s.hidden),
            dense.reshape(keep_layers, le))


def gauss_fill(seed, stream, sigma_raw, n, index0=0):
    out = np.zeros(n, np.int16)
    lib().orc_gauss_fill(seed, stream, sigma_raw, index0, out, n)
    return out


def gauss_table(sigma_raw):
    t = np.zeros(65536, np.uint64)
    kmin = C.c_int(0)
    n = lib().orc_gauss_table(sigma_raw, t, 65536, C.byref(kmin))
    return t[:n].copy(), kmin.value


def gaussian_layer(s: Shape, seed: int, layer: int, w_sigma: float = 0.02):
    """Dense blob of layer `layer` of the synthetic benchmark model (Q,K,V,O,
    Gate,Up,Down from streams 0x1000 + 16*layer + op, N(0, w_sigma) in Q4.12)."""
    H, I, KV = s.hidden, s.inter, s.kv_channels
    sizes = [H * H, KV * H, KV * H, H * H, I * H, I * H, H * I]
    return np.concatenate([gauss_fill(seed, 0x1000 + 16 * layer + op, w_sigma * 4096.0, n)
                           for op, n in enumerate(sizes)])


def gaussian_lm_head(s: Shape, seed: int, w_sigma: float = 0.02):
    """Untied LM head of the synthetic model: N(0, w_sigma) in Q4.12, stream 0x20."""
    return gauss_fill(seed, 0x20, w_sigma * 4096.0, s.vocab * s.hidden).reshape(s.vocab, s.hidden)


def gaussian_embedding_rows(s: Shape, seed: int, tokens):
    """Embedding rows of the synthetic model: N(0, 1) in Q8.8, stream 0x10."""
    return np.stack([gauss_fill(seed, 0x10, 256.0, s.hidden, int(t) * s.hidden) for t in tokens])
