"""ctypes binding of the CPU oracle (oracle/hale_oracle.c).

TEST INFRASTRUCTURE ONLY. Imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's CPU-baseline / --impl reference legs. The CUDA
library never imports, links or calls anything here.

The functions mirror the Rust reference's public operations on the MoE /
sampling path; each wrapper names the reference item it restates.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

F32, F16, BF16, Q8_0, Q4_0 = 0, 1, 2, 3, 4
QK = 32
DTYPES = {"f32": F32, "f16": F16, "bf16": BF16, "q8_0": Q8_0, "q4_0": Q4_0}

_LIBS = {}


class Matrix(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("rows", C.c_uint32), ("cols", C.c_uint32),
                ("data", C.c_void_p)]


class Expert(C.Structure):
    _fields_ = [("gate", Matrix), ("up", Matrix), ("down", Matrix)]


class Layer(C.Structure):
    _fields_ = [("input_norm", C.c_void_p), ("post_norm", C.c_void_p),
                ("q", Matrix), ("k", Matrix), ("v", Matrix), ("o", Matrix),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("is_moe", C.c_int32),
                ("dense", Expert), ("router", Matrix), ("experts", C.c_void_p)]


class Model(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("n_layers", C.c_uint32), ("n_heads", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("vocab", C.c_uint32),
                ("n_experts", C.c_uint32), ("top_k", C.c_uint32), ("normalize_topk", C.c_int32),
                ("eps", C.c_float), ("rope_theta", C.c_float), ("embed", Matrix),
                ("lm_head", Matrix), ("final_norm", C.c_void_p), ("layers", C.c_void_p)]


def lib(native=False):
    """Loads (building if needed) the portable or -march=native oracle."""
    name = "libhale_oracle_native.so" if native else "libhale_oracle.so"
    if name in _LIBS:
        return _LIBS[name]
    path = os.path.join(_build.BUILD, name)
    if not os.path.exists(path) or os.path.exists(_build.SRC) and _build._stale(path):
        _build.build(variants=[name])
    L = C.CDLL(path)
    P = C.c_void_p
    sz = C.c_size_t
    sig = {
        "ho_block_len": (sz, [C.c_int]),
        "ho_block_bytes": (sz, [C.c_int]),
        "ho_row_bytes": (C.c_int64, [C.c_int, sz]),
        "ho_f32_to_f16": (C.c_uint16, [C.c_float]),
        "ho_f16_to_f32": (C.c_float, [C.c_uint16]),
        "ho_f32_to_bf16": (C.c_uint16, [C.c_float]),
        "ho_encode_row": (None, [C.c_int, P, sz, P]),
        "ho_decode_row": (None, [C.c_int, P, sz, P]),
        "ho_quantize_q8": (None, [P, sz, P, P]),
        "ho_dot_quantized": (C.c_float, [C.c_int, P, P, P, sz, P]),
        "ho_dot": (C.c_float, [C.c_int, P, P, sz]),
        "ho_matvec": (None, [C.c_int, P, sz, sz, P, P, C.c_int]),
        "ho_silu": (C.c_float, [C.c_float]),
        "ho_softmax_in_place": (None, [P, sz]),
        "ho_argmax": (sz, [P, sz]),
        "ho_top_k": (sz, [P, sz, sz, P, P]),
        "ho_rms_norm": (None, [P, P, C.c_float, P, sz]),
        "ho_rms_norm_in_place": (None, [P, P, C.c_float, sz]),
        "ho_rope_inv_freq": (None, [sz, C.c_float, P]),
        "ho_rope_angles": (None, [P, sz, sz, P, P]),
        "ho_rope_apply": (None, [P, sz, P, P]),
        "ho_expert_forward": (None, [P, P, P, C.c_int]),
        "ho_moe_route": (sz, [P, sz, C.c_int, P, P, P, C.c_int]),
        "ho_moe_forward": (None, [P, P, sz, sz, C.c_int, P, sz, P, P, P, C.c_int]),
        "ho_xorshift_next_u64": (C.c_uint64, [P]),
        "ho_xorshift_next_f32": (C.c_float, [P]),
        "ho_xorshift_seed": (C.c_uint64, [C.c_uint64]),
        "ho_apply_repetition_penalty": (None, [P, sz, P, sz, C.c_float]),
        "ho_sample": (C.c_uint32, [P, sz, C.c_float, C.c_float, sz, P, P]),
        "ho_model_forward": (C.c_int, [P, C.c_uint32, C.c_uint32, P, P, C.c_uint32, P, P, C.c_int]),
        "ho_expf_batch": (None, [P, P, sz]),
        "ho_num_threads": (C.c_int, []),
        "ho_set_num_threads": (None, [C.c_int]),
    }
    for fn, (res, args) in sig.items():
        f = getattr(L, fn)
        f.restype = res
        f.argtypes = args
    _LIBS[name] = L
    return L


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- formats ---------------------------------------------------------------

def row_bytes(dtype, cols):
    """DType::row_bytes (dtype.rs:53-61); None for a bad length."""
    r = lib().ho_row_bytes(dtype, cols)
    return None if r < 0 else int(r)


def encode(dtype, values):
    """WeightMatrix::from_f32 / encode_row per row (matrix.rs:48-61, quant.rs:274-292)."""
    v = _f32(values)
    rows, cols = (1, v.shape[0]) if v.ndim == 1 else v.shape
    rb = row_bytes(dtype, cols)
    out = np.zeros((rows, rb), dtype=np.uint8)
    L = lib()
    for r in range(rows):
        L.ho_encode_row(dtype, _p(v.reshape(rows, cols)[r]), cols, _p(out[r]))
    return out if v.ndim == 2 else out[0]


def decode(dtype, data, cols):
    """decode_row per row (quant.rs:236-269)."""
    d = np.ascontiguousarray(data, dtype=np.uint8)
    rows = 1 if d.ndim == 1 else d.shape[0]
    out = np.zeros((rows, cols), dtype=np.float32)
    L = lib()
    for r in range(rows):
        L.ho_decode_row(dtype, _p(d.reshape(rows, -1)[r]), cols, _p(out[r]))
    return out if d.ndim == 2 else out[0]


def quantize_q8(x):
    """Q8Activations::quantize (quant.rs:77-93) -> (scales f32[n/32], quants i8[n])."""
    x = _f32(x)
    n = x.shape[-1]
    xs = np.zeros(x.shape[:-1] + (n // QK,), dtype=np.float32)
    xq = np.zeros(x.shape, dtype=np.int8)
    L = lib()
    if x.ndim == 1:
        L.ho_quantize_q8(_p(x), n, _p(xs), _p(xq))
    else:
        for i in range(x.shape[0]):
            L.ho_quantize_q8(_p(x[i]), n, _p(xs[i]), _p(xq[i]))
    return xs, xq


def dot_quantized(dtype, row, xs, xq, want_block_sums=False):
    """dot_quantized (quant.rs:107-144), optionally with per-block int32 sums."""
    row = np.ascontiguousarray(row, dtype=np.uint8)
    xs = _f32(xs)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    n = xq.shape[0]
    sums = np.zeros(n // QK, dtype=np.int32) if want_block_sums else None
    r = lib().ho_dot_quantized(dtype, _p(row), _p(xs), _p(xq), n, _p(sums))
    return (r, sums) if want_block_sums else r


def dot(dtype, row, x):
    """quant::dot (quant.rs:59-66)."""
    row = np.ascontiguousarray(row, dtype=np.uint8)
    x = _f32(x)
    return lib().ho_dot(dtype, _p(row), _p(x), x.shape[0])


def matvec(dtype, w, rows, cols, x, parallel=True):
    """WeightMatrix::matvec / matvec_serial (matrix.rs:115-143)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = _f32(x)
    out = np.zeros(rows, dtype=np.float32)
    lib().ho_matvec(dtype, _p(w), rows, cols, _p(x), _p(out), int(parallel))
    return out


# ---- ops -------------------------------------------------------------------

def silu(v):
    return lib().ho_silu(float(v))


def softmax(x):
    x = _f32(x).copy()
    lib().ho_softmax_in_place(_p(x), x.shape[0])
    return x


def argmax(x):
    x = _f32(x)
    return int(lib().ho_argmax(_p(x), x.shape[0]))


def top_k(scores, k):
    """ops::top_k (topk.rs:44-61) -> (indices, scores), best first."""
    s = _f32(scores)
    idx = np.zeros(max(k, 1), dtype=np.uint32)
    sc = np.zeros(max(k, 1), dtype=np.float32)
    n = lib().ho_top_k(_p(s), s.shape[0], k, _p(idx), _p(sc))
    return idx[:n].copy(), sc[:n].copy()


def rms_norm(x, w, eps):
    x, w = _f32(x), _f32(w)
    out = np.zeros_like(x)
    lib().ho_rms_norm(_p(x), _p(w), eps, _p(out), x.shape[0])
    return out


def rms_norm_in_place(x, w, eps):
    y, w = _f32(x).copy(), _f32(w)
    lib().ho_rms_norm_in_place(_p(y), _p(w), eps, y.shape[0])
    return y


def rope_tables(head_dim, theta, position):
    inv = np.zeros(head_dim // 2, dtype=np.float32)
    L = lib()
    L.ho_rope_inv_freq(head_dim, theta, _p(inv))
    c = np.zeros_like(inv)
    s = np.zeros_like(inv)
    L.ho_rope_angles(_p(inv), head_dim // 2, position, _p(c), _p(s))
    return c, s


def rope_apply(head, c, s):
    h = _f32(head).copy()
    lib().ho_rope_apply(_p(h), h.shape[0], _p(_f32(c)), _p(_f32(s)))
    return h


# ---- experts / MoE -------------------------------------------------------------

class ExpertWeights:
    """One SwiGLU expert's encoded matrices (expert/mod.rs:75-83).

    gate/up are [I, H], down is [H, I]; each a uint8 array of encoded rows.
    """

    def __init__(self, dtype, hidden, inter, gate, up, down):
        self.dtype, self.hidden, self.inter = dtype, hidden, inter
        self.gate = np.ascontiguousarray(gate, dtype=np.uint8)
        self.up = np.ascontiguousarray(up, dtype=np.uint8)
        self.down = np.ascontiguousarray(down, dtype=np.uint8)

    def cstruct(self):
        d, h, i = self.dtype, self.hidden, self.inter
        return Expert(Matrix(d, i, h, _p(self.gate).value), Matrix(d, i, h, _p(self.up).value),
                      Matrix(d, h, i, _p(self.down).value))


def matrix_struct(dtype, rows, cols, data):
    return Matrix(dtype, rows, cols, _p(data).value)


def expert_forward(e, x, parallel=True):
    """Expert::forward (expert/mod.rs:91-103)."""
    x = _f32(x)
    out = np.zeros(e.hidden, dtype=np.float32)
    st = e.cstruct()
    lib().ho_expert_forward(C.byref(st), _p(x), _p(out), int(parallel))
    return out


def moe_forward(router_dtype, router, experts, k, normalize, x, parallel=True, native=False):
    """MoeLayer::forward over rows of x (moe.rs:56-70).

    Returns (out [M,H], expert ids [M,k], weights [M,k]).
    """
    x = _f32(x)
    if x.ndim == 1:
        x = x[None, :]
    m, h = x.shape
    n_exp = len(experts)
    router = np.ascontiguousarray(router, dtype=np.uint8)
    rs = Matrix(router_dtype, n_exp, h, _p(router).value)
    arr = (Expert * n_exp)(*[e.cstruct() for e in experts])
    out = np.zeros((m, h), dtype=np.float32)
    idx = np.zeros((m, k), dtype=np.uint32)
    w = np.zeros((m, k), dtype=np.float32)
    lib(native).ho_moe_forward(C.byref(rs), arr, n_exp, k, int(normalize), _p(x), m, _p(out),
                               _p(idx), _p(w), int(parallel))
    return out, idx, w


def moe_route(router_dtype, router, n_experts, k, normalize, x):
    """MoeLayer::route (moe.rs:36-53) -> (expert ids, weights) best first."""
    x = _f32(x)
    router = np.ascontiguousarray(router, dtype=np.uint8)
    rs = Matrix(router_dtype, n_experts, x.shape[0], _p(router).value)
    idx = np.zeros(k, dtype=np.uint32)
    w = np.zeros(k, dtype=np.float32)
    n = lib().ho_moe_route(C.byref(rs), k, int(normalize), _p(x), _p(idx), _p(w), 1)
    return idx[:n], w[:n]


# ---- sampling ----------------------------------------------------------------

class XorShift64:
    """sampler.rs:128-146."""

    def __init__(self, seed):
        self.state = C.c_uint64(lib().ho_xorshift_seed(seed))

    def next_u64(self):
        return lib().ho_xorshift_next_u64(C.byref(self.state))

    def next_f32(self):
        return lib().ho_xorshift_next_f32(C.byref(self.state))


def apply_repetition_penalty(logits, seen, penalty):
    lg = _f32(logits).copy()
    s = np.ascontiguousarray(seen, dtype=np.int32)
    lib().ho_apply_repetition_penalty(_p(lg), lg.shape[0], _p(s), s.shape[0], penalty)
    return lg


class Sampler:
    """SamplingParams::build() + Sampler::sample (sampler.rs:55-123).

    rng state persists across calls like TopPSampler's XorShift64. A
    repetition penalty (not in the reference) is applied to `seen` ids first.
    """

    def __init__(self, temperature=0.7, top_p=0.9, top_k=40, seed=42):
        self.temperature, self.top_p, self.top_k = temperature, top_p, top_k
        self.state = C.c_uint64(lib().ho_xorshift_seed(seed))

    def sample(self, logits, seen=None, repetition_penalty=1.0):
        lg = _f32(logits)
        if seen is not None and repetition_penalty != 1.0:
            lg = apply_repetition_penalty(lg, seen, repetition_penalty)
        return int(lib().ho_sample(_p(lg), lg.shape[0], self.temperature, self.top_p,
                                   self.top_k, C.byref(self.state), None))


def expf_batch(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().ho_expf_batch(_p(x), _p(y), x.size)
    return y


def num_threads(native=False):
    return lib(native).ho_num_threads()


def set_num_threads(n, native=False):
    """OpenMP threads of the oracle's parallel loops (all host cores, like
    the reference's rayon pool, unless told otherwise)."""
    lib(native).ho_set_num_threads(int(n))
