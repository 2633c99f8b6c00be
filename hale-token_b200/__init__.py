"""hale-token_b200: B200 (sm_100a) implementation of Hale-Token's MoE
quantized-expert forward and sampling tail, behind a C ABI.

The product is libhale_cuda.so (csrc/, declared in include/hale_cuda.h).
This module is a thin ctypes binding of that ABI -- the same calls a Rust
host would make through `extern "C"` -- plus helpers that pass torch device
tensors as raw pointers. There is no CPU fallback: importing this package
without the built library raises.

Because the directory name contains a dash, import it with
``importlib.import_module("hale-token_b200")``.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhale_cuda.so")

# status codes (include/hale_cuda.h)
OK = 0
E_INVALID_ARGUMENT = -1
E_BAD_TENSOR = -2
E_IO = -3
E_CONTEXT_OVERFLOW = -4
E_CUDA = -10
E_NO_DEVICE = -11
E_OUT_OF_MEMORY = -12
E_TIMEOUT = -13
E_DEVICE_CHECK = -14
E_UNSUPPORTED = -15
E_NCCL = -16

F32, F16, BF16, Q8_0, Q4_0 = 0, 1, 2, 3, 4

# Every function the header declares, with its ctypes signature.
P = C.c_void_p
U32, I32, U64, I64, SZ = C.c_uint32, C.c_int32, C.c_uint64, C.c_int64, C.c_size_t


class CacheStats(C.Structure):
    _fields_ = [("pinned_hits", U64), ("lru_hits", U64), ("misses", U64), ("bytes_loaded", U64),
                ("load_seconds", C.c_double), ("pinned_experts", U64), ("pinned_bytes", U64),
                ("lru_experts", U64), ("lru_bytes", U64), ("lru_capacity_bytes", U64),
                ("passthrough", I32)]


class ExpertKey(C.Structure):
    _fields_ = [("layer", U32), ("expert", U32)]


class ExpertView(C.Structure):
    _fields_ = [("gate", P), ("up", P), ("down", P)]


class CachePolicyStruct(C.Structure):
    _fields_ = [("pinned", P), ("n_pinned", U64), ("lru_bytes", U64)]


class MoeLayer(C.Structure):
    _fields_ = [("layer", U32), ("router", P), ("router_dtype", C.c_int), ("n_experts", U32),
                ("top_k", U32), ("normalize_topk", I32)]


class SamplingParams(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", U32),
                ("repetition_penalty", C.c_float)]


class HostMatrix(C.Structure):
    _fields_ = [("dtype", I32), ("rows", U32), ("cols", U32), ("data", P)]


class DecoderLayer(C.Structure):
    _fields_ = [("input_norm", P), ("post_norm", P), ("q_norm", P), ("k_norm", P),
                ("q", HostMatrix), ("k", HostMatrix), ("v", HostMatrix), ("o", HostMatrix),
                ("is_moe", I32), ("router", HostMatrix),
                ("dense_gate", HostMatrix), ("dense_up", HostMatrix), ("dense_down", HostMatrix)]


class DecoderDesc(C.Structure):
    _fields_ = [("hidden", U32), ("n_layers", U32), ("n_heads", U32), ("n_kv_heads", U32),
                ("head_dim", U32), ("vocab", U32), ("n_experts", U32), ("top_k", U32),
                ("normalize_topk", I32), ("eps", C.c_float), ("rope_theta", C.c_float),
                ("embed", HostMatrix), ("lm_head", HostMatrix), ("final_norm", P)]


SIGNATURES = {
    "hale_ctx_create": (I32, [C.c_int, C.POINTER(P)]),
    "hale_ctx_destroy": (None, [P]),
    "hale_last_error": (I32, [P, C.c_char_p, SZ]),
    "hale_ctx_check": (I32, [P, P]),
    "hale_ctx_launch_count": (U64, [P]),
    "hale_ctx_profile": (I32, [P, C.c_int]),
    "hale_ctx_set_expert_kernel": (I32, [P, C.c_int]),
    "hale_ctx_profile_read": (I32, [P, C.c_char_p, C.POINTER(U64), C.POINTER(C.c_double)]),
    "hale_row_bytes": (I64, [C.c_int, U64]),
    "hale_matrix_create": (I32, [P, C.c_int, U32, U32, P, U64, C.c_int, C.POINTER(P)]),
    "hale_matrix_destroy": (None, [P]),
    "hale_matrix_matvec": (I32, [P, P, P, U32, P, P, P]),
    "hale_matrix_matvec_q8": (I32, [P, P, P, P, U32, P, P, P]),
    "hale_quantize_q8": (I32, [P, P, U32, U32, P, P, P]),
    "hale_pool_create": (I32, [P, C.c_int, U32, U32, U32, U32, C.POINTER(P)]),
    "hale_pool_destroy": (None, [P]),
    "hale_pool_upload_expert": (I32, [P, U32, U32, P, U64, C.c_int, P]),
    "hale_pool_fetch": (I32, [P, P, U64, P]),
    "hale_pool_stats": (I32, [P, C.POINTER(CacheStats)]),
    "hale_pool_routing_counts": (I32, [P, P, U64]),
    "hale_pool_expert_bytes": (U64, [P]),
    "hale_pool_create_tiered": (I32, [P, C.c_int, U32, U32, U32, U32, C.POINTER(CachePolicyStruct), C.POINTER(P)]),
    "hale_pool_hbm_slots": (U64, [P]),
    "hale_pool_set_source": (I32, [P, P, P]),
    "hale_moe_forward": (I32, [P, P, C.POINTER(MoeLayer), P, U32, P, P, P, P]),
    "hale_moe_forward_host": (I32, [P, P, C.POINTER(MoeLayer), P, U32, P, P, P, P]),
    "hale_moe_route": (I32, [P, C.POINTER(MoeLayer), U32, P, U32, P, P, P, P]),
    "hale_moe_route_noalloc": (I32, [P, C.c_int, U32, U32, I32, U32, P, U32, P, P, P, P]),
    "hale_q8_aux_pairs": (I32, [U32]),
    "hale_ep_dispatch": (I32, [P, P, U32, P, U32, U32, P, P, P, C.POINTER(U64), P, P, P]),
    "hale_ep_experts": (I32, [P, P, U32, U32, P, P, P, U32, P, P]),
    "hale_ep_combine": (I32, [P, P, P, U32, U32, U32, P, P]),
    "hale_comm_unique_id": (I32, [P]),
    "hale_comm_create": (I32, [P, U32, U32, P, U32, U32, U32, U32, C.POINTER(P)]),
    "hale_comm_destroy": (I32, [P]),
    "hale_moe_forward_ep": (I32, [P, P, P, C.POINTER(MoeLayer), P, U32, P, P, P, P]),
    "hale_decoder_set_comm": (I32, [P, P]),
    "hale_decoder_create": (I32, [P, C.POINTER(DecoderDesc), C.POINTER(DecoderLayer), P, U32, C.POINTER(P)]),
    "hale_decoder_destroy": (None, [P]),
    "hale_decoder_forward": (I32, [P, P, U32, U32, P, P, P]),
    "hale_decoder_create_batched": (I32, [P, C.POINTER(DecoderDesc), C.POINTER(DecoderLayer), P, U32, U32, U32,
                                         C.POINTER(P)]),
    "hale_decoder_step": (I32, [P, P, P, P, P, U32, P, I32, P, P]),
    "hale_decoder_generate": (I32, [P, P, P, U32, P, U64, U32, P, U32, P, P, P, P, P]),
    "hale_lm_head": (I32, [P, P, P, U32, P, P]),
    "hale_sample": (I32, [P, P, U32, U32, C.POINTER(SamplingParams), P, P, U32, P, P]),
    "hale_expf_host": (None, [P, P, U64]),
}

_lib = None


def lib():
    """Loads libhale_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() "
                              "or `python hale-token_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class HaleError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"[{status}] {message}")
        self.status = status


def _check(status, ctx=None):
    if status != OK:
        buf = C.create_string_buffer(512)
        lib().hale_last_error(ctx, buf, 512)
        raise HaleError(status, buf.value.decode(errors="replace"))


def ptr(t):
    """Raw device/host address of a torch tensor or numpy array (or None)."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return C.c_void_p(t.data_ptr())
    return C.c_void_p(t.ctypes.data)


def _stream(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(stream.cuda_stream)


class Context:
    """hale_ctx: one GPU and its workspace.

    expert_kernel picks the expert-kernel family for this context: "auto"
    (by batch shape), "tc" (tcgen05 kernels), "ps" (persistent streaming
    warp-MMA kernels) or "dp4a" (per-CTA kernels); the first two wherever the
    shapes allow (hale_ctx_set_expert_kernel).
    """

    FAMILIES = {"auto": 0, "tc": 1, "dp4a": 2, "ps": 3, "ws": 4}

    def __init__(self, device=0, expert_kernel=None):
        h = P()
        if expert_kernel is not None and expert_kernel not in self.FAMILIES:
            raise ValueError(f"expert_kernel must be one of {sorted(self.FAMILIES)}, not {expert_kernel!r}")
        _check(lib().hale_ctx_create(device, C.byref(h)))
        if expert_kernel is not None:
            _check(lib().hale_ctx_set_expert_kernel(h, self.FAMILIES[expert_kernel]), h)
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().hale_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, stream=None):
        _check(lib().hale_ctx_check(self.h, _stream(stream)), self.h)

    @property
    def launches(self):
        return lib().hale_ctx_launch_count(self.h)

    def profile(self, enable=True):
        """Per-kernel CUDA-event timing of this library's launches."""
        self.call("hale_ctx_profile", self.h, int(enable))

    def profile_read(self, kernel):
        """(launches, total device ms) for a kernel family since the last read."""
        n, ms = U64(), C.c_double()
        self.call("hale_ctx_profile_read", self.h, kernel.encode(), C.byref(n), C.byref(ms))
        return n.value, ms.value

    def call(self, fn, *args):
        _check(getattr(lib(), fn)(*args), self.h)


class Matrix:
    """hale_matrix: WeightMatrix::new over reference-encoded rows."""

    def __init__(self, ctx, dtype, rows, cols, encoded):
        """`encoded`: numpy uint8 [rows, row_bytes] (host) or torch uint8 tensor (device)."""
        h = P()
        on_dev = hasattr(encoded, "is_cuda") and encoded.is_cuda
        nbytes = encoded.numel() if hasattr(encoded, "numel") else encoded.nbytes
        ctx.call("hale_matrix_create", ctx.h, dtype, rows, cols, ptr(encoded), nbytes, int(on_dev),
                 C.byref(h))
        self.ctx, self.h, self.dtype, self.rows, self.cols = ctx, h, dtype, rows, cols

    def __del__(self):
        try:
            if self.h:
                lib().hale_matrix_destroy(self.h)
                self.h = None
        except Exception:
            pass

    def matvec(self, x, out, block_sums=None, stream=None):
        self.ctx.call("hale_matrix_matvec", self.ctx.h, self.h, ptr(x), x.shape[0], ptr(out),
                      ptr(block_sums), _stream(stream))

    def matvec_q8(self, scales, quants, out, block_sums=None, stream=None):
        self.ctx.call("hale_matrix_matvec_q8", self.ctx.h, self.h, ptr(scales), ptr(quants),
                      quants.shape[0], ptr(out), ptr(block_sums), _stream(stream))

    def lm_head(self, hidden, logits, stream=None):
        self.ctx.call("hale_lm_head", self.ctx.h, self.h, ptr(hidden), hidden.shape[0],
                      ptr(logits), _stream(stream))


class CachePolicy:
    """CachePolicy (src/expert/cache.rs:58-64): `pinned` keys (pool layer,
    expert) kept in HBM for good, `lru_bytes` the HBM LRU tier's budget in
    expert-record bytes."""

    def __init__(self, pinned=(), lru_bytes=0):
        self.pinned = [(int(l), int(e)) for l, e in pinned]
        self.lru_bytes = int(lru_bytes)

    def __repr__(self):
        return f"CachePolicy(pinned={len(self.pinned)} experts, lru_bytes={self.lru_bytes})"


class Pool:
    """hale_pool: the ExpertProvider of the MoE layers.

    Without a policy every expert is HBM-resident. With a CachePolicy the
    pool is tiered (ExpertCache, cache.rs:66-194): uploads fill a page-locked
    host tier, HBM holds the pinned experts plus an LRU, and misses are
    copied in as each forward's routes are resolved; results are identical.
    """

    def __init__(self, ctx, dtype, hidden, inter, n_layers, n_experts, policy=None):
        h = P()
        if policy is None:
            ctx.call("hale_pool_create", ctx.h, dtype, hidden, inter, n_layers, n_experts, C.byref(h))
        else:
            keys = (ExpertKey * max(1, len(policy.pinned)))(*[ExpertKey(l, e) for l, e in policy.pinned])
            pol = CachePolicyStruct(C.cast(keys, P), len(policy.pinned), policy.lru_bytes)
            ctx.call("hale_pool_create_tiered", ctx.h, dtype, hidden, inter, n_layers, n_experts, C.byref(pol),
                     C.byref(h))
        self.ctx, self.h, self.policy = ctx, h, policy
        self.dtype, self.hidden, self.inter, self.n_layers, self.n_experts = (
            dtype, hidden, inter, n_layers, n_experts)

    def __del__(self):
        try:
            if self.h:
                lib().hale_pool_destroy(self.h)
                self.h = None
        except Exception:
            pass

    @property
    def expert_bytes(self):
        return lib().hale_pool_expert_bytes(self.h)

    @property
    def hbm_slots(self):
        """Experts HBM holds at once (n_layers * n_experts when resident)."""
        return lib().hale_pool_hbm_slots(self.h)

    def upload(self, layer, expert, record, stream=None):
        on_dev = hasattr(record, "is_cuda") and record.is_cuda
        nbytes = record.numel() if hasattr(record, "numel") else record.nbytes
        self.ctx.call("hale_pool_upload_expert", self.h, layer, expert, ptr(record), nbytes,
                      int(on_dev), _stream(stream))

    SOURCE_FN = C.CFUNCTYPE(I32, P, U32, U32, P, U64)

    def set_source(self, fn):
        """hale_pool_set_source (ExpertSource::load): fn(layer, expert) returns
        the expert's pack record (bytes-like, expert_bytes long); raising (or
        returning None) reports a failed load, which the forward surfaces as
        HaleError E_IO. fn None removes the source."""
        if fn is None:
            self._source = None
            self.ctx.call("hale_pool_set_source", self.h, None, None)
            return

        def load(_user, layer, expert, dst, nbytes):
            try:
                rec = fn(int(layer), int(expert))
                if rec is None:
                    return 1
                mv = memoryview(rec).cast("B")
                if len(mv) != nbytes:
                    return 2
                C.memmove(dst, (C.c_char * nbytes).from_buffer_copy(mv), nbytes)
                return 0
            except Exception:
                return 3

        self._source = self.SOURCE_FN(load)   # kept alive with the pool
        self.ctx.call("hale_pool_set_source", self.h, C.cast(self._source, P), None)

    def fetch(self, keys):
        arr = (ExpertKey * len(keys))(*[ExpertKey(l, e) for l, e in keys])
        out = (ExpertView * len(keys))()
        self.ctx.call("hale_pool_fetch", self.h, C.cast(arr, P), len(keys), C.cast(out, P))
        return [(v.gate, v.up, v.down) for v in out]

    def stats(self):
        s = CacheStats()
        self.ctx.call("hale_pool_stats", self.h, C.byref(s))
        return s

    def routing_counts(self):
        import numpy as np
        n = self.n_layers * self.n_experts
        out = np.zeros(n, dtype=np.uint64)
        self.ctx.call("hale_pool_routing_counts", self.h, ptr(out), n)
        return out.reshape(self.n_layers, self.n_experts)


def moe_layer(layer, router, router_dtype, n_experts, top_k, normalize):
    """hale_moe_layer for a device router tensor; the returned struct keeps
    the tensor alive (the C side only stores its address)."""
    ly = MoeLayer(layer, ptr(router).value if router is not None else None, router_dtype,
                  n_experts, top_k, int(normalize))
    ly._router_ref = router
    return ly


def moe_forward(ctx, pool, layer, x, out, topk_idx=None, topk_w=None, stream=None):
    ctx.call("hale_moe_forward", ctx.h, pool.h, C.byref(layer), ptr(x), x.shape[0], ptr(out),
             ptr(topk_idx), ptr(topk_w), _stream(stream))


def moe_forward_host(ctx, pool, layer, x, out, topk_idx=None, topk_w=None, stream=None):
    ctx.call("hale_moe_forward_host", ctx.h, pool.h, C.byref(layer), ptr(x), x.shape[0],
             ptr(out), ptr(topk_idx), ptr(topk_w), _stream(stream))


def moe_route(ctx, layer, hidden, x, topk_idx, topk_w, probs=None, stream=None):
    ctx.call("hale_moe_route", ctx.h, C.byref(layer), hidden, ptr(x), x.shape[0], ptr(topk_idx),
             ptr(topk_w), ptr(probs), _stream(stream))


def moe_route_noalloc(router, router_dtype, n_experts, top_k, normalize, hidden, x, topk_idx,
                      topk_w, probs=None, stream=None):
    """hale_moe_route_noalloc: routing on the current device with no allocation."""
    _check(lib().hale_moe_route_noalloc(ptr(router), router_dtype, n_experts, top_k, int(normalize),
                                        hidden, ptr(x), x.shape[0], ptr(topk_idx), ptr(topk_w),
                                        ptr(probs), _stream(stream)))


class Decoder:
    """hale_decoder: Transformer::forward (transformer.rs:168-227) on the GPU.

    dims: hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab, n_experts,
    top_k, normalize_topk, eps, rope_theta. layers: one dict per layer with
    input_norm, post_norm, q_norm / k_norm (or None) as float32 arrays; q, k,
    v, o and router (MoE layers) or dense_gate / dense_up / dense_down as
    (dtype, rows, cols, encoded uint8 rows). embed, lm_head: (dtype, rows,
    cols, bytes); final_norm: float32 array. pool: the routed experts of the
    MoE layers in order (pool layer j = j-th MoE layer), or None.
    """

    def __init__(self, ctx, dims, layers, embed, lm_head, final_norm, pool, max_len, n_seqs=1, max_batch=1):
        import numpy as np
        self.ctx, self.dims, self._keep = ctx, dict(dims), []

        def vec(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype=np.float32)
            self._keep.append(a)
            return a.ctypes.data

        def mat(m):
            if m is None:
                return HostMatrix(0, 0, 0, None)
            dt, rows, cols, data = m
            data = np.ascontiguousarray(data, dtype=np.uint8)
            self._keep.append(data)
            return HostMatrix(dt, rows, cols, data.ctypes.data)

        arr = (DecoderLayer * len(layers))()
        for i, L in enumerate(layers):
            moe = L.get("router") is not None
            arr[i] = DecoderLayer(vec(L["input_norm"]), vec(L["post_norm"]), vec(L.get("q_norm")),
                                  vec(L.get("k_norm")), mat(L["q"]), mat(L["k"]), mat(L["v"]), mat(L["o"]),
                                  int(moe), mat(L.get("router")), mat(L.get("dense_gate")),
                                  mat(L.get("dense_up")), mat(L.get("dense_down")))
        d = dims
        desc = DecoderDesc(d["hidden"], d["n_layers"], d["n_heads"], d["n_kv_heads"], d["head_dim"], d["vocab"],
                           d.get("n_experts", 0), d.get("top_k", 0), int(d.get("normalize_topk", 0)), d["eps"],
                           d["rope_theta"], mat(embed), mat(lm_head), vec(final_norm))
        h = P()
        ctx.call("hale_decoder_create_batched", ctx.h, C.byref(desc), arr, pool.h if pool is not None else None,
                 max_len, n_seqs, max_batch, C.byref(h))
        self.n_seqs, self.max_batch, self.max_len = n_seqs, max_batch, max_len
        self.h = h
        self.pool = pool

    def forward(self, token, position, logits=None, hidden=None, stream=None):
        """One decode step; logits / hidden: device tensors or None."""
        self.ctx.call("hale_decoder_forward", self.ctx.h, self.h, int(token), int(position), ptr(logits),
                      ptr(hidden), _stream(stream))

    def step(self, tokens, positions, seqs=None, logits=None, last_logits_only=False, hidden=None, stream=None):
        """hale_decoder_step: one step over rows (tokens[r], positions[r],
        seqs[r]); a prompt's consecutive positions in one call is batched
        prefill, one row per sequence is batched decode. logits: device
        [n, vocab] ([1, vocab] with last_logits_only) or None."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint32)
        sq = None if seqs is None else np.ascontiguousarray(seqs, dtype=np.uint32)
        if p.shape != t.shape or (sq is not None and sq.shape != t.shape):
            raise ValueError("tokens, positions and seqs must have the same length")
        self.ctx.call("hale_decoder_step", self.ctx.h, self.h, t.ctypes.data, p.ctypes.data,
                      None if sq is None else sq.ctypes.data, int(t.size), ptr(logits), int(bool(last_logits_only)),
                      ptr(hidden), _stream(stream))

    def generate(self, prompt, params, seed, max_new_tokens, stop_tokens=(), stream=None):
        """hale_decoder_generate (generate(), generator.rs:55-94): prompt ->
        (new token ids, prefill ms, decode ms)."""
        import numpy as np
        pr = np.ascontiguousarray(prompt, dtype=np.uint32)
        stops = np.ascontiguousarray(stop_tokens, dtype=np.uint32)
        out = np.zeros(max(int(max_new_tokens), 1), dtype=np.uint32)
        n = C.c_uint32()
        pms, dms = C.c_float(), C.c_float()
        self.ctx.call("hale_decoder_generate", self.ctx.h, self.h, pr.ctypes.data, int(pr.size), C.byref(params),
                      int(seed), int(max_new_tokens), stops.ctypes.data if stops.size else None, int(stops.size),
                      out.ctypes.data, C.byref(n), C.byref(pms), C.byref(dms), _stream(stream))
        return out[: n.value].tolist(), pms.value, dms.value

    def set_comm(self, comm):
        """hale_decoder_set_comm: MoE layers expert-parallel over `comm` (this
        decoder's pool holds the rank's share of the experts), or None."""
        self.ctx.call("hale_decoder_set_comm", self.h, comm.h if comm is not None else None)
        self.comm = comm

    def close(self):
        if getattr(self, "h", None):
            lib().hale_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def q8_aux_pairs(cols):
    """int2 entries per Q8Activations aux row: (cols / 32) rounded up to even."""
    return lib().hale_q8_aux_pairs(cols)


def ep_dispatch(ctx, layer, hidden, x, n_ranks, send_q, send_aux, send_meta, topk_idx=None, topk_w=None,
                stream=None):
    """hale_ep_dispatch: route x [M, hidden], pack one record per route in
    owner-rank order. Returns the record count per owner rank (list)."""
    counts = (U64 * n_ranks)()
    ctx.call("hale_ep_dispatch", ctx.h, C.byref(layer), hidden, ptr(x), x.shape[0], n_ranks, ptr(send_q),
             ptr(send_aux), ptr(send_meta), counts, ptr(topk_idx), ptr(topk_w), _stream(stream))
    return [int(c) for c in counts]


def ep_experts(ctx, pool, layer, expert0, recv_q, recv_aux, recv_meta, y, stream=None):
    """hale_ep_experts: y[j] = Expert(record j) for the received records."""
    ctx.call("hale_ep_experts", ctx.h, pool.h, layer, expert0, ptr(recv_q), ptr(recv_aux), ptr(recv_meta),
             recv_meta.shape[0], ptr(y), _stream(stream))


def ep_combine(ctx, send_meta, y_back, m_tokens, top_k, hidden, out, stream=None):
    """hale_ep_combine: out[t] = best-first weighted sum of the token's y rows."""
    ctx.call("hale_ep_combine", ctx.h, ptr(send_meta), ptr(y_back), m_tokens, top_k, hidden, ptr(out),
             _stream(stream))


COMM_ID_BYTES = 128


def comm_unique_id():
    """hale_comm_unique_id: a fresh communicator id (bytes) for hale_comm_create."""
    buf = C.create_string_buffer(COMM_ID_BYTES)
    _check(lib().hale_comm_unique_id(buf))
    return buf.raw


class Comm:
    """hale_comm: this rank's place in an expert-parallel group of n_ranks
    GPUs (collective create / close; one per process and GPU)."""

    def __init__(self, ctx, n_ranks, rank, unique_id, hidden, n_experts, top_k, max_tokens):
        h = P()
        uid = C.create_string_buffer(bytes(unique_id), COMM_ID_BYTES) if unique_id is not None else None
        ctx.call("hale_comm_create", ctx.h, n_ranks, rank, uid, hidden, n_experts, top_k, max_tokens,
                 C.byref(h))
        self.ctx, self.h = ctx, h
        self.n_ranks, self.rank, self.hidden, self.n_experts, self.top_k = n_ranks, rank, hidden, n_experts, top_k
        self.max_tokens = max_tokens

    def close(self):
        if self.h:
            h, self.h = self.h, None
            self.ctx.call("hale_comm_destroy", h)


def moe_forward_ep(ctx, comm, pool, layer, x, out, topk_idx=None, topk_w=None, stream=None):
    """hale_moe_forward_ep: this rank's tokens through the expert-parallel layer."""
    ctx.call("hale_moe_forward_ep", ctx.h, comm.h, pool.h, C.byref(layer), ptr(x), x.shape[0], ptr(out),
             ptr(topk_idx), ptr(topk_w), _stream(stream))


def quantize_q8(ctx, x, scales, quants, stream=None):
    ctx.call("hale_quantize_q8", ctx.h, ptr(x), x.shape[0], x.shape[1], ptr(scales),
             ptr(quants), _stream(stream))


def sample(ctx, logits, params, rng_state, out_tokens, seen_ids=None, stream=None):
    n_seen = seen_ids.shape[1] if seen_ids is not None else 0
    ctx.call("hale_sample", ctx.h, ptr(logits), logits.shape[0], logits.shape[1],
             C.byref(params), ptr(rng_state), ptr(seen_ids), n_seen, ptr(out_tokens),
             _stream(stream))


def row_bytes(dtype, cols):
    r = lib().hale_row_bytes(dtype, cols)
    return None if r < 0 else int(r)


def expf_host(x):
    """The device exp evaluated on the host (same source)."""
    import numpy as np
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().hale_expf_host(ptr(x), ptr(y), x.size)
    return y
