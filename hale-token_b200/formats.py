"""Host-side encoders for the reference's weight formats (numpy, vectorised).

These produce the exact bytes Hale-Token's converter writes
(src/tensor/quant.rs:274-321 via WeightMatrix::from_f32, matrix.rs:48-61)
and the expert-pack record layout gate | up | down
(src/expert/pack.rs:15-16, 125-133). They are data preparation for the
device pool -- the GPU consumes these bytes through the C ABI -- and are
checked byte-for-byte against the CPU oracle in tests/test_formats.py.
"""
import numpy as np

F32, F16, BF16, Q8_0, Q4_0 = 0, 1, 2, 3, 4
QK = 32
BLOCK_BYTES = {F32: 4, F16: 2, BF16: 2, Q8_0: 34, Q4_0: 18}
NAMES = {"f32": F32, "f16": F16, "bf16": BF16, "q8_0": Q8_0, "q4_0": Q4_0}


def row_bytes(dtype, cols):
    """DType::row_bytes (dtype.rs:53-61)."""
    bl = QK if dtype in (Q8_0, Q4_0) else 1
    if cols % bl:
        raise ValueError(f"dtype {dtype} needs row length divisible by {bl}, got {cols}")
    return cols // bl * BLOCK_BYTES[dtype]


def _f16_bytes(v):
    return np.asarray(v, dtype=np.float32).astype(np.float16).view(np.uint8)


def _bf16_bits(v):
    """f32 -> bf16 round-to-nearest-even (NaN kept quiet)."""
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    out = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(v, dtype=np.float32))
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def _sat_trunc(x, lo, hi):
    """Rust `f as i32` then clamp(lo, hi): truncation, NaN -> 0."""
    x = np.where(np.isnan(x), np.float32(0), x)
    return np.clip(np.trunc(x), lo, hi)


def _round_away(x):
    """f32::round: half away from zero (exact: x - trunc(x) is exact)."""
    t = np.trunc(x)
    frac = x - t
    return t + np.where(np.abs(frac) >= np.float32(0.5), np.sign(x), np.float32(0)).astype(np.float32)


def encode_q8_0(values):
    """encode_block_q8_0 (quant.rs:295-305) over rows of 32-multiples."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    rows, cols = v.shape
    b = v.reshape(rows, cols // QK, QK)
    amax = np.fmax.reduce(np.abs(b), axis=2, initial=np.float32(0))
    scale = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, np.float32(1.0) / np.where(scale > 0, scale, 1), 0).astype(np.float32)
    q = _round_away((b * inv[..., None]).astype(np.float32))
    q = np.where(np.isnan(q), 0, np.clip(q, -127, 127)).astype(np.int8)
    out = np.empty((rows, cols // QK, 34), dtype=np.uint8)
    out[..., :2] = _f16_bytes(scale).reshape(rows, cols // QK, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def encode_q4_0(values):
    """encode_block_q4_0 (quant.rs:309-321): the first element of greatest
    magnitude maps to -8; nibble j holds element j (low) and j+16 (high)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    rows, cols = v.shape
    b = v.reshape(rows, cols // QK, QK)
    idx = np.argmax(np.abs(b), axis=2)
    extreme = np.take_along_axis(b, idx[..., None], axis=2)[..., 0]
    scale = (extreme / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(scale != 0, np.float32(1.0) / np.where(scale != 0, scale, 1), 0).astype(np.float32)
    q = _sat_trunc(((b * inv[..., None]).astype(np.float32) + np.float32(8.5)).astype(np.float32), 0, 15)
    q = q.astype(np.uint8)
    out = np.empty((rows, cols // QK, 18), dtype=np.uint8)
    out[..., :2] = _f16_bytes(scale).reshape(rows, cols // QK, 2)
    out[..., 2:] = q[..., :16] | (q[..., 16:] << 4)
    return out.reshape(rows, -1)


def encode(dtype, values):
    """WeightMatrix::from_f32 (matrix.rs:48-61) -> [rows, row_bytes] uint8."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.ndim == 1:
        v = v[None, :]
    if dtype == F32:
        return v.view(np.uint8).reshape(v.shape[0], -1)
    if dtype == F16:
        return v.astype(np.float16).view(np.uint8).reshape(v.shape[0], -1)
    if dtype == BF16:
        return _bf16_bits(v).view(np.uint8).reshape(v.shape[0], -1)
    if dtype == Q8_0:
        return encode_q8_0(v)
    if dtype == Q4_0:
        return encode_q4_0(v)
    raise ValueError(f"unknown dtype {dtype}")


def decode(dtype, rows, cols):
    """decode_row per row (quant.rs:236-269): [rows, row_bytes] uint8 -> f32
    [rows, cols]; quantized values are scale * q in f32."""
    r = np.ascontiguousarray(rows, dtype=np.uint8)
    r = r.reshape(-1, row_bytes(dtype, cols))
    n = r.shape[0]
    if dtype == F32:
        return r.view(np.float32).reshape(n, cols).copy()
    if dtype == F16:
        return r.view(np.float16).astype(np.float32).reshape(n, cols)
    if dtype == BF16:
        return (r.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(n, cols)
    b = r.reshape(n, cols // QK, BLOCK_BYTES[dtype])
    scale = b[..., :2].copy().view(np.float16).astype(np.float32)  # [n, nb, 1]
    if dtype == Q8_0:
        q = b[..., 2:].view(np.int8).astype(np.float32)
    elif dtype == Q4_0:
        nib = b[..., 2:]
        q = np.concatenate([(nib & 0x0F), (nib >> 4)], axis=-1).astype(np.float32) - np.float32(8.0)
    else:
        raise ValueError(f"unknown dtype {dtype}")
    return (scale * q).astype(np.float32).reshape(n, cols)


def pack_record(gate, up, down):
    """One expert-pack record: gate | up | down encoded rows (pack.rs:15-16)."""
    return np.concatenate([np.ascontiguousarray(m, dtype=np.uint8).reshape(-1) for m in (gate, up, down)])


def split_record(record, dtype, hidden, inter):
    """PackHeader::decode_record (pack.rs:125-133) -> (gate, up, down) rows."""
    proj = inter * row_bytes(dtype, hidden)
    r = np.ascontiguousarray(record, dtype=np.uint8)
    gate = r[:proj].reshape(inter, -1)
    up = r[proj:2 * proj].reshape(inter, -1)
    down = r[2 * proj:2 * proj + hidden * row_bytes(dtype, inter)].reshape(hidden, -1)
    return gate, up, down


class SyntheticLayer:
    """A seeded random MoE layer (BASELINE config shapes): router f32
    N(0, 0.02) [E, H]; experts N(0, 0.02) encoded in `dtype`.

    Experts are generated one at a time from per-expert seeds, so any
    subset can be rebuilt identically (the oracle checks a subset)."""

    def __init__(self, seed, n_experts, hidden, inter, dtype=Q4_0, std=0.02):
        self.seed, self.E, self.H, self.I, self.dtype, self.std = seed, n_experts, hidden, inter, dtype, std
        rng = np.random.default_rng([seed, 0xA11CE])
        self.router = (rng.standard_normal((n_experts, hidden), dtype=np.float32) * np.float32(std))

    def expert_f32(self, e):
        rng = np.random.default_rng([self.seed, 1, e])
        s = np.float32(self.std)
        g = rng.standard_normal((self.I, self.H), dtype=np.float32) * s
        u = rng.standard_normal((self.I, self.H), dtype=np.float32) * s
        d = rng.standard_normal((self.H, self.I), dtype=np.float32) * s
        return g, u, d

    def expert_encoded(self, e):
        g, u, d = self.expert_f32(e)
        return encode(self.dtype, g), encode(self.dtype, u), encode(self.dtype, d)

    def record(self, e):
        return pack_record(*self.expert_encoded(e))

    def tokens(self, m, seed=None):
        rng = np.random.default_rng([self.seed, 2, m if seed is None else seed])
        return rng.standard_normal((m, self.H), dtype=np.float32)

    def expert_bytes(self):
        return 2 * self.I * row_bytes(self.dtype, self.H) + self.H * row_bytes(self.dtype, self.I)
