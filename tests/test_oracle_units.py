"""Pins the CPU oracle to the reference's own unit tests.

Each test restates a `#[test]` of the Rust reference (file:line in the
docstring) against the C restatement in oracle/. These run on CPU.
"""
import numpy as np
import pytest

from oracle import oracle as O


def ref_values(n, seed):
    """Deterministic values in [-1, 1) (src/tensor/quant.rs:328-338)."""
    s = np.uint32((seed * 2654435761) & 0xFFFFFFFF)
    s = max(int(s), 1)
    out = np.zeros(n, dtype=np.float32)
    umax = np.float32(4294967295.0)  # `u32::MAX as f32` rounds to 2^32
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        out[i] = (np.float32(s) / umax) * np.float32(2.0) - np.float32(1.0)
    return out


ALL = [O.F32, O.F16, O.BF16, O.Q8_0, O.Q4_0]


def test_row_bytes_match_the_block_layout():
    """dtype.rs:120-127"""
    assert O.row_bytes(O.F32, 64) == 256
    assert O.row_bytes(O.BF16, 64) == 128
    assert O.row_bytes(O.Q8_0, 64) == 68
    assert O.row_bytes(O.Q4_0, 64) == 36
    assert O.row_bytes(O.Q4_0, 33) is None


def test_every_dtype_round_trips_within_its_precision():
    """quant.rs:344-366"""
    v = ref_values(96, 7)
    for dtype, tol in [(O.F32, 0.0), (O.F16, 1e-3), (O.BF16, 1e-2), (O.Q8_0, 1e-2), (O.Q4_0, 0.15)]:
        b = O.encode(dtype, v)
        assert b.shape[0] == O.row_bytes(dtype, 96)
        back = O.decode(dtype, b, 96)
        assert np.abs(v - back).max() <= tol, dtype


def test_dot_equals_dot_of_decoded_row():
    """quant.rs:368-398"""
    w, x = ref_values(64, 3), ref_values(64, 11)
    for dtype in ALL:
        b = O.encode(dtype, w)
        dec = O.decode(dtype, b, 64)
        expect = float(np.sum(dec * x, dtype=np.float32))
        got = O.dot(dtype, b, x)
        tol = 2e-2 * max(abs(expect), 1.0) if dtype in (O.Q8_0, O.Q4_0) else 1e-4
        assert abs(expect - got) < tol, (dtype, expect, got)
    w, x = ref_values(13, 5), ref_values(13, 9)
    b = O.encode(O.F32, w)
    assert abs(O.dot(O.F32, b, x) - float(np.dot(w.astype(np.float64), x))) < 1e-5


def test_unaligned_rows_give_the_same_answer_as_aligned_ones():
    """quant.rs:400-420"""
    w, x = ref_values(100, 4), ref_values(100, 8)
    for dtype in (O.F32, O.F16, O.BF16):
        b = O.encode(dtype, w)
        shifted = np.zeros(b.shape[0] + 1, dtype=np.uint8)
        shifted[1:] = b
        un = shifted[1:]
        assert O.dot(dtype, b, x) == O.dot(dtype, un, x)
        assert np.array_equal(O.decode(dtype, b, 100), O.decode(dtype, un, 100))


def test_zero_block_quantizes_to_zero():
    """quant.rs:422-432"""
    for dtype in (O.Q8_0, O.Q4_0):
        back = O.decode(dtype, O.encode(dtype, np.zeros(32, np.float32)), 32)
        assert np.all(back == 0.0)


def test_matvec_matches_naive_product_and_parallel_equals_serial():
    """matrix.rs:292-316"""
    rows, cols = 70, 64
    i = np.arange(rows * cols)
    w = (((i * 37) % 101).astype(np.float32) - np.float32(50.0)) / np.float32(50.0)
    x = (np.arange(cols, dtype=np.float32) / np.float32(cols)) - np.float32(0.5)
    expect = (w.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64))
    m = O.encode(O.F32, w.reshape(rows, cols))
    par = O.matvec(O.F32, m, rows, cols, x, parallel=True)
    ser = O.matvec(O.F32, m, rows, cols, x, parallel=False)
    assert np.array_equal(par.view(np.uint32), ser.view(np.uint32))
    assert np.abs(par - expect).max() < 1e-4


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q4_0, O.BF16])
def test_parallel_matvec_is_bit_identical_for_every_dtype(dtype):
    """matrix.rs:167-170 (determinism regardless of threading), large shape."""
    rng = np.random.default_rng(5)
    rows, cols = 300, 256
    w = O.encode(dtype, rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal(cols).astype(np.float32)
    par = O.matvec(dtype, w, rows, cols, x, parallel=True)
    ser = O.matvec(dtype, w, rows, cols, x, parallel=False)
    assert np.array_equal(par.view(np.uint32), ser.view(np.uint32))


def test_convert_quantizes_and_keeps_shape():
    """matrix.rs:324-331"""
    w = np.sin(np.arange(4 * 64, dtype=np.float32)).reshape(4, 64)
    q = O.encode(O.Q8_0, w)
    assert q.shape == (4, 68)
    assert q.nbytes < w.nbytes / 3


def test_top_k_matches_full_sort():
    """topk.rs:119-128"""
    scores = (((np.arange(128) * 73) % 128).astype(np.float32) * np.float32(0.37)) - np.float32(20.0)
    order = sorted(range(128), key=lambda a: (-scores[a], a))
    idx, _ = O.top_k(scores, 8)
    assert list(idx) == order[:8]


def test_top_k_ties_prefer_lower_index_and_k_is_clamped():
    """topk.rs:130-139"""
    idx, _ = O.top_k(np.array([1.0, 5.0, 5.0, 5.0], np.float32), 2)
    assert list(idx) == [1, 2]
    assert len(O.top_k(np.array([1.0, 2.0], np.float32), 10)[0]) == 2
    assert len(O.top_k(np.array([1.0], np.float32), 0)[0]) == 0


def test_softmax_sums_to_one_and_survives_huge_logits():
    """activation.rs:38-44"""
    x = O.softmax(np.array([1000.0, 1001.0, 1002.0], np.float32))
    assert abs(float(np.sum(x, dtype=np.float32)) - 1.0) < 1e-6
    assert x[2] > x[1] > x[0]


def test_silu_and_argmax_basics():
    """activation.rs:46-51"""
    assert O.silu(0.0) == 0.0
    assert abs(O.silu(10.0) - 10.0) < 1e-3
    assert O.argmax(np.array([1.0, 3.0, 3.0, -1.0], np.float32)) == 1


def test_rms_norm_normalizes_to_unit_rms():
    """norm.rs:33-46"""
    x = np.array([3.0, -4.0, 0.0, 5.0], np.float32)
    out = O.rms_norm(x, np.ones(4, np.float32), 0.0)
    assert abs(np.sqrt(np.mean(out.astype(np.float64) ** 2)) - 1.0) < 1e-6
    y = O.rms_norm_in_place(x, np.full(4, 2.0, np.float32), 0.0)
    assert np.abs(y - 2.0 * out).max() < 1e-6


def test_rope_position_zero_is_identity_and_rotation_preserves_norm():
    """rope.rs:50-66"""
    c, s = O.rope_tables(8, 10000.0, 0)
    orig = np.arange(1, 9, dtype=np.float32)
    h = O.rope_apply(orig, c, s)
    assert np.array_equal(h, orig)
    c, s = O.rope_tables(8, 10000.0, 17)
    h = O.rope_apply(h, c, s)
    assert abs(float(np.sum(h * h)) - float(np.sum(orig * orig))) < 1e-3
    assert not np.array_equal(h, orig)


def test_greedy_picks_the_argmax():
    """sampler.rs:152-156"""
    assert O.Sampler(temperature=0.0).sample(np.array([0.1, 3.0, -1.0], np.float32)) == 1
    assert O.Sampler(temperature=0.0).sample(np.array([5.0, 1.0], np.float32)) == 0


def test_top_p_only_samples_from_the_nucleus_and_is_reproducible():
    """sampler.rs:158-184"""
    logits = np.array([10.0, 9.5, 0.0, -5.0, -5.0], np.float32)
    a = O.Sampler(temperature=1.0, top_p=0.9, top_k=0, seed=7)
    b = O.Sampler(temperature=1.0, top_p=0.9, top_k=0, seed=7)
    seen = [0] * 5
    for _ in range(500):
        t = a.sample(logits)
        assert t == b.sample(logits)
        seen[t] += 1
    assert seen[0] > 0 and seen[1] > 0
    assert seen[2] + seen[3] + seen[4] == 0


def test_top_k_one_is_greedy():
    """sampler.rs:186-198"""
    s = O.Sampler(temperature=2.0, top_p=1.0, top_k=1, seed=3)
    for _ in range(20):
        assert s.sample(np.array([0.0, 0.1, 0.05], np.float32)) == 1


def test_xorshift_stream_matches_the_published_recurrence():
    """sampler.rs:128-146: xorshift64* (>>12, <<25, >>27, * 0x2545F4914F6CDD1D)."""
    r = O.XorShift64(0)  # seed.max(1)
    s = 1
    M = (1 << 64) - 1
    for _ in range(100):
        s ^= s >> 12
        s ^= (s << 25) & M
        s ^= s >> 27
        assert r.next_u64() == (s * 0x2545F4914F6CDD1D) & M


def test_repetition_penalty_follows_the_hf_convention():
    """Extension (not in the reference): l>0 -> l/p, else l*p, once per id."""
    lg = np.array([2.0, -2.0, 1.0, 0.0], np.float32)
    out = O.apply_repetition_penalty(lg, [0, 1, 1, 3], 2.0)
    assert list(out) == [1.0, -4.0, 1.0, 0.0]


def test_f16_and_bf16_conversions_round_to_nearest_even():
    """half::f16::from_f32 / bf16::from_f32 (used at quant.rs:280-284, 299, 316)."""
    import torch
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                        for s in (1e-7, 1e-5, 1e-3, 1.0, 1e3, 7e4)])
    v = np.concatenate([v, np.array([0.0, -0.0, 65504.0, 65520.0, 6.1e-5, 5.96e-8, 2.98e-8,
                                     np.inf, -np.inf], np.float32)])
    L = O.lib()
    f16 = np.array([L.ho_f32_to_f16(float(x)) for x in v], dtype=np.uint16)
    with np.errstate(over="ignore"):
        ref16 = v.astype(np.float16).view(np.uint16)
    assert np.array_equal(f16, ref16)
    back = np.array([L.ho_f16_to_f32(int(h)) for h in f16], dtype=np.float32)
    assert np.array_equal(back, f16.view(np.float16).astype(np.float32))
    bf = np.array([L.ho_f32_to_bf16(float(x)) for x in v], dtype=np.uint16)
    tb = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bf, tb)
