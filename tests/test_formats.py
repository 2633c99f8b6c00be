"""The package's numpy encoders produce the reference's bytes exactly
(checked against the C oracle's restatement of quant.rs:274-321)."""
import importlib

import numpy as np
import pytest

from oracle import oracle as O

fmt = importlib.import_module("hale-token_b200.formats")


def cases():
    rng = np.random.default_rng(3)
    yield rng.standard_normal((17, 256)).astype(np.float32) * 0.02
    yield rng.standard_normal((5, 64)).astype(np.float32) * 1e3
    z = np.zeros((2, 64), np.float32)
    z[1, 5] = -3.0          # single extreme, negative
    yield z
    t = np.tile(np.float32([1.0, -1.0]), (3, 64))  # ties in |v|: first one wins (q4)
    yield t
    h = (np.arange(4 * 96, dtype=np.float32).reshape(4, 96) - 190.0) / 7.0  # exact .5 steps
    yield h
    tiny = rng.standard_normal((3, 64)).astype(np.float32) * 1e-30
    yield tiny


@pytest.mark.parametrize("dtype", [fmt.F32, fmt.F16, fmt.BF16, fmt.Q8_0, fmt.Q4_0])
def test_numpy_encoders_match_the_oracle_bytes(dtype):
    for v in cases():
        assert np.array_equal(fmt.encode(dtype, v), O.encode(dtype, v)), dtype


def test_pack_record_round_trip():
    layer = fmt.SyntheticLayer(1, 4, 64, 32, fmt.Q4_0)
    rec = layer.record(2)
    assert rec.nbytes == layer.expert_bytes() == 2 * 32 * 36 + 64 * 18
    g, u, d = fmt.split_record(rec, fmt.Q4_0, 64, 32)
    eg, eu, ed = layer.expert_encoded(2)
    assert np.array_equal(g, eg) and np.array_equal(u, eu) and np.array_equal(d, ed)


def test_row_bytes_rejects_ragged_quantized_rows():
    with pytest.raises(ValueError):
        fmt.row_bytes(fmt.Q4_0, 33)
    assert fmt.row_bytes(fmt.Q8_0, 64) == 68
