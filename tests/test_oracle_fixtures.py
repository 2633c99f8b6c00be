"""Pins the CPU oracle to the reference's golden fixtures.

tests/golden/<name>/ holds the reference's tiny random-weight models and the
logits its independent float64 NumPy model produced (copied by
tests/golden/make_golden.py). These restate the reference's integration
tests: tests/litmus.rs:17-59 and tests/tiered_cache.rs:83-102.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import model as OM
from oracle import oracle as O

from conftest import GOLDEN

FIXTURES = ["tiny-qwen3-moe", "tiny-mixtral"]
LOGIT_TOLERANCE = 2e-3  # litmus.rs:15


def expected(name):
    with open(os.path.join(GOLDEN, name, "expected.json")) as f:
        return json.load(f)


def test_golden_files_match_their_manifest():
    with open(os.path.join(GOLDEN, "MANIFEST.json")) as f:
        man = json.load(f)
    for rel, digest in man["files"].items():
        with open(os.path.join(GOLDEN, rel), "rb") as fh:
            assert hashlib.sha256(fh.read()).hexdigest() == digest, rel


@pytest.mark.parametrize("name", FIXTURES)
def test_logits_match_the_reference_for_every_position(name):
    """litmus.rs:17-27"""
    exp = expected(name)
    m = OM.OracleModel(os.path.join(GOLDEN, name))
    got = m.teacher_forced_logits(exp["tokens"])
    diff = np.abs(got - np.asarray(exp["logits"], np.float32)).max()
    assert diff < LOGIT_TOLERANCE, diff


@pytest.mark.parametrize("name", FIXTURES)
def test_greedy_generation_matches_the_reference(name):
    """litmus.rs:29-45"""
    exp = expected(name)
    m = OM.OracleModel(os.path.join(GOLDEN, name))
    assert m.greedy(exp["prompt"], len(exp["greedy_continuation"])) == exp["greedy_continuation"]


def test_prefill_equals_token_by_token_forward():
    """litmus.rs:47-59 (bit-identical)."""
    exp = expected(FIXTURES[0])
    m = OM.OracleModel(os.path.join(GOLDEN, FIXTURES[0]))
    cache = m.new_cache(64)
    prompt = exp["prompt"]
    for i, t in enumerate(prompt[:-1]):
        m.forward(t, i, cache, want_logits=False)
    prefill = m.forward(prompt[-1], len(prompt) - 1, cache)
    step = m.teacher_forced_logits(prompt)[-1]
    assert np.array_equal(prefill.view(np.uint32), step.view(np.uint32))


@pytest.mark.parametrize("name", FIXTURES)
def test_quantized_packs_stay_close_to_the_reference(name):
    """tiered_cache.rs:83-102"""
    exp = expected(name)
    want = np.asarray(exp["logits"], np.float32).astype(np.float64)
    for dtype, max_rms, min_top1 in [(O.Q8_0, 0.01, 0.95), (O.Q4_0, 0.25, 0.6)]:
        m = OM.OracleModel(os.path.join(GOLDEN, name), expert_dtype=dtype)
        got = m.teacher_forced_logits(exp["tokens"]).astype(np.float64)
        rms = np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum())
        top1 = np.mean([O.argmax(g.astype(np.float32)) == O.argmax(w.astype(np.float32))
                        for g, w in zip(got, want)])
        assert rms < max_rms, (dtype, rms)
        assert top1 >= min_top1, (dtype, top1)
