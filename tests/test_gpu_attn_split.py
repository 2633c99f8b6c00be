"""Single-row decode attention spread over the GPU (attn_split_kernel).

A one-row hale_decoder_forward runs attention as score units of 32 positions
and context units of 8 head dims over the whole GPU (Attention::forward,
attention.rs:59-85, in the reference's chain order). Batched steps keep the
per-head-group kernel. Logits at every checked position must equal the
oracle's (ho_model_forward) bit for bit, over GQA ratios 1 to 32, head_dim 32
to 256, contexts that span several softmax chunks, and the first positions
(a single, partial score unit).
"""
import importlib

import numpy as np
import pytest

from oracle import model as OM

import synth
from test_gpu_decoder import build_decoder

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = hale.Context(0)
    yield c
    c.check()
    c.close()


@pytest.mark.parametrize("heads,kv_heads,head_dim,n", [
    (8, 2, 32, 1040),      # G = 4: two 1024-position chunks
    (32, 4, 128, 600),     # Qwen3-30B-A3B attention shape
    (16, 16, 64, 300),     # G = 1 (multi-head attention)
    (32, 2, 64, 700),      # G = 16: 512-position chunks
    (64, 2, 64, 300),      # G = 32: 256-position chunks
    (4, 1, 256, 100),      # head_dim 256
])
def test_single_row_attention_matches_the_oracle(ctx, heads, kv_heads, head_dim, n):
    hf, t, enc = synth.qwen3_moe(40 + heads, 1, 256, heads, kv_heads, head_dim, 4, 2, 64, 256, fmt.Q8_0, "F32")
    om = OM.OracleModel(expert_dtype=fmt.Q8_0, hf_config=hf, tensors=t, expert_encoded=enc)
    tokens = np.random.default_rng(heads * 7 + head_dim).integers(0, 256, n).tolist()
    want = om.teacher_forced_logits(tokens)
    dec = build_decoder(ctx, om, fmt.Q8_0, n, max_batch=256)
    one = torch.empty(256, dtype=torch.float32, device="cuda")
    got = {}
    # the first positions one row at a time (one partial score unit)
    for i in range(4):
        dec.forward(tokens[i], i, one)
        got[i] = one.cpu().numpy().copy()
    # the middle as batched prefill (the per-group kernel), the tail one row
    # at a time again
    tail = n - 6
    for s in range(4, tail, 256):
        e = min(tail, s + 256)
        dec.step(tokens[s:e], list(range(s, e)))
    for i in range(tail, n):
        dec.forward(tokens[i], i, one)
        got[i] = one.cpu().numpy().copy()
    ctx.check()
    dec.close()
    for i, g in got.items():
        diff = g.view(np.uint32) != want[i].view(np.uint32)
        assert not diff.any(), f"position {i}: {diff.sum()} of {diff.size} logits differ"
