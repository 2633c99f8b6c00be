"""Whole-model decode steps on the GPU (hale_decoder) against the oracle.

Transformer::forward (src/model/transformer.rs:168-227) over the reference's
two golden fixture models (tests/golden/, Qwen3-MoE with q/k norms and a
dense layer; Mixtral without), with the routed experts in the pack formats
(q8_0 / q4_0, converted as src/convert.rs does): every position's logits must
equal the oracle's ho_model_forward on the same weights bit for bit, the
greedy continuation must match, and with unquantized-expert tolerance the
logits stay near the fixture's own (the oracle is pinned to those).
"""
import importlib
import json
import os

import numpy as np
import pytest

from oracle import model as OM
from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ST_CODE = {"F32": fmt.F32, "BF16": fmt.BF16, "F16": fmt.F16}


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = hale.Context(0)
    yield c
    c.check()
    c.close()


def build_decoder(ctx, om, expert_dtype, max_len):
    """The fixture's tensors (same names and normalisation as the oracle
    loader) as hale_decoder descriptors, experts encoded like the oracle's."""
    c = om.cfg
    expert_name, router_name, dense_name = OM._names(c["qwen"])

    def hm(name):
        dt, shape, raw = om.raw(name)
        return (ST_CODE[dt], shape[0], shape[1], raw)

    moe_layers = [l for l in range(c["layers"]) if l not in c["dense_layers"]]
    pool = None
    if moe_layers:
        pool = hale.Pool(ctx, expert_dtype, c["hidden"], c["expert_inter"], len(moe_layers), c["experts"])
    layers = []
    for l in range(c["layers"]):
        p = f"model.layers.{l}."
        L = dict(input_norm=om.f32(p + "input_layernorm.weight"), post_norm=om.f32(p + "post_attention_layernorm.weight"),
                 q=hm(p + "self_attn.q_proj.weight"), k=hm(p + "self_attn.k_proj.weight"),
                 v=hm(p + "self_attn.v_proj.weight"), o=hm(p + "self_attn.o_proj.weight"))
        if c["qwen"]:
            L["q_norm"] = om.f32(p + "self_attn.q_norm.weight")
            L["k_norm"] = om.f32(p + "self_attn.k_norm.weight")
        if l in c["dense_layers"]:
            L["dense_gate"] = hm(dense_name(l, "gate"))
            L["dense_up"] = hm(dense_name(l, "up"))
            L["dense_down"] = hm(dense_name(l, "down"))
        else:
            L["router"] = hm(router_name(l))
            j = moe_layers.index(l)
            for e in range(c["experts"]):
                enc = [O.encode(expert_dtype, om.f32(expert_name(l, e, pj))) for pj in ("gate", "up", "down")]
                pool.upload(j, e, fmt.pack_record(*enc))
        layers.append(L)
    embed = hm("model.embed_tokens.weight")
    head = embed if (c["tie"] or "lm_head.weight" not in om.t) else hm("lm_head.weight")
    dims = dict(hidden=c["hidden"], n_layers=c["layers"], n_heads=c["heads"], n_kv_heads=c["kv_heads"],
                head_dim=c["head_dim"], vocab=c["vocab"], n_experts=c["experts"] or 0, top_k=c["top_k"],
                normalize_topk=c["normalize"], eps=c["eps"], rope_theta=c["theta"])
    return hale.Decoder(ctx, dims, layers, embed, head, om.f32("model.norm.weight"), pool, max_len)


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
@pytest.mark.parametrize("expert_dtype", [fmt.Q8_0, fmt.Q4_0])
def test_decoder_logits_are_bit_exact_against_the_oracle(ctx, name, expert_dtype):
    d = os.path.join(GOLDEN, name)
    with open(os.path.join(d, "expected.json")) as f:
        exp = json.load(f)
    tokens = exp["tokens"]
    om = OM.OracleModel(d, expert_dtype=expert_dtype)
    want = om.teacher_forced_logits(tokens)
    dec = build_decoder(ctx, om, expert_dtype, len(tokens) + 4)
    logits = torch.empty(om.cfg["vocab"], dtype=torch.float32, device="cuda")
    got = []
    for i, t in enumerate(tokens):
        dec.forward(t, i, logits)
        got.append(logits.cpu().numpy().copy())
    ctx.check()
    got = np.stack(got)
    diff = got.view(np.uint32) != want.view(np.uint32)
    assert not diff.any(), f"{diff.sum()} of {diff.size} logits differ; first at {np.argwhere(diff)[0]}"
    dec.close()


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
def test_decoder_greedy_generation_matches_the_oracle(ctx, name):
    d = os.path.join(GOLDEN, name)
    with open(os.path.join(d, "expected.json")) as f:
        exp = json.load(f)
    prompt, n = exp["prompt"], len(exp["greedy_continuation"])
    om = OM.OracleModel(d, expert_dtype=fmt.Q8_0)
    want = om.greedy(prompt, n)
    dec = build_decoder(ctx, om, fmt.Q8_0, len(prompt) + n + 1)
    logits = torch.empty(om.cfg["vocab"], dtype=torch.float32, device="cuda")
    for i, t in enumerate(prompt):
        dec.forward(t, i, logits)
    out, pos = [], len(prompt)
    for step in range(n):
        tok = int(torch.argmax(logits).item())   # first index of the max, as argmax (activation.rs:24-32)
        out.append(tok)
        if step + 1 == n:
            break
        dec.forward(tok, pos, logits)
        pos += 1
    assert out == list(want)
    dec.close()


def test_decoder_rejects_positions_beyond_its_cache(ctx):
    d = os.path.join(GOLDEN, "tiny-mixtral")
    om = OM.OracleModel(d, expert_dtype=fmt.Q8_0)
    dec = build_decoder(ctx, om, fmt.Q8_0, 4)
    with pytest.raises(hale.HaleError) as ei:
        dec.forward(1, 4)
    assert ei.value.status == hale.E_CONTEXT_OVERFLOW
    with pytest.raises(hale.HaleError) as ei:
        dec.forward(om.cfg["vocab"], 0)
    assert ei.value.status == hale.E_INVALID_ARGUMENT
    dec.close()


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
def test_checkpoint_loader_builds_a_bit_exact_decoder(ctx, name):
    """load_decoder reads config.json + safetensors itself (config.rs,
    safetensors.rs, arch.rs naming) and converts the experts to q4_0; its
    logits equal the oracle's on the same checkpoint bit for bit."""
    loader = importlib.import_module("hale-token_b200.loader")
    d = os.path.join(GOLDEN, name)
    with open(os.path.join(d, "expected.json")) as f:
        tokens = json.load(f)["tokens"]
    want = OM.OracleModel(d, expert_dtype=fmt.Q4_0).teacher_forced_logits(tokens)
    dec, pool, cfg = loader.load_decoder(ctx, d, fmt.Q4_0, max_len=len(tokens))
    logits = torch.empty(cfg.vocab_size, dtype=torch.float32, device="cuda")
    got = []
    for i, t in enumerate(tokens):
        dec.forward(t, i, logits)
        got.append(logits.cpu().numpy().copy())
    ctx.check()
    got = np.stack(got)
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    dec.close()
