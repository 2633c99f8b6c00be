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

import synth

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


def build_decoder(ctx, om, expert_dtype, max_len, n_seqs=1, max_batch=1, experts=None):
    """The fixture's tensors (same names and normalisation as the oracle
    loader) as hale_decoder descriptors, experts encoded like the oracle's.
    experts: the global expert ids the pool holds (local ids 0..), default
    all of them (an expert-parallel rank holds its own block)."""
    c = om.cfg
    expert_name, router_name, dense_name = OM._names(c["qwen"])

    def hm(name):
        dt, shape, raw = om.raw(name)
        return (ST_CODE[dt], shape[0], shape[1], raw)

    moe_layers = [l for l in range(c["layers"]) if l not in c["dense_layers"]]
    pool = None
    ids = list(range(c["experts"] or 0)) if experts is None else list(experts)
    if moe_layers:
        pool = hale.Pool(ctx, expert_dtype, c["hidden"], c["expert_inter"], len(moe_layers), len(ids))
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
            for le, e in enumerate(ids):
                if om.expert_encoded is not None:
                    enc = [om.expert_encoded(l, e, pj) for pj in ("gate", "up", "down")]
                else:
                    enc = [O.encode(expert_dtype, om.f32(expert_name(l, e, pj))) for pj in ("gate", "up", "down")]
                pool.upload(j, le, fmt.pack_record(*enc))
        layers.append(L)
    embed = hm("model.embed_tokens.weight")
    head = embed if (c["tie"] or "lm_head.weight" not in om.t) else hm("lm_head.weight")
    dims = dict(hidden=c["hidden"], n_layers=c["layers"], n_heads=c["heads"], n_kv_heads=c["kv_heads"],
                head_dim=c["head_dim"], vocab=c["vocab"], n_experts=c["experts"] or 0, top_k=c["top_k"],
                normalize_topk=c["normalize"], eps=c["eps"], rope_theta=c["theta"])
    return hale.Decoder(ctx, dims, layers, embed, head, om.f32("model.norm.weight"), pool, max_len, n_seqs, max_batch)


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


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
@pytest.mark.parametrize("max_batch", [1, 4])
def test_generate_greedy_matches_the_oracle(ctx, name, max_batch):
    """hale_decoder_generate (generate(), generator.rs:55-94) with greedy
    sampling: the fixture's prompt prefilled in steps of max_batch rows, then
    sample -> step on the device; the tokens equal the oracle's greedy run.
    A stop token ends the output right after it; asking for more positions
    than the cache holds is ContextOverflow."""
    d = os.path.join(GOLDEN, name)
    with open(os.path.join(d, "expected.json")) as f:
        exp = json.load(f)
    prompt, n = exp["prompt"], len(exp["greedy_continuation"])
    om = OM.OracleModel(d, expert_dtype=fmt.Q8_0)
    want = list(om.greedy(prompt, n))
    dec = build_decoder(ctx, om, fmt.Q8_0, len(prompt) + n, max_batch=max_batch)
    greedy = hale.SamplingParams(0.0, 1.0, 0, 1.0)
    got, prefill_ms, decode_ms = dec.generate(prompt, greedy, 42, n)
    assert got == want
    assert prefill_ms > 0 and decode_ms > 0
    stop = want[2]
    got_s, _, _ = dec.generate(prompt, greedy, 42, n, stop_tokens=[stop])
    assert got_s == want[: want.index(stop) + 1]
    with pytest.raises(hale.HaleError) as ei:
        dec.generate(prompt, greedy, 42, n + 1)
    assert ei.value.status == hale.E_CONTEXT_OVERFLOW
    ctx.check()
    dec.close()


def test_generate_seeded_top_p_matches_the_oracle_loop(ctx):
    """A seeded temperature / top-k / top-p generation: the device loop's
    tokens equal the oracle's generate() loop (prefill, then TopPSampler with
    the same seed -> forward) token for token."""
    d = os.path.join(GOLDEN, "tiny-qwen3-moe")
    with open(os.path.join(d, "expected.json")) as f:
        exp = json.load(f)
    prompt, n = exp["prompt"], 10
    om = OM.OracleModel(d, expert_dtype=fmt.Q8_0)
    cache = om.new_cache(len(prompt) + n)
    for i, t in enumerate(prompt):
        logits = om.forward(t, i, cache, want_logits=(i == len(prompt) - 1))
    sampler = O.Sampler(temperature=0.8, top_p=0.9, top_k=20, seed=7)
    want = []
    for step in range(n):
        tok = sampler.sample(logits)
        want.append(tok)
        if step + 1 == n:
            break
        logits = om.forward(tok, len(prompt) + step, cache)
    dec = build_decoder(ctx, om, fmt.Q8_0, len(prompt) + n, max_batch=4)
    got, _, _ = dec.generate(prompt, hale.SamplingParams(0.8, 0.9, 20, 1.0), 7, n)
    assert got == want
    ctx.check()
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


def _oracle_logits(name, tokens, expert_dtype=fmt.Q8_0):
    return OM.OracleModel(os.path.join(GOLDEN, name), expert_dtype=expert_dtype).teacher_forced_logits(tokens)


def _bits_equal(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return a.shape == b.shape and bool((a.view(np.uint32) == b.view(np.uint32)).all())


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
@pytest.mark.parametrize("chunk", [1, 5, 0])
def test_batched_prefill_matches_token_by_token(ctx, name, chunk):
    """A prompt in one step (chunk 0) or in chunks of consecutive positions:
    every row's logits equal Transformer::forward token by token (the
    oracle), then single-token decode continues on the same cache."""
    with open(os.path.join(GOLDEN, name, "expected.json")) as f:
        tokens = json.load(f)["tokens"]
    om = OM.OracleModel(os.path.join(GOLDEN, name), expert_dtype=fmt.Q8_0)
    want = om.teacher_forced_logits(tokens)
    n_pre = len(tokens) - 3
    dec = build_decoder(ctx, om, fmt.Q8_0, len(tokens), max_batch=n_pre)
    V = om.cfg["vocab"]
    logits = torch.empty((n_pre, V), dtype=torch.float32, device="cuda")
    step = chunk or n_pre
    for s0 in range(0, n_pre, step):
        s1 = min(n_pre, s0 + step)
        dec.step(tokens[s0:s1], list(range(s0, s1)), logits=logits[s0:s1])
    got = logits.cpu().numpy()
    one = torch.empty(V, dtype=torch.float32, device="cuda")
    tail = []
    for i in range(n_pre, len(tokens)):
        dec.forward(tokens[i], i, one)
        tail.append(one.cpu().numpy().copy())
    ctx.check()
    assert _bits_equal(got, want[:n_pre])
    assert _bits_equal(np.stack(tail), want[n_pre:])
    dec.close()


@pytest.mark.parametrize("name", ["tiny-qwen3-moe", "tiny-mixtral"])
def test_batched_decode_over_sequences(ctx, name):
    """Three sequences with their own caches, one row each per step (plus a
    step that mixes a prefill chunk of one with decode rows of the others):
    each sequence's logits equal the oracle's for that sequence alone."""
    with open(os.path.join(GOLDEN, name, "expected.json")) as f:
        base = json.load(f)["tokens"]
    om = OM.OracleModel(os.path.join(GOLDEN, name), expert_dtype=fmt.Q4_0)
    V = om.cfg["vocab"]
    seqs = [base, base[3:] + base[:3], [(t * 7 + 5) % V for t in base]]
    n = len(base)
    want = [om.teacher_forced_logits(s) for s in seqs]
    dec = build_decoder(ctx, om, fmt.Q4_0, n, n_seqs=3, max_batch=8)
    got = [np.zeros((n, V), np.float32) for _ in seqs]
    # step 0: sequence 2 prefills positions 0..3 while 0 and 1 decode position 0
    rows = [(2, 0), (2, 1), (0, 0), (2, 2), (1, 0), (2, 3)]
    logits = torch.empty((8, V), dtype=torch.float32, device="cuda")
    dec.step([seqs[s][p] for s, p in rows], [p for _, p in rows], [s for s, _ in rows], logits=logits[:len(rows)])
    out = logits.cpu().numpy()
    for r, (s, p) in enumerate(rows):
        got[s][p] = out[r]
    pos = [1, 1, 4]
    while min(pos) < n:
        rows = [(s, pos[s]) for s in range(3) if pos[s] < n]
        dec.step([seqs[s][p] for s, p in rows], [p for _, p in rows], [s for s, _ in rows], logits=logits[:len(rows)])
        out = logits.cpu().numpy()
        for r, (s, p) in enumerate(rows):
            got[s][p] = out[r]
            pos[s] += 1
    ctx.check()
    for s in range(3):
        assert _bits_equal(got[s], want[s]), f"sequence {s}"
    dec.close()


def test_step_last_logits_hidden_and_errors(ctx):
    name = "tiny-qwen3-moe"
    with open(os.path.join(GOLDEN, name, "expected.json")) as f:
        tokens = json.load(f)["tokens"][:6]
    om = OM.OracleModel(os.path.join(GOLDEN, name), expert_dtype=fmt.Q8_0)
    want = om.teacher_forced_logits(tokens)
    dec = build_decoder(ctx, om, fmt.Q8_0, 8, n_seqs=2, max_batch=6)
    V, H = om.cfg["vocab"], om.cfg["hidden"]
    last = torch.empty((1, V), dtype=torch.float32, device="cuda")
    hidden = torch.empty((6, H), dtype=torch.float32, device="cuda")
    dec.step(tokens, list(range(6)), logits=last, last_logits_only=True, hidden=hidden)
    assert _bits_equal(last.cpu().numpy()[0], want[5])
    assert torch.isfinite(hidden).all()
    for bad, status in [(dict(tokens=[1, 2], positions=[3, 3]), hale.E_INVALID_ARGUMENT),
                        (dict(tokens=[1], positions=[0], seqs=[2]), hale.E_INVALID_ARGUMENT),
                        (dict(tokens=[1] * 7, positions=list(range(7))), hale.E_INVALID_ARGUMENT),
                        (dict(tokens=[V], positions=[0]), hale.E_INVALID_ARGUMENT),
                        (dict(tokens=[1], positions=[8]), hale.E_CONTEXT_OVERFLOW)]:
        with pytest.raises(hale.HaleError) as ei:
            dec.step(**bad)
        assert ei.value.status == status
    dec.step([1, 2], [3, 3], seqs=[0, 1])   # same position in two sequences is fine
    ctx.check()
    dec.close()


def test_batched_prefill_through_a_tiered_pool(ctx, tmp_path):
    """Batched rows resolve the tiers one token at a time: same logits."""
    loader = importlib.import_module("hale-token_b200.loader")
    pk = importlib.import_module("hale-token_b200.pack")
    name = "tiny-mixtral"
    with open(os.path.join(GOLDEN, name, "expected.json")) as f:
        tokens = json.load(f)["tokens"]
    dst = str(tmp_path / "c")
    pk.convert_checkpoint(os.path.join(GOLDEN, name), dst, fmt.Q8_0)
    want = _oracle_logits(name, tokens)
    rb = loader.ModelWeights(dst).record_bytes
    dec, pool, cfg = loader.load_decoder(ctx, dst, max_len=len(tokens), policy=hale.CachePolicy([], 2 * rb),
                                         max_batch=len(tokens))
    logits = torch.empty((len(tokens), cfg.vocab_size), dtype=torch.float32, device="cuda")
    dec.step(tokens, list(range(len(tokens))), logits=logits)
    ctx.check()
    assert _bits_equal(logits.cpu().numpy(), want)
    assert pool.stats().misses > 0
    dec.close()


def _decode_and_compare(ctx, om, expert_dtype, prompt, n_new):
    """Greedy decode on the GPU (argmax of its own logits, first index of
    the max as activation.rs:24-32) and on the oracle (generate() with
    greedy sampling, generator.rs:55-94): the generated ids must be equal,
    and the logits of every position (prompt and generated) bit-identical
    to the oracle's teacher-forced logits over the same ids."""
    want_ids = om.greedy(prompt, n_new)
    tokens = list(prompt) + list(want_ids)
    want = om.teacher_forced_logits(tokens)
    dec = build_decoder(ctx, om, expert_dtype, len(tokens) + 1)
    logits = torch.empty(om.cfg["vocab"], dtype=torch.float32, device="cuda")
    got, gen = [], []
    for i, t in enumerate(prompt):
        dec.forward(t, i, logits)
        got.append(logits.cpu().numpy().copy())
    pos = len(prompt)
    for step in range(n_new):
        tok = int(torch.argmax(logits).item())
        gen.append(tok)
        if step + 1 == n_new:
            break
        dec.forward(tok, pos, logits)
        got.append(logits.cpu().numpy().copy())
        pos += 1
    # the last generated id's own logits (position len(tokens) - 1)
    dec.forward(gen[-1], pos, logits)
    got.append(logits.cpu().numpy().copy())
    ctx.check()
    dec.close()
    assert gen == list(want_ids), "greedy ids differ"
    got = np.stack(got)
    diff = got.view(np.uint32) != want.view(np.uint32)
    assert not diff.any(), f"{diff.sum()} of {diff.size} logits differ; first at {np.argwhere(diff)[0]}"


def test_config0_tiny_qwen3_moe_exactly_as_specified(ctx):
    """4 decoder layers, hidden 256, 8 query / 2 KV heads
    of 32, RoPE theta 1e6, RMSNorm eps 1e-6, 16 experts top-4 of
    intermediate 128 with normalised top-k weights, vocab 1024, q8_0
    experts, f32 dense weights, N(0, 0.02) from a seed (norm weights 1.0).
    A 32-token uniform random prompt, then 64 greedy tokens; logits compared
    at all 96 positions."""
    hf, t, enc = synth.qwen3_moe(0, 4, 256, 8, 2, 32, 16, 4, 128, 1024, fmt.Q8_0, "F32")
    om = OM.OracleModel(expert_dtype=fmt.Q8_0, hf_config=hf, tensors=t, expert_encoded=enc)
    prompt = np.random.default_rng(1).integers(0, 1024, 32).tolist()
    _decode_and_compare(ctx, om, fmt.Q8_0, prompt, 64)


def test_config2_shapes_qwen3_30b_a3b_reduced_layers(ctx):
    """BASELINE config 2's shapes (Qwen3-30B-A3B: hidden 2048, 32 query / 4
    KV heads of 128, 128 experts top-8 of intermediate 768 in q4_0, vocab
    151936, bf16 dense weights) at 2 decoder layers: a 4-token prompt and 4
    greedy tokens, every position's logits bit-identical to the oracle."""
    hf, t, enc = synth.qwen3_moe(2, 2, 2048, 32, 4, 128, 128, 8, 768, 151936, fmt.Q4_0, "BF16")
    om = OM.OracleModel(expert_dtype=fmt.Q4_0, hf_config=hf, tensors=t, expert_encoded=enc)
    prompt = np.random.default_rng(3).integers(0, 151936, 4).tolist()
    _decode_and_compare(ctx, om, fmt.Q4_0, prompt, 4)


@pytest.mark.parametrize("head_dim", [384, 512])
def test_wide_heads_take_the_decode_attention_kernel(ctx, head_dim):
    """head_dim above 256 runs attn_decode_kernel (V rows staged three stages
    deep): 20 positions, past several V stages, bit-identical logits."""
    hf, t, enc = synth.qwen3_moe(4, 1, 256, 2, 1, head_dim, 4, 2, 64, 256, fmt.Q8_0, "F32")
    om = OM.OracleModel(expert_dtype=fmt.Q8_0, hf_config=hf, tensors=t, expert_encoded=enc)
    prompt = np.random.default_rng(5).integers(0, 256, 12).tolist()
    _decode_and_compare(ctx, om, fmt.Q8_0, prompt, 8)


def test_expert_parallel_decoder_on_one_rank(ctx):
    """hale_decoder_set_comm with a one-rank communicator: the MoE layers run
    through hale_moe_forward_ep and every position's logits equal the
    oracle's (batched prefill rows, then single rows, eagerly)."""
    hf, t, enc = synth.qwen3_moe(6, 2, 256, 8, 2, 32, 16, 4, 128, 512, fmt.Q8_0, "F32")
    om = OM.OracleModel(expert_dtype=fmt.Q8_0, hf_config=hf, tensors=t, expert_encoded=enc)
    tokens = np.random.default_rng(8).integers(0, 512, 10).tolist()
    want = om.teacher_forced_logits(tokens)
    dec = build_decoder(ctx, om, fmt.Q8_0, len(tokens), max_batch=4)
    comm = hale.Comm(ctx, 1, 0, None, 256, 16, 4, 4)
    try:
        dec.set_comm(comm)
        logits = torch.empty((4, om.cfg["vocab"]), dtype=torch.float32, device="cuda")
        got = []
        dec.step(tokens[:4], list(range(4)), logits=logits)
        got.append(logits.cpu().numpy().copy())
        one = torch.empty(om.cfg["vocab"], dtype=torch.float32, device="cuda")
        for i in range(4, len(tokens)):
            dec.forward(tokens[i], i, one)
            got.append(one.cpu().numpy()[None].copy())
        ctx.check()
        assert _bits_equal(np.concatenate(got), want)
        with pytest.raises(hale.HaleError) as ei:     # a communicator of the wrong shape
            small = hale.Comm(ctx, 1, 0, None, 256, 16, 4, 2)
            try:
                dec.set_comm(small)
            finally:
                small.close()
        assert ei.value.status == hale.E_INVALID_ARGUMENT
    finally:
        dec.set_comm(None)
        comm.close()
        dec.close()
