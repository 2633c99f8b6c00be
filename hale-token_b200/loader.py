"""Hugging Face checkpoints -> a hale_decoder on the GPU.

The reference's load path, restated:
  - ModelConfig::from_hf and validate (src/config.rs:156-240): architecture,
    expert count (num_experts or num_local_experts), expert intermediate size
    (moe_intermediate_size, else intermediate_size), dense layers of Qwen3-MoE
    (mlp_only_layers, or (i + 1) % decoder_sparse_step != 0), normalize_topk
    (always for Mixtral, norm_topk_prob for Qwen3), head_dim default
    hidden / heads, defaults eps 1e-6, rope_theta 1e4, max positions 4096;
  - TensorNaming (src/model/arch.rs:30-118): Qwen3-MoE mlp.experts.N.*_proj,
    Mixtral block_sparse_moe.experts.N.w1/w3/w2;
  - SafetensorsCheckpoint (src/loader/safetensors.rs:60-235): the shards
    listed by model.safetensors.index.json, else every *.safetensors file in
    the directory (sorted); each header validated (length within the file,
    offsets ordered and inside the file); tensors memory-mapped;
  - routed experts converted to the pack formats (q8_0 / q4_0) like
    `hale convert` (src/convert.rs:56-127: rows decoded to f32, re-encoded)
    and uploaded into an HBM expert pool.
"""
import importlib
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

hale = importlib.import_module("hale-token_b200")
fmt = importlib.import_module("hale-token_b200.formats")

QWEN3_MOE, MIXTRAL = "Qwen3MoeForCausalLM", "MixtralForCausalLM"
_DTYPE = {"F32": fmt.F32, "F16": fmt.F16, "BF16": fmt.BF16}


class LoadError(ValueError):
    """A checkpoint or config the engine cannot run (the reference's
    HaleError::InvalidArgument / Safetensors / BadTensor)."""


class MissingTensor(LoadError):
    """A tensor name the checkpoint does not hold (HaleError::MissingTensor)."""


@dataclass
class ModelConfig:
    architecture: str
    hidden_size: int
    expert_intermediate_size: int
    dense_intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    vocab_size: int
    rms_norm_eps: float
    rope_theta: float
    max_position_embeddings: int
    num_experts: int
    experts_per_token: int
    normalize_topk: bool
    tie_word_embeddings: bool
    dense_layers: list = field(default_factory=list)
    bos_token_id: int = None
    eos_token_ids: list = field(default_factory=list)

    @staticmethod
    def from_json_str(text):
        try:
            hf = json.loads(text)
        except json.JSONDecodeError as e:
            raise LoadError(f"config.json: {e}") from None
        return ModelConfig.from_hf(hf)

    @staticmethod
    def from_dir(directory):
        path = os.path.join(directory, "config.json")
        try:
            with open(path) as f:
                text = f.read()
        except OSError as e:
            raise LoadError(f"{path}: {e}") from None
        try:
            return ModelConfig.from_json_str(text)
        except LoadError as e:
            raise LoadError(f"{path}: {e}") from None

    @staticmethod
    def from_hf(hf):
        archs = hf.get("architectures") or []
        if not archs:
            raise LoadError("config.json has no architectures")
        arch = archs[0]
        if arch not in (QWEN3_MOE, MIXTRAL):
            raise LoadError(f"unsupported model architecture `{arch}`")
        for key in ("hidden_size", "num_hidden_layers", "num_attention_heads", "vocab_size", "num_experts_per_tok"):
            if key not in hf:
                raise LoadError(f"config.json: missing field `{key}`")
        n_exp = hf.get("num_experts")
        if n_exp is None:
            n_exp = hf.get("num_local_experts")
        if n_exp is None:
            raise LoadError("config.json has no expert count")
        dense_inter = hf.get("intermediate_size") or 0
        expert_inter = hf.get("moe_intermediate_size") or dense_inter
        layers = hf["num_hidden_layers"]
        if arch == MIXTRAL:
            dense = []
            normalize = True
        else:
            step = max(hf.get("decoder_sparse_step") or 1, 1)
            mlp_only = hf.get("mlp_only_layers") or []
            dense = [i for i in range(layers) if i in mlp_only or (i + 1) % step != 0]
            normalize = bool(hf.get("norm_topk_prob") or False)
        eos = hf.get("eos_token_id")
        eos = [] if eos is None else (list(eos) if isinstance(eos, list) else [eos])
        heads = hf["num_attention_heads"]
        c = ModelConfig(
            architecture=arch, hidden_size=hf["hidden_size"], expert_intermediate_size=expert_inter,
            dense_intermediate_size=dense_inter, num_layers=layers, num_heads=heads,
            num_kv_heads=hf.get("num_key_value_heads") or heads,
            head_dim=hf.get("head_dim") or hf["hidden_size"] // heads, vocab_size=hf["vocab_size"],
            rms_norm_eps=float(hf.get("rms_norm_eps", 1e-6)), rope_theta=float(hf.get("rope_theta", 10000.0)),
            max_position_embeddings=hf.get("max_position_embeddings", 4096), num_experts=n_exp,
            experts_per_token=hf["num_experts_per_tok"], normalize_topk=normalize,
            tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)), dense_layers=dense,
            bos_token_id=hf.get("bos_token_id"), eos_token_ids=eos)
        c.validate()
        return c

    def validate(self):
        if self.num_kv_heads == 0 or self.num_heads % self.num_kv_heads != 0:
            raise LoadError(f"num_attention_heads ({self.num_heads}) must be a multiple of "
                            f"num_key_value_heads ({self.num_kv_heads})")
        if self.head_dim % 2 != 0:
            raise LoadError(f"head_dim ({self.head_dim}) must be even for RoPE")
        if self.experts_per_token == 0 or self.experts_per_token > self.num_experts:
            raise LoadError(f"num_experts_per_tok ({self.experts_per_token}) must be in 1..={self.num_experts}")

    def is_moe_layer(self, layer):
        return layer not in self.dense_layers

    def num_moe_layers(self):
        return self.num_layers - len(self.dense_layers)

    def params_per_expert(self):
        return 3 * self.hidden_size * self.expert_intermediate_size

    def dense_params(self):
        h, q, kv = self.hidden_size, self.num_heads * self.head_dim, self.num_kv_heads * self.head_dim
        attention = h * q + 2 * h * kv + q * h
        norms = 2 * h + (2 * self.head_dim if self.architecture == QWEN3_MOE else 0)
        routers = self.num_moe_layers() * self.num_experts * h
        dense_mlps = len(self.dense_layers) * 3 * h * self.dense_intermediate_size
        embeddings = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
        return self.num_layers * (attention + norms) + routers + dense_mlps + embeddings + h

    def total_params(self):
        return self.dense_params() + self.num_moe_layers() * self.num_experts * self.params_per_expert()

    def active_params(self):
        return self.dense_params() + self.num_moe_layers() * self.experts_per_token * self.params_per_expert()


class Naming:
    """Tensor names of an architecture (arch.rs:30-118)."""

    def __init__(self, architecture):
        self.qwen = architecture == QWEN3_MOE

    def expert(self, layer, e, proj):
        if self.qwen:
            return f"model.layers.{layer}.mlp.experts.{e}.{proj}_proj.weight"
        return f"model.layers.{layer}.block_sparse_moe.experts.{e}.{ {'gate': 'w1', 'down': 'w2', 'up': 'w3'}[proj]}.weight"

    def router(self, layer):
        if self.qwen:
            return f"model.layers.{layer}.mlp.gate.weight"
        return f"model.layers.{layer}.block_sparse_moe.gate.weight"

    def dense_mlp(self, layer, proj):
        return f"model.layers.{layer}.mlp.{proj}_proj.weight"

    embeddings = "model.embed_tokens.weight"
    final_norm = "model.norm.weight"
    lm_head = "lm_head.weight"

    @staticmethod
    def input_norm(layer):
        return f"model.layers.{layer}.input_layernorm.weight"

    @staticmethod
    def post_attention_norm(layer):
        return f"model.layers.{layer}.post_attention_layernorm.weight"

    @staticmethod
    def attention(layer, part):
        return f"model.layers.{layer}.self_attn.{part}.weight"


class Checkpoint:
    """Memory-mapped safetensors shards viewed as one checkpoint."""

    def __init__(self, files):
        self.index = {}
        self.maps = []
        for shard, path in enumerate(files):
            try:
                m = np.memmap(path, dtype=np.uint8, mode="r")
            except (OSError, ValueError) as e:
                raise LoadError(f"{path}: {e}") from None
            for name, info, start in _parse_header(path, m):
                self.index[name] = (shard, info, start)
            self.maps.append(m)

    @staticmethod
    def open_dir(directory):
        idx = os.path.join(directory, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                try:
                    wm = json.load(f)["weight_map"]
                except (json.JSONDecodeError, KeyError) as e:
                    raise LoadError(f"{idx}: {e}") from None
            return Checkpoint(sorted({os.path.join(directory, v) for v in wm.values()}))
        try:
            files = sorted(os.path.join(directory, f) for f in os.listdir(directory) if f.endswith(".safetensors"))
        except OSError as e:
            raise LoadError(f"{directory}: {e}") from None
        if not files:
            raise LoadError(f"no .safetensors files in {directory}")
        return Checkpoint(files)

    def names(self):
        return sorted(self.index)

    def contains(self, name):
        return name in self.index

    def raw(self, name):
        """(dtype string, shape, uint8 view) of a tensor."""
        if name not in self.index:
            raise MissingTensor(f"missing tensor `{name}`")
        shard, info, start = self.index[name]
        b, e = info["data_offsets"]
        return info["dtype"], tuple(info["shape"]), self.maps[shard][start:start + (e - b)]

    def matrix(self, name):
        """TensorSource::matrix: (hale dtype, rows, cols, encoded rows)."""
        dt, shape, raw = self.raw(name)
        if dt not in _DTYPE:
            raise LoadError(f"tensor `{name}`: unsupported dtype {dt}")
        if len(shape) != 2:
            raise LoadError(f"tensor `{name}`: expected 2-D, got shape {list(shape)}")
        if raw.size != shape[0] * shape[1] * (4 if dt == "F32" else 2):
            raise LoadError(f"tensor `{name}`: byte length does not match shape")
        return _DTYPE[dt], shape[0], shape[1], np.asarray(raw)

    def vector(self, name):
        """TensorSource::vector: decoded to f32."""
        dt, shape, raw = self.raw(name)
        if dt not in _DTYPE:
            raise LoadError(f"tensor `{name}`: unsupported dtype {dt}")
        if len(shape) != 1:
            raise LoadError(f"tensor `{name}`: expected 1-D, got shape {list(shape)}")
        return _as_f32(dt, raw, shape[0])

    def f32(self, name):
        dt, shape, raw = self.raw(name)
        return _as_f32(dt, raw, int(np.prod(shape))).reshape(shape)


def _as_f32(dt, raw, n):
    raw = np.asarray(raw)
    if raw.size != n * (4 if dt == "F32" else 2):
        raise LoadError("byte length does not match shape")
    if dt == "F32":
        return raw.view(np.float32).astype(np.float32, copy=True)
    h = raw.view(np.uint16)
    if dt == "BF16":
        return (h.astype(np.uint32) << 16).view(np.float32)
    return h.view(np.float16).astype(np.float32)


def _parse_header(path, m):
    if m.size < 8:
        raise LoadError(f"{path}: file shorter than the 8-byte header length")
    (hlen,) = struct.unpack("<Q", bytes(m[:8]))
    start = 8 + hlen
    if start > m.size:
        raise LoadError(f"{path}: header length exceeds file size")
    try:
        header = json.loads(bytes(m[8:start]))
    except (json.JSONDecodeError, UnicodeDecodeError) as e:
        raise LoadError(f"{path}: {e}") from None
    out = []
    for name, info in header.items():
        if name == "__metadata__":
            continue
        try:
            b, e = info["data_offsets"]
            info["dtype"], info["shape"]
        except (KeyError, TypeError, ValueError):
            raise LoadError(f"{path}: tensor `{name}` has a malformed header entry") from None
        if b > e or start + e > m.size:
            raise LoadError(f"{path}: tensor `{name}` points outside the file")
        out.append((name, info, start + b))
    return out


def write_safetensors(path, tensors):
    """write_safetensors (safetensors.rs:236-275): entries (name, shape,
    dtype string, raw little-endian bytes) in the order given, header keys
    sorted, header padded with spaces to a multiple of 8 bytes."""
    header, offset = {}, 0
    for name, shape, dt, data in tensors:
        if dt not in _DTYPE:
            raise LoadError(f"{name}: {dt} cannot be stored in safetensors")
        n = len(memoryview(data).cast("B"))
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [offset, offset + n]}
        offset += n
    blob = json.dumps(dict(sorted(header.items())), separators=(",", ":")).encode()
    blob += b" " * (-len(blob) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for _, _, _, data in tensors:
            f.write(memoryview(data).cast("B"))


class ModelWeights:
    """A model directory's tensors arranged for hale_decoder (the reference's
    Transformer::load, transformer.rs:58-150, and Engine::load's expert
    source choice, engine.rs:78-86): per-layer norms as f32; projections,
    routers, dense MLPs, embedding and head as stored (dtype, rows, cols,
    bytes); routed experts as pack records (MoE layer j = j-th MoE layer),
    read from experts.hpk when the directory holds one (a converted model),
    else re-encoded from the checkpoint's tensors to expert_dtype.

    expert_dtype: the pool's format (q8_0 / q4_0). Default: the pack's dtype,
    or q8_0 for a plain checkpoint. A pack in another dtype is re-encoded
    from its decoded values (matrix.rs:103-109)."""

    def __init__(self, directory, expert_dtype=None):
        pack = importlib.import_module("hale-token_b200.pack")
        cfg = self.config = ModelConfig.from_dir(directory)
        ck = self.checkpoint = Checkpoint.open_dir(directory)
        names = self.naming = Naming(cfg.architecture)
        self.moe_layers = [l for l in range(cfg.num_layers) if cfg.is_moe_layer(l)]
        pack_path = os.path.join(directory, pack.PACK_FILE_NAME)
        self.pack = pack.PackSource(pack_path) if os.path.exists(pack_path) else None
        if self.pack is not None:
            hd = self.pack.header
            got = (hd.hidden_size, hd.intermediate_size, hd.num_experts, hd.moe_layers)
            want = (cfg.hidden_size, cfg.expert_intermediate_size, cfg.num_experts, self.moe_layers)
            if got != want:
                raise LoadError(f"{pack_path}: pack shape {got} does not match config.json {want}")
            self.expert_dtype = hd.dtype if expert_dtype is None else expert_dtype
        else:
            self.expert_dtype = fmt.Q8_0 if expert_dtype is None else expert_dtype
        if self.expert_dtype not in (fmt.Q8_0, fmt.Q4_0):
            raise LoadError("the expert pool stores q8_0 or q4_0 experts; pass expert_dtype to convert")
        self.layers = []
        for l in range(cfg.num_layers):
            L = dict(input_norm=ck.vector(names.input_norm(l)), post_norm=ck.vector(names.post_attention_norm(l)),
                     q=ck.matrix(names.attention(l, "q_proj")), k=ck.matrix(names.attention(l, "k_proj")),
                     v=ck.matrix(names.attention(l, "v_proj")), o=ck.matrix(names.attention(l, "o_proj")))
            if cfg.architecture == QWEN3_MOE:
                L["q_norm"] = ck.vector(names.attention(l, "q_norm"))
                L["k_norm"] = ck.vector(names.attention(l, "k_norm"))
            if cfg.is_moe_layer(l):
                L["router"] = ck.matrix(names.router(l))
                if self.pack is None:
                    for e in range(cfg.num_experts):
                        for p in ("gate", "up", "down"):
                            if not ck.contains(names.expert(l, e, p)):
                                raise MissingTensor(f"missing tensor `{names.expert(l, e, p)}`")
            else:
                for p in ("gate", "up", "down"):
                    L[f"dense_{p}"] = ck.matrix(names.dense_mlp(l, p))
            self.layers.append(L)
        self.embed = ck.matrix(names.embeddings)
        tied = cfg.tie_word_embeddings or not ck.contains(names.lm_head)
        self.lm_head = self.embed if tied else ck.matrix(names.lm_head)
        self.final_norm = ck.vector(names.final_norm)
        self.dims = dict(hidden=cfg.hidden_size, n_layers=cfg.num_layers, n_heads=cfg.num_heads,
                         n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, vocab=cfg.vocab_size,
                         n_experts=cfg.num_experts, top_k=cfg.experts_per_token,
                         normalize_topk=cfg.normalize_topk, eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta)

    @property
    def record_bytes(self):
        c, d = self.config, self.expert_dtype
        return 2 * c.expert_intermediate_size * fmt.row_bytes(d, c.hidden_size) + \
            c.hidden_size * fmt.row_bytes(d, c.expert_intermediate_size)

    def _values(self, l, e):
        """gate, up, down of expert e of model layer l as f32."""
        if self.pack is None:
            return [self.checkpoint.f32(self.naming.expert(l, e, p)) for p in ("gate", "up", "down")]
        hd = self.pack.header
        parts = self.pack.split(self.pack.record(l, e))
        shapes = [(hd.intermediate_size, hd.hidden_size)] * 2 + [(hd.hidden_size, hd.intermediate_size)]
        return [fmt.decode(hd.dtype, m, sh[1]).reshape(sh) for m, sh in zip(parts, shapes)]

    def expert_record(self, j, e):
        """Expert e of MoE layer j as one pack record gate | up | down."""
        l = self.moe_layers[j]
        if self.pack is not None and self.pack.header.dtype == self.expert_dtype:
            return np.asarray(self.pack.record(l, e))
        enc = [fmt.encode(self.expert_dtype, v) for v in self._values(l, e)]
        for m, p in zip(enc, ("gate", "up", "down")):
            want = (self.config.expert_intermediate_size, self.config.hidden_size) if p != "down" else \
                (self.config.hidden_size, self.config.expert_intermediate_size)
            if m.shape[0] != want[0] or m.shape[1] != fmt.row_bytes(self.expert_dtype, want[1]):
                raise LoadError(f"tensor `{self.naming.expert(l, e, p)}`: expected shape {list(want)}")
        return fmt.pack_record(*enc)


class RoutingStats:
    """RoutingStats (src/expert/stats.rs:15-130): selection counts per (model
    layer, expert), flat at layer * num_experts + expert, saved as the
    reference's JSON ({"num_layers", "num_experts", "counts"}) so a run's
    routing warms the next start's pinned tier."""

    def __init__(self, num_layers, num_experts, counts=None):
        self.num_layers, self.num_experts = int(num_layers), int(num_experts)
        n = self.num_layers * self.num_experts
        self.counts = np.zeros(n, np.uint64) if counts is None else np.asarray(counts, np.uint64).reshape(-1).copy()
        if self.counts.size != n:
            raise LoadError("counter length does not match its shape")

    @staticmethod
    def from_pool(pool, config):
        """The counts a pool recorded (pool layer j = j-th MoE layer) placed
        at their model layers."""
        st = RoutingStats(config.num_layers, config.num_experts)
        c = np.asarray(pool.routing_counts(), np.uint64)
        for j, l in enumerate(l for l in range(config.num_layers) if config.is_moe_layer(l)):
            st.counts[l * st.num_experts:(l + 1) * st.num_experts] = c[j]
        return st

    def pool_counts(self, config):
        """[MoE layers, experts] counts in pool-layer order (for cache_policy)."""
        rows = [self.counts[l * self.num_experts:(l + 1) * self.num_experts]
                for l in range(config.num_layers) if config.is_moe_layer(l)]
        return np.stack(rows) if rows else np.zeros((0, self.num_experts), np.uint64)

    def record(self, layer, expert):
        self.counts[layer * self.num_experts + expert] += 1

    def count(self, layer, expert):
        return int(self.counts[layer * self.num_experts + expert])

    def total(self):
        return int(self.counts.sum())

    def merge(self, other):
        """Adds counters of the same shape (others are ignored, as stats.rs:64-70)."""
        if (other.num_layers, other.num_experts) == (self.num_layers, self.num_experts):
            self.counts += other.counts

    def hottest(self, n):
        return hottest(self.counts.reshape(self.num_layers, self.num_experts), n)

    def coverage(self, n):
        """Fraction of all selections that went to the n hottest experts."""
        t = self.total()
        return 0.0 if t == 0 else sum(self.count(l, e) for l, e in self.hottest(n)) / t

    def save(self, path):
        with open(path, "w") as f:
            json.dump({"num_layers": self.num_layers, "num_experts": self.num_experts,
                       "counts": [int(c) for c in self.counts]}, f, separators=(",", ":"))

    @staticmethod
    def load(path):
        try:
            with open(path) as f:
                d = json.load(f)
            return RoutingStats(d["num_layers"], d["num_experts"], d["counts"])
        except (OSError, json.JSONDecodeError, KeyError, TypeError, ValueError) as e:
            if isinstance(e, LoadError):
                raise
            raise LoadError(f"{path}: {e}") from None

    def __eq__(self, other):
        return isinstance(other, RoutingStats) and (self.num_layers, self.num_experts) == \
            (other.num_layers, other.num_experts) and np.array_equal(self.counts, other.counts)


def split_budget(experts_in_ram, total_experts, per_token_experts):
    """planner::split_budget (src/expert/planner.rs:253-267) -> (pinned, lru)
    expert counts: below twice one token's working set an LRU only thrashes
    on the cyclic layer walk, so every slot is pinned."""
    n = min(experts_in_ram, total_experts)
    if n == total_experts or n < 2 * per_token_experts:
        return n, 0
    return n // 2, n - n // 2


def hottest(counts, n):
    """RoutingStats::hottest (src/expert/stats.rs:77-95): the n most routed
    (layer, expert) keys of a [layers, experts] count array, hotter first,
    ties by index; never-routed keys are left out."""
    flat = np.asarray(counts, dtype=np.uint64).reshape(-1)
    E = np.asarray(counts).shape[-1]
    used = np.flatnonzero(flat)
    order = sorted(used.tolist(), key=lambda i: (-int(flat[i]), i))[:n]
    return [(i // E, i % E) for i in order]


def choose_pinned(counts, n_layers, n_experts, n):
    """choose_pinned (src/engine.rs:266-292): the hottest keys of past runs
    first, then keys expert-major across the layers so every layer gets the
    same share."""
    if n >= n_layers * n_experts:
        return [(l, e) for l in range(n_layers) for e in range(n_experts)]
    chosen = hottest(counts, n) if counts is not None else []
    taken = set(chosen)
    for e in range(n_experts):
        for l in range(n_layers):
            if len(chosen) == n:
                return chosen
            if (l, e) not in taken:
                taken.add((l, e))
                chosen.append((l, e))
    return chosen


def cache_policy(config, record_bytes, budget_bytes, routing_counts=None):
    """cache_policy (src/engine.rs:294-318) for pool layers = MoE ordinals:
    an HBM budget for experts turned into pinned keys plus an LRU budget."""
    hale_mod = hale
    n_moe = config.num_moe_layers()
    total = n_moe * config.num_experts
    per_token = n_moe * config.experts_per_token
    pinned, lru = split_budget(budget_bytes // max(record_bytes, 1), total, per_token)
    keys = choose_pinned(routing_counts, n_moe, config.num_experts, pinned)
    return hale_mod.CachePolicy(keys, lru * record_bytes)


def load_decoder(ctx, directory, expert_dtype=None, max_len=None, policy=None, expert_hbm_bytes=None,
                 routing_counts=None, n_seqs=1, max_batch=1):
    """Builds (decoder, pool, config) from a model directory: a Hugging Face
    checkpoint (config.json + safetensors) or a converted one (config.json,
    dense.safetensors, experts.hpk). Dense weights as stored; experts into an
    HBM-resident pool, or a tiered one when `policy` (a CachePolicy) or
    `expert_hbm_bytes` (planned like the reference's RAM budget, hottest
    experts of `routing_counts` -- a RoutingStats, or [MoE layers, experts]
    counts -- pinned first) is given. max_len: KV-cache
    positions (default the config's max_position_embeddings); n_seqs /
    max_batch: KV caches and rows per Decoder.step."""
    w = ModelWeights(directory, expert_dtype)
    cfg = w.config
    if isinstance(routing_counts, RoutingStats):
        routing_counts = routing_counts.pool_counts(cfg)
    if policy is None and expert_hbm_bytes is not None:
        policy = cache_policy(cfg, w.record_bytes, expert_hbm_bytes, routing_counts)
    pool = None
    if w.moe_layers:
        pool = hale.Pool(ctx, w.expert_dtype, cfg.hidden_size, cfg.expert_intermediate_size, len(w.moe_layers),
                         cfg.num_experts, policy=policy)
        for j in range(len(w.moe_layers)):
            for e in range(cfg.num_experts):
                pool.upload(j, e, w.expert_record(j, e))
    dec = hale.Decoder(ctx, w.dims, w.layers, w.embed, w.lm_head, w.final_norm, pool,
                       max_len or cfg.max_position_embeddings, n_seqs, max_batch)
    return dec, pool, cfg
