"""The Hale expert pack (experts.hpk) and the checkpoint converter.

File layout (src/expert/pack.rs:1-16, 55-123): "HALEPACK", u64 LE length of
a JSON PackHeader, the header, zero padding up to data_offset (a multiple of
16 KiB), then one record per (MoE layer ordinal, expert) at
data_offset + (ordinal * num_experts + expert) * record_stride. A record is
gate | up | down encoded in the pack's dtype (the bytes
hale_pool_upload_expert takes), padded to record_stride.

convert_checkpoint is `hale convert` (src/convert.rs:56-127): every tensor
that is not a routed expert goes to dense.safetensors as stored, every routed
expert to experts.hpk in the requested dtype, config and tokenizer files are
copied.
"""
import importlib
import json
import os
import shutil
import struct
from dataclasses import dataclass, field

import numpy as np

fmt = importlib.import_module("hale-token_b200.formats")
loader = importlib.import_module("hale-token_b200.loader")

PACK_FILE_NAME = "experts.hpk"
DENSE_FILE_NAME = "dense.safetensors"
MAGIC = b"HALEPACK"
FORMAT_VERSION = 1
ALIGN = 16 * 1024
_DTYPE_NAMES = {v: k for k, v in fmt.NAMES.items()}
COPIED_FILES = ("config.json", "tokenizer.json", "tokenizer_config.json", "generation_config.json",
                "special_tokens_map.json")


def _round_up(n, a):
    return -(-n // a) * a


@dataclass
class PackHeader:
    """PackHeader (pack.rs:55-73); serialised with the same field order."""
    version: int
    dtype: int
    hidden_size: int
    intermediate_size: int
    num_experts: int
    moe_layers: list = field(default_factory=list)
    record_bytes: int = 0
    record_stride: int = 0
    data_offset: int = 0

    @staticmethod
    def for_model(config, dtype):
        """PackHeader::for_model (pack.rs:76-99)."""
        h, i = config.hidden_size, config.expert_intermediate_size
        rec = 2 * i * fmt.row_bytes(dtype, h) + h * fmt.row_bytes(dtype, i)
        hd = PackHeader(FORMAT_VERSION, dtype, h, i, config.num_experts,
                        [l for l in range(config.num_layers) if config.is_moe_layer(l)], rec, _round_up(rec, ALIGN), 0)
        hd.data_offset = _round_up(16 + len(hd.to_json()) + 32, ALIGN)
        return hd

    def to_json(self):
        d = {"version": self.version, "dtype": _DTYPE_NAMES[self.dtype], "hidden_size": self.hidden_size,
             "intermediate_size": self.intermediate_size, "num_experts": self.num_experts,
             "moe_layers": list(self.moe_layers), "record_bytes": self.record_bytes,
             "record_stride": self.record_stride, "data_offset": self.data_offset}
        return json.dumps(d, separators=(",", ":")).encode()

    @staticmethod
    def from_json(blob, path="pack"):
        try:
            d = json.loads(blob)
            hd = PackHeader(int(d["version"]), fmt.NAMES[d["dtype"]], int(d["hidden_size"]),
                            int(d["intermediate_size"]), int(d["num_experts"]), [int(x) for x in d["moe_layers"]],
                            int(d["record_bytes"]), int(d["record_stride"]), int(d["data_offset"]))
        except (ValueError, KeyError, TypeError, UnicodeDecodeError) as e:
            raise loader.LoadError(f"{path}: bad pack header: {e}") from None
        return hd

    def file_size(self):
        return self.data_offset + len(self.moe_layers) * self.num_experts * self.record_stride

    def ordinal(self, layer):
        """Position of model layer `layer` among the pack's MoE layers."""
        try:
            return self.moe_layers.index(layer)
        except ValueError:
            raise loader.LoadError(f"layer {layer} has no experts in the pack") from None

    def offset_of(self, layer, expert):
        """PackHeader::offset_of (pack.rs:106-123); `layer` is a model layer."""
        j = self.ordinal(layer)
        if not 0 <= expert < self.num_experts:
            raise loader.LoadError(f"expert L{layer}E{expert} out of range")
        return self.data_offset + (j * self.num_experts + expert) * self.record_stride


class PackWriter:
    """PackWriter (pack.rs:141-200): records go to fixed offsets, in any order."""

    def __init__(self, path, header):
        self.path, self.header = path, header
        js = header.to_json()
        self.f = open(path, "wb")
        self.f.write(MAGIC + struct.pack("<Q", len(js)) + js)
        self.f.truncate(header.file_size())

    def write_record(self, layer, expert, record):
        rec = np.ascontiguousarray(record, dtype=np.uint8).reshape(-1)
        if rec.size != self.header.record_bytes:
            raise loader.LoadError(f"L{layer}E{expert}: record is {rec.size} bytes, expected {self.header.record_bytes}")
        self.f.seek(self.header.offset_of(layer, expert))
        self.f.write(rec.tobytes())

    def finish(self):
        self.f.flush()
        os.fsync(self.f.fileno())
        self.f.close()


class PackSource:
    """PackExpertSource (pack.rs:202-271): the pack memory-mapped read-only,
    its header validated (magic, header size, version, file length)."""

    def __init__(self, path):
        self.path = path
        try:
            with open(path, "rb") as f:
                prefix = f.read(16)
                if len(prefix) < 16 or prefix[:8] != MAGIC:
                    raise loader.LoadError(f"{path} is not a Hale expert pack")
                (n,) = struct.unpack("<Q", prefix[8:])
                if n > ALIGN * 64:
                    raise loader.LoadError(f"{path}: header too large")
                blob = f.read(n)
            if len(blob) != n:
                raise loader.LoadError(f"{path}: truncated header")
            hd = PackHeader.from_json(blob, path)
            if hd.version != FORMAT_VERSION:
                raise loader.LoadError(f"{path}: pack version {hd.version} is not supported "
                                       f"(expected {FORMAT_VERSION})")
            size = os.path.getsize(path)
            if size < hd.file_size():
                raise loader.LoadError(f"{path}: truncated pack ({size} bytes, expected {hd.file_size()})")
            if hd.dtype not in (fmt.F32, fmt.F16, fmt.BF16, fmt.Q8_0, fmt.Q4_0):
                raise loader.LoadError(f"{path}: unknown dtype")
            self.map = np.memmap(path, dtype=np.uint8, mode="r")
        except OSError as e:
            raise loader.LoadError(f"{path}: {e}") from None
        self.header = hd

    @property
    def expert_bytes(self):
        return self.header.record_bytes

    def record(self, layer, expert):
        """One expert's record (gate | up | down) for model layer `layer`."""
        o = self.header.offset_of(layer, expert)
        return self.map[o:o + self.header.record_bytes]

    def record_by_ordinal(self, j, expert):
        return self.record(self.header.moe_layers[j], expert)

    def split(self, record):
        """decode_record (pack.rs:125-133) -> (gate, up, down) encoded rows."""
        h = self.header
        return fmt.split_record(record, h.dtype, h.hidden_size, h.intermediate_size)


def convert_checkpoint(src, dst, expert_dtype=fmt.Q4_0):
    """`hale convert` (convert.rs:56-127). Returns a report dict."""
    if os.path.abspath(src) == os.path.abspath(dst):
        raise loader.LoadError("output directory must differ from the input")
    cfg = loader.ModelConfig.from_dir(src)
    os.makedirs(dst, exist_ok=True)
    ck = loader.Checkpoint.open_dir(src)
    names = loader.Naming(cfg.architecture)
    expert_names = {names.expert(l, e, p) for l in range(cfg.num_layers) if cfg.is_moe_layer(l)
                    for e in range(cfg.num_experts) for p in ("gate", "up", "down")}
    dense = []
    for n in ck.names():
        if n in expert_names:
            continue
        dt, shape, raw = ck.raw(n)
        if dt not in ("F32", "F16", "BF16"):
            continue  # integer buffers some exporters include
        dense.append((n, shape, dt, np.asarray(raw)))
    loader.write_safetensors(os.path.join(dst, DENSE_FILE_NAME), dense)
    hd = PackHeader.for_model(cfg, expert_dtype)
    w = PackWriter(os.path.join(dst, PACK_FILE_NAME), hd)
    for l in hd.moe_layers:
        for e in range(cfg.num_experts):
            enc = [fmt.encode(expert_dtype, ck.f32(names.expert(l, e, p))) for p in ("gate", "up", "down")]
            w.write_record(l, e, fmt.pack_record(*enc))
    w.finish()
    for f in COPIED_FILES:
        if os.path.exists(os.path.join(src, f)):
            shutil.copyfile(os.path.join(src, f), os.path.join(dst, f))
    return {"dense_tensors": len(dense), "dense_bytes": sum(t[3].nbytes for t in dense),
            "experts": len(hd.moe_layers) * cfg.num_experts, "pack_bytes": hd.file_size()}
