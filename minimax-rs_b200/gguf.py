"""GGUF reader, writer and TP / EP shard loader for the MiniMax-M2.7 tensors this library runs.

Host-side counterpart of the reference's weight loading (candle-core's GGUF reader as used by
vendor/candle-transformers/src/quantized_var_builder.rs:52-335, 478-560) and of its tensor-parallel
placement (src/tensor_parallel_model.rs:37-61 `layer_tensor_specs`): it parses a GGUF v2/v3 file
(header, typed metadata, tensor infos, aligned data section), memory-maps tensor bytes, cuts a
rank's shard without dequantising (rows of a quantised matrix, or whole blocks along K), and builds
the library's layer objects from them.

Shapes follow Candle's convention: outermost dimension first (GGUF stores ne[0], the contiguous
one, first).  A quantised tensor's bytes are [rows...][k / block_elems] blocks.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian
GGUF_DEFAULT_ALIGNMENT = 32

# ggml types: (name, elements per block, bytes per block)
GGML_TYPES = {
    0: ("F32", 1, 4),
    1: ("F16", 1, 2),
    8: ("Q8_0", 32, 34),
    12: ("Q4_K", 256, 144),
    13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210),
    30: ("BF16", 1, 2),
}
TYPE_IDS = {v[0]: k for k, v in GGML_TYPES.items()}

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


class GGUFError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    shape: tuple  # Candle order: outermost first
    ggml_type: int
    offset: int   # from the start of the data section

    @property
    def type_name(self) -> str:
        return GGML_TYPES[self.ggml_type][0]

    @property
    def nbytes(self) -> int:
        _, be, bb = GGML_TYPES[self.ggml_type]
        n = int(np.prod(self.shape)) if self.shape else 1
        if n % be or (self.shape and self.shape[-1] % be):
            raise GGUFError(f"{self.name}: rows of {self.shape[-1]} are not whole {self.type_name} blocks")
        return n // be * bb


@dataclass
class GGUFFile:
    path: Path
    version: int
    metadata: dict
    tensors: dict = field(default_factory=dict)
    data_offset: int = 0

    def info(self, name: str) -> TensorInfo:
        if name not in self.tensors:
            raise GGUFError(f"tensor {name!r} not in {self.path}")
        return self.tensors[name]

    def tensor_bytes(self, name: str) -> np.ndarray:
        """uint8 view (memory-mapped) of a tensor's bytes."""
        ti = self.info(name)
        return np.memmap(self.path, dtype=np.uint8, mode="r", offset=self.data_offset + ti.offset,
                         shape=(ti.nbytes,))

    def array(self, name: str) -> np.ndarray:
        """F32 / F16 / BF16 tensors as float32 in Candle shape."""
        ti = self.info(name)
        raw = np.asarray(self.tensor_bytes(name))
        if ti.type_name == "F32":
            a = raw.view(np.float32)
        elif ti.type_name == "F16":
            a = raw.view(np.float16).astype(np.float32)
        elif ti.type_name == "BF16":
            a = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            raise GGUFError(f"{name} is {ti.type_name}, not a float tensor")
        return a.reshape(ti.shape)


def _read_str(f) -> str:
    (n,) = struct.unpack("<Q", f.read(8))
    return f.read(n).decode("utf-8")


def _read_value(f, vt: int):
    if vt in _SCALAR:
        fmt = _SCALAR[vt]
        return struct.unpack(fmt, f.read(struct.calcsize(fmt)))[0]
    if vt == _STR:
        return _read_str(f)
    if vt == _ARR:
        (et,) = struct.unpack("<I", f.read(4))
        (n,) = struct.unpack("<Q", f.read(8))
        return [_read_value(f, et) for _ in range(n)]
    raise GGUFError(f"unknown metadata value type {vt}")


def read(path) -> GGUFFile:
    """Parses header, metadata and tensor infos (tensor bytes stay in the file, memory-mapped)."""
    path = Path(path)
    with open(path, "rb") as f:
        magic, version = struct.unpack("<II", f.read(8))
        if magic != GGUF_MAGIC:
            raise GGUFError(f"{path}: not a GGUF file")
        if version not in (2, 3):
            raise GGUFError(f"{path}: GGUF version {version} is not supported")
        n_tensors, n_kv = struct.unpack("<QQ", f.read(16))
        meta = {}
        for _ in range(n_kv):
            key = _read_str(f)
            (vt,) = struct.unpack("<I", f.read(4))
            meta[key] = _read_value(f, vt)
        infos = {}
        for _ in range(n_tensors):
            name = _read_str(f)
            (nd,) = struct.unpack("<I", f.read(4))
            ne = struct.unpack(f"<{nd}Q", f.read(8 * nd))
            gt, off = struct.unpack("<IQ", f.read(12))
            if gt not in GGML_TYPES:
                raise GGUFError(f"{name}: ggml type {gt} is not supported here")
            infos[name] = TensorInfo(name, tuple(reversed(ne)), gt, off)
        align = int(meta.get("general.alignment", GGUF_DEFAULT_ALIGNMENT))
        data_offset = (f.tell() + align - 1) // align * align
    g = GGUFFile(path, version, meta, infos, data_offset)
    size = path.stat().st_size
    for ti in infos.values():
        if ti.offset % align or data_offset + ti.offset + ti.nbytes > size:
            raise GGUFError(f"{ti.name}: data out of place (offset {ti.offset}, {ti.nbytes} bytes)")
    return g


def _value_bytes(v) -> bytes:
    if isinstance(v, bool):
        return struct.pack("<I?", _BOOL, v)
    if isinstance(v, int):
        return struct.pack("<Iq", _I64, v) if v < 0 else struct.pack("<IQ", _U64, v)
    if isinstance(v, float):
        return struct.pack("<If", _F32, v)
    if isinstance(v, str):
        b = v.encode("utf-8")
        return struct.pack("<IQ", _STR, len(b)) + b
    if isinstance(v, (list, tuple)):
        if not v:
            return struct.pack("<IIQ", _ARR, _U32, 0)
        items = [_value_bytes(x) for x in v]
        et = struct.unpack("<I", items[0][:4])[0]
        return struct.pack("<IIQ", _ARR, et, len(v)) + b"".join(it[4:] for it in items)
    raise GGUFError(f"cannot store metadata value {v!r}")


def write(path, metadata: dict, tensors: dict, alignment: int = GGUF_DEFAULT_ALIGNMENT) -> None:
    """Writes a GGUF v3 file.  tensors: name -> (type name, Candle shape, raw bytes or float array)."""
    meta = dict(metadata)
    if alignment != GGUF_DEFAULT_ALIGNMENT:
        meta["general.alignment"] = alignment
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(meta))
    for k, v in meta.items():
        kb = k.encode("utf-8")
        head += struct.pack("<Q", len(kb)) + kb + _value_bytes(v)
    blobs, off = [], 0
    for name, (tname, shape, data) in tensors.items():
        raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        ti = TensorInfo(name, tuple(shape), TYPE_IDS[tname], off)
        if raw.size != ti.nbytes:
            raise GGUFError(f"{name}: {raw.size} bytes for a {tname} tensor of shape {shape} ({ti.nbytes})")
        nb = name.encode("utf-8")
        ne = tuple(reversed(shape))
        head += struct.pack("<Q", len(nb)) + nb + struct.pack(f"<I{len(ne)}Q", len(ne), *ne)
        head += struct.pack("<IQ", ti.ggml_type, off)
        blobs.append((off, raw))
        off = (off + raw.size + alignment - 1) // alignment * alignment
    data_offset = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_offset - len(head)))
        pos = 0
        for o, raw in blobs:
            f.write(b"\0" * (o - pos))
            f.write(raw.tobytes())
            pos = o + raw.size


# ---- tensor-parallel placement (src/tensor_parallel_model.rs:37-61) ------------------------
# axis of the split in Candle shape, or None for a replicated tensor
LAYER_SHARDS = {
    "attn_q.weight": 0, "attn_k.weight": 0, "attn_v.weight": 0, "attn_output.weight": 1,
    "attn_q_norm.weight": 0, "attn_k_norm.weight": 0, "attn_norm.weight": None, "ffn_norm.weight": None,
    "ffn_gate_inp.weight": None, "exp_probs_b.bias": None,
    "ffn_gate_exps.weight": 1, "ffn_up_exps.weight": 1, "ffn_down_exps.weight": 2,
}


def shard_bytes(g: GGUFFile, name: str, world: int, rank: int) -> tuple:
    """(Candle shape, uint8 bytes) of rank `rank`'s part of a layer tensor, without dequantising:
    a split along an outer axis takes whole rows; a split along the innermost (K) axis takes whole
    blocks of every row (the split must fall on block boundaries)."""
    short = name.split(".", 2)[-1] if name.startswith("blk.") else name
    if short not in LAYER_SHARDS:
        raise GGUFError(f"{name}: no tensor-parallel placement is defined for it")
    axis = LAYER_SHARDS[short]
    ti = g.info(name)
    raw = np.asarray(g.tensor_bytes(name))
    if world == 1 or axis is None:
        return ti.shape, raw
    shape = list(ti.shape)
    if shape[axis] % world:
        raise GGUFError(f"{name}: dimension {axis} ({shape[axis]}) does not split {world} ways")
    _, be, bb = GGML_TYPES[ti.ggml_type]
    per = shape[axis] // world
    if axis == len(shape) - 1:  # K split: whole blocks of every row
        if per % be:
            raise GGUFError(f"{name}: a {per}-wide K shard is not a whole number of {ti.type_name} blocks")
        rows = raw.reshape(-1, shape[-1] // be * bb)
        part = rows[:, rank * per // be * bb:(rank + 1) * per // be * bb]
    else:  # rows of the outer axis
        outer = int(np.prod(shape[:axis])) if axis else 1
        row_bytes = int(np.prod(shape[axis + 1:])) // be * bb
        part = raw.reshape(outer, shape[axis], row_bytes)[:, rank * per:(rank + 1) * per, :]
    shape[axis] = per
    return tuple(shape), np.ascontiguousarray(part).reshape(-1)


# ---- building the library's layer objects ---------------------------------------------------
def _type_code(pkg, tname: str) -> int:
    codes = {"Q4_K": pkg.Q4K, "Q5_K": pkg.Q5K}
    if tname not in codes:
        raise GGUFError(f"expert tensors of type {tname} are not supported by the MoE kernels")
    return codes[tname]


def load_moe_layer(pkg, g: GGUFFile, layer: int, dev, world: int = 1, rank: int = 0, expert_parallel: bool = False):
    """MoeLayer for `blk.{layer}`: router (`ffn_gate_inp`), bias (`exp_probs_b`) and the stacked
    experts: this rank's TP shard (gate / up rows, down K), or with expert_parallel the full tensors
    (the kernels then compute experts e % world == rank)."""
    import torch
    p = f"blk.{layer}."
    router = torch.from_numpy(np.ascontiguousarray(g.array(p + "ffn_gate_inp.weight"))).to(dev)
    bias = torch.from_numpy(np.ascontiguousarray(g.array(p + "exp_probs_b.bias"))).to(dev)
    if g.info(p + "ffn_up_exps.weight").type_name != g.info(p + "ffn_gate_exps.weight").type_name:
        raise GGUFError("gate and up experts must share one type")
    w, r = (1, 0) if expert_parallel else (world, rank)
    parts = {}
    for nm in ("ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight"):
        _, raw = shard_bytes(g, p + nm, w, r)
        parts[nm] = torch.from_numpy(np.array(raw)).to(dev)
    gt = _type_code(pkg, g.info(p + "ffn_gate_exps.weight").type_name)
    dt = _type_code(pkg, g.info(p + "ffn_down_exps.weight").type_name)
    return pkg.MoeLayer(router, bias, parts["ffn_gate_exps.weight"], parts["ffn_up_exps.weight"],
                        parts["ffn_down_exps.weight"], gt, dt)


def load_attn_layer(pkg, g: GGUFFile, layer: int, dev, rope_cos, rope_sin, eps: float = 1e-6):
    """AttnLayer for `blk.{layer}` (one GPU: full Q8_0 projections and norm weights)."""
    import torch
    p = f"blk.{layer}."
    t = {}
    for nm in ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight"):
        ti = g.info(p + nm)
        if ti.type_name != "Q8_0":
            raise GGUFError(f"{p + nm} is {ti.type_name}; the attention kernels take Q8_0")
        t[nm] = torch.from_numpy(np.array(g.tensor_bytes(p + nm))).to(dev)
    qn = torch.from_numpy(np.ascontiguousarray(g.array(p + "attn_q_norm.weight"))).to(dev)
    kn = torch.from_numpy(np.ascontiguousarray(g.array(p + "attn_k_norm.weight"))).to(dev)
    q_rows, hidden = g.info(p + "attn_q.weight").shape
    k_rows = g.info(p + "attn_k.weight").shape[0]
    return pkg.AttnLayer(t["attn_q.weight"], t["attn_k.weight"], t["attn_v.weight"], t["attn_output.weight"], qn, kn,
                         rope_cos, rope_sin, hidden, query_heads=q_rows // 128, kv_heads=k_rows // 128, eps=eps)


def load_lm_head(pkg, g: GGUFFile, dev, eps: float = 1e-6):
    """LmHead from `output.weight` (Q6_K) and `output_norm.weight`."""
    import torch
    ti = g.info("output.weight")
    if ti.type_name != "Q6_K":
        raise GGUFError(f"output.weight is {ti.type_name}; the LM head kernel takes Q6_K")
    w = torch.from_numpy(np.array(g.tensor_bytes("output.weight"))).to(dev)
    nw = torch.from_numpy(np.ascontiguousarray(g.array("output_norm.weight"))).to(dev)
    vocab, hidden = ti.shape
    return pkg.LmHead(w, nw, vocab, hidden, eps)
