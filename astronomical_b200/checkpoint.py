"""SafeTensors ingestion of MLX-quantised Qwen3.5/3.6-MoE checkpoints.

Reads the sparse MoE block of a decoder layer from an MLX checkpoint directory
(config.json + model.safetensors or sharded model-*.safetensors with
model.safetensors.index.json) into the weight dict the block, expert-parallel
and paged front ends take (keys of astronomical_b200.synthetic.make_block_weights),
without copying payloads: every tensor is a read-only numpy memmap of its
byte range in the shard.

Tensor names are the reference's (paths relative to the reference root):
  router          language_model.model.layers.{i}.mlp.gate.{weight[,scales,biases]}
                  (qwen3_5_moe/model/feed_forward_weights.rs:50-70)
  routed experts  ...mlp.switch_mlp.{gate,up,down}_proj.{weight,scales,biases}
                  (qwen3_5_moe/expert_paging/quantized_expert_layer_plan.rs:21-24,107-108)
  shared expert   ...mlp.shared_expert.{gate,up,down}_proj.{weight,scales,biases}
  shared gate     ...mlp.shared_expert_gate.{weight[,scales,biases]}
                  (feed_forward_weights.rs:76-83)
Each module's quantisation is its override in config.json "quantization" (or
"quantization_config"; both present must agree) or the declared default
(qwen3_5/configuration/config.rs:120-155, config_accessors.rs:40-49).  Header
parsing is bounded like the reference's (expert_paging/safetensors_header.rs):
the JSON header is at most 64 MiB, must lie inside the file, every tensor's
byte range must lie inside the payload and match its dtype and shape.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np

MAXIMUM_HEADER_BYTES = 64 * 1024 * 1024
LENGTH_PREFIX_BYTES = 8

# dtype spellings MLX 0.32 accepts (safetensors_header.rs DTYPE_BYTE_WIDTHS) -> numpy
# storage (bf16 is kept as its uint16 bit pattern, the convention of this package)
DTYPES = {"BOOL": np.bool_, "I8": np.int8, "U8": np.uint8, "F8_E4M3": np.uint8,
          "F8_E5M2": np.uint8, "I16": np.int16, "U16": np.uint16, "F16": np.float16,
          "BF16": np.uint16, "I32": np.int32, "U32": np.uint32, "F32": np.float32,
          "I64": np.int64, "U64": np.uint64}
WIDTHS = {k: np.dtype(v).itemsize for k, v in DTYPES.items()}

LAYER_PREFIX = "language_model.model.layers.{layer}.mlp"
# weight-dict key -> module suffix under the layer's mlp prefix
MODULES = {"gate": "switch_mlp.gate_proj", "up": "switch_mlp.up_proj",
           "down": "switch_mlp.down_proj", "sgate": "shared_expert.gate_proj",
           "sup": "shared_expert.up_proj", "sdown": "shared_expert.down_proj",
           "router": "gate", "shared_gate": "shared_expert_gate"}


class SafetensorsHeaderError(ValueError):
    """A shard's framing or header is invalid (mirrors SafetensorsHeaderError)."""


class CheckpointError(ValueError):
    """A tensor the MoE block needs is missing or has the wrong dtype or shape."""


@dataclass(frozen=True)
class TensorEntry:
    dtype: str
    shape: Tuple[int, ...]
    begin: int  # absolute byte offset in the file
    end: int


def read_header(path: str) -> Dict[str, TensorEntry]:
    """Parses and validates one shard's header (payload bytes are not read)."""
    if not os.path.exists(path):
        raise SafetensorsHeaderError(f"safetensors file does not exist: {path}")
    if not os.path.isfile(path):
        raise SafetensorsHeaderError(f"safetensors path is not a regular file: {path}")
    size = os.path.getsize(path)
    if size < LENGTH_PREFIX_BYTES:
        raise SafetensorsHeaderError(
            f"safetensors file is too small to contain a header length prefix: {size} bytes")
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(LENGTH_PREFIX_BYTES))
        if n > MAXIMUM_HEADER_BYTES:
            raise SafetensorsHeaderError(
                f"safetensors header length {n} exceeds the safety limit of "
                f"{MAXIMUM_HEADER_BYTES} bytes")
        if LENGTH_PREFIX_BYTES + n > size:
            raise SafetensorsHeaderError(
                f"safetensors header extends beyond the file: header ends at "
                f"{LENGTH_PREFIX_BYTES + n} but file is {size} bytes")
        raw = f.read(n)
    if len(raw) != n:
        raise SafetensorsHeaderError(
            f"safetensors header is truncated: expected {n} bytes, read {len(raw)}")
    try:
        doc = json.loads(raw.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise SafetensorsHeaderError("safetensors header must contain valid JSON") from e
    if not isinstance(doc, dict):
        raise SafetensorsHeaderError(
            f"safetensors header must be a JSON object, got {type(doc).__name__}")
    base = LENGTH_PREFIX_BYTES + n
    out = {}
    for name, e in doc.items():
        if name == "__metadata__":
            continue
        if not isinstance(e, dict):
            raise SafetensorsHeaderError(f"tensor {name!r} has an invalid entry")
        dtype = e.get("dtype")
        if dtype not in WIDTHS:
            raise SafetensorsHeaderError(f"tensor {name!r} has an unsupported dtype: {dtype!r}")
        shape = e.get("shape")
        if not isinstance(shape, list) or not all(isinstance(d, int) and d >= 0 for d in shape):
            raise SafetensorsHeaderError(f"tensor {name!r} has an invalid shape")
        offs = e.get("data_offsets")
        if (not isinstance(offs, list) or len(offs) != 2 or
                not all(isinstance(o, int) and o >= 0 for o in offs) or offs[0] > offs[1]):
            raise SafetensorsHeaderError(f"tensor {name!r} has invalid data offsets")
        nbytes = int(np.prod(shape, dtype=np.int64)) * WIDTHS[dtype]
        if offs[1] - offs[0] != nbytes:
            raise SafetensorsHeaderError(
                f"tensor {name!r} spans {offs[1] - offs[0]} bytes, its dtype and shape need {nbytes}")
        if base + offs[1] > size:
            raise SafetensorsHeaderError(
                f"tensor {name!r} ends at byte {base + offs[1]}, beyond the {size}-byte file")
        out[name] = TensorEntry(dtype, tuple(shape), base + offs[0], base + offs[1])
    return out


def open_tensor(path: str, entry: TensorEntry) -> np.ndarray:
    """Read-only memmap of one tensor (no copy)."""
    if entry.end == entry.begin:
        return np.zeros(entry.shape, DTYPES[entry.dtype])
    return np.memmap(path, dtype=DTYPES[entry.dtype], mode="r", offset=entry.begin,
                     shape=entry.shape)


def write_safetensors(path: str, tensors: Dict[str, Tuple[str, np.ndarray]],
                      metadata: Optional[Dict[str, str]] = None) -> None:
    """Writes a shard: tensors maps a name to (safetensors dtype, array)."""
    header, chunks, off = {}, [], 0
    for name, (dtype, arr) in tensors.items():
        a = np.ascontiguousarray(arr, dtype=DTYPES[dtype])
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        chunks.append(a.tobytes())
        off += a.nbytes
    if metadata:
        header["__metadata__"] = dict(metadata)
    raw = json.dumps(header).encode("utf-8")
    raw += b" " * (-len(raw) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for c in chunks:
            f.write(c)


class Checkpoint:
    """An MLX checkpoint directory; shard headers are parsed once each and kept
    (the reference shares one header cache across all layers)."""

    def __init__(self, model_dir: str):
        self.model_dir = model_dir
        with open(os.path.join(model_dir, "config.json")) as f:
            self.config = json.load(f)
        self.text = self.config.get("text_config", self.config)
        index = os.path.join(model_dir, "model.safetensors.index.json")
        if os.path.exists(index):
            with open(index) as f:
                self.weight_map = dict(json.load(f)["weight_map"])
        else:
            single = os.path.join(model_dir, "model.safetensors")
            self.weight_map = {n: "model.safetensors" for n in read_header(single)}
        self._headers: Dict[str, Dict[str, TensorEntry]] = {}
        q, qc = self.config.get("quantization"), self.config.get("quantization_config")
        if q is not None and qc is not None and q != qc:
            raise CheckpointError("quantization and quantization_config fields differ")
        self.quantization = q if q is not None else qc

    def _entry(self, name: str):
        shard = self.weight_map.get(name)
        if shard is None:
            return None, None
        path = os.path.join(self.model_dir, shard)
        if path not in self._headers:
            self._headers[path] = read_header(path)
        e = self._headers[path].get(name)
        if e is None:
            raise CheckpointError(f"tensor {name!r} is listed for {shard} but missing from it")
        return path, e

    def has(self, name: str) -> bool:
        return name in self.weight_map

    def tensor(self, name: str, dtype: Optional[str] = None, shape=None) -> np.ndarray:
        path, e = self._entry(name)
        if e is None:
            raise CheckpointError(f"missing tensor entry {name!r}")
        if dtype is not None and e.dtype != dtype:
            raise CheckpointError(f"tensor {name!r} has dtype {e.dtype}, expected {dtype}")
        if shape is not None and tuple(e.shape) != tuple(shape):
            raise CheckpointError(f"tensor {name!r} has shape {list(e.shape)}, expected {list(shape)}")
        return open_tensor(path, e)

    def quantization_profile(self, module: str) -> Tuple[int, int]:
        """(bits, group_size) of a module: its override, else the default."""
        q = self.quantization
        if q is None:
            return 0, 0
        o = q.get(module)
        if isinstance(o, dict):
            return int(o["bits"]), int(o["group_size"])
        return int(q["bits"]), int(q["group_size"])

    def block_config(self) -> dict:
        t = self.text
        bits, group = (int(self.quantization["bits"]), int(self.quantization["group_size"])) \
            if self.quantization else (0, 0)
        return dict(hidden=int(t["hidden_size"]), experts=int(t["num_experts"]),
                    top_k=int(t["num_experts_per_tok"]),
                    intermediate=int(t["moe_intermediate_size"]),
                    shared_intermediate=int(t.get("shared_expert_intermediate_size", 0)),
                    group=group, bits=bits, normalize=bool(t.get("norm_topk_prob", True)),
                    zipf=None)

    def moe_layer(self, layer: int) -> dict:
        """The MoE block of decoder layer `layer` as a weight dict (memmaps)."""
        cfg = self.block_config()
        if not self.quantization:
            raise CheckpointError("the routed experts must be affine-quantised (no quantization "
                                  "configuration found)")
        H, E, I, Is = cfg["hidden"], cfg["experts"], cfg["intermediate"], cfg["shared_intermediate"]
        prefix = LAYER_PREFIX.format(layer=layer)
        w = {"config": cfg}

        def affine(key, rows, in_f, required=True):
            module = f"{prefix}.{MODULES[key]}"
            if not self.has(f"{module}.scales"):
                if not required:
                    return False
                if self.has(f"{module}.weight"):
                    raise CheckpointError(f"{module} is stored unquantised; the expert kernels "
                                          "take affine-quantised projections")
                raise CheckpointError(f"missing tensor entry {module + '.weight'!r}")
            bits, group = self.quantization_profile(module)
            if bits not in (2, 3, 4, 5, 6, 8) or group not in (32, 64, 128) or in_f % group or \
                    (in_f * bits) % 32:
                raise CheckpointError(f"{module}: unsupported quantisation {bits} bits, group {group}")
            w[key + "_q"] = self.tensor(f"{module}.weight", "U32", rows + (in_f * bits // 32,))
            w[key + "_s"] = self.tensor(f"{module}.scales", "BF16", rows + (in_f // group,))
            w[key + "_b"] = self.tensor(f"{module}.biases", "BF16", rows + (in_f // group,))
            if (bits, group) != (cfg["bits"], cfg["group"]):
                w[key + "_bits"], w[key + "_group"] = bits, group
            return True

        affine("gate", (E, I), H)
        affine("up", (E, I), H)
        affine("down", (E, H), I)
        if not affine("router", (E,), H, required=False):
            w["router_w"] = self.tensor(f"{prefix}.gate.weight", "BF16", (E, H))
        if Is:
            affine("sgate", (Is,), H)
            affine("sup", (Is,), H)
            affine("sdown", (H,), Is)
            if not affine("shared_gate", (1,), H, required=False):
                w["shared_gate_w"] = self.tensor(f"{prefix}.shared_expert_gate.weight", "BF16", (1, H))
        return w


def export_moe_layer(weights: dict, layer: int) -> Dict[str, Tuple[str, np.ndarray]]:
    """The tensors of one block's weight dict under the reference's names (for
    writing a checkpoint): the inverse of Checkpoint.moe_layer."""
    prefix = LAYER_PREFIX.format(layer=layer)
    out = {}
    for key, module in MODULES.items():
        if key + "_q" in weights:
            out[f"{prefix}.{module}.weight"] = ("U32", np.asarray(weights[key + "_q"]))
            out[f"{prefix}.{module}.scales"] = ("BF16", np.asarray(weights[key + "_s"]))
            out[f"{prefix}.{module}.biases"] = ("BF16", np.asarray(weights[key + "_b"]))
    if "router_w" in weights:
        out[f"{prefix}.gate.weight"] = ("BF16", np.asarray(weights["router_w"]))
    if "shared_gate_w" in weights:
        out[f"{prefix}.shared_expert_gate.weight"] = ("BF16", np.asarray(weights["shared_gate_w"]))
    return out


def module_overrides(weights: dict, layer: int) -> dict:
    """config.json "quantization" overrides for the projections of a weight dict
    that carry their own bits / group size."""
    prefix = LAYER_PREFIX.format(layer=layer)
    return {f"{prefix}.{module}": {"bits": int(weights[key + "_bits"]),
                                   "group_size": int(weights[key + "_group"])}
            for key, module in MODULES.items() if key + "_bits" in weights}


__all__ = ["SafetensorsHeaderError", "CheckpointError", "TensorEntry", "read_header",
           "open_tensor", "write_safetensors", "Checkpoint", "export_moe_layer",
           "module_overrides"]
