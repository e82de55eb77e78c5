"""HF LLaMA checkpoints in safetensors form, read without copying the file.

The weights path of the reference's compile chain takes an HF ``LlamaForCausalLM``
(tests/test_partition.py:128-167 loads one with ``from_pretrained``) and its
memory planner copies the weight shards into the arenas once
(docs/spec.md:2095-2101).  Here a checkpoint directory (``config.json`` plus
``model.safetensors`` or the sharded ``model.safetensors.index.json`` form) is
opened as a lazy mapping of memory-mapped numpy arrays, and
``runtime.program.load_state_dict`` streams it into the arenas one decoder layer
at a time, so loading a 7B model never holds more than one layer's fused weights
in host memory.

safetensors layout (the format's published specification): an 8-byte
little-endian header length N, N bytes of UTF-8 JSON mapping each tensor name to
``{"dtype", "shape", "data_offsets": [begin, end]}`` (offsets relative to the
byte buffer that follows the header; an optional ``"__metadata__"`` entry), then
the byte buffer.
"""

from __future__ import annotations

import json
import struct
from collections.abc import Mapping
from pathlib import Path

import numpy as np

from comm.plan import np_dtype
from graph.llama import ModelConfig

_DTYPES = {"F64": "float64", "F32": "float32", "F16": "float16", "BF16": "bfloat16", "I64": "int64",
           "I32": "int32", "I16": "int16", "I8": "int8", "U8": "uint8", "BOOL": "bool"}
_INDEX = "model.safetensors.index.json"
_SINGLE = "model.safetensors"


def _read_header(path: Path) -> tuple[dict, int]:
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (shorter than 8 bytes)")
        (n,) = struct.unpack("<Q", raw)
        size = path.stat().st_size
        if n > size - 8:
            raise ValueError(f"{path}: header length {n} exceeds the file ({size} bytes)")
        header = json.loads(f.read(n).decode("utf-8"))
    header.pop("__metadata__", None)
    return header, 8 + n


class SafetensorsFile(Mapping):
    """One safetensors file: ``name -> np.ndarray`` views of a read-only memory map."""

    def __init__(self, path) -> None:
        self.path = Path(path)
        self.header, self._base = _read_header(self.path)
        self._map = None
        buf_bytes = self.path.stat().st_size - self._base
        for name, t in self.header.items():
            if t["dtype"] not in _DTYPES:
                raise ValueError(f"{self.path}: tensor {name} has unsupported dtype {t['dtype']}")
            b, e = t["data_offsets"]
            want = int(np.prod(t["shape"], dtype=np.int64)) * np_dtype(_DTYPES[t["dtype"]]).itemsize
            if not 0 <= b <= e <= buf_bytes or e - b != want:
                raise ValueError(f"{self.path}: tensor {name} has data_offsets {t['data_offsets']} for "
                                 f"shape {t['shape']} {t['dtype']}")

    def __getitem__(self, name: str) -> np.ndarray:
        t = self.header[name]
        if self._map is None:
            self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        b, e = t["data_offsets"]
        raw = self._map[self._base + b:self._base + e]
        return raw.view(np_dtype(_DTYPES[t["dtype"]])).reshape(t["shape"])

    def __iter__(self):
        return iter(self.header)

    def __len__(self) -> int:
        return len(self.header)


class Checkpoint(Mapping):
    """Every tensor of a checkpoint directory (single file or sharded with an index)."""

    def __init__(self, path) -> None:
        self.path = Path(path)
        if self.path.is_file():
            files = {self.path.name: SafetensorsFile(self.path)}
            self._where = {k: self.path.name for k in files[self.path.name]}
        elif (self.path / _INDEX).is_file():
            index = json.loads((self.path / _INDEX).read_text())
            self._where = dict(index["weight_map"])
            files = {f: SafetensorsFile(self.path / f) for f in sorted(set(self._where.values()))}
            for k, f in self._where.items():
                if k not in files[f]:
                    raise ValueError(f"{self.path / _INDEX}: {k} is not in {f}")
        elif (self.path / _SINGLE).is_file():
            files = {_SINGLE: SafetensorsFile(self.path / _SINGLE)}
            self._where = {k: _SINGLE for k in files[_SINGLE]}
        else:
            raise FileNotFoundError(f"{self.path}: no {_SINGLE} or {_INDEX}")
        self._files = files

    def __getitem__(self, name: str) -> np.ndarray:
        return self._files[self._where[name]][name]

    def __iter__(self):
        return iter(self._where)

    def __len__(self) -> int:
        return len(self._where)


def model_config(path, max_seq: int, dtype: str | None = None) -> ModelConfig:
    """``ModelConfig`` from a checkpoint's ``config.json`` (LLaMA family only).

    ``dtype`` defaults to the checkpoint's own (``torch_dtype`` / ``dtype``) when it is
    float32 or bfloat16, else bfloat16.  Features the kernels do not implement (RoPE
    scaling, attention or MLP biases, a head_dim other than hidden / heads) are refused.
    """
    cfg = json.loads((Path(path) / "config.json").read_text())
    if cfg.get("model_type", "llama") != "llama":
        raise ValueError(f"model_type {cfg.get('model_type')!r} is not a LLaMA model")
    if cfg.get("rope_scaling"):
        raise ValueError(f"rope_scaling {cfg['rope_scaling']!r} is not supported")
    if cfg.get("attention_bias") or cfg.get("mlp_bias"):
        raise ValueError("projection biases are not supported")
    heads = cfg["num_attention_heads"]
    if cfg.get("head_dim") not in (None, cfg["hidden_size"] // heads):
        raise ValueError(f"head_dim {cfg['head_dim']} != hidden_size / num_attention_heads")
    if dtype is None:
        stored = cfg.get("torch_dtype") or cfg.get("dtype") or "bfloat16"
        dtype = stored if stored in ("float32", "bfloat16") else "bfloat16"
    if dtype not in ("float32", "bfloat16"):
        raise ValueError(f"dtype {dtype!r}: the kernels run float32 or bfloat16")
    return ModelConfig(cfg["vocab_size"], cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"],
                       heads, cfg.get("num_key_value_heads") or heads, float(cfg["rms_norm_eps"]),
                       float(cfg.get("rope_theta", 10000.0)), dtype, max_seq)


class StateDict(Mapping):
    """HF-named weights of a checkpoint in ``dtype`` (converted on access).

    Tensors already in ``dtype`` stay memory-mapped views; others are converted through
    fp32 (exact from fp16 / bf16) with round-to-nearest-even, as torch's ``.to`` does.
    ``lm_head.weight`` falls back to the embedding when the checkpoint ties them.
    """

    def __init__(self, ckpt: Mapping, dtype: str) -> None:
        self.ckpt, self.dtype = ckpt, np_dtype(dtype)

    def _key(self, name: str) -> str:
        if name == "lm_head.weight" and name not in self.ckpt:
            return "model.embed_tokens.weight"
        return name

    def __getitem__(self, name: str) -> np.ndarray:
        w = self.ckpt[self._key(name)]
        if w.dtype == self.dtype:
            return w
        return np.asarray(w).astype(np.float32).astype(self.dtype)

    def __contains__(self, name) -> bool:
        return self._key(name) in self.ckpt

    def __iter__(self):
        keys = list(self.ckpt)
        if "lm_head.weight" not in self.ckpt and "model.embed_tokens.weight" in self.ckpt:
            keys.append("lm_head.weight")
        return iter(keys)

    def __len__(self) -> int:
        return sum(1 for _ in self)


def state_dict(path, dtype: str) -> StateDict:
    """HF-named weights of the checkpoint at ``path`` (a directory or one .safetensors file)."""
    return StateDict(Checkpoint(path), dtype)
