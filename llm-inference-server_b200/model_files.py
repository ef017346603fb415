"""Synthetic GPT-2 model directories in the reference's on-disk format.

Writes ``weights.bin`` + ``manifest.json`` + ``config.json`` exactly as
gpu-engine/export/export_gpt2.py:98-158 lays them out, so the reference's
WeightsLoader (gpu-engine/src/reference/weights_loader.cpp:14-72: total_bytes,
per-tensor byte ranges, double checksum_sum) and GPT2Config
(gpu-engine/src/model.cpp:7-23) accept them unchanged:

  * tensors back to back as float32, in the order of
    gpu-engine/src/loader.cpp:28-47 (wte, wpe, per layer ln1_g ln1_b qkv_w
    qkv_b proj_w proj_b ln2_g ln2_b fc_w fc_b fc_proj_w fc_proj_b, lnf_g lnf_b);
  * Linear weights row-major [out_features, in_features] (the exporter's
    transposed Conv1D layout, export_gpt2.py:46-56).

There are no pretrained weights or network here, so values are synthetic:
every weight matrix, embedding and bias ~ N(0, std) from one seeded numpy
PCG64 stream (std = 0.02 by default), LayerNorm gamma = 1 and beta = 0.
``eos_token_id`` defaults to -1 so greedy decoding never stops early (the
reference CPU path stops at EOS, cpu_model.cpp:207,213; its GPU engine does not).
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class GPT2Shape:
    n_layer: int = 12
    n_head: int = 12
    d_model: int = 768
    vocab_size: int = 50257
    n_ctx: int = 1024
    layer_norm_epsilon: float = 1e-5
    eos_token_id: int = -1

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_head


GPT2_SMALL = GPT2Shape()
GPT2_MEDIUM = GPT2Shape(n_layer=24, n_head=16, d_model=1024)
GPT2_XL = GPT2Shape(n_layer=48, n_head=25, d_model=1600)


def tensor_specs(shape: GPT2Shape) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) in file order; init is 'normal', 'ones' or 'zeros'."""
    D, V = shape.d_model, shape.vocab_size
    specs: list[tuple[str, tuple[int, ...], str]] = [("wte", (V, D), "normal"), ("wpe", (shape.n_ctx, D), "normal")]
    for i in range(shape.n_layer):
        p = f"layer{i}."
        specs += [
            (p + "ln1_g", (D,), "ones"), (p + "ln1_b", (D,), "zeros"),
            (p + "qkv_w", (3 * D, D), "normal"), (p + "qkv_b", (3 * D,), "normal"),
            (p + "proj_w", (D, D), "normal"), (p + "proj_b", (D,), "normal"),
            (p + "ln2_g", (D,), "ones"), (p + "ln2_b", (D,), "zeros"),
            (p + "fc_w", (4 * D, D), "normal"), (p + "fc_b", (4 * D,), "normal"),
            (p + "fc_proj_w", (D, 4 * D), "normal"), (p + "fc_proj_b", (D,), "normal"),
        ]
    specs += [("lnf_g", (D,), "ones"), ("lnf_b", (D,), "zeros")]
    return specs


def generate_tensors(shape: GPT2Shape, seed: int = 0, std: float = 0.02):
    """Yields (name, float32 array) in file order from one seeded stream."""
    rng = np.random.Generator(np.random.PCG64(seed))
    for name, shp, init in tensor_specs(shape):
        if init == "normal":
            arr = (rng.standard_normal(shp, dtype=np.float32) * np.float32(std)).astype(np.float32)
        elif init == "ones":
            arr = np.ones(shp, dtype=np.float32)
        else:
            arr = np.zeros(shp, dtype=np.float32)
        yield name, arr


def write_model_dir(out_dir: str | Path, shape: GPT2Shape = GPT2_SMALL, seed: int = 0, std: float = 0.02) -> Path:
    """Writes the three files; returns the directory.  Skips the work when a
    directory with the same shape, seed and std is already complete."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    stamp = {"shape": shape.__dict__, "seed": seed, "std": std}
    stamp_path = out / "synthetic.json"
    if stamp_path.exists() and (out / "weights.bin").exists():
        try:
            if json.loads(stamp_path.read_text()) == stamp:
                return out
        except json.JSONDecodeError:
            pass
    manifest = []
    sha = hashlib.sha256()
    checksum = 0.0
    offset = 0
    with open(out / "weights.bin", "wb") as f:
        for name, arr in generate_tensors(shape, seed, std):
            raw = np.ascontiguousarray(arr, dtype=np.float32).tobytes()
            f.write(raw)
            sha.update(raw)
            checksum += float(np.sum(arr.astype(np.float64)))
            manifest.append({"name": name, "dtype": "float32", "shape": list(arr.shape), "byte_offset": offset,
                             "byte_length": len(raw)})
            offset += len(raw)
    (out / "manifest.json").write_text(json.dumps(
        {"tensors": manifest, "checksum_sha256": sha.hexdigest(), "checksum_sum": checksum, "total_bytes": offset},
        indent=1))
    (out / "config.json").write_text(json.dumps({
        "n_layer": shape.n_layer, "n_head": shape.n_head, "d_model": shape.d_model, "head_dim": shape.head_dim,
        "vocab_size": shape.vocab_size, "n_ctx": shape.n_ctx, "layer_norm_epsilon": shape.layer_norm_epsilon,
        "eos_token_id": shape.eos_token_id, "source_model": f"synthetic-seed{seed}-std{std}"}, indent=1))
    stamp_path.write_text(json.dumps(stamp))
    return out


def load_model_dir(model_dir: str | Path) -> tuple[dict, dict[str, np.ndarray]]:
    """Reads (config, {name: float32 array}) back from a model directory."""
    d = Path(model_dir)
    cfg = json.loads((d / "config.json").read_text())
    man = json.loads((d / "manifest.json").read_text())
    blob = np.fromfile(d / "weights.bin", dtype=np.uint8)
    tensors = {}
    for t in man["tensors"]:
        a = blob[t["byte_offset"]: t["byte_offset"] + t["byte_length"]].view(np.float32).reshape(t["shape"])
        tensors[t["name"]] = a
    return cfg, tensors
