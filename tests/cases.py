"""Cache geometries of the golden fixtures, rebuilt as oracle storages (numpy byte buffers).

The same seeds and geometries ``tests/golden/make_golden.py`` fed the reference,
so the oracle and the CUDA path see byte-identical inputs.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))

import kvgen  # noqa: E402
from oracle import oracle  # noqa: E402

GOLDEN = json.loads((HERE / "golden" / "golden.json").read_text())


def storages_5d(seed, layers, num_blocks, block_size=16, heads=8, head_dim=128, prefix="model.layers"):
    """Per layer a flat ``[2, num_blocks, block_size, heads, head_dim]`` bf16 buffer and its two views."""
    storages, views = {}, {}
    per_layer = 2 * num_blocks * block_size * heads * head_dim * 2
    for i in range(layers):
        name = f"{prefix}.{i}"
        storages[name] = kvgen.random_bytes(seed * 1000 + i, per_layer)
        views.update(oracle.split_5d(name, name, 0, num_blocks, block_size, heads, head_dim, 2))
    return storages, views


def storages_vllm031(seed, layers, num_blocks, block_size=16, heads=8, width=256):
    """One buffer ``[layers, num_blocks, block_size, heads, width]`` bf16; per layer a [B,H,N,C] view."""
    nbytes = layers * num_blocks * block_size * heads * width * 2
    storages = {"backing": kvgen.random_bytes(seed, nbytes)}
    per_layer = num_blocks * block_size * heads * width * 2
    pitch = block_size * heads * width * 2
    views = {}
    for i in range(layers):
        name = f"model.layers.{i}.self_attn.attn"
        views[name] = oracle.Span(name, "backing", i * per_layer, pitch, (heads, block_size, width),
                                  (width, heads * width, 1), 2, num_blocks)
    return storages, views


def storages_small(strides, seed):
    """The reference layout tests' tiny cache: (5 blocks, 3 heads, 4 tokens, 8 width) bf16 with ``strides``."""
    storages = {"small": kvgen.random_bytes(seed, 5 * strides[0] * 2)}
    views = {"layer.0": oracle.Span("layer.0", "small", 0, strides[0] * 2, (3, 4, 8), tuple(strides[1:]), 2, 5)}
    return storages, views


def golden_case(key):
    """(fixture entry, storages, layout) for one of the large golden cases."""
    case = GOLDEN[key]
    if case["kind"] == "5d":
        storages, views = storages_5d(case["seed"], case["num_layers"], case["num_blocks"])
    else:
        storages, views = storages_vllm031(case["seed"], case["num_layers"], case["num_blocks"])
    return case, storages, oracle.register(views, 16)


def sha_of(buf: np.ndarray) -> str:
    import hashlib
    return hashlib.sha256(buf.tobytes()).hexdigest()
