"""The golden geometries as CUDA tensors, byte-identical to the oracle's numpy storages."""
from __future__ import annotations

import numpy as np
import torch

from cases import storages_5d, storages_small, storages_vllm031


def to_cuda(buf: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(buf.copy()).cuda()


def cuda_5d(case):
    """Per layer one [2, B, 16, 8, 128] bf16 CUDA tensor (registered 5-D; the data plane splits K/V)."""
    storages, _ = storages_5d(case["seed"], case["num_layers"], case["num_blocks"])
    tensors = {name: to_cuda(buf) for name, buf in storages.items()}
    caches = {name: t.view(torch.bfloat16).view(2, case["num_blocks"], 16, 8, 128) for name, t in tensors.items()}
    return storages, tensors, caches


def cuda_vllm031(case):
    """One [L, B, 16, 8, 256] bf16 buffer, per layer a [B, 8, 16, 256] view (vLLM 0.31.0 registration)."""
    storages, _ = storages_vllm031(case["seed"], case["num_layers"], case["num_blocks"])
    backing = to_cuda(storages["backing"])
    view = backing.view(torch.bfloat16).view(case["num_layers"], case["num_blocks"], 16, 8, 256)
    caches = {f"model.layers.{i}.self_attn.attn": view[i].permute(0, 2, 1, 3) for i in range(case["num_layers"])}
    return storages, {"backing": backing}, caches


def cuda_small(row):
    storages, _ = storages_small(row["strides"], row["seed"])
    tensor = to_cuda(storages["small"])
    cache = tensor.view(torch.bfloat16).as_strided((5, 3, 4, 8), row["strides"])
    return storages, {"small": tensor}, {"layer.0": cache}


def host_bytes(tensors: dict) -> dict:
    torch.cuda.synchronize()
    return {name: t.cpu().numpy().copy() for name, t in tensors.items()}
