"""On-disk cache of the neuron-major down-projection layout (safetensors).

The sparse kernels read the down projections in the neuron-major layout, which a loader
builds from the checkpoint at load time (to_neuron_major: a permutation of the checkpoint's
bytes, hsd/model.py:89-107 of the reference builds it the same way on every load). A cache
file keeps the permuted tensors of every MoE layer, so a later load reads them directly: no
transpose runs, and only the one layout the kernels need is ever resident.

File: one safetensors file. Tensors "layers.{i}.{pw,ps,pb,spw,sps,spb}" for the MoE layers
in order, with the dtypes and shapes to_neuron_major gives. Metadata: "format" (this
module's FORMAT), "key" (the caller's description of the source weights -- a checkpoint
path and revision, a file hash, or a seed for synthetic weights) and "layers" (the count).
A load whose key or format differs raises LayoutCacheMismatch, so a stale cache is never
used silently; the caller rebuilds and saves again.
"""
import os

import torch

NAMES = ("pw", "ps", "pb", "spw", "sps", "spb")
FORMAT = "hsd-neuron-major-1"


class LayoutCacheMismatch(RuntimeError):
    """The cache file was written for other source weights or in another format."""


def save_layout_cache(path, layers, key):
    """Write the neuron-major tensors of every MoE layer to `path`.

    layers: a sequence of (pw, ps, pb, spw, sps, spb) tuples, one per MoE layer, on any
    device (safetensors copies them to host memory). key: a string naming the source
    weights. The file is written next to `path` and renamed into place, so a crash never
    leaves a truncated cache under the final name."""
    tensors = {}
    for i, lay in enumerate(layers):
        if len(lay) != len(NAMES):
            raise ValueError(f"save_layout_cache: layer {i} has {len(lay)} tensors, expected {len(NAMES)}")
        for name, t in zip(NAMES, lay):
            if not isinstance(t, torch.Tensor):
                raise TypeError(f"save_layout_cache: layers.{i}.{name} is not a tensor")
            tensors[f"layers.{i}.{name}"] = t.detach().contiguous()
    from safetensors.torch import save_file
    meta = {"format": FORMAT, "key": str(key), "layers": str(len(layers))}
    tmp = f"{path}.tmp"
    save_file(tensors, tmp, metadata=meta)
    os.replace(tmp, path)


def load_layout_cache(path, key, device="cuda"):
    """Read the cache at `path` onto `device` -> list of (pw, ps, pb, spw, sps, spb) tuples.
    Raises LayoutCacheMismatch when the file's format or key differs from `key`, and
    FileNotFoundError when there is no file."""
    from safetensors import safe_open
    with safe_open(path, framework="pt", device=str(device)) as f:
        meta = f.metadata() or {}
        if meta.get("format") != FORMAT:
            raise LayoutCacheMismatch(f"{path}: format {meta.get('format')!r}, expected {FORMAT!r}")
        if meta.get("key") != str(key):
            raise LayoutCacheMismatch(f"{path}: written for {meta.get('key')!r}, not {str(key)!r}")
        n = int(meta.get("layers", "0"))
        return [tuple(f.get_tensor(f"layers.{i}.{name}") for name in NAMES) for i in range(n)]


def neuron_major_layers(path, key, build, device="cuda"):
    """The MoE layers' neuron-major tensors from the cache at `path` when it holds `key`,
    else from build() (a callable returning the list of (pw, ps, pb, spw, sps, spb) tuples,
    e.g. to_neuron_major over each layer's checkpoint tensors), which are then saved to
    `path` for the next load. Returns (layers, loaded_from_cache)."""
    if path and os.path.exists(path):
        try:
            return load_layout_cache(path, key, device), True
        except LayoutCacheMismatch:
            pass
    layers = build()
    if path:
        save_layout_cache(path, layers, key)
    return layers, False
