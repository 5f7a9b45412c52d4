"""GGUF loading: Q4_K weight tensors of an on-disk model into device memory,
in the layout the GEMV entries take (one row per 256-weight super-block run,
144 bytes per super-block, rows contiguous).

The reference runs llama.cpp on a Q4_K GGUF checkpoint
(`llama-cli ... mistral-7b-v0.3-q4.gguf`); this is the path from such a file
to `q4k_gemv_batch` tasks.  Parsing uses the `gguf` package (gguf-py, the
format's reference reader); the file is memory-mapped and each tensor is
copied to the device once.  GGUF stores a matrix as ne = [K, rows] with rows
contiguous: exactly the Q4_K row layout, so no repacking is needed.

Names follow llama.cpp's tensor naming (`blk.{i}.attn_q.weight`, ...).
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np

QK_K = 256
BLOCK_BYTES = 144

# llama-style decoder layer matrices, in the order of a layer's launch group
# (activation group: attn = attn_norm(x), o = attention output, ffn =
# ffn_norm(h), down = glu(gate, up)).
LLAMA_LAYER = (("q", "attn_q", "attn"), ("k", "attn_k", "attn"), ("v", "attn_v", "attn"),
               ("o", "attn_output", "o"), ("gate", "ffn_gate", "ffn"), ("up", "ffn_up", "ffn"),
               ("down", "ffn_down", "down"))


@dataclass
class Q4KTensor:
    """One Q4_K matrix: `data` is (rows, K/256*144) uint8 (numpy memmap view or device tensor)."""
    name: str
    rows: int
    K: int
    data: object


class GGUFModel:
    """A GGUF file opened for reading (memory-mapped)."""

    def __init__(self, path: str | Path):
        import gguf
        self._gguf = gguf
        self.path = Path(path)
        self.reader = gguf.GGUFReader(str(self.path), "r")
        self.tensors = {t.name: t for t in self.reader.tensors}

    # ---- metadata ---------------------------------------------------------
    def field(self, key: str):
        """A scalar or string metadata value (None when absent)."""
        f = self.reader.fields.get(key)
        if f is None or not f.types:
            return None
        part = f.parts[f.data[0]]
        if f.types[0] == self._gguf.GGUFValueType.STRING:
            return bytes(part).decode("utf-8")
        return part.tolist()[0] if len(part) == 1 else part.tolist()

    @property
    def arch(self) -> str | None:
        return self.field("general.architecture")

    def n_layers(self) -> int:
        n = self.field(f"{self.arch}.block_count") if self.arch else None
        if n is not None:
            return int(n)
        idx = {int(name.split(".")[1]) for name in self.tensors if name.startswith("blk.")}
        return max(idx) + 1 if idx else 0

    # ---- tensors ----------------------------------------------------------
    def q4k(self, name: str) -> Q4KTensor:
        """Host view of one Q4_K matrix; raises for another type or a shape that is not rows x K."""
        t = self.tensors.get(name)
        if t is None:
            raise KeyError(f"{self.path}: no tensor {name!r}")
        if t.tensor_type != self._gguf.GGMLQuantizationType.Q4_K:
            raise TypeError(f"{name}: type {t.tensor_type.name}, not Q4_K")
        dims = [int(d) for d in t.shape]  # ggml order: ne0 = K, ne1 = rows, higher dims 1
        if len(dims) < 2 or any(d != 1 for d in dims[2:]):
            raise ValueError(f"{name}: shape {dims} is not a matrix")
        K, rows = dims[0], dims[1]
        if K % QK_K:
            raise ValueError(f"{name}: K={K} is not a multiple of {QK_K}")
        data = np.asarray(t.data).reshape(rows, K // QK_K * BLOCK_BYTES)
        return Q4KTensor(name, rows, K, data)

    def q4k_names(self) -> list[str]:
        return [n for n, t in self.tensors.items() if t.tensor_type == self._gguf.GGMLQuantizationType.Q4_K]

    def to_device(self, name: str, device="cuda", stream=None) -> Q4KTensor:
        """Copy one Q4_K matrix to the device (16-byte aligned, rows contiguous)."""
        import torch
        h = self.q4k(name)
        src = torch.from_numpy(np.ascontiguousarray(h.data))  # the memmap is read-only: one host copy
        dst = torch.empty(src.shape, dtype=torch.uint8, device=device)
        if stream is None:
            dst.copy_(src)
        else:
            with torch.cuda.stream(stream):
                dst.copy_(src, non_blocking=False)
        return Q4KTensor(name, h.rows, h.K, dst)

    def layer(self, i: int, device="cuda") -> dict[str, Q4KTensor]:
        """The seven Q4_K matrices of decoder layer i (llama naming), on the device."""
        out = {}
        for key, stem, _ in LLAMA_LAYER:
            out[key] = self.to_device(f"blk.{i}.{stem}.weight", device)
        return out


def layer_tasks(q4k, layer: dict[str, Q4KTensor], xs: dict, outs: dict, fuse_ffn: bool = False):
    """Task array for one decoder layer: xs maps activation group -> (ncols, K)
    fp32 device tensor, outs maps matrix key -> (ncols, rows) output.  With
    fuse_ffn the gate and up matrices become one task with the SwiGLU
    epilogue (output in outs["up"]), as llama.cpp's fused Q4_K FFN call."""
    groups = {key: grp for key, _, grp in LLAMA_LAYER}
    if not fuse_ffn:
        keys = [key for key, _, _ in LLAMA_LAYER]
        return q4k.make_tasks([layer[k].data for k in keys], [xs[groups[k]] for k in keys],
                              [outs[k] for k in keys])
    items = []
    for key, _, grp in LLAMA_LAYER:
        if key == "gate":
            continue
        it = dict(W=layer[key].data, x=xs[grp], out=outs[key])
        if key == "up":
            it.update(W_gate=layer["gate"].data, glu="swiglu")
        items.append(it)
    return q4k.make_tasks_ex(items)


def write_q4k_gguf(path: str | Path, tensors: dict[str, np.ndarray], arch: str = "llama",
                   extra_f32: dict[str, np.ndarray] | None = None, n_layers: int | None = None) -> None:
    """Write a GGUF file holding Q4_K matrices given as (rows, K/256*144) uint8
    arrays (and optional fp32 tensors): for tests and for staging synthetic
    weights in the on-disk format."""
    import gguf
    w = gguf.GGUFWriter(str(path), arch)
    if n_layers is not None:
        w.add_block_count(n_layers)
    for name, a in tensors.items():
        a = np.ascontiguousarray(a, dtype=np.uint8)
        if a.ndim != 2 or a.shape[1] % BLOCK_BYTES:
            raise ValueError(f"{name}: expected (rows, K/256*144) uint8, got {a.shape}")
        w.add_tensor(name, a, raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    for name, a in (extra_f32 or {}).items():
        w.add_tensor(name, np.ascontiguousarray(a, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
