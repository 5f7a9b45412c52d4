"""GGUF loading (gemv-q4_k-optimization_b200/gguf_loader.py): a synthetic
llama-style checkpoint written with gguf-py, read back, checked byte for
byte and shape for shape on the CPU, then run through the GEMV on the GPU
against the oracle (plain and with the ffn gate/up fused)."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

from test_gpu_glu import check  # fused-epilogue reference and tolerance

SHAPES = {"attn_q": (256, 512), "attn_k": (64, 512), "attn_v": (64, 512), "attn_output": (256, 512),
          "ffn_gate": (768, 512), "ffn_up": (768, 512), "ffn_down": (256, 768)}


@pytest.fixture(scope="module")
def loader(q4k):
    return importlib.import_module("q4k_b200.gguf_loader")


@pytest.fixture(scope="module")
def model_file(q4k, loader, tmp_path_factory):
    rng = np.random.default_rng(42)
    mats = {}
    for i in range(2):
        for stem, (rows, K) in SHAPES.items():
            mats[f"blk.{i}.{stem}.weight"] = q4k.gen_q4k_numpy(rng, rows, K)
    path = tmp_path_factory.mktemp("gguf") / "tiny-q4k.gguf"
    loader.write_q4k_gguf(path, mats, n_layers=2,
                          extra_f32={"blk.0.attn_norm.weight": np.ones(512, np.float32)})
    return path, mats


def test_gguf_roundtrip_bytes_and_shapes(loader, model_file):
    path, mats = model_file
    m = loader.GGUFModel(path)
    assert m.arch == "llama"
    assert m.n_layers() == 2
    assert sorted(m.q4k_names()) == sorted(mats)
    for name, a in mats.items():
        t = m.q4k(name)
        assert (t.rows, t.K) == (a.shape[0], a.shape[1] // 144 * 256)
        assert np.array_equal(np.asarray(t.data), a), name


def test_gguf_rejects_other_types_and_missing(loader, model_file):
    m = loader.GGUFModel(model_file[0])
    with pytest.raises(TypeError):
        m.q4k("blk.0.attn_norm.weight")
    with pytest.raises(KeyError):
        m.q4k("blk.9.attn_q.weight")


def test_gguf_bytes_dequantize_like_gguf_py(oracle, loader, model_file):
    """The loaded bytes mean to gguf-py's own Q4_K dequantizer what they mean to the oracle."""
    import gguf
    m = loader.GGUFModel(model_file[0])
    t = m.q4k("blk.1.ffn_down.weight")
    W = np.asarray(t.data)
    deq = gguf.quants.dequantize(W, gguf.GGMLQuantizationType.Q4_K).astype(np.float64)  # (rows, K)
    # y = W_deq . e_k picks column k.  A one-hot x quantizes to q = 127 with
    # d8 = fp16(1/127), so the oracle's product is column k times 127 * fp16(1/127).
    K = t.K
    for k in (5, 300, K - 1):
        x = np.zeros((1, K), np.float32)
        x[0, k] = 1.0
        y = oracle.gemv_f32(W, x)[0].astype(np.float64)
        scale = 127.0 * float(np.float16(np.float32(1.0) / np.float32(127.0)))
        assert np.allclose(y, deq[:, k] * scale, rtol=1e-5, atol=1e-6), k


@pytest.mark.gpu
def test_gguf_layer_gemv_on_device(q4k, oracle, loader, model_file):
    import torch
    dev = torch.device("cuda", 0)
    m = loader.GGUFModel(model_file[0])
    layer = m.layer(1, dev)
    rng = np.random.default_rng(3)
    xs_np = {"attn": rng.standard_normal((1, 512)), "o": rng.standard_normal((1, 512)),
             "ffn": rng.standard_normal((1, 512)), "down": rng.standard_normal((1, 768))}
    xs_np = {k: v.astype(np.float32) for k, v in xs_np.items()}
    xs = {k: torch.from_numpy(v).to(dev) for k, v in xs_np.items()}
    groups = {key: grp for key, _, grp in loader.LLAMA_LAYER}
    outs = {key: torch.empty((1, layer[key].rows), device=dev) for key in groups}
    ws = q4k.Workspace()
    q4k.gemv_batch(loader.layer_tasks(q4k, layer, xs, outs), 1, ws)
    for key, grp in groups.items():
        want = oracle.gemv_f32(layer[key].data.cpu().numpy(), xs_np[grp]).astype(np.float64)
        check(outs[key].cpu().numpy(), want, want, "none", key)
    # the same layer with gate/up fused (SwiGLU into outs["up"])
    fused = {key: torch.empty_like(v) for key, v in outs.items()}
    q4k.gemv_batch_ex(loader.layer_tasks(q4k, layer, xs, fused, fuse_ffn=True), 1, ws)
    r = oracle.gemv_f32(layer["up"].data.cpu().numpy(), xs_np["ffn"]).astype(np.float64)
    g = oracle.gemv_f32(layer["gate"].data.cpu().numpy(), xs_np["ffn"]).astype(np.float64)
    check(fused["up"].cpu().numpy(), r, g, "swiglu", "fused ffn from GGUF")
    assert ws.status() == 0
