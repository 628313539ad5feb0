"""Safetensors archives and the Gemma weight loader on the host
(Gemma4WeightLoader.swift semantics): prefix detection, dense vs affine
4-bit tensors, the unaligned-U32 case, shards, and malformed files."""
import json
import struct

import numpy as np
import pytest

import oracle
from popcorn_b200 import safetensors as st

torch = pytest.importorskip("torch")


def _archive(tmp_path, prefix="language_model.model", odd_first=True):
    rng = np.random.default_rng(0)
    w = rng.standard_normal((32, 256)).astype(np.float32) * 0.02
    packed, sc, bi = oracle.aq_quantize(w, sdt="bf16")
    dense = oracle.to_dtype(rng.standard_normal((8, 16)), "bf16")
    t = {}
    if odd_first:  # an odd element count of 16-bit values puts the next tensor at a 2-byte offset
        t[prefix + ".layers.0.input_layernorm.weight"] = (oracle.to_dtype(rng.standard_normal(7), "bf16"), "BF16")
    t[prefix + ".layers.0.self_attn.q_proj.weight"] = (packed, "U32")
    t[prefix + ".layers.0.self_attn.q_proj.scales"] = (sc, "BF16")
    t[prefix + ".layers.0.self_attn.q_proj.biases"] = (bi, "BF16")
    t[prefix + ".embed_tokens.weight"] = (dense, "BF16")
    path = str(tmp_path / "model.safetensors")
    st.save(path, t, metadata={"format": "mlx"})
    return path, packed, sc, bi, dense


def test_roundtrip_and_alignment(tmp_path):
    path, packed, sc, bi, dense = _archive(tmp_path)
    a = st.SafeTensors(path)
    name = "language_model.model.layers.0.self_attn.q_proj.weight"
    dt, shape, off, nb = a.info(name)
    assert dt == "U32" and shape == (32, 32) and off % 4 == 2  # the reference's misaligned case
    assert np.array_equal(a.array(name), packed)
    assert a.metadata == {"format": "mlx"}
    t = a.to_device(name, "cpu")
    assert t.data_ptr() % 16 == 0 and np.array_equal(t.view(torch.int32).numpy().view(np.uint32), packed)


@pytest.mark.parametrize("prefix", ["language_model.model", "model.language_model"])
def test_weight_loader(tmp_path, prefix):
    path, packed, sc, bi, dense = _archive(tmp_path, prefix)
    wl = st.WeightLoader(st.SafeTensors(path), st.Quantization(4, 64), device="cpu")
    assert wl.prefix == prefix
    q = wl.linear(wl.layer_prefix(0) + ".self_attn.q_proj")
    assert (q.out_features, q.in_features, q.bits, q.group_size) == (32, 256, 4, 64)
    assert np.array_equal(q.packed_tensor.numpy().view(np.uint32), packed)
    assert np.array_equal(q.scales.view(torch.int16).numpy().view(np.uint16), sc)
    e = wl.embedding(wl.qualify("embed_tokens"))
    assert e.dtype == torch.bfloat16 and np.array_equal(e.view(torch.int16).numpy().view(np.uint16), dense)
    # without a quantization block every tensor is dense
    wl2 = st.WeightLoader(st.SafeTensors(path), None, device="cpu")
    assert isinstance(wl2.linear(wl2.layer_prefix(0) + ".self_attn.q_proj"), torch.Tensor)


def test_shards(tmp_path):
    st.save(str(tmp_path / "a.safetensors"), {"model.language_model.x.weight": (np.ones(4, np.float32), "F32")})
    st.save(str(tmp_path / "b.safetensors"), {"model.language_model.y.weight": (np.zeros(3, np.int32), "I32")})
    a = st.SafeTensors(str(tmp_path))
    assert sorted(a.names) == ["model.language_model.x.weight", "model.language_model.y.weight"]
    assert a.array("model.language_model.y.weight").dtype == np.int32


def test_errors(tmp_path):
    path = str(tmp_path / "bad.safetensors")
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(st.SafeTensorsError):
        st.SafeTensors(path)
    h = json.dumps({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 8]}}).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(st.SafeTensorsError):  # 4 f32 need 16 bytes
        st.SafeTensors(path)
    good = str(tmp_path / "g.safetensors")
    st.save(good, {"other.weight": (np.ones(2, np.float32), "F32")})
    with pytest.raises(st.SafeTensorsError):  # no Gemma language-model prefix
        st.WeightLoader(st.SafeTensors(good))
    st.save(good, {"model.language_model.p.weight": (np.ones((2, 2), np.float32), "F32"),
                   "model.language_model.p.scales": (np.ones((2, 1), np.float32), "F32"),
                   "model.language_model.p.biases": (np.ones((2, 1), np.float32), "F32")})
    wl = st.WeightLoader(st.SafeTensors(good), st.Quantization(), device="cpu")
    with pytest.raises(st.SafeTensorsError):  # packed weights must be U32
        wl.linear("model.language_model.p")
